"""Tensor-parallel plumbing of a loaded decoder: peer memory and the fused collectives its
launches call (attached once per model, on every rank)."""

from __future__ import annotations


def attach(model, device) -> None:
    raise NotImplementedError("tensor parallelism is not attached yet")


def detach(model) -> None:
    pass
