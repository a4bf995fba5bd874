"""Views of engine device memory as torch tensors (tests and tools): a device address, a shape
and a dtype through the CUDA array interface, no copy."""

from __future__ import annotations

import torch

_TYPESTR = {torch.bfloat16: "<u2", torch.float16: "<f2", torch.float32: "<f4", torch.int32: "<i4",
            torch.uint8: "|u1", torch.int64: "<i8"}


class _View:
    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (ptr, False), "version": 3, "strides": None}


def tensor(ptr: int, shape, dtype: torch.dtype, device: int | None = None) -> torch.Tensor:
    t = torch.as_tensor(_View(ptr, shape, _TYPESTR[dtype]), device="cuda" if device is None else f"cuda:{device}")
    return t.view(torch.bfloat16) if dtype == torch.bfloat16 else t


def weights(model) -> dict[str, torch.Tensor]:
    """Every weight of a loaded decoder, as torch views of its device memory."""
    out = {}
    for name in model.weight_names():
        ptr, shape = model.weight(name)
        out[name] = tensor(ptr, shape, torch.bfloat16, model.device.ordinal)
    return out
