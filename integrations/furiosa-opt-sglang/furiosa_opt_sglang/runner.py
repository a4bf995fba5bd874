"""Runs SGLang-shaped forward batches through the engine: the batch's new tokens staged in one
host-to-device copy a call, kept rows' greedy tokens returned in batch order. `issue` runs SGLang's
scheduled batches themselves (overlap schedule, tokens kept on the device: `steps`)."""

from __future__ import annotations

import numpy as np

from . import batch, paging, steps


class Runner:
    def __init__(self, model, device, cache):
        import furiosa_opt_engine as engine
        from furiosa_opt_engine import decoder as dec

        self.engine, self.dec = engine, dec
        self.model, self.device, self.cache = model, device, cache
        self.steps = steps.State()
        self.speculation = None  # speculative.Speculation when SGLang runs a speculative schedule

    def blocks(self, req_to_token, slot: int, positions: int) -> list[int]:
        """The engine blocks of a request-pool row's first `positions` positions."""
        return paging.blocks(req_to_token[slot], positions)

    def issue(self, schedule_batch, req_to_token, overlap: bool = True):
        """A scheduled generation batch (SGLang's ScheduleBatch fields) as engine calls; returns the
        step's result with its tokens still on the device (`steps.issue`)."""
        return steps.issue(self, schedule_batch, req_to_token, overlap=overlap)

    def forward(self, parts: list[batch.Part], tokens, req_to_token) -> list[int]:
        """Runs `parts` (new tokens in `tokens`, flat) and returns the next token of each kept
        part."""
        flat = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        dev = self.engine.HostTensor.from_dlpack(flat).to_hbm(self.device)
        reqs = []
        for p in parts:
            reqs.append(self.dec.Request([batch.request_blocks(req_to_token, p)], p.cached,
                                         dev[p.start : p.start + p.count],
                                         self.dec.Keep.LAST if p.keep else self.dec.Keep.NONE))
        out = self.model.forward(reqs, self.cache)
        return [int(t) for t in out.to_host().numpy().tolist()] if any(p.keep for p in parts) else []

    def extend(self, req_rows, seq_lens, prefix_lens, new_lens, tokens, req_to_token) -> list[int]:
        return self.forward(batch.parts(req_rows, seq_lens, prefix_lens, new_lens), tokens, req_to_token)

    def decode(self, req_rows, seq_lens, tokens, req_to_token) -> list[int]:
        return self.forward(batch.decode_parts(req_rows, seq_lens), tokens, req_to_token)

    def embed(self, req_rows, seq_lens, prefix_lens, new_lens, tokens, req_to_token, normalize=True):
        """An extend batch of an embedding model (a decoder whose calls return hidden rows, loaded
        as its base model): each request's last row, L2-normalized unless `normalize` is False,
        as an FP32 tensor [requests, hidden] (SGLang's LAST pooling of a causal embedder; the
        reference pools hidden rows the same way:
        integrations/furiosa-opt-sglang/furiosa_opt_sglang/embedding.py)."""
        import torch

        if self.model.output != self.dec.Output.HIDDEN:
            raise ValueError("embedding needs a decoder that returns hidden rows (its base model)")
        parts = batch.parts(req_rows, seq_lens, prefix_lens, new_lens)
        flat = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        dev = self.engine.HostTensor.from_dlpack(flat).to_hbm(self.device)
        reqs = [self.dec.Request([batch.request_blocks(req_to_token, p)], p.cached, dev[p.start : p.start + p.count],
                                 self.dec.Keep.LAST) for p in parts]
        rows = torch.from_numpy(np.asarray(self.model.forward(reqs, self.cache).to_host().numpy(), dtype=np.float32))
        return torch.nn.functional.normalize(rows, p=2, dim=-1) if normalize else rows
