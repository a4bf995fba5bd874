"""Runs SGLang-shaped forward batches through the engine: one engine call per batch, the batch's
new tokens staged in one host-to-device copy, kept rows' greedy tokens returned in batch order."""

from __future__ import annotations

import numpy as np

from . import batch


class Runner:
    def __init__(self, model, device, cache):
        import furiosa_opt_engine as engine
        from furiosa_opt_engine import decoder as dec

        self.engine, self.dec = engine, dec
        self.model, self.device, self.cache = model, device, cache

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
