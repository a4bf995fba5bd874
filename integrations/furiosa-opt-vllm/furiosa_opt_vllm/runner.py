"""The model runner: turns each scheduled step into one engine call.

vLLM's scheduler decides which requests run, how many tokens each feeds and which KV blocks they
hold; this runner keeps each request's known tokens and block table, stages the step's tokens in
one host-to-device copy, calls the engine (`Decoder.forward`) and returns the sampled tokens in
vLLM's order (the reference's runner: integrations/furiosa-opt-vllm/furiosa_opt_vllm/runner.py).
"""

from __future__ import annotations

import numpy as np

from . import pooling, speculation
from .paging import BlockTable, first_group
from .request import State


class Runner:
    def __init__(self, model, device, cache, adapters=None, pooling_config=None):
        import furiosa_opt_engine as engine
        from furiosa_opt_engine import decoder as dec

        self.engine, self.dec = engine, dec
        self.model, self.device, self.cache = model, device, cache
        self.adapters = adapters  # lora.Adapters when vLLM serves LoRA, else None
        # Pooling models: {"task": "embed" | "classify", "method": pooling type, "labels": n}.
        self.pooling_config = pooling_config
        self.pooled: list = []  # each request's pooled output of the last step (None: not yet)
        self.states: dict[str, State] = {}

    # -------------------------------------------------------------------- scheduler bookkeeping
    def update(self, so) -> None:
        for rid in so.finished_req_ids:
            self.states.pop(rid, None)
        for nr in so.scheduled_new_reqs:
            prompt = list(nr.prefill_token_ids if getattr(nr, "prefill_token_ids", None) else nr.prompt_token_ids)
            self.states[nr.req_id] = State(prompt, len(prompt), nr.num_computed_tokens,
                                           BlockTable(first_group(nr.block_ids)),
                                           lora=getattr(nr, "lora_request", None))
            params = getattr(nr, "pooling_params", None)
            if self.pooling_config is not None:
                if params is None:
                    raise ValueError(f"{nr.req_id}: a pooling model serves pooling requests only")
                self.states[nr.req_id].pool = pooling.Pool(params, self.pooling_config.get("method"), len(prompt))
        cr = so.scheduled_cached_reqs
        resumed = getattr(cr, "resumed_req_ids", set()) or set()
        all_tokens = getattr(cr, "all_token_ids", {}) or {}
        for i, rid in enumerate(cr.req_ids):
            st = self.states[rid]
            nb = cr.new_block_ids[i]
            if rid in resumed:
                st.table.replace(first_group(nb))
                if rid in all_tokens:
                    st.tokens = list(all_tokens[rid])
            elif nb is not None:
                st.table.append(first_group(nb))
            st.computed = cr.num_computed_tokens[i]

    # -------------------------------------------------------------------- one call
    def step(self, so) -> tuple[list[str], list[list[int]]]:
        """Runs the scheduled rows; returns (request IDs in order, sampled tokens per request).
        For a pooling model the tokens are empty and `pooled` holds each request's output."""
        if self.pooling_config is not None:
            return self.pool_step(so)
        self.update(so)
        order = list(so.num_scheduled_tokens.keys())
        if not order:
            return [], []
        counts = [int(so.num_scheduled_tokens[r]) for r in order]
        spec = getattr(so, "scheduled_spec_decode_tokens", None) or {}
        drafts = [list(spec.get(r, ())) for r in order]
        flat = np.empty(sum(counts), dtype=np.int32)
        keeps, at = [], 0
        for rid, n, d in zip(order, counts, drafts):
            st = self.states[rid]
            known = n - len(d)
            if d and not st.samples_after(known):
                raise ValueError(f"{rid}: drafts scheduled before the newest token was fed")
            flat[at : at + known] = st.scheduled(known)
            flat[at + known : at + n] = d
            # Rows the call returns: every row of a request with drafts (the target's token after
            # each fed token), else the last row when it samples.
            keeps.append(n if d else int(st.samples_after(known)))
            at += n
        tokens = self.engine.HostTensor.from_dlpack(flat).to_hbm(self.device)
        # Adapters: each sequence naming a LoRA runs with its slot of this call's list.
        slots, adapters = {}, None
        if self.adapters is not None:
            named = {rid: self.states[rid].lora for rid in order
                     if self.states[rid].lora is not None and self.states[rid].lora.lora_int_id}
            if named:
                slots = self.adapters.activate(named)
                adapters = list(self.adapters.slots)
        reqs, at = [], 0
        for rid, n, keep, d in zip(order, counts, keeps, drafts):
            st = self.states[rid]
            mode = self.dec.Keep.ALL if d else (self.dec.Keep.LAST if keep else self.dec.Keep.NONE)
            reqs.append(self.dec.Request([st.table.blocks], st.computed, tokens[at : at + n], mode,
                                         adapter=slots.get(rid)))
            at += n
        out = self.model.forward(reqs, self.cache, adapters)
        picked = out.to_host().numpy().tolist() if any(keeps) else []
        sampled, k = [], 0
        for rid, n, keep, d in zip(order, counts, keeps, drafts):
            st = self.states[rid]
            st.computed += n
            rows = [int(t) for t in picked[k : k + keep]]
            k += keep
            if d:
                # Every fed row came back; the targets start at the newest known token's row.
                got = speculation.accept(d, rows[n - len(d) - 1 :])
                st.computed -= len(d) - (len(got) - 1)
            else:
                got = rows
            st.tokens.extend(got)
            sampled.append(got)
        return order, sampled

    def pool_step(self, so) -> tuple[list[str], list[list[int]]]:
        """A step of a pooling model: prompt chunks whose kept rows (hidden values or label
        scores) feed each request's pooling; a request whose prompt completes gets its output."""
        import torch

        self.update(so)
        order = list(so.num_scheduled_tokens.keys())
        self.pooled = []
        if not order:
            return [], []
        counts = [int(so.num_scheduled_tokens[r]) for r in order]
        flat = np.empty(sum(counts), dtype=np.int32)
        keeps, at = [], 0
        for rid, n in zip(order, counts):
            st = self.states[rid]
            flat[at : at + n] = st.scheduled(n)
            keeps.append(n if st.pool.keep_all(st.computed) else int(st.samples_after(n)))
            at += n
        tokens = self.engine.HostTensor.from_dlpack(flat).to_hbm(self.device)
        reqs, at = [], 0
        for rid, n, keep in zip(order, counts, keeps):
            st = self.states[rid]
            mode = self.dec.Keep.ALL if keep == n and n > 1 else (self.dec.Keep.LAST if keep else self.dec.Keep.NONE)
            reqs.append(self.dec.Request([st.table.blocks], st.computed, tokens[at : at + n], mode))
            at += n
        out = self.model.forward(reqs, self.cache)
        rows = torch.from_numpy(np.asarray(out.to_host().numpy(), dtype=np.float32)) if any(keeps) else None
        k = 0
        cfg = self.pooling_config
        for rid, n, keep in zip(order, counts, keeps):
            st = self.states[rid]
            st.pool.add(rows[k : k + keep] if keep else torch.empty(0), st.computed, n)
            k += keep
            st.computed += n
            if st.pool.done(st.computed):
                v = st.pool.pooled()
                self.pooled.append(pooling.embed(v, st.pool.params) if cfg["task"] == "embed"
                                   else pooling.classify(v, st.pool.params, cfg["labels"]))
            else:
                self.pooled.append(None)
        return order, [[] for _ in order]
