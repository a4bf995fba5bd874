"""The model runner: turns each scheduled step into one engine call.

vLLM's scheduler decides which requests run, how many tokens each feeds and which KV blocks they
hold; this runner keeps each request's known tokens and block table, stages the step's tokens in
one host-to-device copy, calls the engine (`Decoder.forward`) and returns the sampled tokens in
vLLM's order (the reference's runner: integrations/furiosa-opt-vllm/furiosa_opt_vllm/runner.py).
"""

from __future__ import annotations

import numpy as np

from . import batch, pooling, speculation, thinking
from .paging import BlockTable, first_group
from .request import State


class Pending:
    """A step's sampled tokens, still on the device until `collect()` reads them (once; later calls
    return the same result)."""

    def __init__(self, runner: "Runner", order, drafts, kept):
        self.runner, self.order, self.drafts, self.kept = runner, order, drafts, kept
        self.result = None

    def collect(self) -> tuple[list[str], list[list[int]]]:
        if self.result is not None:
            return self.result
        if self in self.runner.uncollected:
            self.runner.uncollected.remove(self)
        self.result = self._read()
        return self.result

    def _read(self) -> tuple[list[str], list[list[int]]]:
        host: dict[int, list[int]] = {}  # one device-to-host read per engine call
        sampled = []
        for rid, d, runs in zip(self.order, self.drafts, self.kept):
            rows = []
            for out, first, n in runs:
                key = id(out)
                if key not in host:
                    host[key] = out.to_host().numpy().tolist()
                rows += [int(t) for t in host[key][first : first + n]]
            st = self.runner.states.get(rid)
            if d:
                # Every fed row came back; the targets start at the newest known token's row.
                fed = len(rows) - len(d)
                got = speculation.accept(d, rows[fed - 1 :])
                if st is not None:
                    st.computed -= len(d) - (len(got) - 1)
            else:
                got = rows
            if st is not None and st.budget is not None:
                forced = thinking.apply(st.budget, got)
                st.computed -= len(got) - len(forced)  # rows verified against a replaced token
                got = forced
            if st is not None:
                st.tokens.extend(got)
            sampled.append(got)
        return self.order, sampled


class Runner:
    def __init__(self, model, device, cache, adapters=None, pooling_config=None, reasoning=None):
        import furiosa_opt_engine as engine
        from furiosa_opt_engine import decoder as dec

        self.engine, self.dec = engine, dec
        self.model, self.device, self.cache = model, device, cache
        self.adapters = adapters  # lora.Adapters when vLLM serves LoRA, else None
        # Pooling models: {"task": "embed" | "classify", "method": pooling type, "labels": n}.
        self.pooling_config = pooling_config
        self.pooled: list = []  # each request's pooled output of the last step (None: not yet)
        # (start marker IDs, end marker IDs) of a reasoning model (vLLM's reasoning config), or None.
        self.reasoning = reasoning
        self.states: dict[str, State] = {}
        # Steps whose tokens are still on the device, oldest first. vLLM collects a step before it
        # issues the second one after it on the driver rank; the other tensor-parallel ranks are
        # never asked, so a step collects every older step but the newest itself (their tokens
        # are long complete) and the newest feeds the next step from the device.
        self.uncollected: list[Pending] = []

    # -------------------------------------------------------------------- scheduler bookkeeping
    def update(self, so) -> None:
        for rid in so.finished_req_ids:
            self.states.pop(rid, None)
        for nr in so.scheduled_new_reqs:
            prompt = list(nr.prefill_token_ids if getattr(nr, "prefill_token_ids", None) else nr.prompt_token_ids)
            self.states[nr.req_id] = State(prompt, len(prompt), nr.num_computed_tokens,
                                           BlockTable(first_group(nr.block_ids)),
                                           lora=getattr(nr, "lora_request", None))
            sampling = getattr(nr, "sampling_params", None)
            budget = getattr(sampling, "thinking_token_budget", None)
            if budget is not None:
                if not getattr(self, "reasoning", None):
                    raise ValueError(f"{nr.req_id}: thinking_token_budget needs the model's reasoning markers "
                                     "(start vLLM with --reasoning-parser)")
                self.states[nr.req_id].budget = thinking.Budget(budget, *self.reasoning)
                self.states[nr.req_id].budget.reset(prompt)
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
                    st.tail = None
                    if st.budget is not None:
                        st.budget.reset(st.tokens, st.prompt)
            elif nb is not None:
                st.table.append(first_group(nb))
            st.computed = cr.num_computed_tokens[i]

    # -------------------------------------------------------------------- one step
    def step(self, so, collect: bool = True):
        """Runs the scheduled rows in calls of at most `decoder.rows` rows.

        With `collect` it returns (request IDs in order, sampled tokens per request). Without it
        (async scheduling, greedy, no drafts) it returns a `Pending` whose `collect()` reads the
        tokens later: each sampling request's token stays on the device, and the next step, which
        vLLM schedules before collecting this one, reads its input token from there. For a pooling
        model the tokens are empty and `pooled` holds each request's output."""
        if self.pooling_config is not None:
            return self.pool_step(so)
        while len(self.uncollected) > 1 or (self.uncollected and collect):
            self.uncollected[0].collect()
        self.update(so)
        order = list(so.num_scheduled_tokens.keys())
        if not order:
            return ([], []) if collect else Pending(self, [], [], [])
        counts = [int(so.num_scheduled_tokens[r]) for r in order]
        spec = getattr(so, "scheduled_spec_decode_tokens", None) or {}
        drafts = [list(spec.get(r, ())) for r in order]
        step, hosts = [], []
        for rid, n, d in zip(order, counts, drafts):
            st = self.states[rid]
            fed = n - len(d)  # rows of tokens the request has (known, or in flight on the device)
            on_device = max(0, st.computed + fed - len(st.tokens))
            if on_device and (st.tail is None or d or on_device > 1):
                raise ValueError(f"{rid}: {fed} rows scheduled after {st.computed} of {len(st.tokens)} known tokens")
            samples = st.computed + fed == len(st.tokens) + on_device
            if d and not samples:
                raise ValueError(f"{rid}: drafts scheduled before the newest token was fed")
            hosts.append(st.scheduled(fed - on_device) + d)
            keep = batch.KEEP_ALL if d else (batch.KEEP_LAST if samples else batch.KEEP_NONE)
            # The device row is the request's last fed row; drafts (host tokens) never follow it.
            step.append(batch.Scheduled(st.computed, n, n - on_device, keep))
        # Adapters: each sequence naming a LoRA runs with its slot of this step's list.
        slots, adapters = {}, None
        if self.adapters is not None:
            named = {rid: self.states[rid].lora for rid in order
                     if self.states[rid].lora is not None and self.states[rid].lora.lora_int_id}
            if named:
                slots = self.adapters.activate(named)
                adapters = list(self.adapters.slots)
        kept: list[list] = [[] for _ in order]  # (output, first row, rows) of each request's kept runs
        for call in batch.plan(step, int(self.model.rows)):
            host_rows = [r for r in call if not r.device]
            flat = np.empty(max(sum(r.rows for r in host_rows), 1), dtype=np.int32)
            at = 0
            for r in host_rows:
                flat[at : at + r.rows] = hosts[r.seq][r.offset : r.offset + r.rows]
                at += r.rows
            tokens = self.engine.HostTensor.from_dlpack(flat).to_hbm(self.device) if host_rows else None
            reqs, at = [], 0
            for r in call:
                st = self.states[order[r.seq]]
                if r.device:
                    src, row = st.tail
                    toks = src[row : row + 1]
                else:
                    toks = tokens[at : at + r.rows]
                    at += r.rows
                mode = (self.dec.Keep.ALL if r.keep == batch.KEEP_ALL else
                        self.dec.Keep.LAST if r.keep == batch.KEEP_LAST else self.dec.Keep.NONE)
                reqs.append(self.dec.Request([st.table.blocks], r.cached, toks, mode, adapter=slots.get(order[r.seq])))
            out = self.model.forward(reqs, self.cache, adapters)
            k = 0
            for r in call:
                n = batch.kept_rows(r)
                if n:
                    kept[r.seq].append((out, k, n))
                k += n
        for i, (rid, n, d) in enumerate(zip(order, counts, drafts)):
            st = self.states[rid]
            st.computed += n
            # The newest sampled token stays on the device until collected; the next step reads it.
            st.tail = (kept[i][-1][0], kept[i][-1][1] + kept[i][-1][2] - 1) if kept[i] and not d else None
        pending = Pending(self, order, drafts, kept)
        if collect:
            return pending.collect()
        self.uncollected.append(pending)
        return pending

    def reads_each_step(self, so) -> bool:
        """Whether a step's tokens must reach the host as it is issued: a scheduled request has a
        thinking budget, which may replace the engine's token."""
        return any(getattr(self.states.get(r), "budget", None) is not None for r in so.num_scheduled_tokens)

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
