"""SGLang's tensor-parallel worker, replaced: its model runner loads the engine decoder on this
rank's GPU and lends SGLang request and token pools over the engine's KV cache (host tables of
16-token pages), and every scheduled batch runs through the engine (`steps.issue`, overlap
schedule with tokens kept on the device). The reference's worker:
integrations/furiosa-opt-sglang/furiosa_opt_sglang/worker.py:30-83 and runner.py.

`Generation` holds the batch entry points and depends on nothing of SGLang's; `worker_class()`
and `model_runner_class()` subclass SGLang's `TpModelWorker` and `ModelRunner` when SGLang is
importable (the hook table installs them).
"""

from __future__ import annotations

import numpy as np

from . import pools


class Generation:
    """The batch entry points of the plugin's worker. `engine_runner` is the plugin's `Runner`;
    `request_table()` is SGLang's request-to-token table (host memory)."""

    engine_runner = None
    enable_overlap = False

    def request_table(self):
        return self.model_runner.req_to_token_pool.req_to_token

    def forward_batch_generation(self, batch, forward_batch=None, pp_proxy_tensors=None, is_verify=False,
                                 skip_attn_backend_init=None, **options):
        # The engine call builds its own operands from the scheduled batch: a prebuilt forward
        # batch, pipeline proxies, verification or captured hidden states are other schedules,
        # which the platform refuses.
        ordinary = (batch is not None and forward_batch is None and pp_proxy_tensors is None and not is_verify
                    and not any(v for v in options.values() if v is not None and v is not False))
        if not ordinary:
            raise ValueError("furiosa-opt-sglang runs ordinary scheduled generation batches only")
        return self.engine_runner.issue(batch, self.request_table(), overlap=bool(self.enable_overlap))

    def forward_batch_embedding(self, batch):
        """An embedding batch: each request's last hidden row, L2-normalized, as SGLang's pooler
        output (a decoder loaded as its base model returns hidden rows)."""
        slots = [int(s) for s in batch.req_pool_indices.tolist()]
        seq_lens = [int(s) for s in batch.seq_lens.tolist()]
        lengths = [int(n) for n in batch.extend_lens]
        prefix = [t - n for t, n in zip(seq_lens, lengths)]
        ids = np.asarray(batch.input_ids.tolist(), dtype=np.int32)
        rows = self.engine_runner.embed(slots, seq_lens, prefix, lengths, ids, self.request_table())
        return pools.pooler_output(rows), False


_made: dict = {}


def model_runner_class():
    """SGLang's ModelRunner with its model, pools and attention setup replaced by the engine's."""
    if "runner" in _made:
        return _made["runner"]
    from sglang.srt.model_executor.model_runner import ModelRunner

    class EngineModelRunner(ModelRunner):
        def initialize(self, *args, **kwargs):
            pools.bind(self)

        def alloc_memory_pool(self, *args, **kwargs):
            pass  # `pools.bind` lends the pools over the engine cache

        def init_attention_backends(self, *args, **kwargs):
            self.attn_backend = None  # the engine runs attention

        def init_cuda_graphs(self, *args, **kwargs):
            # The engine captures its own decode graphs per row bucket.
            self.decode_cuda_graph_runner = None
            self.prefill_cuda_graph_runner = None

    _made["runner"] = EngineModelRunner
    return EngineModelRunner


def worker_class():
    """The TpModelWorker replacement the hook table installs."""
    if "worker" in _made:
        return _made["worker"]
    from sglang.srt.managers.tp_worker import TpModelWorker

    class Worker(Generation, TpModelWorker):
        def _init_model_runner(self, *args, **kwargs):
            runner = model_runner_class()
            self._model_runner = runner(model_config=self.model_config,
                                        mem_fraction_static=self.server_args.mem_fraction_static,
                                        gpu_id=self.gpu_id, nccl_port=self.nccl_port, server_args=self.server_args)

        @property
        def engine_runner(self):
            return self._model_runner.engine_runner

        @property
        def model_runner(self):
            return self._model_runner

    _made["worker"] = Worker
    return Worker
