"""The vLLM worker of one GPU: vLLM's executor calls it as it calls its own GPU worker, and it
answers through the engine. It loads the checkpoint with the engine (every chip of a replica is
one worker process, joined in vLLM's process group), reports the engine's KV layout so vLLM's
cache manager hands out the engine's blocks, allocates the cache once vLLM sized it, and runs
every scheduled step as one engine call (the reference's worker:
integrations/furiosa-opt-vllm/furiosa_opt_vllm/worker.py)."""

from __future__ import annotations

import torch
from vllm.v1.outputs import AsyncModelRunnerOutput, ModelRunnerOutput
from vllm.v1.worker.worker_base import WorkerBase

from . import admission, lora, media, pooling, residency, speculation
from . import cache as kv
from . import load
from .runner import Runner


class Collected(AsyncModelRunnerOutput):
    """A greedy step's output whose tokens are still on the device: `get_output` reads them (vLLM
    calls it after issuing the next step, so the device works while the host schedules)."""

    def __init__(self, pending, worker=None):
        self.pending, self.worker = pending, worker
        self.output = ModelRunnerOutput(req_ids=[], req_id_to_index={})  # filled by get_output

    def get_output(self) -> ModelRunnerOutput:
        try:
            ids, sampled = self.pending.collect()
        except Exception as error:
            # vLLM has issued the next step already; it raises this failure, since its requests
            # lack the tokens this step failed to read.
            if self.worker is not None:
                self.worker.failure = error
            raise
        self.output.req_ids = ids
        self.output.req_id_to_index = {r: i for i, r in enumerate(ids)}
        self.output.sampled_token_ids = sampled
        return self.output


class Worker(WorkerBase):
    def __init__(self, vllm_config, local_rank: int, rank: int, distributed_init_method: str,
                 is_driver_worker: bool = False, **kwargs):
        super().__init__(vllm_config=vllm_config, local_rank=local_rank, rank=rank,
                         distributed_init_method=distributed_init_method, is_driver_worker=is_driver_worker)
        self.model = self.engine_device = self.cache = self.runner = None
        # vLLM's executor threads set this as their CUDA device; the engine's Device is engine_device.
        self.device = None
        self.copy = None  # sleep mode: the host copy of the checkpoint the weights loaded from
        self.adapters = None  # lora.Adapters when vLLM serves LoRA
        self.asleep: dict = {}
        self.pending: ModelRunnerOutput | None = None
        self.proposer = None  # speculation.Proposer when vLLM speculates
        self.pooling = getattr(self.model_config, "runner_type", "generate") == "pooling"
        self.drafts = None  # the drafts proposed after the last step, for take_draft_token_ids
        self.media = None  # media.Media when vLLM runs this instance as a media encoder alone
        self.failure: BaseException | None = None  # the first step whose tokens could not be read

    # ------------------------------------------------------------------------ life cycle
    def init_device(self) -> None:
        from vllm.distributed import ensure_model_parallel_initialized, init_distributed_environment

        torch.cuda.set_device(self.local_rank)
        self.device = torch.device("cuda", self.local_rank)
        pc = self.parallel_config
        init_distributed_environment(pc.world_size, self.rank, self.distributed_init_method, self.local_rank,
                                     backend="nccl")
        ensure_model_parallel_initialized(pc.tensor_parallel_size, pc.pipeline_parallel_size)

    def load_model(self, *args, **kwargs) -> None:
        import os

        from vllm.distributed import get_tensor_model_parallel_rank, get_tp_group

        pc = self.parallel_config
        tp_size = pc.tensor_parallel_size
        tp_rank = get_tensor_model_parallel_rank() if tp_size > 1 else 0
        chips = load.replica_chips(self.local_rank, tp_rank, tp_size, getattr(pc, "data_parallel_rank", 0) or 0,
                                   os.environ.get("FURIOSA_VISIBLE_CHIPS"))
        if media.encoder_only(self.model_config):
            # An encoder-only instance: the checkpoint's media encoder alone, no KV cache.
            import furiosa_opt_engine as engine

            if tp_size > 1:
                raise admission.Refused("tensor_parallel_size", "the media encoder runs on one GPU")
            self.engine_device = engine.Device(engine.Placement(chips, range(8)))
            encoder = engine.LoadOptions().encoder().load(load.checkpoint(self.model_config.model), self.engine_device)
            self.media = media.Media(engine, encoder, self.engine_device)
            return
        architecture = None
        if self.pooling:
            declared = load.architectures(self.model_config.model)
            architecture = next((pooling.base_architecture(a) for a in declared
                                 if pooling.base_architecture(a) is not None), None)
            if architecture is None:
                raise admission.Refused("runner", f"pooling serves Qwen3 causal and classifier checkpoints, "
                                                  f"not {', '.join(declared)}")
        self.architecture = architecture
        self.checkpoint_config = load.overridden(self.model_config.model, getattr(self.model_config, "hf_overrides", None))
        self.model, self.engine_device, self.copy = load.load(
            self.model_config.model, tp_rank, tp_size, keep_copy=bool(self.model_config.enable_sleep_mode),
            chips=chips, group=get_tp_group().cpu_group if tp_size > 1 else None,
            adapters=self.lora_config is not None, architecture=architecture, config=self.checkpoint_config)
        from .additional import Section

        if not Section.parse(self.vllm_config).cuda_graphs:
            self.model.set_graphs(False)
        sc = self.vllm_config.speculative_config
        if sc is not None and str(sc.method) == "draft_model":
            # The draft decoder beside the target on this worker's GPU.
            self.proposer = speculation.DraftModel(
                self.vllm_config, lambda path: load.load_from(load.checkpoint(path), self.engine_device, 1))
        elif sc is not None:
            self.proposer = speculation.Proposer(self.vllm_config)
        if self.lora_config is not None:
            self.adapters = lora.Adapters(self.lora_config.max_loras, self.lora_config.max_cpu_loras,
                                          self.model.adapters)

    # ------------------------------------------------------------------------ sleep mode
    def sleep(self, level: int = 1) -> None:
        residency.sleep(self, level)

    def wake_up(self, tags: list[str] | None = None) -> None:
        residency.wake_up(self, tags)

    def discard(self, tags: tuple[str, ...]) -> None:
        residency.release(self, tags)

    def reload_weights(self, weights_iterator: object = None, weights_path: str | None = None,
                       is_checkpoint_format: bool = True) -> None:
        """Reads the served checkpoint's files again and swaps the weights in; weights from an
        iterator or another path are refused (the engine only loads checkpoints)."""
        for name, value, default in (("weights_iterator", weights_iterator, None),
                                     ("weights_path", weights_path, None),
                                     ("is_checkpoint_format", is_checkpoint_format, True)):
            if value != default:
                raise admission.Refused(name, "the engine reloads the served checkpoint's own files")
        residency.reload(self)

    def determine_available_memory(self) -> int:
        if self.media is not None:
            return 0  # an encoder-only instance caches no keys or values
        free, total = torch.cuda.mem_get_info()
        budget = int(total * self.cache_config.gpu_memory_utilization) - (total - free)
        # The engine addresses each layer's cache with 32-bit byte offsets.
        layers = len(self.model.cache.groups[0].layers)
        budget = max(min(budget, layers * ((1 << 31) - (1 << 20))), 0)
        if isinstance(self.proposer, speculation.DraftModel):
            # vLLM sizes the target's blocks; the draft's cache takes as many blocks of its own size.
            page = int(self.model.cache.pools[0].bytes) * layers
            draft = self.proposer.page_bytes() * len(self.proposer.model.cache.groups[0].layers)
            budget = budget * page // (page + draft)
        return budget

    def get_kv_cache_spec(self):
        if self.media is not None:
            return {}
        return kv.spec(self.model, self.model_config)

    def get_supported_kv_cache_layouts(self) -> list[str]:
        # No torch attention backend runs here for vLLM to ask; the engine's page layout is fixed.
        return list(kv.LAYOUTS)

    def get_cache_block_size_bytes(self) -> int:
        """Bytes of one block across every layer (vLLM's page of each layer's spec)."""
        return sum(int(s.page_size_bytes) for s in self.get_kv_cache_spec().values())

    def initialize_from_config(self, kv_cache_config) -> None:
        from furiosa_opt_engine import decoder as dec

        if self.media is not None:
            if self.vllm_config.ec_transfer_config is not None:
                from vllm.distributed.ec_transfer import ensure_ec_transfer_initialized

                ensure_ec_transfer_initialized(self.vllm_config)
            return

        self.cache = dec.Cache(self.model.cache, int(kv_cache_config.num_blocks))
        rc = getattr(self.vllm_config, "reasoning_config", None)
        markers = None
        if rc is not None and getattr(rc, "reasoning_end_token_ids", None):
            markers = (list(getattr(rc, "reasoning_start_token_ids", None) or []), list(rc.reasoning_end_token_ids))
        self.runner = Runner(self.model, self.engine_device, self.cache, self.adapters, self.pooling_config(),
                             reasoning=markers)
        if self.proposer is not None:
            self.proposer.attach(self.runner, int(kv_cache_config.num_blocks))
        if self.vllm_config.kv_transfer_config is not None:
            # KV offloading: vLLM's connector over the engine's cache pages.
            from vllm.distributed.kv_transfer import ensure_kv_transfer_initialized, get_kv_transfer_group

            from . import offload

            offload.attach(self.cache)
            ensure_kv_transfer_initialized(self.vllm_config, kv_cache_config)
            get_kv_transfer_group().register_kv_caches({})

    # ------------------------------------------------------------------------ LoRA
    def add_lora(self, lora_request) -> bool:
        return self.adapters.add(lora_request)

    def remove_lora(self, lora_id: int) -> bool:
        return self.adapters.remove(lora_id)

    def pin_lora(self, lora_id: int) -> bool:
        return self.adapters.pin(lora_id)

    def list_loras(self) -> set[int]:
        return self.adapters.ids() if self.adapters is not None else set()

    def compile_or_warm_up_model(self):
        from vllm.v1.worker.worker_base import CompilationTimes

        return CompilationTimes(0.0, 0.0)

    def get_supported_tasks(self):
        if media.encoder_only(self.model_config):
            return ("generate",)
        if not self.pooling:
            return ("generate",)
        if self.model is not None:
            return ("classify",) if self.model.output.name == "SCORES" else ("embed",)
        declared = load.architectures(self.model_config.model)
        return ("classify",) if any(a.endswith("ForSequenceClassification") for a in declared) else ("embed",)

    def pooling_config(self) -> dict | None:
        """The runner's pooling settings: the task the model serves, vLLM's pooling type and, for
        a classifier, its labels."""
        if not self.pooling:
            return None
        pc = self.model_config.pooler_config
        method = getattr(pc, "seq_pooling_type", None) or getattr(pc, "pooling_type", None) or "LAST"
        task = self.get_supported_tasks()[0]
        labels = int(getattr(self.model_config.hf_config, "num_labels", 0) or 0) if task == "classify" else 0
        return {"task": task, "method": str(getattr(method, "value", method)), "labels": labels}

    def check_health(self) -> None:
        """Raises when the engine's device failed: a failed launch, copy or bounded device wait
        poisons the device, and every later call (this synchronization included) raises with the
        first failure, so vLLM reports the engine unhealthy instead of scheduling more steps."""
        residency.check_health(self)

    def update_max_model_len(self, max_model_len: int) -> None:
        self.model_config.max_model_len = max_model_len

    def reset_mm_cache(self) -> None:
        pass

    def reset_encoder_cache(self) -> None:
        pass

    def get_kv_connector_handshake_metadata(self):
        return None

    def take_draft_token_ids(self):
        drafts, self.drafts = self.drafts, None
        return drafts

    def shutdown(self) -> None:
        if self.model is not None and self.parallel_config.tensor_parallel_size > 1:
            from furiosa_opt_models_b200.parallel import tp

            tp.detach(self.model)
        self.model = self.runner = self.cache = None

    # ------------------------------------------------------------------------ steps
    def connector(self):
        """vLLM's KV connector of this worker (KV offloading), or None."""
        if self.vllm_config.kv_transfer_config is None:
            return None
        from vllm.distributed.kv_transfer import get_kv_transfer_group, has_kv_transfer_group

        return get_kv_transfer_group() if has_kv_transfer_group() else None

    def execute_model(self, scheduler_output):
        if self.failure is not None:
            raise RuntimeError("an earlier step's tokens could not be read") from self.failure
        if self.media is not None:
            return media.execute(self.media, scheduler_output)
        conn = self.connector()
        meta = getattr(scheduler_output, "kv_connector_metadata", None)
        if conn is not None and meta is not None:
            # Loads from host memory go on the engine's stream ahead of this step's calls.
            conn.handle_preemptions(meta)
            conn.bind_connector_metadata(meta)
            conn.start_load_kv(None)
        try:
            self._run(scheduler_output)
        finally:
            if conn is not None and meta is not None:
                # Stores of the blocks this step filled follow its calls on the same stream.
                from vllm.v1.outputs import KVConnectorOutput

                conn.wait_for_save()
                sending, recving = conn.get_finished(scheduler_output.finished_req_ids)
                kvo = KVConnectorOutput(finished_sending=sending, finished_recving=recving,
                                        kv_connector_stats=conn.get_kv_connector_stats(),
                                        kv_connector_worker_meta=conn.build_connector_worker_meta())
                conn.clear_connector_metadata()
                target = self.pending.output if isinstance(self.pending, Collected) else self.pending
                if target is not None:
                    target.kv_connector_output = kvo
        if scheduler_output.total_num_scheduled_tokens == 0:
            # Nothing ran: vLLM takes this call's return as the step's output (no sampling).
            out, self.pending = self.pending, None
            return out
        return None

    def _run(self, scheduler_output) -> None:
        if scheduler_output.total_num_scheduled_tokens == 0:
            self.runner.update(scheduler_output)
            self.pending = ModelRunnerOutput(req_ids=[], req_id_to_index={})
            return
        if self.asynchronous():
            # The tokens stay on the device; vLLM collects them after it has issued the next step.
            step = self.runner.step(scheduler_output, collect=False)
            if self.runner.reads_each_step(scheduler_output):
                step.collect()  # a thinking budget may replace a token: the next step feeds it from the host
            self.pending = Collected(step, self)
            return
        ids, sampled = self.runner.step(scheduler_output)
        self.pending = ModelRunnerOutput(req_ids=ids, req_id_to_index={r: i for i, r in enumerate(ids)},
                                         sampled_token_ids=sampled,
                                         pooler_output=list(self.runner.pooled) if self.pooling else None)
        if self.proposer is not None:
            from vllm.v1.outputs import DraftTokenIds

            self.drafts = DraftTokenIds(ids, self.proposer.propose(ids, sampled, self.runner))

    def asynchronous(self) -> bool:
        """Greedy steps under vLLM's async scheduling: no pooling, no drafts to propose."""
        sc = getattr(self.vllm_config, "scheduler_config", None)
        return bool(getattr(sc, "async_scheduling", False)) and not self.pooling and self.proposer is None

    def sample_tokens(self, grammar_output=None):
        out, self.pending = self.pending, None
        return out

    def execute_dummy_batch(self) -> None:
        pass
