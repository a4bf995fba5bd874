"""vLLM platform for B200 through the engine: vLLM's CUDA platform, with the plugin's worker,
16-token KV pages, no torch.compile or vLLM CUDA graphs (the engine captures its own), async
scheduling without speculation, and the plugin's refusals (the reference's platform:
integrations/furiosa-opt-vllm/furiosa_opt_vllm/platform.py)."""

from __future__ import annotations

from vllm.platforms.cuda import NvmlCudaPlatform

from . import admission


class B200Platform(NvmlCudaPlatform):
    @classmethod
    def check_and_update_config(cls, vllm_config) -> None:
        pc = vllm_config.parallel_config
        cc = vllm_config.cache_config
        admission.check(vllm_config)
        from .additional import Section

        Section.parse(vllm_config)
        super().check_and_update_config(vllm_config)
        pc.worker_cls = "furiosa_opt_vllm.worker.Worker"
        cc.block_size = 16
        # Async scheduling (vLLM issues step n+1 before it reads step n's tokens; the worker keeps
        # greedy tokens on the device meanwhile) as vLLM decided it, except with speculation: the
        # n-gram proposer reads every step's tokens on the host before the next step.
        if vllm_config.speculative_config is not None:
            vllm_config.scheduler_config.async_scheduling = False
        mc = vllm_config.model_config
        if mc is not None:
            mc.enforce_eager = True
        try:
            from vllm.config import CompilationMode, CUDAGraphMode

            vllm_config.compilation_config.mode = CompilationMode.NONE
            vllm_config.compilation_config.cudagraph_mode = CUDAGraphMode.NONE
        except Exception:
            pass

    @classmethod
    def validate_request(cls, processed_inputs, params) -> None:
        if getattr(params, "temperature", None) is None:
            from . import pooling

            task = getattr(params, "task", None)
            if task is not None and task not in pooling.TASKS:
                raise admission.Refused("task", f"{task}: pooling serves {', '.join(pooling.TASKS)}")
            return
        admission.sampling(params.temperature, params.top_k, params.top_p, params.n, params.logprobs,
                           params.prompt_logprobs)
        admission.unmodified(params)
