"""Stand-ins for the SGLang classes the SGLang plugin subclasses or calls, with the constructor
signatures and fields the plugin relies on (SGLang 0.5.22 as the reference plugin uses it). SGLang
is not installed here or on the GPU hosts; `install(monkeypatch)` puts these modules in
`sys.modules` for one test."""

from __future__ import annotations

import sys
import types


class GenerationBatchResult:
    def __init__(self, logits_output=None, next_token_ids=None, can_run_cuda_graph=False, **kw):
        self.logits_output = logits_output
        self.next_token_ids = next_token_ids
        self.can_run_cuda_graph = can_run_cuda_graph


class LogitsProcessorOutput:
    def __init__(self, next_token_logits=None, **kw):
        self.next_token_logits = next_token_logits


class TpModelWorker:
    def __init__(self, server_args, gpu_id=0, nccl_port=0, model_config=None):
        self.server_args, self.gpu_id, self.nccl_port, self.model_config = server_args, gpu_id, nccl_port, model_config
        self.enable_overlap = not getattr(server_args, "disable_overlap_schedule", False)
        self._init_model_runner()


class ModelRunner:
    def __init__(self, model_config=None, mem_fraction_static=0.9, gpu_id=0, nccl_port=0, server_args=None):
        self.model_config, self.mem_fraction_static, self.gpu_id = model_config, mem_fraction_static, gpu_id
        self.nccl_port, self.server_args = nccl_port, server_args
        self.initialize()

    def initialize(self):
        raise AssertionError("the plugin replaces initialize")


class ReqToTokenPool:
    def __init__(self, size, max_context_len, device, enable_memory_saver):
        import torch

        self.size, self.max_context_len, self.device = size, max_context_len, device
        self.req_to_token = torch.zeros(size, max_context_len, dtype=torch.int32)
        self.free_slots = list(range(size))

    def free_rows(self, indices):
        self.free_slots.extend(int(i) for i in indices)

    def clear(self):
        self.free_slots = list(range(self.size))


class KVCache:
    def __init__(self, size, page_size, dtype, layer_num, device, enable_memory_saver, start_layer=None,
                 end_layer=None):
        self.size, self.page_size, self.dtype, self.layer_num = size, page_size, dtype, layer_num
        self.device, self.start_layer, self.end_layer = device, start_layer, end_layer


class PagedTokenToKVPoolAllocator:
    def __init__(self, size, page_size, dtype, device, kvcache, need_sort):
        self.size, self.page_size, self.dtype, self.device, self.kvcache = size, page_size, dtype, device, kvcache


class HostKVCache:
    def __init__(self, *, dtype, device_capacity_tokens, size_per_token, start_layer, end_layer,
                 host_to_device_ratio, host_size, page_size, layout, pin_memory, device):
        tokens = (host_size * 10**9 // size_per_token if host_size else
                  int(device_capacity_tokens * host_to_device_ratio))
        self.size = tokens // page_size * page_size
        self.page_size, self.layout = page_size, layout
        self.kv_buffer = self.init_kv_buffer()


class EmbeddingPoolerOutput:
    def __init__(self, embeddings):
        self.embeddings = embeddings


class BaseSpecWorker:
    def __init__(self):
        pass


class NgramVerifyInput:
    def __init__(self, draft_token_num, new_seq_lens, accept_tokens, accept_lens):
        self.draft_token_num, self.new_seq_lens = draft_token_num, new_seq_lens
        self.accept_tokens, self.accept_lens = accept_tokens, accept_lens


class HookType:
    REPLACE, BEFORE, AFTER, AROUND = "replace", "before", "after", "around"


class HookRegistry:
    installed: list = []

    @classmethod
    def register(cls, target, function, kind):
        cls.installed.append((target, function, kind))


MODULES = {
    "sglang.srt.managers.utils": {"GenerationBatchResult": GenerationBatchResult},
    "sglang.srt.layers.logits_processor": {"LogitsProcessorOutput": LogitsProcessorOutput},
    "sglang.srt.managers.tp_worker": {"TpModelWorker": TpModelWorker},
    "sglang.srt.model_executor.model_runner": {"ModelRunner": ModelRunner},
    "sglang.srt.mem_cache.memory_pool": {"ReqToTokenPool": ReqToTokenPool, "KVCache": KVCache},
    "sglang.srt.mem_cache.allocator": {"PagedTokenToKVPoolAllocator": PagedTokenToKVPoolAllocator},
    "sglang.srt.mem_cache.pool_host": {"HostKVCache": HostKVCache},
    "sglang.srt.layers.pooler": {"EmbeddingPoolerOutput": EmbeddingPoolerOutput},
    "sglang.srt.plugins.hook_registry": {"HookRegistry": HookRegistry, "HookType": HookType},
    "sglang.srt.speculative.base_spec_worker": {"BaseSpecWorker": BaseSpecWorker},
    "sglang.srt.speculative.ngram_info": {"NgramVerifyInput": NgramVerifyInput},
}


def install(monkeypatch) -> None:
    """Puts the stand-in modules (and their parent packages) into sys.modules and clears the
    plugin's caches of classes made over SGLang's, for the duration of one test."""
    from furiosa_opt_sglang import hicache, pools, speculative, steps, worker

    HookRegistry.installed = []
    for name, members in MODULES.items():
        parts = name.split(".")
        for i in range(1, len(parts)):
            parent = ".".join(parts[:i])
            if parent not in sys.modules:
                monkeypatch.setitem(sys.modules, parent, types.ModuleType(parent))
        mod = types.ModuleType(name)
        for k, v in members.items():
            setattr(mod, k, v)
        monkeypatch.setitem(sys.modules, name, mod)
    monkeypatch.setattr(steps, "_classes", {})
    monkeypatch.setattr(worker, "_made", {})
    monkeypatch.setattr(pools, "_made", {})
    monkeypatch.setattr(hicache, "_made", {})
    monkeypatch.setattr(speculative, "_made", {})
