"""What the plugin serves, checked where vLLM parses its configuration and each request (the
reference's refusals: integrations/furiosa-opt-vllm/furiosa_opt_vllm/admission.py). A refusal
names the option and why, and vLLM reports it before any device work.

Configuration options are a table (`CONTRACTS`): each entry names an option's path in vLLM's
configuration, a predicate on its value and the requirement a refusal states. Request parameters
are checked by `sampling` and `unmodified`."""

from __future__ import annotations

import dataclasses
import types
from typing import Callable


class Refused(ValueError):
    """An option or request the plugin does not serve."""

    def __init__(self, option: str, reason: str):
        super().__init__(f"{option}: {reason}")
        self.option = option
        self.reason = reason

    def __reduce__(self):
        return (Refused, (self.option, self.reason))


CHIPS = (1, 2, 4, 8)

# Speculative methods served: drafts the target verifies greedily (furiosa_opt_vllm.speculation).
SPECULATIVE_METHODS = ("ngram", "draft_model")

# The engine's adapter slots a call holds and the rank every update holds (decoder.AdapterSpec).
LORA_SLOTS = 2
LORA_RANK = 32

# Checkpoint quantization declarations the engine reads itself (block FP8, NVFP4).
QUANTIZATIONS = (None, "fp8", "modelopt_fp4", "modelopt", "compressed-tensors")

_ABSENT = object()


@dataclasses.dataclass(frozen=True)
class Contract:
    """One served-or-refused rule over vLLM's configuration.

    `path` names the option inside `VllmConfig` (dotted attributes); `served(value, config)` says
    whether its value is served; `requirement` is the reason a refusal gives. An option this vLLM
    does not have is skipped; `refuse_as` overrides the option name a refusal reports."""

    path: str
    served: Callable[[object, object], bool]
    requirement: str
    refuse_as: str | None = None

    def option(self) -> str:
        return self.refuse_as or self.path.rsplit(".", 1)[-1]


def _get(config, path: str):
    value = config
    for part in path.split("."):
        value = getattr(value, part, _ABSENT)
        if value is _ABSENT:
            return _ABSENT
    return value


def _tensor(config) -> int:
    v = _get(config, "parallel_config.tensor_parallel_size")
    return 1 if v is _ABSENT else int(v)


def _is(*allowed):
    return lambda v, _cfg: v in allowed


def _at_most(limit):
    return lambda v, _cfg: v is None or int(v) <= limit


def _unset(v, _cfg) -> bool:
    return not v


# Every option the plugin pins or refuses, checked in order when vLLM builds its configuration.
CONTRACTS: tuple[Contract, ...] = (
    # Parallelism: a replica is 1, 2, 4 or 8 GPUs of one node, tensor-parallel.
    Contract("parallel_config.pipeline_parallel_size", _is(1),
             "pipeline parallelism is not served; use tensor parallelism"),
    Contract("parallel_config.tensor_parallel_size", _is(*CHIPS), "a replica runs on 1, 2, 4 or 8 GPUs"),
    Contract("parallel_config.prefill_context_parallel_size", _is(1, None), "context parallelism is not served",
             refuse_as="context_parallel_size"),
    Contract("parallel_config.decode_context_parallel_size", _is(1, None), "context parallelism is not served",
             refuse_as="context_parallel_size"),
    Contract("parallel_config.nnodes", _is(1, None), "a replica runs on one node"),
    Contract("parallel_config.enable_eplb", _unset, "experts keep their placement (no expert load balancing)"),
    Contract("parallel_config.enable_elastic_ep", _unset, "expert parallelism follows the tensor-parallel ranks"),
    Contract("parallel_config.enable_dbo", _unset, "dual-batch overlap is not served; the engine overlaps "
             "communication inside its kernels"),
    # Speculation: n-gram drafts verified greedily.
    Contract("speculative_config", lambda v, _c: v is None or str(getattr(v, "method", None)) in SPECULATIVE_METHODS,
             "drafts come from n-gram prompt lookup (method 'ngram') or a draft model (method 'draft_model')"),
    Contract("speculative_config", lambda v, cfg: v is None or str(getattr(v, "method", None)) != "draft_model"
             or _tensor(cfg) == 1, "a draft model runs beside the target on one GPU a replica",
             refuse_as="speculative_config.method"),
    # LoRA: the engine's two slots, rank 32, one GPU a replica.
    Contract("lora_config.max_loras", _at_most(LORA_SLOTS), f"an engine call holds {LORA_SLOTS} adapters"),
    Contract("lora_config.max_lora_rank", _at_most(LORA_RANK), f"the engine serves ranks up to {LORA_RANK}"),
    Contract("lora_config.fully_sharded_loras", _unset, "adapters are not sharded"),
    Contract("lora_config", lambda v, cfg: v is None or _tensor(cfg) == 1, "adapters are served on one GPU a replica",
             refuse_as="enable_lora"),
    # Cache: BF16 keys and values in 16-token pages of the engine's layout.
    Contract("cache_config.cache_dtype", _is("auto", "bfloat16"), "the engine caches keys and values in BF16",
             refuse_as="kv_cache_dtype"),
    Contract("cache_config.calculate_kv_scales", _unset, "the BF16 cache takes no scales"),
    Contract("cache_config.kv_sharing_fast_prefill", _unset, "every layer keeps its own cache"),
    Contract("offload_config.uva.cpu_offload_gb", lambda v, _c: not v, "weights stay on the GPU",
             refuse_as="cpu_offload_gb"),
    Contract("offload_config.prefetch.offload_group_size", lambda v, _c: not v, "weights stay on the GPU",
             refuse_as="offload_group_size"),
    # Model: the checkpoint as published, BF16 compute, formats the engine reads.
    Contract("model_config.dtype", lambda v, _c: str(v).replace("torch.", "") in ("bfloat16", "auto"),
             "the engine computes in BF16"),
    Contract("model_config.quantization", _is(*QUANTIZATIONS),
             "the engine reads BF16, block FP8 and NVFP4 checkpoints as published"),
    Contract("model_config.hf_overrides", lambda v, _c: not v or isinstance(v, dict),
             "overrides are a mapping of config keys applied to config.json; a function of the config is not served"),
    Contract("model_config.enable_prompt_embeds", _unset, "requests carry token IDs"),
    Contract("model_config.enable_return_routed_experts", _unset, "routing stays on the device"),
    Contract("model_config.override_attention_dtype", _unset, "attention runs in BF16"),
    Contract("load_config.load_format", _is("auto", "safetensors"), "the engine loads safetensors checkpoints"),
    # Transfers: KV offloading to host memory through the plugin's connector, nothing else.
    Contract("ec_transfer_config", lambda v, cfg: v is None or (
        _get(cfg, "model_config.multimodal_config.mm_encoder_only") is True
        and bool(getattr(v, "is_ec_producer", False))),
             "encoder caches are produced only by a media-encoder instance (mm_encoder_only, an EC producer)"),
    Contract("kv_transfer_config.kv_connector", lambda v, _c: v in (None, "FuriosaOffloadingConnector"),
             "KV caches move only to host memory, through FuriosaOffloadingConnector"),
    Contract("kv_transfer_config.kv_load_failure_policy", _is("fail", None),
             "a failed load from host memory fails its requests (the offloaded memory is poisoned)"),
)


def check(config) -> None:
    """Runs every contract on vLLM's configuration; the first one broken is refused."""
    for c in CONTRACTS:
        value = _get(config, c.path)
        if value is _ABSENT:
            continue
        if not c.served(value, config):
            raise Refused(c.option(), f"{value!r} is not served: {c.requirement}")


def options(pipeline: int, tensor: int, speculative: str | None, lora: bool, kv_cache_dtype: str,
            prefill_context: int = 1, decode_context: int = 1, max_loras: int = 1,
            max_lora_rank: int = 16) -> None:
    """The contracts on the engine-level options alone (parallelism, speculation by method name,
    adapters, cache precision), for callers without a full vLLM configuration."""
    ns = types.SimpleNamespace
    check(ns(parallel_config=ns(pipeline_parallel_size=pipeline, tensor_parallel_size=tensor,
                                prefill_context_parallel_size=prefill_context,
                                decode_context_parallel_size=decode_context),
             speculative_config=None if speculative is None else ns(method=speculative),
             lora_config=ns(max_loras=max_loras, max_lora_rank=max_lora_rank) if lora else None,
             cache_config=ns(cache_dtype=kv_cache_dtype)))


def sampling(temperature: float, top_k: int, top_p: float, n: int, logprobs, prompt_logprobs,
             min_tokens: int = 0) -> None:
    """Request-level: the engine's head returns each row's first maximum (greedy decoding)."""
    if temperature > 0:
        raise Refused("temperature", "the engine decodes greedily; use temperature=0")
    if logprobs is not None or prompt_logprobs is not None:
        raise Refused("logprobs", "the engine returns tokens, not log-probabilities")
    if n != 1:
        raise Refused("n", "one sequence per request")


# Sampling parameters that change the distribution a token is drawn from, at their neutral values:
# the engine's head returns each row's first maximum of the unmodified logits, so a request that
# sets any of them is refused rather than answered with tokens that ignore it (the reference's
# greedy predicate: integrations/furiosa-opt-vllm/furiosa_opt_vllm/generation/__init__.py:125-142).
NEUTRAL = (
    ("repetition_penalty", 1.0),
    ("frequency_penalty", 0.0),
    ("presence_penalty", 0.0),
    ("min_tokens", 0),
    ("logit_bias", None),
    ("allowed_token_ids", None),
    ("bad_words", None),
    ("structured_outputs", None),
    ("logprob_token_ids", None),
    ("extra_args", None),
)


def unmodified(params) -> None:
    """Refuses a request whose parameters change the greedy token (penalties, biases, masks,
    grammars); empty lists and dicts count as unset."""
    for name, neutral in NEUTRAL:
        value = getattr(params, name, neutral)
        if neutral is None:
            if value:  # None, [] and {} leave the distribution alone
                raise Refused(name, "the engine returns each row's greedy token of the unmodified logits")
        elif value != neutral:
            raise Refused(name, "the engine returns each row's greedy token of the unmodified logits")
