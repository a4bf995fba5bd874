"""What the plugin serves, checked where vLLM parses its configuration and each request (the
reference's refusals: integrations/furiosa-opt-vllm/furiosa_opt_vllm/admission.py). A refusal
names the option and why, and vLLM reports it before any device work."""

from __future__ import annotations


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
SPECULATIVE_METHODS = ("ngram",)


# The engine's adapter slots a call holds and the rank every update holds (decoder.AdapterSpec).
LORA_SLOTS = 2
LORA_RANK = 32


def options(pipeline: int, tensor: int, speculative: str | None, lora: bool, kv_cache_dtype: str,
            prefill_context: int = 1, decode_context: int = 1, max_loras: int = 1,
            max_lora_rank: int = 16) -> None:
    """Engine-level options: parallelism, speculation (`speculative` is the speculative config's
    method, or None), adapters, cache precision."""
    if pipeline != 1:
        raise Refused("pipeline_parallel_size", "pipeline parallelism is not served; use tensor parallelism")
    if tensor not in CHIPS:
        raise Refused("tensor_parallel_size", f"{tensor} GPUs; a replica runs on 1, 2, 4 or 8")
    if prefill_context != 1 or decode_context != 1:
        raise Refused("context_parallel_size", "context parallelism is not served")
    if speculative is not None and speculative not in SPECULATIVE_METHODS:
        raise Refused("speculative_config",
                      f"method {speculative}: drafts come from n-gram prompt lookup (method 'ngram'); "
                      "draft models are not served")
    if lora:
        if max_loras > LORA_SLOTS:
            raise Refused("max_loras", f"{max_loras} adapters a step; an engine call holds {LORA_SLOTS}")
        if max_lora_rank > LORA_RANK:
            raise Refused("max_lora_rank", f"rank {max_lora_rank}; the engine serves ranks up to {LORA_RANK}")
        if tensor != 1:
            raise Refused("enable_lora", "adapters are served on one GPU a replica")
    if kv_cache_dtype not in ("auto", "bfloat16"):
        raise Refused("kv_cache_dtype", "the engine caches keys and values in BF16")


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
    ("thinking_token_budget", None),
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
