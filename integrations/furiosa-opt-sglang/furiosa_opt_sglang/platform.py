"""The SGLang platform's checks: server arguments the plugin serves, refused with the option's
name otherwise (the reference's platform refusals:
integrations/furiosa-opt-sglang/furiosa_opt_sglang/platform.py)."""

from __future__ import annotations

from . import paging


class Refused(ValueError):
    def __init__(self, option: str, reason: str):
        super().__init__(f"{option}: {reason}")
        self.option = option
        self.reason = reason

    def __reduce__(self):
        return (Refused, (self.option, self.reason))


def check(tp_size: int = 1, pp_size: int = 1, dp_size: int = 1, page_size: int = 16,
          speculative: str | None = None, lora: bool = False, attn_cp_size: int = 1,
          kv_cache_dtype: str = "auto", sampling_backend: str | None = None, draft_model: str | None = None,
          draft_topk: int | None = None) -> None:
    if pp_size != 1:
        raise Refused("pp_size", "pipeline parallelism is not served; use tensor parallelism")
    if tp_size not in (1, 2, 4, 8):
        raise Refused("tp_size", f"{tp_size} GPUs; a replica runs on 1, 2, 4 or 8")
    if attn_cp_size != 1:
        raise Refused("attn_cp_size", "context parallelism is not served")
    if speculative:
        algorithm = str(speculative).upper()
        if algorithm not in ("NGRAM", "STANDALONE"):
            raise Refused("speculative_algorithm", f"{speculative}: the engine drafts by n-grams (NGRAM) or with a "
                          "draft model (STANDALONE); EAGLE and MTP drafts read the target's hidden rows")
        if algorithm == "STANDALONE" and not draft_model:
            raise Refused("speculative_draft_model_path", "STANDALONE drafting loads a draft model")
        if draft_topk not in (None, 1):
            raise Refused("speculative_eagle_topk", "verification runs one chain of drafts a request")
    if lora:
        raise Refused("enable_lora", "adapters are not served through this plugin")
    if kv_cache_dtype not in ("auto", "bfloat16"):
        raise Refused("kv_cache_dtype", "the engine caches keys and values in BF16")
    try:
        paging.check_page_size(page_size)
    except ValueError as e:
        raise Refused("page_size", str(e)) from None


# Request fields whose inputs the engine's calls do not take (token IDs only) or whose outputs they
# do not return (scores).
UNSERVED_INPUTS = ("input_embeds", "image_data", "video_data", "audio_data")


def validate_request(_manager, obj, *args, **kwargs) -> None:
    """Before SGLang's `TokenizerManager._validate_one_request`: refuse a request the plugin does
    not serve, naming the field."""
    for field in UNSERVED_INPUTS:
        if getattr(obj, field, None):
            raise Refused(field, "the engine's decoders take token IDs only")
    if getattr(obj, "return_logprob", False):
        raise Refused("return_logprob", "the engine's decoder calls return tokens, not scores")


class Platform:
    """The class SGLang's platform entry point names: CUDA devices, the plugin's checks."""

    device_name = "cuda"
    device_type = "cuda"

    @classmethod
    def check_server_args(cls, args) -> None:
        check(tp_size=getattr(args, "tp_size", 1), pp_size=getattr(args, "pp_size", 1),
              dp_size=getattr(args, "dp_size", 1), page_size=getattr(args, "page_size", 16) or 16,
              speculative=getattr(args, "speculative_algorithm", None),
              lora=bool(getattr(args, "enable_lora", False)),
              attn_cp_size=getattr(args, "attn_cp_size", 1) or 1,
              kv_cache_dtype=str(getattr(args, "kv_cache_dtype", "auto")),
              draft_model=getattr(args, "speculative_draft_model_path", None),
              draft_topk=getattr(args, "speculative_eagle_topk", None))
