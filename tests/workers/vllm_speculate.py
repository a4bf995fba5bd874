"""Worker of the vLLM speculative-decoding tests: vLLM's LLM with n-gram speculation, or with a
draft model (its checkpoint the fourth argument), through the plugin; writes the greedy
continuations and vLLM's draft counters to a JSON file."""

import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "integrations", "furiosa-opt-vllm"))


def main() -> None:
    from vllm import LLM, SamplingParams
    from vllm.inputs import TokensPrompt

    path, out, prompts = sys.argv[1], sys.argv[2], json.loads(sys.argv[3])
    draft = sys.argv[4] if len(sys.argv) > 4 else None
    spec = ({"method": "draft_model", "model": draft, "num_speculative_tokens": 3} if draft else
            {"method": "ngram", "num_speculative_tokens": 3, "prompt_lookup_max": 3, "prompt_lookup_min": 1})
    llm = LLM(model=path, skip_tokenizer_init=True, gpu_memory_utilization=0.3, max_model_len=1024,
              max_num_seqs=8, max_num_batched_tokens=1024, enforce_eager=True, dtype="bfloat16",
              num_gpu_blocks_override=256, enable_prefix_caching=False, disable_log_stats=False,
              speculative_config=spec)
    params = SamplingParams(temperature=0.0, max_tokens=24, ignore_eos=True, detokenize=False)
    outs = llm.generate([TokensPrompt(prompt_token_ids=p) for p in prompts], params)
    counters = {}
    try:
        for m in llm.get_metrics():
            if m.name.startswith("vllm:spec_decode_num_"):
                counters[m.name] = getattr(m, "value", None)
    except Exception:  # noqa: BLE001 - counters are informative only
        pass
    with open(out, "w") as f:
        json.dump({"tokens": [list(o.outputs[0].token_ids) for o in outs], "counters": counters}, f)


if __name__ == "__main__":
    main()
