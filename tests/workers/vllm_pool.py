"""Worker of the vLLM pooling test: vLLM's LLM with runner "pooling" over a synthetic checkpoint
(with a word-level tokenizer, which vLLM's pooling front end opens) through the plugin; `embed`
writes each prompt's embedding, `classify` its label probabilities."""

import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "integrations", "furiosa-opt-vllm"))


def main() -> None:
    from vllm import LLM
    from vllm.inputs import TokensPrompt

    mode, path, out, prompts = sys.argv[1], sys.argv[2], sys.argv[3], json.loads(sys.argv[4])
    llm = LLM(model=path, runner="pooling", gpu_memory_utilization=0.3,
              max_model_len=1024, max_num_seqs=8, max_num_batched_tokens=1024, enforce_eager=True,
              dtype="bfloat16", num_gpu_blocks_override=256, enable_prefix_caching=False)
    inputs = [TokensPrompt(prompt_token_ids=p) for p in prompts]
    if mode == "embed":
        result = [list(o.outputs.embedding) for o in llm.embed(inputs)]
    else:
        result = [list(o.outputs.probs) for o in llm.classify(inputs)]
    with open(out, "w") as f:
        json.dump(result, f)


if __name__ == "__main__":
    main()
