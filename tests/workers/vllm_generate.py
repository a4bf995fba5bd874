"""Worker of the vLLM plugin test: vLLM's LLM over a synthetic checkpoint with the plugin's
platform; writes the greedy continuations to a JSON file."""

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
    tp = int(sys.argv[4]) if len(sys.argv) > 4 else 1
    llm = LLM(model=path, skip_tokenizer_init=True, gpu_memory_utilization=0.3, max_model_len=1024,
              max_num_seqs=8, max_num_batched_tokens=1024, enforce_eager=True, dtype="bfloat16",
              num_gpu_blocks_override=256, enable_prefix_caching=False, tensor_parallel_size=tp)
    params = SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True, detokenize=False)
    outs = llm.generate([TokensPrompt(prompt_token_ids=p) for p in prompts], params)
    with open(out, "w") as f:
        json.dump([list(o.outputs[0].token_ids) for o in outs], f)
    # A refused request: sampling with temperature.
    try:
        llm.generate([TokensPrompt(prompt_token_ids=prompts[0])], SamplingParams(temperature=0.8, max_tokens=2))
        refused = False
    except Exception as e:  # noqa: BLE001
        refused = "temperature" in str(e)
    with open(out + ".refused", "w") as f:
        json.dump(refused, f)


if __name__ == "__main__":
    main()
