"""Worker of the vLLM LoRA test: greedy continuations of the same prompt with two PEFT adapters
and without any, in one batch, through the plugin."""

import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "integrations", "furiosa-opt-vllm"))


def main() -> None:
    from vllm import LLM, SamplingParams
    from vllm.inputs import TokensPrompt
    from vllm.lora.request import LoRARequest

    path, out, prompt, adapters = sys.argv[1], sys.argv[2], json.loads(sys.argv[3]), json.loads(sys.argv[4])
    llm = LLM(model=path, skip_tokenizer_init=True, gpu_memory_utilization=0.3, max_model_len=1024,
              max_num_seqs=8, max_num_batched_tokens=1024, enforce_eager=True, dtype="bfloat16",
              num_gpu_blocks_override=256, enable_prefix_caching=False, enable_lora=True, max_loras=2,
              max_lora_rank=32)
    params = SamplingParams(temperature=0.0, max_tokens=5, ignore_eos=True, detokenize=False)
    loras = [LoRARequest(f"lora{i}", i + 1, p) for i, p in enumerate(adapters)] + [None]
    outs = llm.generate([TokensPrompt(prompt_token_ids=prompt)] * len(loras), params, lora_request=loras)
    with open(out, "w") as f:
        json.dump([list(o.outputs[0].token_ids) for o in outs], f)


if __name__ == "__main__":
    main()
