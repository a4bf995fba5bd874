"""Worker of the vLLM KV-offload test: vLLM's LLM through the plugin with the engine's offloading
connector and a GPU cache too small to keep a prompt's blocks; the same prompt before and after
others evicted it, and the connector's block counts, go to a JSON file."""

import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "integrations", "furiosa-opt-vllm"))


def main() -> None:
    from vllm import LLM, SamplingParams
    from vllm.inputs import TokensPrompt

    from furiosa_opt_vllm import offload

    path, out, prompts = sys.argv[1], sys.argv[2], json.loads(sys.argv[3])
    llm = LLM(model=path, skip_tokenizer_init=True, gpu_memory_utilization=0.3, max_model_len=512,
              max_num_seqs=4, max_num_batched_tokens=512, enforce_eager=True, dtype="bfloat16",
              num_gpu_blocks_override=48, enable_prefix_caching=True,
              kv_transfer_config={"kv_connector": "FuriosaOffloadingConnector",
                                  "kv_connector_module_path": "furiosa_opt_vllm.offload", "kv_role": "kv_both",
                                  "kv_connector_extra_config": {"cpu_bytes_to_use": 64 << 20}})
    params = SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True, detokenize=False)
    first = llm.generate([TokensPrompt(prompt_token_ids=prompts[0])], params)
    for p in prompts[1:]:  # other prompts take the GPU blocks the first one cached
        llm.generate([TokensPrompt(prompt_token_ids=p)], params)
    again = llm.generate([TokensPrompt(prompt_token_ids=prompts[0])], params)
    with open(out, "w") as f:
        json.dump({"first": list(first[0].outputs[0].token_ids), "again": list(again[0].outputs[0].token_ids),
                   "stats": dict(offload.STATS)}, f)


if __name__ == "__main__":
    main()
