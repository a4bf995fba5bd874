"""Worker of the vLLM sleep-mode test: greedy continuations before sleeping, after waking from
level 1 and level 2, and after reloading the weights; the GPU memory freed while asleep."""

import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "integrations", "furiosa-opt-vllm"))


def main() -> None:
    import torch
    from vllm import LLM, SamplingParams
    from vllm.inputs import TokensPrompt

    path, out, prompts = sys.argv[1], sys.argv[2], json.loads(sys.argv[3])
    llm = LLM(model=path, skip_tokenizer_init=True, gpu_memory_utilization=0.3, max_model_len=1024,
              max_num_seqs=8, max_num_batched_tokens=1024, enforce_eager=True, dtype="bfloat16",
              num_gpu_blocks_override=256, enable_prefix_caching=False, enable_sleep_mode=True)
    params = SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True, detokenize=False)

    def run():
        outs = llm.generate([TokensPrompt(prompt_token_ids=p) for p in prompts], params)
        return [list(o.outputs[0].token_ids) for o in outs]

    result = {"before": run()}
    awake_free = torch.cuda.mem_get_info()[0]
    llm.sleep(level=1)
    result["freed_level1"] = torch.cuda.mem_get_info()[0] - awake_free
    llm.wake_up()
    result["level1"] = run()
    llm.sleep(level=2)
    llm.wake_up(tags=["weights"])
    llm.wake_up(tags=["kv_cache"])
    result["level2"] = run()
    llm.collective_rpc("reload_weights")
    result["reloaded"] = run()
    with open(out, "w") as f:
        json.dump(result, f)


if __name__ == "__main__":
    main()
