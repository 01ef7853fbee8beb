"""One vLLM generation on the Mjolnir backend (run by tests/test_vllm_e2e_gpu.py).

    python tests/vllm_e2e.py <model_dir> <kv_cache_dtype> <scales.json> <calibrate 0|1> <out.json>

A 2-layer Qwen3-shaped model with random weights (``load_format="dummy"``,
no tokenizer) is served in process with ``--attention-backend CUSTOM``; the
script writes the generated token ids and the backend's step counters. With
calibrate = 1 (fp8 cache) it also writes the per-channel K/V amax of every
layer to the scales file, which a later fp6_e2m3 run loads.
"""

import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main() -> None:
    model_dir, kv, scales, calibrate, out_path = sys.argv[1:6]
    os.environ["VLLM_ENABLE_V1_MULTIPROCESSING"] = "0"  # engine in this process: the plugin below applies
    if calibrate == "1":
        os.environ["MJOLNIR_ATTN_KV_CALIBRATE"] = "1"
    else:
        os.environ.pop("MJOLNIR_ATTN_KV_CALIBRATE", None)
        os.environ["MJOLNIR_ATTN_KV_SCALES"] = scales
    import mjolnir_b200

    mjolnir_b200.register()
    from vllm import LLM, SamplingParams

    from mjolnir_b200 import backend, kvscales

    llm = LLM(
        model=model_dir,
        load_format="dummy",
        skip_tokenizer_init=True,
        attention_backend="CUSTOM",
        kv_cache_dtype=kv,
        block_size=16,
        max_model_len=4096,
        max_num_seqs=8,
        gpu_memory_utilization=0.25,
        seed=0,
    )
    prompts = [{"prompt_token_ids": [(7 * i + 13 * j) % 900 + 10 for j in range(300 + 97 * i)]} for i in range(4)]
    outs = llm.generate(prompts, SamplingParams(max_tokens=24, temperature=0.0, ignore_eos=True))
    if calibrate == "1":
        kvscales.dump(scales, model="qwen3-tiny-dummy")
    res = {"tokens": [list(o.outputs[0].token_ids) for o in outs], "stats": dict(backend.STATS)}
    with open(out_path, "w") as f:
        json.dump(res, f)


if __name__ == "__main__":
    main()
