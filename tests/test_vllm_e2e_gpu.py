"""vLLM serving a model on the Mjolnir backend, end to end (B200, vLLM 0.22).

Starts two real vLLM engines (a minute or two; skipped when vLLM does not
import, or with MJOLNIR_VLLM_E2E=0):
a 2-layer Qwen3-shaped model with random weights generates on an fp8 cache
with calibration on (the decode steps on the kernel, the prefill on the
FlashInfer fallback), then on the packed fp6_e2m3 cache with the scales that
calibration wrote (kernel decode, fallback prefill on the expanded e4m3
scratch). Each run is its own process. Both head sizes the kernel takes:
head_dim 128 (Qwen3's) and 256.
"""

import importlib.util
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))

CONFIG = {
    "architectures": ["Qwen3ForCausalLM"],
    "model_type": "qwen3",
    "hidden_size": 1024,
    "intermediate_size": 2048,
    "num_hidden_layers": 2,
    "num_attention_heads": 16,
    "num_key_value_heads": 8,
    "head_dim": 128,
    "vocab_size": 1024,
    "max_position_embeddings": 8192,
    "rms_norm_eps": 1e-6,
    "rope_theta": 1000000.0,
    "tie_word_embeddings": False,
    "torch_dtype": "bfloat16",
    "attention_bias": False,
    "hidden_act": "silu",
    "bos_token_id": 1,
    "eos_token_id": 2,
}


@pytest.mark.skipif(importlib.util.find_spec("vllm") is None or os.environ.get("MJOLNIR_VLLM_E2E") == "0",
                    reason="needs vLLM (and MJOLNIR_VLLM_E2E not 0)")
@pytest.mark.parametrize("head_dim", [128, 256])
def test_vllm_generates_on_the_kernel(tmp_path, head_dim):
    model = tmp_path / "qwen3-tiny"
    model.mkdir()
    (model / "config.json").write_text(json.dumps(dict(CONFIG, head_dim=head_dim)))
    scales = tmp_path / "scales.json"
    results = {}
    for kv, calibrate in (("fp8", "1"), ("fp6_e2m3", "0")):
        out = tmp_path / f"{kv}.json"
        proc = subprocess.run(
            [sys.executable, os.path.join(HERE, "vllm_e2e.py"), str(model), kv, str(scales), calibrate, str(out)],
            capture_output=True, text=True, timeout=1200,
        )
        assert proc.returncode == 0, f"{kv}: exit {proc.returncode}\n{proc.stdout[-3000:]}\n{proc.stderr[-6000:]}"
        results[kv] = json.loads(out.read_text())
        if calibrate == "1":
            doc = json.loads(scales.read_text())
            assert doc["format"] == "mjolnir.kv_scales/2" and len(doc["amax"]) == 2
    for kv, r in results.items():
        print(kv, r["stats"], r["tokens"][0][:8])
        assert all(len(t) == 24 for t in r["tokens"]), kv
        assert r["stats"]["kernel_steps"] > 0, f"{kv}: no decode step ran on the kernel ({r['stats']})"
        assert r["stats"]["fallback_steps"] > 0, f"{kv}: the prefill should run on the fallback ({r['stats']})"
