"""The fp8 quantize-on-write against the op the reference calls for it.

The reference's backend writes fp8 K/V with vLLM's `reshape_and_cache_flash`
(`backend.py:474-483`); this repo's write kernel replaces that call. Here
both write the same bf16 rows, scales and slots into caches that start with
the same random bytes, and the caches must come out byte-identical: every
written slot (including values that saturate at +-448, infinities, NaN and
zeros of both signs), and every byte the padding slots (-1) leave alone.
Skipped when vLLM does not import.
"""

import importlib.util

import pytest
import torch

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(importlib.util.find_spec("vllm") is None, reason="needs vLLM"),
]


@pytest.mark.parametrize("k_scale,v_scale", [(1.0, 1.0), (0.37, 1.9), (0.0123, 57.0)])
def test_fp8_write_matches_vllm_reshape_and_cache_flash(k_scale, v_scale):
    import vllm._custom_ops as ops

    from mjolnir_b200 import kvfp6

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(11)
    T, h_k, d, PS, pages = 700, 8, 128, 16, 64
    key = (torch.randn(T, h_k, d, generator=g, device=dev) * 3).to(torch.bfloat16)
    value = (torch.randn(T, h_k, d, generator=g, device=dev) * 3).to(torch.bfloat16)
    # values far outside e4m3 after scaling, specials, tiny values
    key[0, 0, :4] = torch.tensor([1e4, -1e4, float("inf"), float("-inf")], dtype=torch.bfloat16)
    key[1, 0, :3] = torch.tensor([float("nan"), 0.0, -0.0], dtype=torch.bfloat16)
    value[2, 1, :4] = torch.tensor([3e-6, -3e-6, 1e-30, 448.0], dtype=torch.bfloat16)
    slots = torch.randperm(pages * PS, generator=torch.Generator().manual_seed(3))[:T].to(dev)
    slots[::37] = -1  # padding requests write nothing
    ks = torch.tensor([k_scale], dtype=torch.float32, device=dev)
    vs = torch.tensor([v_scale], dtype=torch.float32, device=dev)

    init = torch.randint(0, 256, (2, pages, PS, h_k, d), dtype=torch.uint8, generator=g, device=dev)
    ref_k, ref_v = init[0].clone(), init[1].clone()
    got_k, got_v = init[0].clone(), init[1].clone()
    ops.reshape_and_cache_flash(key, value, ref_k, ref_v, slots, "fp8", ks, vs)
    kvfp6.reshape_and_cache(key, value, got_k, got_v, slots, ks, vs, "fp8")
    torch.cuda.synchronize()
    for name, got, ref in (("K", got_k, ref_k), ("V", got_v, ref_v)):
        diff = (got != ref).nonzero()
        assert diff.numel() == 0, f"{name}: {diff.shape[0]} bytes differ, first at {diff[:4].tolist()}"
    # the padding slots' bytes are the initial ones in both
    written = torch.zeros(pages * PS, dtype=torch.bool, device=dev)
    written[slots[slots >= 0]] = True
    keep = ~written.view(pages, PS)
    assert torch.equal(got_k[keep], init[0][keep]) and torch.equal(got_v[keep], init[1][keep])
