"""The vLLM boundary end to end on the B200: the builder's plan, the impl's
cache write (``do_kv_cache_update``) and kernel-step ``forward`` on a cache in
the layout vLLM 0.22 allocates for this backend, checked against the oracle
decode over the bytes the write produced. Both KV formats: fp8 with a
per-tensor scale, fp6 with per-channel scales folded into Q and O."""

import json
import math
import types

import numpy as np
import pytest
import torch

from oracle.attention import decode_attention, dequant_pool
from tests.helpers import assert_close_bf16

pytestmark = pytest.mark.gpu
vllm = pytest.importorskip("vllm")


def _setup(kv_cache_dtype, h_q, h_k, d, PS, spec_tokens, tmp_path, monkeypatch):
    import transformers.configuration_utils  # noqa: F401

    from mjolnir_b200 import kvdtype

    kvdtype.register()
    from mjolnir_b200 import backend, builder

    ns = types.SimpleNamespace
    cfg = ns(
        cache_config=ns(cache_dtype=kv_cache_dtype, block_size=PS),
        model_config=ns(dtype=torch.bfloat16, get_num_attention_heads=lambda pc: h_q),
        parallel_config=ns(decode_context_parallel_size=1, prefill_context_parallel_size=1),
        scheduler_config=ns(max_num_seqs=16),
        speculative_config=ns(num_speculative_tokens=spec_tokens) if spec_tokens else None,
    )
    spec = ns(head_size=d, head_size_v=d, block_size=PS, num_kv_heads=h_k, sliding_window=None)
    name = "model.layers.0.self_attn.attn"
    layer = torch.nn.Module()
    layer.num_heads, layer.layer_name = h_q, name
    layer._k_scale = torch.tensor([0.75], device="cuda")
    layer._v_scale = torch.tensor([1.25], device="cuda")
    layer._k_scale_float, layer._v_scale_float = 0.75, 1.25
    if kv_cache_dtype == "fp6_e2m3":
        g = np.random.default_rng(9)
        amax = {"k": (g.random((h_k, d)) * 4 + 0.5).tolist(), "v": (g.random((h_k, d)) * 2 + 0.5).tolist()}
        path = tmp_path / "scales.json"
        path.write_text(json.dumps({"format": "mjolnir.kv_scales/2", "model": "t", "tokens": 1, "amax": {name: amax}}))
        monkeypatch.setenv("MJOLNIR_ATTN_KV_SCALES", str(path))
    monkeypatch.setattr(backend, "layers_of", lambda c, n: {name: layer})
    b = object.__new__(builder.MjolnirMetadataBuilder)
    b._setup(spec, [name], cfg, torch.device("cuda"))
    impl = object.__new__(backend.MjolnirImpl)
    impl.kv_cache_dtype, impl._fp6 = kv_cache_dtype, kv_cache_dtype == "fp6_e2m3"
    impl._kv_layout, impl._layer_reason = None, None
    impl.num_kv_heads, impl.head_size, impl.scale = h_k, d, 1.0 / math.sqrt(d)
    impl.kv_sharing_target_layer_name = None
    shape = backend.MjolnirAttentionBackend.get_kv_cache_shape(64, PS, h_k, d, cache_dtype_str=kv_cache_dtype)
    return backend, b, impl, layer, shape


@pytest.mark.parametrize("kv_cache_dtype", ["fp8", "fp6_e2m3"])
@pytest.mark.parametrize("q_len", [1, 3])
def test_write_then_decode_through_the_impl(kv_cache_dtype, q_len, tmp_path, monkeypatch):
    h_q, h_k, d, PS = 16, 2, 128, 16
    backend, b, impl, layer, shape = _setup(kv_cache_dtype, h_q, h_k, d, PS, 2, tmp_path, monkeypatch)
    g = torch.Generator().manual_seed(21)
    lens = [1 + q_len + 37, 300, 129]
    B = len(lens)
    width = 20  # 3 x 20 of the 64 pages; 300 tokens need 19
    perm = torch.randperm(64, generator=g)[: B * width].to(torch.int32)
    bt = perm.reshape(B, width)
    cache = torch.zeros(shape, dtype=torch.uint8, device="cuda")
    # write every token of every sequence through the impl (prefill-sized write)
    toks = [(s, t) for s in range(B) for t in range(lens[s])]
    slots = torch.tensor([int(bt[s, t // PS]) * PS + t % PS for s, t in toks], dtype=torch.int64)
    key = torch.randn(len(toks), h_k, d, generator=g).to(torch.bfloat16)
    value = torch.randn(len(toks), h_k, d, generator=g).to(torch.bfloat16)
    impl.do_kv_cache_update(layer, key.cuda(), value.cuda(), cache, slots.cuda())
    # one decode step: q_len new tokens per sequence (already written above)
    T = B * q_len
    qsl = torch.arange(0, T + 1, q_len, dtype=torch.int32)
    cam = types.SimpleNamespace(
        num_reqs=B, num_actual_tokens=T, max_query_len=q_len, max_seq_len=max(lens),
        query_start_loc=qsl.cuda(), query_start_loc_cpu=qsl,
        seq_lens=torch.tensor(lens, dtype=torch.int32, device="cuda"),
        seq_lens_cpu_upper_bound=torch.tensor(lens, dtype=torch.int32),
        block_table_tensor=bt.cuda(), slot_mapping=torch.zeros(T, dtype=torch.int64, device="cuda"), causal=True,
    )
    md = b.build(0, cam)
    assert md.kernel_step
    q = torch.randn(T, h_q, d, generator=g).to(torch.bfloat16).cuda()
    out = torch.full((T, h_q * d), float("nan"), dtype=torch.bfloat16, device="cuda")
    ret = impl.forward(layer, q, None, None, cache, md, output=out)
    torch.cuda.synchronize()
    assert ret is out
    b.runner.check_status()
    k_view, v_view = impl.kv_views(cache, h_k, PS, d)
    fmt = "e2m3" if impl._fp6 else "fp8"
    kv_vals = dequant_pool(k_view.cpu(), fmt, d)
    vv_vals = dequant_pool(v_view.cpu(), fmt, d)
    if impl._fp6:
        st = layer._mjolnir_fp6
        ref, _ = decode_attention(q.cpu(), kv_vals, vv_vals, bt, lens, B, q_len, impl.scale,
                                  q_mul=st["k_mul"].cpu(), o_mul=st["v_mul"].cpu())
    else:
        ref, _ = decode_attention(q.cpu(), kv_vals, vv_vals, bt, lens, B, q_len, impl.scale,
                                  k_descale=layer._k_scale.cpu(), v_descale=layer._v_scale.cpu())
    assert_close_bf16(out.view(T, h_q, d), ref, what=f"{kv_cache_dtype} q_len={q_len}")
