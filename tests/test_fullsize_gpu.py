"""Parity at the benchmark's full sizes (the
north-star shape and the reference harness's head_dim-256 shape), through
the public API: one whole step (cache write of the
step's tokens, decode, split merge) over the full resident workload, then
the oracle on a sample of it -- a few sequences, each with a couple of KV
heads, dequantised from the very bytes the write kernel left in the cache.
Size-independent properties ride along: the full batch of outputs is
finite, a second step with the same inputs reproduces the first bit for bit
(the kernels are deterministic), and every output row -- all sequences, all
heads -- agrees with the CUDA-core kernel's (exact fp32 arithmetic, itself
checked against the oracle at small sizes) on the same cache, so a fault in
any work item or head shows, not only in the sampled ones. That comparison
runs both kernels with fp32 outputs at the fp32 tolerance: two bf16 results
may sit one bf16 ulp apart (0.03 at |o| = 4, which the V outliers reach)
when their fp32 values straddle a rounding boundary.
"""

import math

import numpy as np
import pytest
import torch

from oracle.attention import decode_attention, dequant_pool
from tests.helpers import assert_close_bf16, assert_close_fp32

pytestmark = pytest.mark.gpu


def _sampled_reference(wl, seqs, heads):
    """Oracle output (q_len rows x h_r query heads per sampled (seq, head))."""
    PS, d, h_r, ql = wl.PS, wl.d, wl.h_q // wl.h_k, wl.q_len
    bt = wl.block_table.cpu()
    out = {}
    for s in seqs:
        L = wl.lens[s]
        nb = math.ceil(L / PS)
        pages = bt[s, :nb].long()
        for h in heads:
            kb = wl.k_view[pages.to(wl.k_view.device)][:, :, h : h + 1].cpu()
            vb = wl.v_view[pages.to(wl.v_view.device)][:, :, h : h + 1].cpu()
            ks = vs = None
            if wl.fmt == "nvfp4":
                ks = wl.k_scales[pages.to(wl.k_scales.device)][:, :, h : h + 1].cpu()
                vs = wl.v_scales[pages.to(wl.v_scales.device)][:, :, h : h + 1].cpu()
            kv = dequant_pool(kb, wl.fmt, d, ks)
            vv = dequant_pool(vb, wl.fmt, d, vs)
            q = wl.query[s * ql : (s + 1) * ql, h * h_r : (h + 1) * h_r].cpu()
            qm = None if wl.q_mul is None else wl.q_mul[h * h_r : (h + 1) * h_r].cpu()
            om = None if wl.o_mul is None else wl.o_mul[h * h_r : (h + 1) * h_r].cpu()
            kd = wl.kd.reshape(-1)[min(h, wl.kd.numel() - 1)].item()
            vd = wl.vd.reshape(-1)[min(h, wl.vd.numel() - 1)].item()
            ref, _ = decode_attention(q, kv, vv, torch.arange(nb).view(1, nb), [L], 1, ql, wl.scale,
                                      k_descale=kd, v_descale=vd, causal=True, q_mul=qm, o_mul=om)
            out[(s, h)] = ref
    return out


@pytest.mark.parametrize("workload,kv", [("cfg2", "fp8"), ("cfg3", "e2m3"), ("ns", "e2m3"), ("cfg4", "e2m3"),
                                         ("cfg5", "e2m3"), ("cfg5", "fp8"), ("ns", "e3m2"), ("ns", "e2m1"), ("ns", "nvfp4"),
                                         ("hd256", "fp8"), ("hd256", "e2m3"), ("hd256", "nvfp4")])
def test_full_size_step_sampled_parity(workload, kv):
    import bench

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    wl = bench.Workload(workload, kv, 0, 1, dev)
    try:
        _check(wl, workload, kv)
    finally:
        del wl
        torch.cuda.empty_cache()


def _check(wl, workload, kv):
    from mjolnir_b200 import kvfp6

    outs = []
    for _ in range(2):
        kvfp6.reshape_and_cache(wl.new_k, wl.new_v, wl.k_view, wl.v_view, wl.slots, wl.k_scale, wl.v_scale, wl.fmt,
                                k_scales=wl.k_scales, v_scales=wl.v_scales)
        wl.runner.run(wl.plan, wl.query, wl.out, wl.k_view, wl.v_view, wl.kd, wl.vd, wl.scale, k_scales=wl.k_scales,
                      v_scales=wl.v_scales,
                      q_mul=wl.q_mul, o_mul=wl.o_mul)
        torch.cuda.synchronize()
        wl.runner.check_status()
        outs.append(wl.out.clone())
    assert torch.isfinite(outs[0].float()).all()
    assert torch.equal(outs[0], outs[1]), "a repeated step must reproduce its output"
    # the whole batch against the CUDA-core kernel on the same bytes
    from mjolnir_b200.runner import DecodeRunner

    simt = DecodeRunner(num_heads=wl.h_q, num_kv_heads=wl.h_k, head_size=wl.d, page_size=wl.PS, max_num_seqs=wl.b,
                        max_q_len=wl.q_len, kv_format=wl.fmt, device=wl.device, kernel="simt")
    plan = simt.plan(wl.lens, wl.b, wl.q_len, wl.block_table, wl.seq_lens)
    f32 = {}
    for name, r, p in (("tc", wl.runner, wl.plan), ("simt", simt, plan)):
        f32[name] = torch.empty(wl.out.shape, dtype=torch.float32, device=wl.device)
        r.run(p, wl.query, f32[name], wl.k_view, wl.v_view, wl.kd, wl.vd, wl.scale, k_scales=wl.k_scales,
              v_scales=wl.v_scales, q_mul=wl.q_mul, o_mul=wl.o_mul)
        torch.cuda.synchronize()
        r.check_status()
    assert_close_fp32(f32["tc"], f32["simt"], what=f"{workload}/{kv}: every row vs the CUDA-core kernel")
    assert_close_bf16(outs[0], f32["tc"], what=f"{workload}/{kv}: the bf16 step vs its fp32 output")
    del f32
    rng = np.random.default_rng(7)
    b = len(wl.lens)
    seqs = sorted({0, b // 2, b - 1, int(rng.integers(0, b))})
    heads = sorted({0, wl.h_k // 2, wl.h_k - 1})
    ref = _sampled_reference(wl, seqs, heads)
    h_r, ql, d = wl.h_q // wl.h_k, wl.q_len, wl.d
    got = wl.out.view(wl.T, wl.h_q, d)
    for (s, h), r in ref.items():
        g = got[s * ql : (s + 1) * ql, h * h_r : (h + 1) * h_r]
        assert_close_bf16(g, r, what=f"{workload}/{kv} seq {s} (L {wl.lens[s]}) head {h}")
