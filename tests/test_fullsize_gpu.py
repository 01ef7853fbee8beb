"""Parity at the benchmark's full sizes (BASELINE configs 2-5 and the
north-star shape), through the public API: one whole step (cache write of the
step's tokens, decode, split merge) over the full resident workload, then
the oracle on a sample of it -- a few sequences, each with a couple of KV
heads, dequantised from the very bytes the write kernel left in the cache.
A size-independent property rides along: the full batch of outputs is
finite, and a second step with the same inputs reproduces the first bit for
bit (the kernels are deterministic).
"""

import math

import numpy as np
import pytest
import torch

from oracle.attention import decode_attention, dequant_pool
from tests.helpers import assert_close_bf16

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
                                         ("cfg5", "e2m3"), ("cfg5", "fp8"), ("ns", "e3m2"), ("ns", "e2m1"), ("ns", "nvfp4")])
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
    rng = np.random.default_rng(7)
    b = len(wl.lens)
    seqs = sorted({0, b - 1, int(rng.integers(0, b))})
    heads = sorted({0, wl.h_k - 1})
    ref = _sampled_reference(wl, seqs, heads)
    h_r, ql, d = wl.h_q // wl.h_k, wl.q_len, wl.d
    got = wl.out.view(wl.T, wl.h_q, d)
    for (s, h), r in ref.items():
        g = got[s * ql : (s + 1) * ql, h * h_r : (h + 1) * h_r]
        assert_close_bf16(g, r, what=f"{workload}/{kv} seq {s} (L {wl.lens[s]}) head {h}")
