"""nvfp4 KV (e2m1 codes, one e4m3 scale per 16 elements, a global scale) on
the B200: the write kernel reproduces the reference quantizer's bytes (the
golden fixtures of quant.py:68-84), the page expansion gives the e4m3 values
the tensor cores multiply bit for bit, and the decode kernels match the
oracle. The page expansion of the other narrow formats is checked here too."""

import math

import numpy as np
import pytest
import torch

from oracle import quant
from tests.helpers import LAYOUT_SHAPES, Case, assert_close_fp32

pytestmark = pytest.mark.gpu

GOLDEN = __file__.rsplit("/", 1)[0] + "/golden/nvfp4.npz"


def _nvfp4_cache(P, PS, h_k, d, layout="BHN2D", fill=0xA5):
    """Code views in a vLLM layout plus group-scale views (K and V scale rows
    interleaved in one (P, PS, h_k, 2, d / 16) tensor)."""
    from mjolnir_b200.runner import split_kv_cache

    rb = d // 2
    cache = torch.full(LAYOUT_SHAPES[layout](P, PS, h_k, rb), fill, dtype=torch.uint8, device="cuda")
    kv, vv = split_kv_cache(cache, layout, rb)
    sc = torch.full((P, PS, h_k, 2, d // 16), fill, dtype=torch.uint8, device="cuda")
    return kv, vv, sc[:, :, :, 0], sc[:, :, :, 1]


def _write(x_k, x_v, gs_k, gs_v, slots, P, PS, layout="BHN2D"):
    from mjolnir_b200 import kvfp6

    T, h_k, d = x_k.shape
    kv, vv, ks, vs = _nvfp4_cache(P, PS, h_k, d, layout)
    kvfp6.reshape_and_cache(x_k.cuda(), x_v.cuda(), kv, vv, slots.cuda(), gs_k.cuda(), gs_v.cuda(), "nvfp4",
                            k_scales=ks, v_scales=vs)
    torch.cuda.synchronize()
    return kv.cpu().numpy(), vv.cpu().numpy(), ks.cpu().numpy(), vs.cpu().numpy()


@pytest.mark.parametrize("case", ["rand0", "rand1", "rand2", "bf16"])
def test_write_reproduces_reference_bytes(case):
    """Given the reference's global scale, the write kernel's codes and group
    scales equal the reference nvfp4_quantize's, byte for byte."""
    g = np.load(GOLDEN)
    x = torch.from_numpy(g[f"{case}__x"])  # (T, 8, 128) fp32
    gs = torch.tensor([g[f"{case}__gs"][0]], dtype=torch.float32)
    T, h_k, d = x.shape
    PS = 16
    P = (T + PS - 1) // PS
    slots = torch.arange(T, dtype=torch.int64)
    kv, vv, ks, vs = _write(x, x, gs, gs, slots, P, PS)
    codes = kv.reshape(P * PS, h_k, d // 2)[:T]
    scales = ks.reshape(P * PS, h_k, d // 16)[:T]
    np.testing.assert_array_equal(codes, g[f"{case}__codes"])
    np.testing.assert_array_equal(scales, g[f"{case}__sc"])
    np.testing.assert_array_equal(vv.reshape(P * PS, h_k, d // 2)[:T], codes)


@pytest.mark.parametrize("layout", ["BHN2D", "B2NHD", "2BHND"])
def test_write_per_head_scale_padding_and_untouched_slots(layout):
    g = torch.Generator().manual_seed(21)
    h_k, d, PS, T, P = 4, 256, 16, 41, 5
    key = torch.randn(T, h_k, d, generator=g) * 3
    key[2, 1, 32:48] = 0.0  # a zero group
    key[5, 0, 7] = 300.0  # an outlier
    value = (torch.randn(T, h_k, d, generator=g) * 0.01).to(torch.bfloat16)
    key = key.to(torch.bfloat16)
    slots = torch.randperm(P * PS, generator=g)[:T].to(torch.int64)
    slots[[4, 30]] = -1
    gs_k = torch.tensor([quant.nvfp4_global_scale(key[:, h].float().numpy()) for h in range(h_k)], dtype=torch.float32)
    gs_v = torch.tensor([quant.nvfp4_global_scale(value.float().numpy())], dtype=torch.float32)
    kv, vv, ks, vs = _write(key, value, gs_k, gs_v, slots, P, PS, layout)
    ref_k, ref_ks = quant.quantize_rows_nvfp4(key.float().numpy(), gs_k.double().numpy())
    ref_v, ref_vs = quant.quantize_rows_nvfp4(value.float().numpy(), gs_v.double().numpy())
    written = set()
    for t, slot in enumerate(slots.tolist()):
        if slot < 0:
            continue
        blk, off = divmod(slot, PS)
        written.add(slot)
        np.testing.assert_array_equal(kv[blk, off], ref_k[t], err_msg=f"K codes {t}")
        np.testing.assert_array_equal(ks[blk, off], ref_ks[t], err_msg=f"K scales {t}")
        np.testing.assert_array_equal(vv[blk, off], ref_v[t], err_msg=f"V codes {t}")
        np.testing.assert_array_equal(vs[blk, off], ref_vs[t], err_msg=f"V scales {t}")
    for slot in range(P * PS):
        if slot not in written:
            blk, off = divmod(slot, PS)
            for a in (kv, vv, ks, vs):
                assert (a[blk, off] == 0xA5).all(), "wrote a slot it was not given"


def _random_narrow_pool(fmt, P, N, H, d, g):
    bits = 4 if fmt in ("e2m1", "nvfp4") else 6
    codes = torch.randint(0, 1 << bits, (2, P, N, H, d), generator=g, dtype=torch.uint8).numpy()
    packed = quant.pack4(codes) if bits == 4 else quant.pack6(codes)
    sc = None
    if fmt == "nvfp4":
        sc = torch.randint(0, 256, (2, P, N, H, d // 16), generator=g, dtype=torch.uint8).numpy()
        sc[(sc & 0x7F) == 0x7F] = 0x3C  # a written cache holds no NaN scale
    return packed, sc


@pytest.mark.parametrize("fmt", ["e3m2", "e2m1", "nvfp4"])
@pytest.mark.parametrize("ratio", ["none", "head", "channel"])
def test_expand_other_formats_bit_exact(fmt, ratio):
    """Narrow -> e4m3 page expansion for e3m2, e2m1 and nvfp4 (whose bytes
    are then exactly the tensor cores' operand values), every code."""
    from mjolnir_b200 import kvfp6
    from mjolnir_b200.runner import row_bytes, split_kv_cache

    g = torch.Generator().manual_seed(8)
    P, N, H, d = 6, 16, 2, 128
    rb = row_bytes(d, fmt)
    packed, sc = _random_narrow_pool(fmt, P, N, H, d, g)
    cache = torch.zeros(LAYOUT_SHAPES["BHN2D"](P, N, H, rb), dtype=torch.uint8, device="cuda")
    kv, vv = split_kv_cache(cache, "BHN2D", rb)
    kv.copy_(torch.from_numpy(packed[0]))
    vv.copy_(torch.from_numpy(packed[1]))
    ks = vs = None
    if fmt == "nvfp4":
        scd = torch.from_numpy(np.ascontiguousarray(np.moveaxis(sc, 0, 3))).cuda()  # (P, N, H, 2, d/16)
        ks, vs = scd[:, :, :, 0], scd[:, :, :, 1]
    src = torch.tensor([2, 5, 0, 2, 4], dtype=torch.int32)
    rk = rv = None
    if ratio == "head":
        rk, rv = torch.rand(H, generator=g) * 2, torch.rand(H, generator=g) * 90
    elif ratio == "channel":
        rk, rv = torch.rand(H, d, generator=g) * 3, torch.rand(H, d, generator=g) * 80
    out = torch.full(LAYOUT_SHAPES["B2NHD"](len(src), N, H, d), 0x5A, dtype=torch.uint8, device="cuda")
    ok, ov = split_kv_cache(out, "B2NHD", d)
    kvfp6.expand_pages(kv, vv, src.cuda(), ok, ov, None if rk is None else rk.cuda(), None if rv is None else rv.cuda(),
                       kv_format=fmt, k_scales=ks, v_scales=vs)
    torch.cuda.synchronize()
    ok, ov = ok.cpu().numpy(), ov.cpu().numpy()
    for j, p in enumerate(src.tolist()):
        for side, got, r in ((0, ok, rk), (1, ov, rv)):
            ref = quant.expand_rows_e4m3(packed[side, p], d, None if r is None else r.numpy(), fmt=fmt,
                                         sc=None if sc is None else sc[side, p])
            np.testing.assert_array_equal(got[j], ref, err_msg=f"{fmt} out page {j} side {side}")


def _kernel_of(c, **kw):
    from mjolnir_b200 import _lib

    r = c.runner(**kw)
    plan = r.plan(c.seq_lens, c.b, c.q_len, c.block_table, c.seq_lens_t)
    out = torch.empty(c.b * c.q_len, c.h_q * c.d, device="cuda")
    args = r.decode_args(plan, c.query, out, c.k_view, c.v_view, c.dev(c.kd), c.dev(c.vd), 0.1,
                         k_scales=c.k_scales, v_scales=c.v_scales)
    return _lib.KERNEL_NAMES[_lib.decode_kernel(args)]


@pytest.mark.parametrize("kernel", ["simt", "auto"])
@pytest.mark.parametrize("layout", ["BHN2D", "B2NHD", "BHN2R", "2BHND"])
@pytest.mark.parametrize("q_len,h_q", [(1, 16), (1, 32), (1, 64), (3, 32), (8, 32)])
def test_decode_matches_oracle(kernel, layout, q_len, h_q):
    """Decode over an nvfp4 cache (descale gs * 2^3, per tensor as the
    reference harness passes it) against the fp32 oracle on the kernel values."""
    c = Case(seq_lens=(700, 1, 2049, 130, 33), q_len=q_len, h_q=h_q, h_k=4, kv_format="nvfp4", layout=layout,
             seed=13)
    kname = _kernel_of(c, kernel=kernel)
    assert kname == ("decode_simt" if kernel == "simt" else "decode_tc")
    # rows past each sequence's end inside its last page: NaN scale bytes and
    # the largest codes, which no kernel may let into the output
    for s, L in enumerate(c.seq_lens):
        blk, off = divmod(L, c.PS)
        if off:
            page = int(c.block_table_cpu[s, blk])
            for t in (c.k_scales, c.v_scales):
                t[page, off:] = 0x7F
            for t in (c.k_view, c.v_view):
                t[page, off:] = 0x77
    out, _, _ = c.run(kernel=kernel)
    ref, _ = c.oracle()
    T = c.b * c.q_len
    assert_close_fp32(out[:T].view(T, c.h_q, c.d), ref, what=f"nvfp4 {kname} {layout} q_len {q_len}")
    assert torch.isnan(out[T:]).all()  # rows past the batch untouched


def test_decode_after_write_round_trip():
    """Write rows with the kernel, decode them: the output equals the oracle
    on the bytes the write left (a whole step through the public API)."""
    from mjolnir_b200 import kvfp6
    from mjolnir_b200.runner import DecodeRunner

    g = torch.Generator().manual_seed(5)
    h_q, h_k, d, PS = 16, 2, 128, 16
    L = [300, 77]
    n_blocks = [math.ceil(x / PS) for x in L]
    P = sum(n_blocks) + 1
    bt = torch.zeros(len(L), max(n_blocks), dtype=torch.int32)
    perm = torch.randperm(P, generator=g).tolist()
    i = 0
    slots = []
    for s, nb in enumerate(n_blocks):
        bt[s, :nb] = torch.tensor(perm[i:i + nb])
        i += nb
        slots += [int(bt[s, t // PS]) * PS + t % PS for t in range(L[s])]
    T = len(slots)
    k = (torch.randn(T, h_k, d, generator=g)).to(torch.bfloat16)
    v = (torch.randn(T, h_k, d, generator=g)).to(torch.bfloat16)
    gs_k = torch.tensor([quant.nvfp4_global_scale(k.float().numpy())], dtype=torch.float32)
    gs_v = torch.tensor([quant.nvfp4_global_scale(v.float().numpy())], dtype=torch.float32)
    kv, vv, ks, vs = _nvfp4_cache(P, PS, h_k, d, "BHN2R", fill=0)
    kvfp6.reshape_and_cache(k.cuda(), v.cuda(), kv, vv, torch.tensor(slots).cuda(), gs_k.cuda(), gs_v.cuda(), "nvfp4",
                            k_scales=ks, v_scales=vs)
    q = torch.randn(len(L), h_q, d, generator=g).to(torch.bfloat16)
    r = DecodeRunner(num_heads=h_q, num_kv_heads=h_k, head_size=d, page_size=PS, max_num_seqs=len(L), max_q_len=1,
                     kv_format="nvfp4", device=torch.device("cuda"))
    sl = torch.tensor(L, dtype=torch.int32)
    plan = r.plan(L, len(L), 1, bt.cuda(), sl.cuda())
    out = torch.empty(len(L), h_q, d, device="cuda")
    kd, vd = (gs_k.double() * 8).float().cuda(), (gs_v.double() * 8).float().cuda()
    r.run(plan, q.cuda(), out, kv, vv, kd, vd, 1.0 / math.sqrt(d), k_scales=ks, v_scales=vs)
    torch.cuda.synchronize()
    r.check_status()
    from oracle import attention

    kvals = attention.dequant_pool(kv.cpu(), "nvfp4", d, ks.cpu())
    vvals = attention.dequant_pool(vv.cpu(), "nvfp4", d, vs.cpu())
    ref, _ = attention.decode_attention(q, kvals, vvals, bt, L, len(L), 1, 1.0 / math.sqrt(d), kd.cpu(), vd.cpu())
    assert_close_fp32(out, ref, what="nvfp4 write -> decode")
