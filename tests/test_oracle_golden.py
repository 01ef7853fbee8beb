"""Pin the CPU oracle to the reference's own outputs (tests/golden/*.npz)."""

import math
import os

import numpy as np
import pytest
import torch

from oracle import attention, quant
from tests.conftest import GOLDEN


def _load(name):
    return np.load(os.path.join(GOLDEN, name))


def _all_bf16_f32():
    return quant.bf16_to_f32(np.arange(65536, dtype=np.uint32).astype(np.uint16)).reshape(512, 1, 128)


def test_e2m3_exhaustive_bf16_matches_reference():
    g = _load("quant.npz")
    x = _all_bf16_f32()
    for name, s in (("s1", 1.0), ("s037", 0.37), ("s3", 3.0)):
        got = quant.quantize_rows_e2m3(x, np.array([s], np.float32))
        np.testing.assert_array_equal(got, g[f"e2m3_all_{name}"], err_msg=name)


def test_fp8_exhaustive_bf16_matches_reference():
    g = _load("quant.npz")
    x = _all_bf16_f32()
    for name, s in (("s1", 1.0), ("s037", 0.37), ("s3", 3.0)):
        got = quant.quantize_rows_fp8(x, np.array([s], np.float32))
        np.testing.assert_array_equal(got, g[f"fp8_all_{name}"], err_msg=name)


def test_quant_random_scale_modes_match_reference():
    g = _load("quant.npz")
    x = quant.bf16_to_f32(g["rand_head_x"].view(np.uint16))
    np.testing.assert_array_equal(quant.quantize_rows_e2m3(x, g["rand_head_s"]), g["rand_head_e2m3"])
    np.testing.assert_array_equal(quant.quantize_rows_fp8(x, g["rand_head_s"]), g["rand_head_fp8"])
    x = quant.bf16_to_f32(g["rand_chan_x"].view(np.uint16))
    np.testing.assert_array_equal(quant.quantize_rows_e2m3(x, g["rand_chan_s"]), g["rand_chan_e2m3"])
    x = quant.bf16_to_f32(g["cfg3_x"].view(np.uint16))
    np.testing.assert_array_equal(quant.quantize_rows_e2m3(x, g["cfg3_s"]), g["cfg3_e2m3"])
    np.testing.assert_array_equal(quant.decode_rows_e2m3(g["cfg3_e2m3"], 128), g["cfg3_decoded"])


def test_pack_roundtrip_and_table():
    t = quant.e2m3_table()
    assert t[31] == 7.5 and t[8] == 1.0 and t[1] == 0.125 and t[63] == -7.5
    codes = np.random.default_rng(0).integers(0, 64, size=(7, 3, 128), dtype=np.uint8)
    np.testing.assert_array_equal(quant.unpack6(quant.pack6(codes), 128), codes)
    assert quant.pack6(np.array([[1, 2, 3, 4]], np.uint8)).tolist() == [[0x81, 0x30, 0x10]]


def test_scale_mode_rule():
    assert quant.scale_mode(1, 8, 128) == 0
    assert quant.scale_mode(8, 8, 128) == 1
    assert quant.scale_mode(1, 1, 128) == 0
    assert quant.scale_mode(8 * 128, 8, 128) == 2
    assert quant.scale_mode(128, 1, 128) == 2


def _decode_case(g, name):
    ql, h_q, h_k, d, PS, causal, e2m3 = (int(v) for v in g[name + "__meta"])
    fmt = "e2m3" if e2m3 else "fp8"
    kv = attention.dequant_pool(g[name + "__k_bytes"], fmt, d)
    vv = attention.dequant_pool(g[name + "__v_bytes"], fmt, d)
    q = torch.from_numpy(quant.bf16_to_f32(g[name + "__q_bits"].view(np.uint16)))
    sl = g[name + "__seq_lens"]
    o, lse = attention.decode_attention(
        q, kv, vv, torch.from_numpy(g[name + "__block_table"]), sl, len(sl), ql, 1.0 / math.sqrt(d),
        g[name + "__k_descale"], g[name + "__v_descale"], causal=bool(causal),
    )
    return o, lse


def test_decode_oracle_matches_reference():
    g = _load("decode.npz")
    names = sorted({k.split("__")[0] for k in g.files})
    assert len(names) == 5
    for name in names:
        o, lse = _decode_case(g, name)
        ref = torch.from_numpy(g[name + "__o_ref"])
        err = (o - ref).abs().max().item()
        assert err < 2e-6, f"{name}: oracle vs reference max abs {err}"
        assert torch.isfinite(lse).all()


def test_merge_of_split_chunks_equals_whole():
    g = _load("decode.npz")
    name = "fp8_mtp4"
    ql, h_q, h_k, d, PS, causal, _ = (int(v) for v in g[name + "__meta"])
    kv = attention.dequant_pool(g[name + "__k_bytes"], "fp8", d)
    vv = attention.dequant_pool(g[name + "__v_bytes"], "fp8", d)
    q = torch.from_numpy(quant.bf16_to_f32(g[name + "__q_bits"].view(np.uint16)))
    bt = torch.from_numpy(g[name + "__block_table"])
    sl = g[name + "__seq_lens"]
    # one sequence (L = 257), split into key ranges by shrinking the visible
    # context is not expressible with seq_lens; instead merge two halves of the
    # heads' scores directly through merge_splits on synthetic partials.
    s = torch.randn(3, 5, 40)
    v = torch.randn(40, 7)
    p_whole = torch.softmax(s, -1) @ v
    parts_o, parts_l = [], []
    for sl_ in (slice(0, 13), slice(13, 29), slice(29, 40)):
        parts_o.append(torch.softmax(s[..., sl_], -1) @ v[sl_])
        parts_l.append(torch.logsumexp(s[..., sl_], -1))
    o, l = attention.merge_splits(torch.stack(parts_o), torch.stack(parts_l))
    assert torch.allclose(o, p_whole, atol=1e-5)
    assert torch.allclose(l, torch.logsumexp(s, -1), atol=1e-5)
    # an all-masked chunk carries no weight
    o2, _ = attention.merge_splits(
        torch.stack(parts_o + [torch.zeros_like(parts_o[0])]),
        torch.stack(parts_l + [torch.full_like(parts_l[0], -math.inf)]),
    )
    assert torch.allclose(o2, p_whole, atol=1e-5)
    o, _ = attention.decode_attention(q, kv, vv, bt, sl, len(sl), ql, 1.0 / math.sqrt(d), g[name + "__k_descale"], g[name + "__v_descale"])
    assert o.shape == (len(sl) * ql, h_q, d)


def test_empty_causal_rows_are_zero():
    """L < q_len: the first query tokens see no key -> O = 0, LSE = -inf."""
    h_q, h_k, d, PS = 4, 1, 128, 16
    kv = torch.randn(2, PS, h_k, d)
    q = torch.randn(3, h_q, d)
    o, lse = attention.decode_attention(q, kv, kv, torch.tensor([[0, 1]]), [2], 1, 3, 0.1)
    assert (o[0] == 0).all() and torch.isinf(lse[0]).all()
    assert torch.isfinite(lse[1:]).all()


@pytest.mark.parametrize("fmt", ["e3m2", "e2m1"])
def test_narrow_formats_bit_exact_on_every_bf16(fmt):
    """e3m2 and e2m1 (the reference harness's other narrow KV formats): the
    oracle's table and quantizer equal the reference's on every bf16 value."""
    g = np.load(os.path.join(GOLDEN, "narrow.npz"))
    np.testing.assert_array_equal(quant.minifloat_table(fmt), g[f"{fmt}_table"])
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    x = quant.bf16_to_f32(bits).reshape(512, 1, 128)
    for name, s in (("s1", 1.0), ("s037", 0.37), ("s3", 3.0)):
        got = quant.quantize_rows_narrow(x, np.float32(s), fmt)
        np.testing.assert_array_equal(got, g[f"{fmt}_all_{name}"], err_msg=f"{fmt} scale {s}")
        d = quant.decode_rows_narrow(got, 128, fmt)
        assert np.all(np.abs(d) <= quant.minifloat_table(fmt).max())


@pytest.mark.parametrize("case", ["rand0", "rand1", "rand2", "bf16"])
def test_nvfp4_matches_reference(case):
    """nvfp4: the oracle's codes, group scales, global scale, kernel e4m3
    values and descale equal the reference's nvfp4_quantize (quant.py:68-84)."""
    g = np.load(os.path.join(GOLDEN, "nvfp4.npz"))
    x = g[f"{case}__x"]
    codes, sc, gs, kern, desc = quant.nvfp4_quantize(x)
    assert gs == g[f"{case}__gs"][0] and desc == g[f"{case}__gs"][1]
    np.testing.assert_array_equal(quant.pack4(codes), g[f"{case}__codes"])
    np.testing.assert_array_equal(sc, g[f"{case}__sc"])
    np.testing.assert_array_equal(kern, g[f"{case}__kern"])
    # the write form (per-tensor gs) gives the same bytes, and decodes to the kernel values
    packed, sc2 = quant.quantize_rows_nvfp4(x, np.float64(gs))
    np.testing.assert_array_equal(packed, g[f"{case}__codes"])
    np.testing.assert_array_equal(sc2, sc)
    np.testing.assert_array_equal(quant.decode_rows_nvfp4(packed, sc2, x.shape[-1]), quant.decode_fp8(kern))
