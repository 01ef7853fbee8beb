"""Quantize-on-write parity on the B200: cache bytes bit-exact vs the oracle
(which is pinned to the reference quantizer over every bf16 value)."""

import numpy as np
import pytest
import torch

from oracle import quant
from tests.helpers import LAYOUT_SHAPES

pytestmark = pytest.mark.gpu


def _write(key, value, fmt, layout, num_pages, PS, slots, ks, vs):
    from mjolnir_b200 import kvfp6
    from mjolnir_b200.runner import split_kv_cache

    T, h_k, d = key.shape
    from mjolnir_b200.runner import row_bytes

    rb = row_bytes(d, fmt)
    cache = torch.full(LAYOUT_SHAPES[layout](num_pages, PS, h_k, rb), 0xA5, dtype=torch.uint8, device="cuda")
    kv, vv = split_kv_cache(cache, layout, rb)
    kvfp6.reshape_and_cache(key, value, kv, vv, slots.cuda(), ks.cuda(), vs.cuda(), fmt)
    torch.cuda.synchronize()
    return kv.cpu(), vv.cpu()


def _check(kv, vv, key, value, slots, ks, vs, fmt, PS):
    qf = quant.quantize_rows_fp8 if fmt == "fp8" else (lambda x, sc: quant.quantize_rows_narrow(x, sc, fmt))
    ref_k = qf(key.float().cpu().numpy(), ks.numpy())
    ref_v = qf(value.float().cpu().numpy(), vs.numpy())
    written = set()
    for t, slot in enumerate(slots.tolist()):
        if slot < 0:
            continue
        blk, off = divmod(slot, PS)
        written.add(slot)
        np.testing.assert_array_equal(kv[blk, off].numpy(), ref_k[t], err_msg=f"K row {t}")
        np.testing.assert_array_equal(vv[blk, off].numpy(), ref_v[t], err_msg=f"V row {t}")
    for slot in range(kv.shape[0] * PS):
        if slot not in written:
            blk, off = divmod(slot, PS)
            assert (kv[blk, off] == 0xA5).all() and (vv[blk, off] == 0xA5).all(), "wrote a slot it was not given"


@pytest.mark.parametrize("fmt", ["fp8", "e2m3", "e3m2", "e2m1"])
@pytest.mark.parametrize("layout", ["BHN2D", "B2NHD", "2BHND"])
def test_random_rows_all_scale_modes(fmt, layout):
    g = torch.Generator().manual_seed(11)
    h_k, d, PS, T, P = 4, 256, 16, 37, 6
    key = (torch.randn(T, h_k, d, generator=g) * 3).to(torch.bfloat16)
    value = (torch.randn(T, h_k, d, generator=g) * 0.3).to(torch.bfloat16)
    slots = torch.randperm(P * PS, generator=g)[:T].to(torch.int64)
    slots[[3, 17]] = -1
    for ks, vs in (
        (torch.tensor([0.5, 0.4, 0.7, 0.45]), torch.tensor([0.05])),
        (torch.rand(h_k, d, generator=g) * 0.2 + 0.01, torch.rand(h_k, d, generator=g) + 0.1),
    ):
        kv, vv = _write(key.cuda(), value.cuda(), fmt, layout, P, PS, slots, ks, vs)
        _check(kv, vv, key, value, slots, ks, vs, fmt, PS)


@pytest.mark.parametrize("fmt", ["fp8", "e2m3", "e3m2", "e2m1"])
def test_every_bf16_value(fmt):
    """All 65536 bf16 bit patterns (NaN, inf, subnormals, ties) through the kernel."""
    bits = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    x = bits.reshape(512, 1, 128)
    PS = 16
    slots = torch.arange(512, dtype=torch.int64)
    for s in (1.0, 0.37, 3.0):
        sc = torch.tensor([s])
        kv, vv = _write(x.cuda(), x.cuda(), fmt, "BHN2D", 512 // PS, PS, slots, sc, sc)
        qf = quant.quantize_rows_fp8 if fmt == "fp8" else (lambda x, sc: quant.quantize_rows_narrow(x, sc, fmt))
        ref = qf(x.float().numpy(), np.array([s], np.float32))
        got = kv.reshape(512, 1, -1).numpy()
        bad = np.nonzero((got != ref).any(axis=-1))[0]
        assert got.tobytes() == ref.tobytes(), f"scale {s}: {len(bad)} rows differ, first {bad[:4]}"


def test_fp16_and_fp32_sources_and_int32_slots():
    from mjolnir_b200 import kvfp6

    g = torch.Generator().manual_seed(3)
    h_k, d, PS, T, P = 2, 128, 32, 20, 2
    for dt in (torch.float16, torch.float32):
        key = torch.randn(T, h_k, d, generator=g).to(dt)
        slots = torch.randperm(P * PS, generator=g)[:T].to(torch.int32)
        ks = torch.tensor([0.3, 0.6])
        kv, vv = _write(key.cuda(), key.cuda(), "e2m3", "B2HND", P, PS, slots, ks, ks)
        _check(kv, vv, key, key, slots.to(torch.int64), ks, ks, "e2m3", PS)


def test_write_kv_reference_layout_and_decode_roundtrip():
    """write_kv on the reference's (B, H, N, 2*row) layout; decoding the bytes
    returns the quantized values (round trip within the e2m3 grid)."""
    from mjolnir_b200 import kvfp6

    g = torch.Generator().manual_seed(4)
    h_k, d, PS, T, P = 8, 128, 16, 64, 8
    x = torch.randn(T, h_k, d, generator=g)
    x = torch.where(torch.rand(x.shape, generator=g) < 0.01, x * 8, x).to(torch.bfloat16)
    s = x.float().abs().amax(0).clamp(min=1e-6) / 7.5
    cache = torch.zeros(P, h_k, PS, 2 * 96, dtype=torch.uint8, device="cuda")
    slots = torch.randperm(P * PS, generator=g)[:T].to(torch.int64).cuda()
    kvfp6.write_kv(x.cuda(), x.cuda(), cache, slots, s.cuda(), s.cuda())
    torch.cuda.synchronize()
    c = cache.cpu()
    for t, slot in enumerate(slots.tolist()):
        blk, off = divmod(slot, PS)
        ref = quant.quantize_rows_e2m3(x[t].float().numpy(), s.numpy())
        np.testing.assert_array_equal(c[blk, :, off, :96].numpy(), ref)
        back = quant.decode_rows_e2m3(c[blk, :, off, 96:].numpy(), d) * s.numpy()
        assert np.abs(back - x[t].float().numpy()).max() <= (s.numpy() * 0.25 + 1e-6).max()


def test_padding_only_and_bad_slot_flagged():
    from mjolnir_b200 import kvfp6

    key = torch.randn(4, 2, 128, dtype=torch.bfloat16, device="cuda")
    cache = torch.full((2, 2, 16, 256), 0xA5, dtype=torch.uint8, device="cuda")
    kv, vv = cache[..., :128].transpose(1, 2), cache[..., 128:].transpose(1, 2)
    one = torch.ones(1, device="cuda")
    kvfp6.reshape_and_cache(key, key, kv, vv, torch.full((4,), -1, dtype=torch.int64, device="cuda"), one, one, "fp8")
    torch.cuda.synchronize()
    assert (cache == 0xA5).all()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    kvfp6.reshape_and_cache(key, key, kv, vv, torch.tensor([0, 99, 1, 2], device="cuda"), one, one, "fp8", status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 1  # MJ_DEV_BAD_PAGE: slot 99 is past 2 pages of 16
