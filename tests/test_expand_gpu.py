"""e2m3 -> e4m3 page expansion (the fallback scratch) on the B200: output bytes
bit-exact vs the oracle for every code, every ratio mode, any source / output
layout, duplicated and permuted source pages; a bad source page is flagged and
its output page left untouched."""

import numpy as np
import pytest
import torch

from oracle import quant
from tests.helpers import LAYOUT_SHAPES

pytestmark = pytest.mark.gpu


def _pool(layout, P, N, H, d, g):
    """An e2m3 pool in ``layout`` holding random codes (all 64 appear)."""
    from mjolnir_b200.runner import split_kv_cache

    rb = d * 3 // 4
    codes = torch.randint(0, 64, (2, P, N, H, d), generator=g, dtype=torch.uint8)
    packed = quant.pack6(codes.numpy())  # (2, P, N, H, rb)
    cache = torch.zeros(LAYOUT_SHAPES[layout](P, N, H, rb), dtype=torch.uint8, device="cuda")
    kv, vv = split_kv_cache(cache, layout, rb)
    kv.copy_(torch.from_numpy(packed[0]))
    vv.copy_(torch.from_numpy(packed[1]))
    return cache, kv, vv, packed


def _expand(kv, vv, src, out_layout, n_out, ratio_k, ratio_v, status=None, fill=0x5A):
    from mjolnir_b200 import kvfp6
    from mjolnir_b200.runner import split_kv_cache

    _, N, H, rb = kv.shape
    d = rb * 4 // 3
    out = torch.full(LAYOUT_SHAPES[out_layout](n_out, N, H, d), fill, dtype=torch.uint8, device="cuda")
    ok, ov = split_kv_cache(out, out_layout, d)
    kvfp6.expand_pages(kv, vv, src.cuda(), ok, ov, ratio_k, ratio_v, status)
    torch.cuda.synchronize()
    return ok.cpu().numpy(), ov.cpu().numpy()


@pytest.mark.parametrize("src_layout,out_layout", [("BHN2D", "B2NHD"), ("BHN2R", "B2HND"), ("B2NHD", "BHN2D")])
@pytest.mark.parametrize("ratio", ["none", "tensor", "head", "channel"])
def test_expand_bit_exact(src_layout, out_layout, ratio):
    g = torch.Generator().manual_seed(5)
    P, N, H, d = 7, 16, 4, 128
    cache, kv, vv, packed = _pool(src_layout, P, N, H, d, g)
    src = torch.tensor([3, 0, 6, 3, 1, 5, 2, 4, 6], dtype=torch.int32)  # permuted, duplicated
    rk = rv = None
    if ratio == "tensor":
        rk, rv = torch.tensor([0.37]), torch.tensor([21.5])
    elif ratio == "head":
        rk, rv = torch.rand(H, generator=g) * 2, torch.rand(H, generator=g) * 90  # some products pass 448
    elif ratio == "channel":
        rk, rv = torch.rand(H, d, generator=g) * 3, torch.rand(H, d, generator=g) * 80
    ok, ov = _expand(kv, vv, src, out_layout, len(src), None if rk is None else rk.cuda(), None if rv is None else rv.cuda())
    for j, p in enumerate(src.tolist()):
        ref_k = quant.expand_rows_e4m3(packed[0, p], d, None if rk is None else rk.numpy())
        ref_v = quant.expand_rows_e4m3(packed[1, p], d, None if rv is None else rv.numpy())
        np.testing.assert_array_equal(ok[j], ref_k, err_msg=f"K out page {j}")
        np.testing.assert_array_equal(ov[j], ref_v, err_msg=f"V out page {j}")


def test_expand_values_exact_without_ratio():
    """No ratio: every e4m3 byte decodes to the e2m3 code's value."""
    g = torch.Generator().manual_seed(6)
    cache, kv, vv, packed = _pool("BHN2D", 2, 32, 2, 128, g)
    ok, ov = _expand(kv, vv, torch.tensor([1, 0], dtype=torch.int32), "B2NHD", 2, None, None)
    codes = quant.unpack6(packed[0, 1], 128)
    np.testing.assert_array_equal(quant.e4m3_table()[ok[0]], quant.e2m3_table()[codes])


def test_bad_source_page_flagged_and_skipped():
    g = torch.Generator().manual_seed(7)
    cache, kv, vv, packed = _pool("BHN2D", 3, 16, 2, 128, g)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    src = torch.tensor([2, 9, -1, 0], dtype=torch.int32)
    ok, ov = _expand(kv, vv, src, "B2NHD", 4, None, None, status=status)
    assert int(status.item()) == 1  # MJ_DEV_BAD_PAGE
    assert (ok[1] == 0x5A).all() and (ov[2] == 0x5A).all()
    np.testing.assert_array_equal(ok[3], quant.expand_rows_e4m3(packed[0, 0], 128))
