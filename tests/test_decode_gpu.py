"""Decode parity on the B200: the CUDA path through the C ABI vs the CPU oracle
(pinned to the reference) and vs the reference's own outputs (golden)."""

import math
import os

import numpy as np
import pytest
import torch

from oracle import attention, quant
from tests.conftest import GOLDEN
from tests.helpers import Case, assert_close_bf16, assert_close_fp32

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _no_tensor_core_fallback():
    """Every shape the tensor-core kernel takes must find a variant whose
    register split fits the build: a call that silently ran the CUDA-core
    decode instead is counted by the library and fails the test."""
    from mjolnir_b200 import _lib

    before = _lib.load().mj_tc_fallbacks()
    yield
    assert _lib.load().mj_tc_fallbacks() == before, "a decode fell back to the CUDA-core kernel"


def test_golden_reference_outputs():
    """The kernel on the reference's own fixtures vs the reference's ref_decode output."""
    from mjolnir_b200.runner import DecodeRunner

    g = np.load(os.path.join(GOLDEN, "decode.npz"))
    names = sorted({k.split("__")[0] for k in g.files})
    for name in names:
        ql, h_q, h_k, d, PS, causal, e2m3 = (int(v) for v in g[name + "__meta"])
        fmt = "e2m3" if e2m3 else "fp8"
        kb = torch.from_numpy(g[name + "__k_bytes"]).cuda()
        vb = torch.from_numpy(g[name + "__v_bytes"]).cuda()
        sl = torch.from_numpy(g[name + "__seq_lens"]).to(torch.int32)
        bt = torch.from_numpy(g[name + "__block_table"]).to(torch.int32)
        b = len(sl)
        q = torch.from_numpy(g[name + "__q_bits"]).view(torch.bfloat16).cuda()
        kd = torch.from_numpy(g[name + "__k_descale"]).cuda()
        vd = torch.from_numpy(g[name + "__v_descale"]).cuda()
        kernels = ["simt"] + (["tc"] if (d == 128 and ql * h_q // h_k <= 16) or d == 256 else [])
        for sm, kernel in [(sm, k) for sm in (148, 2) for k in kernels]:  # 148 SMs: small batches split
            r = DecodeRunner(num_heads=h_q, num_kv_heads=h_k, head_size=d, page_size=PS, max_num_seqs=b,
                             max_q_len=ql, kv_format=fmt, sm_count=sm, kernel=kernel)
            plan = r.plan(sl.tolist(), b, ql, bt.cuda(), sl.cuda(), causal=bool(causal))
            out = torch.full((b * ql, h_q, d), float("nan"), dtype=torch.float32, device="cuda")
            r.run(plan, q, out, kb, vb, kd, vd, 1.0 / math.sqrt(d))
            torch.cuda.synchronize()
            r.check_status()
            ref = torch.from_numpy(g[name + "__o_ref"])
            assert_close_fp32(out, ref, what=f"{name} {kernel} sm={sm} splits={plan.with_reduction}")


def _kernel_of(c, **kw):
    from mjolnir_b200 import _lib

    r = c.runner(**kw)
    plan = r.plan(c.seq_lens, c.b, c.q_len, c.block_table, c.seq_lens_t)
    out = torch.empty(c.b * c.q_len, c.h_q * c.d, device="cuda")
    args = r.decode_args(plan, c.query, out, c.k_view, c.v_view, c.dev(c.kd), c.dev(c.vd), 0.1,
                         q_mul=c.dev(c.q_mul), o_mul=c.dev(c.o_mul), k_scales=c.k_scales, v_scales=c.v_scales)
    return _lib.KERNEL_NAMES[_lib.decode_kernel(args)]


@pytest.mark.parametrize("kv_format", ["fp8", "e2m3"])
@pytest.mark.parametrize("layout", ["BHN2D", "BNH2D", "B2NHD", "B2HND", "2BNHD", "2BHND"])
@pytest.mark.parametrize("kernel", ["simt", "auto"])
def test_layouts(kv_format, layout, kernel):
    c = Case(seq_lens=(300, 1, 2049, 128), h_q=16, h_k=2, kv_format=kv_format, layout=layout, seed=3)
    # every vLLM layout gives TMA-legal strides here (e2m3 rows are 96 B, a
    # multiple of the 32 B the 16U6 type needs)
    expect = "decode_simt" if kernel == "simt" else "decode_tc"
    assert _kernel_of(c, kernel=kernel) == expect
    out, _, _ = c.run(kernel=kernel)
    ref, _ = c.oracle()
    T = c.b * c.q_len
    assert_close_fp32(out[:T].view(T, c.h_q, c.d), ref, what=f"{kv_format}/{layout}")
    assert torch.isnan(out[T:]).all(), "wrote past the batch"


@pytest.mark.parametrize("kernel", ["simt", "tc"])
def test_config1_shape(kernel):
    """b 4, 8 q / 2 KV heads, d 128, PS 16, L ~ U[1, 2048], fp8 scale 1.0."""
    g = torch.Generator().manual_seed(1)
    lens = torch.randint(1, 2049, (4,), generator=g).tolist()
    c = Case(seq_lens=lens, h_q=8, h_k=2, kv_format="fp8", layout="B2NHD", seed=1)
    for out_dtype in (torch.float32, torch.bfloat16):
        out, lse, plan = c.run(out_dtype=out_dtype, lse=True, kernel=kernel)
        ref, ref_lse = c.oracle()
        T = c.b
        got = out[:T].view(T, c.h_q, c.d)
        if out_dtype == torch.float32:
            assert_close_fp32(got, ref, what="config1 fp32")
            assert torch.allclose(lse.cpu(), ref_lse, atol=1e-4, rtol=1e-5)
        else:
            assert_close_bf16(got, ref, what="config1 bf16")


@pytest.mark.parametrize("kv_format", ["fp8", "e2m3"])
@pytest.mark.parametrize("q_len,causal,h_q,kernel", [(4, True, 16, "simt"), (6, True, 16, "simt"), (3, False, 16, "simt"),
                                                     (4, True, 8, "tc"), (2, False, 16, "tc"), (3, True, 8, "tc"),
                                                     (6, True, 16, "tc"), (4, True, 16, "tc"), (3, False, 16, "tc")])
def test_mtp_rows(kv_format, q_len, causal, h_q, kernel):
    c = Case(seq_lens=(q_len, 700, 1500, 33), q_len=q_len, h_q=h_q, h_k=2, kv_format=kv_format, seed=5,
             descale="head" if kv_format == "fp8" else "tensor", layout="BHN2D")
    out, _, _ = c.run(causal=causal, kernel=kernel)
    ref, _ = c.oracle()
    T = c.b * q_len
    assert_close_fp32(out[:T].view(T, c.h_q, c.d), ref, what=f"mtp q_len {q_len}")


@pytest.mark.parametrize("sm_count", [148, 4])
@pytest.mark.parametrize("kernel", ["simt", "tc"])
def test_split_and_unsplit_agree(sm_count, kernel):
    """Small sm_count: no split; 148 SMs with 3 sequences: every sequence splits."""
    c = Case(seq_lens=(5000, 3000, 129), h_q=32, h_k=8, kv_format="e2m3", seed=7, outliers=0.01, layout="BHN2D")
    out, _, plan = c.run(sm_count=sm_count, kernel=kernel)
    assert plan.with_reduction == (sm_count == 148)
    ref, _ = c.oracle()
    T = c.b
    assert_close_fp32(out[:T].view(T, c.h_q, c.d), ref, what=f"sm {sm_count}")


@pytest.mark.parametrize("kv_format", ["fp8", "e2m3"])
@pytest.mark.parametrize("q_len,h_q", [(1, 8), (2, 8), (3, 4), (1, 32), (3, 16), (6, 16), (8, 16), (5, 16)])
def test_tc_rescale_in_later_tiles(kv_format, q_len, h_q):
    """Scores that grow along the sequence make the running max rise after the
    first tile, so O accumulated in TMEM is rescaled in place. Row counts
    cover the one-warpgroup (4, 8, 16 rows; 6 with padding rows), two- and
    three-warpgroup (24, 48 rows, 40 with padding rows) and row-group (64
    rows) variants."""
    c = Case(seq_lens=(2000, 700, 1290), q_len=q_len, h_q=h_q, h_k=2, kv_format=kv_format, layout="BHN2D",
             seed=43 + q_len, k_ramp=2.5)
    out, _, _ = c.run(kernel="tc", sm_count=8)  # few slots: long chunks, many tiles per job
    ref, _ = c.oracle()
    T = c.b * q_len
    assert_close_fp32(out[:T].view(T, c.h_q, c.d), ref, what=f"rescale {kv_format} n_q {q_len * h_q // 2}")


@pytest.mark.parametrize("kv_format", ["fp8", "e2m3"])
@pytest.mark.parametrize("q_len,h_q", [(1, 8), (2, 16), (4, 16)])
def test_tc_in_kernel_merge_matches_combine_launch(kv_format, q_len, h_q):
    """Split sequences: the last job of each (sequence, KV head) merges the
    partials inside the decode launch; the result equals the separate merge
    launch and the oracle, and stays right on a second launch (the counters
    return to zero)."""
    c = Case(seq_lens=(5000, 3000, 129, 900), q_len=q_len, h_q=h_q, h_k=2, kv_format=kv_format,
             layout="BHN2D", seed=51 + q_len)
    ref, _ = c.oracle()
    T = c.b * q_len
    outs = {}
    for fused in (True, False):
        for rep in range(2):
            out, lse, plan = c.run(kernel="tc", fused_merge=fused, lse=True)
            assert plan.with_reduction
            assert_close_fp32(out[:T].view(T, c.h_q, c.d), ref, what=f"fused={fused} rep={rep}")
        outs[fused] = (out[:T], lse)
    assert torch.allclose(outs[True][0], outs[False][0], atol=1e-5, rtol=1e-5)
    assert torch.allclose(outs[True][1], outs[False][1], atol=1e-4, rtol=1e-5)


@pytest.mark.parametrize("kv_format", ["fp8", "e2m3"])
@pytest.mark.parametrize("h_q,h_k", [(8, 1), (16, 2), (32, 4)])
def test_tc_tensor_parallel_shards(kv_format, h_q, h_k):
    """The per-rank head counts of config 5 under TP 8 / 4 / 2 (64 q / 8 KV
    heads split by KV head): one KV head per rank included."""
    c = Case(seq_lens=(3000, 17, 1290), h_q=h_q, h_k=h_k, kv_format=kv_format, layout="BHN2D", seed=61 + h_k)
    out, _, _ = c.run(kernel="tc")
    ref, _ = c.oracle()
    T = c.b
    assert_close_fp32(out[:T].view(T, c.h_q, c.d), ref, what=f"tp shard {h_q}/{h_k}")


@pytest.mark.parametrize("kv_format", ["e3m2", "e2m1"])
@pytest.mark.parametrize("kernel", ["simt", "tc"])
@pytest.mark.parametrize("q_len,h_q,page_size,layout", [(1, 8, 16, "BHN2D"), (2, 8, 16, "BHN2D"), (1, 16, 32, "B2NHD"),
                                                        (1, 32, 64, "B2NHD"), (3, 16, 32, "BHN2D"), (6, 16, 16, "B2HND")])
def test_other_narrow_formats(kv_format, kernel, q_len, h_q, page_size, layout):
    """e3m2 and e2m1 caches (the reference harness's other narrow formats):
    both kernels, one- and several-warpgroup variants, fused and separate
    K / V boxes, with per-channel scales folded into Q and O."""
    c = Case(seq_lens=(1500, q_len + 3, 777), q_len=q_len, h_q=h_q, h_k=2, page_size=page_size,
             kv_format=kv_format, layout=layout, seed=81 + q_len)
    out, _, _ = c.run(kernel=kernel)
    ref, _ = c.oracle()
    T = c.b * q_len
    assert_close_fp32(out[:T].view(T, c.h_q, c.d), ref, what=f"{kv_format} {kernel} q_len {q_len}")


def test_tc_config4_shape_row_groups():
    """BASELINE config 4 shape (64 q / 8 KV heads, q_len 6 causal: 48 rows per KV
    head in 3 row groups), e2m3, shortened context."""
    c = Case(seq_lens=(3000, 6, 1290), q_len=6, h_q=64, h_k=8, kv_format="e2m3", layout="BHN2D", seed=41)
    out, _, _ = c.run(kernel="tc")
    ref, _ = c.oracle()
    T = c.b * 6
    assert_close_fp32(out[:T].view(T, c.h_q, c.d), ref, what="config4 shape")


def test_descale_per_seq_head_and_d256():
    c = Case(seq_lens=(77, 150, 1000), q_len=2, h_q=8, h_k=1, d=256, page_size=64, kv_format="fp8",
             layout="BHN2D", descale="seqhead", seed=9)
    out, _, _ = c.run()
    ref, _ = c.oracle()
    T = c.b * 2
    assert_close_fp32(out[:T].view(T, c.h_q, c.d), ref, what="d256 seqhead")


@pytest.mark.parametrize("kernel", ["simt", "tc"])
def test_empty_rows_and_fixed_grid(kernel):
    """L < q_len leaves the first draft rows with no visible key: O = 0. A
    padded fixed grid (CUDA-graph mode) gives the same result."""
    c = Case(seq_lens=(2, 400), q_len=4, h_q=8, h_k=2, kv_format="fp8", seed=11)
    out, _, _ = c.run(fixed_grid=True, kernel=kernel)
    ref, _ = c.oracle()
    T = c.b * 4
    got = out[:T].view(T, c.h_q, c.d)
    assert (got[:2] == 0).all()
    assert_close_fp32(got, ref, what="empty rows")


@pytest.mark.parametrize("kernel", ["simt", "tc"])
def test_graph_replay_with_new_plan(kernel):
    """Capture once with a fixed grid, re-plan (different lengths), replay."""
    c = Case(seq_lens=(900, 40, 2100), h_q=16, h_k=2, kv_format="fp8", seed=13, max_num_seqs=4)
    r = c.runner(kernel=kernel)
    T = c.b
    out = torch.zeros(T, c.h_q * c.d, dtype=torch.float32, device="cuda")
    kd, vd = c.dev(c.kd), c.dev(c.vd)
    plan = r.plan(c.seq_lens, c.b, 1, c.block_table, c.seq_lens_t, fixed_grid=True)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        r.run(plan, c.query, out, c.k_view, c.v_view, kd, vd, 1.0 / math.sqrt(c.d))
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        r.run(plan, c.query, out, c.k_view, c.v_view, kd, vd, 1.0 / math.sqrt(c.d))
    new_lens = [700, 40, 1900]
    c.seq_lens_t[: c.b].copy_(torch.tensor(new_lens, dtype=torch.int32))
    r.plan(new_lens, c.b, 1, c.block_table, c.seq_lens_t, fixed_grid=True)
    graph.replay()
    torch.cuda.synchronize()
    c.seq_lens = new_lens
    ref, _ = c.oracle()
    assert_close_fp32(out.view(T, c.h_q, c.d), ref, what="graph replay")


@pytest.mark.parametrize("kernel", ["simt", "tc"])
def test_bad_page_sets_status_not_fault(kernel):
    """A block-table entry past the pool is flagged in the status word and
    skipped (no out-of-bounds read)."""
    from mjolnir_b200 import _lib

    c = Case(seq_lens=(100,), h_q=8, h_k=2, kv_format="fp8", seed=17)
    c.block_table[0, 1] = c.num_pages + 5  # in bounds of the table, out of the pool
    with pytest.raises(_lib.MjolnirError):
        c.run(kernel=kernel)


@pytest.mark.parametrize("kv_format", ["fp8", "e2m3"])
@pytest.mark.parametrize("page_size", [16, 32, 64, 128])
def test_tc_page_sizes(kv_format, page_size):
    lens = (1, 127, 128, 129, 1000, 4097)
    c = Case(seq_lens=lens, h_q=32, h_k=4, page_size=page_size, kv_format=kv_format, layout="BHN2D", seed=page_size)
    out, _, _ = c.run(kernel="tc")
    ref, _ = c.oracle()
    T = c.b
    assert_close_fp32(out[:T].view(T, c.h_q, c.d), ref, what=f"tc {kv_format} PS {page_size}")


def test_tc_nan_bytes_past_sequence_end():
    """fp8 rows after the last token of a sequence's last page may hold NaN
    bytes (0x7F); they get P = 0 and must not reach O."""
    c = Case(seq_lens=(37, 200), h_q=8, h_k=2, kv_format="fp8", layout="BHN2D", seed=31)
    for s, L in enumerate(c.seq_lens):
        page = int(c.block_table_cpu[s, (L - 1) // c.PS])
        c.k_view[page, L % c.PS:] = 0x7F
        c.v_view[page, L % c.PS:] = 0x7F
    out, _, _ = c.run(kernel="tc")
    ref, _ = c.oracle()
    assert_close_fp32(out[: c.b].view(c.b, c.h_q, c.d), ref, what="nan tail")


def test_tc_zero_length_padding_request():
    """A CUDA-graph padding request (seq_len 0) writes O = 0, nothing else moves."""
    c = Case(seq_lens=(300, 0, 50), h_q=8, h_k=2, kv_format="e2m3", layout="BHN2D", seed=33)
    out, _, _ = c.run(kernel="tc")
    ref, _ = c.oracle()
    got = out[: c.b].view(c.b, c.h_q, c.d)
    assert (got[1] == 0).all()
    assert_close_fp32(got, ref, what="padding request")


@pytest.mark.parametrize("kv_format,q_len,h_q", [("e2m3", 1, 32), ("fp8", 1, 16), ("e2m3", 6, 64)])
def test_bounded_wait_runs_out_and_the_next_call_is_exact(kv_format, q_len, h_q):
    """The abort path of the bounded waits: with abort_probe_ns the MMA
    issuer of every CTA first waits 2 us on a phase nothing completes. The
    wait gives up, the launch still ends by itself (every role stops at its
    next wait, lets its copies and MMAs in flight finish and frees its tensor
    memory), the status word reads MJ_DEV_TIMEOUT, and the same call right
    after, without the probe, is exact. One-warpgroup (e2m3 with a converter
    warpgroup, fp8) and three-warpgroup (48 rows per KV head) variants."""
    from mjolnir_b200 import _lib
    from mjolnir_b200.runner import _stream

    c = Case(seq_lens=(3000, 1200, 700), q_len=q_len, h_q=h_q, h_k=8, kv_format=kv_format, seed=31, layout="BHN2D")
    r = c.runner(kernel="tc")
    plan = r.plan(c.seq_lens, c.b, q_len, c.block_table, c.seq_lens_t)
    T = c.b * q_len
    out = torch.zeros(T, c.h_q * c.d, device="cuda")
    args = r.decode_args(plan, c.query, out, c.k_view, c.v_view, c.dev(c.kd), c.dev(c.vd), 1.0 / math.sqrt(c.d),
                         q_mul=c.dev(c.q_mul), o_mul=c.dev(c.o_mul))
    assert _lib.KERNEL_NAMES[_lib.decode_kernel(args)] == "decode_tc"
    args.abort_probe_ns = 2000
    _lib.decode(args, _stream())
    torch.cuda.synchronize()
    with pytest.raises(_lib.MjolnirError, match=f"device status {_lib.MJ_DEV_TIMEOUT}"):
        r.check_status()
    assert int(r.status.item()) == 0  # check_status cleared it
    out, _, _ = c.run(kernel="tc")
    ref, _ = c.oracle()
    assert_close_fp32(out[:T].view(T, c.h_q, c.d), ref, what=f"{kv_format} q_len {q_len} after a timed-out launch")


def test_reset_after_an_error_clears_stale_merge_counts():
    """In-kernel split merge after a device error: a job that stopped early
    never counts itself in, so counters can be left short of a full count.
    check_status clears them with the status word; the same runner and plan
    then merge correctly. The counters are dirtied by hand after a timed-out
    launch (the probe stops every job before it counts)."""
    from mjolnir_b200 import _lib
    from mjolnir_b200.runner import _stream

    c = Case(seq_lens=(6000, 2500, 700), h_q=32, h_k=8, kv_format="e2m3", seed=34, outliers=0.01)
    r = c.runner(fused_merge=True, kernel="tc")
    plan = r.plan(c.seq_lens, c.b, 1, c.block_table, c.seq_lens_t)
    assert plan.with_reduction and int(plan.n_splits.max()) <= 16
    scale = 1.0 / math.sqrt(c.d)
    kd, vd, qm, om = c.dev(c.kd), c.dev(c.vd), c.dev(c.q_mul), c.dev(c.o_mul)
    out = torch.zeros(c.b, c.h_q * c.d, device="cuda")
    args = r.decode_args(plan, c.query, out, c.k_view, c.v_view, kd, vd, scale, q_mul=qm, o_mul=om)
    args.abort_probe_ns = 2000
    _lib.decode(args, _stream())
    torch.cuda.synchronize()
    r.merge_counters.fill_(1)
    with pytest.raises(_lib.MjolnirError, match=f"device status {_lib.MJ_DEV_TIMEOUT}"):
        r.check_status()
    assert int(r.merge_counters.abs().sum()) == 0 and int(r.status.item()) == 0
    got = torch.full((c.b, c.h_q * c.d), float("nan"), device="cuda")
    r.run(plan, c.query, got, c.k_view, c.v_view, kd, vd, scale, q_mul=qm, o_mul=om)
    torch.cuda.synchronize()
    r.check_status()
    ref, _ = c.oracle()
    assert_close_fp32(got.view(c.b, c.h_q, c.d), ref, what="in-kernel merge after a reset")
    assert int(r.merge_counters.abs().sum()) == 0


@pytest.mark.parametrize("kv_format,layout", [("fp8", "BHN2D"), ("e2m3", "BHN2D"), ("e3m2", "BHN2D"), ("e2m1", "BHN2D"),
                                              ("nvfp4", "BHN2D"), ("fp8", "B2NHD"), ("e2m3", "2BHND"), ("nvfp4", "B2NHD")])
@pytest.mark.parametrize("q_len,h_q,h_k", [(1, 16, 4), (1, 24, 4), (2, 16, 4), (1, 64, 4), (2, 64, 4)])
def test_tc_head_dim_256(kv_format, layout, q_len, h_q, h_k):
    """head_dim 256 on the tensor-core kernel (two 128-wide halves per KV row):
    4, 6, 8, 16 and 32 query rows per KV head (32: two row groups), the fused
    K|V box and separate boxes, splits merged by the combine launch and in the
    kernel, scores that grow along the sequence (the O rescale) and, on the
    other pass, 1 % of the values x8 (as the decode tests at head_dim 128,
    one or the other: both together drive |o| to ~20, where the split-fp8
    operands' relative error meets the 2e-3 absolute bound)."""
    for fused_merge, seed, ramp, outl in ((False, 61, 2.0, 0.0), (True, 62, 0.0, 0.01)):
        c = Case(seq_lens=(2100, 700, 129, 33), q_len=q_len, h_q=h_q, h_k=h_k, d=256, kv_format=kv_format,
                 layout=layout, seed=seed + q_len, k_ramp=ramp, outliers=outl)
        assert _kernel_of(c, kernel="tc") == "decode_tc"
        out, _, plan = c.run(kernel="tc", fused_merge=fused_merge)
        assert plan.with_reduction
        ref, _ = c.oracle()
        T = c.b * q_len
        assert_close_fp32(out[:T].view(T, c.h_q, c.d), ref,
                          what=f"d256 {kv_format}/{layout} n_q {q_len * h_q // h_k} merge {fused_merge}")
        assert torch.isnan(out[T:]).all(), "wrote past the batch"


def test_tc_head_dim_256_reference_shape_bf16():
    """The reference harness's own shape (24 q / 4 KV heads, head_dim 256,
    page 128), bf16 output, one long sequence split across the SMs."""
    c = Case(seq_lens=(9000,), h_q=24, h_k=4, d=256, page_size=128, kv_format="fp8", layout="BHN2D", seed=70)
    out, _, plan = c.run(out_dtype=torch.bfloat16, kernel="tc")
    ref, _ = c.oracle()
    assert_close_bf16(out[:1].view(1, c.h_q, c.d), ref, what="d256 reference shape")
