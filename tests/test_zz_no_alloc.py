"""mj_decode_noalloc: the decode entry point for callers that cannot allocate.

Some callers of this library cannot call cudaMalloc: an engine that has
already given all free HBM to its own KV-cache pool, code that runs while a
stream is captured into a CUDA graph in global mode, a plugin host that hands
a plugin only its inputs and outputs. They cannot supply the split-KV partial
buffers that mj_decode takes, so mj_decode_noalloc keeps the partials in a
fixed device array inside the library. These tests call it through the C ABI
and check it against mj_decode on the same inputs, twice in a row (the array
keeps the previous call's contents), and check that a request larger than the
array is refused with a message.

Collected last (file name), so a stop-at-first-failure run has already run
every other test; it also passes alone in a fresh process.
"""

import math

import pytest
import torch

from tests.helpers import Case, assert_close_fp32

pytestmark = pytest.mark.gpu


def _decode_both(c, runner, plan, out_dtype=torch.float32):
    from mjolnir_b200 import _lib
    from mjolnir_b200.runner import _stream

    T = c.b * c.q_len
    ref = torch.full((T, c.h_q * c.d), float("nan"), dtype=out_dtype, device="cuda")
    got = torch.full((T, c.h_q * c.d), float("nan"), dtype=out_dtype, device="cuda")
    kd, vd, qm, om = c.dev(c.kd), c.dev(c.vd), c.dev(c.q_mul), c.dev(c.o_mul)
    runner.run(plan, c.query, ref, c.k_view, c.v_view, kd, vd, 1.0 / math.sqrt(c.d), q_mul=qm, o_mul=om)
    args = runner.decode_args(plan, c.query, got, c.k_view, c.v_view, kd, vd, 1.0 / math.sqrt(c.d), q_mul=qm, o_mul=om)
    args.o_part = None  # the entry point must not need caller scratch
    args.lse_part = None
    args.part_seqs = 0
    _lib.decode_noalloc(args, _stream())
    torch.cuda.synchronize()
    runner.check_status()
    return ref.view(T, c.h_q, c.d), got.view(T, c.h_q, c.d)


def test_noalloc_matches_decode_two_calls_in_a_row():
    # 148 SMs and 3 sequences: every sequence splits, so the partials are used
    first = Case(seq_lens=(5000, 3000, 129), h_q=32, h_k=8, kv_format="e2m3", seed=21, outliers=0.01)
    r1 = first.runner(fused_merge=False)  # partials merged by the combine launch (the next test: in the kernel)
    p1 = r1.plan(first.seq_lens, first.b, 1, first.block_table, first.seq_lens_t)
    assert p1.with_reduction
    ref1, got1 = _decode_both(first, r1, p1)
    assert_close_fp32(got1, ref1, what="noalloc call 1 vs mj_decode")
    # a second call with other shapes and data right after the first: the
    # array still holds call 1's partials, which must not leak into call 2
    second = Case(seq_lens=(2100, 40, 7000, 900), q_len=2, h_q=16, h_k=2, kv_format="fp8", seed=22, descale="head")
    r2 = second.runner(fused_merge=False)
    p2 = r2.plan(second.seq_lens, second.b, 2, second.block_table, second.seq_lens_t)
    assert p2.with_reduction
    ref2, got2 = _decode_both(second, r2, p2)
    assert_close_fp32(got2, ref2, what="noalloc call 2 vs mj_decode")
    oracle2, _ = second.oracle()
    assert_close_fp32(got2, oracle2, what="noalloc call 2 vs oracle")


def test_noalloc_with_in_kernel_merge():
    """With merge counters (a runner built with fused_merge) the tensor-core
    kernel merges the splits itself, reading the partials back from the
    built-in array: the result still equals mj_decode's, on two calls."""
    c = Case(seq_lens=(6000, 2500, 700), h_q=32, h_k=8, kv_format="e2m3", seed=24, outliers=0.01)
    r = c.runner(fused_merge=True)
    plan = r.plan(c.seq_lens, c.b, 1, c.block_table, c.seq_lens_t)
    assert plan.with_reduction and int(plan.n_splits.max()) <= 16  # the in-kernel merge takes <= 16 splits
    for call in (1, 2):
        ref, got = _decode_both(c, r, plan)
        assert_close_fp32(got, ref, what=f"noalloc with the in-kernel merge, call {call}")
    oracle, _ = c.oracle()
    assert_close_fp32(got, oracle, what="noalloc with the in-kernel merge vs oracle")
    assert int(r.merge_counters.abs().sum()) == 0  # the last job of each split group reset its counter


def test_noalloc_refuses_oversized_partials():
    from mjolnir_b200 import _lib

    c = Case(seq_lens=(300, 200), h_q=8, h_k=2, kv_format="fp8", seed=23)
    r = c.runner()
    plan = r.plan(c.seq_lens, c.b, 1, c.block_table, c.seq_lens_t)
    out = torch.empty(c.b, c.h_q * c.d, dtype=torch.float32, device="cuda")
    args = r.decode_args(plan, c.query, out, c.k_view, c.v_view, c.dev(c.kd), c.dev(c.vd), 1.0 / math.sqrt(c.d))
    args.num_seqs = 4096  # 16 splits x 4096 seqs x 2 heads x 4 rows x 129 x 4 B = 270 MB > 16 MiB
    args.max_splits = 16
    with pytest.raises(_lib.MjolnirError, match="built-in scratch holds"):
        _lib.decode_noalloc(args, 0)
