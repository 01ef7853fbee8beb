"""The runner handle of the C ABI on the B200 (mj_create / mj_plan /
mj_runner_fill / mj_decode / mj_destroy): a host that plans and decodes
without the Python runner gets the oracle's output, re-plans into the same
fixed-address buffers under a CUDA graph, and reads the device status."""

import ctypes as C
import math

import numpy as np
import pytest
import torch

from tests.helpers import Case, assert_close_fp32

pytestmark = pytest.mark.gpu


def _runner(lib, c, max_splits=16):
    from mjolnir_b200 import _lib

    h = lib.mj_create(0, c.h_q, c.h_k, c.d, c.PS, c.max_num_seqs, c.q_len, _lib.KV_FORMATS[c.kv_format], max_splits, 2)
    assert h, lib.mj_last_error()
    return h


def _args(c, out):
    """mj_decode_args with the caller's tensors (the plan fields come from the runner)."""
    r = c.runner()
    plan = r.plan(c.seq_lens, c.b, c.q_len, c.block_table, c.seq_lens_t)
    return r, r.decode_args(plan, c.query, out, c.k_view, c.v_view, c.dev(c.kd), c.dev(c.vd), 1.0 / math.sqrt(c.d),
                            q_mul=c.dev(c.q_mul), o_mul=c.dev(c.o_mul))


@pytest.mark.parametrize("kv_format", ["fp8", "e2m3"])
def test_native_runner_plans_and_decodes(kv_format):
    from mjolnir_b200 import _lib

    lib = _lib.load()
    c = Case(seq_lens=(4000, 900, 129, 3000), h_q=16, h_k=2, kv_format=kv_format, layout="BHN2D", seed=71)
    T = c.b
    out = torch.full((T, c.h_q * c.d), float("nan"), dtype=torch.float32, device="cuda")
    keep, a = _args(c, out)
    h = _runner(lib, c)
    try:
        lens = np.asarray(c.seq_lens, dtype=np.int32)
        stream = torch.cuda.current_stream().cuda_stream
        _lib.check(lib.mj_plan(h, lens.ctypes.data_as(C.POINTER(C.c_int32)), c.b, 1, 0, 0, C.c_void_p(stream)))
        _lib.check(lib.mj_runner_fill(h, C.byref(a)))
        assert a.with_combine == 1  # 4 sequences on 296 slots: they split
        _lib.decode(a, stream)
        torch.cuda.synchronize()
        assert lib.mj_runner_status(h) == 0
        ref, _ = c.oracle()
        assert_close_fp32(out[:T].view(T, c.h_q, c.d), ref, what=f"native runner {kv_format}")

        # fixed grid: capture once, re-plan new lengths into the same buffers, replay
        _lib.check(lib.mj_plan(h, lens.ctypes.data_as(C.POINTER(C.c_int32)), c.b, 1, 0, 1, C.c_void_p(stream)))
        _lib.check(lib.mj_runner_fill(h, C.byref(a)))
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            _lib.decode(a, s.cuda_stream)  # warm-up outside capture
            torch.cuda.synchronize()
            with torch.cuda.graph(g, stream=s):
                _lib.decode(a, s.cuda_stream)
        torch.cuda.current_stream().wait_stream(s)
        new = [1500, 800, 40, 2222]  # within the blocks each sequence owns
        c.seq_lens_t[: c.b].copy_(torch.tensor(new, dtype=torch.int32))
        nl = np.asarray(new, dtype=np.int32)
        _lib.check(lib.mj_plan(h, nl.ctypes.data_as(C.POINTER(C.c_int32)), c.b, 1, 0, 1,
                               C.c_void_p(torch.cuda.current_stream().cuda_stream)))
        torch.cuda.synchronize()
        out.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        c.seq_lens = new
        ref2, _ = c.oracle()
        assert_close_fp32(out[:T].view(T, c.h_q, c.d), ref2, what=f"native runner graph replay {kv_format}")
        del g
    finally:
        lib.mj_destroy(h)
    del keep
