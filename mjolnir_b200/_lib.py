"""ctypes binding of libmjolnir_b200.so (the C ABI in include/mjolnir_b200.h).

The library is built in-tree (``python -m mjolnir_b200.build``). There is no
fallback: if the library is missing or a call fails, this module raises.
"""

from __future__ import annotations

import ctypes as C
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmjolnir_b200.so")

MJ_OK = 0
MJ_ERR_INVALID = 1
MJ_ERR_UNSUPPORTED = 2
MJ_ERR_CUDA = 3
MJ_ERR_DEVICE = 4

MJ_DEV_OK = 0
MJ_DEV_BAD_PAGE = 1
MJ_DEV_BAD_SPLIT = 2
MJ_DEV_TIMEOUT = 3

MJ_KV_FP8_E4M3 = 0
MJ_KV_E2M3 = 1
MJ_KV_E3M2 = 2
MJ_KV_E2M1 = 3
MJ_KV_NVFP4 = 4
KV_FORMATS = {"fp8": MJ_KV_FP8_E4M3, "e2m3": MJ_KV_E2M3, "e3m2": MJ_KV_E3M2, "e2m1": MJ_KV_E2M1,
              "nvfp4": MJ_KV_NVFP4}

MJ_DT_BF16 = 0
MJ_DT_FP16 = 1
MJ_DT_FP32 = 2

MJ_KERNEL_AUTO = 0
MJ_KERNEL_SIMT = 1
MJ_KERNEL_TC = 2
KERNEL_NAMES = {MJ_KERNEL_SIMT: "decode_simt", MJ_KERNEL_TC: "decode_tc"}

MJ_SCALE_TENSOR = 0
MJ_SCALE_HEAD = 1
MJ_SCALE_CHANNEL = 2
MJ_SCALE_SEQ_HEAD = 3

EXPORTED = ("mj_last_error", "mj_abi_version", "mj_row_bytes", "mj_cache_write", "mj_decode", "mj_combine",
            "mj_decode_noalloc", "mj_decode_kernel", "mj_expand_pages", "mj_plan_split_kv", "mj_create", "mj_plan",
            "mj_runner_fill", "mj_runner_status", "mj_destroy", "mj_tc_fallbacks")

_i64, _i32, _vp, _f32 = C.c_int64, C.c_int, C.c_void_p, C.c_float


class CacheWriteArgs(C.Structure):
    _fields_ = [
        ("key", _vp), ("value", _vp), ("src_dtype", _i32),
        ("num_tokens", _i64), ("h_k", _i32), ("head_size", _i32),
        ("key_stride_tok", _i64), ("key_stride_head", _i64),
        ("value_stride_tok", _i64), ("value_stride_head", _i64),
        ("k_cache", _vp), ("v_cache", _vp),
        ("k_stride_page", _i64), ("k_stride_row", _i64), ("k_stride_head", _i64),
        ("v_stride_page", _i64), ("v_stride_row", _i64), ("v_stride_head", _i64),
        ("num_pages", _i64), ("page_size", _i32), ("kv_format", _i32),
        ("slot_mapping", _vp),
        ("k_scale", _vp), ("k_scale_mode", _i32),
        ("v_scale", _vp), ("v_scale_mode", _i32),
        ("status", _vp),
        ("k_scales", _vp), ("v_scales", _vp),
        ("ks_stride_page", _i64), ("ks_stride_row", _i64), ("ks_stride_head", _i64),
        ("vs_stride_page", _i64), ("vs_stride_row", _i64), ("vs_stride_head", _i64),
    ]


class ExpandArgs(C.Structure):
    _fields_ = [
        ("k_cache", _vp), ("v_cache", _vp),
        ("k_stride_page", _i64), ("k_stride_row", _i64), ("k_stride_head", _i64),
        ("v_stride_page", _i64), ("v_stride_row", _i64), ("v_stride_head", _i64),
        ("num_pages", _i64),
        ("page_size", _i32), ("h_k", _i32), ("head_size", _i32),
        ("src_pages", _vp), ("num_out_pages", _i64),
        ("k_out", _vp), ("v_out", _vp),
        ("ko_stride_page", _i64), ("ko_stride_row", _i64), ("ko_stride_head", _i64),
        ("vo_stride_page", _i64), ("vo_stride_row", _i64), ("vo_stride_head", _i64),
        ("k_ratio", _vp), ("k_ratio_mode", _i32),
        ("v_ratio", _vp), ("v_ratio_mode", _i32),
        ("status", _vp),
        ("kv_format", _i32),
        ("k_scales", _vp), ("v_scales", _vp),
        ("ks_stride_page", _i64), ("ks_stride_row", _i64), ("ks_stride_head", _i64),
        ("vs_stride_page", _i64), ("vs_stride_row", _i64), ("vs_stride_head", _i64),
    ]


class DecodeArgs(C.Structure):
    _fields_ = [
        ("num_seqs", _i32), ("q_len", _i32), ("h_q", _i32), ("h_k", _i32),
        ("head_size", _i32), ("page_size", _i32), ("kv_format", _i32),
        ("q", _vp), ("q_dtype", _i32), ("q_stride_tok", _i64), ("q_stride_head", _i64),
        ("o", _vp), ("o_dtype", _i32), ("o_stride_tok", _i64), ("o_stride_head", _i64),
        ("k_cache", _vp), ("v_cache", _vp),
        ("k_stride_page", _i64), ("k_stride_row", _i64), ("k_stride_head", _i64),
        ("v_stride_page", _i64), ("v_stride_row", _i64), ("v_stride_head", _i64),
        ("num_pages", _i64),
        ("block_table", _vp), ("block_table_stride", _i64),
        ("seq_lens", _vp),
        ("work", _vp), ("num_work", _i32),
        ("n_splits", _vp), ("max_splits", _i32),
        ("o_part", _vp), ("lse_part", _vp), ("part_seqs", _i32),
        ("lse", _vp),
        ("k_descale", _vp), ("k_descale_mode", _i32),
        ("v_descale", _vp), ("v_descale_mode", _i32),
        ("q_mul", _vp), ("o_mul", _vp),
        ("softmax_scale", _f32), ("causal", _i32), ("with_combine", _i32),
        ("kernel", _i32),
        ("status", _vp),
        ("merge_counters", _vp),
        ("k_scales", _vp), ("v_scales", _vp),
        ("ks_stride_page", _i64), ("ks_stride_row", _i64), ("ks_stride_head", _i64),
        ("vs_stride_page", _i64), ("vs_stride_row", _i64), ("vs_stride_head", _i64),
        ("abort_probe_ns", C.c_uint64),
    ]


class MjolnirError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"mjolnir_b200 status {code}: {msg}")
        self.code = code


_lock = threading.Lock()
_lib = None


def load():
    """Load the in-tree library (build it first if the sources are newer)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m mjolnir_b200.build` "
                "(there is no CPU or PyTorch fallback for the hot path)"
            )
        lib = C.CDLL(LIB_PATH)
        lib.mj_last_error.restype = C.c_char_p
        lib.mj_abi_version.restype = C.c_int
        lib.mj_row_bytes.argtypes = [C.c_int, C.c_int]
        lib.mj_row_bytes.restype = C.c_int
        lib.mj_cache_write.argtypes = [C.POINTER(CacheWriteArgs), _vp]
        lib.mj_cache_write.restype = C.c_int
        for fn in ("mj_decode", "mj_combine", "mj_decode_noalloc"):
            getattr(lib, fn).argtypes = [C.POINTER(DecodeArgs), _vp]
            getattr(lib, fn).restype = C.c_int
        lib.mj_decode_kernel.argtypes = [C.POINTER(DecodeArgs)]
        lib.mj_decode_kernel.restype = C.c_int
        lib.mj_tc_fallbacks.restype = C.c_int
        lib.mj_expand_pages.argtypes = [C.POINTER(ExpandArgs), _vp]
        lib.mj_expand_pages.restype = C.c_int
        _pi = C.POINTER(C.c_int32)
        lib.mj_plan_split_kv.argtypes = [_pi, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                         C.c_float, _pi, C.c_int, _pi, C.POINTER(C.c_int), C.POINTER(C.c_int)]
        lib.mj_plan_split_kv.restype = C.c_int
        lib.mj_create.argtypes = [C.c_int] * 10
        lib.mj_create.restype = _vp
        lib.mj_plan.argtypes = [_vp, _pi, C.c_int, C.c_int, C.c_int, C.c_int, _vp]
        lib.mj_plan.restype = C.c_int
        lib.mj_runner_fill.argtypes = [_vp, C.POINTER(DecodeArgs)]
        lib.mj_runner_fill.restype = C.c_int
        lib.mj_runner_status.argtypes = [_vp]
        lib.mj_runner_status.restype = C.c_int
        lib.mj_destroy.argtypes = [_vp]
        lib.mj_destroy.restype = None
        _lib = lib
    return _lib


def check(rc: int) -> None:
    if rc != MJ_OK:
        msg = load().mj_last_error().decode(errors="replace")
        raise MjolnirError(rc, msg)


def cache_write(args: CacheWriteArgs, stream: int) -> None:
    check(load().mj_cache_write(C.byref(args), _vp(stream)))


def decode(args: DecodeArgs, stream: int) -> None:
    check(load().mj_decode(C.byref(args), _vp(stream)))


def decode_kernel(args: DecodeArgs) -> int:
    """MJ_KERNEL_SIMT or MJ_KERNEL_TC: the kernel mj_decode would launch."""
    rc = load().mj_decode_kernel(C.byref(args))
    if rc < 0:
        check(-rc)
    return rc


def combine(args: DecodeArgs, stream: int) -> None:
    check(load().mj_combine(C.byref(args), _vp(stream)))


def decode_noalloc(args: DecodeArgs, stream: int) -> None:
    """mj_decode with the split-KV partials kept in the library's built-in
    16 MiB device array, for callers that cannot allocate device memory."""
    check(load().mj_decode_noalloc(C.byref(args), _vp(stream)))


def expand_pages(args: ExpandArgs, stream: int) -> None:
    """e2m3 -> e4m3 expansion of cache pages into a fallback's scratch."""
    check(load().mj_expand_pages(C.byref(args), _vp(stream)))


def plan_split_kv(seq_lens, h_k: int, n_q_tiles: int, sm_count: int, ctas_per_sm: int = 1, max_splits: int = 16,
                  pad_to: int = 0, rebalance: bool = True, item_overhead: float = 2.0):
    """The library's host planner (mj_plan_split_kv): (work (n, 4) int32 array,
    n_splits list, chunk_tiles)."""
    import numpy as np

    lens = np.ascontiguousarray(np.asarray(seq_lens, dtype=np.int32))
    n = len(lens)
    tiles = [max(1, -(-int(L) // 128)) for L in lens]
    cap = max(pad_to, sum(tiles))
    work = np.zeros((max(cap, 1), 4), dtype=np.int32)
    ns = np.zeros(n, dtype=np.int32)
    num, chunk = C.c_int(0), C.c_int(0)
    _pi = C.POINTER(C.c_int32)
    check(load().mj_plan_split_kv(lens.ctypes.data_as(_pi), n, h_k, n_q_tiles, sm_count, ctas_per_sm, max_splits,
                                  pad_to, int(rebalance), float(item_overhead), work.ctypes.data_as(_pi), len(work),
                                  ns.ctypes.data_as(_pi), C.byref(num), C.byref(chunk)))
    return work[: num.value], ns.tolist(), chunk.value
