"""Decode runner: plan buffers, KV-cache views and the launch through the C ABI.

Mirrors the reference's shared runner (GoBrrr-ai/mjolnir
``src/mjolnir/mjolnir/runner.py``: ``StepPlan`` :382-397, ``env_flag`` :404-413,
``detect_kv_layout`` / ``split_kv_cache`` :431-484) and the Thor runner
(``arch/thor/runner.py:84-494``: persistent fixed-address plan buffers, a
fixed grid per q_len so CUDA graphs replay, ``plan`` / ``run``). Nothing here
imports vLLM. The kernels are the in-tree sm_100a library; there is no other
compute path.
"""

from __future__ import annotations

import logging
import math
import os
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from .plan import TILE_ROWS, plan_split_kv

_log = logging.getLogger("vllm.mjolnir")

SUPPORTED_PAGE_SIZES = (16, 32, 64, 128)
ENV_PREFIX = "MJOLNIR_ATTN_"
LEGACY_ENV_PREFIX = "THOR_T5_"


def env_flag(name: str, default: str = "") -> str:
    """Read a ``MJOLNIR_ATTN_*`` knob (the legacy ``THOR_T5_*`` spelling is
    honoured as a fallback, as in the reference)."""
    if name in os.environ:
        return os.environ[name].strip()
    if name.startswith(ENV_PREFIX):
        legacy = LEGACY_ENV_PREFIX + name[len(ENV_PREFIX):]
        if legacy in os.environ:
            return os.environ[legacy].strip()
    return default.strip()


@dataclass
class StepPlan:
    """Per-step plan shared by every layer of one KV-cache group."""

    num_seqs: int
    q_len: int
    n_q: int
    num_work: int  # grid.x, fixed per q_len capacity
    with_reduction: bool
    block_table: torch.Tensor  # (>= num_seqs, max_blocks) int32, device
    seq_lens: torch.Tensor  # (>= num_seqs,) int32, device
    work: torch.Tensor  # (num_work, 4) int32 view of a persistent buffer
    n_splits: torch.Tensor  # (num_seqs,) int32 view of a persistent buffer
    chunk_tiles: int
    num_chunks: int
    causal: bool = True
    tile_jobs: int = 0  # 128-row KV tiles x KV heads the step reads


# ---------------------------------------------------------------------------
# KV-cache views
# ---------------------------------------------------------------------------
# BHN2R is the (B, H, N, 2, row) shape the fp6 cache gets on a vLLM without
# the pluggable KV-dtype API (see ``kvdtype``): BHN2D with K|V split into
# their own dim, whatever stride order the fallback backend applied.
KV_LAYOUTS = ("BHN2D", "BNH2D", "B2NHD", "B2HND", "2BNHD", "2BHND", "BHN2R")


def detect_kv_layout(shape, num_kv_heads: int, page_size: int, head_size: int) -> str:
    """Name the layout of a vLLM per-layer KV cache tensor (``head_size`` is
    the per-row element count of the tensor's last dim: d for fp8, the packed
    row bytes for e2m3). Ambiguous shapes (H == N) resolve to the first match;
    MJOLNIR_ATTN_KV_LAYOUT overrides."""
    forced = env_flag("MJOLNIR_ATTN_KV_LAYOUT").upper()
    if forced:
        if forced not in KV_LAYOUTS:
            raise ValueError(f"MJOLNIR_ATTN_KV_LAYOUT must be one of {KV_LAYOUTS}")
        return forced
    H, N, D = num_kv_heads, page_size, head_size
    s = tuple(shape)
    if len(s) == 4 and s[3] == 2 * D:
        if (s[1], s[2]) == (H, N):
            return "BHN2D"
        if (s[1], s[2]) == (N, H):
            return "BNH2D"
    if len(s) == 5 and s[4] == D:
        if s[1] == 2 and (s[2], s[3]) == (N, H):
            return "B2NHD"
        if s[1] == 2 and (s[2], s[3]) == (H, N):
            return "B2HND"
        if s[0] == 2 and (s[2], s[3]) == (N, H):
            return "2BNHD"
        if s[0] == 2 and (s[2], s[3]) == (H, N):
            return "2BHND"
        if s[3] == 2 and (s[1], s[2]) == (H, N):
            return "BHN2R"
    raise ValueError(
        f"unrecognized KV cache shape {s} for H={H} N={N} D={D}; set MJOLNIR_ATTN_KV_LAYOUT to one of {KV_LAYOUTS}"
    )


def split_kv_cache(kv_cache: torch.Tensor, layout: str, row: int):
    """Zero-copy logical (num_pages, page_size, h_k, row) K and V views of any
    supported layout; the physical order is carried in the strides."""
    D = row
    if layout == "BHN2D":
        k, v = kv_cache[..., :D].transpose(1, 2), kv_cache[..., D:].transpose(1, 2)
    elif layout == "BNH2D":
        k, v = kv_cache[..., :D], kv_cache[..., D:]
    elif layout == "B2NHD":
        k, v = kv_cache[:, 0], kv_cache[:, 1]
    elif layout == "B2HND":
        k, v = kv_cache[:, 0].transpose(1, 2), kv_cache[:, 1].transpose(1, 2)
    elif layout == "2BNHD":
        k, v = kv_cache[0], kv_cache[1]
    elif layout == "2BHND":
        k, v = kv_cache[0].transpose(1, 2), kv_cache[1].transpose(1, 2)
    elif layout == "BHN2R":
        k, v = kv_cache[:, :, :, 0].transpose(1, 2), kv_cache[:, :, :, 1].transpose(1, 2)
    else:
        raise ValueError(layout)
    return k, v


def row_bytes(head_size: int, kv_format: str) -> int:
    if head_size % 16:
        raise ValueError(f"head_size {head_size} must be a multiple of 16")
    if kv_format == "fp8":
        return head_size
    if kv_format in ("e2m3", "e3m2"):
        return head_size * 3 // 4
    if kv_format in ("e2m1", "nvfp4"):
        return head_size // 2
    raise ValueError(f"kv_format {kv_format!r}")


NVFP4_GROUP = 16


def scale_row_bytes(head_size: int) -> int:
    """Bytes of one nvfp4 scale row: one e4m3 byte per 16 elements."""
    return head_size // NVFP4_GROUP


def set_scale_views(a, k_scales: torch.Tensor | None, v_scales: torch.Tensor | None, pages: int, page_size: int,
                    h_k: int, head_size: int, kv_format: str) -> None:
    """Point an args struct at the nvfp4 group-scale views (logical
    (pages, page_size, h_k, head_size / 16) bytes, last dim contiguous)."""
    if kv_format != "nvfp4":
        return
    want = (page_size, h_k, scale_row_bytes(head_size))
    for name, t in (("k_scales", k_scales), ("v_scales", v_scales)):
        if t is None:
            raise ValueError("nvfp4 needs k_scales and v_scales")
        if t.dim() != 4 or tuple(t.shape[1:]) != want or t.shape[0] < pages or t.element_size() != 1:
            raise ValueError(f"{name} view {tuple(t.shape)} is not (>= {pages}, {want[0]}, {want[1]}, {want[2]}) bytes")
    a.k_scales, a.v_scales = k_scales.data_ptr(), v_scales.data_ptr()
    a.ks_stride_page, a.ks_stride_row, a.ks_stride_head = kv_byte_strides(k_scales)
    a.vs_stride_page, a.vs_stride_row, a.vs_stride_head = kv_byte_strides(v_scales)


_DT = {torch.bfloat16: _lib.MJ_DT_BF16, torch.float16: _lib.MJ_DT_FP16, torch.float32: _lib.MJ_DT_FP32}


def dtype_code(dt: torch.dtype) -> int:
    if dt not in _DT:
        raise TypeError(f"unsupported dtype {dt} (bf16, fp16 or fp32)")
    return _DT[dt]


def kv_byte_strides(view: torch.Tensor):
    """(page, row, head) byte strides of a logical (pages, PS, h_k, row) view."""
    if view.dim() != 4 or view.stride(3) != 1:
        raise ValueError(f"KV view must be (pages, page_size, h_k, row) with a contiguous row, got {tuple(view.shape)}")
    es = view.element_size()
    st = []
    for n, s in zip(view.shape[:3], view.stride()[:3]):
        st.append(0 if n == 1 else s * es)  # size-1 dims may carry any stride
    return tuple(st)


def scale_mode(t: torch.Tensor, h_k: int, d: int) -> int:
    """Cache-write scale mode (the reference's ``kvfp6._scale_mode``,
    ``kvfp6.py:328-335``)."""
    n = t.numel()
    if n == h_k * d and d > 1 and (h_k > 1 or n > 1):
        if not t.is_contiguous():
            raise ValueError("per-channel KV scales must be contiguous (h_k, d)")
        return _lib.MJ_SCALE_CHANNEL
    if n not in (1, h_k):
        raise ValueError(f"KV scale must be per tensor, per KV head or (h_k, d), got {tuple(t.shape)}")
    return _lib.MJ_SCALE_HEAD if (n == h_k and h_k > 1) else _lib.MJ_SCALE_TENSOR


def descale_mode(t: torch.Tensor, num_seqs: int, h_k: int) -> int:
    """Decode descale mode: 1 element, (h_k,), or (b, h_k) row-major."""
    if t.numel() == 1:
        return _lib.MJ_SCALE_TENSOR
    if t.dim() == 1 and t.shape[0] == h_k:
        if t.stride(0) != 1:
            raise ValueError("per-head descale must be contiguous")
        return _lib.MJ_SCALE_HEAD
    if t.dim() == 2 and t.shape[1] == h_k and t.shape[0] >= num_seqs and t.stride() == (h_k, 1):
        return _lib.MJ_SCALE_SEQ_HEAD
    raise ValueError(f"descale shape {tuple(t.shape)} (1, (h_k,) or contiguous (b, h_k))")


_KERNELS = {"auto": _lib.MJ_KERNEL_AUTO, "simt": _lib.MJ_KERNEL_SIMT, "tc": _lib.MJ_KERNEL_TC}


def _ptr(t):
    return None if t is None else t.data_ptr()


def _stream(device=None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class DecodeRunner:
    """The B200 decode runner (the counterpart of the reference's
    ``T5DecodeRunner``, ``arch/thor/runner.py:84``).

    Owns the persistent, fixed-address plan buffers (work list, per-sequence
    split counts, split-KV partials) so that a captured CUDA graph replays any
    later plan of the same q_len. Q is read and O written in vLLM's
    (tokens, h_q, d) layout directly through strides -- no pack / unpack
    copies -- and the e2m3 channel scales (``q_mul`` / ``o_mul``) are applied
    inside the kernel."""

    def __init__(
        self,
        *,
        num_heads: int,
        num_kv_heads: int,
        head_size: int,
        page_size: int,
        out_dtype: torch.dtype = torch.bfloat16,
        max_num_seqs: int = 256,
        max_q_len: int = 1,
        ctas_per_sm: int = 2,
        max_splits: int = 16,
        kv_format: str = "fp8",
        device: torch.device | str = "cuda",
        sm_count: int | None = None,
        rebalance: bool = True,
        kernel: str | None = None,
        fused_merge: bool | None = None,
    ):
        if num_heads % num_kv_heads:
            raise ValueError("num_heads must be a multiple of num_kv_heads")
        if head_size not in (128, 256):
            raise ValueError(f"head_size {head_size}: the decode kernel runs 128 or 256")
        if page_size not in SUPPORTED_PAGE_SIZES:
            raise ValueError(f"page size {page_size} unsupported (supported: {SUPPORTED_PAGE_SIZES})")
        if kv_format not in _lib.KV_FORMATS:
            raise ValueError(f"kv_format must be one of {tuple(_lib.KV_FORMATS)}")
        self.h_q, self.h_k, self.d = num_heads, num_kv_heads, head_size
        self.h_r = num_heads // num_kv_heads
        if max_q_len * self.h_r > 64:
            raise ValueError(f"q_len * h_q / h_k = {max_q_len * self.h_r} > 64 query rows per KV head")
        self.page_size = page_size
        self.out_dtype = out_dtype
        self.max_num_seqs = max_num_seqs
        self.max_q_len = max_q_len
        self.ctas_per_sm = ctas_per_sm
        self.max_splits = max_splits
        self.kv_format = kv_format
        self.kv_row_bytes = row_bytes(head_size, kv_format)
        self.rebalance = rebalance
        # decode kernel: "auto" (tensor-core kernel where it applies), "simt" or "tc"
        kernel = (kernel or env_flag("MJOLNIR_ATTN_KERNEL", "auto")).lower()
        if kernel not in _KERNELS:
            raise ValueError(f"kernel must be one of {tuple(_KERNELS)}")
        self.kernel = _KERNELS[kernel]
        self.device = torch.device(device)
        if sm_count is None:
            sm_count = torch.cuda.get_device_properties(self.device).multi_processor_count
        self.sm_count = sm_count
        _lib.load()  # fail at construction, not at the first step
        self._cap = max(max_num_seqs * max_splits, self.slots(1))
        nq_max = max_q_len * self.h_r
        dev = self.device
        self.work_buf = torch.zeros(self._cap, 4, dtype=torch.int32, device=dev)
        self.nsplit_buf = torch.ones(max_num_seqs, dtype=torch.int32, device=dev)
        part = max_splits * max_num_seqs * self.h_k * nq_max
        self.o_part = torch.empty(part * head_size, dtype=torch.float32, device=dev)
        self.lse_part = torch.empty(part, dtype=torch.float32, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        # split merge inside the tensor-core kernel (its last job per sequence
        # and KV head merges; the counters return to zero after every launch).
        # It saves the combine launch, which pays on short steps (fp8, batch 4
        # x 4K: 30 -> 21 us per step), but its fences, atomics and serial
        # merges at the ends of jobs cost more on long ones (cfg2 -25 %, cfg3
        # and the north-star shape -9 %). None (MJOLNIR_ATTN_FUSED_MERGE=auto,
        # the default) decides per plan: in the kernel when the step reads at
        # most 16 tiles per SM; 1 / 0 force it on / off.
        if fused_merge is None:
            mode = env_flag("MJOLNIR_ATTN_FUSED_MERGE", "auto").lower()
            fused_merge = True if mode in ("1", "true", "yes") else False if mode in ("0", "false", "no") else None
        self.fused_merge = fused_merge
        self.merge_counters = torch.zeros(max_num_seqs * self.h_k * 64, dtype=torch.int32, device=dev)
        self._one = torch.ones(1, dtype=torch.float32, device=dev)

    # ------------------------------------------------------------------ plan
    def n_tiles(self, q_len: int) -> int:
        """CTA jobs per (work item, KV head): the tensor-core kernel serves up to
        48 query rows per job (16 at head_size 256) and cuts larger GQA x draft
        groups into row groups."""
        n_q = q_len * self.h_r
        rows = 16 if self.d == 256 else 48
        return 1 if n_q <= rows else -(-n_q // rows)

    def ctas(self, q_len: int) -> int:
        """Resident CTAs per SM of the kernel variant for this q_len: two for
        up to 16 query rows per KV head, one (several warpgroups, or head_size
        256) beyond."""
        return self.ctas_per_sm if q_len * self.h_r <= 16 and self.d == 128 else 1

    def slots(self, q_len: int) -> int:
        return max(1, (self.sm_count * self.ctas(q_len)) // (self.h_k * self.n_tiles(q_len)))

    def plan(
        self,
        seq_lens_cpu,
        num_seqs: int,
        q_len: int,
        block_table: torch.Tensor,
        seq_lens: torch.Tensor,
        margin: int = 0,
        causal: bool = True,
        fixed_grid: bool = False,
    ) -> StepPlan:
        """CPU plan + async copy into the persistent device buffers. ``margin``
        plans every sequence that many tokens longer (the kernel masks with the
        device ``seq_lens``, so the plan stays valid while they grow).
        ``fixed_grid`` launches the padded capacity (empty items exit at once)
        so a captured CUDA graph replays any later plan; otherwise the grid is
        the plan's real item count."""
        if not (1 <= q_len <= self.max_q_len and num_seqs <= self.max_num_seqs):
            raise ValueError(f"q_len {q_len} / num_seqs {num_seqs} beyond the runner's capacity")
        lens = [int(x) + margin for x in list(seq_lens_cpu)[:num_seqs]]
        p = plan_split_kv(
            lens,
            self.h_k,
            self.n_tiles(q_len),
            self.sm_count,
            ctas_per_sm=self.ctas(q_len),
            max_splits=self.max_splits,
            pad_to=self._cap,
            rebalance=self.rebalance,
        )
        work_h = torch.from_numpy(p.work_array()).pin_memory() if self.device.type == "cuda" else torch.from_numpy(p.work_array())
        ns_h = torch.tensor(p.n_splits, dtype=torch.int32)
        if self.device.type == "cuda":
            ns_h = ns_h.pin_memory()
        self.work_buf.copy_(work_h, non_blocking=True)
        self.nsplit_buf[:num_seqs].copy_(ns_h, non_blocking=True)
        real = sum(1 for w in p.work if w[2] > w[1])
        return StepPlan(
            num_seqs=num_seqs,
            q_len=q_len,
            n_q=q_len * self.h_r,
            num_work=self._cap if fixed_grid else real,
            # a fixed grid (graph capture) always launches the combine: it skips
            # sequences with one chunk, so any later plan replays correctly
            with_reduction=p.max_splits_used > 1 or fixed_grid,
            block_table=block_table,
            seq_lens=seq_lens,
            work=self.work_buf,
            n_splits=self.nsplit_buf[:num_seqs],
            chunk_tiles=p.chunk_tiles,
            num_chunks=real,
            causal=causal or q_len == 1,
            tile_jobs=sum(-(-L // 128) for L in lens) * self.h_k,
        )

    # ---------------------------------------------------------------- launch
    def decode_args(
        self,
        plan: StepPlan,
        query: torch.Tensor,
        out: torch.Tensor,
        k_cache: torch.Tensor,
        v_cache: torch.Tensor,
        k_scale: torch.Tensor,
        v_scale: torch.Tensor,
        softmax_scale: float,
        q_mul: torch.Tensor | None = None,
        o_mul: torch.Tensor | None = None,
        lse: torch.Tensor | None = None,
        k_scales: torch.Tensor | None = None,
        v_scales: torch.Tensor | None = None,
    ) -> _lib.DecodeArgs:
        b, ql = plan.num_seqs, plan.q_len
        tokens = b * ql
        q3 = query[:tokens]
        if q3.dim() == 2:
            q3 = q3.view(q3.shape[0], self.h_q, self.d)
        o3 = out[:tokens]
        if o3.dim() == 2:
            o3 = o3.view(o3.shape[0], self.h_q, self.d)
        if q3.stride(2) != 1 or o3.stride(2) != 1:
            raise ValueError("query / output head dim must be contiguous")
        if k_cache.dtype not in (torch.uint8, torch.float8_e4m3fn) or v_cache.dtype != k_cache.dtype:
            raise TypeError(f"KV views must be uint8 / float8_e4m3fn, got {k_cache.dtype}")
        if k_cache.shape[1] != self.page_size or k_cache.shape[3] != self.kv_row_bytes:
            raise ValueError(f"KV view {tuple(k_cache.shape)} does not match page {self.page_size} x row {self.kv_row_bytes}")
        ks, vs = kv_byte_strides(k_cache), kv_byte_strides(v_cache)
        for t in (q_mul, o_mul):
            if t is not None and (t.dtype != torch.float32 or not t.is_contiguous() or t.numel() != self.h_q * self.d):
                raise ValueError("q_mul / o_mul must be contiguous fp32 (h_q, d)")
        bt = plan.block_table
        if bt.dtype != torch.int32 or bt.stride(1) != 1 or plan.seq_lens.dtype != torch.int32:
            raise TypeError("block_table / seq_lens must be int32 with contiguous rows")
        a = _lib.DecodeArgs()
        a.num_seqs, a.q_len, a.h_q, a.h_k = b, ql, self.h_q, self.h_k
        a.head_size, a.page_size, a.kv_format = self.d, self.page_size, _lib.KV_FORMATS[self.kv_format]
        a.q, a.q_dtype, a.q_stride_tok, a.q_stride_head = q3.data_ptr(), dtype_code(q3.dtype), q3.stride(0), q3.stride(1)
        a.o, a.o_dtype, a.o_stride_tok, a.o_stride_head = o3.data_ptr(), dtype_code(o3.dtype), o3.stride(0), o3.stride(1)
        a.k_cache, a.v_cache = k_cache.data_ptr(), v_cache.data_ptr()
        a.k_stride_page, a.k_stride_row, a.k_stride_head = ks
        a.v_stride_page, a.v_stride_row, a.v_stride_head = vs
        a.num_pages = k_cache.shape[0]
        a.block_table, a.block_table_stride = bt.data_ptr(), bt.stride(0)
        a.seq_lens = plan.seq_lens.data_ptr()
        a.work, a.num_work = plan.work.data_ptr(), plan.num_work
        a.n_splits, a.max_splits = plan.n_splits.data_ptr(), self.max_splits
        a.o_part, a.lse_part, a.part_seqs = self.o_part.data_ptr(), self.lse_part.data_ptr(), self.max_num_seqs
        a.lse = _ptr(lse)
        a.k_descale, a.k_descale_mode = k_scale.data_ptr(), descale_mode(k_scale, b, self.h_k)
        a.v_descale, a.v_descale_mode = v_scale.data_ptr(), descale_mode(v_scale, b, self.h_k)
        a.q_mul, a.o_mul = _ptr(q_mul), _ptr(o_mul)
        a.softmax_scale = float(softmax_scale)
        a.causal = int(plan.causal)
        a.with_combine = int(plan.with_reduction)
        a.kernel = self.kernel
        a.status = self.status.data_ptr()
        a.merge_counters = self.merge_counters.data_ptr() if self.merges(plan) else None
        set_scale_views(a, k_scales, v_scales, k_cache.shape[0], self.page_size, self.h_k, self.d, self.kv_format)
        return a

    def merges(self, plan: StepPlan) -> bool:
        """Whether this plan's launches carry the in-kernel merge counters."""
        if self.fused_merge is not None:
            return bool(self.fused_merge)
        return plan.tile_jobs <= 16 * self.sm_count

    def merges_in_kernel(self, args: _lib.DecodeArgs) -> bool:
        """True when mj_decode merges the split partials inside the decode
        launch (the one-warpgroup tensor-core variants given counters), so no
        separate mj_combine launch is needed."""
        return (bool(args.merge_counters) and self.kernel_name(args) == "decode_tc"
                and (args.q_len * (self.h_q // self.h_k) <= 16 or self.d == 256) and args.max_splits <= 16)

    def run(
        self,
        plan: StepPlan,
        query: torch.Tensor,  # (>= b*q_len, h_q, d) or (>= b*q_len, h_q*d), any token stride
        out: torch.Tensor,  # same layouts, written in place
        k_cache: torch.Tensor,  # (num_pages, page_size, h_k, row) logical view, fp8 / uint8
        v_cache: torch.Tensor,
        k_scale: torch.Tensor,  # fp32: 1 elem, (h_k,) or (b, h_k)
        v_scale: torch.Tensor,
        softmax_scale: float,
        q_mul: torch.Tensor | None = None,  # (h_q, d) fp32: e2m3 K channel scales folded into Q
        o_mul: torch.Tensor | None = None,  # (h_q, d) fp32: e2m3 V channel scales on O
        lse: torch.Tensor | None = None,  # optional (b*q_len, h_q) fp32
        k_scales: torch.Tensor | None = None,  # nvfp4: (num_pages, page_size, h_k, d / 16) uint8 views
        v_scales: torch.Tensor | None = None,
    ):
        a = self.decode_args(plan, query, out, k_cache, v_cache, k_scale, v_scale, softmax_scale, q_mul, o_mul, lse,
                             k_scales, v_scales)
        _lib.decode(a, _stream(self.device))
        return out

    def kernel_name(self, args: _lib.DecodeArgs) -> str:
        """The decode kernel mj_decode launches for these arguments."""
        return _lib.KERNEL_NAMES[_lib.decode_kernel(args)]

    def check_status(self) -> None:
        """Raise if a kernel flagged a bad page / split index or a wait that
        ran out (synchronizes). The status word is cleared, and so are the
        in-kernel merge counters: a job that stopped early never counted
        itself in, and a stale count would let the next launch merge before
        every split had written its partials."""
        code = int(self.status.item())
        if code != _lib.MJ_DEV_OK:
            self.status.zero_()
            self.merge_counters.zero_()
            raise _lib.MjolnirError(_lib.MJ_ERR_DEVICE, f"device status {code}")


# reference-compatible name
T5DecodeRunner = DecodeRunner
Runner = DecodeRunner
