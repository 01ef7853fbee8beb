"""Quantize-on-write into the paged KV cache (fp8-e4m3 and packed e2m3).

Format (GoBrrr-ai/mjolnir ``src/mjolnir/mjolnir/kvfp6.py:1-20``): one e2m3 code
per element (sign | 2-bit exponent | 3-bit mantissa, bias 1, no inf/nan,
values 0 .. +-7.5), packed little-endian, 4 codes in 3 bytes. A K (or V) row
of d elements is ``d * 3 / 4`` bytes; vLLM's page cell is ``K row | V row``
(``(B, H, N, 2 * d * 3 / 4)`` uint8 in the reference's layout, any stride
order). Values are ``code_value * scale`` with a static scale per tensor, per
KV head or per (KV head, channel).

* :func:`write_kv` -- the reference's e2m3 cache write (``kvfp6.py:218-254``);
* :func:`reshape_and_cache` -- the same kernel on any logical K / V views, for
  both formats (the fp8 path replaces vLLM's ``reshape_and_cache_flash``
  that the reference's ``do_kv_cache_update`` calls, ``backend.py:474-483``).

Both run the sm_100a ``mj_cache_write`` kernel; results are bit-identical to
the reference quantizers (``quant.py:34-65``, ``kvfp6.py:342-355``).
"""

from __future__ import annotations

import torch

from . import _lib
from .runner import _stream, dtype_code, kv_byte_strides, row_bytes as _row_bytes, scale_mode, set_scale_views

E2M3_MAX = 7.5
BITS = 6


def row_bytes(head_size: int) -> int:
    """Bytes of one packed e2m3 K (or V) row."""
    return _row_bytes(head_size, "e2m3")


def cache_write_args(
    key: torch.Tensor,
    value: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
    k_scale: torch.Tensor,
    v_scale: torch.Tensor,
    kv_format: str,
    status: torch.Tensor | None = None,
    k_scales: torch.Tensor | None = None,
    v_scales: torch.Tensor | None = None,
) -> _lib.CacheWriteArgs:
    """Validated ``mj_cache_write`` arguments for these tensors (they must
    stay alive while the returned struct is used)."""
    T = slot_mapping.shape[0]
    _, h_k, d = key.shape
    if key.stride(2) != 1 or value.stride(2) != 1:
        raise ValueError("key / value head dim must be contiguous")
    if key.shape[0] < T or value.shape[0] < T:
        raise ValueError("fewer key/value rows than slots")
    rb = _row_bytes(d, kv_format)
    for t in (k_cache, v_cache):
        if t.dim() != 4 or t.shape[2] != h_k or t.shape[3] != rb:
            raise ValueError(f"cache view {tuple(t.shape)} is not (pages, page_size, {h_k}, {rb})")
        if t.element_size() != 1:
            raise TypeError("cache views must be byte views (uint8 / float8)")
    if slot_mapping.dtype != torch.int64:
        raise TypeError("slot_mapping must be int64")
    if k_scale.dtype != torch.float32 or v_scale.dtype != torch.float32:
        raise TypeError("KV scales must be fp32")
    a = _lib.CacheWriteArgs()
    a.key, a.value, a.src_dtype = key.data_ptr(), value.data_ptr(), dtype_code(key.dtype)
    if value.dtype != key.dtype:
        raise TypeError("key and value must share a dtype")
    a.num_tokens, a.h_k, a.head_size = T, h_k, d
    a.key_stride_tok, a.key_stride_head = key.stride(0), key.stride(1)
    a.value_stride_tok, a.value_stride_head = value.stride(0), value.stride(1)
    a.k_cache, a.v_cache = k_cache.data_ptr(), v_cache.data_ptr()
    a.k_stride_page, a.k_stride_row, a.k_stride_head = kv_byte_strides(k_cache)
    a.v_stride_page, a.v_stride_row, a.v_stride_head = kv_byte_strides(v_cache)
    a.num_pages, a.page_size = k_cache.shape[0], k_cache.shape[1]
    a.kv_format = _lib.KV_FORMATS[kv_format]
    a.slot_mapping = slot_mapping.data_ptr()
    a.k_scale, a.k_scale_mode = k_scale.data_ptr(), scale_mode(k_scale, h_k, d)
    a.v_scale, a.v_scale_mode = v_scale.data_ptr(), scale_mode(v_scale, h_k, d)
    a.status = None if status is None else status.data_ptr()
    set_scale_views(a, k_scales, v_scales, k_cache.shape[0], k_cache.shape[1], h_k, d, kv_format)
    return a


def reshape_and_cache(
    key: torch.Tensor,  # (>= T, h_k, d) bf16/fp16/fp32, d contiguous
    value: torch.Tensor,
    k_cache: torch.Tensor,  # logical (pages, page_size, h_k, row) uint8 / float8 view
    v_cache: torch.Tensor,
    slot_mapping: torch.Tensor,  # (T,) int64 (int32 accepted), -1 = padding
    k_scale: torch.Tensor,  # fp32: 1 elem, (h_k,) or (h_k, d)
    v_scale: torch.Tensor,
    kv_format: str,
    status: torch.Tensor | None = None,
    k_scales: torch.Tensor | None = None,  # nvfp4: (pages, page_size, h_k, d / 16) uint8 group-scale views
    v_scales: torch.Tensor | None = None,
) -> None:
    """Quantize, pack and scatter T new K/V rows into the cache views (nvfp4:
    k_scale / v_scale are the global scales, per tensor or per KV head, and the
    group scale bytes go to k_scales / v_scales)."""
    if slot_mapping.shape[0] == 0:
        return
    if slot_mapping.dtype != torch.int64:
        slot_mapping = slot_mapping.to(torch.int64)
    k_scale = k_scale.to(torch.float32).contiguous()
    v_scale = v_scale.to(torch.float32).contiguous()
    a = cache_write_args(key, value, k_cache, v_cache, slot_mapping, k_scale, v_scale, kv_format, status,
                         k_scales, v_scales)
    _lib.cache_write(a, _stream(key.device))


def write_kv(
    key: torch.Tensor,  # (>= T, h_k, d) bf16/fp16, d contiguous
    value: torch.Tensor,
    kv_cache: torch.Tensor,  # (B, h_k, N, 2 * row_bytes) uint8 layer view, unit last stride
    slot_mapping: torch.Tensor,  # (T,) int, -1 = padding
    k_scale: torch.Tensor,  # fp32: 1 elem, (h_k,) or (h_k, d)
    v_scale: torch.Tensor,
) -> None:
    """Quantize + pack + scatter K/V rows of T tokens into the e2m3 cache
    (the reference's ``kvfp6.write_kv`` contract, ``kvfp6.py:338-374``)."""
    T = slot_mapping.shape[0]
    if T == 0:
        return
    _, h_k, d = key.shape
    _, H, N, Cb = kv_cache.shape
    rb = row_bytes(d)
    if not (h_k == H and 2 * rb == Cb and kv_cache.stride(3) == 1 and kv_cache.dtype == torch.uint8):
        raise ValueError(f"kv_cache {tuple(kv_cache.shape)} is not (B, {h_k}, N, {2 * rb}) uint8")
    k_view = kv_cache[..., :rb].transpose(1, 2)
    v_view = kv_cache[..., rb:].transpose(1, 2)
    reshape_and_cache(key, value, k_view, v_view, slot_mapping, k_scale, v_scale, "e2m3")


def expand_pages(
    k_cache: torch.Tensor,  # narrow logical (pages, page_size, h_k, row_bytes) uint8 view
    v_cache: torch.Tensor,
    src_pages: torch.Tensor,  # (P,) int32: cache page of each output page
    k_out: torch.Tensor,  # e4m3 logical (>= P, page_size, h_k, d) uint8 / float8 view
    v_out: torch.Tensor,
    k_ratio: torch.Tensor | None = None,  # fp32: 1 elem, (h_k,) or (h_k, d)
    v_ratio: torch.Tensor | None = None,
    status: torch.Tensor | None = None,
    kv_format: str = "e2m3",
    k_scales: torch.Tensor | None = None,  # nvfp4: (pages, page_size, h_k, d / 16) uint8 group-scale views
    v_scales: torch.Tensor | None = None,
) -> None:
    """Expand P cache pages (K and V) to e4m3 bytes in output pages 0..P-1.

    Without ratios the bytes are the code values exactly (e2m3, e2m1; e3m2
    rounds to e4m3; nvfp4 gives the e4m3 values its tensor-core MMA reads and
    keeps the gs * 2^3 descale). With per-channel scales s_c and a per-head
    descale S of the reader, ratio = s_c / S makes each byte
    e4m3(code * s_c / S); a reader without descales takes ratio = s_c
    (reference ``kvfp6.py:257-335``)."""
    P = int(src_pages.shape[0])
    if P == 0:
        return
    if kv_format not in ("e2m3", "e3m2", "e2m1", "nvfp4"):
        raise ValueError(f"page expansion reads a narrow format, not {kv_format!r}")
    _, N, h_k, rb = k_cache.shape
    d = rb * 2 if kv_format in ("e2m1", "nvfp4") else rb * 4 // 3
    if rb != _row_bytes(d, kv_format) or v_cache.shape != k_cache.shape:
        raise ValueError(f"{kv_format} views {tuple(k_cache.shape)} / {tuple(v_cache.shape)}")
    for t in (k_out, v_out):
        if t.dim() != 4 or t.shape[0] < P or tuple(t.shape[1:]) != (N, h_k, d) or t.element_size() != 1:
            raise ValueError(f"output view {tuple(t.shape)} is not (>= {P}, {N}, {h_k}, {d}) bytes")
    if src_pages.dtype != torch.int32:
        src_pages = src_pages.to(torch.int32)
    src_pages = src_pages.contiguous()
    a = _lib.ExpandArgs()
    a.k_cache, a.v_cache = k_cache.data_ptr(), v_cache.data_ptr()
    a.k_stride_page, a.k_stride_row, a.k_stride_head = kv_byte_strides(k_cache)
    a.v_stride_page, a.v_stride_row, a.v_stride_head = kv_byte_strides(v_cache)
    a.num_pages, a.page_size, a.h_k, a.head_size = k_cache.shape[0], N, h_k, d
    a.src_pages, a.num_out_pages = src_pages.data_ptr(), P
    a.k_out, a.v_out = k_out.data_ptr(), v_out.data_ptr()
    a.ko_stride_page, a.ko_stride_row, a.ko_stride_head = kv_byte_strides(k_out)
    a.vo_stride_page, a.vo_stride_row, a.vo_stride_head = kv_byte_strides(v_out)
    keep = []
    for side, r in (("k", k_ratio), ("v", v_ratio)):
        if r is None:
            ptr, mode = None, _lib.MJ_SCALE_TENSOR
        else:
            r = r.to(torch.float32).contiguous()
            keep.append(r)
            ptr, mode = r.data_ptr(), scale_mode(r, h_k, d)
        setattr(a, f"{side}_ratio", ptr)
        setattr(a, f"{side}_ratio_mode", mode)
    a.status = None if status is None else status.data_ptr()
    a.kv_format = _lib.KV_FORMATS[kv_format]
    set_scale_views(a, k_scales, v_scales, k_cache.shape[0], N, h_k, d, kv_format)
    _lib.expand_pages(a, _stream(k_cache.device))
