"""Bit-exact CPU restatement of the KV-cache quantizers (test infrastructure).

e2m3 ("fp6_e2m3"): sign | 2-bit exponent | 3-bit mantissa, exponent bias 1, no
inf/nan, magnitudes 0 .. 7.5.  Restates
  * ``minifloat_table`` / ``minifloat_quantize`` (reference
    ``src/mjolnir/mjolnir/quant.py:21-47``): round to nearest, saturating at
    7.5, ties to the SMALLER magnitude (``pick_lo = (ax - lo) <= (hi - ax)``,
    ``quant.py:43``), the sign bit only when the magnitude code is non-zero
    (``quant.py:45``);
  * ``pack_subbyte(codes, 6)`` (``quant.py:50-65``): 4 codes ``c0..c3`` form the
    24-bit little-endian word ``c0 | c1<<6 | c2<<12 | c3<<18`` stored as 3 bytes;
  * ``quantize_rows_reference`` (``src/mjolnir/mjolnir/kvfp6.py:342-355``): the
    input is divided by its scale in fp32 first (per tensor, per KV head, or per
    (KV head, channel));
  * ``decode_rows_reference`` (``kvfp6.py:358-365``): packed bytes -> values.

fp8-e4m3: ``(x.float() / scale)`` rounded to nearest-even e4m3, saturating at
+-448 (the cache write of ``arch/thor/harness.py:588-590`` with the saturation
of vLLM's ``reshape_and_cache_flash``, which ``backend.py:474-483`` calls; the
torch cast alone turns |x| >= 464 into NaN, so the clamp defines saturation).
NaN stays NaN (byte 0x7F / 0xFF keeps its sign bit as torch does).
"""

from __future__ import annotations

import numpy as np

E2M3_MAX = 7.5
FP8_MAX = 448.0


def e2m3_table() -> np.ndarray:
    """(64,) float32: the value of every e2m3 code (code = sign<<5 | e<<3 | m).

    Built from the bit definition: e == 0 -> m/8 (subnormal), else
    (1 + m/8) * 2**(e - 1)."""
    vals = []
    for code in range(64):
        sign = -1.0 if code >> 5 else 1.0
        e = (code >> 3) & 3
        m = code & 7
        v = m / 8.0 if e == 0 else (1.0 + m / 8.0) * 2.0 ** (e - 1)
        vals.append(sign * v)
    return np.asarray(vals, dtype=np.float32)


_TABLE = e2m3_table()
_POS = _TABLE[:32].copy()  # non-negative half, ascending


def e2m3_codes(x: np.ndarray) -> np.ndarray:
    """float32 (already divided by the scale) -> uint8 e2m3 codes.

    Same decision procedure as the reference: ``ax = min(|x|, 7.5)`` (NaN stays
    NaN), ``idx`` = first table entry >= ax (NaN -> past the end), compare the
    two neighbours in fp32, ties to the lower one."""
    x = np.asarray(x, dtype=np.float32)
    ax = np.abs(x)
    ax = np.where(ax > np.float32(E2M3_MAX), np.float32(E2M3_MAX), ax)  # NaN stays NaN
    idx = np.searchsorted(_POS, ax, side="left")  # first pos >= ax; NaN -> 32
    lo = np.clip(idx - 1, 0, 31)
    hi = np.clip(idx, 0, 31)
    with np.errstate(invalid="ignore"):
        pick_lo = (ax - _POS[lo]) <= (_POS[hi] - ax)  # NaN compares False -> hi
    mag = np.where(pick_lo, lo, hi).astype(np.int64)
    neg = (x < 0) & (_POS[mag] > 0)
    return (mag + neg.astype(np.int64) * 32).astype(np.uint8)


def pack6(codes: np.ndarray) -> np.ndarray:
    """(..., d) uint8 codes -> (..., 3d/4) uint8: little-endian 6-bit stream."""
    c = np.asarray(codes).astype(np.uint32)
    d = c.shape[-1]
    assert d % 4 == 0
    c = c.reshape(*c.shape[:-1], d // 4, 4)
    w = c[..., 0] | (c[..., 1] << 6) | (c[..., 2] << 12) | (c[..., 3] << 18)
    out = np.stack([w & 0xFF, (w >> 8) & 0xFF, (w >> 16) & 0xFF], axis=-1)
    return out.reshape(*c.shape[:-2], d // 4 * 3).astype(np.uint8)


def unpack6(packed: np.ndarray, d: int) -> np.ndarray:
    """(..., 3d/4) uint8 -> (..., d) uint8 codes."""
    b = np.asarray(packed).astype(np.uint32).reshape(*packed.shape[:-1], d // 4, 3)
    w = b[..., 0] | (b[..., 1] << 8) | (b[..., 2] << 16)
    codes = np.stack([(w >> (6 * k)) & 63 for k in range(4)], axis=-1)
    return codes.reshape(*packed.shape[:-1], d).astype(np.uint8)


def _expand_scale(scale, h_k: int, d: int) -> np.ndarray:
    """Scale (1 | (h_k,) | (h_k, d)) -> broadcastable (h_k, 1|d) float32, the
    same interpretation as ``kvfp6.quantize_rows_reference``."""
    s = np.asarray(scale, dtype=np.float32)
    if s.size == h_k * d and d > 1:
        return s.reshape(h_k, d)
    s = s.reshape(-1)
    if s.size == 1:
        s = np.repeat(s, h_k)
    return s.reshape(h_k, 1)


def quantize_rows_e2m3(x: np.ndarray, scale) -> np.ndarray:
    """(..., h_k, d) float32 -> (..., h_k, 3d/4) packed e2m3 bytes."""
    x = np.asarray(x, dtype=np.float32)
    h_k, d = x.shape[-2], x.shape[-1]
    with np.errstate(over="ignore", invalid="ignore", divide="ignore"):
        q = (x / _expand_scale(scale, h_k, d)).astype(np.float32)  # IEEE fp32 division
    return pack6(e2m3_codes(q))


def decode_rows_e2m3(packed: np.ndarray, d: int) -> np.ndarray:
    """packed (..., 3d/4) uint8 -> code values (..., d) float32 (no scale)."""
    return _TABLE[unpack6(packed, d).astype(np.int64)]


# ---------------------------------------------------------------------------
# fp8 e4m3 (OCP "e4m3fn": bias 7, no inf, NaN = S.1111.111, max 448)
# ---------------------------------------------------------------------------
def e4m3_table() -> np.ndarray:
    """(256,) float32: value of every e4m3fn byte (NaN for 0x7F / 0xFF)."""
    vals = []
    for b in range(256):
        sign = -1.0 if b >> 7 else 1.0
        e = (b >> 3) & 15
        m = b & 7
        if e == 15 and m == 7:
            vals.append(np.nan)
            continue
        v = (m / 8.0) * 2.0**-6 if e == 0 else (1.0 + m / 8.0) * 2.0 ** (e - 7)
        vals.append(sign * v)
    return np.asarray(vals, dtype=np.float32)


_E4M3 = e4m3_table()
_E4M3_POS = _E4M3[:127].copy()  # 0 .. 448 ascending (bytes 0x00 .. 0x7E)


def e4m3_bytes(x: np.ndarray) -> np.ndarray:
    """float32 -> e4m3fn bytes: round to nearest, ties to even, saturate +-448.

    Ties to even on the byte code: the lower neighbour wins a tie when its
    code is even."""
    x = np.asarray(x, dtype=np.float32)
    nan = np.isnan(x)
    ax = np.minimum(np.abs(np.where(nan, 0, x)), np.float32(FP8_MAX))
    idx = np.searchsorted(_E4M3_POS, ax, side="left")  # first pos >= ax
    lo = np.clip(idx - 1, 0, 126)
    hi = np.clip(idx, 0, 126)
    dl = ax.astype(np.float64) - _E4M3_POS[lo].astype(np.float64)  # exact differences
    dh = _E4M3_POS[hi].astype(np.float64) - ax.astype(np.float64)
    pick_lo = (dl < dh) | ((dl == dh) & (lo % 2 == 0))
    mag = np.where(pick_lo, lo, hi).astype(np.int64)
    mag = np.where(_E4M3_POS[hi] == ax, hi, mag)
    sign = np.signbit(x).astype(np.int64) << 7
    out = (mag | sign).astype(np.int64)
    out = np.where(nan, 0x7F | sign, out)
    return out.astype(np.uint8)


def quantize_rows_fp8(x: np.ndarray, scale) -> np.ndarray:
    """(..., h_k, d) float32 -> (..., h_k, d) e4m3 bytes; scale per tensor,
    per KV head or per (KV head, channel)."""
    x = np.asarray(x, dtype=np.float32)
    h_k, d = x.shape[-2], x.shape[-1]
    with np.errstate(over="ignore", invalid="ignore", divide="ignore"):
        q = (x / _expand_scale(scale, h_k, d)).astype(np.float32)
    return e4m3_bytes(q)


def decode_fp8(b: np.ndarray) -> np.ndarray:
    return _E4M3[np.asarray(b).astype(np.int64)]


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """uint16 bf16 bit patterns -> float32 (exact)."""
    return (np.asarray(bits).astype(np.uint32) << 16).view(np.float32)


def scale_mode(n: int, h_k: int, d: int) -> int:
    """0: per tensor, 1: per KV head, 2: per (KV head, channel) -- the same
    rule as ``kvfp6._scale_mode`` (``kvfp6.py:328-335``)."""
    if n == h_k * d and d > 1 and (h_k > 1 or n > 1):
        return 2
    assert n in (1, h_k)
    return 1 if n == h_k and h_k > 1 else 0


def expand_rows_e4m3(packed: np.ndarray, d: int, ratio=None, fmt: str = "e2m3", sc=None) -> np.ndarray:
    """packed narrow rows (..., h_k, row) -> e4m3 bytes (..., h_k, d):
    ``e4m3(code_value * ratio)`` with the product in float32, round to nearest
    even, saturating at +-448; ratio None gives the code values exactly (e2m3,
    e2m1; e3m2 codes round). nvfp4's code value is its kernel value
    e4m3(code * scale * 2^-3) from the scale bytes ``sc``. Restates the page
    expansion of reference ``kvfp6.py:157-205`` (the RATIO branch of
    ``_expand_kernel``: value LUT x ratio, then the fp8 cast)."""
    if fmt == "nvfp4":
        vals = decode_rows_nvfp4(packed, sc, d).astype(np.float32)
    elif fmt == "e2m3":
        vals = decode_rows_e2m3(packed, d).astype(np.float32)
    else:
        vals = decode_rows_narrow(packed, d, fmt).astype(np.float32)
    if ratio is not None:
        h_k = packed.shape[-2]
        vals = (vals * _expand_scale(ratio, h_k, d)).astype(np.float32)
    return e4m3_bytes(vals)


# ---------------------------------------------------------------------------
# The other narrow formats of the reference's kernel harness (quant.py:14-47,
# arch/thor/decode.py:108-115): e3m2 (6-bit, bias 3, max 28) and e2m1 (4-bit,
# bias 1, max 6); same rounding rule as e2m3 (nearest, ties to the smaller
# magnitude, saturating, no -0), 6-bit codes packed 4 per 3 bytes, 4-bit
# codes 2 per byte, low nibble first (quant.py:50-65).
# ---------------------------------------------------------------------------
MINIFLOAT = {"e3m2": (3, 2, 3), "e2m3": (2, 3, 1), "e2m1": (2, 1, 1)}  # (exponent bits, mantissa bits, bias)
BITS = {"e3m2": 6, "e2m3": 6, "e2m1": 4}


def minifloat_table(fmt: str) -> np.ndarray:
    """Value of every code of a narrow format (code = sign | exponent | mantissa)."""
    eb, mb, bias = MINIFLOAT[fmt]
    vals = []
    for code in range(1 << (1 + eb + mb)):
        sign = -1.0 if code >> (eb + mb) else 1.0
        e = (code >> mb) & ((1 << eb) - 1)
        m = code & ((1 << mb) - 1)
        v = (m / (1 << mb)) * 2.0 ** (1 - bias) if e == 0 else (1 + m / (1 << mb)) * 2.0 ** (e - bias)
        vals.append(sign * v)
    return np.asarray(vals, dtype=np.float32)


def minifloat_codes(x: np.ndarray, fmt: str) -> np.ndarray:
    """float32 (already divided by the scale) -> uint8 codes of `fmt` (the
    procedure of e2m3_codes on that format's table)."""
    table = minifloat_table(fmt)
    pos = table[: len(table) // 2]
    half = len(pos)
    x = np.asarray(x, dtype=np.float32)
    ax = np.abs(x)
    ax = np.where(ax > pos[-1], pos[-1], ax)
    idx = np.searchsorted(pos, ax, side="left")
    lo = np.clip(idx - 1, 0, half - 1)
    hi = np.clip(idx, 0, half - 1)
    with np.errstate(invalid="ignore"):
        pick_lo = (ax - pos[lo]) <= (pos[hi] - ax)
    mag = np.where(pick_lo, lo, hi).astype(np.int64)
    neg = (x < 0) & (pos[mag] > 0)
    return (mag + neg.astype(np.int64) * half).astype(np.uint8)


def pack4(codes: np.ndarray) -> np.ndarray:
    """(..., d) 4-bit codes -> (..., d/2) bytes, low nibble first."""
    c = np.asarray(codes).astype(np.uint8)
    d = c.shape[-1]
    assert d % 2 == 0
    c = c.reshape(*c.shape[:-1], d // 2, 2)
    return (c[..., 0] | (c[..., 1] << 4)).astype(np.uint8)


def unpack4(packed: np.ndarray, d: int) -> np.ndarray:
    b = np.asarray(packed).astype(np.uint8)
    codes = np.stack([b & 15, b >> 4], axis=-1)
    return codes.reshape(*packed.shape[:-1], d).astype(np.uint8)


def quantize_rows_narrow(x: np.ndarray, scale, fmt: str) -> np.ndarray:
    """(..., h_k, d) float32 -> packed (..., h_k, d * bits / 8) bytes of `fmt`."""
    x = np.asarray(x, dtype=np.float32)
    h_k, d = x.shape[-2], x.shape[-1]
    with np.errstate(over="ignore", invalid="ignore", divide="ignore"):
        q = (x / _expand_scale(scale, h_k, d)).astype(np.float32)
    codes = minifloat_codes(q, fmt)
    return pack6(codes) if BITS[fmt] == 6 else pack4(codes)


def decode_rows_narrow(packed: np.ndarray, d: int, fmt: str) -> np.ndarray:
    """Packed rows of `fmt` -> code values (..., d) float32 (no scale)."""
    codes = unpack6(packed, d) if BITS[fmt] == 6 else unpack4(packed, d)
    return minifloat_table(fmt)[codes.astype(np.int64)]


# ---------------------------------------------------------------------------
# nvfp4 (reference quant.py:9-10, :68-84; the kernel-side conversion of
# arch/thor/decode.py:980-1030 and the harness pool of
# arch/thor/harness.py:579-586): e2m1 codes packed two per byte (low nibble
# first), one e4m3 scale per group of 16 elements along d, one fp32 global
# scale gs. The quantizer, in fp32 with gs rounded to fp32 as torch does for a
# Python scalar operand:
#   sc   = e4m3(min(amax_group / 6 / gs, 448))       (round to nearest even)
#   q    = x / (value(sc) * gs)   (0 where that product is 0)
#   code = e2m1(q)                (the narrow formats' rounding rule)
# The tensor cores multiply e4m3(value(code) * value(sc) * 2^-3) -- exact
# product, one rounding to e4m3 -- with the descale gs * 2^3.
# ---------------------------------------------------------------------------
NVFP4_GROUP = 16
NVFP4_SHIFT = 0.125


def nvfp4_global_scale(x: np.ndarray) -> float:
    """gs = max(amax|x|, 1e-12) / (6 * 448), the reference's per-tensor choice
    (the amax in fp32, the division in double)."""
    amax = np.float32(np.max(np.abs(np.asarray(x, dtype=np.float32))))
    return float(max(amax, np.float32(1e-12))) / (6.0 * 448.0)


def nvfp4_quantize(x: np.ndarray, gs: float | None = None, group: int = NVFP4_GROUP):
    """(..., d) float32 -> (codes (..., d) uint8, scale bytes (..., d/group) uint8,
    gs, kernel e4m3 bytes (..., d) uint8, descale gs / 2^-3) -- the outputs of
    the reference's ``nvfp4_quantize`` with the kernel values as e4m3 bytes.
    gs None computes the reference's per-tensor global scale."""
    x = np.asarray(x, dtype=np.float32)
    if gs is None:
        gs = nvfp4_global_scale(x)
    g32 = np.float32(gs)
    *lead, d = x.shape
    xg = x.reshape(*lead, d // group, group)
    amax_g = np.max(np.abs(xg), axis=-1)
    with np.errstate(over="ignore", invalid="ignore", divide="ignore"):
        sc_f = ((amax_g / np.float32(6.0)).astype(np.float32) / g32).astype(np.float32)
        sc_f = np.where(sc_f > np.float32(FP8_MAX), np.float32(FP8_MAX), sc_f)  # NaN stays NaN
        sc = e4m3_bytes(sc_f)
        scf = decode_fp8(sc)
        denom = (scf * g32).astype(np.float32)[..., None]
        q = np.where(denom > 0, xg / np.maximum(denom, np.float32(1e-30)), np.float32(0)).astype(np.float32)
    codes = minifloat_codes(q, "e2m1").reshape(*lead, d)
    kern = nvfp4_kernel_bytes(codes, sc, group)
    return codes, sc, gs, kern, gs / NVFP4_SHIFT


def nvfp4_kernel_bytes(codes: np.ndarray, sc: np.ndarray, group: int = NVFP4_GROUP) -> np.ndarray:
    """e2m1 codes (..., d) and scale bytes (..., d/group) -> the e4m3 bytes the
    tensor cores read: e4m3(value(code) * value(sc) * 2^-3)."""
    codes = np.asarray(codes).astype(np.int64)
    *lead, d = codes.shape
    lut = minifloat_table("e2m1")
    scf = decode_fp8(np.asarray(sc, dtype=np.uint8)).astype(np.float32)
    v = (lut[codes].reshape(*lead, d // group, group) * scf[..., None]).astype(np.float32)
    v = (v * np.float32(NVFP4_SHIFT)).astype(np.float32)
    return e4m3_bytes(v.reshape(*lead, d))


def quantize_rows_nvfp4(x: np.ndarray, gs) -> tuple[np.ndarray, np.ndarray]:
    """(..., h_k, d) float32 -> (packed codes (..., h_k, d/2), scale bytes
    (..., h_k, d/16)) under a global scale per tensor (1 element) or per KV head
    ((h_k,)) -- the quantize-on-write of an nvfp4 cache."""
    x = np.asarray(x, dtype=np.float32)
    g = np.asarray(gs, dtype=np.float64).reshape(-1)
    if g.size == 1:
        codes, sc, *_ = nvfp4_quantize(x, float(g[0]))
        return pack4(codes), sc
    h_k = x.shape[-2]
    assert g.size == h_k, "nvfp4 global scale: 1 element or one per KV head"
    packed = np.empty(x.shape[:-1] + (x.shape[-1] // 2,), dtype=np.uint8)
    sc = np.empty(x.shape[:-1] + (x.shape[-1] // NVFP4_GROUP,), dtype=np.uint8)
    for h in range(h_k):
        c, s, *_ = nvfp4_quantize(x[..., h, :], float(g[h]))
        packed[..., h, :] = pack4(c)
        sc[..., h, :] = s
    return packed, sc


def decode_rows_nvfp4(packed: np.ndarray, sc: np.ndarray, d: int) -> np.ndarray:
    """Packed nvfp4 rows and their scale bytes -> the kernel values (float32,
    before the gs * 2^3 descale)."""
    return decode_fp8(nvfp4_kernel_bytes(unpack4(packed, d), sc))
