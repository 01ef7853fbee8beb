"""vLLM attention backend: the B200 paged decode behind vLLM's backend surface.

The backend class subclasses a stock vLLM backend, the *fallback*
(``MJOLNIR_ATTN_FALLBACK``, default FLASHINFER, which reads fp8 KV on
sm_100), and inherits its KV-cache layout, prefill and mixed-batch path. Two
things change, as in the reference (GoBrrr-ai/mjolnir
``src/mjolnir/mjolnir/backend.py:1-32``):

* the metadata builder (``mjolnir_b200.builder``) gives every uniform decode
  step (q_len <= 1 + speculative tokens, no cascade) a split-KV plan written to
  fixed-address device buffers, so FULL CUDA graphs replay it; every other
  step is built by the fallback's builder;
* the impl runs the sm_100a decode kernel on those steps and the fallback's
  forward on the rest.

KV formats: ``fp8`` / ``fp8_e4m3`` (per-tensor scale) and ``fp6_e2m3`` (packed
6-bit codes with static per-(layer, KV head, channel) scales from a
calibration file, ``mjolnir_b200.kvscales``). The fp6 cache is written by
``mjolnir_b200.kvfp6`` and read directly by the decode kernel, with the K
channel scales folded into Q and the V channel scales into the output; the
steps the fallback runs see the pages they read expanded to an e4m3 scratch.

Select it with ``--attention-backend MJOLNIR`` (a vLLM whose registry has that
member) or ``--attention-backend CUSTOM``; the ``vllm.general_plugins`` entry
point (``mjolnir_b200:register``) registers this class at start-up.
"""

from __future__ import annotations

import logging
from typing import Any, ClassVar

import torch

from . import kvdtype
from .runner import SUPPORTED_PAGE_SIZES, detect_kv_layout, env_flag, row_bytes, split_kv_cache

logger = logging.getLogger("vllm.mjolnir")

try:
    from vllm.v1.attention.backends.registry import AttentionBackendEnum
except ImportError:  # older vLLM layout
    from vllm.attention.backends.registry import AttentionBackendEnum

FP8_CACHE_DTYPES = ("fp8", "fp8_e4m3")
FP6_CACHE_DTYPES = (kvdtype.NAME,)
MJOLNIR_CACHE_DTYPES = FP8_CACHE_DTYPES + FP6_CACHE_DTYPES
# compute capabilities the in-tree kernels are built for (sm_100a only)
SUPPORTED_CAPABILITIES = ((10, 0),)

# Per-process step counters: serving smoke checks read them to see that
# decode steps really ran on the kernel.
STATS = {"kernel_steps": 0, "fallback_steps": 0, "noncausal_steps": 0}


def kv_format(cache_dtype) -> str:
    """'e2m3' for the packed fp6 cache, else 'fp8'."""
    return "e2m3" if str(cache_dtype) in FP6_CACHE_DTYPES else "fp8"


def fallback_name() -> str:
    """The stock backend this one extends (``MJOLNIR_ATTN_FALLBACK``)."""
    name = (env_flag("MJOLNIR_ATTN_FALLBACK", "FLASHINFER") or "FLASHINFER").upper()
    if name in ("CUSTOM", "MJOLNIR"):
        raise ValueError("MJOLNIR_ATTN_FALLBACK must name a stock backend")
    return name


_FALLBACK = fallback_name()
_Base = AttentionBackendEnum[_FALLBACK].get_class()
_BaseBuilder = _Base.get_builder_cls()
_BaseImpl = _Base.get_impl_cls()
_BASE_WRITES_KV_IN_FORWARD = getattr(_Base, "forward_includes_kv_cache_update", True)


def fallback_reads_fp8_scratch() -> bool:
    """Can the fallback read the e4m3 scratch that fp6 pages expand to?"""
    return _FALLBACK in ("FLASHINFER", "FLASH_ATTN")


def unsupported_reason(capability) -> str | None:
    """None on a GPU the in-tree kernels run on, else why not."""
    cap = tuple(capability)
    if cap in SUPPORTED_CAPABILITIES:
        return None
    return f"compute capability {cap[0]}.{cap[1]}: the kernels are built for sm_100a (B200) only"


def max_q_len(vllm_config) -> int:
    """1 + num_speculative_tokens, capped by ``MJOLNIR_ATTN_MAX_QLEN``
    (reference ``backend.py:225-230``)."""
    spec = getattr(vllm_config, "speculative_config", None)
    n = getattr(spec, "num_speculative_tokens", None) if spec is not None else None
    q = 1 + int(n or 0)
    cap = int(env_flag("MJOLNIR_ATTN_MAX_QLEN", "0") or 0)
    return min(q, cap) if cap > 0 else q


def _block_size_ok(sizes, size: int) -> bool:
    """Does a supported-size list (ints and ``MultipleOf``) admit ``size``?"""
    for s in sizes:
        base = getattr(s, "base", None)
        if s == size or (base is not None and size % base == 0):
            return True
    return False


# ---------------------------------------------------------------------------
# Eligibility (config level): None when the kernel can serve, else the reason
# ---------------------------------------------------------------------------
def layers_of(vllm_config, layer_names) -> dict:
    try:
        from vllm.config import get_layers_from_vllm_config
        from vllm.model_executor.layers.attention_layer_base import AttentionLayerBase

        return get_layers_from_vllm_config(vllm_config, AttentionLayerBase, layer_names)
    except Exception:  # noqa: BLE001 - the helper moved between vLLM releases
        return {}


# Attention features a layer may switch on that the decode kernel has no code
# for: the impl attribute, the values that mean "off" and the name reported.
# Tensor-valued features (sinks, ALiBi slopes) are off only when absent.
_LAYER_FEATURES = (
    ("sliding_window", (-1, (-1, -1)), "sliding window"),
    ("logits_soft_cap", (0, 0.0), "logits soft-cap"),
    ("sinks", (), "attention sinks"),
    ("alibi_slopes", (), "ALiBi"),
)


def _feature_on(value, off_values) -> bool:
    if value is None:
        return False
    if isinstance(value, (int, float, tuple)):
        return value not in off_values
    return True  # a tensor or a list of per-head values


def layer_reason(impl) -> str | None:
    """The first per-layer feature of ``impl`` the decode kernel lacks, or
    None (the same features as the reference's ``backend.py:263-273``)."""
    for attr, off_values, name in _LAYER_FEATURES:
        if _feature_on(getattr(impl, attr, None), off_values):
            return name
    return None


def _config_problems(kv_cache_spec, layer_names, vllm_config):
    """Every reason the kernel cannot serve this KV-cache group, cheapest
    checks first (the conditions of the reference's ``backend.py:276-301``)."""
    if env_flag("MJOLNIR_ATTN_DISABLE").lower() in ("1", "true", "yes"):
        yield "MJOLNIR_ATTN_DISABLE set"
    # what the cache holds and how it is paged
    dtype = str(getattr(vllm_config.cache_config, "cache_dtype", "auto"))
    if dtype not in MJOLNIR_CACHE_DTYPES:
        yield f"kv cache dtype {dtype!r} is neither of the kernel's formats {sorted(MJOLNIR_CACHE_DTYPES)}"
    page = getattr(kv_cache_spec, "block_size", None)
    if page not in SUPPORTED_PAGE_SIZES:
        yield f"block size {page} is not a kernel page size {SUPPORTED_PAGE_SIZES}"
    if getattr(kv_cache_spec, "sliding_window", None):
        yield "the KV spec keeps a sliding window"
    # head geometry and model precision
    d_k = getattr(kv_cache_spec, "head_size", None)
    if d_k not in (128, 256):
        yield f"head_size {d_k}: the kernel is built for 128 and 256"
    d_v = getattr(kv_cache_spec, "head_size_v", None) or d_k
    if d_v != d_k:
        yield f"K/V head sizes differ ({d_k} vs {d_v})"
    model_dtype = vllm_config.model_config.dtype
    if model_dtype not in (torch.bfloat16, torch.float16):
        yield f"model dtype {model_dtype} (bf16 or fp16 activations only)"
    # sequences split across ranks need a cross-rank softmax the kernel lacks
    pc = vllm_config.parallel_config
    for kind in ("decode", "prefill"):
        if getattr(pc, f"{kind}_context_parallel_size", 1) > 1:
            yield f"{kind} context parallel"
    # per-layer attention features
    for name, layer in layers_of(vllm_config, layer_names).items():
        why = layer_reason(getattr(layer, "impl", None))
        if why:
            yield f"layer {name}: {why}"


def ineligible_reason(kv_cache_spec, layer_names, vllm_config) -> str | None:
    """The first reason this KV-cache group cannot run on the kernel, or None."""
    return next(_config_problems(kv_cache_spec, layer_names, vllm_config), None)


# ---------------------------------------------------------------------------
# fp6 (e2m3) KV: preconditions and per-channel scales
# ---------------------------------------------------------------------------
def check_fp6(kernel_reason: str | None, layer_names) -> None:
    """An fp6 cache has two readers only: the decode kernel and the fallback's
    e4m3 scratch. Raise ValueError when either is missing (reference
    ``backend.py:308-336``)."""
    try:
        cap = torch.cuda.get_device_capability()
    except (RuntimeError, AssertionError):
        cap = None
    if cap is not None and unsupported_reason(cap):
        raise ValueError(f"{unsupported_reason(cap)} (serve fp8 KV on this GPU)")
    if kernel_reason is not None:
        raise ValueError(
            f"kv cache dtype fp6_e2m3 needs the Mjolnir decode kernel, but it is off for "
            f"{list(layer_names)[:1]}: {kernel_reason}. Serve fp8 KV for this model."
        )
    if not fallback_reads_fp8_scratch():
        raise ValueError(
            f"kv cache dtype fp6_e2m3 needs a fallback that reads fp8 KV (FLASHINFER or FLASH_ATTN); "
            f"MJOLNIR_ATTN_FALLBACK is {_FALLBACK}"
        )
    from . import kvscales

    if kvscales.calibrating():
        raise ValueError("calibrate on fp8 KV (MJOLNIR_ATTN_KV_CALIBRATE), then serve fp6_e2m3 with the file")


def set_layer_scale(layer, name: str, value: torch.Tensor) -> None:
    """Point a layer's ``_k_scale`` / ``_v_scale`` at ``value``.

    The attribute is rebound the way the layer registered it -- checkpoints
    with quantized KV register it as a Parameter, others as a buffer or a
    plain tensor -- so that ``nn.Module.__setattr__`` accepts the new value
    and state-dict consumers still find it; vLLM's float copy
    (``_k_scale_float``) follows when the scale is a single number."""
    registered = getattr(layer, name, None)
    if isinstance(registered, torch.nn.Parameter):
        value = torch.nn.Parameter(value, requires_grad=False)
    if name in getattr(layer, "_buffers", {}):
        layer._buffers[name] = value
    else:
        setattr(layer, name, value)
    mirror = name + "_float"
    if value.numel() == 1 and hasattr(layer, mirror):
        setattr(layer, mirror, float(value.detach().reshape(-1)[0]))


def fp6_layer_state(ks, vs, h_r: int, device, fallback: str) -> dict[str, torch.Tensor]:
    """Tensors one fp6 layer needs, from its (h_k, d) K and V channel scales:

    * ``k_ch`` / ``v_ch`` -- the cache write's quantization scales;
    * ``k_mul`` / ``v_mul`` (h_q, d) -- the kernel's Q and output multipliers;
    * ``k_ratio`` / ``v_ratio`` and ``k_head`` / ``v_head`` -- the fallback
      scratch: e4m3(code * ratio) with descale ``head`` per KV head. FlashAttention
      takes a per-head descale, so ratio = s_c / S_h with S_h = max_c s_c * 7.5 / 448;
      FlashInfer's paged kernels take none, so ratio = s_c and the descale is 1.
    """
    from .kvscales import E2M3_MAX

    st: dict[str, torch.Tensor] = {}
    for side, rows in (("k", ks), ("v", vs)):
        ch = torch.as_tensor(rows, dtype=torch.float32).to(device).contiguous()
        if fallback == "FLASH_ATTN":
            head = ch.amax(dim=1) * (E2M3_MAX / 448.0)
            ratio = ch / head[:, None]
        else:
            head = torch.ones(ch.shape[0], dtype=torch.float32, device=ch.device)
            ratio = ch
        st[f"{side}_ch"] = ch
        st[f"{side}_head"] = head.contiguous()
        st[f"{side}_ratio"] = ratio.contiguous()
        st[f"{side}_mul"] = ch.repeat_interleave(h_r, dim=0).contiguous()
    st["one"] = torch.ones(1, dtype=torch.float32, device=device)
    return st


def install_fp6_scales(vllm_config, layer_names, h_k: int, d: int) -> int:
    """Load the calibration file and attach each layer's fp6 state
    (``layer._mjolnir_fp6``); the layer's k/v scales become the fallback's
    per-head descales. Returns the number of layers set up (reference
    ``backend.py:370-427``)."""
    from . import kvscales

    path = kvscales.scales_path()
    if not path:
        raise ValueError(
            "an fp6_e2m3 cache is written with calibrated scales, and MJOLNIR_ATTN_KV_SCALES names no "
            "scales file; serve the model once on fp8 KV with MJOLNIR_ATTN_KV_CALIBRATE=1 to write one"
        )
    doc = kvscales.load(path)
    missing = kvscales.missing_layers(doc, layer_names)
    if missing:
        shown = ", ".join(missing[:3]) + (", ..." if len(missing) > 3 else "")
        raise ValueError(f"scales file {path} lacks {len(missing)} attention layer(s) of this model: {shown}")
    layers = layers_of(vllm_config, layer_names)
    for name, layer in layers.items():
        ks, vs = kvscales.e2m3_scales(doc, name, h_k, d)
        h_r = max(1, int(getattr(layer, "num_heads", h_k)) // h_k)
        dev = getattr(getattr(layer, "_k_scale", None), "device", None) or torch.device("cpu")
        st = fp6_layer_state(ks, vs, h_r, dev, _FALLBACK)
        layer._mjolnir_fp6 = st
        set_layer_scale(layer, "_k_scale", st["k_head"])
        set_layer_scale(layer, "_v_scale", st["v_head"])
    logger.info("Mjolnir: fp6_e2m3 KV scales for %d layer(s) from %s", len(layers), path)
    return len(layers)


# ---------------------------------------------------------------------------
# fp6 fallback scratch: the e4m3 pages a fallback step reads
# ---------------------------------------------------------------------------
_SCRATCH: dict = {}


def fp6_scratch(pages: int, h_k: int, page_size: int, d: int, device) -> torch.Tensor:
    """A growing per-device e4m3 page buffer in the fallback's own cache shape
    and stride order. Layers run one after another, so one buffer serves all
    of them; it lives outside vLLM's KV budget and grows to the largest step."""
    key = (str(device), h_k, page_size, d)
    buf = _SCRATCH.get(key)
    need = max(1, int(pages))
    if buf is None or buf.shape[0] < need:
        cap = max(need, 2 * buf.shape[0] if buf is not None else need)
        shape = _Base.get_kv_cache_shape(cap, page_size, h_k, d, cache_dtype_str="fp8")
        try:
            order = tuple(_Base.get_kv_cache_stride_order())
            if len(order) != len(shape):
                order = tuple(range(len(shape)))
        except (AttributeError, NotImplementedError):
            order = tuple(range(len(shape)))
        phys = torch.empty(tuple(shape[i] for i in order), dtype=torch.uint8, device=device)
        buf = phys.permute(*[order.index(i) for i in range(len(order))])
        _SCRATCH[key] = buf
    return buf


# ---------------------------------------------------------------------------
# Impl
# ---------------------------------------------------------------------------
class MjolnirImpl(_BaseImpl):  # type: ignore[misc, valid-type]
    """The fallback's impl plus the kernel path (reference ``backend.py:432-785``)."""

    def __init__(self, *args, **kwargs):
        super().__init__(*args, **kwargs)
        cache_dtype = str(getattr(self, "kv_cache_dtype", "auto"))
        self._fp6 = cache_dtype in FP6_CACHE_DTYPES
        if self._fp6:
            # fp6 fallback steps hand the base a scratch tensor chosen per step:
            # they run eager (kernel steps keep their CUDA graphs)
            self.enable_cuda_graph = False
        self._kv_layout: str | None = None
        self._layer_reason = layer_reason(self)
        # the kernel quantizes Q itself (three e4m3 terms per job): the layer
        # keeps handing over bf16 Q; a fallback step that wants fp8 Q gets it
        # quantized here, as the layer would (see _fallback_query)
        self.supports_quant_query_input = False

    def fused_output_quant_supported(self, quant_key) -> bool:
        return False  # the kernel writes bf16 / fp16 output

    # -- KV cache views and write ---------------------------------------------
    def kv_views(self, kv_cache: torch.Tensor, h_k: int, page_size: int, d: int):
        """Logical (pages, page_size, h_k, row) K and V byte views of the layer's cache."""
        row = row_bytes(d, "e2m3" if self._fp6 else "fp8")
        if self._kv_layout is None:
            self._kv_layout = detect_kv_layout(kv_cache.shape, h_k, page_size, row)
        k, v = split_kv_cache(kv_cache, self._kv_layout, row)
        if k.dtype != torch.uint8:
            k, v = k.view(torch.uint8), v.view(torch.uint8)
        return k, v

    def do_kv_cache_update(self, layer, key, value, kv_cache, slot_mapping):
        """Quantize-on-write through the sm_100a cache-write kernel, for both
        formats (reference ``backend.py:473-489``); in calibration mode also
        fold the rows into the layer's running amax."""
        from . import kvfp6, kvscales

        if kvscales.calibrating():
            kvscales.observe(getattr(layer, "layer_name", str(id(layer))), key, value, slot_mapping)
        if getattr(self, "kv_sharing_target_layer_name", None) is not None:
            return None
        if not self._fp6 and str(self.kv_cache_dtype) not in FP8_CACHE_DTYPES:
            return super().do_kv_cache_update(layer, key, value, kv_cache, slot_mapping)
        n = slot_mapping.shape[0]
        if n == 0:
            return None
        _, h_k, d = key.shape
        page_size = self._page_size(kv_cache, h_k, d)
        k_cache, v_cache = self.kv_views(kv_cache, h_k, page_size, d)
        if self._fp6:
            st = layer._mjolnir_fp6
            kvfp6.reshape_and_cache(key, value, k_cache, v_cache, slot_mapping, st["k_ch"], st["v_ch"], "e2m3")
        else:
            kvfp6.reshape_and_cache(key, value, k_cache, v_cache, slot_mapping, layer._k_scale, layer._v_scale, "fp8")
        return None

    def _page_size(self, kv_cache: torch.Tensor, h_k: int, d: int) -> int:
        """The cache's page size, found where the backend's own shape function
        puts the block size (asked once with a sentinel block size)."""
        if getattr(self, "_page_dim", None) is None:
            sentinel = 9973  # a prime no other dim of the probe can equal
            shape = MjolnirAttentionBackend.get_kv_cache_shape(
                3, sentinel, h_k, d, cache_dtype_str=str(self.kv_cache_dtype)
            )
            self._page_dim = list(shape).index(sentinel)
        return int(kv_cache.shape[self._page_dim])

    # -- forward ----------------------------------------------------------------
    def forward(
        self,
        layer,
        query,
        key,
        value,
        kv_cache,
        attn_metadata,
        output=None,
        output_scale=None,
        output_block_scale=None,
        *args: Any,
        **kwargs: Any,
    ):
        if not getattr(attn_metadata, "kernel_step", False):
            query = self._fallback_query(layer, query, attn_metadata)
            if self._fp6 and attn_metadata is not None:
                if getattr(attn_metadata, "mjolnir_fp6_pages", None) is None:
                    raise RuntimeError("Mjolnir: an fp6 fallback step without a page map (not built by MjolnirMetadataBuilder)")
                return self._forward_fp6_fallback(
                    layer, query, key, value, kv_cache, attn_metadata, output, output_scale, output_block_scale,
                    *args, **kwargs,
                )
            return super().forward(
                layer, query, key, value, kv_cache, attn_metadata, output, output_scale, output_block_scale,
                *args, **kwargs,
            )
        if self._layer_reason is not None:
            raise RuntimeError(f"Mjolnir got a layer it cannot run ({self._layer_reason}); set MJOLNIR_ATTN_DISABLE=1")
        if output is None or output_scale is not None:
            raise RuntimeError("Mjolnir kernel steps need a preallocated bf16/fp16 output and no output quantization")
        md = attn_metadata
        runner = md.runner
        k_cache, v_cache = self.kv_views(kv_cache, runner.h_k, runner.page_size, runner.d)
        if k_cache.shape[1] != runner.page_size:
            raise RuntimeError(
                f"Mjolnir: KV page size {k_cache.shape[1]} != planned {runner.page_size}; "
                "set MJOLNIR_ATTN_KV_LAYOUT or MJOLNIR_ATTN_DISABLE=1"
            )
        self._write_kv_in_forward(layer, key, value, kv_cache, md)
        if query.dtype not in (torch.bfloat16, torch.float16):
            # a pre-quantized fp8 query from a layer fusion
            query = (query.float() * layer._q_scale).to(torch.bfloat16)
        if self._fp6:  # channel scales ride Q and O; the codes' descale is 1
            st = layer._mjolnir_fp6
            runner.run(md.plan, query, output, k_cache, v_cache, st["one"], st["one"], self.scale,
                       q_mul=st["k_mul"], o_mul=st["v_mul"])
        else:
            runner.run(md.plan, query, output, k_cache, v_cache, layer._k_scale, layer._v_scale, self.scale)
        return output

    @staticmethod
    def _fallback_query(layer, query, attn_metadata):
        """The fallback's metadata may ask for fp8 Q (FlashInfer's TRTLLM
        kernels with an fp8 cache): quantize with the layer's static q scale,
        as the layer itself would have (reference ``backend.py:609-621``)."""
        want = getattr(attn_metadata, "q_data_type", None)
        if want is None or query.dtype == want or query.dtype not in (torch.bfloat16, torch.float16):
            return query
        if want not in (torch.float8_e4m3fn, torch.float8_e5m2):
            return query.to(want)
        lim = torch.finfo(want).max
        scale = layer._q_scale.float()
        n = query.shape[0]
        q = query.reshape(n, scale.numel(), -1).float() / scale.reshape(1, -1, 1)
        return q.clamp_(-lim, lim).to(want).view(query.shape)

    def _write_kv_in_forward(self, layer, key, value, kv_cache, md) -> None:
        """Only for fallbacks whose forward also writes the cache (older vLLM)."""
        if not _BASE_WRITES_KV_IN_FORWARD or key is None or value is None:
            return
        self.do_kv_cache_update(layer, key, value, kv_cache, md.slot_mapping)

    def _forward_fp6_fallback(self, layer, query, key, value, kv_cache, attn_metadata, *rest, **kwargs):
        """A fallback step on an fp6 cache: expand the pages it reads to the
        e4m3 scratch (codes x channel ratio) and run the base forward on it.
        The builder planned the step against the scratch's page ids."""
        from . import kvfp6

        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError(
                "Mjolnir: an fp6 fallback step inside CUDA-graph capture would replay a stale page map; "
                "serve fp8 KV or report this batch shape"
            )
        pages = attn_metadata.mjolnir_fp6_pages
        h_k, d = self.num_kv_heads, self.head_size
        page_size = self._page_size(kv_cache, h_k, d)
        k_cache, v_cache = self.kv_views(kv_cache, h_k, page_size, d)
        scratch = fp6_scratch(pages["total"], h_k, page_size, d, kv_cache.device)
        sk, sv = split_kv_cache(scratch, detect_kv_layout(scratch.shape, h_k, page_size, d), d)
        st = layer._mjolnir_fp6
        src = pages["src_pages"].clamp(0, k_cache.shape[0] - 1)
        kvfp6.expand_pages(k_cache, v_cache, src, sk, sv, st["k_ratio"], st["v_ratio"])
        view = scratch[: max(1, pages["total"])].view(torch.float8_e4m3fn)
        return super().forward(layer, query, key, value, view, attn_metadata, *rest, **kwargs)


# ---------------------------------------------------------------------------
# Backend
# ---------------------------------------------------------------------------
class MjolnirAttentionBackend(_Base):  # type: ignore[misc, valid-type]
    """The fallback backend with the Mjolnir builder and impl (reference
    ``backend.py:788-866``)."""

    accept_output_buffer: bool = True
    base_backend: ClassVar[type] = _Base
    # the fallback's cache dtypes plus fp6_e2m3 where the fallback reads the e4m3 scratch
    supported_kv_cache_dtypes: ClassVar[list] = list(getattr(_Base, "supported_kv_cache_dtypes", [])) + (
        list(FP6_CACHE_DTYPES) if fallback_reads_fp8_scratch() else []
    )

    @staticmethod
    def get_name() -> str:
        # vLLM maps the name back through AttentionBackendEnum: MJOLNIR exists
        # only in a vLLM that carries that member, CUSTOM everywhere
        from . import BACKEND_NAME, has_native_member

        return BACKEND_NAME if has_native_member() else "CUSTOM"

    @classmethod
    def get_supported_kernel_block_sizes(cls, *args, **kwargs) -> list:
        """16 / 32 / 64 / 128-token pages; FlashInfer's prefill and write take
        any page size, other fallbacks keep their own constraint."""
        if _FALLBACK == "FLASHINFER":
            return list(SUPPORTED_PAGE_SIZES)
        base = _Base.get_supported_kernel_block_sizes(*args, **kwargs)
        ours = [s for s in SUPPORTED_PAGE_SIZES if _block_size_ok(base, s)]
        return ours or list(base)

    @classmethod
    def supports_kv_cache_dtype(cls, kv_cache_dtype) -> bool:
        if kv_cache_dtype in FP6_CACHE_DTYPES:
            return kvdtype.known_to_vllm() and fallback_reads_fp8_scratch() and _Base.supports_kv_cache_dtype("fp8")
        return _Base.supports_kv_cache_dtype(kv_cache_dtype)

    @classmethod
    def supports_combination(cls, head_size, dtype, kv_cache_dtype, block_size, *args, **kwargs):
        # the fallback serves an fp6 cache through its e4m3 scratch
        if kv_cache_dtype in FP6_CACHE_DTYPES:
            kv_cache_dtype = "fp8"
        return _Base.supports_combination(head_size, dtype, kv_cache_dtype, block_size, *args, **kwargs)

    @classmethod
    def customize_spec(cls, spec):
        """Pluggable-dtype vLLM: an fp6 cell is the packed K row then the
        packed V row, ``2 * d * 3 / 4`` bytes."""
        mode = getattr(spec, "kv_quant_mode", None)
        if kvdtype.uses_api() and getattr(mode, "name", None) == "CUSTOM" and getattr(spec, "state_content_bytes", None) is None:
            from dataclasses import replace

            return replace(spec, state_content_bytes=kvdtype.cell_bytes(spec.head_size))
        parent = getattr(super(), "customize_spec", None)
        return parent(spec) if parent is not None else spec

    @staticmethod
    def get_kv_cache_shape(num_blocks, block_size, num_kv_heads, head_size, cache_dtype_str="auto"):
        """fp6 under the in-process shim: (blocks, h_k, page, 2, row bytes) --
        five dims, so the fallback's stride order applies unchanged; with the
        default order it is the K|V-interleaved (B, H, N, 2 * row) cell layout."""
        if cache_dtype_str in FP6_CACHE_DTYPES and kvdtype.shim_installed():
            return (num_blocks, num_kv_heads, block_size, 2, row_bytes(head_size, "e2m3"))
        return _Base.get_kv_cache_shape(num_blocks, block_size, num_kv_heads, head_size, cache_dtype_str=cache_dtype_str)

    @staticmethod
    def get_impl_cls():
        return MjolnirImpl

    @staticmethod
    def get_builder_cls():
        from .builder import MjolnirMetadataBuilder

        return MjolnirMetadataBuilder

    @classmethod
    def supports_device_cpu_query_lens_mismatch(cls) -> bool:
        # the uniform-decode check reads query_start_loc_cpu: it must be exact
        return False
