"""The ``fp6_e2m3`` KV-cache dtype for vLLM: registration and the vLLM 0.22 shim.

Two routes, tried in order by :func:`register` (called from the plugin entry
point):

1. vLLM's pluggable KV-dtype API (``vllm.config.cache.register_kv_cache_dtype``,
   vLLM >= 0.33): register a handler whose storage dtype is uint8 and whose
   quant mode is ``KVQuantMode.CUSTOM`` -- the reference's route
   (GoBrrr-ai/mjolnir ``src/mjolnir/mjolnir/kvdtype.py:21-53``). The backend's
   ``customize_spec`` then sizes the cell at ``2 * d * 3 / 4`` bytes.
2. vLLM without that API (0.22 here): :func:`install_shim` makes the same four
   edits the reference's vLLM image patch hand-applies, in process:
   the ``CacheDType`` literal (CacheConfig validation and the backend
   selector), ``STR_DTYPE_TO_TORCH_DTYPE["fp6_e2m3"] = uint8``, and a KV spec
   whose page is ``page_size * h_k * 2 * row_bytes`` bytes (vLLM 0.22's
   packed-slot ``TQFullAttentionSpec``, which its KV managers treat as a full
   attention spec). ``MJOLNIR_ATTN_FP6_SHIM=0`` turns the shim off.

Both routes are no-ops when vLLM already knows the dtype.
"""

from __future__ import annotations

import logging
import os
import typing

import torch

NAME = "fp6_e2m3"
BITS = 6
_log = logging.getLogger("vllm.mjolnir")
_shim_installed = False


def cell_bytes(head_size: int) -> int:
    """Bytes of one (token, KV head) cell: the packed K row then the packed V row."""
    return 2 * head_size * BITS // 8


def _api_register() -> bool | None:
    """Route 1. None when this vLLM has no pluggable KV-dtype API."""
    try:
        from vllm.config.cache import KV_CACHE_DTYPES, register_kv_cache_dtype
        from vllm.v1.kv_cache_interface import KVQuantMode
    except ImportError:
        return None
    if NAME in KV_CACHE_DTYPES:
        return False

    @register_kv_cache_dtype(NAME)
    class _Fp6E2M3:
        name = NAME

        def torch_dtype(self) -> torch.dtype:
            return torch.uint8  # the packed cell bytes

        def quant_mode(self):
            # quantized, but self-managed: only this package's kernels touch the pool
            return KVQuantMode.CUSTOM

    return True


def shim_installed() -> bool:
    return _shim_installed


def _extend_literal(lit):
    args = typing.get_args(lit)
    return lit if NAME in args else typing.Literal[args + (NAME,)]


def _retype_cache_config(new) -> None:
    """Point CacheConfig's ``cache_dtype`` field at the extended literal and
    rebuild its pydantic validator (the field is validated at construction)."""
    import pydantic
    from vllm.config import cache as cache_mod

    C = cache_mod.CacheConfig
    C.__annotations__["cache_dtype"] = new
    C.__dataclass_fields__["cache_dtype"].type = new
    C.__pydantic_fields__["cache_dtype"].annotation = new
    C.__pydantic_complete__ = False
    pydantic.dataclasses.rebuild_dataclass(C, force=True)


def _patch_layer_spec() -> None:
    """fp6 layers report a packed-slot spec: page = block_size * h_k * cell bytes."""
    from vllm.model_executor.layers.attention import attention as attn_mod
    from vllm.v1.kv_cache_interface import TQFullAttentionSpec

    cls = attn_mod.Attention
    orig = cls.get_kv_cache_spec
    if getattr(orig, "_mjolnir_fp6", False):
        return

    def get_kv_cache_spec(self, vllm_config):
        if getattr(self, "kv_cache_dtype", None) != NAME:
            return orig(self, vllm_config)
        if getattr(self, "sliding_window", None) is not None:
            raise ValueError("kv cache dtype fp6_e2m3: sliding-window layers are not supported")
        hv = getattr(self, "head_size_v", None) or self.head_size
        if hv != self.head_size:
            raise ValueError("kv cache dtype fp6_e2m3 needs equal K and V head sizes")
        return TQFullAttentionSpec(
            block_size=vllm_config.cache_config.block_size,
            num_kv_heads=self.num_kv_heads,
            head_size=self.head_size,
            head_size_v=hv,
            dtype=torch.uint8,
            tq_slot_size=cell_bytes(self.head_size),
        )

    get_kv_cache_spec._mjolnir_fp6 = True  # type: ignore[attr-defined]
    cls.get_kv_cache_spec = get_kv_cache_spec


def install_shim() -> bool:
    """Teach a vLLM without the pluggable KV-dtype API the ``fp6_e2m3`` dtype.
    Returns True when the edits were applied, False when vLLM already knew it
    (or the shim ran before)."""
    global _shim_installed
    if _shim_installed:
        return False
    from vllm.config import cache as cache_mod
    from vllm.utils import torch_utils

    known = NAME in typing.get_args(cache_mod.CacheDType)
    if known and NAME in torch_utils.STR_DTYPE_TO_TORCH_DTYPE:
        return False
    new = _extend_literal(cache_mod.CacheDType)
    cache_mod.CacheDType = new
    _retype_cache_config(new)
    try:
        from vllm.v1.attention import selector

        selector.CacheDType = new  # the selector validates against get_args(CacheDType)
    except ImportError:
        pass
    torch_utils.STR_DTYPE_TO_TORCH_DTYPE.setdefault(NAME, torch.uint8)
    _patch_layer_spec()
    _shim_installed = True
    return True


def known_to_vllm() -> bool:
    """Does the running vLLM accept ``--kv-cache-dtype fp6_e2m3``?"""
    try:
        from vllm.config.cache import get_kv_cache_dtype_handler

        if get_kv_cache_dtype_handler(NAME) is not None:
            return True
    except ImportError:
        pass
    try:
        from vllm.config import cache as cache_mod
        from vllm.utils import torch_utils
    except ImportError:
        return False
    return NAME in typing.get_args(cache_mod.CacheDType) and NAME in torch_utils.STR_DTYPE_TO_TORCH_DTYPE


def uses_api() -> bool:
    """True when fp6 came through vLLM's pluggable API (the spec carries
    ``KVQuantMode.CUSTOM`` and ``customize_spec`` sizes the cell)."""
    try:
        from vllm.config.cache import get_kv_cache_dtype_handler
    except ImportError:
        return False
    return get_kv_cache_dtype_handler(NAME) is not None


def register() -> bool:
    """Plugin-time registration: the pluggable API where vLLM has it, else
    the in-process shim (unless ``MJOLNIR_ATTN_FP6_SHIM=0``). True when this
    call made vLLM aware of the dtype."""
    done = _api_register()
    if done is not None:
        return done
    if os.environ.get("MJOLNIR_ATTN_FP6_SHIM", "1").strip().lower() in ("0", "false", "no"):
        return False
    return install_shim()
