"""mjolnir_b200 -- the MJOLNIR paged decode-attention hot path, native on B200.

A from-scratch sm_100a implementation of GoBrrr-ai/mjolnir's decode-attention
backend: quantize-on-write KV cache (fp8-e4m3 and packed 6-bit e2m3), paged
split-KV decode serving a whole GQA group and all MTP draft positions from one
KV read, and the LSE split combine -- behind a C ABI (include/mjolnir_b200.h)
and the reference's vLLM attention-backend surface.

``register()`` is the vLLM general-plugin entry point (the reference's
``mjolnir.register``, ``src/mjolnir/mjolnir/__init__.py:60-82``): it points
``AttentionBackendEnum.MJOLNIR`` (when the running vLLM has that member) and
``AttentionBackendEnum.CUSTOM`` at ``mjolnir_b200.backend.MjolnirAttentionBackend``.
The backend module, and with it vLLM's attention stack, is imported lazily.
"""

from __future__ import annotations

import os

__all__ = ["BACKEND_NAME", "BACKEND_PATH", "__version__", "register", "has_native_member"]
__version__ = "0.1.0"

BACKEND_NAME = "MJOLNIR"
BACKEND_PATH = "mjolnir_b200.backend.MjolnirAttentionBackend"


def _disabled() -> bool:
    for name in ("MJOLNIR_ATTN_DISABLE", "THOR_T5_DISABLE"):
        if os.environ.get(name, "").strip().lower() in ("1", "true", "yes"):
            return True
    return False


def _registry():
    try:
        from vllm.v1.attention.backends.registry import AttentionBackendEnum, register_backend
    except ImportError:  # older vLLM layout
        from vllm.attention.backends.registry import AttentionBackendEnum, register_backend
    return AttentionBackendEnum, register_backend


def has_native_member() -> bool:
    """True when this vLLM has the ``MJOLNIR`` enum member (a patched vLLM)."""
    try:
        enum, _ = _registry()
    except ImportError:
        return False
    return BACKEND_NAME in enum.__members__


def register() -> None:
    """vLLM ``general_plugins`` entry point."""
    if _disabled():
        return
    try:
        from .kvdtype import register as _register_kv_dtype

        _register_kv_dtype()
    except Exception as e:  # noqa: BLE001 - never break vLLM start-up
        import logging

        logging.getLogger("vllm.mjolnir").warning("Mjolnir fp6 KV dtype not registered: %r", e)
    if os.environ.get("MJOLNIR_ATTN_DEBUG", "").strip():
        os.environ.setdefault("CUDA_LAUNCH_BLOCKING", "1")
    enum, register_backend = _registry()
    if BACKEND_NAME in enum.__members__:
        register_backend(enum[BACKEND_NAME], BACKEND_PATH)
    register_backend(enum.CUSTOM, BACKEND_PATH)
