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

import importlib
import logging
import os

__all__ = ["BACKEND_NAME", "BACKEND_PATH", "__version__", "register", "has_native_member"]
__version__ = "0.1.0"

BACKEND_NAME = "MJOLNIR"
BACKEND_PATH = "mjolnir_b200.backend.MjolnirAttentionBackend"


_ON = ("1", "true", "yes")
# MJOLNIR_ATTN_DISABLE, or THOR_T5_DISABLE (the older name deployments still set)
_SWITCHES = ("MJOLNIR_ATTN_DISABLE", "THOR_T5_DISABLE")


def _switched_off() -> bool:
    return any(os.environ.get(var, "").strip().lower() in _ON for var in _SWITCHES)


def _backend_registry():
    """vLLM's ``AttentionBackendEnum`` and ``register_backend`` (the module
    moved under ``vllm.v1`` in newer releases)."""
    for where in ("vllm.v1.attention.backends.registry", "vllm.attention.backends.registry"):
        try:
            mod = importlib.import_module(where)
        except ImportError:
            continue
        return mod.AttentionBackendEnum, mod.register_backend
    raise ImportError("this vLLM has no attention-backend registry")


def has_native_member() -> bool:
    """True when this vLLM has the ``MJOLNIR`` enum member (a patched vLLM)."""
    try:
        enum, _ = _backend_registry()
    except ImportError:
        return False
    return BACKEND_NAME in enum.__members__


def _register_fp6_dtype() -> None:
    """Add the fp6_e2m3 KV-cache dtype. A failure is logged, not raised: vLLM
    still starts and serves fp8 KV without it."""
    try:
        from .kvdtype import register as register_kv_dtype

        register_kv_dtype()
    except Exception as exc:  # noqa: BLE001 - plugin loading must not abort vLLM
        logging.getLogger("vllm.mjolnir").warning("fp6_e2m3 KV dtype unavailable, fp8 KV still serves: %r", exc)


def register() -> None:
    """vLLM ``general_plugins`` entry point."""
    if _switched_off():
        return
    _register_fp6_dtype()
    if os.environ.get("MJOLNIR_ATTN_DEBUG", "").strip():
        # synchronous launches name a faulting kernel at its launch; the engine
        # processes vLLM starts later inherit the setting
        os.environ.setdefault("CUDA_LAUNCH_BLOCKING", "1")
    enum, register_backend = _backend_registry()
    for member in ([BACKEND_NAME] if BACKEND_NAME in enum.__members__ else []) + ["CUSTOM"]:
        register_backend(enum[member], BACKEND_PATH)
