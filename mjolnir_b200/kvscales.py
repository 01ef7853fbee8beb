"""Static per-(layer, KV head, channel) scales of the packed e2m3 KV cache.

e2m3 covers only +-7.5, so every (layer, KV head, channel) gets its own scale
``s = max(amax, 1e-6) / 7.5 * headroom``. Attention never applies them as
descales: a K channel scale multiplies Q's matching channel
(``q . k = sum_c (q_c s_c) code_c``) and a V channel scale multiplies the
output channel (``O_c = s_c sum_t p_t code_tc``), so the decode kernel reads
raw codes with descale 1.

The amax values come from a calibration pass (``MJOLNIR_ATTN_KV_CALIBRATE=1``
on an fp8 cache: ``observe`` folds every written K/V row into a running
per-channel max, ``dump`` writes the file). The file format is the
reference's, so existing calibration files load unchanged
(GoBrrr-ai/mjolnir ``src/mjolnir/mjolnir/kvscales.py:17-24``, ``:36-37``)::

    {"format": "mjolnir.kv_scales/2", "model": "...", "tokens": N,
     "amax": {"<layer>": {"k": [[d floats] x h_k], "v": [[d floats] x h_k]}}}

Format ``/1`` files carry one amax per head (or one per layer); those
broadcast over the channels.
"""

from __future__ import annotations

import json
import os
import threading
from pathlib import Path

import numpy as np
import torch

FORMAT = "mjolnir.kv_scales/2"
FORMATS = ("mjolnir.kv_scales/1", FORMAT)
E2M3_MAX = 7.5
AMAX_FLOOR = 1e-6

_PATH_VARS = ("MJOLNIR_ATTN_KV_SCALES", "THOR_T5_KV_SCALES")
_loaded: dict[str, dict] = {}


def scales_path() -> str | None:
    """The calibration file named by ``MJOLNIR_ATTN_KV_SCALES`` (legacy
    ``THOR_T5_KV_SCALES``), or None."""
    for var in _PATH_VARS:
        v = os.environ.get(var, "").strip()
        if v:
            return v
    return None


def load(path: str | os.PathLike) -> dict:
    """Parse (once per path) and validate a scales file; ValueError names the
    formats this module reads (reference ``kvscales.py:52-65``)."""
    key = str(path)
    doc = _loaded.get(key)
    if doc is None:
        doc = json.loads(Path(path).read_text())
        fmt = doc.get("format") if isinstance(doc, dict) else None
        if fmt not in FORMATS or not isinstance(doc.get("amax"), dict):
            raise ValueError(f"{path}: format {fmt!r}; readable formats are {', '.join(FORMATS)}")
        _loaded[key] = doc
    return doc


def headroom() -> float:
    """Multiplier on every scale (``MJOLNIR_ATTN_KV_SCALE_HEADROOM``, default 1):
    above 1 leaves room over the calibrated amax before codes saturate."""
    v = os.environ.get("MJOLNIR_ATTN_KV_SCALE_HEADROOM", "").strip()
    return float(v) if v else 1.0


def _amax_matrix(rows, h_k: int, d: int, what: str) -> np.ndarray:
    """(h_k, d) float64 amax from a per-channel, per-head or single entry."""
    if not isinstance(rows, list) or not rows:
        raise ValueError(f"{what}: empty or malformed amax entry")
    if isinstance(rows[0], list):
        a = np.asarray(rows, dtype=np.float64)
    else:
        heads = np.asarray(rows, dtype=np.float64).reshape(-1)
        if heads.size == 1:
            heads = np.repeat(heads, h_k)
        a = np.repeat(heads[:, None], d, axis=1) if heads.size == h_k else heads[:, None]
    if a.shape != (h_k, d):
        raise ValueError(f"{what}: amax is {a.shape[0]}x{a.shape[1] if a.ndim > 1 else 1}, the layer is {h_k}x{d}")
    return a


def e2m3_scales(doc: dict, layer_name: str, h_k: int, d: int) -> tuple[list[list[float]], list[list[float]]]:
    """(K scales, V scales) of one layer, each (h_k, d) nested lists, computed
    as ``max(amax, 1e-6) / 7.5 * headroom`` (reference ``kvscales.py:75-91``).
    KeyError when the file has no entry for the layer."""
    entry = doc["amax"].get(layer_name)
    if entry is None:
        raise KeyError(layer_name)
    hr = headroom()
    out = []
    for side in ("k", "v"):
        a = _amax_matrix(entry.get(side), h_k, d, f"{layer_name}.{side}")
        s = np.maximum(a, AMAX_FLOOR) / E2M3_MAX * hr
        out.append(s.tolist())
    return out[0], out[1]


def missing_layers(doc: dict, layer_names) -> list[str]:
    """Layer names the file has no amax for, in the given order."""
    return [n for n in layer_names if n not in doc["amax"]]


def per_channel(doc: dict, layer_name: str) -> bool:
    """True when the file carries per-channel (format /2) amax for the layer."""
    k = doc["amax"].get(layer_name, {}).get("k")
    return isinstance(k, list) and bool(k) and isinstance(k[0], list)


# ---------------------------------------------------------------------------
# calibration: running per-(KV head, channel) amax of every K/V row written
# ---------------------------------------------------------------------------
class _Observer:
    """Device-resident accumulators of one layer: K amax, V amax (h_k, d)
    float32 and a token count. Updated in place, so a captured CUDA graph
    that contains ``observe`` keeps folding on replay."""

    __slots__ = ("k", "v", "tokens")

    def __init__(self, h_k: int, d: int, device):
        self.k = torch.zeros(h_k, d, dtype=torch.float32, device=device)
        self.v = torch.zeros(h_k, d, dtype=torch.float32, device=device)
        self.tokens = torch.zeros((), dtype=torch.int64, device=device)


_observers: dict[str, _Observer] = {}
_lock = threading.Lock()


def calibrating() -> bool:
    """``MJOLNIR_ATTN_KV_CALIBRATE`` is set: record amax while writing the cache."""
    return os.environ.get("MJOLNIR_ATTN_KV_CALIBRATE", "").strip().lower() in ("1", "true", "yes")


def observe(layer_name: str, key: torch.Tensor, value: torch.Tensor, slot_mapping: torch.Tensor) -> None:
    """Fold the (T, h_k, d) K and V rows whose slot is >= 0 (padding tokens
    carry -1) into the layer's running amax (reference ``kvscales.py:108-129``)."""
    T = int(slot_mapping.shape[0])
    if T == 0:
        return
    h_k, d = int(key.shape[1]), int(key.shape[2])
    with _lock:
        obs = _observers.get(layer_name)
        if obs is None:
            obs = _observers[layer_name] = _Observer(h_k, d, key.device)
    live = (slot_mapping[:T] >= 0).view(T, 1, 1)
    zero = torch.zeros((), dtype=torch.float32, device=key.device)
    for acc, x in ((obs.k, key), (obs.v, value)):
        m = torch.where(live, x[:T].float().abs(), zero).amax(dim=0)
        torch.maximum(acc, m, out=acc)
    obs.tokens.add_(live.sum())


def reset() -> None:
    """Zero every accumulator (e.g. after the engine's warm-up passes, whose
    dummy tokens are not calibration data). The tensors may have been made
    under ``torch.inference_mode``, so they are updated in that mode."""
    with _lock, torch.inference_mode():
        for obs in _observers.values():
            obs.k.zero_()
            obs.v.zero_()
            obs.tokens.zero_()


def snapshot(model: str = "") -> dict:
    """The accumulated amax as a format-/2 document."""
    with _lock, torch.inference_mode():
        amax = {n: {"k": o.k.tolist(), "v": o.v.tolist()} for n, o in sorted(_observers.items())}
        tokens = max((int(o.tokens.item()) for o in _observers.values()), default=0)
    return {"format": FORMAT, "model": model, "tokens": tokens, "amax": amax}


def dump(path: str | os.PathLike, model: str = "") -> dict:
    """Write ``snapshot(model)`` to ``path`` (parents created) and return it."""
    doc = snapshot(model)
    p = Path(path)
    p.parent.mkdir(parents=True, exist_ok=True)
    p.write_text(json.dumps(doc, indent=1) + "\n")
    return doc
