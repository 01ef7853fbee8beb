"""The fp6 scales file and the calibration observer (host only)."""

import json

import numpy as np
import pytest
import torch

from mjolnir_b200 import kvscales


def _doc(amax_k, amax_v, fmt=kvscales.FORMAT):
    return {"format": fmt, "model": "m", "tokens": 10, "amax": {"model.layers.0.attn": {"k": amax_k, "v": amax_v}}}


def test_per_channel_scales_are_amax_over_7_5(tmp_path, monkeypatch):
    monkeypatch.delenv("MJOLNIR_ATTN_KV_SCALE_HEADROOM", raising=False)
    k = [[1.0, 7.5, 0.0, 486.0], [2.0, 3.0, 4.0, 5.0]]
    v = [[0.5] * 4, [15.0] * 4]
    p = tmp_path / "s.json"
    p.write_text(json.dumps(_doc(k, v)))
    doc = kvscales.load(p)
    ks, vs = kvscales.e2m3_scales(doc, "model.layers.0.attn", 2, 4)
    np.testing.assert_allclose(ks, np.maximum(np.array(k), 1e-6) / 7.5)
    np.testing.assert_allclose(vs, np.array(v) / 7.5)
    assert kvscales.per_channel(doc, "model.layers.0.attn")
    assert kvscales.missing_layers(doc, ["model.layers.0.attn", "x"]) == ["x"]
    with pytest.raises(KeyError):
        kvscales.e2m3_scales(doc, "x", 2, 4)


def test_per_head_and_single_entries_broadcast(tmp_path, monkeypatch):
    monkeypatch.setenv("MJOLNIR_ATTN_KV_SCALE_HEADROOM", "1.25")
    p = tmp_path / "s1.json"
    p.write_text(json.dumps(_doc([3.0, 6.0], [9.0], fmt="mjolnir.kv_scales/1")))
    doc = kvscales.load(p)
    ks, vs = kvscales.e2m3_scales(doc, "model.layers.0.attn", 2, 3)
    np.testing.assert_allclose(ks, [[3 / 7.5 * 1.25] * 3, [6 / 7.5 * 1.25] * 3])
    np.testing.assert_allclose(vs, [[9 / 7.5 * 1.25] * 3] * 2)
    assert not kvscales.per_channel(doc, "model.layers.0.attn")


def test_bad_files_rejected(tmp_path):
    p = tmp_path / "bad.json"
    p.write_text(json.dumps({"format": "mjolnir.kv_scales/9", "amax": {}}))
    with pytest.raises(ValueError, match="kv_scales/9"):
        kvscales.load(p)
    q = tmp_path / "shape.json"
    q.write_text(json.dumps(_doc([[1.0, 2.0]], [[1.0, 2.0]])))
    with pytest.raises(ValueError, match="the layer is 2x2"):
        kvscales.e2m3_scales(kvscales.load(q), "model.layers.0.attn", 2, 2)


def test_scales_path_env(monkeypatch):
    monkeypatch.delenv("MJOLNIR_ATTN_KV_SCALES", raising=False)
    monkeypatch.setenv("THOR_T5_KV_SCALES", "/legacy.json")
    assert kvscales.scales_path() == "/legacy.json"
    monkeypatch.setenv("MJOLNIR_ATTN_KV_SCALES", "/new.json")
    assert kvscales.scales_path() == "/new.json"


def test_observer_folds_live_rows_and_dumps_a_loadable_file(tmp_path):
    kvscales.reset()
    g = torch.Generator().manual_seed(0)
    key = torch.randn(6, 2, 8, generator=g)
    value = torch.randn(6, 2, 8, generator=g)
    key[5] = 1000.0  # a padding token: slot -1, must not count
    slots = torch.tensor([3, 4, 9, 1, 0, -1])
    kvscales.observe("L0", key, value, slots)
    kvscales.observe("L0", key[:2] * 3, value[:2], slots[:2])
    doc = kvscales.dump(tmp_path / "out.json", model="toy")
    live = key[:5].abs().amax(0)
    want_k = torch.maximum(live, (key[:2] * 3).abs().amax(0))
    np.testing.assert_allclose(np.array(doc["amax"]["L0"]["k"]), want_k.numpy(), rtol=0, atol=0)
    np.testing.assert_allclose(np.array(doc["amax"]["L0"]["v"]), value[:5].abs().amax(0).numpy())
    assert doc["tokens"] == 7 and doc["format"] == kvscales.FORMAT
    again = kvscales.load(tmp_path / "out.json")
    ks, _ = kvscales.e2m3_scales(again, "L0", 2, 8)
    np.testing.assert_allclose(ks, np.maximum(want_k.numpy(), 1e-6) / 7.5, rtol=1e-6)
    kvscales.reset()
    assert kvscales.snapshot()["amax"]["L0"]["k"][0][0] == 0.0
