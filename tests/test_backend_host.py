"""The vLLM backend surface on the host (vLLM 0.22 as installed, no GPU):
plugin registration, the fp6 dtype shim, the backend class contract, the
builder's step routing and plans, the fp6 page map and layer state, and the
impl's KV views. Kernel launches are covered by the GPU tests."""

import sys
import types

import numpy as np
import pytest
import torch

vllm = pytest.importorskip("vllm")
import transformers.configuration_utils  # noqa: E402,F401 - vLLM config imports need it loaded first

from mjolnir_b200 import kvdtype  # noqa: E402


# ---------------------------------------------------------------- kvdtype
def test_shim_teaches_vllm_the_fp6_dtype():
    kvdtype.register()
    assert kvdtype.known_to_vllm() and kvdtype.shim_installed()
    from vllm.config.cache import CacheConfig
    from vllm.utils.torch_utils import kv_cache_dtype_str_to_dtype

    assert CacheConfig(cache_dtype="fp6_e2m3").cache_dtype == "fp6_e2m3"
    assert CacheConfig(cache_dtype="fp8").cache_dtype == "fp8"
    with pytest.raises(Exception):
        CacheConfig(cache_dtype="fp5_bogus")
    assert kv_cache_dtype_str_to_dtype("fp6_e2m3", None) == torch.uint8
    assert kvdtype.register() is False  # idempotent


def test_shim_spec_has_the_packed_page_size():
    kvdtype.register()
    from vllm.model_executor.layers.attention.attention import Attention
    from vllm.v1.kv_cache_interface import FullAttentionSpec

    layer = types.SimpleNamespace(kv_cache_dtype="fp6_e2m3", sliding_window=None, num_kv_heads=8, head_size=128, head_size_v=128)
    cfg = types.SimpleNamespace(cache_config=types.SimpleNamespace(block_size=16))
    spec = Attention.get_kv_cache_spec(layer, cfg)
    assert spec.page_size_bytes == 16 * 8 * 2 * 96  # page x heads x (K row + V row)
    assert isinstance(spec, FullAttentionSpec)
    layer.sliding_window = 128
    with pytest.raises(ValueError, match="sliding-window"):
        Attention.get_kv_cache_spec(layer, cfg)


def test_api_route_registers_a_custom_handler(monkeypatch):
    """With vLLM's pluggable KV-dtype API: uint8 storage, KVQuantMode.CUSTOM,
    no overwrite of a dtype vLLM already knows."""
    registered = {}
    known = []

    class KVQuantMode:
        CUSTOM = "CUSTOM"

    cache = types.ModuleType("vllm.config.cache")
    cache.KV_CACHE_DTYPES = known

    def register_kv_cache_dtype(name):
        def deco(cls):
            known.append(name)
            registered[name] = cls
            return cls

        return deco

    cache.register_kv_cache_dtype = register_kv_cache_dtype
    iface = types.ModuleType("vllm.v1.kv_cache_interface")
    iface.KVQuantMode = KVQuantMode
    monkeypatch.setitem(sys.modules, "vllm.config.cache", cache)
    monkeypatch.setitem(sys.modules, "vllm.v1.kv_cache_interface", iface)
    assert kvdtype.register() is True
    h = registered["fp6_e2m3"]()
    assert h.torch_dtype() is torch.uint8 and h.quant_mode() == "CUSTOM"
    assert kvdtype.register() is False


def test_shim_can_be_switched_off(monkeypatch):
    monkeypatch.setattr(kvdtype, "_api_register", lambda: None)
    monkeypatch.setenv("MJOLNIR_ATTN_FP6_SHIM", "0")
    assert kvdtype.register() is False


# ---------------------------------------------------------------- registration
def test_register_points_custom_at_the_backend(monkeypatch):
    import mjolnir_b200

    calls = []

    class Enum:
        __members__ = {"CUSTOM": "CUSTOM"}
        CUSTOM = "CUSTOM"

        def __class_getitem__(cls, k):
            return k

    monkeypatch.setattr(mjolnir_b200, "_backend_registry", lambda: (Enum, lambda member, path: calls.append((member, path))))
    mjolnir_b200.register()
    assert calls == [("CUSTOM", "mjolnir_b200.backend.MjolnirAttentionBackend")]
    monkeypatch.setenv("MJOLNIR_ATTN_DISABLE", "1")
    calls.clear()
    mjolnir_b200.register()
    assert calls == []


# ---------------------------------------------------------------- backend class
@pytest.fixture(scope="module")
def backend():
    kvdtype.register()
    from mjolnir_b200 import backend as b

    return b


def test_backend_class_contract(backend):
    B = backend.MjolnirAttentionBackend
    assert B.get_name() == "CUSTOM"  # stock vLLM 0.22 has no MJOLNIR member
    assert B.get_supported_kernel_block_sizes() == [16, 32, 64, 128]
    assert "fp6_e2m3" in B.supported_kv_cache_dtypes and "fp8" in B.supported_kv_cache_dtypes
    assert B.supports_kv_cache_dtype("fp6_e2m3") and B.supports_kv_cache_dtype("fp8")
    assert B.get_kv_cache_shape(10, 16, 8, 128, cache_dtype_str="fp6_e2m3") == (10, 8, 16, 2, 96)
    assert B.get_kv_cache_shape(10, 16, 8, 128, cache_dtype_str="fp8") == (10, 2, 16, 8, 128)
    assert B.get_impl_cls() is backend.MjolnirImpl
    assert B.get_builder_cls().__name__ == "MjolnirMetadataBuilder"
    assert B.supports_device_cpu_query_lens_mismatch() is False
    # the fallback answers fp6 combinations as fp8 ones
    seen = []
    orig = backend._Base.supports_combination
    try:
        backend._Base.supports_combination = classmethod(lambda cls, h, dt, kv, bs, *a, **k: seen.append(kv))
        B.supports_combination(128, torch.bfloat16, "fp6_e2m3", 16, False, False, False, None)
    finally:
        backend._Base.supports_combination = orig
    assert seen == ["fp8"]


def _cfg(cache_dtype="fp8", head=128, block=16, spec_tokens=0, model_dtype=torch.bfloat16):
    ns = types.SimpleNamespace
    return ns(
        cache_config=ns(cache_dtype=cache_dtype, block_size=block),
        model_config=ns(dtype=model_dtype, get_num_attention_heads=lambda pc: 64),
        parallel_config=ns(decode_context_parallel_size=1, prefill_context_parallel_size=1),
        scheduler_config=ns(max_num_seqs=32),
        speculative_config=ns(num_speculative_tokens=spec_tokens) if spec_tokens else None,
    )


def _spec(head=128, block=16, h_k=8):
    return types.SimpleNamespace(head_size=head, head_size_v=head, block_size=block, num_kv_heads=h_k, sliding_window=None)


def test_eligibility_reasons(backend):
    r = backend.ineligible_reason
    assert r(_spec(), [], _cfg()) is None
    assert "kv cache dtype" in r(_spec(), [], _cfg(cache_dtype="auto"))
    assert "head_size" in r(_spec(head=64), [], _cfg())
    assert "block size" in r(_spec(block=8), [], _cfg())
    assert "model dtype" in r(_spec(), [], _cfg(model_dtype=torch.float32))
    impl = types.SimpleNamespace(sliding_window=None, logits_soft_cap=30.0, sinks=None, alibi_slopes=None)
    assert backend.layer_reason(impl) == "logits soft-cap"
    assert backend.unsupported_reason((10, 0)) is None and "sm_100a" in backend.unsupported_reason((9, 0))
    assert backend.max_q_len(_cfg(spec_tokens=5)) == 6


# ---------------------------------------------------------------- builder
class _FakeRunner:
    def __init__(self, **kw):
        self.kw = kw
        self.max_q_len = kw["max_q_len"]
        self.max_num_seqs = kw["max_num_seqs"]
        self.plans = []

    def plan(self, lens, num_seqs, q_len, bt, seq_lens, margin=0, causal=True, fixed_grid=False):
        self.plans.append(dict(lens=list(lens), num_seqs=num_seqs, q_len=q_len, margin=margin, causal=causal, fixed_grid=fixed_grid))
        return types.SimpleNamespace(causal=causal or q_len == 1, q_len=q_len, num_seqs=num_seqs)


def _builder(monkeypatch, backend, cfg, spec=None):
    from mjolnir_b200 import builder as bmod

    monkeypatch.setattr(bmod, "DecodeRunner", _FakeRunner)
    b = object.__new__(bmod.MjolnirMetadataBuilder)
    b._setup(spec or _spec(), ["model.layers.0.self_attn.attn"], cfg, torch.device("cpu"))
    return b


def _cam(q_lens, seq_lens, width=64, causal=True):
    qsl = torch.tensor([0] + list(np.cumsum(q_lens)), dtype=torch.int32)
    n = len(q_lens)
    return types.SimpleNamespace(
        num_reqs=n,
        num_actual_tokens=int(sum(q_lens)),
        max_query_len=max(q_lens),
        max_seq_len=max(seq_lens),
        query_start_loc=qsl,
        query_start_loc_cpu=qsl,
        seq_lens=torch.tensor(seq_lens, dtype=torch.int32),
        seq_lens_cpu_upper_bound=torch.tensor(seq_lens, dtype=torch.int32),
        block_table_tensor=torch.arange(n * width, dtype=torch.int32).reshape(n, width),
        slot_mapping=torch.zeros(int(sum(q_lens)), dtype=torch.int64),
        causal=causal,
    )


def test_builder_routes_uniform_decode_to_the_kernel(monkeypatch, backend):
    from mjolnir_b200 import builder as bmod

    b = _builder(monkeypatch, backend, _cfg(spec_tokens=3))
    assert b.runner.kw["max_q_len"] == 4 and b.runner.kw["num_heads"] == 64 and b.runner.kw["kv_format"] == "fp8"
    assert b.kernel_step_q_len(_cam([1, 1, 1], [5, 9, 100])) == 1
    assert b.kernel_step_q_len(_cam([4, 4, 0, 0], [5, 9, 1, 1])) == 4  # trailing graph padding
    assert b.kernel_step_q_len(_cam([4, 3], [5, 9])) is None  # not uniform
    assert b.kernel_step_q_len(_cam([4, 0, 4], [5, 1, 9])) is None  # padding in the middle
    assert b.kernel_step_q_len(_cam([5, 5], [5, 9])) is None  # beyond 1 + speculative tokens
    assert b.kernel_step_q_len(_cam([3, 3], [5, 9], causal=False)) == 3  # a drafter's block
    calls = []
    monkeypatch.setattr(backend._BaseBuilder, "build", lambda self, cpl, cam, fast=False: calls.append(cpl) or "base-md")
    md = b.build(0, _cam([2, 2], [70, 33]))
    assert md.kernel_step and md.plan.q_len == 2
    assert b.runner.plans[-1] == dict(lens=[70, 33], num_seqs=2, q_len=2, margin=3, causal=True, fixed_grid=True)
    assert b.build(5, _cam([1, 1], [70, 33])) == "base-md" and calls == [5]  # cascade prefix: fallback
    assert b.build(0, _cam([7, 1], [70, 33])) == "base-md"
    assert isinstance(b.build_for_cudagraph_capture(_cam([1] * 4, [9] * 4)), bmod.MjolnirMetadata)


def test_builder_disables_itself_with_a_reason(monkeypatch, backend):
    b = _builder(monkeypatch, backend, _cfg(cache_dtype="auto"))
    assert b.runner is None and "kv cache dtype" in b._reason
    assert b.kernel_step_q_len(_cam([1], [5])) is None
    b2 = _builder(monkeypatch, backend, _cfg(spec_tokens=8))  # 9 x 8 = 72 rows per KV head
    assert b2.runner is None and "query rows" in b2._reason


def test_cudagraph_support(monkeypatch, backend):
    from vllm.v1.attention.backend import AttentionCGSupport

    from mjolnir_b200 import builder as bmod

    monkeypatch.setattr(backend._BaseBuilder, "get_cudagraph_support", classmethod(lambda cls, c, s: AttentionCGSupport.NEVER))
    B = bmod.MjolnirMetadataBuilder
    assert B.get_cudagraph_support(_cfg(), _spec()) == AttentionCGSupport.UNIFORM_SINGLE_TOKEN_DECODE
    assert B.get_cudagraph_support(_cfg(spec_tokens=2), _spec()) == AttentionCGSupport.UNIFORM_BATCH
    monkeypatch.setattr(backend._BaseBuilder, "get_cudagraph_support", classmethod(lambda cls, c, s: AttentionCGSupport.ALWAYS))
    assert B.get_cudagraph_support(_cfg(), _spec()) == AttentionCGSupport.ALWAYS


# ---------------------------------------------------------------- fp6 host logic
def _fp6_builder(monkeypatch, backend, tmp_path, h_k=2, d=128):
    import json

    name = "model.layers.0.self_attn.attn"
    g = np.random.default_rng(3)
    amax_k = (g.random((h_k, d)) * 10 + 0.1).tolist()
    amax_v = (g.random((h_k, d)) * 3 + 0.1).tolist()
    path = tmp_path / "scales.json"
    path.write_text(json.dumps({"format": "mjolnir.kv_scales/2", "model": "t", "tokens": 1, "amax": {name: {"k": amax_k, "v": amax_v}}}))
    monkeypatch.setenv("MJOLNIR_ATTN_KV_SCALES", str(path))
    monkeypatch.delenv("MJOLNIR_ATTN_KV_CALIBRATE", raising=False)
    layer = torch.nn.Module()
    layer.num_heads = 4 * h_k
    layer._k_scale = torch.ones(1)
    layer._v_scale = torch.ones(1)
    layer._k_scale_float = layer._v_scale_float = 1.0
    monkeypatch.setattr(backend, "layers_of", lambda cfg, names: {name: layer})
    b = _builder(monkeypatch, backend, _cfg(cache_dtype="fp6_e2m3"), spec=_spec(h_k=h_k, head=d))
    return b, layer, np.array(amax_k), np.array(amax_v)


def test_fp6_builder_installs_layer_scales(monkeypatch, backend, tmp_path):
    b, layer, ak, av = _fp6_builder(monkeypatch, backend, tmp_path)
    assert b._fp6 and b.runner.kw["kv_format"] == "e2m3"
    st = layer._mjolnir_fp6
    np.testing.assert_allclose(st["k_ch"].numpy(), ak / 7.5, rtol=1e-6)
    np.testing.assert_allclose(st["v_mul"].numpy(), np.repeat(av / 7.5, 4, axis=0), rtol=1e-6)
    if backend._FALLBACK == "FLASHINFER":  # no KV descale: ratio = s_c, layer scales 1
        np.testing.assert_allclose(st["k_ratio"].numpy(), ak / 7.5, rtol=1e-6)
        assert torch.equal(layer._k_scale, torch.ones(2))


def test_fp6_needs_a_scales_file(monkeypatch, backend):
    monkeypatch.delenv("MJOLNIR_ATTN_KV_SCALES", raising=False)
    monkeypatch.delenv("THOR_T5_KV_SCALES", raising=False)
    with pytest.raises(ValueError, match="calibrated scales"):
        _builder(monkeypatch, backend, _cfg(cache_dtype="fp6_e2m3"))


def test_fp6_refuses_an_ineligible_layer(monkeypatch, backend):
    with pytest.raises(ValueError, match="needs the Mjolnir decode kernel"):
        _builder(monkeypatch, backend, _cfg(cache_dtype="fp6_e2m3"), spec=_spec(block=8))


def test_fp6_page_map_and_fallback_build(monkeypatch, backend, tmp_path):
    b, _, _, _ = _fp6_builder(monkeypatch, backend, tmp_path)
    cam = _cam([5, 1, 0], [33, 16, 0], width=4)
    pages = b.fp6_page_map(cam)
    # request 0: 3 pages (0, 1, 2), request 1: 1 page, request 2: none
    assert pages["total"] == 4
    assert pages["src_pages"].tolist() == [0, 1, 2, 4]
    assert pages["block_table"][:2].tolist() == [[0, 1, 2, 0], [3, 0, 0, 0]]
    long = _cam([1], [10_000], width=4)  # an upper bound past the table is capped
    assert b.fp6_page_map(long)["total"] == 4
    seen = []

    def base_build(self, cpl, c, fast=False):
        seen.append(c.block_table_tensor.clone())
        return types.SimpleNamespace()

    monkeypatch.setattr(backend._BaseBuilder, "build", base_build)
    orig = cam.block_table_tensor
    md = b.build(0, cam)  # mixed q_lens: a fallback step
    assert torch.equal(seen[0], pages["block_table"]) and cam.block_table_tensor is orig
    assert md.mjolnir_fp6_pages["total"] == 4
    assert b.use_cascade_attention() is False


def _impl(backend, cache_dtype, h_k=8, d=128):
    impl = object.__new__(backend.MjolnirImpl)
    impl.kv_cache_dtype = cache_dtype
    impl._fp6 = cache_dtype == "fp6_e2m3"
    impl._kv_layout = None
    impl._layer_reason = None
    impl.num_kv_heads, impl.head_size = h_k, d
    impl.kv_sharing_target_layer_name = None
    return impl


@pytest.mark.parametrize("cache_dtype,shape,layout", [
    ("fp8", (10, 2, 32, 8, 128), "B2NHD"),
    ("fp6_e2m3", (10, 8, 32, 2, 96), "BHN2R"),
])
def test_impl_views_and_page_size(backend, cache_dtype, shape, layout):
    impl = _impl(backend, cache_dtype)
    cache = torch.zeros(shape, dtype=torch.uint8)
    assert impl._page_size(cache, 8, 128) == 32
    k, v = impl.kv_views(cache, 8, 32, 128)
    assert impl._kv_layout == layout
    row = 128 if cache_dtype == "fp8" else 96
    assert tuple(k.shape) == (10, 32, 8, row) and tuple(v.shape) == (10, 32, 8, row)
    if cache_dtype == "fp6_e2m3":  # the K|V-interleaved cell: V follows K in the same cell
        assert v.data_ptr() - k.data_ptr() == row and k.stride(1) == 2 * row


def test_impl_cache_write_dispatch(monkeypatch, backend):
    from mjolnir_b200 import kvfp6

    calls = []
    monkeypatch.setattr(kvfp6, "reshape_and_cache", lambda k, v, kc, vc, slots, ks, vs, fmt: calls.append((fmt, ks, tuple(kc.shape))))
    layer = types.SimpleNamespace(_k_scale=torch.tensor([0.5]), _v_scale=torch.tensor([2.0]), layer_name="L")
    key = torch.zeros(3, 8, 128)
    impl = _impl(backend, "fp8")
    impl.do_kv_cache_update(layer, key, key, torch.zeros(4, 2, 16, 8, 128, dtype=torch.uint8), torch.tensor([0, 1, -1]))
    assert calls[-1][0] == "fp8" and calls[-1][1] is layer._k_scale and calls[-1][2] == (4, 16, 8, 128)
    impl6 = _impl(backend, "fp6_e2m3")
    layer._mjolnir_fp6 = {"k_ch": torch.ones(8, 128), "v_ch": torch.ones(8, 128)}
    impl6.do_kv_cache_update(layer, key, key, torch.zeros(4, 8, 16, 2, 96, dtype=torch.uint8), torch.tensor([0, 1, 2]))
    assert calls[-1][0] == "e2m3" and calls[-1][1] is layer._mjolnir_fp6["k_ch"] and calls[-1][2] == (4, 16, 8, 96)
    impl6.kv_sharing_target_layer_name = "other"
    impl6.do_kv_cache_update(layer, key, key, None, torch.tensor([0]))
    assert len(calls) == 2


def test_fallback_step_without_page_map_is_refused(backend):
    impl = _impl(backend, "fp6_e2m3")
    with pytest.raises(RuntimeError, match="page map"):
        impl.forward(None, None, None, None, None, types.SimpleNamespace(), output=None)


def test_fallback_query_quantized_when_the_fallback_wants_fp8(backend):
    layer = types.SimpleNamespace(_q_scale=torch.tensor([0.5]))
    q = torch.randn(3, 4, 128).to(torch.bfloat16)
    md = types.SimpleNamespace(q_data_type=torch.float8_e4m3fn)
    q8 = backend.MjolnirImpl._fallback_query(layer, q, md)
    assert q8.dtype == torch.float8_e4m3fn and q8.shape == q.shape
    assert torch.allclose(q8.float() * 0.5, q.float(), rtol=0.07, atol=0.02)
    assert backend.MjolnirImpl._fallback_query(layer, q, types.SimpleNamespace()) is q
    assert backend.MjolnirImpl._fallback_query(layer, q, types.SimpleNamespace(q_data_type=torch.bfloat16)) is q
