"""The kernel-step metadata and its builder (the vLLM side of the plan).

A step whose batch is a uniform decode -- every request has the same q_len in
``1 .. 1 + num_speculative_tokens`` (trailing CUDA-graph padding requests have
0), causal, no cascade prefix -- gets a split-KV plan from the runner, written
into the runner's fixed-address device buffers with a fixed grid, so FULL
CUDA graphs captured on one plan replay any later one. Every other step is
built by the fallback's builder (reference GoBrrr-ai/mjolnir
``src/mjolnir/mjolnir/builder.py:119-521``); on an fp6 cache such a step also
gets the page map its e4m3 scratch expansion follows.
"""

from __future__ import annotations

import torch

from .backend import (
    _FALLBACK,
    STATS,
    _BaseBuilder,
    check_fp6,
    ineligible_reason,
    install_fp6_scales,
    kv_format,
    logger,
    max_q_len,
    unsupported_reason,
)
from .runner import DecodeRunner, StepPlan, env_flag

try:
    from vllm.v1.attention.backend import AttentionCGSupport
except ImportError:  # older vLLM
    from vllm.v1.attention.backends.utils import AttentionCGSupport

# non-causal uniform blocks (a parallel drafter's block attention) on the kernel
_NONCAUSAL = env_flag("MJOLNIR_ATTN_NONCAUSAL", "1").lower() not in ("0", "false", "no")


class MjolnirMetadata:
    """Kernel-step metadata: the plan and the runner, plus the attributes
    generic vLLM code reads from attention metadata. The fallback's impl
    never sees this object (reference ``builder.py:91-116``)."""

    kernel_step = True

    def __init__(self, *, plan: StepPlan, runner: DecodeRunner, cam):
        self.plan = plan
        self.runner = runner
        self.num_actual_tokens = cam.num_actual_tokens
        self.num_reqs = cam.num_reqs
        self.max_query_len = cam.max_query_len
        self.max_seq_len = cam.max_seq_len
        self.query_start_loc = cam.query_start_loc
        self.seq_lens = cam.seq_lens
        self.block_table = cam.block_table_tensor
        self.slot_mapping = cam.slot_mapping
        self.num_decodes = cam.num_reqs
        self.num_decode_tokens = cam.num_actual_tokens
        self.num_prefills = 0
        self.num_prefill_tokens = 0
        self.use_cascade = False
        self.causal = plan.causal


def uniform_q_len(query_start_loc_cpu, num_reqs: int, q_len: int) -> bool:
    """Every request has ``q_len`` tokens, except trailing padding requests with 0."""
    qsl = query_start_loc_cpu[: num_reqs + 1]
    lens = (qsl[1:] - qsl[:-1]).tolist()
    n = 0
    while n < len(lens) and lens[n] == q_len:
        n += 1
    return all(x == 0 for x in lens[n:])


def fp8_view_of(spec):
    """The KV spec as the fallback sees an fp6 cache: its quant mode fp8
    (the pages it reads are the e4m3 scratch)."""
    try:
        from dataclasses import replace

        from vllm.v1.kv_cache_interface import KVQuantMode
    except ImportError:
        return spec
    mode = getattr(KVQuantMode, "FP8_PER_TENSOR", None)
    if mode is None or not hasattr(spec, "kv_quant_mode"):
        return spec
    return replace(spec, kv_quant_mode=mode)


class MjolnirMetadataBuilder(_BaseBuilder):  # type: ignore[misc, valid-type]
    # a shared-metadata shortcut across KV-cache groups would skip the plan
    supports_update_block_table: bool = False

    def __init__(self, kv_cache_spec, layer_names, vllm_config, device, *args, **kwargs):
        cache_config = vllm_config.cache_config
        saved = cache_config.cache_dtype
        fp6 = kv_format(saved) == "e2m3"
        base_spec = kv_cache_spec
        if fp6:
            # the fallback's builder maps the cache dtype for its kernels and
            # only ever reads the e4m3 scratch: it is built as for fp8 (the
            # cache dtype and the spec's quant mode say fp8 while it runs)
            cache_config.cache_dtype = "fp8"
            base_spec = fp8_view_of(kv_cache_spec)
        try:
            super().__init__(base_spec, layer_names, vllm_config, device, *args, **kwargs)
        finally:
            cache_config.cache_dtype = saved
        self.kv_cache_spec = kv_cache_spec
        self._setup(kv_cache_spec, layer_names, vllm_config, device)

    def _setup(self, kv_cache_spec, layer_names, vllm_config, device) -> None:
        """Everything past the fallback's own construction (separate so host
        tests can run it on a builder made without the fallback)."""
        spec = getattr(vllm_config, "speculative_config", None)
        # a plan made num_speculative_tokens longer stays valid while a fused
        # draft decode advances seq_lens in place (the kernel masks with the
        # live device seq_lens)
        self._plan_margin = int(getattr(spec, "num_speculative_tokens", 0) or 0) if spec is not None else 0
        self._kv_format = kv_format(getattr(vllm_config.cache_config, "cache_dtype", "auto"))
        self._fp6 = self._kv_format == "e2m3"
        self._page = kv_cache_spec.block_size
        mc, pc = vllm_config.model_config, vllm_config.parallel_config
        num_heads = None
        try:
            from vllm.v1.attention.backends.utils import get_num_attention_heads_from_layers

            num_heads = get_num_attention_heads_from_layers(vllm_config, layer_names)
        except Exception:  # noqa: BLE001 - not in every vLLM
            pass
        if num_heads is None:
            num_heads = mc.get_num_attention_heads(pc)
        self._reason = ineligible_reason(kv_cache_spec, layer_names, vllm_config)
        if self._reason is None and torch.device(device).type == "cuda":
            self._reason = unsupported_reason(torch.cuda.get_device_capability(device))
        rows = max_q_len(vllm_config) * (num_heads // max(1, kv_cache_spec.num_kv_heads))
        if self._reason is None and rows > 64:
            self._reason = f"{rows} query rows per KV head (q_len x h_q / h_k > 64)"
        if self._fp6:
            check_fp6(self._reason, layer_names)
            install_fp6_scales(vllm_config, layer_names, kv_cache_spec.num_kv_heads, kv_cache_spec.head_size)
        self.runner: DecodeRunner | None = None
        if self._reason is not None:
            logger.warning("Mjolnir decode disabled for %s: %s -> %s for all steps", list(layer_names)[:1], self._reason, _FALLBACK)
            return
        self.runner = DecodeRunner(
            num_heads=num_heads,
            num_kv_heads=kv_cache_spec.num_kv_heads,
            head_size=kv_cache_spec.head_size,
            page_size=kv_cache_spec.block_size,
            out_dtype=mc.dtype,
            max_num_seqs=vllm_config.scheduler_config.max_num_seqs,
            max_q_len=max_q_len(vllm_config),
            ctas_per_sm=int(env_flag("MJOLNIR_ATTN_CTAS", "2")),
            max_splits=int(env_flag("MJOLNIR_ATTN_MAX_SPLITS", "16")),
            kv_format=self._kv_format,
            device=device,
        )
        logger.info(
            "Mjolnir decode enabled: h_q=%d h_k=%d d=%d page=%d q_len<=%d kv=%s fallback=%s",
            num_heads,
            kv_cache_spec.num_kv_heads,
            kv_cache_spec.head_size,
            kv_cache_spec.block_size,
            self.runner.max_q_len,
            self._kv_format,
            _FALLBACK,
        )

    # -- CUDA graph support ----------------------------------------------------
    @classmethod
    def get_cudagraph_support(cls, vllm_config, kv_cache_spec):
        """Mixed batches go to the fallback, so promise no more than it does
        for those; uniform decode batches are graph-safe on the kernel."""
        base = super().get_cudagraph_support(vllm_config, kv_cache_spec)
        if base == AttentionCGSupport.ALWAYS:
            return base
        want = AttentionCGSupport.UNIFORM_BATCH if max_q_len(vllm_config) > 1 else AttentionCGSupport.UNIFORM_SINGLE_TOKEN_DECODE
        return max(base, want, key=lambda e: e.value)

    @classmethod
    def get_varlen_cudagraph_max_query_len(cls, vllm_config, kv_cache_spec):
        return None  # kernel graphs replay uniform-q_len batches only

    # -- build -------------------------------------------------------------------
    def kernel_step_q_len(self, cam) -> int | None:
        """The q_len of a step the kernel can run, else None.

        A kernel step is a uniform batch -- every request brings q_len query
        tokens (one decode token, or the verified token plus the drafts), with
        CUDA-graph padding requests bringing none -- that fits the runner, under
        a causal mask or, when enabled, a parallel drafter's non-causal block,
        and without decode context parallelism (the step routing of the
        reference's ``builder.py:309-343``)."""
        r = self.runner
        q_len = int(cam.max_query_len)
        mask = getattr(cam, "causal", True)
        fits = (r is not None and 1 <= q_len <= r.max_q_len and cam.num_reqs <= r.max_num_seqs
                and (mask is True or (mask is False and _NONCAUSAL))
                and getattr(cam, "dcp_local_seq_lens", None) is None)
        if not fits:
            return None
        one_token_each = q_len == 1 and cam.num_actual_tokens <= cam.num_reqs
        return q_len if one_token_each or uniform_q_len(cam.query_start_loc_cpu, cam.num_reqs, q_len) else None

    @staticmethod
    def seq_lens_host(cam):
        """Host seq_lens for planning: the upper bound when vLLM offers one
        (the kernel masks with the exact device lengths), else a copy."""
        for name in ("seq_lens_cpu_upper_bound", "seq_lens_cpu"):
            v = getattr(cam, name, None)
            if v is not None:
                return v
        return cam.seq_lens.cpu()

    def build(self, common_prefix_len: int, common_attn_metadata, fast_build: bool = False):
        cam = common_attn_metadata
        q_len = self.kernel_step_q_len(cam) if common_prefix_len == 0 else None
        if q_len is None:
            STATS["fallback_steps"] += 1
            if self._fp6:
                return self._build_fp6_fallback(common_prefix_len, cam, fast_build)
            return super().build(common_prefix_len, cam, fast_build)
        STATS["kernel_steps"] += 1
        causal = getattr(cam, "causal", True) is not False
        if not causal:
            STATS["noncausal_steps"] += 1
        plan = self.runner.plan(
            self.seq_lens_host(cam),
            cam.num_reqs,
            q_len,
            cam.block_table_tensor,
            cam.seq_lens,
            margin=self._plan_margin,
            causal=causal,
            fixed_grid=True,
        )
        return MjolnirMetadata(plan=plan, runner=self.runner, cam=cam)

    def build_for_cudagraph_capture(self, common_attn_metadata):
        return self.build(0, common_attn_metadata)

    def update_draft_decode_metadata(self, metadata) -> None:
        """Fused draft decode: a kernel-step plan already covers every draft
        step (see the plan margin); fallback metadata is the base's."""
        if getattr(metadata, "kernel_step", False):
            return
        parent = getattr(super(), "update_draft_decode_metadata", None)
        if parent is not None:
            parent(metadata)

    def use_cascade_attention(self, *args, **kwargs) -> bool:
        # the fp6 scratch expands per-request pages: no shared-prefix variant
        if self._fp6:
            return False
        return super().use_cascade_attention(*args, **kwargs)

    # -- fp6 fallback steps ------------------------------------------------------
    def fp6_page_map(self, cam) -> dict:
        """Which cache page becomes which scratch page for a fallback step on
        an fp6 cache, and the block table over the scratch: request r's page j
        lands at scratch page ``offset_r + j`` (a shared prefix page is expanded
        once per request that reads it). Page counts are capped at the block
        table's width, so an upper-bound seq_len never indexes past it
        (reference ``builder.py:479-509``)."""
        num_reqs = int(cam.num_reqs)
        lens = [int(x) for x in list(self.seq_lens_host(cam))[:num_reqs]]
        bt = cam.block_table_tensor
        width = int(bt.shape[1])
        counts = [min(-(-L // self._page), width) if L > 0 else 0 for L in lens]
        total = sum(counts)
        remap = torch.zeros(bt.shape[0], width, dtype=torch.int32)
        rows, cols = [], []
        off = 0
        for r, n in enumerate(counts):
            if n:
                remap[r, :n] = torch.arange(off, off + n, dtype=torch.int32)
                rows += [r] * n
                cols += list(range(n))
            off += n
        dev = bt.device
        r_idx = torch.tensor(rows, dtype=torch.long).to(dev)
        c_idx = torch.tensor(cols, dtype=torch.long).to(dev)
        src = bt[r_idx, c_idx].to(torch.int32).contiguous()
        return {"src_pages": src, "block_table": remap.to(dev), "total": total}

    def _build_fp6_fallback(self, common_prefix_len: int, cam, fast_build: bool):
        """The base builder plans against the scratch's page ids (the block
        table is swapped for the remap during its build), and the metadata
        carries the page map the impl expands before the base forward."""
        pages = self.fp6_page_map(cam)
        orig = cam.block_table_tensor
        cam.block_table_tensor = pages["block_table"]
        try:
            md = super().build(common_prefix_len, cam, fast_build)
        finally:
            cam.block_table_tensor = orig
        md.mjolnir_fp6_pages = pages
        return md
