"""Shared builders for the parity tests: seeded paged KV caches in any vLLM
layout, with shuffled pages and poisoned spare pages (the reference's test
fixtures, tests/kernel/_util.py:54-110)."""

from __future__ import annotations

import math

import numpy as np
import torch

from oracle import attention, quant

FP8_NAN = 0x7F  # poisons fp8 pages no sequence owns
E2M3_POISON = 0x7F  # e2m3 bytes of large codes: any stray read shows in the output

LAYOUT_SHAPES = {
    "BHN2D": lambda P, N, H, R: (P, H, N, 2 * R),
    "BNH2D": lambda P, N, H, R: (P, N, H, 2 * R),
    "B2NHD": lambda P, N, H, R: (P, 2, N, H, R),
    "B2HND": lambda P, N, H, R: (P, 2, H, N, R),
    "2BNHD": lambda P, N, H, R: (2, P, N, H, R),
    "2BHND": lambda P, N, H, R: (2, P, H, N, R),
    "BHN2R": lambda P, N, H, R: (P, H, N, 2, R),
}


class Case:
    """A paged decode case: bytes on the device in ``layout``, the same
    pool's values on the host for the oracle."""

    def __init__(self, *, seq_lens, q_len=1, h_q=8, h_k=2, d=128, page_size=16, kv_format="fp8",
                 layout="B2NHD", seed=0, descale="tensor", max_num_seqs=None, outliers=0.0, device="cuda",
                 q_scale=1.0, k_ramp=0.0):
        from mjolnir_b200.runner import detect_kv_layout, split_kv_cache

        g = torch.Generator().manual_seed(seed)
        self.g = g
        self.q_len, self.h_q, self.h_k, self.d, self.PS = q_len, h_q, h_k, d, page_size
        self.kv_format = kv_format
        self.seq_lens = [max(int(L), 0) for L in seq_lens]
        b = self.b = len(self.seq_lens)
        self.max_num_seqs = max_num_seqs or b
        n_blocks = [max(1, math.ceil(L / page_size)) for L in self.seq_lens]
        self.num_pages = sum(n_blocks) + 3
        perm = torch.randperm(self.num_pages, generator=g).tolist()
        bt = torch.zeros(self.max_num_seqs, max(n_blocks) + 1, dtype=torch.int32)
        i = 0
        used = []
        for s, nb in enumerate(n_blocks):
            bt[s, :nb] = torch.tensor(perm[i:i + nb])
            used += perm[i:i + nb]
            i += nb
        unused = perm[i:]
        self.block_table_cpu = bt
        from mjolnir_b200.runner import row_bytes

        rb = self.row = row_bytes(d, kv_format)
        vmax = {"e2m3": 7.5, "e3m2": 28.0, "e2m1": 6.0}.get(kv_format)
        # host pools: raw values -> quantized bytes (oracle) -> code values
        raw = {}
        for side in ("k", "v"):
            x = torch.randn(self.num_pages, page_size, h_k, d, generator=g)
            if outliers:
                m = torch.rand(x.shape, generator=g) < outliers
                x = torch.where(m, x * 8, x)
            raw[side] = x
        if k_ramp:
            # K grows with the token position (x 1 .. 1 + k_ramp over each
            # sequence): later tiles raise the running max, so the kernels
            # rescale what they accumulated from earlier tiles
            for s, nb in enumerate(n_blocks):
                L = max(self.seq_lens[s], 1)
                for bi in range(nb):
                    pos = torch.arange(bi * page_size, (bi + 1) * page_size, dtype=torch.float32)
                    raw["k"][bt[s, bi]] *= (1.0 + k_ramp * pos / L).view(page_size, 1, 1)
        if kv_format == "fp8":
            self.k_scale_w = self.v_scale_w = torch.ones(1)
        elif kv_format == "nvfp4":
            # the reference harness's choice: one global scale per tensor (quant.py:74)
            self.k_scale_w = torch.tensor([quant.nvfp4_global_scale(raw["k"].to(torch.bfloat16).float().numpy())])
            self.v_scale_w = torch.tensor([quant.nvfp4_global_scale(raw["v"].to(torch.bfloat16).float().numpy())])
        else:
            # per (KV head, channel) amax / the format's max (kvscales.e2m3_scales without headroom)
            self.k_scale_w = raw["k"].abs().amax(dim=(0, 1)).clamp(min=1e-6) / vmax
            self.v_scale_w = raw["v"].abs().amax(dim=(0, 1)).clamp(min=1e-6) / vmax
        self.bytes = {}
        self.vals = {}
        self.group_scales = {}
        for side, sc in (("k", self.k_scale_w), ("v", self.v_scale_w)):
            xb = raw[side].to(torch.bfloat16).float().numpy()
            if kv_format == "nvfp4":
                by, gsc = quant.quantize_rows_nvfp4(xb, sc.double().numpy())
                by[unused] = 0x77  # code +6 in both nibbles
                gsc[unused] = 0x7E  # scale 448 (the reference harness's poison, harness.py:581-583)
                self.group_scales[side] = torch.from_numpy(gsc)
                self.bytes[side] = torch.from_numpy(by)
                self.vals[side] = attention.dequant_pool(by, kv_format, d, gsc)
                continue
            if kv_format == "fp8":
                by = quant.quantize_rows_fp8(xb, sc.numpy())
                by[unused] = FP8_NAN
            else:
                by = quant.quantize_rows_narrow(xb, sc.numpy(), kv_format)
                by[unused] = E2M3_POISON
            self.bytes[side] = torch.from_numpy(by)
            self.vals[side] = attention.dequant_pool(by, kv_format, d)
        # device cache in the requested physical layout, byte-initialized to poison
        shape = LAYOUT_SHAPES[layout](self.num_pages, page_size, h_k, rb)
        cache = torch.full(shape, FP8_NAN if kv_format == "fp8" else E2M3_POISON, dtype=torch.uint8, device=device)
        self.layout = detect_kv_layout(cache.shape, h_k, page_size, rb) if h_k != page_size else layout
        assert self.layout == layout or h_k == page_size
        self.kv_cache = cache
        self.k_view, self.v_view = split_kv_cache(cache, layout, rb)
        self.k_view.copy_(self.bytes["k"].to(device))
        self.v_view.copy_(self.bytes["v"].to(device))
        self.k_scales = self.v_scales = None
        if kv_format == "nvfp4":
            # group scales in their own tensor, K and V interleaved per row:
            # (pages, page_size, h_k, 2, d / 16), so both views are strided
            sc_dev = torch.empty(self.num_pages, page_size, h_k, 2, d // 16, dtype=torch.uint8, device=device)
            self.k_scales, self.v_scales = sc_dev[:, :, :, 0], sc_dev[:, :, :, 1]
            self.k_scales.copy_(self.group_scales["k"].to(device))
            self.v_scales.copy_(self.group_scales["v"].to(device))
            self.scale_cache = sc_dev
        self.block_table = bt.to(device)
        sl = torch.zeros(self.max_num_seqs, dtype=torch.int32)
        sl[:b] = torch.tensor(self.seq_lens, dtype=torch.int32)
        self.seq_lens_t = sl.to(device)
        # descales (fp8; nvfp4: gs * 2^3) -- e2m3 uses the channel scales through q_mul / o_mul
        if kv_format == "nvfp4":
            self.kd = (self.k_scale_w.double() / quant.NVFP4_SHIFT).float()
            self.vd = (self.v_scale_w.double() / quant.NVFP4_SHIFT).float()
            self.q_mul = self.o_mul = None
        elif kv_format == "fp8":
            if descale == "tensor":
                self.kd, self.vd = torch.tensor([1.0]), torch.tensor([1.0])
            elif descale == "head":
                self.kd, self.vd = torch.rand(h_k, generator=g) + 0.5, torch.rand(h_k, generator=g) + 0.5
            else:
                self.kd, self.vd = torch.rand(b, h_k, generator=g) + 0.5, torch.rand(b, h_k, generator=g) + 0.5
            self.q_mul = self.o_mul = None
        else:
            self.kd, self.vd = torch.ones(1), torch.ones(1)
            h_r = h_q // h_k
            self.q_mul = self.k_scale_w.repeat_interleave(h_r, 0).contiguous()
            self.o_mul = self.v_scale_w.repeat_interleave(h_r, 0).contiguous()
        T = b * q_len
        self.query_cpu = (torch.randn(T, h_q, d, generator=g) * q_scale).to(torch.bfloat16)
        # Q as a strided view of a wider fused-QKV row
        fused = torch.zeros(T, (h_q + 2 * h_k) * d, dtype=torch.bfloat16, device=device)
        fused[:, : h_q * d] = self.query_cpu.reshape(T, h_q * d).to(device)
        self.query = fused[:, : h_q * d].view(T, h_q, d)

    def dev(self, t):
        return None if t is None else t.to(self.query.device)

    def oracle(self):
        return attention.decode_attention(
            self.query_cpu, self.vals["k"], self.vals["v"], self.block_table_cpu, self.seq_lens, self.b,
            self.q_len, 1.0 / math.sqrt(self.d), self.kd, self.vd, causal=self.causal, q_mul=self.q_mul,
            o_mul=self.o_mul,
        )

    causal = True

    def runner(self, **kw):
        from mjolnir_b200.runner import DecodeRunner

        return DecodeRunner(num_heads=self.h_q, num_kv_heads=self.h_k, head_size=self.d, page_size=self.PS,
                            max_num_seqs=self.max_num_seqs, max_q_len=self.q_len, kv_format=self.kv_format,
                            device=self.query.device, **kw)

    def run(self, out_dtype=torch.float32, causal=True, lse=False, fixed_grid=False, **runner_kw):
        self.causal = causal
        r = self.runner(**runner_kw)
        plan = r.plan(self.seq_lens, self.b, self.q_len, self.block_table, self.seq_lens_t, causal=causal,
                      fixed_grid=fixed_grid)
        T = self.b * self.q_len
        out = torch.full((T + 2, self.h_q * self.d), float("nan"), dtype=out_dtype, device=self.query.device)
        lse_t = torch.full((T, self.h_q), float("nan"), device=self.query.device) if lse else None
        r.run(plan, self.query, out, self.k_view, self.v_view, self.dev(self.kd), self.dev(self.vd),
              1.0 / math.sqrt(self.d), q_mul=self.dev(self.q_mul), o_mul=self.dev(self.o_mul), lse=lse_t,
              k_scales=self.k_scales, v_scales=self.v_scales)
        torch.cuda.synchronize()
        r.check_status()
        return out, lse_t, plan


def assert_close_fp32(got: torch.Tensor, ref: torch.Tensor, max_abs=2e-3, mean_abs=2e-4, what=""):
    """The north-star tolerance: max-abs 2e-3 and mean-abs 2e-4 in fp32."""
    got = got.float().cpu()
    ref = ref.float().cpu()
    assert torch.isfinite(got).all(), f"{what}: non-finite output"
    err = (got - ref).abs()
    assert err.max().item() <= max_abs, f"{what}: max abs {err.max().item():.3g} > {max_abs}"
    assert err.mean().item() <= mean_abs, f"{what}: mean abs {err.mean().item():.3g} > {mean_abs}"
    return err.max().item(), err.mean().item()


def assert_close_bf16(got: torch.Tensor, ref: torch.Tensor, what=""):
    """bf16 output: the fp32 tolerance plus the bf16 rounding of the result
    (half an ulp: |ref| * 2^-8)."""
    got = got.float().cpu()
    ref = ref.float().cpu()
    err = (got - ref).abs()
    bound = 2e-3 + ref.abs() * 2.0**-8
    assert (err <= bound).all(), f"{what}: bf16 error beyond 2e-3 + half-ulp (worst {(err - bound).max().item():.3g})"
