"""Decode-attention benchmark (the BASELINE.json metric): KV GB/s and us/step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload cfg5] [--kv fp8|e2m3|e3m2|e2m1|nvfp4]
    python -m torch.distributed.run --nproc-per-node N bench.py --gpus N ...
    python bench.py --impl reference ...   # the reference's CPU path (oracle port)

A step is one decode-attention step of the workload: the quantize-on-write of
one new token per sequence, the paged split-KV decode, the LSE combine and,
with N > 1, the NCCL all-gather of the per-rank head slices of the output.
KV heads are sharded across ranks (tensor parallel); the per-rank KV stream
is 1/N of the total. ``value`` = total KV bytes of all ranks / the slowest
rank's device time per step.

Workloads (synthetic data of their shapes; the KV
pages are filled by this repo's own quantize-on-write kernel from N(0,1)
bf16 values):
  cfg2  Qwen3-8B shape: 32 q / 8 KV heads, d 128, b 64, L 8192, fp8, PS 16
  cfg3  Qwen3-8B shape: b 128, e2m3, log-normal L (median 8192, sigma 0.75,
        seed 1234) clipped to [512, 32768], 1 % outliers x8, per-channel scales
  cfg4  Qwen3-32B spec decode: 64 q / 8 KV heads, q_len 6 causal, b 32, L 32768, e2m3
  cfg5  long context, TP over KV heads: 64 q / 8 KV heads, b 256, L 131072,
        e2m3 (default) or --kv fp8
The KV stream of every config is larger than the 126 MB L2, so no L2 flush
is needed between steps.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    "cfg2": dict(h_q=32, h_k=8, d=128, b=64, q_len=1, L=8192, kv="fp8", PS=16),
    "cfg3": dict(h_q=32, h_k=8, d=128, b=128, q_len=1, L="lognormal", kv="e2m3", PS=16),
    "cfg4": dict(h_q=64, h_k=8, d=128, b=32, q_len=6, L=32768, kv="e2m3", PS=16),
    "cfg5": dict(h_q=64, h_k=8, d=128, b=256, q_len=1, L=131072, kv="e2m3", PS=16),
    # the north-star target shape: Qwen3-8B e2m3 decode, batch 128 x 32K context
    "ns": dict(h_q=32, h_k=8, d=128, b=128, q_len=1, L=32768, kv="e2m3", PS=16),
    # the reference harness's own default head shape (24 q / 4 KV heads,
    # head_dim 256, page 128), batch 16 x 32K
    "hd256": dict(h_q=24, h_k=4, d=256, b=16, q_len=1, L=32768, kv="fp8", PS=128),
}


def seq_lens_for(w, seed=1234):
    """Context lengths of a workload. cfg3: log-normal with median 8192 and
    sigma 0.75 (the config fixes the median and the clip range, not sigma),
    drawn in float32 from torch's CPU generator seeded 1234 and clipped to
    [512, 32768]: sum 1,317,124 tokens."""
    if w["L"] == "lognormal":
        g = torch.Generator().manual_seed(seed)
        z = torch.randn(w["b"], generator=g)
        L = torch.exp(math.log(8192.0) + 0.75 * z).round().clamp(512, 32768)
        return [int(x) for x in L.tolist()]
    return [int(w["L"])] * w["b"]


def workload_config(name, kv, world, page_size=None, batch=None, seed=1234):
    """The `config` object of a bench line: the workload only (shapes, format,
    lengths, sharding), the same for our arm and the reference arm."""
    w = dict(WORKLOADS[name])
    kv = kv or w["kv"]
    if page_size:
        w["PS"] = page_size
    if batch:
        w["b"] = batch
    lens = seq_lens_for(w, seed)
    return {"workload": name, "kv_format": kv, "batch": w["b"], "h_q": w["h_q"], "h_k": w["h_k"],
            "head_dim": w["d"], "q_len": w["q_len"], "page_size": w["PS"], "sum_seq_len": int(sum(lens)),
            "parallelism": f"tp{world} (KV heads)", "l2": "KV stream per step > 126 MB L2 (no flush needed)",
            "kv_bytes_per_step": kv_bytes(lens, w["h_k"], w["d"], kv)}


VMAX = {"e2m3": 7.5, "e3m2": 28.0, "e2m1": 6.0}  # largest code value of each narrow format


def row_bytes(d, kv):
    """Packed code bytes of one K (or V) row."""
    return {"fp8": d, "e2m3": d * 3 // 4, "e3m2": d * 3 // 4, "e2m1": d // 2, "nvfp4": d // 2}[kv]


def kv_bytes(lens, h_k, d, kv):
    """KV bytes a decode step streams (nvfp4 rows carry d / 16 scale bytes)."""
    return int(sum(lens)) * h_k * 2 * (row_bytes(d, kv) + (d // 16 if kv == "nvfp4" else 0))


class Workload:
    """One rank's shard of a workload, resident on the device."""

    def __init__(self, name, kv, rank, world, device, seed=1234, page_size=None, batch=None):
        from mjolnir_b200 import kvfp6
        from mjolnir_b200.runner import DecodeRunner, split_kv_cache

        w = dict(WORKLOADS[name])
        if kv:
            w["kv"] = kv
        if page_size:
            w["PS"] = page_size
        if batch:  # a smaller batch of the same shape (profiling captures)
            w["b"] = batch
        self.w, self.name = w, name
        if w["h_k"] % world:
            raise SystemExit(f"{w['h_k']} KV heads do not shard over {world} GPUs")
        self.h_k = w["h_k"] // world
        self.h_q = w["h_q"] // world
        self.d, self.PS, self.q_len, self.b, self.fmt = w["d"], w["PS"], w["q_len"], w["b"], w["kv"]
        self.lens = seq_lens_for(w, seed)
        self.device = device
        g = torch.Generator(device=device).manual_seed(seed + 7919 * rank)
        d, PS, h_k = self.d, self.PS, self.h_k
        rb = row_bytes(d, self.fmt)
        n_blocks = [math.ceil(L / PS) for L in self.lens]
        self.num_pages = sum(n_blocks)
        # shuffled physical pages (seeded identically on every rank)
        perm = torch.randperm(self.num_pages, generator=torch.Generator().manual_seed(seed)).to(torch.int32)
        bt = torch.zeros(self.b, max(n_blocks), dtype=torch.int32)
        i = 0
        for s, nb in enumerate(n_blocks):
            bt[s, :nb] = perm[i:i + nb]
            i += nb
        self.block_table = bt.to(device)
        self.seq_lens = torch.tensor(self.lens, dtype=torch.int32, device=device)
        # the vLLM-main / reference layout (B, H, N, 2*row): K|V cell per (page, head, slot)
        self.kv_cache = torch.empty(self.num_pages, h_k, PS, 2 * rb, dtype=torch.uint8, device=device)
        self.k_view, self.v_view = split_kv_cache(self.kv_cache, "BHN2D", rb)
        self.k_scales = self.v_scales = None
        if self.fmt == "nvfp4":
            # group scales (page, head, slot, K|V, d / 16): a page's rows of one head are contiguous
            self.scale_cache = torch.empty(self.num_pages, h_k, PS, 2, d // 16, dtype=torch.uint8, device=device)
            self.k_scales = self.scale_cache[:, :, :, 0].transpose(1, 2)
            self.v_scales = self.scale_cache[:, :, :, 1].transpose(1, 2)
        outliers = 0.01 if name == "cfg3" else 0.0

        def gen(n):
            x = torch.randn(n, h_k, d, generator=g, device=device)
            if outliers:
                x = torch.where(torch.rand(x.shape, generator=g, device=device) < outliers, x * 8, x)
            return x.to(torch.bfloat16)

        # scales: fp8 per tensor 1.0; narrow formats per (KV head, channel) amax / the
        # format's max of a 1M-token sample of the same distribution (kvscales.e2m3_scales,
        # no headroom)
        if self.fmt == "fp8":
            self.k_scale = self.v_scale = torch.ones(1, device=device)
        elif self.fmt == "nvfp4":  # one global scale per tensor: amax / (6 * 448) (quant.py:74)
            self.k_scale = (gen(1 << 20).float().abs().amax().clamp(min=1e-12) / 2688.0).reshape(1)
            self.v_scale = (gen(1 << 20).float().abs().amax().clamp(min=1e-12) / 2688.0).reshape(1)
        else:
            smp = gen(1 << 20).float()
            self.k_scale = (smp.abs().amax(0).clamp(min=1e-6) / VMAX[self.fmt]).contiguous()
            smp = gen(1 << 20).float()
            self.v_scale = (smp.abs().amax(0).clamp(min=1e-6) / VMAX[self.fmt]).contiguous()
            del smp
        chunk = 1 << 19  # tokens per fill step
        total = self.num_pages * PS
        for t0 in range(0, total, chunk):
            n = min(chunk, total - t0)
            slots = torch.arange(t0, t0 + n, dtype=torch.int64, device=device)
            kvfp6.reshape_and_cache(gen(n), gen(n), self.k_view, self.v_view, slots, self.k_scale, self.v_scale, self.fmt,
                                    k_scales=self.k_scales, v_scales=self.v_scales)
        torch.cuda.synchronize(device)
        h_r = self.h_q // self.h_k
        if self.fmt == "nvfp4":  # descale gs * 2^3 (the converted values carry 2^-3)
            self.q_mul = self.o_mul = None
            self.kd, self.vd = self.k_scale * 8.0, self.v_scale * 8.0
        elif self.fmt != "fp8":
            self.q_mul = self.k_scale.repeat_interleave(h_r, 0).contiguous()
            self.o_mul = self.v_scale.repeat_interleave(h_r, 0).contiguous()
            self.kd = self.vd = torch.ones(1, device=device)
        else:
            self.q_mul = self.o_mul = None
            self.kd, self.vd = self.k_scale, self.v_scale
        T = self.b * self.q_len
        self.T = T
        self.query = torch.randn(T, self.h_q, d, generator=g, device=device).to(torch.bfloat16)
        self.new_k = gen(T)
        self.new_v = gen(T)
        # the step's new tokens sit at the end of each sequence
        slots = []
        for s, L in enumerate(self.lens):
            for qi in range(self.q_len):
                t = L - self.q_len + qi
                slots.append(int(bt[s, t // PS]) * PS + t % PS)
        self.slots = torch.tensor(slots, dtype=torch.int64, device=device)
        self.out = torch.empty(T, self.h_q * d, dtype=torch.bfloat16, device=device)
        self.runner = DecodeRunner(num_heads=self.h_q, num_kv_heads=h_k, head_size=d, page_size=PS,
                                   max_num_seqs=self.b, max_q_len=self.q_len, kv_format=self.fmt, device=device)
        self.plan = self.runner.plan(self.lens, self.b, self.q_len, self.block_table, self.seq_lens)
        self.scale = 1.0 / math.sqrt(d)

    def kv_bytes(self):
        return kv_bytes(self.lens, self.h_k, self.d, self.fmt)

    def algorithmic_decode_bytes(self):
        """Bytes the decode launch must move: KV + Q + O + block-table entries."""
        q = self.T * self.h_q * self.d * 2
        bt = sum(math.ceil(L / self.PS) for L in self.lens) * 4
        return self.kv_bytes() + 2 * q + bt


# ---------------------------------------------------------------------------
# measurement helpers
# ---------------------------------------------------------------------------
class ClockSampler:
    """`nvidia-smi` SM clocks and clock-event (throttle) reasons, sampled every
    50 ms from before the warm-up until after the timed region. The summary
    keeps the samples that arrived inside the timed region (marked with
    `mark_start` / `mark_end`); a region shorter than the sampling period is
    represented by the samples nearest to it. Reads settings only."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.samples = []  # (arrival time, sm_mhz, max_mhz, reason names)
        self.t0 = self.t1 = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for ln in self.proc.stdout:
            f = [x.strip() for x in ln.strip().split(",")]
            if len(f) < 9:
                continue
            try:
                self.samples.append((time.monotonic(), float(f[1]), float(f[2]),
                                     {n for n, v in zip(self.NAMES, f[5:9]) if v.lower() == "active"}))
            except ValueError:
                continue

    def mark_start(self):
        self.t0 = time.monotonic()

    def mark_end(self):
        self.t1 = time.monotonic()

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.15)  # the sample covering the end of the region
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        smp = list(self.samples)
        window = "timed region"
        if self.t0 is not None and self.t1 is not None:
            inside = [x for x in smp if self.t0 <= x[0] <= self.t1 + 0.1]
            if not inside and smp:  # region shorter than the period: the nearest samples
                before = [x for x in smp if x[0] < self.t0][-1:]
                after = [x for x in smp if x[0] > self.t1][:1]
                inside, window = before + after, "nearest to the timed region"
            smp = inside
        sm = [x[1] for x in smp]
        reasons = set().union(*[x[3] for x in smp]) if smp else set()
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smp[-1][2] if smp else None,
                "reasons": sorted(reasons), "samples": len(sm), "window": window}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profiled_traffic(kernel, workload, kv, algorithmic):
    """DRAM bytes per decode launch from the committed ncu capture of this
    kernel: the measured bytes when the capture was this workload, else the
    capture's traffic / algorithmic ratio scaled to this launch's bytes."""
    p = os.path.join(ROOT, "profiles", "decode_traffic.json")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        j = json.load(f).get(kernel)
    if not j:
        return None
    if j["captured_on"] == f"{workload}-{kv}":
        return int(j["dram_bytes_per_launch"])
    return int(round(j["traffic_over_algorithmic"] * algorithmic))


# ---------------------------------------------------------------------------
# the reference arm: the reference's CPU path (its torch dequantise-then-attend
# oracle, restated in oracle/), timed on the host cores
# ---------------------------------------------------------------------------
def cpu_reference_step(name, kv, world, n_seqs=1, seed=1234):
    """One bounded CPU sample of the workload: n_seqs sequences (all heads),
    dequantised from quantized bytes and attended in fp32. Returns
    (seconds, kv_bytes of the sample)."""
    from oracle import attention, quant

    w = dict(WORKLOADS[name])
    if kv:
        w["kv"] = kv
    lens = seq_lens_for(w, seed)[:n_seqs]
    h_k, h_q, d, PS, ql = w["h_k"], w["h_q"], w["d"], w["PS"], w["q_len"]
    rng = np.random.default_rng(seed)
    pages = sum(math.ceil(L / PS) for L in lens)
    bt = torch.arange(pages, dtype=torch.int32)
    bt_rows = []
    i = 0
    width = max(math.ceil(L / PS) for L in lens)
    for L in lens:
        n = math.ceil(L / PS)
        row = torch.zeros(width, dtype=torch.int32)
        row[:n] = bt[i:i + n]
        bt_rows.append(row)
        i += n
    btab = torch.stack(bt_rows)
    rb = row_bytes(d, w["kv"])
    kb = rng.integers(0, 256, size=(pages, PS, h_k, rb), dtype=np.uint8)
    vb = rng.integers(0, 256, size=(pages, PS, h_k, rb), dtype=np.uint8)
    ks = vs = None
    if w["kv"] == "fp8":  # no NaN codes in a real cache
        kb[(kb & 0x7F) == 0x7F] = 0
        vb[(vb & 0x7F) == 0x7F] = 0
    if w["kv"] == "nvfp4":  # group scale bytes, no NaN
        ks = rng.integers(0, 0x7F, size=(pages, PS, h_k, d // 16), dtype=np.uint8)
        vs = rng.integers(0, 0x7F, size=(pages, PS, h_k, d // 16), dtype=np.uint8)
    q = torch.from_numpy(rng.standard_normal((len(lens) * ql, h_q, d)).astype(np.float32)).to(torch.bfloat16)
    t0 = time.perf_counter()
    kvals = attention.dequant_pool(kb, w["kv"], d, ks)
    vvals = attention.dequant_pool(vb, w["kv"], d, vs)
    attention.decode_attention(q, kvals, vvals, btab, lens, len(lens), ql, 1.0 / math.sqrt(d))
    dt = time.perf_counter() - t0
    return dt, kv_bytes(lens, h_k, d, w["kv"])


def run_reference_arm(args, rank, world):
    """--impl reference: the reference's CPU path on the host cores (rank 0)."""
    if rank != 0:
        return
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    name, kv = args.workload, args.kv or WORKLOADS[args.workload]["kv"]
    for _ in range(args.warmup):
        cpu_reference_step(name, kv, world, n_seqs=1)
    times, nbytes = [], 0
    for i in range(args.steps):
        dt, nbytes = cpu_reference_step(name, kv, world, n_seqs=1, seed=1234 + i)
        times.append(dt)
    mean = sum(times) / len(times)
    gbs = nbytes / mean / 1e9
    sample = (f"per step 1 sequence of {name} (all {WORKLOADS[name]['h_k']} KV heads, "
              f"L={seq_lens_for(WORKLOADS[name])[0]}, {nbytes} KV bytes): dequantise + fp32 attend")
    line = {
        "impl": "reference", "metric": "decode-attn KV GB/s", "value": round(gbs, 4), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(mean * 1e3, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic", "config": workload_config(name, kv, world, args.page_size, args.batch),
        "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="cfg5", choices=sorted(WORKLOADS))
    ap.add_argument("--kv", default=None, choices=[None, "fp8", "e2m3", "e3m2", "e2m1", "nvfp4"])
    ap.add_argument("--page-size", type=int, default=None, help="override the workload's KV page size")
    ap.add_argument("--batch", type=int, default=None, help="override the workload's batch (small profiling cases)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    from mjolnir_b200 import _lib, kvfp6
    from mjolnir_b200.runner import _stream

    wl = Workload(args.workload, args.kv, rank, world, dev, page_size=args.page_size, batch=args.batch)
    stream = _stream(dev)
    cw = kvfp6.cache_write_args(wl.new_k, wl.new_v, wl.k_view, wl.v_view, wl.slots, wl.k_scale, wl.v_scale, wl.fmt,
                                k_scales=wl.k_scales, v_scales=wl.v_scales)
    da = wl.runner.decode_args(wl.plan, wl.query, wl.out, wl.k_view, wl.v_view, wl.kd, wl.vd, wl.scale,
                               q_mul=wl.q_mul, o_mul=wl.o_mul, k_scales=wl.k_scales, v_scales=wl.v_scales)
    da.with_combine = 0
    combine = wl.plan.with_reduction and not wl.runner.merges_in_kernel(da)
    if world > 1:
        from mjolnir_b200.tp import gather_heads

        # the all-gather buffer and the re-interleaved (T, h_q, d) output, fixed addresses
        gbuf = torch.empty(world, wl.T, wl.h_q, wl.d, dtype=torch.bfloat16, device=dev)
        full_out = torch.empty(wl.T, world * wl.h_q, wl.d, dtype=torch.bfloat16, device=dev)
        local_out = wl.out.view(wl.T, wl.h_q, wl.d)
    launches_per_step = 2 + int(combine)

    def step(ev=None):
        _lib.cache_write(cw, stream)
        if ev is not None:
            ev[0].record()
        _lib.decode(da, stream)
        if ev is not None:
            ev[1].record()
        if combine:
            _lib.combine(da, stream)
        if world > 1:
            gather_heads(local_out, world, buf=gbuf, out=full_out)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    clk = ClockSampler(local)
    clk.__enter__()  # sampling from before the warm-up, so the timed region has samples
    try:
        for _ in range(args.warmup):
            step()
        barrier()
        dec_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        clk.mark_start()
        t0.record()
        for i in range(args.steps):
            step(dec_ev[i])
        t1.record()
        barrier()
        clk.mark_end()
    finally:
        clk.__exit__(None, None, None)
    ms = t0.elapsed_time(t1) / args.steps
    dec_ms = sum(a.elapsed_time(b) for a, b in dec_ev) / args.steps
    ms_t = torch.tensor([ms, dec_ms], device=dev)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms, dec_ms_max = ms_t.tolist()
    total_kv = wl.kv_bytes() * world

    # e2e through the public API: host Q / new K,V in pinned memory copied in,
    # the output copied back, every step inside the timed region
    q_h = wl.query.cpu().pin_memory()
    k_h = wl.new_k.cpu().pin_memory()
    v_h = wl.new_v.cpu().pin_memory()
    o_h = torch.empty((wl.T, world * wl.h_q * wl.d) if world > 1 else wl.out.shape, dtype=torch.bfloat16).pin_memory()

    def e2e_step():
        wl.query.copy_(q_h, non_blocking=True)
        wl.new_k.copy_(k_h, non_blocking=True)
        wl.new_v.copy_(v_h, non_blocking=True)
        kvfp6.reshape_and_cache(wl.new_k, wl.new_v, wl.k_view, wl.v_view, wl.slots, wl.k_scale, wl.v_scale, wl.fmt,
                                k_scales=wl.k_scales, v_scales=wl.v_scales)
        wl.runner.run(wl.plan, wl.query, wl.out, wl.k_view, wl.v_view, wl.kd, wl.vd, wl.scale, q_mul=wl.q_mul, o_mul=wl.o_mul,
                      k_scales=wl.k_scales, v_scales=wl.v_scales)
        if world > 1:
            gather_heads(local_out, world, buf=gbuf, out=full_out)
            o_h.copy_(full_out.view(wl.T, -1), non_blocking=True)
        else:
            o_h.copy_(wl.out, non_blocking=True)

    for _ in range(2):
        e2e_step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        e2e_step()
    e1.record()
    barrier()
    e2e_ms = torch.tensor([e0.elapsed_time(e1) / args.steps], device=dev)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_ms = float(e2e_ms.item())
    h2d = (q_h.numel() + k_h.numel() + v_h.numel()) * 2
    d2h = o_h.numel() * 2

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cores = os.cpu_count() or 1
        torch.set_num_threads(cores)
        dt, nb = cpu_reference_step(args.workload, wl.fmt, world, n_seqs=1)
        cpu = {"value": round(nb / dt / 1e9, 4), "unit": "GB/s", "cores": cores, "kind": "port",
               "sample": f"1 sequence of {args.workload} (all KV heads, L={wl.lens[0]}): dequantise + fp32 attend, {dt:.1f} s"}

    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    peak, peak_kind = peaks()
    alg = wl.algorithmic_decode_bytes()
    achieved = alg / (dec_ms_max * 1e-3) / 1e9
    kname = wl.runner.kernel_name(da)
    traffic = profiled_traffic(kname, args.workload, wl.fmt, alg)
    line = {
        "metric": "decode-attn KV GB/s",
        "value": round(total_kv / (ms * 1e-3) / 1e9, 2),
        "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 4), "us_per_step": round(ms * 1e3, 1),
        "hbm_frac_of_measured_peak": round(total_kv / world / (ms * 1e-3) / 1e9 / peak, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "fp8-e4m3 KV" if wl.fmt == "fp8" else f"{wl.fmt} KV",
        "data": "synthetic (N(0,1) K/V quantized by the repo's write kernel, shuffled pages, random Q)",
        "config": workload_config(args.workload, wl.fmt, world, args.page_size, args.batch),
        "plan": {"chunk_tiles": wl.plan.chunk_tiles, "work_items": wl.plan.num_chunks, "kernel": kname},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic,
                     "kernel": kname, "peak_source": peak_kind,
                     "algorithmic_bytes_per_launch": alg, "launch_ms": round(dec_ms_max, 4)},
        "cpu_baseline": cpu,
        "e2e": {"value": round(total_kv / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s", "ms_per_step": round(e2e_ms, 4),
                "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
