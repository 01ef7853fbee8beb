"""Generate the golden fixtures that pin ``oracle/`` to the reference.

Runs the reference's own Python implementation (GoBrrr-ai/mjolnir, the kernel
package under ``src/mjolnir``) on seeded inputs and writes its outputs as
``tests/golden/*.npz``. It needs the reference checkout, so it runs only in
the development container:

    python tests/golden/make_golden.py [--ref /path/to/mjolnir/src/mjolnir]

Reference functions exercised:
  quant.minifloat_quantize / pack_subbyte     (src/mjolnir/mjolnir/quant.py:34-65)
  quant.nvfp4_quantize                        (src/mjolnir/mjolnir/quant.py:68-84)
  kvfp6.quantize_rows_reference / decode_...  (src/mjolnir/mjolnir/kvfp6.py:342-365)
  the fp8 cache write (x / s).to(e4m3)        (src/mjolnir/mjolnir/arch/thor/harness.py:588-590)
  arch.orin.harness.ref_decode                (src/mjolnir/mjolnir/arch/orin/harness.py:31-79)
  arch.thor.harness.emulate_decode o_exact    (src/mjolnir/mjolnir/arch/thor/harness.py:51-155)
  arch.thor.plan.plan_split_kv                (src/mjolnir/mjolnir/arch/thor/plan.py:140-197)
"""

from __future__ import annotations

import argparse
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _import_ref(path):
    sys.path.insert(0, path)
    from mjolnir import kvfp6, quant  # noqa: F401
    from mjolnir.arch.orin.harness import ref_decode
    from mjolnir.arch.thor.harness import emulate_decode
    from mjolnir.arch.thor.plan import plan_split_kv

    return kvfp6, quant, ref_decode, emulate_decode, plan_split_kv


def all_bf16() -> torch.Tensor:
    bits = torch.arange(65536, dtype=torch.int32).to(torch.int16)
    return bits.view(torch.bfloat16)


def gen_quant(kvfp6):
    out = {}
    x = all_bf16().float().reshape(512, 1, 128)  # every bf16 bit pattern, h_k = 1
    for name, s in (("s1", 1.0), ("s037", 0.37), ("s3", 3.0)):
        out[f"e2m3_all_{name}"] = kvfp6.quantize_rows_reference(x, torch.tensor([s])).numpy()
        xs = (x / s).clamp(-448.0, 448.0)
        out[f"fp8_all_{name}"] = xs.to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    g = torch.Generator().manual_seed(11)
    # per KV head scales (reference test_fp6_write_matches_reference shapes)
    k = (torch.randn(37, 4, 256, generator=g) * 3).to(torch.bfloat16)
    ks = torch.tensor([0.5, 0.4, 0.7, 0.45])
    out["rand_head_x"] = k.view(torch.int16).numpy()
    out["rand_head_s"] = ks.numpy()
    out["rand_head_e2m3"] = kvfp6.quantize_rows_reference(k.float(), ks).numpy()
    out["rand_head_fp8"] = (k.float() / ks.view(1, 4, 1)).clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    # per (KV head, channel) scales with outlier channels
    g = torch.Generator().manual_seed(21)
    ch = torch.rand(4, 128, generator=g) * 0.2 + 0.01
    ch[:, ::17] *= 20.0
    v = (torch.randn(29, 4, 128, generator=g) * ch * 7.5 / 3).to(torch.bfloat16)
    out["rand_chan_x"] = v.view(torch.int16).numpy()
    out["rand_chan_s"] = ch.numpy()
    out["rand_chan_e2m3"] = kvfp6.quantize_rows_reference(v.float(), ch).numpy()
    # config-3 style: N(0,1) with 1 % outliers x8, scales amax / 7.5 per (head, channel)
    g = torch.Generator().manual_seed(1234)
    x3 = torch.randn(64, 8, 128, generator=g)
    mask = torch.rand(x3.shape, generator=g) < 0.01
    x3 = torch.where(mask, x3 * 8, x3).to(torch.bfloat16)
    s3 = (x3.float().abs().amax(dim=0).clamp(min=1e-6) / 7.5)
    out["cfg3_x"] = x3.view(torch.int16).numpy()
    out["cfg3_s"] = s3.numpy()
    out["cfg3_e2m3"] = kvfp6.quantize_rows_reference(x3.float(), s3).numpy()
    # round trip values
    out["cfg3_decoded"] = kvfp6.decode_rows_reference(torch.from_numpy(out["cfg3_e2m3"]), 128).numpy()
    return out


def gen_narrow(quant):
    """e3m2 / e2m1 (and e2m3) codes of every bf16 value at three scales:
    the reference's minifloat_quantize then pack_subbyte (quant.py:34-65)."""
    out = {}
    x = all_bf16().float().reshape(512, 1, 128)
    for fmt, bits in (("e3m2", 6), ("e2m1", 4)):
        for name, s in (("s1", 1.0), ("s037", 0.37), ("s3", 3.0)):
            codes, _ = quant.minifloat_quantize(x / s, fmt)
            out[f"{fmt}_all_{name}"] = quant.pack_subbyte(codes, bits).numpy()
        out[f"{fmt}_table"] = quant.minifloat_table(fmt).numpy()
    return out


def gen_nvfp4(quant):
    """nvfp4 (quant.py:68-84): codes, e4m3 group scales, global scale, kernel
    values and descale of the reference's nvfp4_quantize on seeded inputs --
    random rows at three magnitudes with zeroed elements, zero groups and
    outliers, and every bf16 value of magnitude 2^-27 .. 2^13 (both signs)."""
    out = {}
    g = torch.Generator().manual_seed(4)
    cases = {}
    for i, mag in enumerate((1e-3, 1.0, 50.0)):
        x = torch.randn(3, 8, 128, generator=g) * mag
        x[torch.rand(x.shape, generator=g) < 0.2] = 0.0
        x[0, 0, :16] = 0.0  # a zero group
        x[1, 2, 5] *= 40.0  # an outlier
        cases[f"rand{i}"] = x
    bits = torch.arange(65536, dtype=torch.int32)
    expo = (bits >> 7) & 0xFF
    keep = bits[(expo >= 100) & (expo <= 140)]
    keep = keep[torch.randperm(keep.numel(), generator=g)]
    n = keep.numel() // 1024 * 1024
    cases["bf16"] = (keep[:n].to(torch.int16).view(torch.bfloat16).float()).reshape(-1, 8, 128)
    for name, x in cases.items():
        codes, sc, gs, vals, desc = quant.nvfp4_quantize(x.clone())
        out[f"{name}__x"] = x.numpy()
        out[f"{name}__codes"] = quant.pack_subbyte(codes, 4).numpy()
        out[f"{name}__sc"] = sc.view(torch.uint8).numpy()
        out[f"{name}__gs"] = np.array([gs, desc], dtype=np.float64)
        out[f"{name}__kern"] = vals.to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    return out


def make_pool(g, seq_lens, PS, h_k, d, kv_format, kvfp6, spare=3):
    """Shuffled pages; spare (unreferenced) pages poisoned (0x7F for fp8, 0xFF for e2m3)."""
    n_blocks = [max(1, math.ceil(L / PS)) for L in seq_lens]
    num_pages = sum(n_blocks) + spare
    perm = torch.randperm(num_pages, generator=g).tolist()
    bt = torch.zeros(len(seq_lens), max(n_blocks) + 1, dtype=torch.int32)
    i = 0
    for s, nb in enumerate(n_blocks):
        bt[s, :nb] = torch.tensor(perm[i : i + nb])
        i += nb
    unused = perm[i:]
    x = {}
    for side in ("k", "v"):
        raw = torch.randn(num_pages, PS, h_k, d, generator=g)
        if kv_format == "fp8":
            kd = torch.ones(1)  # the case table below picks the fp8 descales
            b = raw.to(torch.float8_e4m3fn).view(torch.uint8).clone()
            b[unused] = 0x7F
            vals = b.view(torch.float8_e4m3fn).float()
        else:
            kd = raw.abs().amax(dim=(0, 1, 3)).clamp(min=1e-6) / 7.5  # per KV head
            b = kvfp6.quantize_rows_reference(raw, kd).clone()
            b[unused] = 0xFF
            vals = kvfp6.decode_rows_reference(b, d)
        x[side] = (b, vals, kd)
    return bt, x


def gen_decode(kvfp6, ref_decode, emulate_decode):
    cases = {
        # name: (seq_lens, q_len, h_q, h_k, d, PS, kv_format, descale kind, causal)
        "fp8_q1": ((1, 37, 300, 129), 1, 8, 2, 128, 16, "fp8", "tensor", True),
        "fp8_mtp4": ((4, 100, 257), 4, 16, 2, 128, 16, "fp8", "head", True),
        "e2m3_q1": ((513, 18, 130), 1, 8, 2, 128, 16, "e2m3", "head", True),
        "e2m3_mtp3_noncausal": ((40, 200), 3, 12, 2, 128, 32, "e2m3", "head", False),
        "fp8_seqhead_d256": ((77, 150), 2, 8, 1, 256, 64, "fp8", "seqhead", True),
    }
    out = {}
    for ci, (name, (lens, ql, h_q, h_k, d, PS, fmt, dk, causal)) in enumerate(cases.items()):
        g = torch.Generator().manual_seed(100 + ci)
        b = len(lens)
        bt, kv = make_pool(g, lens, PS, h_k, d, fmt, kvfp6)
        kb, kvals, kd = kv["k"]
        vb, vvals, vd = kv["v"]
        if fmt == "fp8":
            if dk == "tensor":
                kd = torch.tensor([1.0])
                vd = torch.tensor([1.0])
            elif dk == "head":
                kd = torch.rand(h_k, generator=g) + 0.5
                vd = torch.rand(h_k, generator=g) + 0.5
            else:
                kd = torch.rand(b, h_k, generator=g) + 0.5
                vd = torch.rand(b, h_k, generator=g) + 0.5
        q = torch.randn(b * ql, h_q, d, generator=g).to(torch.bfloat16)
        scale = 1.0 / math.sqrt(d)

        def exp2(t):
            t = t.float()
            if t.numel() == 1:
                return t.reshape(1, 1).expand(b, h_k)
            if t.dim() == 1:
                return t.reshape(1, h_k).expand(b, h_k)
            return t

        sl = torch.tensor(lens, dtype=torch.int32)
        o_ref = ref_decode(
            q.view(b, ql, h_q, d), kvals, vvals, bt, sl, None, exp2(kd), exp2(vd), scale, causal=causal
        )  # (b, ql, h_q, d)
        # emulate_decode's exact path (packed q rows n = qi * h_r + r)
        h_r = h_q // h_k
        qp = q.float().view(b, ql, h_k, h_r, d).permute(0, 2, 1, 3, 4).reshape(b, h_k, ql * h_r, d)
        _, _, o_ex = emulate_decode(
            qp, kvals, vvals, bt, sl, torch.ones(b, h_k), exp2(kd), exp2(vd), scale, 1.0, ql, 1 << 30, False, causal=causal
        )
        o_ex = o_ex.view(b, h_k, ql, h_r, d).permute(0, 2, 1, 3, 4).reshape(b, ql, h_q, d)
        pre = f"{name}__"
        out[pre + "meta"] = np.array([ql, h_q, h_k, d, PS, int(causal), int(fmt == "e2m3")], dtype=np.int64)
        out[pre + "seq_lens"] = sl.numpy()
        out[pre + "block_table"] = bt.numpy()
        out[pre + "k_bytes"] = kb.numpy()
        out[pre + "v_bytes"] = vb.numpy()
        out[pre + "k_descale"] = kd.float().numpy()
        out[pre + "v_descale"] = vd.float().numpy()
        out[pre + "q_bits"] = q.view(torch.int16).numpy()
        diff = (o_ref - o_ex).abs().max().item()
        assert diff < 1e-5, f"{name}: ref_decode vs emulate_decode exact differ by {diff}"
        print(f"{name}: ref_decode vs emulate_decode o_exact max diff {diff:.3g}")
        out[pre + "o_ref"] = o_ref.reshape(b * ql, h_q, d).numpy()
    return out


def gen_plan(plan_split_kv):
    out = {}
    cases = [
        ((8192,) * 64, 8, 1, 148, 2, 16),
        ((300, 1, 2049, 128), 2, 1, 148, 2, 16),
        ((32768,) * 32, 8, 3, 148, 1, 16),
        ((131072,) * 4, 8, 1, 148, 2, 16),
        ((5, 900, 17000, 3, 64, 12000, 2500), 4, 2, 148, 2, 8),
        ((100000,), 1, 1, 20, 2, 16),
    ]
    for i, (lens, hk, nqt, sm, cps, ms) in enumerate(cases):
        p = plan_split_kv(list(lens), hk, nqt, sm, ctas_per_sm=cps, max_splits=ms)
        out[f"plan{i}__args"] = np.array([hk, nqt, sm, cps, ms], dtype=np.int64)
        out[f"plan{i}__lens"] = np.array(lens, dtype=np.int64)
        out[f"plan{i}__work"] = np.array(p.work, dtype=np.int64).reshape(-1, 4)
        out[f"plan{i}__n_splits"] = np.array(p.n_splits, dtype=np.int64)
        out[f"plan{i}__chunk"] = np.array([p.chunk_tiles, p.slots], dtype=np.int64)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("MJOLNIR_REF_SRC"),
                    help="the reference package directory (src/mjolnir of its checkout)")
    args = ap.parse_args()
    if not args.ref:
        ap.error("pass --ref or set MJOLNIR_REF_SRC")
    kvfp6, quant, ref_decode, emulate_decode, plan_split_kv = _import_ref(args.ref)
    torch.manual_seed(0)
    np.savez_compressed(os.path.join(HERE, "quant.npz"), **gen_quant(kvfp6))
    np.savez_compressed(os.path.join(HERE, "narrow.npz"), **gen_narrow(quant))
    np.savez_compressed(os.path.join(HERE, "nvfp4.npz"), **gen_nvfp4(quant))
    np.savez_compressed(os.path.join(HERE, "decode.npz"), **gen_decode(kvfp6, ref_decode, emulate_decode))
    np.savez_compressed(os.path.join(HERE, "plan.npz"), **gen_plan(plan_split_kv))
    for f in ("quant.npz", "narrow.npz", "nvfp4.npz", "decode.npz", "plan.npz"):
        print(f, os.path.getsize(os.path.join(HERE, f)), "bytes")


if __name__ == "__main__":
    main()
