"""fp32 dequantise-then-attend decode attention on the CPU (test infrastructure).

Restates the reference's exact attention over a paged, quantized KV cache:
``ref_decode`` (GoBrrr-ai/mjolnir ``src/mjolnir/mjolnir/arch/orin/harness.py:31-79``),
which equals the ``o_exact`` output of ``emulate_decode``
(``src/mjolnir/mjolnir/arch/thor/harness.py:51-155``, lines 152-154):

* token ``t`` of sequence ``b`` lives at page ``block_table[b, t // PS]``, row
  ``t % PS``; ``seq_lens`` INCLUDE the step's own ``q_len`` query tokens
  (``arch/thor/decode.py:40``);
* query token ``qi`` of a sequence of length ``L`` sees keys ``0 .. L - q_len + qi``
  when causal (``harness.py:115-117``; ``orin/harness.py:72``), all ``L`` keys
  otherwise;
* scores are ``q . k * softmax_scale * k_descale`` (``q_descale`` is 1 for a
  bf16 query), softmax in fp32, ``O = P V * v_descale``;
* the e2m3 per-channel scales fold as the backend does (``backend.py:370-381``):
  K's into Q (``q_mul``, (h_q, d)), V's into the output (``o_mul``, (h_q, d)).

A query row with no visible key (``L < q_len`` under the causal tail) gets
O = 0 and LSE = -inf, the kernel's empty-row guard (``decode.py:1271-1278``).
"""

from __future__ import annotations

import math

import numpy as np
import torch

from . import quant


def dequant_pool(pool_bytes: np.ndarray | torch.Tensor, kv_format: str, d: int, scales=None) -> torch.Tensor:
    """(pages, PS, h_k, row_bytes) uint8 -> (pages, PS, h_k, d) float32 code values
    (nvfp4: the e4m3 kernel values from the (pages, PS, h_k, d / 16) scale bytes)."""
    b = pool_bytes.numpy() if isinstance(pool_bytes, torch.Tensor) else np.asarray(pool_bytes)
    if kv_format == "nvfp4":
        sc = scales.numpy() if isinstance(scales, torch.Tensor) else np.asarray(scales)
        return torch.from_numpy(quant.decode_rows_nvfp4(b, sc, d))
    if kv_format == "fp8":
        return torch.from_numpy(quant.decode_fp8(b))
    if kv_format == "e2m3":
        return torch.from_numpy(quant.decode_rows_e2m3(b, d))
    if kv_format in ("e3m2", "e2m1"):
        return torch.from_numpy(quant.decode_rows_narrow(b, d, kv_format))
    raise ValueError(kv_format)


def expand_descale(t, num_seqs: int, h_k: int) -> torch.Tensor:
    """1-element | (h_k,) | (b, h_k) -> (b, h_k) float32 (the strides rule of
    ``arch/thor/plan.py:39-47``)."""
    t = torch.as_tensor(t, dtype=torch.float32).cpu()
    if t.numel() == 1:
        return t.reshape(1, 1).expand(num_seqs, h_k)
    if t.dim() == 1:
        return t.reshape(1, h_k).expand(num_seqs, h_k)
    return t[:num_seqs]


def decode_attention(
    q: torch.Tensor,  # (num_seqs * q_len, h_q, d) any float dtype
    k_vals: torch.Tensor,  # (pages, PS, h_k, d) float32 dequantized (no descale)
    v_vals: torch.Tensor,
    block_table: torch.Tensor,  # (>= num_seqs, max_blocks) int
    seq_lens,  # (>= num_seqs,) int, including the q_len new tokens
    num_seqs: int,
    q_len: int,
    softmax_scale: float,
    k_descale=1.0,
    v_descale=1.0,
    causal: bool = True,
    q_mul: torch.Tensor | None = None,  # (h_q, d)
    o_mul: torch.Tensor | None = None,  # (h_q, d)
    num_threads: int | None = None,
):
    """Returns (o (num_seqs * q_len, h_q, d) float32, lse (num_seqs * q_len, h_q) float32)."""
    if num_threads:
        torch.set_num_threads(num_threads)
    T, h_q, d = q.shape[0], q.shape[1], q.shape[2]
    PS, h_k = k_vals.shape[1], k_vals.shape[2]
    h_r = h_q // h_k
    kd = expand_descale(k_descale, num_seqs, h_k)
    vd = expand_descale(v_descale, num_seqs, h_k)
    qf = q[: num_seqs * q_len].float().cpu()
    if q_mul is not None:
        qf = qf * q_mul.float().cpu().view(1, h_q, d)
    out = torch.zeros(num_seqs * q_len, h_q, d)
    lse = torch.full((num_seqs * q_len, h_q), -math.inf)
    bt = torch.as_tensor(block_table).cpu().long()
    lens = [int(x) for x in torch.as_tensor(seq_lens).cpu()[:num_seqs].tolist()]
    for b in range(num_seqs):
        L = lens[b]
        if L <= 0:
            continue
        n_blk = -(-L // PS)
        pages = bt[b, :n_blk]
        K = k_vals[pages].reshape(-1, h_k, d)[:L]  # (L, h_k, d)
        V = v_vals[pages].reshape(-1, h_k, d)[:L]
        qb = qf[b * q_len : (b + 1) * q_len].view(q_len, h_k, h_r, d)
        s = torch.einsum("qkrd,lkd->qkrl", qb, K)
        s = s * (softmax_scale * kd[b]).view(1, h_k, 1, 1)
        if causal:
            lim = torch.arange(q_len) + (L - q_len)  # last visible key per query token
            mask = torch.arange(L).view(1, L) > lim.view(q_len, 1)  # (q_len, L)
            s = s.masked_fill(mask.view(q_len, 1, 1, L), -math.inf)
        m = s.amax(dim=-1, keepdim=True)
        empty = torch.isinf(m) & (m < 0)
        m = torch.where(empty, torch.zeros_like(m), m)
        p = torch.exp(s - m)
        l = p.sum(dim=-1, keepdim=True)
        o = torch.einsum("qkrl,lkd->qkrd", p, V) / torch.where(l > 0, l, torch.ones_like(l))
        o = o * vd[b].view(1, h_k, 1, 1)
        ls = (m + torch.log(l)).squeeze(-1)  # log(0) = -inf for empty rows
        out[b * q_len : (b + 1) * q_len] = o.reshape(q_len, h_q, d)
        lse[b * q_len : (b + 1) * q_len] = ls.reshape(q_len, h_q)
    if o_mul is not None:
        out = out * o_mul.float().cpu().view(1, h_q, d)
    return out, lse


def merge_splits(o_parts: torch.Tensor, lse_parts: torch.Tensor):
    """LSE merge of chunk-normalized partials (the reduction of
    ``arch/thor/decode.py:1473-1541``, in its chunk-normalized form):
    o_parts (S, ..., d) each the softmax-normalized output of one KV chunk,
    lse_parts (S, ...) natural-log sum-exp of that chunk's scaled scores.
    Returns (o (..., d), lse (...)). Chunks with lse = -inf carry no weight."""
    m = lse_parts.amax(dim=0)
    m_safe = torch.where(torch.isinf(m) & (m < 0), torch.zeros_like(m), m)
    w = torch.exp(lse_parts - m_safe)  # (S, ...)
    den = w.sum(dim=0)
    o = (w.unsqueeze(-1) * o_parts).sum(dim=0) / torch.where(den > 0, den, torch.ones_like(den)).unsqueeze(-1)
    lse = m_safe + torch.log(den)
    return o, lse


def kv_bytes(seq_lens, h_k: int, d: int, kv_format: str) -> int:
    """Algorithmic KV bytes one decode step streams: sum(L) * h_k * 2 rows
    (nvfp4 rows carry their d / 16 scale bytes)."""
    row = {"fp8": d, "e2m3": d * 3 // 4, "e3m2": d * 3 // 4, "e2m1": d // 2, "nvfp4": d // 2 + d // 16}[kv_format]
    return int(sum(int(x) for x in seq_lens)) * h_k * 2 * row
