"""Tensor parallelism over KV heads: shard, decode locally, all-gather the output.

Attention never mixes KV heads (a GQA group reads only its own KV head), so
rank r of ``world`` owns KV heads ``[r * h_k / world, (r + 1) * h_k / world)``,
the matching query heads, its own KV pool shard, and runs the cache write,
the decode and the split combine locally with no data-path collective. The
only exchange is one all-gather of the bf16 output, ``(T, h_q / world, d)``
per rank, re-interleaved into ``(T, h_q, d)`` (reference tensor-parallel
serving shards attention heads the same way; the reference itself runs one
GPU, so this layer has no counterpart file there).

The all-gather goes through ``torch.distributed`` (NCCL on the GPUs; gloo on
CPU ranks in the tests); ranks must call :func:`gather_heads` in the same
order, and a rank that fails or never arrives ends the others' collective
with the process group's timeout.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class HeadShard:
    """The heads one rank owns."""

    rank: int
    world: int
    h_q: int  # global query heads
    h_k: int  # global KV heads
    kv_begin: int
    kv_end: int
    q_begin: int
    q_end: int

    @property
    def local_h_k(self) -> int:
        return self.kv_end - self.kv_begin

    @property
    def local_h_q(self) -> int:
        return self.q_end - self.q_begin


def head_shard(h_q: int, h_k: int, rank: int, world: int) -> HeadShard:
    """Rank ``rank``'s KV and query head ranges; ``world`` must divide h_k."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    if h_k % world:
        raise ValueError(f"tensor parallel size {world} does not divide {h_k} KV heads")
    if h_q % h_k:
        raise ValueError(f"{h_q} query heads are not a multiple of {h_k} KV heads")
    per_k = h_k // world
    h_r = h_q // h_k
    k0 = rank * per_k
    return HeadShard(rank, world, h_q, h_k, k0, k0 + per_k, k0 * h_r, (k0 + per_k) * h_r)


def local_query(query: torch.Tensor, shard: HeadShard) -> torch.Tensor:
    """Zero-copy view of this rank's query heads of a (T, h_q, d) query (the
    decode kernel reads Q through its token and head strides)."""
    return query[:, shard.q_begin : shard.q_end, :]


def interleave(gathered: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """(world, T, h_q_local, d) rank-major -> (T, world * h_q_local, d) head-major."""
    world, T, hl, d = gathered.shape
    src = gathered.permute(1, 0, 2, 3)
    if out is None:
        return src.reshape(T, world * hl, d)
    out.view(T, world, hl, d).copy_(src)
    return out


def gather_heads(local_out: torch.Tensor, world: int, group=None, buf: torch.Tensor | None = None,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """All-gather every rank's (T, h_q_local, d) output and return the full
    (T, h_q, d) output. ``buf`` (world, T, h_q_local, d) and ``out`` may be
    preallocated (fixed addresses for CUDA graphs)."""
    import torch.distributed as dist

    T, hl, d = local_out.shape
    if buf is None:
        buf = torch.empty(world, T, hl, d, dtype=local_out.dtype, device=local_out.device)
    dist.all_gather_into_tensor(buf.view(world * T, hl, d), local_out.contiguous(), group=group)
    return interleave(buf, out)
