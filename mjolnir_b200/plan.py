"""Host-side split-KV planning for the decode kernel.

The unit of work is a contiguous chunk of 128-row KV tiles of one sequence,
(seq, tile_begin, tile_end, split); the decode grid runs one CTA per (work
item, KV head), and sequences cut into several chunks are merged by the LSE
combine.

``plan_split_kv`` keeps the reference's occupancy-pinned rule
(GoBrrr-ai/mjolnir ``src/mjolnir/mjolnir/arch/thor/plan.py:140-197``, the
FlashDecoding / FlashInfer scheme): one wave holds
``slots = sm_count * ctas_per_sm // (heads_k * n_q_tiles)`` work items; when
the batch is smaller than a wave, the SMALLEST chunk whose total work fits one
wave is chosen; items are ordered longest first and optionally padded to a
fixed length with empty items so a CUDA graph replays a fixed grid.

B200 addition (``rebalance=True``): when the batch alone fills a wave the
reference does not split at all, which on 148 SMs leaves a ragged last wave
(e.g. 64 sequences x 8 KV heads = 512 CTAs = 1.73 waves of 296). The planner
then evaluates every chunk size ceil(T / k), k = 1 .. max_splits, with a
longest-first wave model -- the sum over waves of the longest item in each
wave, plus a per-item overhead -- and keeps the cheapest. The overhead
(2 tiles) is the tensor-core kernel's measured per-job cost: preparing the
job's Q and writing its O / partials take about as long as two 128-row tiles.
``rebalance=False`` reproduces the reference plan exactly.
"""

from __future__ import annotations

import math

import numpy as np

TILE_ROWS = 128  # KV rows per tile (the kernel's unit)


class SplitPlan:
    def __init__(self, work, n_splits, chunk_tiles, slots):
        self.work = work  # list of (seq, tile_begin, tile_end, split)
        self.n_splits = n_splits  # chunks per sequence
        self.chunk_tiles = chunk_tiles
        self.slots = slots

    @property
    def num_work(self) -> int:
        return len(self.work)

    @property
    def max_splits_used(self) -> int:
        return max(self.n_splits) if self.n_splits else 1

    def work_array(self) -> np.ndarray:
        w = np.asarray(self.work if self.work else [(0, 0, 0, 0)], dtype=np.int32)
        return w.reshape(-1, 4)

    def __repr__(self):
        real = sum(1 for w in self.work if w[2] > w[1])
        pad = self.num_work - real
        return (
            f"SplitPlan(chunk={self.chunk_tiles} tiles, work={real}{f'+{pad} pad' if pad else ''}, "
            f"slots/wave={self.slots}, max chunks/seq={self.max_splits_used})"
        )


def _wave_cost(tiles: np.ndarray, chunk: int, slots: int, item_overhead: float) -> float:
    """Longest-first wave model of the decode time, in tile units."""
    k = np.ceil(tiles / chunk).astype(np.int64)
    full = np.repeat(np.full(len(tiles), chunk, dtype=np.int64), np.maximum(k - 1, 0))
    last = tiles - (k - 1) * chunk
    lens = np.sort(np.concatenate([full, last]))[::-1]
    wave_heads = lens[::slots]  # longest item of each wave
    return float(wave_heads.sum() + item_overhead * len(wave_heads)) + (0.25 if k.max() > 1 else 0.0)


def plan_split_kv(
    seq_lens,
    heads_k: int,
    n_q_tiles: int,
    sm_count: int,
    ctas_per_sm: int = 1,
    max_splits: int = 16,
    force_splits: int = 0,
    min_chunk_tiles: int = 1,
    pad_to: int = 0,
    rebalance: bool = True,
    item_overhead: float = 2.0,
) -> SplitPlan:
    tiles = [max(1, math.ceil(int(L) / TILE_ROWS)) for L in seq_lens]
    T = max(tiles)
    slots = max(1, (sm_count * ctas_per_sm) // (heads_k * n_q_tiles))
    lo = max(min_chunk_tiles, math.ceil(T / max_splits))  # cap chunks per sequence
    if force_splits > 0:
        chunk = max(lo, math.ceil(T / force_splits))
    elif max_splits == 1:
        chunk = T
    elif len(tiles) >= slots:
        chunk = T
        if rebalance:
            t = np.asarray(tiles, dtype=np.int64)
            cands = sorted({max(lo, math.ceil(T / k)) for k in range(1, max_splits + 1)}, reverse=True)
            best = None
            for c in cands:
                cost = _wave_cost(t, c, slots, item_overhead)
                if best is None or cost < best[0] - 1e-9:
                    best = (cost, c)
            chunk = best[1]
    else:
        hi = T
        while lo < hi:  # smallest chunk whose total work fits one wave
            mid = (lo + hi) // 2
            if sum(math.ceil(t / mid) for t in tiles) <= slots:
                hi = mid
            else:
                lo = mid + 1
        chunk = lo
    work, n_splits = [], []
    for b, t in enumerate(tiles):
        k = math.ceil(t / chunk)
        n_splits.append(k)
        work.extend((b, j * chunk, min((j + 1) * chunk, t), j) for j in range(k))
    work.sort(key=lambda w: -(w[2] - w[1]))  # longest first (stable)
    if pad_to:
        if pad_to < len(work):
            raise ValueError(f"pad_to {pad_to} < {len(work)} work items")
        work += [(0, 0, 0, 0)] * (pad_to - len(work))
    assert max(n_splits) <= max_splits
    return SplitPlan(work, n_splits, chunk, slots)
