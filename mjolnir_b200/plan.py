"""Host-side split-KV planning for the decode kernel.

A work item is a contiguous run of 128-row KV tiles of one sequence,
``(seq, tile_begin, tile_end, split)``. The decode runs one job per (work
item, KV head [, row group]) on persistent CTAs that stride through the job
list, and a sequence cut into several items has its partial outputs merged by
the LSE combine.

Every plan is fixed by one number, the chunk length in tiles: sequence ``b``
with ``t_b`` tiles becomes ``ceil(t_b / chunk)`` items of ``chunk`` tiles (the
last one shorter), listed longest first (ties keep sequence order) and
optionally padded with empty items to a fixed length for CUDA-graph replay.

How the chunk is chosen:

* the contract of the reference (GoBrrr-ai/mjolnir
  ``src/mjolnir/mjolnir/arch/thor/plan.py:140-197``), kept exactly with
  ``rebalance=False``: a wave holds ``slots = sm_count * ctas_per_sm //
  (heads_k * n_q_tiles)`` items; a batch of at least one wave is not split,
  a smaller one gets the shortest chunk whose items still fit in one wave;
  ``max_splits`` bounds the items per sequence from below on the chunk.
* the B200 rebalance (``rebalance=True``, the default) scores the
  reference's chunk and every ``ceil(T / k)``, k = 1 .. max_splits, with a
  persistent-grid model: CTA ``j`` runs items ``j, j + slots, ...`` of the
  sorted list, so the step takes the sum over rounds of each round's longest
  item, plus a per-item cost (``item_overhead`` tiles: preparing a job's Q and
  writing its output cost about two tiles on the tensor-core kernel) and a
  quarter tile for the combine launch when anything splits. The cheapest
  chunk wins; on a tie the longer one. This fixes both ragged last rounds of
  large batches (64 sequences x 8 KV heads = 512 jobs on 296 slots) and
  batches a little smaller than a wave, which the reference leaves unsplit
  (256 sequences x 1 KV head on 296 slots idles 40 slots for the whole step).
"""

from __future__ import annotations

import bisect
import math

import numpy as np

TILE_ROWS = 128  # KV rows per tile (the kernel's unit)


class SplitPlan:
    """The work list of one decode step and what was decided to build it."""

    def __init__(self, work, n_splits, chunk_tiles, slots):
        self.work = work  # [(seq, tile_begin, tile_end, split)], longest first, then padding
        self.n_splits = n_splits  # items per sequence
        self.chunk_tiles = chunk_tiles
        self.slots = slots  # items one round of the persistent grid runs at once

    @property
    def num_work(self) -> int:
        return len(self.work)

    @property
    def max_splits_used(self) -> int:
        return max(self.n_splits, default=1)

    def work_array(self) -> np.ndarray:
        rows = self.work or [(0, 0, 0, 0)]
        return np.asarray(rows, dtype=np.int32).reshape(-1, 4)

    def __repr__(self):
        used = [w for w in self.work if w[2] > w[1]]
        extra = self.num_work - len(used)
        pad = f" (+{extra} empty)" if extra else ""
        return (f"<SplitPlan {len(used)} items{pad} of <= {self.chunk_tiles} tiles, {self.slots} per round, "
                f"<= {self.max_splits_used} per sequence>")


def _items_for(tiles, chunk: int) -> int:
    return sum(-(-t // chunk) for t in tiles)


def _reference_chunk(tiles, slots: int, shortest: int) -> int:
    """The reference's choice: no split once the batch fills a round, else the
    shortest chunk (not below `shortest`) whose items fit in one round."""
    longest = max(tiles)
    if len(tiles) >= slots or shortest >= longest:
        return longest
    candidates = range(shortest, longest + 1)  # item count falls as the chunk grows
    return candidates[bisect.bisect_left(candidates, True, key=lambda c: _items_for(tiles, c) <= slots)]


def _round_cost(tiles: np.ndarray, chunk: int, slots: int, item_overhead: float) -> float:
    """Model of a persistent-grid step, in tiles: sum over rounds of each
    round's longest item plus `item_overhead` per round, plus 0.25 for the
    combine launch when some sequence splits."""
    per_seq = -(-tiles // chunk)
    lengths = np.full(int(per_seq.sum()), chunk, dtype=np.int64)
    ends = np.cumsum(per_seq) - 1  # each sequence's last (possibly shorter) item
    lengths[ends] = tiles - (per_seq - 1) * chunk
    lengths[::-1].sort()  # longest first
    leaders = lengths[::slots]  # round r starts with item r * slots, the longest of its round
    return float(leaders.sum()) + item_overhead * len(leaders) + (0.25 if per_seq.max() > 1 else 0.0)


def _cheapest_chunk(tiles, slots: int, shortest: int, max_splits: int, ref_chunk: int, item_overhead: float) -> int:
    longest = max(tiles)
    options = {max(shortest, -(-longest // k)) for k in range(1, max_splits + 1)} | {ref_chunk}
    t = np.asarray(tiles, dtype=np.int64)
    best_chunk, best_cost = None, math.inf
    for chunk in sorted(options, reverse=True):  # a longer chunk keeps a tie
        cost = _round_cost(t, chunk, slots, item_overhead)
        if cost < best_cost - 1e-9:
            best_chunk, best_cost = chunk, cost
    return best_chunk


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
    tiles = [max(1, -(-int(L) // TILE_ROWS)) for L in seq_lens]
    longest = max(tiles)
    slots = max(1, (sm_count * ctas_per_sm) // (heads_k * n_q_tiles))
    shortest = max(min_chunk_tiles, -(-longest // max_splits))  # at most max_splits items per sequence
    if force_splits > 0:
        chunk = max(shortest, -(-longest // force_splits))
    elif max_splits == 1:
        chunk = longest
    else:
        chunk = _reference_chunk(tiles, slots, shortest)
        if rebalance:
            chunk = _cheapest_chunk(tiles, slots, shortest, max_splits, chunk, item_overhead)
    n_splits = [-(-t // chunk) for t in tiles]
    items = [(b, s * chunk, min(t, (s + 1) * chunk), s) for b, t in enumerate(tiles) for s in range(n_splits[b])]
    items.sort(key=lambda w: w[1] - w[2])  # longest first; sort is stable
    if pad_to:
        if pad_to < len(items):
            raise ValueError(f"pad_to {pad_to} is below the {len(items)} work items of this plan")
        items.extend([(0, 0, 0, 0)] * (pad_to - len(items)))
    if max(n_splits) > max_splits:
        raise AssertionError(f"plan cut a sequence into {max(n_splits)} > max_splits {max_splits} items")
    return SplitPlan(items, n_splits, chunk, slots)
