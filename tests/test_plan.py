"""Split-KV planner: the reference's plan reproduced exactly (rebalance off),
and the B200 rebalance's invariants."""

import os

import numpy as np
import pytest

from mjolnir_b200.plan import plan_split_kv
from tests.conftest import GOLDEN


def test_matches_reference_plans():
    g = np.load(os.path.join(GOLDEN, "plan.npz"))
    n = len({k.split("__")[0] for k in g.files})
    for i in range(n):
        hk, nqt, sm, cps, ms = (int(x) for x in g[f"plan{i}__args"])
        p = plan_split_kv(g[f"plan{i}__lens"].tolist(), hk, nqt, sm, ctas_per_sm=cps, max_splits=ms, rebalance=False)
        np.testing.assert_array_equal(np.array(p.work).reshape(-1, 4), g[f"plan{i}__work"])
        np.testing.assert_array_equal(p.n_splits, g[f"plan{i}__n_splits"])
        assert [p.chunk_tiles, p.slots] == g[f"plan{i}__chunk"].tolist()


def _coverage(lens, p):
    tiles = [max(1, -(-L // 128)) for L in lens]
    seen = {b: [] for b in range(len(lens))}
    for s, tb, te, j in p.work:
        if te > tb:
            seen[s].append((j, tb, te))
    for b, t in enumerate(tiles):
        parts = sorted(seen[b])
        assert [j for j, _, _ in parts] == list(range(len(parts))) == list(range(p.n_splits[b]))
        assert parts[0][1] == 0 and parts[-1][2] == t
        for (_, _, e), (_, s, _) in zip(parts, parts[1:]):
            assert e == s


@pytest.mark.parametrize("lens", [[8192] * 64, [8192] * 128, [32768] * 32, [131072] * 256, [5, 900, 17000, 3] * 40])
def test_rebalance_covers_every_tile(lens):
    p = plan_split_kv(lens, 8, 1, 148, ctas_per_sm=2, max_splits=16)
    _coverage(lens, p)
    lengths = [te - tb for _, tb, te, _ in p.work]
    assert lengths == sorted(lengths, reverse=True)


def test_rebalance_fixes_config2_wave_quantization():
    """64 seqs x 8 heads = 512 CTAs on 296 slots: the reference leaves 1.73
    waves; the rebalanced plan fills whole waves better."""
    ref = plan_split_kv([8192] * 64, 8, 1, 148, ctas_per_sm=2, rebalance=False)
    new = plan_split_kv([8192] * 64, 8, 1, 148, ctas_per_sm=2)
    assert ref.chunk_tiles == 64
    assert new.chunk_tiles < 64
    waves_new = -(-len(new.work) // new.slots) * new.chunk_tiles
    waves_ref = -(-len(ref.work) // ref.slots) * ref.chunk_tiles
    assert waves_new < waves_ref


def test_pad_to_and_errors():
    p = plan_split_kv([300, 10], 2, 1, 148, ctas_per_sm=2, pad_to=64)
    assert len(p.work) == 64 and p.work[-1] == (0, 0, 0, 0)
    with pytest.raises(ValueError):
        plan_split_kv([300000] * 8, 2, 1, 148, ctas_per_sm=2, pad_to=3)


def test_native_planner_matches_python():
    """mj_plan_split_kv (C++, for hosts without Python) gives the same plans."""
    import random

    from mjolnir_b200 import _lib

    rng = random.Random(1)
    for _ in range(120):
        n = rng.randint(1, 300)
        lens = [rng.choice([rng.randint(0, 5000), rng.randint(1, 140000), 8192]) for _ in range(n)]
        hk, nt = rng.choice([1, 2, 4, 8]), rng.choice([1, 2, 3])
        sm, cps, ms = rng.choice([148, 132, 8]), rng.choice([1, 2]), rng.choice([1, 4, 16])
        reb, ov, pad = rng.choice([True, False]), rng.choice([0.5, 2.0]), rng.choice([0, n * ms + 5])
        p = plan_split_kv(lens, hk, nt, sm, ctas_per_sm=cps, max_splits=ms, pad_to=pad, rebalance=reb, item_overhead=ov)
        w, ns, chunk = _lib.plan_split_kv(lens, hk, nt, sm, cps, ms, pad, reb, ov)
        assert np.array_equal(w, p.work_array()) and ns == p.n_splits and chunk == p.chunk_tiles
