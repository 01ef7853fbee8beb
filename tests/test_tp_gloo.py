"""Tensor parallelism over KV heads on CPU ranks (gloo, world size 2): head
sharding, the output all-gather and re-interleave against the single-rank
oracle, and host-side failure detection (a rank that raises before the
collective, a rank that never joins) ending in an error, not a hang."""

import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from mjolnir_b200.tp import gather_heads, head_shard, interleave, local_query


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(seed=3, b=3, q_len=2, h_q=8, h_k=4, d=32, PS=4):
    g = torch.Generator().manual_seed(seed)
    lens = [9, 17, 5]
    pages = 16
    k = torch.randn(pages, PS, h_k, d, generator=g)
    v = torch.randn(pages, PS, h_k, d, generator=g)
    bt = torch.randperm(pages, generator=g)[: b * 5].reshape(b, 5)
    q = torch.randn(b * q_len, h_q, d, generator=g)
    return q, k, v, bt, lens, b, q_len


def test_head_shard_ranges():
    s = head_shard(64, 8, 3, 4)
    assert (s.kv_begin, s.kv_end, s.q_begin, s.q_end) == (6, 8, 48, 64)
    assert s.local_h_k == 2 and s.local_h_q == 16
    with pytest.raises(ValueError):
        head_shard(64, 8, 0, 3)
    q = torch.zeros(5, 64, 128)
    lq = local_query(q, s)
    assert lq.data_ptr() == q[:, 48].data_ptr() and lq.stride() == q.stride()


def test_interleave_is_head_major():
    world, T, hl, d = 3, 2, 2, 4
    g = torch.arange(world * T * hl * d, dtype=torch.float32).view(world, T, hl, d)
    full = interleave(g)
    for r in range(world):
        assert torch.equal(full[:, r * hl : (r + 1) * hl], g[r])
    out = torch.empty(T, world * hl, d)
    assert interleave(g, out) is out and torch.equal(out, full)


def _rank_main(rank, world, port, mode, q_out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist

    from oracle.attention import decode_attention

    try:
        if mode == "never_joins" and rank == 1:
            return
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=6))
        q, k, v, bt, lens, b, q_len = _case()
        s = head_shard(q.shape[1], k.shape[2], rank, world)
        o_local, _ = decode_attention(local_query(q, s), k[:, :, s.kv_begin : s.kv_end], v[:, :, s.kv_begin : s.kv_end],
                                      bt, lens, b, q_len, 0.3)
        if mode == "raises" and rank == 1:
            raise RuntimeError("planted failure before the collective")
        full = gather_heads(o_local, world)
        if rank == 0:
            ref, _ = decode_attention(q, k, v, bt, lens, b, q_len, 0.3)
            q_out.put(("ok", float((full - ref).abs().max())))
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001 - reported to the parent
        q_out.put((f"error rank {rank}", type(e).__name__ + ": " + str(e)[:200]))


def _run(mode, timeout=60):
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, mode, q_out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail(f"{mode}: a rank hung past {timeout} s")
    out = []
    while not q_out.empty():
        out.append(q_out.get())
    return out


def test_gloo_world2_matches_single_rank_oracle():
    res = _run("ok")
    assert res and res[0][0] == "ok", res
    assert res[0][1] < 1e-5


@pytest.mark.parametrize("mode", ["raises", "never_joins"])
def test_failed_rank_ends_the_others_with_an_error(mode):
    res = _run(mode)
    kinds = sorted(r[0] for r in res)
    assert "error rank 0" in kinds, res  # the healthy rank reports, it does not hang
