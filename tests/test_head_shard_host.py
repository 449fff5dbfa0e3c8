"""Host side of the head-sharded single stream (recavsr_b200/runtime/head_shard.py),
on CPU: token shards, rank-local spatial tables, the pack / all-to-all / unpack
permutations between token and head shards (in one process for P = 1..8, and
over real gloo ranks for P = 2 and 4), and the composition the stack relies
on: routed attention run per head shard (oracle restatement of
recavsr_infer/kernels/local_attention.py:286-325) and exchanged back equals the
unsharded attention of every token."""
import datetime
import os
import socket
import traceback

import numpy as np
import pytest
import torch

from recavsr_b200.runtime.head_shard import (local_exchange, local_spatial_tables, pack_heads,
                                             token_shard, unpack_heads, unpack_tokens)


def test_token_shard_bounds_and_errors():
    assert [token_shard(48, 4, r) for r in range(4)] == [(0, 12), (12, 12), (24, 12), (36, 12)]
    assert token_shard(16320, 8, 7) == (14280, 2040)
    with pytest.raises(ValueError):
        token_shard(50, 4, 0)
    with pytest.raises(ValueError):
        token_shard(48, 4, 4)


def test_local_spatial_tables_follow_token_positions():
    span, d = 24, 8
    cos = torch.arange(span * d, dtype=torch.float32).reshape(span, d)
    sin = -cos
    for start, count in ((0, 12), (12, 12), (36, 12), (20, 8)):
        lc, ls, sp = local_spatial_tables(cos, sin, span, start, count)
        assert sp == count and lc.shape == (count, d)
        for i in range(count):
            assert torch.equal(lc[i], cos[(start + i) % span])
            assert torch.equal(ls[i], sin[(start + i) % span])


def _emulated_all_to_all(sends):
    """recv_r[j] = send_j[r] for every pair of ranks."""
    world = len(sends)
    return [torch.stack([sends[j][r] for j in range(world)]) for r in range(world)]


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_exchange_permutations_in_one_process(world):
    heads, d, n = 8, 16, 32
    e = heads // world * d
    g = torch.Generator().manual_seed(world)
    q, k, v, o = (torch.randn(n, heads * d, generator=g).bfloat16() for _ in range(4))
    qkv = torch.cat([q, k, v], 1)       # the fused QKV layout: row-strided views
    n_loc = n // world
    sends = []
    for r in range(world):
        s0, _ = token_shard(n, world, r)
        rows = slice(s0, s0 + n_loc)
        send = torch.empty(world, 3, n_loc, e, dtype=torch.bfloat16)
        pack_heads(qkv[rows, :heads * d], qkv[rows, heads * d:2 * heads * d], qkv[rows, 2 * heads * d:], send)
        sends.append(send)
    recvs = _emulated_all_to_all(sends) if world > 1 else [sends[0].clone()]
    backs = []
    for r in range(world):
        qkv_h = torch.empty(3, n, e, dtype=torch.bfloat16)
        unpack_heads(recvs[r], qkv_h)
        cols = slice(r * e, (r + 1) * e)
        for i, x in enumerate((q, k, v)):
            assert torch.equal(qkv_h[i], x[:, cols])
        backs.append(o[:, cols].contiguous().view(world, n_loc, e))
    for r, recv in enumerate(_emulated_all_to_all(backs) if world > 1 else backs):
        out = torch.empty(n_loc, heads * d, dtype=torch.bfloat16)
        unpack_tokens(recv, out)
        s0, _ = token_shard(n, world, r)
        assert torch.equal(out, o[s0:s0 + n_loc])
    with pytest.raises(ValueError):
        pack_heads(q[:n_loc - 1], k[:n_loc - 1], v[:n_loc - 1], sends[0])


def test_local_exchange_copies():
    send = torch.randn(1, 3, 4, 8)
    recv = torch.empty_like(send)
    local_exchange(recv, send)
    assert torch.equal(recv, send)


# ------------------------------------------------------- gloo ranks (CPU)
H, W, FRAMES, HEADS, D = 3, 4, 2, 4, 128
SLOTS, PPOS, QPOS = [1, -1, 0], [4, 0, 5], [6, 7]


def _attention_inputs():
    from oracle.numerics import bf16_round
    rs = np.random.RandomState(77)
    span = H * W
    n, cap = FRAMES * span, len(SLOTS)
    bf = lambda *s: bf16_round(rs.standard_normal(s).astype(np.float32))
    return bf(n, HEADS, D), bf(n, HEADS, D), bf(n, HEADS, D), bf(cap * span, HEADS, D), bf(cap * span, HEADS, D)


def _oracle_attention(q, k, v, pk, pv):
    from oracle import attention as oatt
    from oracle import rope as orope
    tc, ts, _, _ = orope.rolling_tables(D, H, W)
    return oatt.routed_attention(q[None], k[None], v[None], pk[None], pv[None], SLOTS, PPOS, QPOS,
                                 tc, ts, H, W, 22, 40)[0]


def _rank_main(rank, world, port, results):
    import torch.distributed as dist
    from recavsr_b200.runtime.head_shard import AllToAll
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        q, k, v, pk, pv = _attention_inputs()
        n = q.shape[0]
        hl = HEADS // world
        e = hl * D
        s0, n_loc = token_shard(n, world, rank)
        tok = lambda a: torch.from_numpy(a[s0:s0 + n_loc].reshape(n_loc, HEADS * D)).bfloat16()
        send = torch.empty(world, 3, n_loc, e, dtype=torch.bfloat16)
        pack_heads(tok(q), tok(k), tok(v), send)
        recv = torch.empty_like(send)
        exchange = AllToAll()
        exchange(recv, send)
        qkv_h = torch.empty(3, n, e, dtype=torch.bfloat16)
        unpack_heads(recv, qkv_h)
        heads = slice(rank * hl, (rank + 1) * hl)
        for i, a in enumerate((q, k, v)):
            assert np.array_equal(qkv_h[i].float().numpy(), a[:, heads].reshape(n, e)), f"tensor {i}"
        # this rank's heads of every token, its own head shard of the cache planes
        qh, kh, vh = (qkv_h[i].float().numpy().reshape(n, hl, D) for i in range(3))
        out_h = _oracle_attention(qh, kh, vh, pk[:, heads], pv[:, heads])
        attn_h = torch.from_numpy(np.ascontiguousarray(out_h, np.float32).reshape(n, e))
        back = torch.empty(world, n_loc, e)
        exchange(back, attn_h.view(world, n_loc, e))
        attn_tok = torch.empty(n_loc, HEADS * D)
        unpack_tokens(back, attn_tok)
        full = _oracle_attention(q, k, v, pk, pv)[s0:s0 + n_loc].reshape(n_loc, HEADS * D)
        np.testing.assert_allclose(attn_tok.numpy(), full, rtol=1e-5, atol=1e-6)
        dist.barrier()
        results.put((rank, None))
    except Exception:
        results.put((rank, traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_head_shard_exchange_over_gloo_ranks(world):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(world):
            rank, err = results.get(timeout=180)
            got[rank] = err
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert sorted(got) == list(range(world))
    for rank, err in got.items():
        assert err is None, f"rank {rank}:\n{err}"


def _failing_rank_main(rank, world, port, results):
    """Rank 1 leaves before the exchange (a host-side failure); rank 0's
    all-to-all must end with an error, not hang."""
    import time

    import torch.distributed as dist
    from recavsr_b200.runtime.head_shard import AllToAll
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        results.put((rank, "left"))
        return                                   # never joins the collective
    send = torch.zeros(world, 3, 4, 8)
    recv = torch.empty_like(send)
    t0 = time.monotonic()
    try:
        AllToAll()(recv, send)
        results.put((rank, "no error"))
    except Exception as e:                      # noqa: BLE001 - any collective error is the expected outcome
        results.put((rank, f"error after {time.monotonic() - t0:.1f} s: {type(e).__name__}"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:                        # noqa: BLE001
            pass


def test_head_shard_exchange_fails_cleanly_when_a_rank_leaves():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_rank_main, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(2):
            rank, msg = results.get(timeout=120)
            got[rank] = msg
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert got[1] == "left"
    assert got[0].startswith("error after"), got[0]
