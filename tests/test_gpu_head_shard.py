"""Head-sharded single stream on one GPU against the unsharded layer loop.

P ranks are emulated in one process on one device: every rank's token-shard
phase runs, then the all-to-all is done as device copies between the ranks'
exchange buffers, then every rank's head-shard attention, the second exchange
and the token-shard rest of the layer -- the data flow of HeadShardedStack
under torchrun, without kernels that wait on one another. Each kernel
computes a token row or an attention head independently of the others, so the
sharded stream must reproduce the unsharded LayerStack (hidden states and KV
cache planes, by head group) over a prefix block and several body blocks of
routed attention."""
import numpy as np
import pytest
import torch

from tests.golden import recipes
from tests.util import assert_no_device_error, dev_bf16, host

pytestmark = pytest.mark.gpu

DIM, HEADS, FFN, H, W = 512, 4, 1024, 4, 6
ACTIONS = ["recent_2", "recent_2_anchor", "none"]


def _blocks():
    from recavsr_b200.runtime.block import FusedBlock, rope_tables
    tables = rope_tables(128, H, W, "cuda")
    blocks = []
    for i in range(len(ACTIONS)):
        w = {k: dev_bf16(v) for k, v in recipes.block_params(DIM, HEADS, FFN, seed=60 + i).items()}
        w["heads"] = HEADS
        blocks.append(FusedBlock(w, H, W, tables))
    return blocks


def _emulated_step(stacks, shards, frames):
    world = len(stacks)
    n = stacks[0].plan_block(shards[0].shape[0], frames)
    for s in stacks[1:]:
        s.plan_block(shards[0].shape[0], frames)
    sws = [s.shard_workspace(n, frames) for s in stacks]
    for i in range(len(ACTIONS)):
        for s, h, sw in zip(stacks, shards, sws):
            s.layer_pre(i, h, sw)
        for r, sw in enumerate(sws):
            for j in range(world):
                sw.recv[j].copy_(sws[j].send[r])
        for s, sw in zip(stacks, sws):
            s.layer_attend(i, sw, frames)
        for r, sw in enumerate(sws):
            for j in range(world):
                sw.back[j].copy_(sws[j].attn_h.view(world, sw.n_loc, sw.e)[r])
        for s, h, sw in zip(stacks, shards, sws):
            s.layer_post(i, h, sw)


def _close(got, ref, what):
    rel = np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30)
    mx = np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30)
    same = float(np.mean(got == ref))
    # Expected bit-identical; the bound leaves room for a rare NVFP4 code flip,
    # a head or token routed to the wrong place gives errors of order 1.
    assert rel < 2e-3 and mx < 5e-2, f"{what}: rel L2 {rel:.2e}, max {mx:.2e}, identical {same:.4f}"


@pytest.mark.parametrize("world", [2, 4])
def test_head_sharded_stream_matches_unsharded_stack(world):
    from recavsr_b200.runtime.block import LayerStack
    from recavsr_b200.runtime.head_shard import HeadShardedStack
    blocks = _blocks()
    full = LayerStack(blocks, ACTIONS)
    stacks = [HeadShardedStack(blocks, ACTIONS, rank=r, world=world, exchange=lambda *_: None)
              for r in range(world)]
    hl = HEADS // world
    rs = np.random.RandomState(world)
    span = H * W
    for blk_i in range(6):
        frames = 6 if blk_i == 0 else 2
        n = frames * span
        x = recipes.bf16_round(rs.standard_normal((n, DIM)).astype(np.float32))
        hf = dev_bf16(x)
        full.step(hf, frames)
        n_loc = n // world
        shards = [dev_bf16(x[r * n_loc:(r + 1) * n_loc]) for r in range(world)]
        _emulated_step(stacks, shards, frames)
        got = np.concatenate([host(s) for s in shards])
        _close(got, host(hf), f"block {blk_i} hidden")
        for i, c in enumerate(full.caches):
            if not c.capacity:
                continue
            for r, s in enumerate(stacks):
                assert s.route_host.tolist() == full.route_host.tolist()
                for t, (fc, sc) in enumerate(((full.cache_k, s.cache_k), (full.cache_v, s.cache_v))):
                    ref = host(fc[i])[0][:, r * hl:(r + 1) * hl]
                    _close(host(sc[i])[0], ref, f"block {blk_i} layer {i} rank {r} {'kv'[t]} cache")
    assert_no_device_error()


def test_head_sharded_stream_single_rank_step():
    """world = 1 through step(): the exchange is a local copy, one shard holds
    every token and head."""
    from recavsr_b200.runtime.block import LayerStack
    from recavsr_b200.runtime.head_shard import HeadShardedStack
    blocks = _blocks()
    full = LayerStack(blocks, ACTIONS)
    one = HeadShardedStack(blocks, ACTIONS, rank=0, world=1)
    rs = np.random.RandomState(3)
    span = H * W
    for blk_i in range(4):
        frames = 6 if blk_i == 0 else 2
        x = recipes.bf16_round(rs.standard_normal((frames * span, DIM)).astype(np.float32))
        hf, hs = dev_bf16(x), dev_bf16(x)
        full.step(hf, frames)
        one.step(hs, frames)
        _close(host(hs), host(hf), f"block {blk_i}")
    with pytest.raises(ValueError):
        one.step(dev_bf16(x[:span]), 2)
    with pytest.raises(ValueError):
        HeadShardedStack(blocks, ACTIONS, rank=0, world=3)
    assert_no_device_error()
