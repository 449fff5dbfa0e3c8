"""Fused DiT block and layer loop on the GPU against the reference's own block
output (tests/golden) and the oracle's block / router restatement."""
import numpy as np
import pytest
import torch

from oracle import block as oblock
from oracle import rope as orope
from oracle.cache import RouterState, rope_origin
from oracle.numerics import bf16_from_bits, bf16_round
from tests.golden import recipes
from tests.util import assert_no_device_error, dev_bf16, host

pytestmark = pytest.mark.gpu


def _weights(p, heads, device="cuda"):
    w = {k: dev_bf16(v) for k, v in p.items()}
    w["heads"] = heads
    return w


def _oracle_params(p, H, W, heads, cross_k, cross_v, modulation, matmul_dtype=np.float64):
    dim = p["q_w"].shape[1]
    tc, ts, sc, ss = orope.rolling_tables(dim // heads, H, W)
    lin = {n: oblock.QuantLinear(p[n + "_w"], p[n + "_b"], matmul_dtype)
           for n in ("q", "k", "v", "o", "cq", "co", "up", "down")}
    return {"_linears": lin, "modulation": modulation, "norm_q": p["norm_q"], "norm_k": p["norm_k"],
            "cnorm_q": p["cnorm_q"], "norm2_w": p["norm2_w"], "norm2_b": p["norm2_b"],
            "cross_k": cross_k, "cross_v": cross_v, "temporal_cos": tc, "temporal_sin": ts,
            "spatial_cos": sc, "spatial_sin": ss}


def _close(got, ref, rel_l2=1e-2, max_frac=0.1):
    rel = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    mx = np.abs(got - ref).max() / np.abs(ref).max()
    assert rel < rel_l2 and mx < max_frac, (rel, mx)


def test_fused_block_matches_reference_block(golden):
    """Same inputs as the reference PreparedBlock fixture (NVFP4 linears)."""
    from recavsr_b200.runtime.block import FusedBlock, rope_tables
    dim, heads, ffn, H, W, cap = (int(v) for v in golden["block_meta"])
    p = recipes.block_params(dim, heads, ffn)
    blk = FusedBlock(_weights(p, heads), H, W, rope_tables(dim // heads, H, W, "cuda"))
    hidden, pk, pv = recipes.block_inputs(2 * H * W, cap * H * W, dim)
    d = dim // heads
    h, k, v = blk(dev_bf16(hidden), dev_bf16(pk).reshape(1, -1, heads, d),
                  dev_bf16(pv).reshape(1, -1, heads, d),
                  torch.tensor([1, -1, 2], dtype=torch.int32, device="cuda"),
                  torch.tensor([4, 0, 5], dtype=torch.int32, device="cuda"),
                  torch.tensor([6, 7], dtype=torch.int32, device="cuda"))
    assert_no_device_error()
    # cross K/V and modulation are computed on the device like the reference's
    np.testing.assert_allclose(host(blk.modulation), golden["block_modulation"].reshape(6, dim), rtol=0, atol=0)
    ck = bf16_from_bits(golden["block_cross_k"]).reshape(-1, heads, d)
    assert np.abs(host(blk.cross_k) - ck).max() <= 2 ** -6 * np.abs(ck).max()
    ref_h = bf16_from_bits(golden["block_hidden"]).reshape(h.shape)
    ref_k = bf16_from_bits(golden["block_k"]).reshape(k.shape)
    ref_v = bf16_from_bits(golden["block_v"]).reshape(v.shape)
    _close(host(k), ref_k, 5e-3, 2 ** -5)
    _close(host(v), ref_v, 5e-3, 2 ** -5)
    _close(host(h), ref_h)


def test_fused_block_vs_oracle_midsize():
    """dim 768 (6 heads), FFN 2048, 8x12 grid, 2-frame block over 2 cache planes."""
    from recavsr_b200.runtime.block import FusedBlock, rope_tables
    dim, heads, ffn, H, W = 768, 6, 2048, 8, 12
    span = H * W
    p = recipes.block_params(dim, heads, ffn, enc_len=64, seed=21)
    blk = FusedBlock(_weights(p, heads), H, W, rope_tables(128, H, W, "cuda"))
    hidden, pk, pv = recipes.block_inputs(2 * span, 2 * span, dim, seed=22)
    h, k, v = blk(dev_bf16(hidden), dev_bf16(pk).reshape(1, -1, heads, 128),
                  dev_bf16(pv).reshape(1, -1, heads, 128),
                  torch.tensor([1, 0], dtype=torch.int32, device="cuda"),
                  torch.tensor([3, 4], dtype=torch.int32, device="cuda"),
                  torch.tensor([5, 6], dtype=torch.int32, device="cuda"))
    assert_no_device_error()
    params = _oracle_params(p, H, W, heads, host(blk.cross_k), host(blk.cross_v), host(blk.modulation))
    rh, rk, rv = oblock.block_forward(params, hidden[0], pk[0].reshape(-1, heads, 128),
                                      pv[0].reshape(-1, heads, 128), [1, 0], [3, 4], [5, 6], H, W,
                                      (22, 40), heads=heads)
    _close(host(k)[0], rk, 5e-3, 2 ** -5)
    _close(host(h)[0], rh)


def _oracle_stack_step(params_list, routers, caches, hidden, start, frames, H, W, heads):
    origin, qpos = rope_origin(start, frames)
    span = H * W
    d = hidden.shape[1] // heads
    h = hidden
    for i, (prm, rt) in enumerate(zip(params_list, routers)):
        slots, ppos = rt.history(origin)
        cap = rt.capacity
        pk = caches[i][0] if cap else np.zeros((0, heads, d), np.float32)
        pv = caches[i][1] if cap else np.zeros((0, heads, d), np.float32)
        h, k, v = oblock.block_forward(prm, h, pk, pv, list(slots), list(ppos), list(qpos), H, W,
                                       (22, 40), heads=heads)
        for off, slot in rt.commit(frames, start):
            caches[i][0][slot * span:(slot + 1) * span] = k[off * span:(off + 1) * span]
            caches[i][1][slot * span:(slot + 1) * span] = v[off * span:(off + 1) * span]
    return h


def test_layer_stack_streaming_and_graph_replay():
    """3 layers, prefix + 8 body blocks: eager stack vs the oracle's router +
    block loop, and graph replay bit-identical to eager."""
    from recavsr_b200.runtime.block import FusedBlock, LayerStack, rope_tables
    dim, heads, ffn, H, W = 256, 2, 512, 4, 6
    span = H * W
    actions = ["recent_2", "recent_2_anchor", "none"]
    tables = rope_tables(128, H, W, "cuda")
    ps = [recipes.block_params(dim, heads, ffn, seed=40 + i) for i in range(3)]

    def make():
        return LayerStack([FusedBlock(_weights(p, heads), H, W, tables) for p in ps], actions)

    eager, graphed = make(), make()
    params = [_oracle_params(p, H, W, heads, host(b.cross_k), host(b.cross_v), host(b.modulation))
              for p, b in zip(ps, eager.blocks)]
    routers = [RouterState(a) for a in actions]
    caches = [(np.zeros((r.capacity * span, heads, 128), np.float32),
               np.zeros((r.capacity * span, heads, 128), np.float32)) for r in routers]
    rs = np.random.RandomState(5)
    start = 0
    captured = False
    for blk_i in range(9):
        frames = 6 if blk_i == 0 else 2
        x = bf16_round(rs.standard_normal((frames * span, dim)).astype(np.float32))
        he = dev_bf16(x)
        eager.step(he, frames)
        hg = dev_bf16(x)
        if frames == 2 and not captured:
            graphed.step(hg, frames)          # eager first body step sets kernel attributes
            graphed.capture(2 * span, 2)
            captured = True
        else:
            graphed.step(hg, frames, graphs=(frames == 2 and captured))
        ref = _oracle_stack_step(params, routers, caches, x, start, frames, H, W, heads)
        start += frames
        got = host(he)
        _close(got, ref, 2e-2, 0.15)
        np.testing.assert_array_equal(host(hg), got)
    assert_no_device_error()
