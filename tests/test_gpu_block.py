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


def _golden_block(golden, tag):
    from recavsr_b200.runtime.block import FusedBlock, rope_tables
    m = [int(v) for v in golden[f"{tag}_meta"]]
    dim, heads, ffn, H, W, cap = m[:6]
    enc, pseed, iseed = (m[6:9] if len(m) > 6 else (16, 11, 12))
    slots, ppos = (m[9:9 + cap], m[9 + cap:]) if len(m) > 6 else ([1, -1, 2], [4, 0, 5])
    p = recipes.block_params(dim, heads, ffn, enc_len=enc, seed=pseed)
    blk = FusedBlock(_weights(p, heads), H, W, rope_tables(dim // heads, H, W, "cuda"))
    hidden, pk, pv = recipes.block_inputs(2 * H * W, cap * H * W, dim, seed=iseed)
    d = dim // heads
    h, k, v = blk(dev_bf16(hidden), dev_bf16(pk).reshape(1, -1, heads, d),
                  dev_bf16(pv).reshape(1, -1, heads, d),
                  torch.tensor(slots, dtype=torch.int32, device="cuda"),
                  torch.tensor(ppos, dtype=torch.int32, device="cuda"),
                  torch.tensor([6, 7], dtype=torch.int32, device="cuda"))
    assert_no_device_error()
    np.testing.assert_array_equal(host(blk.modulation), golden[f"{tag}_modulation"].reshape(6, dim))
    ck = bf16_from_bits(golden[f"{tag}_cross_k"]).reshape(-1, heads, d)
    assert np.abs(host(blk.cross_k) - ck).max() <= 2 ** -6 * np.abs(ck).max()
    ref = {n: bf16_from_bits(golden[f"{tag}_{n}"]) for n in ("hidden", "k", "v")}
    return host(h), host(k), host(v), ref


# The block output passes through six NVFP4 GEMMs whose E2M1 codes flip on
# 1-ulp differences of their bf16 inputs (SDPA vs online softmax, LayerNorm
# reduction order). Two faithful implementations therefore differ at the
# block level: the CPU oracle itself is 4.1% (relative L2) from the
# reference's own output at dim 768 while its K/V are bit-exact. The block
# checks bound that spread; kernel parity is proven stage by stage below.
BLOCK_REL_L2 = 0.06
BLOCK_MAX_FRAC = 0.15


@pytest.mark.parametrize("tag", ["block", "block768"])
def test_fused_block_matches_reference_block(golden, tag):
    """Same inputs as the reference PreparedBlock fixtures (NVFP4 linears)."""
    h, k, v, ref = _golden_block(golden, tag)
    _close(k.reshape(-1), ref["k"].reshape(-1), 5e-3, 2 ** -5)
    _close(v.reshape(-1), ref["v"].reshape(-1), 5e-3, 2 ** -5)
    _close(h.reshape(-1), ref["hidden"].reshape(-1), BLOCK_REL_L2, BLOCK_MAX_FRAC)


def test_fused_block_stagewise_vs_oracle():
    """Every kernel of the block, fed the block's own intermediates, against the
    oracle step it replaces (dim 768, 6 heads, FFN 2048, 8x12 grid, 2 planes)."""
    import ctypes as C
    from recavsr_b200 import _lib
    from recavsr_b200.runtime.block import FusedBlock, Workspace, rope_tables
    from oracle import nvfp4 as onv
    from oracle.attention import plain_attention, routed_attention
    dim, heads, ffn, H, W = 768, 6, 2048, 8, 12
    span, n = H * W, 2 * H * W
    p = recipes.block_params(dim, heads, ffn, enc_len=64, seed=21)
    blk = FusedBlock(_weights(p, heads), H, W, rope_tables(128, H, W, "cuda"))
    hidden, pk, pv = recipes.block_inputs(n, 2 * span, dim, seed=22)
    ws = Workspace(blk, n)
    lib, st = _lib.library(), _lib.stream()
    mod = host(blk.modulation)
    lin = {nm: oblock.QuantLinear(p[nm + "_w"], p[nm + "_b"]) for nm in ("o", "cq", "co", "up", "down")}
    tc, ts, sc, ss = orope.rolling_tables(128, H, W)
    h = dev_bf16(hidden[0]).contiguous()
    shift, scale, gate, cshift, cscale, cgate = (blk.modulation[i] for i in range(6))
    sync = torch.cuda.synchronize

    def ln_codes(x_host, w=None, b=None, sh=None, scl=None):
        y = oblock.layer_norm(x_host, w, b)
        if scl is not None:
            y = y * (1 + scl) + sh
        return onv.quantize(bf16_round(y))

    # LN1 + AdaLN + NVFP4 (bf16 LN outputs may differ by 1 ulp -> compare dequantized)
    _lib.check(lib.rc_ln_modulate_quant(h.data_ptr(), dim, n, dim, None, None, shift.data_ptr(),
                                        scale.data_ptr(), 1e-6, None, 0, ws.a_codes.data_ptr(),
                                        ws.a_scales.data_ptr(), 1.0, st), "ln1")
    sync()
    rc_, rs_ = ln_codes(hidden[0], sh=mod[0], scl=mod[1])
    a_dev = onv.dequantize(ws.a_codes.cpu().numpy(), ws.a_scales.cpu().numpy(), n, dim)
    a_ref = onv.dequantize(rc_, rs_, n, dim)
    assert np.mean(a_dev != a_ref) < 0.01
    # QKV GEMM on the kernel's own codes: 1e-2 rel of the dequantized matmul
    blk._gemm(lib, ws, ws.a_codes, ws.a_scales, blk.qkv, n, _lib.EPI_BIAS, ws.qkv, st)
    sync()
    wq = np.concatenate([p["q_w"], p["k_w"], p["v_w"]], 0)
    bq = np.concatenate([p["q_b"], p["k_b"], p["v_b"]])
    wc, wsf = onv.quantize(wq)
    qkv_ref = onv.nvfp4_mm(ws.a_codes.cpu().numpy(), ws.a_scales.cpu().numpy(), wc, wsf, bq, n, 3 * dim, dim)
    qkv = host(ws.qkv)
    assert np.abs(qkv - qkv_ref).max() <= 1e-2 * np.abs(qkv_ref).max()
    # RMSNorm + spatial RoPE
    q_in, k_in = ws.qkv[:, :dim], ws.qkv[:, dim:2 * dim]
    _lib.check(lib.rc_rmsnorm_rope(2, (C.c_void_p * 2)(q_in.data_ptr(), k_in.data_ptr()),
                                   (C.c_longlong * 2)(3 * dim, 3 * dim),
                                   (C.c_void_p * 2)(blk.norm_q.data_ptr(), blk.norm_k.data_ptr()),
                                   (C.c_void_p * 2)(ws.q_rot.data_ptr(), ws.k_rot.data_ptr()),
                                   (C.c_longlong * 2)(dim, dim), n, dim, 128, span,
                                   blk.tables["spatial_cos"].data_ptr(),
                                   blk.tables["spatial_sin"].data_ptr(), 1e-6, st), "rms")
    sync()
    cs = np.tile(sc, (2, 1))[:, None, :]
    sn = np.tile(ss, (2, 1))[:, None, :]
    for got, x, w in ((ws.q_rot, qkv[:, :dim], p["norm_q"]), (ws.k_rot, qkv[:, dim:2 * dim], p["norm_k"])):
        ref = orope.apply_rotary(oblock.rms_norm(x, w).reshape(n, heads, 128), cs, sn).reshape(n, dim)
        assert np.abs(host(got) - ref).max() <= 2 ** -7 * np.abs(ref).max()
    # routed attention
    slots = torch.tensor([1, 0], dtype=torch.int32, device="cuda")
    pp = torch.tensor([3, 4], dtype=torch.int32, device="cuda")
    qp = torch.tensor([5, 6], dtype=torch.int32, device="cuda")
    dpk, dpv = dev_bf16(pk).reshape(1, -1, heads, 128), dev_bf16(pv).reshape(1, -1, heads, 128)
    blk._attention(lib, ws, dpk, dpv, slots, pp, qp, n, st)
    sync()
    att = host(ws.attn)
    ra = routed_attention(host(ws.q_rot).reshape(1, n, heads, 128), host(ws.k_rot).reshape(1, n, heads, 128),
                          qkv[:, 2 * dim:].reshape(1, n, heads, 128), pk.reshape(1, -1, heads, 128),
                          pv.reshape(1, -1, heads, 128), [1, 0], [3, 4], [5, 6], tc, ts, H, W, 22, 40)
    assert np.abs(att - ra[0].reshape(n, dim)).max() <= 2e-2
    # o-proj, gated residual (exact on identical inputs)
    _lib.check(lib.rc_nvfp4_quantize(ws.attn.data_ptr(), n, dim, dim, 1.0, ws.a_codes.data_ptr(),
                                     ws.a_scales.data_ptr(), st), "q")
    blk._gemm(lib, ws, ws.a_codes, ws.a_scales, blk.o, n, _lib.EPI_GATED_RESIDUAL, h, st, gate)
    sync()
    h1 = bf16_round(hidden[0] + lin["o"](att) * mod[2])
    assert np.abs(host(h) - h1).max() <= 1e-2 * np.abs(h1).max()
    h1 = host(h)
    # LN2 -> cross q -> RMSNorm -> cross attention -> cross-o residual
    _lib.check(lib.rc_ln_modulate_quant(h.data_ptr(), dim, n, dim, blk.norm2_w.data_ptr(),
                                        blk.norm2_b.data_ptr(), None, None, 1e-6, None, 0,
                                        ws.a_codes.data_ptr(), ws.a_scales.data_ptr(), 1.0, st), "ln2")
    blk._gemm(lib, ws, ws.a_codes, ws.a_scales, blk.cq, n, _lib.EPI_BIAS, ws.cq, st)
    sync()
    cq_ref = onv.nvfp4_mm(ws.a_codes.cpu().numpy(), ws.a_scales.cpu().numpy(), *onv.quantize(p["cq_w"]),
                          p["cq_b"], n, dim, dim)
    assert np.abs(host(ws.cq) - cq_ref).max() <= 1e-2 * np.abs(cq_ref).max()
    _lib.check(lib.rc_rmsnorm_rope(1, (C.c_void_p * 1)(ws.cq.data_ptr()), (C.c_longlong * 1)(dim),
                                   (C.c_void_p * 1)(blk.cnorm_q.data_ptr()),
                                   (C.c_void_p * 1)(ws.q_rot.data_ptr()), (C.c_longlong * 1)(dim),
                                   n, dim, 128, 1, None, None, 1e-6, st), "crms")
    strides = (C.c_longlong * 9)(0, dim, 128, 0, dim, 128, 0, dim, 128)
    _lib.check(lib.rc_cross_attention(ws.q_rot.data_ptr(), blk.cross_k.data_ptr(),
                                      blk.cross_v.data_ptr(), strides, 1, n, blk.cross_k.shape[0],
                                      heads, 128, ws.attn.data_ptr(), dim, None, None, st), "cross")
    sync()
    ca = host(ws.attn)
    rca = plain_attention(host(ws.q_rot).reshape(n, heads, 128), host(blk.cross_k), host(blk.cross_v))
    assert np.abs(ca - rca.reshape(n, dim)).max() <= 2e-2
    _lib.check(lib.rc_nvfp4_quantize(ws.attn.data_ptr(), n, dim, dim, 1.0, ws.a_codes.data_ptr(),
                                     ws.a_scales.data_ptr(), st), "q2")
    blk._gemm(lib, ws, ws.a_codes, ws.a_scales, blk.co, n, _lib.EPI_RESIDUAL, h, st)
    sync()
    h2 = bf16_round(h1 + lin["co"](ca))
    assert np.abs(host(h) - h2).max() <= 1e-2 * np.abs(h2).max()
    h2 = host(h)
    # LN3 -> ffn_up (GELU + NVFP4 epilogue) -> ffn_down gated residual
    _lib.check(lib.rc_ln_modulate_quant(h.data_ptr(), dim, n, dim, None, None, cshift.data_ptr(),
                                        cscale.data_ptr(), 1e-6, None, 0, ws.a_codes.data_ptr(),
                                        ws.a_scales.data_ptr(), 1.0, st), "ln3")
    _lib.check(lib.rc_nvfp4_gemm(ws.a_codes.data_ptr(), ws.a_scales.data_ptr(), blk.up.codes.data_ptr(),
                                 blk.up.scales.data_ptr(), blk.up.bias.data_ptr(), n, ffn, dim, 1.0,
                                 _lib.EPI_GELU_NVFP4, None, 0, None, ws.f_codes.data_ptr(),
                                 ws.f_scales.data_ptr(), 1.0, st), "up")
    sync()
    up_ref = bf16_round(oblock.gelu_tanh(onv.nvfp4_mm(ws.a_codes.cpu().numpy(), ws.a_scales.cpu().numpy(),
                                                      *onv.quantize(p["up_w"]), p["up_b"], n, ffn, dim)))
    up_dev = onv.dequantize(ws.f_codes.cpu().numpy(), ws.f_scales.cpu().numpy(), n, ffn)
    uc, us = onv.quantize(up_ref)
    assert np.mean(up_dev != onv.dequantize(uc, us, n, ffn)) < 0.01
    blk._gemm(lib, ws, ws.f_codes, ws.f_scales, blk.down, n, _lib.EPI_GATED_RESIDUAL, h, st, cgate)
    sync()
    y = onv.nvfp4_mm(ws.f_codes.cpu().numpy(), ws.f_scales.cpu().numpy(), *onv.quantize(p["down_w"]),
                     p["down_b"], n, dim, ffn)
    h3 = bf16_round(h2 + y * mod[5])
    assert np.abs(host(h) - h3).max() <= 1e-2 * np.abs(h3).max()
    assert_no_device_error()


def _oracle_stack_step(params_list, routers, caches, hidden, start, frames, H, W, heads):
    origin, qpos = rope_origin(start, frames)
    span = H * W
    d = hidden.shape[1] // heads
    h = hidden
    routes = []
    for i, (prm, rt) in enumerate(zip(params_list, routers)):
        slots, ppos = rt.history(origin)
        routes.append((list(slots), list(ppos)))
        cap = rt.capacity
        pk = caches[i][0] if cap else np.zeros((0, heads, d), np.float32)
        pv = caches[i][1] if cap else np.zeros((0, heads, d), np.float32)
        h, k, v = oblock.block_forward(prm, h, pk, pv, list(slots), list(ppos), list(qpos), H, W,
                                       (22, 40), heads=heads)
        for off, slot in rt.commit(frames, start):
            caches[i][0][slot * span:(slot + 1) * span] = k[off * span:(off + 1) * span]
            caches[i][1][slot * span:(slot + 1) * span] = v[off * span:(off + 1) * span]
    return h, routes


def test_layer_stack_streaming_and_graph_replay():
    """3 layers, prefix + 8 body blocks. Per block the oracle starts from the
    stack's own cache contents (teacher forcing, so NVFP4 code flips do not
    compound across blocks); routing tables must equal the oracle router's
    exactly, graph replay must be bit-identical to eager launches, and so must
    the host-to-host streaming path (step_host, copies overlapping the
    neighbouring blocks, no host sync until the end). The K / V planes each
    block commits to the cache must match the oracle's k / v of that layer
    (K is a column range of its own buffer, V of the fused QKV output, so the
    two source row strides differ)."""
    from recavsr_b200.runtime.block import FusedBlock, LayerStack, rope_tables
    dim, heads, ffn, H, W = 256, 2, 512, 4, 6
    span = H * W
    actions = ["recent_2", "recent_2_anchor", "none"]
    tables = rope_tables(128, H, W, "cuda")
    ps = [recipes.block_params(dim, heads, ffn, seed=40 + i) for i in range(3)]

    def make():
        return LayerStack([FusedBlock(_weights(p, heads), H, W, tables) for p in ps], actions)

    eager, graphed, streamed = make(), make(), make()
    pending = []   # (pinned input, pinned output, eager result) of streamed body blocks
    params = [_oracle_params(p, H, W, heads, host(b.cross_k), host(b.cross_v), host(b.modulation))
              for p, b in zip(ps, eager.blocks)]
    routers = [RouterState(a) for a in actions]
    rs = np.random.RandomState(5)
    start = 0
    captured = False
    for blk_i in range(9):
        frames = 6 if blk_i == 0 else 2
        x = bf16_round(rs.standard_normal((frames * span, dim)).astype(np.float32))
        caches = [(host(eager.cache_k[i])[0].copy(), host(eager.cache_v[i])[0].copy())
                  for i in range(3)]
        he = dev_bf16(x)
        eager.step(he, frames)
        hg = dev_bf16(x)
        stream_now = frames == 2 and captured
        if frames == 2 and not captured:
            graphed.step(hg, frames)          # eager first body step sets kernel attributes
            graphed.capture(2 * span, 2)
            hs = dev_bf16(x)
            streamed.step(hs, frames)
            streamed.capture(2 * span, 2)
            captured = True
        else:
            graphed.step(hg, frames, graphs=(frames == 2 and captured))
            if not stream_now:
                streamed.step(dev_bf16(x), frames)
        if stream_now:
            hin = torch.tensor(x).bfloat16().pin_memory()
            hout = torch.empty_like(hin).pin_memory()
            streamed.step_host(hin, hout, frames)
        ref, routes = _oracle_stack_step(params, routers, caches, x, start, frames, H, W, heads)
        start += frames
        for i in range(3):
            if eager.caches[i].capacity:
                for t, dev_cache in enumerate((eager.cache_k, eager.cache_v)):
                    _close(host(dev_cache[i])[0].reshape(-1), caches[i][t].reshape(-1),
                           BLOCK_REL_L2, BLOCK_MAX_FRAC)
        for i, (slots, ppos) in enumerate(routes):
            o = i * eager._row
            cap = eager.caches[i].capacity
            assert eager.route_host[o:o + cap].tolist() == (slots or [-1] * cap)
            if slots:
                assert eager.route_host[o + 8:o + 8 + cap].tolist() == ppos
        got = host(he)
        _close(got, ref, BLOCK_REL_L2, BLOCK_MAX_FRAC)
        np.testing.assert_array_equal(host(hg), got)
        if stream_now:
            pending.append((hin, hout, got))
    streamed.sync_host()
    torch.cuda.synchronize()
    assert len(pending) == 7
    for hin, hout, got in pending:
        np.testing.assert_array_equal(hout.float().numpy(), got)
    assert_no_device_error()


def test_layer_stack_step_host_reuses_one_pinned_buffer():
    """LayerStack.step_host with one pinned input buffer refilled with new data
    every block once the previous block's HostStep.input_consumed completed,
    and each result read after its output_ready: bit-identical to step()."""
    from recavsr_b200.runtime.block import FusedBlock, LayerStack, rope_tables
    dim, heads, ffn, H, W = 256, 2, 512, 4, 6
    span = H * W
    actions = ["recent_2", "recent_2_anchor", "none"]
    tables = rope_tables(128, H, W, "cuda")
    ps = [recipes.block_params(dim, heads, ffn, seed=40 + i) for i in range(3)]

    def make():
        return LayerStack([FusedBlock(_weights(p, heads), H, W, tables) for p in ps], actions)

    ref, streamed = make(), make()
    rs = np.random.RandomState(8)
    xs = [bf16_round(rs.standard_normal(((6 if i == 0 else 2) * span, dim)).astype(np.float32))
          for i in range(10)]
    want = []
    for i, x in enumerate(xs):
        h = dev_bf16(x)
        ref.step(h, 6 if i == 0 else 2)
        want.append(host(h))
    streamed.step(dev_bf16(xs[0]), 6)
    h = dev_bf16(xs[1])
    streamed.step(h, 2)                       # eager first body step, then capture
    streamed.capture(2 * span, 2)
    np.testing.assert_array_equal(host(h), want[1])
    hin = torch.empty((2 * span, dim), dtype=torch.bfloat16).pin_memory()
    outs, handles = [], []
    for x in xs[2:]:
        if handles:
            handles[-1].input_consumed.synchronize()
        hin.copy_(torch.from_numpy(x))
        outs.append(torch.empty_like(hin).pin_memory())
        handles.append(streamed.step_host(hin, outs[-1], 2))
    for i, (o, hd) in enumerate(zip(outs, handles)):
        hd.output_ready.synchronize()
        np.testing.assert_array_equal(o.float().numpy(), want[i + 2], err_msg=f"block {i + 2}")
    streamed.sync_host()
    assert_no_device_error()
