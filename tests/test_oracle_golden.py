"""Pins the CPU oracle to outputs recorded from the reference itself
(tests/golden/make_golden.py). CPU only."""
import numpy as np
import pytest

from oracle import attention, block, cache, fp8, nvfp4, rope
from oracle.numerics import bf16_from_bits, bf16_round
from tests.golden import recipes


@pytest.mark.parametrize("case", ["special", "ragged", "weights", "cfg3_small"])
def test_nvfp4_quantize_bit_exact(golden, case):
    x = bf16_from_bits(golden[f"quant_{case}_x"])
    codes, scales = nvfp4.quantize(x)
    np.testing.assert_array_equal(codes, golden[f"quant_{case}_codes"])
    np.testing.assert_array_equal(scales, golden[f"quant_{case}_scales"])


def test_nvfp4_recipes_regenerate_inputs(golden):
    x = recipes.cfg3_activation(300, 512, seed=2)
    np.testing.assert_array_equal(bf16_from_bits(golden["quant_cfg3_small_x"]), x)


def test_nvfp4_dequant_roundtrip():
    x = recipes.cfg3_activation(64, 256, seed=4)
    c, s = nvfp4.quantize(x)
    d = nvfp4.dequantize(c, s, 64, 256)
    c2, s2 = nvfp4.quantize(d)   # dequantized values re-quantize to themselves
    np.testing.assert_array_equal(nvfp4.dequantize(c2, s2, 64, 256), d)  # (-0 codes aside)


@pytest.mark.parametrize("case", ["act", "weight"])
def test_fp8_quantize_bit_exact(golden, case):
    q, scale = fp8.quantize(bf16_from_bits(golden[f"fp8_{case}_x"]))
    assert np.float32(scale) == golden[f"fp8_{case}_scale"]
    np.testing.assert_array_equal(q, golden[f"fp8_{case}_q"])


def test_router_matches_reference(router_golden):
    for action, rec in router_golden.items():
        st = cache.RouterState(action, initial=5, stride=6, anchors=2)
        assert st.capacity == rec["capacity"]
        content = {}
        for step in rec["steps"]:
            origin, qpos = cache.rope_origin(step["start"], step["frames"])
            assert origin == step["origin"] and list(qpos) == step["qpos"]
            slots, ppos = st.history(origin)
            assert list(slots) == step["slots"] and list(ppos) == step["ppos"], (action, step)
            for off, slot in st.commit(step["frames"], step["start"]):
                content[slot] = step["start"] + off
            if step["slot_frames"]:
                for slot, fid in content.items():
                    assert step["slot_frames"][slot] == fid
            assert sorted(st.frame_to_slot) == step["frame_ids"]


def test_rope_tables(golden):
    tc, ts, sc, ss = rope.rolling_tables(128, 11, 20)
    np.testing.assert_array_equal(tc, golden["rope_tcos"])
    np.testing.assert_array_equal(ts, golden["rope_tsin"])
    np.testing.assert_array_equal(sc, golden["rope_scos"])
    np.testing.assert_array_equal(ss, golden["rope_ssin"])
    for h, w in ((22, 40), (34, 60)):
        t = rope.rolling_tables(128, h, w)
        sums = [t[2].astype(np.float64).sum(), t[3].astype(np.float64).sum(),
                t[0].astype(np.float64).sum(), t[1].astype(np.float64).sum()]
        np.testing.assert_allclose(sums, golden[f"rope_sum_{h}x{w}"], rtol=0, atol=1e-9)


def test_rope_apply(golden):
    x = bf16_from_bits(golden["rope_x"]).reshape(1, 440, 3, 128)
    _, _, sc, ss = rope.rolling_tables(128, 11, 20)
    tc, ts = golden["rope_tcos"], golden["rope_tsin"]
    sp = rope.apply_rotary(x.reshape(1, 2, 220, 3, 128), sc[None, None, :, None, :],
                           ss[None, None, :, None, :])
    np.testing.assert_array_equal(sp.reshape(-1), bf16_from_bits(golden["rope_spatial"]).reshape(-1))
    np.testing.assert_array_equal(sp.reshape(-1), bf16_from_bits(golden["rope_rotary"]).reshape(-1))
    tp = rope.apply_temporal(x[0], [4, 17], tc, ts, 220)
    np.testing.assert_array_equal(tp.reshape(-1), bf16_from_bits(golden["rope_temporal"]).reshape(-1))


def test_attention_dense_matches_sdpa(golden):
    g = {n: bf16_from_bits(golden[f"attn_dense_{n}"]) for n in ("q", "ck", "cv", "pk", "pv")}
    tc, ts, _, _ = rope.rolling_tables(128, 4, 6)
    out = attention.routed_attention(g["q"], g["ck"], g["cv"], g["pk"], g["pv"], [2, -1, 0],
                                     [5, 0, 3], [6, 7], tc, ts, 4, 6, 22, 40)
    ref32 = golden["attn_dense_f32"]
    assert np.abs(out - ref32).max() < 2e-2
    assert np.abs(out - ref32).max() <= 2 * np.abs(bf16_round(ref32) - ref32).max() + 1e-6
    assert np.abs(out - golden["attn_dense_bf16"]).max() < 2e-2


@pytest.mark.parametrize("tag", ["win_a", "win_b"])
def test_attention_window_matches_triton(golden, tag):
    if f"attn_{tag}_out" not in golden:
        pytest.skip("fixture generated without TRITON_INTERPRET=1")
    H, W, wh, ww, d, cap = (int(v) for v in golden[f"attn_{tag}_meta"][:6])
    rest = [int(v) for v in golden[f"attn_{tag}_meta"][6:]]
    slots, ppos = rest[:cap], rest[cap:]
    a = {n: golden[f"attn_{tag}_{n}"].astype(np.float32) for n in ("q", "ck", "cv", "pk", "pv")}
    tc, ts, _, _ = rope.rolling_tables(d, H, W)
    out = attention.routed_attention(a["q"], a["ck"], a["cv"], a["pk"], a["pv"], slots, ppos,
                                     [7, 8], tc, ts, H, W, wh, ww, dtype="fp16")
    # fp16 kernel rounds probabilities before PV; the oracle does not.
    assert np.abs(out - golden[f"attn_{tag}_out"]).max() < 5e-3


def _block_setup(golden, tag="block"):
    m = [int(v) for v in golden[f"{tag}_meta"]]
    dim, heads, ffn, H, W, cap = m[:6]
    p = recipes.block_params(dim, heads, ffn, enc_len=m[6], seed=m[7])
    tc, ts, sc, ss = rope.rolling_tables(dim // heads, H, W)
    lin = {n: block.QuantLinear(p[n + "_w"], p[n + "_b"])
           for n in ("q", "k", "v", "o", "cq", "co", "up", "down")}
    params = {"_linears": lin, "modulation": golden[f"{tag}_modulation"].reshape(6, dim),
              "norm_q": p["norm_q"], "norm_k": p["norm_k"], "cnorm_q": p["cnorm_q"],
              "norm2_w": p["norm2_w"], "norm2_b": p["norm2_b"],
              "cross_k": bf16_from_bits(golden[f"{tag}_cross_k"]).reshape(-1, heads, dim // heads),
              "cross_v": bf16_from_bits(golden[f"{tag}_cross_v"]).reshape(-1, heads, dim // heads),
              "temporal_cos": tc, "temporal_sin": ts, "spatial_cos": sc, "spatial_sin": ss}
    hidden, pk, pv = recipes.block_inputs(2 * H * W, cap * H * W, dim, seed=m[8])
    slots, ppos = m[9:9 + cap], m[9 + cap:]
    return dim, heads, H, W, params, hidden, pk, pv, slots, ppos


@pytest.mark.parametrize("tag", ["block", "block768"])
def test_block_forward_matches_reference(golden, tag):
    dim, heads, H, W, params, hidden, pk, pv, slots, ppos = _block_setup(golden, tag)
    d = dim // heads
    h, k, v = block.block_forward(params, hidden[0], pk[0].reshape(-1, heads, d),
                                  pv[0].reshape(-1, heads, d), slots, ppos, [6, 7],
                                  H, W, (22, 40), heads=heads)
    ref_h = bf16_from_bits(golden[f"{tag}_hidden"]).reshape(h.shape)
    ref_k = bf16_from_bits(golden[f"{tag}_k"]).reshape(k.shape)
    ref_v = bf16_from_bits(golden[f"{tag}_v"]).reshape(v.shape)
    # K/V come straight from the first quantized GEMMs + RMSNorm/RoPE: near bit-exact.
    assert np.abs(k - ref_k).max() <= 2 ** -6 * np.abs(ref_k).max()
    assert np.abs(v - ref_v).max() <= 2 ** -7 * np.abs(ref_v).max()
    # The block output passes through 5 more quantized GEMMs whose E2M1 codes can
    # flip on 1-ulp bf16 differences (fp64 exact softmax here vs the reference's
    # fp32 SDPA); compare in relative L2 and max-abs: measured 0.5% at dim 256,
    # 4.1% at dim 768.
    rel = np.linalg.norm(h - ref_h) / np.linalg.norm(ref_h)
    assert rel < 0.06, rel
    assert np.abs(h - ref_h).max() < 0.15 * np.abs(ref_h).max()


def test_refined_quotient_e2m1_codes_are_exact():
    """The kernels code NVFP4 (global scale 1) as e2m1_rn(q1) with q0 = x*r,
    q1 = fma(fma(-q0, s, x), r, q0) and r the hardware's approximate 1/s; the
    e2m1 conversion rounds to nearest even. For every bf16 x and every E4M3
    scale s with |x| <= 16 s (a block's scale is e4m3(amax / 6), so its
    elements satisfy |x| / s <= 6.4), and r up to 64 ulps away from 1/s,
    this equals the reference ladder applied to fl32(x / s) (exhaustive; the
    hardware conversion itself is checked exhaustively on the GPU by
    test_gpu_quant)."""
    from oracle.numerics import bf16_from_bits, e4m3_decode
    x = bf16_from_bits(np.arange(65536, dtype=np.uint32).astype(np.uint16))
    x = x[np.isfinite(x)]
    scales = e4m3_decode(np.arange(1, 127, dtype=np.uint8)).astype(np.float32)
    for s in scales:
        xs = x[np.abs(x) <= np.float32(16) * s]
        ref = nvfp4.e2m1_codes((xs / s).astype(np.float32))
        r0 = np.float32(1.0) / s
        ulp = np.spacing(r0)
        for r in r0 + ulp * np.array([-64, -1, 0, 1, 64], np.float32):   # MUFU rcp is within 1 ulp
            q0 = (xs * r).astype(np.float32)
            rem = (xs.astype(np.float64) - q0.astype(np.float64) * np.float64(s)).astype(np.float32)  # exact
            q1 = (rem.astype(np.float64) * np.float64(r) + q0.astype(np.float64)).astype(np.float32)
            # e2m1 round-to-nearest-even (the ladder is RNE), sign from the sign bit
            code = nvfp4.e2m1_codes(np.abs(q1)) | (np.signbit(q1).astype(np.uint8) * 8)
            np.testing.assert_array_equal(code, ref)


def test_div6_is_exact_for_bf16():
    """The kernels compute the NVFP4 block scale amax / 6 without dividing:
    q = amax * fl(1/6), refined once by the exact residual. For every finite
    non-negative bf16 amax this equals IEEE fp32 division (exhaustive, with the
    final fma rounded exactly)."""
    from fractions import Fraction
    from oracle.numerics import bf16_from_bits
    a = bf16_from_bits(np.arange(0, 0x7F80, dtype=np.uint32).astype(np.uint16)).astype(np.float32)
    ref = (a / np.float32(6)).astype(np.float32)
    r6 = np.float32(1) / np.float32(6)
    q = (a * r6).astype(np.float32)
    rem = (a.astype(np.float64) - q.astype(np.float64) * 6.0).astype(np.float32)   # exact
    approx = (rem.astype(np.float64) * np.float64(r6) + q.astype(np.float64)).astype(np.float32)
    # Double rounding through float64 can only matter next to an fp32 midpoint:
    # re-round those few candidates exactly.
    fr6 = Fraction(float(r6))
    for i in np.nonzero(approx != ref)[0].tolist() + list(range(0, len(a), 997)):
        exact = Fraction(float(rem[i])) * fr6 + Fraction(float(q[i]))
        cands = [np.nextafter(approx[i], np.float32(-np.inf)), approx[i], np.nextafter(approx[i], np.float32(np.inf))]
        dist = [abs(Fraction(float(c)) - exact) for c in cands]
        best = min(range(3), key=lambda k: (dist[k], int(np.float32(cands[k]).view(np.uint32)) & 1))
        approx[i] = cands[best]
    np.testing.assert_array_equal(approx, ref)
