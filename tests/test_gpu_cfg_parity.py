"""Parity at the BASELINE configurations' full sizes, checked against the
oracle on sampled rows / heads / blocks so the CPU side stays bounded.

* cfg3: the NVFP4 linear at M in {3520, 7040} x (K, N) in {(3072, 3072),
  (3072, 14336), (14336, 3072)} through the runtime's GEMM entry (split-K tail,
  grouped raster at 7040), ffn_up's GELU + NVFP4 epilogue at 3520 and 7040,
  and the FP8 per-tensor linear at all nine shapes.
* cfg2: the 75-block streaming run of the routed-attention microbenchmark:
  one layer per scope {0, 1, 2, 4, 8} over an 8-plane ring, append / evict
  every block on the device, sampled blocks and heads against the oracle.
* cfg5-ii: one 120 x 68 (3840 x 2176) local-window launch, 2 sampled heads,
  sampled query rows (edges, corners and the interior).
Tolerances are the spec's: GEMM outputs within 1e-2 of the dequantized fp32
matmul (relative to max |ref|), attention within 2e-2 max-abs / 1e-2 relative.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import fp8 as ofp8
from oracle import nvfp4 as onv
from oracle import rope as orope
from oracle.block import gelu_tanh
from oracle.numerics import bf16_round, e4m3_encode
from tests.golden import recipes
from tests.util import assert_no_device_error, dev_bf16, host, max_rel

pytestmark = pytest.mark.gpu
TOL = 1e-2
ABS, REL = 2e-2, 1e-2
CFG3 = [(3072, 3072), (3072, 14336), (14336, 3072)]


def _sample_rows(m):
    """Three 128-row blocks: the first, one in the middle, the last (ragged)."""
    mid = (m // 2) // 128 * 128
    return np.r_[0:128, mid:mid + 128, m - 128:m]


_WCACHE = {}


def _weight(n, k):
    if (n, k) not in _WCACHE:
        w = recipes.cfg3_weight(n, k, seed=3)
        wc, wsf = onv.quantize(w)
        _WCACHE[(n, k)] = (w, wc, wsf, onv.dequantize(wc, wsf, n, k).astype(np.float64))
    return _WCACHE[(n, k)]


def _bias(n):
    return recipes.bf16_normal(np.random.RandomState(n), (n,), 0.1)


@pytest.mark.parametrize("m", [3520, 7040])
@pytest.mark.parametrize("k,n", CFG3)
def test_cfg3_nvfp4_linear(m, k, n):
    from recavsr_b200.runtime import nvfp4
    a = recipes.cfg3_activation(m, k, seed=2)
    w, wc, wsf, wdeq = _weight(n, k)
    bias = _bias(n)
    ac, asf = nvfp4.quantize(dev_bf16(a))
    bc, bsf = nvfp4.quantize(dev_bf16(w))
    out = host(nvfp4.gemm(ac, bc, asf, bsf, dev_bf16(bias)))
    assert_no_device_error()
    np.testing.assert_array_equal(bc.cpu().numpy(), wc)
    rows = _sample_rows(m)
    rc, rsf = onv.quantize(a[rows])
    ref = onv.nvfp4_mm(rc, rsf, wc, wsf, bias, len(rows), n, k, b_dequantized=wdeq)
    err = max_rel(out[rows], ref)
    assert err < TOL, err


@pytest.mark.parametrize("m", [3520, 7040])
def test_cfg3_ffn_up_gelu_nvfp4_epilogue(m):
    """ffn_up (K 3072 -> N 14336) with the fused GELU(tanh) + NVFP4 epilogue at
    M = 3520 and 7040 (the latter in the grouped tile order): bf16 GELU output
    within 1e-2, and the fused codes / scales equal the oracle's quantization
    of the kernel's own bf16 output on the sampled 128-row blocks."""
    from recavsr_b200 import _lib
    from recavsr_b200.runtime import nvfp4
    k, n = 3072, 14336
    a = recipes.cfg3_activation(m, k, seed=4)
    w, wc, wsf, wdeq = _weight(n, k)
    bias = _bias(n)
    ac, asf = nvfp4.quantize(dev_bf16(a))
    bc, bsf = nvfp4.quantize(dev_bf16(w))
    out = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    qc = torch.empty(m, n // 2, dtype=torch.uint8, device="cuda")
    qs = torch.full((nvfp4.scale_numel(m, n),), 0xAB, dtype=torch.uint8, device="cuda")
    ws = nvfp4.split_workspace(ac.device)
    db = dev_bf16(bias)
    _lib.call("rc_nvfp4_gemm_ws", ac.data_ptr(), asf.data_ptr(), bc.data_ptr(), bsf.data_ptr(),
              db.data_ptr(), m, n, k, 1.0, _lib.EPI_GELU_NVFP4, out.data_ptr(), n, None,
              qc.data_ptr(), qs.data_ptr(), 1.0, ws.data_ptr(), ws.numel(), _lib.stream())
    assert_no_device_error()
    rows = _sample_rows(m)
    rc, rsf = onv.quantize(a[rows])
    y = bf16_round(gelu_tanh(onv.nvfp4_mm(rc, rsf, wc, wsf, bias, len(rows), n, k, b_dequantized=wdeq)))
    yo = host(out)
    assert max_rel(yo[rows], y) < TOL
    codes, scales = qc.cpu().numpy(), qs.cpu().numpy()
    got_sf = onv.unswizzle_scales(scales, m, n)
    for r0 in (0, (m // 2) // 128 * 128, m - 128):
        blk = slice(r0, r0 + 128)
        ec, es = onv.quantize(yo[blk])
        np.testing.assert_array_equal(codes[blk], ec)
        np.testing.assert_array_equal(got_sf[blk], onv.unswizzle_scales(es, 128, n))


def _fp8_rows(x, scale):
    """oracle.fp8.quantize's arithmetic for rows of a matrix whose per-tensor
    scale comes from the whole matrix."""
    z = np.clip((np.asarray(x, np.float32) / np.float32(scale)).astype(np.float32),
                -ofp8.FP8_MAX, ofp8.FP8_MAX)
    return e4m3_encode(z)


@pytest.mark.parametrize("m", [1760, 3520, 7040])
@pytest.mark.parametrize("k,n", CFG3)
def test_cfg3_fp8_linear(m, k, n):
    from recavsr_b200.runtime import fp8
    a = recipes.cfg3_activation(m, k, seed=2)
    w = recipes.cfg3_weight(n, k, seed=3)
    bias = _bias(n)
    aq, sa = fp8.quantize(dev_bf16(a))
    wq, sw = fp8.quantize(dev_bf16(w))
    out = host(fp8.fp8_mm(aq, sa, wq, sw, dev_bf16(bias)))
    assert_no_device_error()
    ref_wq, ref_sw = ofp8.quantize(w)
    ref_sa = np.float32(max(np.float32(np.abs(a).max()), np.float32(1e-12)) / np.float32(ofp8.FP8_MAX))
    assert float(sa) == float(ref_sa) and float(sw) == float(ref_sw)
    np.testing.assert_array_equal(wq.cpu().numpy(), ref_wq)
    rows = _sample_rows(m)
    ref_aq = _fp8_rows(a[rows], ref_sa)
    np.testing.assert_array_equal(aq.cpu().numpy()[rows], ref_aq)
    ref = ofp8.fp8_mm(ref_aq, ref_sa, ref_wq, ref_sw, bias)
    assert max_rel(out[rows], ref) < TOL


def test_cfg2_streaming_75_blocks():
    """cfg2: 24 heads x 128, T = 880 (22 x 40), 2-frame query blocks, 75 blocks.
    Five layers, one per scope {0, 1, 2, 4, 8}: each keeps an 8-plane ring of
    past K / V on the device, attends to its `scope` most recent frames
    (slot = frame % 8) plus the current two, then appends the current frames
    with the device commit (the two oldest planes are evicted by overwrite).
    Q/K/V ~ N(0,1)/sqrt(128). Blocks 0, 1, 4, 37 and 74, heads 0 and 17,
    against the oracle fed with a host copy of the same ring."""
    from recavsr_b200 import _lib
    from recavsr_b200.runtime.block import rope_tables
    from recavsr_b200.runtime.ops import routed_attention
    H, W, heads, ring, blocks = 22, 40, 24, 8, 75
    span = H * W
    scopes = (0, 1, 2, 4, 8)
    check_blocks, check_heads = {0, 1, 4, 37, 74}, [0, 17]
    tb = rope_tables(128, H, W, "cuda")
    tc, ts, _, _ = orope.rolling_tables(128, H, W)
    ring_k = [torch.zeros(1, ring * span, heads, 128, dtype=torch.bfloat16, device="cuda") for _ in scopes]
    ring_v = [torch.zeros_like(r) for r in ring_k]
    host_k = [np.zeros((1, ring * span, 2, 128), np.float32) for _ in scopes]
    host_v = [np.zeros_like(r) for r in host_k]
    g = torch.Generator(device="cuda").manual_seed(1)
    rnd = lambda: (torch.randn(1, 2 * span, heads, 128, generator=g, device="cuda") / 128 ** 0.5).bfloat16()
    i32 = lambda v: torch.tensor(v, dtype=torch.int32, device="cuda")
    out = torch.empty(1, 2 * span, heads, 128, dtype=torch.bfloat16, device="cuda")
    lib = _lib.library()
    checked = 0
    for blk in range(blocks):
        start = 2 * blk
        origin = max(0, start + 2 - 22)
        for li, scope in enumerate(scopes):
            q, k, v = rnd(), rnd(), rnd()
            frames = list(range(max(0, start - scope), start))
            slots = [f % ring for f in frames] + [-1] * (ring - len(frames))
            ppos = [f - origin for f in frames] + [0] * (ring - len(frames))
            qpos = [start - origin, start + 1 - origin]
            routed_attention(q, k, v, ring_k[li], ring_v[li], i32(slots), i32(ppos), i32(qpos),
                             tb["temporal_cos"], tb["temporal_sin"], H, W, H, W, out=out)
            if blk in check_blocks:
                sel = lambda t: host(t[:, :, check_heads])
                ref = oatt.routed_attention(sel(q), sel(k), sel(v), host_k[li], host_v[li], slots, ppos,
                                            qpos, tc, ts, H, W, H, W)
                got = sel(out)
                err = np.abs(got - ref).max()
                assert err <= ABS and max_rel(got, ref) <= REL, (blk, scope, err)
                checked += 1
            # append the current two frames (slots start % 8, start + 1 % 8)
            src = (C.c_int * 2)(0, 1)                              # host arrays (read at launch)
            dst = (C.c_int * 2)(start % ring, (start + 1) % ring)
            _lib.check(lib.rc_kv_commit(k.data_ptr(), v.data_ptr(), heads * 256, ring_k[li].data_ptr(),
                                        ring_v[li].data_ptr(), heads * 256, heads * 256, span, 2,
                                        src, dst, _lib.stream()), "kv_commit")
            kh, vh = host(k[:, :, check_heads]), host(v[:, :, check_heads])
            for f in range(2):
                s = (start + f) % ring
                host_k[li][:, s * span:(s + 1) * span] = kh[:, f * span:(f + 1) * span]
                host_v[li][:, s * span:(s + 1) * span] = vh[:, f * span:(f + 1) * span]
    assert_no_device_error()
    assert checked == len(check_blocks) * len(scopes)
    # the device ring holds the same planes as the host copy after 75 blocks
    for li in range(len(scopes)):
        np.testing.assert_array_equal(host(ring_k[li][:, :, check_heads]), host_k[li])
        np.testing.assert_array_equal(host(ring_v[li][:, :, check_heads]), host_v[li])


def test_cfg5_4k_local_window_sampled():
    """cfg5-ii geometry: 3840x2176 -> 68 x 120 tokens (T = 8160), 2-frame query
    block, 22 x 40 windows, 4 routed planes; all 24 heads on the device, heads
    3 and 20 checked on 320 query rows (both frames' corners, edges, interior)."""
    from recavsr_b200.runtime.block import rope_tables
    from recavsr_b200.runtime.ops import routed_attention
    H, W, heads, cap = 68, 120, 24, 4
    span = H * W
    g = torch.Generator(device="cuda").manual_seed(11)
    r = lambda n: (torch.randn(1, n * span, heads, 128, generator=g, device="cuda") / 128 ** 0.5 * 3).bfloat16()
    q, ck, cv, pk, pv = r(2), r(2), r(2), r(cap), r(cap)
    tb = rope_tables(128, H, W, "cuda")
    slots, ppos, qpos = [2, 0, 3, 1], [4, 5, 6, 7], [8, 9]
    i32 = lambda v: torch.tensor(v, dtype=torch.int32, device="cuda")
    out = routed_attention(q, ck, cv, pk, pv, i32(slots), i32(ppos), i32(qpos), tb["temporal_cos"],
                           tb["temporal_sin"], H, W, 22, 40)
    assert_no_device_error()
    hs = [3, 20]
    rs = np.random.RandomState(0)
    ys = np.r_[0, 1, 10, 11, 12, 33, 34, 56, 57, 66, 67, rs.randint(0, H, 21)]
    xs = np.r_[0, 1, 19, 20, 21, 59, 60, 99, 100, 118, 119, rs.randint(0, W, 21)]
    grid = (ys[:, None] * W + xs[None, :]).reshape(-1)[:160]
    rows = np.r_[grid, grid + span]
    sel = lambda t: host(t[:, :, hs])
    tc, ts, _, _ = orope.rolling_tables(128, H, W)
    ref = oatt.routed_attention(sel(q), sel(ck), sel(cv), sel(pk), sel(pv), slots, ppos, qpos, tc, ts,
                                H, W, 22, 40, query_rows=rows)
    got = host(out[:, :, hs])[:, rows]
    err = np.abs(got - ref).max()
    assert err <= ABS and max_rel(got, ref) <= REL, err
