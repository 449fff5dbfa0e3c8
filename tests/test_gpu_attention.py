"""Routed attention on the GPU against the oracle (which is pinned to the
reference's sdpa_attention and Triton kernel): max-abs <= 2e-2 and
normwise relative <= 1e-2 in bf16, the tolerances the spec states."""
import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import rope as orope
from oracle.numerics import bf16_from_bits, bf16_round
from tests.golden import recipes
from tests.util import assert_no_device_error, dev_bf16, host, max_rel

pytestmark = pytest.mark.gpu
ABS, REL = 2e-2, 1e-2


def _run(H, W, wh, ww, cap, slots, ppos, qpos, heads=2, seed=0, check_heads=None, std=1.0,
         fused=False, abs_scale=False):
    from recavsr_b200.kernels.local_attention import routed_attention
    span = H * W
    frames = len(qpos)
    rs = np.random.RandomState(seed)
    q, ck, cv = (recipes.bf16_normal(rs, (1, frames * span, heads, 128), std) for _ in range(3))
    pk, pv = (recipes.bf16_normal(rs, (1, cap * span, heads, 128), std) for _ in range(2))
    tc, ts, _, _ = orope.rolling_tables(128, H, W)
    dev = lambda a: dev_bf16(a)
    if fused:
        qkv = torch.cat([dev(q), dev(ck), dev(cv)], dim=2)   # [1, tok, 3*heads, d]
        dq, dck, dcv = qkv[:, :, :heads], qkv[:, :, heads:2 * heads], qkv[:, :, 2 * heads:]
    else:
        dq, dck, dcv = dev(q), dev(ck), dev(cv)
    dpk, dpv = dev(pk), dev(pv)
    out = routed_attention(dq, dck, dcv, dpk, dpv,
                           torch.tensor(slots, dtype=torch.int32, device="cuda"),
                           torch.tensor(ppos, dtype=torch.int32, device="cuda"),
                           torch.tensor(qpos, dtype=torch.int32, device="cuda"),
                           torch.from_numpy(tc).cuda(), torch.from_numpy(ts).cuda(), H, W, wh, ww)
    assert_no_device_error()
    got = host(out)
    hs = list(range(heads)) if check_heads is None else check_heads
    ref = oatt.routed_attention(q[:, :, hs], ck[:, :, hs], cv[:, :, hs], pk[:, :, hs],
                                pv[:, :, hs], slots, ppos, qpos, tc, ts, H, W, wh, ww)
    g = got[:, :, hs]
    err_abs = np.abs(g - ref).max()
    err_rel = max_rel(g, ref)
    # abs_scale: outputs far from unit scale are compared at the same relative
    # bf16 precision (the absolute bound is stated for unit-scale values).
    bound = ABS * max(1.0, float(np.abs(ref).max())) if abs_scale else ABS
    assert err_abs <= bound and err_rel <= REL, (err_abs, err_rel)
    return err_abs


def test_dense_golden_fixture(golden):
    """Against the reference's own sdpa_attention (fp32, CPU) outputs."""
    from recavsr_b200.kernels.local_attention import sdpa_attention
    g = {n: dev_bf16(bf16_from_bits(golden[f"attn_dense_{n}"])) for n in ("q", "ck", "cv", "pk", "pv")}
    tc, ts, _, _ = orope.rolling_tables(128, 4, 6)
    out = sdpa_attention(g["q"], g["ck"], g["cv"], g["pk"], g["pv"],
                         torch.tensor([2, -1, 0], dtype=torch.int32, device="cuda"),
                         torch.tensor([5, 0, 3], dtype=torch.int32, device="cuda"),
                         torch.tensor([6, 7], dtype=torch.int32, device="cuda"),
                         torch.from_numpy(tc).cuda(), torch.from_numpy(ts).cuda(), 4, 6, 22, 40)
    ref = golden["attn_dense_f32"]
    assert np.abs(host(out) - ref).max() <= ABS
    assert max_rel(host(out), ref) <= REL


def test_window_golden_fixture(golden):
    """Windowed case of the reference Triton kernel (fixture win_b, d=128), inputs
    re-rounded to bf16; checked against the oracle on the same bf16 inputs and
    loosely against the fp16 Triton output itself."""
    from recavsr_b200.kernels.local_attention import paired_attention
    if "attn_win_b_out" not in golden:
        pytest.skip("fixture generated without TRITON_INTERPRET=1")
    H, W, wh, ww, d, cap = (int(v) for v in golden["attn_win_b_meta"][:6])
    rest = [int(v) for v in golden["attn_win_b_meta"][6:]]
    slots, ppos = rest[:cap], rest[cap:]
    a = {n: bf16_round(golden[f"attn_win_b_{n}"].astype(np.float32)) for n in ("q", "ck", "cv", "pk", "pv")}
    tc, ts, _, _ = orope.rolling_tables(d, H, W)
    out = paired_attention(*(dev_bf16(a[n]) for n in ("q", "ck", "cv", "pk", "pv")),
                           torch.tensor(slots, dtype=torch.int32, device="cuda"),
                           torch.tensor(ppos, dtype=torch.int32, device="cuda"),
                           torch.tensor([7, 8], dtype=torch.int32, device="cuda"),
                           torch.from_numpy(tc).cuda(), torch.from_numpy(ts).cuda(), H, W, wh, ww)
    got = host(out)
    ref = oatt.routed_attention(a["q"], a["ck"], a["cv"], a["pk"], a["pv"], slots, ppos, [7, 8],
                                tc, ts, H, W, wh, ww)
    assert np.abs(got - ref).max() <= ABS
    assert np.abs(got - golden["attn_win_b_out"]).max() <= 5e-2


@pytest.mark.parametrize("H,W,wh,ww,cap,slots,ppos,qpos", [
    (4, 6, 22, 40, 3, [2, -1, 0], [5, 0, 3], [6, 7]),          # dense, one empty slot
    (22, 40, 22, 40, 2, [0, 1], [6, 7], [8, 9]),                # cfg4 geometry, recent_2
    (22, 40, 22, 40, 0, [], [], [0, 1]),                        # empty cache
    (22, 40, 22, 40, 4, [-1, -1, -1, -1], [0, 0, 0, 0], [2, 3]),  # all slots empty
    (11, 20, 22, 40, 0, [], [], [0, 1, 2, 3, 4, 5]),            # 6-frame prefix
    (8, 16, 4, 8, 3, [2, -1, 0], [3, 0, 5], [7, 8]),            # local windows
    (34, 60, 22, 40, 3, [1, 0, 2], [3, 4, 5], [6, 7]),          # cfg5 1080p local
    (13, 45, 22, 40, 1, [0], [2], [3, 4]),                      # local on one axis only
])
def test_routed_attention(H, W, wh, ww, cap, slots, ppos, qpos):
    _run(H, W, wh, ww, cap, slots, ppos, qpos, check_heads=[0, 1])


def test_cfg2_eight_plane_scope():
    """cfg2 shape: 24 heads, T=880, an 8-plane ring with all planes routed."""
    slots = [3, 0, 7, 1, 6, 2, 5, 4]
    ppos = [1, 2, 3, 4, 5, 6, 7, 8]
    _run(22, 40, 22, 40, 8, slots, ppos, [9, 10], heads=24, check_heads=[0, 13, 23],
         std=1.0 / np.sqrt(128) * 4)


def test_strided_qkv_views():
    """q/k/v as head slices of one fused QKV activation (token stride 3*heads*d)."""
    _run(22, 40, 22, 40, 2, [1, 0], [4, 5], [6, 7], heads=4, fused=True)


def test_peaked_scores_rescale():
    """Large logits force the lazy running-max rescale path."""
    _run(22, 40, 22, 40, 2, [0, 1], [3, 4], [5, 6], heads=2, std=3.0, abs_scale=True)


def test_rejects_bad_geometry():
    from recavsr_b200.kernels.local_attention import paired_attention
    q = torch.zeros(1, 3 * 24, 2, 128, dtype=torch.bfloat16, device="cuda")
    e = torch.zeros(1, 0, 2, 128, dtype=torch.bfloat16, device="cuda")
    i = torch.zeros(0, dtype=torch.int32, device="cuda")
    qp = torch.zeros(3, dtype=torch.int32, device="cuda")
    c = torch.zeros(22, 22, device="cuda")
    with pytest.raises(ValueError):
        paired_attention(q, q, q, e, e, i, i, qp, c, c, 4, 6, 2, 2)   # 3 frames


@pytest.mark.parametrize("split", [False, True])
@pytest.mark.parametrize("nq,nk,heads", [(192, 64, 6), (1760, 512, 24), (1760, 2048, 24), (48, 16, 2)])
def test_cross_attention(nq, nk, heads, split):
    """Unmasked, rotary-free attention over the prompt keys (transformer.py:123-128);
    split=True passes a tail-split workspace, twice in a row (1760 x 24 heads
    over 2048 keys: the last wave's 40 query tiles run as three key-range
    pieces each; over 512 keys the units are too short to split)."""
    import ctypes as C
    from recavsr_b200 import _lib
    rs = np.random.RandomState(nq + nk)
    q = recipes.bf16_normal(rs, (nq, heads, 128))
    k = recipes.bf16_normal(rs, (nk, heads, 128))
    v = recipes.bf16_normal(rs, (nk, heads, 128))
    dq, dk, dv = dev_bf16(q), dev_bf16(k), dev_bf16(v)
    out = torch.empty(nq, heads, 128, dtype=torch.bfloat16, device="cuda")
    hd = heads * 128
    st = (C.c_longlong * 9)(0, hd, 128, 0, hd, 128, 0, hd, 128)
    if split:
        wsb = _lib.library().rc_cross_attention_workspace()
        ws = torch.zeros(wsb, dtype=torch.uint8, device="cuda")
        for _ in range(2):
            _lib.call("rc_cross_attention_ws", dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), st, 1, nq,
                      nk, heads, 128, out.data_ptr(), hd, None, None, ws.data_ptr(), wsb, _lib.stream())
        assert int(ws[-640:].count_nonzero()) == 0   # the arrival counters are back at zero
    else:
        _lib.call("rc_cross_attention", dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), st, 1, nq, nk,
                  heads, 128, out.data_ptr(), hd, None, None, _lib.stream())
    assert_no_device_error()
    hs = [0, 13 % heads, heads - 1]
    ref = oatt.plain_attention(q[:, hs], k[:, hs], v[:, hs])
    got = host(out)[:, hs]
    assert np.abs(got - ref).max() <= ABS and max_rel(got, ref) <= REL


def test_routed_attention_six_heads_small_plane():
    _run(8, 12, 22, 40, 2, [1, 0], [3, 4], [5, 6], heads=6)


def test_attention_fused_nvfp4_output():
    """The optional NVFP4 output equals rc_nvfp4_quantize of the bf16 output."""
    import ctypes as C
    from recavsr_b200 import _lib
    from recavsr_b200.runtime.block import rope_tables
    from recavsr_b200.runtime.nvfp4 import quantize, scale_numel
    H, W, heads = 22, 40, 24
    t = H * W
    rs = np.random.RandomState(9)
    q, k, v = (dev_bf16(recipes.bf16_normal(rs, (1, 2 * t, heads, 128))) for _ in range(3))
    pk, pv = (dev_bf16(recipes.bf16_normal(rs, (1, 2 * t, heads, 128))) for _ in range(2))
    tb = rope_tables(128, H, W, "cuda")
    slots = torch.tensor([1, 0], dtype=torch.int32, device="cuda")
    ppos = torch.tensor([3, 4], dtype=torch.int32, device="cuda")
    qpos = torch.tensor([5, 6], dtype=torch.int32, device="cuda")
    n, dim = 2 * t, heads * 128
    out = torch.empty(1, n, heads, 128, dtype=torch.bfloat16, device="cuda")
    codes = torch.empty(n, dim // 2, dtype=torch.uint8, device="cuda")
    sf = torch.full((scale_numel(n, dim),), 0x5A, dtype=torch.uint8, device="cuda")
    wsb = _lib.library().rc_paired_attention_workspace(1, 2, 2, H, W, heads, 128)
    ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
    st = []
    for x in (q, k, v, pk, pv):
        st += [x.stride(0), x.stride(1), x.stride(2)]
    _lib.call("rc_paired_attention", q.data_ptr(), k.data_ptr(), v.data_ptr(), pk.data_ptr(),
              pv.data_ptr(), (C.c_longlong * 15)(*st), slots.data_ptr(), ppos.data_ptr(),
              qpos.data_ptr(), tb["temporal_cos"].data_ptr(), tb["temporal_sin"].data_ptr(), 1, 2, 2,
              H, W, heads, 128, 44, H, W, ws.data_ptr(), wsb, out.data_ptr(), dim, codes.data_ptr(),
              sf.data_ptr(), _lib.stream())
    rc_, rs_ = quantize(out.reshape(n, dim))
    assert_no_device_error()
    assert torch.equal(codes, rc_) and torch.equal(sf, rs_)
