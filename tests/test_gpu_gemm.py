"""tcgen05 GEMM parity (NVFP4 block-scaled, FP8 per-tensor, bf16) against the
oracle's dequantized fp32 matmul: |out - ref| <= 1e-2 * max|ref| (the
tolerance the spec states for the GEMMs), plus the fused epilogues."""
import numpy as np
import pytest
import torch

from oracle import fp8 as ofp8
from oracle import nvfp4 as onv
from oracle.block import gelu_tanh
from oracle.numerics import bf16_round
from tests.golden import recipes
from tests.util import assert_no_device_error, dev_bf16, dev_u8, host, max_rel

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _operands(m, n, k, seed=2):
    a = recipes.cfg3_activation(m, k, seed=seed)
    w = recipes.cfg3_weight(n, k, seed=seed + 1)
    bias = recipes.bf16_normal(np.random.RandomState(seed + 2), (n,), 0.1)
    ac, asf = onv.quantize(a)
    wc, wsf = onv.quantize(w)
    return a, w, bias, ac, asf, wc, wsf


SHAPES = [(1760, 3072, 3072), (1760, 9216, 3072), (1760, 3072, 14336), (300, 256, 512),
          (128, 128, 64), (77, 384, 320), (1, 16, 64)]


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_nvfp4_gemm_bias(m, n, k):
    from recavsr_b200.runtime import nvfp4
    a, w, bias, ac, asf, wc, wsf = _operands(m, n, k)
    ref = onv.nvfp4_mm(ac, asf, wc, wsf, bias, m, n, k)
    out = nvfp4.nvfp4_mm(dev_u8(ac), dev_u8(wc).view(torch.bfloat16), dev_u8(asf),
                         dev_u8(wsf).view(torch.bfloat16), dev_bf16(bias))
    assert_no_device_error()
    err = max_rel(host(out), ref)
    assert err < TOL, err


def test_nvfp4_linear_end_to_end():
    """NVFP4Linear (quantize on device + GEMM) equals the oracle's NVFP4Linear."""
    from recavsr_b200.runtime.nvfp4 import NVFP4Linear
    m, n, k = 440, 768, 512
    a, w, bias, *_ = _operands(m, n, k, seed=5)
    lin = torch.nn.Linear(k, n).cuda().bfloat16()
    with torch.no_grad():
        lin.weight.copy_(dev_bf16(w))
        lin.bias.copy_(dev_bf16(bias))
    q = NVFP4Linear(lin)
    from oracle.block import QuantLinear
    ref = QuantLinear(w, bias)(a)
    out = host(q(dev_bf16(a)[None])[0])
    assert max_rel(out, ref) < TOL


def test_nvfp4_gemm_alpha_global_scale():
    from recavsr_b200.runtime import nvfp4
    m, n, k = 256, 512, 1024
    a = recipes.cfg3_activation(m, k, seed=7)
    w = recipes.cfg3_weight(n, k, seed=8)
    ga = float(2688.0 / np.abs(a).max())
    gw = float(2688.0 / np.abs(w).max())
    ac, asf = nvfp4.quantize(dev_bf16(a), global_scale=ga)
    wc, wsf = nvfp4.quantize(dev_bf16(w), global_scale=gw)
    out = nvfp4.gemm(ac, wc, asf, wsf, None, alpha=1.0 / (ga * gw))
    ref = a.astype(np.float64) @ w.astype(np.float64).T
    # NVFP4 quantization error itself dominates: compare against the oracle path.
    rc, rs = onv.quantize(a, ga)
    wc2, ws2 = onv.quantize(w, gw)
    oref = onv.nvfp4_mm(rc, rs, wc2, ws2, None, m, n, k, alpha=1.0 / (ga * gw))
    assert max_rel(host(out), oref) < TOL
    assert max_rel(host(out), ref) < 0.2


def _lib_gemm(epi, m, n, k, ac, asf, wc, wsf, bias, out, gate=None, qc=None, qs=None, split=True):
    """rc_nvfp4_gemm_ws (tail split-K with a workspace) or, split=False, rc_nvfp4_gemm."""
    from recavsr_b200 import _lib
    from recavsr_b200.runtime.nvfp4 import split_workspace
    args = [ac.data_ptr(), asf.data_ptr(), wc.data_ptr(), wsf.data_ptr(), _lib.ptr(bias), m, n, k, 1.0,
            epi, _lib.ptr(out), 0 if out is None else out.stride(0), _lib.ptr(gate), _lib.ptr(qc),
            _lib.ptr(qs), 1.0]
    if split:
        ws = split_workspace(ac.device)
        _lib.call("rc_nvfp4_gemm_ws", *args, ws.data_ptr(), ws.numel(), _lib.stream())
    else:
        _lib.call("rc_nvfp4_gemm", *args, _lib.stream())


@pytest.mark.parametrize("split", [True, False])
@pytest.mark.parametrize("m,n,k", [(1760, 3072, 3072), (200, 256, 512), (256, 3072, 14336)])
def test_nvfp4_gemm_gated_residual(m, n, k, split):
    from recavsr_b200 import _lib
    a, w, bias, ac, asf, wc, wsf = _operands(m, n, k, seed=9)
    h = recipes.bf16_normal(np.random.RandomState(3), (m, n))
    gate = np.random.RandomState(4).standard_normal(n).astype(np.float32)
    y = onv.nvfp4_mm(ac, asf, wc, wsf, bias, m, n, k)
    ref = bf16_round(h + y * gate)
    hd = dev_bf16(h)
    _lib_gemm(_lib.EPI_GATED_RESIDUAL, m, n, k, dev_u8(ac), dev_u8(asf), dev_u8(wc), dev_u8(wsf),
              dev_bf16(bias), hd, gate=torch.from_numpy(gate).cuda(), split=split)
    assert max_rel(host(hd), ref) < TOL
    hd2 = dev_bf16(h)
    _lib_gemm(_lib.EPI_RESIDUAL, m, n, k, dev_u8(ac), dev_u8(asf), dev_u8(wc), dev_u8(wsf),
              dev_bf16(bias), hd2, split=split)
    assert max_rel(host(hd2), bf16_round(h + y)) < TOL
    assert_no_device_error()


def test_nvfp4_gemm_split_back_to_back():
    """Split-K GEMMs queued back to back on one workspace (each merge resets its
    tile counter for the next call) give identical results; split and unsplit
    results differ only by the fp32 summation order."""
    from recavsr_b200 import _lib
    from recavsr_b200.runtime.nvfp4 import split_workspace
    m, n, k = 1760, 3072, 14336            # 336 tiles: the last 40 run as 3 k-ranges each
    a, w, bias, ac, asf, wc, wsf = _operands(m, n, k, seed=21)
    y = onv.nvfp4_mm(ac, asf, wc, wsf, bias, m, n, k)
    dac, dasf, dwc, dwsf, db = dev_u8(ac), dev_u8(asf), dev_u8(wc), dev_u8(wsf), dev_bf16(bias)
    outs = [torch.empty(m, n, dtype=torch.bfloat16, device="cuda") for _ in range(6)]
    for o in outs:
        _lib_gemm(_lib.EPI_BIAS, m, n, k, dac, dasf, dwc, dwsf, db, o)
    plain = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    _lib_gemm(_lib.EPI_BIAS, m, n, k, dac, dasf, dwc, dwsf, db, plain, split=False)
    assert_no_device_error()
    for o in outs:
        assert max_rel(host(o), y) < TOL
        assert torch.equal(o, outs[0])                       # fixed summation order
    assert max_rel(host(outs[0]), host(plain)) < 2 ** -8      # summation order only
    assert int(split_workspace(dac.device)[-640:].count_nonzero()) == 0   # counters back at zero


@pytest.mark.parametrize("m,n,k", [(1760, 14336, 3072), (130, 512, 256), (256, 3072, 8192)])
def test_nvfp4_gemm_gelu_requantize(m, n, k):
    """ffn_up epilogue: GELU(tanh) then NVFP4 codes/scales for ffn_down. The
    re-quantized operand must dequantize to the oracle's within one E2M1 step
    per element where the bf16 GELU outputs agree."""
    from recavsr_b200 import _lib
    from recavsr_b200.runtime.nvfp4 import scale_numel
    a, w, bias, ac, asf, wc, wsf = _operands(m, n, k, seed=12)
    y = bf16_round(gelu_tanh(onv.nvfp4_mm(ac, asf, wc, wsf, bias, m, n, k)))
    out = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    qc = torch.empty(m, n // 2, dtype=torch.uint8, device="cuda")
    qs = torch.full((scale_numel(m, n),), 0xAB, dtype=torch.uint8, device="cuda")
    _lib_gemm(_lib.EPI_GELU_NVFP4, m, n, k, dev_u8(ac), dev_u8(asf), dev_u8(wc), dev_u8(wsf),
              dev_bf16(bias), out, qc=qc, qs=qs)
    assert_no_device_error()
    yo = host(out)
    assert max_rel(yo, y) < TOL
    # Quantizing the kernel's own bf16 output with the oracle must give its codes exactly.
    rc, rs = onv.quantize(yo)
    np.testing.assert_array_equal(qc.cpu().numpy(), rc)
    np.testing.assert_array_equal(qs.cpu().numpy(), rs)


@pytest.mark.parametrize("m,n,k", [(1760, 3072, 3072), (300, 256, 512), (64, 128, 128)])
def test_fp8_gemm(m, n, k):
    from recavsr_b200 import _lib
    a = recipes.cfg3_activation(m, k, seed=21)
    w = recipes.cfg3_weight(n, k, seed=22)
    bias = recipes.bf16_normal(np.random.RandomState(23), (n,), 0.1)
    aq, sa = ofp8.quantize(a)
    wq, sw = ofp8.quantize(w)
    ref = ofp8.fp8_mm(aq, sa, wq, sw, bias)
    out = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    sad = torch.tensor(sa, dtype=torch.float32, device="cuda")
    swd = torch.tensor(sw, dtype=torch.float32, device="cuda")
    ad, wd, bd = dev_u8(aq), dev_u8(wq), dev_bf16(bias)   # keep alive across the call
    _lib.call("rc_fp8_gemm", ad.data_ptr(), sad.data_ptr(), wd.data_ptr(),
              swd.data_ptr(), bd.data_ptr(), m, n, k, 1.0, _lib.EPI_BIAS,
              out.data_ptr(), n, None, _lib.stream())
    assert_no_device_error()
    assert max_rel(host(out), ref) < TOL


def test_fp8_linear_module():
    from recavsr_b200.runtime.fp8 import FP8Linear
    m, n, k = 300, 512, 768
    a = recipes.cfg3_activation(m, k, seed=31)
    w = recipes.cfg3_weight(n, k, seed=32)
    lin = torch.nn.Linear(k, n).cuda().bfloat16()
    with torch.no_grad():
        lin.weight.copy_(dev_bf16(w))
        lin.bias.zero_()
    out = host(FP8Linear(lin)(dev_bf16(a)))
    aq, sa = ofp8.quantize(a)
    wq, sw = ofp8.quantize(w)
    assert max_rel(out, ofp8.fp8_mm(aq, sa, wq, sw, None)) < TOL


@pytest.mark.parametrize("m,n,k", [(1760, 3072, 3072), (100, 256, 320)])
def test_bf16_gemm(m, n, k):
    from recavsr_b200 import _lib
    rs = np.random.RandomState(41)
    a = recipes.bf16_normal(rs, (m, k))
    w = recipes.bf16_normal(rs, (n, k), 0.02)
    bias = recipes.bf16_normal(rs, (n,), 0.1)
    ref = bf16_round(a.astype(np.float64) @ w.astype(np.float64).T + bias)
    out = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    ad, wd, bd = dev_bf16(a), dev_bf16(w), dev_bf16(bias)   # keep alive across the call
    _lib.call("rc_bf16_gemm", ad.data_ptr(), wd.data_ptr(), bd.data_ptr(), m, n, k,
              _lib.EPI_BIAS, out.data_ptr(), n, None, _lib.stream())
    assert_no_device_error()
    assert max_rel(host(out), ref) < TOL


def test_gemm_rejects_bad_k():
    from recavsr_b200.runtime import nvfp4
    a = torch.zeros(16, 24, dtype=torch.uint8, device="cuda")
    with pytest.raises(ValueError):
        nvfp4.gemm(a, a, torch.zeros(512, dtype=torch.uint8, device="cuda"),
                   torch.zeros(512, dtype=torch.uint8, device="cuda"))


def test_bf16_gemm_grouped_tile_raster():
    """Operands beyond half the L2 (here 2 x 64 MB) run in the grouped tile
    order (12 row blocks per group; 2000 rows = 16 row blocks, so the last
    group is partial): every output tile must still land where it belongs.
    Reference: fp32 matmul of the same bf16 operands, rounded to bf16."""
    from recavsr_b200 import _lib
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    m, n, k = 2000, 2048, 16384
    a = torch.randn(m, k, generator=g, device="cuda").bfloat16()
    w = (torch.randn(n, k, generator=g, device="cuda") * 0.02).bfloat16()
    bias = (torch.randn(n, generator=g, device="cuda") * 0.1).bfloat16()
    out = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    _lib.call("rc_bf16_gemm", a.data_ptr(), w.data_ptr(), bias.data_ptr(), m, n, k, _lib.EPI_BIAS,
              out.data_ptr(), n, None, _lib.stream())
    ref = (a.float() @ w.float().T + bias.float()).bfloat16().float()
    assert_no_device_error()
    err = (out.float() - ref).abs()
    assert float(err.max() / ref.abs().max()) < TOL
    # a misplaced tile would be off by O(1) in some 128 x 128 block
    tiles = torch.nn.functional.pad(err, (0, 0, 0, 2048 - m)).reshape(16, 128, 16, 128).amax((1, 3))
    assert float(tiles.max()) < TOL * float(ref.abs().max()), tiles


def test_nvfp4_gemm_grouped_raster_matches_row_chunks():
    """cfg3's 7040 x 3072 x 14336 NVFP4 GEMM has 72 MB of operands, so it runs in
    the grouped tile order (55 row blocks: four groups of 12 and one of 7); the
    same GEMM as four 1760-row chunks (35 MB each) runs row-fastest. Neither
    splits K (rc_nvfp4_gemm), so every output element is accumulated the same
    way and the two must agree bit for bit."""
    from recavsr_b200 import _lib
    from recavsr_b200.runtime import nvfp4
    g = torch.Generator(device="cuda")
    g.manual_seed(7)
    m, n, k = 7040, 3072, 14336
    a = torch.randn(m, k, generator=g, device="cuda").bfloat16()
    w = (torch.randn(n, k, generator=g, device="cuda") * 0.02).bfloat16()
    bias = (torch.randn(n, generator=g, device="cuda") * 0.1).bfloat16()
    wc, wsf = nvfp4.quantize(w)

    def run(rows):
        ac, asf = nvfp4.quantize(rows)
        out = torch.empty(rows.shape[0], n, dtype=torch.bfloat16, device="cuda")
        _lib.call("rc_nvfp4_gemm", ac.data_ptr(), asf.data_ptr(), wc.data_ptr(), wsf.data_ptr(),
                  bias.data_ptr(), rows.shape[0], n, k, 1.0, _lib.EPI_BIAS, out.data_ptr(), n, None,
                  None, None, 1.0, _lib.stream())
        return out
    full = run(a)
    chunks = torch.cat([run(a[r:r + 1760]) for r in range(0, m, 1760)])
    assert_no_device_error()
    assert torch.equal(full, chunks)


def _pair_rows(m):
    """Sampled 128-row blocks: first, middle, last (ragged)."""
    mid = (m // 2) // 128 * 128
    return np.r_[0:128, mid:mid + 128, m - 128:m]


@pytest.mark.parametrize("epi", ["gated", "residual"])
def test_nvfp4_gemm_pair_residual_epilogues(epi):
    """3520 x 3072 x 14336 runs on CTA pairs (256 x 256 tiles over two SMs):
    the in-place residual epilogues against the oracle on sampled rows."""
    from recavsr_b200 import _lib
    from recavsr_b200.runtime import nvfp4
    m, n, k = 3520, 3072, 14336
    a, w, bias, ac, asf, wc, wsf = _operands(m, n, k, seed=51)
    rs = np.random.RandomState(52)
    h0 = recipes.bf16_normal(rs, (m, n))
    gate = rs.standard_normal(n).astype(np.float32)
    out = dev_bf16(h0)
    gd = torch.from_numpy(gate).cuda()
    code = _lib.EPI_GATED_RESIDUAL if epi == "gated" else _lib.EPI_RESIDUAL
    da, dsa, dw, dsw, db = dev_u8(ac), dev_u8(asf), dev_u8(wc), dev_u8(wsf), dev_bf16(bias)
    ws = nvfp4.split_workspace(da.device)
    _lib.call("rc_nvfp4_gemm_ws", da.data_ptr(), dsa.data_ptr(), dw.data_ptr(), dsw.data_ptr(), db.data_ptr(),
              m, n, k, 1.0, code, out.data_ptr(), n, gd.data_ptr() if epi == "gated" else None, None, None, 1.0,
              ws.data_ptr(), ws.numel(), _lib.stream())
    assert_no_device_error()
    rows = _pair_rows(m)
    rc_, rsf = onv.quantize(a[rows])
    y = onv.nvfp4_mm(rc_, rsf, wc, wsf, bias, len(rows), n, k)
    add = y * gate[None, :] if epi == "gated" else y
    ref = bf16_round(h0[rows] + bf16_round(add))
    assert max_rel(host(out)[rows], ref) < TOL


def test_nvfp4_gemm_pair_gelu_ragged_rows():
    """M = 3400 has 27 row blocks of 128, so the last 256-row pair tile's
    second CTA lies wholly past the matrix: its rows must be skipped, the
    scale atoms of the padding rows (3400..3455) written as zero and nothing
    written past them. GELU + NVFP4 epilogue, N = 14336 (pair path)."""
    from recavsr_b200 import _lib
    from recavsr_b200.runtime.nvfp4 import scale_numel
    m, n, k = 3400, 14336, 3072
    a, w, bias, ac, asf, wc, wsf = _operands(m, n, k, seed=53)
    pad = 4096                                   # canary bytes after the scale buffer
    qs_all = torch.full((scale_numel(m, n) + pad,), 0xAB, dtype=torch.uint8, device="cuda")
    qc = torch.empty(m, n // 2, dtype=torch.uint8, device="cuda")
    out = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    _lib_gemm(_lib.EPI_GELU_NVFP4, m, n, k, dev_u8(ac), dev_u8(asf), dev_u8(wc), dev_u8(wsf),
              dev_bf16(bias), out, qc=qc, qs=qs_all)
    assert_no_device_error()
    qs = qs_all[:scale_numel(m, n)].cpu().numpy()
    assert (qs_all[scale_numel(m, n):].cpu().numpy() == 0xAB).all()          # nothing past the buffer
    sf = onv.unswizzle_scales(qs, (m + 127) // 128 * 128, n)
    assert (sf[m:] == 0).all()                                               # padding rows zeroed
    rows = _pair_rows(m)
    rc_, rsf = onv.quantize(a[rows])
    y = bf16_round(gelu_tanh(onv.nvfp4_mm(rc_, rsf, wc, wsf, bias, len(rows), n, k)))
    yo = host(out)
    assert max_rel(yo[rows], y) < TOL
    ec, es = onv.quantize(yo[m - 128:m])
    np.testing.assert_array_equal(qc.cpu().numpy()[m - 128:m], ec)


def test_bf16_gemm_swiglu_epilogue():
    """RC_EPI_SWIGLU: weights with gate / up rows interleaved in blocks of 8;
    the fused output equals torch's bf16 SiLU(gate) * up applied to the same
    GEMM's bias-epilogue output (within one bf16 rounding on <= 0.1% of the
    values); ragged M, output row stride wider than N / 2."""
    from recavsr_b200 import _lib
    from recavsr_b200.runtime.decoder import _swiglu_rows
    import torch.nn.functional as F
    g = torch.Generator(device="cuda").manual_seed(21)
    m, k, h = 1003, 512, 1024
    x = torch.randn(m, k, generator=g, device="cuda").bfloat16()
    wg, wu = (torch.randn(h, k, generator=g, device="cuda") / k ** 0.5 for _ in range(2))
    bg, bu = (torch.randn(h, generator=g, device="cuda") * 0.1 for _ in range(2))
    w, b = _swiglu_rows(wg, wu, x.device), _swiglu_rows(bg, bu, x.device)
    y = torch.empty(m, 2 * h, dtype=torch.bfloat16, device="cuda")
    _lib.call("rc_bf16_gemm", x.data_ptr(), w.data_ptr(), b.data_ptr(), m, 2 * h, k, _lib.EPI_BIAS, y.data_ptr(),
              2 * h, None, _lib.stream())
    out = torch.full((m, h + 64), 3.0, dtype=torch.bfloat16, device="cuda")
    _lib.call("rc_bf16_gemm", x.data_ptr(), w.data_ptr(), b.data_ptr(), m, 2 * h, k, _lib.EPI_SWIGLU,
              out.data_ptr(), h + 64, None, _lib.stream())
    yy = y.view(m, h // 8, 2, 8)
    ref = (F.silu(yy[:, :, 0]) * yy[:, :, 1]).reshape(m, h)
    got = out[:, :h]
    diff = (got.float() - ref.float()).abs() / ref.float().abs().clamp_min(1e-20)
    assert (diff > 0).float().mean().item() <= 1e-3 and diff.max().item() <= 2 ** -7
    assert torch.all(out[:, h:] == 3.0)
    with pytest.raises(ValueError):
        _lib.call("rc_bf16_gemm", x.data_ptr(), w.data_ptr(), b.data_ptr(), m, 2 * h, k, _lib.EPI_SWIGLU,
                  out.data_ptr(), h // 2, None, _lib.stream())


def test_bf16_gemm_split_workspace_matches_plain():
    """rc_bf16_gemm_ws (the session glue's convolution GEMMs): 336 tiles of
    128 x 128, the last 40 run as 3 k-ranges; the result equals rc_bf16_gemm's
    up to the fp32 summation order, repeats exactly, and leaves the workspace's
    counters at zero. Both against the fp32 matmul."""
    from recavsr_b200 import _lib
    from recavsr_b200.runtime.ops import split_workspace
    m, n, k = 1760, 3072, 4096
    rs = np.random.RandomState(31)
    a = recipes.bf16_normal(rs, (m, k))
    w = recipes.bf16_normal(rs, (n, k), 0.02)
    b = recipes.bf16_normal(rs, (n,), 0.1)
    ad, wd, bd = dev_bf16(a), dev_bf16(w), dev_bf16(b)
    ws = split_workspace(ad.device)
    outs = []
    for _ in range(3):
        o = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
        _lib.call("rc_bf16_gemm_ws", ad.data_ptr(), wd.data_ptr(), bd.data_ptr(), m, n, k, _lib.EPI_BIAS,
                  o.data_ptr(), n, None, ws.data_ptr(), ws.numel(), _lib.stream())
        outs.append(o)
    plain = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    _lib.call("rc_bf16_gemm", ad.data_ptr(), wd.data_ptr(), bd.data_ptr(), m, n, k, _lib.EPI_BIAS,
              plain.data_ptr(), n, None, _lib.stream())
    assert_no_device_error()
    ref = a.astype(np.float64) @ w.astype(np.float64).T + b
    for o in outs:
        assert torch.equal(o, outs[0])
    assert max_rel(host(outs[0]), ref) < TOL
    assert max_rel(host(outs[0]), host(plain)) < 2 ** -8
    assert int(ws[-640:].count_nonzero()) == 0


def test_bf16_gemm_wide_tiles_long_k():
    """bf16 GEMMs with K >= 16384 and at least four waves of 128 x 256 tiles
    (the LQ projector's conv1 shape class) run on the wide single-accumulator
    tiles: 9472 x 2048 x 16384 with bias and with the residual epilogue
    against torch's fp32 matmul of the same bf16 operands."""
    from recavsr_b200 import _lib
    g = torch.Generator(device="cuda").manual_seed(41)
    m, n, k = 9472, 2048, 16384
    a = torch.randn(m, k, generator=g, device="cuda").bfloat16()
    w = (torch.randn(n, k, generator=g, device="cuda") * 0.02).bfloat16()
    b = (torch.randn(n, generator=g, device="cuda") * 0.1).bfloat16()
    ref = a.float() @ w.float().T + b.float()
    out = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    _lib.call("rc_bf16_gemm", a.data_ptr(), w.data_ptr(), b.data_ptr(), m, n, k, _lib.EPI_BIAS, out.data_ptr(), n,
              None, _lib.stream())
    h = (torch.randn(m, n, generator=g, device="cuda")).bfloat16()
    res = h.clone()
    _lib.call("rc_bf16_gemm", a.data_ptr(), w.data_ptr(), b.data_ptr(), m, n, k, _lib.EPI_RESIDUAL, res.data_ptr(),
              n, None, _lib.stream())
    assert_no_device_error()
    scale = ref.abs().max().item()
    assert (out.float() - ref).abs().max().item() < TOL * scale
    ref_res = h.float() + ref.bfloat16().float()
    assert (res.float() - ref_res).abs().max().item() < TOL * ref_res.abs().max().item()
