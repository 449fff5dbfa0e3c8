"""Quantizer parity on the GPU: bit-exact against the reference's own outputs
(tests/golden) and against the oracle on cfg3-sized inputs."""
import numpy as np
import pytest
import torch

from oracle import fp8 as ofp8
from oracle import nvfp4 as onv
from oracle.numerics import bf16_from_bits, bf16_round
from tests.golden import recipes
from tests.util import assert_no_device_error, dev_bf16

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("case", ["special", "ragged", "weights", "cfg3_small"])
def test_nvfp4_quantize_matches_reference(golden, case):
    from recavsr_b200.runtime import nvfp4
    x = dev_bf16(bf16_from_bits(golden[f"quant_{case}_x"]))
    codes, scales = nvfp4.quantize(x)
    np.testing.assert_array_equal(codes.cpu().numpy(), golden[f"quant_{case}_codes"])
    np.testing.assert_array_equal(scales.cpu().numpy(), golden[f"quant_{case}_scales"])
    assert_no_device_error()


@pytest.mark.parametrize("m,k", [(1760, 3072), (3520, 3072), (1760, 14336), (1, 64), (129, 80)])
def test_nvfp4_quantize_cfg3_shapes(m, k):
    from recavsr_b200.runtime import nvfp4
    x = recipes.cfg3_activation(m, k, seed=2)
    codes, scales = nvfp4.quantize(dev_bf16(x))
    rc, rs = onv.quantize(x)
    np.testing.assert_array_equal(codes.cpu().numpy(), rc)
    np.testing.assert_array_equal(scales.cpu().numpy(), rs)


def test_nvfp4_quantize_strided_rows():
    from recavsr_b200.runtime import nvfp4
    x = recipes.cfg3_activation(200, 512, seed=3)
    big = torch.zeros(200, 768, dtype=torch.bfloat16, device="cuda")
    big[:, 128:640] = dev_bf16(x)
    codes, scales = nvfp4.quantize(big[:, 128:640])
    rc, rs = onv.quantize(x)
    np.testing.assert_array_equal(codes.cpu().numpy(), rc)
    np.testing.assert_array_equal(scales.cpu().numpy(), rs)


def test_nvfp4_global_scale_mode():
    from recavsr_b200.runtime import nvfp4
    x = recipes.cfg3_activation(256, 512, seed=4)
    g = float(448.0 * 6.0 / np.abs(x).max())
    codes, scales = nvfp4.quantize(dev_bf16(x), global_scale=g)
    rc, rs = onv.quantize(x, global_scale=g)
    np.testing.assert_array_equal(codes.cpu().numpy(), rc)
    np.testing.assert_array_equal(scales.cpu().numpy(), rs)


@pytest.mark.parametrize("case", ["act", "weight"])
def test_fp8_quantize_matches_reference(golden, case):
    from recavsr_b200.runtime import fp8
    q, scale = fp8.quantize(dev_bf16(bf16_from_bits(golden[f"fp8_{case}_x"])))
    assert np.float32(scale.item()) == golden[f"fp8_{case}_scale"]
    np.testing.assert_array_equal(q.cpu().numpy(), golden[f"fp8_{case}_q"])


def test_fp8_quantize_cfg3():
    from recavsr_b200.runtime import fp8
    x = recipes.cfg3_activation(1760, 3072, seed=2)
    q, scale = fp8.quantize(dev_bf16(x))
    rq, rscale = ofp8.quantize(x)
    assert np.float32(scale.item()) == rscale
    np.testing.assert_array_equal(q.cpu().numpy(), rq)


def test_fp8_quantize_back_to_back():
    """Many quantizations queued without a host sync: the quantize kernel of
    each call starts while its amax kernel still runs (programmatic dependent
    launch) and must read the finished amax, never a partial one."""
    from recavsr_b200.runtime import fp8
    x = recipes.cfg3_activation(1760, 3072, seed=5)
    rq, rscale = ofp8.quantize(x)
    xd = dev_bf16(x)
    outs = [fp8.quantize(xd) for _ in range(40)]
    for q, scale in outs:
        assert np.float32(scale.item()) == rscale
        np.testing.assert_array_equal(q.cpu().numpy(), rq)


def test_fp8_quantize_strided_rows():
    """Rows with a pitch larger than K take the indexed (non-packed) path."""
    from recavsr_b200.runtime import fp8
    x = recipes.cfg3_activation(300, 1024, seed=6)
    big = torch.zeros(300, 1280, dtype=torch.bfloat16, device="cuda")
    big[:, 256:1280] = dev_bf16(x)
    q, scale = fp8.quantize(big[:, 256:1280])
    rq, rscale = ofp8.quantize(x)
    assert np.float32(scale.item()) == rscale
    np.testing.assert_array_equal(q.cpu().numpy(), rq)
    assert_no_device_error()


@pytest.mark.parametrize("amax", [448.0, 1.0, 3.0e-3, 6.0e4, 2.0 ** -100, 3.0e38])
def test_fp8_quantize_every_bf16_value(amax):
    """Every finite bf16 x with |x| <= amax, quantized with scale amax/448:
    covers each E4M3 rounding boundary, the subnormal codes and the zeros."""
    from recavsr_b200.runtime import fp8
    from oracle.numerics import bf16_from_bits
    amax = bf16_round(np.array([amax], np.float32))[0]
    allx = bf16_from_bits(np.arange(65536, dtype=np.uint32).astype(np.uint16)).astype(np.float32)
    xs = allx[np.abs(allx) <= amax]
    xs = np.concatenate([[amax], xs])
    xs = np.concatenate([xs, np.zeros((-len(xs)) % 1024, np.float32)]).reshape(-1, 1024)
    q, scale = fp8.quantize(dev_bf16(xs))
    rq, rscale = ofp8.quantize(xs)
    assert np.float32(scale.item()) == rscale
    np.testing.assert_array_equal(q.cpu().numpy(), rq)


def test_fp8_quantize_many_scales():
    """64 amax values spread over the bf16 range (each a separate call, so
    each its own per-tensor scale), every bf16 |x| <= amax of both signs."""
    from recavsr_b200.runtime import fp8
    from oracle.numerics import bf16_from_bits
    allx = bf16_from_bits(np.arange(65536, dtype=np.uint32).astype(np.uint16)).astype(np.float32)
    allx = allx[np.isfinite(allx)]
    pos = np.sort(allx[allx > 0])
    rng = np.random.default_rng(11)
    for amax in pos[np.sort(rng.choice(len(pos), 64, replace=False))]:
        xs = np.concatenate([[amax], allx[np.abs(allx) <= amax]])
        xs = np.concatenate([xs, np.zeros((-len(xs)) % 512, np.float32)]).reshape(-1, 512)
        q, scale = fp8.quantize(dev_bf16(xs))
        rq, rscale = ofp8.quantize(xs)
        assert np.float32(scale.item()) == rscale, amax
        np.testing.assert_array_equal(q.cpu().numpy(), rq, err_msg=f"amax={amax}")


@pytest.mark.parametrize("special", [np.inf, -np.inf, np.nan])
def test_fp8_quantize_non_finite(special):
    """An inf makes the scale inf (finite values -> signed zeros, inf/inf ->
    NaN code); a NaN makes the scale NaN and every code the NaN code. The
    sign of a NaN that a division creates is the platform's default NaN
    (negative on x86, positive on the GPU), so NaN codes compare by
    magnitude; every other code is bit-exact."""
    from recavsr_b200.runtime import fp8
    x = recipes.cfg3_activation(64, 256, seed=7)
    x[5, 17] = special
    q, scale = fp8.quantize(dev_bf16(x))
    rq, rscale = ofp8.quantize(x)
    got = np.float32(scale.item())
    assert got == rscale or (np.isnan(got) and np.isnan(rscale))
    q = q.cpu().numpy()
    nan_code = (rq & 0x7F) == 0x7F
    np.testing.assert_array_equal(q[~nan_code], rq[~nan_code])
    np.testing.assert_array_equal(q[nan_code] & 0x7F, rq[nan_code] & 0x7F)


def test_nvfp4_quantize_every_bf16_value_every_scale():
    """Blocks [6s, x, ...] pin the block scale to each E4M3 value s in turn and
    run every bf16 x with |x| <= 6s through the device quantizer."""
    from recavsr_b200.runtime import nvfp4
    from oracle.numerics import bf16_from_bits, e4m3_decode
    allx = bf16_from_bits(np.arange(65536, dtype=np.uint32).astype(np.uint16))
    allx = allx[np.isfinite(allx)]
    rows = []
    for s in e4m3_decode(np.arange(1, 127, dtype=np.uint8)):
        amax = np.float32(6.0) * s
        if amax != bf16_round(amax) or amax / np.float32(6.0) < 2.0 ** -9:
            continue
        xs = allx[np.abs(allx) <= amax]
        pad = (-len(xs)) % 15
        xs = np.concatenate([xs, np.zeros(pad, np.float32)]).reshape(-1, 15)
        rows.append(np.concatenate([np.full((len(xs), 1), amax, np.float32), xs], 1))
    blocks = np.concatenate(rows, 0)
    n = (len(blocks) // 64) * 64
    x = blocks[:n].reshape(-1, 16 * 64)              # 64 blocks per row
    codes, scales = nvfp4.quantize(dev_bf16(x))
    rc, rs = onv.quantize(x)
    np.testing.assert_array_equal(codes.cpu().numpy(), rc)
    np.testing.assert_array_equal(scales.cpu().numpy(), rs)


def test_nvfp4_quantize_every_bf16_amax():
    """Blocks [a, a/3, -a/7, 0, ...] for every finite positive bf16 a (plus inf
    and NaN blocks): the block scale e4m3(max(a/6, 2^-9)) is computed without
    division on the device and must match the oracle's bytes exactly."""
    from recavsr_b200.runtime import nvfp4
    from oracle.numerics import bf16_from_bits
    amax = bf16_from_bits(np.arange(1, 0x7F80, dtype=np.uint32).astype(np.uint16)).astype(np.float32)
    amax = np.concatenate([amax, np.array([np.inf, np.nan], np.float32)])
    blocks = np.zeros((len(amax), 16), np.float32)
    blocks[:, 0] = amax
    with np.errstate(invalid="ignore"):
        blocks[:, 1] = bf16_round(amax / 3)
        blocks[:, 2] = bf16_round(-amax / 7)
    n = (len(blocks) + 63) // 64 * 64
    blocks = np.concatenate([blocks, np.zeros((n - len(blocks), 16), np.float32)])
    x = blocks.reshape(-1, 16 * 64)
    codes, scales = nvfp4.quantize(dev_bf16(x))
    rc, rs = onv.quantize(x)
    np.testing.assert_array_equal(scales.cpu().numpy(), rs)
    np.testing.assert_array_equal(codes.cpu().numpy(), rc)


@pytest.mark.parametrize("m,k", [(7040, 14336), (7040, 3072)])
def test_quantizers_bit_exact_at_full_size(m, k):
    """The device NVFP4 and FP8 quantizers on cfg3's full-size activations
    produce the reference's exact bytes: SHA-256 of codes and swizzled scales
    (and the FP8 scale) against tests/golden/fullsize_hashes.json, recorded
    from the reference's own quantizers."""
    from recavsr_b200.runtime import fp8, nvfp4
    from tests.test_oracle_fullsize import fullsize_hashes, sha
    ref = fullsize_hashes()
    x = torch.from_numpy(recipes.cfg3_activation_large(m, k)).cuda().bfloat16()   # bf16 values: exact
    codes, scales = nvfp4.quantize(x)
    assert sha(codes.cpu().numpy()) == ref[f"nvfp4_{m}x{k}"]["codes"]
    assert sha(scales.cpu().numpy()) == ref[f"nvfp4_{m}x{k}"]["scales"]
    q, scale = fp8.quantize(x)
    assert np.float32(scale.item()) == np.float32(ref[f"fp8_{m}x{k}"]["scale"])
    assert sha(q.cpu().numpy()) == ref[f"fp8_{m}x{k}"]["codes"]
    assert_no_device_error()
