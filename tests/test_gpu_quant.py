"""Quantizer parity on the GPU: bit-exact against the reference's own outputs
(tests/golden) and against the oracle on cfg3-sized inputs."""
import numpy as np
import pytest
import torch

from oracle import fp8 as ofp8
from oracle import nvfp4 as onv
from oracle.numerics import bf16_from_bits
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
