"""One process driving two GPUs: the kernels' shared-memory attributes are set
per device (cudaFuncSetAttribute applies to the current device only), so the
attention and the GEMM launch on the second device after running on the first.
Skipped with fewer than two GPUs."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _run_on(dev):
    from oracle import nvfp4 as onv
    from recavsr_b200.kernels.local_attention import routed_attention
    from recavsr_b200.runtime import nvfp4
    from recavsr_b200.runtime.rope import RollingRoPE
    g = torch.Generator(device=dev).manual_seed(3)
    r = lambda *s, std=1.0: (torch.randn(*s, generator=g, device=dev) * std).bfloat16()
    with torch.cuda.device(dev):
        x, w = r(256, 512), r(384, 512, std=0.05)
        xq, xs = nvfp4.quantize(x)
        wq, ws = nvfp4.quantize(w)
        y = nvfp4.gemm(xq, wq, xs, ws, None)
        rq, rsc = onv.quantize(x.float().cpu().numpy())
        wq_ref, ws_ref = onv.quantize(w.float().cpu().numpy())
        y_ref = onv.nvfp4_mm(rq, rsc, wq_ref, ws_ref, None, 256, 384, 512)
        err = np.abs(y.float().cpu().numpy() - y_ref).max() / np.abs(y_ref).max()
        assert err <= 1e-2, (dev, err)
        H, W, heads = 22, 40, 4
        rope = RollingRoPE(128, H, W, device=dev)
        q, k, v = (r(1, 2 * H * W, heads, 128) for _ in range(3))
        pk, pv = r(1, H * W, heads, 128), r(1, H * W, heads, 128)
        i32 = lambda vals: torch.tensor(vals, dtype=torch.int32, device=dev)
        out = routed_attention(q, k, v, pk, pv, i32([0]), i32([3]), i32([4, 5]), rope.temporal_cos,
                               rope.temporal_sin, H, W, H, W)
        torch.cuda.synchronize(dev)
        return out.float().cpu()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_kernels_run_on_a_second_device_in_one_process():
    from recavsr_b200 import _lib
    a = _run_on(torch.device("cuda", 0))
    b = _run_on(torch.device("cuda", 1))
    assert torch.equal(a, b)           # same inputs, same deterministic kernels
    with torch.cuda.device(1):
        assert _lib.read_device_error() == 0
    with torch.cuda.device(0):
        assert _lib.read_device_error() == 0
