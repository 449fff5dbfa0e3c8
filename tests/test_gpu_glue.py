"""Glue kernels on the GPU against the oracle / reference fixtures:
LayerNorm+modulation(+NVFP4), RMSNorm+spatial RoPE, temporal RoPE, KV commit."""
import numpy as np
import pytest
import torch

from oracle import nvfp4 as onv
from oracle import rope as orope
from oracle.block import layer_norm, rms_norm
from oracle.numerics import bf16_from_bits, bf16_round
from tests.golden import recipes
from tests.util import assert_no_device_error, dev_bf16, host, max_rel

pytestmark = pytest.mark.gpu


def _ln_call(x, shift=None, scale=None, weight=None, bias=None, quant=False):
    from recavsr_b200 import _lib
    from recavsr_b200.runtime.nvfp4 import scale_numel
    m, n = x.shape
    out = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    qc = torch.empty(m, n // 2, dtype=torch.uint8, device="cuda") if quant else None
    qs = torch.full((scale_numel(m, n),), 0xCD, dtype=torch.uint8, device="cuda") if quant else None
    _lib.call("rc_ln_modulate_quant", x.data_ptr(), x.stride(0), m, n, _lib.ptr(weight),
              _lib.ptr(bias), _lib.ptr(shift), _lib.ptr(scale), 1e-6, out.data_ptr(), n,
              _lib.ptr(qc), _lib.ptr(qs), 1.0, _lib.stream())
    return out, qc, qs


@pytest.mark.parametrize("m,n", [(1760, 3072), (130, 256), (1, 64)])
def test_ln_modulate_quant(m, n):
    rs = np.random.RandomState(3)
    x = recipes.bf16_normal(rs, (m, n)) * 3 + 0.5
    x = bf16_round(x)
    shift = rs.standard_normal(n).astype(np.float32)
    scale = rs.standard_normal(n).astype(np.float32)
    ref = bf16_round(layer_norm(x) * (1 + scale) + shift)
    out, qc, qs = _ln_call(dev_bf16(x), torch.from_numpy(shift).cuda(),
                           torch.from_numpy(scale).cuda(), quant=True)
    assert_no_device_error()
    o = host(out)
    assert max_rel(o, ref) < 1e-2
    # ulp-level agreement on almost every element
    assert np.mean(o != ref) < 0.02
    rc, rsf = onv.quantize(o)
    np.testing.assert_array_equal(qc.cpu().numpy(), rc)
    np.testing.assert_array_equal(qs.cpu().numpy(), rsf)


def test_native_layer_norm_affine():
    from recavsr_b200.kernels.native_norm import native_layer_norm
    rs = np.random.RandomState(4)
    x = recipes.bf16_normal(rs, (3, 50, 3072))
    w = recipes.bf16_normal(rs, (3072,), 1.0)
    b = recipes.bf16_normal(rs, (3072,), 1.0)
    out = host(native_layer_norm(dev_bf16(x), dev_bf16(w), dev_bf16(b), 1e-6))
    ref = bf16_round(layer_norm(x.reshape(-1, 3072), w, b)).reshape(x.shape)
    assert max_rel(out, ref) < 1e-2


def test_native_rms_norm():
    from recavsr_b200.kernels.native_norm import native_rms_norm
    rs = np.random.RandomState(5)
    x = recipes.bf16_normal(rs, (2, 70, 3072), 2.0)
    w = bf16_round(1 + 0.1 * rs.standard_normal(3072).astype(np.float32))
    out = host(native_rms_norm(dev_bf16(x), dev_bf16(w), 1e-6))
    ref = rms_norm(x.reshape(-1, 3072), w).reshape(x.shape)
    assert max_rel(out, ref) < 1e-2
    assert np.mean(out != ref) < 0.01


def test_rmsnorm_rope_qk():
    """RMSNorm across heads then spatial RoPE (PreparedBlock.forward :99-100)."""
    from recavsr_b200 import _lib
    import ctypes as C
    H, W, heads, d = 22, 40, 24, 128
    span = H * W
    m = 2 * span
    rs = np.random.RandomState(6)
    qkv = recipes.bf16_normal(rs, (m, 3 * heads * d))
    wq = bf16_round(1 + 0.1 * rs.standard_normal(heads * d).astype(np.float32))
    wk = bf16_round(1 + 0.1 * rs.standard_normal(heads * d).astype(np.float32))
    _, _, sc, ss = orope.rolling_tables(d, H, W)
    qd = dev_bf16(qkv)
    outs = [torch.empty(m, heads * d, dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    wqd, wkd = dev_bf16(wq), dev_bf16(wk)
    scd, ssd = torch.from_numpy(sc).cuda(), torch.from_numpy(ss).cuda()
    n = heads * d
    _lib.call("rc_rmsnorm_rope", 2, (C.c_void_p * 2)(qd.data_ptr(), qd.data_ptr() + 2 * n),
              (C.c_longlong * 2)(3 * n, 3 * n), (C.c_void_p * 2)(wqd.data_ptr(), wkd.data_ptr()),
              (C.c_void_p * 2)(outs[0].data_ptr(), outs[1].data_ptr()), (C.c_longlong * 2)(n, n),
              m, n, d, span, scd.data_ptr(), ssd.data_ptr(), 1e-6, _lib.stream())
    assert_no_device_error()
    tile_c = np.tile(sc, (2, 1))[:, None, :]
    tile_s = np.tile(ss, (2, 1))[:, None, :]
    for i, w in enumerate((wq, wk)):
        x = qkv[:, i * n:(i + 1) * n]
        ref = orope.apply_rotary(rms_norm(x, w).reshape(m, heads, d), tile_c, tile_s)
        got = host(outs[i]).reshape(m, heads, d)
        assert max_rel(got, ref) < 1e-2
        assert np.mean(got != ref) < 0.01


def test_rope_modules_match_reference(golden):
    from recavsr_b200.runtime.rope import RollingRoPE, apply_temporal
    r = RollingRoPE(128, 11, 20, device="cuda")
    np.testing.assert_array_equal(r.temporal_cos.cpu().numpy(), golden["rope_tcos"])
    np.testing.assert_array_equal(r.spatial_cos.reshape(220, 128).cpu().numpy(), golden["rope_scos"])
    x = dev_bf16(bf16_from_bits(golden["rope_x"]).reshape(1, 440, 3, 128))
    sp = r.spatial(x)
    np.testing.assert_array_equal(host(sp).reshape(-1), bf16_from_bits(golden["rope_spatial"]).reshape(-1))
    pos = torch.tensor([4, 17], dtype=torch.int32, device="cuda")
    tp = apply_temporal(x, pos, r.temporal_cos, r.temporal_sin, span=220)
    np.testing.assert_array_equal(host(tp).reshape(-1), bf16_from_bits(golden["rope_temporal"]).reshape(-1))


def test_cache_commit_matches_router(router_golden):
    """FixedKVCache on the device: slot ids / positions bit-identical to the
    reference over 75 blocks for every action, and plane contents = frame ids."""
    from recavsr_b200.runtime.cache import FixedKVCache
    from recavsr_b200.runtime.rope import RollingRoPE
    span, heads, d = 6, 2, 8
    rope = RollingRoPE(128, 1, 1, device="cuda")
    for action, rec in router_golden.items():
        c = FixedKVCache(action)
        for step in rec["steps"]:
            frames, start = step["frames"], step["start"]
            origin, qpos = rope.positions(start, frames)
            dummy = torch.zeros(1, frames * span, heads, d, device="cuda", dtype=torch.bfloat16)
            _, _, slots, ppos = c.history(dummy, origin=origin)
            assert slots.tolist() == step["slots"] and ppos.tolist() == step["ppos"]
            ids = torch.arange(start, start + frames, device="cuda", dtype=torch.float32)
            k = ids.view(1, frames, 1, 1).expand(1, frames, span, heads * d).reshape(1, frames * span, heads, d)
            k = k.bfloat16().contiguous()
            c.commit(k, (-k).contiguous(), frames=frames, start=start)
            if step["slot_frames"]:
                kk = c.key.float().view(c.capacity, span * heads * d)
                vv = c.value.float().view(c.capacity, span * heads * d)
                for slot, fid in enumerate(step["slot_frames"]):
                    if slot in c.frame_to_slot.values():
                        assert torch.all(kk[slot] == fid) and torch.all(vv[slot] == -fid)
    assert_no_device_error()
