"""The drop-in operator surface composed the way the reference composes it.

`DropInBlock` restates recavsr_infer/runtime/transformer.py:28-134
(PreparedBlock with native_norms=True and NVFP4 linears) line for line, but
every operator it calls is this package's drop-in: native_layer_norm on the
fp32 rows the reference passes (:91,121,130), native_rms_norm, apply_rotary,
sdpa_attention, NVFP4Linear (quantize + nvfp4_mm). Only the reference's own
torch calls stay torch (the fp32 modulation arithmetic, GELU, the
cross-attention SDPA, :88-133). The block runs eagerly and under
torch.compile(fullgraph=True, dynamic=False) with the reference's Inductor
options (transformer.py:229-246), which traces through the ops' fake
implementations, and is checked against the reference PreparedBlock fixtures.
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F
from torch import nn

from oracle.numerics import bf16_from_bits
from tests.golden import recipes
from tests.util import assert_no_device_error, dev_bf16, host

pytestmark = pytest.mark.gpu

BLOCK_REL_L2 = 0.06       # NVFP4 code flips between faithful implementations (test_gpu_block.py)
BLOCK_MAX_FRAC = 0.15


class _Norm(nn.Module):
    """The attributes PreparedBlock.layer_norm / rms_norm read (weight, bias, eps)."""

    def __init__(self, dim, weight=None, bias=None, eps=1e-6):
        super().__init__()
        self.weight = None if weight is None else nn.Parameter(weight, requires_grad=False)
        self.bias = None if bias is None else nn.Parameter(bias, requires_grad=False)
        self.eps = eps


class DropInBlock(nn.Module):
    """PreparedBlock.forward (transformer.py:81-134) over the drop-in ops."""

    def __init__(self, p, heads, H, W, modulation, cross_k, cross_v, window=(22, 40)):
        super().__init__()
        from recavsr_b200.runtime.nvfp4 import NVFP4Linear
        from recavsr_b200.runtime.rope import RollingRoPE
        dim = p["q_w"].shape[1]
        self.heads, self.height, self.width, self.window = heads, H, W, window
        self.local = H > window[0] or W > window[1]

        def lin(name):
            m = nn.Linear(p[name + "_w"].shape[1], p[name + "_w"].shape[0], device="cuda",
                          dtype=torch.bfloat16)
            with torch.no_grad():
                m.weight.copy_(dev_bf16(p[name + "_w"]))
                m.bias.copy_(dev_bf16(p[name + "_b"]))
            return NVFP4Linear(m)

        self.q, self.k, self.v, self.o = lin("q"), lin("k"), lin("v"), lin("o")
        self.cq, self.co, self.up, self.down = lin("cq"), lin("co"), lin("up"), lin("down")
        self.norm1 = _Norm(dim)
        self.norm2 = _Norm(dim, dev_bf16(p["norm2_w"]), dev_bf16(p["norm2_b"]))
        self.norm3 = _Norm(dim)
        self.norm_q = _Norm(dim, dev_bf16(p["norm_q"]))
        self.norm_k = _Norm(dim, dev_bf16(p["norm_k"]))
        self.cnorm_q = _Norm(dim, dev_bf16(p["cnorm_q"]))
        rope = RollingRoPE(dim // heads, H, W, device="cuda")
        self.register_buffer("modulation", modulation)
        self.register_buffer("cross_k", cross_k)
        self.register_buffer("cross_v", cross_v)
        self.register_buffer("spatial_cos", rope.spatial_cos)
        self.register_buffer("spatial_sin", rope.spatial_sin)
        self.register_buffer("temporal_cos", rope.temporal_cos)
        self.register_buffer("temporal_sin", rope.temporal_sin)

    def layer_norm(self, module, x):
        from recavsr_b200.kernels.native_norm import native_layer_norm
        return native_layer_norm(x, module.weight, module.bias, module.eps)

    def rms_norm(self, module, x):
        from recavsr_b200.kernels.native_norm import native_rms_norm
        return native_rms_norm(x, module.weight, module.eps)

    def spatial(self, x):
        from recavsr_b200.runtime.rope import apply_rotary
        shape = x.shape
        x = x.reshape(shape[0], -1, self.height * self.width, shape[2], shape[3])
        return apply_rotary(x, self.spatial_cos, self.spatial_sin).reshape(shape)

    def forward(self, hidden, past_key, past_value, slots, past_positions, query_positions):
        from recavsr_b200.kernels.local_attention import paired_attention, sdpa_attention
        shift, scale, gate, cshift, cscale, cgate = [
            part.squeeze(2) for part in self.modulation.chunk(6, dim=2)]
        norm = (self.layer_norm(self.norm1, hidden.float()) * (1 + scale) + shift).to(hidden.dtype)
        q, k, v = self.q(norm), self.k(norm), self.v(norm)
        q = self.spatial(self.rms_norm(self.norm_q, q).unflatten(2, (self.heads, -1)))
        k = self.spatial(self.rms_norm(self.norm_k, k).unflatten(2, (self.heads, -1)))
        v = v.unflatten(2, (self.heads, -1))
        attention = paired_attention if self.local else sdpa_attention
        out = attention(q, k, v, past_key, past_value, slots, past_positions, query_positions,
                        self.temporal_cos, self.temporal_sin, self.height, self.width, *self.window)
        out = self.o(out.flatten(2).to(q.dtype))
        hidden = (hidden.float() + out * gate).to(hidden.dtype)
        norm = self.layer_norm(self.norm2, hidden.float()).to(hidden.dtype)
        q = self.rms_norm(self.cnorm_q, self.cq(norm)).unflatten(2, (self.heads, -1))
        out = F.scaled_dot_product_attention(q.transpose(1, 2), self.cross_k.transpose(1, 2),
                                             self.cross_v.transpose(1, 2), dropout_p=0.0).transpose(1, 2)
        hidden = hidden + self.co(out.flatten(2).to(q.dtype))
        norm = (self.layer_norm(self.norm3, hidden.float()) * (1 + cscale) + cshift).to(hidden.dtype)
        ffn = self.down(F.gelu(self.up(norm), approximate="tanh"))
        hidden = (hidden.float() + ffn.float() * cgate).to(hidden.dtype)
        return hidden, k, v


def _close(got, ref, rel_l2, max_frac):
    rel = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    mx = np.abs(got - ref).max() / np.abs(ref).max()
    assert rel < rel_l2 and mx < max_frac, (rel, mx)


def _setup(golden, tag):
    m = [int(v) for v in golden[f"{tag}_meta"]]
    dim, heads, ffn, H, W, cap, enc, pseed, iseed = m[:9]
    slots, ppos = m[9:9 + cap], m[9 + cap:]
    p = recipes.block_params(dim, heads, ffn, enc_len=enc, seed=pseed)
    d = dim // heads
    modulation = torch.from_numpy(golden[f"{tag}_modulation"]).reshape(1, 1, 6, dim).cuda()
    ck = torch.from_numpy(bf16_from_bits(golden[f"{tag}_cross_k"])).reshape(1, -1, heads, d)
    cv = torch.from_numpy(bf16_from_bits(golden[f"{tag}_cross_v"])).reshape(1, -1, heads, d)
    core = DropInBlock(p, heads, H, W, modulation, ck.cuda().bfloat16(), cv.cuda().bfloat16()).eval()
    hidden, pk, pv = recipes.block_inputs(2 * H * W, cap * H * W, dim, seed=iseed)
    args = (dev_bf16(hidden).reshape(1, 2 * H * W, dim), dev_bf16(pk).reshape(1, -1, heads, d),
            dev_bf16(pv).reshape(1, -1, heads, d),
            torch.tensor(slots, dtype=torch.int32, device="cuda"),
            torch.tensor(ppos, dtype=torch.int32, device="cuda"),
            torch.tensor([6, 7], dtype=torch.int32, device="cuda"))
    ref = {n: bf16_from_bits(golden[f"{tag}_{n}"]) for n in ("hidden", "k", "v")}
    return core, args, ref


def _check(outs, ref):
    h, k, v = (host(t).reshape(-1) for t in outs)
    _close(k, ref["k"].reshape(-1), 5e-3, 2 ** -5)
    _close(v, ref["v"].reshape(-1), 5e-3, 2 ** -5)
    _close(h, ref["hidden"].reshape(-1), BLOCK_REL_L2, BLOCK_MAX_FRAC)


@pytest.mark.parametrize("tag", ["block", "block768"])
def test_dropin_block_eager_matches_reference_block(golden, tag):
    core, args, ref = _setup(golden, tag)
    with torch.inference_mode():
        outs = core(*args)
    assert_no_device_error()
    _check(outs, ref)


def test_dropin_block_compiled_fullgraph_matches_eager(golden):
    """torch.compile(fullgraph=True, dynamic=False) with the Inductor options of
    transformer.py:229-246: every drop-in op traces through its fake, the
    compiled block runs the same kernels and equals the eager block."""
    core, args, ref = _setup(golden, "block768")
    with torch.inference_mode():
        eager = core(*args)
    known = torch._inductor.config.get_config_copy()
    opts = {k: v for k, v in {**torch._inductor.list_mode_options("default"),
                              "emulate_precision_casts": True,
                              "force_same_precision": True}.items() if k in known}
    torch._dynamo.reset()
    compiled = torch.compile(core, fullgraph=True, dynamic=False, options=opts)
    with torch.inference_mode():
        outs = compiled(*args)
        again = compiled(*args)
    assert_no_device_error()
    _check(outs, ref)
    for a, b, c in zip(eager, outs, again):
        assert torch.equal(b, c)
        # Inductor may fuse the fp32 modulation arithmetic differently from eager
        # (one fp32 rounding apart), which can flip an NVFP4 code downstream.
        _close(host(b).reshape(-1), host(a).reshape(-1), 2e-2, 0.1)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("affine", [False, True])
def test_native_layer_norm_any_dtype(dtype, affine):
    """native_norm.py:7-17: layer_norm(x.float(), w.float(), b.float(), eps).to(x.dtype),
    against torch's fp32 layer_norm of the same rows."""
    from recavsr_b200.kernels.native_norm import native_layer_norm
    g = torch.Generator(device="cuda").manual_seed(5)
    x = (torch.randn(1, 440, 3072, generator=g, device="cuda") * 3 + 0.5).to(dtype)
    w = (1 + 0.1 * torch.randn(3072, generator=g, device="cuda")) if affine else None
    b = 0.1 * torch.randn(3072, generator=g, device="cuda") if affine else None
    if affine and dtype != torch.float32:
        w, b = w.to(dtype), b.to(dtype)
    got = native_layer_norm(x, w, b, 1e-6)
    assert got.dtype == dtype and got.shape == x.shape
    ref = F.layer_norm(x.float(), (3072,), None if w is None else w.float(),
                       None if b is None else b.float(), 1e-6)
    err = (got.float() - ref).abs().max().item()
    tol = 2e-5 if dtype == torch.float32 else (2 ** -7 if dtype == torch.bfloat16 else 2 ** -10) * 8
    assert err <= tol, err
    if dtype != torch.float32:   # one rounding of a value within fp32 noise of the reference
        assert (got.float() - ref.to(dtype).float()).abs().max().item() <= tol


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_native_rms_norm_any_dtype(dtype):
    from recavsr_b200.kernels.native_norm import native_rms_norm
    g = torch.Generator(device="cuda").manual_seed(6)
    x = torch.randn(880, 3072, generator=g, device="cuda").to(dtype)
    w = (1 + 0.1 * torch.randn(3072, generator=g, device="cuda")).to(dtype)
    got = native_rms_norm(x, w, 1e-6)
    assert got.dtype == dtype
    ref = F.rms_norm(x.float(), (3072,), w.float(), 1e-6)
    tol = 1e-5 if dtype == torch.float32 else 2 ** -9 * 4
    assert (got.float() - ref).abs().max().item() <= tol


@pytest.mark.parametrize("n", [256, 512, 1024])
@pytest.mark.parametrize("rms", [False, True])
def test_layer_norm_bf16_warp_rows(n, rms):
    """rc_layer_norm's warp-per-row path (bf16 rows of 256 / 512 / 1024, the
    FlashDecoder's RMSNorm over 512): against torch's fp32 norm of the same
    rows, within one bf16 rounding; a ragged row count (not a multiple of 8)
    and a row stride wider than the row."""
    from recavsr_b200 import _lib
    g = torch.Generator(device="cuda").manual_seed(7 + n)
    m = 1003
    base = (torch.randn(m, n + 64, generator=g, device="cuda") * 2 + 0.3).bfloat16()
    x = base[:, :n]
    w = 1 + 0.1 * torch.randn(n, generator=g, device="cuda")
    b = 0.1 * torch.randn(n, generator=g, device="cuda")
    out = torch.full((m, n + 32), 7.0, dtype=torch.bfloat16, device="cuda")
    _lib.call("rc_layer_norm", x.data_ptr(), 1, n + 64, m, n, w.data_ptr(), None if rms else b.data_ptr(), 1e-5,
              int(rms), out.data_ptr(), n + 32, _lib.stream())
    ref = (F.rms_norm(x.float(), (n,), w, 1e-5) if rms else F.layer_norm(x.float(), (n,), w, b, 1e-5))
    err = (out[:, :n].float() - ref).abs() / ref.abs().clamp_min(1e-3)
    assert err.max().item() <= 2 ** -7
    assert torch.all(out[:, n:] == 7.0)
