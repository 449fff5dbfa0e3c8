"""FlashDecoder decode step on the device (recavsr_b200.runtime.decoder.DecoderSession)
against the oracle's DecoderOracle (pinned to the reference's
FlashDecoderSession on the CPU): every RGB chunk of a stream long enough to
trim both caches, on a small model and on the released widths (dim 512,
8 / 2 heads, SwiGLU 2048); CUDA-graph replay equal to eager launches bit for
bit; the layout kernels (pixel unshuffle / shuffle) and the SwiGLU SiLU
against torch's own CUDA ops.

Tolerance of the decode: the device runs the reference's CUDA arithmetic (bf16
activations and weights, fp32 accumulation, fp32 norms and RoPE), the oracle
fp32 throughout, so the RGB differ by bf16 rounding propagated through the
blocks: max |err| <= 0.1 and mean |err| <= 6e-3 (RGB in [-1, 1]; measured on
a B200: 0.066 / 0.0052 on the released widths). Against the reference's own
bf16 FlashDecoderSession on the GPU (baseline/compare.py decoder_step) the
largest RGB difference measured 0.012."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import flashdecoder as ofd
from tests.golden import recipes
from tests.util import assert_no_device_error

pytestmark = pytest.mark.gpu


def _session(tag, **kw):
    from recavsr_b200.runtime.decoder import DecoderSession
    c = recipes.DECODER_CASES[tag]
    _, mean, std, _ = recipes.decoder_inputs(tag)
    params = recipes.decoder_params(tag)
    return DecoderSession(params, height=c["h"], width=c["w"], mean=mean, std=std, dim=c["dim"],
                          num_heads=c["num_heads"], num_kv_groups=c["num_kv_groups"], depth=c["depth"],
                          refinement_depth=c["refinement_depth"], mlp_ratio=c["mlp_ratio"], window=c["window"],
                          **kw)


def _oracle(tag):
    c = recipes.DECODER_CASES[tag]
    _, mean, std, _ = recipes.decoder_inputs(tag)
    return ofd.DecoderOracle(recipes.decoder_params(tag), dim=c["dim"], num_heads=c["num_heads"],
                             num_kv_groups=c["num_kv_groups"], depth=c["depth"],
                             refinement_depth=c["refinement_depth"], window=c["window"], mean=mean, std=std)


@pytest.mark.parametrize("tag", sorted(recipes.DECODER_CASES))
def test_decode_stream_matches_oracle(tag):
    lat, _, _, lr = recipes.decoder_inputs(tag)
    sess, orc = _session(tag), _oracle(tag)
    got = [r.float().cpu().numpy()[0] for r in sess.step(torch.from_numpy(lat).cuda(),
                                                          lr_up=torch.from_numpy(lr).cuda())]
    off = 0
    for i, g in enumerate(got):
        take = 1 if i == 0 else 4
        ref, _, _ = orc.step(lat[0, :, i], lr[0, :, off:off + take])
        off += take
        assert g.shape == ref.shape
        err = np.abs(g - ref)
        assert err.max() <= 0.1 and err.mean() <= 6e-3, (i, float(err.max()), float(err.mean()))
    assert_no_device_error()


def test_graph_replay_equals_eager():
    """Two sessions on the same stream of 6 latent frames: eager launches, and
    graphs captured after frame 2 (both ring parities) -- equal bit for bit,
    including after reset() and a second stream."""
    tag = "s"
    c = recipes.DECODER_CASES[tag]
    g = torch.Generator().manual_seed(9)
    frames = 6
    lat = torch.randn(1, 48, frames, c["h"], c["w"], generator=g).cuda()
    lr = (torch.rand(1, 3, 1 + 4 * (frames - 1), 16 * c["h"], 16 * c["w"], generator=g) * 2 - 1).cuda()
    eager, graphed = _session(tag), _session(tag)
    a = [r.clone() for r in eager.step(lat, lr_up=lr)]
    b = [r.clone() for r in graphed.step(lat[:, :, :2], lr_up=lr[:, :, :5])]
    graphed.capture()
    assert len(graphed.graphs) == 2
    b += [r.clone() for r in graphed.step(lat[:, :, 2:], lr_up=lr[:, :, 5:])]
    assert len(a) == len(b) == frames
    for x, y in zip(a, b):
        assert torch.equal(x, y)
    eager.reset()
    graphed.reset()
    a2 = [r.clone() for r in eager.step(lat, lr_up=lr)]
    b2 = [r.clone() for r in graphed.step(lat, lr_up=lr)]
    for x, y in zip(a2, b2):
        assert torch.equal(x, y)
    assert torch.equal(a2[3], a[3])
    assert_no_device_error()


def test_layout_kernels_match_torch():
    """rc_fd_lr_unshuffle = F.pixel_unshuffle(., 16) cast to bf16;
    rc_fd_pixel_shuffle = F.pixel_shuffle(., 16) + clamp; rc_fd_silu = bf16
    F.silu(gate) * up and F.silu, as torch computes them on CUDA."""
    import ctypes as C
    from recavsr_b200 import _lib
    h, w, frames = 3, 5, 4
    g = torch.Generator(device="cuda").manual_seed(3)
    lr = torch.randn(3, frames, 16 * h, 16 * w, generator=g, device="cuda")
    out = torch.empty(frames * h * w, 768, dtype=torch.bfloat16, device="cuda")
    st = (C.c_longlong * 3)(lr.stride(0), lr.stride(1), lr.stride(2))
    _lib.call("rc_fd_lr_unshuffle", lr.data_ptr(), 0, st, frames, h, w, out.data_ptr(), _lib.stream())
    ref = F.pixel_unshuffle(lr.transpose(0, 1), 16).permute(0, 2, 3, 1).reshape(frames * h * w, 768)
    assert torch.equal(out, ref.bfloat16())
    y = (torch.randn(4 * h * w, 768, generator=g, device="cuda") * 1.5).bfloat16()
    rgb = torch.empty(3, 4, 16 * h, 16 * w, dtype=torch.bfloat16, device="cuda")
    _lib.call("rc_fd_pixel_shuffle", y.data_ptr(), 768, 0, 4, 4, h, w, rgb.data_ptr(), _lib.stream())
    ref = F.pixel_shuffle(y.view(4, h, w, 768).permute(0, 3, 1, 2), 16).permute(1, 0, 2, 3).clamp(-1, 1)
    assert torch.equal(rgb, ref)
    gu = (torch.randn(64, 2 * 256, generator=g, device="cuda") * 3).bfloat16()
    act = torch.empty(64, 256, dtype=torch.bfloat16, device="cuda")
    _lib.call("rc_fd_silu", gu.data_ptr(), 64, 256, 0, act.data_ptr(), _lib.stream())
    ref = F.silu(gu[:, :256]) * gu[:, 256:]
    diff = (act.float() - ref.float()).abs() / ref.float().abs().clamp_min(1e-30)
    assert (diff > 0).float().mean() <= 1e-3 and diff.max() <= 2 ** -7, float(diff.max())
    x = gu[:, :256].clone()
    _lib.call("rc_fd_silu", x.data_ptr(), 64, 256, 1, None, _lib.stream())
    assert (x != F.silu(gu[:, :256])).float().mean() <= 1e-3
    assert_no_device_error()


def test_step_host_equals_step():
    """DecoderSession.step_host (RGB copies to pinned host memory on a copy
    stream, overlapping the next frame) delivers the frames step() returns, bit
    for bit, over a stream of blocks with graphs captured mid-stream, reusing
    one pinned buffer per block size after output_ready."""
    tag = "s"
    c = recipes.DECODER_CASES[tag]
    g = torch.Generator().manual_seed(11)
    blocks = 4
    h16, w16 = 16 * c["h"], 16 * c["w"]
    lats = [torch.randn(1, 48, 2, c["h"], c["w"], generator=g).cuda() for _ in range(blocks)]
    lrs = [(torch.rand(1, 3, 5 if i == 0 else 8, h16, w16, generator=g) * 2 - 1).cuda() for i in range(blocks)]
    ref, got = _session(tag), _session(tag)
    first = torch.empty((3, 5, h16, w16), dtype=torch.bfloat16).pin_memory()
    body = torch.empty((3, 8, h16, w16), dtype=torch.bfloat16).pin_memory()
    for i in range(blocks):
        want = torch.cat([r[0].clone() for r in ref.step(lats[i], lr_up=lrs[i])], dim=1).cpu()
        if i == 2:
            got.capture()
        out = first if i == 0 else body
        st = got.step_host(lats[i], lrs[i], out)
        st.output_ready.synchronize()
        assert torch.equal(out, want), i
    got.sync_host()
    assert_no_device_error()
