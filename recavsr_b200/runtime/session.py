"""Session glue around the DiT layer loop on B200.

TransformerSession.step (recavsr_infer/runtime/transformer.py:279-349) turns
one block of normalized LQ RGB frames plus noise into the next latent block:

  hidden = patch_embedding(noise) + lq_proj.forward_streaming(lq)
           + sr_proj(patch_embedding(recycle))               (:317-328)
  30 x (history -> block -> commit)                          (:330-337)
  norm_out + modulation -> proj_out -> unpatchify            (:338-345)
  result = noise - prediction; recycle = result[:, :, -2:]   (:346-349)

Here every piece runs on the library: the linears (patch embedding as a GEMM
over gathered 1x2x2 patches, the LQ projector's out_proj, sr_proj, proj_out)
on the tcgen05 bf16 GEMM, the residual adds in its epilogue; the LQ
projector's two causal strided Conv3d layers (models/lq_proj.py:44-139) as
im2col (pixel unshuffle fused for the first) + the bf16 GEMM + channel
RMSNorm / SiLU; norm_out + modulation in the LayerNorm row kernel; unpatchify,
`noise - prediction` and the bf16 recycle copy in one kernel. The layer loop is
a LayerStack. Temporal history of the causal convolutions follows
CausalConv3d.forward_streaming's index arithmetic exactly.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import _lib
from .block import HostStep
from .constants import (BODY_LATENT_FRAMES, BODY_RGB_FRAMES, PREFIX_LATENT_FRAMES, PREFIX_RGB_FRAMES,
                        SPATIAL_TOKEN_STRIDE, VAE_SPATIAL_STRIDE)

_EPS = 1e-6
_KT = 4                      # temporal kernel of both causal convolutions (lq_proj.py:51-61)
_UNSHUFFLE = 16              # pixel unshuffle factor (lq_proj.py:168)


_GLUE_WS: dict = {}


def _glue_workspace(device: torch.device) -> torch.Tensor:
    """The glue GEMMs' split-K workspace, one per device (allocated on first
    use, zero-filled; the glue issues its GEMMs in order on one stream)."""
    key = torch.device(device).index
    ws = _GLUE_WS.get(key)
    if ws is None:
        ws = torch.zeros((_lib.library().rc_gemm_split_workspace(),), dtype=torch.uint8, device=device)
        _GLUE_WS[key] = ws
    return ws


def _gemm(a: torch.Tensor, w: torch.Tensor, bias, out: torch.Tensor, epi: int) -> torch.Tensor:
    """out[M, N] (epilogue epi) = a[M, K] @ w[N, K]^T + bias on the tcgen05 bf16
    GEMM (tail split-K through the glue's workspace)."""
    if not a.is_contiguous():
        raise ValueError("GEMM operand rows must be contiguous")
    ws = _glue_workspace(a.device)
    _lib.call("rc_bf16_gemm_ws", a.data_ptr(), w.data_ptr(), _lib.ptr(bias), a.shape[0], w.shape[0],
              a.shape[1], epi, out.data_ptr(), out.stride(0), None, ws.data_ptr(), ws.numel(),
              _lib.stream(a.device))
    return out


@dataclass
class ConvStreamState:
    """Temporal history of one strided causal convolution (lq_proj.py:11-16)."""
    history: torch.Tensor | None = None
    seen_frames: int = 0


def streaming_window(seen: int, chunk: int, stride: int, kernel: int = _KT):
    """(first output endpoint, last endpoint, first needed input frame, outputs)
    of CausalConv3d.forward_streaming (lq_proj.py:84-100, 125)."""
    if chunk <= 0:
        raise ValueError("A streaming convolution chunk cannot be empty.")
    next_end = (seen + stride - 1) // stride * stride
    last_in = seen + chunk - 1
    if next_end > last_in:
        raise ValueError("Streaming LQ chunk is too short to emit the next strided "
                         f"convolution output: seen={seen}, chunk={chunk}.")
    last_end = last_in // stride * stride
    return next_end, last_end, next_end - (kernel - 1), 1 + (last_end - next_end) // stride


def conv_input(x: torch.Tensor, state: ConvStreamState, frame_dim: int, stride: int,
               kernel: int = _KT) -> tuple[torch.Tensor, int]:
    """The frames one streaming causal convolution reads for chunk x (history,
    first frame replicated where the causal window starts before frame 0:
    lq_proj.py:102-122), as one contiguous tensor, and its output count; the
    state keeps the last kernel-1 frames (lq_proj.py:133-135)."""
    chunk = x.shape[frame_dim]
    next_end, last_end, needed, n_out = streaming_window(state.seen_frames, chunk, stride, kernel)
    if state.history is None:
        combined, cstart = x, state.seen_frames
    else:
        h = state.history
        keep = [s for i, s in enumerate(h.shape) if i != frame_dim]
        if keep != [s for i, s in enumerate(x.shape) if i != frame_dim]:
            raise ValueError("Streaming convolution history shape changed.")
        combined = torch.cat((h, x), frame_dim)
        cstart = state.seen_frames - h.shape[frame_dim]
    lo = max(needed, 0) - cstart
    inp = combined.narrow(frame_dim, lo, last_end - cstart + 1 - lo)
    if needed < 0:
        first = combined.narrow(frame_dim, 0, 1)
        reps = [1] * combined.dim()
        reps[frame_dim] = -needed
        inp = torch.cat((first.repeat(*reps), inp), frame_dim)
    length = combined.shape[frame_dim]
    tail = min(kernel - 1, length)
    state.history = combined.narrow(frame_dim, length - tail, tail).clone()
    state.seen_frames += chunk
    return inp.contiguous(), n_out


def _device(device) -> torch.device:
    """A CUDA device with its index ("cuda" -> the current device)."""
    dev = torch.device(device)
    if dev.type == "cuda" and dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    return dev


def _conv_weight(w: torch.Tensor, device) -> torch.Tensor:
    """[cout, cin, kt, kh, kw] -> [cout, kt*kh*kw*cin] bf16 (the im2col column order)."""
    cout = w.shape[0]
    return w.to(device=device, dtype=torch.bfloat16).permute(0, 2, 3, 4, 1).reshape(cout, -1).contiguous()


class LQProjector:
    """LQ4xProj.forward_streaming (models/lq_proj.py:231-246) on B200.

    weights: conv1_w [h1, 768, 4, 3, 3], conv1_b, norm1_w [h1], conv2_w
    [h2, h1, 4, 3, 3], conv2_b, norm2_w [h2], out_w [out, h2], out_b."""

    def __init__(self, weights: dict, device):
        device = _device(device)
        bf = lambda t: t.to(device=device, dtype=torch.bfloat16).reshape(-1).contiguous()
        self.device = device
        self.w1, self.b1 = _conv_weight(weights["conv1_w"], device), bf(weights["conv1_b"])
        self.w2, self.b2 = _conv_weight(weights["conv2_w"], device), bf(weights["conv2_b"])
        self.n1, self.n2 = bf(weights["norm1_w"]), bf(weights["norm2_w"])
        self.wo = weights["out_w"].to(device=device, dtype=torch.bfloat16).contiguous()
        self.bo = bf(weights["out_b"])
        self.h1, self.h2, self.out_dim = self.w1.shape[0], self.w2.shape[0], self.wo.shape[0]
        self.cin = weights["conv1_w"].shape[1]
        if self.cin % (_UNSHUFFLE * _UNSHUFFLE) or self.w1.shape[1] != 36 * self.cin:
            raise ValueError("conv1 must read 16x16-unshuffled RGB with a (4, 3, 3) kernel")
        if self.h1 % 16 or self.h2 % 64 or self.out_dim % 16:
            raise ValueError("LQ projector widths: hidden_dim1 % 16, hidden_dim2 % 64 and out_dim % 16 "
                             "must be 0 (GEMM K and N granules)")

    def create_streaming_state(self):
        return (ConvStreamState(), ConvStreamState())

    def forward_streaming(self, video: torch.Tensor, state, residual: torch.Tensor | None = None):
        """video [1, 3, T, H, W] bf16 on the device. Returns the projected tokens
        [T' * H/32 * W/32, out_dim] bf16, or adds them into `residual` (same
        shape, bf16(residual + tokens)) and returns it."""
        if video.dim() != 5 or video.shape[0] != 1:
            raise ValueError(f"video must have shape [1, C, T, H, W], got {tuple(video.shape)}.")
        _, c, frames, height, width = video.shape
        if c * _UNSHUFFLE * _UNSHUFFLE != self.cin:
            raise ValueError(f"Expected {self.cin // (_UNSHUFFLE * _UNSHUFFLE)} input channels, got {c}.")
        if height % SPATIAL_TOKEN_STRIDE or width % SPATIAL_TOKEN_STRIDE:
            raise ValueError("Input height and width must be divisible by 32, "
                             f"got {(height, width)}.")
        _lib.require_cuda(video, "LQProjector")
        s1, s2 = state
        dev = video.device
        st = _lib.stream(dev)
        # conv1: stride (2, 1, 1) over the 16x16-unshuffled RGB frames
        x1, n1 = conv_input(video[0].to(torch.bfloat16), s1, frame_dim=1, stride=2)
        h1, w1 = height // _UNSHUFFLE, width // _UNSHUFFLE
        tc = x1.shape[1]
        a1 = torch.empty((n1 * h1 * w1, 36 * self.cin), dtype=torch.bfloat16, device=dev)
        _lib.call("rc_conv3d_im2col", x1.data_ptr(), height * width, tc * height * width, width, 0, _UNSHUFFLE,
                  self.cin, tc, h1, w1, 2, 1, n1, a1.data_ptr(), a1.stride(0), st)
        y1 = _gemm(a1, self.w1, self.b1, torch.empty((a1.shape[0], self.h1), dtype=torch.bfloat16, device=dev),
                   _lib.EPI_BIAS)
        del a1
        _lib.call("rc_channel_rmsnorm_silu", y1.data_ptr(), self.h1, y1.shape[0], self.h1, self.n1.data_ptr(),
                  _EPS, y1.data_ptr(), self.h1, st)
        # conv2: stride (2, 2, 2) over conv1's channels-last frames
        x2, n2 = conv_input(y1.view(n1, h1, w1, self.h1), s2, frame_dim=0, stride=2)
        h2, w2 = (h1 - 1) // 2 + 1, (w1 - 1) // 2 + 1
        a2 = torch.empty((n2 * h2 * w2, 36 * self.h1), dtype=torch.bfloat16, device=dev)
        _lib.call("rc_conv3d_im2col", x2.data_ptr(), h1 * w1 * self.h1, 0, w1 * self.h1, self.h1, 0, self.h1,
                  x2.shape[0], h1, w1, 2, 2, n2, a2.data_ptr(), a2.stride(0), st)
        y2 = _gemm(a2, self.w2, self.b2, torch.empty((a2.shape[0], self.h2), dtype=torch.bfloat16, device=dev),
                   _lib.EPI_BIAS)
        del a2
        _lib.call("rc_channel_rmsnorm_silu", y2.data_ptr(), self.h2, y2.shape[0], self.h2, self.n2.data_ptr(),
                  _EPS, y2.data_ptr(), self.h2, st)
        if residual is None:
            out = torch.empty((y2.shape[0], self.out_dim), dtype=torch.bfloat16, device=dev)
            return _gemm(y2, self.wo, self.bo, out, _lib.EPI_BIAS)
        if residual.shape != (y2.shape[0], self.out_dim) or residual.dtype != torch.bfloat16:
            raise ValueError("residual must be [tokens, out_dim] bf16")
        return _gemm(y2, self.wo, self.bo, residual, _lib.EPI_RESIDUAL)


class SessionGlue:
    """The non-layer parts of TransformerSession.step on B200.

    weights: patch_w [dim, C, 1, 2, 2], patch_b, sr_w [dim, dim], sr_b,
    proj_out_w [C*4, dim], proj_out_b, head_shift / head_scale fp32 [dim]
    (scale_shift_table + temb, transformer.py:338-341), and the LQ projector's
    weights (LQProjector)."""

    def __init__(self, weights: dict, device):
        dev = _device(device)
        bf = lambda t: t.to(device=dev, dtype=torch.bfloat16).contiguous()
        self.device = dev
        pw = weights["patch_w"]
        self.dim, self.channels = pw.shape[0], pw.shape[1]
        if tuple(pw.shape[2:]) != (1, 2, 2):
            raise ValueError("patch embedding must be a (1, 2, 2) Conv3d")
        if (self.channels * 4) % 64 or self.dim % 64:
            raise ValueError("latent channels * 4 and the model width must be multiples of 64 "
                             "(GEMM K granule)")
        self.patch_w, self.patch_b = bf(pw.reshape(self.dim, -1)), bf(weights["patch_b"])
        self.sr_w, self.sr_b = bf(weights["sr_w"]), bf(weights["sr_b"])
        self.out_w, self.out_b = bf(weights["proj_out_w"]), bf(weights["proj_out_b"])
        self.shift = weights["head_shift"].to(device=dev, dtype=torch.float32).reshape(-1).contiguous()
        self.scale = weights["head_scale"].to(device=dev, dtype=torch.float32).reshape(-1).contiguous()
        self.lq = LQProjector(weights, dev)

    def _patches(self, x: torch.Tensor) -> torch.Tensor:
        """[1, C, F, h, w] fp32 / bf16 -> patch rows [F*h/2*w/2, C*4] bf16."""
        _, c, f, h, w = x.shape
        x = x.contiguous()
        out = torch.empty((f * (h // 2) * (w // 2), c * 4), dtype=torch.bfloat16, device=x.device)
        _lib.call("rc_patchify", x.data_ptr(), int(x.dtype == torch.bfloat16), f * h * w, h * w, w, c, f, h, w,
                  2, 2, out.data_ptr(), out.stride(0), _lib.stream(x.device))
        return out

    def embed(self, noise: torch.Tensor, lq: torch.Tensor, recycle: torch.Tensor, lq_state) -> torch.Tensor:
        """hidden [tokens, dim] bf16 = patch(noise) + lq_proj(lq) + sr_proj(patch(recycle)),
        summed in the reference's order with a bf16 rounding after each add."""
        hidden = _gemm(self._patches(noise), self.patch_w, self.patch_b, self._new_hidden(noise),
                       _lib.EPI_BIAS)
        self.lq.forward_streaming(lq, lq_state, residual=hidden)
        rec = _gemm(self._patches(recycle), self.patch_w, self.patch_b, self._new_hidden(recycle), _lib.EPI_BIAS)
        return _gemm(rec, self.sr_w, self.sr_b, hidden, _lib.EPI_RESIDUAL)

    def _new_hidden(self, lat: torch.Tensor) -> torch.Tensor:
        _, _, f, h, w = lat.shape
        return torch.empty((f * (h // 2) * (w // 2), self.dim), dtype=torch.bfloat16, device=self.device)

    def head(self, hidden: torch.Tensor, noise: torch.Tensor, recycle_frames: int = BODY_LATENT_FRAMES):
        """(noise - unpatchify(proj_out(norm_out(hidden) * (1 + scale) + shift)),
        its last recycle_frames frames in bf16) -- transformer.py:338-348."""
        n, dim = hidden.shape
        st = _lib.stream(hidden.device)
        normed = torch.empty_like(hidden)
        _lib.call("rc_ln_modulate_quant", hidden.data_ptr(), hidden.stride(0), n, dim, None, None,
                  self.shift.data_ptr(), self.scale.data_ptr(), _EPS, normed.data_ptr(), dim, None, None, 1.0, st)
        pred = _gemm(normed, self.out_w, self.out_b,
                     torch.empty((n, self.out_w.shape[0]), dtype=torch.bfloat16, device=hidden.device),
                     _lib.EPI_BIAS)
        _, c, f, h, w = noise.shape
        noise = noise.contiguous()
        result = torch.empty_like(noise)
        rf = min(recycle_frames, f)
        recycle = torch.empty((1, c, rf, h, w), dtype=torch.bfloat16, device=hidden.device)
        _lib.call("rc_unpatchify_residual", pred.data_ptr(), pred.stride(0), noise.data_ptr(), result.data_ptr(),
                  recycle.data_ptr(), c, f, h, w, 2, 2, rf, st)
        return result, recycle


class StreamingSession:
    """TransformerSession.step (transformer.py:279-349) over a LayerStack and
    SessionGlue: step(lq [1, 3, T, H, W]) -> result [1, C, frames, H/16, W/16]
    fp32; prefix block first (21 RGB -> 6 latent frames), then body blocks
    (8 RGB -> 2 latent frames)."""

    def __init__(self, stack, glue: SessionGlue, height: int, width: int, *, seed: int = 42,
                 graphs: bool = False):
        if height % SPATIAL_TOKEN_STRIDE or width % SPATIAL_TOKEN_STRIDE or min(height, width) < SPATIAL_TOKEN_STRIDE:
            raise ValueError("Transformer geometry must be a positive multiple of 32.")
        self.stack, self.glue, self.height, self.width = stack, glue, height, width
        self.graphs = graphs
        self.generator = torch.Generator(device=glue.device)
        self.reset(seed)

    def reset(self, seed: int = 42) -> None:
        self.stack.reset()
        self.lq_state = self.glue.lq.create_streaming_state()
        self.generator.manual_seed(seed)
        self.latent_offset, self.previous_latents = 0, None

    def step(self, lq: torch.Tensor, *, noise: torch.Tensor | None = None) -> torch.Tensor:
        frames = PREFIX_LATENT_FRAMES if self.latent_offset == 0 else BODY_LATENT_FRAMES
        rgb = PREFIX_RGB_FRAMES if self.latent_offset == 0 else BODY_RGB_FRAMES
        if tuple(lq.shape) != (1, 3, rgb, self.height, self.width):
            raise ValueError(f"Expected LQ block [1,3,{rgb},{self.height},{self.width}].")
        shape = (1, self.glue.channels, frames, self.height // VAE_SPATIAL_STRIDE,
                 self.width // VAE_SPATIAL_STRIDE)
        dev = self.glue.device
        if noise is None:
            noise = torch.randn(shape, generator=self.generator, device=dev, dtype=torch.float32)
        if tuple(noise.shape) != shape or noise.dtype != torch.float32 or noise.device != dev:
            raise ValueError("Explicit noise must match the block in FP32 on the model device.")
        recycle = (torch.zeros(shape, dtype=torch.bfloat16, device=dev) if self.previous_latents is None
                   else self.previous_latents)
        hidden = self.glue.embed(noise, lq.to(device=dev, dtype=torch.bfloat16), recycle, self.lq_state)
        n = hidden.shape[0]
        if self.graphs and frames == BODY_LATENT_FRAMES:
            if n not in self.stack._graphs:
                self.stack.step(hidden, frames)            # eager first body block, then capture
                self.stack.capture(n, frames)
            else:
                self.stack.step(hidden, frames, graphs=True)
        else:
            self.stack.step(hidden, frames)
        result, self.previous_latents = self.glue.head(hidden, noise)
        self.latent_offset += frames
        return result

    def step_host(self, host_lq: torch.Tensor, host_out: torch.Tensor) -> HostStep:
        """step() from pinned host LQ frames to pinned host latents: the
        host-to-device copy of this block's frames and the device-to-host copy
        of its result run on two copy streams (inputs, outputs) with
        double-buffered staging, so they overlap the neighbouring blocks' work:
        the next block's input copy does not queue behind this block's output
        copy, which has to wait for this block's compute.

        Asynchronous: the call returns before either copy has run. host_lq must
        not be rewritten before the returned HostStep's `input_consumed` has
        completed, and host_out holds the latents once `output_ready` has
        completed; sync_host() waits for every copy issued so far."""
        dev = self.glue.device
        if getattr(self, "_copy", None) is None:
            self._copy, self._copy_out, self._stage = torch.cuda.Stream(dev), torch.cuda.Stream(dev), {}
        comp, cs, co = torch.cuda.current_stream(dev), self._copy, self._copy_out
        key = tuple(host_lq.shape)
        if key not in self._stage:
            st = {"lq": [torch.empty(key, dtype=torch.bfloat16, device=dev) for _ in range(2)], "k": 0,
                  "ready": [torch.cuda.Event() for _ in range(2)],
                  "consumed": [torch.cuda.Event() for _ in range(2)]}
            for e in st["consumed"]:
                e.record(comp)
            self._stage[key] = st
        st = self._stage[key]
        k = st["k"] & 1
        handle = HostStep(torch.cuda.Event(), torch.cuda.Event())
        with torch.cuda.stream(cs):
            cs.wait_event(st["consumed"][k])          # the block two steps back has read this buffer
            st["lq"][k].copy_(host_lq, non_blocking=True)
            st["ready"][k].record(cs)
            handle.input_consumed.record(cs)
        comp.wait_event(st["ready"][k])
        result = self.step(st["lq"][k])
        st["consumed"][k].record(comp)
        done = torch.cuda.Event()
        done.record(comp)
        with torch.cuda.stream(co):
            co.wait_event(done)
            host_out.copy_(result, non_blocking=True)
            handle.output_ready.record(co)
        result.record_stream(co)
        st["k"] += 1
        return handle

    def sync_host(self) -> None:
        """Block the host until every step_host copy issued so far has run; the
        current stream also waits for them."""
        if getattr(self, "_copy", None) is not None:
            for s in (self._copy, self._copy_out):
                torch.cuda.current_stream(self.glue.device).wait_stream(s)
                s.synchronize()
