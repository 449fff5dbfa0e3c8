"""FlashDecoder's streaming decode on B200 (drop-in for
recavsr_infer/runtime/flashdecoder.py:54-175 `FlashDecoderSession` and the
`FlashDecoder.decode_step` it drives, models/flashdecoder/flashdecoder_wan22.py:759-874).

`DecoderSession(params, height=..., width=..., mean=..., std=..., ...)` holds the
decoder's weights (the reference's state-dict names, fp32 master values cast to
bf16 once, as bf16 autocast casts them per call) and, per layer, its K / V
cache as frame rings. `step(latents, lr_up=...)` yields the RGB chunks of
`FlashDecoderSession.step`: one frame for the first latent frame of a stream,
then four per latent frame, bf16 in [-1, 1].

Per decode step (one latent frame): the LR stem (pixel unshuffle -> linear ->
grouping), the latent projection, 12 backbone blocks over the frame's n
tokens (1 current frame, a 2-frame window), the temporal projection into 4
frames, 2 refinement blocks over 4n tokens (an 8-frame window), the spatial
projection and the pixel shuffle. A block is RMSNorm -> fused q|k|v GEMM ->
K / V RMSNorm into the rings -> 3D RoPE of q and of the window's keys ->
rc_local_gqa_attention -> output GEMM (+ residual) -> RMSNorm -> fused
gate|up GEMM with the SwiGLU epilogue -> down GEMM (+ residual): nine launches, all of
this library's kernels. Steady-state steps are replayed from CUDA graphs
(capture(): one per parity of the ring positions, which repeat every two steps).
"""
from __future__ import annotations

import ctypes as C
import math

import numpy as np
import torch

from .. import _lib

EPI_BIAS, EPI_RESIDUAL, EPI_SWIGLU = 0, 2, 4
HEAD_DIM = 64


def _dev(x, device, dtype):
    if isinstance(x, np.ndarray):
        x = torch.from_numpy(x)
    return x.detach().to(device=device, dtype=dtype).contiguous()


def _pad_k(w: torch.Tensor, k: int) -> torch.Tensor:
    """[N, K0] -> [N, k] with zero columns (the GEMM's K granule is 64)."""
    out = torch.zeros((w.shape[0], k), dtype=w.dtype, device=w.device)
    out[:, :w.shape[1]] = w
    return out


def _swiglu_rows(gate, up, device) -> torch.Tensor:
    """Gate and up rows (or biases) interleaved in blocks of 8, the layout of
    the GEMM's SwiGLU epilogue: [g0..g7, u0..u7, g8..g15, u8..u15, ...]."""
    g, u = torch.as_tensor(gate), torch.as_tensor(up)
    n = g.shape[0]
    both = torch.stack([g.reshape(n // 8, 8, *g.shape[1:]), u.reshape(n // 8, 8, *u.shape[1:])], 1)
    return _dev(both.reshape(2 * n, *g.shape[1:]), device, torch.bfloat16)


def rope_tables(height: int, width: int, max_t: int, device, theta: float = 10000.0, dims=(16, 24, 24)):
    """flashdecoder_wan22.py:158-224 as one fp32 buffer: cos_t [max_t, 8] |
    sin_t | cos_h [height, 12] | sin_h | cos_w [width, 12] | sin_w, each pair's
    angle computed as the reference computes it (positions.float() * inv_freq
    on the device, inv_freq built on the host)."""
    parts = []
    for n, d in zip((max_t, height, width), dims):
        inv = (1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.float32) / d))).to(device)
        ang = torch.arange(n, device=device).to(torch.float32).unsqueeze(-1) * inv
        parts += [torch.cos(ang).reshape(-1), torch.sin(ang).reshape(-1)]
    return torch.cat(parts).contiguous()


class _Stack:
    """One _StreamingTransformer (flashdecoder_wan22.py:380-497): its blocks'
    weights, its frame rings and the count of frames written."""

    def __init__(self, owner, prefix, depth, max_frames, cur):
        d, dev = owner, owner.device
        self.max_frames, self.cur, self.total = max_frames, cur, 0
        self.layers = []
        ring_tokens = max_frames * d.n
        for i in range(depth):
            pre = f"{prefix}.blocks.{i}."
            a = pre + "attention."
            w = d.params
            self.layers.append(dict(
                attn_w=_dev(w[pre + "attention_norm.weight"], dev, torch.float32),
                ffn_w=_dev(w[pre + "feed_forward_norm.weight"], dev, torch.float32),
                qkv_w=_dev(torch.cat([torch.as_tensor(w[a + x + ".weight"]) for x in ("query", "key", "value")]),
                           dev, torch.bfloat16),
                qkv_b=_dev(torch.cat([torch.as_tensor(w[a + x + ".bias"]) for x in ("query", "key", "value")]),
                           dev, torch.bfloat16),
                kn=_dev(w[a + "key_norm.weight"], dev, torch.float32),
                vn=_dev(w[a + "value_norm.weight"], dev, torch.float32),
                o_w=_dev(w[a + "output.weight"], dev, torch.bfloat16),
                o_b=_dev(w[a + "output.bias"], dev, torch.bfloat16),
                gu_w=_swiglu_rows(w[pre + "feed_forward.gate.weight"], w[pre + "feed_forward.up.weight"],
                                  dev),
                gu_b=_swiglu_rows(w[pre + "feed_forward.gate.bias"], w[pre + "feed_forward.up.bias"], dev),
                d_w=_dev(w[pre + "feed_forward.down.weight"], dev, torch.bfloat16),
                d_b=_dev(w[pre + "feed_forward.down.bias"], dev, torch.bfloat16),
                k_ring=torch.zeros((d.hk, ring_tokens, HEAD_DIM), dtype=torch.float32, device=dev),
                v_ring=torch.zeros((d.hk, ring_tokens, HEAD_DIM), dtype=torch.bfloat16, device=dev)))
        self.ring_head = ring_tokens * HEAD_DIM

    def positions(self):
        """(prev, nf, slot0, slot_w) of the next step: the trimmed cache keeps
        the last max_frames - cur frames written (flashdecoder_wan22.py:428-437),
        key frame t lives in ring slot (slot0 + t) % max_frames and the current
        frames are written from slot slot_w on."""
        keep = self.max_frames - self.cur
        prev = min(self.total, keep)
        return prev, prev + self.cur, (self.total - prev) % self.max_frames, self.total % self.max_frames


class DecoderSession:
    """B200 FlashDecoderSession for one stream at a fixed latent grid (B = 1).

    params: the FlashDecoder state dict (tensors or arrays, reference names);
    mean / std: the 48 latent normalization values (vae_config latents_mean /
    latents_std); height / width: the latent grid (output 16x that)."""

    def __init__(self, params, *, height, width, mean, std, dim=512, num_heads=8, num_kv_groups=2, depth=12,
                 refinement_depth=2, mlp_ratio=4.0, window=(24, 24), window_size=2, eps=1e-5,
                 rope_theta=10000.0, device=None):
        from .flashdecoder import validate_spatial_window
        self.window = validate_spatial_window(tuple(window))
        if dim % num_heads or num_heads % num_kv_groups or dim // num_heads != HEAD_DIM:
            raise ValueError("FlashDecoder on B200 needs 64-dimensional heads and whole KV groups.")
        self.device = torch.device(device or "cuda")
        if self.device.type != "cuda":
            raise ValueError("DecoderSession runs on a CUDA device.")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.h, self.w, self.n = height, width, height * width
        self.dim, self.hq, self.hk, self.eps = dim, num_heads, num_kv_groups, float(eps)
        self.hidden = int(dim * mlp_ratio)
        if self.hidden % 64 or dim % 64:
            raise ValueError("dim and the SwiGLU width must be multiples of 64.")
        self.params = params
        dev, n, bf = self.device, self.n, torch.bfloat16
        w = params
        self.lat_w = _pad_k(_dev(w["latent_projection.weight"], dev, bf), 64)
        self.lat_b = _dev(w["latent_projection.bias"], dev, bf)
        self.stem_w = _dev(w["lr_stem.weight"], dev, bf)
        self.stem_b = _dev(w["lr_stem.bias"], dev, bf)
        self.early_w = _dev(w["lr_early_projection.weight"], dev, bf)
        self.late_w = _pad_k(_dev(w["lr_late_projection.weight"], dev, bf), 64)
        self.tp_w = _dev(w["temporal_projection.weight"], dev, bf)
        self.tp_b = _dev(w["temporal_projection.bias"], dev, bf)
        self.s0_w = _dev(w["spatial_projection.0.weight"], dev, bf)
        self.s0_b = _dev(w["spatial_projection.0.bias"], dev, bf)
        self.s2_w = _dev(w["spatial_projection.2.weight"], dev, bf)
        self.s2_b = _dev(w["spatial_projection.2.bias"], dev, bf)
        self.mean = _dev(mean, dev, bf)
        self.std = _dev(std, dev, bf)
        self.backbone = _Stack(self, "backbone", depth, window_size, 1)
        self.refinement = _Stack(self, "temporal_refinement", refinement_depth, 4 * window_size, 4)
        self.tables = rope_tables(height, width, 4 * window_size, dev, rope_theta)
        self.max_t = 4 * window_size
        qkv_n = dim + 2 * self.hk * HEAD_DIM
        t4 = 4 * n
        e = lambda *s, dt=bf: torch.empty(s, dtype=dt, device=dev)
        self.x, self.hr, self.xn = e(n, dim), e(t4, dim), e(t4, dim)
        self.qkv, self.q_rot, self.att = e(t4, qkv_n), e(t4, dim), e(t4, dim)
        self.act = e(t4, self.hidden)
        self.s2 = e(t4, 768)
        self.lat_in, self.unsh, self.feats = e(n, 64), e(t4, 768), e(t4, 48)
        self.grouped, self.late_in = e(n, 192), e(t4, 64)
        kv_tokens = 4 * window_size * n
        self.kbuf, self.vbuf = e(self.hk, kv_tokens, HEAD_DIM), e(self.hk, kv_tokens, HEAD_DIM)
        # RGB output per frame parity: a frame's copy to the host can overlap the
        # next frame's decode (step_host).
        self.rgb_bufs = [e(3, 4, 16 * height, 16 * width), e(3, 4, 16 * height, 16 * width)]
        self._copied = [None, None]         # copy-finished event per buffer
        self._copy = None
        self.lat_stage = e(48, n, dt=torch.float32)
        self.lr_stage = e(3, 4, 16 * height, 16 * width, dt=torch.float32)
        self.frame_index = 0
        self.graphs = {}

    # ------------------------------------------------------------------ pieces
    def _gemm(self, a, w, b, m, n, k, epi, out, ldo):
        _lib.call("rc_bf16_gemm", a.data_ptr(), w.data_ptr(), None if b is None else b.data_ptr(), m, n, k, epi,
                  out.data_ptr(), ldo, None, self.stream)

    def _rms(self, x, weight, rows, out):
        _lib.call("rc_layer_norm", x.data_ptr(), 1, self.dim, rows, self.dim, weight.data_ptr(), None, self.eps, 1,
                  out.data_ptr(), self.dim, self.stream)

    def _stack(self, st: _Stack, x: torch.Tensor, positions):
        prev, nf, slot0, slot_w = positions
        cur, n, dim = st.cur, self.n, self.dim
        tokens = cur * n
        qkv_n = self.qkv.shape[1]
        q_str = (C.c_longlong * 9)(tokens * dim, HEAD_DIM, dim,
                                   self.hk * nf * n * HEAD_DIM, nf * n * HEAD_DIM, HEAD_DIM,
                                   self.hk * nf * n * HEAD_DIM, nf * n * HEAD_DIM, HEAD_DIM)
        o_str = (C.c_longlong * 3)(tokens * dim, HEAD_DIM, dim)
        for L in st.layers:
            self._rms(x, L["attn_w"], tokens, self.xn)
            self._gemm(self.xn, L["qkv_w"], L["qkv_b"], tokens, qkv_n, dim, EPI_BIAS, self.qkv, qkv_n)
            _lib.call("rc_fd_kv_norm", self.qkv.data_ptr(), qkv_n, tokens, dim, self.hk, L["kn"].data_ptr(),
                      L["vn"].data_ptr(), self.eps, L["k_ring"].data_ptr(), L["v_ring"].data_ptr(), st.ring_head,
                      slot_w * n, self.stream)
            _lib.call("rc_fd_rope_gather", self.qkv.data_ptr(), qkv_n, self.hq, self.hk, cur, prev, nf, slot0,
                      st.max_frames, self.h, self.w, L["k_ring"].data_ptr(), L["v_ring"].data_ptr(), st.ring_head,
                      self.tables.data_ptr(), self.max_t, self.q_rot.data_ptr(), self.kbuf.data_ptr(),
                      self.vbuf.data_ptr(), self.stream)
            _lib.call("rc_local_gqa_attention", self.q_rot.data_ptr(), self.kbuf.data_ptr(), self.vbuf.data_ptr(),
                      q_str, 1, self.hq, self.hk, cur, nf, self.h, self.w, HEAD_DIM, self.window[0],
                      self.window[1], cur, st.max_frames // cur, 0, self.att.data_ptr(), o_str, self.stream)
            self._gemm(self.att, L["o_w"], L["o_b"], tokens, dim, dim, EPI_RESIDUAL, x, dim)
            self._rms(x, L["ffn_w"], tokens, self.xn)
            # gate | up GEMM with the SwiGLU epilogue: act = bf16(bf16(silu(gate)) * up)
            self._gemm(self.xn, L["gu_w"], L["gu_b"], tokens, 2 * self.hidden, dim, EPI_SWIGLU, self.act,
                       self.hidden)
            self._gemm(self.act, L["d_w"], L["d_b"], tokens, dim, self.hidden, EPI_RESIDUAL, x, dim)
        st.total += cur

    def _decode(self, first: bool, bpos, rpos, rgb):
        """One decode step from the staged latent frame (lat_stage) and LR
        frames (lr_stage[:, :F]) into rgb[:, :F]."""
        n, dim, h, w = self.n, self.dim, self.h, self.w
        f_lr = 1 if first else 4
        _lib.call("rc_fd_latent_in", self.lat_stage.data_ptr(), n, n, self.mean.data_ptr(), self.std.data_ptr(),
                  self.lat_in.data_ptr(), self.stream)
        s = self.lr_stage
        strides = (C.c_longlong * 3)(s.stride(0), s.stride(1), s.stride(2))
        _lib.call("rc_fd_lr_unshuffle", s.data_ptr(), 0, strides, f_lr, h, w, self.unsh.data_ptr(), self.stream)
        self._gemm(self.unsh, self.stem_w, self.stem_b, f_lr * n, 48, 768, EPI_BIAS, self.feats, 48)
        _lib.call("rc_fd_lr_group", self.feats.data_ptr(), 48, n, int(first), self.grouped.data_ptr(),
                  self.late_in.data_ptr(), self.stream)
        self._gemm(self.grouped, self.early_w, None, n, dim, 192, EPI_BIAS, self.x, dim)
        self._gemm(self.lat_in, self.lat_w, self.lat_b, n, dim, 64, EPI_RESIDUAL, self.x, dim)
        self._stack(self.backbone, self.x, bpos)
        self._gemm(self.late_in, self.late_w, None, 4 * n, dim, 64, EPI_BIAS, self.hr, dim)
        for t in range(4):
            self._gemm(self.x, self.tp_w[t * dim:(t + 1) * dim], self.tp_b[t * dim:(t + 1) * dim], n, dim, dim,
                       EPI_RESIDUAL, self.hr[t * n:(t + 1) * n], dim)
        self._stack(self.refinement, self.hr, rpos)
        self._gemm(self.hr, self.s0_w, self.s0_b, 4 * n, self.hidden, dim, EPI_BIAS, self.act, self.hidden)
        _lib.call("rc_fd_silu", self.act.data_ptr(), 4 * n, self.hidden, 1, None, self.stream)
        self._gemm(self.act, self.s2_w, self.s2_b, 4 * n, 768, self.hidden, EPI_BIAS, self.s2, 768)
        _lib.call("rc_fd_pixel_shuffle", self.s2.data_ptr(), 768, 3 if first else 0, f_lr, 4, h, w,
                  rgb.data_ptr(), self.stream)

    # -------------------------------------------------------------- public API
    @property
    def stream(self):
        return torch.cuda.current_stream(self.device).cuda_stream

    def reset(self):
        """Start a new stream (runtime/flashdecoder.py:99-102); captured graphs are kept."""
        self.frame_index = 0
        for st in (self.backbone, self.refinement):
            st.total = 0

    def _key(self):
        """Graph key of the next step: the first step, or the parity of a
        steady-state step (ring positions repeat every two steps)."""
        bp, rp = self.backbone.positions(), self.refinement.positions()
        steady = bp[0] == self.backbone.max_frames - 1 and rp[0] == self.refinement.max_frames - 4
        return ("steady", bp, rp) if steady else None

    def decode_frame(self, latent: torch.Tensor, lr_up: torch.Tensor) -> torch.Tensor:
        """One latent frame: latent [48, h, w] (normalized, as the DiT emits it),
        lr_up [3, F, 16h, 16w] (F = 1 on the first frame of a stream, else 4) ->
        rgb [3, F, 16h, 16w] bf16 in [-1, 1] (a view of an internal buffer,
        valid until the next call)."""
        first = self.frame_index == 0
        f_lr = 1 if first else 4
        if tuple(latent.shape) != (48, self.h, self.w) or tuple(lr_up.shape) != (3, f_lr, 16 * self.h, 16 * self.w):
            raise ValueError("Latent frame or lr_up does not match the session geometry.")
        parity = self.frame_index % 2
        rgb = self.rgb_bufs[parity]
        with torch.cuda.device(self.device):
            if self._copied[parity] is not None:       # the buffer's previous frame has reached the host
                torch.cuda.current_stream(self.device).wait_event(self._copied[parity])
            self.lat_stage.copy_(latent.reshape(48, self.n), non_blocking=True)
            self.lr_stage[:, :f_lr].copy_(lr_up, non_blocking=True)
            bpos, rpos = self.backbone.positions(), self.refinement.positions()
            key = None if first else self._key()
            g = self.graphs.get(key) if key is not None else None
            if g is not None:
                g.replay()
                self.backbone.total += 1
                self.refinement.total += 4
            else:
                self._decode(first, bpos, rpos, rgb)
        self.frame_index += 1
        return rgb[:, :f_lr]

    def capture(self):
        """Record the two steady-state steps (one per ring parity) as CUDA
        graphs, replayed by later decode_frame calls. Needs a stream past its
        first two latent frames (the windows are full). Capturing runs no
        kernel; the frame counters are restored afterwards."""
        if self.frame_index < 2:
            raise RuntimeError("capture() needs a stream past its first two latent frames.")
        saved = (self.backbone.total, self.refinement.total)
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.device(self.device), torch.cuda.stream(side):
            for i in range(2):
                key = self._key()
                bpos, rpos = self.backbone.positions(), self.refinement.positions()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=side):
                    self._decode(False, bpos, rpos, self.rgb_bufs[(self.frame_index + i) % 2])
                self.graphs[key] = g        # _decode advanced the stacks' frame counters
        torch.cuda.current_stream(self.device).wait_stream(side)
        self.backbone.total, self.refinement.total = saved

    def step(self, latents: torch.Tensor, *, lr_up: torch.Tensor):
        """runtime/flashdecoder.py:140-175: normalized latents [1, 48, T, h, w]
        and the aligned target-resolution LR frames lr_up [1, 3, F, 16h, 16w]
        (F = 4T, minus 3 on a stream's first block) -> yields one RGB chunk
        [1, 3, 1 | 4, 16h, 16w] (bf16, [-1, 1]) per latent frame."""
        if latents.ndim != 5 or latents.shape[1] != 48 or min(latents.shape) < 1:
            raise ValueError("FlashDecoder expects nonempty [B,48,T,H,W] latents.")
        if latents.shape[0] != 1 or tuple(latents.shape[3:]) != (self.h, self.w):
            raise ValueError("This session decodes one stream at its latent grid.")
        expected = 4 * latents.shape[2] - (3 if self.frame_index == 0 else 0)
        if lr_up is None or tuple(lr_up.shape) != (1, 3, expected, 16 * self.h, 16 * self.w):
            raise ValueError(f"lr_up must have target-resolution shape {(1, 3, expected, 16 * self.h, 16 * self.w)}.")
        offset = 0
        for i in range(latents.shape[2]):
            take = 1 if self.frame_index == 0 else 4
            rgb = self.decode_frame(latents[0, :, i], lr_up[0, :, offset:offset + take])
            offset += take
            yield rgb.unsqueeze(0)

    def step_host(self, latents: torch.Tensor, lr_up: torch.Tensor, host_out: torch.Tensor):
        """step() into pinned host memory: host_out [3, F, 16h, 16w] bf16 (F =
        4T, minus 3 on a stream's first block) receives the block's RGB frames.
        Each frame's device-to-host copy runs on a copy stream and overlaps the
        next frame's decode (the two frame parities have their own RGB buffer).
        Asynchronous: returns a HostStep whose `input_consumed` completes once
        latents / lr_up have been read and `output_ready` once host_out holds
        every frame of the block; sync_host() waits for every copy issued."""
        from .block import HostStep
        if not host_out.is_pinned() or host_out.dtype != torch.bfloat16:
            raise ValueError("host_out must be pinned bf16 memory.")
        expected = 4 * latents.shape[2] - (3 if self.frame_index == 0 else 0)
        if tuple(host_out.shape) != (3, expected, 16 * self.h, 16 * self.w):
            raise ValueError(f"host_out must have shape {(3, expected, 16 * self.h, 16 * self.w)}.")
        if self._copy is None:
            self._copy = torch.cuda.Stream(self.device)
        compute = torch.cuda.current_stream(self.device)
        off = 0
        for chunk in self.step(latents, lr_up=lr_up):
            f = chunk.shape[2]
            parity = (self.frame_index - 1) % 2
            decoded = torch.cuda.Event()
            decoded.record(compute)
            self._copy.wait_event(decoded)
            with torch.cuda.stream(self._copy):
                # per channel: each channel's frame range is contiguous on both
                # sides, so every copy is one asynchronous DMA (a strided pinned
                # destination would be staged through a synchronous copy)
                for c in range(3):
                    host_out[c, off:off + f].copy_(chunk[0, c], non_blocking=True)
            done = torch.cuda.Event()
            done.record(self._copy)
            self._copied[parity] = done
            off += f
        consumed = torch.cuda.Event()
        consumed.record(compute)
        return HostStep(input_consumed=consumed, output_ready=self._copied[(self.frame_index - 1) % 2])

    def sync_host(self):
        """Block the host until every copy step_host issued has finished."""
        if self._copy is not None:
            self._copy.synchronize()

    @classmethod
    def from_module(cls, model, *, height, width, mean, std, device=None):
        """From a reference FlashDecoder module (its state dict and sizes)."""
        return cls({k: v.float() for k, v in model.state_dict().items()}, height=height, width=width, mean=mean,
                   std=std, dim=model.dim, num_heads=model.num_heads, num_kv_groups=model.num_kv_groups,
                   depth=model.depth, refinement_depth=model.refinement_depth,
                   mlp_ratio=model.backbone.blocks[0].feed_forward.gate.out_features / model.dim,
                   window=model.spatial_window_size, window_size=model.window_size, device=device)


def random_params(device, seed=0, *, dim=512, hidden=2048, depth=12, refinement_depth=2, kv_dim=128):
    """Random-init FlashDecoder weights with the reference's state-dict names
    (for benchmarks and profiling; the released variant's sizes by default):
    linear weights N(0, 1/fan_in), biases N(0, 0.02), norm weights 1 + N(0, 0.1)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    p = {}

    def lin(name, n, k, bias=True):
        p[name + ".weight"] = torch.randn(n, k, generator=g, device=device) / k ** 0.5
        if bias:
            p[name + ".bias"] = torch.randn(n, generator=g, device=device) * 0.02

    def norm(name, n):
        p[name + ".weight"] = 1 + torch.randn(n, generator=g, device=device) * 0.1

    for prefix, n_blocks in (("backbone", depth), ("temporal_refinement", refinement_depth)):
        for i in range(n_blocks):
            b = f"{prefix}.blocks.{i}."
            norm(b + "attention_norm", dim)
            for name, n in (("query", dim), ("key", kv_dim), ("value", kv_dim), ("output", dim)):
                lin(b + "attention." + name, n, dim)
            norm(b + "attention.key_norm", HEAD_DIM)
            norm(b + "attention.value_norm", HEAD_DIM)
            norm(b + "feed_forward_norm", dim)
            lin(b + "feed_forward.gate", hidden, dim)
            lin(b + "feed_forward.up", hidden, dim)
            lin(b + "feed_forward.down", dim, hidden)
    lin("latent_projection", dim, 48)
    lin("temporal_projection", 4 * dim, dim)
    lin("spatial_projection.0", hidden, dim)
    lin("spatial_projection.2", 768, hidden)
    lin("lr_stem", 48, 768)
    lin("lr_early_projection", dim, 192, bias=False)
    lin("lr_late_projection", dim, 48, bias=False)
    return p

