"""Fused DiT block and layer loop on B200.

``FusedBlock`` computes what recavsr_infer/runtime/transformer.py:81-134
(PreparedBlock.forward with NVFP4 linears) computes, with fewer passes:

  LN1+AdaLN -> NVFP4 codes (one quantization shared by q, k and v)
  one QKV GEMM (N = 3*dim, bias)             [the reference runs 3 GEMMs + 3 quantizers]
  RMSNorm(q), RMSNorm(k) + spatial RoPE      (one kernel, both tensors)
  routed attention (temporal RoPE, cache planes read in place via slot ids),
      output quantized to NVFP4 in its epilogue -> o-proj GEMM, epilogue h = h + y * gate
  LN2(affine) -> NVFP4 -> cross-q GEMM -> RMSNorm -> cross attention (512 keys),
      NVFP4 epilogue -> cross-o GEMM, epilogue h = h + y
  LN3+AdaLN -> NVFP4 -> ffn_up GEMM, epilogue GELU(tanh) -> NVFP4 codes for ffn_down
  ffn_down GEMM, epilogue h = h + y * cgate
All intermediate roundings (bf16 outputs of every linear, of the norms and of
GELU) happen where the reference rounds.

``LayerStack`` is the 30-layer loop of TransformerSession.step
(transformer.py:311-318): routing per layer with the reference's
FixedKVCache bookkeeping, attention over the routed planes, KV commit. Its
routing metadata (slot ids, positions, commit plans) lives in one device
table, so a whole body block can be captured once as a CUDA graph and
replayed while the router state advances.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from .. import _lib
from .cache import FixedKVCache
from .constants import DEFAULT_SPATIAL_WINDOW
from .ops import quantize as nvfp4_quantize
from .ops import scale_numel

_EPS = 1e-6


def _bf16_linear(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None) -> torch.Tensor:
    """bf16 nn.Linear on the tcgen05 GEMM (used for the cross K/V precompute)."""
    m = x.reshape(-1, x.shape[-1]).contiguous()
    out = torch.empty((m.shape[0], w.shape[0]), dtype=torch.bfloat16, device=x.device)
    _lib.call("rc_bf16_gemm", m.data_ptr(), w.contiguous().data_ptr(), _lib.ptr(b), m.shape[0],
              w.shape[0], m.shape[1], _lib.EPI_BIAS, out.data_ptr(), out.stride(0), None,
              _lib.stream(x.device))
    return out.reshape(*x.shape[:-1], w.shape[0])


def _rms(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    from .ops import rms_norm_rope
    return rms_norm_rope(x, w, _EPS)


def block_weights_from_module(block, conditioning) -> dict:
    """Extract the tensors FusedBlock needs from a block with the reference's
    module layout (models/transformer_wan.py:786-822) and the streaming
    conditioning (timestep projection, encoder states)."""
    a1, a2 = block.attn1, block.attn2
    w = {
        "q_w": a1.to_q.weight, "q_b": a1.to_q.bias, "k_w": a1.to_k.weight, "k_b": a1.to_k.bias,
        "v_w": a1.to_v.weight, "v_b": a1.to_v.bias, "o_w": a1.to_out[0].weight, "o_b": a1.to_out[0].bias,
        "cq_w": a2.to_q.weight, "cq_b": a2.to_q.bias, "ck_w": a2.to_k.weight, "ck_b": a2.to_k.bias,
        "cv_w": a2.to_v.weight, "cv_b": a2.to_v.bias, "co_w": a2.to_out[0].weight, "co_b": a2.to_out[0].bias,
        "up_w": block.ffn.net[0].proj.weight, "up_b": block.ffn.net[0].proj.bias,
        "down_w": block.ffn.net[2].weight, "down_b": block.ffn.net[2].bias,
        "norm_q": a1.norm_q.weight, "norm_k": a1.norm_k.weight,
        "cnorm_q": a2.norm_q.weight, "cnorm_k": a2.norm_k.weight,
        "norm2_w": block.norm2.weight, "norm2_b": block.norm2.bias,
        "scale_shift_table": block.scale_shift_table,
        "timestep_proj": conditioning.timestep_proj,
        "encoder": conditioning.encoder_hidden_states,
        "heads": a1.heads,
    }
    return {k: (v.detach() if isinstance(v, torch.Tensor) else v) for k, v in w.items()}


@dataclass
class HostStep:
    """Events of one step_host call: `input_consumed` completes once the
    pinned input buffer has been copied to the device (the caller may then
    refill it), `output_ready` once the result has reached the pinned output
    buffer. Wait with .synchronize() or test with .query()."""
    input_consumed: torch.cuda.Event
    output_ready: torch.cuda.Event


@dataclass
class _Quantized:
    codes: torch.Tensor
    scales: torch.Tensor
    bias: torch.Tensor | None
    n: int
    k: int


class FusedBlock(torch.nn.Module):
    """B200 PreparedBlock with NVFP4 linears (see module docstring)."""

    def __init__(self, weights: dict, height: int, width: int, rope_tables: dict, *,
                 window=DEFAULT_SPATIAL_WINDOW):
        super().__init__()
        dev = weights["q_w"].device
        self.device = dev
        self.height, self.width = height, width
        self.window = tuple(window)
        self.heads = int(weights["heads"])
        self.dim = weights["q_w"].shape[1]
        self.head_dim = self.dim // self.heads
        self.ffn = weights["up_w"].shape[0]
        bf = lambda t: None if t is None else t.to(device=dev, dtype=torch.bfloat16).contiguous()
        modulation = (weights["scale_shift_table"].reshape(1, 6, self.dim).float()
                      + weights["timestep_proj"].reshape(1, 6, self.dim).float())
        self.modulation = modulation.reshape(6, self.dim).to(dev).contiguous()
        # Cross K/V precomputed once with the bf16 linears, before quantization
        # (transformer.py:52-56 runs before quantize_block_linears).
        enc = bf(weights["encoder"])
        ck = _bf16_linear(enc, bf(weights["ck_w"]), bf(weights["ck_b"]))
        self.cross_k = _rms(ck, bf(weights["cnorm_k"])).reshape(-1, self.heads, self.head_dim).contiguous()
        self.cross_v = _bf16_linear(enc, bf(weights["cv_w"]), bf(weights["cv_b"])).reshape(
            -1, self.heads, self.head_dim).contiguous()

        def quant(wname, bname):
            w = bf(weights[wname])
            codes, scales = nvfp4_quantize(w)
            return _Quantized(codes, scales, bf(weights[bname]), w.shape[0], w.shape[1])

        wqkv = torch.cat([bf(weights["q_w"]), bf(weights["k_w"]), bf(weights["v_w"])], 0)
        qkv_codes, qkv_scales = nvfp4_quantize(wqkv)
        self.qkv = _Quantized(qkv_codes, qkv_scales,
                              torch.cat([bf(weights["q_b"]), bf(weights["k_b"]), bf(weights["v_b"])]),
                              wqkv.shape[0], wqkv.shape[1])
        del wqkv
        self.o = quant("o_w", "o_b")
        self.cq = quant("cq_w", "cq_b")
        self.co = quant("co_w", "co_b")
        self.up = quant("up_w", "up_b")
        self.down = quant("down_w", "down_b")
        self.norm_q, self.norm_k = bf(weights["norm_q"]), bf(weights["norm_k"])
        self.cnorm_q = bf(weights["cnorm_q"])
        self.norm2_w, self.norm2_b = bf(weights["norm2_w"]), bf(weights["norm2_b"])
        self.tables = rope_tables
        self.local = height > self.window[0] or width > self.window[1]

    # ------------------------------------------------------------------ api
    def forward(self, hidden, past_key, past_value, slots, past_positions, query_positions):
        """PreparedBlock.forward signature: returns (hidden, k, v) without
        modifying the caller's hidden state."""
        n = hidden.shape[1]
        ws = Workspace(self, n)
        h = hidden.reshape(n, self.dim).contiguous().clone()
        self.run(h, ws, past_key, past_value, slots, past_positions, query_positions)
        k = ws.k_rot.reshape(1, n, self.heads, self.head_dim).clone()
        v = ws.qkv[:, 2 * self.dim:].reshape(1, n, self.heads, self.head_dim).clone()
        return h.reshape(1, n, self.dim), k, v

    def run(self, h, ws, past_key, past_value, slots, past_positions, query_positions):
        """In-place layer on h [N, dim]; leaves k (ws.k_rot) and v (ws.qkv) for the commit."""
        lib = _lib.library()
        st = _lib.stream(h.device)
        self.pre_attention(lib, h, ws, st)
        # 4. routed attention, output NVFP4-quantized in its epilogue
        self._attention(lib, ws, past_key, past_value, slots, past_positions, query_positions,
                        h.shape[0], st, quantized=True)
        self.post_attention(lib, h, ws, st)

    def pre_attention(self, lib, h, ws, st, spatial=None):
        """Steps 1-3 of the layer on h [N, dim]: LN1 + AdaLN -> NVFP4, the fused
        QKV GEMM (ws.qkv), RMSNorm + spatial RoPE of q and k (ws.q_rot, ws.k_rot).
        spatial = (cos, sin, span) replaces the block's own spatial tables (a
        token shard passes the rows of its own tokens with span = N)."""
        n, dim = h.shape
        mod = self.modulation
        chk = _lib.check
        if spatial is None:
            spatial = (self.tables["spatial_cos"], self.tables["spatial_sin"], self.height * self.width)
        scos, ssin, span = spatial
        # 1. LN1 + AdaLN -> NVFP4
        chk(lib.rc_ln_modulate_quant(h.data_ptr(), dim, n, dim, None, None, mod[0].data_ptr(),
                                     mod[1].data_ptr(), _EPS, None, 0, ws.a_codes.data_ptr(),
                                     ws.a_scales.data_ptr(), 1.0, st), "ln1")
        # 2. fused QKV
        self._gemm(lib, ws, ws.a_codes, ws.a_scales, self.qkv, n, _lib.EPI_BIAS, ws.qkv, st)
        # 3. RMSNorm + spatial RoPE of q and k
        q_in, k_in = ws.qkv[:, :dim], ws.qkv[:, dim:2 * dim]
        chk(lib.rc_rmsnorm_rope(2, (C.c_void_p * 2)(q_in.data_ptr(), k_in.data_ptr()),
                                (C.c_longlong * 2)(ws.qkv.stride(0), ws.qkv.stride(0)),
                                (C.c_void_p * 2)(self.norm_q.data_ptr(), self.norm_k.data_ptr()),
                                (C.c_void_p * 2)(ws.q_rot.data_ptr(), ws.k_rot.data_ptr()),
                                (C.c_longlong * 2)(dim, dim), n, dim, self.head_dim,
                                span, scos.data_ptr(), ssin.data_ptr(), _EPS, st), "rmsnorm_rope")

    def post_attention(self, lib, h, ws, st):
        """Steps 5-7 of the layer on h [N, dim], with the attention output's NVFP4
        operand in ws.a_codes / ws.a_scales: o-proj with gated residual, cross
        attention block, FFN block."""
        n, dim = h.shape
        mod = self.modulation
        gate, cshift, cscale, cgate = mod[2], mod[3], mod[4], mod[5]
        chk = _lib.check
        # 5. o-proj with gated residual
        self._gemm(lib, ws, ws.a_codes, ws.a_scales, self.o, n, _lib.EPI_GATED_RESIDUAL, h, st, gate)
        # 6. cross attention
        chk(lib.rc_ln_modulate_quant(h.data_ptr(), dim, n, dim, self.norm2_w.data_ptr(),
                                     self.norm2_b.data_ptr(), None, None, _EPS, None, 0,
                                     ws.a_codes.data_ptr(), ws.a_scales.data_ptr(), 1.0, st), "ln2")
        self._gemm(lib, ws, ws.a_codes, ws.a_scales, self.cq, n, _lib.EPI_BIAS, ws.cq, st)
        chk(lib.rc_rmsnorm_rope(1, (C.c_void_p * 1)(ws.cq.data_ptr()), (C.c_longlong * 1)(dim),
                                (C.c_void_p * 1)(self.cnorm_q.data_ptr()),
                                (C.c_void_p * 1)(ws.q_rot.data_ptr()), (C.c_longlong * 1)(dim),
                                n, dim, self.head_dim, 1, None, None, _EPS, st), "cross_rms")
        hd = self.head_dim
        strides = (C.c_longlong * 9)(0, dim, hd, 0, dim, hd, 0, dim, hd)
        chk(lib.rc_cross_attention_ws(ws.q_rot.data_ptr(), self.cross_k.data_ptr(),
                                      self.cross_v.data_ptr(), strides, 1, n, self.cross_k.shape[0],
                                      self.heads, hd, None, dim, ws.a_codes.data_ptr(),
                                      ws.a_scales.data_ptr(), ws.cross_ws.data_ptr(), ws.cross_ws.numel(),
                                      st), "cross_attn")
        self._gemm(lib, ws, ws.a_codes, ws.a_scales, self.co, n, _lib.EPI_RESIDUAL, h, st)
        # 7. FFN
        chk(lib.rc_ln_modulate_quant(h.data_ptr(), dim, n, dim, None, None, cshift.data_ptr(),
                                     cscale.data_ptr(), _EPS, None, 0, ws.a_codes.data_ptr(),
                                     ws.a_scales.data_ptr(), 1.0, st), "ln3")
        chk(lib.rc_nvfp4_gemm_ws(ws.a_codes.data_ptr(), ws.a_scales.data_ptr(), self.up.codes.data_ptr(),
                                 self.up.scales.data_ptr(), _lib.ptr(self.up.bias), n, self.up.n,
                                 self.up.k, 1.0, _lib.EPI_GELU_NVFP4, None, 0, None,
                                 ws.f_codes.data_ptr(), ws.f_scales.data_ptr(), 1.0,
                                 ws.gemm_ws.data_ptr(), ws.gemm_ws.numel(), st), "ffn_up")
        self._gemm(lib, ws, ws.f_codes, ws.f_scales, self.down, n, _lib.EPI_GATED_RESIDUAL, h, st, cgate)

    # ------------------------------------------------------------ helpers
    def _gemm(self, lib, ws, codes, scales, w: _Quantized, m, epi, out, st, gate=None):
        _lib.check(lib.rc_nvfp4_gemm_ws(codes.data_ptr(), scales.data_ptr(), w.codes.data_ptr(),
                                        w.scales.data_ptr(), _lib.ptr(w.bias), m, w.n, w.k, 1.0, epi,
                                        out.data_ptr(), out.stride(0), _lib.ptr(gate), None, None,
                                        1.0, ws.gemm_ws.data_ptr(), ws.gemm_ws.numel(), st),
                   "nvfp4_gemm")

    def _attention(self, lib, ws, past_key, past_value, slots, ppos, qpos, n, st, quantized=False):
        """Routed attention into ws.attn (bf16) or, with quantized=True, straight
        into the NVFP4 operand of the o-proj (ws.a_codes / ws.a_scales)."""
        dim, hd, heads = self.dim, self.head_dim, self.heads
        span = self.height * self.width
        frames = n // span
        cap = int(slots.numel())
        kv_tok = past_key.stride(1) if cap else 0
        strides = (C.c_longlong * 15)(
            0, dim, hd,                      # q (spatially rotated)
            0, dim, hd,                      # current k
            0, ws.qkv.stride(0), hd,         # current v: view into qkv
            0, kv_tok, hd, 0, kv_tok, hd)    # cache planes
        wh, ww = (self.height, self.width) if not self.local else self.window
        _lib.check(lib.rc_paired_attention(
            ws.q_rot.data_ptr(), ws.k_rot.data_ptr(), ws.qkv[:, 2 * dim:].data_ptr(),
            past_key.data_ptr() if cap else None, past_value.data_ptr() if cap else None, strides,
            slots.data_ptr() if cap else None, ppos.data_ptr() if cap else None, qpos.data_ptr(),
            self.tables["temporal_cos"].data_ptr(), self.tables["temporal_sin"].data_ptr(),
            1, frames, cap, self.height, self.width, heads, hd, self.tables["temporal_cos"].shape[1] * 2,
            wh, ww, ws.attn_ws.data_ptr(), ws.attn_ws.numel(),
            None if quantized else ws.attn.data_ptr(), dim,
            ws.a_codes.data_ptr() if quantized else None,
            ws.a_scales.data_ptr() if quantized else None, st),
            "attention")


class Workspace:
    """Per-token-count scratch shared by all layers of a stack."""

    def __init__(self, block: FusedBlock, n: int, max_cap: int = 8, attention: bool = True):
        dev, dim = block.device, block.dim
        span = block.height * block.width
        frames = n // span
        self.n = n
        self.a_codes = torch.empty((n, dim // 2), dtype=torch.uint8, device=dev)
        self.a_scales = torch.empty((scale_numel(n, dim),), dtype=torch.uint8, device=dev)
        self.qkv = torch.empty((n, 3 * dim), dtype=torch.bfloat16, device=dev)
        self.q_rot = torch.empty((n, dim), dtype=torch.bfloat16, device=dev)
        self.k_rot = torch.empty((n, dim), dtype=torch.bfloat16, device=dev)
        self.attn = torch.empty((n, dim), dtype=torch.bfloat16, device=dev)
        self.cq = torch.empty((n, dim), dtype=torch.bfloat16, device=dev)
        self.f_codes = torch.empty((n, block.ffn // 2), dtype=torch.uint8, device=dev)
        self.f_scales = torch.empty((scale_numel(n, block.ffn),), dtype=torch.uint8, device=dev)
        if attention:       # a token shard of a head-sharded stack attends elsewhere
            ws = _lib.library().rc_paired_attention_workspace(1, frames, max_cap, block.height,
                                                              block.width, block.heads, block.head_dim)
            self.attn_ws = torch.empty((ws,), dtype=torch.uint8, device=dev)
        # Split-K partials and arrival counters of the NVFP4 GEMMs (zero-filled;
        # the GEMMs leave it zero-filled).
        self.gemm_ws = torch.zeros((_lib.library().rc_gemm_split_workspace(),), dtype=torch.uint8,
                                   device=dev)
        # Tail-split partials and counters of the cross-attention (zero-filled;
        # the kernel leaves it zero-filled).
        self.cross_ws = torch.zeros((_lib.library().rc_cross_attention_workspace(),), dtype=torch.uint8,
                                    device=dev)


def rope_tables(head_dim: int, height: int, width: int, device) -> dict:
    """RollingRoPE tables in the layouts the kernels read: temporal [22, td/2],
    spatial [H*W, d] (transformer.py:57-60, rope.py:50-82)."""
    from .rope import RollingRoPE
    r = RollingRoPE(head_dim, height, width, device=device)
    return {"temporal_cos": r.temporal_cos.float().contiguous(),
            "temporal_sin": r.temporal_sin.float().contiguous(),
            "spatial_cos": r.spatial_cos.reshape(height * width, head_dim).float().contiguous(),
            "spatial_sin": r.spatial_sin.reshape(height * width, head_dim).float().contiguous(),
            "rope": r}


class LayerStack:
    """The layer loop of TransformerSession.step (transformer.py:311-318) over
    FusedBlocks with one FixedKVCache router per layer.

    step(hidden, frames) runs one latent block; with graphs=True, body blocks
    (same token count every step) replay one captured CUDA graph whose routing
    metadata is refreshed by a single host-to-device copy per block.
    """

    def __init__(self, blocks: list[FusedBlock], actions: list[str], *, initial=5, stride=6,
                 anchors=2):
        if len(blocks) != len(actions):
            raise ValueError("A static KV router action is required for every DiT block.")
        self.blocks, self.actions = blocks, list(actions)
        self.router = (initial, stride, anchors)
        b0 = blocks[0]
        self.device, self.dim, self.heads, self.head_dim = b0.device, b0.dim, b0.heads, b0.head_dim
        if not hasattr(self, "cache_heads"):
            self.cache_heads = self.heads        # a head-sharded stack caches its own heads only
        self.span = b0.height * b0.width
        self.rope = b0.tables["rope"]
        self._ws: dict[int, Workspace] = {}
        self._io: dict[int, dict] = {}          # step_host staging buffers and events per token count
        self._copy_stream = None          # host -> device inputs of step_host
        self._copy_out_stream = None      # device -> host results of step_host
        self._graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self.reset()

    def reset(self):
        """Start a new stream: fresh routers and zeroed caches. Graphs captured
        before hold the old cache pointers and are dropped."""
        self._graphs.clear()
        ini, st, an = self.router
        self.caches = [FixedKVCache(a, initial=ini, stride=st, anchors=an) for a in self.actions]
        self.max_cap = max(c.capacity for c in self.caches)
        L = len(self.blocks)
        # Device routing table: per layer [slots(8) | ppos(8) | plan(1+2*8)] + qpos(8).
        self._row = 8 + 8 + 17
        # Pinned routing tables in a ring: the host may run several blocks ahead
        # of the device, and a block's host-to-device copy reads its table when
        # the stream reaches it, so a table is rewritten only after its copy ran.
        self._route_ring = [torch.zeros((L * self._row + 8,), dtype=torch.int32, pin_memory=True)
                            for _ in range(4)]
        self._route_copied = [None] * len(self._route_ring)
        self._route_i = 0
        self.route_host = self._route_ring[0]
        self.route_dev = torch.zeros_like(self.route_host, device=self.device)
        shape = lambda c: (1, max(c.capacity, 1) * self.span, self.cache_heads, self.head_dim)
        self.cache_k = [torch.zeros(shape(c), dtype=torch.bfloat16, device=self.device) for c in self.caches]
        self.cache_v = [torch.zeros(shape(c), dtype=torch.bfloat16, device=self.device) for c in self.caches]
        self.latent_offset = 0

    def workspace(self, n):
        if n not in self._ws:
            self._ws[n] = Workspace(self.blocks[0], n, max(self.max_cap, 1))
        return self._ws[n]

    def _plan(self, frames):
        """Host routing for one block: fills the next table of the ring (route_host),
        advances the routers."""
        j = self._route_i % len(self._route_ring)
        if self._route_copied[j] is not None:
            self._route_copied[j].synchronize()        # its previous upload has run
        self.route_host = self._route_ring[j]
        origin, _ = self.rope.positions(self.latent_offset, frames)
        qpos = [self.latent_offset - origin + f for f in range(frames)]
        r = self.route_host
        base_q = len(self.blocks) * self._row
        r[base_q:base_q + 8] = 0
        r[base_q:base_q + frames] = torch.tensor(qpos, dtype=torch.int32)
        for i, c in enumerate(self.caches):
            o = i * self._row
            slots, ppos = c.route(origin)
            r[o:o + 8] = -1
            r[o + 8:o + 16] = 0
            if slots:
                r[o:o + len(slots)] = torch.tensor(slots, dtype=torch.int32)
                r[o + 8:o + 8 + len(ppos)] = torch.tensor(ppos, dtype=torch.int32)
            copies = c.plan_commit(frames, self.latent_offset)
            r[o + 16] = len(copies)
            for j, (src, dst) in enumerate(copies):
                r[o + 17 + 2 * j] = src
                r[o + 18 + 2 * j] = dst
        self.latent_offset += frames

    def _layers(self, h, n, frames):
        lib = _lib.library()
        st = _lib.stream(self.device)
        ws = self.workspace(n)
        rd = self.route_dev
        qpos = rd[len(self.blocks) * self._row:]
        row_bytes = self.dim * 2
        for i, (blk, c) in enumerate(zip(self.blocks, self.caches)):
            o = i * self._row
            cap = c.capacity
            slots, ppos = rd[o:o + cap], rd[o + 8:o + 8 + cap]
            blk.run(h, ws, self.cache_k[i], self.cache_v[i], slots, ppos, qpos, )
            if cap:
                _lib.check(lib.rc_kv_commit_planned(
                    ws.k_rot.data_ptr(), ws.qkv[:, 2 * self.dim:].data_ptr(), ws.k_rot.stride(0) * 2,
                    ws.qkv.stride(0) * 2, self.cache_k[i].data_ptr(), self.cache_v[i].data_ptr(),
                    row_bytes, row_bytes, self.span, frames, cap, rd[o + 16:].data_ptr(), st),
                    "kv_commit")

    def step(self, hidden: torch.Tensor, frames: int, *, graphs: bool = False) -> torch.Tensor:
        """hidden [N, dim] bf16 on the device, updated in place through all layers."""
        n = hidden.shape[0]
        if n != frames * self.span:
            raise ValueError("hidden must hold `frames` complete planes.")
        self._plan(frames)
        self._upload_route()
        if not graphs:
            self._layers(hidden, n, frames)
            return hidden
        g = self._graphs.get(n)
        if g is None:
            raise RuntimeError("capture() the graph for this token count first")
        self._static[n].copy_(hidden)
        g.replay()
        hidden.copy_(self._static[n])
        return hidden

    def step_host(self, host_in: torch.Tensor, host_out: torch.Tensor, frames: int) -> "HostStep":
        """One body block from pinned host memory to pinned host memory through
        the captured graph: the host-to-device copy of this block's hidden state
        and the device-to-host copy of its result run on two copy streams
        (inputs, outputs), so they overlap the previous / next block's layer
        loop (double-buffered staging) and the next input copy never queues
        behind an output copy waiting for its block's compute.

        Asynchronous: the call returns before either copy has run. The returned
        HostStep says when the caller may touch the buffers again: host_in must
        not be rewritten before `input_consumed` has completed (the copy reads
        it on the device's schedule, possibly after later step_host calls were
        issued), and host_out holds the result once `output_ready` has
        completed. sync_host() waits for every copy issued so far."""
        n = host_in.shape[0]
        if n != frames * self.span or host_out.shape != host_in.shape:
            raise ValueError("host_in / host_out must hold `frames` complete planes.")
        if n not in self._graphs:
            raise RuntimeError("capture() the graph for this token count first")
        io = self._io.get(n)
        if io is None:
            mk = lambda: torch.empty((n, self.dim), dtype=torch.bfloat16, device=self.device)
            io = {"in": [mk(), mk()], "out": [mk(), mk()], "k": 0,
                  "in_ready": [torch.cuda.Event() for _ in range(2)],
                  "consumed": [torch.cuda.Event() for _ in range(2)],
                  "done": [torch.cuda.Event() for _ in range(2)],
                  "drained": [torch.cuda.Event() for _ in range(2)]}
            for e in io["consumed"] + io["drained"]:
                e.record(torch.cuda.current_stream(self.device))
            self._io[n] = io
        if self._copy_stream is None:
            self._copy_stream = torch.cuda.Stream(self.device)
            self._copy_out_stream = torch.cuda.Stream(self.device)
        k = io["k"] & 1
        comp, cs, co = torch.cuda.current_stream(self.device), self._copy_stream, self._copy_out_stream
        handle = HostStep(torch.cuda.Event(), torch.cuda.Event())
        with torch.cuda.stream(cs):
            cs.wait_event(io["consumed"][k])          # the block two steps back has read this buffer
            io["in"][k].copy_(host_in, non_blocking=True)
            io["in_ready"][k].record(cs)
            handle.input_consumed.record(cs)
        self._plan(frames)
        self._upload_route()
        comp.wait_event(io["in_ready"][k])
        self._static[n].copy_(io["in"][k])
        io["consumed"][k].record(comp)
        self._graphs[n].replay()
        comp.wait_event(io["drained"][k])             # its previous result has left the device
        io["out"][k].copy_(self._static[n])
        io["done"][k].record(comp)
        with torch.cuda.stream(co):
            co.wait_event(io["done"][k])
            host_out.copy_(io["out"][k], non_blocking=True)
            io["drained"][k].record(co)
            handle.output_ready.record(co)
        io["k"] += 1
        return handle

    def _upload_route(self) -> None:
        """Host-to-device copy of the table _plan just filled, on the current stream."""
        j = self._route_i % len(self._route_ring)
        self.route_dev.copy_(self.route_host, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        self._route_copied[j] = ev
        self._route_i += 1

    def sync_host(self) -> None:
        """Block the host until every step_host copy issued so far has run (every
        host_in was read, every host_out written); the current stream also
        waits for them."""
        if self._copy_stream is not None:
            for s in (self._copy_stream, self._copy_out_stream):
                torch.cuda.current_stream(self.device).wait_stream(s)
                s.synchronize()

    def capture(self, n: int, frames: int):
        """Capture one block of the layer loop for a token count n (after at
        least one eager step so every kernel attribute is set)."""
        if not hasattr(self, "_static"):
            self._static = {}
        self._static[n] = torch.zeros((n, self.dim), dtype=torch.bfloat16, device=self.device)
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                self._layers(self._static[n], n, frames)
        torch.cuda.current_stream(self.device).wait_stream(s)
        self._graphs[n] = g
        return g
