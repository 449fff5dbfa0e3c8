"""Generate the golden fixtures of tests/golden/ by running the REFERENCE itself.

Run where a checkout of the reference exists:
    python tests/golden/make_golden.py <reference checkout>            # reference_outputs.npz, router.json
    python tests/golden/make_golden.py <reference checkout> --session  # session_outputs.npz
    TRITON_INTERPRET=1 python tests/golden/make_golden.py <reference checkout> --flashdecoder
    python tests/golden/make_golden.py <reference checkout> --fullsize  # fullsize_hashes.json
    python tests/golden/make_golden.py <reference checkout> --pipeline  # pipeline_outputs.npz
    python tests/golden/make_golden.py <reference checkout> --decoder-step  # decoder_step_outputs.npz
    python tests/golden/make_golden.py <reference checkout> --colorfix      # colorfix_outputs.npz
    python tests/golden/make_golden.py <reference checkout> --pipeline-cuda [out.npz]
                                        # pipeline_cuda_outputs.npz (needs a CUDA device)
                                                                        # flashdecoder_outputs.npz
(or set RECAVSR_REFERENCE). Under TRITON_INTERPRET=1 it also records the
reference's Triton kernel on windowed cases. The --session fixtures come from
the reference's TransformerSession.step on a stand-in model (its own LQ4xProj
and torch modules; weights and inputs from recipes.py).

The reference is imported with two import shims and no other change:
* ``diffusers.models.embeddings.get_1d_rotary_pos_embed`` (diffusers 0.37.1 is
  not installed): the standard rotary table -- theta 10000, float64
  frequencies theta^(-2i/dim), cos/sin of pos*freq with every pair frequency
  repeated twice, cast to float32.
* ``recavsr_infer.weights`` (imports the diffusers model): a stub, since only
  ``PreparedBlock`` is needed from runtime/transformer.py.
Nothing here is shipped: it records what the reference computes so that the
oracle (oracle/) can be checked against it on any machine.
"""
from __future__ import annotations

import json
import os
import sys
import types

import numpy as np
import torch
from torch import nn
from torch.nn import functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
from tests.golden import recipes  # noqa: E402


def _install_shims(ref_root: str):
    def get_1d_rotary_pos_embed(dim, pos, theta=10000.0, use_real=False, linear_factor=1.0,
                                ntk_factor=1.0, repeat_interleave_real=True,
                                freqs_dtype=torch.float32):
        if isinstance(pos, int):
            pos = torch.arange(pos)
        freqs = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=freqs_dtype)[: dim // 2] / dim))
        freqs = torch.outer(pos, freqs)
        return (freqs.cos().repeat_interleave(2, dim=1).float(),
                freqs.sin().repeat_interleave(2, dim=1).float())

    for name in ("diffusers", "diffusers.models", "diffusers.models.embeddings"):
        sys.modules.setdefault(name, types.ModuleType(name))
    sys.modules["diffusers.models.embeddings"].get_1d_rotary_pos_embed = get_1d_rotary_pos_embed
    sys.path.insert(0, ref_root)
    import recavsr_infer  # noqa: F401
    stub = types.ModuleType("recavsr_infer.weights")
    stub.load_block = lambda *a, **k: None
    sys.modules["recavsr_infer.weights"] = stub


def t16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).bfloat16()


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


# --------------------------------------------------------------------- NVFP4
def gen_quant(out):
    from recavsr_infer.runtime import nvfp4
    cases = {
        "special": recipes.quant_special_rows(64),
        "ragged": recipes.bf16_normal(np.random.RandomState(5), (130, 96)),
        "weights": recipes.cfg3_weight(192, 320, seed=6),
        "cfg3_small": recipes.cfg3_activation(300, 512, seed=2),
    }
    for name, x in cases.items():
        packed, scales = nvfp4.quantize(t16(x))
        out[f"quant_{name}_x"] = bits(t16(x))
        out[f"quant_{name}_codes"] = packed.numpy()
        out[f"quant_{name}_scales"] = scales.numpy()


def gen_fp8(out):
    from recavsr_infer.runtime import fp8
    captured = {}

    def fake_scaled_mm(a, b, scale_a, scale_b, bias, out_dtype, use_fast_accum):
        captured["q"], captured["scale"] = a, scale_a
        return torch.zeros(a.shape[0], b.shape[1], dtype=out_dtype)

    layer = object.__new__(fp8.FP8Linear)
    nn.Module.__init__(layer)
    layer.in_features, layer.out_features = 96, 32
    layer.weight_packed = torch.zeros(32, 96, dtype=torch.float8_e4m3fn).view(torch.bfloat16)
    layer.bias = None
    layer.weight_scale = torch.tensor(1.0)
    real = torch._scaled_mm
    torch._scaled_mm = fake_scaled_mm
    try:
        for name, x in {"act": recipes.cfg3_activation(64, 96, seed=8),
                        "weight": recipes.cfg3_weight(48, 96, seed=9)}.items():
            layer.forward(t16(x))
            out[f"fp8_{name}_x"] = bits(t16(x))
            out[f"fp8_{name}_q"] = captured["q"].view(torch.uint8).numpy().copy()
            out[f"fp8_{name}_scale"] = np.float32(captured["scale"].item())
    finally:
        torch._scaled_mm = real


# -------------------------------------------------------------------- router
def gen_router():
    from recavsr_infer.runtime.cache import ACTIONS, FixedKVCache
    from recavsr_infer.runtime.rope import RollingRoPE
    rope = RollingRoPE(128, 1, 1, device="cpu")
    result = {}
    for action in ACTIONS:
        cache = FixedKVCache(action, initial=5, stride=6, anchors=2)
        start, steps = 0, []
        for block in range(75):
            frames = 6 if block == 0 else 2
            origin, qpos = rope.positions(start, frames)
            dummy = torch.zeros(1, frames, 1, 1)
            _, _, slots, ppos = cache.history(dummy, origin=origin)
            key = torch.arange(start, start + frames, dtype=torch.float32).view(1, frames, 1, 1)
            cache.commit(key, key.clone(), frames=frames, start=start)
            content = [] if cache.key is None else [int(v) for v in cache.key.view(-1).tolist()]
            steps.append({"start": start, "frames": frames, "origin": origin,
                          "qpos": qpos.tolist(), "slots": slots.tolist(), "ppos": ppos.tolist(),
                          "slot_frames": content, "frame_ids": list(cache.frame_indices)})
            start += frames
        result[action] = {"capacity": cache.capacity, "steps": steps}
    return result


# ---------------------------------------------------------------------- RoPE
def gen_rope(out):
    from recavsr_infer.runtime.rope import RollingRoPE, apply_rotary, apply_temporal
    r = RollingRoPE(128, 11, 20, device="cpu")
    out["rope_tcos"], out["rope_tsin"] = r.temporal_cos.numpy(), r.temporal_sin.numpy()
    out["rope_scos"] = r.spatial_cos.reshape(220, 128).numpy()
    out["rope_ssin"] = r.spatial_sin.reshape(220, 128).numpy()
    rs = np.random.RandomState(21)
    x = recipes.bf16_normal(rs, (1, 2 * 220, 3, 128))
    out["rope_x"] = bits(t16(x))
    out["rope_spatial"] = bits(r.spatial(t16(x)))
    pos = torch.tensor([4, 17], dtype=torch.int32)
    out["rope_temporal"] = bits(apply_temporal(t16(x), pos, r.temporal_cos, r.temporal_sin, span=220))
    c, s = r.spatial_cos, r.spatial_sin
    out["rope_rotary"] = bits(apply_rotary(t16(x).reshape(1, 2, 220, 3, 128), c, s))
    for h, w in ((22, 40), (34, 60)):
        rr = RollingRoPE(128, h, w, device="cpu")
        out[f"rope_sum_{h}x{w}"] = np.array([rr.spatial_cos.double().sum().item(),
                                             rr.spatial_sin.double().sum().item(),
                                             rr.temporal_cos.double().sum().item(),
                                             rr.temporal_sin.double().sum().item()])


# ----------------------------------------------------------------- attention
def gen_attention(out):
    import triton
    from recavsr_infer.kernels import local_attention as la
    from recavsr_infer.runtime.rope import RollingRoPE
    # (a) dense path: sdpa_attention in fp32 and bf16 on CPU
    H, W, heads, d, frames, cap = 4, 6, 2, 128, 2, 3
    span = H * W
    rs = np.random.RandomState(31)
    q, ck, cv = (recipes.bf16_normal(rs, (1, frames * span, heads, d)) for _ in range(3))
    pk, pv = (recipes.bf16_normal(rs, (1, cap * span, heads, d)) for _ in range(2))
    slots = torch.tensor([2, -1, 0], dtype=torch.int32)
    ppos = torch.tensor([5, 0, 3], dtype=torch.int32)
    qpos = torch.tensor([6, 7], dtype=torch.int32)
    r = RollingRoPE(d, H, W, device="cpu")
    for dt, tag in ((torch.float32, "f32"), (torch.bfloat16, "bf16")):
        o = la.sdpa_attention(*(t16(a).to(dt) for a in (q, ck, cv, pk, pv)), slots, ppos, qpos,
                              r.temporal_cos, r.temporal_sin, H, W, 22, 40)
        out[f"attn_dense_{tag}"] = o.float().numpy()
    for n, a in zip(("q", "ck", "cv", "pk", "pv"), (q, ck, cv, pk, pv)):
        out[f"attn_dense_{n}"] = bits(t16(a))
    # (b) windowed path: the reference's Triton kernel under TRITON_INTERPRET=1 (fp16 only)
    if os.environ.get("TRITON_INTERPRET") == "1":
        for tag, (H, W, wh, ww, d, cap, sl, pp) in {
            "win_a": (8, 16, 4, 8, 64, 3, [2, -1, 0], [3, 0, 5]),
            "win_b": (6, 10, 3, 5, 128, 2, [1, 0], [4, 6]),
        }.items():
            span = H * W
            rs = np.random.RandomState(41 + len(tag))
            qh = [rs.standard_normal((1, 2 * span, 2, d)).astype(np.float16) for _ in range(3)]
            ph = [rs.standard_normal((1, cap * span, 2, d)).astype(np.float16) for _ in range(2)]
            tq = [torch.from_numpy(a) for a in qh + ph]
            slots = torch.tensor(sl, dtype=torch.int32)
            ppos = torch.tensor(pp, dtype=torch.int32)
            qpos = torch.tensor([7, 8], dtype=torch.int32)
            r = RollingRoPE(d, H, W, device="cpu")
            o = torch.empty_like(tq[0])
            bh, bw, bt = 4, 8, 2
            la._paired_local[(triton.cdiv(H, bh) * triton.cdiv(W, bw), 1, 2)](
                *tq, slots, ppos, qpos, r.temporal_cos, r.temporal_sin, o,
                *tq[0].stride()[:3], *tq[1].stride()[:3], *tq[2].stride()[:3],
                *tq[3].stride()[:3], *tq[4].stride()[:3],
                H, W, 2, cap, 2, d, r.temporal_cos.shape[1] * 2, min(H, wh), min(W, ww),
                bh, bw, bt, bh * bw * bt, 64, min(H, min(H, wh) + bh - 1),
                min(W, min(W, ww) + bw - 1), num_warps=4, num_stages=2)
            out[f"attn_{tag}_out"] = o.float().numpy()
            for n, a in zip(("q", "ck", "cv", "pk", "pv"), qh + ph):
                out[f"attn_{tag}_{n}"] = a
            out[f"attn_{tag}_meta"] = np.array([H, W, wh, ww, d, cap] + sl + pp, np.int64)


# --------------------------------------------------------------------- block
class _FP32LayerNorm(nn.LayerNorm):
    """diffusers FP32LayerNorm: layer_norm of x.float() (affine params cast to
    float), cast back to the input dtype."""

    def forward(self, x):
        return F.layer_norm(x.float(), self.normalized_shape,
                            None if self.weight is None else self.weight.float(),
                            None if self.bias is None else self.bias.float(),
                            self.eps).to(x.dtype)


class _Attention(nn.Module):
    """Module layout PreparedBlock reads from WanAttention
    (models/transformer_wan.py:515-626), unfused projections."""

    def __init__(self, dim, heads, cross):
        super().__init__()
        self.to_q, self.to_k, self.to_v = (nn.Linear(dim, dim) for _ in range(3))
        self.to_out = nn.ModuleList([nn.Linear(dim, dim), nn.Dropout(0.0)])
        self.norm_q = nn.RMSNorm(dim, eps=1e-6)
        self.norm_k = nn.RMSNorm(dim, eps=1e-6)
        self.heads, self.fused_projections, self.is_cross_attention = heads, False, cross

    def precompute_cross_attention_kv(self, enc):
        key = self.norm_k(self.to_k(enc)).unflatten(2, (self.heads, -1))
        return key, self.to_v(enc).unflatten(2, (self.heads, -1))


class _GeluProj(nn.Module):
    def __init__(self, dim, inner):
        super().__init__()
        self.proj = nn.Linear(dim, inner)

    def forward(self, x):
        return F.gelu(self.proj(x), approximate="tanh")


class _FeedForward(nn.Module):
    def __init__(self, dim, inner):
        super().__init__()
        self.net = nn.ModuleList([_GeluProj(dim, inner), nn.Dropout(0.0), nn.Linear(inner, dim)])

    def forward(self, x):
        for m in self.net:
            x = m(x)
        return x


class _Block(nn.Module):
    def __init__(self, dim, heads, ffn):
        super().__init__()
        self.norm1 = _FP32LayerNorm(dim, 1e-6, elementwise_affine=False)
        self.attn1 = _Attention(dim, heads, False)
        self.attn2 = _Attention(dim, heads, True)
        self.norm2 = _FP32LayerNorm(dim, 1e-6, elementwise_affine=True)
        self.ffn = _FeedForward(dim, ffn)
        self.norm3 = _FP32LayerNorm(dim, 1e-6, elementwise_affine=False)
        self.scale_shift_table = nn.Parameter(torch.zeros(1, 6, dim))


class _QuantLinear(nn.Module):
    """NVFP4Linear with the GEMM replaced by its defining math: the reference's
    own quantize() of activations and weights, dequantized, fp32 matmul + bias,
    bf16 out (the GEMM's defining math, the parity target for the GEMM)."""

    LUT = torch.tensor([0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6])

    def __init__(self, linear):
        super().__init__()
        from recavsr_infer.runtime import nvfp4
        self.q = nvfp4.quantize
        self.n, self.k = linear.out_features, linear.in_features
        self.w = self.deq(*self.q(linear.weight.detach()), self.n, self.k)
        self.bias = linear.bias

    def deq(self, packed, flat, m, k):
        codes = torch.stack((packed & 15, packed >> 4), -1).reshape(m, k).long()
        pm, pk = (m + 127) // 128 * 128, ((k // 16 + 3) // 4) * 4
        sc = flat.reshape(pm // 128, pk // 4, 32, 4, 4).permute(0, 3, 2, 1, 4).reshape(pm, pk)
        sc = sc[:m, : k // 16].contiguous().view(torch.float8_e4m3fn).float()
        return (self.LUT[codes].reshape(m, k // 16, 16) * sc[..., None]).reshape(m, k)

    def forward(self, x):
        a = x.reshape(-1, self.k)
        acc = self.deq(*self.q(a), a.shape[0], self.k).double() @ self.w.double().T
        if self.bias is not None:
            acc = acc + self.bias.double()
        return acc.float().to(torch.bfloat16).reshape(*x.shape[:-1], self.n)


def gen_block(out, tag="block", dim=256, heads=2, ffn=512, H=4, W=6, enc_len=16, pseed=11,
              iseed=12, cap=3, slots=(1, -1, 2), ppos=(4, 0, 5)):
    from recavsr_infer.runtime.rope import RollingRoPE
    from recavsr_infer.runtime.transformer import PreparedBlock
    span = H * W
    p = recipes.block_params(dim, heads, ffn, enc_len=enc_len, seed=pseed)
    b = _Block(dim, heads, ffn)
    with torch.no_grad():
        names = {"q": b.attn1.to_q, "k": b.attn1.to_k, "v": b.attn1.to_v, "o": b.attn1.to_out[0],
                 "cq": b.attn2.to_q, "ck": b.attn2.to_k, "cv": b.attn2.to_v, "co": b.attn2.to_out[0],
                 "up": b.ffn.net[0].proj, "down": b.ffn.net[2]}
        for n, lin in names.items():
            lin.weight.copy_(torch.from_numpy(p[n + "_w"]))
            lin.bias.copy_(torch.from_numpy(p[n + "_b"]))
        b.attn1.norm_q.weight.copy_(torch.from_numpy(p["norm_q"]))
        b.attn1.norm_k.weight.copy_(torch.from_numpy(p["norm_k"]))
        b.attn2.norm_q.weight.copy_(torch.from_numpy(p["cnorm_q"]))
        b.attn2.norm_k.weight.copy_(torch.from_numpy(p["cnorm_k"]))
        b.norm2.weight.copy_(torch.from_numpy(p["norm2_w"]))
        b.norm2.bias.copy_(torch.from_numpy(p["norm2_b"]))
        b.scale_shift_table.copy_(torch.from_numpy(p["scale_shift_table"]))
    b = b.to(torch.bfloat16)
    cond = types.SimpleNamespace(timestep_proj=t16(p["timestep_proj"]),
                                 encoder_hidden_states=t16(p["encoder"]))
    rope = RollingRoPE(dim // heads, H, W, device="cpu")
    core = PreparedBlock(b, cond, rope, window=(22, 40)).eval()
    for mod in list(b.modules()):          # quantize_block_linears order (transformer.py:217-224)
        for name, child in list(mod.named_children()):
            if isinstance(child, nn.Linear):
                setattr(mod, name, _QuantLinear(child))
    hidden, pk, pv = recipes.block_inputs(2 * span, cap * span, dim, seed=iseed)
    slots = torch.tensor(list(slots), dtype=torch.int32)
    ppos = torch.tensor(list(ppos), dtype=torch.int32)
    qpos = torch.tensor([6, 7], dtype=torch.int32)
    with torch.inference_mode():
        h, k, v = core(t16(hidden), t16(pk).unflatten(2, (heads, -1)),
                       t16(pv).unflatten(2, (heads, -1)), slots, ppos, qpos)
    out[f"{tag}_hidden"] = bits(h)
    out[f"{tag}_k"] = bits(k)
    out[f"{tag}_v"] = bits(v)
    out[f"{tag}_modulation"] = core.modulation.detach().float().numpy()
    out[f"{tag}_cross_k"] = bits(core.cross_k.detach())
    out[f"{tag}_cross_v"] = bits(core.cross_v.detach())
    out[f"{tag}_meta"] = np.array([dim, heads, ffn, H, W, cap, enc_len, pseed, iseed] + list(slots)
                                  + list(ppos), np.int64)


class _SessionModel(nn.Module):
    """The attributes TransformerSession (runtime/transformer.py:148-349) reads
    from the Wan model: patch_embedding, lq_proj (the reference's own LQ4xProj),
    sr_proj, blocks, norm_out (FP32LayerNorm without affine), proj_out,
    scale_shift_table, config, the static KV router and the streaming
    conditioning cache (here given directly: temb, timestep projection and the
    already projected prompt states)."""

    def __init__(self, blocks, actions, channels, dim, heads, h1, h2, temb, timestep_proj):
        super().__init__()
        from recavsr_infer.models.lq_proj import LQ4xProj
        self.patch_embedding = nn.Conv3d(channels, dim, kernel_size=(1, 2, 2), stride=(1, 2, 2))
        self.lq_proj = LQ4xProj(3, dim, h1, h2)
        self.sr_proj = nn.Linear(dim, dim)
        self.blocks = nn.ModuleList(blocks)
        self.norm_out = _FP32LayerNorm(dim, 1e-6, elementwise_affine=False)
        self.proj_out = nn.Linear(dim, channels * 4)
        self.scale_shift_table = nn.Parameter(torch.zeros(1, 2, dim))
        self.config = types.SimpleNamespace(in_channels=channels, patch_size=(1, 2, 2),
                                            num_attention_heads=heads, attention_head_dim=dim // heads)
        self._static_kv_router = types.SimpleNamespace(layer_actions=list(actions), anchor_initial_index=5,
                                                       anchor_stride_latents=6, anchor_capacity_latents=2)
        self._temb, self._tproj = temb, timestep_proj

    def _cache_streaming_conditioning(self, timestep, prompt):
        return types.SimpleNamespace(temb=self._temb, timestep_proj=self._tproj, encoder_hidden_states=prompt)


def gen_session(out, dim=256, heads=2, ffn=512, channels=16, height=128, width=192, h1=64, h2=128,
                enc_len=16, actions=("recent_2", "none")):
    """Three TransformerSession.step calls (prefix 21 RGB frames, then two
    8-frame body blocks) of a 2-layer stand-in model, NVFP4 block linears
    emulated as in gen_block; weights and inputs from tests/golden/recipes.py
    (session_params, block_params, session_inputs). Records the LQ projector's
    outputs, the hidden state entering the first block, the hidden state
    leaving the last block and the step results."""
    from recavsr_infer.runtime.transformer import TransformerSession
    bp = [recipes.block_params(dim, heads, ffn, enc_len=enc_len, seed=70 + i) for i in range(len(actions))]
    blocks = []
    for p in bp:
        b = _Block(dim, heads, ffn)
        with torch.no_grad():
            names = {"q": b.attn1.to_q, "k": b.attn1.to_k, "v": b.attn1.to_v, "o": b.attn1.to_out[0],
                     "cq": b.attn2.to_q, "ck": b.attn2.to_k, "cv": b.attn2.to_v, "co": b.attn2.to_out[0],
                     "up": b.ffn.net[0].proj, "down": b.ffn.net[2]}
            for n, lin in names.items():
                lin.weight.copy_(torch.from_numpy(p[n + "_w"]))
                lin.bias.copy_(torch.from_numpy(p[n + "_b"]))
            b.attn1.norm_q.weight.copy_(torch.from_numpy(p["norm_q"]))
            b.attn1.norm_k.weight.copy_(torch.from_numpy(p["norm_k"]))
            b.attn2.norm_q.weight.copy_(torch.from_numpy(p["cnorm_q"]))
            b.attn2.norm_k.weight.copy_(torch.from_numpy(p["cnorm_k"]))
            b.norm2.weight.copy_(torch.from_numpy(p["norm2_w"]))
            b.norm2.bias.copy_(torch.from_numpy(p["norm2_b"]))
            b.scale_shift_table.copy_(torch.from_numpy(p["scale_shift_table"]))
        blocks.append(b)
    g = recipes.session_params(dim, channels, h1, h2)
    temb = g["temb"]
    model = _SessionModel(blocks, actions, channels, dim, heads, h1, h2, t16(temb),
                          t16(bp[0]["timestep_proj"]))
    with torch.no_grad():
        model.patch_embedding.weight.copy_(torch.from_numpy(g["patch_w"]))
        model.patch_embedding.bias.copy_(torch.from_numpy(g["patch_b"]))
        model.sr_proj.weight.copy_(torch.from_numpy(g["sr_w"]))
        model.sr_proj.bias.copy_(torch.from_numpy(g["sr_b"]))
        model.proj_out.weight.copy_(torch.from_numpy(g["proj_out_w"]))
        model.proj_out.bias.copy_(torch.from_numpy(g["proj_out_b"]))
        lq = model.lq_proj
        lq.conv1.weight.copy_(torch.from_numpy(g["conv1_w"]))
        lq.conv1.bias.copy_(torch.from_numpy(g["conv1_b"]))
        lq.norm1.weight.copy_(torch.from_numpy(g["norm1_w"]).reshape(-1, 1, 1, 1))
        lq.conv2.weight.copy_(torch.from_numpy(g["conv2_w"]))
        lq.conv2.bias.copy_(torch.from_numpy(g["conv2_b"]))
        lq.norm2.weight.copy_(torch.from_numpy(g["norm2_w"]).reshape(-1, 1, 1, 1))
        lq.out_proj.weight.copy_(torch.from_numpy(g["out_w"]))
        lq.out_proj.bias.copy_(torch.from_numpy(g["out_b"]))
    model = model.to(torch.bfloat16)
    model.scale_shift_table = nn.Parameter(torch.from_numpy(g["scale_shift_table"]))   # fp32, as the
    # reference keeps scale_shift_table in fp32 (models/transformer_wan.py:945)
    session = TransformerSession(model, t16(bp[0]["encoder"]), height, width, seed=0)
    for b in model.blocks:                 # quantize_block_linears (transformer.py:217-224), emulated
        for mod in list(b.modules()):
            for name, child in list(mod.named_children()):
                if isinstance(child, nn.Linear):
                    setattr(mod, name, _QuantLinear(child))
    seen = {"lq": [], "first_in": [], "last_out": []}
    lq_fwd = model.lq_proj.forward_streaming
    model.lq_proj.forward_streaming = lambda v, s: seen["lq"].append(lq_fwd(v, s)) or seen["lq"][-1]
    first, last = session.cores[0], session.cores[-1]
    first_fwd, last_fwd = first.forward, last.forward

    def first_hook(hidden, *a):
        seen["first_in"].append(hidden.clone())
        return first_fwd(hidden, *a)

    def last_hook(*a):
        r = last_fwd(*a)
        seen["last_out"].append(r[0].clone())
        return r
    first.forward, last.forward = first_hook, last_hook
    out["session_meta"] = np.array([dim, heads, ffn, channels, height, width, h1, h2, enc_len], np.int64)
    with torch.inference_mode():
        for i, (video, noise) in enumerate(recipes.session_inputs(channels, height, width)):
            result = session.step(t16(video), noise=torch.from_numpy(noise))
            out[f"session_step{i}_result"] = result.float().numpy()
            out[f"session_step{i}_lqproj"] = bits(seen["lq"][-1])
            out[f"session_step{i}_hidden_in"] = bits(seen["first_in"][-1])
            out[f"session_step{i}_hidden_out"] = bits(seen["last_out"][-1])


def gen_flashdecoder(out):
    """FlashDecoder's local GQA attention (models/flashdecoder/flashdecoder_wan22.py:38-119):
    the reference's CPU path (fp32 SDPA under the visibility mask) on the three
    geometries of recipes.LOCAL_GQA_CASES, and under TRITON_INTERPRET=1 its Triton forward
    (_local_attention_triton.py:21-131, fp16) on the first."""
    from recavsr_infer.models.flashdecoder.flashdecoder_wan22 import _local_attention
    for tag, (b, hq, hk, d, h, w, win, grp, tw, qf, nf) in recipes.LOCAL_GQA_CASES.items():
        q, k, v = recipes.local_gqa_inputs(tag)
        res = _local_attention(torch.from_numpy(q), torch.from_numpy(k), torch.from_numpy(v), height=h,
                               width=w, window=win, group_size=grp, temporal_window=tw)
        out[f"fd_{tag}_out"] = res.numpy()
    if os.environ.get("TRITON_INTERPRET") == "1":
        import triton
        from recavsr_infer.models.flashdecoder import _local_attention_triton as fl
        b, hq, hk, d, h, w, win, grp, tw, qf, nf = recipes.LOCAL_GQA_CASES["a"]
        q16, k16, v16 = (torch.from_numpy(x).half() for x in recipes.local_gqa_inputs("a"))
        res = torch.empty_like(q16)
        lse = torch.empty((b, hq, qf * h * w), dtype=torch.float32)
        fl._forward[(qf * triton.cdiv(h, 4), triton.cdiv(w, 16), b * hq)](
            q16, k16, v16, res, lse, h, w, hq, hk, d, (win[0],) * (tw * grp), (win[1],) * (tw * grp),
            min(triton.next_power_of_2(win[1] + 15), triton.next_power_of_2(w)), qf, nf, nf - qf, tw, grp,
            4, 16, 64, 64)
        out["fd_a_triton_fp16"] = res.numpy()          # fp16 values, stored as fp16


def gen_decoder_step(out):
    """FlashDecoder's streaming decode (models/flashdecoder/flashdecoder_wan22.py:759-874
    through runtime/flashdecoder.py:140-175 FlashDecoderSession.step) on the CPU in
    fp32, for each recipes.DECODER_CASES entry: the RGB chunk of every step (the
    first step 1 frame, then 4), the hidden states leaving the backbone and the
    temporal refinement of every step (forward hooks)."""
    from recavsr_infer.models.flashdecoder.flashdecoder_wan22 import FlashDecoder
    from recavsr_infer.runtime.flashdecoder import FlashDecoderSession
    for tag, c in recipes.DECODER_CASES.items():
        model = FlashDecoder(dim=c["dim"], depth=c["depth"], num_heads=c["num_heads"],
                             num_kv_groups=c["num_kv_groups"], refinement_depth=c["refinement_depth"],
                             mlp_ratio=c["mlp_ratio"], spatial_window_size=c["window"])
        params = recipes.decoder_params(tag)
        model.load_state_dict({k: torch.from_numpy(v) for k, v in params.items()}, strict=True)
        model.eval()
        latents, mean, std, lr_up = recipes.decoder_inputs(tag)
        model.vae_config = {"latents_mean": mean.tolist(), "latents_std": std.tolist()}
        seen = {"backbone": [], "refinement": []}
        model.backbone.register_forward_hook(lambda m, a, o: seen["backbone"].append(o[0].detach().clone()))
        model.temporal_refinement.register_forward_hook(
            lambda m, a, o: seen["refinement"].append(o[0].detach().clone()))
        session = FlashDecoderSession(model)
        rgb = list(session.step(torch.from_numpy(latents), lr_up=torch.from_numpy(lr_up)))
        for i, r in enumerate(rgb):
            out[f"dec_{tag}_rgb{i}"] = r.numpy()
            out[f"dec_{tag}_backbone{i}"] = seen["backbone"][i].numpy()
            out[f"dec_{tag}_refine{i}"] = seen["refinement"][i].numpy()


def gen_colorfix(out):
    """recavsr_infer/color_fix.py:58-117 on the CPU: adain_color_fix and
    wavelet_color_fix on recipes.COLORFIX_CASES."""
    from recavsr_infer.color_fix import adain_color_fix, wavelet_color_fix
    for tag in recipes.COLORFIX_CASES:
        dec, ref, lq = recipes.colorfix_inputs(tag)
        out[f"cf_{tag}_adain"] = adain_color_fix(torch.from_numpy(dec), torch.from_numpy(ref)).numpy()
        out[f"cf_{tag}_wavelet"] = wavelet_color_fix(torch.from_numpy(dec), lq)


FULLSIZE_SHAPES = ((7040, 14336), (7040, 3072))     # cfg3's largest activations


def gen_fullsize():
    """SHA-256 of the reference's NVFP4 codes / swizzled scales
    (runtime/nvfp4.py:49-68) and FP8 codes + scale (runtime/fp8.py:41-42) of
    the cfg3 activations at full size (recipes.cfg3_activation_large): a
    size-independent pin of bit-exactness where the arrays are too large to
    keep as fixtures."""
    import hashlib
    from recavsr_infer.runtime import fp8, nvfp4
    sha = lambda a: hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()
    result = {}
    for m, k in FULLSIZE_SHAPES:
        x = t16(recipes.cfg3_activation_large(m, k))
        packed, scales = nvfp4.quantize(x)
        result[f"nvfp4_{m}x{k}"] = {"codes": sha(packed.numpy()), "scales": sha(scales.numpy())}
        layer = object.__new__(fp8.FP8Linear)
        nn.Module.__init__(layer)
        captured = {}

        def fake_scaled_mm(a, b, scale_a, scale_b, bias, out_dtype, use_fast_accum):
            captured["q"], captured["scale"] = a, scale_a
            return torch.zeros(a.shape[0], b.shape[1], dtype=out_dtype)
        layer.in_features, layer.out_features = k, 16
        layer.weight_packed = torch.zeros(16, k, dtype=torch.float8_e4m3fn).view(torch.bfloat16)
        layer.bias, layer.weight_scale = None, torch.tensor(1.0)
        real, torch._scaled_mm = torch._scaled_mm, fake_scaled_mm
        try:
            layer.forward(x)
        finally:
            torch._scaled_mm = real
        result[f"fp8_{m}x{k}"] = {"codes": sha(captured["q"].view(torch.uint8).numpy()),
                                  "scale": float(captured["scale"].item())}
    return result


# ------------------------------------------------------------ host pipeline
PIPELINE_ENLARGE = [            # (LQ frames, h, w, block, output size or None for x4 scale)
    (5, 22, 40, 8, None),       # x4 -> 88 x 160: height padded by 8 (reflect)
    (3, 13, 21, 3, (50, 75)),   # non-integer scale, both axes reflect-padded
    (2, 5, 6, 4, (10, 12)),     # pads >= size: replicate
]
PIPELINE_BLEND = [              # (LQ width, strips, overlap, scale, out height, frames)
    (40, 3, 6, 4.0, 24, 2),
    (33, 2, 5, 2.0, 16, 2),
]


def gen_pipeline(out):
    """The reference's video.prepare_block pieces (enlarge_block: cv2.resize
    INTER_LINEAR + block padding; block_tensor: normalize + pad) and
    strips.blend_strips (its own canvas loop, fed in-memory frames in place of
    the decoded strip videos). `av` (PyAV) is not installed and only opens
    files, so it is stubbed; cv2 is the real opencv-python-headless."""
    import hashlib
    sys.modules.setdefault("av", types.ModuleType("av"))
    from recavsr_infer import strips, video
    for i, (n, h, w, block, size) in enumerate(PIPELINE_ENLARGE):
        frames = recipes.lq_frames_u8(n, h, w, seed=60 + i)
        size = size or video.scaled_size(h, w, 4.0)
        enlarged = video.enlarge_block(frames, size, block=block)
        x = video.block_tensor(enlarged, block, device="cpu")
        out[f"enlarge{i}_u8"] = enlarged.numpy()                  # [1, 3, block, H, W] uint8
        out[f"enlarge{i}_sha256"] = np.frombuffer(
            hashlib.sha256(x.contiguous().numpy().tobytes()).digest(), np.uint8)
        out[f"enlarge{i}_shape"] = np.array(x.shape, np.int64)
        if x.numel() <= 65536:
            out[f"enlarge{i}_f32"] = x.numpy()
    for i, (lq_w, n_strips, overlap, scale, height, n_frames) in enumerate(PIPELINE_BLEND):
        cols = strips.strip_columns(lq_w, n_strips, overlap, scale)
        width = strips.scaled_size(1, lq_w, scale)[1]
        widths = [round(x1 * scale) - round(x0 * scale) for x0, x1 in cols]
        rs = np.random.RandomState(80 + i)
        strip_frames = [[rs.randint(0, 256, (height, sw, 3)).astype(np.uint8) for _ in range(n_frames)]
                        for sw in widths]
        feed = dict(zip(map(str, range(n_strips)), strip_frames))
        saved = strips._decode
        strips._decode = lambda p: iter(feed[str(p)])
        try:
            blended = list(strips.blend_strips([str(k) for k in range(n_strips)], cols, scale, height, width))
        finally:
            strips._decode = saved
        out[f"blend{i}_columns"] = np.array(cols, np.int64)
        out[f"blend{i}_out"] = np.stack(blended)
        for s_i, fr in enumerate(strip_frames):
            out[f"blend{i}_strip{s_i}"] = np.stack(fr)


def gen_pipeline_cuda(out):
    """block_tensor as the reference's inference runs it (device="cuda",
    inference.py:285): torch normalizes there by multiplying with the fp32
    reciprocal of 127.5 instead of dividing, so its output differs from the
    CPU fixture by one fp32 ulp on some byte values. The enlarged frames come
    from the reference's own enlarge_block (cv2, CPU), as in inference."""
    import hashlib
    sys.modules.setdefault("av", types.ModuleType("av"))
    from recavsr_infer import video
    for i, (n, h, w, block, size) in enumerate(PIPELINE_ENLARGE):
        frames = recipes.lq_frames_u8(n, h, w, seed=60 + i)
        size = size or video.scaled_size(h, w, 4.0)
        x = video.block_tensor(video.enlarge_block(frames, size, block=block), block, device="cuda").cpu()
        out[f"enlarge{i}_sha256"] = np.frombuffer(
            hashlib.sha256(x.contiguous().numpy().tobytes()).digest(), np.uint8)
        out[f"enlarge{i}_shape"] = np.array(x.shape, np.int64)
        if x.numel() <= 65536:
            out[f"enlarge{i}_f32"] = x.numpy()


def main():
    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    ref = args[0] if args else os.environ.get("RECAVSR_REFERENCE")
    if not ref:
        raise SystemExit("usage: make_golden.py <reference checkout> [--session]  (or set RECAVSR_REFERENCE)")
    _install_shims(ref)
    if "--fullsize" in sys.argv:
        with open(os.path.join(HERE, "fullsize_hashes.json"), "w") as f:
            json.dump(gen_fullsize(), f, indent=1)
        print("wrote fullsize_hashes.json")
        return
    if "--pipeline-cuda" in sys.argv:
        out = {}
        gen_pipeline_cuda(out)
        path = args[1] if len(args) > 1 else os.path.join(HERE, "pipeline_cuda_outputs.npz")
        np.savez_compressed(path, **out)
        print("wrote", len(out), "pipeline (cuda) arrays to", path)
        return
    if "--pipeline" in sys.argv:
        out = {}
        gen_pipeline(out)
        np.savez_compressed(os.path.join(HERE, "pipeline_outputs.npz"), **out)
        print("wrote", len(out), "pipeline arrays")
        return
    if "--colorfix" in sys.argv:
        out = {}
        gen_colorfix(out)
        np.savez_compressed(os.path.join(HERE, "colorfix_outputs.npz"), **out)
        print("wrote", len(out), "colour-correction arrays")
        return
    if "--decoder-step" in sys.argv:
        torch.manual_seed(0)
        out = {}
        gen_decoder_step(out)
        np.savez_compressed(os.path.join(HERE, "decoder_step_outputs.npz"), **out)
        print("wrote", len(out), "decoder step arrays")
        return
    if "--flashdecoder" in sys.argv:
        out = {}
        gen_flashdecoder(out)
        np.savez_compressed(os.path.join(HERE, "flashdecoder_outputs.npz"), **out)
        print("wrote", len(out), "flashdecoder arrays")
        return
    if "--session" in sys.argv:
        # The session-glue fixtures live in their own file (the reference's
        # TransformerSession.step with a stand-in model; CPU only).
        torch.manual_seed(0)
        out = {}
        gen_session(out)
        np.savez_compressed(os.path.join(HERE, "session_outputs.npz"), **out)
        print("wrote", len(out), "session arrays")
        return
    torch.manual_seed(0)
    out = {}
    gen_quant(out)
    gen_fp8(out)
    gen_rope(out)
    gen_attention(out)
    gen_block(out)
    gen_block(out, "block768", dim=768, heads=6, ffn=2048, H=8, W=12, enc_len=64, pseed=21,
              iseed=22, cap=2, slots=(1, 0), ppos=(3, 4))
    np.savez_compressed(os.path.join(HERE, "reference_outputs.npz"), **out)
    with open(os.path.join(HERE, "router.json"), "w") as f:
        json.dump(gen_router(), f, separators=(",", ":"))
    print("wrote", len(out), "arrays")


if __name__ == "__main__":
    main()
