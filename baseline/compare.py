"""This library next to the reference's own GPU build, on the same B200.

The reference (chariot2658/ReCaVSR, installed unmodified into baseline/_ref by
`python -m pip install --no-index --no-build-isolation --no-deps --target
baseline/_ref <reference checkout>`) is imported with two import shims and no
other change: diffusers' rotary-table helper (diffusers is not installed; the
stub computes the standard table) and `recavsr_infer.weights` (imports the
diffusers model; only PreparedBlock is needed). Everything the reference runs
on the GPU is its own code: the Triton `_paired_local` kernel, `sdpa_attention`
(gather / cat / temporal RoPE / masked torch SDPA), `nvfp4.quantize` +
`nvfp4_mm` (torch._scaled_mm_v2, cuBLASLt), `FP8Linear` (torch._scaled_mm),
`PreparedBlock` compiled with torch.compile as TransformerSession compiles it.

    python baseline/compare.py gemm        # cfg3: NVFP4 / FP8 linears and quantizers, 9 shapes
    python baseline/compare.py attention   # cfg2/cfg4: routed attention at 1280x704, scopes 0..8 planes
    python baseline/compare.py local       # cfg5: 22x40-window attention at 1920x1088 and 3840x2176
    python baseline/compare.py layers      # cfg4: the 30-layer DiT loop, PreparedBlock x 30 compiled
    python baseline/compare.py pipeline    # frame preparation (enlarge + normalize + pad) and strip blend
    python baseline/compare.py decoder     # FlashDecoder local GQA attention (its Triton forward)
    python baseline/compare.py decoder_step  # FlashDecoder decode step (its FlashDecoderSession, eager and compiled)
    python baseline/compare.py colorfix    # AdaIN / wavelet colour correction of a body block's 8 frames
    python baseline/compare.py all

This library's side is imported from recavsr_b200.runtime (ops, fp8, block):
those modules register no operator under the reference's op names, so both
live in one process. Per-op times are CUDA-graph replays of `--reps` calls on the same buffers
(inputs L2-warm where they fit, as for both sides alike); the layer loop is
timed as each side runs it (the reference: its Python loop over compiled
blocks and FixedKVCache; this library: LayerStack's CUDA graph), with CUDA
events, after warm-up. Prints one JSON line per measurement and a table.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time
import types

import torch
import torch.nn.functional as F
from torch import nn

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")
sys.path.insert(0, ROOT)


def install_reference():
    """Import the installed reference with its two shims; returns its package."""
    if not os.path.isdir(os.path.join(REF, "recavsr_infer")):
        raise SystemExit(f"reference not installed in {REF} (see the module docstring)")

    def get_1d_rotary_pos_embed(dim, pos, theta=10000.0, use_real=False, linear_factor=1.0,
                                ntk_factor=1.0, repeat_interleave_real=True, freqs_dtype=torch.float32):
        if isinstance(pos, int):
            pos = torch.arange(pos)
        freqs = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=freqs_dtype)[: dim // 2] / dim))
        freqs = torch.outer(pos.to(freqs_dtype), freqs)
        return (freqs.cos().repeat_interleave(2, dim=1).float(),
                freqs.sin().repeat_interleave(2, dim=1).float())

    for name in ("diffusers", "diffusers.models", "diffusers.models.embeddings"):
        sys.modules.setdefault(name, types.ModuleType(name))
    sys.modules["diffusers.models.embeddings"].get_1d_rotary_pos_embed = get_1d_rotary_pos_embed
    sys.path.insert(0, REF)
    import recavsr_infer
    stub = types.ModuleType("recavsr_infer.weights")
    stub.load_block = lambda *a, **k: None
    sys.modules["recavsr_infer.weights"] = stub
    return recavsr_infer


def emit(rows, **kv):
    rows.append(kv)
    print(json.dumps(kv), flush=True)


def graph_time(fn, reps):
    """Mean device time per call of fn, from a CUDA graph of `reps` calls."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side), torch.cuda.graph(g, stream=side):
        for _ in range(reps):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    g.replay()
    b.record()
    b.synchronize()
    return a.elapsed_time(b) / reps * 1e-3


def event_time(fn, reps):
    """Mean device time per call of fn launched eagerly (no graph)."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        fn()
    b.record()
    b.synchronize()
    return a.elapsed_time(b) / reps * 1e-3


def _inductor_opts():
    known = torch._inductor.config.get_config_copy()
    opts = {**torch._inductor.list_mode_options("default"), "emulate_precision_casts": True,
            "force_same_precision": True}
    return {k: v for k, v in opts.items() if k in known}


# ---------------------------------------------------------------- cfg3 linears
def case_gemm(rows, reps):
    from recavsr_b200 import _lib
    from recavsr_b200.runtime import fp8 as our_fp8
    from recavsr_b200.runtime import ops as our_nv
    from recavsr_infer.runtime import nvfp4 as ref_nv
    lib = _lib.library()
    ref_quant = torch.compile(ref_nv.quantize, fullgraph=True, dynamic=False, options=_inductor_opts())
    g = torch.Generator(device="cuda").manual_seed(2)
    ws = torch.zeros(lib.rc_gemm_split_workspace(), dtype=torch.uint8, device="cuda")
    for m in (1760, 3520, 7040):
        for k, n in ((3072, 3072), (3072, 14336), (14336, 3072)):
            a = torch.randn(m, k, generator=g, device="cuda")
            mask = torch.rand(m, k, generator=g, device="cuda") < 1e-3
            a = torch.where(mask, a * 20, a).bfloat16()
            w = (torch.randn(n, k, generator=g, device="cuda") * 0.02).bfloat16()
            bias = (torch.randn(n, generator=g, device="cuda") * 0.02).bfloat16()
            ac, asf = our_nv.quantize(a)
            wc, wsf = our_nv.quantize(w)
            rac, rasf = ref_quant(a)
            eac, easf = ref_nv.quantize(a)          # the reference's formula, eager (the parity target)
            torch.cuda.synchronize()
            codes_equal = bool(torch.equal(ac, eac) and torch.equal(asf, easf))
            compiled_code_diff = int((ac != rac).sum()) + int((asf != rasf).sum())
            compiled_vs_eager = int((eac != rac).sum()) + int((easf != rasf).sum())
            out = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")

            def ours():
                _lib.check(lib.rc_nvfp4_gemm_ws(ac.data_ptr(), asf.data_ptr(), wc.data_ptr(), wsf.data_ptr(),
                                                bias.data_ptr(), m, n, k, 1.0, _lib.EPI_BIAS, out.data_ptr(),
                                                n, None, None, None, 1.0, ws.data_ptr(), ws.numel(),
                                                _lib.stream()), "nvfp4_gemm")

            def theirs():
                return ref_nv.nvfp4_mm(ac.view(torch.bfloat16), wc.view(torch.bfloat16),
                                       asf.view(torch.bfloat16), wsf.view(torch.bfloat16), bias)
            ref_out = theirs()
            ours()
            torch.cuda.synchronize()
            diff = float((out.float() - ref_out.float()).abs().max() / ref_out.float().abs().max())
            t_o, t_r = graph_time(ours, reps), graph_time(theirs, reps)
            tq_o = graph_time(lambda: our_nv.quantize(a), reps)
            tq_r = graph_time(lambda: ref_quant(a), reps)
            fl = 2.0 * m * n * k
            emit(rows, case="gemm", path="nvfp4", M=m, K=k, N=n, ours_us=t_o * 1e6, ref_us=t_r * 1e6,
                 ours_tflops=fl / t_o / 1e12, ref_tflops=fl / t_r / 1e12, speedup=t_r / t_o,
                 max_rel_diff=diff, quant_ours_us=tq_o * 1e6, quant_ref_us=tq_r * 1e6,
                 quant_equal_to_ref_eager=codes_equal, quant_bytes_differing_from_ref_compiled=compiled_code_diff,
                 ref_compiled_vs_ref_eager_bytes_differing=compiled_vs_eager,
                 ref="recavsr_infer.runtime.nvfp4.nvfp4_mm (torch._scaled_mm_v2) / quantize (torch.compile)")
            # FP8 per-tensor path: the same e4m3 operands through both GEMMs.
            aq, sa = our_fp8.quantize(a)
            wq, sw = our_fp8.quantize(w)
            out8 = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")

            def ours8():
                _lib.check(lib.rc_fp8_gemm(aq.data_ptr(), sa.data_ptr(), wq.data_ptr(), sw.data_ptr(),
                                           bias.data_ptr(), m, n, k, 1.0, _lib.EPI_BIAS, out8.data_ptr(), n,
                                           None, _lib.stream()), "fp8_gemm")

            def theirs8():   # recavsr_infer/runtime/fp8.py:44-47
                return torch._scaled_mm(aq.view(torch.float8_e4m3fn), wq.view(torch.float8_e4m3fn).t(),
                                        scale_a=sa, scale_b=sw, bias=bias, out_dtype=torch.bfloat16,
                                        use_fast_accum=False)
            r8 = theirs8()
            ours8()
            torch.cuda.synchronize()
            d8 = float((out8.float() - r8.float()).abs().max() / r8.float().abs().max())
            t_o, t_r = graph_time(ours8, reps), graph_time(theirs8, reps)
            emit(rows, case="gemm", path="fp8", M=m, K=k, N=n, ours_us=t_o * 1e6, ref_us=t_r * 1e6,
                 ours_tflops=fl / t_o / 1e12, ref_tflops=fl / t_r / 1e12, speedup=t_r / t_o,
                 max_rel_diff=d8, ref="torch._scaled_mm as recavsr_infer/runtime/fp8.py:44-47 calls it")
            del a, w, ac, asf, wc, wsf, rac, rasf, eac, easf, out, ref_out, aq, wq, out8, r8


# ------------------------------------------------------------ routed attention
def _attn_inputs(h, w, heads, cap, g):
    t = h * w
    r = lambda *s: (torch.randn(*s, generator=g, device="cuda") / 128 ** 0.5).bfloat16()
    return (r(1, 2 * t, heads, 128), r(1, 2 * t, heads, 128), r(1, 2 * t, heads, 128),
            r(1, cap * t, heads, 128), r(1, cap * t, heads, 128))


def _routing(cap, visible):
    slots = [cap - visible + i for i in range(visible)] + [-1] * (cap - visible)
    ppos = [12 - visible + i for i in range(visible)] + [0] * (cap - visible)
    i32 = lambda v: torch.tensor(v, dtype=torch.int32, device="cuda")
    return i32(slots), i32(ppos), i32([12, 13])


def case_attention(rows, reps):
    """cfg4 / cfg2 geometry: 1280x704 (22x40 tokens), 2-frame query block, 24
    heads; the window covers the grid, so the reference runs sdpa_attention
    (runtime/transformer.py:46,102). Visible routed planes 0, 1, 2, 4, 6, 8."""
    from recavsr_b200.runtime.ops import routed_attention
    from recavsr_infer.kernels import local_attention as ref_la
    from recavsr_infer.runtime.rope import RollingRoPE
    h, w, heads = 22, 40, 24
    t = h * w
    rope = RollingRoPE(128, h, w, device="cuda")
    ref_c = torch.compile(ref_la.sdpa_attention, fullgraph=True, dynamic=False, options=_inductor_opts())
    g = torch.Generator(device="cuda").manual_seed(1)
    for vis in (0, 1, 2, 4, 6, 8):
        cap = vis
        q, ck, cv, pk, pv = _attn_inputs(h, w, heads, cap, g)
        slots, ppos, qpos = _routing(cap, vis)
        args = (q, ck, cv, pk, pv, slots, ppos, qpos, rope.temporal_cos, rope.temporal_sin, h, w, h, w)
        out = torch.empty_like(q)
        ours = lambda: routed_attention(*args, out=out)
        theirs = lambda: ref_la.sdpa_attention(*args)
        theirs_c = lambda: ref_c(*args)
        ref_out = theirs()
        ours()
        torch.cuda.synchronize()
        diff = float((out.float() - ref_out.float()).abs().max())
        t_o, t_r, t_c = graph_time(ours, reps), graph_time(theirs, reps), graph_time(theirs_c, reps)
        fl = 4.0 * 128 * heads * (2 * t) * t * (vis + 2)
        emit(rows, case="attention", geometry="1280x704 (22x40), 1760 queries, 24 heads", visible_planes=vis + 2,
             ours_us=t_o * 1e6, ref_eager_us=t_r * 1e6, ref_compiled_us=t_c * 1e6,
             ours_tflops=fl / t_o / 1e12, ref_compiled_tflops=fl / t_c / 1e12,
             speedup_vs_compiled=t_c / t_o, max_abs_diff=diff,
             ref="recavsr_infer.kernels.local_attention.sdpa_attention (eager and torch.compile)")
        del q, ck, cv, pk, pv, out, ref_out


def case_local(rows, reps):
    """cfg5 geometries: 1920x1088 (34x60) and 3840x2176 (68x120), 22x40
    windows, 4 routed planes + 2 current; the reference runs its Triton
    paired_attention (the Triton `_paired_local` kernel)."""
    from recavsr_b200.runtime.ops import routed_attention
    from recavsr_infer.kernels import local_attention as ref_la
    from recavsr_infer.runtime.rope import RollingRoPE
    g = torch.Generator(device="cuda").manual_seed(3)
    for h, w, heads in ((34, 60, 24), (68, 120, 24), (68, 120, 3)):
        t = h * w
        rope = RollingRoPE(128, h, w, device="cuda")
        q, ck, cv, pk, pv = _attn_inputs(h, w, heads, 4, g)
        slots, ppos, qpos = _routing(4, 4)
        args = (q, ck, cv, pk, pv, slots, ppos, qpos, rope.temporal_cos, rope.temporal_sin, h, w, 22, 40)
        out = torch.empty_like(q)
        ours = lambda: routed_attention(*args, out=out)
        theirs = lambda: ref_la.paired_attention(*args)
        ref_out = theirs()
        ours()
        torch.cuda.synchronize()
        diff = float((out.float() - ref_out.float()).abs().max())
        t_o, t_r = graph_time(ours, reps), graph_time(theirs, reps)
        fl = 4.0 * 128 * heads * (2 * t) * (min(h, 22) * min(w, 40)) * 6
        emit(rows, case="local", geometry=f"{w * 32}x{h * 32} ({h}x{w} tokens), 22x40 window, {heads} heads",
             visible_planes=6, ours_us=t_o * 1e6, ref_us=t_r * 1e6, ours_tflops=fl / t_o / 1e12,
             ref_tflops=fl / t_r / 1e12, speedup=t_r / t_o, max_abs_diff=diff,
             ref="recavsr_infer.kernels.local_attention.paired_attention (Triton _paired_local)")
        del q, ck, cv, pk, pv, out, ref_out


def visible_pairs(h, w, qf, nf, window, group_size, temporal_window):
    """(query, key) pairs the FlashDecoder mask admits, counted per axis."""
    import numpy as np

    def axis(n, win):
        d = np.arange(n)[:, None] - np.arange(n)[None, :]      # key - query
        return int(((d >= -(win // 2)) & (d < win // 2)).sum())
    frames = 0
    for qt in range(qf):
        qg = (qt + nf - qf) // group_size
        frames += sum(1 for kt in range(nf) if qg - temporal_window < kt // group_size <= qg)
    return frames * axis(h, window[0]) * axis(w, window[1])


def case_decoder(rows, reps):
    """FlashDecoder's local attention (flashdecoder_wan22.py:38-119) at its
    decoder geometry: 8 query heads on 2 KV heads, head_dim 64, 24x24 window;
    the backbone step (1 new frame, 2-frame window) and the temporal
    refinement (4 new frames, 8-frame window), at 704x1280 (44x80 latent) and
    1088x1920 (68x120) frames, bf16. The reference runs its Triton forward
    (_local_attention_triton.py:21-131)."""
    from recavsr_b200.runtime.flashdecoder import local_attention as ours_fd
    from recavsr_infer.models.flashdecoder.flashdecoder_wan22 import _local_attention as ref_fd
    g = torch.Generator(device="cuda").manual_seed(4)
    for h, w in ((44, 80), (68, 120)):
        n = h * w
        for qf, nf, batch in ((1, 2, 1), (4, 8, 1), (4, 8, 4)):
            kw = dict(height=h, width=w, window=(24, 24), group_size=qf, temporal_window=2)
            q = torch.randn(batch, 8, qf * n, 64, device="cuda", generator=g).to(torch.bfloat16)
            k = torch.randn(batch, 2, nf * n, 64, device="cuda", generator=g).to(torch.bfloat16)
            v = torch.randn(batch, 2, nf * n, 64, device="cuda", generator=g).to(torch.bfloat16)
            ref_out = ref_fd(q, k, v, **kw)
            out = ours_fd(q, k, v, **kw)
            torch.cuda.synchronize()
            diff = float((out.float() - ref_out.float()).abs().max())
            t_o = graph_time(lambda: ours_fd(q, k, v, **kw), reps)
            t_r = graph_time(lambda: ref_fd(q, k, v, **kw), reps)
            fl = 4.0 * 64 * 8 * batch * visible_pairs(h, w, qf, nf, (24, 24), qf, 2)
            emit(rows, case="decoder", geometry=f"{w * 16}x{h * 16} ({h}x{w} latent), batch {batch}, "
                 f"{qf} query frames on {nf}", ours_us=t_o * 1e6, ref_us=t_r * 1e6,
                 ours_tflops=fl / t_o / 1e12, ref_tflops=fl / t_r / 1e12, speedup=t_r / t_o,
                 max_abs_diff=diff, ref="flashdecoder_wan22._local_attention (Triton forward)")
            del q, k, v, out, ref_out


def case_decoder_step(rows, steps, warmup, h=44, w=80):
    """The FlashDecoder decode step (flashdecoder_wan22.py:759-874) of the
    released S variant (12 backbone + 2 refinement blocks, dim 512), random
    weights, on a 704x1280 stream (44x80 latent grid): the reference's own
    FlashDecoderSession (runtime/flashdecoder.py:54-175; bf16 autocast, eager
    and torch.compile'd as --compile-decoder does) against DecoderSession with
    CUDA-graph replay, per latent frame in the steady state (4 RGB frames out),
    CUDA events; plus the largest RGB difference over the stream."""
    from recavsr_b200.runtime.decoder import DecoderSession
    from recavsr_infer.models.flashdecoder.flashdecoder_wan22 import FlashDecoder
    from recavsr_infer.runtime.flashdecoder import FlashDecoderSession
    torch.manual_seed(0)
    model = FlashDecoder.from_variant("S").cuda().eval()
    g = torch.Generator().manual_seed(1)
    mean, std = torch.randn(48, generator=g) * 0.5, torch.rand(48, generator=g) * 1.5 + 0.5
    model.vae_config = {"latents_mean": mean.tolist(), "latents_std": std.tolist()}
    frames = warmup + steps + 2
    lat = torch.randn(1, 48, frames, h, w, generator=g).cuda()
    lr = (torch.rand(1, 3, 1 + 4 * (frames - 1), 16 * h, 16 * w, generator=g) * 2 - 1).cuda()
    ours = DecoderSession.from_module(model, height=h, width=w, mean=mean, std=std)

    def run(session, capture_at=None):
        outs, times = [], []
        off = 0
        for i in range(frames):
            take = 1 if i == 0 else 4
            if capture_at is not None and i == capture_at:
                session.capture()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            out = next(iter(session.step(lat[:, :, i:i + 1], lr_up=lr[:, :, off:off + take])))
            b.record()
            b.synchronize()
            outs.append(out.float().clone())
            times.append(a.elapsed_time(b) * 1e-3)
            off += take
        return outs, times[warmup + 2:]

    with torch.inference_mode():
        o_out, o_t = run(ours, capture_at=2)
        r_out, r_t = run(FlashDecoderSession(model))
        rc_out, rc_t = run(FlashDecoderSession(model, compile_decoder=True))
    diff = max(float((a - b).abs().max()) for a, b in zip(o_out, r_out))
    mean_diff = max(float((a - b).abs().mean()) for a, b in zip(o_out, r_out))
    t_o, t_r, t_c = (statistics.median(t) for t in (o_t, r_t, rc_t))
    emit(rows, case="decoder_step", geometry=f"{16 * w}x{16 * h} ({h}x{w} latent), S variant (12 + 2 blocks)",
         ours_ms=t_o * 1e3, ref_eager_ms=t_r * 1e3, ref_compiled_ms=t_c * 1e3,
         ours_out_fps=4 / t_o, ref_compiled_out_fps=4 / t_c, speedup_vs_compiled=t_c / t_o,
         speedup_vs_eager=t_r / t_o, max_abs_diff=diff, max_mean_abs_diff=mean_diff,
         ref="recavsr_infer.runtime.flashdecoder.FlashDecoderSession (bf16 autocast)")


def case_colorfix(rows, reps):
    """The colour correction of one body block's output (8 RGB frames at
    704x1280, bf16 from the decoder; LQ 176x320 uint8): the reference's own
    adain_color_fix / wavelet_color_fix (color_fix.py:58-117, torch on the GPU)
    against this library's drop-ins, through the same public calls (the
    wavelet's uint8 result comes back to the host on both sides); wall time per
    call with a device sync, and the device-only wavelet beside it."""
    import numpy as np
    from recavsr_b200.runtime import colorfix as ours
    from recavsr_infer import color_fix as theirs
    g = torch.Generator(device="cuda").manual_seed(5)
    dec = (torch.rand(1, 3, 8, 704, 1280, generator=g, device="cuda") * 2 - 1).bfloat16()
    ref = torch.rand(1, 3, 8, 704, 1280, generator=g, device="cuda") * 2 - 1
    lq = np.random.RandomState(5).randint(0, 256, (8, 176, 320, 3)).astype(np.uint8)
    lq_dev = torch.from_numpy(lq).cuda()

    def wall(fn):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(reps):
            fn()
        torch.cuda.synchronize()
        return (time.perf_counter() - t0) / reps
    a_o, a_r = ours.adain_color_fix(dec, ref), theirs.adain_color_fix(dec, ref)
    w_o, w_r = ours.wavelet_color_fix(dec, lq), theirs.wavelet_color_fix(dec, lq)
    d = np.abs(w_o.astype(np.int16) - w_r.astype(np.int16))
    emit(rows, case="colorfix", step="adain, 8 frames 704x1280", ours_ms=wall(lambda: ours.adain_color_fix(dec, ref)) * 1e3,
         ref_ms=wall(lambda: theirs.adain_color_fix(dec, ref)) * 1e3,
         max_abs_diff=float((a_o - a_r.float()).abs().max()))
    emit(rows, case="colorfix", step="wavelet, 8 frames 704x1280 -> uint8 on the host",
         ours_ms=wall(lambda: ours.wavelet_color_fix(dec, lq)) * 1e3,
         ref_ms=wall(lambda: theirs.wavelet_color_fix(dec, lq)) * 1e3,
         ours_device_ms=graph_time(lambda: ours.wavelet_color_fix_device(dec, lq_dev), reps) * 1e3,
         max_abs_diff=int(d.max()), frac_differing=float((d > 0).mean()))


# ------------------------------------------------------------- the layer loop
class _FP32LayerNorm(nn.LayerNorm):
    """diffusers FP32LayerNorm as the released block uses it (norm1/norm3 without
    affine, norm2 with): layer_norm of x.float(), cast back to x's dtype."""

    def forward(self, x):
        return F.layer_norm(x.float(), self.normalized_shape,
                            None if self.weight is None else self.weight.float(),
                            None if self.bias is None else self.bias.float(), self.eps).to(x.dtype)


class _Attention(nn.Module):
    """The WanAttention attributes PreparedBlock reads (models/transformer_wan.py:515-626)."""

    def __init__(self, dim, heads):
        super().__init__()
        self.to_q, self.to_k, self.to_v = (nn.Linear(dim, dim) for _ in range(3))
        self.to_out = nn.ModuleList([nn.Linear(dim, dim), nn.Dropout(0.0)])
        self.norm_q, self.norm_k = nn.RMSNorm(dim, eps=1e-6), nn.RMSNorm(dim, eps=1e-6)
        self.heads, self.fused_projections = heads, False

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
    """The released DiT block's module layout (models/transformer_wan.py:786-822)."""

    def __init__(self, dim, heads, ffn):
        super().__init__()
        self.norm1 = _FP32LayerNorm(dim, 1e-6, elementwise_affine=False)
        self.attn1 = _Attention(dim, heads)
        self.attn2 = _Attention(dim, heads)
        self.norm2 = _FP32LayerNorm(dim, 1e-6, elementwise_affine=True)
        self.ffn = _FeedForward(dim, ffn)
        self.norm3 = _FP32LayerNorm(dim, 1e-6, elementwise_affine=False)
        self.scale_shift_table = nn.Parameter(torch.randn(1, 6, dim) / dim ** 0.5)


def reference_layers(steps, warmup, compiled=True):
    """The reference's layer loop of TransformerSession.step (runtime/transformer.py:
    311-318) over 30 PreparedBlocks (native norms, NVFP4 linears, compiled as
    :229-246) with the released static router, at 1280x704, random-init weights.
    Returns seconds per body block (device time, CUDA events; the host loop
    included, as the reference runs it)."""
    import bench
    from recavsr_infer.runtime.cache import FixedKVCache
    from recavsr_infer.runtime.nvfp4 import quantize_block_linears
    from recavsr_infer.runtime.rope import RollingRoPE
    from recavsr_infer.runtime.transformer import PreparedBlock
    dim, heads, ffn = bench.DIM, bench.HEADS, bench.FFN
    torch.manual_seed(0)
    rope = RollingRoPE(128, bench.H_TOK, bench.W_TOK, device="cuda")
    enc = torch.randn(1, bench.ENC_LEN, dim, device="cuda").bfloat16()
    cores, eager = [], []
    with torch.no_grad():
        for _ in range(bench.LAYERS):
            b = _Block(dim, heads, ffn).cuda()
            for mod in b.modules():
                if isinstance(mod, nn.Linear):
                    nn.init.normal_(mod.weight, std=0.02)
                    nn.init.normal_(mod.bias, std=0.02)
            b = b.bfloat16()
            cond = types.SimpleNamespace(timestep_proj=torch.randn(1, 1, 6, dim, device="cuda").bfloat16(),
                                         encoder_hidden_states=enc)
            core = PreparedBlock(b, cond, rope, window=(22, 40), native_norms=True).eval()
            quantize_block_linears(b)
            eager.append(core)
    torch._dynamo.config.recompile_limit = 64
    cores = [torch.compile(c, fullgraph=True, dynamic=False, options=_inductor_opts()) if compiled else c
             for c in eager]
    caches = [FixedKVCache(a, initial=5, stride=6, anchors=2) for a in bench.ACTIONS]
    state = {"offset": 0}

    @torch.inference_mode()
    def step(hidden, frames, use):
        origin, positions = rope.positions(state["offset"], frames)
        dummy = hidden.unflatten(2, (heads, -1))
        for core, cache in zip(use, caches):
            history = cache.history(dummy, origin=origin)
            hidden, k, v = core(hidden, *history, positions)
            cache.commit(k, v, frames=frames, start=state["offset"])
        state["offset"] += frames
        return hidden

    g = torch.Generator(device="cuda").manual_seed(99)
    prefix = torch.randn(1, bench.PREFIX * bench.T, dim, generator=g, device="cuda").bfloat16()
    body = torch.randn(1, bench.BODY * bench.T, dim, generator=g, device="cuda").bfloat16()
    step(prefix, bench.PREFIX, eager)                  # warm-up block, uncompiled
    t0 = time.time()
    for _ in range(max(warmup, 3)):
        step(body, bench.BODY, cores)
    torch.cuda.synchronize()
    compile_s = time.time() - t0
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        out = step(body, bench.BODY, cores)
    b.record()
    b.synchronize()
    assert torch.isfinite(out.float()).all()
    return a.elapsed_time(b) * 1e-3 / steps, compile_s


def our_layers(steps, warmup):
    import bench
    stack = bench.build_stack(torch.device("cuda"), seed=1234)
    g = torch.Generator(device="cuda").manual_seed(99)
    stack.step(torch.randn(bench.PREFIX * bench.T, bench.DIM, generator=g, device="cuda").bfloat16(),
               bench.PREFIX)
    body = torch.randn(bench.BODY * bench.T, bench.DIM, generator=g, device="cuda").bfloat16()
    h = body.clone()
    stack.step(h, bench.BODY)
    stack.capture(bench.BODY * bench.T, bench.BODY)
    for _ in range(max(warmup, 3)):
        h.copy_(body)
        stack.step(h, bench.BODY, graphs=True)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        stack.step(h, bench.BODY, graphs=True)
    b.record()
    b.synchronize()
    return a.elapsed_time(b) * 1e-3 / steps


def case_layers(rows, steps, warmup):
    import bench
    tokens = bench.BODY * bench.T
    t_ours = our_layers(steps, warmup)
    torch.cuda.empty_cache()
    t_ref, compile_s = reference_layers(steps, warmup)
    emit(rows, case="layers", geometry="cfg4: 30 layers, 1280x704 (22x40), 2-frame body block, released router",
         ours_ms=t_ours * 1e3, ref_ms=t_ref * 1e3, ours_tokens_s=tokens / t_ours, ref_tokens_s=tokens / t_ref,
         ours_out_fps=tokens / t_ours * 4 / bench.T, ref_out_fps=tokens / t_ref * 4 / bench.T,
         speedup=t_ref / t_ours, ref_warmup_and_compile_s=compile_s,
         ref="PreparedBlock x 30 (native norms, NVFP4Linear, torch.compile fullgraph default mode) + "
             "FixedKVCache, as TransformerSession.step runs them")


# ----------------------------------------------------------- host pipeline
def case_pipeline(rows, reps):
    """One body block (8 LQ frames) to the model input, from uint8 frames in
    pinned host memory: the reference's prepare_block (video.py:138-150: CPU
    cv2.resize of every frame into a pinned buffer, its upload, block_tensor on
    the GPU) next to recavsr_b200.runtime.pipeline (upload of the LQ frames,
    one rc_enlarge_block launch); wall time per block, host included, with a
    device sync per block. Then one blended 1920x1080 frame from 4 strips: the
    reference's CPU canvas loop (strips.py:85-97) next to rc_strip_blend
    (device frames; device time)."""
    import numpy as np
    from recavsr_b200.runtime import pipeline as ours
    from recavsr_infer import strips as ref_strips
    from recavsr_infer import video as ref_video
    rs = np.random.RandomState(0)
    for (h, w) in ((176, 320), (270, 480)):
        lq = rs.randint(0, 256, (8, h, w, 3)).astype(np.uint8)
        lq_pinned = torch.from_numpy(lq).pin_memory()
        size = ref_video.scaled_size(h, w, 4.0)

        def theirs():
            x = ref_video.enlarge_block(lq, size, block=8, pin=True)
            return ref_video.block_tensor(x, 8, device="cuda")

        def mine():
            return ours.enlarge_block(lq_pinned.to("cuda", non_blocking=True), size, block=8)
        r, o = theirs(), mine()
        torch.cuda.synchronize()
        equal = bool(torch.equal(r, o))

        def wall(fn):
            for _ in range(2):
                fn()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            for _ in range(reps):
                fn()
                torch.cuda.synchronize()
            return (time.perf_counter() - t0) / reps
        t_r, t_o = wall(theirs), wall(mine)
        dev = lq_pinned.cuda()
        t_k = graph_time(lambda: ours.enlarge_block(dev, size, block=8), reps)
        out_bytes = 3 * 8 * (-(-size[0] // 32) * 32) * size[1] * 4
        emit(rows, case="pipeline", step=f"prepare_block 8 frames {w}x{h} -> {size[1]}x{size[0]} fp32",
             ours_ms=t_o * 1e3, ref_ms=t_r * 1e3, speedup=t_r / t_o, outputs_equal=equal,
             kernel_us=t_k * 1e6, kernel_gbs=(out_bytes + lq.nbytes) / t_k / 1e9,
             ref="recavsr_infer.video.enlarge_block (cv2, CPU) + block_tensor (torch, GPU)")
    cols = ref_strips.strip_columns(480, 4, 48, 4.0)
    width = 1920
    weights = ref_strips.column_weights(cols, 4.0, width)
    frames = [rs.randint(0, 256, (1080, len(w), 3)).astype(np.uint8) for _, w in weights]
    total = np.zeros(width, dtype=np.float32)
    for o0, w in weights:
        total[o0:o0 + len(w)] += w

    def ref_blend():
        canvas = np.zeros((1080, width, 3), dtype=np.float32)
        for f, (o0, w) in zip(frames, weights):
            canvas[:, o0:o0 + len(w)] += f * w[None, :, None]
        canvas /= total[None, :, None]
        return np.clip(canvas + 0.5, 0, 255).astype(np.uint8)
    t0 = time.perf_counter()
    for _ in range(reps):
        want = ref_blend()
    t_r = (time.perf_counter() - t0) / reps
    blender = ours.StripBlender(cols, 4.0, 1080, width, device="cuda")
    dframes = [torch.from_numpy(f).cuda() for f in frames]
    got = blender.blend(dframes)
    t_o = graph_time(lambda: blender.blend(dframes), reps)
    emit(rows, case="pipeline", step="strip blend, 4 strips -> 1920x1080 uint8", ours_us=t_o * 1e6,
         ref_us=t_r * 1e6, speedup=t_r / t_o, outputs_equal=bool(np.array_equal(got.cpu().numpy(), want)),
         ref="the canvas loop of recavsr_infer.strips.blend_strips (numpy, CPU)")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["gemm", "attention", "local", "layers", "pipeline", "decoder", "decoder_step",
                                     "colorfix", "all"])
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    args = ap.parse_args()
    install_reference()
    sys.modules.setdefault("av", types.ModuleType("av"))   # PyAV only opens video files; not needed here
    torch.cuda.set_device(0)
    torch._dynamo.config.recompile_limit = 64     # one compiled graph per shape, as the reference allows
    rows = []
    todo = (["gemm", "attention", "local", "layers", "pipeline", "decoder", "decoder_step", "colorfix"]
            if args.case == "all" else [args.case])
    for c in todo:
        if c == "gemm":
            case_gemm(rows, args.reps)
        elif c == "attention":
            case_attention(rows, args.reps)
        elif c == "local":
            case_local(rows, args.reps)
        elif c == "pipeline":
            case_pipeline(rows, args.reps)
        elif c == "decoder":
            case_decoder(rows, args.reps)
        elif c == "decoder_step":
            case_decoder_step(rows, args.steps, args.warmup)
        elif c == "colorfix":
            case_colorfix(rows, args.reps)
        else:
            case_layers(rows, args.steps, args.warmup)
        torch.cuda.empty_cache()
    from recavsr_b200 import _lib
    if _lib.read_device_error():
        raise SystemExit("device error word set")


if __name__ == "__main__":
    main()
