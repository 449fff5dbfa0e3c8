"""Run one hot-path kernel at the benchmark's shapes, for profiling.

    python -m recavsr_b200.profile_case gemm_up      # NVFP4 ffn_up 1760x14336x3072 (+GELU/NVFP4 epilogue)
    python -m recavsr_b200.profile_case gemm_qkv     # NVFP4 QKV 1760x9216x3072
    python -m recavsr_b200.profile_case gemm_down    # NVFP4 ffn_down 1760x3072x14336 (+gated residual)
    python -m recavsr_b200.profile_case attention    # routed attention, 1760 queries, 4 past planes
    python -m recavsr_b200.profile_case quant        # NVFP4 quantizer 1760x3072
    python -m recavsr_b200.profile_case ln           # LayerNorm+AdaLN+NVFP4 1760x3072
    python -m recavsr_b200.profile_case rms          # RMSNorm+spatial RoPE of q and k, 1760x3072 each
    python -m recavsr_b200.profile_case gemm_sweep   # NVFP4 / FP8 linears, M x (K, N) sweep + quantizers
    python -m recavsr_b200.profile_case attention_sweep  # 30-layer routed attention, scopes 0/1/2/4/8
    python -m recavsr_b200.profile_case lq_conv1     # LQ projector conv1: im2col + bf16 GEMM, body block
    python -m recavsr_b200.profile_case lq_conv2     # LQ projector conv2: im2col + bf16 GEMM, body block
    python -m recavsr_b200.profile_case lq_norm      # channel RMSNorm + SiLU, 14080 x 2048
    python -m recavsr_b200.profile_case gemm_vs_cublas   # NVFP4 GEMM vs the reference's _scaled_mm_v2 (cuBLASLt)

Each case allocates fresh inputs (a few hundred MB at most), captures `--reps`
launches in a CUDA graph, replays it and prints the mean CUDA-event time per
launch (inputs stay L2-resident between launches, as in the layer loop).
"""
from __future__ import annotations

import argparse
import ctypes as C

import torch

from . import _lib
from .runtime.ops import quantize, scale_numel

M, DIM, FFN, HEADS, HD, H, W = 1760, 3072, 14336, 24, 128, 22, 40


def _gemm(n, k, epi):
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    a = torch.randn(M, k, generator=g, device="cuda").bfloat16()
    w = (torch.randn(n, k, generator=g, device="cuda") * 0.02).bfloat16()
    ac, asf = quantize(a)
    wc, wsf = quantize(w)
    bias = torch.zeros(n, dtype=torch.bfloat16, device="cuda")
    out = torch.randn(M, n, generator=g, device="cuda").bfloat16()
    gate = torch.ones(n, device="cuda")
    qc = torch.empty(M, n // 2, dtype=torch.uint8, device="cuda")
    qs = torch.empty(scale_numel(M, n), dtype=torch.uint8, device="cuda")
    lib = _lib.library()
    sws = torch.zeros(lib.rc_gemm_split_workspace(), dtype=torch.uint8, device="cuda")

    def run():
        _lib.check(lib.rc_nvfp4_gemm_ws(ac.data_ptr(), asf.data_ptr(), wc.data_ptr(), wsf.data_ptr(),
                                        bias.data_ptr(), M, n, k, 1.0, epi,
                                        None if epi == _lib.EPI_GELU_NVFP4 else out.data_ptr(), n,
                                        gate.data_ptr(), qc.data_ptr(), qs.data_ptr(), 1.0,
                                        sws.data_ptr(), sws.numel(), _lib.stream()), "gemm")
    return run, 2.0 * M * n * k, "TFLOP/s"


def _attention(planes=4, h=H, w=W, window=None):
    """Routed attention of a 2-frame query block over `planes` routed planes
    plus the 2 current frames; window None = the grid (the sdpa path), else
    (wh, ww) local windows. FLOPs count visible keys only."""
    from .runtime.ops import routed_attention
    from .runtime.block import rope_tables
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    t = h * w
    wh, ww = window if window else (h, w)
    r = lambda *s: torch.randn(*s, generator=g, device="cuda").bfloat16()
    q, k, v = r(1, 2 * t, HEADS, HD), r(1, 2 * t, HEADS, HD), r(1, 2 * t, HEADS, HD)
    pk, pv = r(1, planes * t, HEADS, HD), r(1, planes * t, HEADS, HD)
    slots = torch.arange(planes, dtype=torch.int32, device="cuda")
    ppos = torch.arange(planes, dtype=torch.int32, device="cuda")
    qpos = torch.tensor([planes, planes + 1], dtype=torch.int32, device="cuda")
    tb = rope_tables(HD, h, w, "cuda")
    out = torch.empty_like(q)

    def run():
        routed_attention(q, k, v, pk, pv, slots, ppos, qpos, tb["temporal_cos"], tb["temporal_sin"],
                         h, w, wh, ww, out=out)
    keys = min(h, wh) * min(w, ww)          # per query and visible plane
    return run, 4.0 * HD * HEADS * (2 * t) * keys * (planes + 2), "TFLOP/s"


def _quant():
    x = torch.randn(M, DIM, device="cuda").bfloat16()
    codes = torch.empty(M, DIM // 2, dtype=torch.uint8, device="cuda")
    sf = torch.empty(scale_numel(M, DIM), dtype=torch.uint8, device="cuda")
    lib = _lib.library()

    def run():
        _lib.check(lib.rc_nvfp4_quantize(x.data_ptr(), M, DIM, DIM, 1.0, codes.data_ptr(), sf.data_ptr(),
                                         _lib.stream()), "quant")
    return run, M * DIM * 2.5625, "GB/s"


def _quant_fp8(m=M, k=DIM):
    """Per-tensor FP8 quantizer (amax pass + quantize pass); GB/s of
    algorithmic bytes (bf16 in once, e4m3 out)."""
    x = torch.randn(m, k, device="cuda").bfloat16()
    q = torch.empty(m, k, dtype=torch.uint8, device="cuda")
    scratch = torch.empty(2, dtype=torch.int32, device="cuda")
    scale = torch.empty((), dtype=torch.float32, device="cuda")
    lib = _lib.library()

    def run():
        _lib.check(lib.rc_fp8_quantize(x.data_ptr(), m, k, k, scratch.data_ptr(), scale.data_ptr(),
                                       q.data_ptr(), _lib.stream()), "quant_fp8")
    return run, m * k * 3.0, "GB/s"


def _ln():
    x = torch.randn(M, DIM, device="cuda").bfloat16()
    sh, sc = torch.randn(DIM, device="cuda"), torch.randn(DIM, device="cuda")
    codes = torch.empty(M, DIM // 2, dtype=torch.uint8, device="cuda")
    sf = torch.empty(scale_numel(M, DIM), dtype=torch.uint8, device="cuda")
    lib = _lib.library()

    def run():
        _lib.check(lib.rc_ln_modulate_quant(x.data_ptr(), DIM, M, DIM, None, None, sh.data_ptr(),
                                            sc.data_ptr(), 1e-6, None, 0, codes.data_ptr(),
                                            sf.data_ptr(), 1.0, _lib.stream()), "ln")
    return run, M * DIM * 2.5625, "GB/s"


def _rms():
    qkv = torch.randn(M, 3 * DIM, device="cuda").bfloat16()
    wq, wk = torch.rand(DIM, device="cuda").bfloat16(), torch.rand(DIM, device="cuda").bfloat16()
    q_rot, k_rot = (torch.empty(M, DIM, dtype=torch.bfloat16, device="cuda") for _ in range(2))
    cos, sin = (torch.rand(H * W, HD, device="cuda") for _ in range(2))
    lib = _lib.library()

    def run():
        _lib.check(lib.rc_rmsnorm_rope(2, (C.c_void_p * 2)(qkv.data_ptr(), qkv[:, DIM:].data_ptr()),
                                       (C.c_longlong * 2)(3 * DIM, 3 * DIM),
                                       (C.c_void_p * 2)(wq.data_ptr(), wk.data_ptr()),
                                       (C.c_void_p * 2)(q_rot.data_ptr(), k_rot.data_ptr()),
                                       (C.c_longlong * 2)(DIM, DIM), M, DIM, HD, H * W,
                                       cos.data_ptr(), sin.data_ptr(), 1e-6, _lib.stream()), "rms")
    return run, 2 * M * DIM * 4, "GB/s"


def _cross_attention(nk=512):
    """Cross-attention of the body block over the prompt keys, NVFP4 output
    (as the block runs it), with the tail-split workspace."""
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    r = lambda *sh: torch.randn(*sh, generator=g, device="cuda").bfloat16()
    q, k, v = r(M, HEADS, HD), r(nk, HEADS, HD), r(nk, HEADS, HD)
    dim = HEADS * HD
    codes = torch.empty(M, dim // 2, dtype=torch.uint8, device="cuda")
    sf = torch.empty(scale_numel(M, dim), dtype=torch.uint8, device="cuda")
    lib = _lib.library()
    ws = torch.zeros(lib.rc_cross_attention_workspace(), dtype=torch.uint8, device="cuda")
    st = (C.c_longlong * 9)(0, dim, HD, 0, dim, HD, 0, dim, HD)

    def run():
        _lib.check(lib.rc_cross_attention_ws(q.data_ptr(), k.data_ptr(), v.data_ptr(), st, 1, M, nk, HEADS,
                                             HD, None, dim, codes.data_ptr(), sf.data_ptr(), ws.data_ptr(),
                                             ws.numel(), _lib.stream()), "cross")
    return run, 4.0 * HD * HEADS * M * nk, "TFLOP/s"


def _lq_conv(which):
    """One body block of the LQ projector's causal Conv3d at 1280x704 (the
    frames a body chunk reads): conv1 = im2col of 16x16-unshuffled RGB
    (10 frames -> 4 outputs of 44 x 80) + bf16 GEMM 14080 x 2048 x 27648;
    conv2 = im2col of conv1's channels-last output (6 frames -> 2 outputs of
    22 x 40) + bf16 GEMM 1760 x 3072 x 73728. Time covers both launches."""
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    lib = _lib.library()
    if which == 1:
        src = torch.randn(3, 10, 704, 1280, generator=g, device="cuda").bfloat16()
        cin, cout, fin, hin, win, ss, fout = 768, 2048, 10, 44, 80, 1, 4
        strides = (704 * 1280, 10 * 704 * 1280, 1280, 0, 16)
    else:
        src = torch.randn(6, 44, 80, 2048, generator=g, device="cuda").bfloat16()
        cin, cout, fin, hin, win, ss, fout = 2048, 3072, 6, 44, 80, 2, 2
        strides = (44 * 80 * 2048, 0, 80 * 2048, 2048, 0)
    ho, wo = (hin - 1) // ss + 1, (win - 1) // ss + 1
    rows, k = fout * ho * wo, 36 * cin
    cols = torch.empty(rows, k, dtype=torch.bfloat16, device="cuda")
    w = (torch.randn(cout, k, generator=g, device="cuda") * 0.02).bfloat16()
    bias = torch.zeros(cout, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(rows, cout, dtype=torch.bfloat16, device="cuda")

    def run():
        _lib.check(lib.rc_conv3d_im2col(src.data_ptr(), *strides, cin, fin, hin, win, 2, ss, fout,
                                        cols.data_ptr(), k, _lib.stream()), "im2col")
        _lib.check(lib.rc_bf16_gemm(cols.data_ptr(), w.data_ptr(), bias.data_ptr(), rows, cout, k,
                                    _lib.EPI_BIAS, out.data_ptr(), cout, None, _lib.stream()), "gemm")
    return run, 2.0 * rows * cout * k, "TFLOP/s"


def _lq_norm():
    """Channel RMSNorm + SiLU in place on conv1's body-block output (14080 x 2048)."""
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    x = torch.randn(14080, 2048, generator=g, device="cuda").bfloat16()
    w = torch.ones(2048, dtype=torch.bfloat16, device="cuda")
    lib = _lib.library()

    def run():
        _lib.check(lib.rc_channel_rmsnorm_silu(x.data_ptr(), 2048, 14080, 2048, w.data_ptr(), 1e-6,
                                               x.data_ptr(), 2048, _lib.stream()), "rmsnorm_silu")
    return run, 2.0 * 2 * 14080 * 2048, "GB/s"


CASES = {
    "lq_conv1": lambda: _lq_conv(1),
    "lq_conv2": lambda: _lq_conv(2),
    "lq_norm": _lq_norm,
    "gemm_up": lambda: _gemm(FFN, DIM, _lib.EPI_GELU_NVFP4),
    "gemm_qkv": lambda: _gemm(3 * DIM, DIM, _lib.EPI_BIAS),
    "gemm_o": lambda: _gemm(DIM, DIM, _lib.EPI_GATED_RESIDUAL),
    "gemm_cq": lambda: _gemm(DIM, DIM, _lib.EPI_BIAS),
    "gemm_down": lambda: _gemm(DIM, FFN, _lib.EPI_GATED_RESIDUAL),
    "attention": _attention,
    # cfg5 stream: 1080p output (34 x 60 tokens), 22 x 40 local windows
    "attention_local_1080p": lambda: _attention(planes=4, h=34, w=60, window=(22, 40)),
    "cross_attention": _cross_attention,
    "quant": _quant,
    "quant_fp8": _quant_fp8,
    "quant_fp8_large": lambda: _quant_fp8(7040, 14336),
    "ln": _ln,
    "rms": _rms,
}


def _graph_time(run, reps):
    """Mean device time per call of `run`, replayed from a CUDA graph."""
    for _ in range(3):
        run()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph, stream=side):
            for _ in range(reps):
                run()
    torch.cuda.current_stream().wait_stream(side)
    graph.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    graph.replay()
    b.record()
    b.synchronize()
    return a.elapsed_time(b) / reps * 1e-3


def _cfg3_operands(m, n, k, g):
    """Activation N(0,1) with 0.1% of the entries x20 (outliers), weight N(0, 0.02)."""
    a = torch.randn(m, k, generator=g, device="cuda")
    mask = torch.rand(m, k, generator=g, device="cuda") < 1e-3
    a = torch.where(mask, a * 20, a).bfloat16()
    w = (torch.randn(n, k, generator=g, device="cuda") * 0.02).bfloat16()
    return a, w


def gemm_sweep(reps=10):
    """NVFP4 / FP8 linear sweep: M in {1760, 3520, 7040} x (K, N) in {(3072, 3072),
    (3072, 14336), (14336, 3072)}, bias epilogue, plus the NVFP4 and FP8
    quantizers on the activation (GB/s of algorithmic bytes)."""
    from .runtime import fp8
    lib = _lib.library()
    g = torch.Generator(device="cuda")
    g.manual_seed(2)
    print("path   M     K      N      us       TFLOP/s  | quant us  GB/s")
    for m in (1760, 3520, 7040):
        for k, n in ((3072, 3072), (3072, 14336), (14336, 3072)):
            a, w = _cfg3_operands(m, n, k, g)
            bias = torch.zeros(n, dtype=torch.bfloat16, device="cuda")
            out = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
            ac, asf = quantize(a)
            wc, wsf = quantize(w)

            def nvf4():
                _lib.check(lib.rc_nvfp4_gemm(ac.data_ptr(), asf.data_ptr(), wc.data_ptr(), wsf.data_ptr(),
                                             bias.data_ptr(), m, n, k, 1.0, _lib.EPI_BIAS, out.data_ptr(), n,
                                             None, None, None, 1.0, _lib.stream()), "nvfp4_gemm")

            def nvf4_quant():
                quantize(a)
            t = _graph_time(nvf4, reps)
            tq = _graph_time(nvf4_quant, reps)
            print(f"nvfp4 {m:5d} {k:6d} {n:6d} {t * 1e6:8.1f} {2.0 * m * n * k / t / 1e12:9.1f}"
                  f"  | {tq * 1e6:7.1f} {m * k * 2.5625 / tq / 1e9:7.1f}")
            aq, sa = fp8.quantize(a)
            wq, sw = fp8.quantize(w)

            def f8():
                _lib.check(lib.rc_fp8_gemm(aq.data_ptr(), sa.data_ptr(), wq.data_ptr(), sw.data_ptr(),
                                           bias.data_ptr(), m, n, k, 1.0, _lib.EPI_BIAS, out.data_ptr(), n,
                                           None, _lib.stream()), "fp8_gemm")

            def f8_quant():
                fp8.quantize(a)
            t = _graph_time(f8, reps)
            tq = _graph_time(f8_quant, reps)
            print(f"fp8   {m:5d} {k:6d} {n:6d} {t * 1e6:8.1f} {2.0 * m * n * k / t / 1e12:9.1f}"
                  f"  | {tq * 1e6:7.1f} {m * k * 3.0 / tq / 1e9:7.1f}")
            del a, w, ac, asf, wc, wsf, aq, wq, out


def gemm_vs_cublas(reps=10):
    """The reference's own NVFP4 GEMM call (recavsr_infer/runtime/nvfp4.py:22-39:
    torch._scaled_mm_v2, BlockWise1x16 scales in the 32x4x4 swizzle, bias, bf16
    out -- cuBLASLt) next to rc_nvfp4_gemm on the same codes and scales (the
    quantizer's output is byte-identical to the reference's), cfg3 shapes; also
    the largest difference between the two outputs relative to max |cuBLAS|."""
    lib = _lib.library()
    if not hasattr(torch, "_scaled_mm_v2") or not hasattr(torch, "float4_e2m1fn_x2"):
        raise SystemExit("this torch has no _scaled_mm_v2 / float4_e2m1fn_x2")
    g = torch.Generator(device="cuda")
    g.manual_seed(2)
    print("M     K      N      ours us  TFLOP/s | cuBLAS us  TFLOP/s | ours/cuBLAS time  max diff")
    for m in (1760, 3520, 7040):
        for k, n in ((3072, 3072), (3072, 14336), (14336, 3072)):
            a, w = _cfg3_operands(m, n, k, g)
            bias = (torch.randn(n, generator=g, device="cuda") * 0.02).bfloat16()
            out = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
            ac, asf = quantize(a)
            wc, wsf = quantize(w)

            def ours():
                _lib.check(lib.rc_nvfp4_gemm(ac.data_ptr(), asf.data_ptr(), wc.data_ptr(), wsf.data_ptr(),
                                             bias.data_ptr(), m, n, k, 1.0, _lib.EPI_BIAS, out.data_ptr(), n,
                                             None, None, None, 1.0, _lib.stream()), "nvfp4_gemm")

            def cublas():
                return torch._scaled_mm_v2(
                    ac.view(torch.float4_e2m1fn_x2), wc.view(torch.float4_e2m1fn_x2).t(),
                    [asf.view(torch.float8_e4m3fn)], [2], [1], [wsf.view(torch.float8_e4m3fn)], [2], [1],
                    bias, torch.bfloat16)
            ref = cublas()
            ours()
            torch.cuda.synchronize()
            diff = float((out.float() - ref.float()).abs().max() / ref.float().abs().max())
            t, tc = _graph_time(ours, reps), _graph_time(cublas, reps)
            fl = 2.0 * m * n * k
            print(f"{m:5d} {k:6d} {n:6d} {t * 1e6:8.1f} {fl / t / 1e12:8.1f} | {tc * 1e6:8.1f} "
                  f"{fl / tc / 1e12:8.1f} | {t / tc:6.3f}  {diff:.2e}")
            del a, w, ac, asf, wc, wsf, out, ref


def attention_sweep(reps=5):
    """Routed-attention microbenchmark: 30 layers x 24 heads x 128, T = 880
    (22 x 40), 2-frame query block (1760 queries), layer i attends to
    [0, 1, 2, 4, 8][i % 5] routed planes of an 8-plane ring plus the 2 current
    frames; FLOPs count visible keys only: 4 d heads Nq T sum(scope + 2)."""
    from .runtime.ops import routed_attention
    from .runtime.block import rope_tables
    g = torch.Generator(device="cuda")
    g.manual_seed(1)
    t = H * W
    r = lambda *sh: (torch.randn(*sh, generator=g, device="cuda") / HD ** 0.5).bfloat16()
    q, k, v = r(1, 2 * t, HEADS, HD), r(1, 2 * t, HEADS, HD), r(1, 2 * t, HEADS, HD)
    ring_k, ring_v = r(1, 8 * t, HEADS, HD), r(1, 8 * t, HEADS, HD)
    tb = rope_tables(HD, H, W, "cuda")
    out = torch.empty_like(q)
    calls = []
    for layer in range(30):
        scope = (0, 1, 2, 4, 8)[layer % 5]
        slots = torch.full((8,), -1, dtype=torch.int32, device="cuda")
        slots[:scope] = torch.arange(8 - scope, 8, dtype=torch.int32, device="cuda")
        ppos = torch.zeros(8, dtype=torch.int32, device="cuda")
        ppos[:scope] = torch.arange(12 - scope, 12, dtype=torch.int32, device="cuda")
        calls.append((slots, ppos))
    qpos = torch.tensor([12, 13], dtype=torch.int32, device="cuda")

    def run():
        for slots, ppos in calls:
            routed_attention(q, k, v, ring_k, ring_v, slots, ppos, qpos, tb["temporal_cos"],
                             tb["temporal_sin"], H, W, H, W, out=out)
    flops = 4.0 * HD * HEADS * (2 * t) * t * sum((0, 1, 2, 4, 8)[i % 5] + 2 for i in range(30))
    dt = _graph_time(run, reps)
    print(f"attention sweep: {dt * 1e3:.3f} ms per 30-layer block, {flops / dt / 1e12:.1f} TFLOP/s "
          f"({flops:.3e} FLOP, {flops / (2 * t):.3e} FLOP/token)")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=sorted(CASES) + ["gemm_sweep", "attention_sweep", "gemm_vs_cublas"])
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--seconds", type=float, default=0.0,
                    help="also replay for this long and report the sustained per-launch time "
                         "(sample clocks / power alongside to see the power cap)")
    args = ap.parse_args()
    if args.case == "gemm_sweep":
        return gemm_sweep()
    if args.case == "attention_sweep":
        return attention_sweep()
    if args.case == "gemm_vs_cublas":
        return gemm_vs_cublas()
    run, work, unit = CASES[args.case]()
    for _ in range(3):
        run()
    torch.cuda.synchronize()
    # Replay the launches from a CUDA graph so host launch overhead stays out
    # of the per-launch device time.
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph, stream=side):
            for _ in range(args.reps):
                run()
    torch.cuda.current_stream().wait_stream(side)
    graph.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    graph.replay()
    b.record()
    b.synchronize()
    dt = a.elapsed_time(b) / args.reps * 1e-3
    rate = work / dt / (1e12 if unit == "TFLOP/s" else 1e9)
    print(f"{args.case}: {dt * 1e6:.1f} us/launch, {rate:.1f} {unit}")
    if args.seconds > 0:
        n = max(1, int(args.seconds / (dt * args.reps)))
        a.record()
        for _ in range(n):
            graph.replay()
        b.record()
        b.synchronize()
        ds = a.elapsed_time(b) / (n * args.reps) * 1e-3
        rs = work / ds / (1e12 if unit == "TFLOP/s" else 1e9)
        print(f"{args.case} sustained {a.elapsed_time(b) / 1e3:.1f} s: {ds * 1e6:.1f} us/launch, {rs:.1f} {unit}")
    if _lib.read_device_error():
        raise SystemExit("device error word set")


if __name__ == "__main__":
    main()
