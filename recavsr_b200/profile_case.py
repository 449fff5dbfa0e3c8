"""Run one hot-path kernel at the benchmark's shapes, for profiling.

    python -m recavsr_b200.profile_case gemm_up      # NVFP4 ffn_up 1760x14336x3072 (+GELU/NVFP4 epilogue)
    python -m recavsr_b200.profile_case gemm_qkv     # NVFP4 QKV 1760x9216x3072
    python -m recavsr_b200.profile_case gemm_down    # NVFP4 ffn_down 1760x3072x14336 (+gated residual)
    python -m recavsr_b200.profile_case attention    # routed attention, 1760 queries, 4 past planes
    python -m recavsr_b200.profile_case quant        # NVFP4 quantizer 1760x3072
    python -m recavsr_b200.profile_case ln           # LayerNorm+AdaLN+NVFP4 1760x3072
    python -m recavsr_b200.profile_case rms          # RMSNorm+spatial RoPE of q and k, 1760x3072 each
    python -m recavsr_b200.profile_case gemm_cfg3_long_k   # NVFP4 7040x3072x14336 (CTA-pair tiles)
    python -m recavsr_b200.profile_case decoder      # FlashDecoder local GQA attention, 704x1280 refinement step
    python -m recavsr_b200.profile_case decoder_step # one FlashDecoder-S decode step at 704x1280 (eager launches)
    python -m recavsr_b200.profile_case lq_conv1     # LQ projector conv1: im2col + bf16 GEMM, body block
    python -m recavsr_b200.profile_case lq_conv2     # LQ projector conv2: im2col + bf16 GEMM, body block
    python -m recavsr_b200.profile_case lq_norm      # channel RMSNorm + SiLU, 14080 x 2048

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


def _gemm(n, k, epi, m=M):
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    a = torch.randn(m, k, generator=g, device="cuda").bfloat16()
    w = (torch.randn(n, k, generator=g, device="cuda") * 0.02).bfloat16()
    ac, asf = quantize(a)
    wc, wsf = quantize(w)
    bias = torch.zeros(n, dtype=torch.bfloat16, device="cuda")
    out = torch.randn(m, n, generator=g, device="cuda").bfloat16()
    gate = torch.ones(n, device="cuda")
    qc = torch.empty(m, n // 2, dtype=torch.uint8, device="cuda")
    qs = torch.empty(scale_numel(m, n), dtype=torch.uint8, device="cuda")
    lib = _lib.library()
    sws = torch.zeros(lib.rc_gemm_split_workspace(), dtype=torch.uint8, device="cuda")

    def run():
        _lib.check(lib.rc_nvfp4_gemm_ws(ac.data_ptr(), asf.data_ptr(), wc.data_ptr(), wsf.data_ptr(),
                                        bias.data_ptr(), m, n, k, 1.0, epi,
                                        None if epi == _lib.EPI_GELU_NVFP4 else out.data_ptr(), n,
                                        gate.data_ptr(), qc.data_ptr(), qs.data_ptr(), 1.0,
                                        sws.data_ptr(), sws.numel(), _lib.stream()), "gemm")
    return run, 2.0 * m * n * k, "TFLOP/s"


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


def _decoder(h=44, w=80, qf=4, nf=8, batch=1):
    """FlashDecoder local attention (8 query heads on 2 KV heads, head_dim
    64, 24x24 window, groups of qf frames, 2 groups visible), bf16."""
    from .runtime.flashdecoder import local_attention
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    n = h * w
    q = torch.randn(batch, 8, qf * n, 64, generator=g, device="cuda").bfloat16()
    k = torch.randn(batch, 2, nf * n, 64, generator=g, device="cuda").bfloat16()
    v = torch.randn(batch, 2, nf * n, 64, generator=g, device="cuda").bfloat16()
    kw = dict(height=h, width=w, window=(24, 24), group_size=qf, temporal_window=2)

    def axis(size):
        d = torch.arange(size)[:, None] - torch.arange(size)[None, :]
        return int(((d >= -12) & (d < 12)).sum())
    frames = sum(min(nf, ((t + nf - qf) // qf + 1) * qf) - max(0, ((t + nf - qf) // qf - 1) * qf)
                 for t in range(qf))
    return (lambda: local_attention(q, k, v, **kw)), 4.0 * 64 * 8 * batch * frames * axis(h) * axis(w), "TFLOP/s"


def _decoder_step(h=44, w=80):
    """One steady-state FlashDecoder-S decode step (12 + 2 blocks, random
    weights) at a 44x80 latent grid, launched eagerly (one unit = one latent
    frame, 0.91 TFLOP)."""
    from .runtime.decoder import DecoderSession, random_params
    dev = torch.device("cuda", torch.cuda.current_device())
    sess = DecoderSession(random_params(dev, 0), height=h, width=w, mean=torch.zeros(48), std=torch.ones(48),
                          device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(1)
    lat = torch.randn(1, 48, 1, h, w, generator=g, device=dev)
    lr1 = torch.rand(1, 3, 1, 16 * h, 16 * w, generator=g, device=dev) * 2 - 1
    lr4 = torch.rand(1, 3, 4, 16 * h, 16 * w, generator=g, device=dev) * 2 - 1
    list(sess.step(lat, lr_up=lr1))
    for _ in range(2):
        list(sess.step(lat, lr_up=lr4))
    return (lambda: list(sess.step(lat, lr_up=lr4))), 0.91e12, "TFLOP/s"


CASES = {
    "decoder": _decoder,
    "decoder_step": _decoder_step,
    "decoder_backbone": lambda: _decoder(qf=1, nf=2),
    "gemm_cfg3_long_k": lambda: _gemm(DIM, FFN, _lib.EPI_BIAS, m=7040),
    "gemm_cfg3_wide_n": lambda: _gemm(FFN, DIM, _lib.EPI_BIAS, m=7040),
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=sorted(CASES))
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--seconds", type=float, default=0.0,
                    help="also replay for this long and report the sustained per-launch time "
                         "(sample clocks / power alongside to see the power cap)")
    args = ap.parse_args()
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
