"""Benchmark: DiT latent tokens/s of the ReCaVSR hot path on B200.

Workload (the 720p x4 streaming configuration): the 30-layer streaming DiT
layer loop (routed self-attention over the released static KV router, cross
attention over 512 prompt tokens, NVFP4 linears, modulation / LayerNorm /
RMSNorm / RoPE glue, KV-cache commit) on 1280x704 output = 22x40 latent
tokens per frame (T = 880), body blocks of 2 latent frames (1760 tokens).
Random-init weights of the released architecture (dim 3072, 24 heads x 128,
FFN 14336), synthetic N(0,1) hidden states, prompt states and timestep
projection. One step = one body block through all 30 layers; the 6-frame
prefix block and enough body blocks to fill every layer's cache run as
warm-up. Inputs/weights/caches (~4 GB) exceed L2 (126 MB), so no flush.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference] [--head-shard | --session]

The default line also times, per stream, the whole one-step DiT step through
its host-buffer entry (`e2e`, `out_fps`) and the whole pipeline of a body
block (`pipeline`: LQ uint8 frames in -> enlarge -> DiT step -> FlashDecoder ->
RGB frames out, the "720p x4 out frames/s" of the metric).

Under torchrun each rank runs an independent stream (weak scaling, no
collective); rank 0 prints one JSON line with the max-over-ranks time.
--head-shard instead runs one 3840x2176 stream split by heads over the ranks
(NCCL all-to-all at the attention boundary; strong scaling); --session times the
whole one-step DiT stream step (LQ projector, patch embedding, layers, head).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

DIM, HEADS, HEAD_DIM, FFN, LAYERS = 3072, 24, 128, 14336, 30
H_TOK, W_TOK = 22, 40                  # 1280x704 / 32
T = H_TOK * W_TOK
BODY, PREFIX = 2, 6
ENC_LEN = 512
# Layer actions of the released static KV router (checkpoints/model_config.json).
ACTIONS = ["none", "none", "recent_1", "none", "recent_2", "none", "recent_2", "recent_4", "none",
           "recent_2_anchor", "recent_4", "recent_4_anchor", "recent_2", "recent_4_anchor", "anchor",
           "recent_4_anchor", "recent_2", "recent_4_anchor", "recent_2_anchor", "recent_4", "recent_2",
           "none", "recent_2_anchor", "recent_2", "none", "recent_2", "none", "recent_1", "none", "none"]
METRIC = "DiT latent tokens/s/GPU (routed attn+NVFP4 linears); 720p x4 out frames/s"

# DRAM bytes per launch of the roofline kernels (dram__bytes_read.sum +
# dram__bytes_write.sum, one ncu capture of the same shapes through
# `python -m recavsr_b200.profile_case gemm_up|attention`); a profiler figure,
# not measured by this script.
PROFILED_DRAM = {
    "ffn_up": {"read": 28039936, "write": 129280,
               "source": "ncu on profile_case gemm_up (1760x14336x3072, GELU+NVFP4 epilogue, 256x256 CTA-pair tiles)"},
    "attention": {"read": 75758080, "write": 2477824,
                  "source": "ncu on profile_case attention (1760 queries, 4 routed + 2 current planes)"},
}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            m = json.load(f)
        return m["hbm_gbs"], m["bf16_tflops"], m.get("bf16_tflops_sustained", m["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, 1400.0, "fallback"


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """SM clock, power and clock-event reasons sampled during the timed region:
    NVML read every 10 ms from a thread (read-only queries; the GPU is found
    by the PCI bus id of the torch device, so CUDA_VISIBLE_DEVICES remapping
    does not matter), or `nvidia-smi -lms 100` where NVML is unavailable."""

    REASONS = (("hw_slowdown", 0x8 | 0x80), ("sw_power_cap", 0x4), ("sw_thermal_slowdown", 0x20),
               ("hw_thermal_slowdown", 0x40))
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index, self.rows, self.proc, self.nvml, self.stop = index, [], None, None, False
        self.max_mhz = None

    def __enter__(self):
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            pr = torch.cuda.get_device_properties(self.index)
            bus = f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0"
            self.nvml = (pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus))
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.nvml[1], pynvml.NVML_CLOCK_SM))
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
            return self
        except Exception:
            self.nvml = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _poll(self):
        nv, h = self.nvml
        while not self.stop:
            try:
                sm = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                mask = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                power = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
            except Exception:
                break
            self.rows.append((sm, power, mask))
            time.sleep(0.01)

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == 7:
                try:
                    self.max_mhz = float(parts[1])
                    mask = sum(bit for (name, bit), v in zip(
                        (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
                         ("sw_power_cap", 0x4)), parts[3:]) if v.lower() == "active")
                    self.rows.append((float(parts[0]), float(parts[2]), mask))
                except ValueError:
                    pass

    def __exit__(self, *exc):
        self.stop = True
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        elif self.nvml:
            self.thread.join(timeout=1)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"]}
        reasons = sorted({name for _, _, m in self.rows for name, bits in self.REASONS if m & bits})
        return {"sm_mhz": statistics.median(r[0] for r in self.rows), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.rows),
                "power_w": statistics.median(r[1] for r in self.rows),
                "source": "nvml" if self.nvml else "nvidia-smi"}


# -------------------------------------------------------------- model setup
def build_stack(device, seed):
    from recavsr_b200.runtime.block import LayerStack
    return LayerStack(build_blocks(device, seed, H_TOK, W_TOK), ACTIONS)


def build_blocks(device, seed, h_tok, w_tok):
    import torch
    from recavsr_b200.runtime.block import FusedBlock, rope_tables
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    tables = rope_tables(HEAD_DIM, h_tok, w_tok, device)
    rnd = lambda *s, std=1.0: (torch.randn(*s, generator=g, device=device) * std).bfloat16()
    encoder = rnd(1, ENC_LEN, DIM)
    blocks = []
    for _ in range(LAYERS):
        w = {}
        for name, (n, k) in {"q": (DIM, DIM), "k": (DIM, DIM), "v": (DIM, DIM), "o": (DIM, DIM),
                             "cq": (DIM, DIM), "ck": (DIM, DIM), "cv": (DIM, DIM), "co": (DIM, DIM),
                             "up": (FFN, DIM), "down": (DIM, FFN)}.items():
            w[name + "_w"] = rnd(n, k, std=0.02)
            w[name + "_b"] = rnd(n, std=0.02)
        for name in ("norm_q", "norm_k", "cnorm_q", "cnorm_k", "norm2_w"):
            w[name] = (1 + 0.1 * torch.randn(DIM, generator=g, device=device)).bfloat16()
        w["norm2_b"] = rnd(DIM, std=0.1)
        w["scale_shift_table"] = rnd(1, 6, DIM, std=DIM ** -0.5)
        w["timestep_proj"] = rnd(1, 1, 6, DIM)
        w["encoder"] = encoder
        w["heads"] = HEADS
        blocks.append(FusedBlock(w, h_tok, w_tok, tables))
        del w
    torch.cuda.synchronize(device)
    return blocks


def algorithmic_flops_per_token():
    """Linears per token (30 layers): q,k,v,o,cross-q,cross-o = 6*2*dim^2, FFN 2*2*dim*ffn."""
    return LAYERS * (6 * 2 * DIM * DIM + 2 * 2 * DIM * FFN)


def attention_flops_per_block(stack):
    """Visible keys only: 4 * d * heads * Nq * T * sum over layers of (planes),
    counted from the last block's routing table."""
    planes = 0
    for i, c in enumerate(stack.caches):
        o = i * stack._row
        planes += int((stack.route_host[o:o + c.capacity] >= 0).sum())
    return 4 * HEAD_DIM * HEADS * (BODY * T) * T * (planes + BODY * LAYERS), planes


# ------------------------------------------------------- kernel-level timing
def time_kernel(fn, reps, torch):
    s = torch.cuda.current_stream()
    for _ in range(3):
        fn()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a.record(s)
    for _ in range(reps):
        fn()
    b.record(s)
    b.synchronize()
    return a.elapsed_time(b) / reps * 1e-3


def kernel_roofline(stack, torch):
    """Time the ffn_up NVFP4 GEMM (the largest launch of the step) and the
    routed attention of the recent_4_anchor layers on the step's own buffers,
    as the layer loop runs them: each call uses the next layer's weights (30 x
    25 MB of ffn_up weights) or the next recent_4_anchor layer's KV cache (4 x
    65 MB), so those operands come from HBM as in the step, not from L2. The
    activations (32 MB or less) are L2-resident, as they are in the step, where
    the kernel before wrote them. Also the same launches on one layer's
    operands repeated (L2-warm), for comparison."""
    from recavsr_b200 import _lib
    lib = _lib.library()
    n = BODY * T
    ws = stack.workspace(n)
    st = _lib.stream()
    cursor = {"up": 0, "att": 0}

    def up_on(blk):
        _lib.check(lib.rc_nvfp4_gemm_ws(ws.a_codes.data_ptr(), ws.a_scales.data_ptr(), blk.up.codes.data_ptr(),
                                        blk.up.scales.data_ptr(), blk.up.bias.data_ptr(), n, FFN, DIM, 1.0,
                                        _lib.EPI_GELU_NVFP4, None, 0, None, ws.f_codes.data_ptr(),
                                        ws.f_scales.data_ptr(), 1.0, ws.gemm_ws.data_ptr(),
                                        ws.gemm_ws.numel(), st), "up")

    def up_rot():
        up_on(stack.blocks[cursor["up"] % LAYERS])
        cursor["up"] += 1
    t_up = time_kernel(up_rot, 60, torch)
    t_up_warm = time_kernel(lambda: up_on(stack.blocks[11]), 50, torch)
    rd = stack.route_dev
    qpos = rd[LAYERS * stack._row:]
    att_layers = [i for i, a in enumerate(ACTIONS) if a == "recent_4_anchor"]

    def att_on(i):
        o = i * stack._row
        cap = stack.caches[i].capacity
        stack.blocks[i]._attention(lib, ws, stack.cache_k[i], stack.cache_v[i], rd[o:o + cap],
                                   rd[o + 8:o + 8 + cap], qpos, n, st)

    def att_rot():
        att_on(att_layers[cursor["att"] % len(att_layers)])
        cursor["att"] += 1
    t_att = time_kernel(att_rot, 20, torch)
    t_att_warm = time_kernel(lambda: att_on(11), 20, torch)
    o = 11 * stack._row
    vis = int((stack.route_host[o:o + stack.caches[11].capacity] >= 0).sum())
    att_flops = 4 * HEAD_DIM * HEADS * n * T * (vis + BODY)
    return {"ffn_up_s": t_up, "ffn_up_warm_s": t_up_warm, "ffn_up_flops": 2.0 * n * FFN * DIM,
            "attn_s": t_att, "attn_warm_s": t_att_warm, "attn_flops": float(att_flops),
            "attn_planes": vis + BODY, "attn_layers": att_layers}


def ffn_up_bytes():
    """Algorithmic bytes of one ffn_up launch: NVFP4 activation and weight codes
    + scales in, NVFP4 codes + scales of the GELU output out, bf16 bias."""
    n = BODY * T
    codes = lambda m, k: m * k // 2
    scales = lambda m, k: (m + 127) // 128 * 128 * ((k // 16 + 3) // 4 * 4)
    return (codes(n, DIM) + scales(n, DIM) + codes(FFN, DIM) + scales(FFN, DIM) + 2 * FFN
            + codes(n, FFN) + scales(n, FFN))


# ---------------------------------------------------------------- CPU side
def cpu_baseline(sample_tokens_note=True):
    """Oracle port of one DiT block forward in the reference's CPU formulation
    (fp32 linears as nn.Linear runs them there -- its NVFP4 GEMM needs CUDA --,
    fp32 attention and softmax; numpy/BLAS on all host cores) at the bench
    geometry; tokens/s is extrapolated to the 30-layer step."""
    from oracle import block as oblock
    from oracle import rope as orope
    rs = np.random.RandomState(0)
    f32 = lambda *s, std=1.0: (rs.standard_normal(s).astype(np.float32) * np.float32(std))
    lin = {}
    for name, (n, k) in {"q": (DIM, DIM), "k": (DIM, DIM), "v": (DIM, DIM), "o": (DIM, DIM),
                         "cq": (DIM, DIM), "co": (DIM, DIM), "up": (FFN, DIM), "down": (DIM, FFN)}.items():
        lin[name] = oblock.QuantLinear(f32(n, k, std=0.02), f32(n, std=0.02), matmul_dtype=np.float32,
                                       quantized=False)
    tc, ts, sc, ss = orope.rolling_tables(HEAD_DIM, H_TOK, W_TOK)
    p = {"_linears": lin, "modulation": f32(6, DIM), "norm_q": 1 + f32(DIM, std=0.1),
         "norm_k": 1 + f32(DIM, std=0.1), "cnorm_q": 1 + f32(DIM, std=0.1),
         "norm2_w": 1 + f32(DIM, std=0.1), "norm2_b": f32(DIM, std=0.1),
         "cross_k": f32(ENC_LEN, HEADS, HEAD_DIM), "cross_v": f32(ENC_LEN, HEADS, HEAD_DIM),
         "temporal_cos": tc, "temporal_sin": ts, "spatial_cos": sc, "spatial_sin": ss}
    hidden = f32(BODY * T, DIM)
    pk, pv = f32(2 * T, HEADS, HEAD_DIM), f32(2 * T, HEADS, HEAD_DIM)
    t0 = time.perf_counter()
    oblock.block_forward(p, hidden, pk, pv, [0, 1], [6, 7], [8, 9], H_TOK, W_TOK, (22, 40),
                         heads=HEADS, matmul_dtype=np.float32)
    dt = time.perf_counter() - t0
    tokens_per_s = BODY * T / (dt * LAYERS)
    return {"value": tokens_per_s, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"1 of 30 layers (recent_2 cache, 1760 tokens, fp32 linears and attention), {dt:.2f} s, "
                      "extrapolated x30"}


def run_reference(args, rank, world):
    """--impl reference: the reference's CPU formulation (oracle port) timed on
    the host cores; rank 0 only."""
    if rank != 0:
        return
    os.environ.setdefault("OMP_NUM_THREADS", str(os.cpu_count()))
    vals = []
    for i in range(args.warmup + args.steps):
        r = cpu_baseline()
        if i >= args.warmup:
            vals.append(r["value"])
    v = statistics.median(vals)
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": BODY * T / v * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic",
        "config": {"workload": "cfg4 DiT layer loop, 1280x704 (22x40 tokens), 2-frame body block",
                   "global_batch": 1, "seq_len": BODY * T, "parallelism": "cpu"},
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
                         "sample": r["sample"]},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ------------------------------------------------- single stream, head-sharded
H_4K, W_4K = 68, 120                   # 3840x2176 model raster / 32
T_4K = H_4K * W_4K


def run_head_shard(args, rank, world, local):
    """--head-shard: one 3840x2176 stream (T = 8160 tokens per latent frame,
    2-frame body blocks of 16320 tokens, 22x40 local windows) split over the
    torchrun ranks by heads (24 / N per rank) with two NCCL all-to-alls per
    layer; tokens/s of the one stream (strong scaling). Every rank builds the
    same weights and the same block inputs and works on its own shard."""
    import datetime

    import torch
    import torch.distributed as dist
    from recavsr_b200 import _lib
    from recavsr_b200.runtime.head_shard import HeadShardedStack
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    stack = HeadShardedStack(build_blocks(device, 1234, H_4K, W_4K), ACTIONS, rank=rank, world=world)
    g = torch.Generator(device=device)
    g.manual_seed(99)
    shard = lambda x: x[rank * (x.shape[0] // world):(rank + 1) * (x.shape[0] // world)].contiguous()
    prefix = shard(torch.randn(PREFIX * T_4K, DIM, generator=g, device=device).bfloat16())
    stack.step(prefix, PREFIX)
    body = shard(torch.randn(BODY * T_4K, DIM, generator=g, device=device).bfloat16())
    h = body.clone()
    warm = max(args.warmup, 3)
    for _ in range(warm):
        h.copy_(body)
        stack.step(h, BODY)
    torch.cuda.synchronize(device)
    if not torch.isfinite(h.float()).all():
        raise RuntimeError("non-finite hidden state after warm-up")
    dev_err = _lib.read_device_error()
    if dev_err:
        raise RuntimeError(f"device error word 0x{dev_err:08x}")
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        start.record()
        for _ in range(args.steps):
            stack.step(h, BODY)
        end.record()
        end.synchronize()
    t = start.elapsed_time(end) * 1e-3
    host_in = torch.empty(body.shape, dtype=torch.bfloat16, pin_memory=True)
    host_in.copy_(body.cpu())
    host_out = torch.empty_like(host_in, pin_memory=True)
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        h.copy_(host_in, non_blocking=True)
        stack.step(h, BODY)
        host_out.copy_(h, non_blocking=True)
    e1.record()
    e1.synchronize()
    te = e0.elapsed_time(e1) * 1e-3
    if world > 1:
        tt = torch.tensor([t, te], device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t, te = float(tt[0]), float(tt[1])
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    tokens = BODY * T_4K * args.steps
    value = tokens / t
    launches_per_layer = 15   # LN x3, GEMM x6, RMSNorm x2, gather + attention, NVFP4 quantize, cross attention
    print(json.dumps({
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": warm, "ms_per_step": t / args.steps * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "nvfp4 linears / bf16 attention",
        "data": "synthetic (random-init weights, N(0,1) hidden/prompt states)",
        "config": {"workload": "cfg5 single stream 3840x2176 -> 68x120 tokens (T=8160), 2-frame body "
                               "block (16320 tokens), 30 layers, released router, 22x40 local windows",
                   "global_batch": 1, "seq_len": BODY * T_4K,
                   "parallelism": f"heads x{world} (token-sharded linears, all-to-all at attention)",
                   "l2": "working set > 126 MB L2 (no flush)", "cuda_graph": False},
        "out_fps": value * 4 / T_4K,
        "e2e": {"value": tokens / te, "unit": "tokens/s",
                "h2d_bytes_per_step": body.numel() * 2 * world, "d2h_bytes_per_step": body.numel() * 2 * world,
                "path": "per rank: copy shard in, HeadShardedStack.step, copy shard out (one stream)"},
        "gpu_launches": args.steps * (LAYERS * launches_per_layer + sum(
            1 for c in stack.caches if c.capacity)),
        "clocks": clk.summary(),
    }), flush=True)


# ------------------------------------------- whole one-step DiT stream (glue)
LQ_H1, LQ_H2, LATENT_C = 2048, 3072, 48


def build_glue(device, seed):
    """Random-init session glue of the released architecture: patch embedding
    Conv3d(48 -> 3072, 1x2x2), the LQ projector (768 -> 2048 -> 3072 causal
    Conv3d (4, 3, 3) + out_proj 3072 -> 3072), sr_proj, proj_out 3072 -> 192, the
    output scale_shift_table + temb."""
    import torch
    from recavsr_b200.runtime.session import SessionGlue
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    rnd = lambda *s, std=0.02: (torch.randn(*s, generator=g, device=device) * std).bfloat16()
    w = {"patch_w": rnd(DIM, LATENT_C, 1, 2, 2, std=0.05), "patch_b": rnd(DIM),
         "sr_w": rnd(DIM, DIM), "sr_b": rnd(DIM), "proj_out_w": rnd(LATENT_C * 4, DIM),
         "proj_out_b": rnd(LATENT_C * 4),
         "conv1_w": rnd(LQ_H1, 768, 4, 3, 3), "conv1_b": rnd(LQ_H1), "norm1_w": 1 + rnd(LQ_H1, std=0.1),
         "conv2_w": rnd(LQ_H2, LQ_H1, 4, 3, 3), "conv2_b": rnd(LQ_H2), "norm2_w": 1 + rnd(LQ_H2, std=0.1),
         "out_w": rnd(DIM, LQ_H2), "out_b": rnd(DIM),
         "head_shift": rnd(DIM, std=DIM ** -0.5).float(), "head_scale": rnd(DIM, std=DIM ** -0.5).float()}
    return SessionGlue(w, device)


def synthetic_lq(frames, device, seed):
    """LQ RGB frames as the reference's pipeline feeds them (video.py:103-179):
    uint8 uniform noise at 320x176, 5x5 box filter, bilinear x4 to 1280x704,
    normalized to [-1, 1], bf16 [1, 3, frames, 704, 1280]."""
    import torch
    import torch.nn.functional as F
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    lr = torch.randint(0, 256, (frames, 3, 176, 320), generator=g, device=device).float()
    lr = F.avg_pool2d(F.pad(lr, (2, 2, 2, 2), mode="replicate"), 5, stride=1)
    hr = F.interpolate(lr, size=(704, 1280), mode="bilinear", align_corners=False)
    return (hr / 127.5 - 1.0).clamp(-1, 1).permute(1, 0, 2, 3).unsqueeze(0).bfloat16().contiguous()


def measure_session(session, device, rank, world, steps, warm):
    """Time `steps` body blocks of the whole streaming one-step DiT through its
    public host-buffer entry, StreamingSession.step_host: each step's 8 LQ RGB
    frames are copied from pinned host memory and its 2 latent frames back to
    pinned host memory inside the timed region (copies on a side stream,
    overlapping the neighbouring blocks). A fresh stream (reset, prefix block)
    precedes the warm-up. Returns (seconds, h2d bytes, d2h bytes, clocks, host LQ frames)."""
    import torch
    import torch.distributed as dist
    from recavsr_b200 import _lib
    session.reset(seed=rank)
    prefix = synthetic_lq(21, device, 5 + rank)
    body = synthetic_lq(8, device, 6 + rank)
    host_lq = torch.empty(body.shape, dtype=torch.bfloat16, pin_memory=True)
    host_lq.copy_(body.cpu())
    host_out = torch.empty((1, LATENT_C, BODY, 44, 80), dtype=torch.float32, pin_memory=True)
    session.step(prefix)
    for _ in range(warm):
        session.step_host(host_lq, host_out)
    session.sync_host()
    torch.cuda.synchronize(device)
    dev_err = _lib.read_device_error()
    if dev_err:
        raise RuntimeError(f"device error word 0x{dev_err:08x}")
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device.index or 0) as clk:
        start.record()
        for _ in range(steps):
            session.step_host(host_lq, host_out)
        session.sync_host()
        end.record()
        end.synchronize()
    t = start.elapsed_time(end) * 1e-3
    if not torch.isfinite(host_out).all():
        raise RuntimeError("non-finite session output")
    return t, host_lq.numel() * 2, host_out.numel() * 4, clk.summary(), host_lq


SESSION_GLUE_LAUNCHES = 15   # 2 im2col, 2 channel norms, 7 bf16 GEMMs, 2 patch gathers, 1 LayerNorm, 1 unpatchify
DEC_DIM, DEC_HIDDEN, DEC_DEPTH, DEC_REFINE = 512, 2048, 12, 2   # FlashDecoder-S (flashdecoder_wan22.py:590-600)
# Launches of one decode step: 6 before the backbone, 9 per block, 5 between the
# stacks, 4 after the refinement.
DECODER_LAUNCHES = 6 + 9 * (DEC_DEPTH + DEC_REFINE) + 5 + 4


def build_decoder(device, seed, h=44, w=80):
    """Random-init FlashDecoder-S (the released variant: dim 512, 8 query / 2
    KV heads, 12 backbone + 2 refinement blocks, SwiGLU 2048, 24x24 windows)
    as a DecoderSession at the 704x1280 latent grid (weights from
    runtime.decoder.random_params); latent normalization mean N(0, 0.5),
    std U(0.5, 2)."""
    import torch
    from recavsr_b200.runtime.decoder import DecoderSession, random_params
    g = torch.Generator(device=device)
    g.manual_seed(seed + 1)
    mean = torch.randn(LATENT_C, generator=g, device=device) * 0.5
    std = torch.rand(LATENT_C, generator=g, device=device) * 1.5 + 0.5
    return DecoderSession(random_params(device, seed), height=h, width=w, mean=mean, std=std, dim=DEC_DIM,
                          num_heads=8, num_kv_groups=2, depth=DEC_DEPTH, refinement_depth=DEC_REFINE,
                          mlp_ratio=DEC_HIDDEN / DEC_DIM, device=device)


def lq_u8(frames, seed):
    """LQ RGB frames as a video decoder delivers them, uint8 [frames, 176, 320, 3]:
    uniform noise smoothed by a 5x5 box filter (integer mean)."""
    rs = np.random.RandomState(seed)
    x = rs.randint(0, 256, (frames, 180, 324, 3)).astype(np.int32)
    acc = sum(x[:, dy:dy + 176, dx:dx + 320] for dy in range(5) for dx in range(5))
    return (acc // 25).astype(np.uint8)


def measure_pipeline(session, decoder, device, rank, world, steps, warm):
    """The whole per-block pipeline of one stream, timed end to end with CUDA
    events: the block's 8 LQ uint8 frames (320x176) copied from pinned host
    memory, enlarged, normalized and padded on the device (rc_enlarge_block,
    video.py:138-179), the one-step DiT (StreamingSession.step: LQ projector,
    patch embedding, 30 layers as a CUDA graph, head), the FlashDecoder on its
    2 latent frames (DecoderSession, CUDA graphs) and the 8 RGB output frames
    (704x1280, bf16) copied to pinned host memory on a copy stream that
    overlaps the next frames' decode (DecoderSession.step_host); the decoder
    runs on a second stream, overlapping the next block's DiT step. The
    stream starts with its 21-frame prefix block; the decoder's graphs are
    captured during warm-up. Returns (seconds, decoder seconds per body block,
    h2d bytes, d2h bytes, clocks)."""
    import torch
    import torch.distributed as dist
    from recavsr_b200 import _lib
    from recavsr_b200.runtime.pipeline import enlarge_block
    session.reset(seed=rank)
    decoder.reset()
    prefix = torch.from_numpy(lq_u8(21, 8 + rank)).pin_memory()
    body = torch.from_numpy(lq_u8(8, 9 + rank)).pin_memory()
    rgb_host = torch.empty((3, 8, 704, 1280), dtype=torch.bfloat16, pin_memory=True)
    rgb_prefix = torch.empty((3, 21, 704, 1280), dtype=torch.bfloat16, pin_memory=True)

    dec_stream = torch.cuda.Stream(device)

    def block(host, n_rgb, out):
        x = enlarge_block(host.to(device, non_blocking=True), (704, 1280), block=n_rgb, dtype=torch.bfloat16)
        lat = session.step(x)
        # The decoder runs on its own stream, overlapping the next block's DiT
        # step; its RGB copies to the host overlap the next frames.
        ready = torch.cuda.Event()
        ready.record()
        dec_stream.wait_event(ready)
        x.record_stream(dec_stream)
        lat.record_stream(dec_stream)
        with torch.cuda.stream(dec_stream):
            return decoder.step_host(lat, x, out)

    block(prefix, 21, rgb_prefix)
    for i in range(warm):
        if i == 1:
            decoder.capture()
        block(body, 8, rgb_host)
    decoder.sync_host()
    torch.cuda.synchronize(device)
    dev_err = _lib.read_device_error()
    if dev_err:
        raise RuntimeError(f"device error word 0x{dev_err:08x}")
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device.index or 0) as clk:
        start.record()
        for _ in range(steps):
            st = block(body, 8, rgb_host)
        torch.cuda.current_stream(device).wait_event(st.output_ready)
        end.record()
        end.synchronize()
    t = start.elapsed_time(end) * 1e-3
    if not torch.isfinite(rgb_host.float()).all():
        raise RuntimeError("non-finite decoder output")
    # The decoder alone on the same inputs (steady-state body blocks, graphs).
    lat = torch.randn((1, LATENT_C, BODY, 44, 80), device=device)
    x = enlarge_block(body.to(device), (704, 1280), block=8, dtype=torch.bfloat16)
    for _ in range(2):
        list(decoder.step(lat, lr_up=x))
    torch.cuda.synchronize(device)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        list(decoder.step(lat, lr_up=x))
    b.record()
    b.synchronize()
    t_dec = a.elapsed_time(b) * 1e-3 / steps
    return t, t_dec, body.numel(), rgb_host.numel() * 2, clk.summary()


def run_session(args, rank, world, local):
    """--session: the whole streaming one-step DiT (TransformerSession.step) at
    1280x704 output: LQ projector + patch embedding + sr_proj, the 30-layer loop
    (CUDA graph), output head, noise - prediction, timed through step_host
    (pinned host frames in, latents out), plus the glue's per-phase device
    times; one independent stream per rank."""
    import datetime

    import torch
    import torch.distributed as dist
    from recavsr_b200.runtime.session import StreamingSession
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    session = StreamingSession(build_stack(device, seed=1234 + rank), build_glue(device, 77 + rank),
                               704, 1280, seed=rank, graphs=True)
    warm = max(args.warmup, 3)
    t, h2d, d2h, clocks, host_lq = measure_session(session, device, rank, world, args.steps, warm)
    # Per-phase device time of the glue on body blocks (a fresh LQ stream
    # primed with a prefix, so every timed call is a valid streaming step).
    glue = session.glue
    out_shape = (1, LATENT_C, BODY, 44, 80)
    nz = torch.randn(out_shape, device=device)
    rec = torch.zeros(out_shape, dtype=torch.bfloat16, device=device)
    lq_dev = host_lq.to(device)
    lq_state = glue.lq.create_streaming_state()
    glue.lq.forward_streaming(synthetic_lq(21, device, 5 + rank), lq_state)
    t_embed = time_kernel(lambda: glue.embed(nz, lq_dev, rec, lq_state), 5, torch)
    hidden = torch.randn(BODY * T, DIM, device=device).bfloat16()
    t_head = time_kernel(lambda: glue.head(hidden, nz), 5, torch)
    m1, m2 = 4 * 44 * 80, BODY * T                       # conv1 / conv2 output rows per body block
    embed_flops = (2.0 * m1 * LQ_H1 * 36 * 768 + 2.0 * m2 * LQ_H2 * 36 * LQ_H1 + 2.0 * m2 * DIM * LQ_H2
                   + 2 * 2.0 * m2 * DIM * LATENT_C * 4 + 2.0 * m2 * DIM * DIM)
    _, bf16_peak, _, src = peaks()
    if world > 1:
        tt = torch.tensor([t], device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t = float(tt[0])
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    tokens = BODY * T * args.steps * world
    value = tokens / t
    print(json.dumps({
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": warm, "ms_per_step": t / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "nvfp4 DiT linears / bf16 attention and glue",
        "data": "synthetic (random-init weights; LQ frames: uint8 noise, 5x5 box filter, bilinear x4)",
        "config": {"workload": "cfg4 whole one-step DiT stream step (LQ projector, patch embedding, "
                               "30 layers, output head), 1280x704, 8 LQ frames -> 2 latent frames",
                   "global_batch": world, "seq_len": BODY * T, "parallelism": f"streams x{world}",
                   "l2": "working set > 126 MB L2 (no flush)", "cuda_graph": "layer loop"},
        "value_is": "aggregate tokens/s over all GPUs; tokens_per_s_per_gpu is the metric's per-GPU figure",
        "tokens_per_s_per_gpu": value / world,
        "out_fps": value * 4 / T,
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "path": "StreamingSession.step_host: LQ frames from pinned host, latents to pinned host "
                        "(copies on a side stream, overlapping the neighbouring blocks)"},
        "gpu_launches": args.steps * (LAYERS * 14 + sum(1 for c in session.stack.caches if c.capacity)
                                      + SESSION_GLUE_LAUNCHES),
        "glue": {"embed_ms": t_embed * 1e3, "head_ms": t_head * 1e3,
                 "embed_tflops": embed_flops / t_embed / 1e12,
                 "embed_frac": embed_flops / t_embed / 1e12 / bf16_peak,
                 "peak": f"{src} bf16 dense {bf16_peak} TFLOP/s",
                 "embed": "LQ projector (im2col + bf16 GEMMs + channel RMSNorm/SiLU), patch embedding x2, sr_proj"},
        "clocks": clocks,
    }), flush=True)


# ------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--eager", action="store_true", help="no CUDA graph (launch from Python)")
    ap.add_argument("--no-kernel-timing", action="store_true",
                    help="skip the per-kernel roofline timing (e.g. for an ncu launch list)")
    ap.add_argument("--head-shard", action="store_true",
                    help="one 3840x2176 stream split by heads over the ranks (strong scaling)")
    ap.add_argument("--session", action="store_true",
                    help="only the whole one-step DiT stream step (LQ projector, layers, head) per block")
    ap.add_argument("--no-session", action="store_true",
                    help="skip the whole-step session and pipeline measurements of the default line")
    ap.add_argument("--no-decoder", action="store_true",
                    help="skip the whole-pipeline measurement (DiT step + FlashDecoder) of the default line")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.head_shard:
        return run_head_shard(args, rank, world, local)
    if args.session:
        return run_session(args, rank, world, local)

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    from recavsr_b200 import _lib
    stack = build_stack(device, seed=1234 + rank)
    g = torch.Generator(device=device)
    g.manual_seed(99 + rank)
    warm = max(args.warmup, 3)
    # Prefix (6 frames) then body blocks; the caches fill within a few blocks.
    prefix = torch.randn(PREFIX * T, DIM, generator=g, device=device).bfloat16()
    stack.step(prefix, PREFIX)
    body = torch.randn(BODY * T, DIM, generator=g, device=device).bfloat16()
    h = body.clone()
    stack.step(h, BODY)                       # eager body step: sets kernel attributes
    use_graph = not args.eager
    if use_graph:
        stack.capture(BODY * T, BODY)
    for _ in range(warm):
        h.copy_(body)
        stack.step(h, BODY, graphs=use_graph)
    torch.cuda.synchronize(device)
    if not torch.isfinite(h.float()).all():
        raise RuntimeError("non-finite hidden state after warm-up")
    dev_err = _lib.read_device_error()
    if dev_err:
        raise RuntimeError(f"device error word 0x{dev_err:08x}")

    # ---- timed region: device-resident inputs
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        start.record()
        for _ in range(args.steps):
            stack.step(h, BODY, graphs=use_graph)
        end.record()
        end.synchronize()
    t = start.elapsed_time(end) * 1e-3
    # ---- e2e: host buffers, copies inside the timed region
    host_in = torch.empty((BODY * T, DIM), dtype=torch.bfloat16, pin_memory=True)
    host_in.copy_(body.cpu())
    host_out = torch.empty_like(host_in, pin_memory=True)
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if use_graph:
        # Streaming path of the public API: each block's host->device input copy
        # and device->host result copy overlap the neighbouring blocks' layer loops.
        outs = [host_out, torch.empty_like(host_out, pin_memory=True)]
        stack.step_host(host_in, outs[1], BODY)    # warm the staging buffers
        stack.sync_host()
        torch.cuda.synchronize(device)
        e0.record()
        for i in range(args.steps):
            stack.step_host(host_in, outs[i & 1], BODY)
        stack.sync_host()
        e1.record()
    else:
        e0.record()
        for _ in range(args.steps):
            h.copy_(host_in, non_blocking=True)
            stack.step(h, BODY, graphs=use_graph)
            host_out.copy_(h, non_blocking=True)
        e1.record()
    e1.synchronize()
    te = e0.elapsed_time(e1) * 1e-3
    kr = kernel_roofline(stack, torch) if rank == 0 and not args.no_kernel_timing else None
    att_flops, planes = attention_flops_per_block(stack)
    layer_launches = LAYERS * 14 + sum(1 for c in stack.caches if c.capacity)
    # ---- the whole streaming step (TransformerSession.step) through its public
    # host-buffer entry: LQ frames in from pinned host memory, latents out.
    ts = None
    if not args.no_session:
        from recavsr_b200.runtime.session import StreamingSession
        session = StreamingSession(stack, build_glue(device, 77 + rank), 704, 1280, seed=rank, graphs=True)
        ts, s_h2d, s_d2h, s_clk, _ = measure_session(session, device, rank, world, args.steps, warm)
    # ---- the whole pipeline of a stream: LQ uint8 frames in, RGB frames out
    tp = None
    if not args.no_session and not args.no_decoder:
        decoder = build_decoder(device, 91 + rank)
        tp, t_dec, p_h2d, p_d2h, p_clk = measure_pipeline(session, decoder, device, rank, world, args.steps, warm)
    if world > 1:
        tt = torch.tensor([t, te, ts or 0.0, tp or 0.0], device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t, te = float(tt[0]), float(tt[1])
        ts = float(tt[2]) if ts is not None else None
        tp = float(tt[3]) if tp is not None else None
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    tokens = BODY * T * args.steps * world
    value = tokens / t
    hbm, bf16_peak, bf16_sus, src = peaks()
    fp4_peak = 4 * bf16_peak
    if kr is None:
        kr = {"ffn_up_flops": 1.0, "ffn_up_s": float("inf"), "ffn_up_warm_s": float("inf"), "attn_flops": 1.0,
              "attn_s": float("inf"), "attn_warm_s": float("inf"), "attn_planes": 0, "attn_layers": []}
    achieved = kr["ffn_up_flops"] / kr["ffn_up_s"] / 1e12
    cpu = None if args.no_cpu_baseline else cpu_baseline()
    layer_e2e = {"value": tokens / te, "unit": "tokens/s",
                 "h2d_bytes_per_step": BODY * T * DIM * 2 + stack.route_dev.numel() * 4,   # block + routing table
                 "d2h_bytes_per_step": BODY * T * DIM * 2,
                 "path": "LayerStack.step_host (pinned host -> device -> pinned host; copies overlap the "
                         "neighbouring blocks)" if not args.eager else "copy, step, copy on one stream"}
    out = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": warm, "ms_per_step": t / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "nvfp4 linears / bf16 attention",
        "data": "synthetic (random-init weights, N(0,1) hidden/prompt states; LQ frames: uint8 noise, "
                "5x5 box filter, bilinear x4)",
        "config": {"workload": "cfg4 DiT layer loop (30 layers, released router), 1280x704 -> 22x40 "
                               "tokens, 2-frame body block (1760 tokens), B=1; e2e / out_fps: the whole "
                               "one-step stream step (LQ projector, patch embedding, layers, head)",
                   "global_batch": world, "seq_len": BODY * T, "parallelism": f"streams x{world}",
                   "l2": "working set > 126 MB L2 (no flush)", "cuda_graph": use_graph},
        "value_is": "aggregate tokens/s over all GPUs; tokens_per_s_per_gpu is the metric's per-GPU figure",
        "tokens_per_s_per_gpu": value / world,
        "out_fps_layer_loop": value * 4 / T,
        "linear_tflops": value * algorithmic_flops_per_token() / 1e12,
        "attention_tflops": att_flops * (value / (BODY * T)) / 1e12,
        "roofline": {"bound": "tensor", "kernel": "nvfp4 ffn_up GEMM 1760x14336x3072 (+GELU+NVFP4 epilogue)",
                     "achieved": achieved, "peak": fp4_peak, "unit": "TFLOP/s", "frac": achieved / fp4_peak,
                     "peak_source": f"4 x {src} bf16 dense ({bf16_peak} TFLOP/s): FP4:BF16 dense ratio 4",
                     "timing": "CUDA events over 60 launches, each on the next layer's weights (HBM-resident "
                               "as in the step); L2-warm (one layer repeated): "
                               f"{kr['ffn_up_flops'] / kr['ffn_up_warm_s'] / 1e12:.1f} TFLOP/s",
                     "traffic": PROFILED_DRAM["ffn_up"]["read"] + PROFILED_DRAM["ffn_up"]["write"],
                     "traffic_source": PROFILED_DRAM["ffn_up"]["source"],
                     "algorithmic_bytes": ffn_up_bytes(),
                     "attention": {"achieved": kr["attn_flops"] / kr["attn_s"] / 1e12, "peak": bf16_peak,
                                   "frac": kr["attn_flops"] / kr["attn_s"] / 1e12 / bf16_peak,
                                   "planes": kr["attn_planes"], "unit": "TFLOP/s",
                                   "timing": f"each launch on the next recent_4_anchor layer's KV cache "
                                             f"(layers {kr['attn_layers']}); L2-warm: "
                                             f"{kr['attn_flops'] / kr['attn_warm_s'] / 1e12:.1f} TFLOP/s",
                                   "traffic": PROFILED_DRAM["attention"]["read"] + PROFILED_DRAM["attention"]["write"],
                                   "traffic_source": PROFILED_DRAM["attention"]["source"]}},
        "cpu_baseline": cpu,
        "e2e": layer_e2e,
        "gpu_launches": args.steps * layer_launches,
        "clocks": clk.summary(),
        "attention_planes_per_block": planes + BODY * LAYERS,
    }
    if ts is not None:
        stokens = BODY * T * args.steps * world
        out["out_fps"] = stokens / ts * 4 / T
        out["e2e"] = {"value": stokens / ts, "unit": "tokens/s", "h2d_bytes_per_step": s_h2d,
                      "d2h_bytes_per_step": s_d2h,
                      "path": "StreamingSession.step_host: the whole one-step DiT stream step (LQ projector, "
                              "patch embedding, 30 layers, head, noise - prediction) from 8 LQ RGB frames in "
                              "pinned host memory to 2 latent frames in pinned host memory"}
        out["e2e_layer_loop"] = layer_e2e
        out["session"] = {"ms_per_step": ts / args.steps * 1e3, "tokens_s": stokens / ts,
                          "gpu_launches": args.steps * (layer_launches + SESSION_GLUE_LAUNCHES),
                          "clocks": s_clk}
    else:
        out["out_fps"] = value * 4 / T
    if tp is not None:
        frames = 4 * BODY * args.steps * world
        out["pipeline"] = {
            "out_fps": frames / tp, "ms_per_body_block": tp / args.steps * 1e3,
            "out_fps_per_gpu": frames / tp / world,
            "decoder_ms_per_latent_frame": t_dec / BODY * 1e3,
            "decoder_out_fps": 4 * BODY / t_dec,
            "h2d_bytes_per_step": p_h2d, "d2h_bytes_per_step": p_d2h,
            "gpu_launches": args.steps * (1 + layer_launches + SESSION_GLUE_LAUNCHES + BODY * DECODER_LAUNCHES),
            "path": "per body block of one stream: 8 LQ uint8 frames 320x176 from pinned host -> rc_enlarge_block "
                    "(bf16 704x1280) -> StreamingSession.step (one-step DiT) -> DecoderSession.step_host "
                    "(FlashDecoder-S, 2 latent frames, CUDA graphs, on a second stream overlapping the next "
                    "block's DiT step) -> 8 RGB frames 704x1280 bf16 to pinned host (copies on a third stream); "
                    "timed to the last frame's arrival",
            "excluded": "video decode / encode and colour correction",
            "clocks": p_clk,
        }
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
