// FlashDecoder decode step: the glue kernels around its linears and local
// attention (recavsr_infer/models/flashdecoder/flashdecoder_wan22.py:245-874,
// runtime/flashdecoder.py:140-175), in the arithmetic the reference runs on
// CUDA under bf16 autocast:
//
//   rc_fd_latent_in     raw = bf16(bf16(bf16(latent) * std) + mean)  (runtime/flashdecoder.py:168),
//                       as [n, 64] GEMM rows (channels 48..63 zero)
//   rc_fd_lr_unshuffle  F.pixel_unshuffle(lr_up, 16) channels (c, i, j) -> bf16 [F*n, 768]  (:704-707)
//   rc_fd_lr_group      the first chunk's frame repetition and the 4-frame grouping of the
//                       LR features (:708-719): [n, 192] early and [4n, 64] late GEMM rows
//   rc_fd_kv_norm       key_norm / value_norm (RMSNorm over each 64-dim head, fp32) of the
//                       current tokens into the layer's K (fp32) / V (bf16) frame rings (:310-322)
//   rc_fd_rope_gather   3D RoPE (:198-242, fp32 math, no fused multiply-add) of the queries
//                       and of every key frame of the window, in temporal order, plus the
//                       window's V frames: the attention operands (:324-331)
//   rc_fd_silu          SwiGLU's bf16(bf16(silu(gate)) * up) (:344-345) or an in-place SiLU
//                       (spatial_projection, :680-684)
//   rc_fd_pixel_shuffle pixel_shuffle(16) of the spatial projection into RGB frames,
//                       clamped to [-1, 1] (:845-866, runtime/flashdecoder.py:175)
//
// Frame rings: a layer's cache of `slots` frames is [heads][slots * n][64]; the
// frame with global index g lives in slot g % slots, so a step writes its
// current frames without moving the kept ones, and rc_fd_rope_gather reads the
// window's frames in temporal order (slot (slot0 + t) % slots for key frame t).
#include "common.cuh"

namespace {

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__global__ void __launch_bounds__(256) fd_latent_in_kernel(const float* lat, long long cs, int n,
                                                           const __nv_bfloat16* mean,
                                                           const __nv_bfloat16* stdv, __nv_bfloat16* out) {
  rc::pdl_trigger();
  rc::pdl_wait();
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)n * 64) return;
  const int p = (int)(i >> 6), c = (int)(i & 63);
  float v = 0.f;
  if (c < 48) {
    const float x = bf16r(rc::ld_in(lat + c * cs + p));
    const float prod = bf16r(__fmul_rn(x, __bfloat162float(rc::ld_in(stdv + c))));
    v = __fadd_rn(prod, __bfloat162float(rc::ld_in(mean + c)));
  }
  out[i] = __float2bfloat16_rn(v);
}

// One thread per 8 output columns (8 consecutive pixels of one patch row).
template <typename T>
__global__ void __launch_bounds__(256) fd_lr_unshuffle_kernel(const T* lr, long long sc, long long sf,
                                                              long long sy, int frames, int h, int w,
                                                              __nv_bfloat16* out) {
  rc::pdl_trigger();
  rc::pdl_wait();
  const long long n = (long long)h * w;
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;   // over frames*n*96
  if (i >= frames * n * 96) return;
  const int ch = (int)(i % 96);                  // 8-column chunk of the 768 columns
  const long long row = i / 96;                  // f * n + p
  const int f = (int)(row / n), p = (int)(row % n);
  const int c = ch >> 5, ii = (ch >> 1) & 15, j0 = (ch & 1) * 8;
  const int y = (p / w) * 16 + ii, x = (p % w) * 16 + j0;
  const T* src = lr + c * sc + f * sf + y * sy + x;
  uint32_t wv[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    float a, b;
    if constexpr (sizeof(T) == 4) {
      a = rc::ld_in(reinterpret_cast<const float*>(src) + 2 * k);
      b = rc::ld_in(reinterpret_cast<const float*>(src) + 2 * k + 1);
    } else {
      a = __bfloat162float(rc::ld_in(reinterpret_cast<const __nv_bfloat16*>(src) + 2 * k));
      b = __bfloat162float(rc::ld_in(reinterpret_cast<const __nv_bfloat16*>(src) + 2 * k + 1));
    }
    wv[k] = rc::pack_bf16x2(a, b);
  }
  *reinterpret_cast<uint4*>(out + row * 768 + ch * 8) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
}

// One thread per (token, frame of the group, 8-column chunk of 64).
__global__ void __launch_bounds__(256) fd_lr_group_kernel(const __nv_bfloat16* feats, long long ldf, int n,
                                                          int first, __nv_bfloat16* grouped,
                                                          __nv_bfloat16* late) {
  rc::pdl_trigger();
  rc::pdl_wait();
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;   // over 4*n*8
  if (i >= 4LL * n * 8) return;
  const int ch = (int)(i & 7);
  const long long fp = i >> 3;
  const int f = (int)(fp / n), p = (int)(fp % n);
  const int src_f = first ? 0 : f;
  uint4 v = make_uint4(0, 0, 0, 0);
  if (ch < 6) {
    const __nv_bfloat16* s = feats + ((long long)src_f * n + p) * ldf + ch * 8;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t lo = __bfloat16_as_ushort(rc::ld_in(s + 2 * k));
      const uint32_t hi = __bfloat16_as_ushort(rc::ld_in(s + 2 * k + 1));
      (&v.x)[k] = lo | (hi << 16);
    }
    *reinterpret_cast<uint4*>(grouped + (long long)p * 192 + f * 48 + ch * 8) = v;
  }
  *reinterpret_cast<uint4*>(late + ((long long)f * n + p) * 64 + ch * 8) = v;
}

// One warp per (token, KV head): RMSNorm of the head's 64 K and 64 V values.
__global__ void __launch_bounds__(256) fd_kv_norm_kernel(const __nv_bfloat16* qkv, long long ldq, int tokens,
                                                         int q_cols, int hk, const float* wk, const float* wv,
                                                         float eps, float* k_ring, __nv_bfloat16* v_ring,
                                                         long long ring_head, long long token0) {
  rc::pdl_trigger();
  rc::pdl_wait();
  const long long wid = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= (long long)tokens * hk) return;
  const int t = (int)(wid / hk), h = (int)(wid % hk);
  const __nv_bfloat16* row = qkv + (long long)t * ldq + q_cols;
  const long long dst = h * ring_head + (token0 + t) * 64 + 2 * lane;
#pragma unroll
  for (int which = 0; which < 2; ++which) {
    const __nv_bfloat16* src = row + (which * hk + h) * 64 + 2 * lane;
    const float a = __bfloat162float(rc::ld_in(src)), b = __bfloat162float(rc::ld_in(src + 1));
    float ss = __fadd_rn(__fmul_rn(a, a), __fmul_rn(b, b));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    const float r = rsqrtf(__fadd_rn(__fmul_rn(ss, 1.0f / 64.0f), eps));
    const float* wt = which ? wv : wk;
    const float ya = __fmul_rn(__fmul_rn(a, r), rc::ld_in(wt + 2 * lane));
    const float yb = __fmul_rn(__fmul_rn(b, r), rc::ld_in(wt + 2 * lane + 1));
    if (which == 0) {
      *reinterpret_cast<float2*>(k_ring + dst) = make_float2(ya, yb);
    } else {
      *reinterpret_cast<uint32_t*>(v_ring + dst) = rc::pack_bf16x2(ya, yb);
    }
  }
}

struct RopeArgs {
  const __nv_bfloat16* qkv;
  long long ldq;
  int hq, hk, cur, prev, nf, slot0, slots, h, w;
  const float* k_ring;
  const __nv_bfloat16* v_ring;
  long long ring_head;
  const float* tab;            // cos_t [max_t][8] | sin_t | cos_h [h][12] | sin_h | cos_w [w][12] | sin_w
  int max_t;
  __nv_bfloat16* q_out;        // [cur*n, hq*64]
  __nv_bfloat16* k_out;        // [hk][nf*n][64]
  __nv_bfloat16* v_out;        // [hk][nf*n][64]
};

// cos / sin of rotary pair j (0..31) of the token at (t, y, x).
__device__ __forceinline__ void rope_cs(const RopeArgs& a, int j, int t, int y, int x, float& c, float& s) {
  const float* ct = a.tab;
  const float* st = ct + a.max_t * 8;
  const float* chh = st + a.max_t * 8;
  const float* sh = chh + a.h * 12;
  const float* cw = sh + a.h * 12;
  const float* sw = cw + a.w * 12;
  if (j < 8) {
    c = rc::ld_in(ct + t * 8 + j);
    s = rc::ld_in(st + t * 8 + j);
  } else if (j < 20) {
    c = rc::ld_in(chh + y * 12 + j - 8);
    s = rc::ld_in(sh + y * 12 + j - 8);
  } else {
    c = rc::ld_in(cw + x * 12 + j - 20);
    s = rc::ld_in(sw + x * 12 + j - 20);
  }
}

// Rotates 4 (even, odd) pairs: even' = e c - o s, odd' = e s + o c in fp32
// (separately rounded products, as the reference's tensor expressions).
__device__ __forceinline__ uint4 rotate4(const RopeArgs& a, const float (&e)[8], int j0, int t, int y, int x) {
  uint32_t wv[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    float c, s;
    rope_cs(a, j0 + k, t, y, x, c, s);
    const float ev = e[2 * k], od = e[2 * k + 1];
    wv[k] = rc::pack_bf16x2(__fsub_rn(__fmul_rn(ev, c), __fmul_rn(od, s)),
                            __fadd_rn(__fmul_rn(ev, s), __fmul_rn(od, c)));
  }
  return make_uint4(wv[0], wv[1], wv[2], wv[3]);
}

// Flat index over three ranges of 8-element chunks: rotated queries,
// rotated key frames, copied value frames.
__global__ void __launch_bounds__(256) fd_rope_gather_kernel(RopeArgs a) {
  rc::pdl_trigger();
  rc::pdl_wait();
  const long long n = (long long)a.h * a.w;
  const long long nq = (long long)a.cur * n * a.hq * 8, nk = (long long)a.nf * n * a.hk * 8;
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < nq) {
    const int ch = (int)(i & 7);
    const long long th = i >> 3;
    const int head = (int)(th % a.hq);
    const long long tok = th / a.hq;
    const int f = (int)(tok / n), p = (int)(tok % n);
    const __nv_bfloat16* src = a.qkv + tok * a.ldq + head * 64 + ch * 8;
    const uint4 raw = rc::ld_in(reinterpret_cast<const uint4*>(src));
    float e[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t wv = (&raw.x)[k];
      e[2 * k] = __uint_as_float(wv << 16);
      e[2 * k + 1] = __uint_as_float(wv & 0xffff0000u);
    }
    *reinterpret_cast<uint4*>(a.q_out + tok * (a.hq * 64) + head * 64 + ch * 8) =
        rotate4(a, e, ch * 4, a.prev + f, p / a.w, p % a.w);
    return;
  }
  i -= nq;
  const bool is_v = i >= nk;
  if (is_v) i -= nk;
  if (i >= nk) return;
  const int ch = (int)(i & 7);
  const long long hr = i >> 3;                      // head * nf*n + key row
  const int head = (int)(hr / (a.nf * n));
  const long long kr = hr % (a.nf * n);
  const int kf = (int)(kr / n), p = (int)(kr % n);
  const long long slot = (a.slot0 + kf) % a.slots;
  const long long src = head * a.ring_head + (slot * n + p) * 64 + ch * 8;
  const long long dst = ((long long)head * a.nf * n + kr) * 64 + ch * 8;
  if (is_v) {
    *reinterpret_cast<uint4*>(a.v_out + dst) = rc::ld_in(reinterpret_cast<const uint4*>(a.v_ring + src));
  } else {
    const float4 lo = rc::ld_in(reinterpret_cast<const float4*>(a.k_ring + src));
    const float4 hi = rc::ld_in(reinterpret_cast<const float4*>(a.k_ring + src) + 1);
    const float e[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
    *reinterpret_cast<uint4*>(a.k_out + dst) = rotate4(a, e, ch * 4, kf, p / a.w, p % a.w);
  }
}

// SiLU as the reference's CUDA kernel forms it: x / (1 + exp(-x)) in fp32.
__device__ __forceinline__ float silu(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x))); }

// mode 0: out[m, j] = bf16(bf16(silu(x[m, j])) * x[m, H + j]) from [M, 2H];
// mode 1: x[m, j] = bf16(silu(x[m, j])) in place on [M, H]. 8 columns per thread.
__global__ void __launch_bounds__(256) fd_silu_kernel(__nv_bfloat16* x, int M, int H, int mode,
                                                      __nv_bfloat16* out) {
  rc::pdl_trigger();
  rc::pdl_wait();
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int per_row = H / 8;
  if (i >= (long long)M * per_row) return;
  const long long m = i / per_row;
  const int c = (int)(i % per_row) * 8;
  const long long ld = mode == 0 ? 2LL * H : H;
  const uint4 g = rc::ld_in(reinterpret_cast<const uint4*>(x + m * ld + c));
  uint4 u = make_uint4(0, 0, 0, 0);
  if (mode == 0) u = rc::ld_in(reinterpret_cast<const uint4*>(x + m * ld + H + c));
  uint32_t wv[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t gw = (&g.x)[k];
    float s0 = bf16r(silu(__uint_as_float(gw << 16)));
    float s1 = bf16r(silu(__uint_as_float(gw & 0xffff0000u)));
    if (mode == 0) {
      const uint32_t uw = (&u.x)[k];
      s0 = __fmul_rn(s0, __uint_as_float(uw << 16));
      s1 = __fmul_rn(s1, __uint_as_float(uw & 0xffff0000u));
    }
    wv[k] = rc::pack_bf16x2(s0, s1);
  }
  __nv_bfloat16* dst = mode == 0 ? out + m * H + c : x + m * ld + c;
  *reinterpret_cast<uint4*>(dst) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
}

// One thread per 8 horizontally adjacent output pixels of one channel.
__global__ void __launch_bounds__(256) fd_pixel_shuffle_kernel(const __nv_bfloat16* y, long long ldy, int f0,
                                                               int frames, int out_frames, int h, int w,
                                                               __nv_bfloat16* out) {
  rc::pdl_trigger();
  rc::pdl_wait();
  const int W = 16 * w, Hp = 16 * h;
  const long long per_frame = (long long)Hp * (W / 8);
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;   // over 3 * frames * Hp * W/8
  if (i >= 3LL * frames * per_frame) return;
  const int cf = (int)(i / per_frame);             // c * frames + f
  const long long r = i % per_frame;
  const int Y = (int)(r / (W / 8)), X = (int)(r % (W / 8)) * 8;
  const int c = cf / frames, f = cf % frames;
  const long long tok = (long long)(f0 + f) * h * w + (Y / 16) * w + X / 16;
  const uint4 v = rc::ld_in(reinterpret_cast<const uint4*>(y + tok * ldy + c * 256 + (Y & 15) * 16 + (X & 15)));
  uint32_t wv[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t ww = (&v.x)[k];
    const float a = fminf(fmaxf(__uint_as_float(ww << 16), -1.0f), 1.0f);
    const float b = fminf(fmaxf(__uint_as_float(ww & 0xffff0000u), -1.0f), 1.0f);
    wv[k] = rc::pack_bf16x2(a, b);
  }
  *reinterpret_cast<uint4*>(out + ((long long)(c * out_frames + f) * Hp + Y) * W + X) =
      make_uint4(wv[0], wv[1], wv[2], wv[3]);
}

int grid1(long long items) { return (int)((items + 255) / 256); }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

extern "C" {

int rc_fd_latent_in(const float* latent, long long channel_stride, int n, const void* mean, const void* stdv,
                    void* out, cudaStream_t stream) {
  if (!latent || !mean || !stdv || !out || n < 1 || channel_stride < n)
    return rc::set_error(RC_ERR_ARG, "rc_fd_latent_in: bad arguments");
  return rc::check_launch(rc::launch_pdl(fd_latent_in_kernel, dim3(grid1(64LL * n)), dim3(256), 0, stream, latent,
                                         channel_stride, n, reinterpret_cast<const __nv_bfloat16*>(mean),
                                         reinterpret_cast<const __nv_bfloat16*>(stdv),
                                         reinterpret_cast<__nv_bfloat16*>(out)),
                          "rc_fd_latent_in");
}

int rc_fd_lr_unshuffle(const void* lr, int dtype, const long long* strides, int frames, int h, int w, void* out,
                       cudaStream_t stream) {
  if (!lr || !out || !strides || frames < 1 || h < 1 || w < 1 || (dtype != 0 && dtype != 1) || !aligned16(out))
    return rc::set_error(RC_ERR_ARG, "rc_fd_lr_unshuffle: bad arguments");
  const int esz = dtype == 0 ? 4 : 2;
  for (int k = 0; k < 3; ++k)
    if ((strides[k] * esz) % 16) return rc::set_error(RC_ERR_ARG, "rc_fd_lr_unshuffle: strides must be 16-byte multiples");
  if (reinterpret_cast<uintptr_t>(lr) % 16) return rc::set_error(RC_ERR_ARG, "rc_fd_lr_unshuffle: input must be 16-byte aligned");
  const long long items = (long long)frames * h * w * 96;
  cudaError_t e = dtype == 0
      ? rc::launch_pdl(fd_lr_unshuffle_kernel<float>, dim3(grid1(items)), dim3(256), 0, stream,
                       reinterpret_cast<const float*>(lr), strides[0], strides[1], strides[2], frames, h, w,
                       reinterpret_cast<__nv_bfloat16*>(out))
      : rc::launch_pdl(fd_lr_unshuffle_kernel<__nv_bfloat16>, dim3(grid1(items)), dim3(256), 0, stream,
                       reinterpret_cast<const __nv_bfloat16*>(lr), strides[0], strides[1], strides[2], frames, h,
                       w, reinterpret_cast<__nv_bfloat16*>(out));
  return rc::check_launch(e, "rc_fd_lr_unshuffle");
}

int rc_fd_lr_group(const void* feats, long long ldf, int n, int first, void* grouped, void* late,
                   cudaStream_t stream) {
  if (!feats || !grouped || !late || n < 1 || ldf < 48 || ldf % 8 || !aligned16(feats) || !aligned16(grouped) ||
      !aligned16(late))
    return rc::set_error(RC_ERR_ARG, "rc_fd_lr_group: bad arguments");
  return rc::check_launch(rc::launch_pdl(fd_lr_group_kernel, dim3(grid1(32LL * n)), dim3(256), 0, stream,
                                         reinterpret_cast<const __nv_bfloat16*>(feats), ldf, n, first ? 1 : 0,
                                         reinterpret_cast<__nv_bfloat16*>(grouped),
                                         reinterpret_cast<__nv_bfloat16*>(late)),
                          "rc_fd_lr_group");
}

int rc_fd_kv_norm(const void* qkv, long long ldq, int tokens, int q_cols, int hk, const float* wk,
                  const float* wv, float eps, float* k_ring, void* v_ring, long long ring_head, long long token0,
                  cudaStream_t stream) {
  if (!qkv || !wk || !wv || !k_ring || !v_ring || tokens < 1 || hk < 1 || q_cols < 0 ||
      ldq < q_cols + 128LL * hk || ring_head < 64LL * (token0 + tokens) || token0 < 0)
    return rc::set_error(RC_ERR_ARG, "rc_fd_kv_norm: bad arguments");
  return rc::check_launch(rc::launch_pdl(fd_kv_norm_kernel, dim3(grid1(32LL * tokens * hk)), dim3(256), 0, stream,
                                         reinterpret_cast<const __nv_bfloat16*>(qkv), ldq, tokens, q_cols, hk, wk,
                                         wv, eps, k_ring, reinterpret_cast<__nv_bfloat16*>(v_ring), ring_head,
                                         token0),
                          "rc_fd_kv_norm");
}

int rc_fd_rope_gather(const void* qkv, long long ldq, int hq, int hk, int cur, int prev, int nf, int slot0,
                      int slots, int h, int w, const float* k_ring, const void* v_ring, long long ring_head,
                      const float* tables, int max_t, void* q_out, void* k_out, void* v_out,
                      cudaStream_t stream) {
  if (!qkv || !k_ring || !v_ring || !tables || !q_out || !k_out || !v_out || hq < 1 || hk < 1 || cur < 1 ||
      prev < 0 || nf < cur || slots < nf || slot0 < 0 || h < 1 || w < 1 || max_t < prev + cur || max_t < nf ||
      ldq % 8 || ring_head < (long long)slots * h * w * 64 || !aligned16(qkv) || !aligned16(q_out) ||
      !aligned16(k_out) || !aligned16(v_out) || !aligned16(k_ring) || !aligned16(v_ring))
    return rc::set_error(RC_ERR_ARG, "rc_fd_rope_gather: bad arguments");
  RopeArgs a{reinterpret_cast<const __nv_bfloat16*>(qkv), ldq, hq, hk, cur, prev, nf, slot0, slots, h, w,
             k_ring, reinterpret_cast<const __nv_bfloat16*>(v_ring), ring_head, tables, max_t,
             reinterpret_cast<__nv_bfloat16*>(q_out), reinterpret_cast<__nv_bfloat16*>(k_out),
             reinterpret_cast<__nv_bfloat16*>(v_out)};
  const long long n = (long long)h * w;
  const long long items = (long long)cur * n * hq * 8 + 2LL * nf * n * hk * 8;
  return rc::check_launch(rc::launch_pdl(fd_rope_gather_kernel, dim3(grid1(items)), dim3(256), 0, stream, a),
                          "rc_fd_rope_gather");
}

int rc_fd_silu(void* x, int M, int H, int mode, void* out, cudaStream_t stream) {
  if (!x || M < 1 || H < 8 || H % 8 || (mode != 0 && mode != 1) || (mode == 0 && !out) || !aligned16(x) ||
      (mode == 0 && !aligned16(out)))
    return rc::set_error(RC_ERR_ARG, "rc_fd_silu: bad arguments");
  return rc::check_launch(rc::launch_pdl(fd_silu_kernel, dim3(grid1((long long)M * (H / 8))), dim3(256), 0, stream,
                                         reinterpret_cast<__nv_bfloat16*>(x), M, H, mode,
                                         reinterpret_cast<__nv_bfloat16*>(out)),
                          "rc_fd_silu");
}

int rc_fd_pixel_shuffle(const void* y, long long ldy, int f0, int frames, int out_frames, int h, int w, void* out,
                        cudaStream_t stream) {
  if (!y || !out || ldy < 768 || ldy % 8 || f0 < 0 || frames < 1 || f0 + frames > 4 || out_frames < frames ||
      h < 1 || w < 1 ||
      !aligned16(y) || !aligned16(out))
    return rc::set_error(RC_ERR_ARG, "rc_fd_pixel_shuffle: bad arguments");
  const long long items = 3LL * frames * 16 * h * 2 * w;
  return rc::check_launch(rc::launch_pdl(fd_pixel_shuffle_kernel, dim3(grid1(items)), dim3(256), 0, stream,
                                         reinterpret_cast<const __nv_bfloat16*>(y), ldy, f0, frames, out_frames, h,
                                         w, reinterpret_cast<__nv_bfloat16*>(out)),
                          "rc_fd_pixel_shuffle");
}

}  // extern "C"
