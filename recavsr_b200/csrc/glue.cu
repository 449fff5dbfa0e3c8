// Row-wise glue around the DiT linears: LayerNorm (+affine) (+AdaLN
// modulation) with an optional fused NVFP4 quantizer, RMSNorm across heads
// with the spatial rotary embedding, the temporal rotary embedding, and the
// KV-cache plane commit. Row kernels run one 128-thread CTA per row with up to
// four 8-element chunks per thread (a lane pair per 16-element quantization
// block, N <= 4096), so the row stays in registers and each input byte is read
// from HBM once.
//
// Numerics follow recavsr_infer/runtime/transformer.py:88-133 in eager order:
//   LN in fp32 (two-pass mean / variance, rsqrt(var + eps)), then
//   y * (1 + scale) + shift as separate fp32 roundings, then bf16;
//   RMSNorm: bf16(x * rsqrt(mean(x^2) + eps) * w) with one rounding;
//   rotary: (e*c - o*s, e*s + o*c) in fp32, then bf16 (runtime/rope.py:23-30).
#include "common.cuh"
#include <cuda_fp16.h>

namespace {


__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    f[2 * j] = __uint_as_float(w[j] << 16);
    f[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
  }
}
// Same as unpack8, but opaque to common-subexpression elimination: a row
// kernel re-expands its packed bf16 registers in each pass instead of keeping
// every expanded fp32 value alive across passes (which would spill).
__device__ __forceinline__ void unpack8_fresh(const uint4& v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t lo, hi;
    asm volatile("shl.b32 %0, %2, 16;\n\tand.b32 %1, %2, 0xffff0000;" : "=r"(lo), "=r"(hi) : "r"(w[j]));
    f[2 * j] = __uint_as_float(lo);
    f[2 * j + 1] = __uint_as_float(hi);
  }
}
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int j = 0; j < 4; ++j)
    w[j] = (uint32_t)rc::bf16_bits(f[2 * j]) | ((uint32_t)rc::bf16_bits(f[2 * j + 1]) << 16);
  return make_uint4(w[0], w[1], w[2], w[3]);
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

struct LnArgs {
  const __nv_bfloat16* x; long long ldx;
  const __nv_bfloat16* weight; const __nv_bfloat16* bias;   // affine (nullable)
  const float* shift; const float* scale;                    // modulation (nullable)
  float eps;
  __nv_bfloat16* out; long long ldo;                         // bf16 output (nullable)
  uint8_t* codes; uint8_t* sf; float g;                      // NVFP4 output (nullable)
  int M, N;
};

__device__ __forceinline__ void loadf8(const float* p, float (&f)[8]) {
  const float4* q = reinterpret_cast<const float4*>(p);
  const float4 a = rc::ld_in(q), b = rc::ld_in(q + 1);
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

__device__ __forceinline__ void loadf8_plain(const float* p, float (&f)[8]) {
  const float4* q = reinterpret_cast<const float4*>(p);
  const float4 a = q[0], b = q[1];
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

// NVFP4 encode of one 16-element block split over a lane pair (lanes 2b and
// 2b+1 hold elements 0-7 and 8-15). Returns this lane's 4 code bytes; both
// lanes get the block's scale byte.
__device__ __forceinline__ uint32_t quant8_pair(const float (&f)[8], float g, uint8_t& sfb) {
  float amax = rc::absmax3_nan(rc::absmax3_nan(f[0], f[1], f[2]), rc::absmax3_nan(f[3], f[4], f[5]),
                               rc::absmax3_nan(f[6], f[7], 0.0f));
  amax = rc::absmax3_nan(amax, __shfl_xor_sync(0xffffffffu, amax, 1), 0.0f);
  if (g == 1.0f) {
    sfb = rc::nvfp4_scale_byte(amax);
    return sfb == 0x7f ? 0u : rc::nvfp4_codes8(f, rc::e4m3_nonneg_to_float(sfb));
  }
  float sc = __fmul_rn(__fdiv_rn(amax, 6.0f), g);
  sc = sc < 0.001953125f ? 0.001953125f : sc;
  sfb = rc::e4m3_from_float(sc);
  const float sd = rc::e4m3_to_float(sfb);
  uint32_t w = 0;
  {
#pragma unroll
    for (int j = 0; j < 8; ++j) w |= rc::e2m1_code(__fdiv_rn(__fmul_rn(f[j], g), sd)) << (4 * j);
  }
  return w;
}

// Scale bytes of 4 consecutive k-blocks = lanes 8a, 8a+2, 8a+4, 8a+6: one word.
__device__ __forceinline__ void store_sf4_pairs(uint8_t* sf, int row, int kb, int katoms, uint8_t b,
                                                bool live) {
  const uint32_t b0 = b;
  const uint32_t b1 = __shfl_down_sync(0xffffffffu, b0, 2);
  const uint32_t b2 = __shfl_down_sync(0xffffffffu, b0, 4);
  const uint32_t b3 = __shfl_down_sync(0xffffffffu, b0, 6);
  if (live && (threadIdx.x & 7) == 0)
    *reinterpret_cast<uint32_t*>(sf + rc::sf_offset(row, kb, katoms)) =
        b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
}

// Row kernels: one CTA of kRowThreads threads per row; thread t owns the
// 8-element chunks t, t + kRowThreads, ... (at most kRowChunks of them, so
// N <= 4096) and issues all of its loads before the first reduction. The
// straight-line code per row is short (a few chunks per thread), so thousands
// of small CTAs stay resident and hide the load -> reduce -> store latency.
// Lanes (2m, 2m+1) of a warp hold one 16-element quantization block and lanes
// 8a..8a+7 one scale-atom column.
constexpr int kRowThreads = 128;
constexpr int kRowChunks = 4;

__device__ __forceinline__ float row_sum(float v, float* red) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  const float t = (red[0] + red[1]) + (red[2] + red[3]);
  __syncthreads();   // red is reused by the next reduction
  return t;
}

// CH = chunks per thread (ceil(N / 8 / kRowThreads)); AFF / MOD: whether an
// affine weight / bias or a modulation scale / shift may be present (register
// arrays are sized for the inputs the launch has).
template <int CH, bool AFF, bool MOD>
constexpr int ln_min_blocks() {   // 6 resident CTAs where the registers allow it
  return (CH * ((AFF ? 8 : 0) + (MOD ? 16 : 0)) > 48) ? 4 : 6;
}
template <int CH, bool AFF, bool MOD>
__global__ void __launch_bounds__(kRowThreads, ln_min_blocks<CH, AFF, MOD>()) ln_modulate_kernel(LnArgs a) {
  __shared__ float red[4];
  rc::pdl_trigger();
  rc::pdl_wait();
  const int row = blockIdx.x;
  const int t = threadIdx.x;
  if (row >= a.M) {
    // One extra CTA (launched when M % 128 != 0): zero the scale words of the
    // padding rows [M, ceil(M/128)*128) so the next GEMM reads zeros there.
    const int katoms = ((a.N >> 4) + 3) >> 2;
    const int pad = (a.M + 127) / 128 * 128 - a.M;
    for (int i = t; i < pad * katoms; i += kRowThreads)
      *reinterpret_cast<uint32_t*>(a.sf + rc::sf_offset(a.M + i / katoms, (i % katoms) * 4, katoms)) = 0u;
    return;
  }
  const int nch = a.N >> 3;
  uint4 raw[CH];
#pragma unroll
  for (int i = 0; i < CH; ++i) {
    const int c = t + i * kRowThreads;
    raw[i] = c < nch ? rc::ld_in(reinterpret_cast<const uint4*>(a.x + (size_t)row * a.ldx) + c)
                     : make_uint4(0, 0, 0, 0);
  }
  // Every per-column vector of this thread's chunks, loaded with the row,
  // before the reductions (their latency overlaps the two block barriers)
  // and before the first store (a store through a byte pointer may alias
  // them, so a load inside the chunk loop would wait behind the previous
  // chunk's stores).
  uint4 wraw[AFF ? CH : 1], braw[AFF ? CH : 1];
  float sc[MOD ? CH : 1][8], sh[MOD ? CH : 1][8];
#pragma unroll
  for (int i = 0; i < CH; ++i) {
    const int c = t + i * kRowThreads;
    const bool live = c < nch;
    const int n0 = c * 8;
    if constexpr (AFF) {
      wraw[i] = live && a.weight ? rc::ld_in(reinterpret_cast<const uint4*>(a.weight + n0)) : make_uint4(0, 0, 0, 0);
      braw[i] = live && a.bias ? rc::ld_in(reinterpret_cast<const uint4*>(a.bias + n0)) : make_uint4(0, 0, 0, 0);
    }
    if constexpr (MOD) {
      if (live && a.scale) loadf8(a.scale + n0, sc[i]);
      if (live && a.shift) loadf8(a.shift + n0, sh[i]);
    }
  }
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < CH; ++i) {
    float f[8];
    unpack8(raw[i], f);
#pragma unroll
    for (int j = 0; j < 8; ++j) s += f[j];
  }
  const float mean = __fdiv_rn(row_sum(s, red), (float)a.N);
  float m2 = 0.f;
#pragma unroll
  for (int i = 0; i < CH; ++i) {
    if (t + i * kRowThreads < nch) {
      float f[8];
      unpack8_fresh(raw[i], f);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = f[j] - mean;
        m2 = fmaf(d, d, m2);
      }
    }
  }
  const float rstd = rsqrtf(__fdiv_rn(row_sum(m2, red), (float)a.N) + a.eps);
  const int katoms = ((a.N >> 4) + 3) >> 2;
  const float2 nmean = make_float2(-mean, -mean), rstd2 = make_float2(rstd, rstd);
  const float2 one2 = make_float2(1.0f, 1.0f);
#pragma unroll
  for (int i = 0; i < CH; ++i) {
    if (i * kRowThreads >= nch) break;                 // CTA-uniform
    const int c = t + i * kRowThreads;
    const bool live = c < nch;
    const int n0 = c * 8;
    float f[8];
    unpack8_fresh(raw[i], f);
    if (live) {
      float w[8], b[8];
      if constexpr (AFF) {
        if (a.weight) unpack8(wraw[i], w);
        if (a.bias) unpack8(braw[i], b);
      }
      // fl(fl(x - mean) * rstd), then each affine / modulation step rounded
      // separately, two columns per packed fp32 op; bf16 at the end.
      uint32_t h[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 y = __fmul2_rn(__fadd2_rn(make_float2(f[2 * j], f[2 * j + 1]), nmean), rstd2);
        if constexpr (AFF) {
          if (a.weight) y = __fmul2_rn(y, make_float2(w[2 * j], w[2 * j + 1]));
          if (a.bias) y = __fadd2_rn(y, make_float2(b[2 * j], b[2 * j + 1]));
        }
        if constexpr (MOD) {
          if (a.scale) y = __fmul2_rn(y, __fadd2_rn(one2, make_float2(sc[i][2 * j], sc[i][2 * j + 1])));
          if (a.shift) y = __fadd2_rn(y, make_float2(sh[i][2 * j], sh[i][2 * j + 1]));
        }
        h[j] = rc::pack_bf16x2(y.x, y.y);
        f[2 * j] = __uint_as_float(h[j] << 16);
        f[2 * j + 1] = __uint_as_float(h[j] & 0xffff0000u);
      }
      if (a.out) *reinterpret_cast<uint4*>(a.out + (size_t)row * a.ldo + n0) = make_uint4(h[0], h[1], h[2], h[3]);
    }
    if (a.codes) {
      uint8_t sfb;
      const uint32_t wq = quant8_pair(f, a.g, sfb);
      if (live) *reinterpret_cast<uint32_t*>(a.codes + (size_t)row * (a.N >> 1) + (size_t)c * 4) = wq;
      store_sf4_pairs(a.sf, row, c >> 1, katoms, live ? sfb : 0, live);
    }
  }
}

struct RmsArgs {
  const __nv_bfloat16* x[2]; long long ldx[2];
  const __nv_bfloat16* w[2];
  __nv_bfloat16* out[2]; long long ldo[2];
  const float* cos; const float* sin;  // [span, d] spatial tables (nullable -> no rotary)
  float eps;
  int M, N, d, span;
};

// One CTA of kRowThreads threads per (row, tensor); thread t owns chunks
// t, t + kRowThreads, ... of 8 elements. When 8 * kRowThreads is a whole
// number of heads, all of a thread's chunks sit at the same offset within a
// head and its rotary coefficients are loaded once.
__global__ void __launch_bounds__(kRowThreads, 8) rmsnorm_rope_kernel(RmsArgs a) {
  __shared__ float red[4];
  rc::pdl_trigger();
  rc::pdl_wait();
  const int row = blockIdx.x, t = threadIdx.x;
  const bool second = blockIdx.y != 0;            // select, not index: keeps the params in registers
  const __nv_bfloat16* xp = second ? a.x[1] : a.x[0];
  const long long ldx = second ? a.ldx[1] : a.ldx[0];
  __nv_bfloat16* op = second ? a.out[1] : a.out[0];
  const long long ldo = second ? a.ldo[1] : a.ldo[0];
  const __nv_bfloat16* w = second ? a.w[1] : a.w[0];
  const int nch = a.N >> 3;
  uint4 raw[kRowChunks];
#pragma unroll
  for (int i = 0; i < kRowChunks; ++i) {
    const int c = t + i * kRowThreads;
    raw[i] = c < nch ? rc::ld_in(reinterpret_cast<const uint4*>(xp + (size_t)row * ldx) + c)
                     : make_uint4(0, 0, 0, 0);
  }
  // The norm weights of this thread's chunks, loaded with the row (a store
  // through `op` could alias them and would keep later loads behind it).
  uint4 wraw[kRowChunks];
  if (w) {
#pragma unroll
    for (int i = 0; i < kRowChunks; ++i) {
      const int c = t + i * kRowThreads;
      wraw[i] = c < nch ? rc::ld_in(reinterpret_cast<const uint4*>(w) + c) : make_uint4(0, 0, 0, 0);
    }
  }
  const int pos = row % a.span;
  const bool same_dd = ((8 * kRowThreads) % a.d) == 0;
  float cs[8], sn[8];
  if (a.cos && same_dd) {
    const int dd = (t * 8) % a.d;
    loadf8(a.cos + (size_t)pos * a.d + dd, cs);
    loadf8(a.sin + (size_t)pos * a.d + dd, sn);
  }
  float r = 0.f;
  if (w) {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kRowChunks; ++i) {
      float f[8];
      unpack8(raw[i], f);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(f[j], f[j], ss);
    }
    r = rsqrtf(__fdiv_rn(row_sum(ss, red), (float)a.N) + a.eps);
  }
#pragma unroll
  for (int i = 0; i < kRowChunks; ++i) {
    const int c = t + i * kRowThreads;
    if (c >= nch) break;
    const int n0 = c * 8;
    float f[8];
    unpack8_fresh(raw[i], f);
    if (w) {
      float wf[8];
      unpack8(wraw[i], wf);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 y = __fmul2_rn(__fmul2_rn(make_float2(f[2 * j], f[2 * j + 1]), make_float2(r, r)),
                                    make_float2(wf[2 * j], wf[2 * j + 1]));
        const uint32_t h = rc::pack_bf16x2(y.x, y.y);
        f[2 * j] = __uint_as_float(h << 16);
        f[2 * j + 1] = __uint_as_float(h & 0xffff0000u);
      }
    }
    if (a.cos) {
      if (!same_dd) {
        const int dd = n0 % a.d;   // 8 | d: a chunk never straddles heads
        loadf8(a.cos + (size_t)pos * a.d + dd, cs);
        loadf8(a.sin + (size_t)pos * a.d + dd, sn);
      }
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        const float e = f[j], o = f[j + 1];
        f[j] = __fsub_rn(__fmul_rn(e, cs[j]), __fmul_rn(o, sn[j]));
        f[j + 1] = __fadd_rn(__fmul_rn(e, sn[j]), __fmul_rn(o, cs[j]));
      }
    }
    *reinterpret_cast<uint4*>(op + (size_t)row * ldo + n0) = pack8(f);
  }
}

// Temporal rotary on the first `td` dims of every head of `planes` planes of
// `span` tokens; plane p uses position pos[p] (runtime/rope.py:33-47).
__global__ void temporal_rope_kernel(const __nv_bfloat16* x, long long ldx,
                                     __nv_bfloat16* out, long long ldo,
                                     const int* pos, const float* cos,
                                     const float* sin, int rows, int span, int heads,
                                     int d, int td) {
  rc::pdl_trigger();
  rc::pdl_wait();
  const long long pairs_per_row = (long long)heads * (d / 2);
  const long long total = (long long)rows * pairs_per_row;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / pairs_per_row;
    const int rem = (int)(i % pairs_per_row);
    const int h = rem / (d / 2), pr = rem % (d / 2);
    const __nv_bfloat162 v =
        *reinterpret_cast<const __nv_bfloat162*>(x + row * ldx + (long long)h * d + 2 * pr);
    float e = __low2float(v), o = __high2float(v);
    if (2 * pr < td) {
      const int p = pos[row / span];
      const float c = cos[p * (td / 2) + pr], s = sin[p * (td / 2) + pr];
      const float ne = __fsub_rn(__fmul_rn(e, c), __fmul_rn(o, s));
      const float no = __fadd_rn(__fmul_rn(e, s), __fmul_rn(o, c));
      e = ne;
      o = no;
    }
    *reinterpret_cast<__nv_bfloat162*>(out + row * ldo + (long long)h * d + 2 * pr) =
        __floats2bfloat162_rn(e, o);
  }
}

// KV commit: copy `n` planes of `span` rows (`row_bytes` each) for K and V.
struct CommitArgs {
  const uint8_t* src[2]; long long src_ld[2];
  uint8_t* dst[2]; long long dst_ld[2];
  int src_plane[8]; int dst_plane[8];
  int n, span, row_bytes;
};

__global__ void kv_commit_kernel(CommitArgs a) {
  rc::pdl_trigger();
  rc::pdl_wait();
  const int vec_per_row = a.row_bytes >> 4;
  const long long per_plane = (long long)a.span * vec_per_row;
  const long long total = 2LL * a.n * per_plane;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int t = (int)(i / (a.n * per_plane));
    const long long r = i % (a.n * per_plane);
    const int c = (int)(r / per_plane);
    const long long q = r % per_plane;
    const long long row = q / vec_per_row, v = q % vec_per_row;
    const uint4* s = reinterpret_cast<const uint4*>(
        a.src[t] + ((long long)a.src_plane[c] * a.span + row) * a.src_ld[t]);
    uint4* dd = reinterpret_cast<uint4*>(
        a.dst[t] + ((long long)a.dst_plane[c] * a.span + row) * a.dst_ld[t]);
    dd[v] = rc::ld_in(s + v);
  }
}

// Same copy with the plane plan read from device memory:
// plan = [n, src0, dst0, src1, dst1, ...] (n <= max_planes), so a captured
// graph stays valid while the routing changes between replays. One CTA =
// kCommitRows rows of one plan entry (blockIdx.y) of K or V (blockIdx.z): the
// plan is read once per CTA and the row loop uses 32-bit offsets, with all of
// a thread's row loads in flight before its stores.
constexpr int kCommitRows = 8;
constexpr int kCommitThreads = 128;

__global__ void __launch_bounds__(kCommitThreads) kv_commit_planned_kernel(CommitArgs a, const int* plan) {
  rc::pdl_trigger();
  rc::pdl_wait();
  const int c = blockIdx.y, t = blockIdx.z;
  if (c >= min(plan[0], a.n)) return;
  const int sp = plan[1 + 2 * c], dp = plan[2 + 2 * c];
  if (sp < 0 || dp < 0 || dp >= a.dst_plane[0]) return;   // dst_plane[0] = slot capacity
  const int vec = a.row_bytes >> 4;
  const int r0 = blockIdx.x * kCommitRows;
  const int rows = min(kCommitRows, a.span - r0);
  const uint8_t* src = a.src[t] + ((long long)sp * a.span + r0) * a.src_ld[t];
  uint8_t* dst = a.dst[t] + ((long long)dp * a.span + r0) * a.dst_ld[t];
  for (int v = threadIdx.x; v < vec; v += kCommitThreads) {
    uint4 val[kCommitRows];
#pragma unroll
    for (int r = 0; r < kCommitRows; ++r)
      if (r < rows) val[r] = rc::ld_in(reinterpret_cast<const uint4*>(src + r * a.src_ld[t]) + v);
#pragma unroll
    for (int r = 0; r < kCommitRows; ++r)
      if (r < rows) reinterpret_cast<uint4*>(dst + r * a.dst_ld[t])[v] = val[r];
  }
}

// Row norm of any floating input type, result in the same type: the drop-in
// recavsr_math::layer_norm / rms_norm contract (kernels/native_norm.py:7-28
// returns .to(x.dtype) of an fp32 computation; PreparedBlock.layer_norm passes
// fp32 rows, runtime/transformer.py:91,121,130). One CTA per row; the row is
// read three times (sum, centred squares, output), the re-reads hit L1.
// dtype: 0 fp32, 1 bf16, 2 fp16. weight / bias: fp32 (nullable).
constexpr int kNormThreads = 256;

__device__ __forceinline__ float load_any(const void* p, size_t i, int dtype) {
  if (dtype == 0) return rc::ld_in(reinterpret_cast<const float*>(p) + i);
  const unsigned short h = rc::ld_in(reinterpret_cast<const unsigned short*>(p) + i);
  if (dtype == 1) return __uint_as_float((uint32_t)h << 16);
  return __half2float(__ushort_as_half(h));
}
__device__ __forceinline__ void store_any(void* p, size_t i, int dtype, float v) {
  if (dtype == 0) reinterpret_cast<float*>(p)[i] = v;
  else if (dtype == 1) reinterpret_cast<unsigned short*>(p)[i] = rc::bf16_bits(v);
  else reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
}
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) t += red[i];
  __syncthreads();
  return t;
}

struct NormArgs {
  const void* x; long long ldx; int dtype;
  const float* weight; const float* bias; float eps; int rms;
  void* out; long long ldo;
  int M, N;
};

__global__ void __launch_bounds__(kNormThreads) row_norm_kernel(NormArgs a) {
  __shared__ float red[kNormThreads / 32];
  rc::pdl_trigger();
  rc::pdl_wait();
  const size_t row = blockIdx.x;
  const size_t xo = row * (size_t)a.ldx, oo = row * (size_t)a.ldo;
  float mean = 0.f;
  if (!a.rms) {
    float s = 0.f;
    for (int i = threadIdx.x; i < a.N; i += kNormThreads) s += load_any(a.x, xo + i, a.dtype);
    mean = __fdiv_rn(block_sum(s, red), (float)a.N);
  }
  float m2 = 0.f;
  for (int i = threadIdx.x; i < a.N; i += kNormThreads) {
    const float d = load_any(a.x, xo + i, a.dtype) - mean;
    m2 = fmaf(d, d, m2);
  }
  const float rstd = rsqrtf(__fdiv_rn(block_sum(m2, red), (float)a.N) + a.eps);
  for (int i = threadIdx.x; i < a.N; i += kNormThreads) {
    float y = __fmul_rn(__fsub_rn(load_any(a.x, xo + i, a.dtype), mean), rstd);
    if (a.weight) y = __fmul_rn(y, rc::ld_in(a.weight + i));
    if (a.bias) y = __fadd_rn(y, rc::ld_in(a.bias + i));
    store_any(a.out, oo + i, a.dtype, y);
  }
}

// bf16 rows of N = 256 V: one warp per row, V 16-byte vectors per lane
// (vector c = v * 32 + lane covers columns 8c .. 8c + 7), the same formula as
// row_norm_kernel with warp-shuffle sums.
template <int V>
__global__ void __launch_bounds__(256) row_norm_warp_kernel(NormArgs a) {
  rc::pdl_trigger();
  rc::pdl_wait();
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= a.M) return;
  const uint4* xp = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(a.x) + row * a.ldx);
  float f[V * 8];
#pragma unroll
  for (int v = 0; v < V; ++v) {
    const uint4 w = rc::ld_in(xp + v * 32 + lane);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t u = (&w.x)[k];
      f[8 * v + 2 * k] = __uint_as_float(u << 16);
      f[8 * v + 2 * k + 1] = __uint_as_float(u & 0xffff0000u);
    }
  }
  auto warp_sum = [](float x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    return x;
  };
  float mean = 0.f;
  if (!a.rms) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < V * 8; ++i) s += f[i];
    mean = __fdiv_rn(warp_sum(s), (float)a.N);
  }
  float m2 = 0.f;
#pragma unroll
  for (int i = 0; i < V * 8; ++i) {
    const float d = f[i] - mean;
    m2 = fmaf(d, d, m2);
  }
  const float rstd = rsqrtf(__fdiv_rn(warp_sum(m2), (float)a.N) + a.eps);
  uint4* op = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.out) + row * a.ldo);
#pragma unroll
  for (int v = 0; v < V; ++v) {
    const int c0 = (v * 32 + lane) * 8;
    float y[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) y[k] = __fmul_rn(__fsub_rn(f[8 * v + k], mean), rstd);
    if (a.weight) {
      const float4 w0 = rc::ld_in(reinterpret_cast<const float4*>(a.weight + c0));
      const float4 w1 = rc::ld_in(reinterpret_cast<const float4*>(a.weight + c0) + 1);
      const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int k = 0; k < 8; ++k) y[k] = __fmul_rn(y[k], wv[k]);
    }
    if (a.bias) {
      const float4 b0 = rc::ld_in(reinterpret_cast<const float4*>(a.bias + c0));
      const float4 b1 = rc::ld_in(reinterpret_cast<const float4*>(a.bias + c0) + 1);
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int k = 0; k < 8; ++k) y[k] = __fadd_rn(y[k], bv[k]);
    }
    op[v * 32 + lane] = make_uint4(rc::pack_bf16x2(y[0], y[1]), rc::pack_bf16x2(y[2], y[3]),
                                   rc::pack_bf16x2(y[4], y[5]), rc::pack_bf16x2(y[6], y[7]));
  }
}

int grid_for(long long work, int threads) {
  long long b = (work + threads - 1) / threads;
  return (int)(b < 1 ? 1 : (b > 148LL * 16 ? 148LL * 16 : b));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

RC_DEVICE_ERROR_ACCESSOR(glue)

extern "C" {

// LayerNorm over the last dim N of x [M, N] (fp32 math), optional affine
// weight/bias (bf16), optional AdaLN modulation y*(1+scale)+shift (fp32 [N]),
// rounded to bf16 into `out` (nullable) and/or NVFP4-quantized into
// codes [M, N/2] + swizzled scales (nullable) with global scale g.
int rc_ln_modulate_quant(const void* x, long long ldx, int M, int N, const void* weight,
                         const void* bias, const float* shift, const float* scale, float eps,
                         void* out, long long ldo, uint8_t* codes, uint8_t* scales_swizzled,
                         float global_scale, cudaStream_t stream) {
  if (M < 0 || N <= 0 || N % 64 || N > 4096)
    return rc::set_error(RC_ERR_ARG, "rc_ln_modulate_quant: N must be a multiple of 64 and <= 4096 (N=%d)", N);
  if (!x || (!out && !codes) || (codes && !scales_swizzled))
    return rc::set_error(RC_ERR_ARG, "rc_ln_modulate_quant: missing pointer");
  if (!aligned16(x) || ldx % 8 || (out && (!aligned16(out) || ldo % 8)) ||
      (shift && reinterpret_cast<uintptr_t>(shift) % 16) || (scale && reinterpret_cast<uintptr_t>(scale) % 16) ||
      (weight && !aligned16(weight)) || (bias && !aligned16(bias)) ||
      (codes && (reinterpret_cast<uintptr_t>(codes) % 8 || reinterpret_cast<uintptr_t>(scales_swizzled) % 4)))
    return rc::set_error(RC_ERR_ARG, "rc_ln_modulate_quant: rows must be 16-byte aligned");
  if (!(global_scale > 0.f)) return rc::set_error(RC_ERR_ARG, "rc_ln_modulate_quant: bad global scale");
  if (M == 0) return RC_OK;
  LnArgs a{reinterpret_cast<const __nv_bfloat16*>(x), ldx,
           reinterpret_cast<const __nv_bfloat16*>(weight), reinterpret_cast<const __nv_bfloat16*>(bias),
           shift, scale, eps, reinterpret_cast<__nv_bfloat16*>(out), ldo, codes, scales_swizzled,
           global_scale, M, N};
  const int ch = ((N >> 3) + kRowThreads - 1) / kRowThreads;   // 1..kRowChunks
  const bool aff = weight || bias, mod = shift || scale;
  using K = void (*)(LnArgs);
  static const K table[kRowChunks][4] = {
      {ln_modulate_kernel<1, false, false>, ln_modulate_kernel<1, true, false>, ln_modulate_kernel<1, false, true>, ln_modulate_kernel<1, true, true>},
      {ln_modulate_kernel<2, false, false>, ln_modulate_kernel<2, true, false>, ln_modulate_kernel<2, false, true>, ln_modulate_kernel<2, true, true>},
      {ln_modulate_kernel<3, false, false>, ln_modulate_kernel<3, true, false>, ln_modulate_kernel<3, false, true>, ln_modulate_kernel<3, true, true>},
      {ln_modulate_kernel<4, false, false>, ln_modulate_kernel<4, true, false>, ln_modulate_kernel<4, false, true>, ln_modulate_kernel<4, true, true>}};
  const K kern = table[ch - 1][(aff ? 1 : 0) + (mod ? 2 : 0)];
  return rc::check_launch(rc::launch_pdl(kern, dim3(M + ((codes && M % 128) ? 1 : 0)), dim3(kRowThreads), 0, stream, a),
                          "rc_ln_modulate_quant");
}

// LayerNorm (rms = 0) or RMSNorm (rms = 1) over the last dim N of x [M, N]
// in fp32 with fp32 affine weight / bias (nullable; bias ignored for RMS),
// output in x's type (dtype 0 fp32, 1 bf16, 2 fp16).
int rc_layer_norm(const void* x, int dtype, long long ldx, int M, int N, const float* weight,
                  const float* bias, float eps, int rms, void* out, long long ldo,
                  cudaStream_t stream) {
  if (dtype < 0 || dtype > 2 || M < 0 || N <= 0 || ldx < N || ldo < N)
    return rc::set_error(RC_ERR_ARG, "rc_layer_norm: bad shape or dtype (dtype=%d M=%d N=%d)", dtype, M, N);
  if (!x || !out) return rc::set_error(RC_ERR_ARG, "rc_layer_norm: missing pointer");
  const int es = dtype == 0 ? 4 : 2;
  if (reinterpret_cast<uintptr_t>(x) % es || reinterpret_cast<uintptr_t>(out) % es ||
      (weight && reinterpret_cast<uintptr_t>(weight) % 4) || (bias && reinterpret_cast<uintptr_t>(bias) % 4))
    return rc::set_error(RC_ERR_ARG, "rc_layer_norm: misaligned pointer");
  if (M == 0) return RC_OK;
  NormArgs a{x, ldx, dtype, weight, rms ? nullptr : bias, eps, rms, out, ldo, M, N};
  // bf16 rows of 256 / 512 / 1024 with 16-byte aligned rows and vectors: a warp per row.
  const bool vec = dtype == 1 && (N == 256 || N == 512 || N == 1024) && aligned16(x) && aligned16(out) &&
                   ldx % 8 == 0 && ldo % 8 == 0 && (!weight || aligned16(weight)) &&
                   (rms || !bias || aligned16(bias));
  if (vec) {
    const dim3 grid((unsigned)((M + 7) / 8));
    cudaError_t e = N == 256 ? rc::launch_pdl(row_norm_warp_kernel<1>, grid, dim3(256), 0, stream, a)
                  : N == 512 ? rc::launch_pdl(row_norm_warp_kernel<2>, grid, dim3(256), 0, stream, a)
                             : rc::launch_pdl(row_norm_warp_kernel<4>, grid, dim3(256), 0, stream, a);
    return rc::check_launch(e, "rc_layer_norm");
  }
  return rc::check_launch(rc::launch_pdl(row_norm_kernel, dim3(M), dim3(kNormThreads), 0, stream, a),
                          "rc_layer_norm");
}

// RMSNorm across the full row (eps, affine bf16 weight) of up to two tensors
// (n_tensors = 1 or 2, e.g. q and k), optionally followed by the interleaved
// rotary embedding with per-token tables cos/sin [span, d] (token = row % span).
// A null weight skips the norm (rotary only).
int rc_rmsnorm_rope(int n_tensors, const void* const* xs, const long long* ldx,
                    const void* const* weights, void* const* outs, const long long* ldo, int M,
                    int N, int d, int span, const float* cos, const float* sin, float eps,
                    cudaStream_t stream) {
  if (n_tensors < 1 || n_tensors > 2 || M < 0 || N <= 0 || N % 8 || N > 4096 ||
      d <= 0 || d % 8 || N % d || span <= 0)
    return rc::set_error(RC_ERR_ARG, "rc_rmsnorm_rope: bad shape (N=%d d=%d span=%d)", N, d, span);
  RmsArgs a{};
  for (int t = 0; t < n_tensors; ++t) {
    if (!xs[t] || !outs[t] || !aligned16(xs[t]) || !aligned16(outs[t]) ||
        (weights[t] && !aligned16(weights[t])) || ldx[t] % 8 || ldo[t] % 8 ||
        (cos && (reinterpret_cast<uintptr_t>(cos) % 16 || reinterpret_cast<uintptr_t>(sin) % 16)))
      return rc::set_error(RC_ERR_ARG, "rc_rmsnorm_rope: tensor %d must be 16-byte aligned", t);
    a.x[t] = reinterpret_cast<const __nv_bfloat16*>(xs[t]);
    a.ldx[t] = ldx[t];
    a.w[t] = reinterpret_cast<const __nv_bfloat16*>(weights[t]);  // null: rotary only
    a.out[t] = reinterpret_cast<__nv_bfloat16*>(outs[t]);
    a.ldo[t] = ldo[t];
  }
  if ((cos == nullptr) != (sin == nullptr))
    return rc::set_error(RC_ERR_ARG, "rc_rmsnorm_rope: cos and sin go together");
  a.cos = cos;
  a.sin = sin;
  a.eps = eps;
  a.M = M;
  a.N = N;
  a.d = d;
  a.span = span;
  if (M == 0) return RC_OK;
  return rc::check_launch(
      rc::launch_pdl(rmsnorm_rope_kernel, dim3(M, n_tensors), dim3(kRowThreads), 0, stream, a),
      "rc_rmsnorm_rope");
}

int rc_temporal_rope(const void* x, long long ldx, void* out, long long ldo, const int* positions,
                     const float* cos, const float* sin, int rows, int span, int heads, int d,
                     int td, cudaStream_t stream) {
  if (rows < 0 || span <= 0 || rows % span || heads <= 0 || d <= 0 || d % 2 || td % 2 || td > d ||
      ldx < heads * d || ldo < heads * d)
    return rc::set_error(RC_ERR_ARG, "rc_temporal_rope: bad shape");
  if (rows == 0) return RC_OK;
  if (reinterpret_cast<uintptr_t>(x) % 4 || reinterpret_cast<uintptr_t>(out) % 4 || ldx % 2 || ldo % 2)
    return rc::set_error(RC_ERR_ARG, "rc_temporal_rope: rows must be 4-byte aligned");
  return rc::check_launch(
      rc::launch_pdl(temporal_rope_kernel, dim3(grid_for((long long)rows * heads * (d / 2), 256)), dim3(256), 0,
                     stream, reinterpret_cast<const __nv_bfloat16*>(x), ldx,
                     reinterpret_cast<__nv_bfloat16*>(out), ldo, positions, cos, sin, rows, span, heads, d, td),
      "rc_temporal_rope");
}

// Copy n_planes retained planes of `span` rows from the block's K/V
// (src plane index = frame offset in the block) into cache slots.
int rc_kv_commit(const void* src_k, const void* src_v, long long src_ld_bytes, void* dst_k,
                 void* dst_v, long long dst_ld_bytes, int row_bytes, int span, int n_planes,
                 const int* src_planes, const int* dst_slots, cudaStream_t stream) {
  if (n_planes < 0 || n_planes > 8 || span <= 0 || row_bytes <= 0 || row_bytes % 16)
    return rc::set_error(RC_ERR_ARG, "rc_kv_commit: bad shape (planes=%d row_bytes=%d)", n_planes, row_bytes);
  if (n_planes == 0) return RC_OK;
  if (!aligned16(src_k) || !aligned16(src_v) || !aligned16(dst_k) || !aligned16(dst_v) ||
      src_ld_bytes % 16 || dst_ld_bytes % 16)
    return rc::set_error(RC_ERR_ARG, "rc_kv_commit: rows must be 16-byte aligned");
  CommitArgs a{};
  a.src[0] = reinterpret_cast<const uint8_t*>(src_k);
  a.src[1] = reinterpret_cast<const uint8_t*>(src_v);
  a.dst[0] = reinterpret_cast<uint8_t*>(dst_k);
  a.dst[1] = reinterpret_cast<uint8_t*>(dst_v);
  a.src_ld[0] = a.src_ld[1] = src_ld_bytes;
  a.dst_ld[0] = a.dst_ld[1] = dst_ld_bytes;
  for (int i = 0; i < n_planes; ++i) {
    if (src_planes[i] < 0 || dst_slots[i] < 0)
      return rc::set_error(RC_ERR_ARG, "rc_kv_commit: negative plane index");
    a.src_plane[i] = src_planes[i];
    a.dst_plane[i] = dst_slots[i];
  }
  a.n = n_planes;
  a.span = span;
  a.row_bytes = row_bytes;
  return rc::check_launch(rc::launch_pdl(kv_commit_kernel, dim3(grid_for(2LL * n_planes * span * (row_bytes / 16), 256)),
                                         dim3(256), 0, stream, a),
                          "rc_kv_commit");
}

// Device-planned variant: plan = [n, (src plane, dst slot) x n] in device
// memory, at most max_planes copies, slots < capacity.
int rc_kv_commit_planned(const void* src_k, const void* src_v, long long src_ld_k_bytes,
                         long long src_ld_v_bytes, void* dst_k, void* dst_v, long long dst_ld_bytes,
                         int row_bytes, int span, int max_planes, int capacity, const int* plan,
                         cudaStream_t stream) {
  if (max_planes < 0 || max_planes > 8 || span <= 0 || row_bytes <= 0 || row_bytes % 16 || capacity < 0)
    return rc::set_error(RC_ERR_ARG, "rc_kv_commit_planned: bad shape");
  if (max_planes == 0 || capacity == 0) return RC_OK;
  if (!plan || !aligned16(src_k) || !aligned16(src_v) || !aligned16(dst_k) || !aligned16(dst_v) ||
      src_ld_k_bytes % 16 || src_ld_v_bytes % 16 || dst_ld_bytes % 16)
    return rc::set_error(RC_ERR_ARG, "rc_kv_commit_planned: rows must be 16-byte aligned");
  if (src_ld_k_bytes < row_bytes || src_ld_v_bytes < row_bytes || dst_ld_bytes < row_bytes)
    return rc::set_error(RC_ERR_ARG, "rc_kv_commit_planned: row stride below row_bytes");
  CommitArgs a{};
  a.src[0] = reinterpret_cast<const uint8_t*>(src_k);
  a.src[1] = reinterpret_cast<const uint8_t*>(src_v);
  a.dst[0] = reinterpret_cast<uint8_t*>(dst_k);
  a.dst[1] = reinterpret_cast<uint8_t*>(dst_v);
  a.src_ld[0] = src_ld_k_bytes;
  a.src_ld[1] = src_ld_v_bytes;
  a.dst_ld[0] = a.dst_ld[1] = dst_ld_bytes;
  a.dst_plane[0] = capacity;
  a.n = max_planes;
  a.span = span;
  a.row_bytes = row_bytes;
  return rc::check_launch(
      rc::launch_pdl(kv_commit_planned_kernel, dim3((span + kCommitRows - 1) / kCommitRows, max_planes, 2),
                     dim3(kCommitThreads), 0, stream, a, plan),
      "rc_kv_commit_planned");
}

}  // extern "C"
