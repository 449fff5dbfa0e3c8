// Activation / weight quantizers. HBM-bound; every output byte is written once.
//
// NVFP4 (recavsr_infer/runtime/nvfp4.py:49-68): per row, per 16-element block,
//   s = e4m3(max(amax(x_blk) / 6 * g, 2^-9)),  z = (x * g) / float(s),
//   code = e2m1 ladder of z, two codes per byte (even element in the low nibble),
//   scales zero-padded to (ceil(M/128)*128, ceil(K/64)*4) and stored in the
//   128x4 blocked order. g = 1 is the reference formula bit for bit; g != 1 is
//   the per-tensor global-scale mode (GEMM then multiplies by 1/(g_a*g_b)).
//
// FP8 (recavsr_infer/runtime/fp8.py:38-42): per-tensor
//   scale = max(amax(|x|), 1e-12) / 448,  q = e4m3(clamp(x / scale, -448, 448)).
#include "common.cuh"

namespace {

constexpr int kQRows = 128;       // rows per CTA (one scale-atom row block)
constexpr int kQThreads = 512;    // 128 rows x 4 k-blocks (one 64-column k-atom)

// One thread per 16-element block; the CTA covers one scale atom (128 rows x
// 4 k-blocks = 512 bytes of scales, written as 32 coalesced 16-byte lines).
__global__ void __launch_bounds__(kQThreads)
nvfp4_quantize_kernel(const __nv_bfloat16* x, int M, int K, long long ldx, float g,
                      uint8_t* codes, uint8_t* scales) {
  __shared__ __align__(16) uint8_t s_line[32][16];
  rc::pdl_trigger();
  rc::pdl_wait();
  const int nkb = K >> 4;
  const int katoms = (nkb + 3) >> 2;
  const int kt = blockIdx.x;
  const int t = threadIdx.x;
  const int r = t >> 2, kk = t & 3;         // row in the atom, k-block in the atom
  const int row = blockIdx.y * kQRows + r, kb = kt * 4 + kk;
  uint8_t sf = 0;
  if (row < M && kb < nkb) {
    const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)row * ldx + (size_t)kb * 16);
    uint4 v0 = rc::ld_in(src), v1 = rc::ld_in(src + 1);
    const uint32_t w[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    float f[16];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      f[2 * j] = __uint_as_float(w[j] << 16);
      f[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
    }
    uint32_t lo = 0, hi = 0;
    if (g == 1.0f) {
      rc::nvfp4_encode16(f, sf, lo, hi);
    } else {
      float amax = 0.0f;
#pragma unroll
      for (int j = 0; j < 16; ++j) amax = rc::absmax_nan(amax, f[j]);
      float sc = __fmul_rn(__fdiv_rn(amax, 6.0f), g);
      sc = sc < 0.001953125f ? 0.001953125f : sc;   // clamp_min(2^-9); NaN passes through
      sf = rc::e4m3_from_float(sc);
      const float sd = rc::e4m3_to_float(sf);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const uint32_t c = rc::e2m1_code(__fdiv_rn(__fmul_rn(f[j], g), sd));
        if (j < 8) lo |= c << (4 * j);
        else hi |= c << (4 * (j - 8));
      }
    }
    *reinterpret_cast<uint2*>(codes + (size_t)row * (K >> 1) + (size_t)kb * 8) = make_uint2(lo, hi);
  }
  // Atom line m0 holds rows {m0, m0+32, m0+64, m0+96} x 4 k-blocks.
  s_line[r & 31][(r >> 5) * 4 + kk] = sf;
  __syncthreads();
  if (t < 32) {
    const uint4 line = *reinterpret_cast<const uint4*>(s_line[t]);
    *reinterpret_cast<uint4*>(scales + ((size_t)(blockIdx.y * katoms + kt) * 32 + t) * 16) = line;
  }
}

// ---------------------------------------------------------------- FP8
// Both passes walk the matrix as 16-byte vectors of 8 bf16 (index i = row *
// K/8 + column vector), kF8Unroll vectors in flight per thread. kDense: rows
// are packed (ldx == K), so vector i sits at x + 8 i and no division is needed.
constexpr int kF8Threads = 256;
constexpr int kF8Unroll = 4;

template <bool kDense>
__device__ __forceinline__ uint4 f8_load(const __nv_bfloat16* x, long long kv, long long ldx, long long i) {
  if (kDense) return rc::ld_in(reinterpret_cast<const uint4*>(x) + i);
  const long long row = i / kv;
  return rc::ld_in(reinterpret_cast<const uint4*>(x + row * ldx) + (i - row * kv));
}

// max over the 8 elements of |x| as fp32 bit patterns: a bf16 is the high half
// of its fp32, clearing the sign gives |x|, and unsigned order of non-negative
// fp32 patterns is numeric order with NaN above +inf (torch's amax propagates
// NaN, so NaN must win).
__device__ __forceinline__ uint32_t absmax8_bits(uint4 v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t m = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) m = max(m, max((w[j] << 16) & 0x7fffffffu, w[j] & 0x7fff0000u));
  return m;
}

template <bool kDense>
__global__ void __launch_bounds__(kF8Threads) absmax_bf16_kernel(const __nv_bfloat16* x, int M, int K,
                                                                  long long ldx, unsigned int* amax_bits) {
  rc::pdl_trigger();
  rc::pdl_wait();
  const long long kv = K >> 3, total = (long long)M * kv;
  const long long stride = (long long)gridDim.x * kF8Threads;
  long long i = blockIdx.x * (long long)kF8Threads + threadIdx.x;
  uint32_t m = 0;
  for (; i + (kF8Unroll - 1) * stride < total; i += kF8Unroll * stride) {
    uint4 v[kF8Unroll];
#pragma unroll
    for (int u = 0; u < kF8Unroll; ++u) v[u] = f8_load<kDense>(x, kv, ldx, i + u * stride);
#pragma unroll
    for (int u = 0; u < kF8Unroll; ++u) m = max(m, absmax8_bits(v[u]));
  }
  for (; i < total; i += stride) m = max(m, absmax8_bits(f8_load<kDense>(x, kv, ldx, i)));
#pragma unroll
  for (int o = 16; o; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ uint32_t s_max[kF8Threads / 32];
  if ((threadIdx.x & 31) == 0) s_max[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < kF8Threads / 32 ? s_max[threadIdx.x] : 0u;
#pragma unroll
    for (int o = 4; o; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (threadIdx.x == 0 && m) atomicMax(amax_bits, m);
  }
}

// Four fp32 -> four E4M3 bytes (element 0 in the low byte). The clamp to
// +-448 of the reference is the conversion's satfinite (finite values above
// 448 and +-inf give +-448, the same codes the clamp gives); only NaN differs:
// the reference's encoder gives sign | 0x7f, the conversion a fixed NaN code.
// Clamped finite values never produce a 0x7f magnitude (448 is 0x7e), so the
// 0x7f magnitudes are exactly the NaN inputs and are patched from the signs.
__device__ __forceinline__ uint32_t e4m3x4(const float (&z)[4]) {
  uint16_t lo, hi;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(lo) : "f"(z[1]), "f"(z[0]));
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(hi) : "f"(z[3]), "f"(z[2]));
  uint32_t q = (uint32_t)lo | ((uint32_t)hi << 16);
  if (__vcmpeq4(q & 0x7f7f7f7fu, 0x7f7f7f7fu)) {
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (z[j] != z[j]) {
        const uint32_t code = 0x7fu | ((__float_as_uint(z[j]) >> 24) & 0x80u);
        q = (q & ~(0xffu << (8 * j))) | (code << (8 * j));
      }
  }
  return q;
}

// x / scale for the 8 elements of one vector, IEEE-rounded like torch's
// division. kRecip (scale finite and normal, every call whose input is
// finite): with y = RN(1/scale), q = RN(|x| y) and one step of Markstein's
// correction (P. Markstein, IBM J. Res. Develop. 34(1), 1990: r = |x| - scale
// q exactly by one fma, q' = RN(q + r y)) give RN(|x| / scale); the sign is
// put back afterwards so that -0 and negative underflow keep it. An
// exhaustive CPU replay of this sequence over every bf16 |x| <= amax and
// every scale a bf16 amax yields (4.7e8 pairs) matches correctly rounded
// division bit for bit. Otherwise (scale inf or NaN) a full division.
template <bool kRecip>
__device__ __forceinline__ uint2 fp8_codes8(uint4 v, float scale, float recip) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  float z[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t h = (j & 1) ? (w[j >> 1] & 0xffff0000u) : (w[j >> 1] << 16);
    if (kRecip) {
      const float ax = __uint_as_float(h & 0x7fffffffu);
      const float q = __fmul_rn(ax, recip);
      const float r = __fmaf_rn(-q, scale, ax);
      z[j] = __uint_as_float(__float_as_uint(__fmaf_rn(r, recip, q)) | (h & 0x80000000u));
    } else {
      z[j] = __fdiv_rn(__uint_as_float(h), scale);
    }
  }
  const float z0[4] = {z[0], z[1], z[2], z[3]}, z1[4] = {z[4], z[5], z[6], z[7]};
  return make_uint2(e4m3x4(z0), e4m3x4(z1));
}

template <bool kDense, bool kRecip>
__device__ __forceinline__ void fp8_quantize_rows(const __nv_bfloat16* x, long long kv, long long ldx,
                                                  long long total, float scale, uint2* out) {
  const float recip = kRecip ? __frcp_rn(scale) : 0.0f;
  const long long stride = (long long)gridDim.x * kF8Threads;
  long long i = blockIdx.x * (long long)kF8Threads + threadIdx.x;
  for (; i + (kF8Unroll - 1) * stride < total; i += kF8Unroll * stride) {
    uint4 v[kF8Unroll];
#pragma unroll
    for (int u = 0; u < kF8Unroll; ++u) v[u] = f8_load<kDense>(x, kv, ldx, i + u * stride);
#pragma unroll
    for (int u = 0; u < kF8Unroll; ++u) out[i + u * stride] = fp8_codes8<kRecip>(v[u], scale, recip);
  }
  for (; i < total; i += stride) out[i] = fp8_codes8<kRecip>(f8_load<kDense>(x, kv, ldx, i), scale, recip);
}

template <bool kDense>
__global__ void __launch_bounds__(kF8Threads) fp8_quantize_kernel(const __nv_bfloat16* x, int M, int K,
                                                                   long long ldx, const unsigned int* amax_bits,
                                                                   float* scale_out, uint8_t* q) {
  rc::pdl_trigger();
  rc::pdl_wait();
  float amax = __uint_as_float(rc::ld_in(amax_bits));
  amax = amax < 1e-12f ? 1e-12f : amax;         // clamp_min(1e-12); NaN passes through
  const float scale = __fdiv_rn(amax, 448.0f);
  if (blockIdx.x == 0 && threadIdx.x == 0 && scale_out) *scale_out = scale;
  const long long kv = K >> 3, total = (long long)M * kv;
  uint2* out = reinterpret_cast<uint2*>(q);     // q is packed M x K: vector i -> bytes 8i..8i+7
  if (isfinite(scale) && scale >= 0x1p-126f)    // normal and finite; uniform over the grid
    fp8_quantize_rows<kDense, true>(x, kv, ldx, total, scale, out);
  else
    fp8_quantize_rows<kDense, false>(x, kv, ldx, total, scale, out);
}

}  // namespace

RC_DEVICE_ERROR_ACCESSOR(quant)

extern "C" {

int rc_nvfp4_quantize(const void* x, int M, int K, long long ldx, float global_scale,
                      uint8_t* codes, uint8_t* scales_swizzled, cudaStream_t stream) {
  if (M < 0 || K <= 0 || K % 16)
    return rc::set_error(RC_ERR_ARG, "rc_nvfp4_quantize: K must be a positive multiple of 16 (M=%d K=%d)", M, K);
  if (!x || !codes || !scales_swizzled)
    return rc::set_error(RC_ERR_ARG, "rc_nvfp4_quantize: null pointer");
  if (ldx < K || (ldx * 2) % 16 || reinterpret_cast<uintptr_t>(x) % 16 ||
      reinterpret_cast<uintptr_t>(codes) % 8 || reinterpret_cast<uintptr_t>(scales_swizzled) % 16)
    return rc::set_error(RC_ERR_ARG, "rc_nvfp4_quantize: rows must be 16-byte aligned (ldx=%lld)", ldx);
  if (!(global_scale > 0.0f))
    return rc::set_error(RC_ERR_ARG, "rc_nvfp4_quantize: global scale must be positive");
  if (M == 0) return RC_OK;
  const int nkb = K / 16;
  dim3 grid((nkb + 3) / 4, (M + kQRows - 1) / kQRows);
  return rc::check_launch(
      rc::launch_pdl(nvfp4_quantize_kernel, grid, dim3(kQThreads), 0, stream,
                     reinterpret_cast<const __nv_bfloat16*>(x), M, K, ldx, global_scale, codes, scales_swizzled),
      "rc_nvfp4_quantize");
}

// amax_scratch: one 32-bit device word, overwritten by this call.
int rc_fp8_quantize(const void* x, int M, int K, long long ldx, unsigned int* amax_scratch,
                    float* scale_out, uint8_t* q, cudaStream_t stream) {
  if (M < 0 || K <= 0 || K % 8)
    return rc::set_error(RC_ERR_ARG, "rc_fp8_quantize: K must be a positive multiple of 8");
  if (!x || !q || !amax_scratch || !scale_out)
    return rc::set_error(RC_ERR_ARG, "rc_fp8_quantize: null pointer");
  if (ldx < K || (ldx * 2) % 16 || reinterpret_cast<uintptr_t>(x) % 16 ||
      reinterpret_cast<uintptr_t>(q) % 8)
    return rc::set_error(RC_ERR_ARG, "rc_fp8_quantize: rows must be 16-byte aligned");
  if (cudaMemsetAsync(amax_scratch, 0, sizeof(unsigned int), stream) != cudaSuccess)
    return rc::set_error(RC_ERR_CUDA, "rc_fp8_quantize: memset failed");
  if (M == 0) return RC_OK;
  // kF8Unroll vectors per thread per pass, at most 4 CTAs per SM (one wave).
  const long long work = (long long)M * (K / 8);
  long long blocks = (work + kF8Threads * kF8Unroll - 1) / (kF8Threads * kF8Unroll);
  const long long cap = 4LL * rc::sm_count();
  const dim3 grid((unsigned)(blocks > cap ? cap : blocks));
  const bool dense = ldx == K;
  const auto* xb = reinterpret_cast<const __nv_bfloat16*>(x);
  int rc_ = rc::check_launch(dense ? rc::launch_pdl(absmax_bf16_kernel<true>, grid, dim3(kF8Threads), 0, stream,
                                                    xb, M, K, ldx, amax_scratch)
                                   : rc::launch_pdl(absmax_bf16_kernel<false>, grid, dim3(kF8Threads), 0, stream,
                                                    xb, M, K, ldx, amax_scratch),
                             "rc_fp8_quantize(amax)");
  if (rc_) return rc_;
  const auto* amax = static_cast<const unsigned int*>(amax_scratch);
  return rc::check_launch(dense ? rc::launch_pdl(fp8_quantize_kernel<true>, grid, dim3(kF8Threads), 0, stream,
                                                 xb, M, K, ldx, amax, scale_out, q)
                                : rc::launch_pdl(fp8_quantize_kernel<false>, grid, dim3(kF8Threads), 0, stream,
                                                 xb, M, K, ldx, amax, scale_out, q),
                          "rc_fp8_quantize");
}

}  // extern "C"
