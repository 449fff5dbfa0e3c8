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
__global__ void absmax_bf16_kernel(const __nv_bfloat16* x, int M, int K, long long ldx,
                                   unsigned int* amax_bits) {
  rc::pdl_trigger();
  rc::pdl_wait();
  float m = 0.0f;
  const int kv = K >> 3;  // uint4 per row
  const long long total = (long long)M * kv;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / kv, c = i % kv;
    uint4 v = rc::ld_in(reinterpret_cast<const uint4*>(x + row * ldx) + c);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float a = __uint_as_float(w[j] << 16), b = __uint_as_float(w[j] & 0xffff0000u);
      // NaN must win (torch amax propagates NaN): compare on the bit pattern.
      m = __uint_as_float(max(__float_as_uint(m), __float_as_uint(fabsf(a))));
      m = __uint_as_float(max(__float_as_uint(m), __float_as_uint(fabsf(b))));
    }
  }
  unsigned int mb = __float_as_uint(m);
#pragma unroll
  for (int o = 16; o; o >>= 1) mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, o));
  if ((threadIdx.x & 31) == 0 && mb) atomicMax(amax_bits, mb);
}

__global__ void fp8_quantize_kernel(const __nv_bfloat16* x, int M, int K, long long ldx,
                                    const unsigned int* amax_bits, float* scale_out, uint8_t* q) {
  rc::pdl_trigger();
  rc::pdl_wait();
  float amax = __uint_as_float(rc::ld_in(amax_bits));
  amax = amax < 1e-12f ? 1e-12f : amax;         // clamp_min(1e-12); NaN passes through
  const float scale = __fdiv_rn(amax, 448.0f);
  if (blockIdx.x == 0 && threadIdx.x == 0 && scale_out) *scale_out = scale;
  const int kv = K >> 3;
  const long long total = (long long)M * kv;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / kv, c = i % kv;
    uint4 v = rc::ld_in(reinterpret_cast<const uint4*>(x + row * ldx) + c);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t out[2] = {0, 0};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t h = (j & 1) ? (w[j >> 1] & 0xffff0000u) : (w[j >> 1] << 16);
      float z = __fdiv_rn(__uint_as_float(h), scale);
      z = z > 448.0f ? 448.0f : (z < -448.0f ? -448.0f : z);
      out[j >> 2] |= (uint32_t)rc::e4m3_from_float(z) << (8 * (j & 3));
    }
    *reinterpret_cast<uint2*>(q + row * (long long)K + c * 8) = make_uint2(out[0], out[1]);
  }
}

int grid_for(long long work, int threads) {
  long long b = (work + threads - 1) / threads;
  int sms = 148;
  long long cap = (long long)sms * 8;
  return (int)(b < 1 ? 1 : (b > cap ? cap : b));
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
  const long long work = (long long)M * (K / 8);
  int rc_ = rc::check_launch(rc::launch_pdl(absmax_bf16_kernel, dim3(grid_for(work, 256)), dim3(256), 0, stream,
                                            reinterpret_cast<const __nv_bfloat16*>(x), M, K, ldx, amax_scratch),
                             "rc_fp8_quantize(amax)");
  if (rc_) return rc_;
  return rc::check_launch(rc::launch_pdl(fp8_quantize_kernel, dim3(grid_for(work, 256)), dim3(256), 0, stream,
                                         reinterpret_cast<const __nv_bfloat16*>(x), M, K, ldx,
                                         static_cast<const unsigned int*>(amax_scratch), scale_out, q),
                          "rc_fp8_quantize");
}

}  // extern "C"
