// Shared host/device helpers for the ReCaVSR B200 kernels.
//
// Status convention of every extern "C" entry point (include/recavsr_b200.h):
//   0 = ok, 1 = invalid argument, 2 = CUDA error, 3 = device wait timed out,
//   4 = unsupported configuration. The message of the last failure on the
//   calling host thread is kept for rc_get_last_error().
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>
#include <math.h>

#define RC_OK 0
#define RC_ERR_ARG 1
#define RC_ERR_CUDA 2
#define RC_ERR_TIMEOUT 3
#define RC_ERR_UNSUPPORTED 4

// Device-side error word, one per translation unit. A kernel whose bounded
// wait gives up (or that sees an impossible index) stores a non-zero code here
// and returns early; the host reads and clears every unit's word with
// rc_read_device_error().
//   bits 0..7  = kernel id, bits 8..15 = site, bits 16..31 = block id (low bits)
static __device__ unsigned int g_rc_device_error;

// Defines `unsigned int rc_take_device_error_<tag>()` for this unit.
#define RC_DEVICE_ERROR_ACCESSOR(tag)                                              \
  unsigned int rc_take_device_error_##tag() {                                      \
    unsigned int v = 0, zero = 0;                                                  \
    if (cudaMemcpyFromSymbol(&v, g_rc_device_error, sizeof(v)) != cudaSuccess)     \
      return 0xffffffffu;                                                          \
    if (v) cudaMemcpyToSymbol(g_rc_device_error, &zero, sizeof(zero));            \
    return v;                                                                      \
  }

// Kernel ids stored in the low byte of the error word.
enum RcKernelId : unsigned int {
  kKernQuant = 1, kKernGemmNvf4 = 2, kKernGemmFp8 = 3, kKernAttention = 4,
  kKernGlue = 5, kKernCache = 6, kKernDecoderAttention = 7,
};

namespace rc {

int set_error(int code, const char* fmt, ...);
int check_launch(const char* what);
int check_launch(cudaError_t launched, const char* what);   // result of launch_pdl
int sm_count();   // streaming multiprocessors of the current device (cached per device)

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) applies to the current
// device only, so each kernel keeps one flag per device. A flag is set after
// the attribute call succeeded; two threads may both make the (idempotent)
// call before either sets it.
constexpr int kMaxDevices = 64;
struct SmemAttrFlags {
  volatile int set[kMaxDevices];
};
int ensure_smem_attr(SmemAttrFlags& flags, const void* func, int bytes, const char* what);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
// dims/strides: innermost first; strides are in bytes for dims 1..rank-1.
int encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, void* base,
                const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                CUtensorMapSwizzle swizzle, const char* what);

// Programmatic dependent launch. Every kernel of the library is launched with
// launch_pdl (below) and starts with pdl_trigger(); pdl_wait(): the next
// kernel in the stream may begin launching onto SMs this grid frees up (its
// prologue -- barrier init, TMEM allocation, tensor-map prefetch -- overlaps
// this grid's tail), and no kernel reads global memory before pdl_wait(),
// which returns once the preceding grid has completed and its writes are
// visible. Because every kernel waits on its predecessor before finishing,
// the ordering is transitive along the stream.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Global loads of kernel inputs. With programmatic dependent launch a kernel
// is resident while the kernels before it in the stream still write its
// inputs, so the read-only non-coherent path (ld.global.nc, which __ldg and
// `const __restrict__` pointers select) does not apply: it is defined only for
// data that nothing writes during the kernel's lifetime, and the compiler may
// schedule such loads ahead of pdl_wait(). These are ordinary coherent loads
// through a pointer the compiler cannot prove read-only; the "memory" clobber
// of pdl_wait() keeps them after it, and independent loads still overlap.
template <typename T>
__device__ __forceinline__ T ld_in(const T* p) {
  return *p;
}

// Pull the 128-byte line holding p into L1 (no register result, no wait).
__device__ __forceinline__ void prefetch_l1(const void* p) {
  asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
}

// launch_pdl with thread-block clusters of `cluster_x` CTAs along x.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                      cudaStream_t stream, unsigned cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cluster_x;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Launch `kernel` on `stream` with programmatic stream serialization allowed.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Device: record the first error only.
__device__ __forceinline__ void device_fail(unsigned int kernel_id, unsigned int site) {
  unsigned int word = (kernel_id & 0xffu) | ((site & 0xffu) << 8) |
                      ((blockIdx.x & 0xffffu) << 16);
  atomicCAS(&g_rc_device_error, 0u, word);
}

// Wall-clock bound of any device-side wait (mbarrier phase, flag): far above
// any legitimate wait inside one kernel, yet it guarantees that a kernel never
// hangs the GPU. Measured on %globaltimer (nanoseconds).
constexpr unsigned long long kWaitNs = 4000000000ull;

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------
// FP8 E4M3 (fn variant: no infinities, 0x7f / 0xff are NaN, max finite 448).
// Round-to-nearest-even, subnormals kept, magnitudes >= 480 (and NaN) map to
// the NaN code 0x7f with the input's sign: the same results as PyTorch's
// float -> float8_e4m3fn cast that the reference quantizers use.
// Derivation: subnormal grid is k * 2^-9 (k = 0..7); the normal grid within
// [2^e, 2^(e+1)) is 2^e * (1 + j/8). Rounding a*2^9 or the mantissa fraction
// with rintf (RNE) gives the code directly; a carry rolls into the exponent.
// ---------------------------------------------------------------------------
__host__ __device__ __forceinline__ uint8_t e4m3_from_float(float v) {
  uint32_t bits;
#ifdef __CUDA_ARCH__
  bits = __float_as_uint(v);
#else
  memcpy(&bits, &v, 4);
#endif
  const uint8_t sign = (uint8_t)((bits >> 24) & 0x80u);
  const float a = fabsf(v);
  if (!(a < 480.0f)) return (uint8_t)(sign | 0x7fu);
  if (a < 0.015625f) {  // below 2^-6: subnormal grid of 2^-9
    const int k = (int)rintf(a * 512.0f);
    return (uint8_t)(sign | (uint8_t)k);  // k == 8 is exactly the min normal 0x08
  }
  int e;
  const float m = frexpf(a, &e);  // a = m * 2^e, m in [0.5, 1)
  // a = (2m) * 2^(e-1), 2m in [1, 2); biased exponent = e - 1 + 7
  const int j = (int)rintf((2.0f * m - 1.0f) * 8.0f);
  const int code = ((e + 6) << 3) + j;  // a carry (j == 8) bumps the exponent
  return (uint8_t)(sign | (uint8_t)code);
}

__host__ __device__ __forceinline__ float e4m3_to_float(uint8_t c) {
  const int s = c >> 7, e = (c >> 3) & 0xf, m = c & 7;
  float v;
  if (e == 0xf && m == 7) {
    v = NAN;
  } else if (e == 0) {
    v = ldexpf((float)m, -9);
  } else {
    v = ldexpf(1.0f + (float)m * 0.125f, e - 7);
  }
  return s ? -v : v;
}

// E2M1 code of z (magnitudes 0, .5, 1, 1.5, 2, 3, 4, 6; ties to even) as the
// count of thresholds passed, strict at .25/1.25/2.5/5 and inclusive at
// .75/1.75/3.5, with the sign bit (8) set for z < 0 only (so -0 and NaN give
// code 0). Same decision ladder as recavsr_infer/runtime/nvfp4.py:56-61.
__host__ __device__ __forceinline__ uint32_t e2m1_code(float z) {
  const float a = fabsf(z);
  uint32_t c = (a > 0.25f) + (a >= 0.75f) + (a > 1.25f) + (a >= 1.75f) + (a > 2.5f) +
               (a >= 3.5f) + (a > 5.0f);
  return c | (z < 0.0f ? 8u : 0u);
}

// NaN-propagating max of |x| (torch's amax propagates NaN).
__host__ __device__ __forceinline__ float absmax_nan(float m, float x) {
  const float a = fabsf(x);
  return (a > m || a != a) ? a : m;
}

// (a, b) -> bf16x2 word with a in the low half (one cvt.rn.bf16x2.f32).
__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// NaN-propagating max of three magnitudes (three-input max.NaN, sm_100).
__device__ __forceinline__ float absmax3_nan(float a, float b, float c) {
  float d;
  asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(fabsf(a)), "f"(fabsf(b)), "f"(fabsf(c)));
  return d;
}

// Eight fp32 values -> eight E2M1 codes (round to nearest even, saturating to
// +-6), value j in nibble j, by the hardware e2m1x2 conversion.
__device__ __forceinline__ uint32_t e2m1x8_rn(const float* q) {
  uint32_t out;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
      "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
      : "=r"(out)
      : "f"(q[0]), "f"(q[1]), "f"(q[2]), "f"(q[3]), "f"(q[4]), "f"(q[5]), "f"(q[6]), "f"(q[7]));
  return out;
}

// NVFP4 encoding of bf16-valued x with global scale 1
// (recavsr_infer/runtime/nvfp4.py:49-61): scale byte e4m3(max(amax/6, 2^-9))
// and codes e2m1(fl(x / s)), bit for bit. nvfp4_codes8 codes 8 values for a
// finite scale s; nvfp4_encode16 does a whole 16-element block.
//   The quotient: q = x * r with r ~ 1/s (MUFU reciprocal), refined once by the
//   exact residual, q' = q + (x - q*s) * r. The codes only depend on which side
//   of each E2M1 rounding threshold t (0.25, 0.75, ..., 5) fl(x/s) falls, and on
//   exact ties x = t*s. Away from ties x/s lies at least 2^-9 (relative) from
//   every t (x has 8 significant bits, t*s at most 7), far beyond the ~2^-21
//   error of q'; at a tie the residual is exact and q' rounds to t itself, where
//   the conversion's round-to-nearest-even breaks the tie as the reference's
//   strict / inclusive thresholds do. x = -0 gives q' = +0 (code 0, no sign,
//   like the reference's z < 0 test); a NaN scale (NaN or huge amax) gives code
//   0 for every element, as x / NaN does.
__device__ __forceinline__ uint32_t nvfp4_codes8(const float* x, float s) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(s));
  const float2 r2 = make_float2(r, r), ns2 = make_float2(-s, -s);
  float q[8];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 xv = make_float2(x[2 * j], x[2 * j + 1]);
    const float2 q0 = __fmul2_rn(xv, r2);
    const float2 rem = __ffma2_rn(q0, ns2, xv);
    const float2 q1 = __ffma2_rn(rem, r2, q0);
    q[2 * j] = q1.x;
    q[2 * j + 1] = q1.y;
  }
  return e2m1x8_rn(q);
}

// fl32(a / 6) for a bf16-valued a >= 0 without a division: q = a * fl(1/6),
// refined once by the exact residual. Bit-identical to IEEE division for every
// finite non-negative bf16 a (checked exhaustively by
// tests/test_oracle_golden.py::test_div6_is_exact_for_bf16); NaN and inf give NaN.
__device__ __forceinline__ float div6_bf16(float a) {
  constexpr float r6 = 1.0f / 6.0f;
  const float q = a * r6;
  return fmaf(fmaf(-q, 6.0f, a), r6, q);
}

// E4M3 code of v >= 0 (or NaN), round to nearest even, subnormals kept; as
// e4m3_from_float: above 464 (the tie between 448 and the next step, which is
// the NaN code) and for NaN the result is the NaN code 0x7f. The hardware
// conversion saturates instead, so it only sees v <= 464.
__device__ __forceinline__ uint8_t e4m3_rn_nonneg(float v) {
  if (!(v <= 464.0f)) return 0x7f;
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(0.0f), "f"(v));
  return (uint8_t)(r & 0xff);
}

// Value of a non-negative, non-NaN E4M3 code: its 7 magnitude bits placed at
// bit 20 of an fp32 read as 2^(E-127) (1 + M/8) (or the fp32 subnormal M 2^-129
// when E = 0), times 2^120 -> 2^(E-7) (1 + M/8) (or M 2^-9). Needs fp32
// subnormals kept (no flush-to-zero), which is the default.
__device__ __forceinline__ float e4m3_nonneg_to_float(uint8_t c) {
  return __uint_as_float((uint32_t)(c & 0x7f) << 20) * 0x1p120f;
}

// Scale byte of a block from its (NaN-propagating) amax, global scale 1.
__device__ __forceinline__ uint8_t nvfp4_scale_byte(float amax) {
  float sc = div6_bf16(amax);
  sc = sc < 0.001953125f ? 0.001953125f : sc;   // clamp_min(2^-9); NaN passes through
  return e4m3_rn_nonneg(sc);
}

__device__ __forceinline__ void nvfp4_encode16(const float (&x)[16], uint8_t& sfb, uint32_t& lo,
                                               uint32_t& hi) {
  float m[5];
#pragma unroll
  for (int j = 0; j < 5; ++j) m[j] = absmax3_nan(x[3 * j], x[3 * j + 1], x[3 * j + 2]);
  const float amax = absmax3_nan(absmax3_nan(m[0], m[1], m[2]), absmax3_nan(m[3], m[4], x[15]), 0.0f);
  sfb = nvfp4_scale_byte(amax);
  if (sfb == 0x7f) {   // NaN scale
    lo = hi = 0;
    return;
  }
  const float s = e4m3_nonneg_to_float(sfb);
  lo = nvfp4_codes8(x, s);
  hi = nvfp4_codes8(x + 8, s);
}

// ---- softmax helpers shared by the attention kernels
__device__ __forceinline__ float max3(float a, float b, float c) {   // three-input max (sm_100)
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float fast_exp2(float x) {   // MUFU ex2 (as tl.exp2)
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x for two x <= 2^7 on the FMA pipe: x = j + f with j = rint(x) (by the
// 1.5 * 2^23 rounding constant) and |f| <= 1/2; 2^f by a degree-4 polynomial
// (coefficients fitted here: relative error <= 8.5e-6 on [-1/2, 1/2], far
// below the bf16 rounding of P) and j added to the exponent field. x < -126
// gives 0, as the flush-to-zero MUFU exp2 does.
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  constexpr float kRound = 12582912.0f;
  const float2 xc = make_float2(fmaxf(x.x, -127.0f), fmaxf(x.y, -127.0f));
  const float2 t = __fadd2_rn(xc, make_float2(kRound, kRound));
  const float2 j = __fadd2_rn(t, make_float2(-kRound, -kRound));
  const float2 f = __ffma2_rn(j, make_float2(-1.0f, -1.0f), xc);
  float2 q = __ffma2_rn(make_float2(0.00925496f, 0.00925496f), f, make_float2(0.05585603f, 0.05585603f));
  q = __ffma2_rn(q, f, make_float2(0.24031252f, 0.24031252f));
  q = __ffma2_rn(q, f, make_float2(0.6931306f, 0.6931306f));
  q = __ffma2_rn(q, f, make_float2(0.9999978f, 0.9999978f));
  const float ex = __uint_as_float(__float_as_uint(q.x) + (__float_as_uint(t.x) << 23));
  const float ey = __uint_as_float(__float_as_uint(q.y) + (__float_as_uint(t.y) << 23));
  return make_float2(x.x < -126.0f ? 0.0f : ex, x.y < -126.0f ? 0.0f : ey);
}

// Offset of the scale byte for (row, k-block) in the 128x4 blocked layout
// (recavsr_infer/runtime/nvfp4.py:64-67): atoms of 128 rows x 4 k-blocks,
// k-atoms innermost; inside an atom, row r = 32*m1 + m0 and k-block kk sit at
// m0*16 + m1*4 + kk.
__host__ __device__ __forceinline__ size_t sf_offset(int row, int kb, int katoms) {
  const int mb = row >> 7, r = row & 127, m0 = r & 31, m1 = r >> 5;
  const int kt = kb >> 2, kk = kb & 3;
  return ((size_t)(mb * katoms + kt) * 32 + m0) * 16 + m1 * 4 + kk;
}

// Round-to-nearest-even float -> bf16 bits (NaN kept quiet).
__host__ __device__ __forceinline__ uint16_t bf16_bits(float f) {
#ifdef __CUDA_ARCH__
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
#else
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
#endif
}
__host__ __device__ __forceinline__ float bf16_to_float(uint16_t h) {
#ifdef __CUDA_ARCH__
  return __uint_as_float((uint32_t)h << 16);
#else
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
#endif
}

}  // namespace rc
