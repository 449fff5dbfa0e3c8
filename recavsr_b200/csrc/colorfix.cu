// Colour correction of decoded frames (recavsr_infer/color_fix.py:18-117).
//
// rc_cf_adain: AdaIN per frame and RGB channel (color_fix.py:18-29,58-81). A
// first pass writes per-(plane, chunk) sums and sums of squares of content and
// reference in fp64 (content = (x + 1) * 0.5 in fp32, as the reference maps
// [-1, 1] to [0, 1]); the apply pass reduces its plane's chunks, forms the
// sample variance (plain variance for one-pixel planes), and writes
// ((c - mean_c) * sqrt((var_r + 1e-5) / (var_c + 1e-5)) + mean_r) * 2 - 1 (fp32).
//
// rc_cf_bicubic_u8 + rc_cf_wavelet_level: wavelet correction (:32-55,84-117).
// The LQ uint8 frames are upsampled to the decoded size by cubic convolution
// (Keys, A = -0.75; torch's upsample_bicubic2d with align_corners=False: source
// x = (dst + 0.5) * in / out - 0.5, the 4 taps clamped to the image) of
// lq / 255, clamped to [0, 1]. Each of the 5 levels (dilations 1, 2, 4, 8, 16)
// blurs the content and the reference lows with [1, 2, 1]^T [1, 2, 1] / 16
// (replicate padding) and adds low - blur into the content's high part; the
// first level reads the content as clamp((decoded + 1) * 0.5, 0, 1) from the
// decoded [3, T, H, W] frames, the last writes uint8 round(clamp(high +
// blurred reference, 0, 1) * 255) as [T, H, W, 3]. Internal planes are
// [T * 3, H, W] fp32 (frame-major, as the reference permutes).
#include "common.cuh"

namespace {

constexpr int kChunk = 16384;          // elements per partial-sum chunk

__device__ __forceinline__ float load_as_float(const void* p, long long i, int dtype) {
  if (dtype == 0) return rc::ld_in(reinterpret_cast<const float*>(p) + i);
  return __bfloat162float(rc::ld_in(reinterpret_cast<const __nv_bfloat16*>(p) + i));
}

__device__ __forceinline__ double block_sum_d(double v, double* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  double s = 0.0;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) s += red[i];
  return s;
}

// grid (chunks, planes): sums of c, c^2, r, r^2 over one chunk of one plane.
__global__ void __launch_bounds__(256) adain_partial_kernel(const void* content, int dc, const void* ref, int dr,
                                                            long long hw, double* part, int chunks) {
  __shared__ double red[8];
  rc::pdl_trigger();
  rc::pdl_wait();
  const long long plane = blockIdx.y, base = plane * hw;
  const long long lo = (long long)blockIdx.x * kChunk, hi = min(lo + kChunk, hw);
  double s[4] = {0, 0, 0, 0};
  for (long long i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    const float c = __fmul_rn(__fadd_rn(load_as_float(content, base + i, dc), 1.0f), 0.5f);
    const float r = __fmul_rn(__fadd_rn(load_as_float(ref, base + i, dr), 1.0f), 0.5f);
    s[0] += c;
    s[1] += (double)c * c;
    s[2] += r;
    s[3] += (double)r * r;
  }
  double* dst = part + (plane * chunks + blockIdx.x) * 4;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const double t = block_sum_d(s[k], red);
    if (threadIdx.x == 0) dst[k] = t;
  }
}

// grid (blocks, planes): reduce the plane's chunks, then apply.
__global__ void __launch_bounds__(256) adain_apply_kernel(const void* content, int dc, long long hw,
                                                          const double* part, int chunks, float* out) {
  __shared__ float coef[3];                 // mean_c, gain, mean_r
  rc::pdl_trigger();
  rc::pdl_wait();
  const long long plane = blockIdx.y;
  if (threadIdx.x == 0) {
    double s[4] = {0, 0, 0, 0};
    for (int q = 0; q < chunks; ++q)
      for (int k = 0; k < 4; ++k) s[k] += rc::ld_in(part + (plane * chunks + q) * 4 + k);
    const double n = (double)hw, den = hw > 1 ? n - 1.0 : n;
    const double mc = s[0] / n, mr = s[2] / n;
    const double vc = fmax(s[1] - s[0] * mc, 0.0) / den, vr = fmax(s[3] - s[2] * mr, 0.0) / den;
    coef[0] = (float)mc;
    coef[1] = (float)sqrt((vr + 1e-5) / (vc + 1e-5));
    coef[2] = (float)mr;
  }
  __syncthreads();
  const float mc = coef[0], gain = coef[1], mr = coef[2];
  const long long base = plane * hw;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < hw; i += (long long)gridDim.x * blockDim.x) {
    const float c = __fmul_rn(__fadd_rn(load_as_float(content, base + i, dc), 1.0f), 0.5f);
    const float y = __fadd_rn(__fmul_rn(__fsub_rn(c, mc), gain), mr);
    out[base + i] = __fsub_rn(__fmul_rn(y, 2.0f), 1.0f);
  }
}

// Keys' cubic convolution weights (A = -0.75) of taps -1, 0, 1, 2 at fraction t.
__device__ __forceinline__ void cubic_coeffs(float t, float (&c)[4]) {
  constexpr float A = -0.75f;
  auto conv1 = [](float x) { return __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(__fmul_rn(A + 2.0f, x), A + 3.0f), x), x), 1.0f); };
  auto conv2 = [](float x) {
    return __fsub_rn(__fmul_rn(__fadd_rn(__fmul_rn(__fsub_rn(__fmul_rn(A, x), 5.0f * A), x), 8.0f * A), x), 4.0f * A);
  };
  c[0] = conv2(__fadd_rn(t, 1.0f));
  c[1] = conv1(t);
  c[2] = conv1(__fsub_rn(1.0f, t));
  c[3] = conv2(__fadd_rn(__fsub_rn(1.0f, t), 1.0f));
}

// One thread per output pixel of one (frame, channel) plane: out [T*3, H, W].
__global__ void __launch_bounds__(256) bicubic_u8_kernel(const uint8_t* lq, int T, int h, int w, int H, int W,
                                                         float* out) {
  __shared__ float inv255[256];          // k / 255 (the same IEEE division per byte value)
  inv255[threadIdx.x] = __fdiv_rn((float)threadIdx.x, 255.0f);
  __syncthreads();
  rc::pdl_trigger();
  rc::pdl_wait();
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)T * 3 * H * W) return;
  const int x = (int)(i % W), y = (int)((i / W) % H);
  const long long p = i / ((long long)H * W);
  const int t = (int)(p / 3), c = (int)(p % 3);
  const float sx = __fsub_rn(__fmul_rn(__fadd_rn((float)x, 0.5f), (float)w / (float)W), 0.5f);
  const float sy = __fsub_rn(__fmul_rn(__fadd_rn((float)y, 0.5f), (float)h / (float)H), 0.5f);
  const float fx = floorf(sx), fy = floorf(sy);
  float cx[4], cy[4];
  cubic_coeffs(__fsub_rn(sx, fx), cx);
  cubic_coeffs(__fsub_rn(sy, fy), cy);
  const int ix = (int)fx, iy = (int)fy;
  const uint8_t* frame = lq + (long long)t * h * w * 3 + c;
  float acc = 0.f;
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int yy = min(max(iy - 1 + a, 0), h - 1);
    float row = 0.f;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int xx = min(max(ix - 1 + b, 0), w - 1);
      const float v = inv255[rc::ld_in(frame + ((long long)yy * w + xx) * 3)];
      row = __fadd_rn(row, __fmul_rn(v, cx[b]));
    }
    acc = __fadd_rn(acc, __fmul_rn(row, cy[a]));
  }
  out[i] = fminf(fmaxf(acc, 0.f), 1.f);
}

struct LevelArgs {
  const void* decoded;   // first level: [3, T, H, W] in [-1, 1] (dtype)
  int dtype;
  const float* low_c;    // later levels: [T*3, H, W]
  const float* low_r;
  float* blur_c;
  float* blur_r;
  float* high;
  uint8_t* out;          // last level: [T, H, W, 3]
  int T, H, W, r, first, last;
};

__device__ __forceinline__ float content_at(const LevelArgs& a, int t, int c, int y, int x) {
  if (a.first) {
    const long long i = (((long long)c * a.T + t) * a.H + y) * a.W + x;
    return fminf(fmaxf(__fmul_rn(__fadd_rn(load_as_float(a.decoded, i, a.dtype), 1.0f), 0.5f), 0.f), 1.f);
  }
  return rc::ld_in(a.low_c + (((long long)t * 3 + c) * a.H + y) * a.W + x);
}

// One thread per pixel of one (frame, channel) plane.
__global__ void __launch_bounds__(256) wavelet_level_kernel(LevelArgs a) {
  rc::pdl_trigger();
  rc::pdl_wait();
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)a.T * 3 * a.H * a.W) return;
  const int x = (int)(i % a.W), y = (int)((i / a.W) % a.H);
  const long long p = i / ((long long)a.H * a.W);
  const int t = (int)(p / 3), c = (int)(p % 3);
  const int ys[3] = {max(y - a.r, 0), y, min(y + a.r, a.H - 1)};
  const int xs[3] = {max(x - a.r, 0), x, min(x + a.r, a.W - 1)};
  constexpr float k[3] = {0.25f, 0.5f, 0.25f};
  float bc = 0.f, br = 0.f;
  const float* lr = a.low_r + p * a.H * a.W;
#pragma unroll
  for (int u = 0; u < 3; ++u)
#pragma unroll
    for (int v = 0; v < 3; ++v) {
      const float wgt = k[u] * k[v];
      bc = __fadd_rn(bc, __fmul_rn(content_at(a, t, c, ys[u], xs[v]), wgt));
      br = __fadd_rn(br, __fmul_rn(rc::ld_in(lr + (long long)ys[u] * a.W + xs[v]), wgt));
    }
  const float lc = content_at(a, t, c, y, x);
  const float hi = __fadd_rn(a.first ? 0.f : rc::ld_in(a.high + i), __fsub_rn(lc, bc));
  if (a.last) {
    const float fixed = fminf(fmaxf(__fadd_rn(hi, br), 0.f), 1.f);
    a.out[(((long long)t * a.H + y) * a.W + x) * 3 + c] = (uint8_t)__float2int_rn(__fmul_rn(fixed, 255.0f));
  } else {
    a.blur_c[i] = bc;
    a.blur_r[i] = br;
    a.high[i] = hi;
  }
}

int blocks_for(long long items) { return (int)((items + 255) / 256); }

}  // namespace

extern "C" {

long long rc_cf_adain_workspace(int planes, long long hw) {
  return (long long)planes * ((hw + kChunk - 1) / kChunk) * 4 * (long long)sizeof(double);
}

int rc_cf_adain(const void* content, int content_dtype, const void* reference, int reference_dtype, int planes,
                long long hw, void* workspace, long long workspace_bytes, float* out, cudaStream_t stream) {
  if (!content || !reference || !out || !workspace || planes < 1 || hw < 1 || (content_dtype != 0 && content_dtype != 1) ||
      (reference_dtype != 0 && reference_dtype != 1) || planes > 65535)
    return rc::set_error(RC_ERR_ARG, "rc_cf_adain: bad arguments");
  const int chunks = (int)((hw + kChunk - 1) / kChunk);
  if (workspace_bytes < rc_cf_adain_workspace(planes, hw) || (reinterpret_cast<uintptr_t>(workspace) & 7))
    return rc::set_error(RC_ERR_ARG, "rc_cf_adain: workspace too small or misaligned");
  double* part = reinterpret_cast<double*>(workspace);
  int r = rc::check_launch(rc::launch_pdl(adain_partial_kernel, dim3(chunks, planes), dim3(256), 0, stream, content,
                                          content_dtype, reference, reference_dtype, hw, part, chunks),
                           "rc_cf_adain");
  if (r) return r;
  const int bx = (int)std::min<long long>((hw + 256LL * 8 - 1) / (256LL * 8), 1024);
  return rc::check_launch(rc::launch_pdl(adain_apply_kernel, dim3(bx, planes), dim3(256), 0, stream, content,
                                         content_dtype, hw, part, chunks, out),
                          "rc_cf_adain");
}

int rc_cf_bicubic_u8(const uint8_t* lq, int T, int h, int w, int H, int W, float* out, cudaStream_t stream) {
  if (!lq || !out || T < 1 || h < 1 || w < 1 || H < 1 || W < 1)
    return rc::set_error(RC_ERR_ARG, "rc_cf_bicubic_u8: bad arguments");
  return rc::check_launch(rc::launch_pdl(bicubic_u8_kernel, dim3(blocks_for((long long)T * 3 * H * W)), dim3(256), 0,
                                         stream, lq, T, h, w, H, W, out),
                          "rc_cf_bicubic_u8");
}

int rc_cf_wavelet_level(const void* decoded, int dtype, const float* low_c, const float* low_r, float* blur_c,
                        float* blur_r, float* high, uint8_t* out, int T, int H, int W, int radius, int first,
                        int last, cudaStream_t stream) {
  if (T < 1 || H < 1 || W < 1 || radius < 1 || !low_r || (first && !decoded) || (!first && !low_c) ||
      (dtype != 0 && dtype != 1) || (last && !out) || (!last && (!blur_c || !blur_r || !high)) ||
      (!first && !high))
    return rc::set_error(RC_ERR_ARG, "rc_cf_wavelet_level: bad arguments");
  LevelArgs a{decoded, dtype, low_c, low_r, blur_c, blur_r, high, out, T, H, W, radius, first ? 1 : 0, last ? 1 : 0};
  return rc::check_launch(rc::launch_pdl(wavelet_level_kernel, dim3(blocks_for((long long)T * 3 * H * W)), dim3(256),
                                         0, stream, a),
                          "rc_cf_wavelet_level");
}

}  // extern "C"
