// Session glue around the DiT layer loop (recavsr_infer/runtime/transformer.py:279-349):
// the LQ projector's causal strided Conv3d layers as im2col + the tcgen05 bf16
// GEMM (models/lq_proj.py:75-139, 231-246), its channel RMSNorm + SiLU
// (lq_proj.py:26-40, 196-204), the patch embedding's patch gather (a Conv3d with
// kernel = stride = (1, 2, 2), transformer_wan.py:1020-1022), and the output
// head's unpatchify fused with `noise - prediction` and the bf16 recycle copy
// (transformer.py:330-349). The linears themselves (patch embedding, out_proj,
// sr_proj, proj_out) run on rc_bf16_gemm.
#include "common.cuh"

namespace {

__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    f[2 * j] = __uint_as_float(w[j] << 16);
    f[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
  }
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int j = 0; j < 4; ++j)
    w[j] = (uint32_t)rc::bf16_bits(f[2 * j]) | ((uint32_t)rc::bf16_bits(f[2 * j + 1]) << 16);
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// im2col of a Conv3d with kernel (4, 3, 3), padding (0, 1, 1) and stride
// (stride_t, stride_s, stride_s) -- lq_proj.py:51-61 -- over a source whose
// temporal padding / history the host has already laid out. Row m = output
// position (o, yo, xo); column k = tap * cin + c with tap = (dt * 3 + dy) * 3 + dx,
// the order of the weight permuted to [cout, kt, kh, kw, cin]. Source element
// (frame t, row y, column x, channel c):
//   r == 0 (channels-last): src + t*st + y*sy + x*sx + c;
//   r  > 0 (pixel unshuffle by r of planar RGB, lq_proj.py:279-285, channel
//          c = (rgb * r + i) * r + j): src + t*st + rgb*sc + (y*r + i)*sy + x*r + j.
// One CTA per output row; each thread moves 8 channels (16 bytes) per step.
struct Im2colArgs {
  const __nv_bfloat16* src;
  long long st, sc, sy, sx;
  int r, cin, hin, win, stride_t, stride_s, ho, wo;
  __nv_bfloat16* out;
  long long ldo;
};

__global__ void __launch_bounds__(256) im2col_kernel(Im2colArgs a) {
  rc::pdl_trigger();
  rc::pdl_wait();
  const int m = blockIdx.x;
  const int xo = m % a.wo, t1 = m / a.wo;
  const int yo = t1 % a.ho, o = t1 / a.ho;
  uint4* dst = reinterpret_cast<uint4*>(a.out + (long long)m * a.ldo);
  const int cv = a.cin >> 3;
  const int chunks = 36 * cv;
  const int rr = a.r * a.r;
  for (int q = threadIdx.x; q < chunks; q += blockDim.x) {
    const int tap = q / cv, c0 = (q - tap * cv) << 3;
    const int dt = tap / 9, rem = tap - dt * 9;
    const int dy = rem / 3, dx = rem - dy * 3;
    const int y = yo * a.stride_s + dy - 1, x = xo * a.stride_s + dx - 1;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (y >= 0 && y < a.hin && x >= 0 && x < a.win) {
      const __nv_bfloat16* f = a.src + (long long)(o * a.stride_t + dt) * a.st;
      const __nv_bfloat16* p;
      if (a.r) {
        const int c = c0 / rr, rem2 = c0 - c * rr;
        const int i = rem2 / a.r, j = rem2 - i * a.r;
        p = f + c * a.sc + (long long)(y * a.r + i) * a.sy + x * a.r + j;
      } else {
        p = f + (long long)y * a.sy + (long long)x * a.sx + c0;
      }
      v = rc::ld_in(reinterpret_cast<const uint4*>(p));
    }
    dst[q] = v;
  }
}

// Channel RMSNorm + SiLU of lq_proj.py:26-40 followed by nn.SiLU on the bf16
// result: y = bf16(x * rsqrt(mean(x^2) + eps) * w), out = bf16(y * sigmoid(y)),
// one 256-thread CTA per row of C <= 8192 channels (C % 8 == 0), in place
// allowed (the row is in registers before the first store).
__global__ void __launch_bounds__(256) rmsnorm_silu_kernel(const __nv_bfloat16* x, long long ldx,
                                                           const __nv_bfloat16* w, float eps,
                                                           __nv_bfloat16* out, long long ldo, int C) {
  rc::pdl_trigger();
  rc::pdl_wait();
  __shared__ float red[8];
  const int nv = C >> 3;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (long long)blockIdx.x * ldx);
  uint4 xv[4];
  float ss = 0.0f;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int q = threadIdx.x + k * 256;
    if (q < nv) {
      xv[k] = rc::ld_in(xr + q);
      float f[8];
      unpack8(xv[k], f);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(f[j], f[j], ss);
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float rinv = rsqrtf(tot / (float)C + eps);
  uint4* orow = reinterpret_cast<uint4*>(out + (long long)blockIdx.x * ldo);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int q = threadIdx.x + k * 256;
    if (q < nv) {
      float f[8], g[8];
      unpack8(xv[k], f);
      unpack8(rc::ld_in(wr + q), g);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float y = rc::bf16_to_float(rc::bf16_bits((f[j] * rinv) * g[j]));
        f[j] = y / (1.0f + expf(-y));
      }
      orow[q] = pack8(f);
    }
  }
}

// Patch gather of a Conv3d with kernel = stride = (1, ph, pw): token
// n = (f, yy, xx), column k = (c * ph + i) * pw + j (the weight's [cout, c, 1, ph, pw]
// order), value bf16(src[c, f, yy*ph + i, xx*pw + j]) from fp32 or bf16 input.
template <typename T>
__device__ __forceinline__ float load_val(const T* p);
template <>
__device__ __forceinline__ float load_val<float>(const float* p) { return rc::ld_in(p); }
template <>
__device__ __forceinline__ float load_val<__nv_bfloat16>(const __nv_bfloat16* p) {
  return rc::bf16_to_float(rc::ld_in(reinterpret_cast<const uint16_t*>(p)));
}

template <typename T>
__global__ void __launch_bounds__(256) patchify_kernel(const T* src, long long sc, long long sf, long long sy,
                                                       int C, int hh, int ww, int ph, int pw,
                                                       __nv_bfloat16* out, long long ldo) {
  rc::pdl_trigger();
  rc::pdl_wait();
  const int n = blockIdx.x;
  const int xx = n % ww, t1 = n / ww;
  const int yy = t1 % hh, f = t1 / hh;
  const int K = C * ph * pw;
  uint16_t* orow = reinterpret_cast<uint16_t*>(out + (long long)n * ldo);
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    const int c = k / (ph * pw), r = k - c * ph * pw;
    const int i = r / pw, j = r - i * pw;
    const float v = load_val(src + c * sc + f * sf + (long long)(yy * ph + i) * sy + xx * pw + j);
    orow[k] = rc::bf16_bits(v);
  }
}

// out[c, f, y, x] = noise[c, f, y, x] - float(pred[n, ((y % ph) * pw + x % pw) * C + c])
// with n = (f * hh + y / ph) * ww + x / pw (transformer.py:330-345), and for
// the last `rf` frames recycle[c, f - (F - rf), y, x] = bf16(out) (:346-348).
// noise / out / recycle contiguous [C, F, H, W] ([C, rf, H, W]); one thread per element.
__global__ void __launch_bounds__(256) unpatchify_residual_kernel(const __nv_bfloat16* pred, long long ldp,
                                                                  const float* noise, float* out,
                                                                  __nv_bfloat16* recycle, int C, int F, int H,
                                                                  int W, int ph, int pw, int rf) {
  rc::pdl_trigger();
  rc::pdl_wait();
  const long long total = (long long)C * F * H * W;
  const int hh = H / ph, ww = W / pw;
  const uint16_t* pr = reinterpret_cast<const uint16_t*>(pred);
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const int x = (int)(e % W);
    const long long t1 = e / W;
    const int y = (int)(t1 % H);
    const long long t2 = t1 / H;
    const int f = (int)(t2 % F), c = (int)(t2 / F);
    const long long n = ((long long)f * hh + y / ph) * ww + x / pw;
    const int col = ((y % ph) * pw + x % pw) * C + c;
    const float p = rc::bf16_to_float(rc::ld_in(pr + n * ldp + col));
    const float v = rc::ld_in(noise + e) - p;
    out[e] = v;
    if (recycle && f >= F - rf)
      reinterpret_cast<uint16_t*>(recycle)[(((long long)c * rf + (f - (F - rf))) * H + y) * W + x] = rc::bf16_bits(v);
  }
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

extern "C" {

int rc_conv3d_im2col(const void* src, long long frame_stride, long long chan_stride, long long row_stride,
                     long long col_stride, int unshuffle, int cin, int frames_in, int h_in, int w_in,
                     int stride_t, int stride_s, int frames_out, void* out, long long ldo,
                     cudaStream_t stream) {
  const char* what = "rc_conv3d_im2col";
  if (cin <= 0 || cin % 8 || frames_in <= 0 || h_in <= 0 || w_in <= 0 || stride_t <= 0 || stride_s <= 0 ||
      frames_out < 0 || unshuffle < 0 || (unshuffle && unshuffle % 8) ||
      (unshuffle && cin % (unshuffle * unshuffle)))
    return rc::set_error(RC_ERR_ARG, "%s: bad geometry", what);
  if (frames_out && (long long)(frames_out - 1) * stride_t + 4 > frames_in)
    return rc::set_error(RC_ERR_ARG, "%s: %d output frames need %d input frames, got %d", what, frames_out,
                         (frames_out - 1) * stride_t + 4, frames_in);
  const int ho = (h_in - 1) / stride_s + 1, wo = (w_in - 1) / stride_s + 1;
  const long long rows = (long long)frames_out * ho * wo;
  if (rows == 0) return RC_OK;
  if (rows > 0x7fffffffLL) return rc::set_error(RC_ERR_ARG, "%s: too many output rows", what);
  if (!src || !out || !al16(src) || !al16(out) || ldo % 8 || ldo < 36LL * cin || frame_stride % 8 ||
      row_stride % 8 || (unshuffle ? chan_stride % 8 : col_stride % 8))
    return rc::set_error(RC_ERR_ARG, "%s: tensors and strides must be 16-byte aligned", what);
  Im2colArgs a{reinterpret_cast<const __nv_bfloat16*>(src), frame_stride, chan_stride, row_stride, col_stride,
               unshuffle, cin, h_in, w_in, stride_t, stride_s, ho, wo,
               reinterpret_cast<__nv_bfloat16*>(out), ldo};
  return rc::check_launch(rc::launch_pdl(im2col_kernel, dim3((unsigned)rows), dim3(256), 0, stream, a), what);
}

int rc_channel_rmsnorm_silu(const void* x, long long ldx, int M, int C, const void* weight, float eps, void* out,
                            long long ldo, cudaStream_t stream) {
  const char* what = "rc_channel_rmsnorm_silu";
  if (M < 0 || C <= 0 || C % 8 || C > 8192 || ldx < C || ldo < C)
    return rc::set_error(RC_ERR_ARG, "%s: bad shape (M=%d C=%d)", what, M, C);
  if (M == 0) return RC_OK;
  if (!x || !weight || !out || !al16(x) || !al16(weight) || !al16(out) || ldx % 8 || ldo % 8)
    return rc::set_error(RC_ERR_ARG, "%s: rows must be 16-byte aligned", what);
  return rc::check_launch(
      rc::launch_pdl(rmsnorm_silu_kernel, dim3(M), dim3(256), 0, stream,
                     reinterpret_cast<const __nv_bfloat16*>(x), ldx, reinterpret_cast<const __nv_bfloat16*>(weight),
                     eps, reinterpret_cast<__nv_bfloat16*>(out), ldo, C),
      what);
}

int rc_patchify(const void* src, int src_is_bf16, long long chan_stride, long long frame_stride,
                long long row_stride, int C, int F, int H, int W, int ph, int pw, void* out, long long ldo,
                cudaStream_t stream) {
  const char* what = "rc_patchify";
  if (C <= 0 || F < 0 || H <= 0 || W <= 0 || ph <= 0 || pw <= 0 || H % ph || W % pw ||
      ldo < (long long)C * ph * pw)
    return rc::set_error(RC_ERR_ARG, "%s: bad shape", what);
  const long long tokens = (long long)F * (H / ph) * (W / pw);
  if (tokens == 0) return RC_OK;
  if (tokens > 0x7fffffffLL) return rc::set_error(RC_ERR_ARG, "%s: too many tokens", what);
  if (!src || !out) return rc::set_error(RC_ERR_ARG, "%s: null pointer", what);
  cudaError_t e;
  if (src_is_bf16)
    e = rc::launch_pdl(patchify_kernel<__nv_bfloat16>, dim3((unsigned)tokens), dim3(256), 0, stream,
                       reinterpret_cast<const __nv_bfloat16*>(src), chan_stride, frame_stride, row_stride, C,
                       H / ph, W / pw, ph, pw, reinterpret_cast<__nv_bfloat16*>(out), ldo);
  else
    e = rc::launch_pdl(patchify_kernel<float>, dim3((unsigned)tokens), dim3(256), 0, stream,
                       reinterpret_cast<const float*>(src), chan_stride, frame_stride, row_stride, C, H / ph,
                       W / pw, ph, pw, reinterpret_cast<__nv_bfloat16*>(out), ldo);
  return rc::check_launch(e, what);
}

int rc_unpatchify_residual(const void* pred, long long ldp, const float* noise, float* out, void* recycle,
                           int C, int F, int H, int W, int ph, int pw, int recycle_frames, cudaStream_t stream) {
  const char* what = "rc_unpatchify_residual";
  if (C <= 0 || F < 0 || H <= 0 || W <= 0 || ph <= 0 || pw <= 0 || H % ph || W % pw ||
      ldp < (long long)C * ph * pw || recycle_frames < 0 || recycle_frames > F)
    return rc::set_error(RC_ERR_ARG, "%s: bad shape", what);
  const long long total = (long long)C * F * H * W;
  if (total == 0) return RC_OK;
  if (!pred || !noise || !out || (recycle_frames && !recycle))
    return rc::set_error(RC_ERR_ARG, "%s: null pointer", what);
  long long blocks = (total + 255) / 256;
  if (blocks > 148LL * 16) blocks = 148LL * 16;
  return rc::check_launch(
      rc::launch_pdl(unpatchify_residual_kernel, dim3((unsigned)blocks), dim3(256), 0, stream,
                     reinterpret_cast<const __nv_bfloat16*>(pred), ldp, noise, out,
                     recycle_frames ? reinterpret_cast<__nv_bfloat16*>(recycle) : nullptr, C, F, H, W, ph, pw,
                     recycle_frames),
      what);
}

}  // extern "C"
