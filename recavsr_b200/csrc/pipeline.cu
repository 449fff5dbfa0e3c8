// Frame preparation and strip blending around the DiT, on the device.
//
// rc_enlarge_block: one LQ block of uint8 RGB frames (as decoded, [h, w, 3])
// -> the model input [3, block, Hp, Wp] (fp32 or bf16): the bilinear enlarge
// of recavsr_infer/video.py:153-174 (cv2.resize INTER_LINEAR, 8-bit fixed
// point), the last valid frame repeated to fill the block, x / 127.5 - 1 and
// the pad of the width then the height to the 32-pixel token stride (reflect,
// or replicate when the pad is not smaller than the size, video.py:165-179),
// in one pass. The host uploads only the small LQ frames (1/16 of the
// enlarged bytes at x4) and the enlarged block never exists in uint8.
// The reference's block_tensor normalizes with torch, whose CUDA kernel
// multiplies by the fp32 reciprocal of a scalar divisor (x * fl32(1/127.5))
// while its CPU kernel divides (x / 127.5): the two differ by one fp32 ulp for
// 111 of the 256 byte values. Both are offered (flags bit RC_ENLARGE_RECIPROCAL);
// the reference's inference runs block_tensor on CUDA.
//
// rc_strip_blend: one output frame of recavsr_infer/strips.py:72-99 -- the
// strips' uint8 frames weighted by their feather ramps, summed in strip order
// in fp32, divided by the per-column total, + 0.5, clipped and truncated.
//
// The 8-bit bilinear arithmetic (the weights of one output column or row):
//   f = fl32((i + 0.5) * (1 / (dst / src)) - 0.5)    (the scale in double)
//   s = floor(f), f -= s; columns only: s < 0 -> (s, f) = (0, 0),
//   s >= src - 1 -> (s, f) = (src - 1, 0); rows keep f and clip s, s + 1;
//   w0 = rint((1 - f) * 2048), w1 = rint(f * 2048)  (ties to even)
//   S = src[s] * w0 + src[s + 1] * w1 along x, then along y
//   v = ((S0 >> 4) * b0 >> 16) + ((S1 >> 4) * b1 >> 16), out = sat_u8((v + 2) >> 2).
// Everything is integer or IEEE fp32 / fp64 with explicit rounding, so the
// result is the same bytes on every run.
#include "common.cuh"

namespace {

struct Tap {
  int i0, i1, w0, w1;
};

// Weights of output coordinate `o` along an axis of `src` inputs scaled to `dst`.
__device__ __forceinline__ Tap axis_tap(int o, int src, int dst, bool clamp_fraction) {
  const double scale = 1.0 / ((double)dst / (double)src);
  float f = __double2float_rn(__dsub_rn(__dmul_rn((double)o + 0.5, scale), 0.5));
  const float fl = floorf(f);
  int s = (int)fl;
  f = __fsub_rn(f, fl);
  if (clamp_fraction) {
    if (s < 0) { s = 0; f = 0.f; }
    if (s >= src - 1) { s = src - 1; f = 0.f; }
  }
  Tap t;
  t.w0 = __float2int_rn(__fmul_rn(__fsub_rn(1.0f, f), 2048.0f));
  t.w1 = __float2int_rn(__fmul_rn(f, 2048.0f));
  t.i0 = min(max(s, 0), src - 1);
  t.i1 = min(max(s + 1, 0), src - 1);
  return t;
}

// Source index of padded position p of an axis of n values padded at the end
// by `pad` (reflect without repeating the edge when pad < n, else replicate).
__device__ __forceinline__ int pad_source(int p, int n, int pad) {
  if (p < n) return p;
  return pad < n ? 2 * (n - 1) - p : n - 1;
}

struct EnlargeArgs {
  const uint8_t* src;
  long long frame_stride, row_stride;   // bytes
  int valid, block, h, w, out_h, out_w, hp, wp;
  int bf16, reciprocal;
  void* out;                            // [3, block, hp, wp]
};

constexpr int kEnlargeCols = 8;         // output columns per thread

__global__ void __launch_bounds__(256) enlarge_block_kernel(EnlargeArgs a) {
  rc::pdl_trigger();
  rc::pdl_wait();
  const int x0 = (blockIdx.x * blockDim.x + threadIdx.x) * kEnlargeCols;
  const int y = blockIdx.y, t = blockIdx.z;
  if (x0 >= a.wp) return;
  const int pw = a.wp - a.out_w, ph = a.hp - a.out_h;
  const Tap ty = axis_tap(pad_source(y, a.out_h, ph), a.h, a.out_h, false);
  const uint8_t* frame = a.src + (long long)min(t, a.valid - 1) * a.frame_stride;
  const uint8_t* r0 = frame + (long long)ty.i0 * a.row_stride;
  const uint8_t* r1 = frame + (long long)ty.i1 * a.row_stride;
  float v[3][kEnlargeCols];
#pragma unroll
  for (int j = 0; j < kEnlargeCols; ++j) {
    const Tap tx = axis_tap(pad_source(x0 + j, a.out_w, pw), a.w, a.out_w, true);
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      const int s0 = (int)rc::ld_in(r0 + 3 * tx.i0 + c) * tx.w0 + (int)rc::ld_in(r0 + 3 * tx.i1 + c) * tx.w1;
      const int s1 = (int)rc::ld_in(r1 + 3 * tx.i0 + c) * tx.w0 + (int)rc::ld_in(r1 + 3 * tx.i1 + c) * tx.w1;
      const int q = (((s0 >> 4) * ty.w0) >> 16) + (((s1 >> 4) * ty.w1) >> 16);
      const int u = min(max((q + 2) >> 2, 0), 255);
      const float x = a.reciprocal ? __fmul_rn((float)u, 1.0f / 127.5f) : __fdiv_rn((float)u, 127.5f);
      v[c][j] = __fsub_rn(x, 1.0f);
    }
  }
  // wp is a multiple of 32, so every thread's 8 columns lie inside the row.
  const long long plane = (long long)a.block * a.hp * a.wp;
  const long long base = ((long long)t * a.hp + y) * a.wp + x0;
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    if (a.bf16) {
      uint32_t w[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) w[j] = rc::pack_bf16x2(v[c][2 * j], v[c][2 * j + 1]);
      *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.out) + c * plane + base) =
          make_uint4(w[0], w[1], w[2], w[3]);
    } else {
      float4* o = reinterpret_cast<float4*>(reinterpret_cast<float*>(a.out) + c * plane + base);
      o[0] = make_float4(v[c][0], v[c][1], v[c][2], v[c][3]);
      o[1] = make_float4(v[c][4], v[c][5], v[c][6], v[c][7]);
    }
  }
}

constexpr int kMaxStrips = 16;

struct BlendArgs {
  const uint8_t* frame[kMaxStrips];     // [height, width_s, 3] per strip, row stride row_stride[s]
  const float* weight[kMaxStrips];      // [width_s]
  long long row_stride[kMaxStrips];
  int offset[kMaxStrips], width_s[kMaxStrips];
  int n, height, width;
  const float* total;                   // [width]
  uint8_t* out;                         // [height, width, 3]
  long long out_row_stride;
};

__global__ void __launch_bounds__(256) strip_blend_kernel(BlendArgs a) {
  rc::pdl_trigger();
  rc::pdl_wait();
  const int x = blockIdx.x * blockDim.x + threadIdx.x, y = blockIdx.y;
  if (x >= a.width) return;
  float c0 = 0.f, c1 = 0.f, c2 = 0.f;
  for (int s = 0; s < a.n; ++s) {
    const int xs = x - a.offset[s];
    if (xs < 0 || xs >= a.width_s[s]) continue;
    const float w = rc::ld_in(a.weight[s] + xs);
    const uint8_t* p = a.frame[s] + (long long)y * a.row_stride[s] + 3 * xs;
    c0 = __fadd_rn(c0, __fmul_rn((float)rc::ld_in(p), w));
    c1 = __fadd_rn(c1, __fmul_rn((float)rc::ld_in(p + 1), w));
    c2 = __fadd_rn(c2, __fmul_rn((float)rc::ld_in(p + 2), w));
  }
  const float tot = rc::ld_in(a.total + x);
  auto to_u8 = [&](float c) -> uint8_t {
    const float v = __fadd_rn(__fdiv_rn(c, tot), 0.5f);
    return (uint8_t)(int)fminf(fmaxf(v, 0.f), 255.f);   // clip, then truncate toward zero
  };
  uint8_t* o = a.out + (long long)y * a.out_row_stride + 3 * x;
  o[0] = to_u8(c0);
  o[1] = to_u8(c1);
  o[2] = to_u8(c2);
}

}  // namespace

extern "C" {

int rc_enlarge_block(const uint8_t* src, long long frame_stride, long long row_stride, int valid,
                     int block, int h, int w, int out_h, int out_w, int flags, void* out,
                     cudaStream_t stream) {
  if (!src || !out)
    return rc::set_error(RC_ERR_ARG, "rc_enlarge_block: missing pointer");
  if (valid < 1 || block < valid || h < 1 || w < 1 || out_h < 1 || out_w < 1 ||
      row_stride < 3LL * w || frame_stride < row_stride * h)
    return rc::set_error(RC_ERR_ARG, "rc_enlarge_block: bad geometry (valid=%d block=%d %dx%d -> %dx%d)",
                         valid, block, h, w, out_h, out_w);
  const int hp = (out_h + 31) / 32 * 32, wp = (out_w + 31) / 32 * 32;
  if ((reinterpret_cast<uintptr_t>(out) & 15) != 0)
    return rc::set_error(RC_ERR_ARG, "rc_enlarge_block: output must be 16-byte aligned");
  if (hp > 65535 || block > 65535)
    return rc::set_error(RC_ERR_ARG, "rc_enlarge_block: raster too tall (%d rows)", hp);
  if (flags & ~3) return rc::set_error(RC_ERR_ARG, "rc_enlarge_block: unknown flags 0x%x", flags);
  EnlargeArgs a{src, frame_stride, row_stride, valid, block, h, w, out_h, out_w, hp, wp,
                (flags & 1) ? 1 : 0, (flags & 2) ? 1 : 0, out};
  const int per_row = wp / kEnlargeCols;
  const dim3 grid((per_row + 255) / 256, hp, block);
  return rc::check_launch(rc::launch_pdl(enlarge_block_kernel, grid, dim3(256), 0, stream, a),
                          "rc_enlarge_block");
}

int rc_strip_blend(int n_strips, const uint8_t* const* frames, const long long* row_strides,
                   const int* offsets, const int* widths, const float* const* weights,
                   const float* total, int height, int width, uint8_t* out, long long out_row_stride,
                   cudaStream_t stream) {
  if (n_strips < 1 || n_strips > kMaxStrips || height < 1 || width < 1 || out_row_stride < 3LL * width)
    return rc::set_error(RC_ERR_ARG, "rc_strip_blend: bad shape (strips=%d %dx%d)", n_strips, height, width);
  if (!frames || !offsets || !widths || !weights || !total || !out || !row_strides)
    return rc::set_error(RC_ERR_ARG, "rc_strip_blend: missing pointer");
  BlendArgs a{};
  for (int s = 0; s < n_strips; ++s) {
    if (!frames[s] || !weights[s] || widths[s] < 1 || offsets[s] < 0 || offsets[s] + widths[s] > width ||
        row_strides[s] < 3LL * widths[s])
      return rc::set_error(RC_ERR_ARG, "rc_strip_blend: strip %d does not fit the frame", s);
    a.frame[s] = frames[s];
    a.weight[s] = weights[s];
    a.row_stride[s] = row_strides[s];
    a.offset[s] = offsets[s];
    a.width_s[s] = widths[s];
  }
  a.n = n_strips;
  a.height = height;
  a.width = width;
  a.total = total;
  a.out = out;
  a.out_row_stride = out_row_stride;
  const dim3 grid((width + 255) / 256, height);
  return rc::check_launch(rc::launch_pdl(strip_blend_kernel, grid, dim3(256), 0, stream, a),
                          "rc_strip_blend");
}

}  // extern "C"
