/*
 * recavsr_b200 -- C ABI of the B200 (sm_100a) kernels behind ReCaVSR's DiT hot path.
 *
 * Every entry point is asynchronous on `stream` (a cudaStream_t passed as a
 * plain pointer), takes raw device pointers, sizes and strides (in elements
 * unless the name says bytes), and returns a status:
 *   0 RC_OK, 1 RC_ERR_ARG (invalid argument; Python raises ValueError),
 *   2 RC_ERR_CUDA, 3 RC_ERR_TIMEOUT (a bounded device wait gave up),
 *   4 RC_ERR_UNSUPPORTED (valid but unimplemented geometry).
 * The text of the last failure on the calling thread is returned by
 * rc_get_last_error(). Device-side faults that kernels detect themselves are
 * latched in an error word read (and cleared) by rc_read_device_error().
 * bf16 tensors are passed as `const void*` (IEEE bfloat16, row-major).
 * None of these calls allocates device memory.
 */
#ifndef RECAVSR_B200_H_
#define RECAVSR_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* rc_stream_t;

/* ---- library ---------------------------------------------------------- */
int rc_abi_version(void);
int rc_get_last_error(char* buf, size_t size);
int rc_read_device_error(unsigned int* word);

/* ---- NVFP4 / FP8 quantizers ------------------------------------------ */
/* Replaces recavsr_infer/runtime/nvfp4.py:49-68 `quantize(matrix)`.
 * x: bf16 [M, K] with row stride ldx (K % 16 == 0). codes: u8 [M, K/2]
 * (even element in the low nibble). scales_swizzled: u8
 * [ceil(M/128)*128 * ceil(K/64)*4] in the 128x4 blocked order, padding zeroed.
 * global_scale = 1 reproduces the reference bit for bit. */
int rc_nvfp4_quantize(const void* x, int M, int K, long long ldx, float global_scale,
                      uint8_t* codes, uint8_t* scales_swizzled, rc_stream_t stream);

/* Replaces the activation quantization of recavsr_infer/runtime/fp8.py:41-42
 * (and the weight quantization of :32-34): scale = max(amax,1e-12)/448 written
 * to *scale_out (device), q = e4m3(clamp(x/scale)). amax_scratch: one device
 * u32, overwritten. */
int rc_fp8_quantize(const void* x, int M, int K, long long ldx, unsigned int* amax_scratch,
                    float* scale_out, uint8_t* q, rc_stream_t stream);

/* ---- GEMMs (tcgen05) --------------------------------------------------- */
/* Epilogues: 0 out = bf16(alpha*acc + bias); 1 out = bf16(out + bf16(alpha*acc+bias)*gate[n]);
 * 2 out = bf16(out + bf16(alpha*acc+bias)); 3 (NVFP4 only) y = bf16(gelu_tanh(bf16(alpha*acc+bias)))
 * quantized to NVFP4 into q_codes / q_scales (out optional). K % 64 == 0, N % 16 == 0. */
#define RC_EPI_BIAS 0
#define RC_EPI_GATED_RESIDUAL 1
#define RC_EPI_RESIDUAL 2
#define RC_EPI_GELU_NVFP4 3
/* bf16 only: the columns come as 16-column chunks of 8 gate then 8 up
 * columns; out [M, N/2] = bf16(bf16(silu(y_gate)) * y_up) (the SwiGLU of
 * recavsr_infer/models/flashdecoder/flashdecoder_wan22.py:344-345). */
#define RC_EPI_SWIGLU 4

/* Replaces recavsr_infer/runtime/nvfp4.py:22-39 `nvfp4_mm` (torch._scaled_mm_v2,
 * BlockWise1x16 / SWIZZLE_32_4_4, bias, bf16 out). */
int rc_nvfp4_gemm(const uint8_t* a_codes, const uint8_t* a_scales, const uint8_t* b_codes,
                  const uint8_t* b_scales, const void* bias, int M, int N, int K, float alpha,
                  int epilogue, void* out, long long ldo, const float* gate, uint8_t* q_codes,
                  uint8_t* q_scales, float q_global_scale, rc_stream_t stream);

/* rc_nvfp4_gemm with a split-K workspace: the tiles of the last, partial wave
 * of the persistent grid run as up to 4 k-ranges each (fp32 partials in the
 * workspace, summed in a fixed order by the last range to finish). workspace:
 * rc_gemm_split_workspace() bytes, 16-byte aligned, zero-filled before first
 * use (each successful call leaves it zero-filled); calls sharing one
 * workspace must be ordered on one stream. */
long long rc_gemm_split_workspace(void);
int rc_nvfp4_gemm_ws(const uint8_t* a_codes, const uint8_t* a_scales, const uint8_t* b_codes,
                     const uint8_t* b_scales, const void* bias, int M, int N, int K, float alpha,
                     int epilogue, void* out, long long ldo, const float* gate, uint8_t* q_codes,
                     uint8_t* q_scales, float q_global_scale, void* workspace,
                     long long workspace_bytes, rc_stream_t stream);

/* Replaces the torch._scaled_mm call of recavsr_infer/runtime/fp8.py:44-47
 * (per-tensor scales are device pointers, use_fast_accum=False semantics). */
int rc_fp8_gemm(const uint8_t* a, const float* scale_a, const uint8_t* b, const float* scale_b,
                const void* bias, int M, int N, int K, float alpha, int epilogue, void* out,
                long long ldo, const float* gate, rc_stream_t stream);

/* bf16 nn.Linear (the default, unquantized DiT linears of
 * recavsr_infer/runtime/transformer.py:95-133). */
int rc_bf16_gemm(const void* a, const void* b, const void* bias, int M, int N, int K, int epilogue,
                 void* out, long long ldo, const float* gate, rc_stream_t stream);
/* rc_bf16_gemm with a split-K workspace (the rules of rc_nvfp4_gemm_ws): the
 * LQ projector's long-K convolution GEMMs (recavsr_infer/models/lq_proj.py:80-139
 * as TransformerSession runs them, transformer.py:279-300). */
int rc_bf16_gemm_ws(const void* a, const void* b, const void* bias, int M, int N, int K, int epilogue,
                    void* out, long long ldo, const float* gate, void* workspace, long long workspace_bytes,
                    rc_stream_t stream);

/* ---- glue --------------------------------------------------------------- */
/* LayerNorm (+affine) (+AdaLN modulation) (+fused NVFP4 quantize) of
 * recavsr_infer/runtime/transformer.py:91-93,121,130-132 and
 * kernels/native_norm.py:7-17. */
int rc_ln_modulate_quant(const void* x, long long ldx, int M, int N, const void* weight,
                         const void* bias, const float* shift, const float* scale, float eps,
                         void* out, long long ldo, uint8_t* codes, uint8_t* scales_swizzled,
                         float global_scale, rc_stream_t stream);

/* Replaces recavsr_infer/kernels/native_norm.py:7-17 (`native_layer_norm`,
 * rms = 0) and :25-28 (`native_rms_norm`, rms = 1) for any floating input:
 * the norm of each row of x [M, N] (row stride ldx) in fp32 with the fp32
 * affine weight / bias (nullable; bias unused when rms = 1), written in x's
 * type into out (row stride ldo). dtype: 0 fp32, 1 bf16, 2 fp16. The
 * reference's only caller passes fp32 rows (runtime/transformer.py:91,121,130). */
int rc_layer_norm(const void* x, int dtype, long long ldx, int M, int N, const float* weight,
                  const float* bias, float eps, int rms, void* out, long long ldo,
                  rc_stream_t stream);

/* RMSNorm across heads (+ spatial rotary) of up to two tensors:
 * recavsr_infer/runtime/transformer.py:99-100,122 (norm_q/norm_k, PreparedBlock.spatial),
 * kernels/native_norm.py:25-28, runtime/rope.py:23-30. */
int rc_rmsnorm_rope(int n_tensors, const void* const* xs, const long long* ldx,
                    const void* const* weights, void* const* outs, const long long* ldo, int M,
                    int N, int d, int span, const float* cos, const float* sin, float eps,
                    rc_stream_t stream);

/* Temporal rotary embedding of recavsr_infer/runtime/rope.py:33-47 (apply_temporal). */
int rc_temporal_rope(const void* x, long long ldx, void* out, long long ldo, const int* positions,
                     const float* cos, const float* sin, int rows, int span, int heads, int d,
                     int td, rc_stream_t stream);

/* ---- KV cache ------------------------------------------------------------ */
/* Plane copies of recavsr_infer/runtime/cache.py:121-134 (FixedKVCache.commit):
 * plane src_planes[i] of the block's K/V -> slot dst_slots[i] of the cache. */
int rc_kv_commit(const void* src_k, const void* src_v, long long src_ld_bytes, void* dst_k,
                 void* dst_v, long long dst_ld_bytes, int row_bytes, int span, int n_planes,
                 const int* src_planes, const int* dst_slots, rc_stream_t stream);

/* Same copies with the plan in device memory: plan = [n, (src plane, dst slot) x n],
 * n <= max_planes <= 8, slots < capacity. Lets a captured CUDA graph of the
 * layer loop follow the router without re-capture. K and V have their own
 * source row strides (the block's V is a column range of the fused QKV output,
 * cache.py:85-133 takes key and value as separate tensors). */
int rc_kv_commit_planned(const void* src_k, const void* src_v, long long src_ld_k_bytes,
                         long long src_ld_v_bytes, void* dst_k, void* dst_v, long long dst_ld_bytes,
                         int row_bytes, int span, int max_planes, int capacity, const int* plan,
                         rc_stream_t stream);

/* ---- routed attention (tcgen05) ------------------------------------------ */
/* Replaces recavsr_infer/kernels/local_attention.py:172-260 `paired_attention`
 * (custom op recavsr_local::paired, Triton `_paired_local`) and :286-325
 * `sdpa_attention` (window covering the grid). q/ck/cv [B, QT*H*W, heads, d],
 * pk/pv [B, CAP*H*W, heads, d] bf16 with strides[15] = (batch, token, head)
 * element strides of q, ck, cv, pk, pv; slots/past_positions int32 [CAP]
 * (slot -1 = empty), query_positions int32 [QT], cos/sin fp32 [frames, td/2]
 * (the rolling temporal table), all on the device. out: [B, QT*H*W, heads, d]
 * bf16 with token stride out_ld (nullable when out_codes is given).
 * out_codes/out_scales (optional, B = 1): the output also NVFP4-quantized as
 * rc_nvfp4_quantize would quantize it ([QT*H*W, heads*d/2] codes + swizzled
 * scales), ready for the o-proj GEMM. workspace: caller-provided device scratch
 * of rc_paired_attention_workspace(...) bytes (rotated K planes, then about
 * 10.6 MB of tail-split partials and counters). d = 128. */
long long rc_paired_attention_workspace(int B, int QT, int CAP, int H, int W, int heads, int d);
int rc_paired_attention(const void* q, const void* ck, const void* cv, const void* pk, const void* pv,
                        const long long* strides, const int* slots, const int* past_positions,
                        const int* query_positions, const float* cos, const float* sin, int B,
                        int QT, int CAP, int H, int W, int heads, int d, int td, int window_h,
                        int window_w, void* workspace, long long workspace_bytes, void* out,
                        long long out_ld, uint8_t* out_codes, uint8_t* out_scales,
                        rc_stream_t stream);

/* Allocation-free form of rc_paired_attention (no counterpart in the
 * reference, which always lets PyTorch allocate). For callers that must not
 * call cudaMalloc -- for example code that launches while another thread of the
 * process holds a CUDA-graph capture in global mode (device allocation is not
 * permitted then), or a host framework that hands this library no allocator
 * and a fixed memory budget. It takes the same arguments minus the workspace
 * and uses a scratch array built into the library instead: 64 MiB of device
 * memory per GPU that loads the library, held until the process exits.
 * Geometries needing more than 64 MiB of scratch (rc_paired_attention_workspace)
 * are rejected with RC_ERR_ARG. The first call on each device looks the array
 * up (cudaGetSymbolAddress with that device current), so make that first call
 * before any stream capture. All calls share the one array: calls whose work
 * overlaps on the GPU (concurrent streams) race on it; calls ordered on one
 * stream are safe. Nothing in the scratch needs to start at zero -- every
 * scratch byte the kernels read is written earlier in the same call. */
int rc_paired_attention_static_scratch(const void* q, const void* ck, const void* cv, const void* pk,
                                       const void* pv, const long long* strides, const int* slots,
                                       const int* past_positions, const int* query_positions,
                                       const float* cos, const float* sin, int B, int QT, int CAP,
                                       int H, int W, int heads, int d, int td, int window_h,
                                       int window_w, void* out, long long out_ld, uint8_t* out_codes,
                                       uint8_t* out_scales, rc_stream_t stream);

/* Unmasked attention without rotary embedding or cache (the cross-attention of
 * recavsr_infer/runtime/transformer.py:123-128 over the precomputed prompt K/V):
 * q [B, Nq, heads, d], k/v [B, Nk, heads, d] with strides[9] = (batch, token,
 * head) element strides of q, k, v; out [B, Nq, heads, d] (token stride out_ld),
 * optional NVFP4 copy of the output in out_codes/out_scales (B = 1). */
int rc_cross_attention(const void* q, const void* k, const void* v, const long long* strides, int B,
                       int Nq, int Nk, int heads, int d, void* out, long long out_ld,
                       uint8_t* out_codes, uint8_t* out_scales, rc_stream_t stream);

/* rc_cross_attention with a tail-split workspace of rc_cross_attention_workspace()
 * bytes (16-byte aligned, zero-filled before its first use; each successful call
 * leaves it zero-filled; calls sharing one must be ordered on one stream): the
 * query tiles of the last partial wave run as key-range pieces. */
long long rc_cross_attention_workspace(void);
int rc_cross_attention_ws(const void* q, const void* k, const void* v, const long long* strides, int B,
                          int Nq, int Nk, int heads, int d, void* out, long long out_ld,
                          uint8_t* out_codes, uint8_t* out_scales, void* workspace,
                          long long workspace_bytes, rc_stream_t stream);

/* ---- session glue around the layer loop ---------------------------------- */
/* im2col of the LQ projector's CausalConv3d (recavsr_infer/models/lq_proj.py:44-139:
 * kernel (4, 3, 3), padding (0, 1, 1), stride (stride_t, stride_s, stride_s)) over
 * frames_in source frames the caller has already laid out (history, replicated
 * first frame), for the tcgen05 bf16 GEMM against the weight permuted to
 * [cout, kt, kh, kw, cin]. out: [frames_out * Ho * Wo, 36 * cin] bf16 (row stride
 * ldo), Ho = (h_in - 1) / stride_s + 1. Source element (frame t, row y, column x,
 * channel c), bf16, 16-byte aligned strides:
 *   unshuffle == 0: channels-last, src + t*frame_stride + y*row_stride + x*col_stride + c;
 *   unshuffle == r: planar RGB pixel-unshuffled by r (lq_proj.py:279-285, c = (rgb*r + i)*r + j),
 *                   src + t*frame_stride + rgb*chan_stride + (y*r + i)*row_stride + x*r + j. */
int rc_conv3d_im2col(const void* src, long long frame_stride, long long chan_stride,
                     long long row_stride, long long col_stride, int unshuffle, int cin,
                     int frames_in, int h_in, int w_in, int stride_t, int stride_s, int frames_out,
                     void* out, long long ldo, rc_stream_t stream);

/* ChannelRMSNorm3d + SiLU of lq_proj.py:26-40,196-204 on channels-last rows:
 * out = bf16(silu(bf16(x * rsqrt(mean(x^2) + eps) * weight))), C <= 8192,
 * C % 8 == 0, in place allowed. */
int rc_channel_rmsnorm_silu(const void* x, long long ldx, int M, int C, const void* weight, float eps,
                            void* out, long long ldo, rc_stream_t stream);

/* Patch gather of the patch embedding Conv3d (kernel = stride = (1, ph, pw);
 * recavsr_infer/models/transformer_wan.py:1020-1022, used at runtime/transformer.py:321-328):
 * src [C, F, H, W] (fp32 or bf16, element strides chan / frame / row, unit column
 * stride) -> out [F*(H/ph)*(W/pw), C*ph*pw] bf16, column (c*ph + i)*pw + j. */
int rc_patchify(const void* src, int src_is_bf16, long long chan_stride, long long frame_stride,
                long long row_stride, int C, int F, int H, int W, int ph, int pw, void* out,
                long long ldo, rc_stream_t stream);

/* Output head tail of recavsr_infer/runtime/transformer.py:333-348: unpatchify the
 * proj_out rows pred [F*(H/ph)*(W/pw), ph*pw*C] bf16 and return
 * out = noise - float(prediction) (fp32 [C, F, H, W]); the last recycle_frames
 * frames of out also as bf16 into recycle [C, recycle_frames, H, W]. */
int rc_unpatchify_residual(const void* pred, long long ldp, const float* noise, float* out,
                           void* recycle, int C, int F, int H, int W, int ph, int pw,
                           int recycle_frames, rc_stream_t stream);

/* ---- FlashDecoder ----------------------------------------------------------- */
/* Replaces recavsr_infer/models/flashdecoder/_local_attention_triton.py:21-131
 * (the Triton forward called by flashdecoder_wan22.py:38-119 `_local_attention`):
 * streaming local grouped-query attention. q [B, HQ, QF*H*W, D], k / v
 * [B, HK, NF*H*W, D], fp16 (fp16 = 1) or bf16, head dim contiguous, element
 * strides[9] = (batch, head, token) of q, k, v (multiples of 8). Query head h
 * reads key / value head h / (HQ / HK); a query of frame qt sees the key frames
 * of temporal groups (qg - temporal_window, qg], qg = (qt + NF - QF) / group_size,
 * and within a frame the keys at dy in [-window_h/2, window_h/2), dx in
 * [-window_w/2, window_w/2), truncated at the grid border. out [B, HQ, QF*H*W, D]
 * contiguous, in q's type. D = 64 (RC_ERR_UNSUPPORTED otherwise). */
int rc_local_gqa_attention(const void* q, const void* k, const void* v, const long long* strides, int B,
                           int HQ, int HK, int QF, int NF, int H, int W, int D, int window_h, int window_w,
                           int group_size, int temporal_window, int fp16, void* out, rc_stream_t stream);

/* FlashDecoder decode step glue (recavsr_infer/models/flashdecoder/flashdecoder_wan22.py,
 * runtime/flashdecoder.py:140-175), bf16 in the reference's CUDA autocast arithmetic.
 * Frame rings: a layer's K (fp32) / V (bf16) cache of `slots` frames is
 * [heads][slots * n][64], element head stride ring_head; global frame g lives
 * in slot g % slots. */

/* runtime/flashdecoder.py:168: raw = bf16(bf16(bf16(latent) * std) + mean) of a
 * normalized latent frame (fp32, channel c at latent + c * channel_stride, n
 * tokens contiguous) as GEMM rows out [n, 64] bf16 (columns 48..63 zero). */
int rc_fd_latent_in(const float* latent, long long channel_stride, int n, const void* mean, const void* stdv,
                    void* out, rc_stream_t stream);

/* flashdecoder_wan22.py:704-707: F.pixel_unshuffle(lr_up, 16) of `frames` LR
 * frames (dtype 0 fp32 / 1 bf16; element strides[3] = channel, frame, row;
 * pixels contiguous) -> bf16 [frames * h * w, 768], columns (c, i, j). */
int rc_fd_lr_unshuffle(const void* lr, int dtype, const long long* strides, int frames, int h, int w, void* out,
                       rc_stream_t stream);

/* flashdecoder_wan22.py:708-719: LR features [F, n, 48] (row stride ldf) ->
 * grouped [n, 192] (4 frames x 48) and late [4n, 64] (columns 48..63 zero);
 * first != 0 repeats frame 0 four times (the first chunk). */
int rc_fd_lr_group(const void* feats, long long ldf, int n, int first, void* grouped, void* late,
                   rc_stream_t stream);

/* flashdecoder_wan22.py:310-322: key_norm / value_norm (RMSNorm over each
 * 64-dim head, fp32 weights) of the K / V columns of fused q|k|v rows (K at
 * column q_cols, V at q_cols + 64 hk) into ring rows token0 .. token0 + tokens. */
int rc_fd_kv_norm(const void* qkv, long long ldq, int tokens, int q_cols, int hk, const float* wk,
                  const float* wv, float eps, float* k_ring, void* v_ring, long long ring_head, long long token0,
                  rc_stream_t stream);

/* flashdecoder_wan22.py:198-242,324-331: 3D RoPE of the current queries
 * (temporal position prev + frame) into q_out [cur*n, hq*64], of the window's
 * nf key frames (temporal positions 0..nf-1, ring slots (slot0 + t) % slots)
 * into k_out [hk][nf*n][64] bf16, and the window's V frames into v_out.
 * tables: fp32 cos_t [max_t][8] | sin_t | cos_h [h][12] | sin_h | cos_w [w][12] | sin_w. */
int rc_fd_rope_gather(const void* qkv, long long ldq, int hq, int hk, int cur, int prev, int nf, int slot0,
                      int slots, int h, int w, const float* k_ring, const void* v_ring, long long ring_head,
                      const float* tables, int max_t, void* q_out, void* k_out, void* v_out, rc_stream_t stream);

/* flashdecoder_wan22.py:344-345 (mode 0: out [M, H] = bf16(bf16(silu(x[:, :H])) * x[:, H:])
 * from x [M, 2H]) and :680-684 (mode 1: x [M, H] = bf16(silu(x)) in place). */
int rc_fd_silu(void* x, int M, int H, int mode, void* out, rc_stream_t stream);

/* flashdecoder_wan22.py:845-866 + runtime/flashdecoder.py:175: frames f0 .. f0+frames-1
 * of the spatial projection y [4n, 768] (row stride ldy) pixel-shuffled by 16
 * into out [3, out_frames, 16h, 16w] bf16 (frames 0 .. frames-1), clamped to [-1, 1]. */
int rc_fd_pixel_shuffle(const void* y, long long ldy, int f0, int frames, int out_frames, int h, int w, void* out,
                        rc_stream_t stream);

/* ---- colour correction (recavsr_infer/color_fix.py) ------------------------ */
/* color_fix.py:18-29,58-81 (adain_color_fix): per plane (frame, RGB channel) of
 * `planes` planes of hw values (content / reference in [-1, 1], dtype 0 fp32,
 * 1 bf16, same plane order), mean and sample variance of (x + 1) * 0.5, out
 * fp32 = ((c - mean_c) * sqrt((var_r + 1e-5) / (var_c + 1e-5)) + mean_r) * 2 - 1.
 * workspace: rc_cf_adain_workspace(planes, hw) bytes, 8-byte aligned. */
long long rc_cf_adain_workspace(int planes, long long hw);
int rc_cf_adain(const void* content, int content_dtype, const void* reference, int reference_dtype, int planes,
                long long hw, void* workspace, long long workspace_bytes, float* out, rc_stream_t stream);

/* color_fix.py:102-110: clamp(bicubic(lq / 255), 0, 1) of uint8 frames
 * [T, h, w, 3] at H x W (torch's upsample_bicubic2d, align_corners = false)
 * into out [T * 3, H, W] fp32. */
int rc_cf_bicubic_u8(const uint8_t* lq, int T, int h, int w, int H, int W, float* out, rc_stream_t stream);

/* color_fix.py:32-55,111-117: one level (dilation `radius`) of the wavelet
 * correction over [T * 3, H, W] fp32 planes: blur_c / blur_r = the [1,2,1]^2 / 16
 * blur (replicate padding) of low_c / low_r, high += low_c - blur_c. first:
 * the content is clamp((decoded + 1) * 0.5, 0, 1) read from decoded
 * [3, T, H, W] (dtype 0 fp32, 1 bf16) and high starts at 0. last: writes
 * uint8 round(clamp(high + blur_r, 0, 1) * 255) into out [T, H, W, 3]
 * (blur_c, blur_r and high are not written). */
int rc_cf_wavelet_level(const void* decoded, int dtype, const float* low_c, const float* low_r, float* blur_c,
                        float* blur_r, float* high, uint8_t* out, int T, int H, int W, int radius, int first,
                        int last, rc_stream_t stream);

/* ---- frame preparation and strip blending -------------------------------- */
/* Replaces recavsr_infer/video.py:153-179 (`enlarge_block` + `block_tensor`,
 * called by `prepare_block` :138-150): src = `valid` uint8 RGB frames [h, w, 3]
 * (byte strides frame_stride / row_stride, contiguous pixels), bilinearly
 * enlarged to out_h x out_w exactly as cv2.resize INTER_LINEAR does for 8-bit
 * images, the last frame repeated up to `block` frames, normalized to
 * x / 127.5 - 1 and padded to Hp x Wp (out_h, out_w rounded up to multiples of
 * 32; reflect, or replicate when the pad is not smaller than the size). out:
 * [3, block, Hp, Wp] contiguous, 16-byte aligned; fp32, or bf16 with
 * RC_ENLARGE_BF16. The normalization divides by 127.5 as the reference's
 * block_tensor does on the CPU, or with RC_ENLARGE_RECIPROCAL multiplies by
 * fl32(1/127.5) as it does on CUDA (torch's scalar division there), the
 * device the reference's inference uses. */
#define RC_ENLARGE_BF16 1
#define RC_ENLARGE_RECIPROCAL 2
int rc_enlarge_block(const uint8_t* src, long long frame_stride, long long row_stride, int valid,
                     int block, int h, int w, int out_h, int out_w, int flags, void* out,
                     rc_stream_t stream);

/* One output frame of recavsr_infer/strips.py:72-99 (`blend_strips`): strip s's
 * uint8 frame [height, widths[s], 3] (device pointer frames[s], row stride
 * row_strides[s] bytes) placed at column offsets[s] and weighted by its feather
 * ramp weights[s] (device fp32 [widths[s]]); canvas summed in strip order in
 * fp32, divided by total (device fp32 [width]), + 0.5, clipped to [0, 255] and
 * truncated into out (device uint8 [height, width, 3], row stride
 * out_row_stride bytes). frames / row_strides / offsets / widths / weights are
 * host arrays of n_strips (<= 16) entries. */
int rc_strip_blend(int n_strips, const uint8_t* const* frames, const long long* row_strides,
                   const int* offsets, const int* widths, const float* const* weights,
                   const float* total, int height, int width, uint8_t* out, long long out_row_stride,
                   rc_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* RECAVSR_B200_H_ */
