// Local grouped-query attention of the FlashDecoder on tcgen05
// (replaces recavsr_infer/models/flashdecoder/_local_attention_triton.py:21-131,
// the Triton forward `_forward`, and the masked SDPA of
// flashdecoder_wan22.py:38-119 `_local_attention`).
//
// Semantics: q [B, HQ, QF*n, D], k / v [B, HK, NF*n, D] with n = H*W tokens per
// frame (row-major y, x); query head h reads key / value head h / (HQ / HK). A
// query of frame qt belongs to temporal group qg = (qt + NF - QF) / R and sees
// the key frames of groups (qg - TW, qg]; within a frame it sees the keys at
// dy in [-wh/2, wh/2), dx in [-ww/2, ww/2) around its own position, truncated
// at the grid border (no window clamping). Softmax with scale D^-0.5.
//
// One CTA per (8 x 16-query tile of one frame, query head): the queries'
// union of windows in a visible frame is covered by 8 x 16 key boxes, loaded
// by TMA from a 5-D view (d, x, y, frame, head) that zero-fills past the grid.
// Per key box: S = Q K^T on the tensor core (M 128 queries, N 128 keys, K =
// D) into one of two TMEM buffers; four softmax warps (one query row per
// thread, its TMEM lane) mask the truncated window, update the running max
// and sum, write P (bf16 / fp16 pairs) into TMEM; P V (M 128, N = D, K 128
// keys, A from TMEM) lands in a TMEM tile that the softmax threads fold into
// their register accumulator with the online rescale. Warp 4 loads, warp 5
// issues the MMAs. Every wait is bounded; on expiry the kernel records an
// error word and unwinds.
#include <cuda_fp16.h>

#include "sm100.cuh"

namespace {

constexpr int kD = 64;                 // head dim
constexpr int kBM = 128;               // queries (and keys) per tile: 8 rows x 16 columns
constexpr int kBH = 8, kBW = 16;
constexpr int kStages = 3;             // K / V ring
constexpr int kTile = kBM * kD * 2;    // 16 KB: 128 rows of 128 B
constexpr int kThreads = 192;          // 4 softmax warps, producer, MMA
constexpr int kTmemCols = 512;
constexpr uint32_t kTmS = 0, kTmP = 256, kTmPV = 320;   // S x2 (128 cols each), P (64), PV (64)

struct Layout {
  static constexpr int offQ = 0;
  static constexpr int offK = offQ + kTile;
  static constexpr int offV = offK + kStages * kTile;
  static constexpr int offBar = offV + kStages * kTile;
  static constexpr int kBars = 1 + 2 * kStages + 2 + 2 + 1 + 1 + 1;
  static constexpr int kAlloc = offBar + kBars * 8 + 32 + 1024;   // + alignment slack
};

struct FdParams {
  int H, W, QF, NF, HQ, HK, R, TW, wh, ww;
  int tiles_y, tiles_x;
  float scale_log2;                    // D^-0.5 * log2(e)
  int fp16;
  void* out;                           // [HQ, QF*n, D] of this batch item, contiguous
};

// Instruction descriptor, kind::f16, fp32 accumulator, A / B bf16 or fp16.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, int fp16, int b_mn_major) {
  return (1u << 4) | ((fp16 ? 0u : 1u) << 7) | ((fp16 ? 0u : 1u) << 10) | ((uint32_t)b_mn_major << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// The key boxes of one query tile: visible frames [f0, f1), rows from r0 in
// nrb boxes of 8, columns from c0 in ncb boxes of 16.
struct KeyTiles {
  int f0, f1, r0, c0, nrb, ncb;
  __device__ int count() const { return (f1 - f0) * nrb * ncb; }
  __device__ void at(int j, int& f, int& ky0, int& kx0) const {
    const int per = nrb * ncb;
    f = f0 + j / per;
    const int r = j % per;
    ky0 = r0 + (r / ncb) * kBH;
    kx0 = c0 + (r % ncb) * kBW;
  }
};

__device__ KeyTiles key_tiles(const FdParams& p, int qt, int ty, int tx) {
  KeyTiles t;
  const int qg = (qt + p.NF - p.QF) / p.R;
  t.f0 = max((qg - p.TW + 1) * p.R, 0);
  t.f1 = min((qg + 1) * p.R, p.NF);
  // Rows / columns any query of the tile can see (half-open window, truncated).
  const int rlo = max(ty * kBH - p.wh / 2, 0), rhi = min(ty * kBH + kBH - 1 + p.wh / 2 - 1, p.H - 1);
  const int clo = max(tx * kBW - p.ww / 2, 0), chi = min(tx * kBW + kBW - 1 + p.ww / 2 - 1, p.W - 1);
  t.r0 = rlo;
  t.c0 = clo;
  t.nrb = rhi >= rlo ? (rhi - rlo + kBH) / kBH : 0;
  t.ncb = chi >= clo ? (chi - clo + kBW) / kBW : 0;
  return t;
}

// 2^x with the MUFU approximation (flushes denormal results to zero; a few
// ulp, far below the bf16 / fp16 rounding of P).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b, int fp16) {
  if (fp16) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
  return rc::pack_bf16x2(a, b);
}

__global__ void __launch_bounds__(kThreads, 1)
fd_attention_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                    const __grid_constant__ CUtensorMap tmap_v, const FdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Layout::offBar);
  uint64_t* q_full = bars;
  uint64_t* kv_full = q_full + 1;          // [kStages]
  uint64_t* kv_empty = kv_full + kStages;  // [kStages]
  uint64_t* s_full = kv_empty + kStages;   // [2]
  uint64_t* s_free = s_full + 2;           // [2]
  uint64_t* p_full = s_free + 2;
  uint64_t* pv_full = p_full + 1;
  uint64_t* done = pv_full + 1;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(done + 1);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, hq = blockIdx.y;
  const int per_frame = p.tiles_y * p.tiles_x;
  const int qt = tile / per_frame, ty = (tile % per_frame) / p.tiles_x, tx = tile % p.tiles_x;
  const int hk = hq / (p.HQ / p.HK);

  if (threadIdx.x == 0) {
    sm100::mbar_init(q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      sm100::mbar_init(&kv_full[s], 1);
      sm100::mbar_init(&kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      sm100::mbar_init(&s_full[b], 1);
      sm100::mbar_init(&s_free[b], kBM);
    }
    sm100::mbar_init(p_full, kBM);
    sm100::mbar_init(pv_full, 1);
    sm100::mbar_init(done, 1);
    *abort_flag = 0;
    sm100::fence_mbar_init();
  }
  if (warp == 5) {
    sm100::tmem_alloc(tmem_slot, kTmemCols);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  rc::pdl_trigger();
  rc::pdl_wait();
  const uint32_t tmem = *tmem_slot;
  const KeyTiles kt = key_tiles(p, qt, ty, tx);
  const int T = kt.count();

  auto fail = [&](unsigned int site) {
    if (!*abort_flag) rc::device_fail(kKernDecoderAttention, site);
    *abort_flag = 1;
  };
  auto wait = [&](uint64_t* bar, uint32_t parity, unsigned int site) -> bool {
    if (sm100::mbar_wait(bar, parity, abort_flag)) return true;
    if (!*abort_flag) fail(site);
    return false;
  };

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    if (sm100::elect_one_sync()) {
      sm100::tma_prefetch_desc(&tmap_q);
      sm100::tma_prefetch_desc(&tmap_k);
      sm100::tma_prefetch_desc(&tmap_v);
      sm100::mbar_arrive_expect_tx(q_full, kTile);
      sm100::tma_load_5d(smem + Layout::offQ, &tmap_q, q_full, 0, tx * kBW, ty * kBH, qt, hq);
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      for (int j = 0; j < T; ++j) {
        if (!wait(&kv_empty[stage], phase ^ 1, 1)) break;
        int f, ky0, kx0;
        kt.at(j, f, ky0, kx0);
        sm100::mbar_arrive_expect_tx(&kv_full[stage], 2 * kTile);
        sm100::tma_load_5d(smem + Layout::offK + stage * kTile, &tmap_k, &kv_full[stage], 0, kx0, ky0, f, hk);
        sm100::tma_load_5d(smem + Layout::offV + stage * kTile, &tmap_v, &kv_full[stage], 0, kx0, ky0, f, hk);
        ++issued;
        if (++stage == kStages) { stage = 0; phase ^= 1; }
      }
      // Drain: the loads this thread issued land before the CTA exits.
      sm100::mbar_wait(q_full, 0);
      for (int s = 0; s < kStages && issued > 0; ++s, --issued) {
        if (stage == 0) { stage = kStages; phase ^= 1; }
        --stage;
        sm100::mbar_wait(&kv_full[stage], phase);
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (sm100::elect_one_sync()) {
      const uint32_t idesc_qk = idesc_f16(kBM, kBM, p.fp16, 0);
      const uint32_t idesc_pv = idesc_f16(kBM, kD, p.fp16, 1);
      const uint64_t dq = sm100::desc_kmajor_sw128(sm100::smem_u32(smem + Layout::offQ));
      const uint64_t dk0 = sm100::desc_kmajor_sw128(sm100::smem_u32(smem + Layout::offK));
      const uint64_t dv0 = sm100::desc_mnmajor_sw128(sm100::smem_u32(smem + Layout::offV), kTile);
      bool ok = wait(q_full, 0, 2);
      int stage = 0, prev_stage = 0;
      uint32_t phase = 0;
      for (int j = 0; ok && j <= T; ++j) {
        if (j < T) {
          const int b = j & 1;
          if (!wait(&kv_full[stage], phase, 3)) { ok = false; break; }
          if (j >= 2 && !wait(&s_free[b], ((j >> 1) - 1) & 1, 4)) { ok = false; break; }
          sm100::tc_fence_after();
          const uint64_t dk = sm100::desc_add(dk0, stage * kTile);
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk)
            sm100::mma_f16_ss(tmem + kTmS + b * 128, sm100::desc_add(dq, 32 * kk), sm100::desc_add(dk, 32 * kk),
                              idesc_qk, kk > 0 ? 1u : 0u);
          sm100::tc_commit(&s_full[b]);
        }
        if (j >= 1) {
          const int i = j - 1;
          if (!wait(p_full, i & 1, 5)) { ok = false; break; }
          sm100::tc_fence_after();
          const uint64_t dv = sm100::desc_add(dv0, prev_stage * kTile);
#pragma unroll
          for (int kk = 0; kk < kBM / 16; ++kk)
            sm100::mma_f16_ts(tmem + kTmPV, tmem + kTmP + 8 * kk, sm100::desc_add(dv, kk * 16 * 128), idesc_pv,
                              kk > 0 ? 1u : 0u);
          sm100::tc_commit(pv_full);
          sm100::tc_commit(&kv_empty[prev_stage]);
        }
        prev_stage = stage;
        if (j < T && ++stage == kStages) { stage = 0; phase ^= 1; }
      }
      sm100::tc_commit(done);
      sm100::mbar_wait(done, 0);
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int r = threadIdx.x;                       // query row = TMEM lane
    const int qy = ty * kBH + (r >> 4), qx = tx * kBW + (r & 15);
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    const int lo_y = max(qy - p.wh / 2, 0), hi_y = min(qy + p.wh / 2 - 1, p.H - 1);
    const int lo_x = max(qx - p.ww / 2, 0), hi_x = min(qx + p.ww / 2 - 1, p.W - 1);
    const float sc = p.scale_log2;
    float o[kD];
#pragma unroll
    for (int d = 0; d < kD; ++d) o[d] = 0.f;
    float m = -INFINITY, l = 0.f, alpha_prev = 0.f;
    bool ok = true;
    // o = o * a + (the P V tile in TMEM)
    auto fold = [&](float a) {
#pragma unroll
      for (int c = 0; c < kD; c += 16) {
        uint32_t w[16];
        sm100::tmem_ld16(tmem + kTmPV + c + lane_off, w);
        sm100::tmem_ld_wait();
#pragma unroll
        for (int d = 0; d < 16; ++d) o[c + d] = fmaf(o[c + d], a, __uint_as_float(w[d]));
      }
    };
    for (int j = 0; j < T && ok; ++j) {
      int f, ky0, kx0;
      kt.at(j, f, ky0, kx0);
      (void)f;
      const int b = j & 1;
      ok = __all_sync(0xffffffffu, wait(&s_full[b], (j >> 1) & 1, 6));
      if (!ok) break;
      sm100::tc_fence_after();
      // Visible rows / columns of this 8 x 16 key box for this query (key c
      // of the box is row c / 16, column c % 16).
      uint32_t rowmask = 0, colmask = 0;
#pragma unroll
      for (int i = 0; i < kBH; ++i) rowmask |= (uint32_t)(ky0 + i >= lo_y && ky0 + i <= hi_y) << i;
#pragma unroll
      for (int i = 0; i < kBW; ++i) colmask |= (uint32_t)(kx0 + i >= lo_x && kx0 + i <= hi_x) << i;
      const uint32_t sb = tmem + kTmS + b * 128 + lane_off;
      // Pass 1: the row maximum over the visible keys.
      float mj = -INFINITY;
#pragma unroll
      for (int c = 0; c < kBM; c += 16) {
        uint32_t w[16];
        sm100::tmem_ld16(sb + c, w);
        sm100::tmem_ld_wait();
        if ((rowmask >> (c >> 4)) & 1u) {
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if ((colmask >> i) & 1u) mj = fmaxf(mj, __uint_as_float(w[i]));
        }
      }
      const float mn = fmaxf(m, mj == -INFINITY ? -INFINITY : __fmul_rn(mj, sc));
      const float alpha = mn == -INFINITY ? 1.f : fast_exp2(m - mn);
      // The previous box's P V: fold it in (this also frees P).
      if (j >= 1) {
        ok = __all_sync(0xffffffffu, wait(pv_full, (j - 1) & 1, 7));
        if (!ok) break;
        sm100::tc_fence_after();
        fold(alpha_prev);
      }
      // Pass 2: P = 2^(s * scale - max) on visible keys, 32 keys per TMEM store.
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < kBM; c += 32) {
        uint32_t w[32], pk[16];
        sm100::tmem_ld16(sb + c, *reinterpret_cast<uint32_t(*)[16]>(&w[0]));
        sm100::tmem_ld16(sb + c + 16, *reinterpret_cast<uint32_t(*)[16]>(&w[16]));
        sm100::tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const int c0 = c + i;
          const bool v0 = ((rowmask >> (c0 >> 4)) & (colmask >> (c0 & 15)) & 1u) != 0;
          const bool v1 = ((rowmask >> ((c0 + 1) >> 4)) & (colmask >> ((c0 + 1) & 15)) & 1u) != 0;
          const float p0 = v0 ? fast_exp2(__fmaf_rn(__uint_as_float(w[i]), sc, -mn)) : 0.f;
          const float p1 = v1 ? fast_exp2(__fmaf_rn(__uint_as_float(w[i + 1]), sc, -mn)) : 0.f;
          sum += p0 + p1;
          pk[i / 2] = pack_half2(p0, p1, p.fp16);
        }
        sm100::tmem_st16(tmem + kTmP + c / 2 + lane_off, pk);
      }
      l = l * alpha + sum;
      m = mn;
      alpha_prev = alpha;
      sm100::tmem_st_wait();
      sm100::tc_fence_before();
      sm100::mbar_arrive(&s_free[b]);
      sm100::mbar_arrive(p_full);
    }
    if (ok && T > 0) ok = __all_sync(0xffffffffu, wait(pv_full, (T - 1) & 1, 8));
    if (ok && T > 0) {
      sm100::tc_fence_after();
      fold(alpha_prev);
      if (qy < p.H && qx < p.W) {
        const float inv = 1.f / l;
        const long long n = (long long)p.H * p.W;
        uint8_t* dst = reinterpret_cast<uint8_t*>(p.out) +
                       (((long long)hq * p.QF * n + (long long)qt * n + (long long)qy * p.W + qx) * kD) * 2;
#pragma unroll
        for (int d = 0; d < kD; d += 8) {
          uint4 w;
          w.x = pack_half2(o[d] * inv, o[d + 1] * inv, p.fp16);
          w.y = pack_half2(o[d + 2] * inv, o[d + 3] * inv, p.fp16);
          w.z = pack_half2(o[d + 4] * inv, o[d + 5] * inv, p.fp16);
          w.w = pack_half2(o[d + 6] * inv, o[d + 7] * inv, p.fp16);
          *reinterpret_cast<uint4*>(dst + d * 2) = w;
        }
      }
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    __syncwarp();
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, kTmemCols);
  }
}

// 5-D view (d, x, y, frame, head) of one batch item's [heads, frames*H*W, D]
// tensor with element strides token_stride / head_stride (d contiguous).
int make_map(CUtensorMap* m, const void* base, int fp16, int W, int H, int frames, int heads,
             long long token_stride, long long head_stride, const char* what) {
  const uint64_t dims[5] = {(uint64_t)kD, (uint64_t)W, (uint64_t)H, (uint64_t)frames, (uint64_t)heads};
  const uint64_t str[4] = {(uint64_t)token_stride * 2, (uint64_t)token_stride * 2 * W,
                           (uint64_t)token_stride * 2 * W * H, (uint64_t)head_stride * 2};
  const uint32_t box[5] = {kD, kBW, kBH, 1, 1};
  return rc::encode_tmap(m, fp16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5,
                         const_cast<void*>(base), dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B, what);
}

}  // namespace

RC_DEVICE_ERROR_ACCESSOR(decoder_attention)

extern "C" {

int rc_local_gqa_attention(const void* q, const void* k, const void* v, const long long* strides, int B,
                           int HQ, int HK, int QF, int NF, int H, int W, int D, int window_h, int window_w,
                           int group_size, int temporal_window, int fp16, void* out, cudaStream_t stream) {
  const char* what = "rc_local_gqa_attention";
  if (D != kD) return rc::set_error(RC_ERR_UNSUPPORTED, "%s: head_dim %d (64 supported)", what, D);
  if (B < 1 || HQ < 1 || HK < 1 || HQ % HK || H < 1 || W < 1 || QF < 1 || NF < QF || group_size < 1 ||
      temporal_window < 1 || QF % group_size || NF % group_size || window_h < 2 || window_w < 2 ||
      window_h % 2 || window_w % 2)
    return rc::set_error(RC_ERR_ARG, "%s: invalid local grid, GQA heads or temporal group alignment", what);
  if (!q || !k || !v || !out || !strides) return rc::set_error(RC_ERR_ARG, "%s: missing pointer", what);
  for (int i = 0; i < 9; ++i)
    if (strides[i] % 8) return rc::set_error(RC_ERR_ARG, "%s: strides must be multiples of 8 elements", what);
  const int ty = (H + kBH - 1) / kBH, tx = (W + kBW - 1) / kBW;
  if ((long long)QF * ty * tx > 2147483647LL || HQ > 65535)
    return rc::set_error(RC_ERR_ARG, "%s: grid too large", what);
  static rc::SmemAttrFlags attr_flags = {};
  if (const int st = rc::ensure_smem_attr(attr_flags, reinterpret_cast<const void*>(fd_attention_kernel),
                                          Layout::kAlloc, what))
    return st;
  const long long n = (long long)H * W;
  for (int b = 0; b < B; ++b) {
    // strides: (batch, head, token) of q, k, v in elements.
    const uint8_t* qb = reinterpret_cast<const uint8_t*>(q) + strides[0] * 2 * b;
    const uint8_t* kb = reinterpret_cast<const uint8_t*>(k) + strides[3] * 2 * b;
    const uint8_t* vb = reinterpret_cast<const uint8_t*>(v) + strides[6] * 2 * b;
    CUtensorMap mq, mk, mv;
    int r = make_map(&mq, qb, fp16, W, H, QF, HQ, strides[2], strides[1], what);
    if (!r) r = make_map(&mk, kb, fp16, W, H, NF, HK, strides[5], strides[4], what);
    if (!r) r = make_map(&mv, vb, fp16, W, H, NF, HK, strides[8], strides[7], what);
    if (r) return r;
    FdParams p{H, W, QF, NF, HQ, HK, group_size, temporal_window, window_h, window_w, ty, tx,
               1.4426950408889634f / sqrtf((float)kD), fp16 ? 1 : 0,
               reinterpret_cast<uint8_t*>(out) + (long long)b * HQ * QF * n * kD * 2};
    r = rc::check_launch(rc::launch_pdl(fd_attention_kernel, dim3(QF * ty * tx, HQ), dim3(kThreads),
                                        Layout::kAlloc, stream, mq, mk, mv, p),
                         what);
    if (r) return r;
  }
  return RC_OK;
}

}  // extern "C"
