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
// One CTA per (8 x 16-query tile of one frame, query head), two CTAs per SM.
// The union of the tile's windows in a visible frame is covered by 16 x 8 key
// boxes (16 rows x 8 columns: 1280 keys for the 31 x 39 union of a 24 x 24
// window, against 1536 for 8 x 16 boxes), loaded by TMA from a 5-D view
// (d, x, y, frame, head) that zero-fills past the grid. Per key box: S = Q K^T
// (M 128 queries, N 128 keys, K = D) into one of two 128-column TMEM buffers;
// four softmax warps (one query row per thread, its TMEM lane) take the row
// maximum over the visible keys, write P = 2^(s - max) (bf16 / fp16 pairs)
// over the first 64 columns of the same buffer, and the P V product (M 128,
// N = D, K 128 keys, A from TMEM) lands in the buffer's last 64 columns, which
// the threads fold into their register accumulator with the online rescale.
// A buffer is reused two boxes later, after that fold. Each warp covers two
// query rows, so whole key rows outside both rows' windows are skipped (no
// exponentials, P = 0), and chunks of rows both see take a path without row
// masks. The kernel is issue-bound (not MUFU-bound) at this size, so every
// exponential runs on the MUFU. Warp 4 loads, warp 5 issues the MMAs. Every wait is
// bounded; on expiry the kernel records an error word and unwinds.
#include <cuda_fp16.h>

#include "sm100.cuh"

namespace {

constexpr int kD = 64;                 // head dim
constexpr int kBM = 128;               // queries (and keys) per tile
constexpr int kBH = 8, kBW = 16;       // query tile: 8 rows x 16 columns
constexpr int kKH = 16, kKW = 8;       // key box: 16 rows x 8 columns
constexpr int kStages = 3;             // K / V ring
constexpr int kTile = kBM * kD * 2;    // 16 KB: 128 rows of 128 B
constexpr int kThreads = 192;          // 4 softmax warps, producer, MMA
constexpr int kTmemCols = 256;         // two S buffers; P and P.V alias their halves

struct Layout {
  static constexpr int offQ = 0;
  static constexpr int offK = offQ + kTile;
  static constexpr int offV = offK + kStages * kTile;
  static constexpr int offBar = offV + kStages * kTile;
  static constexpr int kBars = 1 + 2 * kStages + 2 + 2 + 1 + 1 + 1;
  static constexpr int kAlloc = offBar + kBars * 8 + 32;
};

struct FdParams {
  int H, W, QF, NF, HQ, HK, R, TW, wh, ww;
  int tiles_y, tiles_x;
  float scale_log2;                    // D^-0.5 * log2(e)
  int fp16;
  long long out_head, out_token;       // element strides of the output
  void* out;                           // this batch item's output
};

// Instruction descriptor, kind::f16, fp32 accumulator, A / B bf16 or fp16.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, int fp16, int b_mn_major) {
  return (1u << 4) | ((fp16 ? 0u : 1u) << 7) | ((fp16 ? 0u : 1u) << 10) | ((uint32_t)b_mn_major << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// The key boxes of one query tile: visible frames [f0, f1), rows from r0 in
// nrb boxes of 16, columns from c0 in ncb boxes of 8.
struct KeyTiles {
  int f0, f1, r0, c0, nrb, ncb;
  __device__ int count() const { return (f1 - f0) * nrb * ncb; }
  __device__ void at(int j, int& f, int& ky0, int& kx0) const {
    const int per = nrb * ncb;
    f = f0 + j / per;
    const int r = j % per;
    ky0 = r0 + (r / ncb) * kKH;
    kx0 = c0 + (r % ncb) * kKW;
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
  t.nrb = rhi >= rlo ? (rhi - rlo + kKH) / kKH : 0;
  t.ncb = chi >= clo ? (chi - clo + kKW) / kKW : 0;
  return t;
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b, int fp16) {
  if (fp16) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
  return rc::pack_bf16x2(a, b);
}

__global__ void __launch_bounds__(kThreads, 2)
fd_attention_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                    const __grid_constant__ CUtensorMap tmap_v, const FdParams p) {
  // 1024-byte alignment: the 128-byte TMA swizzle pattern repeats every 1024 bytes.
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Layout::offBar);
  uint64_t* q_full = bars;
  uint64_t* kv_full = q_full + 1;          // [kStages]
  uint64_t* kv_empty = kv_full + kStages;  // [kStages]
  uint64_t* s_full = kv_empty + kStages;   // [2] S of the buffer's box computed
  uint64_t* s_free = s_full + 2;           // [2] buffer folded and free (128 arrivals)
  uint64_t* p_full = s_free + 2;           // P written (128 arrivals)
  uint64_t* pv_full = p_full + 1;          // P V finished
  uint64_t* done = pv_full + 1;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(done + 1);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 2);

  const int warp = threadIdx.x >> 5;
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
    // The swizzled TMA tiles need a 1024-byte aligned dynamic shared memory
    // base; record an error (and load nothing) if the launch did not give one.
    *abort_flag = (sm100::smem_u32(smem) & 1023u) ? 1 : 0;
    if (*abort_flag) rc::device_fail(kKernDecoderAttention, 15);
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
  const int T = *abort_flag ? 0 : kt.count();

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
    if (T > 0 && sm100::elect_one_sync()) {
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
    if (T > 0 && sm100::elect_one_sync()) {
      const uint32_t idesc_qk = idesc_f16(kBM, kBM, p.fp16, 0);
      const uint32_t idesc_pv = idesc_f16(kBM, kD, p.fp16, 1);
      const uint64_t dq = sm100::desc_kmajor_sw128(sm100::smem_u32(smem + Layout::offQ));
      const uint64_t dk0 = sm100::desc_kmajor_sw128(sm100::smem_u32(smem + Layout::offK));
      const uint64_t dv0 = sm100::desc_mnmajor_sw128(sm100::smem_u32(smem + Layout::offV), kTile);
      bool ok = wait(q_full, 0, 2);
      int stage = 0, prev_stage = 0;
      uint32_t phase = 0;
      // Per step j: S(j) into buffer j & 1 (once box j - 2's P V there has
      // been folded), then P(j-1) V into the last 64 columns of buffer
      // (j - 1) & 1 (once P(j-1) is written over its first 64 columns).
      for (int j = 0; ok && j <= T; ++j) {
        if (j < T) {
          const int b = j & 1;
          if (!wait(&kv_full[stage], phase, 3)) { ok = false; break; }
          if (j >= 2 && !wait(&s_free[b], ((j >> 1) - 1) & 1, 4)) { ok = false; break; }
          sm100::tc_fence_after();
          const uint64_t dk = sm100::desc_add(dk0, stage * kTile);
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk)
            sm100::mma_f16_ss(tmem + b * 128, sm100::desc_add(dq, 32 * kk), sm100::desc_add(dk, 32 * kk),
                              idesc_qk, kk > 0 ? 1u : 0u);
          sm100::tc_commit(&s_full[b]);
        }
        if (j >= 1) {
          const int i = j - 1, b = i & 1;
          if (!wait(p_full, i & 1, 5)) { ok = false; break; }
          sm100::tc_fence_after();
          const uint64_t dv = sm100::desc_add(dv0, prev_stage * kTile);
#pragma unroll
          for (int kk = 0; kk < kBM / 16; ++kk)
            sm100::mma_f16_ts(tmem + b * 128 + 64, tmem + b * 128 + 8 * kk, sm100::desc_add(dv, kk * 16 * 128),
                              idesc_pv, kk > 0 ? 1u : 0u);
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
    // Thread r = query (ty*8 + r/16, tx*16 + r%16); warp w holds query rows
    // 2w and 2w + 1 of the tile (lanes 0-15 / 16-31).
    const int r = threadIdx.x;
    const int qy = ty * kBH + (r >> 4), qx = tx * kBW + (r & 15);
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    const int lo_y = max(qy - p.wh / 2, 0), hi_y = min(qy + p.wh / 2 - 1, p.H - 1);
    const int lo_x = max(qx - p.ww / 2, 0), hi_x = min(qx + p.ww / 2 - 1, p.W - 1);
    // Key rows either query row of the warp sees ([any_lo, any_hi]: the upper
    // row's start, the lower row's end) and rows both see ([all_lo, all_hi]).
    const int any_lo = __shfl_sync(0xffffffffu, lo_y, 0), any_hi = __shfl_sync(0xffffffffu, hi_y, 16);
    const int all_lo = __shfl_sync(0xffffffffu, lo_y, 16), all_hi = __shfl_sync(0xffffffffu, hi_y, 0);
    const float sc = p.scale_log2;
    const float2 sc2 = make_float2(sc, sc);
    float o[kD];
#pragma unroll
    for (int d = 0; d < kD; ++d) o[d] = 0.f;
    float m = -INFINITY, l = 0.f, alpha_prev = 0.f;
    bool ok = T > 0;
    // o = o * a + (the P V tile in TMEM buffer b), which frees buffer b.
    auto fold = [&](float a, int b) {
      uint32_t w[4][16];
#pragma unroll
      for (int c = 0; c < 4; ++c) sm100::tmem_ld16(tmem + b * 128 + 64 + 16 * c + lane_off, w[c]);
      sm100::tmem_ld_wait();
      const float2 a2 = make_float2(a, a);
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int d = 0; d < 16; d += 2) {
          const float2 t = __ffma2_rn(make_float2(o[16 * c + d], o[16 * c + d + 1]), a2,
                                      make_float2(__uint_as_float(w[c][d]), __uint_as_float(w[c][d + 1])));
          o[16 * c + d] = t.x;
          o[16 * c + d + 1] = t.y;
        }
    };
    // 32 S values (4 box rows x 8 columns) of chunk c of buffer sb.
    auto load_chunk = [&](uint32_t sb, int c, uint32_t (&w)[32]) {
      sm100::tmem_ld16(sb + c, *reinterpret_cast<uint32_t(*)[16]>(&w[0]));
      sm100::tmem_ld16(sb + c + 16, *reinterpret_cast<uint32_t(*)[16]>(&w[16]));
      sm100::tmem_ld_wait();
    };
    for (int j = 0; j < T && ok; ++j) {
      int f, ky0, kx0;
      kt.at(j, f, ky0, kx0);
      (void)f;
      const int b = j & 1;
      ok = __all_sync(0xffffffffu, wait(&s_full[b], (j >> 1) & 1, 6));
      if (!ok) break;
      sm100::tc_fence_after();
      const uint32_t sb = tmem + b * 128 + lane_off;
      // Pass 1: per key column, the maximum over the key rows this query
      // sees (key c of the box is row c / 8, column c % 8); then the maximum
      // over the columns it sees.
      float cm[kKW];
#pragma unroll
      for (int k = 0; k < kKW; ++k) cm[k] = -INFINITY;
#pragma unroll
      for (int c = 0; c < kBM; c += 32) {
        const int y0 = ky0 + c / 8;                             // the chunk's rows y0 .. y0 + 3
        if (y0 + 3 < any_lo || y0 > any_hi) continue;           // warp-uniform: none visible
        uint32_t w[32];
        load_chunk(sb, c, w);
        if (y0 >= all_lo && y0 + 3 <= all_hi) {                // warp-uniform: all visible
#pragma unroll
          for (int k = 0; k < kKW; ++k) {
            cm[k] = rc::max3(cm[k], __uint_as_float(w[k]), __uint_as_float(w[8 + k]));
            cm[k] = rc::max3(cm[k], __uint_as_float(w[16 + k]), __uint_as_float(w[24 + k]));
          }
        } else {
#pragma unroll
          for (int rr = 0; rr < 4; ++rr) {
            const bool vis = y0 + rr >= lo_y && y0 + rr <= hi_y;
#pragma unroll
            for (int k = 0; k < kKW; ++k) cm[k] = vis ? fmaxf(cm[k], __uint_as_float(w[8 * rr + k])) : cm[k];
          }
        }
      }
      // Column bias: 0 for the key columns this query sees, -inf otherwise.
      float cneg[kKW];
#pragma unroll
      for (int k = 0; k < kKW; ++k) cneg[k] = (kx0 + k >= lo_x && kx0 + k <= hi_x) ? 0.f : -INFINITY;
      const float mj = rc::max3(rc::max3(cm[0] + cneg[0], cm[1] + cneg[1], cm[2] + cneg[2]),
                                rc::max3(cm[3] + cneg[3], cm[4] + cneg[4], cm[5] + cneg[5]),
                                fmaxf(cm[6] + cneg[6], cm[7] + cneg[7]));
      const float mn = fmaxf(m, mj == -INFINITY ? -INFINITY : __fmul_rn(mj, sc));
      const float alpha = mn == -INFINITY ? 1.f : rc::fast_exp2(m - mn);
      // The previous box's P V: fold it in, then its buffer is free for S(j + 1).
      if (j >= 1) {
        ok = __all_sync(0xffffffffu, wait(pv_full, (j - 1) & 1, 7));
        if (!ok) break;
        sm100::tc_fence_after();
        fold(alpha_prev, b ^ 1);
        sm100::tc_fence_before();
        sm100::mbar_arrive(&s_free[b ^ 1]);
      }
      // Pass 2: P = 2^(s * scale - max) over the visible keys, written over
      // the S columns already read (32 keys -> 16 P words per chunk).
      const float nm = mn == -INFINITY ? 0.f : -mn;
      float2 cb[kKW / 2];
#pragma unroll
      for (int k = 0; k < kKW / 2; ++k) cb[k] = make_float2(cneg[2 * k] + nm, cneg[2 * k + 1] + nm);
      float2 sum2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
      for (int c = 0; c < kBM; c += 32) {
        const int y0 = ky0 + c / 8;
        uint32_t pk[16];
        if (y0 + 3 < any_lo || y0 > any_hi) {                   // warp-uniform: none visible
#pragma unroll
          for (int i = 0; i < 16; ++i) pk[i] = 0u;
        } else {
          uint32_t w[32];
          load_chunk(sb, c, w);
          const bool all = y0 >= all_lo && y0 + 3 <= all_hi;   // warp-uniform
#pragma unroll
          for (int rr = 0; rr < 4; ++rr) {
            const float rneg = (all || (y0 + rr >= lo_y && y0 + rr <= hi_y)) ? 0.f : -INFINITY;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const float2 s2 = make_float2(__uint_as_float(w[8 * rr + 2 * k]), __uint_as_float(w[8 * rr + 2 * k + 1]));
              float2 xv = __ffma2_rn(s2, sc2, cb[k]);
              if (!all) xv = __fadd2_rn(xv, make_float2(rneg, rneg));
              float2 e;
              e.x = rc::fast_exp2(xv.x);
              e.y = rc::fast_exp2(xv.y);
              sum2[k & 1] = __fadd2_rn(sum2[k & 1], e);
              pk[4 * rr + k] = pack_half2(e.x, e.y, p.fp16);
            }
          }
        }
        sm100::tmem_st16(sb + c / 2, pk);
      }
      l = __fmaf_rn(l, alpha, (sum2[0].x + sum2[0].y) + (sum2[1].x + sum2[1].y));
      m = mn;
      alpha_prev = alpha;
      sm100::tmem_st_wait();
      sm100::tc_fence_before();
      sm100::mbar_arrive(p_full);
    }
    if (ok) ok = __all_sync(0xffffffffu, wait(pv_full, (T - 1) & 1, 8));
    if (ok) {
      sm100::tc_fence_after();
      fold(alpha_prev, (T - 1) & 1);
      if (qy < p.H && qx < p.W) {
        const float inv = 1.f / l;
        const long long n = (long long)p.H * p.W;
        uint8_t* dst = reinterpret_cast<uint8_t*>(p.out) +
                       ((long long)hq * p.out_head + ((long long)qt * n + (long long)qy * p.W + qx) * p.out_token) * 2;
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
             long long token_stride, long long head_stride, int box_w, int box_h, const char* what) {
  const uint64_t dims[5] = {(uint64_t)kD, (uint64_t)W, (uint64_t)H, (uint64_t)frames, (uint64_t)heads};
  const uint64_t str[4] = {(uint64_t)token_stride * 2, (uint64_t)token_stride * 2 * W,
                           (uint64_t)token_stride * 2 * W * H, (uint64_t)head_stride * 2};
  const uint32_t box[5] = {kD, (uint32_t)box_w, (uint32_t)box_h, 1, 1};
  return rc::encode_tmap(m, fp16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5,
                         const_cast<void*>(base), dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B, what);
}

}  // namespace

RC_DEVICE_ERROR_ACCESSOR(decoder_attention)

extern "C" {

int rc_local_gqa_attention(const void* q, const void* k, const void* v, const long long* strides, int B,
                           int HQ, int HK, int QF, int NF, int H, int W, int D, int window_h, int window_w,
                           int group_size, int temporal_window, int fp16, void* out,
                           const long long* out_strides, cudaStream_t stream) {
  const char* what = "rc_local_gqa_attention";
  if (D != kD) return rc::set_error(RC_ERR_UNSUPPORTED, "%s: head_dim %d (64 supported)", what, D);
  if (B < 1 || HQ < 1 || HK < 1 || HQ % HK || H < 1 || W < 1 || QF < 1 || NF < QF || group_size < 1 ||
      temporal_window < 1 || QF % group_size || NF % group_size || window_h < 2 || window_w < 2 ||
      window_h % 2 || window_w % 2)
    return rc::set_error(RC_ERR_ARG, "%s: invalid local grid, GQA heads or temporal group alignment", what);
  if (!q || !k || !v || !out || !strides) return rc::set_error(RC_ERR_ARG, "%s: missing pointer", what);
  for (int i = 0; i < 9; ++i)
    if (strides[i] % 8) return rc::set_error(RC_ERR_ARG, "%s: strides must be multiples of 8 elements", what);
  const long long n = (long long)H * W;
  // Output strides (batch, head, token) in elements; NULL = contiguous [B, HQ, QF*n, D].
  const long long ob = out_strides ? out_strides[0] : (long long)HQ * QF * n * kD;
  const long long oh = out_strides ? out_strides[1] : (long long)QF * n * kD;
  const long long ot = out_strides ? out_strides[2] : kD;
  if (ob % 8 || oh % 8 || ot % 8 || ot < kD || (reinterpret_cast<uintptr_t>(out) & 15))
    return rc::set_error(RC_ERR_ARG, "%s: output must be 16-byte aligned with strides in multiples of 8", what);
  const int ty = (H + kBH - 1) / kBH, tx = (W + kBW - 1) / kBW;
  if ((long long)QF * ty * tx > 2147483647LL || HQ > 65535)
    return rc::set_error(RC_ERR_ARG, "%s: grid too large", what);
  static rc::SmemAttrFlags attr_flags = {};
  if (const int st = rc::ensure_smem_attr(attr_flags, reinterpret_cast<const void*>(fd_attention_kernel),
                                          Layout::kAlloc, what))
    return st;
  for (int b = 0; b < B; ++b) {
    // strides: (batch, head, token) of q, k, v in elements.
    const uint8_t* qb = reinterpret_cast<const uint8_t*>(q) + strides[0] * 2 * b;
    const uint8_t* kb = reinterpret_cast<const uint8_t*>(k) + strides[3] * 2 * b;
    const uint8_t* vb = reinterpret_cast<const uint8_t*>(v) + strides[6] * 2 * b;
    CUtensorMap mq, mk, mv;
    int r = make_map(&mq, qb, fp16, W, H, QF, HQ, strides[2], strides[1], kBW, kBH, what);
    if (!r) r = make_map(&mk, kb, fp16, W, H, NF, HK, strides[5], strides[4], kKW, kKH, what);
    if (!r) r = make_map(&mv, vb, fp16, W, H, NF, HK, strides[8], strides[7], kKW, kKH, what);
    if (r) return r;
    FdParams p{H, W, QF, NF, HQ, HK, group_size, temporal_window, window_h, window_w, ty, tx,
               1.4426950408889634f / sqrtf((float)kD), fp16 ? 1 : 0, oh, ot,
               reinterpret_cast<uint8_t*>(out) + b * ob * 2};
    r = rc::check_launch(rc::launch_pdl(fd_attention_kernel, dim3(QF * ty * tx, HQ), dim3(kThreads),
                                        Layout::kAlloc, stream, mq, mk, mv, p),
                         what);
    if (r) return r;
  }
  return RC_OK;
}

}  // extern "C"
