// Cache-routed self-attention of a QT-frame query block over the current
// frames plus the routed past planes of the KV cache
// (recavsr_infer/kernels/local_attention.py:18-169 `_paired_local` and
// :286-325 `sdpa_attention`), and the rotary-free cross-attention of
// recavsr_infer/runtime/transformer.py:123-128.
//
// Semantics (one batch element, one head):
//   planes = [past planes i with slots[i] >= 0 (position past_positions[i])]
//            + [current frames f (position query_positions[f])]
//   q and every key get the temporal rotary embedding of their plane position
//   on the first `td` dims (fp32 math, bf16 rounding), exactly as the reference;
//   a query at (qy, qx) sees, in every plane, the keys of rows
//   [top, top+WH) x cols [left, left+WW), top = clamp(qy - WH/2, 0, H - WH),
//   left = clamp(qx - WW/2, 0, W - WW), WH = min(H, window_h), WW = min(W, window_w)
//   (a window covering the grid = every key, the sdpa path);
//   out = softmax(q k^T / sqrt(d)) v with fp32 accumulation.
//
// Two kernels per launch:
//  1. rope_gather: temporally rotated copies of the current K frames and the
//     routed past K planes into a caller-provided workspace (the slot
//     indirection is applied here, so the attention kernel reads K densely).
//  2. attention: one CTA per (128-query tile, head) = one unit. With one CTA
//     per SM the units run in waves; the units of the last, partial wave are
//     split over their key tiles into up to four pieces (CTAs) that write
//     unnormalised partials, and the last piece of a unit to finish merges
//     them (flash-decoding style split-K, applied to the tail wave only).
//     Warp 0 = TMA producer: K tiles (workspace) and V tiles (read in place
//     from the cache slot / current frame) of 128 keys in a 4-stage K ring and
//     a 3-stage V ring, K three tiles ahead of V.
//     The keys of every tile are split between two independent softmax slots:
//     slot 0 (warps 2-5) takes keys 0-63, slot 1 (warps 6-9) keys 64-127. Each
//     slot keeps its own S, P and O in tensor memory and its own running max /
//     sum per row, one thread per query row (TMEM lane): per 64-key block it
//     loads S, applies the window mask, keeps a lazily rescaled running max,
//     computes exp2 and stores P (bf16). The two warps of a TMEM lane quadrant
//     (one per slot) never wait for each other until the end, where they
//     combine (O_0, m_0, l_0) and (O_1, m_1, l_1) into the output. First, each
//     slot loads half of every thread's Q row from global memory, rotates it
//     and stores it into tensor memory.
//     Warp 1 = MMA issuer: S_x = Q K_x^T and O_x += P_x V_x, A operands (Q, P)
//     in tensor memory. Slot 1 starts one block behind slot 0, so the slots
//     run out of phase and one slot's softmax overlaps the other's MMAs; the
//     issuer waits (suspending) on each MMA's inputs in the order they become
//     ready.
//   TMEM columns: S_0 [0,64) | S_1 [64,128) | P_0 [128,160) | P_1 [160,192) |
//   Q [192,256) | O_0 [256,384) | O_1 [384,512).
//   Dense mode (window covers the grid): a query tile = 128 consecutive tokens,
//   a key tile = 128 consecutive tokens of a plane (4-D TMA view; the plane
//   tail reads as zeros). Local mode: a query tile = 2 frames x 8 x 8 tokens, a
//   key tile = an 8 x 16 box of the union of the tile's windows (5-D TMA
//   view); slot 0 / 1 take its box rows 0-3 / 4-7.
#include <stdlib.h>

#include <mutex>

#include "sm100.cuh"

namespace {

constexpr int kD = 128;             // head dim supported by the tcgen05 kernel
constexpr int kBM = 128;            // queries per CTA (one TMEM lane each)
constexpr int kBN = 128;            // keys per K / V tile
constexpr int kSB = 64;             // keys per slot and tile
constexpr int kThreads = 320;       // producer, MMA, 2 slots x 4 softmax warps
constexpr int kLocalQH = 8, kLocalQW = 8;   // local query tile: 2 frames x 8 x 8
constexpr int kLocalKH = 8, kLocalKW = 16;  // local key box: 8 rows x 16 cols
constexpr int kMaxPlanes = 16;
constexpr float kRescaleThreshold = 8.0f;   // log2 units

// Tensor-memory column map (512 columns allocated); slot x adds x * width.
constexpr uint32_t kTmS = 0, kTmP = 128, kTmQ = 192, kTmO = 256;

struct AttnParams {
  const __nv_bfloat16* q;       // raw queries (head dim contiguous)
  long long q_ld, q_hs;         // elements between tokens / heads
  int T, H, W, heads, QT, CAP;
  int Tq;                       // query tokens (dense mode validity)
  int wh, ww;                   // effective window (clamped to the grid)
  int local;                    // 0 dense, 1 local
  int n_qtiles;                 // query tiles per head
  int qtiles_x, qtiles_y;       // local: tiles along x / y per frame pair
  float scale_log2;             // d^-0.5 * log2(e)
  const int* slots;             // [CAP] device
  const int* qpos;              // [QT] device query plane positions (null: no query rotation)
  const float* cos;             // [positions, td/2] temporal rotary table
  const float* sin;
  int td;                       // rotated leading dims of each head (even, <= d)
  __nv_bfloat16* out;           // [Tq, heads, d] (nullable when q_codes is set)
  long long out_ld;             // elements between tokens
  uint8_t* q_codes;             // optional NVFP4 output [Tq, heads*d/2]
  uint8_t* q_sf;                // its swizzled scales (heads*d as K)
  // Tail split: units (query tile, head) [0, n_regular) run whole, one CTA
  // each; every later unit runs as `split` CTAs ("pieces"), each over a
  // contiguous range of its key tiles. A piece writes its unnormalised partial
  // (O, running max m, sum l) to `part`; the last piece of a unit to finish
  // (per-unit arrival counter) merges them into the outputs.
  int n_regular, split;
  float* part;                  // [pieces][kPartFloats]
  int* counters;                // [tail units], zero at launch
};

// Partial of one piece: O as [d/4][128 rows][4] floats (a warp's float4 stores
// of one column quad are contiguous), then m[128] and l[128] (log2 units).
constexpr int kPartO = kD * kBM, kPartFloats = kPartO + 2 * kBM;
constexpr int kMaxSplit = 4;          // pieces per unit
constexpr int kMaxPieces = 160;       // pieces per launch (>= SMs of a B200)

struct SmemLayout {
  static constexpr int kChunk = 128 * 128;           // 128 rows x 128 bytes
  static constexpr int kStagesK = 4;                 // K ring depth
  static constexpr int kStagesV = 3;                 // V ring depth
  static constexpr int offK = 0;                     // kStagesK x 2 chunks
  static constexpr int offV = offK + 2 * kStagesK * kChunk;
  static constexpr int offBar = offV + 2 * kStagesV * kChunk;
  static constexpr int kBars = 24;
  static constexpr int offMisc = offBar + kBars * 8;
  static constexpr int offRed = offMisc + 16 + kMaxPlanes * 4;   // [2 slots][2][128] floats
  static constexpr int kTotal = offRed + 2 * 2 * 128 * 4;
  static constexpr int kAlloc = kTotal;
};

// Key rectangle of one query tile (local mode) and the key tiles per plane.
struct TileIter {
  const AttnParams& p;
  int ry0, ry1, rx0, rx1;       // local-mode key rectangle
  __device__ TileIter(const AttnParams& p_, int qy0, int qx0) : p(p_) {
    if (p.local) {
      const int qy1 = min(qy0 + kLocalQH, p.H) - 1, qx1 = min(qx0 + kLocalQW, p.W) - 1;
      ry0 = min(max(qy0 - p.wh / 2, 0), p.H - p.wh);
      ry1 = min(max(qy1 - p.wh / 2, 0), p.H - p.wh) + p.wh;
      rx0 = min(max(qx0 - p.ww / 2, 0), p.W - p.ww);
      rx1 = min(max(qx1 - p.ww / 2, 0), p.W - p.ww) + p.ww;
    } else {
      ry0 = ry1 = rx0 = rx1 = 0;
    }
  }
  // Tiles per plane: dense = nx runs of 128 tokens; local = nx x ny boxes.
  __device__ int tiles_x() const {
    return !p.local ? (p.T + kBN - 1) / kBN : (rx1 - rx0 + kLocalKW - 1) / kLocalKW;
  }
  __device__ int tiles_y() const { return !p.local ? 1 : (ry1 - ry0 + kLocalKH - 1) / kLocalKH; }
};

// Position of a key tile in the enumeration (visible-plane index, box column,
// box row), advanced incrementally; origin() gives the first token (dense) or
// the box origin (ky0, kx0) (local).
struct TileCursor {
  int plane = 0, tx = 0, ty = 0;
  __device__ void seek(int t, int nx, int ny) {   // the t-th tile of the enumeration
    plane = t / (nx * ny);
    const int r = t - plane * nx * ny;
    ty = r / nx;
    tx = r - ty * nx;
  }
  __device__ void advance(int nx, int ny) {
    if (++tx == nx) {
      tx = 0;
      if (++ty == ny) {
        ty = 0;
        ++plane;
      }
    }
  }
  __device__ void origin(const TileIter& it, int& a, int& b) const {
    if (!it.p.local) {
      a = tx * kBN;
      b = 0;
    } else {
      a = it.ry0 + ty * kLocalKH;
      b = it.rx0 + tx * kLocalKW;
    }
  }
};

// Position in a ring of buffers: stage index and phase parity.
struct Ring {
  int stage = 0;
  uint32_t phase = 0;
  __device__ void advance(int n) {
    if (++stage == n) {
      stage = 0;
      phase ^= 1u;
    }
  }
};

using rc::pack_bf16x2;
using rc::exp2_poly2;
using rc::fast_exp2;
using rc::max3;

// Rotates the bf16 pairs (even, odd) = (lo, hi) half of each word by the
// angle of `pair0 + j` (fp32 math, bf16 rounding of each output).
template <int N>
__device__ __forceinline__ void rotate_pairs(uint32_t (&w)[N], int pair0, int td, const float* cs,
                                             const float* sn) {
#pragma unroll
  for (int j = 0; j < N; ++j) {
    const int pr = pair0 + j;
    if (2 * pr < td) {
      const float e = __uint_as_float(w[j] << 16), o = __uint_as_float(w[j] & 0xffff0000u);
      const float c = rc::ld_in(cs + pr), s = rc::ld_in(sn + pr);
      w[j] = pack_bf16x2(__fsub_rn(__fmul_rn(e, c), __fmul_rn(o, s)),
                         __fadd_rn(__fmul_rn(e, s), __fmul_rn(o, c)));
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1)
attention_kernel(const __grid_constant__ CUtensorMap tm_k,
                 const __grid_constant__ CUtensorMap tm_pv, const __grid_constant__ CUtensorMap tm_cv,
                 const AttnParams p) {
  using L = SmemLayout;
  constexpr int kSK = L::kStagesK, kSV = L::kStagesV;
  // 1024-byte alignment: the 128-byte TMA swizzle pattern repeats every 1024 bytes.
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::offBar);
  uint64_t* q_tmem = bars + 0;             // rotated Q stored in tensor memory (256 arrivals)
  uint64_t* k_full = bars + 1;             // [kSK] K tile landed
  uint64_t* k_empty = k_full + kSK;        // [kSK] both slots' Q K^T read the K stage
  uint64_t* v_full = k_empty + kSK;        // [kSV] V tile landed
  uint64_t* v_empty = v_full + kSV;        // [kSV] both slots' P.V read the V stage
  uint64_t* s_full = v_empty + kSV;        // [2] S_x of the slot's current block finished
  uint64_t* s_free = s_full + 2;           // [2] S_x loaded by the slot's threads (128 arrivals)
  uint64_t* p_full = s_free + 2;           // [2] P_x written (128 arrivals)
  uint64_t* o_done = p_full + 2;           // [2] P_x.V finished
  uint64_t* done = o_done + 2;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::offMisc);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::offMisc + 4);
  int* s_nplanes = reinterpret_cast<int*>(smem + L::offMisc + 8);
  int* s_planes = reinterpret_cast<int*>(smem + L::offMisc + 16);   // kMaxPlanes

  rc::pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Unit (query tile, head) and key-tile piece of this CTA.
  int unit = blockIdx.x, piece = 0, nsplit = 1;
  if (unit >= p.n_regular) {
    const int t = unit - p.n_regular;
    unit = p.n_regular + t / p.split;
    piece = t - (unit - p.n_regular) * p.split;
    nsplit = p.split;
  }
  const int head = unit / p.n_qtiles;
  const int qtile = unit - head * p.n_qtiles;

  // Query tile origin.
  int q_row0 = 0, qf0 = 0, qy0 = 0, qx0 = 0;
  if (!p.local) {
    q_row0 = qtile * kBM;
  } else {
    const int per_pair = p.qtiles_x * p.qtiles_y;
    qf0 = (qtile / per_pair) * 2;
    const int r = qtile % per_pair;
    qy0 = (r / p.qtiles_x) * kLocalQH;
    qx0 = (r % p.qtiles_x) * kLocalQW;
  }

  if (threadIdx.x == 0) {
    sm100::mbar_init(q_tmem, 256);
    for (int s2 = 0; s2 < kSK; ++s2) {
      sm100::mbar_init(&k_full[s2], 1);
      sm100::mbar_init(&k_empty[s2], 1);
    }
    for (int s2 = 0; s2 < kSV; ++s2) {
      sm100::mbar_init(&v_full[s2], 1);
      sm100::mbar_init(&v_empty[s2], 1);
    }
    for (int x = 0; x < 2; ++x) {
      sm100::mbar_init(&s_full[x], 1);
      sm100::mbar_init(&s_free[x], 128);
      sm100::mbar_init(&p_full[x], 128);
      sm100::mbar_init(&o_done[x], 1);
    }
    sm100::mbar_init(done, 1);
    *abort_flag = 0;
    sm100::fence_mbar_init();
  }
  if (warp == 1) {
    sm100::tmem_alloc(tmem_slot, 512);
    sm100::tmem_relinquish();
  }
  // The set-up above (barriers, tensor memory) overlaps the previous kernel's
  // tail; its outputs, and the routing table, are read only from here.
  rc::pdl_wait();
  if (threadIdx.x == 0) {
    // Visible planes: routed past planes (slot >= 0), then the current frames.
    int n = 0;
    for (int i = 0; i < p.CAP; ++i)
      if (p.slots[i] >= 0 && p.slots[i] < p.CAP) s_planes[n++] = i;
    for (int f = 0; f < p.QT; ++f) s_planes[n++] = p.CAP + f;
    *s_nplanes = n;
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int nplanes = *s_nplanes;
  TileIter it(p, qy0, qx0);
  const int nx = it.tiles_x(), ny = it.tiles_y();
  // This CTA's key tiles: [t0, t0 + n_tiles) of the unit's nplanes * nx * ny.
  const int n_all = nplanes * nx * ny;
  const int t0 = piece * n_all / nsplit;
  const int n_tiles = (piece + 1) * n_all / nsplit - t0;

  auto fail = [&](unsigned int site) {
    if (!*abort_flag) rc::device_fail(kKernAttention, site);
    *abort_flag = 1;
  };
  auto wait = [&](uint64_t* bar, uint32_t parity, unsigned int site) -> bool {
    if (sm100::mbar_wait(bar, parity, abort_flag)) return true;
    fail(site);
    return false;
  };

  if (warp == 0) {
    // ----------------------------------------------------------- producer
    if (sm100::elect_one_sync()) {
      // K runs three tiles ahead of V: Q K^T of a tile comes a pipeline step
      // before its P.V, and a K stage frees up as soon as both slots' Q K^T on
      // it finish (slot 1 trails slot 0 by about one block).
      TileCursor kc;
      kc.seek(t0, nx, ny);
      TileCursor vc = kc;
      Ring kr, vr;
      int nk = 0, nv = 0;
      bool ok = true;
      auto load = [&](bool is_k, const TileCursor& c, const Ring& r) -> bool {
        uint64_t* full = is_k ? &k_full[r.stage] : &v_full[r.stage];
        if (!wait(is_k ? &k_empty[r.stage] : &v_empty[r.stage], r.phase ^ 1u, is_k ? 1 : 11)) return false;
        const int plane = s_planes[c.plane];
        int a, b;
        c.origin(it, a, b);
        uint8_t* dst = smem + (is_k ? L::offK : L::offV) + r.stage * 2 * L::kChunk;
        const CUtensorMap* map;
        int src_plane;
        if (is_k) {
          map = &tm_k;
          src_plane = plane;
        } else if (plane < p.CAP) {
          map = &tm_pv;
          src_plane = p.slots[plane];
        } else {
          map = &tm_cv;
          src_plane = plane - p.CAP;
        }
        sm100::mbar_arrive_expect_tx(full, 2 * L::kChunk);
        for (int ch = 0; ch < 2; ++ch) {
          if (!p.local) sm100::tma_load_4d(dst + ch * L::kChunk, map, full, ch * 64, head, a, src_plane);
          else sm100::tma_load_5d(dst + ch * L::kChunk, map, full, ch * 64, head, b, a, src_plane);
        }
        return true;
      };
      constexpr int kLead = kSK - 1;
      for (int i = 0; i < n_tiles + kLead && ok; ++i) {
        if (i < n_tiles) {
          if (!(ok = load(true, kc, kr))) break;
          kc.advance(nx, ny);
          kr.advance(kSK);
          ++nk;
        }
        if (i >= kLead) {
          if (!(ok = load(false, vc, vr))) break;
          vc.advance(nx, ny);
          vr.advance(kSV);
          ++nv;
        }
      }
      // Drain the loads still in flight (at most one ring's depth) before teardown.
      for (int j = max(0, nk - kSK); j < nk; ++j) sm100::mbar_wait(&k_full[j % kSK], (j / kSK) & 1);
      for (int j = max(0, nv - kSV); j < nv; ++j) sm100::mbar_wait(&v_full[j % kSV], (j / kSV) & 1);
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issuer
    if (sm100::elect_one_sync()) {
      constexpr uint32_t idesc_qk = sm100::idesc_bf16(kBM, kSB, 0, 0);
      constexpr uint32_t idesc_pv = sm100::idesc_bf16(kBM, kD, 0, 1);
      bool ok = wait(q_tmem, 0, 2);
      sm100::tc_fence_after();
      // Issue order, per key tile i: S_0(i+1), S_1(i+1), P_0(i).V, P_1(i).V --
      // the order in which their inputs become ready once slot 1 trails slot 0
      // (its first Q K^T waits for slot 0's first P). S_x(i) needs K tile i and
      // S_x(i-1) read; P_x(i).V needs V tile i and P_x(i) written. A ring stage
      // is released after both slots' MMAs on it.
      // Base descriptors of K stage 0 / V stage 0; every MMA adds constant offsets.
      const uint64_t dk0 = sm100::desc_kmajor_sw128(sm100::smem_u32(smem + L::offK));
      const uint64_t dv0 = sm100::desc_mnmajor_sw128(sm100::smem_u32(smem + L::offV), L::kChunk);
      auto issue_s = [&](int x, int i) -> bool {
        if (i > 0 && !wait(&s_free[x], (i - 1) & 1, 5)) return false;
        if (!wait(&k_full[i % kSK], (i / kSK) & 1, 4)) return false;
        sm100::tc_fence_after();
        const uint64_t dk = sm100::desc_add(dk0, (i % kSK) * 2 * L::kChunk + x * kSB * 128);
        const uint32_t ts = tmem + kTmS + x * kSB;
#pragma unroll
        for (int k = 0; k < kD / 16; ++k)
          sm100::mma_f16_ts(ts, tmem + kTmQ + 8 * k, sm100::desc_add(dk, (k >> 2) * L::kChunk + (k & 3) * 32),
                            idesc_qk, k > 0 ? 1u : 0u);
        sm100::tc_commit(&s_full[x]);
        if (x == 1) sm100::tc_commit(&k_empty[i % kSK]);   // both slots done with K tile i
        return true;
      };
      auto issue_pv = [&](int x, int j) -> bool {
        if (!wait(&p_full[x], j & 1, 3)) return false;
        if (x == 0 && !wait(&v_full[j % kSV], (j / kSV) & 1, 12)) return false;
        sm100::tc_fence_after();
        const uint64_t dv = sm100::desc_add(dv0, (j % kSV) * 2 * L::kChunk + x * kSB * 128);
        const uint32_t to = tmem + kTmO + x * kD, tp = tmem + kTmP + x * 32;
#pragma unroll
        for (int k = 0; k < kSB / 16; ++k)
          sm100::mma_f16_ts(to, tp + 8 * k, sm100::desc_add(dv, k * 16 * 128), idesc_pv, (j > 0 || k > 0) ? 1u : 0u);
        sm100::tc_commit(&o_done[x]);
        if (x == 1) sm100::tc_commit(&v_empty[j % kSV]);   // both slots done with V tile j
        return true;
      };
      if (ok && n_tiles > 0) {
        ok = issue_s(0, 0);
        // Slot 1 starts one softmax block behind slot 0: the slots then run out
        // of phase, one in its exp2 loop while the other loads S, reduces and
        // stores P.
        if (ok && n_tiles > 1) ok = wait(&p_full[0], 0, 13);
        ok = ok && issue_s(1, 0);
      }
      for (int i = 0; i < n_tiles && ok; ++i) {
        if (i + 1 < n_tiles) ok = issue_s(0, i + 1) && issue_s(1, i + 1);
        ok = ok && issue_pv(0, i) && issue_pv(1, i);
      }
      sm100::tc_commit(done);
      sm100::mbar_wait(done, 0);
    }
  } else {
    // ----------------------------------------------------------- softmax
    // Slot x = (warp - 2) / 4; the warp's TMEM lane quadrant is warp % 4 and
    // each thread owns one query row; the two warps of a quadrant (one per
    // slot) hold the same rows.
    const int quad = warp & 3;
    const int x = (warp - 2) >> 2;
    const int r = quad * 32 + lane;               // query row within the tile / TMEM lane
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t t_s = tmem + kTmS + x * kSB + lane_off;
    const uint32_t t_p = tmem + kTmP + x * 32 + lane_off;
    int qrow = -1, qf = 0, qy = 0, qx = 0;
    if (!p.local) {
      const int t = q_row0 + r;
      if (t < p.Tq) qrow = t;
      qf = t / p.T;
    } else {
      const int f = qf0 + (r >> 6), yy = qy0 + ((r >> 3) & 7), xx = qx0 + (r & 7);
      if (f < p.QT && yy < p.H && xx < p.W) qrow = f * p.T + yy * p.W + xx;
      qf = f;
      qy = yy;
      qx = xx;
    }
    bool ok = true;
    {
      // Slot x loads head dims [64x, 64x + 64) of its Q row (zeros past the
      // last query) and rotates them (temporal RoPE, fp32 math, bf16 rounding)
      // into tensor memory.
      uint32_t qv[32];
      const uint4* src = qrow >= 0 ? reinterpret_cast<const uint4*>(p.q + (size_t)qrow * p.q_ld +
                                                                      (size_t)head * p.q_hs + x * 64)
                                   : nullptr;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const uint4 w = src ? rc::ld_in(src + u) : make_uint4(0, 0, 0, 0);
        qv[4 * u] = w.x;
        qv[4 * u + 1] = w.y;
        qv[4 * u + 2] = w.z;
        qv[4 * u + 3] = w.w;
      }
      if (p.qpos && qrow >= 0 && x * 64 < p.td) {
        const int pos = p.qpos[qf];
        rotate_pairs(qv, x * 32, p.td, p.cos + (size_t)pos * (p.td >> 1), p.sin + (size_t)pos * (p.td >> 1));
      }
      sm100::tmem_st32(tmem + kTmQ + x * 32 + lane_off, qv);
      sm100::tmem_st_wait();
    }
    sm100::tc_fence_before();
    sm100::mbar_arrive(q_tmem);
    const int top = min(max(qy - p.wh / 2, 0), p.H - p.wh);
    const int left = min(max(qx - p.ww / 2, 0), p.W - p.ww);
    const float scale = p.scale_log2;
    const uint32_t t_o = tmem + kTmO + x * kD + lane_off;
    float m_used = -INFINITY, l = 0.f;
    TileCursor cur;
    cur.seek(t0, nx, ny);
    for (int i = 0; i < n_tiles && ok; ++i, cur.advance(nx, ny)) {
      int a, b;
      cur.origin(it, a, b);
      if (!__all_sync(0xffffffffu, wait(&s_full[x], i & 1, 6))) { ok = false; break; }
      sm100::tc_fence_after();
      float v[64];
      {
        uint32_t r0[16], r1[16], r2[16], r3[16];
        sm100::tmem_ld16(t_s, r0);
        sm100::tmem_ld16(t_s + 16, r1);
        sm100::tmem_ld16(t_s + 32, r2);
        sm100::tmem_ld16(t_s + 48, r3);
        sm100::tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          v[j] = __uint_as_float(r0[j]);
          v[16 + j] = __uint_as_float(r1[j]);
          v[32 + j] = __uint_as_float(r2[j]);
          v[48 + j] = __uint_as_float(r3[j]);
        }
      }
      // S_x is in registers: the MMA may write the slot's next block.
      sm100::tc_fence_before();
      sm100::mbar_arrive(&s_free[x]);
      if (p.local || a + (x + 1) * kSB > p.T) {
        // Validity of the slot's 64 keys as a bit mask: dense = a prefix of
        // the plane; local = 4 box rows x 16 box columns intersected with the window.
        uint64_t mask;
        if (!p.local) {
          const int cnt = min(max(p.T - (a + x * kSB), 0), 64);
          mask = cnt >= 64 ? ~0ull : ((1ull << cnt) - 1ull);
        } else {
          uint32_t cols = 0;
#pragma unroll
          for (int j = 0; j < kLocalKW; ++j) {
            const int kx = b + j;
            cols |= (kx < p.W && kx >= left && kx < left + p.ww) ? (1u << j) : 0u;
          }
          mask = 0;
#pragma unroll
          for (int y = 0; y < 4; ++y) {
            const int ky = a + x * 4 + y;
            if (ky < p.H && ky >= top && ky < top + p.wh) mask |= (uint64_t)cols << (16 * y);
          }
        }
        if (mask != ~0ull) {
#pragma unroll
          for (int j = 0; j < 64; ++j) v[j] = ((mask >> j) & 1ull) ? v[j] : -INFINITY;
        }
      }
      // Row max of the block: 8 independent three-input chains.
      float mx[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mx[k] = max3(v[k], v[k + 8], v[k + 16]);
#pragma unroll
      for (int k = 0; k < 8; ++k) mx[k] = max3(mx[k], v[k + 24], v[k + 32]);
#pragma unroll
      for (int k = 0; k < 8; ++k) mx[k] = max3(mx[k], v[k + 40], v[k + 48]);
#pragma unroll
      for (int k = 0; k < 8; ++k) mx[k] = fmaxf(mx[k], v[k + 56]);
      float mt = max3(max3(mx[0], mx[1], mx[2]), max3(mx[3], mx[4], mx[5]), fmaxf(mx[6], mx[7]));
      mt = mt == -INFINITY ? -INFINITY : mt * scale;   // scale > 0 commutes with max
      // Lazy rescaling: move the reference max only when it grows by > 2^8.
      float corr = 1.0f;
      bool rescale = false;
      if (mt > m_used + kRescaleThreshold || (m_used == -INFINITY && mt > -INFINITY)) {
        corr = m_used == -INFINITY ? 0.f : fast_exp2(m_used - mt);
        rescale = (i > 0) && m_used != -INFINITY;
        m_used = mt;
      }
      const float mref = m_used == -INFINITY ? 0.f : m_used;
      // P = exp2(s * scale - mref), two columns per packed op: three of every
      // four column pairs on the MUFU, the fourth by the FMA-pipe polynomial.
      // Masked scores (-inf) give 0 either way.
      const float2 scale2 = make_float2(scale, scale), nmref2 = make_float2(-mref, -mref);
      float2 sum2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      uint32_t pk[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float2 xv = __ffma2_rn(make_float2(v[2 * j], v[2 * j + 1]), scale2, nmref2);
        float2 e;
        if ((j & 3) == 3) {
          e = exp2_poly2(xv);
        } else {
          e.x = fast_exp2(xv.x);
          e.y = fast_exp2(xv.y);
        }
        sum2[j & 1] = __fadd2_rn(sum2[j & 1], e);
        pk[j] = pack_bf16x2(e.x, e.y);
      }
      l = __fmul_rn(l, corr) + ((sum2[0].x + sum2[0].y) + (sum2[1].x + sum2[1].y));
      // P_x of the previous block was read by its P.V (which also leaves O_x stable).
      if (i > 0 && !__all_sync(0xffffffffu, wait(&o_done[x], (i - 1) & 1, 7))) { ok = false; break; }
      sm100::tc_fence_after();
      sm100::tmem_st32(t_p, pk);
      // O changes only when a row's reference max moved (rare).
      if (__any_sync(0xffffffffu, rescale)) {
        const float f = rescale ? corr : 1.0f;
#pragma unroll 1
        for (int c = 0; c < kD; c += 16) {
          uint32_t w[16];
          sm100::tmem_ld16(t_o + c, w);
          sm100::tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) w[j] = __float_as_uint(__uint_as_float(w[j]) * f);
          sm100::tmem_st16(t_o + c, w);
        }
      }
      sm100::tmem_st_wait();
      sm100::tc_fence_before();
      sm100::mbar_arrive(&p_full[x]);
    }
    // Combine the two slots: out = (O_0 2^(m_0 - m) + O_1 2^(m_1 - m)) /
    // (l_0 2^(m_0 - m) + l_1 2^(m_1 - m)), m = max(m_0, m_1); slot x writes
    // head dims [64x, 64x + 64).
    const bool fin = ok && n_tiles > 0 && __all_sync(0xffffffffu, wait(&o_done[x], (n_tiles - 1) & 1, 8));
    float* red = reinterpret_cast<float*>(smem + L::offRed);   // [slot][m, l][row]
    red[(x * 2 + 0) * 128 + r] = fin ? m_used : NAN;
    red[(x * 2 + 1) * 128 + r] = l;
    sm100::tc_fence_before();
    asm volatile("bar.sync %0, 64;" ::"r"(1 + quad) : "memory");
    sm100::tc_fence_after();
    const float m0 = red[0 * 128 + r], l0 = red[1 * 128 + r];
    const float m1 = red[2 * 128 + r], l1 = red[3 * 128 + r];
    const bool valid = fin && m0 == m0 && m1 == m1;
    const float m = valid ? fmaxf(m0, m1) : -INFINITY;
    const float a0 = (!valid || m0 == -INFINITY) ? 0.f : fast_exp2(m0 - m);
    const float a1 = (!valid || m1 == -INFINITY) ? 0.f : fast_exp2(m1 - m);
    const float lsum = valid ? __fadd_rn(__fmul_rn(l0, a0), __fmul_rn(l1, a1)) : 0.f;
    const uint32_t o0 = tmem + kTmO + lane_off, o1 = tmem + kTmO + kD + lane_off;
    __nv_bfloat16* dst = (qrow >= 0 && p.out) ? p.out + (size_t)qrow * p.out_ld + (size_t)head * kD : nullptr;
    const int katoms = (p.heads * kD) >> 6;
    // Writes output columns [c, c + 16) of this row: bf16, and NVFP4 of the
    // bf16 values (16 columns = one block) for the o-proj GEMM.
    auto emit = [&](int c, const float (&o)[16]) {
      float y[16];
      uint32_t w[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        w[j] = pack_bf16x2(o[2 * j], o[2 * j + 1]);
        y[2 * j] = __uint_as_float(w[j] << 16);
        y[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
      }
      if (dst) {
        reinterpret_cast<uint4*>(dst + c)[0] = make_uint4(w[0], w[1], w[2], w[3]);
        reinterpret_cast<uint4*>(dst + c)[1] = make_uint4(w[4], w[5], w[6], w[7]);
      }
      if (p.q_codes && qrow >= 0) {
        uint8_t sfb;
        uint32_t lo, hi;
        rc::nvfp4_encode16(y, sfb, lo, hi);
        const int kb = (head * kD + c) >> 4;
        *reinterpret_cast<uint2*>(p.q_codes + (size_t)qrow * (p.heads * kD / 2) + (kb << 3)) = make_uint2(lo, hi);
        p.q_sf[rc::sf_offset(qrow, kb, katoms)] = sfb;
      }
    };
    if (nsplit == 1) {
      if (valid) {
        const float inv = 1.0f / fmaxf(lsum, 1e-20f);
        const float2 c0 = make_float2(a0 * inv, a0 * inv), c1 = make_float2(a1 * inv, a1 * inv);
#pragma unroll 1
        for (int c = x * 64; c < x * 64 + 64; c += 16) {
          uint32_t w0[16], w1[16];
          sm100::tmem_ld16(o0 + c, w0);
          sm100::tmem_ld16(o1 + c, w1);
          sm100::tmem_ld_wait();
          float o[16];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float2 s0 = make_float2(__uint_as_float(w0[2 * j]), __uint_as_float(w0[2 * j + 1]));
            const float2 s1 = make_float2(__uint_as_float(w1[2 * j]), __uint_as_float(w1[2 * j + 1]));
            const float2 v = __ffma2_rn(s1, c1, __fmul2_rn(s0, c0));
            o[2 * j] = v.x;
            o[2 * j + 1] = v.y;
          }
          emit(c, o);
        }
      }
    } else {
      // Piece of a split unit: store the partial (O_0 a_0 + O_1 a_1, m, l);
      // the last piece to arrive merges all of the unit's partials:
      // out = sum_q O_q 2^(m_q - M) / sum_q l_q 2^(m_q - M), M = max_q m_q.
      // A piece without keys (or whose rows saw only masked keys) stores
      // m = -inf and no O.
      const int tail_unit = unit - p.n_regular;
      float* mine = p.part + (size_t)(tail_unit * nsplit + piece) * kPartFloats;
      if (m > -INFINITY) {
        const float2 c0 = make_float2(a0, a0), c1 = make_float2(a1, a1);
#pragma unroll 1
        for (int c = x * 64; c < x * 64 + 64; c += 16) {
          uint32_t w0[16], w1[16];
          sm100::tmem_ld16(o0 + c, w0);
          sm100::tmem_ld16(o1 + c, w1);
          sm100::tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float4 v;
            float2 s0 = make_float2(__uint_as_float(w0[4 * j]), __uint_as_float(w0[4 * j + 1]));
            float2 s1 = make_float2(__uint_as_float(w1[4 * j]), __uint_as_float(w1[4 * j + 1]));
            const float2 lo = __ffma2_rn(s1, c1, __fmul2_rn(s0, c0));
            s0 = make_float2(__uint_as_float(w0[4 * j + 2]), __uint_as_float(w0[4 * j + 3]));
            s1 = make_float2(__uint_as_float(w1[4 * j + 2]), __uint_as_float(w1[4 * j + 3]));
            const float2 hi = __ffma2_rn(s1, c1, __fmul2_rn(s0, c0));
            v = make_float4(lo.x, lo.y, hi.x, hi.y);
            __stcg(reinterpret_cast<float4*>(mine) + ((c >> 2) + j) * kBM + r, v);
          }
        }
      }
      if (x == 0) {
        __stcg(mine + kPartO + r, m);
        __stcg(mine + kPartO + kBM + r, lsum);
      }
      // Release the partial, then count the arrival (one thread per CTA).
      __threadfence();
      int* s_last = reinterpret_cast<int*>(smem + L::offMisc + 12);
      asm volatile("bar.sync 5, 256;" ::: "memory");
      if (threadIdx.x == 64) *s_last = atomicAdd(&p.counters[tail_unit], 1) == nsplit - 1;
      asm volatile("bar.sync 5, 256;" ::: "memory");
      if (*s_last) {
        __threadfence();   // acquire: the other pieces' partials are visible from here
        if (threadIdx.x == 64) p.counters[tail_unit] = 0;   // every piece has arrived: ready for the next launch
        const float* base = p.part + (size_t)tail_unit * nsplit * kPartFloats;
        float mq[kMaxSplit], cq[kMaxSplit];
        float mm = -INFINITY;
#pragma unroll
        for (int q = 0; q < kMaxSplit; ++q) {
          mq[q] = q < nsplit ? __ldcg(base + q * kPartFloats + kPartO + r) : -INFINITY;
          mm = fmaxf(mm, mq[q]);
        }
        float ls = 0.f;
#pragma unroll
        for (int q = 0; q < kMaxSplit; ++q) {
          cq[q] = mq[q] == -INFINITY ? 0.f : fast_exp2(mq[q] - mm);
          if (mq[q] > -INFINITY) ls = __fadd_rn(ls, __fmul_rn(__ldcg(base + q * kPartFloats + kPartO + kBM + r), cq[q]));
        }
        const float inv = 1.0f / fmaxf(ls, 1e-20f);
#pragma unroll
        for (int q = 0; q < kMaxSplit; ++q) cq[q] *= inv;
#pragma unroll 1
        for (int c = x * 64; c < x * 64 + 64; c += 16) {
          float o[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) o[j] = 0.f;
#pragma unroll
          for (int q = 0; q < kMaxSplit; ++q) {
            if (mq[q] == -INFINITY) continue;
            const float4* src = reinterpret_cast<const float4*>(base + q * kPartFloats) + (c >> 2) * kBM + r;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float4 v = __ldcg(src + j * kBM);
              o[4 * j] = fmaf(v.x, cq[q], o[4 * j]);
              o[4 * j + 1] = fmaf(v.y, cq[q], o[4 * j + 1]);
              o[4 * j + 2] = fmaf(v.z, cq[q], o[4 * j + 2]);
              o[4 * j + 3] = fmaf(v.w, cq[q], o[4 * j + 3]);
            }
          }
          emit(c, o);
        }
      }
    }
  }
  // Zero the scale bytes of the padding rows (to a multiple of 128) for this head.
  if (p.q_sf && qtile == 0 && piece == 0) {
    const int pm = (p.Tq + 127) / 128 * 128, katoms = (p.heads * kD) >> 6;
    for (int i = threadIdx.x; i < (pm - p.Tq) * 8; i += blockDim.x)
      p.q_sf[rc::sf_offset(p.Tq + i / 8, head * 8 + i % 8, katoms)] = 0;
  }

  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------ pre-pass
struct GatherParams {
  const __nv_bfloat16* ck; long long ck_ld, ck_hs;   // token / head strides (elements)
  const __nv_bfloat16* pk; long long pk_ld, pk_hs;
  const int* slots; const int* ppos; const int* qpos;
  const float* cos; const float* sin;                 // [*, td/2]
  __nv_bfloat16* k_out;                               // [(CAP+QT)*T, heads*d]
  int T, QT, CAP, hd, td, d;
  int* counters;                                      // tail-split arrival counters to zero
  int n_counters;
};

// One CTA = kGatherRows token rows of one plane (blockIdx.y): the plane's
// source (cache slot or current frame) and position are read once per CTA.
// Thread t owns 16-byte vectors t, t + blockDim.x, ... of every row, so its
// head, offset within the head and rotary coefficients are fixed for the CTA;
// a vector's row loads are all in flight before its stores (32-bit offsets
// within the plane). Workspace plane order: routed past planes [0, CAP) (slot
// indirection applied), then the current frames.
constexpr int kGatherRows = 8;

__global__ void rope_gather_kernel(GatherParams g) {
  rc::pdl_trigger();
  rc::pdl_wait();
  if (blockIdx.x == 0 && blockIdx.y == 0)
    for (int i = threadIdx.x; i < g.n_counters; i += blockDim.x) g.counters[i] = 0;
  const int plane = blockIdx.y;
  const __nv_bfloat16* src_base;
  long long ld, hs;
  int pos;
  if (plane < g.CAP) {
    const int slot = g.slots[plane];
    if (slot < 0 || slot >= g.CAP) return;   // not visible: the attention never reads this plane
    src_base = g.pk + (long long)slot * g.T * g.pk_ld;
    ld = g.pk_ld;
    hs = g.pk_hs;
    pos = g.ppos[plane];
  } else {
    const int f = plane - g.CAP;
    src_base = g.ck + (long long)f * g.T * g.ck_ld;
    ld = g.ck_ld;
    hs = g.ck_hs;
    pos = g.qpos[f];
  }
  const int t0 = blockIdx.x * kGatherRows;
  const int rows = min(kGatherRows, g.T - t0);
  __nv_bfloat16* dst_base = g.k_out + ((long long)plane * g.T + t0) * g.hd;
  src_base += (long long)t0 * ld;
  const int vec = g.hd >> 3, dvec = g.d >> 3;
  for (int v = threadIdx.x; v < vec; v += blockDim.x) {
    const int head = v / dvec, dd = (v - head * dvec) * 8;
    const __nv_bfloat16* src = src_base + head * hs + dd;
    __nv_bfloat16* dst = dst_base + v * 8;
    uint4 raw[kGatherRows];
#pragma unroll
    for (int r = 0; r < kGatherRows; ++r)
      if (r < rows) raw[r] = rc::ld_in(reinterpret_cast<const uint4*>(src + r * ld));
    const bool rot = dd < g.td;
    float c[4] = {1.f, 1.f, 1.f, 1.f}, sn[4] = {0.f, 0.f, 0.f, 0.f};
    if (rot) {
      const float* cs = g.cos + (size_t)pos * (g.td >> 1);
      const float* ss = g.sin + (size_t)pos * (g.td >> 1);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int pr = (dd >> 1) + j;
        if (2 * pr < g.td) {
          c[j] = rc::ld_in(cs + pr);
          sn[j] = rc::ld_in(ss + pr);
        }
      }
    }
#pragma unroll
    for (int r = 0; r < kGatherRows; ++r) {
      if (r >= rows) continue;
      uint4 r4 = raw[r];
      if (rot) {
        uint32_t w[4] = {r4.x, r4.y, r4.z, r4.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (2 * ((dd >> 1) + j) < g.td) {
            const float e = __uint_as_float(w[j] << 16), o = __uint_as_float(w[j] & 0xffff0000u);
            w[j] = pack_bf16x2(__fsub_rn(__fmul_rn(e, c[j]), __fmul_rn(o, sn[j])),
                               __fadd_rn(__fmul_rn(e, sn[j]), __fmul_rn(o, c[j])));
          }
        }
        r4 = make_uint4(w[0], w[1], w[2], w[3]);
      }
      *reinterpret_cast<uint4*>(dst + (long long)r * g.hd) = r4;
    }
  }
}

// Key / value views (innermost first): dense (d, heads, tokens, planes) with
// 128-token boxes, local (d, heads, W, H, planes) with 8 x 16 boxes;
// `ld` = elements between tokens, `hs` = between heads.
int make_view(CUtensorMap* m, const void* base, long long ld, long long hs, int heads, int T, int H,
              int W, int planes, bool local, const char* what) {
  if (local) {
    const uint64_t dims[5] = {(uint64_t)kD, (uint64_t)heads, (uint64_t)W, (uint64_t)H, (uint64_t)planes};
    const uint64_t str[4] = {(uint64_t)hs * 2, (uint64_t)ld * 2, (uint64_t)ld * 2 * W,
                             (uint64_t)ld * 2 * T};
    const uint32_t box[5] = {64, 1, kLocalKW, kLocalKH, 1};
    return rc::encode_tmap(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, const_cast<void*>(base), dims, str, box,
                           CU_TENSOR_MAP_SWIZZLE_128B, what);
  }
  const uint64_t dims[4] = {(uint64_t)kD, (uint64_t)heads, (uint64_t)T, (uint64_t)planes};
  const uint64_t str[3] = {(uint64_t)hs * 2, (uint64_t)ld * 2, (uint64_t)ld * 2 * T};
  const uint32_t box[4] = {64, 1, kBN, 1};
  return rc::encode_tmap(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, str, box,
                         CU_TENSOR_MAP_SWIZZLE_128B, what);
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Workspace tail after the rotated K planes: the pieces' partials, then one
// arrival counter per split unit (at most one per piece).
constexpr long long kSplitBytes = (long long)kMaxPieces * kPartFloats * 4 + kMaxPieces * 4;
long long split_offset(long long planes_bytes) { return (planes_bytes + 255) / 256 * 256; }

// Tail split of `units` equal units over the SMs (one CTA per SM at a time):
// the units of the last, partial wave run as `split` pieces each, so that wave
// ends about `split` times sooner. `max_tiles` bounds the key tiles of a unit.
void plan_split(int units, int max_tiles, bool can_split, int& n_regular, int& split) {
  constexpr int cap = kMaxSplit;
  n_regular = units;
  split = 1;
  if (!can_split) return;
  const int sms = rc::sm_count();
  const int tail = units % sms;
  if (!tail) return;
  int s = sms / tail;
  s = s < cap ? s : cap;
  s = s < max_tiles / 4 ? s : max_tiles / 4;   // at least four key tiles per piece
  while (s > 1 && tail * s > kMaxPieces) --s;
  if (s < 2) return;
  n_regular = units - tail;
  split = s;
}

rc::SmemAttrFlags g_attr_flags = {};

int ensure_smem_attr(const char* what) {
  return rc::ensure_smem_attr(g_attr_flags, reinterpret_cast<const void*>(attention_kernel),
                              SmemLayout::kAlloc, what);
}

// ---------------------------------------------------------------------------
// Allocation-free variant. Its scratch (the rotated K planes the attention
// kernel reads) lives in this file-scope device array instead of a caller
// buffer. Every GPU that loads the library holds these 64 MiB until the
// process exits. Host code cannot pass the array's name to a kernel: that name
// is only a host-side handle, so the device address is looked up with
// cudaGetSymbolAddress once per device (with that device current) and cached.
constexpr long long kStaticScratchBytes = 64LL << 20;
static __device__ __align__(256) uint8_t g_attention_scratch[kStaticScratchBytes];
using rc::kMaxDevices;
void* g_scratch_addr[kMaxDevices] = {};   // per-device cache of the array's address
std::mutex g_scratch_mu;

}  // namespace

RC_DEVICE_ERROR_ACCESSOR(attention)

extern "C" {

long long rc_paired_attention_workspace(int B, int QT, int CAP, int H, int W, int heads, int d) {
  if (B <= 0 || QT <= 0 || CAP < 0 || H <= 0 || W <= 0 || heads <= 0 || d <= 0) return -1;
  return split_offset((long long)B * (QT + CAP) * H * W * heads * d * 2) + kSplitBytes;
}

// strides[15]: (batch, token, head) strides in elements of q, ck, cv, pk, pv
// (the head dim itself must be contiguous). slots / positions / rotary tables
// live on the device; the workspace holds the rotated K planes.
int rc_paired_attention(const void* q, const void* ck, const void* cv, const void* pk, const void* pv,
                        const long long* strides, const int* slots, const int* past_positions,
                        const int* query_positions, const float* cos, const float* sin, int B,
                        int QT, int CAP, int H, int W, int heads, int d, int td, int window_h,
                        int window_w, void* workspace, long long workspace_bytes, void* out,
                        long long out_ld, uint8_t* out_codes, uint8_t* out_scales,
                        cudaStream_t stream) {
  const char* what = "rc_paired_attention";
  if (B <= 0 || QT <= 0 || CAP < 0 || H <= 0 || W <= 0 || heads <= 0)
    return rc::set_error(RC_ERR_ARG, "%s: bad geometry", what);
  if (d != kD)
    return rc::set_error(RC_ERR_UNSUPPORTED, "%s: head_dim %d (the tcgen05 kernel supports 128)", what, d);
  if (td < 0 || td > d || td % 2 || window_h <= 0 || window_w <= 0 || CAP > kMaxPlanes - 8 || QT > 8)
    return rc::set_error(RC_ERR_ARG, "%s: bad rotary / window / plane count", what);
  if (!q || !ck || !cv || (!out && !out_codes) || !query_positions || !cos || !sin || !strides ||
      (CAP && (!pk || !pv || !slots || !past_positions)) || (!out_codes != !out_scales))
    return rc::set_error(RC_ERR_ARG, "%s: null pointer", what);
  if (out_codes && ((heads * d) % 64 || reinterpret_cast<uintptr_t>(out_codes) % 8))
    return rc::set_error(RC_ERR_ARG, "%s: NVFP4 output needs heads*d %% 64 == 0 and 8-byte alignment", what);
  const long long need = rc_paired_attention_workspace(B, QT, CAP, H, W, heads, d);
  if (!workspace || workspace_bytes < need || !al16(workspace))
    return rc::set_error(RC_ERR_ARG, "%s: workspace of %lld bytes (16-byte aligned) required", what, need);
  for (int t = 0; t < 5; ++t) {
    if (t >= 3 && !CAP) continue;
    if ((B > 1 && strides[3 * t] % 8) || strides[3 * t + 1] % 8 || strides[3 * t + 2] % 8)
      return rc::set_error(RC_ERR_ARG, "%s: strides must be multiples of 8 elements (16 bytes)", what);
  }
  const void* ptrs[5] = {q, ck, cv, pk, pv};
  for (int i = 0; i < 5; ++i)
    if (ptrs[i] && !al16(ptrs[i])) return rc::set_error(RC_ERR_ARG, "%s: tensors must be 16-byte aligned", what);
  if (out && (!al16(out) || out_ld % 8)) return rc::set_error(RC_ERR_ARG, "%s: output must be 16-byte aligned", what);
  const int T = H * W;
  const int wh = window_h < H ? window_h : H, ww = window_w < W ? window_w : W;
  const bool local = wh < H || ww < W;
  if (local && QT % 2) return rc::set_error(RC_ERR_UNSUPPORTED, "%s: local windows need an even frame count", what);
  if (out_codes && B > 1) return rc::set_error(RC_ERR_UNSUPPORTED, "%s: NVFP4 output needs B == 1", what);
  int r = ensure_smem_attr(what);
  if (r) return r;
  const long long hd = (long long)heads * d;
  const long long per_batch = (long long)(QT + CAP) * T * hd;
  // Split region (reused by every batch element: the launches are stream-ordered).
  uint8_t* split_base = reinterpret_cast<uint8_t*>(workspace) + split_offset((long long)B * per_batch * 2);
  float* part = reinterpret_cast<float*>(split_base);
  int* counters = reinterpret_cast<int*>(split_base + (long long)kMaxPieces * kPartFloats * 4);
  for (int b = 0; b < B; ++b) {
    __nv_bfloat16* ks = reinterpret_cast<__nv_bfloat16*>(workspace) + b * per_batch;
    const __nv_bfloat16* qb = reinterpret_cast<const __nv_bfloat16*>(q) + b * strides[0];
    const __nv_bfloat16* ckb = reinterpret_cast<const __nv_bfloat16*>(ck) + b * strides[3];
    const __nv_bfloat16* cvb = reinterpret_cast<const __nv_bfloat16*>(cv) + b * strides[6];
    const __nv_bfloat16* pkb = CAP ? reinterpret_cast<const __nv_bfloat16*>(pk) + b * strides[9] : nullptr;
    const __nv_bfloat16* pvb = CAP ? reinterpret_cast<const __nv_bfloat16*>(pv) + b * strides[12] : nullptr;
    GatherParams g{ckb, strides[4], strides[5], pkb, strides[10], strides[11], slots, past_positions,
                   query_positions, cos, sin, ks, T, QT, CAP, (int)hd, td, d, counters, kMaxPieces};
    const int vec = (int)(hd / 8);
    const int threads = vec < 512 ? (vec + 31) / 32 * 32 : 512;
    if ((r = rc::check_launch(rc::launch_pdl(rope_gather_kernel, dim3((T + kGatherRows - 1) / kGatherRows, QT + CAP),
                                             dim3(threads), 0, stream, g),
                              "rc_paired_attention(rope)")))
      return r;
    CUtensorMap tk, tpv, tcv;
    if ((r = make_view(&tk, ks, hd, d, heads, T, H, W, CAP + QT, local, what))) return r;
    if ((r = make_view(&tcv, cvb, strides[7], strides[8], heads, T, H, W, QT, local, what))) return r;
    if (CAP) {
      if ((r = make_view(&tpv, pvb, strides[13], strides[14], heads, T, H, W, CAP, local, what))) return r;
    } else {
      tpv = tcv;
    }
    AttnParams p{};
    p.q = qb; p.q_ld = strides[1]; p.q_hs = strides[2];
    p.T = T; p.H = H; p.W = W; p.heads = heads; p.QT = QT; p.CAP = CAP; p.Tq = QT * T;
    p.wh = wh; p.ww = ww; p.local = local;
    p.scale_log2 = (float)(1.0 / sqrt((double)d) * 1.4426950408889634);
    p.slots = slots;
    p.qpos = query_positions;
    p.cos = cos;
    p.sin = sin;
    p.td = td;
    p.out = out ? reinterpret_cast<__nv_bfloat16*>(out) + (long long)b * QT * T * out_ld : nullptr;
    p.out_ld = out_ld;
    p.q_codes = out_codes;
    p.q_sf = out_scales;
    if (!local) {
      p.n_qtiles = (QT * T + kBM - 1) / kBM;
    } else {
      p.qtiles_x = (W + kLocalQW - 1) / kLocalQW;
      p.qtiles_y = (H + kLocalQH - 1) / kLocalQH;
      p.n_qtiles = (QT / 2) * p.qtiles_x * p.qtiles_y;
    }
    // Key tiles of a unit: every visible plane x the tiles of its key rectangle.
    const int per_plane = !local ? (T + kBN - 1) / kBN
                                 : ((wh + kLocalQH - 1 + kLocalKH - 1) / kLocalKH) *
                                       ((ww + kLocalQW - 1 + kLocalKW - 1) / kLocalKW);
    const int units = p.n_qtiles * heads;
    plan_split(units, (CAP + QT) * per_plane, true, p.n_regular, p.split);
    p.part = part;
    p.counters = counters;
    dim3 grid(p.n_regular + (units - p.n_regular) * p.split);
    if ((r = rc::check_launch(
             rc::launch_pdl(attention_kernel, grid, dim3(kThreads), SmemLayout::kAlloc, stream, tk, tpv, tcv, p),
             what)))
      return r;
  }
  return RC_OK;
}

// Unmasked attention without rotary embedding and without cache, e.g. the
// cross-attention of recavsr_infer/runtime/transformer.py:123-128 (queries
// over the 512 precomputed prompt keys). strides[9]: (batch, token, head)
// element strides of q, k, v. Runs the same tcgen05 kernel on the inputs
// directly (no workspace).
long long rc_cross_attention_workspace(void) { return kSplitBytes; }

int rc_cross_attention_ws(const void* q, const void* k, const void* v, const long long* strides, int B,
                          int Nq, int Nk, int heads, int d, void* out, long long out_ld,
                          uint8_t* out_codes, uint8_t* out_scales, void* workspace,
                          long long workspace_bytes, cudaStream_t stream);

int rc_cross_attention(const void* q, const void* k, const void* v, const long long* strides, int B,
                       int Nq, int Nk, int heads, int d, void* out, long long out_ld,
                       uint8_t* out_codes, uint8_t* out_scales, cudaStream_t stream) {
  return rc_cross_attention_ws(q, k, v, strides, B, Nq, Nk, heads, d, out, out_ld, out_codes, out_scales,
                               nullptr, 0, stream);
}

// Same, with a tail-split workspace (rc_cross_attention_workspace() bytes,
// 16-byte aligned, zero-filled before its first use; every successful call
// leaves it zero-filled): the query tiles of the last partial wave run as
// key-range pieces. A null workspace runs every unit whole.
int rc_cross_attention_ws(const void* q, const void* k, const void* v, const long long* strides, int B,
                          int Nq, int Nk, int heads, int d, void* out, long long out_ld,
                          uint8_t* out_codes, uint8_t* out_scales, void* workspace,
                          long long workspace_bytes, cudaStream_t stream) {
  const char* what = "rc_cross_attention";
  if (workspace && (workspace_bytes < kSplitBytes || !al16(workspace)))
    return rc::set_error(RC_ERR_ARG, "%s: workspace of %lld bytes (16-byte aligned) required", what, kSplitBytes);
  if (B <= 0 || Nq < 0 || Nk <= 0 || heads <= 0 || !strides)
    return rc::set_error(RC_ERR_ARG, "%s: bad geometry", what);
  if (d != kD)
    return rc::set_error(RC_ERR_UNSUPPORTED, "%s: head_dim %d (the tcgen05 kernel supports 128)", what, d);
  if (!q || !k || !v || (!out && !out_codes) || (!out_codes != !out_scales))
    return rc::set_error(RC_ERR_ARG, "%s: null pointer", what);
  if (out_codes && (B > 1 || (heads * d) % 64 || reinterpret_cast<uintptr_t>(out_codes) % 8))
    return rc::set_error(RC_ERR_ARG, "%s: NVFP4 output needs B == 1 and heads*d %% 64 == 0", what);
  for (int t = 0; t < 3; ++t)
    if ((B > 1 && strides[3 * t] % 8) || strides[3 * t + 1] % 8 || strides[3 * t + 2] % 8)
      return rc::set_error(RC_ERR_ARG, "%s: strides must be multiples of 8 elements (16 bytes)", what);
  if (!al16(q) || !al16(k) || !al16(v) || (out && (!al16(out) || out_ld % 8)))
    return rc::set_error(RC_ERR_ARG, "%s: tensors must be 16-byte aligned", what);
  if (Nq == 0) return RC_OK;
  int r = ensure_smem_attr(what);
  if (r) return r;
  for (int b = 0; b < B; ++b) {
    const __nv_bfloat16* qb = reinterpret_cast<const __nv_bfloat16*>(q) + b * strides[0];
    const __nv_bfloat16* kb = reinterpret_cast<const __nv_bfloat16*>(k) + b * strides[3];
    const __nv_bfloat16* vb = reinterpret_cast<const __nv_bfloat16*>(v) + b * strides[6];
    CUtensorMap tk, tv;
    if ((r = make_view(&tk, kb, strides[4], strides[5], heads, Nk, 1, Nk, 1, false, what))) return r;
    if ((r = make_view(&tv, vb, strides[7], strides[8], heads, Nk, 1, Nk, 1, false, what))) return r;
    AttnParams p{};
    p.q = qb; p.q_ld = strides[1]; p.q_hs = strides[2];
    p.T = Nk; p.H = 1; p.W = Nk; p.heads = heads; p.QT = 1; p.CAP = 0; p.Tq = Nq;
    p.wh = 1; p.ww = Nk; p.local = 0;
    p.scale_log2 = (float)(1.0 / sqrt((double)d) * 1.4426950408889634);
    p.slots = nullptr;
    p.qpos = nullptr;       // no rotary embedding
    p.td = 0;
    p.out = out ? reinterpret_cast<__nv_bfloat16*>(out) + (long long)b * Nq * out_ld : nullptr;
    p.out_ld = out_ld;
    p.q_codes = out_codes;
    p.q_sf = out_scales;
    p.n_qtiles = (Nq + kBM - 1) / kBM;
    const int units = p.n_qtiles * heads;
    plan_split(units, (Nk + kBN - 1) / kBN, workspace != nullptr, p.n_regular, p.split);
    p.part = reinterpret_cast<float*>(workspace);
    p.counters = workspace ? reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(workspace) +
                                                    (long long)kMaxPieces * kPartFloats * 4)
                           : nullptr;
    dim3 grid(p.n_regular + (units - p.n_regular) * p.split);
    if ((r = rc::check_launch(
             rc::launch_pdl(attention_kernel, grid, dim3(kThreads), SmemLayout::kAlloc, stream, tk, tv, tv, p),
             what)))
      return r;
  }
  return RC_OK;
}

// Same computation as rc_paired_attention, for callers that cannot allocate
// device memory; see include/recavsr_b200.h for the contract.
int rc_paired_attention_static_scratch(const void* q, const void* ck, const void* cv, const void* pk,
                                       const void* pv, const long long* strides, const int* slots,
                                       const int* past_positions, const int* query_positions,
                                       const float* cos, const float* sin, int B, int QT, int CAP,
                                       int H, int W, int heads, int d, int td, int window_h,
                                       int window_w, void* out, long long out_ld, uint8_t* out_codes,
                                       uint8_t* out_scales, cudaStream_t stream) {
  const char* what = "rc_paired_attention_static_scratch";
  const long long need = rc_paired_attention_workspace(B, QT, CAP, H, W, heads, d);
  if (need < 0) return rc::set_error(RC_ERR_ARG, "%s: bad geometry", what);
  if (need > kStaticScratchBytes)
    return rc::set_error(RC_ERR_ARG,
                         "%s: this geometry needs %lld bytes of scratch; the built-in scratch holds %lld "
                         "bytes (use rc_paired_attention with a caller buffer)",
                         what, need, kStaticScratchBytes);
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return rc::set_error(RC_ERR_CUDA, "%s: no usable current device", what);
  void* scratch;
  {
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_addr[dev]) {
      void* addr = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&addr, g_attention_scratch);
      if (e != cudaSuccess || !addr)
        return rc::set_error(RC_ERR_CUDA, "%s: cudaGetSymbolAddress failed: %s", what, cudaGetErrorString(e));
      g_scratch_addr[dev] = addr;
    }
    scratch = g_scratch_addr[dev];
  }
  return rc_paired_attention(q, ck, cv, pk, pv, strides, slots, past_positions, query_positions, cos,
                             sin, B, QT, CAP, H, W, heads, d, td, window_h, window_w, scratch,
                             kStaticScratchBytes, out, out_ld, out_codes, out_scales, stream);
}

}  // extern "C"
