// tcgen05 GEMM for the DiT linears: D[M,N] = epilogue(alpha * A[M,K] . B[N,K]^T + bias).
//
// Operand kinds (both operands K-major, 128-byte rows staged by TMA with the
// 128-byte swizzle, 32 bytes of K per MMA instruction):
//   NVF4 : E2M1 codes (2 per byte) with UE4M3 scales per 16 elements in the
//          128x4 blocked layout of recavsr_infer/runtime/nvfp4.py:64-67 (the
//          same layout the MMA consumes, so scale atoms are copied verbatim:
//          global -> smem with a bulk copy -> TMEM with tcgen05.cp 32x128b.warpx4)
//          -- replaces torch._scaled_mm_v2 in runtime/nvfp4.py:22-39.
//   E4M3 : per-tensor scaled FP8, alpha = scale_a * scale_b read on device
//          -- replaces torch._scaled_mm in runtime/fp8.py:44-47.
//   BF16 : plain bf16 linears.
// Accumulation is fp32 in TMEM. One CTA per SM runs a persistent loop over
// 128 x BN output tiles with warp roles: warp 0 = TMA producer, warp 1 = MMA
// issuer (+ TMEM owner), the other warps = epilogue (TMEM -> registers ->
// global; two or four warps per TMEM lane quadrant, each on an equal share of
// the tile's columns, see epi_warps). With
// BN = 128 the accumulator is double-buffered in TMEM so the epilogue of one
// tile overlaps the MMAs of the next, and the bf16 output tile is staged in
// shared memory and written by TMA stores (residual epilogues TMA-load the
// residual tile into the same boxes first); with BN = 256 the epilogue drains
// the accumulator into registers first and releases it, which gives the same
// overlap with a single accumulator.
// Epilogues fuse the block's follow-up element-wise work:
//   BIAS           out = bf16(acc*alpha + bias)
//   GATED_RESIDUAL h   = bf16(h + bf16(acc*alpha + bias) * gate[n])   (in place)
//   RESIDUAL       h   = bf16(h + bf16(acc*alpha + bias))            (in place)
//   GELU_NVF4      y   = bf16(gelu_tanh(bf16(acc*alpha + bias))), quantized to
//                  NVFP4 (16 columns = one block) for the next linear.
//   SWIGLU (bf16)  each 16-column chunk is 8 gate then 8 up columns (weights
//                  interleaved by the caller): out[:, n/2 ..] =
//                  bf16(bf16(silu(y_gate)) * y_up), y = bf16(acc + bias).
#include <stdlib.h>

#include "sm100.cuh"

namespace {

enum Kind : int { KIND_NVF4 = 0, KIND_E4M3 = 1, KIND_BF16 = 2 };
enum Epi : int { EPI_BIAS = 0, EPI_GATED_RESIDUAL = 1, EPI_RESIDUAL = 2, EPI_GELU_NVF4 = 3, EPI_SWIGLU = 4 };

constexpr int BM = 128;
constexpr int kRowBytes = 128;                     // K bytes per smem row / k-tile
// Epilogue warps per CTA: 4 per TMEM lane quadrant for the GELU + NVFP4
// epilogue (latency-bound math), 2 per quadrant for the light epilogues (more
// warps there only compete with the MMA issuer for its SM sub-partition).
// A CTA pair (PAIR) drains a 128 x 256 accumulator per CTA into registers, so
// it always uses 16 epilogue warps (64 accumulator columns per thread).
template <int EPI, bool PAIR = false>
constexpr int epi_warps() { return (PAIR || EPI == EPI_GELU_NVF4) ? 16 : 8; }
template <int EPI, bool PAIR = false>
constexpr int gemm_threads() { return 64 + 32 * epi_warps<EPI, PAIR>(); }   // producer, MMA, epilogue
constexpr int kSfAtomBytes = 512;                  // 128 rows x 4 scale bytes

template <int KIND>
struct KindTraits;
template <>
struct KindTraits<KIND_NVF4> {
  static constexpr int kElemsPerTile = 256;   // K elements per 128-byte row
  static constexpr bool kScaled = true;
};
template <>
struct KindTraits<KIND_E4M3> {
  static constexpr int kElemsPerTile = 128;
  static constexpr bool kScaled = false;
};
template <>
struct KindTraits<KIND_BF16> {
  static constexpr int kElemsPerTile = 64;
  static constexpr bool kScaled = false;
};

struct GemmParams {
  int M, N, K;
  int k_tiles;                 // ceil(K / elems per tile)
  int m_blocks, n_blocks;
  const uint8_t* sfa;          // NVF4: swizzled scales of A (padded)
  const uint8_t* sfb;          // NVF4: swizzled scales of B
  int sf_katoms;               // ceil(K/64): 4-block atoms along K
  float alpha;
  const float* alpha_ptr_a;    // E4M3: device scale of A (nullable)
  const float* alpha_ptr_b;    // E4M3: device scale of B (nullable)
  const __nv_bfloat16* bias;   // [N] (nullable)
  __nv_bfloat16* out;          // [M, ldo] (BIAS / GELU_NVF4 bf16 out, nullable for GELU)
  long long ldo;
  const float* gate;           // [N] (GATED_RESIDUAL)
  uint8_t* q_codes;            // GELU_NVF4: [M, N/2]
  uint8_t* q_sf;               // GELU_NVF4: swizzled scales (N as K)
  float q_g;                   // GELU_NVF4: global scale
  // Tail split-K: tiles [0, n_regular) run whole; every later tile runs as
  // `split` work units over contiguous k-tile ranges. Each unit stores its fp32
  // partial tile in `part`; the last unit of a tile to finish (per-tile arrival
  // counter) sums the partials in unit order and runs the epilogue.
  int n_regular, split;
  float* part;                 // [units of split tiles][BM x BN] as [BN/4][BM][4]
  int* counters;               // [split tiles]; zero between launches (the merging unit resets it)
  // Tile raster: tiles run in groups of group_m row blocks, row block fastest
  // within a group, then column block. group_m = m_blocks is the plain
  // row-fastest order; a smaller group keeps the operand panels one wave
  // touches few enough to be served from L2 when A and B do not fit in it.
  int group_m;
};

constexpr int kMaxSplit = 4;       // units per split tile
constexpr int kMaxPieces = 160;    // split units per launch (>= SMs of a B200)

// Work unit u of the persistent schedule: tile, k-tile range and the index of
// the unit among the split units (-1 for a whole tile).
struct Unit {
  int tile, kt0, kt1, piece;
};
__device__ __forceinline__ Unit unit_of(const GemmParams& p, int u) {
  if (u < p.n_regular) return {u, 0, p.k_tiles, -1};
  const int t = u - p.n_regular, tt = t / p.split, pc = t - tt * p.split;
  return {p.n_regular + tt, pc * p.k_tiles / p.split, (pc + 1) * p.k_tiles / p.split, t};
}
// Row / column block of a tile index under the grouped raster (a bijection
// onto [0, m_blocks) x [0, n_blocks); the last group may hold fewer rows).
__device__ __forceinline__ void tile_coords(const GemmParams& p, int tile, int& mb, int& nb) {
  const int per_group = p.group_m * p.n_blocks;
  const int g = tile / per_group, r = tile - g * per_group;
  const int gm = min(p.group_m, p.m_blocks - g * p.group_m);
  mb = g * p.group_m + r % gm;
  nb = r / gm;
}

template <int KIND, int BN, int STAGES, bool PAIR = false>
struct Smem {
  static constexpr int kA = BM * kRowBytes;
  static constexpr int kB = (PAIR ? BN / 2 : BN) * kRowBytes;   // a pair splits B's rows between its CTAs
  static constexpr int kSfa = KindTraits<KIND>::kScaled ? 4 * kSfAtomBytes : 0;
  static constexpr int kSfb = KindTraits<KIND>::kScaled ? (BN / 128) * 4 * kSfAtomBytes : 0;
  static constexpr int offA = 0;
  static constexpr int offB = offA + STAGES * kA;
  static constexpr int offSfa = offB + STAGES * kB;
  static constexpr int offSfb = offSfa + STAGES * kSfa;
  // Single-CTA 128-column tiles stage the epilogue's bf16 output (and the
  // residual input) in shared memory: BN / 64 boxes of 128 rows x 128 bytes.
  static constexpr int kOut = (!PAIR && BN == 128) ? BM * BN * 2 : 0;
  static constexpr int offOut = offSfb + STAGES * kSfb;
  static constexpr int offBar = offOut + kOut;
  static constexpr int kBars = 2 * STAGES + 6 + 2;
  static constexpr int kTotal = offBar + kBars * 8 + 16;
  static constexpr int kAlloc = kTotal;
};

// GELU(tanh) of two bf16-valued inputs: 0.5 x (1 + tanh(u)), u = sqrt(2/pi)
// (x + 0.044715 x^3), evaluated as the identical x / (1 + 2^(x (k1 + k3 x^2)))
// with k1 = -2 sqrt(2/pi) log2(e), k3 = 0.044715 k1, on packed fp32 pairs with
// the MUFU exp2 / reciprocal: a few fp32 ulps from tanhf, invisible after the
// bf16 rounding in all but ~1e-3 of elements (one bf16 ulp there). Large
// negative x gives -0 (exp2 overflows to inf, its reciprocal is 0).
__device__ __forceinline__ float2 gelu_tanh2(float2 x) {
  constexpr float k1 = -2.0f * 0.7978845608028654f * 1.4426950408889634f;
  constexpr float k3 = 0.044715f * k1;
  const float2 t = __fmul2_rn(x, x);
  const float2 z = __fmul2_rn(__ffma2_rn(t, make_float2(k3, k3), make_float2(k1, k1)), x);
  float2 e, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e.x) : "f"(z.x));
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e.y) : "f"(z.y));
  const float2 d = __fadd2_rn(e, make_float2(1.0f, 1.0f));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r.x) : "f"(d.x));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r.y) : "f"(d.y));
  return __fmul2_rn(x, r);
}

// bf16x2 word -> the two values as fp32 (low half first).
__device__ __forceinline__ void unpack_bf16x2(uint32_t w, float& a, float& b) {
  a = __uint_as_float(w << 16);
  b = __uint_as_float(w & 0xffff0000u);
}

template <int KIND, int BN, int STAGES, int EPI, bool PAIR>
__global__ void __launch_bounds__(gemm_threads<EPI, PAIR>(), 1)
gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
            const __grid_constant__ CUtensorMap tmap_sfa, const __grid_constant__ CUtensorMap tmap_sfb,
            const __grid_constant__ CUtensorMap tmap_out, const GemmParams p) {
  using S = Smem<KIND, BN, STAGES, PAIR>;
  static_assert(!PAIR || (KIND == KIND_NVF4 && BN == 256), "CTA pairs run 256 x 256 NVFP4 tiles");
  constexpr bool kScaled = KindTraits<KIND>::kScaled;
  constexpr int kMmaPerTile = 4;                     // 4 x 32 bytes of K per 128-byte row
  constexpr int kTmemCols = 512;
  constexpr int kSfaCols = 16;                       // 4 k-steps x 4 columns
  constexpr int kSfbCols = 4 * (BN / 32);            // 4 k-steps x BN/32 columns
  constexpr int kAcc = BN == 128 ? 2 : 1;            // accumulator stages in TMEM
  static_assert(kAcc * BN + 2 * (kSfaCols + kSfbCols) <= kTmemCols, "TMEM budget");

  // 1024-byte alignment: the 128-byte TMA swizzle pattern repeats every 1024 bytes.
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::offBar);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;     // [2]
  uint64_t* acc_empty = acc_full + 2;      // [2]
  uint64_t* done = acc_empty + 2;          // [1]
  volatile int* abort_flag = reinterpret_cast<volatile int*>(done + 2);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 3);
  uint64_t* h_full = done + 5;             // [1] residual tile staged (kStaged)
  // Epilogues that stage their bf16 output tile in shared memory and write it
  // with TMA stores (residual epilogues first TMA-load the residual tile into
  // the same boxes): one 128-byte line per row per box instead of each lane
  // storing its own row, which kept the SM's memory pipeline busy enough to
  // slow the next tile's operand loads and MMAs.
  constexpr bool kStaged = !PAIR && BN == 128 && EPI != EPI_GELU_NVF4;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_units = p.n_regular + (p.m_blocks * p.n_blocks - p.n_regular) * p.split;
  // CTA pair: both CTAs of a cluster walk the same units (256-row tiles); the
  // even one (leader) issues the MMAs, each CTA owns 128 of the rows.
  const uint32_t rank = PAIR ? sm100::cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  const int unit0 = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int unit_step = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      sm100::mbar_init(&full[s], 1);
      sm100::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      sm100::mbar_init(&acc_full[a], 1);
      // A pair's leader counts one arrival per epilogue warp of both CTAs.
      sm100::mbar_init(&acc_empty[a], PAIR ? 2 * epi_warps<EPI, PAIR>() : 32 * epi_warps<EPI, PAIR>());
    }
    sm100::mbar_init(done, 1);
    sm100::mbar_init(h_full, 1);
    *abort_flag = 0;
    sm100::fence_mbar_init();
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      sm100::tmem_alloc_pair(tmem_slot, kTmemCols);
      sm100::tmem_relinquish_pair();
    } else {
      sm100::tmem_alloc(tmem_slot, kTmemCols);
      sm100::tmem_relinquish();
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) sm100::cluster_sync();   // both CTAs' barriers initialised before any remote use
  sm100::tc_fence_after();
  rc::pdl_trigger();
  rc::pdl_wait();   // the previous kernel's outputs (our A operand) are visible from here
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_acc = tmem;                                 // kAcc x BN columns
  const uint32_t tmem_sfa = tmem + kAcc * BN;                     // 2 x kSfaCols
  const uint32_t tmem_sfb = tmem + kAcc * BN + 2 * kSfaCols;      // 2 x kSfbCols

  auto fail = [&](unsigned int site) {
    rc::device_fail(kKernGemmNvf4 + (KIND == KIND_NVF4 ? 0 : 1), site);
    *abort_flag = 1;
  };
  auto wait = [&](uint64_t* bar, uint32_t parity, unsigned int site) -> bool {
    if (sm100::mbar_wait(bar, parity, abort_flag)) return true;
    if (!*abort_flag) fail(site);
    return false;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (sm100::elect_one_sync()) {
      sm100::tma_prefetch_desc(&tmap_a);
      sm100::tma_prefetch_desc(&tmap_b);
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      bool ok = true;
      for (int u = unit0; u < num_units && ok; u += unit_step) {
        const Unit un = unit_of(p, u);
        int mb, nb;
        tile_coords(p, un.tile, mb, nb);
        if constexpr (PAIR) {
          // Each CTA loads its own 128 A rows, its half of B's rows, its A
          // scale atoms and all of B's; the loads count on the leader's full
          // barrier, which the leader arms with both CTAs' bytes.
          constexpr uint32_t kSfBox = 4 * kSfAtomBytes;
          constexpr uint32_t kCtaBytes = S::kA + S::kB + kSfBox + (BN / 128) * kSfBox;
          const int mrow = mb * 2 + (int)rank;
          for (int kt = un.kt0; kt < un.kt1; ++kt) {
            if (!wait(&empty[stage], phase ^ 1, 1)) { ok = false; break; }
            const uint32_t full_leader = sm100::mapa(sm100::smem_u32(&full[stage]), 0);
            if (leader) sm100::mbar_arrive_expect_tx(&full[stage], 2 * kCtaBytes);
            sm100::tma_load_2d_pair(smem + S::offA + stage * S::kA, &tmap_a, full_leader, kt * kRowBytes, mrow * BM);
            sm100::tma_load_2d_pair(smem + S::offB + stage * S::kB, &tmap_b, full_leader, kt * kRowBytes,
                                    nb * BN + (int)rank * (BN / 2));
            sm100::tma_load_3d_pair(smem + S::offSfa + stage * S::kSfa, &tmap_sfa, full_leader, 0, kt * 16, mrow);
            for (int r = 0; r < BN / 128; ++r)
              sm100::tma_load_3d_pair(smem + S::offSfb + stage * S::kSfb + r * kSfBox, &tmap_sfb, full_leader, 0,
                                      kt * 16, nb * (BN / 128) + r);
            ++issued;
            if (++stage == STAGES) { stage = 0; phase ^= 1; }
          }
        } else {
        for (int kt = un.kt0; kt < un.kt1; ++kt) {
          if (!wait(&empty[stage], phase ^ 1, 1)) { ok = false; break; }
          uint32_t bytes = S::kA + S::kB;
          int sfa_bytes = 0, sfb_bytes = 0;
          if constexpr (kScaled) {
            const int atoms = min(4, p.sf_katoms - kt * 4);
            sfa_bytes = atoms * kSfAtomBytes;
            bytes += sfa_bytes;
            for (int r = 0; r < BN / 128; ++r) sfb_bytes += atoms * kSfAtomBytes;
            bytes += sfb_bytes;
          }
          sm100::mbar_arrive_expect_tx(&full[stage], bytes);
          sm100::tma_load_2d(smem + S::offA + stage * S::kA, &tmap_a, &full[stage], kt * kRowBytes, mb * BM);
          sm100::tma_load_2d(smem + S::offB + stage * S::kB, &tmap_b, &full[stage], kt * kRowBytes, nb * BN);
          if constexpr (kScaled) {
            const int atoms = sfa_bytes / kSfAtomBytes;
            const uint8_t* src_a = p.sfa + ((size_t)mb * p.sf_katoms + kt * 4) * kSfAtomBytes;
            asm volatile(
                "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                    sm100::smem_u32(smem + S::offSfa + stage * S::kSfa)),
                "l"(src_a), "r"(sfa_bytes), "r"(sm100::smem_u32(&full[stage]))
                : "memory");
            for (int r = 0; r < BN / 128; ++r) {
              const uint8_t* src_b =
                  p.sfb + ((size_t)(nb * (BN / 128) + r) * p.sf_katoms + kt * 4) * kSfAtomBytes;
              asm volatile(
                  "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                      sm100::smem_u32(smem + S::offSfb + stage * S::kSfb + r * 4 * kSfAtomBytes)),
                  "l"(src_b), "r"(atoms * kSfAtomBytes), "r"(sm100::smem_u32(&full[stage]))
                  : "memory");
            }
            (void)atoms;
          }
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        }
      }
      // Drain: every load this thread issued must land before the CTA exits.
      // (In a pair the loads of both CTAs count on the leader's barriers, so
      // the leader drains for both; the final cluster barrier keeps the other
      // CTA resident until then.)
      if (PAIR && !leader) issued = 0;
      for (int s = 0; s < STAGES && issued > 0; ++s, --issued) {
        if (stage == 0) { stage = STAGES; phase ^= 1; }
        --stage;
        sm100::mbar_wait(&full[stage], phase);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (leader && sm100::elect_one_sync()) {
      uint32_t idesc;
      if constexpr (KIND == KIND_NVF4) idesc = sm100::idesc_nvf4(PAIR ? 2 * BM : BM, BN);
      else if constexpr (KIND == KIND_E4M3) idesc = sm100::idesc_e4m3(BM, BN);
      else idesc = sm100::idesc_bf16(BM, BN, 0, 0);
      int stage = 0;
      uint32_t phase = 0;
      int sf_buf = 0;
      bool ok = true;
      int local = 0;
      // Base descriptors of stage 0; every MMA / scale copy adds constant
      // offsets, which keeps the issuing thread's instruction stream short.
      const uint64_t da0 = sm100::desc_kmajor_sw128(sm100::smem_u32(smem + S::offA));
      const uint64_t db0 = sm100::desc_kmajor_sw128(sm100::smem_u32(smem + S::offB));
      uint64_t dsa0 = 0, dsb0 = 0;
      if constexpr (kScaled) {
        dsa0 = sm100::desc_sf_rows(sm100::smem_u32(smem + S::offSfa));
        dsb0 = sm100::desc_sf_rows(sm100::smem_u32(smem + S::offSfb));
      }
      // One k-step j (0..3) of a k-tile: its scale copies (block-scaled kinds)
      // and its MMA.
      auto copy_sf = [&](int j, uint32_t sfa_t, uint32_t sfb_t, uint64_t dsa, uint64_t dsb) {
        if constexpr (PAIR) {
          sm100::tmem_cp_32x128b_warpx4_pair(sfa_t + 4 * j, sm100::desc_add(dsa, j * kSfAtomBytes));
#pragma unroll
          for (int r = 0; r < BN / 128; ++r)
            sm100::tmem_cp_32x128b_warpx4_pair(sfb_t + j * (BN / 32) + 4 * r,
                                               sm100::desc_add(dsb, (r * 4 + j) * kSfAtomBytes));
        } else {
          sm100::tmem_cp_32x128b_warpx4(sfa_t + 4 * j, sm100::desc_add(dsa, j * kSfAtomBytes));
#pragma unroll
          for (int r = 0; r < BN / 128; ++r)
            sm100::tmem_cp_32x128b_warpx4(sfb_t + j * (BN / 32) + 4 * r,
                                          sm100::desc_add(dsb, (r * 4 + j) * kSfAtomBytes));
        }
      };
      auto mma = [&](int j, uint32_t d_tmem, uint64_t da, uint64_t db, uint32_t sfa_t, uint32_t sfb_t,
                     uint32_t acc) {
        const uint64_t a = sm100::desc_add(da, 32 * j), b = sm100::desc_add(db, 32 * j);
        if constexpr (KIND == KIND_NVF4 && PAIR)
          sm100::mma_nvf4_ss_pair(d_tmem, a, b, idesc, sfa_t + 4 * j, sfb_t + j * (BN / 32), acc);
        else if constexpr (KIND == KIND_NVF4)
          sm100::mma_nvf4_ss(d_tmem, a, b, idesc, sfa_t + 4 * j, sfb_t + j * (BN / 32), acc);
        else if constexpr (KIND == KIND_E4M3)
          sm100::mma_f8f6f4_ss(d_tmem, a, b, idesc, acc);
        else
          sm100::mma_f16_ss(d_tmem, a, b, idesc, acc);
      };
      auto commit = [&](uint64_t* bar) {
        if constexpr (PAIR) sm100::tc_commit_pair(bar);   // arrives in both CTAs
        else sm100::tc_commit(bar);
      };
      for (int u = unit0; u < num_units && ok; u += unit_step, ++local) {
        const Unit un = unit_of(p, u);
        const int as = local % kAcc;
        const uint32_t acc_parity = (uint32_t)((local / kAcc) & 1);
        if (!wait(&acc_empty[as], acc_parity ^ 1, 2)) { ok = false; break; }
        sm100::tc_fence_after();
        const uint32_t d_tmem = tmem_acc + as * BN;
        for (int kt = un.kt0; kt < un.kt1; ++kt) {
          if (!wait(&full[stage], phase, 3)) { ok = false; break; }
          sm100::tc_fence_after();
          const uint64_t da = sm100::desc_add(da0, stage * S::kA);
          const uint64_t db = sm100::desc_add(db0, stage * S::kB);
          uint32_t sfa_t = 0, sfb_t = 0;
          uint64_t dsa = 0, dsb = 0;
          int steps;
          if constexpr (kScaled) {
            steps = min(4, p.sf_katoms - kt * 4);   // K % 64 == 0: one atom per k-step
            sfa_t = tmem_sfa + sf_buf * kSfaCols;
            sfb_t = tmem_sfb + sf_buf * kSfbCols;
            dsa = sm100::desc_add(dsa0, stage * S::kSfa);
            dsb = sm100::desc_add(dsb0, stage * S::kSfb);
            sf_buf ^= 1;
          } else {
            const int rem = (p.K - kt * KindTraits<KIND>::kElemsPerTile) /
                            (KindTraits<KIND>::kElemsPerTile / kMmaPerTile);
            steps = min(kMmaPerTile, rem);
          }
          if (steps == kMmaPerTile) {          // full k-tile: straight-line issue
            if constexpr (kScaled) {
#pragma unroll
              for (int j = 0; j < kMmaPerTile; ++j) copy_sf(j, sfa_t, sfb_t, dsa, dsb);
            }
#pragma unroll
            for (int j = 0; j < kMmaPerTile; ++j) mma(j, d_tmem, da, db, sfa_t, sfb_t, (kt != un.kt0) | (j != 0));
          } else {
            if constexpr (kScaled) {
              for (int j = 0; j < steps; ++j) copy_sf(j, sfa_t, sfb_t, dsa, dsb);
            }
            for (int j = 0; j < steps; ++j) mma(j, d_tmem, da, db, sfa_t, sfb_t, (kt != un.kt0) | (j != 0));
          }
          commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        commit(&acc_full[as]);
      }
      // Make sure no MMA is still writing TMEM when the CTA (pair) tears down.
      commit(done);
      sm100::mbar_wait(done, 0);
    } else if (PAIR && !leader && sm100::elect_one_sync()) {
      // The leader's last commit also arrives here: let it land before leaving.
      sm100::mbar_wait(done, 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Each thread owns one accumulator row (TMEM lane) and a share of the
    // tile's columns. It first drains its columns from TMEM into registers and releases
    // the accumulator, so the next tile's MMAs overlap this tile's epilogue math.
    const int quad = warp & 3;                 // TMEM lane quadrant of this warp
    const int part = (warp - 2) >> 2;          // which share of the tile's columns
    const int row_in_tile = quad * 32 + lane;
    constexpr int kCols = BN / (epi_warps<EPI, PAIR>() / 4);
    int local = 0;
    float alpha = p.alpha;
    if constexpr (KIND == KIND_E4M3) {
      if (p.alpha_ptr_a) alpha = __fmul_rn(alpha, *p.alpha_ptr_a);
      if (p.alpha_ptr_b) alpha = __fmul_rn(alpha, *p.alpha_ptr_b);
    }
    int* s_flags = reinterpret_cast<int*>(done + 4);   // [0] last unit of the tile, [1] a warp failed
    if (threadIdx.x == 64) s_flags[1] = 0;
    asm volatile("bar.sync 1, %0;" ::"r"(32 * epi_warps<EPI, PAIR>()) : "memory");
    // Accumulator release: every epilogue thread has read its columns. In a
    // pair the arrival is relaxed: the MMA needs only the TMEM reads, which
    // tcgen05.wait::ld has completed; a release at cluster scope would first
    // wait for the warp's earlier global stores (the previous tile's outputs)
    // to be performed, with the MMA idle meanwhile.
    auto release = [&](int as) {
      sm100::tc_fence_before();
      if constexpr (PAIR) {
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive_cluster_relaxed(sm100::mapa(sm100::smem_u32(&acc_empty[as]), 0));
      } else {
        sm100::mbar_arrive(&acc_empty[as]);
      }
    };
    constexpr bool kRes = EPI == EPI_GATED_RESIDUAL || EPI == EPI_RESIDUAL;
    // Staged output: BN / 64 boxes of 128 rows x 64 bf16 columns (the SwiGLU
    // epilogue writes half as many columns: one box).
    uint8_t* const out_smem = smem + S::offOut;
    constexpr int kOutBoxes = EPI == EPI_SWIGLU ? BN / 128 : BN / 64;
    static_assert(!kStaged || kCols == 64, "staged epilogue: 64 columns per thread");
    // Address in the staging boxes of bf16 column c (a multiple of 8) of this thread's row.
    auto stage_at = [&](int c) -> uint8_t* {
      return out_smem + (c >> 6) * (BM * 128) + sm100::sw128_offset(row_in_tile, (c & 63) >> 3);
    };
    int h_issued = 0, h_used = 0;               // residual tiles loaded into / consumed from the boxes
    // Residual tile of (mb, nb) into the boxes (one elected thread), once the
    // previous tile's TMA stores have finished reading them.
    auto stage_residual = [&](int mb, int nb) {
      ++h_issued;
      if (threadIdx.x != 64) return;
      sm100::bulk_wait_group_read0();
      sm100::mbar_arrive_expect_tx(h_full, kOutBoxes * BM * 128);
      for (int b = 0; b < kOutBoxes; ++b)
        sm100::tma_load_2d(out_smem + b * (BM * 128), &tmap_out, h_full, nb * BN + 64 * b, mb * BM);
    };
    if constexpr (kStaged) {
      if (threadIdx.x == 64) sm100::tma_prefetch_desc(&tmap_out);
    }
    for (int u = unit0; u < num_units; u += unit_step, ++local) {
      const Unit un = unit_of(p, u);
      int mb, nb;
      tile_coords(p, un.tile, mb, nb);
      if constexpr (PAIR) mb = mb * 2 + (int)rank;   // this CTA's 128-row block of the pair's tile
      const int as = local % kAcc;
      const int row = mb * BM + row_in_tile;
      const bool row_ok = row < p.M;
      const int ncol0 = nb * BN + part * kCols;   // first column of this thread's share
      // Before the accumulator is ready, start this tile's epilogue operand
      // loads (the residual tile into the staging boxes, the bias / gate lines
      // into L1), so their L2 round trips overlap the tile's last MMAs. (A
      // split tile's merging unit loads the residual after the merge.)
      if constexpr (kStaged && kRes)
        if (un.piece < 0) stage_residual(mb, nb);
      if (lane == 0 && ncol0 < p.N) {
        const int ncols = min(kCols, p.N - ncol0);
        if (p.bias)
          for (int c = 0; c < ncols; c += 64) rc::prefetch_l1(p.bias + ncol0 + c);
        if constexpr (EPI == EPI_GATED_RESIDUAL)
          for (int c = 0; c < ncols; c += 32) rc::prefetch_l1(p.gate + ncol0 + c);
      }
      const bool got = __all_sync(0xffffffffu, wait(&acc_full[as], (uint32_t)((local / kAcc) & 1), 4));
      // (Staged epilogues decide at their first barrier, all warps alike.)
      if (!kStaged && !got && (BN != 128 || un.piece < 0)) break;
      const uint32_t t_row = tmem_acc + as * BN + part * kCols + ((uint32_t)(quad * 32) << 16);
      // Per 16-column chunk: the bias / residual / gate operands (zero-filled
      // past the matrix edge).
      struct Ops {
        uint4 b0, b1, h0, h1;
        float4 g[4];
      };
      auto load_ops = [&](int cc) -> Ops {
        Ops o{};
        const int n0 = nb * BN + part * kCols + cc;
        if (!row_ok || n0 >= p.N) return o;
        if (p.bias) {
          const uint4* bp = reinterpret_cast<const uint4*>(p.bias + n0);
          o.b0 = rc::ld_in(bp);
          o.b1 = rc::ld_in(bp + 1);
        }
        if constexpr (kStaged && kRes) {
          o.h0 = *reinterpret_cast<const uint4*>(stage_at(part * kCols + cc));
          o.h1 = *reinterpret_cast<const uint4*>(stage_at(part * kCols + cc + 8));
        } else if constexpr (kRes) {
          const uint4* hp = reinterpret_cast<const uint4*>(p.out + (size_t)row * p.ldo + n0);
          o.h0 = hp[0];
          o.h1 = hp[1];
        }
        if constexpr (EPI == EPI_GATED_RESIDUAL) {
          const float4* gp = reinterpret_cast<const float4*>(p.gate + n0);
#pragma unroll
          for (int j = 0; j < 4; ++j) o.g[j] = rc::ld_in(gp + j);
        }
        return o;
      };
      // Epilogue math of one chunk from its accumulator words; the bf16
      // results go to the staging boxes (kStaged) or straight to global memory.
      auto emit_chunk = [&](int cc, const uint32_t* a16, const Ops& o) {
        const int n0 = nb * BN + part * kCols + cc;
        if (n0 >= p.N) return;
        if (!row_ok) {
          // Padding rows of the next linear's scale atoms must read as zero
          // (a pair's last tile may reach past the padded rows: skip those).
          if constexpr (EPI == EPI_GELU_NVF4)
            if (row < ((p.M + 127) & ~127)) p.q_sf[rc::sf_offset(row, n0 >> 4, (p.N + 63) >> 6)] = 0;
          return;
        }
        // y = bf16(acc * alpha + bias), two columns per packed fp32 op.
        float v[16];
        uint32_t w[8];
        {
          const uint32_t bw[8] = {o.b0.x, o.b0.y, o.b0.z, o.b0.w, o.b1.x, o.b1.y, o.b1.z, o.b1.w};
          const float2 alpha2 = make_float2(alpha, alpha);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            float2 x = __fmul2_rn(make_float2(__uint_as_float(a16[2 * j]), __uint_as_float(a16[2 * j + 1])), alpha2);
            if (p.bias) {
              float2 b;
              unpack_bf16x2(bw[j], b.x, b.y);
              x = __fadd2_rn(x, b);
            }
            w[j] = rc::pack_bf16x2(x.x, x.y);
            unpack_bf16x2(w[j], v[2 * j], v[2 * j + 1]);
          }
        }
        if constexpr (EPI == EPI_SWIGLU) {
          // Columns n0 .. n0 + 7 hold gate, n0 + 8 .. n0 + 15 up for output
          // columns n0 / 2 .. n0 / 2 + 7: bf16(bf16(silu(gate)) * up), SiLU as
          // x / (1 + exp(-x)) in fp32 with the MUFU exp2 (of -x log2 e) and
          // reciprocal, without flush to zero: a few fp32 ulps from the IEEE
          // quotient, which the bf16 rounding hides on all but ~1e-4 of the
          // values (the exact quotient made this epilogue, not the MMA, bound
          // the decoder's K = 512 gate|up GEMMs).
          uint32_t sw[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float s2[2];
#pragma unroll
            for (int k = 0; k < 2; ++k) {
              const float g = v[2 * j + k];
              float e, r;
              asm("ex2.approx.f32 %0, %1;" : "=f"(e) : "f"(__fmul_rn(g, -1.4426950408889634f)));
              asm("rcp.approx.f32 %0, %1;" : "=f"(r) : "f"(__fadd_rn(1.0f, e)));
              const float sg = __bfloat162float(__float2bfloat16_rn(__fmul_rn(g, r)));
              s2[k] = __fmul_rn(sg, v[8 + 2 * j + k]);
            }
            sw[j] = rc::pack_bf16x2(s2[0], s2[1]);
          }
          const uint4 r = make_uint4(sw[0], sw[1], sw[2], sw[3]);
          if constexpr (kStaged) *reinterpret_cast<uint4*>(stage_at((part * kCols + cc) >> 1)) = r;
          else *reinterpret_cast<uint4*>(p.out + (size_t)row * p.ldo + (n0 >> 1)) = r;
          return;
        }
        if constexpr (kRes) {
          const uint32_t hw[8] = {o.h0.x, o.h0.y, o.h0.z, o.h0.w, o.h1.x, o.h1.y, o.h1.z, o.h1.w};
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            float2 h;
            unpack_bf16x2(hw[j], h.x, h.y);
            float2 add = make_float2(v[2 * j], v[2 * j + 1]);
            if constexpr (EPI == EPI_GATED_RESIDUAL) {
              const float4 g4 = o.g[j >> 1];
              add = __fmul2_rn(add, (j & 1) ? make_float2(g4.z, g4.w) : make_float2(g4.x, g4.y));
            }
            const float2 r = __fadd2_rn(h, add);
            w[j] = rc::pack_bf16x2(r.x, r.y);
          }
        }
        if constexpr (EPI == EPI_GELU_NVF4) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float2 g = gelu_tanh2(make_float2(v[2 * j], v[2 * j + 1]));
            w[j] = rc::pack_bf16x2(g.x, g.y);
            unpack_bf16x2(w[j], v[2 * j], v[2 * j + 1]);
          }
          uint8_t sfb;
          uint32_t lo = 0, hi = 0;
          if (p.q_g == 1.0f) {
            rc::nvfp4_encode16(v, sfb, lo, hi);
          } else {
            float amax = 0.f;
#pragma unroll
            for (int j = 0; j < 16; ++j) amax = rc::absmax_nan(amax, v[j]);
            float sc = __fmul_rn(__fdiv_rn(amax, 6.0f), p.q_g);
            sc = sc < 0.001953125f ? 0.001953125f : sc;
            sfb = rc::e4m3_from_float(sc);
            const float sd = rc::e4m3_to_float(sfb);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const uint32_t code = rc::e2m1_code(__fdiv_rn(__fmul_rn(v[j], p.q_g), sd));
              if (j < 8) lo |= code << (4 * j);
              else hi |= code << (4 * (j - 8));
            }
          }
          *reinterpret_cast<uint2*>(p.q_codes + (size_t)row * (p.N >> 1) + (n0 >> 1)) = make_uint2(lo, hi);
          p.q_sf[rc::sf_offset(row, n0 >> 4, (p.N + 63) >> 6)] = sfb;
          if (!p.out) return;
        }
        if constexpr (kStaged) {
          *reinterpret_cast<uint4*>(stage_at(part * kCols + cc)) = make_uint4(w[0], w[1], w[2], w[3]);
          *reinterpret_cast<uint4*>(stage_at(part * kCols + cc + 8)) = make_uint4(w[4], w[5], w[6], w[7]);
        } else {
          uint4* dst = reinterpret_cast<uint4*>(p.out + (size_t)row * p.ldo + n0);
          dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
          dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
        }
      };
      if (BN == 128 && un.piece >= 0) {   // (the host splits 128-column tiles only)
        // Split tile: store this unit's partial, count the arrival. The last
        // unit to arrive sums every unit's partial in unit order (per chunk,
        // all units' words loaded together) into its own accumulator in TMEM
        // and then runs the whole-tile epilogue below on it.
        float4* mine = reinterpret_cast<float4*>(p.part + (size_t)un.piece * (BM * BN));
        if (got) {
          sm100::tc_fence_after();
#pragma unroll
          for (int cc = 0; cc < kCols; cc += 16) {
            uint32_t a16[16];
            sm100::tmem_ld16(t_row + cc, a16);
            sm100::tmem_ld_wait();
#pragma unroll
            for (int c = 0; c < 16; c += 4)
              __stcg(mine + ((part * kCols + cc + c) >> 2) * BM + row_in_tile,
                     make_float4(__uint_as_float(a16[c]), __uint_as_float(a16[c + 1]),
                                 __uint_as_float(a16[c + 2]), __uint_as_float(a16[c + 3])));
          }
        } else if (lane == 0) {
          s_flags[1] = 1;
        }
        __threadfence();
        asm volatile("bar.sync 1, %0;" ::"r"(32 * epi_warps<EPI, PAIR>()) : "memory");
        const int tail_tile = un.tile - p.n_regular;
        if (threadIdx.x == 64)
          s_flags[0] = !s_flags[1] && atomicAdd(&p.counters[tail_tile], 1) == p.split - 1;
        asm volatile("bar.sync 1, %0;" ::"r"(32 * epi_warps<EPI, PAIR>()) : "memory");
        if (s_flags[1]) break;
        if (!s_flags[0]) {
          release(as);                             // accumulator free: next tile may start
          continue;
        }
        if constexpr (kStaged && kRes) stage_residual(mb, nb);
        __threadfence();   // acquire: the other units' partials are visible from here
        const float4* src = reinterpret_cast<const float4*>(p.part + (size_t)tail_tile * p.split * (BM * BN)) +
                            ((part * kCols) >> 2) * BM + row_in_tile;
#pragma unroll 1
        for (int cc = 0; cc < kCols; cc += 16) {
          float4 q4[kMaxSplit][4];
#pragma unroll
          for (int q = 0; q < kMaxSplit; ++q)
#pragma unroll
            for (int i = 0; i < 4; ++i)
              if (q < p.split) q4[q][i] = __ldcg(src + (size_t)q * (BM * BN / 4) + ((cc >> 2) + i) * BM);
          uint32_t a16[16];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            float4 sum = q4[0][i];
#pragma unroll
            for (int q = 1; q < kMaxSplit; ++q) {
              if (q < p.split) {
                sum.x += q4[q][i].x; sum.y += q4[q][i].y; sum.z += q4[q][i].z; sum.w += q4[q][i].w;
              }
            }
            a16[4 * i] = __float_as_uint(sum.x);
            a16[4 * i + 1] = __float_as_uint(sum.y);
            a16[4 * i + 2] = __float_as_uint(sum.z);
            a16[4 * i + 3] = __float_as_uint(sum.w);
          }
          sm100::tmem_st16(t_row + cc, a16);
        }
        sm100::tmem_st_wait();
        if (threadIdx.x == 64) p.counters[tail_tile] = 0;   // ready for the next launch
      }
      if constexpr (kStaged) {
        // Staged epilogue: the boxes are free (residual: its tile has landed
        // in them; otherwise: the previous tile's stores have read them), then
        // per 16-column chunk a TMEM load, the operands, the math into the
        // boxes; the accumulator is released after the last chunk (with two
        // accumulator stages the MMA needs it again only two tiles later) and
        // one thread stores the boxes.
        bool ok = got;
        if constexpr (kRes) {
          ++h_used;
          ok = wait(h_full, (uint32_t)((h_used - 1) & 1), 5) && ok;
        } else {
          if (threadIdx.x == 64) sm100::bulk_wait_group_read0();
        }
        if (!sm100::bar_and(1, 32 * epi_warps<EPI, PAIR>(), ok)) break;
        sm100::tc_fence_after();
#pragma unroll
        for (int cc = 0; cc < kCols; cc += 16) {
          uint32_t a16[16];
          sm100::tmem_ld16(t_row + cc, a16);
          const Ops o = load_ops(cc);
          sm100::tmem_ld_wait();
          emit_chunk(cc, a16, o);
        }
        release(as);                             // accumulator free
        sm100::fence_proxy_async_smem();         // the boxes' writes, visible to the TMA stores
        asm volatile("bar.sync 1, %0;" ::"r"(32 * epi_warps<EPI, PAIR>()) : "memory");
        if (threadIdx.x == 64) {
          const int x0 = EPI == EPI_SWIGLU ? nb * (BN / 2) : nb * BN;
          const int n_out = EPI == EPI_SWIGLU ? p.N / 2 : p.N;
          for (int b = 0; b < kOutBoxes; ++b)
            if (x0 + 64 * b < n_out) sm100::tma_store_2d(&tmap_out, out_smem + b * (BM * 128), x0 + 64 * b, mb * BM);
          sm100::bulk_commit_group();
        }
      } else {
        // Other epilogues: drain the tile's columns from TMEM into registers
        // and release the accumulator first, so the next tile's MMAs overlap
        // this tile's epilogue math (essential with a single accumulator).
        uint32_t acc[kCols];
        sm100::tc_fence_after();
#pragma unroll
        for (int c = 0; c < kCols; c += 16)
          sm100::tmem_ld16(t_row + c, *reinterpret_cast<uint32_t(*)[16]>(&acc[c]));
        sm100::tmem_ld_wait();
        release(as);                             // accumulator free: next tile may start
#pragma unroll
        for (int cc = 0; cc < kCols; cc += 16) emit_chunk(cc, &acc[cc], load_ops(cc));
      }
    }
    if constexpr (kStaged) {
      if (threadIdx.x == 64) {
        // A residual tile still in flight (a wait gave up) lands before the
        // CTA leaves; every TMA store has completed.
        if (h_issued > 0) sm100::mbar_wait(h_full, (uint32_t)((h_issued - 1) & 1));
        sm100::bulk_wait_group0();
      }
    }
  }

  sm100::tc_fence_before();
  __syncthreads();
  // A pair's CTAs leave together: the leader's MMAs read the other CTA's
  // shared memory and write its tensor memory until its `done` wait returns.
  if constexpr (PAIR) sm100::cluster_sync();
  if (warp == 1) {
    __syncwarp();
    sm100::tc_fence_after();
    if constexpr (PAIR) sm100::tmem_dealloc_pair(tmem, kTmemCols);
    else sm100::tmem_dealloc(tmem, kTmemCols);
  }
}

// Tail split-K. The persistent CTAs take the tiles round-robin, so the last
// `tiles % sms` tiles form a partial wave; those run as `split` k-ranges each,
// so that wave ends about `split` times sooner. Storing and merging the fp32
// partials costs about as much as 4-8 k-tiles of MMA, so every range keeps at
// least 8 k-tiles (measured on M = 1760: the split gains 3% on ffn_down,
// K = 14336, and loses 16% on o-proj, K = 3072, which therefore stays whole).
void plan_split(int tiles, int sms, bool can_split, GemmParams& p) {
  constexpr int cap = kMaxSplit;
  p.n_regular = tiles;
  p.split = 1;
  const int tail = tiles % sms;
  if (!can_split || !tail) return;
  int s = sms / tail;
  s = s < cap ? s : cap;
  s = s < p.k_tiles / 8 ? s : p.k_tiles / 8;
  while (s > 1 && tail * s > kMaxPieces) --s;
  if (s < 2) return;
  p.n_regular = tiles - tail;
  p.split = s;
}

constexpr long long kSplitPartBytes = (long long)kMaxPieces * BM * 128 * 4;
constexpr long long kSplitWorkspaceBytes = kSplitPartBytes + kMaxPieces * 4;

// The tensor maps of a launch: A and B operand rows, (CTA pairs only) A's
// and B's scale atoms viewed as [row blocks][4 * k atoms][128 B], and (staged
// epilogues only) the bf16 output as boxes of 128 rows x 64 columns.
struct Maps {
  CUtensorMap a, b, sfa, sfb, out;
};

template <int KIND, int BN, int STAGES, int EPI, bool PAIR>
int launch(const Maps& m, const GemmParams& p, cudaStream_t stream, const char* what) {
  using S = Smem<KIND, BN, STAGES, PAIR>;
  auto kern = gemm_kernel<KIND, BN, STAGES, EPI, PAIR>;
  static rc::SmemAttrFlags attr_flags = {};
  if (const int st = rc::ensure_smem_attr(attr_flags, reinterpret_cast<const void*>(kern), S::kAlloc, what))
    return st;
  const int tiles = p.m_blocks * p.n_blocks;
  const int sms = rc::sm_count();
  GemmParams q = p;
  if constexpr (PAIR) {
    // One 2-CTA cluster per pair of SMs, each walking whole 256 x 256 tiles.
    q.n_regular = tiles;
    q.split = 1;
    const int pairs = tiles < sms / 2 ? tiles : sms / 2;
    return rc::check_launch(rc::launch_pdl_cluster(kern, dim3(2 * pairs), dim3(gemm_threads<EPI, PAIR>()), S::kAlloc,
                                                   stream, 2, m.a, m.b, m.sfa, m.sfb, m.a, q),
                            what);
  }
  plan_split(tiles, sms, BN == 128 && p.part != nullptr, q);
  const int units = q.n_regular + (tiles - q.n_regular) * q.split;
  const int grid = units < sms ? units : sms;
  return rc::check_launch(rc::launch_pdl(kern, grid, dim3(gemm_threads<EPI>()), S::kAlloc, stream, m.a, m.b,
                                         m.a, m.b, m.out, q), what);
}

template <int KIND, int BN, int STAGES, bool PAIR = false>
int dispatch_epi(int epi, const Maps& m, const GemmParams& p, cudaStream_t stream, const char* what) {
  switch (epi) {
    case EPI_BIAS: return launch<KIND, BN, STAGES, EPI_BIAS, PAIR>(m, p, stream, what);
    case EPI_GATED_RESIDUAL: return launch<KIND, BN, STAGES, EPI_GATED_RESIDUAL, PAIR>(m, p, stream, what);
    case EPI_RESIDUAL: return launch<KIND, BN, STAGES, EPI_RESIDUAL, PAIR>(m, p, stream, what);
    case EPI_GELU_NVF4: return launch<KIND, BN, STAGES, EPI_GELU_NVF4, PAIR>(m, p, stream, what);
    case EPI_SWIGLU:
      if constexpr (KIND == KIND_BF16 && !PAIR) return launch<KIND, BN, STAGES, EPI_SWIGLU, PAIR>(m, p, stream, what);
      break;
  }
  return rc::set_error(RC_ERR_ARG, "%s: unknown epilogue %d", what, epi);
}

// Whether an NVFP4 GEMM runs on CTA pairs (256 x 256 tiles over two SMs):
// one MMA-issuing thread feeds 256 rows, each SM stages only half of B and a
// quarter less operand data per FLOP crosses L2. Measured (B200, same box,
// A/B against the single-CTA kernel; per-k-tile timestamps of the issuing
// thread): a pair keeps its tensor pipes busy to within ~15% once a tile has
// many k-tiles (7040 x 3072 x 14336: 118.7 vs 145.0 us, 5.2 PFLOP/s), but its
// single 256-column accumulator (two would not fit tensor memory beside the
// scale factors) is handed to the epilogue with the tensor pipe idle for
// ~2-3k cycles per tile, which a 12-k-tile tile (K = 3072) does not amortize,
// and 256 x 256 tiles quantize coarsely onto 74 SM pairs. So pairs take the
// GEMMs with at least two waves of pair tiles and a long K or a wide N
// (ffn_up 1760 x 14336 x 3072: 44.7 vs 46.2 us; M = 3520 / 7040 with K or
// N = 14336: 7-18% faster); the N = 3072 linears at M = 1760 (o-proj, cross,
// ffn_down with its tail split) and QKV stay on single CTAs.
bool gemm_use_pair(int kind, int M, int N, int K) {
  if (kind != KIND_NVF4 || N % 256) return false;
  const long long pair_tiles = (long long)((M + 255) / 256) * (N / 256);
  return pair_tiles >= rc::sm_count() && (K >= 8192 || N >= 12288);
}

// Tile width. 128 x 256 tiles (single accumulator, register-drained
// epilogue) move a third less operand data per FLOP than 128 x 128 tiles, but
// the 128 x 128 tiles overlap each tile's epilogue with the next tile's
// mainloop (double-buffered accumulator) and quantize better onto 148 SMs.
bool gemm_prefer_wide(int epi, int M, int N, int K) {
  if (N % 256) return false;
  // Measured on M = 1760 (same box, A/B): the 256-column tile wins only for
  // the wide GELU + NVFP4 GEMM (ffn_up, N = 14336: 45.9 vs 48.0 us), where
  // halving the MMA and scale-copy instructions per FLOP outweighs the
  // exposed epilogue; it loses on o-proj / ffn_down (wave quantization at
  // N = 3072) and ties on QKV.
  (void)M; (void)K;
  return epi == EPI_GELU_NVF4 && N >= 12288;
}
// bf16 GEMMs with a long K and at least four waves of 128 x 256 tiles (the LQ
// projector's first convolution, 14080 x 2048 x 27648).
bool gemm_prefer_wide_bf16(int epi, int M, int N, int K) {
  if (N % 256 || epi == EPI_SWIGLU) return false;
  const long long wide_tiles = (long long)((M + 127) / 128) * (N / 256);
  return K >= 16384 && wide_tiles >= 4LL * rc::sm_count();
}

// Shared argument checks + tensor maps; `elem_bytes_x2` = 2 * bytes/element
// (1 for fp4, 2 for fp8, 4 for bf16).
int run_gemm(int kind, int epi, const void* a, const void* b, int M, int N, int K,
             GemmParams& p, cudaStream_t stream, const char* what) {
  const int ebx2 = kind == KIND_NVF4 ? 1 : (kind == KIND_E4M3 ? 2 : 4);
  if (M < 0 || N <= 0 || K <= 0 || N % 16)
    return rc::set_error(RC_ERR_ARG, "%s: bad shape M=%d N=%d K=%d (N %% 16 == 0)", what, M, N, K);
  if (K % 64)
    return rc::set_error(RC_ERR_UNSUPPORTED, "%s: K must be a multiple of 64 (K=%d)", what, K);
  if (!a || !b) return rc::set_error(RC_ERR_ARG, "%s: null operand", what);
  if (epi == EPI_SWIGLU && (kind != KIND_BF16 || N % 16))
    return rc::set_error(RC_ERR_ARG, "%s: the SwiGLU epilogue is bf16-only", what);
  if (epi != EPI_GELU_NVF4 || p.out) {
    if (!p.out || p.ldo < (epi == EPI_SWIGLU ? N / 2 : N) || p.ldo % 8 || reinterpret_cast<uintptr_t>(p.out) % 16)
      return rc::set_error(RC_ERR_ARG, "%s: output rows must be 16-byte aligned (ldo=%lld)", what, p.ldo);
  }
  if (epi == EPI_GATED_RESIDUAL && !p.gate) return rc::set_error(RC_ERR_ARG, "%s: gate missing", what);
  if (epi == EPI_GELU_NVF4 && (!p.q_codes || !p.q_sf || N % 64))
    return rc::set_error(RC_ERR_ARG, "%s: GELU/NVFP4 epilogue needs codes, scales and N %% 64 == 0", what);
  if (M == 0) return RC_OK;
  const uint64_t row_bytes = (uint64_t)K * ebx2 / 2;
  Maps maps;
  const uint64_t da[2] = {row_bytes, (uint64_t)M}, db[2] = {row_bytes, (uint64_t)N};
  const uint64_t sa[1] = {row_bytes}, sb[1] = {row_bytes};
  const bool pair = gemm_use_pair(kind, M, N, K);
  const bool wide = !pair && (kind == KIND_BF16 ? gemm_prefer_wide_bf16(epi, M, N, K) : gemm_prefer_wide(epi, M, N, K));
  const bool staged = !pair && !wide && epi != EPI_GELU_NVF4;   // the kernel's kStaged
  const uint32_t boxa[2] = {128, 128}, boxb[2] = {128, (uint32_t)(wide ? 256 : 128)};
  int r = rc::encode_tmap(&maps.a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(a), da, sa, boxa,
                          CU_TENSOR_MAP_SWIZZLE_128B, what);
  if (r) return r;
  r = rc::encode_tmap(&maps.b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(b), db, sb, boxb,
                      CU_TENSOR_MAP_SWIZZLE_128B, what);
  if (r) return r;
  maps.out = maps.a;
  if (staged) {
    // bf16 output [M, N] (SwiGLU: N / 2) with row stride ldo, 128 x 64 boxes.
    const uint64_t dout[2] = {(uint64_t)(epi == EPI_SWIGLU ? N / 2 : N), (uint64_t)M};
    const uint64_t sout[1] = {(uint64_t)p.ldo * 2};
    const uint32_t boxo[2] = {64, 128};
    r = rc::encode_tmap(&maps.out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p.out, dout, sout, boxo,
                        CU_TENSOR_MAP_SWIZZLE_128B, what);
    if (r) return r;
  }
  if (pair) {
    // Scale atoms (512 B = 128 rows x 4 k-blocks) as 128-byte lines: one box
    // is a k-tile's 4 atoms of one 128-row block; lines past the last atom
    // (K % 256 != 0) and row blocks past the matrix read as zero.
    const uint64_t katoms = (uint64_t)(K + 63) / 64;
    const uint64_t dsa[3] = {128, 4 * katoms, (uint64_t)(M + 127) / 128};
    const uint64_t dsb[3] = {128, 4 * katoms, (uint64_t)(N + 127) / 128};
    const uint64_t ss[2] = {128, katoms * kSfAtomBytes};
    const uint32_t box[3] = {128, 16, 1};
    r = rc::encode_tmap(&maps.sfa, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t*>(p.sfa), dsa, ss, box,
                        CU_TENSOR_MAP_SWIZZLE_NONE, what);
    if (r) return r;
    r = rc::encode_tmap(&maps.sfb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t*>(p.sfb), dsb, ss, box,
                        CU_TENSOR_MAP_SWIZZLE_NONE, what);
    if (r) return r;
  }
  const int ept = kind == KIND_NVF4 ? 256 : (kind == KIND_E4M3 ? 128 : 64);
  p.M = M;
  p.N = N;
  p.K = K;
  p.k_tiles = (K + ept - 1) / ept;
  p.m_blocks = (M + BM - 1) / BM;
  p.sf_katoms = (K + 63) / 64;
  // Operands beyond half the 126 MB L2 (the LQ projector's convolutions, K up
  // to 73728): groups of 12 row blocks, so a wave of 148 tiles reads ~12 A
  // and ~13 B panels instead of up to 110 A panels (measured on the
  // 14080 x 2048 x 27648 bf16 GEMM: 9.8 GB of DRAM reads for 0.9 GB of
  // operands in row-fastest order). Smaller GEMMs keep row-fastest order.
  const double operand_bytes = ((double)M + (double)N) * (double)row_bytes;
  p.group_m = operand_bytes > 64e6 && p.m_blocks > 12 ? 12 : p.m_blocks;
  if (pair) {
    p.m_blocks = (M + 2 * BM - 1) / (2 * BM);     // 256-row tiles
    p.n_blocks = N / 256;
    p.group_m = operand_bytes > 64e6 && p.m_blocks > 6 ? 6 : p.m_blocks;
    p.part = nullptr;                             // no split-K on pairs
    return dispatch_epi<KIND_NVF4, 256, 5, true>(epi, maps, p, stream, what);
  }
  if (wide) {
    p.n_blocks = N / 256;
    if (kind == KIND_NVF4) return dispatch_epi<KIND_NVF4, 256, 4>(epi, maps, p, stream, what);
    if (kind == KIND_E4M3) return dispatch_epi<KIND_E4M3, 256, 4>(epi, maps, p, stream, what);
    return dispatch_epi<KIND_BF16, 256, 4>(epi, maps, p, stream, what);
  }
  p.n_blocks = (N + 127) / 128;
  if (kind == KIND_NVF4) return dispatch_epi<KIND_NVF4, 128, 5>(epi, maps, p, stream, what);
  if (kind == KIND_E4M3) return dispatch_epi<KIND_E4M3, 128, 6>(epi, maps, p, stream, what);
  return dispatch_epi<KIND_BF16, 128, 6>(epi, maps, p, stream, what);
}

}  // namespace

RC_DEVICE_ERROR_ACCESSOR(gemm_nvf4)
unsigned int rc_take_device_error_gemm_fp8() { return 0; }

extern "C" {

// NVFP4 block-scaled GEMM (see file header). a_codes [M, K/2], b_codes
// [N, K/2] (row-major, K-major), scales in the swizzled layout produced by
// rc_nvfp4_quantize. epilogue: 0 bias, 1 gated residual (out += y * gate),
// 2 residual (out += y), 3 GELU + NVFP4 requantize into q_codes/q_scales.
int rc_nvfp4_gemm(const uint8_t* a_codes, const uint8_t* a_scales, const uint8_t* b_codes,
                  const uint8_t* b_scales, const void* bias, int M, int N, int K, float alpha,
                  int epilogue, void* out, long long ldo, const float* gate, uint8_t* q_codes,
                  uint8_t* q_scales, float q_global_scale, cudaStream_t stream) {
  if (!a_scales || !b_scales) return rc::set_error(RC_ERR_ARG, "rc_nvfp4_gemm: null scales");
  if (reinterpret_cast<uintptr_t>(a_scales) % 16 || reinterpret_cast<uintptr_t>(b_scales) % 16)
    return rc::set_error(RC_ERR_ARG, "rc_nvfp4_gemm: scale buffers must be 16-byte aligned");
  GemmParams p{};
  p.sfa = a_scales;
  p.sfb = b_scales;
  p.alpha = alpha;
  p.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  p.gate = gate;
  p.q_codes = q_codes;
  p.q_sf = q_scales;
  p.q_g = q_global_scale;
  return run_gemm(KIND_NVF4, epilogue, a_codes, b_codes, M, N, K, p, stream, "rc_nvfp4_gemm");
}

long long rc_gemm_split_workspace(void) { return kSplitWorkspaceBytes; }

// rc_nvfp4_gemm with a split-K workspace (rc_gemm_split_workspace() bytes,
// 16-byte aligned, zero-filled before its first use; every successful call
// leaves it zero-filled). Calls that share a workspace must be ordered on one
// stream.
int rc_nvfp4_gemm_ws(const uint8_t* a_codes, const uint8_t* a_scales, const uint8_t* b_codes,
                     const uint8_t* b_scales, const void* bias, int M, int N, int K, float alpha,
                     int epilogue, void* out, long long ldo, const float* gate, uint8_t* q_codes,
                     uint8_t* q_scales, float q_global_scale, void* workspace, long long workspace_bytes,
                     cudaStream_t stream) {
  const char* what = "rc_nvfp4_gemm_ws";
  if (!a_scales || !b_scales) return rc::set_error(RC_ERR_ARG, "%s: null scales", what);
  if (reinterpret_cast<uintptr_t>(a_scales) % 16 || reinterpret_cast<uintptr_t>(b_scales) % 16)
    return rc::set_error(RC_ERR_ARG, "%s: scale buffers must be 16-byte aligned", what);
  if (!workspace || workspace_bytes < kSplitWorkspaceBytes || reinterpret_cast<uintptr_t>(workspace) % 16)
    return rc::set_error(RC_ERR_ARG, "%s: workspace of %lld bytes (16-byte aligned) required", what,
                         kSplitWorkspaceBytes);
  GemmParams p{};
  p.sfa = a_scales;
  p.sfb = b_scales;
  p.alpha = alpha;
  p.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  p.gate = gate;
  p.q_codes = q_codes;
  p.q_sf = q_scales;
  p.q_g = q_global_scale;
  p.part = reinterpret_cast<float*>(workspace);
  p.counters = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(workspace) + kSplitPartBytes);
  return run_gemm(KIND_NVF4, epilogue, a_codes, b_codes, M, N, K, p, stream, what);
}

// Per-tensor FP8 (E4M3) GEMM: alpha * scale_a * scale_b * A.B^T + bias.
int rc_fp8_gemm(const uint8_t* a, const float* scale_a, const uint8_t* b, const float* scale_b,
                const void* bias, int M, int N, int K, float alpha, int epilogue, void* out,
                long long ldo, const float* gate, cudaStream_t stream) {
  GemmParams p{};
  p.alpha = alpha;
  p.alpha_ptr_a = scale_a;
  p.alpha_ptr_b = scale_b;
  p.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  p.gate = gate;
  if (epilogue == EPI_GELU_NVF4) return rc::set_error(RC_ERR_ARG, "rc_fp8_gemm: GELU/NVFP4 epilogue is NVFP4-only");
  return run_gemm(KIND_E4M3, epilogue, a, b, M, N, K, p, stream, "rc_fp8_gemm");
}

// bf16 GEMM with the same epilogues (plain nn.Linear path).
int rc_bf16_gemm(const void* a, const void* b, const void* bias, int M, int N, int K, int epilogue,
                 void* out, long long ldo, const float* gate, cudaStream_t stream) {
  GemmParams p{};
  p.alpha = 1.0f;
  p.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  p.gate = gate;
  if (epilogue == EPI_GELU_NVF4) return rc::set_error(RC_ERR_ARG, "rc_bf16_gemm: GELU/NVFP4 epilogue is NVFP4-only");
  return run_gemm(KIND_BF16, epilogue, a, b, M, N, K, p, stream, "rc_bf16_gemm");
}

// rc_bf16_gemm with the split-K workspace of rc_nvfp4_gemm_ws (same size,
// alignment, zero-fill and ordering rules): the tiles of the partial last
// wave run as k-ranges (the LQ projector's K = 73728 convolution GEMM).
int rc_bf16_gemm_ws(const void* a, const void* b, const void* bias, int M, int N, int K, int epilogue,
                    void* out, long long ldo, const float* gate, void* workspace, long long workspace_bytes,
                    cudaStream_t stream) {
  const char* what = "rc_bf16_gemm_ws";
  if (!workspace || workspace_bytes < kSplitWorkspaceBytes || reinterpret_cast<uintptr_t>(workspace) % 16)
    return rc::set_error(RC_ERR_ARG, "%s: workspace of %lld bytes (16-byte aligned) required", what,
                         kSplitWorkspaceBytes);
  GemmParams p{};
  p.alpha = 1.0f;
  p.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  p.gate = gate;
  p.part = reinterpret_cast<float*>(workspace);
  p.counters = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(workspace) + kSplitPartBytes);
  if (epilogue == EPI_GELU_NVF4) return rc::set_error(RC_ERR_ARG, "%s: GELU/NVFP4 epilogue is NVFP4-only", what);
  return run_gemm(KIND_BF16, epilogue, a, b, M, N, K, p, stream, what);
}

}  // extern "C"
