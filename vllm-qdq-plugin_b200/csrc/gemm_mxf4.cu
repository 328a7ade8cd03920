// Block-scaled MXFP4 GEMM on the sm_100a tensor cores:
//   C[M, N] (bf16) = A[M, K] . W[N, K]^T (+ bias[N]),  fp32 accumulation,
// where A and W are E2M1 codes (two per byte, element 2j in the low nibble)
// with one E8M0 scale per 32 consecutive K elements.
//
// This replaces "MXFP4 QDQ of the activation, then Marlin's bf16 x
// dequantised-FP4 GEMM" (reference: src/vllm_qdq_plugin/patch.py:51-57 +
// vllm/_custom_ops.py:1277 marlin_gemm): because QDQ'd activations are exactly
// MXFP4-representable, the activation can be fed to kind::mxf4 MMAs as codes
// + scales, and every product is the same exact value Marlin forms.
//
// Kernel structure: persistent, one CTA per SM walking 128 x 256 output
// tiles (tile t: m block t % num_m, n block t / num_m, so the CTAs in flight
// share W tiles in L2), 10 warps:
//   warp 0 / one lane   TMA producer: A and W code tiles (128-byte swizzle)
//                       and their scale-factor chunks (bulk copies) into a
//                       4-stage shared-memory ring; it runs ahead across tiles
//   warp 1 / one lane   MMA issuer: waits until the epilogue has drained the
//                       TMEM accumulator, then per stage tcgen05.cp scale
//                       factors smem -> TMEM and 4 x tcgen05.mma.kind::mxf4
//                       (K = 64 each); tcgen05.commit frees the stage and,
//                       after the last stage, hands the tile to the epilogue
//   warps 2-9           epilogue: warp w reads TMEM lanes 32 (w % 4) .. +31 and
//                       columns 128 ((w - 2) / 4) .. +127 into registers, frees
//                       the accumulator (the next tile's MMAs start), then adds
//                       the bias, converts and stores while they run
//
// Scale factors use the tcgen05 "tiled" layout in global memory (see
// qdq_sf_tile): rows are grouped by 128 and K-scales by 4 into 512-byte
// chunks, chunk (rb, kc) at ((rb * kchunks) + kc) * 512, byte
// (r % 32) * 16 + ((r / 32) % 4) * 4 + (ks % 4).  Rows are padded to a
// multiple of 128 and the K-scale count to one stage's worth (8 for E8M0 per
// 32, 16 for E4M3 per 16).
//
// NVFP4 variant (kNV): E2M1 codes with one UE4M3 scale per 16 K elements and
// an fp32 tensor scale per operand, on tcgen05.mma.kind::mxf4nvf4.block16.
// A K-256 stage then carries four scale chunks per 128-row block instead of
// two, each MMA (K = 64) reads one whole chunk column, and the epilogue
// multiplies the fp32 accumulator by alpha = w_global_scale / a_global_scale
// (vLLM's conventions: the activation is dequantised as code * s / gs_a, the
// weight as code * s * gs_w).
#include <cmath>
#include <cstring>

#include "sm100.cuh"

namespace qdqb200 {
namespace {

using namespace sm100;

constexpr int BM = 128;             // rows of A per tile (UMMA M)
constexpr int BN = 256;             // rows of W per tile (UMMA N)
constexpr int BK = 256;             // K elements per stage
constexpr int BKB = BK / 2;         // bytes per row per stage (128: one swizzle row)
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BKB;   // 16 KB
constexpr int B_BYTES = BN * BKB;   // 32 KB
constexpr int TMEM_COLS = 512;
constexpr int ACC_COL = 0;          // 256 fp32 columns
constexpr int SFA_COL = 256;        // 8 columns (2 K-chunks x 4), NVFP4 16
constexpr int SFB_COL = 272;        // 16 columns (2 K-chunks x 2 row blocks x 4), NVFP4 32
constexpr int EPI_WARPS = 8;
constexpr int THREADS = 32 * (2 + EPI_WARPS);

// Per-format stage geometry: 512-byte scale chunks per 128-row block and
// stage (CPS), stage bytes, and the ring depths that fit 227 KB.
template <bool kNV>
struct Fmt {
  static constexpr int CPS = kNV ? 4 : 2;
  static constexpr int SFA = CPS * 512;        // 128 rows of A
  static constexpr int SFB = 2 * CPS * 512;    // 256 rows of W
  static constexpr int STAGE = BM * (BK / 2) + BN * (BK / 2) + SFA + SFB;
  static constexpr uint32_t IDESC1 = idesc_mxf4(BM, BN, !kNV);
  static constexpr uint32_t IDESC2 = idesc_mxf4(256, BN, !kNV);
};

struct __align__(8) Barriers {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t acc_full;    // MMA -> epilogue: the tile's accumulator is complete
  uint64_t acc_empty;   // epilogue -> MMA: the accumulator has been read out
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

template <bool kNV>
constexpr size_t smem_bytes() { return 1024 + STAGES * Fmt<kNV>::STAGE + sizeof(Barriers); }
static_assert(smem_bytes<true>() <= 227 * 1024, "NVFP4 GEMM shared memory");

// The 4 MMAs (K = 64 each) of one K-256 stage.  MXFP4: scale chunk j = kk / 2
// holds the stage's K-scales 4j..4j+3, of which the MMA reads the pair sf_id.
// NVFP4: chunk kk holds the MMA's four K-scales.  sfb: chunk j of W rows
// 0-127 at column 8 j, of rows 128-255 at 8 j + 4.
template <bool kNV, bool kPair>
__device__ __forceinline__ void issue_stage(uint32_t acc, uint64_t da, uint64_t db, uint32_t sfa, uint32_t sfb,
                                            bool first) {
  constexpr uint32_t idesc = kPair ? Fmt<kNV>::IDESC2 : Fmt<kNV>::IDESC1;
#pragma unroll
  for (int kk = 0; kk < BK / 64; ++kk) {
    const uint32_t acc_on = (!first || kk != 0) ? 1u : 0u;
    // K step of 64 E2M1 = 32 bytes inside the 128-byte swizzled row
    const uint64_t a = da + ((kk * 32) >> 4), b = db + ((kk * 32) >> 4);
    if constexpr (kNV) {
      if constexpr (kPair) mma_nvf4_pair(acc, a, b, idesc, sfa + 4 * kk, sfb + 8 * kk, acc_on);
      else mma_nvf4(acc, a, b, idesc, sfa + 4 * kk, sfb + 8 * kk, acc_on);
    } else {
      const uint32_t j = kk >> 1, sf_id = (kk & 1) * 2;
      const uint32_t id = idesc_with_sf_ids(idesc, sf_id, sf_id);
      if constexpr (kPair) mma_mxf4_pair(acc, a, b, id, (sfa + 4 * j) | (sf_id << 30), (sfb + 8 * j) | (sf_id << 30), acc_on);
      else mma_mxf4(acc, a, b, id, (sfa + 4 * j) | (sf_id << 30), (sfb + 8 * j) | (sf_id << 30), acc_on);
    }
  }
}

// Output element type: bf16 (kF16 = false) or fp16; bias has the same type.
template <bool kF16>
struct OutT {
  using T = __nv_bfloat16;
  __device__ static float load(const T* p) { return __bfloat162float(*p); }
  __device__ static uint32_t pack(float a, float b) { return pack_bf16x2(a, b); }
  __device__ static T one(float a) { return __float2bfloat16_rn(a); }
};
template <>
struct OutT<true> {
  using T = __half;
  __device__ static float load(const T* p) { return __half2float(*p); }
  __device__ static uint32_t pack(float a, float b) { return pack_f16x2(a, b); }
  __device__ static T one(float a) { return __float2half_rn(a); }
};

template <bool kF16, bool kNV>
__global__ void __launch_bounds__(THREADS, 1)
mxf4_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                 const uint8_t* __restrict__ sfa, const uint8_t* __restrict__ sfb,
                 const void* __restrict__ bias_v, void* __restrict__ C_v, int M, int N,
                 int K, int64_t ldc, int kchunks, const float* __restrict__ a_gs, float w_gs, int* status) {
  using O = OutT<kF16>;
  using F = Fmt<kNV>;
  constexpr int STAGE_BYTES = F::STAGE, SFA_BYTES = F::SFA, CPS = F::CPS;
  using T = typename O::T;
  const T* bias = static_cast<const T*>(bias_v);
  T* C = static_cast<T*>(C_v);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Barriers* bars = reinterpret_cast<Barriers*>(smem + STAGES * STAGE_BYTES);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (M + BM - 1) / BM;
  const int num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kt = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    mbar_init(&bars->acc_full, 1);
    mbar_init(&bars->acc_empty, 32 * EPI_WARPS);
    mbar_init(&bars->drain, 1);
    bars->abort = 0;
    fence_barrier_init();
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
  }
  if (warp == 0) {
    tmem_alloc(&bars->tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0) {
    // ---------------- producer
    if (elect_one()) {
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        const int m_blk = tile % num_m, n_blk = tile / num_m;
        const bool second_rb = (n_blk * 2 + 1) * 128 < N;
        for (int kt = 0; kt < num_kt; ++kt, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(&bars->empty[s], ((it / STAGES) & 1) ^ 1, status, 0x101)) {
            bars->abort = 1;
            ok = false;
            break;
          }
          if (*(volatile int*)&bars->abort) { ok = false; break; }
          uint8_t* st = smem + s * STAGE_BYTES;
          mbar_arrive_expect_tx(&bars->full[s], A_BYTES + B_BYTES + SFA_BYTES + (second_rb ? 2 : 1) * CPS * 512);
          tma_load_2d(st, &tmap_a, kt * BKB, m_blk * BM, &bars->full[s]);
          tma_load_2d(st + A_BYTES, &tmap_b, kt * BKB, n_blk * BN, &bars->full[s]);
          bulk_load(st + A_BYTES + B_BYTES, sfa + (static_cast<int64_t>(m_blk) * kchunks + CPS * kt) * 512,
                    CPS * 512, &bars->full[s]);
          bulk_load(st + A_BYTES + B_BYTES + SFA_BYTES,
                    sfb + (static_cast<int64_t>(2 * n_blk) * kchunks + CPS * kt) * 512, CPS * 512, &bars->full[s]);
          if (second_rb)
            bulk_load(st + A_BYTES + B_BYTES + SFA_BYTES + CPS * 512,
                      sfb + (static_cast<int64_t>(2 * n_blk + 1) * kchunks + CPS * kt) * 512, CPS * 512,
                      &bars->full[s]);
        }
      }
      // Drain: every issued copy has landed before the CTA may exit.
      for (int j = (it > STAGES ? it - STAGES : 0); j < it; ++j)
        mbar_wait(&bars->full[j % STAGES], (j / STAGES) & 1, status, 0x102);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (elect_one()) {
      int it = 0, i = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x, ++i) {
        // the epilogue has read the previous tile's accumulator out of TMEM
        if (i > 0 && !mbar_wait(&bars->acc_empty, (i - 1) & 1, status, 0x202)) { ok = false; break; }
        tc_fence_after();
        for (int kt = 0; kt < num_kt; ++kt, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(&bars->full[s], (it / STAGES) & 1, status, 0x201)) { ok = false; break; }
          if (*(volatile int*)&bars->abort) { ok = false; break; }
          tc_fence_after();
          uint8_t* st = smem + s * STAGE_BYTES;
          const uint8_t* sa = st + A_BYTES + B_BYTES;
          const uint8_t* sb = sa + SFA_BYTES;
          // scale factors: chunk j of each 128-row block (MXFP4: K-scales
          // 4j..4j+3 of this stage; NVFP4: the four K-scales of MMA j)
#pragma unroll
          for (int j = 0; j < CPS; ++j) {
            tmem_cp_sf(tmem + SFA_COL + 4 * j, smem_desc_sf(sa + 512 * j));
            tmem_cp_sf(tmem + SFB_COL + 8 * j, smem_desc_sf(sb + 512 * j));                // rows 0-127
            tmem_cp_sf(tmem + SFB_COL + 8 * j + 4, smem_desc_sf(sb + CPS * 512 + 512 * j));  // rows 128-255
          }
          issue_stage<kNV, false>(tmem + ACC_COL, smem_desc_sw128(st), smem_desc_sw128(st + A_BYTES),
                                  tmem + SFA_COL, tmem + SFB_COL, kt == 0);
          tc_commit(&bars->empty[s]);
        }
        if (!ok) break;
        tc_commit(&bars->acc_full);
      }
      if (!ok) bars->abort = 1;
      // every issued tcgen05 op has completed before TMEM is released
      tc_commit(&bars->drain);
      mbar_wait(&bars->drain, 0, status, 0x203);
    }
  } else {
    // ---------------- epilogue: TMEM lanes 32 (warp % 4).. = tile rows, columns 128 h ..
    const int q = warp & 3, h = (warp - 2) >> 2;
    const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16) + ACC_COL + h * 128;
    const float alpha = kNV ? w_gs / *a_gs : 1.0f;
    bool ok = true;
    int i = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++i) {
      const int m_blk = tile % num_m, n_blk = tile / num_m;
      if (ok) ok = mbar_wait(&bars->acc_full, i & 1, status, 0x301);
      ok = __all_sync(0xffffffffu, ok);  // the TMEM loads below are warp-collective
      tc_fence_after();
      uint32_t r[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(taddr + 32 * c, r[c]);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&bars->acc_empty);  // the next tile's MMAs may overwrite the accumulator
      if (!ok || *(volatile int*)&bars->abort || num_kt == 0) continue;
      const int row = m_blk * BM + q * 32 + lane;
      if (row >= M) continue;
      const int n0 = n_blk * BN + h * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int ncols = min(32, N - n0 - 32 * c);
        if (ncols <= 0) continue;
        T* crow = C + static_cast<int64_t>(row) * ldc + n0 + 32 * c;
        float v[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] = kNV ? __uint_as_float(r[c][e]) * alpha : __uint_as_float(r[c][e]);
        if (bias != nullptr) {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (e < ncols) v[e] += O::load(bias + n0 + 32 * c + e);
        }
        if (ncols == 32 && (reinterpret_cast<uintptr_t>(crow) & 15) == 0) {
          uint4* dst = reinterpret_cast<uint4*>(crow);
#pragma unroll
          for (int w4 = 0; w4 < 4; ++w4)
            dst[w4] = make_uint4(O::pack(v[8 * w4 + 0], v[8 * w4 + 1]), O::pack(v[8 * w4 + 2], v[8 * w4 + 3]),
                                 O::pack(v[8 * w4 + 4], v[8 * w4 + 5]), O::pack(v[8 * w4 + 6], v[8 * w4 + 7]));
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (e < ncols) crow[e] = O::one(v[e]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// CTA-pair variant: a cluster of two CTAs computes 256 x 256 tiles with
// tcgen05.mma.cta_group::2 (M = 256: CTA r holds A rows [128 r, 128 r + 128)
// and W rows [128 r, 128 r + 128) of the tile, and its TMEM the accumulator
// of its 128 rows over all 256 columns).  Per SM and K stage this streams
// 32 KB of codes instead of 48 KB, so the ring holds 6 stages.
//   rank 0 and 1, warp 0   TMA producer of the CTA's own halves and scale
//                          chunks (W scales for all 256 columns, which each
//                          CTA's MMA half reads), completing on the leader's
//                          full barrier
//   rank 0, warp 1         MMA issuer for the pair; commits arrive on both
//                          CTAs' barriers
//   warps 2-9              epilogue of the CTA's 128 rows
// Scale chunks arrive by TMA (2-D maps of 512-byte rows) so that they, too,
// complete on the leader's barrier.
// ---------------------------------------------------------------------------
constexpr int P_STAGES_MAX = 6;
constexpr int P_A = 128 * BKB;      // 16 KB: the CTA's 128 A rows
constexpr int P_B = 128 * BKB;      // 16 KB: the CTA's 128 W rows
// Per format: the CTA's 128 A rows' and all 256 W rows' scale chunks; MXFP4
// stages are 35 KB (6 in the ring), NVFP4 stages 38 KB (5).
template <bool kNV>
struct PairFmt {
  static constexpr int STAGES = kNV ? 5 : 6;
  static constexpr int SFA = Fmt<kNV>::SFA;
  static constexpr int SFB = Fmt<kNV>::SFB;
  static constexpr int STAGE = P_A + P_B + SFA + SFB;
  static constexpr int TX = 2 * STAGE;  // bytes both CTAs land on the leader's barrier per stage
};

struct __align__(8) PairBars {
  uint64_t full[P_STAGES_MAX];   // leader: both CTAs' stage bytes landed
  uint64_t empty[P_STAGES_MAX];  // each CTA: the pair's MMAs on the stage completed
  uint64_t acc_full;             // each CTA: its accumulator half is complete
  uint64_t acc_empty;            // leader: both CTAs' epilogues read their halves (512 arrivals)
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};
template <bool kNV>
constexpr size_t pair_smem_bytes() { return 1024 + PairFmt<kNV>::STAGES * PairFmt<kNV>::STAGE + sizeof(PairBars); }
static_assert(pair_smem_bytes<false>() <= 227 * 1024, "pair GEMM shared memory");
static_assert(pair_smem_bytes<true>() <= 227 * 1024, "NVFP4 pair GEMM shared memory");

template <bool kF16, bool kNV>
__global__ void __launch_bounds__(THREADS, 1)
mxf4_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                      const __grid_constant__ CUtensorMap tmap_sfa, const __grid_constant__ CUtensorMap tmap_sfb,
                      const void* __restrict__ bias_v, void* __restrict__ C_v, int M, int N, int K, int64_t ldc,
                      int kchunks, const float* __restrict__ a_gs, float w_gs, int* status) {
  using O = OutT<kF16>;
  using PF = PairFmt<kNV>;
  constexpr int P_STAGES = PF::STAGES, P_STAGE = PF::STAGE, P_SFA = PF::SFA, P_TX = PF::TX;
  constexpr int CPS = Fmt<kNV>::CPS;
  using T = typename O::T;
  const T* bias = static_cast<const T*>(bias_v);
  T* C = static_cast<T*>(C_v);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  PairBars* bars = reinterpret_cast<PairBars*>(smem + P_STAGES * P_STAGE);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int pair = blockIdx.x >> 1, num_pairs = gridDim.x >> 1;
  const int num_m = (M + 255) / 256;
  const int num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kt = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    mbar_init(&bars->acc_full, 1);
    mbar_init(&bars->acc_empty, 2 * 32 * EPI_WARPS);
    mbar_init(&bars->drain, 1);
    bars->abort = 0;
    fence_barrier_init();
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
    prefetch_tmap(&tmap_sfa);
    prefetch_tmap(&tmap_sfb);
  }
  if (warp == 0) {
    tmem_alloc_pair(&bars->tmem_base, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers are initialised and the TMEM is allocated
  tc_fence_after();
  pdl_launch_dependents();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0) {
    // ---------------- producer (both CTAs): own halves, landing on the leader's barrier
    if (elect_one()) {
      // A stage's weight loads (W codes and both W scale chunks) and its
      // activation loads (codes and scales: the previous kernel on the stream
      // writes them).
      auto load_w = [&](int s, int n_blk, int kt) {
        uint8_t* st = smem + s * P_STAGE;
        const uint32_t full0 = cluster_addr(&bars->full[s], 0);
        if (rank == 0) mbar_arrive_expect_tx(&bars->full[s], P_TX);
        tma_load_2d_pair(st + P_A, &tmap_b, kt * BKB, n_blk * BN + static_cast<int>(rank) * 128, full0);
        tma_load_2d_pair(st + P_A + P_B + P_SFA, &tmap_sfb, 0, (n_blk * 2) * kchunks + CPS * kt, full0);
        tma_load_2d_pair(st + P_A + P_B + P_SFA + CPS * 512, &tmap_sfb, 0, (n_blk * 2 + 1) * kchunks + CPS * kt,
                         full0);
      };
      auto load_a = [&](int s, int m_blk, int kt) {
        uint8_t* st = smem + s * P_STAGE;
        const uint32_t full0 = cluster_addr(&bars->full[s], 0);
        tma_load_2d_pair(st, &tmap_a, kt * BKB, m_blk * 256 + static_cast<int>(rank) * 128, full0);
        tma_load_2d_pair(st + P_A + P_B, &tmap_sfa, 0, (m_blk * 2 + static_cast<int>(rank)) * kchunks + CPS * kt,
                         full0);
      };
      // The first ring of the first tile's weight loads goes out before
      // griddepcontrol.wait (programmatic dependent launch): it overlaps the
      // tail of the kernel that produces the activation codes.
      const int pre = pair < num_tiles ? min(P_STAGES, num_kt) : 0;
      for (int kt = 0; kt < pre; ++kt) load_w(kt, pair / num_m, kt);
      pdl_wait();
      for (int kt = 0; kt < pre; ++kt) load_a(kt, pair % num_m, kt);
      int it = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < num_tiles; tile += num_pairs) {
        const int m_blk = tile % num_m, n_blk = tile / num_m;
        for (int kt = 0; kt < num_kt; ++kt, ++it) {
          if (it < pre) continue;  // issued above
          const int s = it % P_STAGES;
          if (!mbar_wait(&bars->empty[s], ((it / P_STAGES) & 1) ^ 1, status, 0x111)) {
            bars->abort = 1;
            ok = false;
            break;
          }
          load_w(s, n_blk, kt);
          load_a(s, m_blk, kt);
        }
      }
      // The leader's MMA waits on every stage either CTA issued; its final
      // full waits (below) cover the pair's copies still in flight.
      if (rank == 0)
        for (int j = (it > P_STAGES ? it - P_STAGES : 0); j < it; ++j)
          mbar_wait(&bars->full[j % P_STAGES], (j / P_STAGES) & 1, status, 0x112);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader)
    if (rank == 0 && elect_one()) {
      pdl_wait();
      int it = 0, i = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < num_tiles; tile += num_pairs, ++i) {
        // both CTAs' epilogues have read the previous tile's accumulator
        if (i > 0 && !mbar_wait(&bars->acc_empty, (i - 1) & 1, status, 0x212)) { ok = false; break; }
        tc_fence_after();
        for (int kt = 0; kt < num_kt; ++kt, ++it) {
          const int s = it % P_STAGES;
          if (!mbar_wait(&bars->full[s], (it / P_STAGES) & 1, status, 0x211)) { ok = false; break; }
          tc_fence_after();
          uint8_t* st = smem + s * P_STAGE;
          const uint8_t* sa = st + P_A + P_B;
          const uint8_t* sb = sa + P_SFA;
#pragma unroll
          for (int j = 0; j < CPS; ++j) {
            tmem_cp_sf_pair(tmem + SFA_COL + 4 * j, smem_desc_sf(sa + 512 * j));
            tmem_cp_sf_pair(tmem + SFB_COL + 8 * j, smem_desc_sf(sb + 512 * j));                // W rows 0-127
            tmem_cp_sf_pair(tmem + SFB_COL + 8 * j + 4, smem_desc_sf(sb + CPS * 512 + 512 * j));  // W rows 128-255
          }
          issue_stage<kNV, true>(tmem + ACC_COL, smem_desc_sw128(st), smem_desc_sw128(st + P_A), tmem + SFA_COL,
                                 tmem + SFB_COL, kt == 0);
          tc_commit_pair(&bars->empty[s]);
        }
        if (!ok) break;
        tc_commit_pair(&bars->acc_full);
      }
      if (!ok) bars->abort = 1;
      tc_commit_pair_local(&bars->drain);  // tracks the pair's tcgen05 ops
      mbar_wait(&bars->drain, 0, status, 0x213);
    }
  } else {
    // ---------------- epilogue (both CTAs): TMEM lanes = the CTA's 128 tile rows
    pdl_wait();  // C, the bias and the activation's global scale belong to the stream's order
    const int q = warp & 3, h = (warp - 2) >> 2;
    const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16) + ACC_COL + h * 128;
    const float alpha = kNV ? w_gs / *a_gs : 1.0f;
    const uint32_t acc_empty0 = cluster_addr(&bars->acc_empty, 0);
    bool ok = true;
    int i = 0;
    for (int tile = pair; tile < num_tiles; tile += num_pairs, ++i) {
      const int m_blk = tile % num_m, n_blk = tile / num_m;
      if (ok) ok = mbar_wait(&bars->acc_full, i & 1, status, 0x311);
      ok = __all_sync(0xffffffffu, ok);  // the TMEM loads below are warp-collective
      tc_fence_after();
      uint32_t r[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(taddr + 32 * c, r[c]);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive_cluster(acc_empty0);  // the pair's next MMAs may overwrite the accumulator
      if (!ok || *(volatile int*)&bars->abort) continue;
      const int row = m_blk * 256 + static_cast<int>(rank) * 128 + q * 32 + lane;
      if (row >= M) continue;
      const int n0 = n_blk * BN + h * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int ncols = min(32, N - n0 - 32 * c);
        if (ncols <= 0) continue;
        T* crow = C + static_cast<int64_t>(row) * ldc + n0 + 32 * c;
        float v[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] = kNV ? __uint_as_float(r[c][e]) * alpha : __uint_as_float(r[c][e]);
        if (bias != nullptr) {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (e < ncols) v[e] += O::load(bias + n0 + 32 * c + e);
        }
        if (ncols == 32 && (reinterpret_cast<uintptr_t>(crow) & 15) == 0) {
          uint4* dst = reinterpret_cast<uint4*>(crow);
#pragma unroll
          for (int w4 = 0; w4 < 4; ++w4)
            dst[w4] = make_uint4(O::pack(v[8 * w4 + 0], v[8 * w4 + 1]), O::pack(v[8 * w4 + 2], v[8 * w4 + 3]),
                                 O::pack(v[8 * w4 + 4], v[8 * w4 + 5]), O::pack(v[8 * w4 + 6], v[8 * w4 + 7]));
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (e < ncols) crow[e] = O::one(v[e]);
        }
      }
    }
  }

  // Neither CTA releases the pair's TMEM or exits while the other may still
  // arrive on its barriers or read its shared memory.
  tc_fence_before();
  cluster_sync();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, TMEM_COLS);
  }
}

// Row-major E8M0/E4M3 scales [rows, ks] (row stride ld) -> tiled layout
// (rows padded to 128, ks padded to a multiple of 8, pad bytes = pad_value).
__global__ void sf_tile_kernel(const uint8_t* __restrict__ sf, uint8_t* __restrict__ out, int rows, int ks,
                               int64_t ld, int rows_p, int ks_p, uint8_t pad_value) {
  const int64_t total = static_cast<int64_t>(rows_p) * ks_p;
  const int kchunks = ks_p / 4;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / ks_p);
    const int k = static_cast<int>(i - static_cast<int64_t>(r) * ks_p);
    const uint8_t v = (r < rows && k < ks) ? sf[static_cast<int64_t>(r) * ld + k] : pad_value;
    const int64_t off = (static_cast<int64_t>(r / 128) * kchunks + k / 4) * 512 + (r % 32) * 16 +
                        ((r / 32) % 4) * 4 + (k % 4);
    out[off] = v;
  }
}

}  // namespace

// ---------------------------------------------------------------------------
// host helpers
// ---------------------------------------------------------------------------
typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                    CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                    CUtensorMapFloatOOBfill);

static PFN_encodeTiled encode_fn() {
  static PFN_encodeTiled fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled>(p);
  }
  return fn;
}

int make_tmap_u8_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t row_bytes, uint64_t ld_bytes,
                    uint32_t box_bytes, uint32_t box_rows, int swizzle_bytes) {
  PFN_encodeTiled fn = encode_fn();
  if (fn == nullptr) return fail(QDQ_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (ld_bytes & 15))
    return fail(QDQ_ERR_ALIGNMENT, "TMA operand needs 16-byte aligned base and row stride");
  const cuuint64_t dims[2] = {row_bytes, rows};
  const cuuint64_t strides[1] = {ld_bytes};
  const cuuint32_t box[2] = {box_bytes, box_rows};
  const cuuint32_t elem[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, elem,
                  CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                  : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                        : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(QDQ_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return QDQ_OK;
}

int make_tmap_u16_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld_bytes,
                     uint32_t box_cols, uint32_t box_rows, int swizzle_bytes) {
  PFN_encodeTiled fn = encode_fn();
  if (fn == nullptr) return fail(QDQ_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (ld_bytes & 15))
    return fail(QDQ_ERR_ALIGNMENT, "TMA operand needs 16-byte aligned base and row stride");
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {ld_bytes};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t elem[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base), dims, strides, box, elem,
                  CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(QDQ_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return QDQ_OK;
}

int make_tmap_u32_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld_bytes,
                     uint32_t box_cols, uint32_t box_rows) {
  PFN_encodeTiled fn = encode_fn();
  if (fn == nullptr) return fail(QDQ_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (ld_bytes & 15))
    return fail(QDQ_ERR_ALIGNMENT, "TMA operand needs 16-byte aligned base and row stride");
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {ld_bytes};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t elem[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void*>(base), dims, strides, box, elem,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(QDQ_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return QDQ_OK;
}

}  // namespace qdqb200

using namespace qdqb200;

extern "C" int64_t qdq_sf_tiled_bytes(int64_t rows, int64_t k) {
  if (rows <= 0 || k <= 0) return 0;
  const int64_t rows_p = (rows + 127) / 128 * 128;
  const int64_t ks_p = ((k + 31) / 32 + 7) / 8 * 8;
  return rows_p * ks_p;
}

extern "C" int qdq_sf_tile(const void* sf, void* sf_tiled, int64_t rows, int64_t k, int64_t ld, int block,
                           void* stream) {
  if (rows < 0 || k < 0) return fail(QDQ_ERR_INVALID_ARG, "qdq_sf_tile: negative shape");
  if (block != 32 && block != 16)
    return fail(QDQ_ERR_UNSUPPORTED, "qdq_sf_tile: block must be 32 (MXFP4, E8M0) or 16 (NVFP4, E4M3)");
  if (rows == 0 || k == 0) return QDQ_OK;
  if (!sf || !sf_tiled) return fail(QDQ_ERR_INVALID_ARG, "qdq_sf_tile: null pointer");
  const int64_t ks = (k + block - 1) / block;
  if (ld < ks) return fail(QDQ_ERR_INVALID_ARG, "qdq_sf_tile: ld < number of scales per row");
  const int rows_p = static_cast<int>((rows + 127) / 128 * 128);
  // one K-256 GEMM stage: 8 E8M0 scales per 32, or 16 E4M3 scales per 16
  const int per_stage = 256 / block;
  const int ks_p = static_cast<int>((ks + per_stage - 1) / per_stage * per_stage);
  const int64_t total = static_cast<int64_t>(rows_p) * ks_p;
  const int grid = static_cast<int>(std::min<int64_t>((total + 255) / 256, 148 * 16));
  sf_tile_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(sf), static_cast<uint8_t*>(sf_tiled), static_cast<int>(rows),
      static_cast<int>(ks), ld, rows_p, ks_p, 0);
  return check_launch("qdq_sf_tile");
}

namespace qdqb200 {
namespace {

// One block-scaled GEMM launch: CTA pairs on 256 x 256 tiles when A has two
// or more 128-row blocks, else one CTA per 128 x 256 tile.  kchunks = 512-byte
// scale chunks per 128-row block (per K).
template <bool kNV>
int launch_gemm(const char* who, const void* a_codes, const void* a_sf_tiled, const void* w_codes,
                const void* w_sf_tiled, const float* a_gs, float w_gs, const void* bias, void* c, int64_t M,
                int64_t N, int64_t K, int64_t lda_bytes, int64_t ldw_bytes, int64_t ldc, int out_dtype,
                int kchunks, cudaStream_t s) {
  int* status = device_status_ptr();
  if (status == nullptr) return QDQ_ERR_CUDA;
  const int sms = device_sm_count();
  const int of = out_dtype == QDQ_DTYPE_FP16 ? 1 : 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (M > BM && sms >= 2) {
    CUtensorMap ta, tb, tsa, tsb;
    constexpr int CPS = Fmt<kNV>::CPS;
    if (int st = make_tmap_u8_2d(&ta, a_codes, M, K / 2, lda_bytes, BKB, 128, 128)) return st;
    if (int st = make_tmap_u8_2d(&tb, w_codes, N, K / 2, ldw_bytes, BKB, 128, 128)) return st;
    if (int st = make_tmap_u32_2d(&tsa, a_sf_tiled, (M + 127) / 128 * kchunks, 128, 512, 128, CPS)) return st;
    if (int st = make_tmap_u32_2d(&tsb, w_sf_tiled, (N + 127) / 128 * kchunks, 128, 512, 128, CPS)) return st;
    static bool pair_attr[2][64] = {{false}};
    const void* pfn = of ? reinterpret_cast<const void*>(&mxf4_gemm_pair_kernel<true, kNV>)
                         : reinterpret_cast<const void*>(&mxf4_gemm_pair_kernel<false, kNV>);
    constexpr size_t smem = pair_smem_bytes<kNV>();
    if (dev >= 0 && dev < 64 && !pair_attr[of][dev]) {
      cudaError_t e = cudaFuncSetAttribute(pfn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      if (e != cudaSuccess) return fail(QDQ_ERR_CUDA, "%s: smem attribute: %s", who, cudaGetErrorString(e));
      pair_attr[of][dev] = true;
    }
    const int64_t tiles = ((M + 255) / 256) * ((N + BN - 1) / BN);
    const int64_t pairs = std::min<int64_t>(tiles, sms / 2);
    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs));
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    // programmatic dependent launch: weight prefetch overlaps the previous kernel
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    const int m_ = static_cast<int>(M), n_ = static_cast<int>(N), k_ = static_cast<int>(K);
    cudaError_t e = of ? cudaLaunchKernelEx(&cfg, mxf4_gemm_pair_kernel<true, kNV>, ta, tb, tsa, tsb, bias, c, m_,
                                            n_, k_, ldc, kchunks, a_gs, w_gs, status)
                       : cudaLaunchKernelEx(&cfg, mxf4_gemm_pair_kernel<false, kNV>, ta, tb, tsa, tsb, bias, c, m_,
                                            n_, k_, ldc, kchunks, a_gs, w_gs, status);
    if (e != cudaSuccess) return fail(QDQ_ERR_CUDA, "%s: pair launch: %s", who, cudaGetErrorString(e));
    return check_launch(who);
  }
  CUtensorMap ta, tb;
  if (int st = make_tmap_u8_2d(&ta, a_codes, M, K / 2, lda_bytes, BKB, BM, 128)) return st;
  if (int st = make_tmap_u8_2d(&tb, w_codes, N, K / 2, ldw_bytes, BKB, BN, 128)) return st;
  static bool attr_set[2][64] = {{false}};
  const void* fn = of ? reinterpret_cast<const void*>(&mxf4_gemm_kernel<true, kNV>)
                      : reinterpret_cast<const void*>(&mxf4_gemm_kernel<false, kNV>);
  constexpr size_t smem = smem_bytes<kNV>();
  if (dev >= 0 && dev < 64 && !attr_set[of][dev]) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return fail(QDQ_ERR_CUDA, "%s: smem attribute: %s", who, cudaGetErrorString(e));
    attr_set[of][dev] = true;
  }
  const int64_t tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  dim3 grid(static_cast<unsigned>(std::min<int64_t>(tiles, sms > 0 ? sms : 148)));
  auto* sfa = static_cast<const uint8_t*>(a_sf_tiled);
  auto* sfb = static_cast<const uint8_t*>(w_sf_tiled);
  const int m_ = static_cast<int>(M), n_ = static_cast<int>(N), k_ = static_cast<int>(K);
  if (of)
    mxf4_gemm_kernel<true, kNV><<<grid, THREADS, smem, s>>>(ta, tb, sfa, sfb, bias, c, m_, n_, k_, ldc, kchunks,
                                                           a_gs, w_gs, status);
  else
    mxf4_gemm_kernel<false, kNV><<<grid, THREADS, smem, s>>>(ta, tb, sfa, sfb, bias, c, m_, n_, k_, ldc, kchunks,
                                                            a_gs, w_gs, status);
  return check_launch(who);
}

int check_gemm_args(const char* who, const void* a_codes, const void* a_sf_tiled, const void* w_codes,
                    const void* w_sf_tiled, const void* c, int64_t M, int64_t N, int64_t K, int64_t lda_bytes,
                    int64_t ldw_bytes, int64_t ldc, int out_dtype) {
  if (out_dtype != QDQ_DTYPE_BF16 && out_dtype != QDQ_DTYPE_FP16)
    return fail(QDQ_ERR_INVALID_ARG, "%s: out_dtype must be bf16 (0) or fp16 (1)", who);
  if (M < 0 || N < 0 || K < 0) return fail(QDQ_ERR_INVALID_ARG, "%s: negative shape", who);
  if (M == 0 || N == 0) return QDQ_OK;
  if (!a_codes || !a_sf_tiled || !w_codes || !w_sf_tiled || !c)
    return fail(QDQ_ERR_INVALID_ARG, "%s: null pointer", who);
  if (K == 0) return fail(QDQ_ERR_UNSUPPORTED, "%s: K == 0", who);
  if (K % 32 != 0) return fail(QDQ_ERR_UNSUPPORTED, "%s: K=%lld must be a multiple of 32", who, (long long)K);
  if (M > (1ll << 30) || N > (1ll << 30) || K > (1ll << 30))
    return fail(QDQ_ERR_UNSUPPORTED, "%s: dimension too large", who);
  if (lda_bytes < K / 2 || ldw_bytes < K / 2 || ldc < N)
    return fail(QDQ_ERR_INVALID_ARG, "%s: leading dimension too small", who);
  if ((reinterpret_cast<uintptr_t>(a_sf_tiled) & 15) || (reinterpret_cast<uintptr_t>(w_sf_tiled) & 15))
    return fail(QDQ_ERR_ALIGNMENT, "%s: scale-factor buffers must be 16-byte aligned", who);
  return QDQ_OK;
}

}  // namespace
}  // namespace qdqb200

extern "C" int fp4_gemm_mxf4(const void* a_codes, const void* a_sf_tiled, const void* w_codes,
                             const void* w_sf_tiled, const void* bias, void* c, int64_t M, int64_t N,
                             int64_t K, int64_t lda_bytes, int64_t ldw_bytes, int64_t ldc, int out_dtype,
                             void* stream) {
  if (int st = check_gemm_args("fp4_gemm_mxf4", a_codes, a_sf_tiled, w_codes, w_sf_tiled, c, M, N, K, lda_bytes,
                               ldw_bytes, ldc, out_dtype))
    return st;
  if (M == 0 || N == 0) return QDQ_OK;
  const int kchunks = static_cast<int>(((K / 32) + 7) / 8 * 8 / 4);
  return launch_gemm<false>("fp4_gemm_mxf4", a_codes, a_sf_tiled, w_codes, w_sf_tiled, nullptr, 1.0f, bias, c, M,
                            N, K, lda_bytes, ldw_bytes, ldc, out_dtype, kchunks, static_cast<cudaStream_t>(stream));
}

extern "C" int64_t qdq_sf16_tiled_bytes(int64_t rows, int64_t k) {
  if (rows <= 0 || k <= 0) return 0;
  const int64_t rows_p = (rows + 127) / 128 * 128;
  const int64_t ks_p = ((k + 15) / 16 + 15) / 16 * 16;
  return rows_p * ks_p;
}

extern "C" int fp4_gemm_nvf4(const void* a_codes, const void* a_sf_tiled, const float* a_global_scale,
                             const void* w_codes, const void* w_sf_tiled, float w_global_scale, const void* bias,
                             void* c, int64_t M, int64_t N, int64_t K, int64_t lda_bytes, int64_t ldw_bytes,
                             int64_t ldc, int out_dtype, void* stream) {
  if (int st = check_gemm_args("fp4_gemm_nvf4", a_codes, a_sf_tiled, w_codes, w_sf_tiled, c, M, N, K, lda_bytes,
                               ldw_bytes, ldc, out_dtype))
    return st;
  if (M == 0 || N == 0) return QDQ_OK;
  if (a_global_scale == nullptr) return fail(QDQ_ERR_INVALID_ARG, "fp4_gemm_nvf4: null a_global_scale");
  if (!(w_global_scale > 0.0f) || !std::isfinite(w_global_scale))
    return fail(QDQ_ERR_INVALID_ARG, "fp4_gemm_nvf4: w_global_scale must be finite and positive");
  const int kchunks = static_cast<int>(((K / 16) + 15) / 16 * 16 / 4);
  return launch_gemm<true>("fp4_gemm_nvf4", a_codes, a_sf_tiled, w_codes, w_sf_tiled, a_global_scale,
                           w_global_scale, bias, c, M, N, K, lda_bytes, ldw_bytes, ldc, out_dtype, kchunks,
                           static_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------------------
// Fused linear: bf16/fp16 activation -> MXFP4 codes + tiled scales (exactly
// the reference's mxfp4_qdq quantisation) -> block-scaled GEMM.  Scratch for
// the activation codes comes from the caller's workspace.
// ---------------------------------------------------------------------------
extern "C" int64_t fp4_linear_workspace_bytes(int64_t M, int64_t K) {
  if (M <= 0 || K <= 0) return 0;
  const int64_t kp = (K + 31) / 32 * 32;
  auto up = [](int64_t v) { return (v + 255) / 256 * 256; };
  return up(M * kp / 2) + up(M * kp / 32) + up(qdq_sf_tiled_bytes(M, K));
}

extern "C" int fp4_linear_mxf4(const void* a, int64_t lda, int dtype, const void* w_codes,
                               const void* w_sf_tiled, const void* bias, void* c, int64_t M, int64_t N,
                               int64_t K, int64_t ldw_bytes, int64_t ldc, void* workspace,
                               int64_t workspace_bytes, void* stream) {
  if (M < 0 || N < 0 || K < 0) return fail(QDQ_ERR_INVALID_ARG, "fp4_linear_mxf4: negative shape");
  if (M == 0 || N == 0) return QDQ_OK;
  if (K % 32 != 0) return fail(QDQ_ERR_UNSUPPORTED, "fp4_linear_mxf4: K=%lld must be a multiple of 32", (long long)K);
  if (workspace == nullptr || workspace_bytes < fp4_linear_workspace_bytes(M, K))
    return fail(QDQ_ERR_INVALID_ARG, "fp4_linear_mxf4: workspace smaller than fp4_linear_workspace_bytes()");
  // Small M: one launch that quantises the activation inside the GEMM producer.
  if (M <= 64 && (dtype == QDQ_DTYPE_BF16 || dtype == QDQ_DTYPE_FP16) &&
      (reinterpret_cast<uintptr_t>(a) & 15) == 0 && ((lda * 2) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(w_sf_tiled) & 15) == 0 && lda >= K && ldc >= N && ldw_bytes >= K / 2)
    return fp4_linear_decode(a, lda, dtype, w_codes, w_sf_tiled, bias, c, M, N, K, ldw_bytes, ldc, stream);
  auto up = [](int64_t v) { return (v + 255) / 256 * 256; };
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint8_t* a_codes = ws;
  uint8_t* a_sf = a_codes + up(M * K / 2);
  uint8_t* a_sf_t = a_sf + up(M * K / 32);
  if (K % 256 == 0 && (dtype == QDQ_DTYPE_BF16 || dtype == QDQ_DTYPE_FP16) &&
      (reinterpret_cast<uintptr_t>(a) & 15) == 0 && lda % 8 == 0) {
    // one pass: codes and tiled scales (no padded K chunk to clear)
    if (int st = qdq_mxfp4_codes_tiled(a, a_codes, a_sf_t, M, K, lda, dtype, stream)) return st;
  } else {
    if (int st = qdq_mxfp4(a, nullptr, a_codes, a_sf, M, K, lda, K, dtype, 32, stream)) return st;
    if (int st = qdq_sf_tile(a_sf, a_sf_t, M, K, K / 32, 32, stream)) return st;
  }
  return fp4_gemm_mxf4(a_codes, a_sf_t, w_codes, w_sf_tiled, bias, c, M, N, K, K / 2, ldw_bytes, ldc, dtype,
                       stream);
}

// ---------------------------------------------------------------------------
// Fused NVFP4 linear: bf16/fp16 activation -> (global amax) -> NVFP4 codes +
// E4M3 scales per 16 (exactly vLLM's NVFP4 quantisation, the codes of
// nvfp4_qdq) -> tiled scales -> block16 GEMM with alpha = gs_w / gs_a.
// ---------------------------------------------------------------------------
extern "C" int64_t fp4_linear_nvf4_workspace_bytes(int64_t M, int64_t K) {
  if (M <= 0 || K <= 0) return 0;
  auto up = [](int64_t v) { return (v + 255) / 256 * 256; };
  return 256 + up(M * K / 2) + up(M * K / 16) + up(qdq_sf16_tiled_bytes(M, K));
}

extern "C" int fp4_linear_nvf4(const void* a, int64_t lda, int dtype, const float* a_global_scale,
                               const void* w_codes, const void* w_sf_tiled, float w_global_scale,
                               const void* bias, void* c, int64_t M, int64_t N, int64_t K, int64_t ldw_bytes,
                               int64_t ldc, void* workspace, int64_t workspace_bytes, void* stream) {
  if (M < 0 || N < 0 || K < 0) return fail(QDQ_ERR_INVALID_ARG, "fp4_linear_nvf4: negative shape");
  if (M == 0 || N == 0) return QDQ_OK;
  if (dtype != QDQ_DTYPE_BF16 && dtype != QDQ_DTYPE_FP16)
    return fail(QDQ_ERR_INVALID_ARG, "fp4_linear_nvf4: dtype must be bf16 (0) or fp16 (1)");
  if (K % 32 != 0) return fail(QDQ_ERR_UNSUPPORTED, "fp4_linear_nvf4: K=%lld must be a multiple of 32", (long long)K);
  if (workspace == nullptr || workspace_bytes < fp4_linear_nvf4_workspace_bytes(M, K) ||
      (reinterpret_cast<uintptr_t>(workspace) & 255))
    return fail(QDQ_ERR_INVALID_ARG,
                "fp4_linear_nvf4: workspace must be 256-byte aligned and hold fp4_linear_nvf4_workspace_bytes()");
  auto up = [](int64_t v) { return (v + 255) / 256 * 256; };
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  float* gs = reinterpret_cast<float*>(ws);           // 4 bytes of gs, then 16 bytes of amax scratch
  uint8_t* a_codes = ws + 256;
  uint8_t* a_sf = a_codes + up(M * K / 2);
  uint8_t* a_sf_t = a_sf + up(M * K / 16);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Small M: the swap-AB decode kernel quantises the activation in its
  // producer.  Without a given scale, up to 24 rows it also takes their global
  // amax, split over clusters of 4 CTAs (each reads a quarter of the rows from
  // L2 while its weight ring fills), when N / 128 is a multiple of 4.
  // Otherwise one 8-CTA cluster pass takes it first, overlapped with the
  // decode kernel's prologue through programmatic dependent launch.  At
  // N = 14336, K = 4096 the first takes M = 8 / 16 / 24 to 11.1 / 13.4 /
  // 16.7 us against 11.8 / 13.8 / 17.0 us for the second; from M = 32 the
  // second is faster (M = 64: 28.2 against 29.4 us).
  const bool decode = M <= 64 && (reinterpret_cast<uintptr_t>(a) & 15) == 0 && ((lda * 2) & 15) == 0 &&
                      (reinterpret_cast<uintptr_t>(w_sf_tiled) & 15) == 0 && lda >= K && ldc >= N &&
                      ldw_bytes >= K / 2;
  const float* gs_a = a_global_scale;
  if (decode) {
    if (gs_a == nullptr && (M > 24 || ((N + 127) / 128) % 4 != 0)) {
      if (int st = launch_global_scale_small(a, gs, M, K, lda, dtype, s)) return st;
      gs_a = gs;
    }
    return fp4_linear_decode_nvf4(a, lda, dtype, gs_a, w_codes, w_sf_tiled, w_global_scale, bias, c, M, N, K,
                                  ldw_bytes, ldc, stream);
  }
  if (gs_a == nullptr) {
    if (int st = qdq_nvfp4_global_scale(a, gs, ws + 16, M, K, lda, dtype, stream)) return st;
    gs_a = gs;
  }
  // codes and tiled scales in one pass when K % 256 == 0 (rows 16-byte aligned), else codes, scales and
  // their tiling
  if (K % 256 == 0 && (reinterpret_cast<uintptr_t>(a) & 15) == 0 && lda % 8 == 0) {
    if (int st = qdq_nvfp4_codes_tiled(a, gs_a, a_codes, a_sf_t, M, K, lda, dtype, stream)) return st;
  } else {
    if (int st = qdq_nvfp4(a, nullptr, a_codes, a_sf, gs_a, M, K, lda, K, dtype, stream)) return st;
    if (int st = qdq_sf_tile(a_sf, a_sf_t, M, K, K / 16, 16, stream)) return st;
  }
  return fp4_gemm_nvf4(a_codes, a_sf_t, gs_a, w_codes, w_sf_tiled, w_global_scale, bias, c, M, N, K, K / 2,
                       ldw_bytes, ldc, dtype, s);
}
