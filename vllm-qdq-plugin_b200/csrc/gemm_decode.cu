// Fused MXFP4 linear for small M (decode and small batches), one launch:
//   C[M, N] = mxfp4(A)[M, K] . W[N, K]^T (+ bias[N]),  fp32 accumulation,
// with A bf16/fp16 and W E2M1 codes + E8M0 scales in the tiled layout of
// qdq_sf_tile.  The activation is quantised inside the GEMM's producer with
// the same group rule as the QDQ kernel (mx_quant.cuh), so the products are
// those of the reference's mxfp4_qdq(A) against W (reference:
// src/vllm_qdq_plugin/patch.py:51-57 + vllm/_custom_ops.py:1277 marlin_gemm).
//
// NVFP4 mode (kNV): W carries E4M3 scales per 16 (block16 tiled layout) and a
// tensor scale w_gs, the activation is quantised with vLLM's NVFP4 rule
// against the per-tensor scale gs_a (given, or 2688 / max |a| computed by
// the kernel, split over clusters of CTAs), the MMAs are kind::mxf4nvf4.block16 and the
// output is scaled by w_gs / gs_a (reference: the NVFP4 Marlin path of
// vllm/model_executor/layers/quantization/utils/marlin_utils_fp4.py:149-202).
//
// "Swap AB": the tcgen05 MMA's M side is 128 rows of W and its N side the
// activation rows, padded to NA = 16, 32 or 64.  One CTA per 128 rows of W
// streams that slice of W once (N / 128 CTAs: 112 for N = 14336), so the
// kernel is bound by HBM reading W, not by the tensor pipe.
//
// CTA, 10 warps:
//   warp 0 / one lane   TMA producer: W code tile [128 rows x 128 B] (128-byte
//                       swizzle), its scale chunks and the raw [NA, 256]
//                       bf16/fp16 slice of A into a ring of 3-8 stages
//   warp 1 / one lane   MMA issuer: per stage 4 x tcgen05.mma.kind::mxf4
//                       (M = 128, N = NA, K = 64), commit frees the stage
//   warps 2-9           activation quantiser in 1, 2 or 4 teams (decode_teams),
//                       team t taking the stages of ring slots s = t (mod
//                       teams), so several stages are quantised at once (each
//                       slot's barrier phases are observed in order by one team) (the stage's raw A slice in shared
//                       memory -> E2M1 codes in the swizzled operand layout +
//                       E8M0 scales in the scale-chunk layout); then the
//                       epilogue (TMEM lanes = W rows, columns = activation rows)
#include "mx_quant.cuh"
#include "sm100.cuh"

namespace qdqb200 {
namespace {

using namespace sm100;

constexpr int DBM = 128;                 // W rows per CTA (UMMA M)
constexpr int DBK = 256;                 // K elements per stage
constexpr int DBKB = DBK / 2;            // code bytes per row per stage (one 128-byte swizzle row)
constexpr int NA_MAX = 64;               // activation rows per launch (UMMA N)
constexpr int W_TILE = DBM * DBKB;       // 16 KB
constexpr int SF_STAGE = 1024;           // two 512-byte scale chunks (8 scales per row)
// NVFP4 (block16): four 512-byte scale chunks per stage (16 E4M3 scales per row)
__host__ __device__ constexpr int sf_stage(bool nv) { return nv ? 2 * SF_STAGE : SF_STAGE; }
constexpr int D_QUANT_THREADS = 256;                 // 8 quantiser / epilogue warps
constexpr int D_THREADS = 64 + D_QUANT_THREADS;      // + producer and MMA warps
// Quantiser teams (one stage each in flight) for M activation rows: few rows
// make a stage's quantisation latency-bound, so more stages run at once;
// many rows make it throughput-bound, so more threads share one stage.
__host__ __device__ constexpr int decode_teams(int M) { return M <= 16 ? 4 : (M <= 32 ? 2 : 1); }
constexpr int D_TMEM_COLS = 128;
constexpr uint32_t T_ACC = 0, T_SFW = 64, T_SFA = 80;  // scale columns: 4 per 512-byte chunk

// Stage layout for NA activation rows: W codes | A codes | W scales | A scales | raw A.
template <int kNA, bool kNV = false>
struct DLayout {
  static constexpr int A_TILE = kNA * DBKB;
  static constexpr int RAW = kNA * DBK * 2;
  static constexpr int SFS = sf_stage(kNV);
  static constexpr int ST_W = 0, ST_A = W_TILE, ST_SFW = W_TILE + A_TILE, ST_SFA = ST_SFW + SFS,
                       ST_RAW = ST_SFA + SFS;
  static constexpr int STAGE = (ST_RAW + RAW + 1023) / 1024 * 1024;
  // as many stages as fit 227 KB (MXFP4 at NA = 16: 8 x 28 KB; NVFP4 7 x 30 KB)
  static constexpr int STAGES = kNA == 16 ? (kNV ? 7 : 8) : (kNA == 32 ? 5 : 3);
};

struct __align__(8) DBars {
  uint64_t raw[8];     // W, its scales and the raw A slice landed (1 arrival + tx)
  uint64_t ready[8];   // the activation slice is quantised (one team's arrivals)
  uint64_t empty[8];   // the stage's MMAs completed
  uint64_t acc_full;
  uint32_t tmem_base;
  int abort;
  int preissued;       // stages whose loads thread 0 issued before the CTA-wide sync
  uint32_t amax[8];    // NVFP4 without a given activation scale: per-warp |x| maxima (bit patterns)
  uint32_t camax[4];   // ... and the maxima of the cluster's CTAs, written by each of them
};
// NVFP4 without a given activation scale (the host passes none up to 24
// rows): the kernel runs in clusters of kDecCluster CTAs that split the
// activation rows' global amax between them.
constexpr int kDecCluster = 4;
template <int kNA, bool kNV = false>
constexpr size_t d_smem_bytes() {
  return 1024 + static_cast<size_t>(DLayout<kNA, kNV>::STAGES) * DLayout<kNA, kNV>::STAGE + sizeof(DBars);
}
static_assert(d_smem_bytes<16, true>() <= 227 * 1024 && d_smem_bytes<32, true>() <= 227 * 1024 &&
              d_smem_bytes<64, true>() <= 227 * 1024, "decode stages exceed shared memory");

template <bool kF16>
struct DOut {
  using T = __nv_bfloat16;
  __device__ static float load(const T* p) { return __bfloat162float(*p); }
  __device__ static T one(float a) { return __float2bfloat16_rn(a); }
};
template <>
struct DOut<true> {
  using T = __half;
  __device__ static float load(const T* p) { return __half2float(*p); }
  __device__ static T one(float a) { return __float2half_rn(a); }
};

// kNV: NVFP4 weights (E4M3 scales per 16, tensor scale w_gs) and the
// activation quantised to NVFP4 with the per-tensor scale *a_gs (vLLM's
// NVFP4 rule, nv_group_codes), block16 MMAs, output times w_gs / *a_gs.
template <int kDtype, int kNA, bool kNV>
__global__ void __launch_bounds__(D_THREADS, 1)
mxf4_decode_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_a,
                   const uint8_t* __restrict__ sfw, const void* __restrict__ bias_v, void* __restrict__ c_v,
                   int M, int N, int K, int64_t ldc, int kchunks, const float* __restrict__ a_gs, float w_gs,
                   float zero, const uint16_t* __restrict__ a_raw, int64_t lda, int* status) {
  using Lay = DLayout<kNA, kNV>;
  constexpr int SFS = Lay::SFS, CPS = SFS / 512;  // scale bytes / chunks per stage
  constexpr int S = Lay::STAGES;
  constexpr bool kF16 = kDtype == QDQ_DTYPE_FP16;
  using O = DOut<kF16>;
  using T = typename O::T;
  const T* bias = static_cast<const T*>(bias_v);
  T* C = static_cast<T*>(c_v);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  DBars* bars = reinterpret_cast<DBars*>(smem + S * Lay::STAGE);
  const int warp = threadIdx.x >> 5;
  const int n_blk = blockIdx.x;
  const int num_kt = (K + DBK - 1) / DBK;

  // One stage's loads: the W tile and its scales (weights), then the raw A
  // slice (the activation, which the previous kernel on the stream may write).
  auto issue_w = [&](int kt) {
    const int s = kt % S;
    uint8_t* st = smem + s * Lay::STAGE;
    mbar_arrive_expect_tx(&bars->raw[s], W_TILE + SFS + Lay::RAW);
    tma_load_2d(st + Lay::ST_W, &tmap_w, kt * DBKB, n_blk * DBM, &bars->raw[s]);
    bulk_load(st + Lay::ST_SFW, sfw + (static_cast<int64_t>(n_blk) * kchunks + CPS * kt) * 512, SFS,
              &bars->raw[s]);
  };
  auto issue_a = [&](int kt) {
    const int s = kt % S;
    tma_load_2d(smem + s * Lay::STAGE + Lay::ST_RAW, &tmap_a, kt * DBK, 0, &bars->raw[s]);
  };
  auto issue_stage = [&](int kt) {
    issue_w(kt);
    issue_a(kt);
  };
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&bars->raw[s], 1);
      mbar_init(&bars->ready[s], D_QUANT_THREADS / decode_teams(M));
      mbar_init(&bars->empty[s], 1);
    }
    mbar_init(&bars->acc_full, 1);
    bars->abort = 0;
    fence_barrier_init();
    prefetch_tmap(&tmap_w);
    prefetch_tmap(&tmap_a);
    // The first ring of weight loads needs neither TMEM nor the cleared tiles,
    // nor the previous kernel on the stream, so it starts before all of them:
    // the HBM latency overlaps the prologue (and, under programmatic dependent
    // launch, the previous kernel's tail).
    const int pre = min(S, num_kt);
    for (int kt = 0; kt < pre; ++kt) issue_w(kt);
    bars->preissued = pre;
  }
  pdl_launch_dependents();
  // Activation rows >= M and their scales stay zero for the whole launch
  // (disjoint from the W, W-scale and raw-A bytes the loads above write).
  constexpr int kZero = (Lay::A_TILE + 2 * SFS) / 16;  // A codes + W and A scale chunks
  for (int i = threadIdx.x; i < S * kZero; i += D_THREADS) {
    const int s = i / kZero, o = (i % kZero) * 16;
    if (o < Lay::A_TILE || o >= Lay::A_TILE + SFS)  // skip the W scales (loaded every stage)
      *reinterpret_cast<uint4*>(smem + s * Lay::STAGE + Lay::ST_A + o) = make_uint4(0, 0, 0, 0);
  }
  if (warp == 0) {
    tmem_alloc(&bars->tmem_base, D_TMEM_COLS);
    tmem_relinquish();
  }
  // Everything below reads the activation or writes C: the previous kernel
  // on the stream must have completed (programmatic dependent launch).
  pdl_wait();
  if (threadIdx.x == 0)
    for (int kt = 0; kt < bars->preissued; ++kt) issue_a(kt);
  fence_proxy_async_smem();  // the zeroed operand bytes are read by the tensor core
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0) {
    // ---------------- producer: W, its scales, raw A
    if (kNV && a_gs == nullptr) cluster_sync();  // the quantiser warps' amax exchange (every thread joins)
    if (elect_one()) {
      int issued = bars->preissued;
      for (int kt = issued; kt < num_kt; ++kt) {
        const int s = kt % S;
        if (!mbar_wait(&bars->empty[s], ((kt / S) & 1) ^ 1, status, 0x401)) {
          bars->abort = 1;
          break;
        }
        if (*(volatile int*)&bars->abort) break;
        issue_stage(kt);
        ++issued;
      }
      for (int kt = (issued > S ? issued - S : 0); kt < issued; ++kt)
        mbar_wait(&bars->raw[kt % S], (kt / S) & 1, status, 0x402);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (kNV && a_gs == nullptr) cluster_sync();  // the quantiser warps' amax exchange (every thread joins)
    if (elect_one()) {
      constexpr uint32_t idesc = idesc_mxf4(DBM, kNA, !kNV);
      bool ok = true;
      for (int kt = 0; kt < num_kt; ++kt) {
        const int s = kt % S;
        if (!mbar_wait(&bars->ready[s], (kt / S) & 1, status, 0x403)) { ok = false; break; }
        if (*(volatile int*)&bars->abort) { ok = false; break; }
        tc_fence_after();
        uint8_t* st = smem + s * Lay::STAGE;
#pragma unroll
        for (int j = 0; j < CPS; ++j) {  // chunk j: scales 4j .. 4j+3 of the stage, W rows / activation rows
          tmem_cp_sf(tmem + T_SFW + 4 * j, smem_desc_sf(st + Lay::ST_SFW + 512 * j));
          tmem_cp_sf(tmem + T_SFA + 4 * j, smem_desc_sf(st + Lay::ST_SFA + 512 * j));
        }
        const uint64_t dw = smem_desc_sw128(st + Lay::ST_W);
        const uint64_t da = smem_desc_sw128(st + Lay::ST_A);
#pragma unroll
        for (int kk = 0; kk < DBK / 64; ++kk) {
          if (kNV) {  // block16: K-64 step kk reads the whole chunk kk
            mma_nvf4(tmem + T_ACC, dw + ((kk * 32) >> 4), da + ((kk * 32) >> 4), idesc, tmem + T_SFW + 4 * kk,
                     tmem + T_SFA + 4 * kk, (kt | kk) != 0);
          } else {    // block32: chunk kk / 2, scale bytes 2 (kk % 2), +1
            const uint32_t j = kk >> 1, sf_id = (kk & 1) * 2;
            mma_mxf4(tmem + T_ACC, dw + ((kk * 32) >> 4), da + ((kk * 32) >> 4),
                     idesc_with_sf_ids(idesc, sf_id, sf_id), (tmem + T_SFW + 4 * j) | (sf_id << 30),
                     (tmem + T_SFA + 4 * j) | (sf_id << 30), (kt | kk) != 0);
          }
        }
        tc_commit(&bars->empty[s]);
      }
      if (!ok) bars->abort = 1;
      tc_commit(&bars->acc_full);  // also on abort: the epilogue waits for the issued MMAs
    }
  } else {
    // ---------------- activation quantiser (teams), then epilogue
    const int teams = decode_teams(M);
    const int team_threads = D_QUANT_THREADS / teams;
    const int team = (threadIdx.x - 64) / team_threads;
    const int tq = (threadIdx.x - 64) % team_threads;
    const int lane = threadIdx.x & 31;
    bool ok = true;
    // NVFP4 activation scale, written by the previous kernel or computed here
    // (after pdl_wait either way): gs = 2688 / max |a| over the whole [M, K]
    // activation, the formula of qdq_nvfp4_global_scale, from the same
    // maximum bit pattern, so the same fp32 value.  Computed here, the CTAs
    // of a cluster each reduce every kDecCluster-th 16-byte chunk of the
    // rows (from L2, while their weight rings fill), write their maximum
    // into every CTA of the cluster (distributed shared memory) and meet at
    // the cluster barrier.
    float gs = 0.f;
    if (kNV) {
      if (a_gs != nullptr) {
        gs = __ldg(a_gs);
      } else {
        const uint32_t crank = cluster_rank();
        const int qt = threadIdx.x - 64, cpr = K / 8;  // 16-byte chunks per row
        uint32_t m8 = 0;
        for (int i = qt + D_QUANT_THREADS * static_cast<int>(crank); i < M * cpr;
             i += D_QUANT_THREADS * kDecCluster) {
          const int row = i / cpr, c = i - row * cpr;
          m8 = max(m8, absmax8(ld_stream(reinterpret_cast<const uint4*>(a_raw + row * lda + c * 8))));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m8 = max(m8, __shfl_xor_sync(0xffffffffu, m8, o));
        if (lane == 0) bars->amax[warp - 2] = m8;
        asm volatile("bar.sync 1, %0;" ::"n"(D_QUANT_THREADS) : "memory");  // the quantiser warps only
        if (qt == 0) {
          uint32_t cta = 0;
#pragma unroll
          for (int w = 0; w < 8; ++w) cta = max(cta, bars->amax[w]);
#pragma unroll
          for (int r = 0; r < kDecCluster; ++r)
            asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(cluster_addr(&bars->camax[crank], r)), "r"(cta)
                         : "memory");
        }
        cluster_sync();  // every CTA's maximum is in every CTA's camax
        uint32_t all = 0;
#pragma unroll
        for (int r = 0; r < kDecCluster; ++r) all = max(all, bars->camax[r]);
        gs = __fdiv_rn(2688.0f, Fmt<kDtype>::amax_value(all));
      }
    }
    const float rgs = kNV ? zero_safe_recip(gs) : 0.f;
    for (int kt = 0; kt < num_kt; ++kt) {
      const int s = kt % S;
      // A parity wait can only tell the current phase from the previous one,
      // so every stage of a slot goes to the same team, in order.
      if (s % teams != team) continue;
      if (ok) ok = mbar_wait(&bars->raw[s], (kt / S) & 1, status, 0x404);
      uint8_t* st = smem + s * Lay::STAGE;
      // groups (row m, 32-block g) of this stage's [M, 256] slice; columns past K read as zero
      if (kNV) {  // 16-blocks: 8 code bytes (half a 16-byte chunk) and one E4M3 scale each
        for (int it = tq; it < M * (DBK / 16); it += team_threads) {
          const int m = it >> 4, g = it & 15;
          const uint4* src = reinterpret_cast<const uint4*>(st + Lay::ST_RAW + m * (DBK * 2) + g * 32);
          uint4 v[2] = {src[0], src[1]};
          uint32_t code[2];
          const uint32_t sb = nv_group_codes<kDtype>(v, gs, rgs, zero, code);
          *reinterpret_cast<uint2*>(st + Lay::ST_A + m * DBKB + (((g >> 1) ^ (m & 7)) << 4) + (g & 1) * 8) =
              make_uint2(code[0], code[1]);
          st[Lay::ST_SFA + (g >> 2) * 512 + (m & 31) * 16 + ((m >> 5) & 3) * 4 + (g & 3)] = static_cast<uint8_t>(sb);
        }
      }
      for (int it = tq; !kNV && it < M * (DBK / 32); it += team_threads) {
        const int m = it >> 3, g = it & 7;
        const uint4* src = reinterpret_cast<const uint4*>(st + Lay::ST_RAW + m * (DBK * 2) + g * 64);
        uint4 v[4] = {src[0], src[1], src[2], src[3]};
        uint32_t code[4];
        const int e = mx_group_codes<kDtype>(v, code);
        // 128-byte swizzle: 16-byte chunk g of row m sits at chunk g ^ (m % 8)
        *reinterpret_cast<uint4*>(st + Lay::ST_A + m * DBKB + ((g ^ (m & 7)) << 4)) =
            make_uint4(code[0], code[1], code[2], code[3]);
        st[Lay::ST_SFA + (g >> 2) * 512 + (m & 31) * 16 + ((m >> 5) & 3) * 4 + (g & 3)] =
            static_cast<uint8_t>(e);
      }
      fence_proxy_async_smem();
      mbar_arrive(&bars->ready[s]);
    }
    // epilogue: warp w reads TMEM lanes 32 (w % 4).. (W rows); warps 2-5 take
    // the activation-row columns [0, 32), warps 6-9 [32, 64)
    if (ok) ok = mbar_wait(&bars->acc_full, 0, status, 0x405);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    const int q = warp & 3;
    const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16) + T_ACC;
    constexpr int NC = kNA > 32 ? 2 : 1;
    const int half = (warp - 2) >> 2;
    if (half < NC && 32 * half < M) {
      uint32_t r[32];
      tmem_ld32(taddr + 32 * half, r);
      tmem_ld_wait();
      const int n = n_blk * DBM + q * 32 + lane;
      if (ok && !*(volatile int*)&bars->abort && n < N) {
        const float b = bias != nullptr ? O::load(bias + n) : 0.f;
        const float alpha = kNV ? w_gs / gs : 1.0f;  // as the block16 GEMM's epilogue
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int m = 32 * half + i;
          const float v = kNV ? __uint_as_float(r[i]) * alpha : __uint_as_float(r[i]);
          if (m < M) C[static_cast<int64_t>(m) * ldc + n] = O::one(v + b);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, D_TMEM_COLS);
  }
}

template <int kDtype, int kNA, bool kNV>
int launch_decode(const CUtensorMap& tw, const CUtensorMap& ta, const uint8_t* sf, const void* bias, void* c,
                  int64_t M, int64_t N, int64_t K, int64_t ldc, int kchunks, const float* a_gs, float w_gs,
                  const void* a_raw, int64_t lda, int* status, cudaStream_t s) {
  constexpr size_t smem = d_smem_bytes<kNA, kNV>();
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(&mxf4_decode_kernel<kDtype, kNA, kNV>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return fail(QDQ_ERR_CUDA, "fp4_linear_decode: smem attribute: %s", cudaGetErrorString(e));
    attr_set[dev] = true;
  }
  // Programmatic dependent launch: the kernel streams its first weight tiles
  // while the previous kernel on the stream finishes (griddepcontrol.wait
  // guards every activation read and output write).
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>((N + DBM - 1) / DBM));
  cfg.blockDim = dim3(D_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  if (kNV && a_gs == nullptr) {  // the activation's amax split over clusters of kDecCluster CTAs
    if (cfg.gridDim.x % kDecCluster != 0)
      return fail(QDQ_ERR_INVALID_ARG, "fp4_linear_decode: in-kernel amax needs N / 128 to be a multiple of %d",
                  kDecCluster);
    at[1].id = cudaLaunchAttributeClusterDimension;
    at[1].val.clusterDim.x = kDecCluster;
    at[1].val.clusterDim.y = 1;
    at[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
  }
  const float zero = 0.0f;  // +0.0 as an operand the compiler cannot fold (see nv_scale8)
  const cudaError_t e = cudaLaunchKernelEx(&cfg, mxf4_decode_kernel<kDtype, kNA, kNV>, tw, ta, sf, bias, c,
                                           static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), ldc,
                                           kchunks, a_gs, w_gs, zero, static_cast<const uint16_t*>(a_raw), lda,
                                           status);
  if (e != cudaSuccess) return fail(QDQ_ERR_CUDA, "fp4_linear_decode: launch: %s", cudaGetErrorString(e));
  return check_launch("fp4_linear_decode");
}

// ---------------------------------------------------------------------------
// Grouped MXFP4 MoE GEMM (replaces moe_wna16_marlin_gemm for MXFP4 experts)
// ---------------------------------------------------------------------------
// Pre-pass (moe_gather_quant_kernel): the activation rows in sorted-slot
// order (vLLM's moe_align_block_size layout), quantised to MXFP4 once: codes
// [num_sorted, K/2] and, per block of moe_block_size slots, the E8M0 scales in
// the tiled layout (rows 0..bs-1 of one 128-row chunk set).  Padding slots are
// zero.  Its first CTA also cuts the live blocks into segments: runs of at
// most MOE_SEG_MAX consecutive blocks that name the same local expert.
//
// Then the grouped GEMM walks (segment, 128 rows of the expert's W) items: a
// stage holds one W tile and the codes of the segment's blocks (NA rows each,
// back to back), and ONE swap-AB MMA per K step covers the whole segment
// (M = 128 W rows, N = NA x blocks <= 192), so W is read from shared memory
// once per segment.  The MMA's B-side scales for a segment starting at block
// b are the scale chunk of block b, which the pre-pass fills with the rows of
// blocks b, b+1, b+2 at their segment rows NA*i + r (rows 128-191 of a
// three-block NA = 64 segment come from block b+2's chunk): every segment,
// wherever it starts, finds its scales in 4-column TMEM copies.
// Stage: W codes | A codes x 3 | W scales | A scales (rows 0-127, 128-255).
constexpr int MOE_SEG_MAX = 3;

// Segment table in the workspace: [0] = count, [1 + i] = first block << 2 | blocks.
__device__ void moe_segments(const int32_t* __restrict__ expert_ids, int nlive, int num_experts,
                             int32_t* __restrict__ seg_tab) {
  __shared__ int s_max[8], s_sum[8];
  __shared__ int s_carry_rs, s_carry_cnt;
  const int t = threadIdx.x, lane = t & 31, wid = t >> 5;
  if (t == 0) {
    s_carry_rs = -1;
    s_carry_cnt = 0;
  }
  __syncthreads();
  for (int base = 0; base < nlive; base += 256) {
    const int b = base + t;
    const int e = b < nlive ? __ldg(expert_ids + b) : -1;
    const bool valid = b < nlive && e >= 0 && e < num_experts;
    const int ep = (b > 0 && b <= nlive) ? __ldg(expert_ids + b - 1) : -1;
    const bool start_run = valid && (b == 0 || ep != e);
    // inclusive max-scan of run starts: the first block of b's run
    int v = start_run ? b : -1;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, v, off);
      if (lane >= off) v = max(v, o);
    }
    if (lane == 31) s_max[wid] = v;
    __syncthreads();
    if (wid == 0) {
      int w = lane < 8 ? s_max[lane] : -1;
#pragma unroll
      for (int off = 1; off < 8; off <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, w, off);
        if (lane >= off) w = max(w, o);
      }
      if (lane < 8) s_max[lane] = w;
    }
    __syncthreads();
    v = max(v, wid > 0 ? s_max[wid - 1] : -1);
    v = max(v, s_carry_rs);
    const bool seg_start = valid && ((b - v) % MOE_SEG_MAX) == 0;
    // exclusive sum-scan of segment starts
    const unsigned bal = __ballot_sync(0xffffffffu, seg_start);
    if (lane == 0) s_sum[wid] = __popc(bal);
    __syncthreads();
    int before = s_carry_cnt + __popc(bal & ((1u << lane) - 1u));
    for (int w = 0; w < wid; ++w) before += s_sum[w];
    if (seg_start) {
      int nb = 1;
      if (b + 1 < nlive && __ldg(expert_ids + b + 1) == e) {
        ++nb;
        if (MOE_SEG_MAX > 2 && b + 2 < nlive && __ldg(expert_ids + b + 2) == e) ++nb;
      }
      seg_tab[1 + before] = (b << 2) | nb;
    }
    __syncthreads();
    if (t == 255) {
      s_carry_rs = v;
      int tot = 0;
      for (int w = 0; w < 8; ++w) tot += s_sum[w];
      s_carry_cnt += tot;
    }
    __syncthreads();
  }
  if (t == 0) seg_tab[0] = s_carry_cnt;
}

// Item index type: 32-bit when num_sorted * gpr_p < 2^31 (the divisions by
// gpr_p and bs per item are then 32-bit), else 64-bit.
template <int kDtype, typename Idx>
__global__ void __launch_bounds__(256)
moe_gather_quant_kernel(const uint16_t* __restrict__ a, int64_t lda, const int32_t* __restrict__ sorted_ids,
                        const int32_t* __restrict__ expert_ids, const int32_t* __restrict__ num_post_padded,
                        int64_t num_sorted, int bs, int na, int top_k, int n_slots, int num_experts, int K,
                        int kchunks, uint8_t* __restrict__ codes, uint8_t* __restrict__ sf,
                        int32_t* __restrict__ seg_tab) {
  // Every scale byte the GEMM reads is written here, the padding groups past
  // K / 32 (up to kchunks * 4 per row, one K-256 stage) as E8M0 0 (2^-127):
  // the workspace may hold stale bytes, and a stale 0xFF (NaN) would turn the
  // padding's zero codes into NaN products.
  const int gpr = K / 32;
  const Idx gpr_p = static_cast<Idx>(kchunks) * 4;
  const Idx total = static_cast<Idx>(num_sorted) * gpr_p;
  const int npp = __ldg(num_post_padded);
  if (blockIdx.x == 0) {
    const int64_t nb = num_sorted / bs;
    const int64_t live = npp <= 0 ? 0 : (static_cast<int64_t>(npp) + bs - 1) / bs;
    moe_segments(expert_ids, static_cast<int>(live < nb ? live : nb), num_experts, seg_tab);
  }
  for (Idx it = static_cast<Idx>(blockIdx.x) * blockDim.x + threadIdx.x; it < total;
       it += static_cast<Idx>(gridDim.x) * blockDim.x) {
    const Idx p = it / gpr_p;
    const int g = static_cast<int>(it - p * gpr_p);
    const int s = p < static_cast<Idx>(max(npp, 0)) ? __ldg(sorted_ids + p) : -1;
    uint32_t code[4] = {0u, 0u, 0u, 0u};
    int e = 0;
    if (g < gpr && s >= 0 && s < n_slots) {
      const uint4* src = reinterpret_cast<const uint4*>(a + static_cast<int64_t>(s / top_k) * lda + g * 32);
      uint4 v[4] = {src[0], src[1], src[2], src[3]};
      e = mx_group_codes<kDtype>(v, code);
    }
    if (g < gpr)
      *reinterpret_cast<uint4*>(codes + static_cast<int64_t>(p) * (K / 2) + g * 16) =
          make_uint4(code[0], code[1], code[2], code[3]);
    const Idx b = p / static_cast<Idx>(bs);
    const int r = static_cast<int>(p - b * static_cast<Idx>(bs));
    // row r of block b sits at segment row na*i + r of the chunk of block b - i
#pragma unroll
    for (int i = 0; i < MOE_SEG_MAX; ++i) {
      const int row = i * na + r;
      if (row >= 128 || b < static_cast<Idx>(i)) break;
      sf[(static_cast<int64_t>(b - i) * kchunks + g / 4) * 512 + (row & 31) * 16 + (row >> 5) * 4 + (g & 3)] =
          static_cast<uint8_t>(e);
    }
  }
}

template <int kNA>
struct MLayout {
  static constexpr int A_TILE = kNA * DBKB;  // one block's codes per stage
  static constexpr int ST_W = 0, ST_A = W_TILE, ST_SFW = ST_A + MOE_SEG_MAX * A_TILE, ST_SFA = ST_SFW + SF_STAGE;
  static constexpr int STAGE = (ST_SFA + 2 * SF_STAGE + 1023) / 1024 * 1024;
  static constexpr int STAGES = kNA == 64 ? 5 : (kNA == 32 ? 7 : 8);
};
struct __align__(8) MBars {
  uint64_t full[8];       // W, the segment's codes and the scale chunks landed (1 arrival + tx)
  uint64_t empty[8];      // the stage's MMAs completed
  uint64_t acc_full[2];   // MMA -> epilogue, per accumulator buffer
  uint64_t acc_empty[2];  // epilogue -> MMA (256 arrivals)
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};
template <int kNA>
constexpr size_t m_smem_bytes() {
  return 1024 + static_cast<size_t>(MLayout<kNA>::STAGES) * MLayout<kNA>::STAGE + sizeof(MBars);
}
static_assert(m_smem_bytes<16>() <= 227 * 1024 && m_smem_bytes<32>() <= 227 * 1024 &&
              m_smem_bytes<64>() <= 227 * 1024, "MoE stages exceed shared memory");
// TMEM of the MoE kernel: two accumulators of MOE_SEG_MAX x 64 columns, the
// W scales (4 columns per K chunk) and the segment scales (8 columns per K
// chunk: rows 0-127, then 128-255).
constexpr uint32_t M_ACC = 0, M_ACC_STRIDE = 64 * MOE_SEG_MAX, M_SFW = 2 * M_ACC_STRIDE, M_SFA = M_SFW + 8,
                   M_TMEM_COLS = 512;
static_assert(M_SFA + 16 <= M_TMEM_COLS, "MoE TMEM columns");
constexpr int M_EPI_WARPS = 8;
constexpr int M_THREADS = 32 * (2 + M_EPI_WARPS);

// Persistent: CTA c takes work items c, c + gridDim.x, ...; item i is segment
// i / n_tiles against 128-row W tile i % n_tiles, so the CTAs in flight cover
// every W tile of a few consecutive segments: each W tile of an expert streams
// from HBM once while its segments' codes stay in L2.  The stage ring runs across
// items and the accumulator is double-buffered, so an item's epilogue overlaps
// the next item's MMAs.
template <int kDtype, int kNA>
__global__ void __launch_bounds__(M_THREADS, 1)
mxf4_moe_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_a,
                const uint8_t* __restrict__ sfw, int64_t sf_per_expert, const uint8_t* __restrict__ sfa,
                const int32_t* __restrict__ seg_tab, const int32_t* __restrict__ sorted_ids,
                const int32_t* __restrict__ expert_ids, const float* __restrict__ topk_w, int mul_topk, int top_k,
                int bs, int num_blocks, int num_experts, void* __restrict__ c_v, int64_t ldc, int size_m, int N, int K, int kchunks, int* status) {
  using Lay = MLayout<kNA>;
  constexpr int S = Lay::STAGES;
  constexpr bool kF16 = kDtype == QDQ_DTYPE_FP16;
  using O = DOut<kF16>;
  using T = typename O::T;
  T* C = static_cast<T*>(c_v);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  MBars* bars = reinterpret_cast<MBars*>(smem + S * Lay::STAGE);
  const int warp = threadIdx.x >> 5;
  const int num_kt = (K + DBK - 1) / DBK;
  const int n_slots = size_m * top_k;
  const int nseg = min(max(seg_tab[0], 0), num_blocks);
  const int n_tiles = (N + DBM - 1) / DBM;
  const int num_items = nseg * n_tiles;
  // A segment entry every role decodes alike; a malformed one is skipped.
  auto seg_of = [&](int item, int& blk0, int& nb, int& e) -> bool {
    const int seg = seg_tab[1 + item / n_tiles];
    blk0 = seg >> 2;
    nb = seg & 3;
    if (blk0 < 0 || nb < 1 || blk0 + nb > num_blocks) return false;
    e = __ldg(expert_ids + blk0);
    return e >= 0 && e < num_experts;
  };

  if (threadIdx.x == 0) {
    for (int st = 0; st < S; ++st) {
      mbar_init(&bars->full[st], 1);
      mbar_init(&bars->empty[st], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->acc_full[i], 1);
      mbar_init(&bars->acc_empty[i], 32 * M_EPI_WARPS);
    }
    mbar_init(&bars->drain, 1);
    bars->abort = 0;
    fence_barrier_init();
    prefetch_tmap(&tmap_w);
    prefetch_tmap(&tmap_a);
  }
  if (warp == 0) {
    tmem_alloc(&bars->tmem_base, M_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0) {
    // ---------------- producer: W_e tile, the segment's codes and scale chunks
    if (elect_one()) {
      int it = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < num_items; item += gridDim.x) {
        int blk0, nb, e;
        if (!seg_of(item, blk0, nb, e)) continue;
        const int n_tile = item % n_tiles;
        const int64_t w_row0 = static_cast<int64_t>(e) * N + static_cast<int64_t>(n_tile) * DBM;
        const uint8_t* sfw_e = sfw + e * sf_per_expert + static_cast<int64_t>(n_tile) * kchunks * 512;
        for (int kt = 0; kt < num_kt; ++kt, ++it) {
          const int st = it % S;
          if (!mbar_wait(&bars->empty[st], ((it / S) & 1) ^ 1, status, 0x501)) {
            bars->abort = 1;
            ok = false;
            break;
          }
          if (*(volatile int*)&bars->abort) { ok = false; break; }
          uint8_t* sp = smem + st * Lay::STAGE;
          const bool wide = kNA * nb > 128;
          mbar_arrive_expect_tx(&bars->full[st],
                                W_TILE + nb * Lay::A_TILE + (wide ? 3 : 2) * SF_STAGE);
          tma_load_2d(sp + Lay::ST_W, &tmap_w, kt * DBKB, static_cast<int32_t>(w_row0), &bars->full[st]);
          bulk_load(sp + Lay::ST_SFW, sfw_e + 2 * kt * 512, SF_STAGE, &bars->full[st]);
          for (int i = 0; i < nb; ++i)
            tma_load_2d(sp + Lay::ST_A + i * Lay::A_TILE, &tmap_a, kt * DBKB, (blk0 + i) * bs, &bars->full[st]);
          bulk_load(sp + Lay::ST_SFA, sfa + (static_cast<int64_t>(blk0) * kchunks + 2 * kt) * 512, SF_STAGE,
                    &bars->full[st]);
          if (wide)  // segment rows 128-191: block blk0 + 2's chunk
            bulk_load(sp + Lay::ST_SFA + SF_STAGE, sfa + (static_cast<int64_t>(blk0 + 2) * kchunks + 2 * kt) * 512,
                      SF_STAGE, &bars->full[st]);
        }
      }
      for (int j = (it > S ? it - S : 0); j < it; ++j)
        mbar_wait(&bars->full[j % S], (j / S) & 1, status, 0x502);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (elect_one()) {
      int it = 0, j = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < num_items; item += gridDim.x) {
        int blk0, nb, e;
        if (!seg_of(item, blk0, nb, e)) continue;
        const uint32_t idesc = idesc_mxf4(DBM, kNA * nb, true);  // N = the segment's rows
        const bool wide = kNA * nb > 128;
        const int buf = j & 1;
        // the epilogue has read this buffer's previous item out of TMEM
        if (!mbar_wait(&bars->acc_empty[buf], ((j >> 1) & 1) ^ 1, status, 0x506)) { ok = false; break; }
        tc_fence_after();
        const uint32_t acc = tmem + M_ACC + M_ACC_STRIDE * buf;
        for (int kt = 0; kt < num_kt; ++kt, ++it) {
          const int st = it % S;
          if (!mbar_wait(&bars->full[st], (it / S) & 1, status, 0x503)) { ok = false; break; }
          if (*(volatile int*)&bars->abort) { ok = false; break; }
          tc_fence_after();
          uint8_t* sp = smem + st * Lay::STAGE;
          tmem_cp_sf(tmem + M_SFW + 0, smem_desc_sf(sp + Lay::ST_SFW));
          tmem_cp_sf(tmem + M_SFW + 4, smem_desc_sf(sp + Lay::ST_SFW + 512));
          tmem_cp_sf(tmem + M_SFA + 0, smem_desc_sf(sp + Lay::ST_SFA));        // K chunk 0, rows 0-127
          tmem_cp_sf(tmem + M_SFA + 8, smem_desc_sf(sp + Lay::ST_SFA + 512));  // K chunk 1, rows 0-127
          if (wide) {
            tmem_cp_sf(tmem + M_SFA + 4, smem_desc_sf(sp + Lay::ST_SFA + 1024));   // K chunk 0, rows 128-191
            tmem_cp_sf(tmem + M_SFA + 12, smem_desc_sf(sp + Lay::ST_SFA + 1536));  // K chunk 1
          }
          const uint64_t dw = smem_desc_sw128(sp + Lay::ST_W);
          const uint64_t da = smem_desc_sw128(sp + Lay::ST_A);
#pragma unroll
          for (int kk = 0; kk < DBK / 64; ++kk) {
            const uint32_t jj = kk >> 1, sf_id = (kk & 1) * 2;
            mma_mxf4(acc, dw + ((kk * 32) >> 4), da + ((kk * 32) >> 4), idesc_with_sf_ids(idesc, sf_id, sf_id),
                     (tmem + M_SFW + 4 * jj) | (sf_id << 30), (tmem + M_SFA + 8 * jj) | (sf_id << 30),
                     (kt | kk) != 0);
          }
          tc_commit(&bars->empty[st]);
        }
        if (!ok) break;
        tc_commit(&bars->acc_full[buf]);
        ++j;
      }
      if (!ok) bars->abort = 1;
      tc_commit(&bars->drain);
      mbar_wait(&bars->drain, 0, status, 0x507);
    }
  } else {
    // ---------------- epilogue: TMEM lanes = W rows, columns = the segment's slots
    // Eight warps: warp w reads TMEM lanes 32 (w % 4).. and the 32-column
    // chunks c = half, half + 2, half + 4 of the segment's NA * nb columns.
    const int lane = threadIdx.x & 31;
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    constexpr int CH = (64 * MOE_SEG_MAX / 32 + 1) / 2;  // chunks per warp at most
    bool ok = true;
    int j = 0;
    for (int item = blockIdx.x; item < num_items; item += gridDim.x) {
      int blk0, nb, e;
      if (!seg_of(item, blk0, nb, e)) continue;
      const int n_tile = item % n_tiles;
      const int nchunks = (kNA * nb + 31) / 32;
      // Routing of this warp's columns, fetched while the MMAs run: lane l
      // holds the slot of column 32 c + l (-1 for padding) and its weight.
      int slot[CH];
      float wt[CH];
#pragma unroll
      for (int t = 0; t < CH; ++t) {
        const int col = 32 * (half + 2 * t) + lane;
        const int i = col / kNA, r = col % kNA;
        int s = (i < nb && r < bs) ? __ldg(sorted_ids + static_cast<int64_t>(blk0 + i) * bs + r) : -1;
        if (s >= n_slots) s = -1;
        slot[t] = s;
        wt[t] = (mul_topk && s >= 0) ? __ldg(topk_w + s) : 1.0f;
      }
      const int buf = j & 1;
      if (ok) ok = mbar_wait(&bars->acc_full[buf], (j >> 1) & 1, status, 0x505);
      ok = __all_sync(0xffffffffu, ok);
      tc_fence_after();
      const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16) + M_ACC + M_ACC_STRIDE * buf;
      const int n = n_tile * DBM + q * 32 + lane;
      const bool in_n = n < N;
      // warp-uniform: every lane takes part in the shuffles below
      const bool store = __all_sync(0xffffffffu, ok && !*(volatile int*)&bars->abort);
      if (half >= nchunks) {
        tc_fence_before();
        mbar_arrive(&bars->acc_empty[buf]);
      }
#pragma unroll
      for (int t = 0; t < CH; ++t) {
        const int c = half + 2 * t;
        if (c >= nchunks) break;
        uint32_t r[32];
        tmem_ld32(taddr + 32 * c, r);
        tmem_ld_wait();
        if (c + 2 >= nchunks) {  // this warp's last chunk of the item
          tc_fence_before();
          mbar_arrive(&bars->acc_empty[buf]);  // the next item on this buffer may start
        }
        if (!store) continue;
#pragma unroll
        for (int l = 0; l < 32; ++l) {
          const int s = __shfl_sync(0xffffffffu, slot[t], l);
          const float w = __shfl_sync(0xffffffffu, wt[t], l);
          if (s >= 0 && in_n) C[static_cast<int64_t>(s) * ldc + n] = O::one(__uint_as_float(r[l]) * w);
        }
      }
      ++j;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, M_TMEM_COLS);
  }
}

template <int kDtype, int kNA>
int launch_moe(const CUtensorMap& tw, const CUtensorMap& ta, const uint8_t* sf, int64_t sf_per_expert,
               const uint8_t* sfa, const int32_t* seg_tab, const int32_t* sorted_ids, const int32_t* expert_ids,
               const float* topk_w, int mul, int top_k, int bs, int64_t num_blocks, int num_experts, void* c,
               int64_t ldc,
               int64_t size_m, int64_t N, int64_t K, int kchunks, int* status, cudaStream_t s) {
  constexpr size_t smem = m_smem_bytes<kNA>();
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(&mxf4_moe_kernel<kDtype, kNA>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return fail(QDQ_ERR_CUDA, "fp4_moe_mxf4: smem attribute: %s", cudaGetErrorString(e));
    attr_set[dev] = true;
  }
  // at most one segment per block; the kernel reads the actual count
  const int64_t items = num_blocks * ((N + DBM - 1) / DBM);
  const int sms = device_sm_count();
  dim3 grid(static_cast<unsigned>(std::min<int64_t>(items, sms > 0 ? sms : 148)));
  mxf4_moe_kernel<kDtype, kNA><<<grid, M_THREADS, smem, s>>>(
      tw, ta, sf, sf_per_expert, sfa, seg_tab, sorted_ids, expert_ids, topk_w, mul, top_k, bs,
      static_cast<int>(num_blocks), num_experts, c, ldc,
      static_cast<int>(size_m), static_cast<int>(N), static_cast<int>(K), kchunks, status);
  return check_launch("fp4_moe_mxf4");
}

}  // namespace

// Host entry used by fp4_linear_mxf4 for M <= 64 (declared in common.cuh).
// Small-M fused linear, MXFP4 (nv == false) or NVFP4 (nv: E4M3 weight scales
// per 16 with tensor scale w_gs; the activation quantised with the device
// scalar *a_gs).  One launch.
static int decode_common(const void* a, int64_t lda, int dtype, const void* w_codes, const void* w_sf_tiled,
                         const void* bias, void* c, int64_t M, int64_t N, int64_t K, int64_t ldw_bytes,
                         int64_t ldc, bool nv, const float* a_gs, float w_gs, void* stream) {
  if (M < 1 || M > NA_MAX) return fail(QDQ_ERR_INVALID_ARG, "fp4_linear_decode: M must be in [1, 64]");
  if ((reinterpret_cast<uintptr_t>(a) & 15) || ((lda * 2) & 15))
    return fail(QDQ_ERR_ALIGNMENT, "fp4_linear_decode: activation rows must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(w_sf_tiled) & 15)
    return fail(QDQ_ERR_ALIGNMENT, "fp4_linear_decode: scale-factor buffer must be 16-byte aligned");
  int* status = device_status_ptr();
  if (status == nullptr) return QDQ_ERR_CUDA;
  const int na = M <= 16 ? 16 : (M <= 32 ? 32 : 64);
  CUtensorMap tw, ta;
  if (int st = make_tmap_u8_2d(&tw, w_codes, N, K / 2, ldw_bytes, DBKB, DBM, 128)) return st;
  if (int st = make_tmap_u16_2d(&ta, a, M, K, lda * 2, DBK, na)) return st;
  // 512-byte chunks of 4 scales per 128 rows, scales per row padded to one K-256 stage
  const int kchunks = nv ? static_cast<int>(((K / 16) + 15) / 16 * 16 / 4)
                         : static_cast<int>(((K / 32) + 7) / 8 * 8 / 4);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto* sf = static_cast<const uint8_t*>(w_sf_tiled);
  const bool f16 = dtype == QDQ_DTYPE_FP16;
#define QDQ_DECODE(NA, NV)                                                                                  \
  return f16 ? launch_decode<QDQ_DTYPE_FP16, NA, NV>(tw, ta, sf, bias, c, M, N, K, ldc, kchunks, a_gs, w_gs, \
                                                      a, lda, status, s)                                      \
             : launch_decode<QDQ_DTYPE_BF16, NA, NV>(tw, ta, sf, bias, c, M, N, K, ldc, kchunks, a_gs, w_gs, \
                                                      a, lda, status, s);
  if (nv) {
    if (na == 16) { QDQ_DECODE(16, true) }
    if (na == 32) { QDQ_DECODE(32, true) }
    QDQ_DECODE(64, true)
  }
  if (na == 16) { QDQ_DECODE(16, false) }
  if (na == 32) { QDQ_DECODE(32, false) }
  QDQ_DECODE(64, false)
#undef QDQ_DECODE
}

int fp4_linear_decode(const void* a, int64_t lda, int dtype, const void* w_codes, const void* w_sf_tiled,
                      const void* bias, void* c, int64_t M, int64_t N, int64_t K, int64_t ldw_bytes,
                      int64_t ldc, void* stream) {
  return decode_common(a, lda, dtype, w_codes, w_sf_tiled, bias, c, M, N, K, ldw_bytes, ldc, false, nullptr, 0.f,
                       stream);
}

int fp4_linear_decode_nvf4(const void* a, int64_t lda, int dtype, const float* a_gs, const void* w_codes,
                           const void* w_sf_tiled, float w_gs, const void* bias, void* c, int64_t M, int64_t N,
                           int64_t K, int64_t ldw_bytes, int64_t ldc, void* stream) {
  return decode_common(a, lda, dtype, w_codes, w_sf_tiled, bias, c, M, N, K, ldw_bytes, ldc, true, a_gs, w_gs,
                       stream);
}

}  // namespace qdqb200

using namespace qdqb200;

static int64_t moe_kchunks(int64_t K) { return ((K / 32) + 7) / 8 * 8 / 4; }

extern "C" int64_t fp4_moe_workspace_bytes(int64_t num_sorted, int moe_block_size, int64_t K) {
  if (num_sorted <= 0 || moe_block_size <= 0 || K <= 0) return 0;
  auto up = [](int64_t v) { return (v + 255) / 256 * 256; };
  const int64_t blocks = (num_sorted + moe_block_size - 1) / moe_block_size;
  return up(num_sorted * ((K + 31) / 32 * 16)) + up(blocks * moe_kchunks(K) * 512) + up(4 * (blocks + 1));
}

extern "C" int fp4_moe_mxf4(const void* a, int64_t lda, int dtype, const void* w_codes, const void* w_sf_tiled,
                            int64_t num_experts, const int32_t* sorted_token_ids, const int32_t* expert_ids,
                            const int32_t* num_tokens_post_padded, const float* topk_weights, int64_t num_sorted,
                            int moe_block_size, int top_k, int mul_topk_weights, void* c, int64_t ldc,
                            int64_t size_m, int64_t N, int64_t K, void* workspace, int64_t workspace_bytes,
                            void* stream) {
  if (dtype != QDQ_DTYPE_BF16 && dtype != QDQ_DTYPE_FP16)
    return fail(QDQ_ERR_INVALID_ARG, "fp4_moe_mxf4: dtype must be bf16 (0) or fp16 (1)");
  if (size_m < 0 || N < 0 || K < 0 || num_sorted < 0 || num_experts < 0)
    return fail(QDQ_ERR_INVALID_ARG, "fp4_moe_mxf4: negative size");
  if (moe_block_size < 1 || moe_block_size > NA_MAX)
    return fail(QDQ_ERR_UNSUPPORTED, "fp4_moe_mxf4: moe_block_size must be in [1, 64] (got %d)", moe_block_size);
  if (top_k < 1) return fail(QDQ_ERR_INVALID_ARG, "fp4_moe_mxf4: top_k must be >= 1");
  if (size_m == 0 || N == 0 || num_sorted == 0 || num_experts == 0) return QDQ_OK;
  if (K == 0 || K % 32 != 0)
    return fail(QDQ_ERR_UNSUPPORTED, "fp4_moe_mxf4: K=%lld must be a positive multiple of 32", (long long)K);
  if (!a || !w_codes || !w_sf_tiled || !sorted_token_ids || !expert_ids || !num_tokens_post_padded || !c ||
      (mul_topk_weights && !topk_weights))
    return fail(QDQ_ERR_INVALID_ARG, "fp4_moe_mxf4: null pointer");
  if (lda < K || ldc < N) return fail(QDQ_ERR_INVALID_ARG, "fp4_moe_mxf4: leading dimension too small");
  if ((reinterpret_cast<uintptr_t>(a) & 15) || ((lda * 2) & 15) || (reinterpret_cast<uintptr_t>(w_sf_tiled) & 15))
    return fail(QDQ_ERR_ALIGNMENT, "fp4_moe_mxf4: activation rows and scale buffer must be 16-byte aligned");
  if (num_experts * N > (1ll << 31) || size_m * top_k > (1ll << 31) || num_sorted > (1ll << 31))
    return fail(QDQ_ERR_UNSUPPORTED, "fp4_moe_mxf4: too many rows");
  if (workspace == nullptr || workspace_bytes < fp4_moe_workspace_bytes(num_sorted, moe_block_size, K) ||
      (reinterpret_cast<uintptr_t>(workspace) & 255))
    return fail(QDQ_ERR_INVALID_ARG, "fp4_moe_mxf4: workspace missing, unaligned or smaller than "
                                     "fp4_moe_workspace_bytes()");
  int* status = device_status_ptr();
  if (status == nullptr) return QDQ_ERR_CUDA;
  const int kchunks = static_cast<int>(moe_kchunks(K));
  const int64_t num_blocks = num_sorted / moe_block_size;
  if (num_blocks == 0) return QDQ_OK;
  auto up = [](int64_t v) { return (v + 255) / 256 * 256; };
  uint8_t* a_codes = static_cast<uint8_t*>(workspace);
  uint8_t* a_sf = a_codes + up(num_sorted * (K / 2));
  const int64_t sf_blocks = (num_sorted + moe_block_size - 1) / moe_block_size;  // the gather writes a tail block
  int32_t* seg_tab = reinterpret_cast<int32_t*>(a_sf + up(sf_blocks * kchunks * 512));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto* ap = static_cast<const uint16_t*>(a);
  const int na = moe_block_size <= 16 ? 16 : (moe_block_size <= 32 ? 32 : 64);  // the GEMM's rows per block
  // 1) gather + quantise the routed rows in sorted order (zero at padding)
  {
    const int64_t items = num_sorted * (K / 32);
    const int grid = static_cast<int>(std::min<int64_t>((items + 255) / 256, static_cast<int64_t>(device_sm_count()) * 8));
    // 32-bit items while the last grid-stride step cannot wrap
    const bool narrow = num_sorted * kchunks * 4 < (int64_t(1) << 31);
#define QDQ_MOE_GATHER(DT, IDX)                                                                                  \
  moe_gather_quant_kernel<DT, IDX><<<grid, 256, 0, s>>>(                                                         \
      ap, lda, sorted_token_ids, expert_ids, num_tokens_post_padded, num_sorted, moe_block_size, na, top_k,      \
      static_cast<int>(size_m * top_k), static_cast<int>(num_experts), static_cast<int>(K), kchunks, a_codes, a_sf, \
      seg_tab)
    if (dtype == QDQ_DTYPE_FP16) {
      if (narrow) QDQ_MOE_GATHER(QDQ_DTYPE_FP16, uint32_t);
      else QDQ_MOE_GATHER(QDQ_DTYPE_FP16, int64_t);
    } else {
      if (narrow) QDQ_MOE_GATHER(QDQ_DTYPE_BF16, uint32_t);
      else QDQ_MOE_GATHER(QDQ_DTYPE_BF16, int64_t);
    }
#undef QDQ_MOE_GATHER
    if (int st = check_launch("fp4_moe_mxf4 (gather)")) return st;
  }
  // 2) grouped GEMM
  CUtensorMap tw, ta;
  if (int st = make_tmap_u8_2d(&tw, w_codes, num_experts * N, K / 2, K / 2, DBKB, DBM, 128)) return st;
  if (int st = make_tmap_u8_2d(&ta, a_codes, num_sorted, K / 2, K / 2, DBKB, na, 128)) return st;
  const int64_t sf_per_expert = qdq_sf_tiled_bytes(N, K);
  auto* sf = static_cast<const uint8_t*>(w_sf_tiled);
#define QDQ_MOE_LAUNCH(DT, NA)                                                                                  \
  return launch_moe<DT, NA>(tw, ta, sf, sf_per_expert, a_sf, seg_tab, sorted_token_ids, expert_ids, topk_weights, \
                            mul_topk_weights, top_k, moe_block_size, num_blocks, static_cast<int>(num_experts), c, \
                            ldc, size_m, N, K, kchunks,                                                          \
                            status, s)
  if (dtype == QDQ_DTYPE_FP16) {
    if (na == 16) QDQ_MOE_LAUNCH(QDQ_DTYPE_FP16, 16);
    if (na == 32) QDQ_MOE_LAUNCH(QDQ_DTYPE_FP16, 32);
    QDQ_MOE_LAUNCH(QDQ_DTYPE_FP16, 64);
  }
  if (na == 16) QDQ_MOE_LAUNCH(QDQ_DTYPE_BF16, 16);
  if (na == 32) QDQ_MOE_LAUNCH(QDQ_DTYPE_BF16, 32);
  QDQ_MOE_LAUNCH(QDQ_DTYPE_BF16, 64);
#undef QDQ_MOE_LAUNCH
}
