// Sage3 FP4 flash attention on sm_100a tensor cores, D = 128, one 128-row
// query tile per CTA.  MXFP4 (E2M1 + E8M0 per 32, tcgen05 kind::mxf4) or
// NVFP4 (E2M1 + E4M3 per 16, kind::mxf4nvf4 block16).
//
// Reference semantics: the mxfp4_hw kernel (sage3/mxfp4_hw_kernel.py:167-393)
//   S  = dot_scaled(Q, K^T) (+ delta_s[group of the query tile, key]),
//   online softmax in base 2 with qk_scale = sm_scale * log2(e),
//   l += sum of the unquantised p,
//   P quantised per row and 32 keys: e = clamp(ceil(log2(max(p)/6)), -127, 127),
//     codes = cvt.rn.satfinite.e2m1x2(p * 2^-e),
//   O += dot_scaled(P, V), O / l at the end.
// Keys beyond L are masked (the reference attends to its zero padding; see
// DESIGN.md for the size of that difference).
//
// CTA (10 warps):
//   warp 0        TMA producer: K tile [128 keys x 64 B], V^T tile [128 d x 64 B]
//                 (64-byte swizzle), their E8M0 chunks and the delta_s row slice
//                 into a 4-stage ring; the Q tile once
//   warp 1        MMA issuer: S[j%2] = Q K_j^T (tcgen05.mma kind::mxf4, 2 x K=64),
//                 then O += P_{j-1} V_{j-1}; scale factors via tcgen05.cp
//   warps 2-9     softmax, two threads per query row (TMEM lane), 64 keys each:
//                 S -> registers, + delta_s, row max (partner exchange through
//                 shared memory), O rescale in TMEM when the max grows, exp2, row
//                 sum, P -> E2M1 codes + E8M0 scales in shared memory;
//                 epilogue O / l -> bf16 NHD
// TMEM: S0 [0,128) S1 [128,256) O [256,384) scale factors [384,400).
#include "attn_common.cuh"

namespace qdqb200 {
namespace attn {
namespace {

using namespace sm100;

constexpr int BM = 128, BN = 128, HD = 128;
constexpr int STAGES = 4;
constexpr int CODE_TILE = 128 * 64;  // 8 KB: 128 rows x 128 E2M1
constexpr int SF_CHUNK = 512;
constexpr int SF_TILE = 1024;        // scale bytes per 128-row tile in global memory (two chunks)
constexpr int DS_BYTES = BN * 2;
// stage: K codes | V codes | K sf | V sf | delta_s (bf16)
constexpr int ST_K = 0, ST_V = CODE_TILE, ST_KSF = 2 * CODE_TILE, ST_VSF = ST_KSF + SF_TILE,
              ST_DS = ST_VSF + SF_TILE;
constexpr int STAGE_BYTES = 19 * 1024;
static_assert(ST_DS + DS_BYTES <= STAGE_BYTES, "stage layout");
// CTA smem: Q codes | P codes | stages | Q sf | P sf | barriers
constexpr int OFF_Q = 0, OFF_P = CODE_TILE, OFF_STAGE = 2 * CODE_TILE;
constexpr int OFF_QSF = OFF_STAGE + STAGES * STAGE_BYTES;
constexpr int OFF_PSF = OFF_QSF + SF_TILE;
constexpr int OFF_RED = OFF_PSF + SF_TILE;              // [3][2][128] floats: row max / row sum exchange
constexpr int OFF_BAR = OFF_RED + 3 * 2 * 128 * 4;
constexpr int THREADS = 320;                             // producer, MMA, 8 softmax warps
constexpr int TMEM_COLS = 512;
// scale-factor columns: 8 per operand (NVFP4: two chunks; MXFP4 uses the first 4)
constexpr uint32_t T_S0 = 0, T_O = 256, T_SFQ = 384, T_SFK = 392, T_SFP = 400, T_SFV = 408;
static_assert(HD == BN, "PV uses the same instruction shape as QK");

struct Bars {
  uint64_t q_full;
  uint64_t kv_full[STAGES];
  uint64_t kv_empty[STAGES];
  uint64_t s_full[2];
  uint64_t s_free[2];
  uint64_t p_full;
  uint64_t o_done;
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};
constexpr size_t SMEM_BYTES = 1024 + OFF_BAR + sizeof(Bars);

struct Params {
  int H, L, Lp, T;  // T = Lp / 128
  int64_t o_sb, o_sn, o_sh;
  float qk_scale;   // sm_scale * log2(e)
  int causal;
  int smoothing;
  float p_prescale;  // 1, or 448*6 for the reference's emulated configs
  int l_quant;       // l = sum of quantised P (emulated configs) instead of unquantised p
};

// Sum of the eight E2M1 values packed in a 32-bit word (exact in fp16).
__device__ __forceinline__ float e2m1_word_sum(uint32_t w) {
  __half2 acc = __floats2half2_rn(0.f, 0.f);
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    const uint32_t h = e2m1x2_to_f16x2((w >> (8 * b)) & 0xFFu);
    acc = __hadd2(acc, *reinterpret_cast<const __half2*>(&h));
  }
  return __low2float(acc) + __high2float(acc);
}

// Issue the two K=64 block-scaled MMAs of a 128 x 128 x 128 product.
template <bool kNV>
__device__ __forceinline__ void mma_k128(uint32_t d, uint64_t da, uint64_t db, uint32_t sfa, uint32_t sfb,
                                         bool accumulate_first) {
  constexpr uint32_t idesc = idesc_mxf4(BM, BN, !kNV);
#pragma unroll
  for (int kk = 0; kk < 2; ++kk) {
    if (kNV) {  // UE4M3 per 16: MMA kk reads scale chunk kk (4 scales per row)
      mma_nvf4(d, da + kk * 2, db + kk * 2, idesc, sfa + 4 * kk, sfb + 4 * kk, accumulate_first || kk);
    } else {    // UE8M0 per 32: scale bytes 2kk, 2kk+1 of the chunk
      const uint32_t sf_id = kk * 2;
      mma_mxf4(d, da + kk * 2, db + kk * 2, idesc_with_sf_ids(idesc, sf_id, sf_id), sfa | (sf_id << 30),
               sfb | (sf_id << 30), accumulate_first || kk);
    }
  }
}
template <bool kNV>
__device__ __forceinline__ void cp_sf(uint32_t taddr, const uint8_t* smem_sf) {
  tmem_cp_sf(taddr, smem_desc_sf(smem_sf));
  if (kNV) tmem_cp_sf(taddr + 4, smem_desc_sf(smem_sf + SF_CHUNK));
}

template <bool kNV>
__global__ void __launch_bounds__(THREADS, 1)
sage3_fp4_flash_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                         const __grid_constant__ CUtensorMap map_v, const uint8_t* __restrict__ qsf,
                         const uint8_t* __restrict__ ksf, const uint8_t* __restrict__ vsf,
                         const __nv_bfloat16* __restrict__ ds, __nv_bfloat16* __restrict__ out, Params p,
                         int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + OFF_BAR);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int qt = blockIdx.x;       // query tile
  const int bh = blockIdx.y;
  const int G = p.T;
  const int nkv = p.causal ? qt + 1 : p.T;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bars->kv_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->s_free[i], 256);
    }
    mbar_init(&bars->p_full, 256);
    mbar_init(&bars->o_done, 1);
    mbar_init(&bars->drain, 1);
    bars->abort = 0;
    fence_barrier_init();
    prefetch_tmap(&map_q);
    prefetch_tmap(&map_k);
    prefetch_tmap(&map_v);
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
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      constexpr int kSfBytes = kNV ? SF_TILE : SF_CHUNK;
      mbar_arrive_expect_tx(&bars->q_full, CODE_TILE + kSfBytes);
      tma_load_2d(smem + OFF_Q, &map_q, 0, bh * p.Lp + qt * BM, &bars->q_full);
      bulk_load(smem + OFF_QSF, qsf + (static_cast<int64_t>(bh) * p.T + qt) * SF_TILE, kSfBytes, &bars->q_full);
      int issued = 0;
      for (int j = 0; j < nkv; ++j) {
        const int s = j % STAGES;
        if (!mbar_wait(&bars->kv_empty[s], ((j / STAGES) & 1) ^ 1, status, 0x1101)) {
          bars->abort = 1;
          break;
        }
        if (*(volatile int*)&bars->abort) break;
        uint8_t* st = smem + OFF_STAGE + s * STAGE_BYTES;
        const uint32_t bytes = 2 * CODE_TILE + 2 * kSfBytes + (p.smoothing ? DS_BYTES : 0);
        mbar_arrive_expect_tx(&bars->kv_full[s], bytes);
        tma_load_2d(st + ST_K, &map_k, 0, bh * p.Lp + j * BN, &bars->kv_full[s]);
        tma_load_2d(st + ST_V, &map_v, j * (BN / 2), bh * HD, &bars->kv_full[s]);
        bulk_load(st + ST_KSF, ksf + (static_cast<int64_t>(bh) * p.T + j) * SF_TILE, kSfBytes, &bars->kv_full[s]);
        bulk_load(st + ST_VSF, vsf + (static_cast<int64_t>(bh) * p.T + j) * SF_TILE, kSfBytes, &bars->kv_full[s]);
        if (p.smoothing)
          bulk_load(st + ST_DS, ds + (static_cast<int64_t>(bh) * G + qt) * p.Lp + j * BN, DS_BYTES,
                    &bars->kv_full[s]);
        ++issued;
      }
      mbar_wait(&bars->q_full, 0, status, 0x1102);
      for (int j = (issued > STAGES ? issued - STAGES : 0); j < issued; ++j)
        mbar_wait(&bars->kv_full[j % STAGES], (j / STAGES) & 1, status, 0x1103);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      bool ok = mbar_wait(&bars->q_full, 0, status, 0x1201);
      if (ok) {
        tc_fence_after();
        cp_sf<kNV>(tmem + T_SFQ, smem + OFF_QSF);
      }
      const uint64_t dq = smem_desc_sw64(smem + OFF_Q);
      const uint64_t dp = smem_desc_sw64(smem + OFF_P);
      auto issue_pv = [&](int t) -> bool {
        const int s = t % STAGES;
        if (!mbar_wait(&bars->p_full, t & 1, status, 0x1202)) return false;
        tc_fence_after();
        uint8_t* st = smem + OFF_STAGE + s * STAGE_BYTES;
        cp_sf<kNV>(tmem + T_SFP, smem + OFF_PSF);
        cp_sf<kNV>(tmem + T_SFV, st + ST_VSF);
        mma_k128<kNV>(tmem + T_O, dp, smem_desc_sw64(st + ST_V), tmem + T_SFP, tmem + T_SFV, t != 0);
        tc_commit(&bars->kv_empty[s]);
        tc_commit(&bars->o_done);
        return true;
      };
      for (int j = 0; ok && j < nkv; ++j) {
        const int s = j % STAGES, sb = j & 1;
        if (!mbar_wait(&bars->kv_full[s], (j / STAGES) & 1, status, 0x1203)) { ok = false; break; }
        if (j >= 2 && !mbar_wait(&bars->s_free[sb], ((j >> 1) - 1) & 1, status, 0x1204)) { ok = false; break; }
        if (*(volatile int*)&bars->abort) { ok = false; break; }
        tc_fence_after();
        uint8_t* st = smem + OFF_STAGE + s * STAGE_BYTES;
        cp_sf<kNV>(tmem + T_SFK, st + ST_KSF);
        mma_k128<kNV>(tmem + T_S0 + sb * 128, dq, smem_desc_sw64(st + ST_K), tmem + T_SFQ, tmem + T_SFK, false);
        tc_commit(&bars->s_full[sb]);
        if (j >= 1 && !issue_pv(j - 1)) { ok = false; break; }
      }
      if (ok && nkv > 0) ok = issue_pv(nkv - 1);
      if (!ok) bars->abort = 1;
      // every issued tcgen05 op has completed before TMEM is released
      tc_commit(&bars->drain);
      mbar_wait(&bars->drain, 0, status, 0x1205);
    }
  } else {
    // ------------------------------------------------------------ softmax / epilogue
    // 8 warps: two threads per query row, each owning 64 of the tile's 128 keys
    // (and 64 of O's 128 columns).  Warp w reads TMEM lane quadrant w % 4.
    const int sw = warp - 2;                   // 0..7
    const int half = sw >> 2;                  // which 64 columns
    const int quad = warp & 3;
    const int r = quad * 32 + lane;            // query row within the tile
    const int c0 = half * 64;                  // first column owned
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    uint8_t* prow = smem + OFF_P + r * 64;
    const int swz = (r >> 1) & 3;              // 64-byte swizzle of this row's 16-byte chunks
    float* red = reinterpret_cast<float*>(smem + OFF_RED);  // [2 tile parities][2 halves][128 rows]
    const float qk = p.qk_scale;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      const int s = j % STAGES, sb = j & 1;
      // After a failed (timed-out) wait the thread stops waiting but keeps
      // iterating, so every softmax warp reaches every named barrier.
      if (ok) ok = mbar_wait(&bars->s_full[sb], (j >> 1) & 1, status, 0x1301) &&
                   mbar_wait(&bars->kv_full[s], (j / STAGES) & 1, status, 0x1302);
      ok = __all_sync(0xffffffffu, ok);  // warp-uniform: the TMEM loads below are .sync.aligned
      tc_fence_after();
      float x[64];
      {
        uint32_t u[32], u2[32];
        tmem_ld32(tmem + lane_base + T_S0 + sb * 128 + c0, u);
        tmem_ld32(tmem + lane_base + T_S0 + sb * 128 + c0 + 32, u2);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          x[i] = __uint_as_float(u[i]);
          x[32 + i] = __uint_as_float(u2[i]);
        }
      }
      tc_fence_before();
      mbar_arrive(&bars->s_free[sb]);
      const uint8_t* st = smem + OFF_STAGE + s * STAGE_BYTES;
      if (p.smoothing) {
        const uint4* dsv = reinterpret_cast<const uint4*>(st + ST_DS + c0 * 2);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 w = dsv[c];
          const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 a = add_f32x2(make_float2(x[c * 8 + 2 * i], x[c * 8 + 2 * i + 1]),
                                       make_float2(bf16lo(ww[i]), bf16hi(ww[i])));
            x[c * 8 + 2 * i] = a.x;
            x[c * 8 + 2 * i + 1] = a.y;
          }
        }
      }
      // masking: keys beyond L (last tile) and, if causal, keys after the query
      const int key0 = j * BN + c0;
      const int qrow = qt * BM + r;
      const int lim = p.causal ? min(p.L - key0, qrow - key0 + 1) : p.L - key0;
      if (lim < 64) {
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (i >= lim) x[i] = -INFINITY;
      }
      // row max over this thread's 64 keys (8 independent chains), then with the partner
      float mx8[8];
#pragma unroll
      for (int a = 0; a < 8; ++a) mx8[a] = x[a];
#pragma unroll
      for (int i = 8; i < 64; i += 8)
#pragma unroll
        for (int a = 0; a < 8; ++a) mx8[a] = fmaxf(mx8[a], x[i + a]);
      const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                             fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      red[(sb * 2 + half) * 128 + r] = mx;
      named_barrier(1, 256);
      const float mx_row = fmaxf(mx, red[(sb * 2 + (half ^ 1)) * 128 + r]);
      const float m_new = fmaxf(m_run, mx_row * qk);
      // PV(j-1) must be complete before O is rescaled or P is overwritten
      if (ok && j >= 1) ok = mbar_wait(&bars->o_done, (j - 1) & 1, status, 0x1303);
      ok = __all_sync(0xffffffffu, ok);
      const bool grow = (m_new > m_run) && (m_run != -INFINITY);
      const float alpha = grow ? ex2_approx(m_run - m_new) : 1.0f;
      if (__any_sync(0xffffffffu, grow)) {
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < 64; c += 32) {
          uint32_t u[32];
          tmem_ld32(tmem + lane_base + T_O + c0 + c, u);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const float2 v = mul_f32x2(make_float2(__uint_as_float(u[i]), __uint_as_float(u[i + 1])),
                                       make_float2(alpha, alpha));
            u[i] = __float_as_uint(v.x);
            u[i + 1] = __float_as_uint(v.y);
          }
          tmem_st32(tmem + lane_base + T_O + c0 + c, u);
        }
        tmem_st_wait();
      }
      l_run *= alpha;
      m_run = m_new;
      // p = exp2(x * qk_scale - m); partial row sum in 8 chains
      const float2 qk2 = make_float2(qk, qk), mneg2 = make_float2(-m_new, -m_new);
      float ls8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < 64; i += 2) {
        const float2 t = fma_f32x2(make_float2(x[i], x[i + 1]), qk2, mneg2);
        x[i] = ex2_approx(t.x);
        x[i + 1] = ex2_approx(t.y);
        ls8[(i >> 1) & 7] += x[i] + x[i + 1];
      }
      const float lsum_tile = ((ls8[0] + ls8[1]) + (ls8[2] + ls8[3])) + ((ls8[4] + ls8[5]) + (ls8[6] + ls8[7]));
      if (!p.l_quant) l_run += lsum_tile;
      // P -> E2M1 codes (round-to-nearest-even) with per-block scales:
      // MXFP4: E8M0 2^e per 32 keys, e = clamp(ceil(log2(max / 6)), -127, 127);
      // NVFP4: E4M3 per 16 keys, s = e4m3(max(max / 6, 1e-8)).
      // The emulated configs first scale p by 448*6 (it cancels in O / l).
      float lq = 0.f;  // sum of the quantised values (emulated configs)
      if (p.p_prescale != 1.0f) {
        const float2 ps = make_float2(p.p_prescale, p.p_prescale);
#pragma unroll
        for (int i = 0; i < 64; i += 2) {
          const float2 v = mul_f32x2(make_float2(x[i], x[i + 1]), ps);
          x[i] = v.x;
          x[i + 1] = v.y;
        }
      }
      if (!kNV) {
        uint32_t sfh = 0;
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          float a8[8];
#pragma unroll
          for (int a = 0; a < 8; ++a) a8[a] = x[g * 32 + a];
#pragma unroll
          for (int i = 8; i < 32; i += 8)
#pragma unroll
            for (int a = 0; a < 8; ++a) a8[a] = fmaxf(a8[a], x[g * 32 + i + a]);
          const float amax = fmaxf(fmaxf(fmaxf(a8[0], a8[1]), fmaxf(a8[2], a8[3])),
                                   fmaxf(fmaxf(a8[4], a8[5]), fmaxf(a8[6], a8[7])));
          const uint32_t rb = __float_as_uint(__fdiv_rn(amax, 6.0f));
          const int e = min(max(static_cast<int>(rb >> 23) - 127 + ((rb & 0x7FFFFFu) != 0), -127), 127);
          const int be = 127 - e;  // biased exponent of 2^-e, in [0, 254]
          const float inv = __uint_as_float(be > 0 ? static_cast<uint32_t>(be) << 23 : 0x00400000u);
          const float2 inv2 = make_float2(inv, inv);
          uint32_t w[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t word = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int n = g * 32 + q * 8 + 2 * i;
              const float2 sc = mul_f32x2(make_float2(x[n], x[n + 1]), inv2);
              word |= cvt_e2m1x2(sc.x, sc.y) << (8 * i);
            }
            w[q] = word;
          }
          if (p.l_quant) {
            const float sum = (e2m1_word_sum(w[0]) + e2m1_word_sum(w[1])) + (e2m1_word_sum(w[2]) + e2m1_word_sum(w[3]));
            lq += sum * __uint_as_float(e + 127 > 0 ? static_cast<uint32_t>(e + 127) << 23 : 0x00400000u);
          }
          const int chunk = half * 2 + g;
          *reinterpret_cast<uint4*>(prow + ((chunk ^ swz) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
          sfh |= static_cast<uint32_t>(e + 127) << (8 * g);
        }
        *reinterpret_cast<uint16_t*>(smem + OFF_PSF + (r & 31) * 16 + (r >> 5) * 4 + half * 2) =
            static_cast<uint16_t>(sfh);
      } else {
        uint32_t sfw = 0;
        uint32_t w[8];
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          float a8[8];
#pragma unroll
          for (int a = 0; a < 8; ++a) a8[a] = fmaxf(x[g * 16 + a], x[g * 16 + 8 + a]);
          const float amax = fmaxf(fmaxf(fmaxf(a8[0], a8[1]), fmaxf(a8[2], a8[3])),
                                   fmaxf(fmaxf(a8[4], a8[5]), fmaxf(a8[6], a8[7])));
          const float scl = fmaxf(__fdiv_rn(amax, 6.0f), 1e-8f);
          const uint32_t sb8 = e4m3_byte(scl);
          const float sv = round_e4m3(scl);
          const float inv = sv > 0.f ? __fdiv_rn(1.0f, sv) : 0.f;
          const float2 inv2 = make_float2(inv, inv);
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            uint32_t word = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int n = g * 16 + q * 8 + 2 * i;
              const float2 sc = mul_f32x2(make_float2(x[n], x[n + 1]), inv2);
              word |= cvt_e2m1x2(sc.x, sc.y) << (8 * i);
            }
            w[g * 2 + q] = word;
          }
          if (p.l_quant) lq += (e2m1_word_sum(w[g * 2]) + e2m1_word_sum(w[g * 2 + 1])) * sv;
          sfw |= sb8 << (8 * g);
        }
        *reinterpret_cast<uint4*>(prow + (((half * 2) ^ swz) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
        *reinterpret_cast<uint4*>(prow + (((half * 2 + 1) ^ swz) << 4)) = make_uint4(w[4], w[5], w[6], w[7]);
        *reinterpret_cast<uint32_t*>(smem + OFF_PSF + half * SF_CHUNK + (r & 31) * 16 + (r >> 5) * 4) = sfw;
      }
      if (p.l_quant) l_run += lq;
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&bars->p_full);
    }
    // ---------------- epilogue: combine the two partial row sums, O / l -> bf16
    red[(2 * 2 + half) * 128 + r] = l_run;
    named_barrier(1, 256);
    const float l_row = l_run + red[(2 * 2 + (half ^ 1)) * 128 + r];
    if (ok && nkv > 0) ok = mbar_wait(&bars->o_done, (nkv - 1) & 1, status, 0x1304);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    const int qrow = qt * BM + r;
    const bool store = ok && !*(volatile int*)&bars->abort && qrow < p.L;
    const float inv_l = 1.0f / l_row;
    const int b = bh / p.H, h = bh % p.H;
    __nv_bfloat16* orow = out + b * p.o_sb + static_cast<int64_t>(qrow) * p.o_sn + h * p.o_sh + c0;
#pragma unroll 1
    for (int c = 0; c < 64; c += 32) {
      uint32_t u[32];
      tmem_ld32(tmem + lane_base + T_O + c0 + c, u);
      tmem_ld_wait();
      if (store) {
        uint4* dst = reinterpret_cast<uint4*>(orow + c);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t w[4];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            w[i] = pack_bf16x2(__uint_as_float(u[q * 8 + 2 * i]) * inv_l, __uint_as_float(u[q * 8 + 2 * i + 1]) * inv_l);
          dst[q] = make_uint4(w[0], w[1], w[2], w[3]);
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

}  // namespace

int launch_flash(const Problem& pr, const Workspace& w, cudaStream_t s) {
  int* status = device_status_ptr();
  if (status == nullptr) return QDQ_ERR_CUDA;
  const int64_t BH = static_cast<int64_t>(pr.B) * pr.H;
  CUtensorMap mq, mk, mv;
  if (int st = make_tmap_u8_2d(&mq, w.qc, BH * pr.Lp, 64, 64, 64, 128, 64)) return st;
  if (int st = make_tmap_u8_2d(&mk, w.kc, BH * pr.Lp, 64, 64, 64, 128, 64)) return st;
  if (int st = make_tmap_u8_2d(&mv, w.vt, BH * HD, pr.Lp / 2, pr.Lp / 2, 64, 128, 64)) return st;
  static bool attr[2][64] = {{false}};
  int dev = 0;
  cudaGetDevice(&dev);
  const void* fn = pr.nv ? reinterpret_cast<const void*>(&sage3_fp4_flash_kernel<true>)
                         : reinterpret_cast<const void*>(&sage3_fp4_flash_kernel<false>);
  if (dev >= 0 && dev < 64 && !attr[pr.nv][dev]) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(SMEM_BYTES));
    if (e != cudaSuccess) return fail(QDQ_ERR_CUDA, "sage3 flash: smem attribute: %s", cudaGetErrorString(e));
    attr[pr.nv][dev] = true;
  }
  Params p;
  p.H = pr.H;
  p.L = pr.L;
  p.Lp = pr.Lp;
  p.T = pr.Lp / 128;
  p.o_sb = pr.o_sb;
  p.o_sn = pr.o_sn;
  p.o_sh = pr.o_sh;
  p.qk_scale = pr.sm_scale * 1.4426950408889634f;
  p.causal = pr.causal;
  p.smoothing = pr.smoothing;
  p.p_prescale = pr.emulated ? 2688.0f : 1.0f;
  p.l_quant = pr.emulated;
  dim3 grid(static_cast<unsigned>(p.T), static_cast<unsigned>(BH));
  if (pr.nv)
    sage3_fp4_flash_kernel<true><<<grid, THREADS, SMEM_BYTES, s>>>(mq, mk, mv, w.qsf, w.ksf, w.vsf, w.ds, pr.o, p,
                                                                  status);
  else
    sage3_fp4_flash_kernel<false><<<grid, THREADS, SMEM_BYTES, s>>>(mq, mk, mv, w.qsf, w.ksf, w.vsf, w.ds, pr.o,
                                                                   p, status);
  return check_launch("sage3 flash");
}

}  // namespace attn
}  // namespace qdqb200
