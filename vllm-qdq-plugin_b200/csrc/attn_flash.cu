// Sage3 FP4 flash attention on sm_100a tensor cores, D = 128.
// MXFP4 (E2M1 + E8M0 per 32, tcgen05 kind::mxf4) or NVFP4 (E2M1 + E4M3 per
// 16, kind::mxf4nvf4 block16).
//
// Reference semantics: the mxfp4_hw kernel (sage3/mxfp4_hw_kernel.py:167-393)
//   S  = dot_scaled(Q, K^T) (+ delta_s[group of the query tile, key]),
//   online softmax in base 2 with qk_scale = sm_scale * log2(e),
//   l += sum of the unquantised p,
//   P quantised per row and 32 keys: e = clamp(ceil(log2(max(p)/6)), -127, 127),
//     codes = cvt.rn.satfinite.e2m1x2(p * 2^-e),
//   O += dot_scaled(P, V), O / l at the end;
// and, for the emulated configs (p_quant_kernels.py:37-150,
// attention_kernel.py:176-186), P scaled by 448*6 before block scaling and
// l = sum of the dequantised P.  Keys beyond L are masked (the reference
// attends to its zero padding).
//
// CTA = two 128-row query tiles (A, B) of one (batch, head) that share every
// K/V tile, 12 warps:
//   warps 0-3     softmax A: one thread per query row (TMEM lane): S -> registers,
//                 + delta_s, row max, O_A rescale in TMEM when the max grows,
//                 exp2, row sum, P -> E2M1 codes + block scales in shared
//                 memory; epilogue O_A / l -> bf16 NHD
//   warps 4-7     softmax B (the same for tile B)
//   warp 8        MMA issuer: per key tile j, S = Q_A K_j^T, then (once A has
//                 read S) S = Q_B K_j^T, then O_A += P_A V_{j-1}, O_B += P_B V_{j-1}
//   warp 9        TMA producer: K tile [128 keys x 64 B], V^T tile [128 d x 64 B]
//                 (64-byte swizzle), their scale chunks and both tiles' delta_s
//                 slices into a 4-stage ring; Q_A, Q_B once
//   warps 10-11   idle (they complete the third warpgroup for setmaxnreg)
// The single S buffer alternates between the two softmax warpgroups, which
// therefore run out of phase and overlap their MUFU / FMA / ALU work.
// Registers: softmax warpgroups 224 per thread, the rest 56 (setmaxnreg;
// 2 x 128 x 224 + 128 x 56 = 384 x 168, the launch allocation).
// TMEM: S [0,128) O_A [128,256) O_B [256,384), scale factors [384,432).
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
// stage: K codes | V codes | K sf | V sf | delta_s A | delta_s B
constexpr int ST_K = 0, ST_V = CODE_TILE, ST_KSF = 2 * CODE_TILE, ST_VSF = ST_KSF + SF_TILE,
              ST_DS = ST_VSF + SF_TILE;
constexpr int STAGE_BYTES = 19 * 1024;
static_assert(ST_DS + 2 * DS_BYTES <= STAGE_BYTES, "stage layout");
// CTA smem: Q_A | Q_B | P_A | P_B | stages | Q sf A,B | P sf A,B | barriers
constexpr int OFF_Q = 0, OFF_P = 2 * CODE_TILE, OFF_STAGE = 4 * CODE_TILE;
constexpr int OFF_QSF = OFF_STAGE + STAGES * STAGE_BYTES;
constexpr int OFF_PSF = OFF_QSF + 2 * SF_TILE;
constexpr int OFF_BAR = OFF_PSF + 2 * SF_TILE;
constexpr int THREADS = 384;
constexpr int TMEM_COLS = 512;
// scale-factor columns: 8 per operand (NVFP4: two chunks; MXFP4 uses the first 4)
constexpr uint32_t T_S = 0, T_O = 128, T_SFQ = 384, T_SFK = 400, T_SFP = 408, T_SFV = 416;

struct Bars {
  uint64_t q_full;
  uint64_t kv_full[STAGES];
  uint64_t kv_empty[STAGES];
  uint64_t s_full[2];   // per warpgroup: S holds its tile's scores
  uint64_t s_free[2];   // per warpgroup: its scores are in registers
  uint64_t p_full[2];   // per warpgroup: its P codes / scales are in shared memory
  uint64_t o_done[2];   // per warpgroup: its PV MMA completed
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

// The two K=64 block-scaled MMAs of a 128 x 128 x 128 product.
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

__device__ __forceinline__ void reg_alloc_224() { asm volatile("setmaxnreg.inc.sync.aligned.u32 224;"); }
__device__ __forceinline__ void reg_dealloc_56() { asm volatile("setmaxnreg.dec.sync.aligned.u32 56;"); }

// max of v[base .. base+32) in 8 independent chains
__device__ __forceinline__ float max32(const float* v) {
  float m8[8];
#pragma unroll
  for (int a = 0; a < 8; ++a) m8[a] = fmaxf(fmaxf(v[a], v[8 + a]), fmaxf(v[16 + a], v[24 + a]));
  return fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])), fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
}

// ---------------------------------------------------------------------------
// softmax warpgroup: one query tile, thread = row
// ---------------------------------------------------------------------------
template <bool kNV>
__device__ __forceinline__ void softmax_wg(uint8_t* smem, Bars* bars, uint32_t tmem, const Params& p, int wg,
                                           int qt, int bh, int nkv, __nv_bfloat16* __restrict__ out,
                                           int* status) {
  const int warp = (threadIdx.x >> 5) & 3;
  const int lane = threadIdx.x & 31;
  const int r = warp * 32 + lane;            // query row in the tile = TMEM lane
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
  const uint32_t t_o = tmem + T_O + wg * 128;
  uint8_t* prow = smem + OFF_P + wg * CODE_TILE + r * 64;
  uint8_t* psf = smem + OFF_PSF + wg * SF_TILE;
  const int swz = (r >> 1) & 3;              // 64-byte swizzle of this row's 16-byte chunks
  const float qk = p.qk_scale;
  const int qrow = qt * BM + r;
  float m_run = -INFINITY, l_run = 0.f;
  bool ok = true;
  for (int j = 0; j < nkv; ++j) {
    const int s = j % STAGES;
    // After a failed (timed-out) wait the thread stops waiting but keeps
    // iterating, so the other roles are never left waiting on it.
    if (ok) ok = mbar_wait(&bars->s_full[wg], j & 1, status, 0x1301) &&
                 mbar_wait(&bars->kv_full[s], (j / STAGES) & 1, status, 0x1302);
    ok = __all_sync(0xffffffffu, ok);  // warp-uniform: the TMEM accesses below are .sync.aligned
    tc_fence_after();
    float x[BN];
#pragma unroll
    for (int c = 0; c < BN; c += 32) {
      uint32_t u[32];
      tmem_ld32(tmem + lane_base + T_S + c, u);
#pragma unroll
      for (int i = 0; i < 32; ++i) x[c + i] = __uint_as_float(u[i]);
    }
    tmem_ld_wait();
    tc_fence_before();
    mbar_arrive(&bars->s_free[wg]);
    const uint8_t* st = smem + OFF_STAGE + s * STAGE_BYTES;
    if (p.smoothing) {
      const uint4* dsv = reinterpret_cast<const uint4*>(st + ST_DS + wg * DS_BYTES);
#pragma unroll
      for (int c = 0; c < BN / 8; ++c) {
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
    const int key0 = j * BN;
    const int lim = p.causal ? min(p.L - key0, qrow - key0 + 1) : p.L - key0;
    if (lim < BN) {
#pragma unroll
      for (int i = 0; i < BN; ++i)
        if (i >= lim) x[i] = -INFINITY;
    }
    const float mx = fmaxf(fmaxf(max32(x), max32(x + 32)), fmaxf(max32(x + 64), max32(x + 96)));
    const float m_new = fmaxf(m_run, mx * qk);
    // PV(j-1) of this tile must be complete before O is rescaled or P is overwritten
    if (ok && j >= 1) ok = mbar_wait(&bars->o_done[wg], (j - 1) & 1, status, 0x1303);
    ok = __all_sync(0xffffffffu, ok);
    const bool grow = (m_new > m_run) && (m_run != -INFINITY);
    const float alpha = grow ? ex2_approx(m_run - m_new) : 1.0f;
    if (__any_sync(0xffffffffu, grow)) {
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < HD; c += 32) {
        uint32_t u[32];
        tmem_ld32(t_o + lane_base + c, u);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float2 v = mul_f32x2(make_float2(__uint_as_float(u[i]), __uint_as_float(u[i + 1])),
                                     make_float2(alpha, alpha));
          u[i] = __float_as_uint(v.x);
          u[i + 1] = __float_as_uint(v.y);
        }
        tmem_st32(t_o + lane_base + c, u);
      }
      tmem_st_wait();
    }
    l_run *= alpha;
    m_run = m_new;
    // p = exp2(x * qk_scale - m); row sum in 8 chains
    const float2 qk2 = make_float2(qk, qk), mneg2 = make_float2(-m_new, -m_new);
    float ls8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < BN; i += 2) {
      const float2 t = fma_f32x2(make_float2(x[i], x[i + 1]), qk2, mneg2);
      x[i] = ex2_approx(t.x);
      x[i + 1] = ex2_approx(t.y);
      ls8[(i >> 1) & 7] += x[i] + x[i + 1];
    }
    if (!p.l_quant) l_run += ((ls8[0] + ls8[1]) + (ls8[2] + ls8[3])) + ((ls8[4] + ls8[5]) + (ls8[6] + ls8[7]));
    // P -> E2M1 codes (round-to-nearest-even) with per-block scales:
    // MXFP4: E8M0 2^e per 32 keys, e = clamp(ceil(log2(max / 6)), -127, 127);
    // NVFP4: E4M3 per 16 keys, s = e4m3(max(max / 6, 1e-8)).
    // The emulated configs first scale p by 448*6 (it cancels in O / l).
    if (p.p_prescale != 1.0f) {
      const float2 ps = make_float2(p.p_prescale, p.p_prescale);
#pragma unroll
      for (int i = 0; i < BN; i += 2) {
        const float2 v = mul_f32x2(make_float2(x[i], x[i + 1]), ps);
        x[i] = v.x;
        x[i + 1] = v.y;
      }
    }
    float lq = 0.f;
    if (!kNV) {
      uint32_t sfw = 0;
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        const float amax = max32(x + g * 32);
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
        *reinterpret_cast<uint4*>(prow + ((g ^ swz) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
        sfw |= static_cast<uint32_t>(e + 127) << (8 * g);
      }
      *reinterpret_cast<uint32_t*>(psf + (r & 31) * 16 + (r >> 5) * 4) = sfw;
    } else {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t sfw = 0;
        uint32_t w[8];
#pragma unroll
        for (int g4 = 0; g4 < 4; ++g4) {
          const int g = h * 4 + g4;
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
            w[g4 * 2 + q] = word;
          }
          if (p.l_quant) lq += (e2m1_word_sum(w[g4 * 2]) + e2m1_word_sum(w[g4 * 2 + 1])) * sv;
          sfw |= sb8 << (8 * g4);
        }
        *reinterpret_cast<uint4*>(prow + (((h * 2) ^ swz) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
        *reinterpret_cast<uint4*>(prow + (((h * 2 + 1) ^ swz) << 4)) = make_uint4(w[4], w[5], w[6], w[7]);
        *reinterpret_cast<uint32_t*>(psf + h * SF_CHUNK + (r & 31) * 16 + (r >> 5) * 4) = sfw;
      }
    }
    if (p.l_quant) l_run += lq;
    fence_proxy_async_smem();
    tc_fence_before();
    mbar_arrive(&bars->p_full[wg]);
  }
  // ---------------- epilogue: O / l -> bf16 NHD
  if (ok && nkv > 0) ok = mbar_wait(&bars->o_done[wg], (nkv - 1) & 1, status, 0x1304);
  ok = __all_sync(0xffffffffu, ok);
  tc_fence_after();
  const bool store = ok && !*(volatile int*)&bars->abort && qrow < p.L;
  const float inv_l = 1.0f / l_run;
  const int b = bh / p.H, h = bh % p.H;
  __nv_bfloat16* orow = out + b * p.o_sb + static_cast<int64_t>(qrow) * p.o_sn + h * p.o_sh;
#pragma unroll 1
  for (int c = 0; c < HD; c += 32) {
    uint32_t u[32];
    tmem_ld32(t_o + lane_base + c, u);
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
  const int qtA = 2 * blockIdx.x;
  const int qtB = qtA + 1;
  const bool hasB = qtB < p.T;
  const int nq = hasB ? 2 : 1;
  const int bh = blockIdx.y;
  const int nkv = p.causal ? qtA + nq : p.T;  // causal: keys up to the last query row of the CTA
  constexpr int kSfBytes = kNV ? SF_TILE : SF_CHUNK;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bars->kv_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->s_free[i], 128);
      mbar_init(&bars->p_full[i], 128);
      mbar_init(&bars->o_done[i], 1);
    }
    mbar_init(&bars->drain, 1);
    bars->abort = 0;
    fence_barrier_init();
    prefetch_tmap(&map_q);
    prefetch_tmap(&map_k);
    prefetch_tmap(&map_v);
  }
  if (warp == 8) {
    tmem_alloc(&bars->tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp < 8) {
    reg_alloc_224();
    const int wg = warp >> 2;
    if (wg < nq) softmax_wg<kNV>(smem, bars, tmem, p, wg, qtA + wg, bh, nkv, out, status);
  } else {
    reg_dealloc_56();
    if (warp == 9) {
      // ------------------------------------------------------------ producer
      if (elect_one()) {
        mbar_arrive_expect_tx(&bars->q_full, nq * (CODE_TILE + kSfBytes));
        for (int t = 0; t < nq; ++t) {
          tma_load_2d(smem + OFF_Q + t * CODE_TILE, &map_q, 0, bh * p.Lp + (qtA + t) * BM, &bars->q_full);
          bulk_load(smem + OFF_QSF + t * SF_TILE, qsf + (static_cast<int64_t>(bh) * p.T + qtA + t) * SF_TILE,
                    kSfBytes, &bars->q_full);
        }
        int issued = 0;
        for (int j = 0; j < nkv; ++j) {
          const int s = j % STAGES;
          if (!mbar_wait(&bars->kv_empty[s], ((j / STAGES) & 1) ^ 1, status, 0x1101)) {
            bars->abort = 1;
            break;
          }
          if (*(volatile int*)&bars->abort) break;
          uint8_t* st = smem + OFF_STAGE + s * STAGE_BYTES;
          const uint32_t bytes = 2 * CODE_TILE + 2 * kSfBytes + (p.smoothing ? nq * DS_BYTES : 0);
          mbar_arrive_expect_tx(&bars->kv_full[s], bytes);
          tma_load_2d(st + ST_K, &map_k, 0, bh * p.Lp + j * BN, &bars->kv_full[s]);
          tma_load_2d(st + ST_V, &map_v, j * (BN / 2), bh * HD, &bars->kv_full[s]);
          bulk_load(st + ST_KSF, ksf + (static_cast<int64_t>(bh) * p.T + j) * SF_TILE, kSfBytes, &bars->kv_full[s]);
          bulk_load(st + ST_VSF, vsf + (static_cast<int64_t>(bh) * p.T + j) * SF_TILE, kSfBytes, &bars->kv_full[s]);
          if (p.smoothing)
            for (int t = 0; t < nq; ++t)
              bulk_load(st + ST_DS + t * DS_BYTES, ds + (static_cast<int64_t>(bh) * p.T + qtA + t) * p.Lp + j * BN,
                        DS_BYTES, &bars->kv_full[s]);
          ++issued;
        }
        mbar_wait(&bars->q_full, 0, status, 0x1102);
        for (int j = (issued > STAGES ? issued - STAGES : 0); j < issued; ++j)
          mbar_wait(&bars->kv_full[j % STAGES], (j / STAGES) & 1, status, 0x1103);
      }
    } else if (warp == 8) {
      // ------------------------------------------------------------ MMA issuer
      if (elect_one()) {
        bool ok = mbar_wait(&bars->q_full, 0, status, 0x1201);
        if (ok) {
          tc_fence_after();
          for (int t = 0; t < nq; ++t) cp_sf<kNV>(tmem + T_SFQ + t * 8, smem + OFF_QSF + t * SF_TILE);
        }
        auto issue_pv = [&](int t) -> bool {
          const int s = t % STAGES;
          uint8_t* st = smem + OFF_STAGE + s * STAGE_BYTES;
          for (int w = 0; w < nq; ++w) {
            if (!mbar_wait(&bars->p_full[w], t & 1, status, 0x1202)) return false;
            tc_fence_after();
            if (w == 0) cp_sf<kNV>(tmem + T_SFV, st + ST_VSF);
            cp_sf<kNV>(tmem + T_SFP, smem + OFF_PSF + w * SF_TILE);
            mma_k128<kNV>(tmem + T_O + w * 128, smem_desc_sw64(smem + OFF_P + w * CODE_TILE),
                          smem_desc_sw64(st + ST_V), tmem + T_SFP, tmem + T_SFV, t != 0);
            tc_commit(&bars->o_done[w]);
          }
          tc_commit(&bars->kv_empty[s]);
          return true;
        };
        for (int j = 0; ok && j < nkv; ++j) {
          const int s = j % STAGES;
          if (!mbar_wait(&bars->kv_full[s], (j / STAGES) & 1, status, 0x1203)) { ok = false; break; }
          if (*(volatile int*)&bars->abort) { ok = false; break; }
          uint8_t* st = smem + OFF_STAGE + s * STAGE_BYTES;
          for (int w = 0; w < nq && ok; ++w) {
            // S is free once the warpgroup that used it last has read its scores:
            // for A that is B (or A alone) at key tile j-1, for B it is A at key tile j.
            const int prev = w == 0 ? nq - 1 : 0;
            const int prev_j = w == 0 ? j - 1 : j;
            if (prev_j >= 0 && !mbar_wait(&bars->s_free[prev], prev_j & 1, status, 0x1204)) { ok = false; break; }
            tc_fence_after();
            if (w == 0) cp_sf<kNV>(tmem + T_SFK, st + ST_KSF);
            mma_k128<kNV>(tmem + T_S, smem_desc_sw64(smem + OFF_Q + w * CODE_TILE), smem_desc_sw64(st + ST_K),
                          tmem + T_SFQ + w * 8, tmem + T_SFK, false);
            tc_commit(&bars->s_full[w]);
          }
          if (!ok) break;
          if (j >= 1 && !issue_pv(j - 1)) { ok = false; break; }
        }
        if (ok && nkv > 0) ok = issue_pv(nkv - 1);
        if (!ok) bars->abort = 1;
        // every issued tcgen05 op has completed before TMEM is released
        tc_commit(&bars->drain);
        mbar_wait(&bars->drain, 0, status, 0x1205);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
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
  dim3 grid(static_cast<unsigned>((p.T + 1) / 2), static_cast<unsigned>(BH));
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
