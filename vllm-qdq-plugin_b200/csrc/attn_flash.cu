// Sage3 FP4 flash attention on sm_100a tensor cores (MXFP4: E2M1 data, E8M0
// scales per 32), D = 128, one 128-row query tile per CTA.
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
constexpr int DS_BYTES = BN * 2;
// stage: K codes | V codes | K sf | V sf | delta_s (bf16)
constexpr int ST_K = 0, ST_V = CODE_TILE, ST_KSF = 2 * CODE_TILE, ST_VSF = ST_KSF + SF_CHUNK,
              ST_DS = ST_VSF + SF_CHUNK;
constexpr int STAGE_BYTES = 18 * 1024;
static_assert(ST_DS + DS_BYTES <= STAGE_BYTES, "stage layout");
// CTA smem: Q codes | P codes | stages | Q sf | P sf | barriers
constexpr int OFF_Q = 0, OFF_P = CODE_TILE, OFF_STAGE = 2 * CODE_TILE;
constexpr int OFF_QSF = OFF_STAGE + STAGES * STAGE_BYTES;
constexpr int OFF_PSF = OFF_QSF + SF_CHUNK;
constexpr int OFF_RED = OFF_PSF + SF_CHUNK;              // [3][2][128] floats: row max / row sum exchange
constexpr int OFF_BAR = OFF_RED + 3 * 2 * 128 * 4;
constexpr int THREADS = 320;                             // producer, MMA, 8 softmax warps
constexpr int TMEM_COLS = 512;
constexpr uint32_t T_S0 = 0, T_O = 256, T_SFQ = 384, T_SFK = 388, T_SFP = 392, T_SFV = 396;
constexpr uint32_t IDESC = idesc_mxf4(BM, BN, true);  // also N = HD for PV
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
};

__global__ void __launch_bounds__(THREADS, 1)
sage3_mxfp4_flash_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
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
      mbar_arrive_expect_tx(&bars->q_full, CODE_TILE + SF_CHUNK);
      tma_load_2d(smem + OFF_Q, &map_q, 0, bh * p.Lp + qt * BM, &bars->q_full);
      bulk_load(smem + OFF_QSF, qsf + (static_cast<int64_t>(bh) * p.T + qt) * SF_CHUNK, SF_CHUNK, &bars->q_full);
      int issued = 0;
      for (int j = 0; j < nkv; ++j) {
        const int s = j % STAGES;
        if (!mbar_wait(&bars->kv_empty[s], ((j / STAGES) & 1) ^ 1, status, 0x1101)) {
          bars->abort = 1;
          break;
        }
        if (*(volatile int*)&bars->abort) break;
        uint8_t* st = smem + OFF_STAGE + s * STAGE_BYTES;
        const uint32_t bytes = 2 * CODE_TILE + 2 * SF_CHUNK + (p.smoothing ? DS_BYTES : 0);
        mbar_arrive_expect_tx(&bars->kv_full[s], bytes);
        tma_load_2d(st + ST_K, &map_k, 0, bh * p.Lp + j * BN, &bars->kv_full[s]);
        tma_load_2d(st + ST_V, &map_v, j * (BN / 2), bh * HD, &bars->kv_full[s]);
        bulk_load(st + ST_KSF, ksf + (static_cast<int64_t>(bh) * p.T + j) * SF_CHUNK, SF_CHUNK, &bars->kv_full[s]);
        bulk_load(st + ST_VSF, vsf + (static_cast<int64_t>(bh) * p.T + j) * SF_CHUNK, SF_CHUNK, &bars->kv_full[s]);
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
        tmem_cp_sf(tmem + T_SFQ, smem_desc_sf(smem + OFF_QSF));
      }
      const uint64_t dq = smem_desc_sw64(smem + OFF_Q);
      const uint64_t dp = smem_desc_sw64(smem + OFF_P);
      auto issue_pv = [&](int t) -> bool {
        const int s = t % STAGES;
        if (!mbar_wait(&bars->p_full, t & 1, status, 0x1202)) return false;
        tc_fence_after();
        uint8_t* st = smem + OFF_STAGE + s * STAGE_BYTES;
        tmem_cp_sf(tmem + T_SFP, smem_desc_sf(smem + OFF_PSF));
        tmem_cp_sf(tmem + T_SFV, smem_desc_sf(st + ST_VSF));
        const uint64_t dv = smem_desc_sw64(st + ST_V);
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
          const uint32_t sf_id = kk * 2;
          mma_mxf4(tmem + T_O, dp + kk * 2, dv + kk * 2, idesc_with_sf_ids(IDESC, sf_id, sf_id),
                   (tmem + T_SFP) | (sf_id << 30), (tmem + T_SFV) | (sf_id << 30), (t | kk) != 0);
        }
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
        tmem_cp_sf(tmem + T_SFK, smem_desc_sf(st + ST_KSF));
        const uint64_t dk = smem_desc_sw64(st + ST_K);
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
          const uint32_t sf_id = kk * 2;
          mma_mxf4(tmem + T_S0 + sb * 128, dq + kk * 2, dk + kk * 2, idesc_with_sf_ids(IDESC, sf_id, sf_id),
                   (tmem + T_SFQ) | (sf_id << 30), (tmem + T_SFK) | (sf_id << 30), kk != 0);
        }
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
      l_run += ((ls8[0] + ls8[1]) + (ls8[2] + ls8[3])) + ((ls8[4] + ls8[5]) + (ls8[6] + ls8[7]));
      // P -> E2M1 codes (RNE) with one E8M0 scale per 32 keys
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
        // e = clamp(ceil(log2(amax / 6)), -127, 127); 0 -> -127
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
        const int chunk = half * 2 + g;
        *reinterpret_cast<uint4*>(prow + ((chunk ^ swz) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
        sfh |= static_cast<uint32_t>(e + 127) << (8 * g);
      }
      *reinterpret_cast<uint16_t*>(smem + OFF_PSF + (r & 31) * 16 + (r >> 5) * 4 + half * 2) =
          static_cast<uint16_t>(sfh);
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
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    cudaError_t e = cudaFuncSetAttribute(sage3_mxfp4_flash_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(SMEM_BYTES));
    if (e != cudaSuccess) return fail(QDQ_ERR_CUDA, "sage3 flash: smem attribute: %s", cudaGetErrorString(e));
    attr[dev] = true;
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
  dim3 grid(static_cast<unsigned>(p.T), static_cast<unsigned>(BH));
  sage3_mxfp4_flash_kernel<<<grid, THREADS, SMEM_BYTES, s>>>(mq, mk, mv, w.qsf, w.ksf, w.vsf, w.ds, pr.o, p,
                                                            status);
  return check_launch("sage3 flash");
}

}  // namespace attn
}  // namespace qdqb200
