// Sage3 FP4 / FP8 flash attention on sm_100a tensor cores, D = 128.
// MXFP4 (E2M1 + E8M0 per 32, tcgen05 kind::mxf4), NVFP4 (E2M1 + E4M3 per
// 16, kind::mxf4nvf4 block16) or MXFP8 (E4M3 + E8M0 per 32, kind::mxf8f6f4).
//
// Reference semantics: the mxfp4_hw kernel (sage3/mxfp4_hw_kernel.py:167-393)
//   S  = dot_scaled(Q, K^T) (+ delta_s[group of the query tile, key]),
//   online softmax in base 2 with qk_scale = sm_scale * log2(e),
//   l += sum of the unquantised p,
//   P quantised per row and 32 keys: e = clamp(ceil(log2(max(p)/6)), -127, 127),
//     codes = cvt.rn.satfinite.e2m1x2(p * 2^-e),
//   O += dot_scaled(P, V), O / l at the end;
// and, for the emulated configs (p_quant_kernels.py:37-283,
// attention_kernel.py:176-186), P scaled by 448*6 (two-level configs) before
// block scaling and l = sum of the dequantised P; those with E8M0 scales
// encode P on the reference's 9-level grid as E4M3 codes (P/V format F_G9),
// their Q / K / V arriving from the pre-pass the same way.  The mxfp8_hw kernel
// (sage3/mxfp8_hw_kernel.py:88-246) is the mxfp4_hw one with E4M3 operands:
// P scale e = clamp(ceil(log2(max(p)/448)), -127, 127), codes
// E4M3(min(p * 2^-e, 448)) round-to-nearest-even.  Keys beyond L are masked
// (the reference attends to its zero padding).
//
// CTA = two 128-row query tiles (A, B) of one (batch, head) that share every
// K/V tile, 20 warps:
//   warps 0-7     softmax A: two threads per query row (TMEM lane), warps
//                 0-3 on keys 0-63 of every key tile and warps 4-7 on keys
//                 64-127 (warps w and w + 4 share TMEM lanes 32 (w % 4) ..):
//                 S half-row -> registers, half-row block maxima and the row
//                 max through the partner thread, O_A half-row rescale in TMEM
//                 when the max grows, exp2, partial row sum, P -> codes +
//                 block scales in shared memory; epilogue O_A / l -> bf16 (or fp16) NHD
//   warps 8-15    softmax B (the same for tile B)
//   warp 16       QK MMA issuer: per key tile j, S = delta_s_A + Q_A K_j^T, then
//                 (once A has read S) S = delta_s_B + Q_B K_j^T
//   warp 17       TMA producer: K tile [128 keys x 64 B], V^T tile [128 d x 64 B]
//                 (64-byte swizzle; E4M3: 128 B rows, 128-byte swizzle), their
//                 scale chunks and the two tiles' delta_s rows (bf16 / fp16) into a
//                 4-stage ring (3 for E4M3); Q_A, Q_B once
//   warp 18       PV MMA issuer: O_A += P_A V_j, O_B += P_B V_j as each P tile
//                 is complete (warp 19 idle)
// Four softmax warps per SM sub-partition (instead of two with one thread
// per row) hide the latency of the exp2 / convert / sum chains; the partner
// threads of a row exchange their half-row maxima (and at the end their
// partial row sums) through shared memory and a 64-thread named barrier.
// The single S buffer alternates between the two softmax warpgroups, which
// therefore run out of phase and overlap their MUFU / FMA / ALU work.
// delta_s on the tensor core: with QK smoothing, S starts as one bf16 (fp16) MMA
// (kind::f16, K = 16) of a constant "ones" operand by the stage's delta_s tile,
// and the block-scaled QK MMAs accumulate onto it.  A_t (128 x 16, K-major, no
// swizzle) is 1 in column t and 0 elsewhere; B (128 keys x 16, MN-major,
// 128-byte swizzle) holds delta_s of query group qtA in K-row 0 and of qtA + 1
// in K-row 1 (one 2-row TMA box per 64 keys), rows 2-15 zero, so
// A_t x B^T = delta_s of tile t broadcast over its 128 query rows.  The
// reference adds delta_s to the fp32 scores after the QK product; here it is
// the accumulator's initial value, the same sum in another order.
// Registers: 96 per thread at launch (640 x 96); setmaxnreg moves them to
// 104 for the four softmax warpgroups and 64 for the fifth (the two MMA
// issuers, the producer and an idle warp that completes the warpgroup): 512 x 104 + 128 x 64 = 640 x 96.
// TMEM: S [0,128) O_A [128,256) O_B [256,384), scale factors [384,432).
#include <cmath>

#include "attn_common.cuh"

namespace qdqb200 {
namespace attn {
namespace {

using namespace sm100;

constexpr int BM = 128, BN = 128, HD = 128;
constexpr int MAX_STAGES = 4;
constexpr int SF_CHUNK = 512;
constexpr int SF_TILE = 1024;        // scale bytes per 128-row tile in global memory (two chunks)
constexpr int DS_TILE = 2048;        // delta_s MMA operand: two 1 KB 128-byte-swizzle atoms of 64 keys
constexpr int DS_TX = 2 * 2 * 64 * 2;  // bytes the two 64-key x 2-row delta_s boxes bring per stage
constexpr int ONES_TILE = 2048;      // "ones" MMA operand of one query tile: 128 rows x 16 B
constexpr int ZERO_TILE = 2048;      // zero K-rows 8-15 of both delta_s MMA operands
constexpr uint32_t IDESC_DS = idesc_bf16(BM, BN, true);
// the same with fp16 A and B (format code 0 in bits 7-9 and 10-12), for fp16 inputs
constexpr uint32_t IDESC_DS_F16 = IDESC_DS & ~((7u << 7) | (7u << 10));
constexpr int THREADS = 640;         // 16 softmax warps; the two MMA issuers, TMA producer and an idle warp
constexpr int MMA_WARP = 16, TMA_WARP = 17, PV_WARP = 18;
constexpr int TMEM_COLS = 512;
// scale-factor columns: 8 per operand (NVFP4: two chunks; MXFP4 uses the first 4)
constexpr uint32_t T_S = 0, T_O = 128, T_SFQ = 384, T_SFK = 400, T_SFP = 408, T_SFV = 416;

struct Bars {
  uint64_t q_full;
  uint64_t kv_full[MAX_STAGES];
  uint64_t kv_empty[MAX_STAGES];
  uint64_t s_full[2];   // per warpgroup: S holds its tile's scores
  uint64_t s_free[2];   // per warpgroup: its scores are in registers
  uint64_t p_full[2];   // per warpgroup: its P codes / scales are in shared memory
  uint64_t o_done[2];   // per warpgroup: its PV MMA completed
  uint64_t drain[2];    // per MMA issuer: its last tcgen05 op completed
  float xslot[2][2][2][BM];       // [tile][phase & 1][half][row]: exchanged row maxima, then l
  uint32_t tmem_base;
  int abort;
};

// Shared-memory layout for Q/K rows of QKR bytes and P/V rows of PVR bytes
// (64 for E2M1, 128 for E4M3).
// stage: K codes | V codes | K sf | V sf | delta_s tile
// CTA: Q_A | Q_B | P_A[2] | P_B[2] | stages | Q sf A,B | P sf A[2],B[2] | ones A,B | zeros | barriers
// P (codes and scales) is double-buffered per query tile: key tile j writes
// buffer j & 1 while PV(j-1) may still read the other one.
template <int QKR, int PVR>
struct FL {
  static constexpr int QK_TILE = 128 * QKR;   // a Q or K tile
  static constexpr int PV_TILE = 128 * PVR;   // a P or V^T tile
  static constexpr int ST_K = 0, ST_V = QK_TILE, ST_KSF = QK_TILE + PV_TILE, ST_VSF = ST_KSF + SF_TILE,
                       ST_DS = ST_VSF + SF_TILE;
  static constexpr int STAGE_BYTES = (ST_DS + DS_TILE + 1023) / 1024 * 1024;
  static constexpr int OFF_Q = 0, OFF_P = 2 * QK_TILE, OFF_STAGE = 2 * QK_TILE + 4 * PV_TILE;
  static constexpr int FIXED =
      1024 + OFF_STAGE + 6 * SF_TILE + 2 * ONES_TILE + ZERO_TILE + static_cast<int>(sizeof(Bars));
  static constexpr int STAGES = (227 * 1024 - FIXED) / STAGE_BYTES < MAX_STAGES
                                    ? (227 * 1024 - FIXED) / STAGE_BYTES : MAX_STAGES;
  static constexpr int OFF_QSF = OFF_STAGE + STAGES * STAGE_BYTES;
  static constexpr int OFF_PSF = OFF_QSF + 2 * SF_TILE;
  static constexpr int OFF_ONES = OFF_PSF + 4 * SF_TILE;
  static constexpr int OFF_ZERO = OFF_ONES + 2 * ONES_TILE;  // above every tile whose descriptor points here
  static constexpr int OFF_BAR = OFF_ZERO + ZERO_TILE;
  static constexpr size_t SMEM_BYTES = 1024 + OFF_BAR + sizeof(Bars);
  static_assert(STAGES >= 2 && SMEM_BYTES <= 227 * 1024, "flash layout");
  static_assert(ST_DS % 1024 == 0 && STAGE_BYTES % 1024 == 0 && OFF_STAGE % 1024 == 0 && OFF_ZERO % 1024 == 0,
                "128-byte-swizzle atoms of the delta_s operands must be 1024-byte aligned");
  static_assert(OFF_ZERO - OFF_STAGE < (1 << 18), "descriptor byte offsets are 14-bit multiples of 16");
};
__host__ __device__ constexpr int fmt_row(int f) { return fmt_e4m3(f) ? 128 : 64; }
template <int kQK, int kPV>
using FLay = FL<fmt_row(kQK), fmt_row(kPV)>;
__device__ __forceinline__ uint64_t code_desc(bool f8, const void* p) {
  return f8 ? smem_desc_sw128(p) : smem_desc_sw64(p);
}

struct Params {
  int H, L, Lp, T;  // T = Lp / 128
  int D;            // head dim stored (32, 64, 96 or 128; the channels above D are zero)
  int64_t o_sb, o_sn, o_sh;
  float qk_scale;   // sm_scale * log2(e)
  int causal;
  int smoothing;
  float p_prescale;      // emulated-config P prescale: 448*6 (two-level) or 1 (single-level _s1)
  float p_prescale_lg2;  // log2(p_prescale)
  int vsmooth;           // the V mean was subtracted before quantisation: add it back to O / l
  const float* vmean;    // [BH, 128] the V means (values of the input dtype), when vsmooth
  int f16;               // inputs, delta_s and the output are fp16, else bf16
};

// Kernel variants are <Q/K format, P/V format, emulated P handling>:
//   hardware-kernel P (kEmu = false): P quantised per 32 keys with E8M0
//     2^ceil(log2(max p / fmt_max)), l = sum of the unquantised p
//     (mxfp4_hw_kernel.py / mxfp8_hw_kernel.py and the mixed _hw kernels);
//   emulated-config P (kEmu = true): p times a prescale (448*6 for the
//     two-level configs, 1 for the single-level _s1 ones), block-quantised,
//     l = sum of the dequantised P (p_quant_kernels.py, attention_kernel.py).
// F_NV4B32 (mxfp4_s1_e4m3) runs on the block16 MMA with each per-32 E4M3
// scale in both of its 16-element slots, which multiplies every element by
// the same scale as one per-32 slot would.

// acc + the sum of 2 * value over eight non-negative E2M1 codes (one per
// nibble of w): prmt looks each 3-bit magnitude up in {0, 1, 2, 3, 4, 6, 8,
// 12} (twice the E2M1 values, one byte each) and dp4a adds the bytes; exact.
__device__ __forceinline__ uint32_t e2m1x8_sum2(uint32_t w, uint32_t acc) {
  const uint32_t lo = __byte_perm(0x03020100u, 0x0C080604u, w & 0xFFFFu);
  const uint32_t hi = __byte_perm(0x03020100u, 0x0C080604u, w >> 16);
  return __dp4a(hi, 0x01010101u, __dp4a(lo, 0x01010101u, acc));
}
// A small non-negative integer (< 2^23) as a float, without the I2F unit.
__device__ __forceinline__ float small_u2f(uint32_t v) {
  return __uint_as_float(0x4B000000u | v) - 8388608.0f;
}

// Shared-memory accesses through 32-bit shared-window addresses.
__device__ __forceinline__ void sts128(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w) : "memory");
}
__device__ __forceinline__ void sts64(uint32_t a, uint32_t x, uint32_t y) {
  asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(a), "r"(x), "r"(y) : "memory");
}
__device__ __forceinline__ void reg_alloc_softmax() { asm volatile("setmaxnreg.inc.sync.aligned.u32 104;"); }
__device__ __forceinline__ void reg_dealloc_others() { asm volatile("setmaxnreg.dec.sync.aligned.u32 64;"); }
__device__ __forceinline__ void sts16(uint32_t a, uint32_t x) {
  asm volatile("st.shared.u16 [%0], %1;" ::"r"(a), "h"(static_cast<unsigned short>(x)) : "memory");
}
__device__ __forceinline__ void sts32(uint32_t a, uint32_t x) {
  asm volatile("st.shared.b32 [%0], %1;" ::"r"(a), "r"(x) : "memory");
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ float lg2_approx(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^e as a float for e in [-127, 127] (2^-127 is the subnormal 0x00400000).
__device__ __forceinline__ float exp2i(int e) {
  return __uint_as_float(e + 127 > 0 ? static_cast<uint32_t>(e + 127) << 23 : 0x00400000u);
}

// E8M0 block exponent of the reference for a finite amax >= 0:
// e = clamp(ceil(log2(q)), -127, 127) with q = amax / 6 rounded to fp32 and
// the ceiling read from q's bits (exponent field - 127, plus 1 if the
// mantissa is nonzero).  Without the division: for amax = M * 2^E
// (1 <= M < 2), q = (M / 1.5) * 2^(E-2) and its rounded value has a zero
// mantissa iff M == 1.5 or rounds up to 2^(E-2), so the ceiling is
// E - 2 + (M > 1.5) whenever q is normal (amax exponent field >= 3).  Below
// that q is subnormal (ceiling read as -126) or rounds to 0 (-127, amax at
// most 3 * 2^-149).
__device__ __forceinline__ int mx_block_exp(float amax) {
  const uint32_t b = __float_as_uint(amax);
  const int ex = static_cast<int>(b >> 23);
  const int e = ex < 3 ? (b > 3u ? -126 : -127) : ex - 129 + ((b & 0x7FFFFFu) > 0x400000u);
  return min(e, 127);
}

// E8M0 block exponent of the mxfp8_hw kernel's P for a finite amax >= 0:
// e = clamp(ceil(log2(amax / 448)), -127, 127).  For amax = M * 2^E
// (1 <= M < 2) the quotient is (M / 1.75) * 2^(E-8) with a zero mantissa only
// at M == 1.75, so the ceiling is E - 8 + (M > 1.75); amax exponent fields
// below 8 (a quotient under 2^-127) clamp to -127, and so does amax = 0.
__device__ __forceinline__ int mx8_block_exp(float amax) {
  const uint32_t b = __float_as_uint(amax);
  const int e = static_cast<int>(b >> 23) - 135 + ((b & 0x7FFFFFu) > 0x600000u ? 1 : 0);
  return min(max(e, -127), 127);
}

// The block-scaled MMAs of a 128 x 128 x 128 product: two K=64 (E2M1) or
// four K=32 (E4M3) instructions.
template <int kFmt>
__device__ __forceinline__ void mma_k128(uint32_t d, uint64_t da, uint64_t db, uint32_t sfa, uint32_t sfb,
                                         bool accumulate_first) {
  constexpr bool kNV = fmt_block16(kFmt);
  if (fmt_e4m3(kFmt)) {
    constexpr uint32_t idesc8 = idesc_mxf8(BM, BN);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {  // 32 E4M3 = 32 bytes per step; scale byte kk of the chunk
      const uint32_t sf_id = kk;
      mma_mxf8(d, da + kk * 2, db + kk * 2, idesc_with_sf_ids(idesc8, sf_id, sf_id), sfa | (sf_id << 30),
               sfb | (sf_id << 30), accumulate_first || kk);
    }
    return;
  }
  constexpr uint32_t idesc = idesc_mxf4(BM, BN, !kNV);
#pragma unroll
  for (int kk = 0; kk < 2; ++kk) {
    if (kNV) {  // UE4M3 per 16 (F_NV4B32: each scale twice): MMA kk reads scale chunk kk
      mma_nvf4(d, da + kk * 2, db + kk * 2, idesc, sfa + 4 * kk, sfb + 4 * kk, accumulate_first || kk);
    } else {    // UE8M0 per 32: scale bytes 2kk, 2kk+1 of the chunk
      const uint32_t sf_id = kk * 2;
      mma_mxf4(d, da + kk * 2, db + kk * 2, idesc_with_sf_ids(idesc, sf_id, sf_id), sfa | (sf_id << 30),
               sfb | (sf_id << 30), accumulate_first || kk);
    }
  }
}
// Scale chunk(s) at shared-memory descriptor d -> TMEM (NVFP4: two chunks).
template <bool kNV>
__device__ __forceinline__ void cp_sf_d(uint32_t taddr, uint64_t d) {
  tmem_cp_sf(taddr, d);
  if (kNV) tmem_cp_sf(taddr + 4, d + (SF_CHUNK >> 4));
}
template <bool kNV>
__device__ __forceinline__ void cp_sf(uint32_t taddr, const uint8_t* smem_sf) {
  cp_sf_d<kNV>(taddr, smem_desc_sf(smem_sf));
}


// max of v[0 .. 16) and of v[0 .. 32), three-input max (sm_100)
__device__ __forceinline__ float max16(const float* v) {
  const float a0 = fmax3(v[0], v[1], v[2]), a1 = fmax3(v[3], v[4], v[5]), a2 = fmax3(v[6], v[7], v[8]);
  const float a3 = fmax3(v[9], v[10], v[11]), a4 = fmax3(v[12], v[13], v[14]);
  return fmaxf(fmax3(a0, a1, a2), fmax3(a3, a4, v[15]));
}
__device__ __forceinline__ float max32(const float* v) {
  float a[10];
#pragma unroll
  for (int i = 0; i < 10; ++i) a[i] = fmax3(v[3 * i], v[3 * i + 1], v[3 * i + 2]);
  const float b0 = fmax3(a[0], a[1], a[2]), b1 = fmax3(a[3], a[4], a[5]), b2 = fmax3(a[6], a[7], a[8]);
  const float b3 = fmax3(a[9], v[30], v[31]);
  return fmaxf(fmax3(b0, b1, b2), b3);
}

// ---------------------------------------------------------------------------
// softmax warpgroup: one query tile, thread = row
// ---------------------------------------------------------------------------
// Sum of four E4M3 bytes (exact in fp32).
__device__ __forceinline__ float e4m3x4_sum(uint32_t w) {
  uint32_t h0, h1;
  asm("{\n\t.reg .b16 lo, hi;\n\t"
      "mov.b32 {lo, hi}, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, lo;\n\t"
      "cvt.rn.f16x2.e4m3x2 %1, hi;\n\t}"
      : "=r"(h0), "=r"(h1)
      : "r"(w));
  return (f16lo(h0) + f16hi(h0)) + (f16lo(h1) + f16hi(h1));
}

// A row's value from the partner thread (same query tile and row, other half
// of the keys): both warps write theirs into slot ph & 1 and meet at the
// pair's named barrier (1 + 4 wg + quad, 64 threads), which also orders the
// shared-memory writes before the reads.  A thread cannot reach exchange
// ph + 2, which reuses the slot, before its partner has passed exchange
// ph + 1, i.e. has read exchange ph's value.  The barrier cannot be left
// waiting: the two warps run the same nkv + 1 exchanges on every path (a
// timed-out wait stops waiting but never leaves the loop), and warps of an
// unused query tile skip softmax_wg together.
__device__ __forceinline__ float pair_exchange(Bars* bars, int wg, int hf, int quad, int r, float v, int ph) {
  volatile float* slot = &bars->xslot[wg][ph & 1][0][0];
  slot[hf * BM + r] = v;
  asm volatile("bar.sync %0, 64;" ::"r"(1 + wg * 4 + quad) : "memory");
  return slot[(hf ^ 1) * BM + r];
}

// One softmax thread: query row r of tile wg and keys [64 hf, 64 hf + 64) of
// every key tile.  Warps (wg, hf = 0, quad) and (wg, hf = 1, quad) share TMEM
// lanes 32 quad .. 32 quad + 31 (the rows) and split the 128 S / O columns.
template <int kQK, int kPV, bool kEmu>
__device__ __forceinline__ void softmax_wg(uint8_t* smem, Bars* bars, uint32_t tmem, const Params& p, int wg, int hf,
                                           int quad, int qt, int bh, int nkv, __nv_bfloat16* __restrict__ out,
                                           int* status) {
  constexpr bool kNV = kPV == F_NV4;
  constexpr bool kP8 = fmt_e4m3(kPV);
  constexpr bool kG9 = kPV == F_G9;          // the reference's 9-level grid, as E4M3 codes
  constexpr bool kE4S32 = kPV == F_NV4B32;   // E4M3 scale per 32 keys
  using Lay = FLay<kQK, kPV>;
  constexpr int NG = kNV ? 8 : 4;            // scale blocks per row of 128 keys
  constexpr int NGH = NG / 2;                // of them in this thread's half
  constexpr int HB = BN / 2;                 // keys per half
  const int warp = quad;
  const int lane = threadIdx.x & 31;
  const int r = warp * 32 + lane;            // query row in the tile = TMEM lane
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
  const uint32_t t_o = tmem + T_O + wg * 128 + hf * HB;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t prow0 = sbase + Lay::OFF_P + 2 * wg * Lay::PV_TILE + r * fmt_row(kPV);      // this row of P
  const uint32_t psf0 = sbase + Lay::OFF_PSF + 2 * wg * SF_TILE + (r & 31) * 16 + (r >> 5) * 4;  // its scale word
  // swizzle of this row's 16-byte chunks: 64-byte (E2M1) or 128-byte (E4M3) pattern
  const int swz = kP8 ? (r & 7) : ((r >> 1) & 3);
  const float qk = p.qk_scale;
  const int qrow = qt * BM + r;
  float m_run = -INFINITY, l_run = 0.f;
  bool ok = true;
  for (int j = 0; j < nkv; ++j) {
    // After a failed (timed-out) wait the thread stops waiting but keeps
    // iterating, so the other roles are never left waiting on it.
    if (ok) ok = mbar_wait(&bars->s_full[wg], j & 1, status, 0x1301);
    ok = __all_sync(0xffffffffu, ok);  // warp-uniform: the TMEM accesses below are .sync.aligned
    tc_fence_after();
    float x[HB];
#pragma unroll
    for (int c = 0; c < HB; c += 32) {
      uint32_t u[32];
      tmem_ld32(tmem + lane_base + T_S + hf * HB + c, u);
#pragma unroll
      for (int i = 0; i < 32; ++i) x[c + i] = __uint_as_float(u[i]);
    }
    tmem_ld_wait();
    tc_fence_before();
    mbar_arrive(&bars->s_free[wg]);
    // masking: keys beyond L (last tile) and, if causal, keys after the query
    const int key0 = j * BN + hf * HB;
    const int lim = p.causal ? min(p.L - key0, qrow - key0 + 1) : p.L - key0;
    if (lim < HB) {
#pragma unroll
      for (int i = 0; i < HB; ++i)
        if (i >= lim) x[i] = -INFINITY;
    }
    // block maxima of the scores; the row max (with the partner's half) and
    // each block's max of p (p = exp2(x * qk - m) is monotone in x) follow
    float gm[NGH];
#pragma unroll
    for (int g = 0; g < NGH; ++g) gm[g] = kNV ? max16(x + 16 * g) : max32(x + 32 * g);
    const float mh = kNV ? fmaxf(fmaxf(gm[0], gm[1]), fmaxf(gm[2], gm[3])) : fmaxf(gm[0], gm[1]);
    const float mx = fmaxf(mh, pair_exchange(bars, wg, hf, quad, r, mh, j));
    const float m_new = fmaxf(m_run, mx * qk);
    const bool grow = (m_new > m_run) && (m_run != -INFINITY);
    const float alpha = grow ? ex2_approx(m_run - m_new) : 1.0f;
    l_run *= alpha;
    m_run = m_new;
    // P(j) goes to buffer j & 1; PV(j-2), its previous reader, completed before
    // p_full(j-1) was signalled (the o_done wait below, one tile earlier).
    // Block g below is this half's block g (the row's block hf * NGH + g).
    const uint32_t prow = prow0 + (j & 1) * Lay::PV_TILE;
    const uint32_t psf = psf0 + (j & 1) * SF_TILE;
    const float2 qk2 = make_float2(qk, qk);
    if (!kEmu && kP8) {
      // P -> E4M3 codes (round-to-nearest-even, saturating at 448 as the
      // reference's min(., 448)) with E8M0 2^e per 32 keys,
      // e = clamp(ceil(log2(max p / 448)), -127, 127), folded into the
      // exponent as for E2M1; l += sum of the unquantised p.
      uint32_t sfw = 0;
      float lsum = 0.f;
#pragma unroll
      for (int g = 0; g < NGH; ++g) {
        const int gg = hf * NGH + g;
        const int e = mx8_block_exp(ex2_approx(fmaf(gm[g], qk, -m_new)));
        const float cg = -m_new - static_cast<float>(e);
        const float2 c2 = make_float2(cg, cg);
        float2 acc[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
        uint32_t w[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          float v[4];
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int n = g * 32 + q * 4 + 2 * i;
            const float2 t = fma_f32x2(make_float2(x[n], x[n + 1]), qk2, c2);
            v[2 * i] = ex2_approx(t.x);
            v[2 * i + 1] = ex2_approx(t.y);
            acc[i] = add_f32x2(acc[i], make_float2(v[2 * i], v[2 * i + 1]));
          }
          w[q] = cvt_e4m3x4(v[0], v[1], v[2], v[3]);
        }
        const float2 a = add_f32x2(acc[0], acc[1]);
        lsum = fmaf(a.x + a.y, exp2i(e), lsum);
        sts128(prow + (((2 * gg) ^ swz) << 4), w[0], w[1], w[2], w[3]);
        sts128(prow + (((2 * gg + 1) ^ swz) << 4), w[4], w[5], w[6], w[7]);
        sfw |= static_cast<uint32_t>(e + 127) << (8 * g);
      }
      l_run += lsum;
      sts16(psf + 2 * hf, sfw);
    } else if (!kEmu) {
      // P -> E2M1 codes (round-to-nearest-even) with E8M0 2^e per 32 keys,
      // e = clamp(ceil(log2(max p / 6)), -127, 127).  The block scale is folded
      // into the exponent: p * 2^-e = exp2(x * qk - m - e).  l += sum of p
      // = sum over blocks of 2^e * sum(p * 2^-e).
      uint32_t sfw = 0;
      float lsum = 0.f;
#pragma unroll
      for (int g = 0; g < NGH; ++g) {
        const int gg = hf * NGH + g;
        const int e = mx_block_exp(ex2_approx(fmaf(gm[g], qk, -m_new)));
        const float cg = -m_new - static_cast<float>(e);
        const float2 c2 = make_float2(cg, cg);
        float2 acc[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
        uint32_t w[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float v[8];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int n = g * 32 + q * 8 + 2 * i;
            const float2 t = fma_f32x2(make_float2(x[n], x[n + 1]), qk2, c2);
            v[2 * i] = ex2_approx(t.x);
            v[2 * i + 1] = ex2_approx(t.y);
            acc[i & 1] = add_f32x2(acc[i & 1], make_float2(v[2 * i], v[2 * i + 1]));
          }
          w[q] = cvt_e2m1x8(v[0], v[1], v[2], v[3], v[4], v[5], v[6], v[7]);
        }
        const float2 a = add_f32x2(acc[0], acc[1]);
        lsum = fmaf(a.x + a.y, exp2i(e), lsum);
        sts128(prow + ((gg ^ swz) << 4), w[0], w[1], w[2], w[3]);
        sfw |= static_cast<uint32_t>(e + 127) << (8 * g);
      }
      l_run += lsum;
      sts16(psf + 2 * hf, sfw);
    } else if (kP8) {
      // Emulated single-level MXFP8 P (p_quant_mxfp8_s1): E8M0 2^e per 32 keys,
      // e = clamp(ceil(log2(max(max p / 448, 1e-8))), -127, 127), E4M3 codes
      // of p * 2^-e (the fp8 cast, round-to-nearest-even); l += sum of the
      // dequantised P.
      // kG9 (p_quant_mxfp4 / p_quant_mxfp4_s1): the same with max / 6 and the
      // reference's 9-level grid (ties upward), held as E4M3 codes.
      // The prescale and 2^-e are folded into the exponent:
      // p * prescale * 2^-e = exp2(x * qk - m + log2(prescale) - e).
      uint32_t sfw = 0;
      float lq = 0.f;
#pragma unroll
      for (int g = 0; g < NGH; ++g) {
        const int gg = hf * NGH + g;
        const float amax = __fmul_rn(ex2_approx(fmaf(gm[g], qk, -m_new)), p.p_prescale);
        const int e = max(kG9 ? mx_block_exp(amax) : mx8_block_exp(amax), -26);  // ceil(log2(1e-8)) = -26
        const float cg = p.p_prescale_lg2 - m_new - static_cast<float>(e);
        const float2 c2 = make_float2(cg, cg);
        uint32_t w[8];
        float gsum = 0.f;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          float v[4];
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int n = g * 32 + q * 4 + 2 * i;
            const float2 t = fma_f32x2(make_float2(x[n], x[n + 1]), qk2, c2);
            v[2 * i] = ex2_approx(t.x);
            v[2 * i + 1] = ex2_approx(t.y);
          }
          if (kG9) {
#pragma unroll
            for (int i = 0; i < 4; ++i) v[i] = grid9_mag(v[i]);
          }
          w[q] = cvt_e4m3x4(v[0], v[1], v[2], v[3]);
          gsum += e4m3x4_sum(w[q]);
        }
        lq = fmaf(gsum, exp2i(e), lq);
        sts128(prow + (((2 * gg) ^ swz) << 4), w[0], w[1], w[2], w[3]);
        sts128(prow + (((2 * gg + 1) ^ swz) << 4), w[4], w[5], w[6], w[7]);
        sfw |= static_cast<uint32_t>(e + 127) << (8 * g);
      }
      l_run += lq;
      sts16(psf + 2 * hf, sfw);
    } else {
      // Emulated configs: p = exp2(x * qk - m), times the prescale (448*6 for
      // the two-level configs, which cancels in O / l; 1 for the single-level
      // _s1 ones), block-quantised; l += sum of the dequantised P.
      //   MXFP4: E8M0 2^e per 32, e = clamp(ceil(log2(max / 6)), -127, 127);
      //   NVFP4: E4M3 per 16, s = e4m3(max(max / 6, 1e-8));
      //   E4M3 per 32: s = max(e4m3(max(max / 6, 1e-8)), 2^-9).
      // The block max of p * prescale is round(max p * prescale) (rounding is
      // monotone).  prescale / s is folded into the exponent:
      // p * prescale / s = exp2(x * qk - m + log2(prescale) - log2(s)), log2(s)
      // exact for the power-of-two scales and lg2.approx for the E4M3 ones
      // (a zero E4M3 scale zeroes its block in the MMA; its codes are then
      // taken at 2^-9).
      float lq = 0.f;
      uint32_t sfw = 0u;
#pragma unroll
      for (int g = 0; g < NGH; ++g) {
        constexpr int GS = BN / NG;
        const int gg = hf * NGH + g;
        const float amax = __fmul_rn(ex2_approx(fmaf(gm[g], qk, -m_new)), p.p_prescale);
        float deq, lg2s;
        uint32_t sbyte;
        if (kNV || kE4S32) {
          const float scl = fmaxf(amax * (1.0f / 6.0f), 1e-8f);
          sbyte = e4m3_byte(scl);
          deq = round_e4m3(scl);
          if (kE4S32) {  // p_quant_mxfp4_s1_e4m3 clamps at the smallest E4M3 subnormal (byte 1)
            sbyte = max(sbyte, 1u);
            deq = fmaxf(deq, 1.953125e-3f);
          }
          lg2s = lg2_approx(fmaxf(deq, 1.953125e-3f));
        } else {
          const int e = max(mx_block_exp(amax), -26);  // the scale's max(., 1e-8): ceil(log2(1e-8)) = -26
          sbyte = static_cast<uint32_t>(e + 127);
          deq = exp2i(e);
          lg2s = static_cast<float>(e);
        }
        const float cg = p.p_prescale_lg2 - m_new - lg2s;
        const float2 c2 = make_float2(cg, cg);
        uint32_t isum = 0;  // sum of 2 * the block's E2M1 values (p >= 0: no sign bits)
        uint32_t w[GS / 8];
#pragma unroll
        for (int q = 0; q < GS / 8; ++q) {
          float v[8];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int n = g * GS + q * 8 + 2 * i;
            const float2 t = fma_f32x2(make_float2(x[n], x[n + 1]), qk2, c2);
            v[2 * i] = ex2_approx(t.x);
            v[2 * i + 1] = ex2_approx(t.y);
          }
          w[q] = cvt_e2m1x8(v[0], v[1], v[2], v[3], v[4], v[5], v[6], v[7]);
          isum = e2m1x8_sum2(w[q], isum);
        }
        lq = fmaf(small_u2f(isum), 0.5f * deq, lq);
        if (kNV) {
          // 16-byte chunk gg/2 of the row holds blocks 2*(gg/2), 2*(gg/2)+1
          sts64(prow + (((gg >> 1) ^ swz) << 4) + (gg & 1) * 8, w[0], w[1]);
          sfw |= sbyte << (8 * g);  // scale chunk hf holds this half's 4 blocks
        } else if (kE4S32) {
          // block gg fills 16-element scale slots 2gg and 2gg+1 (chunk hf)
          sts128(prow + ((gg ^ swz) << 4), w[0], w[1], w[2], w[3]);
          sfw |= (sbyte * 0x101u) << (16 * g);
        } else {
          sts128(prow + ((gg ^ swz) << 4), w[0], w[1], w[2], w[3]);
          sfw |= sbyte << (8 * g);
        }
      }
      l_run += lq;
      if (kNV || kE4S32) sts32(psf + hf * SF_CHUNK, sfw);
      else sts16(psf + 2 * hf, sfw);
    }
    // O holds PV(0 .. j-1): rescale it by alpha once PV(j-1) has completed and
    // before PV(j) is issued (p_full).  All four column chunks in flight at once.
    if (ok && j >= 1) ok = mbar_wait(&bars->o_done[wg], (j - 1) & 1, status, 0x1303);
    ok = __all_sync(0xffffffffu, ok);
    if (__any_sync(0xffffffffu, grow)) {
      tc_fence_after();
      uint32_t u[HD / 64][32];
#pragma unroll
      for (int c = 0; c < HD / 64; ++c) tmem_ld32(t_o + lane_base + 32 * c, u[c]);
      tmem_ld_wait();
#pragma unroll
      for (int c = 0; c < HD / 64; ++c) {
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float2 v = mul_f32x2(make_float2(__uint_as_float(u[c][i]), __uint_as_float(u[c][i + 1])),
                                     make_float2(alpha, alpha));
          u[c][i] = __float_as_uint(v.x);
          u[c][i + 1] = __float_as_uint(v.y);
        }
        tmem_st32(t_o + lane_base + 32 * c, u[c]);
      }
      tmem_st_wait();
    }
    fence_proxy_async_smem();
    tc_fence_before();
    mbar_arrive(&bars->p_full[wg]);
  }
  // ---------------- epilogue: O / l -> bf16 / fp16 NHD
  const float l_row = l_run + pair_exchange(bars, wg, hf, quad, r, l_run, nkv);
  if (ok && nkv > 0) ok = mbar_wait(&bars->o_done[wg], (nkv - 1) & 1, status, 0x1304);
  ok = __all_sync(0xffffffffu, ok);
  tc_fence_after();
  const bool store = ok && !*(volatile int*)&bars->abort && qrow < p.L;
  const float inv_l = 1.0f / l_row;
  const int b = bh / p.H, h = bh % p.H;
  __nv_bfloat16* orow = out + b * p.o_sb + static_cast<int64_t>(qrow) * p.o_sn + h * p.o_sh + hf * HB;
#pragma unroll 1
  for (int c = 0; c < HB; c += 32) {
    uint32_t u[32];
    tmem_ld32(t_o + lane_base + c, u);
    tmem_ld_wait();
    if (store && hf * HB + c < p.D) {
      float add[32];
      if (p.vsmooth) {  // softmax rows sum to 1: O + v_mean is the attention of the uncentred V
        const float4* vm = reinterpret_cast<const float4*>(p.vmean + static_cast<int64_t>(bh) * HD + hf * HB + c);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 t = __ldg(vm + i);
          add[4 * i] = t.x;
          add[4 * i + 1] = t.y;
          add[4 * i + 2] = t.z;
          add[4 * i + 3] = t.w;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) add[i] = 0.f;
      }
      uint4* dst = reinterpret_cast<uint4*>(orow + c);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float lo = fmaf(__uint_as_float(u[q * 8 + 2 * i]), inv_l, add[q * 8 + 2 * i]);
          const float hi = fmaf(__uint_as_float(u[q * 8 + 2 * i + 1]), inv_l, add[q * 8 + 2 * i + 1]);
          w[i] = p.f16 ? pack_f16x2(lo, hi) : pack_bf16x2(lo, hi);
        }
        dst[q] = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
  }
}

template <int kQK, int kPV, bool kEmu>
__global__ void __launch_bounds__(THREADS, 1)
sage3_fp4_flash_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                       const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_ds,
                       const uint8_t* __restrict__ qsf, const uint8_t* __restrict__ ksf,
                       const uint8_t* __restrict__ vsf, __nv_bfloat16* __restrict__ out, Params p, int* status) {
  constexpr bool kNVq = fmt_block16(kQK), kNVp = fmt_block16(kPV);   // two scale chunks per tile
  constexpr bool kQ8 = fmt_e4m3(kQK), kP8 = fmt_e4m3(kPV);  // 128-byte code rows
  using Lay = FLay<kQK, kPV>;
  constexpr int STAGES = Lay::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + Lay::OFF_BAR);
  const int warp = threadIdx.x >> 5;
  const int qtA = 2 * blockIdx.x;
  const int qtB = qtA + 1;
  const bool hasB = qtB < p.T;
  const int nq = hasB ? 2 : 1;
  const int bh = blockIdx.y;
  const int nkv = p.causal ? qtA + nq : p.T;  // causal: keys up to the last query row of the CTA
  constexpr int kSfQK = kNVq ? SF_TILE : SF_CHUNK, kSfPV = kNVp ? SF_TILE : SF_CHUNK;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bars->kv_full[s], 1);
      mbar_init(&bars->kv_empty[s], 2);  // one commit from each MMA issuer
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->s_free[i], 2 * BM);
      mbar_init(&bars->p_full[i], 2 * BM);
      mbar_init(&bars->o_done[i], 1);
    }
    mbar_init(&bars->drain[0], 1);
    mbar_init(&bars->drain[1], 1);
    bars->abort = 0;
    fence_barrier_init();
    prefetch_tmap(&map_q);
    prefetch_tmap(&map_k);
    prefetch_tmap(&map_v);
    if (p.smoothing) prefetch_tmap(&map_ds);
  }
  if (p.smoothing) {
    // delta_s MMA operands: every stage's delta_s tile and the zero tile start
    // at zero (the TMA writes only K-rows 0-1 of each atom); ones tile t has
    // 1.0 (the input dtype) in column t of each 16-byte row
    for (int s = 0; s < STAGES; ++s)
      for (int i = threadIdx.x; i < DS_TILE / 16; i += THREADS)
        *reinterpret_cast<uint4*>(smem + Lay::OFF_STAGE + s * Lay::STAGE_BYTES + Lay::ST_DS + 16 * i) =
            make_uint4(0, 0, 0, 0);
    for (int i = threadIdx.x; i < (2 * ONES_TILE + ZERO_TILE) / 16; i += THREADS) {
      const int t = i / (ONES_TILE / 16);  // 0, 1: ones tiles; 2: zero tile
      const uint32_t one = p.f16 ? 0x3C00u : 0x3F80u;  // 1.0 in fp16 / bf16, the delta_s rows' type
      *reinterpret_cast<uint4*>(smem + Lay::OFF_ONES + 16 * i) =  // element t of the row = 1.0
          make_uint4(t == 0 ? one : (t == 1 ? one << 16 : 0u), 0u, 0u, 0u);
    }
    fence_proxy_async_smem();  // visible to the TMA unit and the tensor core
  }
  if (warp == MMA_WARP) {
    tmem_alloc(&bars->tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp < MMA_WARP) {
    reg_alloc_softmax();
    const int wg = warp >> 3;  // query tile
    if (wg < nq)
      softmax_wg<kQK, kPV, kEmu>(smem, bars, tmem, p, wg, (warp >> 2) & 1, warp & 3, qtA + wg, bh, nkv, out, status);
  } else {
    reg_dealloc_others();
    if (warp == TMA_WARP) {
      // ------------------------------------------------------------ producer
      if (elect_one()) {
        mbar_arrive_expect_tx(&bars->q_full, nq * (Lay::QK_TILE + kSfQK));
        for (int t = 0; t < nq; ++t) {
          tma_load_2d(smem + Lay::OFF_Q + t * Lay::QK_TILE, &map_q, 0, bh * p.Lp + (qtA + t) * BM, &bars->q_full);
          bulk_load(smem + Lay::OFF_QSF + t * SF_TILE, qsf + (static_cast<int64_t>(bh) * p.T + qtA + t) * SF_TILE,
                    kSfQK, &bars->q_full);
        }
        int issued = 0;
        for (int j = 0; j < nkv; ++j) {
          const int s = j % STAGES;
          if (!mbar_wait(&bars->kv_empty[s], ((j / STAGES) & 1) ^ 1, status, 0x1101)) {
            bars->abort = 1;
            break;
          }
          if (*(volatile int*)&bars->abort) break;
          uint8_t* st = smem + Lay::OFF_STAGE + s * Lay::STAGE_BYTES;
          const uint32_t bytes = Lay::QK_TILE + Lay::PV_TILE + kSfQK + kSfPV + (p.smoothing ? DS_TX : 0);
          mbar_arrive_expect_tx(&bars->kv_full[s], bytes);
          tma_load_2d(st + Lay::ST_K, &map_k, 0, bh * p.Lp + j * BN, &bars->kv_full[s]);
          tma_load_2d(st + Lay::ST_V, &map_v, j * (kP8 ? BN : BN / 2), bh * HD, &bars->kv_full[s]);
          bulk_load(st + Lay::ST_KSF, ksf + (static_cast<int64_t>(bh) * p.T + j) * SF_TILE, kSfQK,
                    &bars->kv_full[s]);
          bulk_load(st + Lay::ST_VSF, vsf + (static_cast<int64_t>(bh) * p.T + j) * SF_TILE, kSfPV,
                    &bars->kv_full[s]);
          if (p.smoothing)  // delta_s rows qtA, qtA + 1 (zero-filled past the last row) of keys j*128 + [0, 128)
            for (int h = 0; h < 2; ++h)
              tma_load_2d(st + Lay::ST_DS + h * 1024, &map_ds, j * BN + h * 64, bh * p.T + qtA, &bars->kv_full[s]);
          ++issued;
        }
        mbar_wait(&bars->q_full, 0, status, 0x1102);
        for (int j = (issued > STAGES ? issued - STAGES : 0); j < issued; ++j)
          mbar_wait(&bars->kv_full[j % STAGES], (j / STAGES) & 1, status, 0x1103);
      }
    } else if (warp == MMA_WARP) {
      // ---------------------------------------------------- QK (S) MMA issuer
      if (elect_one()) {
        bool ok = mbar_wait(&bars->q_full, 0, status, 0x1201);
        if (ok) {
          tc_fence_after();
          for (int t = 0; t < nq; ++t) cp_sf<kNVq>(tmem + T_SFQ + t * 8, smem + Lay::OFF_QSF + t * SF_TILE);
        }
        // Descriptors are computed once: a shared-memory descriptor's start
        // address counts 16-byte units (14 bits, no carry out for addresses
        // below 256 KB), so the tile in stage s, or query tile w, is the
        // stage-0 (tile-0) descriptor plus its byte offset / 16.  The delta_s
        // B descriptor's SBO (bits 32-45) is the distance to the zero tile,
        // which shrinks by the same amount as the start grows.
        constexpr uint64_t kStage = Lay::STAGE_BYTES >> 4;
        constexpr uint64_t kDsStep = kStage - (kStage << 32);
        const uint64_t kd0 = code_desc(kQ8, smem + Lay::OFF_STAGE + Lay::ST_K);
        const uint64_t ksf0 = smem_desc_sf(smem + Lay::OFF_STAGE + Lay::ST_KSF);
        const uint64_t qd0 = code_desc(kQ8, smem + Lay::OFF_Q);
        const uint32_t z_addr = smem_u32(smem + Lay::OFF_ZERO);
        const uint32_t a_addr = smem_u32(smem + Lay::OFF_ONES);
        const uint32_t b_addr = smem_u32(smem + Lay::OFF_STAGE + Lay::ST_DS);
        // A: K-major, no swizzle: 8-row core matrices 128 B apart (SBO), K-rows 8-15 -> zeros (LBO)
        // B: MN-major, 128-byte swizzle: 64-key atoms 1024 B apart (LBO), K-rows 8-15 -> zeros (SBO)
        const uint64_t dsa[2] = {smem_desc(a_addr, z_addr - a_addr, 128, 0),
                                 smem_desc(a_addr + ONES_TILE, z_addr - a_addr - ONES_TILE, 128, 0)};
        const uint64_t dsb0 = smem_desc(b_addr, 1024, z_addr - b_addr, 2);
        for (int j = 0; ok && j < nkv; ++j) {
          const int s = j % STAGES;
          if (!mbar_wait(&bars->kv_full[s], (j / STAGES) & 1, status, 0x1203)) { ok = false; break; }
          if (*(volatile int*)&bars->abort) { ok = false; break; }
          const uint64_t su = static_cast<uint64_t>(s);
          for (int w = 0; w < nq && ok; ++w) {
            // S is free once the warpgroup that used it last has read its scores:
            // for A that is B (or A alone) at key tile j-1, for B it is A at key tile j.
            const int prev = w == 0 ? nq - 1 : 0;
            const int prev_j = w == 0 ? j - 1 : j;
            if (prev_j >= 0 && !mbar_wait(&bars->s_free[prev], prev_j & 1, status, 0x1204)) { ok = false; break; }
            tc_fence_after();
            if (w == 0) cp_sf_d<kNVq>(tmem + T_SFK, ksf0 + su * kStage);
            if (p.smoothing)  // S = delta_s of this tile's query group
              mma_f16(tmem + T_S, dsa[w], dsb0 + su * kDsStep, p.f16 ? IDESC_DS_F16 : IDESC_DS, 0);
            mma_k128<kQK>(tmem + T_S, qd0 + static_cast<uint64_t>(w) * (Lay::QK_TILE >> 4), kd0 + su * kStage,
                          tmem + T_SFQ + w * 8, tmem + T_SFK, p.smoothing != 0);
            tc_commit(&bars->s_full[w]);
          }
          if (!ok) break;
          tc_commit(&bars->kv_empty[s]);  // the stage's K side (K, its scales, delta_s) is read
        }
        if (!ok) bars->abort = 1;
        // every tcgen05 op this thread issued has completed before TMEM is released
        tc_commit(&bars->drain[0]);
        mbar_wait(&bars->drain[0], 0, status, 0x1205);
      }
    } else if (warp == PV_WARP) {
      // ------------------------------------------------------ PV MMA issuer
      // A thread of its own, so that a PV issue never delays the next S and
      // each P tile goes to the tensor core as soon as it is complete.  Both
      // issuers' MMAs touch disjoint TMEM (S, SFQ, SFK here; O, SFP, SFV there)
      // and only read the stage, which kv_empty (two commits) releases.
      if (elect_one()) {
        bool ok = true;
        constexpr uint64_t kStage = Lay::STAGE_BYTES >> 4;
        const uint64_t vd0 = code_desc(kP8, smem + Lay::OFF_STAGE + Lay::ST_V);
        const uint64_t vsf0 = smem_desc_sf(smem + Lay::OFF_STAGE + Lay::ST_VSF);
        const uint64_t pd0 = code_desc(kP8, smem + Lay::OFF_P);
        const uint64_t psf0 = smem_desc_sf(smem + Lay::OFF_PSF);
        for (int t = 0; ok && t < nkv; ++t) {
          const int s = t % STAGES;
          // the stage cannot be refilled before this thread's kv_empty commit for tile t
          if (!mbar_wait(&bars->kv_full[s], (t / STAGES) & 1, status, 0x1206)) { ok = false; break; }
          const uint64_t so = static_cast<uint64_t>(s) * kStage;
          for (int w = 0; w < nq; ++w) {
            if (!mbar_wait(&bars->p_full[w], t & 1, status, 0x1202)) { ok = false; break; }
            if (*(volatile int*)&bars->abort) { ok = false; break; }
            tc_fence_after();
            if (w == 0) cp_sf_d<kNVp>(tmem + T_SFV, vsf0 + so);
            const uint64_t pb = static_cast<uint64_t>(2 * w + (t & 1));  // P buffer of key tile t
            cp_sf_d<kNVp>(tmem + T_SFP, psf0 + pb * (SF_TILE >> 4));
            mma_k128<kPV>(tmem + T_O + w * 128, pd0 + pb * (Lay::PV_TILE >> 4), vd0 + so, tmem + T_SFP, tmem + T_SFV,
                          t != 0);
            tc_commit(&bars->o_done[w]);
          }
          if (!ok) break;
          tc_commit(&bars->kv_empty[s]);  // the stage's V side is read
        }
        if (!ok) bars->abort = 1;
        tc_commit(&bars->drain[1]);
        mbar_wait(&bars->drain[1], 0, status, 0x1207);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

template <int kQK, int kPV, bool kEmu>
int launch_mode(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mds,
                const Workspace& w, const Problem& pr, const Params& p, dim3 grid, int* status, cudaStream_t s) {
  constexpr size_t smem = FLay<kQK, kPV>::SMEM_BYTES;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    cudaError_t e = cudaFuncSetAttribute(&sage3_fp4_flash_kernel<kQK, kPV, kEmu>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return fail(QDQ_ERR_CUDA, "sage3 flash: smem attribute: %s", cudaGetErrorString(e));
    attr[dev] = true;
  }
  sage3_fp4_flash_kernel<kQK, kPV, kEmu><<<grid, THREADS, smem, s>>>(mq, mk, mv, mds, w.qsf, w.ksf, w.vsf, pr.o,
                                                                     p, status);
  return check_launch("sage3 flash");
}

int code_map(CUtensorMap* map, const uint8_t* base, int64_t rows, int64_t row_bytes, bool f8) {
  // E2M1 rows of 64 bytes (64-byte swizzle) or E4M3 rows of 128 (128-byte swizzle); 128-row boxes
  return make_tmap_u8_2d(map, base, rows, row_bytes, row_bytes, f8 ? 128 : 64, 128, f8 ? 128 : 64);
}

}  // namespace

int launch_flash(const Problem& pr, const Workspace& w, cudaStream_t s) {
  int* status = device_status_ptr();
  if (status == nullptr) return QDQ_ERR_CUDA;
  const int64_t BH = static_cast<int64_t>(pr.B) * pr.H;
  const bool q8 = fmt_e4m3(pr.qk_fmt), p8 = fmt_e4m3(pr.pv_fmt);
  CUtensorMap mq, mk, mv, mds;
  if (int st = code_map(&mq, w.qc, BH * pr.Lp, q8 ? 128 : 64, q8)) return st;
  if (int st = code_map(&mk, w.kc, BH * pr.Lp, q8 ? 128 : 64, q8)) return st;
  if (int st = code_map(&mv, w.vt, BH * HD, p8 ? pr.Lp : pr.Lp / 2, p8)) return st;
  // delta_s [BH * G, Lp] bf16 / fp16, boxes of 64 keys x 2 query groups, 128-byte swizzle
  if (int st = make_tmap_u16_2d(&mds, w.ds, BH * (pr.Lp / 128), pr.Lp, static_cast<uint64_t>(pr.Lp) * 2, 64, 2, 128))
    return st;
  Params p;
  p.H = pr.H;
  p.L = pr.L;
  p.Lp = pr.Lp;
  p.T = pr.Lp / 128;
  p.D = pr.D;
  p.o_sb = pr.o_sb;
  p.o_sn = pr.o_sn;
  p.o_sh = pr.o_sh;
  p.qk_scale = pr.sm_scale * 1.4426950408889634f;
  p.causal = pr.causal;
  p.smoothing = pr.smoothing;
  p.p_prescale = pr.p_prescale;
  p.p_prescale_lg2 = static_cast<float>(std::log2(static_cast<double>(pr.p_prescale)));
  p.vsmooth = pr.vsmooth;
  p.vmean = w.vmean;
  p.f16 = pr.f16;
  dim3 grid(static_cast<unsigned>((p.T + 1) / 2), static_cast<unsigned>(BH));
  // The flash kernel sees Q / K codes of every E4M3 format alike (F_G9, F_E8
  // and F_MX8 differ only in how the pre-pass quantised them), and P / V of
  // F_E8 like F_MX8; F_G9 P / V keeps its own P quantiser.
  const int qk_fmt = fmt_e4m3(pr.qk_fmt) ? static_cast<int>(F_MX8) : pr.qk_fmt;
  const int pv_fmt = pr.pv_fmt == F_E8 ? static_cast<int>(F_MX8) : pr.pv_fmt;
#define QDQ_FLASH(QK, PV, EMU)                                                             \
  if (qk_fmt == QK && pv_fmt == PV && (pr.emulated != 0) == EMU)                           \
    return launch_mode<QK, PV, EMU>(mq, mk, mv, mds, w, pr, p, grid, status, s);
  QDQ_FLASH(F_MX4, F_MX4, false)   // mxfp4_hw
  QDQ_FLASH(F_NV4, F_NV4, true)    // nvfp4
  QDQ_FLASH(F_MX8, F_MX8, false)   // mxfp8_hw
  QDQ_FLASH(F_MX8, F_MX8, true)    // mxfp8_s1, mixed_fp4qk_fp8pv (+ _vs)
  QDQ_FLASH(F_MX8, F_G9, true)     // mxfp4, mxfp4_s1 (+ vsmooth), mixed_fp8qk_fp4pv (+ _vs)
  QDQ_FLASH(F_MX8, F_MX4, false)   // mixed_mxfp8qk_mxfp4pv_hw
  QDQ_FLASH(F_MX4, F_MX8, false)   // mixed_mxfp4qk_mxfp8pv_hw
  QDQ_FLASH(F_NV4B32, F_NV4B32, true)  // mxfp4_s1_e4m3
#undef QDQ_FLASH
  return fail(QDQ_ERR_UNSUPPORTED, "sage3 flash: no kernel for formats (%d, %d, emulated %d)", pr.qk_fmt, pr.pv_fmt,
              pr.emulated);
}

}  // namespace attn
}  // namespace qdqb200
