// Pre-pass of the Sage3 FP4 attention: QK smoothing + FP4 quantisation of
// Q, K and V, and the delta_s correction, for inputs in the NHD layout
// vllm-omni hands the backend ([B, L, H, D], reference
// sage3_attn/impl.py:102-104 transposes these to HND; here the kernels read
// NHD strides directly).
//
// Reference semantics (mxfp4_hw branch, sage3/api.py:161-206):
//   qk_smoothing (sage3/transforms.py:47-95), applied before padding:
//     k_c  = k - mean_L(k)                      (ops in the input dtype)
//     q_m  = mean over each 128-row group of q, the last group zero-padded
//     q_s  = q - q_m[group]
//     delta_s[g, n] = (q_m[g] . k_c[n]) rounded to the input dtype (its matmul)
//   The input dtype is bf16 or fp16 (kernels templated on kF16); every
//   rounding above is to that dtype, as the reference's torch ops round.
//   quantize_to_mxfp4 (sage3/mxfp4_hw_kernel.py:73-116) of q_s and k_c along
//   D and of V along the sequence, per 32-group:
//     e = clamp(ceil(log2(max(amax, 6*2^-126) / 6)), -127, 127), byte e+127
//     code of x / 2^e with round-half-away thresholds
//   (ceil(log2(.)) is evaluated exactly from the float's bits).
//   mxfp8_hw (sage3/api.py:114-160) quantises the same q_s, k_c and V with
//   quantize_to_mxfp8 (sage3/mxfp8_hw_kernel.py:37-65):
//     e = ceil(log2(max(amax, 1e-12) / 448)), byte clamp(e + 127, 0, 254),
//     code = E4M3 of x / 2^e, round-to-nearest-even (torch's float8_e4m3fn cast).
//   The emulated E8M0 configs (mxfp4, mxfp4_s1, mxfp8_s1 and the mixed ones,
//   formats F_G9 / F_E8) quantise q_s, k_c and V with the reference's own
//   quantize_qk / quantize_v steps instead (emu8_quant32 below), into E4M3
//   codes with E8M0 scales.
//
// Head dims D < 128 (32, 64, 96) are zero-extended to 128 as the rows are
// loaded: the extra channels are zero in Q, K and V, so they add nothing to
// Q K^T, delta_s or P V, and their quantisation groups (whole groups of 32,
// or of 16 for NVFP4) hold only zeros and leave the real groups' scales
// alone.  The flash kernel stores only the first D output channels.
//
// Outputs (workspace), with Lp = L rounded up to 128, BH = B*H, G = Lp/128:
//   ksum   fp32 [BH, D]           per-channel sums of k (mean = dtype(ksum / L))
//   (kernels: colsum_kernel for the K (and V) sums; the Q pass; the K pass,
//   which also writes delta_s; the V pass)
//   qmean  bf16/fp16 [BH, G, D]   Q group means (input dtype)
//   qc, kc uint8 [BH*Lp, D/2]     E2M1 codes (element 2j low nibble), or [BH*Lp, D] E4M3
//   qsf, ksf                      block scales, 1024 bytes per 128 rows: two 512-byte tcgen05
//                                 scale chunks (NVFP4: 8 E4M3 per row; MXFP4: 4 E8M0 in the first;
//                                 E4M3 per 32: 4 scales, each in two adjacent 16-element slots)
//   vt     uint8 [BH*D, Lp/2]     V transposed: row (bh, d), keys packed along the row
//                                 ([BH*D, Lp] for E4M3)
//   vsf                           1024 bytes per (bh, key tile): 128 d-rows x (4 E8M0 | 8 E4M3)
//   ds     bf16/fp16 [BH, G, Lp]  delta_s (the reference's dtype: the input's)
#include "attn_common.cuh"

namespace qdqb200 {
namespace attn {
namespace {

// ---------------------------------------------------------------- helpers
__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}
// The 16-bit input type: bf16 (kF16 = false) or fp16.  lo / hi read the two
// halves of a 32-bit word, round rounds to the type (nearest even), pack
// rounds two floats into one word, bits / val convert one element.
template <bool kF16>
struct In16 {
  __device__ static float lo(uint32_t w) { return kF16 ? f16lo(w) : bf16lo(w); }
  __device__ static float hi(uint32_t w) { return kF16 ? f16hi(w) : bf16hi(w); }
  __device__ static float round(float x) { return kF16 ? __half2float(__float2half_rn(x)) : bf16_round(x); }
  __device__ static uint32_t pack(float a, float b) { return kF16 ? pack_f16x2(a, b) : pack_bf16x2(a, b); }
  __device__ static uint16_t bits(float x) {
    return kF16 ? __half_as_ushort(__float2half_rn(x)) : __bfloat16_as_ushort(__float2bfloat16_rn(x));
  }
  __device__ static float val(uint16_t b) {
    return kF16 ? __half2float(__ushort_as_half(b)) : __uint_as_float(static_cast<uint32_t>(b) << 16);
  }
};

// Exact ceil(log2(r)) for r > 0 (r finite).
__device__ __forceinline__ int ceil_log2(float r) {
  const uint32_t b = __float_as_uint(r);
  const int ef = static_cast<int>((b >> 23) & 0xFF);
  const uint32_t man = b & 0x7FFFFFu;
  if (ef == 0) {  // subnormal: r = man * 2^-149
    const int msb = 31 - __clz(man);
    return (man == (1u << msb)) ? msb - 149 : msb - 148;
  }
  return (ef - 127) + (man != 0 ? 1 : 0);
}

// E8M0 exponent e for a group whose |x| max is amax (mxfp4_hw_kernel.py:96-100).
__device__ __forceinline__ int mx_group_exp(float amax) {
  const float amax_safe = fmaxf(amax, 6.0f * 1.1754943508222875e-38f);  // 6 * 2^-126
  int e = ceil_log2(__fdiv_rn(amax_safe, 6.0f));
  return min(max(e, -127), 127);
}


// 2^-e as an exact float (e in [-127, 127]; 2^127 for e = -127).
__device__ __forceinline__ float exp2_neg(int e) {
  const int be = 127 - e;  // biased exponent of 2^-e
  return be >= 1 ? __uint_as_float(static_cast<uint32_t>(be) << 23)
                 : __uint_as_float(1u << (22 + be));
}


// E8M0 exponent of quantize_to_mxfp8 for a group whose |x| max is amax:
// e = ceil(log2(a / 448)) with a = max(amax, 1e-12).  For a = M * 2^E
// (1 <= M < 2) the fp32 quotient is (M / 1.75) * 2^(E-8), normal for every
// a >= 1e-12, and has a zero mantissa only when M == 1.75 (M just below 1.75
// rounds to 1 - 2^-24, not 1), so the ceiling is E - 8 + (M > 1.75).
__device__ __forceinline__ int mx8_group_exp(float amax) {
  const uint32_t b = __float_as_uint(fmaxf(amax, 1e-12f));
  return static_cast<int>(b >> 23) - 135 + ((b & 0x7FFFFFu) > 0x600000u ? 1 : 0);
}

// Quantise 32 floats (one MXFP8 group): 32 E4M3 bytes into out[0..31]
// (16-byte aligned), returns the E8M0 byte.  x * 2^-e equals the
// reference's x / 2^e exactly (a power-of-two scale, both rounded once).
__device__ __forceinline__ uint32_t mx8_quant32(const float* v, uint8_t* out) {
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
  const int e = mx8_group_exp(amax);
  const float inv = exp2_neg(e);
  uint32_t w[8];
#pragma unroll
  for (int q = 0; q < 8; ++q)
    w[q] = cvt_e4m3x4(v[4 * q] * inv, v[4 * q + 1] * inv, v[4 * q + 2] * inv, v[4 * q + 3] * inv);
  reinterpret_cast<uint4*>(out)[0] = make_uint4(w[0], w[1], w[2], w[3]);
  reinterpret_cast<uint4*>(out)[1] = make_uint4(w[4], w[5], w[6], w[7]);
  return static_cast<uint32_t>(min(max(e + 127, 0), 254));
}



// One 32-element group of the reference's emulated E8M0 QuantConfigs
// (quantize_qk / quantize_v, quantize.py:21-141, with round_to_e8m0_torch,
// quant_primitives.py:140-151), every step in the input dtype T:
//   sc = max(T(amax / fp_max), T(1e-8));
//   e  = clamp(ceil(T(log2(sc))), -127, 127): the logarithm rounded to fp32
//        and then to T, as torch evaluates it on a T tensor (computed here in
//        double precision and rounded once to fp32; over every bf16 and fp16
//        sc its bf16 / fp16 rounding equals torch's);
//   codes = grid9(T(x / 2^e)) (kGrid9, fp_max 6) or the E4M3 cast of T(x / 2^e)
//        (fp_max 448, round to nearest even), stored as E4M3 bytes;
// returns the E8M0 byte e + 127.  x / 2^e is exact, so T(x / 2^e) is x * 2^-e
// rounded to T (a no-op except at the bottom of fp16's range).  With fp16
// inputs an all-zero group has sc = 0, for which the reference divides by a
// zero scale; its codes here are 0 (so is the reference's E2M1 result).
template <bool kGrid9, bool kF16>
__device__ __forceinline__ uint32_t emu8_quant32(const float* v, uint8_t* out) {
  using E = In16<kF16>;
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
  const float sc = fmaxf(E::round(__fdiv_rn(amax, kGrid9 ? 6.0f : 448.0f)), E::round(1e-8f));
  int e = -127;
  if (sc > 0.f) {
    const float lg = E::round(static_cast<float>(log2(static_cast<double>(sc))));
    e = min(max(static_cast<int>(ceilf(lg)), -127), 127);
  }
  const float inv = sc > 0.f ? exp2_neg(e) : 0.f;
  uint32_t w[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    float t[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float xn = E::round(v[4 * q + i] * inv);
      t[i] = kGrid9 ? copysignf(grid9_mag(fabsf(xn)), xn) : xn;
    }
    w[q] = cvt_e4m3x4(t[0], t[1], t[2], t[3]);
  }
  reinterpret_cast<uint4*>(out)[0] = make_uint4(w[0], w[1], w[2], w[3]);
  reinterpret_cast<uint4*>(out)[1] = make_uint4(w[4], w[5], w[6], w[7]);
  return static_cast<uint32_t>(e + 127);
}

__device__ __forceinline__ int64_t nhd_row(int b, int n, int h, int64_t sb, int64_t sn, int64_t sh) {
  return b * sb + n * sn + h * sh;
}

// E8M0 group quantisers for inputs of bf16 or fp16 precision (at most 8 or 11
// significant bits: q_s, k_c and V are values of the input dtype).  x * 2^-e
// is then exact, and its distance to a midpoint between E2M1 values (0.25,
// 0.75, ... 5, at most 3 significant bits) is zero or at least 2^-11
// relative (2^-8 for bf16).  Scaling by
// (1 + 2^-12), also exact, lifts the midpoints themselves just above and moves
// nothing else across one, so the hardware's round-to-nearest-even cvt yields
// the reference's round-half-away codes (mxfp4_hw_kernel.py:43-61).  The
// product is formed as fma(x, inv, +0), so an input of -0 encodes as +0 like
// the reference's sign test x < 0 (a negative product that underflows to
// zero keeps the negative-zero code; both dequantise to 0).
__device__ __forceinline__ uint32_t mx_quant32_bf(const float* v, uint8_t* out) {
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
  const int e = mx_group_exp(amax);
  const float inv = exp2_neg(e) * (1.0f + 1.0f / 4096.0f);
  float s[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) s[i] = __fmaf_rn(v[i], inv, 0.0f);
  uint32_t w[4];
#pragma unroll
  for (int q = 0; q < 4; ++q)
    w[q] = cvt_e2m1x8(s[8 * q], s[8 * q + 1], s[8 * q + 2], s[8 * q + 3], s[8 * q + 4], s[8 * q + 5],
                      s[8 * q + 6], s[8 * q + 7]);
  *reinterpret_cast<uint4*>(out) = make_uint4(w[0], w[1], w[2], w[3]);
  return static_cast<uint32_t>(e + 127);
}

// E4M3-scaled blocks (the reference's nvfp4 / mxfp4_s1_e4m3 QuantConfigs,
// quantize.py:21-81 with round_to_e4m3, on the hardware E2M1 grid): scale
// s = e4m3(max(dtype(amax / 6), 1e-8)), codes of the quotient x / s rounded
// half away from zero.  x has bf16 or fp16 precision (8 or 11 significant
// bits) and s at most 4, so x / s is either exactly an E2M1 midpoint (a value
// with at most 7 significant bits times s) or at least 2^-11 relative away
// from every midpoint (x and midpoint * s then differ by at least one unit in
// x's last place).  x * (RN(1 / s) * (1 + 2^-12)) is within 3 * 2^-24
// relative of x / s * (1 + 2^-12): above a midpoint that x / s equals, on the
// same side of every other, so the round-to-nearest-even cvt gives the
// round-half-away code (checked exhaustively on the CPU for every bf16 x and
// E4M3 s, and for every fp16 x and E4M3 s).
// fma(x, inv, +0) turns an exact -0 into +0 (the reference's sign is x < 0).
// KB elements, KB / 2 code bytes; returns the scale byte (0: the block is 0).
template <int KB, bool kF16>
__device__ __forceinline__ uint32_t nv_quant_fast(const float* v, uint8_t* out) {
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < KB; ++i) amax = fmaxf(amax, fabsf(v[i]));
  const float sc = fmaxf(In16<kF16>::round(amax / 6.0f), 1e-8f);
  const uint32_t sbyte = e4m3_byte(sc);
  const float s = round_e4m3(sc);
  const float inv = s > 0.f ? (1.0f / s) * (1.0f + 1.0f / 4096.0f) : 0.f;
  float t[KB];
#pragma unroll
  for (int i = 0; i < KB; ++i) t[i] = __fmaf_rn(v[i], inv, 0.0f);
  uint32_t w[KB / 8];
#pragma unroll
  for (int q = 0; q < KB / 8; ++q)
    w[q] = cvt_e2m1x8(t[8 * q], t[8 * q + 1], t[8 * q + 2], t[8 * q + 3], t[8 * q + 4], t[8 * q + 5],
                      t[8 * q + 6], t[8 * q + 7]);
  if (KB == 16) *reinterpret_cast<uint2*>(out) = make_uint2(w[0], w[1]);
  else *reinterpret_cast<uint4*>(out) = make_uint4(w[0], w[1], w[2 % (KB / 8)], w[3 % (KB / 8)]);
  return sbyte;
}

// One group of a row in format kFmt: codes to `crow`, the scale byte(s) to the
// tcgen05 scale chunk(s) at sft (row r, group g of the tile).
template <int kFmt, bool kF16>
__device__ __forceinline__ void quant_group(const float* v, uint8_t* crow, uint8_t* sft, int r, int g) {
  const int slot = (r % 32) * 16 + (r / 32) * 4;
  if (kFmt == F_MX8) {
    sft[slot + g] = static_cast<uint8_t>(mx8_quant32(v, crow));
  } else if (kFmt == F_G9 || kFmt == F_E8) {
    sft[slot + g] = static_cast<uint8_t>(emu8_quant32<kFmt == F_G9, kF16>(v, crow));
  } else if (kFmt == F_NV4) {
    sft[(g / 4) * 512 + slot + (g % 4)] = static_cast<uint8_t>(nv_quant_fast<16, kF16>(v, crow));
  } else if (kFmt == F_NV4B32) {
    *reinterpret_cast<uint16_t*>(sft + (g / 2) * 512 + slot + 2 * (g % 2)) =
        static_cast<uint16_t>(nv_quant_fast<32, kF16>(v, crow) * 0x101u);
  } else {
    sft[slot + g] = static_cast<uint8_t>(mx_quant32_bf(v, crow));
  }
}

// ---------------------------------------------------------------- channel sums
// sum[bh, d] += sum over keys of x[b, n, h, d] (K for its mean; V for V
// smoothing).  grid (BH, ceil(L / 256)), 256 threads: thread t sums the 8
// channels of 16-byte chunk t % 16 over rows t / 16 + 16 i of the block's 256
// rows (16 independent loads in flight), then the 16 partial sums per channel
// meet in shared memory.
template <bool kF16>
__global__ void __launch_bounds__(256) colsum_kernel(const __nv_bfloat16* __restrict__ x, int H, int L, int D,
                                                     int64_t sb, int64_t sn, int64_t sh, float* __restrict__ sum) {
  __shared__ __align__(16) float part[16][128];
  const int bh = blockIdx.x, b = bh / H, h = bh % H;
  const int c = threadIdx.x & 15, r0 = threadIdx.x >> 4;
  const int n0 = blockIdx.y * 256;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int n = n0 + r0 + 16 * i;
    if (n < L && c * 8 < D) {
      const uint4 u = ld_stream(reinterpret_cast<const uint4*>(x + nhd_row(b, n, h, sb, sn, sh) + c * 8));
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[2 * j] += In16<kF16>::lo(w[j]);
        acc[2 * j + 1] += In16<kF16>::hi(w[j]);
      }
    }
  }
  *reinterpret_cast<float4*>(&part[r0][c * 8]) = make_float4(acc[0], acc[1], acc[2], acc[3]);
  *reinterpret_cast<float4*>(&part[r0][c * 8 + 4]) = make_float4(acc[4], acc[5], acc[6], acc[7]);
  __syncthreads();
  if (threadIdx.x < 128) {
    float t = 0.f;
#pragma unroll
    for (int r = 0; r < 16; ++r) t += part[r][threadIdx.x];
    atomicAdd(&sum[bh * 128 + threadIdx.x], t);
  }
}

// ---------------------------------------------------------------- Q / K passes
// grid (BH, Lp/128), 256 threads, one 128-row x 128-d tile per CTA:
//   load the tile into shared memory (thread t: 16-byte chunk t % 16 of rows
//   t / 16 + 16 i; Q also sums its columns on the way, for the group mean);
//   the mean (Q: the tile's zero-padded group mean, written to qmean; K:
//   bf16(ksum / L)); the centred bf16 tile in place (padding rows stay 0);
//   each row's groups along D quantised in format kFmt.
// K with smoothing also computes this key tile's delta_s rows for every query
// group from the centred tile (see ds_tile), so K is read once here.
constexpr int DS_LD = 136;  // padded row length (bf16) -> conflict-free ldmatrix
constexpr int QK_TILE_BYTES = 128 * DS_LD * 2;
constexpr int QK_SMEM_Q = QK_TILE_BYTES + 16 * 128 * 4;   // tile + column partial sums
constexpr int QK_SMEM_K = QK_TILE_BYTES + 64 * DS_LD * 2;  // tile + 64 query-group means

template <bool kF16>
__device__ void ds_tile(const __nv_bfloat16* kcs, __nv_bfloat16* qms, const __nv_bfloat16* __restrict__ qmean,
                        __nv_bfloat16* __restrict__ ds, int bh, int G, int Lp, int n0);

// 16-byte global -> shared copy that bypasses registers (src_size 0: zero fill).
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sm100::smem_u32(smem)), "l"(gmem),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// Rows [g0, g0 + 64) of this head's query-group means -> qms ([64][DS_LD]),
// zero past G: four 16-byte copies per thread of the 256.
__device__ __forceinline__ void qmean_chunk_async(__nv_bfloat16* qms, const __nv_bfloat16* __restrict__ qmean, int bh,
                                                  int G, int g0) {
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int i = threadIdx.x + 256 * k, r = i >> 4, c = i & 15;
    const bool valid = g0 + r < G;
    cp_async16(qms + r * DS_LD + c * 8,
               qmean + (static_cast<int64_t>(bh) * G + (valid ? g0 + r : 0)) * 128 + c * 8, valid);
  }
  cp_async_commit();
}

template <bool kIsQ, int kFmt, bool kF16>
__global__ void __launch_bounds__(256) qk_quant_kernel(const __nv_bfloat16* __restrict__ x, int H, int L, int Lp, int D,
                                                       int64_t sb, int64_t sn, int64_t sh,
                                                       const float* __restrict__ ksum, __nv_bfloat16* __restrict__ qmean,
                                                       uint8_t* __restrict__ codes, uint8_t* __restrict__ sf,
                                                       int smoothing, __nv_bfloat16* __restrict__ ds) {
  extern __shared__ __align__(16) uint8_t qk_smem[];
  __nv_bfloat16* tile = reinterpret_cast<__nv_bfloat16*>(qk_smem);  // [128][DS_LD]
  __shared__ float mean[128];
  const int bh = blockIdx.x, b = bh / H, h = bh % H;
  const int t0 = blockIdx.y * 128;
  const int c = threadIdx.x & 15, r0 = threadIdx.x >> 4;
  if (!kIsQ && smoothing)  // the first 64 query-group means for delta_s, fetched while K is quantised
    qmean_chunk_async(reinterpret_cast<__nv_bfloat16*>(qk_smem + QK_TILE_BYTES), qmean, bh, Lp / 128, 0);
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = r0 + 16 * i;
    const int n = t0 + r;
    uint4 u = make_uint4(0, 0, 0, 0);
    if (n < L && c * 8 < D) u = ld_stream(reinterpret_cast<const uint4*>(x + nhd_row(b, n, h, sb, sn, sh) + c * 8));
    *reinterpret_cast<uint4*>(tile + r * DS_LD + c * 8) = u;
    if (kIsQ) {
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[2 * j] += In16<kF16>::lo(w[j]);
        acc[2 * j + 1] += In16<kF16>::hi(w[j]);
      }
    }
  }
  if (kIsQ) {
    float* part = reinterpret_cast<float*>(qk_smem + QK_TILE_BYTES);  // [16][128]
    *reinterpret_cast<float4*>(part + r0 * 128 + c * 8) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    *reinterpret_cast<float4*>(part + r0 * 128 + c * 8 + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
  }
  __syncthreads();
  if (threadIdx.x < 128) {
    const int d = threadIdx.x;
    float m = 0.f;
    if (smoothing) {
      if (kIsQ) {
        // torch mean over the zero-padded 128-row group (transforms.py:72-80)
        const float* part = reinterpret_cast<const float*>(qk_smem + QK_TILE_BYTES);
        float sum = 0.f;
#pragma unroll
        for (int r = 0; r < 16; ++r) sum += part[r * 128 + d];
        m = In16<kF16>::round(sum / 128.0f);
        reinterpret_cast<uint16_t*>(qmean)[(static_cast<int64_t>(bh) * (Lp / 128) + blockIdx.y) * 128 + d] =
            In16<kF16>::bits(m);
      } else {
        m = In16<kF16>::round(ksum[bh * 128 + d] / static_cast<float>(L));
      }
    }
    mean[d] = m;
  }
  __syncthreads();
  if (smoothing) {  // centre in place: dtype(x - mean) on real rows, padding rows stay 0
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = r0 + 16 * i;
      if (t0 + r < L) {
        uint4* pu = reinterpret_cast<uint4*>(tile + r * DS_LD + c * 8);
        const uint4 u = *pu;
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          o[j] = In16<kF16>::pack(In16<kF16>::lo(w[j]) - mean[c * 8 + 2 * j],
                                  In16<kF16>::hi(w[j]) - mean[c * 8 + 2 * j + 1]);
        *pu = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
    __syncthreads();
  }
  // (row, group) items: 4 groups of 32 per row, NVFP4 8 groups of 16.
  // Scale chunks: 1024 bytes per 128-row tile (the E8M0 formats use the first
  // 512; F_NV4B32 writes each scale into both 16-element slots of its group).
  uint8_t* sft = sf + (static_cast<int64_t>(bh) * (Lp / 128) + blockIdx.y) * 1024;
  constexpr int kGroups = kFmt == F_NV4 ? 8 : 4, kGs = kFmt == F_NV4 ? 16 : 32;
  for (int it = threadIdx.x; it < 128 * kGroups; it += 256) {
    const int r = it / kGroups, g = it % kGroups;
    const int n = t0 + r;
    float v[kGs];
#pragma unroll
    for (int q = 0; q < kGs / 8; ++q) {
      const uint4 u = *reinterpret_cast<const uint4*>(tile + r * DS_LD + g * kGs + q * 8);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[q * 8 + 2 * j] = In16<kF16>::lo(w[j]);
        v[q * 8 + 2 * j + 1] = In16<kF16>::hi(w[j]);
      }
    }
    uint8_t* crow = fmt_e4m3(kFmt) ? codes + (static_cast<int64_t>(bh) * Lp + n) * 128 + g * 32
                                  : codes + (static_cast<int64_t>(bh) * Lp + n) * 64 + g * (kGs / 2);
    quant_group<kFmt, kF16>(v, crow, sft, r, g);
  }
  if (!kIsQ && smoothing) {
    __syncthreads();  // (the tile was only read above; ds_tile reuses the rest of the buffer)
    ds_tile<kF16>(tile, reinterpret_cast<__nv_bfloat16*>(qk_smem + QK_TILE_BYTES), qmean, ds, bh, Lp / 128, Lp,
                  t0);
  }
}

// ---------------------------------------------------------------- V quantisation
// grid (BH, Lp/128), 128 threads: thread d quantises V[:, d] over the tile's
// 128 keys in groups of 32 (NVFP4: 16) in format kFmt into 64 (E2M1) or 128
// (E4M3) code bytes of row (bh, d) of V^T, staged in shared memory and then
// written row by row in 16-byte pieces (coalesced).
constexpr int V_TILE_BYTES = 128 * (128 + 8) * 2;
template <int kFmt>
__host__ __device__ constexpr int v_code_ld() { return (fmt_e4m3(kFmt) ? 128 : 64) + 16; }  // staged code row (bytes, padded)
template <int kFmt>
__host__ __device__ constexpr int v_smem_bytes() { return V_TILE_BYTES + 128 * v_code_ld<kFmt>(); }

template <int kFmt, bool kF16>
__global__ void __launch_bounds__(128) v_quant_kernel(const __nv_bfloat16* __restrict__ v, int H, int L, int Lp, int D,
                                                      int64_t sb, int64_t sn, int64_t sh,
                                                      uint8_t* __restrict__ vt, uint8_t* __restrict__ vsf,
                                                      const float* __restrict__ vsum, float* __restrict__ vmean) {
  extern __shared__ __align__(16) uint8_t v_smem[];
  auto tile = reinterpret_cast<uint16_t (*)[128 + 8]>(v_smem);
  uint8_t* cst = v_smem + V_TILE_BYTES;  // [128][v_code_ld] staged code rows
  const int bh = blockIdx.x, b = bh / H, h = bh % H;
  const int t0 = blockIdx.y * 128;
  {
    uint4 u[16];  // all 16 loads in flight before the first shared-memory store
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const int i = threadIdx.x + 128 * k, r = i >> 4, c = i & 15;
      const int n = t0 + r;
      u[k] = (n < L && c * 8 < D) ? ld_stream(reinterpret_cast<const uint4*>(v + nhd_row(b, n, h, sb, sn, sh) + c * 8))
                                  : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const int i = threadIdx.x + 128 * k;
      *reinterpret_cast<uint4*>(&tile[i >> 4][(i & 15) * 8]) = u[k];
    }
  }
  __syncthreads();
  const int d = threadIdx.x;
  constexpr bool kF8 = fmt_e4m3(kFmt);
  // V smoothing (transforms.py v_smoothing): quantise dtype(v - mean_L(v)); the
  // flash epilogue adds the mean back.  Padding rows stay zero.
  using E = In16<kF16>;
  float vm = 0.f;
  if (vsum != nullptr) {
    vm = E::round(vsum[bh * 128 + d] / static_cast<float>(L));
    if (blockIdx.y == 0) vmean[bh * 128 + d] = vm;
    for (int r = 0; r < 128 && t0 + r < L; ++r) tile[r][d] = E::bits(E::val(tile[r][d]) - vm);
  }
  uint8_t* row = cst + d * v_code_ld<kFmt>();
  uint8_t* sft = vsf + (static_cast<int64_t>(bh) * (Lp / 128) + blockIdx.y) * 1024 + (d % 32) * 16 + (d / 32) * 4;
  if (kFmt == F_NV4B32) {
    uint32_t sfw[2] = {0, 0};
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
      float x[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) x[i] = E::val(tile[g * 32 + i][d]);
      sfw[g / 2] |= (nv_quant_fast<32, kF16>(x, row + g * 16) * 0x101u) << (16 * (g % 2));
    }
    *reinterpret_cast<uint32_t*>(sft) = sfw[0];
    *reinterpret_cast<uint32_t*>(sft + 512) = sfw[1];
  } else if (kFmt == F_NV4) {
    uint32_t sfw[2] = {0, 0};
#pragma unroll 1
    for (int g = 0; g < 8; ++g) {
      float x[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) x[i] = E::val(tile[g * 16 + i][d]);
      sfw[g / 4] |= nv_quant_fast<16, kF16>(x, row + g * 8) << (8 * (g % 4));
    }
    *reinterpret_cast<uint32_t*>(sft) = sfw[0];
    *reinterpret_cast<uint32_t*>(sft + 512) = sfw[1];
  } else {
    uint32_t sfw = 0;
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
      float x[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) x[i] = E::val(tile[g * 32 + i][d]);
      uint32_t sb;
      if (kFmt == F_G9 || kFmt == F_E8) sb = emu8_quant32<kFmt == F_G9, kF16>(x, row + g * 32);
      else sb = kF8 ? mx8_quant32(x, row + g * 32) : mx_quant32_bf(x, row + g * 16);
      sfw |= sb << (8 * g);
    }
    *reinterpret_cast<uint32_t*>(sft) = sfw;
  }
  __syncthreads();
  constexpr int kRow = kF8 ? 128 : 64, kChunks = kRow / 16;
  const int64_t vld = kF8 ? Lp : Lp / 2;  // V^T row length in bytes
  for (int i = threadIdx.x; i < 128 * kChunks; i += 128) {
    const int rr = i / kChunks, c = i % kChunks;
    *reinterpret_cast<uint4*>(vt + (static_cast<int64_t>(bh) * 128 + rr) * vld + blockIdx.y * kRow + c * 16) =
        *reinterpret_cast<const uint4*>(cst + rr * v_code_ld<kFmt>() + c * 16);
  }
}

// ---------------------------------------------------------------- delta_s
// ds[bh, g, n] = dtype( sum_d qmean[bh, g, d] * kc[bh, n, d] ), kc = dtype(k - mean),
// with bf16 or fp16 tensor-core MMAs (mma.sync m16n8k16, fp32 accumulation),
// stored as rows of the input dtype that the flash kernel loads by TMA as an
// MMA operand.
// Run by the K pass's 256 threads (8 warps) on its centred key tile kcs
// ([128][DS_LD] bf16 in shared memory): walks the G query groups 64 at a
// time through qms ([64][DS_LD]); each warp owns a 32 (g) x 32 (n) block of
// the 64 x 128 output chunk.

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(sm100::smem_u32(p)));
}
template <bool kF16>
__device__ __forceinline__ void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if (kF16)
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  else
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <bool kF16>
__device__ void ds_tile(const __nv_bfloat16* kcs, __nv_bfloat16* qms, const __nv_bfloat16* __restrict__ qmean,
                        __nv_bfloat16* __restrict__ ds, int bh, int G, int Lp, int n0) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wm = warp >> 2;        // 0..1: g rows [32 wm, 32 wm + 32)
  const int wn = warp & 3;         // 0..3: keys [32 wn, 32 wn + 32)
  for (int g0 = 0; g0 < G; g0 += 64) {
    __syncthreads();  // previous chunk's qms reads are done (and kcs is ready on the first pass)
    if (g0 > 0) qmean_chunk_async(qms, qmean, bh, G, g0);  // chunk 0 was issued at kernel start
    cp_async_wait_all();
    __syncthreads();
    float acc[2][4][4] = {};
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {  // 8 x 16 = 128 = D
      uint32_t a[2][4];
#pragma unroll
      for (int mi = 0; mi < 2; ++mi) {
        const int row = wm * 32 + mi * 16 + (lane & 15);
        const int col = kk * 16 + (lane >> 4) * 8;
        ldsm_x4(a[mi], qms + row * DS_LD + col);
      }
#pragma unroll
      for (int nj = 0; nj < 2; ++nj) {  // two pairs of n8 tiles
        uint32_t bb[4];
        // matrices: (n 0-7, k 0-7), (n 0-7, k 8-15), (n 8-15, k 0-7), (n 8-15, k 8-15)
        const int nrow = wn * 32 + nj * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int col = kk * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(bb, kcs + nrow * DS_LD + col);
#pragma unroll
        for (int mi = 0; mi < 2; ++mi) {
          mma_16816<kF16>(acc[mi][nj * 2 + 0], a[mi], bb[0], bb[1]);
          mma_16816<kF16>(acc[mi][nj * 2 + 1], a[mi], bb[2], bb[3]);
        }
      }
    }
    // The chunk's 64 x 128 outputs are staged in qms (its query means are no
    // longer read once every warp is past the MMAs) and leave as whole
    // 256-byte rows: c fragment rows (lane/4) and (lane/4 + 8), cols
    // 2*(lane%4) + {0,1}.
    __syncthreads();
#pragma unroll
    for (int mi = 0; mi < 2; ++mi)
#pragma unroll
      for (int ni = 0; ni < 4; ++ni)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int gl = wm * 32 + mi * 16 + (lane >> 2) + hh * 8;
          const int nl = wn * 32 + ni * 8 + (lane & 3) * 2;
          *reinterpret_cast<uint32_t*>(qms + gl * DS_LD + nl) =
              In16<kF16>::pack(acc[mi][ni][hh * 2], acc[mi][ni][hh * 2 + 1]);
        }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 4; ++k) {  // 64 rows x 16 chunks of 16 bytes, four per thread
      const int i = threadIdx.x + 256 * k, gl = i >> 4, c = i & 15;
      if (g0 + gl < G)
        *reinterpret_cast<uint4*>(ds + (static_cast<int64_t>(bh) * G + g0 + gl) * Lp + n0 + c * 8) =
            *reinterpret_cast<const uint4*>(qms + gl * DS_LD + c * 8);
    }
  }
}

}  // namespace

// The Q and K passes of format kFmt; their dynamic shared memory (above the
// 48 KB default) is enabled once per device for this instantiation.
template <int kFmt, bool kF16>
int launch_qk(const Problem& p, const Workspace& w, cudaStream_t s) {
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    if (cudaFuncSetAttribute(qk_quant_kernel<true, kFmt, kF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             QK_SMEM_Q) != cudaSuccess ||
        cudaFuncSetAttribute(qk_quant_kernel<false, kFmt, kF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             QK_SMEM_K) != cudaSuccess)
      return fail(QDQ_ERR_CUDA, "sage3 prepass: smem attribute");
    attr[dev] = true;
  }
  const int BH = p.B * p.H, T = p.Lp / 128;
  qk_quant_kernel<true, kFmt, kF16><<<dim3(BH, T), 256, QK_SMEM_Q, s>>>(
      p.q, p.H, p.L, p.Lp, p.D, p.q_sb, p.q_sn, p.q_sh, w.ksum, w.qmean, w.qc, w.qsf, p.smoothing, w.ds);
  qk_quant_kernel<false, kFmt, kF16><<<dim3(BH, T), 256, QK_SMEM_K, s>>>(
      p.k, p.H, p.L, p.Lp, p.D, p.k_sb, p.k_sn, p.k_sh, w.ksum, w.qmean, w.kc, w.ksf, p.smoothing, w.ds);
  return QDQ_OK;
}

// The V pass of format kFmt (dynamic shared memory above the 48 KB default).
template <int kFmt, bool kF16>
int launch_v(const Problem& p, const Workspace& w, const float* vs, cudaStream_t s) {
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    if (cudaFuncSetAttribute(v_quant_kernel<kFmt, kF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             v_smem_bytes<kFmt>()) != cudaSuccess)
      return fail(QDQ_ERR_CUDA, "sage3 prepass: smem attribute");
    attr[dev] = true;
  }
  v_quant_kernel<kFmt, kF16><<<dim3(p.B * p.H, p.Lp / 128), 128, v_smem_bytes<kFmt>(), s>>>(
      p.v, p.H, p.L, p.Lp, p.D, p.v_sb, p.v_sn, p.v_sh, w.vt, w.vsf, vs, w.vmean);
  return QDQ_OK;
}

template <bool kF16>
int launch_prepass_t(const Problem& p, const Workspace& w, cudaStream_t s) {
  const int BH = p.B * p.H;
  if (cudaMemsetAsync(w.ksum, 0, sizeof(float) * BH * 128, s) != cudaSuccess)
    return fail(QDQ_ERR_CUDA, "sage3 prepass: memset failed");
  if (p.smoothing)
    colsum_kernel<kF16><<<dim3(BH, (p.L + 255) / 256), 256, 0, s>>>(p.k, p.H, p.L, p.D, p.k_sb, p.k_sn, p.k_sh,
                                                                    w.ksum);
  if (p.vsmooth) {
    if (cudaMemsetAsync(w.vsum, 0, sizeof(float) * BH * 128, s) != cudaSuccess)
      return fail(QDQ_ERR_CUDA, "sage3 prepass: memset failed");
    colsum_kernel<kF16><<<dim3(BH, (p.L + 255) / 256), 256, 0, s>>>(p.v, p.H, p.L, p.D, p.v_sb, p.v_sn, p.v_sh,
                                                                    w.vsum);
  }
  // Q (group means first: the K pass's delta_s reads them), then K, in the Q/K format
  int st = QDQ_OK;
  switch (p.qk_fmt) {
    case F_MX8: st = launch_qk<F_MX8, kF16>(p, w, s); break;
    case F_G9: st = launch_qk<F_G9, kF16>(p, w, s); break;
    case F_E8: st = launch_qk<F_E8, kF16>(p, w, s); break;
    case F_NV4: st = launch_qk<F_NV4, kF16>(p, w, s); break;
    case F_NV4B32: st = launch_qk<F_NV4B32, kF16>(p, w, s); break;
    default: st = launch_qk<F_MX4, kF16>(p, w, s); break;
  }
  if (st != QDQ_OK) return st;
  // V^T in the P/V format
  const float* vs = p.vsmooth ? w.vsum : nullptr;
  switch (p.pv_fmt) {
    case F_MX8: st = launch_v<F_MX8, kF16>(p, w, vs, s); break;
    case F_G9: st = launch_v<F_G9, kF16>(p, w, vs, s); break;
    case F_E8: st = launch_v<F_E8, kF16>(p, w, vs, s); break;
    case F_NV4: st = launch_v<F_NV4, kF16>(p, w, vs, s); break;
    case F_NV4B32: st = launch_v<F_NV4B32, kF16>(p, w, vs, s); break;
    default: st = launch_v<F_MX4, kF16>(p, w, vs, s); break;
  }
  if (st != QDQ_OK) return st;
  return check_launch("sage3 prepass");
}

int launch_prepass(const Problem& p, const Workspace& w, cudaStream_t s) {
  return p.f16 ? launch_prepass_t<true>(p, w, s) : launch_prepass_t<false>(p, w, s);
}

}  // namespace attn
}  // namespace qdqb200
