/*
 * qdq_oracle.c — CPU restatement of the reference's quantisation arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * kernels under vllm-qdq-plugin_b200/csrc; it is loaded only by tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference leg.
 * The product path never calls it.
 *
 * Each function restates, step by step, one routine of the reference:
 *   oracle_mxfp4_qdq        vllm_qdq_plugin/qdq/mxfp4.py:98-156 (+ :35-95)
 *   oracle_nvfp4_qdq        vLLM 0.22 quantization/utils/nvfp4_emulation_utils.py
 *                           ref_nvfp4_quant (:439-452), cast_to_fp4 (:425-436),
 *                           get_reciprocal (:415-421), ref_nvfp4_quant_dequant
 *                           CPU branch (:467-478)
 *   oracle_mxfp4_hw_quant   vllm_qdq_plugin/sage3_attn/sage3/mxfp4_hw_kernel.py:43-116
 *                           (quantize_to_mxfp4 / _float_to_e2m1_nibble)
 *   oracle_mxfp8_hw_quant   vllm_qdq_plugin/sage3_attn/sage3/mxfp8_hw_kernel.py:37-65
 *                           (quantize_to_mxfp8)
 *   oracle_mxfp8_qdq        vllm_qdq_plugin/qdq/mxfp8.py:73-125 (+ _round_half_to_even
 *                           :24-37, _quantize_to_e4m3fn_no_fp8_dtype :40-70)
 * Pinned against fixtures produced by importing the reference itself
 * (tests/golden/make_golden.py).
 *
 * Rounding model: the reference's bf16/fp16 tensor ops on CPU compute in fp32
 * and round the result to the 16-bit type with round-to-nearest-even; fp32
 * ops are single IEEE operations.  This file is compiled with
 * -ffp-contract=off and without -ffast-math so each C expression rounds the
 * way the corresponding torch op does.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ */
/* 16-bit float helpers                                                 */
/* ------------------------------------------------------------------ */
static inline float f32_from_bits(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }
static inline uint32_t bits_from_f32(float f) { uint32_t b; memcpy(&b, &f, 4); return b; }

static inline float bf16_to_f32(uint16_t h) { return f32_from_bits((uint32_t)h << 16); }
static inline uint16_t f32_to_bf16(float f) {               /* round-to-nearest-even */
  uint32_t b = bits_from_f32(f);
  if ((b & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((b >> 16) | 0x0040u);  /* quiet NaN */
  b += 0x7FFFu + ((b >> 16) & 1u);
  return (uint16_t)(b >> 16);
}
static inline float fp16_to_f32(uint16_t h) { _Float16 v; memcpy(&v, &h, 2); return (float)v; }
static inline uint16_t f32_to_fp16(float f) { _Float16 v = (_Float16)f; uint16_t h; memcpy(&h, &v, 2); return h; }

static inline float h_to_f32(uint16_t h, int is_fp16) { return is_fp16 ? fp16_to_f32(h) : bf16_to_f32(h); }
static inline uint16_t f32_to_h(float f, int is_fp16) { return is_fp16 ? f32_to_fp16(f) : f32_to_bf16(f); }

/* torch's float -> int32 cast of a non-finite value on x86 (cvttss2si): INT32_MIN. */
static inline int32_t x86_f32_to_i32(float f) {
  if (!(f >= -2147483648.0f && f < 2147483648.0f)) return INT32_MIN;
  return (int32_t)f;
}

/* ------------------------------------------------------------------ */
/* MXFP4 QDQ (mxfp4.py)                                                 */
/* ------------------------------------------------------------------ */

/* _fp_to_fp4_simulate (mxfp4.py:35-95) on one 16-bit pattern. */
static uint16_t fp4_simulate(uint16_t hbits, int mbits, int ebits, int bias) {
  const int32_t v = (int16_t)hbits;                         /* val.view(int16) */
  const int32_t exp = (v >> mbits) & ((1 << ebits) - 1);
  const int32_t sign = (v >> (mbits + ebits)) & 1;
  const int32_t mlast = (v >> (mbits - 1)) & 1;
  const int32_t unb = exp - bias + 1;                       /* new_exp, :53-54 */
  const int32_t shift = (unb <= 0) ? (1 - unb) : 0;
  int32_t tail_bits = mbits - 1 + shift;
  if (tail_bits >= 16) tail_bits = 16;
  const int32_t mant_plus_one = v & ((1 << (mbits + 1)) - 1);
  const int32_t half = 1 << (tail_bits - 1);
  const int32_t tail = mant_plus_one & ((1 << tail_bits) - 1);
  const int close = tail < half, away = tail > half, tie = tail == half;

  const int32_t m_close = (unb > 0) * mlast;
  const int32_t e_close = exp;
  const int32_t m_away = (unb > 0) && (mlast == 0);
  const int32_t e_away = exp + ((unb <= 0) || (mlast == 1));
  const int32_t e_tie = (exp > bias - 2) * (exp + (mlast == 1));

  int32_t e = away * e_away + close * e_close + tie * e_tie;              /* :76-78 */
  int32_t m = away * m_away + close * m_close;                            /* :79 */
  m = m + (e > 2 + bias) * (m == 0);                                      /* :80 */
  if (e >= bias - 2) {                                                    /* :82-84 */
    if (e < bias - 2) e = bias - 2;
    if (e > bias + 2) e = bias + 2;
  } else {
    e = 0;
  }
  const int32_t q = (sign << 15) + (e << mbits) + (m << (mbits - 1));
  return (uint16_t)(q & 0xFFFF);
}

static uint8_t e2m1_code_of(float q) {
  float a = fabsf(q);
  int c = 0;
  if (a >= 6.0f) c = 7; else if (a >= 4.0f) c = 6; else if (a >= 3.0f) c = 5;
  else if (a >= 2.0f) c = 4; else if (a >= 1.5f) c = 3; else if (a >= 1.0f) c = 2;
  else if (a >= 0.5f) c = 1;
  if (signbit(q)) c |= 8;
  return (uint8_t)c;
}

/* One 32-group of mxfp4_qdq (mxfp4.py:135-155); n <= 32 real elements, the
 * rest behave as the zero padding of :117-120. */
static void mxfp4_group(const uint16_t* x, uint16_t* y, int n, int is_fp16,
                        uint8_t* codes /*16 bytes or NULL*/, uint8_t* scale_out) {
  const int mbits = is_fp16 ? 10 : 7, ebits = is_fp16 ? 5 : 8, bias = is_fp16 ? 15 : 127;
  const int32_t val_to_add = 1 << (mbits - 1 - 1);
  const int32_t se_mask = ((1 << (ebits + 1)) - 1) << mbits;
  /* block_max = max(|x|) in the 16-bit type (:137) */
  float bmax = 0.0f;
  for (int i = 0; i < n; ++i) {
    float a = fabsf(h_to_f32(x[i], is_fp16));
    if (a > bmax || isnan(a)) bmax = a;
  }
  const uint16_t bm_bits = f32_to_h(bmax, is_fp16);
  const int32_t r = ((int32_t)bm_bits + val_to_add) & se_mask;            /* :138-140 */
  const float bm_r = h_to_f32((uint16_t)r, is_fp16);
  /* floor(log2(block_max)) in the 16-bit type: exact for a power of two */
  float lg;
  if (bm_r == 0.0f) lg = -INFINITY;
  else if (isinf(bm_r) || isnan(bm_r)) lg = bm_r;  /* log2(inf)=inf, NaN stays NaN */
  else lg = (float)ilogbf(bm_r);
  int64_t se = (int64_t)127 + (int64_t)x86_f32_to_i32(floorf(lg)) - 2;    /* :142-144, int32 add */
  se = (int32_t)(uint32_t)se;                                             /* int32 wrap */
  if (se < 0) se = 0;                                                     /* :145 */
  if (se > 254) se = 254;
  const float scale_f32 = ldexpf(1.0f, (int)se - 127);                    /* 2.0 ** (e-127), fp32 */
  const float scale = h_to_f32(f32_to_h(scale_f32, is_fp16), is_fp16);   /* .to(dtype) (:146) */
  for (int i = 0; i < 32; ++i) {
    const uint16_t xi = i < n ? x[i] : (uint16_t)0;
    const uint16_t v = f32_to_h(h_to_f32(xi, is_fp16) / scale, is_fp16);  /* :148 */
    const uint16_t q = fp4_simulate(v, mbits, ebits, bias);                /* :149-154 */
    const float out = h_to_f32(q, is_fp16) * scale;                        /* :155 */
    if (i < n) y[i] = f32_to_h(out, is_fp16);
    if (codes) {
      /* E2M1 code of the dequantised result divided by the E8M0 scale 2^(se-127):
       * the simulated grid value q for every finite group, a signed zero for
       * fp16 groups whose 16-bit scale underflowed to 0. */
      const float qv = i < n ? h_to_f32(y[i], is_fp16) / ldexpf(1.0f, (int)se - 127) : 0.0f;
      const uint8_t c = e2m1_code_of(qv);
      if (i & 1) codes[i >> 1] = (uint8_t)(codes[i >> 1] | (c << 4));
      else codes[i >> 1] = c;
    }
  }
  if (scale_out) *scale_out = (uint8_t)se;
}

/*
 * x, y: [M, K] 16-bit patterns with row strides ldx/ldy.
 * codes (optional): [M, Kp/2] bytes; scales (optional): [M, Kp/32] bytes.
 */
void oracle_mxfp4_qdq(const uint16_t* x, uint16_t* y, uint8_t* codes, uint8_t* scales,
                      int64_t M, int64_t K, int64_t ldx, int64_t ldy, int is_fp16,
                      int nthreads) {
  const int64_t gpr = (K + 31) / 32;
  const int64_t ldc = gpr * 16, lds = gpr;
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(static) if (nthreads != 1)
#endif
  for (int64_t r = 0; r < M; ++r) {
    for (int64_t g = 0; g < gpr; ++g) {
      const int64_t k0 = g * 32;
      const int n = (int)((K - k0) < 32 ? (K - k0) : 32);
      mxfp4_group(x + r * ldx + k0, y + r * ldy + k0, n, is_fp16,
                  codes ? codes + r * ldc + g * 16 : 0, scales ? scales + r * lds + g : 0);
    }
  }
}

/* ------------------------------------------------------------------ */
/* NVFP4 QDQ (vLLM nvfp4_emulation_utils.py, CPU branch)                */
/* ------------------------------------------------------------------ */

/* fp32 -> float8_e4m3fn -> fp32, round-to-nearest-even (torch's cast). Finite,
 * |v| <= 448 on every call site here (the caller clamps first). */
float oracle_round_e4m3(float v) {
  if (isnan(v)) return v;
  const float a = fabsf(v);
  float q;
  if (a < 0.015625f) {                 /* below 2^-6: subnormal step 2^-9 */
    q = nearbyintf(a * 512.0f) / 512.0f;
  } else {
    int e = ilogbf(a);                 /* 2^e <= a < 2^(e+1) */
    const float step = ldexpf(1.0f, e - 3);
    q = nearbyintf(a / step) * step;
  }
  if (q > 448.0f) q = NAN;             /* not reached after clamp */
  return copysignf(q, v);
}

/* E4M3 byte of a value that oracle_round_e4m3 returns. */
static uint8_t e4m3_byte_of(float q) {
  uint8_t s = signbit(q) ? 0x80 : 0;
  float a = fabsf(q);
  if (a == 0.0f) return s;
  if (a < 0.015625f) return (uint8_t)(s | (uint8_t)nearbyintf(a * 512.0f));
  int e = ilogbf(a);
  int m = (int)nearbyintf(a / ldexpf(1.0f, e - 3)) - 8;
  return (uint8_t)(s | ((e + 7) << 3) | m);
}

/* cast_to_fp4 (:425-436): sequential in-place thresholds == RNE onto E2M1. */
static float cast_to_fp4(float x) {
  const float sgn = (x > 0.0f) ? 1.0f : ((x < 0.0f) ? -1.0f : (isnan(x) ? x : 0.0f));
  float a = fabsf(x);
  if (a >= 0.0f && a <= 0.25f) a = 0.0f;
  if (a > 0.25f && a < 0.75f) a = 0.5f;
  if (a >= 0.75f && a <= 1.25f) a = 1.0f;
  if (a > 1.25f && a < 1.75f) a = 1.5f;
  if (a >= 1.75f && a <= 2.5f) a = 2.0f;
  if (a > 2.5f && a < 3.5f) a = 3.0f;
  if (a >= 3.5f && a <= 5.0f) a = 4.0f;
  if (a > 5.0f) a = 6.0f;
  return a * sgn;
}

static inline float get_reciprocal(float t) {           /* 1 / (t + (t == 0) * 1e8) */
  return 1.0f / (t + (t == 0.0f ? 1e8f : 0.0f));
}

void oracle_nvfp4_qdq(const uint16_t* x, uint16_t* y, uint8_t* codes, uint8_t* scales,
                      float gs, int64_t M, int64_t K, int64_t ldx, int64_t ldy, int is_fp16,
                      int nthreads) {
  const float recip6 = (float)(1.0 / 6.0);           /* FLOAT4_E2M1_MAX_RECIPROCAL as fp32 */
  const float rgs = get_reciprocal(gs);
  const int64_t gpr = K / 16;
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(static) if (nthreads != 1)
#endif
  for (int64_t r = 0; r < M; ++r) {
    for (int64_t g = 0; g < gpr; ++g) {
      const uint16_t* xg = x + r * ldx + g * 16;
      uint16_t* yg = y + r * ldy + g * 16;
      float vmax = 0.0f;
      for (int i = 0; i < 16; ++i) {
        float a = fabsf(h_to_f32(xg[i], is_fp16));
        if (a > vmax || isnan(a)) vmax = a;
      }
      float s = gs * (vmax * recip6);                           /* :445 */
      if (s > 448.0f) s = 448.0f;                                /* :446 */
      if (s < -448.0f) s = -448.0f;
      s = oracle_round_e4m3(s);                                  /* :447 */
      const float out_scale = get_reciprocal(s * rgs);           /* :448 */
      const float deq = s / gs;                                  /* :475 */
      for (int i = 0; i < 16; ++i) {
        float sx = h_to_f32(xg[i], is_fp16) * out_scale;         /* :450 */
        if (sx < -6.0f) sx = -6.0f;                              /* :451 */
        if (sx > 6.0f) sx = 6.0f;
        const float q = cast_to_fp4(sx);
        yg[i] = f32_to_h(q * deq, is_fp16);                      /* :476-478 */
        if (codes) {
          const uint8_t c = e2m1_code_of(q);
          uint8_t* cb = codes + r * (K / 2) + g * 8 + (i >> 1);
          if (i & 1) *cb = (uint8_t)(*cb | (c << 4)); else *cb = c;
        }
      }
      if (scales) scales[r * gpr + g] = e4m3_byte_of(s);
    }
  }
}

/* gs = 2688 / amax(|x|) in fp32. */
float oracle_nvfp4_global_scale(const uint16_t* x, int64_t M, int64_t K, int64_t ldx, int is_fp16) {
  float m = 0.0f;
  for (int64_t r = 0; r < M; ++r)
    for (int64_t k = 0; k < K; ++k) {
      float a = fabsf(h_to_f32(x[r * ldx + k], is_fp16));
      if (a > m) m = a;
    }
  return 2688.0f / m;
}

/* ------------------------------------------------------------------ */
/* quantize_to_mxfp4 (mxfp4_hw_kernel.py:73-116): fp32 rows of length K   */
/* (K % 32 == 0) -> packed codes [rows, K/2] + E8M0 bytes [rows, K/32].   */
/* ceil(log2(r)) is evaluated exactly from r's bits; torch.log2 can round */
/* a value a few ulps above a power of two down to the integer.           */
/* ------------------------------------------------------------------ */
static int ceil_log2_exact(float r) {
  int e;
  const float m = frexpf(r, &e);       /* r = m * 2^e, m in [0.5, 1) */
  return (m == 0.5f) ? e - 1 : e;
}

void oracle_mxfp4_hw_quant(const float* x, uint8_t* codes, uint8_t* scales, int64_t rows,
                           int64_t K, int nthreads) {
  const float min_amax = 6.0f * ldexpf(1.0f, -126);
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(static) if (nthreads != 1)
#endif
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t g = 0; g < K / 32; ++g) {
      const float* xg = x + r * K + g * 32;
      float amax = 0.0f;
      for (int i = 0; i < 32; ++i) { float a = fabsf(xg[i]); if (a > amax) amax = a; }
      if (amax < min_amax) amax = min_amax;
      int e = ceil_log2_exact(amax / 6.0f);
      if (e < -127) e = -127;
      if (e > 127) e = 127;
      scales[r * (K / 32) + g] = (uint8_t)(e + 127);
      const float sc = ldexpf(1.0f, e);
      for (int i = 0; i < 32; i += 2) {
        uint8_t nib[2];
        for (int j = 0; j < 2; ++j) {
          const float v = xg[i + j] / sc;
          float a = fabsf(v);
          if (a > 6.0f) a = 6.0f;
          int c = 0;
          if (a >= 0.25f) c = 1;
          if (a >= 0.75f) c = 2;
          if (a >= 1.25f) c = 3;
          if (a >= 1.75f) c = 4;
          if (a >= 2.5f) c = 5;
          if (a >= 3.5f) c = 6;
          if (a >= 5.0f) c = 7;
          nib[j] = (uint8_t)(c | (v < 0.0f ? 8 : 0));
        }
        codes[r * (K / 2) + g * 16 + i / 2] = (uint8_t)(nib[0] | (nib[1] << 4));
      }
    }
  }
}

/* ------------------------------------------------------------------ */
/* quantize_to_mxfp8 (sage3/mxfp8_hw_kernel.py:37-65): fp32 rows of length */
/* K (K % 32 == 0) -> E4M3 bytes [rows, K] + E8M0 bytes [rows, K/32]:      */
/*   e = ceil(log2(max(amax, 1e-12) / 448)), byte clamp(e + 127, 0, 254),  */
/*   code = torch's float8_e4m3fn cast of x / 2^e (round-to-nearest-even). */
/* ------------------------------------------------------------------ */
static uint8_t e4m3_rne_byte(float x) {   /* |x| <= 448 */
  const uint8_t sgn = signbit(x) ? 0x80 : 0;
  const float a = fabsf(x);
  if (a < 0x1p-6f) return (uint8_t)(sgn | (int)nearbyintf(a * 512.0f));  /* 8 -> 0x08, the min normal */
  int e = ilogbf(a);
  int m = (int)nearbyintf(a / ldexpf(1.0f, e - 3));                     /* 8 .. 16 */
  if (m == 16) { m = 8; ++e; }
  if (e > 8 || (e == 8 && m > 14)) { e = 8; m = 14; }                    /* 448 */
  return (uint8_t)(sgn | ((e + 7) << 3) | (m - 8));
}

void oracle_mxfp8_hw_quant(const float* x, uint8_t* codes, uint8_t* scales, int64_t rows, int64_t K,
                           int nthreads) {
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(static) if (nthreads != 1)
#endif
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t g = 0; g < K / 32; ++g) {
      const float* xg = x + r * K + g * 32;
      float amax = 0.0f;
      for (int i = 0; i < 32; ++i) { float a = fabsf(xg[i]); if (a > amax) amax = a; }
      if (amax < 1e-12f) amax = 1e-12f;
      int b = ceil_log2_exact(amax / 448.0f) + 127;
      if (b < 0) b = 0;
      if (b > 254) b = 254;
      scales[r * (K / 32) + g] = (uint8_t)b;
      const float sc = ldexpf(1.0f, b - 127);
      for (int i = 0; i < 32; ++i) codes[r * K + g * 32 + i] = e4m3_rne_byte(xg[i] / sc);
    }
  }
}

/* ------------------------------------------------------------------ */
/* MXFP8 QDQ (vllm_qdq_plugin/qdq/mxfp8.py)                             */
/* ------------------------------------------------------------------ */

/* _round_half_to_even (mxfp8.py:24-37): floor, then +1 above one half or, on
 * an exact half, when the floor is odd.  fp32 throughout. */
static float rhte(float x) {
  const float f = floorf(x);
  const float frac = x - f;
  const int tie = frac == 0.5f;
  const int up = frac > 0.5f;
  const int odd = fmodf(f, 2.0f) != 0.0f;
  return f + (float)(up | (tie & odd));
}

static inline float clampf(float v, float lo, float hi) {  /* torch.clamp: NaN stays NaN */
  if (isnan(v)) return v;
  return v < lo ? lo : (v > hi ? hi : v);
}

/* _quantize_to_e4m3fn_no_fp8_dtype (mxfp8.py:40-70), fp32 in and out. */
static float e4m3_sim(float x) {
  const float sign = x > 0.0f ? 1.0f : (x < 0.0f ? -1.0f : (isnan(x) ? x : 0.0f));   /* torch.sign */
  const float ax = clampf(fabsf(x), 0.0f, 448.0f);
  const float sub_step = 0x1p-9f, min_normal = 0x1p-6f;
  float sub_q = rhte(ax / sub_step) * sub_step;
  sub_q = clampf(sub_q, 0.0f, 7.0f * sub_step);                         /* :57 */
  const float safe = isnan(ax) ? ax : (ax < min_normal ? min_normal : ax);
  float e = floorf(log2f(safe));
  e = clampf(e, -6.0f, 8.0f);
  const float step = exp2f(e - 3.0f);
  float norm_q = rhte(ax / step) * step;
  norm_q = clampf(norm_q, min_normal, 448.0f);                          /* :66 */
  const float q = ax < min_normal ? sub_q : norm_q;
  return q * sign;
}

/* E4M3 byte of a value e4m3_sim returns (finite, |v| <= 448, on the grid). */
static uint8_t e4m3_byte_exact(float q) {
  const uint8_t sgn = signbit(q) ? 0x80 : 0;
  const float a = fabsf(q);
  if (a == 0.0f) return sgn;
  if (a < 0x1p-6f) return (uint8_t)(sgn | (uint8_t)(a * 512.0f));
  const int e = ilogbf(a);
  const int m = (int)(a / ldexpf(1.0f, e - 3)) - 8;
  return (uint8_t)(sgn | ((e + 7) << 3) | m);
}

/* One group of n <= gs elements (a partial last group is zero-padded). */
static void mxfp8_group(const uint16_t* x, uint16_t* y, int n, int gs, int is_fp16, uint8_t* codes,
                        uint8_t* scale_out) {
  /* block max in the input dtype, then fp32, clamped below at FLT_MIN (:104-105) */
  float bm = 0.0f;
  int has_nan = 0;
  for (int i = 0; i < n; ++i) {
    const float a = fabsf(h_to_f32(x[i], is_fp16));
    if (isnan(a)) has_nan = 1;
    if (a > bm) bm = a;
  }
  (void)gs;
  if (has_nan) bm = NAN;                                 /* torch.max propagates NaN */
  if (!(bm >= 0x1p-126f) && !isnan(bm)) bm = 0x1p-126f;  /* clamp(min=finfo(float32).tiny) */
  /* 127 + floor(log2(bm)).to(int32) - 8, clamped to [0, 254] (:107-112); the
   * float->int32 cast of +-inf / NaN is x86's INT_MIN */
  const int32_t fl = x86_f32_to_i32(floorf(log2f(bm)));
  int64_t se = 127 + (int64_t)fl - 8;
  if (se < 0) se = 0;
  if (se > 254) se = 254;
  const float scale = ldexpf(1.0f, (int)se - 127);       /* 2.0 ** (scale_exp - 127) */
  for (int i = 0; i < n; ++i) {
    const float xs = h_to_f32(x[i], is_fp16) / scale;    /* :117 */
    const float q = e4m3_sim(xs);                         /* :118 */
    y[i] = f32_to_h(q * scale, is_fp16);                  /* :119 */
    if (codes) codes[i] = isnan(q) ? 0x7F : e4m3_byte_exact(q);
  }
  if (scale_out) *scale_out = (uint8_t)se;
}

/*
 * x, y: [M, K] 16-bit patterns with row strides ldx/ldy; group gs (32 in the
 * plugin's calls).  codes (optional): [M, K] E4M3 bytes; scales (optional):
 * [M, ceil(K/gs)] E8M0 bytes.
 */
void oracle_mxfp8_qdq(const uint16_t* x, uint16_t* y, uint8_t* codes, uint8_t* scales, int64_t M,
                      int64_t K, int64_t ldx, int64_t ldy, int is_fp16, int gs, int nthreads) {
  const int64_t gpr = (K + gs - 1) / gs;
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(static) if (nthreads != 1)
#endif
  for (int64_t r = 0; r < M; ++r) {
    for (int64_t g = 0; g < gpr; ++g) {
      const int64_t k0 = g * gs;
      const int n = (int)((K - k0) < gs ? (K - k0) : gs);
      mxfp8_group(x + r * ldx + k0, y + r * ldy + k0, n, gs, is_fp16, codes ? codes + r * K + k0 : 0,
                  scales ? scales + r * gpr + g : 0);
    }
  }
}

int oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
