// MXFP4 / NVFP4 activation quant-dequant for sm_100a.
//
// Both are single-pass HBM-bound kernels: every element is read once (2 B) and
// written once (2 B).  A lane owns one 16-byte chunk (8 bf16/fp16); the lanes
// of one scale group (4 for MXFP4's 32, 2 for NVFP4's 16) exchange their
// partial |x| maxima with warp shuffles, so no shared memory or second pass is
// needed.  E2M1 encoding uses the sm_100a `cvt.rn.satfinite.e2m1x2.f32`
// instruction (round-to-nearest-even, saturating at 6), decoding uses
// `cvt.rn.f16x2.e2m1x2` (exact).
//
// Semantics follow
//   - MXFP4: vllm_qdq_plugin/qdq/mxfp4.py:98-156 (reference plugin), bit-exact;
//   - NVFP4: vLLM 0.22 nvfp4_emulation_utils.py:439-478 (CPU branch), bit-exact.
// All float arithmetic that the references round step by step is written with
// __fmul_rn/__fadd_rn/__fdiv_rn so that no FMA contraction changes a rounding.
#include <algorithm>

#include "mx_quant.cuh"
#include "sm100.cuh"

namespace qdqb200 {
namespace {

constexpr uint32_t kFull = 0xFFFFFFFFu;
constexpr int kThreads = 256;
constexpr int kUnroll = 4;           // 16-byte chunks in flight per lane

// Resident CTAs per SM asked of the y-only MXFP4 kernel: at <= 32 registers
// 8 CTAs fit instead of 6, keeping more 16-byte loads in flight (config 1:
// 6012-6041 -> 6177-6181 GB/s).  The same cap measured no gain for MXFP8 and
// a 1.5% loss for NVFP4 (capped at 40), so those keep the compiler's choice.
constexpr int kMxMinBlocks = 8;
// 16-byte chunks in flight per lane of the MXFP4 kernel: 2 for the y-only
// variant under its 32-register cap (config 1: 6337 against 6210 GB/s at 4;
// 8 spills and drops to 4139), kUnroll otherwise.
__host__ __device__ constexpr int mx_unroll(bool y, bool codes, bool scales) {
  return (y && !codes && !scales) ? 2 : kUnroll;
}

// ---------------------------------------------------------------------------
// MXFP4: vectorised kernel (K % 32 == 0, 16-byte aligned rows)
// ---------------------------------------------------------------------------
// kTiledSF: the E8M0 bytes go straight to the block-scaled GEMM's tiled
// scale layout (qdq_sf_tile; `lds` then holds its K-chunk count).
template <int kDtype, bool kContig, bool kY, bool kCodes, bool kScales, bool kTiledSF = false>
__global__ void __launch_bounds__(kThreads, (kY && !kCodes && !kScales) ? kMxMinBlocks : 0)
mxfp4_vec_kernel(const uint16_t* __restrict__ x, uint16_t* __restrict__ y,
                 uint8_t* __restrict__ codes, uint8_t* __restrict__ scales,
                 uint32_t cpr, uint64_t total, int64_t ldx, int64_t ldy, int64_t ldc,
                 int64_t lds) {
  using F = Fmt<kDtype>;
  constexpr int kU = mx_unroll(kY, kCodes, kScales);
  if (kTiledSF) {
    // The fused linear's activation pass, launched with programmatic dependent
    // launch: the GEMM after it may start (and prefetch its weights) at once;
    // this pass reads the activation and overwrites the codes the previous
    // GEMM read, so it waits for the previous kernel first.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
  }
  const uint32_t lane = threadIdx.x & 31u;
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x * kU;
  for (uint64_t base = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + (threadIdx.x & ~31u)) * kU;
       base < total; base += stride) {
    uint4 v[kU];
    uint64_t xo[kU], yo[kU], co[kU], so[kU];
    bool ok[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const uint64_t c = base + static_cast<uint64_t>(u) * 32u + lane;
      ok[u] = c < total;
      if (kContig) {
        xo[u] = c * 8u;
        yo[u] = c * 8u;
        co[u] = c * 4u;
        so[u] = c >> 2;
      } else {
        const uint32_t row = static_cast<uint32_t>(c) / cpr;
        const uint32_t col = static_cast<uint32_t>(c) - row * cpr;
        xo[u] = row * static_cast<uint64_t>(ldx) + col * 8u;
        yo[u] = row * static_cast<uint64_t>(ldy) + col * 8u;
        co[u] = row * static_cast<uint64_t>(ldc) + col * 4u;
        so[u] = row * static_cast<uint64_t>(lds) + (col >> 2);
      }
      if (kTiledSF) {  // 32-bit division while the chunk index fits
        const uint32_t row = total <= 0xFFFFFFFFull ? static_cast<uint32_t>(c) / cpr : static_cast<uint32_t>(c / cpr);
        const uint32_t gi = static_cast<uint32_t>(c - static_cast<uint64_t>(row) * cpr) >> 2;
        so[u] = (static_cast<uint64_t>(row >> 7) * static_cast<uint64_t>(lds) + (gi >> 2)) * 512u +
                (row & 31u) * 16u + ((row >> 5) & 3u) * 4u + (gi & 3u);
      }
      v[u] = ok[u] ? ld_stream(reinterpret_cast<const uint4*>(x + xo[u])) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      uint32_t amax = absmax8(v[u]);
      amax = max(amax, __shfl_xor_sync(kFull, amax, 1));
      amax = max(amax, __shfl_xor_sync(kFull, amax, 2));
      const int e = F::mx_exp(amax);
      const float inv = __uint_as_float(static_cast<uint32_t>(254 - e) << 23);  // 1/scale, exact
      const float sc = F::mx_scale(e);
      const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
      float sv[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 t = mul_f32x2(make_float2(F::lo(w[j]), F::hi(w[j])), make_float2(inv, inv));
        sv[2 * j] = t.x;
        sv[2 * j + 1] = t.y;
      }
      uint32_t h[4];
      uint32_t code_word = e2m1_roundtrip8(sv, h);
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 d = mul_f32x2(make_float2(f16lo(h[j]), f16hi(h[j])), make_float2(sc, sc));
        o[j] = F::pack(d.x, d.y);
      }
      if (F::kScaleCanBeZero && e == 0) {
        code_word = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          o[j] = fp16_zero_scale_word(w[j]);
          code_word |= zero_codes_of(o[j]) << (8 * j);
        }
      }
      if (ok[u]) {
        if (kY) st_stream(reinterpret_cast<uint4*>(y + yo[u]), make_uint4(o[0], o[1], o[2], o[3]));
        if (kCodes) *reinterpret_cast<uint32_t*>(codes + co[u]) = code_word;
        if (kScales && (lane & 3u) == 0) scales[so[u]] = static_cast<uint8_t>(e);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// MXFP4: generic kernel (any K, any alignment); one thread per 32-group.
// A partial last group behaves as if zero-padded (mxfp4.py:117-120).
// ---------------------------------------------------------------------------
template <int kDtype>
__global__ void __launch_bounds__(kThreads)
mxfp4_generic_kernel(const uint16_t* __restrict__ x, uint16_t* __restrict__ y,
                     uint8_t* __restrict__ codes, uint8_t* __restrict__ scales, int64_t M,
                     int64_t K, int64_t ldx, int64_t ldy, int64_t ldc, int64_t lds) {
  using F = Fmt<kDtype>;
  const int64_t gpr = (K + 31) / 32;
  const int64_t ngroups = M * gpr;
  for (int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < ngroups;
       g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = g / gpr;
    const int64_t gi = g - r * gpr;
    const int64_t k0 = gi * 32;
    const int n = static_cast<int>((K - k0) < 32 ? (K - k0) : 32);
    const uint16_t* xr = x + r * ldx + k0;
    uint16_t* yr = y ? y + r * ldy + k0 : nullptr;
    uint32_t amax = 0;
    for (int i = 0; i < n; ++i) amax = max(amax, static_cast<uint32_t>(xr[i] & 0x7FFFu));
    const int e = F::mx_exp(amax);
    const float inv = __uint_as_float(static_cast<uint32_t>(254 - e) << 23);
    const float sc = F::mx_scale(e);
    for (int i = 0; i < 32; i += 2) {
      uint32_t byte = 0;
      if (i < n) {
        const uint16_t x0 = xr[i];
        const bool has1 = (i + 1) < n;
        const uint16_t x1 = has1 ? xr[i + 1] : static_cast<uint16_t>(0);
        byte = cvt_e2m1x2(__fmul_rn(F::one(x0), inv), __fmul_rn(F::one(x1), inv));
        if (!has1) byte &= 0x0Fu;
        const uint32_t h = e2m1x2_to_f16x2(byte);
        uint16_t y0 = F::pack1(__fmul_rn(f16lo(h), sc));
        uint16_t y1 = F::pack1(__fmul_rn(f16hi(h), sc));
        if (F::kScaleCanBeZero && e == 0) {
          y0 = fp16_zero_scale_result(x0);
          y1 = fp16_zero_scale_result(x1);
          byte = zero_codes_of(static_cast<uint32_t>(y0) | (static_cast<uint32_t>(y1) << 16));
          if (!has1) byte &= 0x0Fu;
        }
        if (y) {
          yr[i] = y0;
          if (has1) yr[i + 1] = y1;
        }
      }
      if (codes) codes[r * ldc + gi * 16 + i / 2] = static_cast<uint8_t>(byte);
    }
    if (scales) scales[r * lds + gi] = static_cast<uint8_t>(e);
  }
}

// kTiledSF: the E4M3 bytes go straight to the block16 GEMM's tiled scale
// layout (qdq_sf_tile with block 16; `lds` then holds its K-chunk count,
// K / 64), and the kernel takes part in programmatic dependent launch as
// the MXFP4 one does.
template <int kDtype, bool kContig, bool kY, bool kCodes, bool kScales, bool kTiledSF = false>
__global__ void __launch_bounds__(kThreads)
nvfp4_vec_kernel(const uint16_t* __restrict__ x, uint16_t* __restrict__ y,
                 uint8_t* __restrict__ codes, uint8_t* __restrict__ scales,
                 const float* __restrict__ gsp, uint32_t cpr, uint64_t total, int64_t ldx,
                 int64_t ldy, int64_t ldc, int64_t lds, float zero) {
  using F = Fmt<kDtype>;
  if (kTiledSF) {
    // the fused linear's activation pass: the GEMM after it may launch at
    // once; the activation and gs come from the kernels before it
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
  }
  const float gs = __ldg(gsp);
  const float rgs = zero_safe_recip(gs);
  const uint32_t lane = threadIdx.x & 31u;
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x * kUnroll;
  for (uint64_t base = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + (threadIdx.x & ~31u)) * kUnroll;
       base < total; base += stride) {
    uint4 v[kUnroll];
    uint64_t xo[kUnroll], yo[kUnroll], co[kUnroll], so[kUnroll];
    bool ok[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const uint64_t c = base + static_cast<uint64_t>(u) * 32u + lane;
      ok[u] = c < total;
      if (kContig) {
        xo[u] = c * 8u;
        yo[u] = c * 8u;
        co[u] = c * 4u;
        so[u] = c >> 1;
      } else {
        const uint32_t row = static_cast<uint32_t>(c) / cpr;
        const uint32_t col = static_cast<uint32_t>(c) - row * cpr;
        xo[u] = row * static_cast<uint64_t>(ldx) + col * 8u;
        yo[u] = row * static_cast<uint64_t>(ldy) + col * 8u;
        co[u] = row * static_cast<uint64_t>(ldc) + col * 4u;
        so[u] = row * static_cast<uint64_t>(lds) + (col >> 1);
      }
      if (kTiledSF) {  // 16-element group gi of row `row`: chunk (row / 128, gi / 4) of the tiled layout
        const uint32_t row = total <= 0xFFFFFFFFull ? static_cast<uint32_t>(c) / cpr : static_cast<uint32_t>(c / cpr);
        const uint32_t gi = static_cast<uint32_t>(c - static_cast<uint64_t>(row) * cpr) >> 1;
        so[u] = (static_cast<uint64_t>(row >> 7) * static_cast<uint64_t>(lds) + (gi >> 2)) * 512u +
                (row & 31u) * 16u + ((row >> 5) & 3u) * 4u + (gi & 3u);
      }
      v[u] = ok[u] ? ld_stream(reinterpret_cast<const uint4*>(x + xo[u])) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      uint32_t amax = absmax8(v[u]);
      amax = max(amax, __shfl_xor_sync(kFull, amax, 1));
      const NvGroup g = nv_group(F::amax_value(amax), gs, rgs);
      const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
      uint32_t h[4];
      uint32_t code_word;
      if (g.out_scale >= kNoUnderflowScale) {
        float sv[8];
        nv_scale8(w, g.out_scale, zero, sv, kDtype == QDQ_DTYPE_FP16);
        code_word = e2m1_roundtrip8(sv, h);
      } else {
        code_word = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t byte = nv_codes(F::lo(w[j]), F::hi(w[j]), g.out_scale);
          code_word |= byte << (8 * j);
          h[j] = e2m1x2_to_f16x2(byte);
        }
      }
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 d = mul_f32x2(make_float2(f16lo(h[j]), f16hi(h[j])), make_float2(g.deq, g.deq));
        o[j] = F::pack(d.x, d.y);
      }
      if (ok[u]) {
        if (kY) st_stream(reinterpret_cast<uint4*>(y + yo[u]), make_uint4(o[0], o[1], o[2], o[3]));
        if (kCodes) *reinterpret_cast<uint32_t*>(codes + co[u]) = code_word;
        if (kScales && (lane & 1u) == 0) scales[so[u]] = static_cast<uint8_t>(g.sbyte);
      }
    }
  }
}

// NVFP4 generic kernel: one thread per 16-group (K % 16 == 0, any alignment).
template <int kDtype>
__global__ void __launch_bounds__(kThreads)
nvfp4_generic_kernel(const uint16_t* __restrict__ x, uint16_t* __restrict__ y,
                     uint8_t* __restrict__ codes, uint8_t* __restrict__ scales,
                     const float* __restrict__ gsp, int64_t M, int64_t K, int64_t ldx,
                     int64_t ldy, int64_t ldc, int64_t lds) {
  using F = Fmt<kDtype>;
  const float gs = __ldg(gsp);
  const float rgs = zero_safe_recip(gs);
  const int64_t gpr = K / 16;
  for (int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < M * gpr;
       g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = g / gpr;
    const int64_t gi = g - r * gpr;
    const uint16_t* xr = x + r * ldx + gi * 16;
    uint16_t* yr = y ? y + r * ldy + gi * 16 : nullptr;
    uint32_t amax = 0;
    for (int i = 0; i < 16; ++i) amax = max(amax, static_cast<uint32_t>(xr[i] & 0x7FFFu));
    const NvGroup ng = nv_group(F::amax_value(amax), gs, rgs);
    for (int i = 0; i < 16; i += 2) {
      const uint32_t byte = nv_codes(F::one(xr[i]), F::one(xr[i + 1]), ng.out_scale);
      const uint32_t h = e2m1x2_to_f16x2(byte);
      if (yr) {
        yr[i] = F::pack1(__fmul_rn(f16lo(h), ng.deq));
        yr[i + 1] = F::pack1(__fmul_rn(f16hi(h), ng.deq));
      }
      if (codes) codes[r * ldc + gi * 8 + i / 2] = static_cast<uint8_t>(byte);
    }
    if (scales) scales[r * lds + gi] = static_cast<uint8_t>(ng.sbyte);
  }
}

// ---------------------------------------------------------------------------
// global amax -> gs = 2688 / amax   (one pass; last block finalises)
// ws[0] = running max of |x| bit patterns, ws[1] = finished-block ticket.
// ---------------------------------------------------------------------------
template <int kDtype, bool kVec>
__global__ void __launch_bounds__(kThreads)
amax_gs_kernel(const uint16_t* __restrict__ x, int64_t M, int64_t K, int64_t ldx,
               uint32_t* __restrict__ ws, float* __restrict__ gs_out) {
  using F = Fmt<kDtype>;
  uint32_t m = 0;
  if (kVec && ldx == K) {
    // contiguous rows: one flat run of 16-byte chunks, four loads in flight per thread
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    const uint64_t total = static_cast<uint64_t>(M) * static_cast<uint64_t>(K / 8);
    const uint64_t step = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    uint64_t c = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    for (; c + 3 * step < total; c += 4 * step) {
      const uint4 v0 = ld_stream(xv + c), v1 = ld_stream(xv + c + step), v2 = ld_stream(xv + c + 2 * step),
                  v3 = ld_stream(xv + c + 3 * step);
      m = max(m, max(max(absmax8(v0), absmax8(v1)), max(absmax8(v2), absmax8(v3))));
    }
    for (; c < total; c += step) m = max(m, absmax8(ld_stream(xv + c)));
  } else if (kVec) {
    const uint32_t cpr = static_cast<uint32_t>(K / 8);
    const uint64_t total = static_cast<uint64_t>(M) * cpr;
    for (uint64_t c = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; c < total;
         c += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
      const uint64_t row = c / cpr;
      const uint64_t col = c - row * cpr;
      m = max(m, absmax8(ld_stream(reinterpret_cast<const uint4*>(x + row * ldx + col * 8))));
    }
  } else {
    const int64_t total = M * K;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
      const int64_t row = i / K;
      m = max(m, static_cast<uint32_t>(x[row * ldx + (i - row * K)] & 0x7FFFu));
    }
  }
  m = __reduce_max_sync(kFull, m);
  __shared__ uint32_t warp_max[kThreads / 32];
  __shared__ bool last;
  if ((threadIdx.x & 31u) == 0) warp_max[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    uint32_t b = threadIdx.x < (kThreads / 32) ? warp_max[threadIdx.x] : 0u;
    b = __reduce_max_sync(kFull, b);
    if (threadIdx.x == 0) {
      atomicMax(&ws[0], b);
      __threadfence();
      last = atomicAdd(&ws[1], 1u) == gridDim.x - 1;
    }
  }
  __syncthreads();
  if (last && threadIdx.x == 0) {
    __threadfence();
    const uint32_t bits = atomicOr(&ws[0], 0u);
    *gs_out = __fdiv_rn(2688.0f, F::amax_value(bits));
    ws[0] = 0;
    ws[1] = 0;
  }
}

// ---------------------------------------------------------------------------
// global amax of a small activation (the NVFP4 decode linear's rows): one
// cluster of kAmaxCtas CTAs, each reducing a strided share of the 16-byte
// chunks; the CTAs' maxima meet in CTA 0's shared memory (distributed shared
// memory and one cluster barrier), so neither a cleared workspace nor
// atomics are needed.  gs = 2688 / amax from the same maximum bit pattern as
// amax_gs_kernel, so the same fp32 value.  Launched with programmatic
// dependent launch, it waits for the previous kernel on the stream (which may
// write x) before reading, and lets the next kernel launch at once: that
// kernel's prologue and weight prefetch overlap this pass, and its
// griddepcontrol.wait orders its read of gs after this kernel's write.
// ---------------------------------------------------------------------------
constexpr int kAmaxCtas = 8;

template <int kDtype>
__global__ void __cluster_dims__(kAmaxCtas, 1, 1) __launch_bounds__(kThreads)
amax_gs_small_kernel(const uint16_t* __restrict__ x, int M, int K, int64_t ldx, float* __restrict__ gs_out) {
  using F = Fmt<kDtype>;
  __shared__ uint32_t warp_max[kThreads / 32];
  __shared__ uint32_t cta_max[kAmaxCtas];
  sm100::pdl_launch_dependents();
  sm100::pdl_wait();
  const uint32_t rank = sm100::cluster_rank();
  const int cpr = K / 8, total = M * cpr;
  uint32_t m = 0;
#pragma unroll 4
  for (int c = static_cast<int>(rank) * kThreads + threadIdx.x; c < total; c += kAmaxCtas * kThreads) {
    const int row = c / cpr, col = c - row * cpr;
    m = max(m, absmax8(ld_stream(reinterpret_cast<const uint4*>(x + row * ldx + col * 8))));
  }
  m = __reduce_max_sync(kFull, m);
  if ((threadIdx.x & 31u) == 0) warp_max[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    uint32_t b = threadIdx.x < (kThreads / 32) ? warp_max[threadIdx.x] : 0u;
    b = __reduce_max_sync(kFull, b);
    if (threadIdx.x == 0)
      asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(sm100::cluster_addr(&cta_max[rank], 0)), "r"(b)
                   : "memory");
  }
  sm100::cluster_sync();  // every CTA's maximum is in CTA 0's cta_max
  if (rank == 0 && threadIdx.x == 0) {
    uint32_t bits = 0;
#pragma unroll
    for (int i = 0; i < kAmaxCtas; ++i) bits = max(bits, cta_max[i]);
    *gs_out = __fdiv_rn(2688.0f, F::amax_value(bits));
  }
}

// ---------------------------------------------------------------------------
// MXFP8: E4M3 elements, E8M0 scale per 32 (vllm_qdq_plugin/qdq/mxfp8.py:73-125),
// bit-exact.
// ---------------------------------------------------------------------------
// Scale exponent 127 + floor(log2(max(amax, FLT_MIN))) - 8, clamped to
// [0, 254] (mxfp8.py:104-112).  For a bf16/fp16 maximum, floor(log2) is the
// fp32 exponent field (their mantissas are too short for log2 to round up to
// the next integer); a zero or sub-FLT_MIN maximum sits at FLT_MIN (-126);
// inf / NaN give 0, the x86 float->int32 cast of +-inf / NaN.
template <int kDtype>
__device__ __forceinline__ int mx8_exp(uint32_t amax_bits) {
  const uint32_t b = __float_as_uint(Fmt<kDtype>::amax_value(amax_bits));
  const int ef = static_cast<int>(b >> 23);
  if (ef == 255) return 0;
  return min(max((ef == 0 ? -126 : ef - 127) + 119, 0), 254);
}
__device__ __forceinline__ float pow2f(int e) {  // 2^e, e in [-127, 127]
  return __uint_as_float(e > -127 ? static_cast<uint32_t>(e + 127) << 23 : 0x00400000u);
}
// The reference's E4M3 grid (mxfp8.py:40-70) is round-to-nearest-even with
// saturation at 448, except that its subnormal branch is clamped to 7 * 2^-9
// (:57): magnitudes in [7.5, 8) * 2^-9 give 7 * 2^-9 where RNE gives 2^-6.
// Lowering [7, 8) * 2^-9 to 7 * 2^-9 before the hardware conversion
// reproduces that.
__device__ __forceinline__ float mx8_sub_clamp(float v) {
  const uint32_t u = __float_as_uint(v);
  return ((u & 0x7FFFFFFFu) - 0x3C600000u < 0x00200000u) ? __uint_as_float((u & 0x80000000u) | 0x3C600000u) : v;
}
// Two values -> E4M3 pair (a in the low byte) and its exact fp16x2 decode.
__device__ __forceinline__ uint32_t e4m3x2_roundtrip(float a, float b, uint32_t& h) {
  uint32_t out;
  asm("{\n\t.reg .b16 t;\n\t"
      "cvt.rn.satfinite.e4m3x2.f32 t, %3, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %1, t;\n\t"
      "cvt.u32.u16 %0, t;\n\t}"
      : "=r"(out), "=r"(h)
      : "f"(a), "f"(b));
  return out;
}
// The same two steps on an f16x2 pair of quotients: magnitudes in
// [7, 8) * 2^-9 (fp16 0x2300 .. 0x23FF) lose their low mantissa bits, which
// leaves 7 * 2^-9 with the sign; then E4M3 with the exact fp16x2 decode.  The
// quotients of the fast path fit fp16 exactly: |x / scale| < 2^9, at most 11
// significant bits, and those below 2^-14 (fp16 subnormals, rounded) are far
// below 2^-10, where every E4M3 code is zero.
__device__ __forceinline__ uint32_t mx8_pair_f16(uint32_t h, uint32_t& dec) {
  uint32_t eq, out;
  asm("{\n\t.reg .b32 m;\n\t"
      "and.b32 m, %1, 0x7F007F00;\n\t"
      "set.eq.u32.f16x2 %0, m, %2;\n\t}"
      : "=r"(eq)
      : "r"(h), "r"(0x23002300u));
  h &= ~(eq & 0x00FF00FFu);
  asm("{\n\t.reg .b16 t;\n\t"
      "cvt.rn.satfinite.e4m3x2.f16x2 t, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %1, t;\n\t"
      "cvt.u32.u16 %0, t;\n\t}"
      : "=r"(out), "=r"(dec)
      : "r"(h));
  return out;
}
// x / scale for a pair.  torch.sign makes a zero quotient +0 (mxfp8.py:46,
// :70): with fma(x, inv, zero), zero = +0.0 a kernel argument, an exact -0
// becomes +0.  That covers every zero quotient while no nonzero input can
// underflow: inv >= 2^-16 (scale exponent <= 143), always so for fp16.
// Above it, zero quotients are cleared by comparison.
__device__ __forceinline__ float2 mx8_scaled(float a, float b, float inv, float zero, bool fast) {
  if (fast) return fma_f32x2(make_float2(a, b), make_float2(inv, inv), make_float2(zero, zero));
  float2 t = mul_f32x2(make_float2(a, b), make_float2(inv, inv));
  if (t.x == 0.0f) t.x = 0.0f;
  if (t.y == 0.0f) t.y = 0.0f;
  return t;
}

template <int kDtype, bool kContig, bool kY, bool kCodes, bool kScales>
__global__ void __launch_bounds__(kThreads)
mxfp8_vec_kernel(const uint16_t* __restrict__ x, uint16_t* __restrict__ y,
                 uint8_t* __restrict__ codes, uint8_t* __restrict__ scales,
                 uint32_t cpr, uint64_t total, int64_t ldx, int64_t ldy, int64_t ldc,
                 int64_t lds, float zero) {
  using F = Fmt<kDtype>;
  const uint32_t lane = threadIdx.x & 31u;
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x * kUnroll;
  for (uint64_t base = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + (threadIdx.x & ~31u)) * kUnroll;
       base < total; base += stride) {
    uint4 v[kUnroll];
    uint64_t xo[kUnroll], yo[kUnroll], co[kUnroll], so[kUnroll];
    bool ok[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const uint64_t c = base + static_cast<uint64_t>(u) * 32u + lane;
      ok[u] = c < total;
      if (kContig) {
        xo[u] = c * 8u;
        yo[u] = c * 8u;
        co[u] = c * 8u;
        so[u] = c >> 2;
      } else {
        const uint32_t row = static_cast<uint32_t>(c) / cpr;
        const uint32_t col = static_cast<uint32_t>(c) - row * cpr;
        xo[u] = row * static_cast<uint64_t>(ldx) + col * 8u;
        yo[u] = row * static_cast<uint64_t>(ldy) + col * 8u;
        co[u] = row * static_cast<uint64_t>(ldc) + col * 8u;
        so[u] = row * static_cast<uint64_t>(lds) + (col >> 2);
      }
      v[u] = ok[u] ? ld_stream(reinterpret_cast<const uint4*>(x + xo[u])) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      uint32_t amax = absmax8(v[u]);
      amax = max(amax, __shfl_xor_sync(kFull, amax, 1));
      amax = max(amax, __shfl_xor_sync(kFull, amax, 2));
      const int e = mx8_exp<kDtype>(amax);
      const float inv = pow2f(127 - e), sc = pow2f(e - 127);
      const bool fast = e <= 143;
      const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
      uint32_t o[4], cw[2] = {0u, 0u};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 t = mx8_scaled(F::lo(w[j]), F::hi(w[j]), inv, zero, fast);
        uint32_t h, pair;
        if (fast) pair = mx8_pair_f16(pack_f16x2(t.x, t.y), h);
        else pair = e4m3x2_roundtrip(mx8_sub_clamp(t.x), mx8_sub_clamp(t.y), h);
        cw[j >> 1] |= pair << (16 * (j & 1));
        const float2 d = mul_f32x2(make_float2(f16lo(h), f16hi(h)), make_float2(sc, sc));
        o[j] = F::pack(d.x, d.y);
      }
      if (ok[u]) {
        if (kY) st_stream(reinterpret_cast<uint4*>(y + yo[u]), make_uint4(o[0], o[1], o[2], o[3]));
        if (kCodes) *reinterpret_cast<uint2*>(codes + co[u]) = make_uint2(cw[0], cw[1]);
        if (kScales && (lane & 3u) == 0) scales[so[u]] = static_cast<uint8_t>(e);
      }
    }
  }
}

// Any K, any alignment: one thread per 32-group (a partial last group is
// zero-padded, mxfp8.py:97-100).
template <int kDtype>
__global__ void __launch_bounds__(kThreads)
mxfp8_generic_kernel(const uint16_t* __restrict__ x, uint16_t* __restrict__ y, uint8_t* __restrict__ codes,
                     uint8_t* __restrict__ scales, int64_t M, int64_t K, int64_t ldx, int64_t ldy,
                     int64_t ldc, int64_t lds, float zero) {
  using F = Fmt<kDtype>;
  const int64_t gpr = (K + 31) / 32;
  const int64_t ngroups = M * gpr;
  for (int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < ngroups;
       g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = g / gpr;
    const int64_t gi = g - r * gpr;
    const int64_t k0 = gi * 32;
    const int n = static_cast<int>((K - k0) < 32 ? (K - k0) : 32);
    const uint16_t* xr = x + r * ldx + k0;
    uint32_t amax = 0;
    for (int i = 0; i < n; ++i) amax = max(amax, static_cast<uint32_t>(xr[i] & 0x7FFFu));
    const int e = mx8_exp<kDtype>(amax);
    const float inv = pow2f(127 - e), sc = pow2f(e - 127);
    const bool fast = e <= 143;
    for (int i = 0; i < n; i += 2) {
      const bool has1 = (i + 1) < n;
      const float2 t = mx8_scaled(F::one(xr[i]), has1 ? F::one(xr[i + 1]) : 0.0f, inv, zero, fast);
      uint32_t h;
      const uint32_t pair = e4m3x2_roundtrip(mx8_sub_clamp(t.x), mx8_sub_clamp(t.y), h);
      if (y) {
        y[r * ldy + k0 + i] = F::pack1(__fmul_rn(f16lo(h), sc));
        if (has1) y[r * ldy + k0 + i + 1] = F::pack1(__fmul_rn(f16hi(h), sc));
      }
      if (codes) {
        codes[r * ldc + k0 + i] = static_cast<uint8_t>(pair & 0xFFu);
        if (has1) codes[r * ldc + k0 + i + 1] = static_cast<uint8_t>(pair >> 8);
      }
    }
    if (codes)
      for (int i = n; i < 32; ++i) codes[r * ldc + k0 + i] = 0;  // zero padding
    if (scales) scales[r * lds + gi] = static_cast<uint8_t>(e);
  }
}

// Grid of the QDQ kernels: one CTA per `per_block` work items, so the block
// scheduler keeps every SM at full occupancy until the last wave, with the
// grid-stride loop only as a guard for grids beyond the hardware limit.
// Measured on B200 against a persistent grid of 8 CTAs per SM: config 2
// 5958 -> 6572 GB/s, config 1 5675 -> 6041 GB/s (a persistent grid with
// equal rounds per CTA was slower still, 5222 GB/s at config 1).
int grid_for(uint64_t work_items, int per_block) {
  const uint64_t need = (work_items + per_block - 1) / per_block;
  constexpr uint64_t kMaxGrid = 1u << 30;
  return static_cast<int>(need < 1 ? 1 : (need < kMaxGrid ? need : kMaxGrid));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool aligned4(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; }

// Output sets the vectorised kernels are instantiated for; any other mix of
// (y, codes, scales) goes through the generic kernel.
enum OutSet { kOutY = 0, kOutAll = 1, kOutCodes = 2, kOutOther = 3 };

OutSet out_set(const void* y, const void* codes, const void* scales) {
  if (y && !codes && !scales) return kOutY;
  if (y && codes && scales) return kOutAll;
  if (!y && codes && scales) return kOutCodes;
  return kOutOther;
}

template <int kDtype, bool kContig, typename... Args>
void dispatch_mx_vec(OutSet o, int grid, cudaStream_t s, Args... args) {
  if (o == kOutY) mxfp4_vec_kernel<kDtype, kContig, true, false, false><<<grid, kThreads, 0, s>>>(args...);
  else if (o == kOutAll) mxfp4_vec_kernel<kDtype, kContig, true, true, true><<<grid, kThreads, 0, s>>>(args...);
  else mxfp4_vec_kernel<kDtype, kContig, false, true, true><<<grid, kThreads, 0, s>>>(args...);
}

template <int kDtype, bool kContig, typename... Args>
void dispatch_nv_vec(OutSet o, int grid, cudaStream_t s, Args... args) {
  if (o == kOutY) nvfp4_vec_kernel<kDtype, kContig, true, false, false><<<grid, kThreads, 0, s>>>(args...);
  else if (o == kOutAll) nvfp4_vec_kernel<kDtype, kContig, true, true, true><<<grid, kThreads, 0, s>>>(args...);
  else nvfp4_vec_kernel<kDtype, kContig, false, true, true><<<grid, kThreads, 0, s>>>(args...);
}

template <int kDtype, bool kContig, typename... Args>
void dispatch_mx8_vec(OutSet o, int grid, cudaStream_t s, Args... args) {
  if (o == kOutY) mxfp8_vec_kernel<kDtype, kContig, true, false, false><<<grid, kThreads, 0, s>>>(args...);
  else if (o == kOutAll) mxfp8_vec_kernel<kDtype, kContig, true, true, true><<<grid, kThreads, 0, s>>>(args...);
  else mxfp8_vec_kernel<kDtype, kContig, false, true, true><<<grid, kThreads, 0, s>>>(args...);
}

int check_common(const void* x, const void* y, const void* codes, int64_t M, int64_t K,
                 int64_t ldx, int64_t ldy, int dtype, const char* who) {
  if (M < 0 || K < 0) return fail(QDQ_ERR_INVALID_ARG, "%s: negative shape [%lld, %lld]", who, (long long)M, (long long)K);
  if (dtype != QDQ_DTYPE_BF16 && dtype != QDQ_DTYPE_FP16)
    return fail(QDQ_ERR_INVALID_ARG, "%s: dtype must be bf16 (0) or fp16 (1), got %d", who, dtype);
  if (M == 0 || K == 0) return QDQ_OK;
  if (x == nullptr) return fail(QDQ_ERR_INVALID_ARG, "%s: null input pointer", who);
  if (y == nullptr && codes == nullptr) return fail(QDQ_ERR_INVALID_ARG, "%s: neither y nor codes requested", who);
  if (ldx < K || (y != nullptr && ldy < K)) return fail(QDQ_ERR_INVALID_ARG, "%s: row stride smaller than K", who);
  if (x == y && ldx != ldy) return fail(QDQ_ERR_INVALID_ARG, "%s: in-place call needs ldx == ldy", who);
  return QDQ_OK;
}

}  // namespace
}  // namespace qdqb200

using namespace qdqb200;

extern "C" int qdq_mxfp4(const void* x, void* y, void* codes, void* scales, int64_t M, int64_t K,
                         int64_t ldx, int64_t ldy, int dtype, int group_size, void* stream) {
  if (int st = check_common(x, y, codes, M, K, ldx, ldy, dtype, "qdq_mxfp4")) return st;
  if (group_size != 32)
    return fail(QDQ_ERR_UNSUPPORTED, "qdq_mxfp4: group_size must be 32 (got %d)", group_size);
  if (M == 0 || K == 0) return QDQ_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t Kp = (K + 31) / 32 * 32;
  const int64_t ldc = Kp / 2, lds = Kp / 32;
  auto* xp = static_cast<const uint16_t*>(x);
  auto* yp = static_cast<uint16_t*>(y);
  auto* cp = static_cast<uint8_t*>(codes);
  auto* sp = static_cast<uint8_t*>(scales);
  const uint64_t cpr = static_cast<uint64_t>(K / 8);
  const uint64_t total = static_cast<uint64_t>(M) * cpr;
  const OutSet o = out_set(y, codes, scales);
  if (y == nullptr) ldy = K;
  const bool vec = (K % 32 == 0) && aligned16(x) && (y == nullptr || aligned16(y)) && (ldx % 8 == 0) &&
                   (ldy % 8 == 0) && (codes == nullptr || aligned4(codes)) && o != kOutOther;
  const bool contig = (ldx == K) && (ldy == K);
  if (vec && (contig || total < (1ull << 32))) {
    const int grid = grid_for(total, kThreads * (o == kOutY ? mx_unroll(true, false, false) : kUnroll));
    if (dtype == QDQ_DTYPE_BF16) {
      if (contig) dispatch_mx_vec<QDQ_DTYPE_BF16, true>(o, grid, s, xp, yp, cp, sp, (uint32_t)cpr, total, ldx, ldy, ldc, lds);
      else dispatch_mx_vec<QDQ_DTYPE_BF16, false>(o, grid, s, xp, yp, cp, sp, (uint32_t)cpr, total, ldx, ldy, ldc, lds);
    } else {
      if (contig) dispatch_mx_vec<QDQ_DTYPE_FP16, true>(o, grid, s, xp, yp, cp, sp, (uint32_t)cpr, total, ldx, ldy, ldc, lds);
      else dispatch_mx_vec<QDQ_DTYPE_FP16, false>(o, grid, s, xp, yp, cp, sp, (uint32_t)cpr, total, ldx, ldy, ldc, lds);
    }
  } else {
    const uint64_t ngroups = static_cast<uint64_t>(M) * static_cast<uint64_t>((K + 31) / 32);
    const int grid = grid_for(ngroups, kThreads);
    if (dtype == QDQ_DTYPE_BF16)
      mxfp4_generic_kernel<QDQ_DTYPE_BF16><<<grid, kThreads, 0, s>>>(xp, yp, cp, sp, M, K, ldx, ldy, ldc, lds);
    else
      mxfp4_generic_kernel<QDQ_DTYPE_FP16><<<grid, kThreads, 0, s>>>(xp, yp, cp, sp, M, K, ldx, ldy, ldc, lds);
  }
  return check_launch("qdq_mxfp4");
}

namespace qdqb200 {
// MXFP4 codes [M, K/2] (row stride K/2) and E8M0 scales written directly in
// the GEMM's tiled layout (qdq_sf_tile), one pass.  K % 256 == 0 (no padded
// K chunk), 16-byte aligned rows; scale bytes of pad rows (>= M) are left as
// they are: the GEMM multiplies them only with the zero codes TMA fills in.
int qdq_nvfp4_codes_tiled(const void* x, const float* global_scale, void* codes, void* sf_tiled, int64_t M,
                          int64_t K, int64_t ldx, int dtype, void* stream) {
  if (M <= 0 || K <= 0) return QDQ_OK;
  if (K % 256 != 0 || !aligned16(x) || ldx % 8 != 0 || !aligned4(codes))
    return fail(QDQ_ERR_UNSUPPORTED, "qdq_nvfp4_codes_tiled: K %% 256 and 16-byte aligned rows required");
  const uint64_t cpr = static_cast<uint64_t>(K / 8);
  const uint64_t total = static_cast<uint64_t>(M) * cpr;
  if (total >= (1ull << 32) && ldx != K)
    return fail(QDQ_ERR_UNSUPPORTED, "qdq_nvfp4_codes_tiled: too many elements for a strided input");
  const int64_t kchunks = K / 64;  // 512-byte chunks (4 E4M3 scales of 16 elements each) per 128 rows
  const int grid = grid_for(total, kThreads * kUnroll);
  auto* xp = static_cast<const uint16_t*>(x);
  auto* cp = static_cast<uint8_t*>(codes);
  auto* sp = static_cast<uint8_t*>(sf_tiled);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kThreads);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see the kernel's griddepcontrol
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  uint16_t* const no_y = nullptr;
  const int64_t ldy_ = K, ldc_ = K / 2;
  const uint32_t cpr32 = static_cast<uint32_t>(cpr);
  const float zero = 0.0f;
  const bool contig = ldx == K;
  cudaError_t e = cudaSuccess;
#define QDQ_NV_TILED(DT, CONTIG)                                                                                 \
  e = cudaLaunchKernelEx(&cfg, nvfp4_vec_kernel<DT, CONTIG, false, true, true, true>, xp, no_y, cp, sp,           \
                         global_scale, cpr32, total, static_cast<int64_t>(ldx), ldy_, ldc_, kchunks, zero)
  if (dtype == QDQ_DTYPE_BF16) {
    if (contig) QDQ_NV_TILED(QDQ_DTYPE_BF16, true);
    else QDQ_NV_TILED(QDQ_DTYPE_BF16, false);
  } else {
    if (contig) QDQ_NV_TILED(QDQ_DTYPE_FP16, true);
    else QDQ_NV_TILED(QDQ_DTYPE_FP16, false);
  }
#undef QDQ_NV_TILED
  if (e != cudaSuccess) return fail(QDQ_ERR_CUDA, "qdq_nvfp4_codes_tiled: launch: %s", cudaGetErrorString(e));
  return check_launch("qdq_nvfp4_codes_tiled");
}

int qdq_mxfp4_codes_tiled(const void* x, void* codes, void* sf_tiled, int64_t M, int64_t K, int64_t ldx,
                          int dtype, void* stream) {
  if (M <= 0 || K <= 0) return QDQ_OK;
  if (K % 256 != 0 || !aligned16(x) || ldx % 8 != 0 || !aligned4(codes))
    return fail(QDQ_ERR_UNSUPPORTED, "qdq_mxfp4_codes_tiled: K %% 256 and 16-byte aligned rows required");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint64_t cpr = static_cast<uint64_t>(K / 8);
  const uint64_t total = static_cast<uint64_t>(M) * cpr;
  if (total >= (1ull << 32) && ldx != K)
    return fail(QDQ_ERR_UNSUPPORTED, "qdq_mxfp4_codes_tiled: too many elements for a strided input");
  const int64_t kchunks = K / 128;
  const int grid = grid_for(total, kThreads * kUnroll);
  auto* xp = static_cast<const uint16_t*>(x);
  auto* cp = static_cast<uint8_t*>(codes);
  auto* sp = static_cast<uint8_t*>(sf_tiled);
  const bool contig = ldx == K;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kThreads);
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see the kernel's griddepcontrol
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  uint16_t* const no_y = nullptr;
  const int64_t ldy_ = K, ldc_ = K / 2;
  const uint32_t cpr32 = static_cast<uint32_t>(cpr);
  cudaError_t e = cudaSuccess;
#define QDQ_TILED(DT, CONTIG)                                                                                 \
  e = cudaLaunchKernelEx(&cfg, mxfp4_vec_kernel<DT, CONTIG, false, true, true, true>, xp, no_y, cp, sp, cpr32, \
                         total, ldx, ldy_, ldc_, kchunks)
  if (dtype == QDQ_DTYPE_BF16) {
    if (contig) QDQ_TILED(QDQ_DTYPE_BF16, true);
    else QDQ_TILED(QDQ_DTYPE_BF16, false);
  } else {
    if (contig) QDQ_TILED(QDQ_DTYPE_FP16, true);
    else QDQ_TILED(QDQ_DTYPE_FP16, false);
  }
#undef QDQ_TILED
  if (e != cudaSuccess) return fail(QDQ_ERR_CUDA, "qdq_mxfp4_codes_tiled: launch: %s", cudaGetErrorString(e));
  return check_launch("qdq_mxfp4_codes_tiled");
}
}  // namespace qdqb200

extern "C" int qdq_mxfp8(const void* x, void* y, void* codes, void* scales, int64_t M, int64_t K,
                         int64_t ldx, int64_t ldy, int dtype, int group_size, void* stream) {
  if (int st = check_common(x, y, codes, M, K, ldx, ldy, dtype, "qdq_mxfp8")) return st;
  if (group_size != 32)
    return fail(QDQ_ERR_UNSUPPORTED, "qdq_mxfp8: group_size must be 32 (got %d)", group_size);
  if (M == 0 || K == 0) return QDQ_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t Kp = (K + 31) / 32 * 32;
  const int64_t ldc = Kp, lds = Kp / 32;
  auto* xp = static_cast<const uint16_t*>(x);
  auto* yp = static_cast<uint16_t*>(y);
  auto* cp = static_cast<uint8_t*>(codes);
  auto* sp = static_cast<uint8_t*>(scales);
  const uint64_t cpr = static_cast<uint64_t>(K / 8);
  const uint64_t total = static_cast<uint64_t>(M) * cpr;
  const OutSet o = out_set(y, codes, scales);
  if (y == nullptr) ldy = K;
  const bool vec = (K % 32 == 0) && aligned16(x) && (y == nullptr || aligned16(y)) && (ldx % 8 == 0) &&
                   (ldy % 8 == 0) && (codes == nullptr || (reinterpret_cast<uintptr_t>(codes) & 7u) == 0) &&
                   o != kOutOther;
  const bool contig = (ldx == K) && (ldy == K);
  if (vec && (contig || total < (1ull << 32))) {
    const int grid = grid_for(total, kThreads * kUnroll);
    if (dtype == QDQ_DTYPE_BF16) {
      if (contig) dispatch_mx8_vec<QDQ_DTYPE_BF16, true>(o, grid, s, xp, yp, cp, sp, (uint32_t)cpr, total, ldx, ldy, ldc, lds, 0.0f);
      else dispatch_mx8_vec<QDQ_DTYPE_BF16, false>(o, grid, s, xp, yp, cp, sp, (uint32_t)cpr, total, ldx, ldy, ldc, lds, 0.0f);
    } else {
      if (contig) dispatch_mx8_vec<QDQ_DTYPE_FP16, true>(o, grid, s, xp, yp, cp, sp, (uint32_t)cpr, total, ldx, ldy, ldc, lds, 0.0f);
      else dispatch_mx8_vec<QDQ_DTYPE_FP16, false>(o, grid, s, xp, yp, cp, sp, (uint32_t)cpr, total, ldx, ldy, ldc, lds, 0.0f);
    }
  } else {
    const uint64_t ngroups = static_cast<uint64_t>(M) * static_cast<uint64_t>((K + 31) / 32);
    const int grid = grid_for(ngroups, kThreads);
    if (dtype == QDQ_DTYPE_BF16)
      mxfp8_generic_kernel<QDQ_DTYPE_BF16><<<grid, kThreads, 0, s>>>(xp, yp, cp, sp, M, K, ldx, ldy, ldc, lds, 0.0f);
    else
      mxfp8_generic_kernel<QDQ_DTYPE_FP16><<<grid, kThreads, 0, s>>>(xp, yp, cp, sp, M, K, ldx, ldy, ldc, lds, 0.0f);
  }
  return check_launch("qdq_mxfp8");
}

extern "C" int qdq_nvfp4(const void* x, void* y, void* codes, void* scales, const float* global_scale,
                         int64_t M, int64_t K, int64_t ldx, int64_t ldy, int dtype, void* stream) {
  if (int st = check_common(x, y, codes, M, K, ldx, ldy, dtype, "qdq_nvfp4")) return st;
  if (K % 16 != 0) return fail(QDQ_ERR_INVALID_ARG, "qdq_nvfp4: K=%lld is not a multiple of 16", (long long)K);
  if (M == 0 || K == 0) return QDQ_OK;
  if (global_scale == nullptr) return fail(QDQ_ERR_INVALID_ARG, "qdq_nvfp4: null global_scale");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t ldc = K / 2, lds = K / 16;
  auto* xp = static_cast<const uint16_t*>(x);
  auto* yp = static_cast<uint16_t*>(y);
  auto* cp = static_cast<uint8_t*>(codes);
  auto* sp = static_cast<uint8_t*>(scales);
  const uint64_t cpr = static_cast<uint64_t>(K / 8);
  const uint64_t total = static_cast<uint64_t>(M) * cpr;
  const OutSet o = out_set(y, codes, scales);
  if (y == nullptr) ldy = K;
  const bool vec = aligned16(x) && (y == nullptr || aligned16(y)) && (ldx % 8 == 0) && (ldy % 8 == 0) &&
                   (codes == nullptr || aligned4(codes)) && o != kOutOther;
  const bool contig = (ldx == K) && (ldy == K);
  if (vec && (contig || total < (1ull << 32))) {
    const int grid = grid_for(total, kThreads * kUnroll);
    if (dtype == QDQ_DTYPE_BF16) {
      if (contig) dispatch_nv_vec<QDQ_DTYPE_BF16, true>(o, grid, s, xp, yp, cp, sp, global_scale, (uint32_t)cpr, total, ldx, ldy, ldc, lds, 0.0f);
      else dispatch_nv_vec<QDQ_DTYPE_BF16, false>(o, grid, s, xp, yp, cp, sp, global_scale, (uint32_t)cpr, total, ldx, ldy, ldc, lds, 0.0f);
    } else {
      if (contig) dispatch_nv_vec<QDQ_DTYPE_FP16, true>(o, grid, s, xp, yp, cp, sp, global_scale, (uint32_t)cpr, total, ldx, ldy, ldc, lds, 0.0f);
      else dispatch_nv_vec<QDQ_DTYPE_FP16, false>(o, grid, s, xp, yp, cp, sp, global_scale, (uint32_t)cpr, total, ldx, ldy, ldc, lds, 0.0f);
    }
  } else {
    const uint64_t ngroups = static_cast<uint64_t>(M) * static_cast<uint64_t>(K / 16);
    const int grid = grid_for(ngroups, kThreads);
    if (dtype == QDQ_DTYPE_BF16)
      nvfp4_generic_kernel<QDQ_DTYPE_BF16><<<grid, kThreads, 0, s>>>(xp, yp, cp, sp, global_scale, M, K, ldx, ldy, ldc, lds);
    else
      nvfp4_generic_kernel<QDQ_DTYPE_FP16><<<grid, kThreads, 0, s>>>(xp, yp, cp, sp, global_scale, M, K, ldx, ldy, ldc, lds);
  }
  return check_launch("qdq_nvfp4");
}

namespace qdqb200 {
// Shared by the public entry below and by any caller that owns its scratch.
int launch_global_scale(const void* x, float* gs_out, uint32_t* ws, int64_t M, int64_t K,
                        int64_t ldx, int dtype, cudaStream_t s) {
  if (cudaMemsetAsync(ws, 0, 2 * sizeof(uint32_t), s) != cudaSuccess)
    return fail(QDQ_ERR_CUDA, "qdq_nvfp4_global_scale: clearing workspace failed: %s",
                cudaGetErrorString(cudaGetLastError()));
  auto* xp = static_cast<const uint16_t*>(x);
  const bool vec = aligned16(x) && (K % 8 == 0) && (ldx % 8 == 0);
  const uint64_t work = vec ? static_cast<uint64_t>(M) * (K / 8) : static_cast<uint64_t>(M) * K;
  // a persistent grid (8 CTAs per SM): one pair of atomics per CTA on ws
  const int grid = std::min(grid_for(work, kThreads * 4), device_sm_count() * 8);
  if (dtype == QDQ_DTYPE_BF16) {
    if (vec) amax_gs_kernel<QDQ_DTYPE_BF16, true><<<grid, kThreads, 0, s>>>(xp, M, K, ldx, ws, gs_out);
    else amax_gs_kernel<QDQ_DTYPE_BF16, false><<<grid, kThreads, 0, s>>>(xp, M, K, ldx, ws, gs_out);
  } else {
    if (vec) amax_gs_kernel<QDQ_DTYPE_FP16, true><<<grid, kThreads, 0, s>>>(xp, M, K, ldx, ws, gs_out);
    else amax_gs_kernel<QDQ_DTYPE_FP16, false><<<grid, kThreads, 0, s>>>(xp, M, K, ldx, ws, gs_out);
  }
  return check_launch("qdq_nvfp4_global_scale");
}
}  // namespace qdqb200

namespace qdqb200 {
// gs of a small [M, K] activation (M * K / 8 < 2^31 chunks, 16-byte aligned
// rows, K % 8 == 0) by one CTA cluster, for the NVFP4 decode linear.
int launch_global_scale_small(const void* x, float* gs_out, int64_t M, int64_t K, int64_t ldx, int dtype,
                              cudaStream_t s) {
  if (!aligned16(x) || K % 8 != 0 || ldx % 8 != 0 || M * (K / 8) >= (int64_t(1) << 31))
    return fail(QDQ_ERR_INVALID_ARG, "global scale (small): rows must be 16-byte aligned and M*K/8 < 2^31");
  auto* xp = static_cast<const uint16_t*>(x);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kAmaxCtas);
  cfg.blockDim = dim3(kThreads);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int m = static_cast<int>(M), k = static_cast<int>(K);
  cudaError_t e = dtype == QDQ_DTYPE_BF16
                      ? cudaLaunchKernelEx(&cfg, amax_gs_small_kernel<QDQ_DTYPE_BF16>, xp, m, k, ldx, gs_out)
                      : cudaLaunchKernelEx(&cfg, amax_gs_small_kernel<QDQ_DTYPE_FP16>, xp, m, k, ldx, gs_out);
  if (e != cudaSuccess) return fail(QDQ_ERR_CUDA, "global scale (small): launch failed: %s", cudaGetErrorString(e));
  return check_launch("global scale (small)");
}
}  // namespace qdqb200

extern "C" int qdq_nvfp4_global_scale(const void* x, float* global_scale_out, void* workspace,
                                      int64_t M, int64_t K, int64_t ldx, int dtype, void* stream) {
  if (M <= 0 || K <= 0) return fail(QDQ_ERR_INVALID_ARG, "qdq_nvfp4_global_scale: empty tensor has no amax");
  if (dtype != QDQ_DTYPE_BF16 && dtype != QDQ_DTYPE_FP16)
    return fail(QDQ_ERR_INVALID_ARG, "qdq_nvfp4_global_scale: bad dtype %d", dtype);
  if (!x || !global_scale_out || !workspace)
    return fail(QDQ_ERR_INVALID_ARG, "qdq_nvfp4_global_scale: null pointer");
  if (ldx < K) return fail(QDQ_ERR_INVALID_ARG, "qdq_nvfp4_global_scale: ldx < K");
  if (!aligned4(workspace)) return fail(QDQ_ERR_ALIGNMENT, "qdq_nvfp4_global_scale: workspace not 4-byte aligned");
  return launch_global_scale(x, global_scale_out, static_cast<uint32_t*>(workspace), M, K, ldx, dtype,
                             static_cast<cudaStream_t>(stream));
}
