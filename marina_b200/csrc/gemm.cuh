// Persistent warp-specialised tcgen05 GEMM for the encoder's linear layers:
//
//     D[M, N] = A[M, K] · B[N, K]^T        (A = activations, B = a Linear's weight, both K-major)
//
// followed by a fused epilogue (bias, GELU, residual add into the f16 stream, re-quantisation). One CTA per SM
// walks the output tiles (128 rows x BN columns) in n-fastest order, so the CTAs working on
// the same 128-row block of A at the same time share it through L2.
//
// Roles (64 + 32 x epilogue warps threads):
//   warp 0, one lane : TMA producer. A 128x128-byte tile and a BNx128-byte tile per stage,
//                      128-byte swizzled, into a STAGES-deep ring of shared-memory buffers.
//   warp 1, one lane : MMA issuer. 4 tcgen05.mma (K = 32 bytes each) per stage into a TMEM
//                      accumulator; two accumulators of BN columns (four for BN <= 128)
//                      cycle between tiles so the epilogue of one tile overlaps the MMAs of
//                      the next.
//   warps 2..        : epilogue (8 warps, 16 for the GELU epilogue). Warp w reads TMEM lanes
//                      32*(w%4).. (one output row per thread) in its share of the tile's
//                      columns, 32 at a time, applies the epilogue functor, writes the
//                      32x32 block into one of its two swizzled shared-memory staging blocks and
//                      one lane issues a TMA tile store (or, for the residual stream, a TMA
//                      reduce-add), so global writes are whole swizzle rows issued by the copy
//                      engine and a store drains while the next chunk is packed.
//
// Operands are bf16 (kind::f16, K-step 64 per stage) or e4m3 (kind::f8f6f4, K-step 128 per
// stage); either way a stage row is 128 bytes. K tails and M tails are zero-filled by TMA
// on load and clipped by TMA on store.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "e4m3x2.cuh"
#include "ptx.cuh"

namespace mrn {

constexpr int kTileM = 128;
constexpr int kStageRowBytes = 128;  // one swizzle row: 64 bf16 or 128 e4m3 values of K
constexpr uint32_t kTmemCols = 512;  // two accumulators of up to 256 f32 columns
constexpr int kEpiChunk = 32;        // columns per epilogue step
constexpr int kMaxSmem = 232448;     // 227 KB per CTA

// Shared memory of one (BN, epilogue) instantiation: the operand ring plus one 32 x 32 staging
// block per epilogue warp. A_TERMS = 2 for two-term e4m3 activations (hi and lo A tiles per stage).
template <int BN, int EPI_WARPS, int OUT_BYTES, int A_TERMS = 1>
struct GemmShape {
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN must be a multiple of 32 in [32, 256]");
  static constexpr int kABytes = A_TERMS * kTileM * kStageRowBytes;
  static constexpr int kBBytes = BN * kStageRowBytes;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kEpiBufBytes = 32 * kEpiChunk * OUT_BYTES;
  static constexpr int kBarrierBytes = 256;
  // Two staging blocks per warp (a chunk's store drains while the next chunk is packed) unless
  // that costs the operand ring a stage below four.
  static constexpr int kFit2 = (kMaxSmem - 1024 - kBarrierBytes - 2 * EPI_WARPS * kEpiBufBytes) / kStageBytes;
  static constexpr int kFit1 = (kMaxSmem - 1024 - kBarrierBytes - EPI_WARPS * kEpiBufBytes) / kStageBytes;
  static constexpr int kEpiBuffers = (kFit2 >= 4 || kFit2 == kFit1) ? 2 : 1;
  static constexpr int kEpiBytes = kEpiBuffers * EPI_WARPS * kEpiBufBytes;
  static constexpr int kFit = (kMaxSmem - 1024 - kBarrierBytes - kEpiBytes) / kStageBytes;
  static constexpr int kStages = kFit > 8 ? 8 : kFit;
  static_assert(kStages >= 2, "not enough shared memory for a 2-stage pipeline");
  static constexpr int kSmemBytes = 1024 /*alignment slack*/ + kStages * kStageBytes + kEpiBytes + kBarrierBytes;
  static constexpr int kThreads = 64 + 32 * EPI_WARPS;
};

__device__ __forceinline__ float rcp_approx(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ float ex2_approx(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ __half2 ex2_approx_h2(__half2 x) {
  uint32_t r;
  asm("ex2.approx.f16x2 %0, %1;" : "=r"(r) : "r"(*reinterpret_cast<const uint32_t*>(&x)));
  return *reinterpret_cast<const __half2*>(&r);
}

// (lo, hi) -> f16x2, saturating to +-65504 instead of overflowing to infinity.
__device__ __forceinline__ __half2 f32x2_to_h2_sat(float2 v) {
  uint32_t r;
  asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(v.y), "f"(v.x));
  return *reinterpret_cast<const __half2*>(&r);
}

// Exact GELU, x Phi(x) with Phi the standard normal CDF (torch.nn.GELU(); the reference's
// gelu_exact, src/net/cuda/kernels.cu:62-65), written as
//
//     GELU(x) = relu(x) - |x| Phi(-|x|),    Phi(-a) = 2^(-g(a)),   g(a) = -log2 Phi(-a),
//
// so an element costs one hardware exponential (ex2) plus a polynomial for g, which is smooth
// and convex on a >= 0. The coefficients (negated, so the Horner chain gives -g) are
// least-squares fits on Chebyshev nodes made by gelu_fit.py beside this file; a is clamped
// at the fit's bound, past which Phi(-a) no longer moves the output by half an ulp.
//   f32 form (bf16 outputs): degree 7, |relative GELU error| <= 4.3e-6.
//   packed f16 form (outputs rounded to e4m3 next, 12.5% steps): degree 4, <= 1.0e-2,
//   most of it the f16 rounding of x itself.
// kGeluF32: degree 7 on [0, 5.5], max relative GELU error 4.21e-06 in float32
constexpr float kGeluF32Bound = 5.5f;
constexpr float kGeluF32_0 = -9.999938561e-01f;
constexpr float kGeluF32_1 = -1.151278331e+00f;
constexpr float kGeluF32_2 = -4.583817849e-01f;
constexpr float kGeluF32_3 = -5.405228293e-02f;
constexpr float kGeluF32_4 = 8.556272268e-03f;
constexpr float kGeluF32_5 = -9.434208502e-04f;
constexpr float kGeluF32_6 = 6.328849712e-05f;
constexpr float kGeluF32_7 = -1.921234625e-06f;
// kGeluF16: degree 4 on [0, 4.5], max relative GELU error 1.00e-02 in float16
constexpr float kGeluF16Bound = 4.5f;
constexpr float kGeluF16_0 = -1.001255186e+00f;
constexpr float kGeluF16_1 = -1.136516071e+00f;
constexpr float kGeluF16_2 = -4.867097285e-01f;
constexpr float kGeluF16_3 = -3.413367701e-02f;
constexpr float kGeluF16_4 = 2.233444850e-03f;

// GELU of two f32 values, packed arithmetic for the polynomial.
__device__ __forceinline__ float2 gelu2(float2 x) {
  const float2 a = make_float2(fabsf(x.x), fabsf(x.y));
  const float2 t = make_float2(fminf(a.x, kGeluF32Bound), fminf(a.y, kGeluF32Bound));
  float2 p = fma2(t, make_float2(kGeluF32_7, kGeluF32_7), make_float2(kGeluF32_6, kGeluF32_6));
  p = fma2(t, p, make_float2(kGeluF32_5, kGeluF32_5));
  p = fma2(t, p, make_float2(kGeluF32_4, kGeluF32_4));
  p = fma2(t, p, make_float2(kGeluF32_3, kGeluF32_3));
  p = fma2(t, p, make_float2(kGeluF32_2, kGeluF32_2));
  p = fma2(t, p, make_float2(kGeluF32_1, kGeluF32_1));
  p = fma2(t, p, make_float2(kGeluF32_0, kGeluF32_0));
  const float2 q = make_float2(ex2_approx(p.x), ex2_approx(p.y));  // Phi(-|x|)
  return fma2(make_float2(-a.x, -a.y), q, make_float2(fmaxf(x.x, 0.f), fmaxf(x.y, 0.f)));
}

// The same on a packed f16 pair.
__device__ __forceinline__ __half2 gelu_h2(__half2 x) {
  const __half2 a = __habs2(x);
  const __half2 t = __hmin2(a, __float2half2_rn(kGeluF16Bound));
  __half2 p = __hfma2(t, __float2half2_rn(kGeluF16_4), __float2half2_rn(kGeluF16_3));
  p = __hfma2(t, p, __float2half2_rn(kGeluF16_2));
  p = __hfma2(t, p, __float2half2_rn(kGeluF16_1));
  p = __hfma2(t, p, __float2half2_rn(kGeluF16_0));
  const __half2 q = ex2_approx_h2(p);
  return __hfma2(__hneg2(a), q, __hmax2(x, __float2half2_rn(0.f)));
}

// Byte offset of 16-byte chunk `j` of row `r` in a staging block whose rows are RB bytes and
// which the TMA map reads with the matching swizzle (RB 128 -> 128B, 64 -> 64B, 32 -> 32B):
// the swizzle XORs address bits [4, 4+log2(RB/16)) with bits [7, ...).
template <int RB>
__device__ __forceinline__ int staged_offset(int r, int j) {
  if constexpr (RB == 128) return r * 128 + ((j ^ (r & 7)) << 4);
  if constexpr (RB == 64) return r * 64 + ((j ^ ((r >> 1) & 3)) << 4);
  return r * 32 + ((j ^ ((r >> 2) & 1)) << 4);
}

// ---- epilogues -------------------------------------------------------------------------
// `pack` turns one row's 32 accumulator columns (starting at output column `col`) into the
// row's kOutBytes*32 output bytes as 16-byte chunks.

// out = bf16(acc * scale + bias)
struct EpiBiasBf16 {
  static constexpr int kOutBytes = 2;
  static constexpr bool kReduce = false;
  static constexpr int kWarps = 8;
  static constexpr int kTerms = 1;
  const float* bias;
  float scale;
  __device__ __forceinline__ void pack(int col, const float (&v)[32], uint4 (&o)[4]) const {
    const float2 s2 = make_float2(scale, scale);
#pragma unroll
    for (int c = 0; c < 32; c += 4) {
      const float4 b = __ldg(reinterpret_cast<const float4*>(bias + col + c));
      const float2 y0 = fma2(make_float2(v[c], v[c + 1]), s2, make_float2(b.x, b.y));
      const float2 y1 = fma2(make_float2(v[c + 2], v[c + 3]), s2, make_float2(b.z, b.w));
      __nv_bfloat162 p[2] = {__floats2bfloat162_rn(y0.x, y0.y), __floats2bfloat162_rn(y1.x, y1.y)};
      reinterpret_cast<uint2*>(o)[c / 4] = *reinterpret_cast<const uint2*>(p);
    }
  }
};

// The 32 bias values of an epilogue chunk starting at column `col`, as 8 vectors (loaded ahead of
// the accumulator where a kernel has the registers to spare).
__device__ __forceinline__ void load_bias32(const float* bias, int col, float4 (&b)[8]) {
#pragma unroll
  for (int k = 0; k < 8; ++k) b[k] = __ldg(reinterpret_cast<const float4*>(bias + col) + k);
}

// out = GELU(acc * scale + bias) as bf16, or as e4m3 codes of value * inv_q (saturating).
// The GELU is the bulk of the epilogue's arithmetic, so it gets 16 warps.
template <bool E4M3>
struct EpiGelu {
  static constexpr int kOutBytes = E4M3 ? 1 : 2;
  static constexpr bool kReduce = false;
  static constexpr int kWarps = 16;
  static constexpr int kTerms = 1;
  const float* bias;
  float scale;
  float inv_q;
  __device__ __forceinline__ void pack(int col, const float (&v)[32], uint4 (&o)[kOutBytes * 2]) const {
    float4 b[8];
    load_bias32(bias, col, b);
    pack_with(b, v, o);
  }
  __device__ __forceinline__ void pack_with(const float4 (&b)[8], const float (&v)[32],
                                            uint4 (&o)[kOutBytes * 2]) const {
    const float2 s2 = make_float2(scale, scale);
    if constexpr (E4M3) {
      const __half2 iq = __float2half2_rn(inv_q);
#pragma unroll
      for (int c = 0; c < 32; c += 16) {
        __nv_fp8x2_storage_t q[8];
#pragma unroll
        for (int j = 0; j < 8; j += 2) {
          const float4 bb = b[(c + 2 * j) / 4];
          const float2 x0 = fma2(make_float2(v[c + 2 * j], v[c + 2 * j + 1]), s2, make_float2(bb.x, bb.y));
          const float2 x1 = fma2(make_float2(v[c + 2 * j + 2], v[c + 2 * j + 3]), s2, make_float2(bb.z, bb.w));
          const __half2 y0 = __hmul2(gelu_h2(f32x2_to_h2_sat(x0)), iq);
          const __half2 y1 = __hmul2(gelu_h2(f32x2_to_h2_sat(x1)), iq);
          q[j] = __nv_cvt_halfraw2_to_fp8x2(y0, __NV_SATFINITE, __NV_E4M3);
          q[j + 1] = __nv_cvt_halfraw2_to_fp8x2(y1, __NV_SATFINITE, __NV_E4M3);
        }
        o[c / 16] = *reinterpret_cast<const uint4*>(q);
      }
    } else {
#pragma unroll
      for (int c = 0; c < 32; c += 4) {
        const float4 bb = b[c / 4];
        const float2 y0 = gelu2(fma2(make_float2(v[c], v[c + 1]), s2, make_float2(bb.x, bb.y)));
        const float2 y1 = gelu2(fma2(make_float2(v[c + 2], v[c + 3]), s2, make_float2(bb.z, bb.w)));
        __nv_bfloat162 p[2] = {__floats2bfloat162_rn(y0.x, y0.y), __floats2bfloat162_rn(y1.x, y1.y)};
        reinterpret_cast<uint2*>(o)[c / 4] = *reinterpret_cast<const uint2*>(p);
      }
    }
  }
};

// The tanh-form GELU (Gelu::Tanh, src/net/cpu.rs:270-276 in the reference):
//     0.5 x (1 + tanh(u)),  u = sqrt(2/pi) (x + 0.044715 x^3),
// written as relu(x) - |x| s(-2 u(|x|)) with the logistic s(-z) = 1 / (1 + e^z) (since
// 0.5 (1 + tanh(u)) = s(2u) and u is odd), so the negative tail keeps its relative accuracy
// where 1 + tanh(u) would cancel. One ex2 and one reciprocal per element; for large |x| the
// exponential overflows to infinity and the tail term is exactly 0.
constexpr float kGeluTanhC1 = 0.7978845608028654f * 2.8853900817779268f;  // sqrt(2/pi) * 2 log2(e)
constexpr float kGeluTanhC3 = kGeluTanhC1 * 0.044715f;
__device__ __forceinline__ float gelu_tanh(float x) {
  const float a = fabsf(x);
  const float z = a * fmaf(kGeluTanhC3, a * a, kGeluTanhC1);  // 2 u(|x|) log2(e)
  const float q = rcp_approx(1.f + ex2_approx(z));
  return fmaf(-a, q, fmaxf(x, 0.f));
}

// out = GELU_tanh(acc * scale + bias) as bf16, or as e4m3 codes of value * inv_q.
template <bool E4M3>
struct EpiGeluTanh {
  static constexpr int kOutBytes = E4M3 ? 1 : 2;
  static constexpr bool kReduce = false;
  static constexpr int kWarps = 16;
  static constexpr int kTerms = 1;
  const float* bias;
  float scale;
  float inv_q;
  __device__ __forceinline__ void pack(int col, const float (&v)[32], uint4 (&o)[kOutBytes * 2]) const {
    float4 b[8];
    load_bias32(bias, col, b);
    pack_with(b, v, o);
  }
  __device__ __forceinline__ void pack_with(const float4 (&b)[8], const float (&v)[32],
                                            uint4 (&o)[kOutBytes * 2]) const {
    const float2 s2 = make_float2(scale, scale);
#pragma unroll
    for (int c = 0; c < 32; c += 4) {
      const float4 bb = b[c / 4];
      const float2 x0 = fma2(make_float2(v[c], v[c + 1]), s2, make_float2(bb.x, bb.y));
      const float2 x1 = fma2(make_float2(v[c + 2], v[c + 3]), s2, make_float2(bb.z, bb.w));
      const float y0 = gelu_tanh(x0.x), y1 = gelu_tanh(x0.y), y2 = gelu_tanh(x1.x), y3 = gelu_tanh(x1.y);
      if constexpr (E4M3) {
        __nv_fp8x2_storage_t q[2] = {
            __nv_cvt_float2_to_fp8x2(make_float2(y0 * inv_q, y1 * inv_q), __NV_SATFINITE, __NV_E4M3),
            __nv_cvt_float2_to_fp8x2(make_float2(y2 * inv_q, y3 * inv_q), __NV_SATFINITE, __NV_E4M3)};
        reinterpret_cast<uint32_t*>(o)[c / 4] = *reinterpret_cast<const uint32_t*>(q);
      } else {
        __nv_bfloat162 p[2] = {__floats2bfloat162_rn(y0, y1), __floats2bfloat162_rn(y2, y3)};
        reinterpret_cast<uint2*>(o)[c / 4] = *reinterpret_cast<const uint2*>(p);
      }
    }
  }
};

// out = GELU(acc * scale + bias) * inv_q as two-term e4m3 (hi = e4m3(v), lo = e4m3(v - hi)), the
// erf form or (TANH) the tanh form, in f32: the row's 32 hi codes go to out[0..1] and its 32 lo codes
// to out[2..3]. The kernel stores them as two 32-column blocks, the lo block lo_col columns to the
// right of the hi block (an [M, 2N] output holding the hi codes, then the lo codes, of each row).
template <bool TANH>
struct EpiGeluE4m3x2 {
  static constexpr int kOutBytes = 2;
  static constexpr bool kReduce = false;
  static constexpr int kWarps = 16;
  static constexpr int kTerms = 2;
  const float* bias;
  float scale;
  float inv_q;
  int lo_col;
  __device__ __forceinline__ void pack(int col, const float (&v)[32], uint4 (&o)[4]) const {
    float4 b[8];
    load_bias32(bias, col, b);
    const float2 s2 = make_float2(scale, scale), q2 = make_float2(inv_q, inv_q);
    uint32_t* hi = reinterpret_cast<uint32_t*>(o);
    uint32_t* lo = hi + 8;
#pragma unroll
    for (int c = 0; c < 32; c += 4) {
      const float4 bb = b[c / 4];
      float2 y0 = fma2(make_float2(v[c], v[c + 1]), s2, make_float2(bb.x, bb.y));
      float2 y1 = fma2(make_float2(v[c + 2], v[c + 3]), s2, make_float2(bb.z, bb.w));
      if constexpr (TANH) {
        y0 = make_float2(gelu_tanh(y0.x), gelu_tanh(y0.y));
        y1 = make_float2(gelu_tanh(y1.x), gelu_tanh(y1.y));
      } else {
        y0 = gelu2(y0);
        y1 = gelu2(y1);
      }
      split_e4m3x4(mul2(y0, q2), mul2(y1, q2), hi[c / 4], lo[c / 4]);
    }
  }
};

// x += acc * scale + bias on the f16 residual stream, as a TMA reduce-add of the f16 values.
struct EpiResidual {
  static constexpr int kOutBytes = 2;
  static constexpr bool kReduce = true;
  static constexpr int kWarps = 8;
  static constexpr int kTerms = 1;
  const float* bias;
  float scale;
  __device__ __forceinline__ void pack(int col, const float (&v)[32], uint4 (&o)[4]) const {
    const float2 s2 = make_float2(scale, scale);
#pragma unroll
    for (int c = 0; c < 32; c += 4) {
      const float4 b = __ldg(reinterpret_cast<const float4*>(bias + col + c));
      const float2 y0 = fma2(make_float2(v[c], v[c + 1]), s2, make_float2(b.x, b.y));
      const float2 y1 = fma2(make_float2(v[c + 2], v[c + 3]), s2, make_float2(b.z, b.w));
      __half2 h[2] = {__floats2half2_rn(y0.x, y0.y), __floats2half2_rn(y1.x, y1.y)};
      reinterpret_cast<uint2*>(o)[c / 4] = *reinterpret_cast<const uint2*>(h);
    }
  }
};

// ---- the kernel ------------------------------------------------------------------------
// X2: two-term e4m3 A (e4m3 operands only): map_a reads the hi codes and map_a2 the lo codes of
// each A tile; every MMA step runs on both into the same accumulator. Otherwise map_a2 is unused.
template <int BN, bool FP8, class Epi, bool X2 = false>
__global__ void __launch_bounds__(64 + 32 * Epi::kWarps, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_a2,
                   const __grid_constant__ CUtensorMap map_b, const __grid_constant__ CUtensorMap map_out, Epi epi,
                   int M, int N, int K, int* status) {
  static_assert(FP8 || !X2, "two-term activations need e4m3 operands");
  using S = GemmShape<BN, Epi::kWarps, Epi::kOutBytes, X2 ? 2 : 1>;
  constexpr int kStages = S::kStages;
  constexpr int kEpiWarps = Epi::kWarps;
  constexpr int kEpiBufBytes = S::kEpiBufBytes;
  constexpr int kEpiBytes = S::kEpiBytes;
  constexpr int kElemsPerStage = FP8 ? 128 : 64;
  constexpr uint32_t kIdesc = FP8 ? idesc_e4m3(kTileM, BN) : idesc_bf16(kTileM, BN);
  // TMEM accumulators cycled between tiles: four of 128 columns for BN <= 128 (the epilogue
  // may trail the MMAs by three tiles), else two.
  constexpr int kAccs = BN <= 128 ? 4 : 2;
  constexpr int kRowBytes = kEpiChunk * Epi::kOutBytes;  // staged bytes per output row

  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the 128-byte swizzle atoms.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sm_a = smem;
  uint8_t* sm_b = smem + kStages * S::kABytes;
  uint8_t* sm_epi = smem + kStages * S::kStageBytes;  // 1024-aligned: stage sizes are multiples of 1024
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm_epi + kEpiBytes);
  uint64_t* full = bars;                      // [kStages] TMA -> MMA
  uint64_t* empty = bars + kStages;           // [kStages] MMA -> TMA
  uint64_t* tmem_full = bars + 2 * kStages;   // [kAccs] MMA -> epilogue
  uint64_t* tmem_empty = tmem_full + kAccs;   // [kAccs] epilogue -> MMA
  uint64_t* drain = tmem_empty + kAccs;       // [1] MMA completion on abort
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_tiles = N / BN;
  const int m_tiles = (M + kTileM - 1) / kTileM;
  const int total = m_tiles * n_tiles;
  const int k_blocks = (K + kElemsPerStage - 1) / kElemsPerStage;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < kAccs; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], kEpiWarps);
    }
    mbar_init(drain, 1);
    *abort = 0;
    fence_barrier_init();
    tma_prefetch_map(&map_a);
    if constexpr (X2) tma_prefetch_map(&map_a2);
    tma_prefetch_map(&map_b);
    tma_prefetch_map(&map_out);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dep_wait();
  grid_dep_launch();

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, parity_mask = 0;  // per stage: a load was issued, and in which phase
#ifdef MRN_TEST_HOOKS
      const int first_tile = g_test_no_loads ? total : static_cast<int>(blockIdx.x);
#else
      const int first_tile = blockIdx.x;
#endif
      for (int tile = first_tile; tile < total && !*abort; tile += gridDim.x) {
        const int m0 = (tile / n_tiles) * kTileM;
        const int n0 = (tile % n_tiles) * BN;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort)) {
            raise_error(status, abort, kErrTimeoutProducer);
            break;
          }
          mbar_arrive_expect_tx(&full[stage], S::kStageBytes);
          tma_load_2d(sm_a + stage * S::kABytes, &map_a, &full[stage], kb * kElemsPerStage, m0);
          if constexpr (X2)
            tma_load_2d(sm_a + stage * S::kABytes + kTileM * kStageRowBytes, &map_a2, &full[stage],
                        kb * kElemsPerStage, m0);
          tma_load_2d(sm_b + stage * S::kBBytes, &map_b, &full[stage], kb * kElemsPerStage, n0);
          issued_mask |= 1u << stage;
          parity_mask = (parity_mask & ~(1u << stage)) | (phase << stage);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (*abort) {
        // Let the copies still in flight land before the CTA's shared memory goes away.
        for (int s = 0; s < kStages; ++s)
          if (issued_mask & (1u << s)) mbar_wait_bounded(&full[s], (parity_mask >> s) & 1u);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool issued = false;
      for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
        if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1u, abort)) {
          raise_error(status, abort, kErrTimeoutMma);
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(acc * BN);
        bool ok = true;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort)) {
            raise_error(status, abort, kErrTimeoutMma);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sm_a + stage * S::kABytes);
          const uint32_t b_addr = smem_u32(sm_b + stage * S::kBBytes);
#pragma unroll
          for (int k = 0; k < kStageRowBytes / 32; ++k) {
            const uint64_t ad = desc_sw128(a_addr + 32u * k);
            const uint64_t bd = desc_sw128(b_addr + 32u * k);
            if constexpr (FP8) {
              mma_e4m3(d, ad, bd, kIdesc, (kb | k) != 0);
              if constexpr (X2) mma_e4m3(d, desc_sw128(a_addr + kTileM * kStageRowBytes + 32u * k), bd, kIdesc, 1);
            } else {
              mma_bf16(d, ad, bd, kIdesc, (kb | k) != 0);
            }
          }
          issued = true;
          tc_commit(&empty[stage]);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(&tmem_full[acc]);
        if (++acc == kAccs) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (*abort && issued) {
        // Let the MMAs already issued finish before their buffers and TMEM go away.
        tc_commit(drain);
        if (!mbar_wait_bounded(drain, 0) && status) atomicCAS(status, 0, kErrTimeoutDrain);
      }
    }
  } else {
    // ---- epilogue: warps 2..; warp w reads TMEM lane quarter w % 4 and takes every
    // kParts-th 32-column chunk of the tile, starting at its part index.
    constexpr int kParts = kEpiWarps / 4;
    const int quarter = warp & 3;
    const int part = (warp - 2) >> 2;
    uint8_t* const sb0 = sm_epi + (warp - 2) * S::kEpiBuffers * kEpiBufBytes;
    int buf = 0;  // staging block of the next chunk
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
      const int m0 = (tile / n_tiles) * kTileM;
      const int n0 = (tile % n_tiles) * BN;
      if (!mbar_wait(&tmem_full[acc], acc_phase, abort)) {
        if (lane == 0) raise_error(status, abort, kErrTimeoutEpilogue);
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN);
      const int row0 = m0 + quarter * 32;
#pragma unroll 1
      for (int c = part * kEpiChunk; c < BN; c += kParts * kEpiChunk) {
        float v[32];
        tmem_ld32(taddr + c, v);
        if (c + kParts * kEpiChunk >= BN) {
          // Last TMEM read of this tile by this warp: hand the accumulator back.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tmem_empty[acc]);
        }
        uint4 out[Epi::kOutBytes * 2];
        epi.pack(n0 + c, v, out);
        // The staging block must no longer be read by this warp's store from it (the previous
        // chunk's with one block, the one before with two).
        uint8_t* sb = sb0 + buf * kEpiBufBytes;
        buf = buf + 1 == S::kEpiBuffers ? 0 : buf + 1;
        if (lane == 0) bulk_wait_read<S::kEpiBuffers - 1>();
        __syncwarp();
        if constexpr (Epi::kTerms == 2) {
          // Two 32 x 32-byte blocks: the hi codes, then the lo codes.
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            *reinterpret_cast<uint4*>(sb + staged_offset<32>(lane, j)) = out[j];
            *reinterpret_cast<uint4*>(sb + 1024 + staged_offset<32>(lane, j)) = out[2 + j];
          }
        } else {
#pragma unroll
          for (int j = 0; j < Epi::kOutBytes * 2; ++j)
            *reinterpret_cast<uint4*>(sb + staged_offset<kRowBytes>(lane, j)) = out[j];
        }
        fence_async_shared();
        __syncwarp();
        if (lane == 0) {
          if (row0 < M) {
            if constexpr (Epi::kReduce) {
              tma_reduce_add_2d(&map_out, sb, n0 + c, row0);
            } else if constexpr (Epi::kTerms == 2) {
              tma_store_2d(&map_out, sb, n0 + c, row0);
              tma_store_2d(&map_out, sb + 1024, epi.lo_col + n0 + c, row0);
            } else {
              tma_store_2d(&map_out, sb, n0 + c, row0);
            }
          }
          bulk_commit();
        }
      }
      if (part * kEpiChunk >= BN) {
        // A warp without a chunk in this tile still releases the accumulator.
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tmem_empty[acc]);
      }
      if (++acc == kAccs) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---- the CTA-pair kernel ------------------------------------------------------------------
// The same GEMM on 256 x 256 output tiles computed by a cluster of two CTAs with tcgen05
// cta_group::2: each CTA loads its own 128 rows of A and 128 rows (output columns) of B into
// its shared memory, the even CTA (leader) issues M = 256, N = 256 MMAs that read both CTAs'
// operands, and each CTA's TMEM receives the 128 x 256 accumulator of its own rows. Per CTA a
// stage is 32 KB (against 48 KB for the same FLOPs on one CTA), so the ring is 6 deep.
//
// Barriers: the leader's full[s] counts both CTAs' TMA bytes (expect_tx posted by the leader);
// the leader's MMA commits to empty[s] and tmem_full[a] of both CTAs at once (multicast
// commit); tmem_empty[a] lives in the leader and counts the epilogue warps of both CTAs (the
// peer arrives remotely). Every wait is bounded as in the single-CTA kernel.
template <int OUT_BYTES, int EPI_WARPS, int A_TERMS = 1>
struct PairShape {
  static constexpr int kBN = 256;       // output columns per pair tile
  static constexpr int kBHalf = 128;    // B rows loaded by each CTA
  static constexpr int kABytes = A_TERMS * kTileM * kStageRowBytes;
  static constexpr int kBBytes = kBHalf * kStageRowBytes;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kEpiBufBytes = 32 * kEpiChunk * OUT_BYTES;
  static constexpr int kBarrierBytes = 256;
  static constexpr int kFit2 = (kMaxSmem - 1024 - kBarrierBytes - 2 * EPI_WARPS * kEpiBufBytes) / kStageBytes;
  static constexpr int kFit1 = (kMaxSmem - 1024 - kBarrierBytes - EPI_WARPS * kEpiBufBytes) / kStageBytes;
  static constexpr int kEpiBuffers = (kFit2 >= 4 || kFit2 == kFit1) ? 2 : 1;
  static constexpr int kEpiBytes = kEpiBuffers * EPI_WARPS * kEpiBufBytes;
  static constexpr int kFit = (kMaxSmem - 1024 - kBarrierBytes - kEpiBytes) / kStageBytes;
  static constexpr int kStages = kFit > 8 ? 8 : kFit;
  static_assert(kStages >= 2, "not enough shared memory for a 2-stage pipeline");
  static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + kEpiBytes + kBarrierBytes;
  static constexpr int kThreads = 64 + 32 * EPI_WARPS;
};

template <bool FP8, class Epi, bool X2 = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(64 + 32 * Epi::kWarps, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_a2,
                     const __grid_constant__ CUtensorMap map_b, const __grid_constant__ CUtensorMap map_out, Epi epi,
                     int M, int N, int K, int* status) {
  static_assert(FP8 || !X2, "two-term activations need e4m3 operands");
  using S = PairShape<Epi::kOutBytes, Epi::kWarps, X2 ? 2 : 1>;
  constexpr int BN = S::kBN;
  constexpr int kStages = S::kStages;
  constexpr int kEpiWarps = Epi::kWarps;
  constexpr int kEpiBufBytes = S::kEpiBufBytes;
  constexpr int kEpiBytes = S::kEpiBytes;
  constexpr int kElemsPerStage = FP8 ? 128 : 64;
  constexpr uint32_t kIdesc = FP8 ? idesc_e4m3(2 * kTileM, BN) : idesc_bf16(2 * kTileM, BN);
  constexpr int kRowBytes = kEpiChunk * Epi::kOutBytes;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sm_a = smem;
  uint8_t* sm_b = smem + kStages * S::kABytes;
  uint8_t* sm_epi = smem + kStages * S::kStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm_epi + kEpiBytes);
  uint64_t* full = bars;                     // [kStages] both CTAs' TMA -> leader's MMA (leader's copy used)
  uint64_t* empty = bars + kStages;          // [kStages] MMA -> each CTA's producer
  uint64_t* tmem_full = bars + 2 * kStages;  // [2] MMA -> each CTA's epilogue
  uint64_t* tmem_empty = tmem_full + 2;      // [2] both CTAs' epilogues -> MMA (leader's copy used)
  uint64_t* drain = tmem_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1;
  const int pairs = gridDim.x >> 1;
  const int n_tiles = N / BN;
  const int m_tiles = (M + 2 * kTileM - 1) / (2 * kTileM);
  const int total = m_tiles * n_tiles;
  const int k_blocks = (K + kElemsPerStage - 1) / kElemsPerStage;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], 2 * kEpiWarps);
    }
    mbar_init(drain, 1);
    *abort = 0;
    fence_barrier_init();
    tma_prefetch_map(&map_a);
    if constexpr (X2) tma_prefetch_map(&map_a2);
    tma_prefetch_map(&map_b);
    tma_prefetch_map(&map_out);
  }
  // Both CTAs' barriers exist before either signals the other's.
  cluster_sync();
  if (warp == 0) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dep_wait();
  grid_dep_launch();

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer (both CTAs): own A rows, own half of B; bytes counted on the leader
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, parity_mask = 0;
      for (int tile = pair; tile < total && !*abort; tile += pairs) {
        const int m0 = (tile / n_tiles) * 2 * kTileM + static_cast<int>(rank) * kTileM;
        const int nb = (tile % n_tiles) * BN + static_cast<int>(rank) * S::kBHalf;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort)) {
            raise_error(status, abort, kErrTimeoutProducer);
            break;
          }
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * S::kStageBytes);
          const uint32_t bar = map_to_rank(smem_u32(&full[stage]), 0);
          tma_load_2d_pair(sm_a + stage * S::kABytes, &map_a, bar, kb * kElemsPerStage, m0);
          if constexpr (X2)
            tma_load_2d_pair(sm_a + stage * S::kABytes + kTileM * kStageRowBytes, &map_a2, bar, kb * kElemsPerStage,
                             m0);
          tma_load_2d_pair(sm_b + stage * S::kBBytes, &map_b, bar, kb * kElemsPerStage, nb);
          issued_mask |= 1u << stage;
          parity_mask = (parity_mask & ~(1u << stage)) | (phase << stage);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (*abort && leader) {
        for (int s = 0; s < kStages; ++s)
          if (issued_mask & (1u << s)) mbar_wait_bounded(&full[s], (parity_mask >> s) & 1u);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---- MMA issuer (leader only)
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool issued = false;
      for (int tile = pair; tile < total; tile += pairs) {
        if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1u, abort)) {
          raise_error(status, abort, kErrTimeoutMma);
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(acc * BN);
        bool ok = true;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort)) {
            raise_error(status, abort, kErrTimeoutMma);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sm_a + stage * S::kABytes);
          const uint32_t b_addr = smem_u32(sm_b + stage * S::kBBytes);
#pragma unroll
          for (int k = 0; k < kStageRowBytes / 32; ++k) {
            const uint64_t ad = desc_sw128(a_addr + 32u * k);
            const uint64_t bd = desc_sw128(b_addr + 32u * k);
            if constexpr (FP8) {
              mma_pair_e4m3(d, ad, bd, kIdesc, (kb | k) != 0);
              if constexpr (X2)
                mma_pair_e4m3(d, desc_sw128(a_addr + kTileM * kStageRowBytes + 32u * k), bd, kIdesc, 1);
            } else {
              mma_pair_bf16(d, ad, bd, kIdesc, (kb | k) != 0);
            }
          }
          issued = true;
          tc_commit_pair(&empty[stage], 0x3);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit_pair(&tmem_full[acc], 0x3);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      if (*abort && issued) {
        tc_commit_pair(drain, 0x1);
        if (!mbar_wait_bounded(drain, 0) && status) atomicCAS(status, 0, kErrTimeoutDrain);
      }
    }
  } else {
    // ---- epilogue (both CTAs): this CTA's 128 rows x 256 columns
    constexpr int kParts = kEpiWarps / 4;
    const int quarter = warp & 3;
    const int part = (warp - 2) >> 2;
    uint8_t* const sb0 = sm_epi + (warp - 2) * S::kEpiBuffers * kEpiBufBytes;
    int buf = 0;  // staging block of the next chunk
    const uint32_t empty_addr0 = map_to_rank(smem_u32(&tmem_empty[0]), 0);
    const uint32_t empty_addr1 = map_to_rank(smem_u32(&tmem_empty[1]), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = pair; tile < total; tile += pairs) {
      const int m0 = (tile / n_tiles) * 2 * kTileM + static_cast<int>(rank) * kTileM;
      const int n0 = (tile % n_tiles) * BN;
      if (!mbar_wait(&tmem_full[acc], acc_phase, abort)) {
        if (lane == 0) raise_error(status, abort, kErrTimeoutEpilogue);
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN);
      const int row0 = m0 + quarter * 32;
#pragma unroll 1
      for (int c = part * kEpiChunk; c < BN; c += kParts * kEpiChunk) {
        float v[32];
        tmem_ld32(taddr + c, v);
        if (c + kParts * kEpiChunk >= BN) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(acc ? empty_addr1 : empty_addr0);
        }
        uint4 out[Epi::kOutBytes * 2];
        epi.pack(n0 + c, v, out);
        uint8_t* sb = sb0 + buf * kEpiBufBytes;
        buf = buf + 1 == S::kEpiBuffers ? 0 : buf + 1;
        if (lane == 0) bulk_wait_read<S::kEpiBuffers - 1>();
        __syncwarp();
        if constexpr (Epi::kTerms == 2) {
          // Two 32 x 32-byte blocks: the hi codes, then the lo codes.
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            *reinterpret_cast<uint4*>(sb + staged_offset<32>(lane, j)) = out[j];
            *reinterpret_cast<uint4*>(sb + 1024 + staged_offset<32>(lane, j)) = out[2 + j];
          }
        } else {
#pragma unroll
          for (int j = 0; j < Epi::kOutBytes * 2; ++j)
            *reinterpret_cast<uint4*>(sb + staged_offset<kRowBytes>(lane, j)) = out[j];
        }
        fence_async_shared();
        __syncwarp();
        if (lane == 0) {
          if (row0 < M) {
            if constexpr (Epi::kReduce) {
              tma_reduce_add_2d(&map_out, sb, n0 + c, row0);
            } else if constexpr (Epi::kTerms == 2) {
              tma_store_2d(&map_out, sb, n0 + c, row0);
              tma_store_2d(&map_out, sb + 1024, epi.lo_col + n0 + c, row0);
            } else {
              tma_store_2d(&map_out, sb, n0 + c, row0);
            }
          }
          bulk_commit();
        }
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  tc_fence_before();
  __syncwarp();
  // Neither CTA leaves (or frees TMEM) while the other may still signal its barriers.
  cluster_sync();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, kTmemCols);
  }
}

}  // namespace mrn
