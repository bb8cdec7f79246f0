// Rows of d values held by one warp, and the LayerNorm arithmetic on them: shared by the
// embedding, LayerNorm and heads kernels, so that every LayerNorm of the evaluator rounds the
// same way.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include <type_traits>

#include "e4m3x2.cuh"
#include "kernels.cuh"
#include "ptx.cuh"

namespace mrn {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---- one row of d values held by a warp -------------------------------------------------
// Lane l holds VPL = d/32 values as VPL/VEC chunks of VEC consecutive elements; chunk c sits
// at element (c*32 + l)*VEC, so every chunk step is one coalesced warp-wide access.
template <int VPL, int VEC>
struct WarpRow {
  static constexpr int kChunks = VPL / VEC;
  float v[VPL];

  __device__ __forceinline__ static int col(int c, int lane) { return (c * 32 + lane) * VEC; }

  __device__ __forceinline__ void load(const float* __restrict__ src, int lane) {
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      if constexpr (VEC == 4) {
        const float4 q = *reinterpret_cast<const float4*>(src + col(c, lane));
        v[c * 4 + 0] = q.x, v[c * 4 + 1] = q.y, v[c * 4 + 2] = q.z, v[c * 4 + 3] = q.w;
      } else {
        const float2 q = *reinterpret_cast<const float2*>(src + col(c, lane));
        v[c * 2 + 0] = q.x, v[c * 2 + 1] = q.y;
      }
    }
  }

  // The same from / to the f16 residual stream.
  __device__ __forceinline__ void load(const __half* __restrict__ src, int lane) {
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      if constexpr (VEC == 4) {
        const uint2 q = *reinterpret_cast<const uint2*>(src + col(c, lane));
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&q.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&q.y));
        v[c * 4 + 0] = a.x, v[c * 4 + 1] = a.y, v[c * 4 + 2] = b.x, v[c * 4 + 3] = b.y;
      } else {
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(src + col(c, lane)));
        v[c * 2 + 0] = a.x, v[c * 2 + 1] = a.y;
      }
    }
  }

  // Round every value to f16 in place (what a store to the residual stream keeps).
  __device__ __forceinline__ void round_to_half() {
#pragma unroll
    for (int i = 0; i < VPL; ++i) v[i] = __half2float(__float2half_rn(v[i]));
  }

  __device__ __forceinline__ void store(__half* __restrict__ dst, int lane) const {
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      if constexpr (VEC == 4) {
        __half2 h[2] = {__floats2half2_rn(v[c * 4], v[c * 4 + 1]), __floats2half2_rn(v[c * 4 + 2], v[c * 4 + 3])};
        *reinterpret_cast<uint2*>(dst + col(c, lane)) = *reinterpret_cast<const uint2*>(h);
      } else {
        *reinterpret_cast<__half2*>(dst + col(c, lane)) = __floats2half2_rn(v[c * 2], v[c * 2 + 1]);
      }
    }
  }

  __device__ __forceinline__ void store(float* __restrict__ dst, int lane) const {
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      if constexpr (VEC == 4)
        *reinterpret_cast<float4*>(dst + col(c, lane)) = make_float4(v[c * 4], v[c * 4 + 1], v[c * 4 + 2], v[c * 4 + 3]);
      else
        *reinterpret_cast<float2*>(dst + col(c, lane)) = make_float2(v[c * 2], v[c * 2 + 1]);
    }
  }

  __device__ __forceinline__ void store_act(void* dst, ActType type, float inv_q, int lane) const {
    if (type == ActType::kE4m3x2)
      store_act<ActType::kE4m3x2>(dst, inv_q, lane);
    else if (type == ActType::kBf16)
      store_act<ActType::kBf16>(dst, inv_q, lane);
    else
      store_act<ActType::kE4m3>(dst, inv_q, lane);
  }

  // The same for an output type known at compile time.
  template <ActType OUT>
  __device__ __forceinline__ void store_act(void* dst, float inv_q, int lane) const {
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      const float* x = v + c * VEC;
      if constexpr (OUT == ActType::kE4m3x2) {
        // hi codes at the element's column, lo codes d = 32 VPL bytes further on (inv_q applied).
        uint8_t* o = static_cast<uint8_t*>(dst) + col(c, lane);
        if constexpr (VEC == 4) {
          uint32_t hi, lo;
          split_e4m3x4(make_float2(x[0] * inv_q, x[1] * inv_q), make_float2(x[2] * inv_q, x[3] * inv_q), hi, lo);
          *reinterpret_cast<uint32_t*>(o) = hi;
          *reinterpret_cast<uint32_t*>(o + 32 * VPL) = lo;
        } else {
          uint16_t hi, lo;
          split_e4m3x2(make_float2(x[0] * inv_q, x[1] * inv_q), hi, lo);
          *reinterpret_cast<uint16_t*>(o) = hi;
          *reinterpret_cast<uint16_t*>(o + 32 * VPL) = lo;
        }
      } else if constexpr (OUT == ActType::kBf16) {
        __nv_bfloat16* o = static_cast<__nv_bfloat16*>(dst) + col(c, lane);
        if constexpr (VEC == 4) {
          __nv_bfloat162 p[2] = {__floats2bfloat162_rn(x[0], x[1]), __floats2bfloat162_rn(x[2], x[3])};
          *reinterpret_cast<uint2*>(o) = *reinterpret_cast<const uint2*>(p);
        } else {
          *reinterpret_cast<__nv_bfloat162*>(o) = __floats2bfloat162_rn(x[0], x[1]);
        }
      } else {
        uint8_t* o = static_cast<uint8_t*>(dst) + col(c, lane);
        if constexpr (VEC == 4) {
          __nv_fp8x2_storage_t p[2] = {
              __nv_cvt_float2_to_fp8x2(make_float2(x[0] * inv_q, x[1] * inv_q), __NV_SATFINITE, __NV_E4M3),
              __nv_cvt_float2_to_fp8x2(make_float2(x[2] * inv_q, x[3] * inv_q), __NV_SATFINITE, __NV_E4M3)};
          *reinterpret_cast<uint32_t*>(o) = *reinterpret_cast<const uint32_t*>(p);
        } else {
          *reinterpret_cast<__nv_fp8x2_storage_t*>(o) =
              __nv_cvt_float2_to_fp8x2(make_float2(x[0] * inv_q, x[1] * inv_q), __NV_SATFINITE, __NV_E4M3);
        }
      }
    }
  }
};

// ---- LayerNorm arithmetic shared by the embedding and LayerNorm kernels -------------------
// (mean, 1/sqrt(var + eps)) of a warp-held row: biased two-pass variance as src/net/cpu.rs:331-336,
// on packed f32x2 arithmetic; d = 32 VPL, and a power-of-two d makes 1/d exact, so the mean is the
// reference's sum / d.
template <int VPL, int VEC>
__device__ __forceinline__ float2 ln_stats(const WarpRow<VPL, VEC>& cur, int d, float eps) {
  constexpr bool kPow2 = (VPL & (VPL - 1)) == 0;
  const float inv_d = 1.f / static_cast<float>(d);
  float2 s2 = make_float2(cur.v[0], cur.v[1]);
#pragma unroll
  for (int i = 2; i < VPL; i += 2) s2 = add2(s2, make_float2(cur.v[i], cur.v[i + 1]));
  const float s = warp_sum(s2.x + s2.y);
  const float mean = kPow2 ? s * inv_d : s / static_cast<float>(d);
  const float2 nm = make_float2(-mean, -mean);
  float2 q2 = make_float2(0.f, 0.f);
#pragma unroll
  for (int i = 0; i < VPL; i += 2) {
    const float2 c = add2(make_float2(cur.v[i], cur.v[i + 1]), nm);
    q2 = fma2(c, c, q2);
  }
  const float q = warp_sum(q2.x + q2.y);
  return make_float2(mean, rsqrtf((kPow2 ? q * inv_d : q / static_cast<float>(d)) + eps));
}

// In place: y = ((v - mean) * inv) * gamma + beta, gamma/beta read as vectors from `g`/`b`
// (shared or global memory, element k of the row at g[k]).
template <int VPL, int VEC>
__device__ __forceinline__ void ln_apply(WarpRow<VPL, VEC>& cur, const float* g, const float* b, float2 stats,
                                         int lane) {
  using Row = WarpRow<VPL, VEC>;
  const float inv = stats.y, mean = stats.x;
  const float2 i2 = make_float2(inv, inv), mi2 = make_float2(-mean * inv, -mean * inv);
#pragma unroll
  for (int k = 0; k < Row::kChunks; ++k) {
    const int col = Row::col(k, lane);
    if constexpr (VEC == 4) {
      const float4 g4 = *reinterpret_cast<const float4*>(g + col);
      const float4 b4 = *reinterpret_cast<const float4*>(b + col);
      const float2 t0 = fma2(make_float2(cur.v[k * 4], cur.v[k * 4 + 1]), i2, mi2);
      const float2 t1 = fma2(make_float2(cur.v[k * 4 + 2], cur.v[k * 4 + 3]), i2, mi2);
      const float2 y0 = fma2(t0, make_float2(g4.x, g4.y), make_float2(b4.x, b4.y));
      const float2 y1 = fma2(t1, make_float2(g4.z, g4.w), make_float2(b4.z, b4.w));
      cur.v[k * 4] = y0.x, cur.v[k * 4 + 1] = y0.y, cur.v[k * 4 + 2] = y1.x, cur.v[k * 4 + 3] = y1.y;
    } else {
      const float2 g2 = *reinterpret_cast<const float2*>(g + col);
      const float2 b2 = *reinterpret_cast<const float2*>(b + col);
      const float2 y = fma2(fma2(make_float2(cur.v[k * 2], cur.v[k * 2 + 1]), i2, mi2), g2, b2);
      cur.v[k * 2] = y.x, cur.v[k * 2 + 1] = y.y;
    }
  }
}

// One row of the f16 stream as loaded (VEC halves per chunk), kept packed until it is used.
template <int VPL, int VEC>
struct RawRow {
  static constexpr int kChunks = VPL / VEC;
  using Chunk = typename std::conditional<VEC == 4, uint2, uint32_t>::type;
  Chunk c[kChunks];
  __device__ __forceinline__ void load(const __half* __restrict__ src, int lane) {
#pragma unroll
    for (int k = 0; k < kChunks; ++k) c[k] = *reinterpret_cast<const Chunk*>(src + WarpRow<VPL, VEC>::col(k, lane));
  }
  __device__ __forceinline__ void unpack(WarpRow<VPL, VEC>& r) const {
#pragma unroll
    for (int k = 0; k < kChunks; ++k) {
      const __half2* h = reinterpret_cast<const __half2*>(&c[k]);
#pragma unroll
      for (int e = 0; e < VEC / 2; ++e) {
        const float2 f = __half22float2(h[e]);
        r.v[k * VEC + 2 * e] = f.x, r.v[k * VEC + 2 * e + 1] = f.y;
      }
    }
  }
};

}  // namespace mrn
