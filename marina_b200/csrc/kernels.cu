// The evaluator's non-GEMM kernels: token embedding (fused with layer 0's norm1), warp-per-row
// LayerNorm, per-(position, head) attention on the tensor cores, the legal-move policy head
// and the value head's output layer. See kernels.cuh for the data layout.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include <type_traits>

#include "kernels.cuh"
#include "ptx.cuh"

namespace mrn {

namespace {

constexpr int kPlanes = 73;
constexpr int kActions = 64 * kPlanes;

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
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      const float* x = v + c * VEC;
      if (type == ActType::kBf16) {
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

// ---- embedding + layer 0 norm1 (src/net/cpu.rs:59-84, src/net/cuda/kernels.cu:69-100) ----
template <int VPL, int VEC>
__global__ void __launch_bounds__(256) embed_ln_kernel(EmbedParams e, NormParams n, int rows, int d) {
  // gamma [d], beta [d], both times the output's 1/scale (1 for bf16 outputs)
  extern __shared__ __align__(16) float gb[];
  const float oq = n.out_type == ActType::kE4m3 ? n.inv_q : 1.f;
  for (int k = threadIdx.x; k < d; k += blockDim.x) {
    gb[k] = n.gamma[k] * oq;
    gb[d + k] = n.beta[k] * oq;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  using Row = WarpRow<VPL, VEC>;
  Row r;
  const int pos = row / e.t, i = row - pos * e.t;
  const uint8_t* b = e.boards + static_cast<size_t>(pos) * 66;
  if (i == 0) {
    const uint8_t castling = b[64];
    const int ep = b[65] < 8 ? b[65] : 8;
#pragma unroll
    for (int c = 0; c < Row::kChunks; ++c)
#pragma unroll
      for (int k = 0; k < VEC; ++k) {
        const int o = Row::col(c, lane) + k;
        const float* w = e.castling_w + static_cast<size_t>(o) * 4;
        float s = 0.f;
#pragma unroll
        for (int bit = 0; bit < 4; ++bit) s += __ldg(w + bit) * static_cast<float>((castling >> bit) & 1);
        r.v[c * VEC + k] = (__ldg(e.state_embed + o) + (__ldg(e.castling_b + o) + s)) +
                           __ldg(e.ep_embed + static_cast<size_t>(ep) * d + o);
      }
  } else if (i >= e.square_start && i < e.square_start + 64) {
    const int s = i - e.square_start;
    const int piece = b[s] < 13 ? b[s] : 0;
    Row sq;
    r.load(e.piece_embed + static_cast<size_t>(piece) * d, lane);
    sq.load(e.square_embed + static_cast<size_t>(s) * d, lane);
#pragma unroll
    for (int k = 0; k < VPL; ++k) r.v[k] += sq.v[k];
  } else {
#pragma unroll
    for (int k = 0; k < VPL; ++k) r.v[k] = 0.f;
  }
  // norm1 sees the f16 values the residual stream keeps
  r.round_to_half();
  r.store(e.x + static_cast<size_t>(row) * d, lane);
  ln_apply(r, gb, gb + d, ln_stats(r, d, n.eps), lane);
  const size_t off = static_cast<size_t>(row) * d * (n.out_type == ActType::kBf16 ? 2 : 1);
  r.store_act(static_cast<uint8_t*>(n.out) + off, n.out_type, 1.f, lane);
}

// ---- LayerNorm, one warp per row (src/net/cpu.rs:323-343) --------------------------------
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

// Warps stride over rows; gamma and beta sit in shared memory and the next three rows are in
// flight (packed f16, VPL/2 registers each) while the current row is reduced. At 64 registers
// a thread (d <= 512), four 256-thread blocks fit on an SM: 32 warps x 3 rows of reads
// outstanding; wider rows get 128 registers and two blocks.
template <int VPL>
constexpr int ln_blocks_per_sm() {
  return VPL > 16 ? 2 : 4;
}

template <int VPL, int VEC>
__global__ void __launch_bounds__(256, ln_blocks_per_sm<VPL>()) layernorm_kernel(const __half* __restrict__ x,
                                                                                 NormParams n, int rows, int d) {
  // gamma [d], beta [d], both times the output's 1/scale (1 for bf16 outputs)
  extern __shared__ __align__(16) float gb[];
  const float oq = n.out_type == ActType::kE4m3 ? n.inv_q : 1.f;
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    gb[i] = n.gamma[i] * oq;
    gb[d + i] = n.beta[i] * oq;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int stride = gridDim.x * 8;
  int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const size_t out_bytes = n.out_type == ActType::kBf16 ? 2 : 1;
  using Row = WarpRow<VPL, VEC>;
  using Raw = RawRow<VPL, VEC>;
  Raw r0, r1, r2;
  r0.load(x + static_cast<size_t>(row) * d, lane);
  if (row + stride < rows) r1.load(x + static_cast<size_t>(row + stride) * d, lane);
  if (row + 2 * stride < rows) r2.load(x + static_cast<size_t>(row + 2 * stride) * d, lane);
  for (;;) {
    Row cur;
    r0.unpack(cur);
    r0 = r1;
    r1 = r2;
    if (row + 3 * stride < rows) r2.load(x + static_cast<size_t>(row + 3 * stride) * d, lane);
    ln_apply(cur, gb, gb + d, ln_stats(cur, d, n.eps), lane);
    cur.store_act(static_cast<uint8_t*>(n.out) + static_cast<size_t>(row) * d * out_bytes, n.out_type, 1.f, lane);
    row += stride;
    if (row >= rows) break;
  }
}

// ---- heads -----------------------------------------------------------------------------
// One CTA (8 warps) per position. Each warp takes legal slots in turn: the slot's square token
// gets the final norm and the policy norm in registers (src/net/cpu.rs:137,140-152) and its
// logit is bias[plane] + <token, W[plane]> (src/net/cuda/kernels.cu:407-444 gathers the same
// logits). Warp 0 also normalises the state token for the value head's first layer. The
// softmax over the legal slots is block-wide (src/net/cpu.rs:177-178).
constexpr int kHeadsWarps = 8;

template <int VPL, int VEC>
__global__ void __launch_bounds__(kHeadsWarps * 32) heads_kernel(HeadsParams p, int d) {
  extern __shared__ float logits[];  // [slots] when p.softmax
  __shared__ float red[kHeadsWarps];
  using Row = WarpRow<VPL, VEC>;
  const int pos = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t row0 = static_cast<size_t>(pos) * p.t;

  if (warp == 0) {
    Row r;
    r.load(p.x + row0 * d, lane);
    ln_apply(r, p.final_g, p.final_b, ln_stats(r, d, p.eps), lane);
    ln_apply(r, p.value_g, p.value_b, ln_stats(r, d, p.eps), lane);
    r.store_act(static_cast<__nv_bfloat16*>(p.value_in) + static_cast<size_t>(pos) * d, ActType::kBf16, 1.f, lane);
  }

  for (int slot = warp; slot < p.slots; slot += kHeadsWarps) {
    const int action = p.legal ? p.legal[static_cast<size_t>(pos) * p.slots + slot] : slot;
    float logit = -INFINITY;
    if (action >= kActions) {
      if (lane == 0 && p.status) atomicCAS(p.status, 0, kErrBadAction);
    } else if (action >= 0) {
      const int square = action / kPlanes, plane = action - square * kPlanes;
      Row r;
      r.load(p.x + (row0 + p.square_start + square) * d, lane);
      ln_apply(r, p.final_g, p.final_b, ln_stats(r, d, p.eps), lane);
      ln_apply(r, p.policy_g, p.policy_b, ln_stats(r, d, p.eps), lane);
      Row w;  // the plane's weight row, vector loads
      w.load(p.policy_w + static_cast<size_t>(plane) * d, lane);
      float2 acc = make_float2(0.f, 0.f);
#pragma unroll
      for (int k = 0; k < VPL; k += 2)
        acc = fma2(make_float2(r.v[k], r.v[k + 1]), make_float2(w.v[k], w.v[k + 1]), acc);
      logit = warp_sum(acc.x + acc.y) + __ldg(p.policy_bias + plane);
    }
    if (lane == 0) {
      if (p.softmax)
        logits[slot] = logit;
      else
        p.priors[static_cast<size_t>(pos) * p.slots + slot] = logit;
    }
  }
  if (!p.softmax) return;
  __syncthreads();

  float m = -INFINITY;
  for (int i = threadIdx.x; i < p.slots; i += blockDim.x) m = fmaxf(m, logits[i]);
  m = warp_max(m);
  if (lane == 0) red[warp] = m;
  __syncthreads();
  m = red[0];
#pragma unroll
  for (int w = 1; w < kHeadsWarps; ++w) m = fmaxf(m, red[w]);
  __syncthreads();
  float sum = 0.f;
  for (int i = threadIdx.x; i < p.slots; i += blockDim.x) {
    const float e = logits[i] == -INFINITY ? 0.f : expf(logits[i] - m);
    logits[i] = e;
    sum += e;
  }
  sum = warp_sum(sum);
  if (lane == 0) red[warp] = sum;
  __syncthreads();
  sum = 0.f;
#pragma unroll
  for (int w = 0; w < kHeadsWarps; ++w) sum += red[w];
  const float inv = 1.f / fmaxf(sum, 1.17549435e-38f);
  for (int i = threadIdx.x; i < p.slots; i += blockDim.x)
    p.priors[static_cast<size_t>(pos) * p.slots + i] = logits[i] * inv;
}

// Value head output layer and softmax, one warp per position (src/net/cpu.rs:161-162,179-180).
template <int VPL, int VEC>
__global__ void __launch_bounds__(256) value_out_kernel(ValueOutParams p, int positions, int d) {
  const int lane = threadIdx.x & 31;
  const int pos = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (pos >= positions) return;
  using Row = WarpRow<VPL, VEC>;
  const __nv_bfloat16* h = static_cast<const __nv_bfloat16*>(p.hidden) + static_cast<size_t>(pos) * d;
  float acc[3] = {0.f, 0.f, 0.f};
#pragma unroll
  for (int c = 0; c < Row::kChunks; ++c)
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      const int k = Row::col(c, lane) + e;
      const float hv = __bfloat162float(h[k]);
#pragma unroll
      for (int o = 0; o < 3; ++o) acc[o] += hv * __ldg(p.w2 + o * d + k);
    }
  float z[3];
#pragma unroll
  for (int o = 0; o < 3; ++o) z[o] = warp_sum(acc[o]) + __ldg(p.b2 + o);
  if (lane == 0) {
    float* out = p.wdl + static_cast<size_t>(pos) * 3;
    if (p.softmax) {
      const float m = fmaxf(z[0], fmaxf(z[1], z[2]));
      const float e0 = expf(z[0] - m), e1 = expf(z[1] - m), e2 = expf(z[2] - m);
      const float inv = 1.f / (e0 + e1 + e2);
      out[0] = e0 * inv, out[1] = e1 * inv, out[2] = e2 * inv;
    } else {
      out[0] = z[0], out[1] = z[1], out[2] = z[2];
    }
  }
}

// Dispatch on d (a multiple of 64 up to 1024): values per lane and vector width.
template <template <int, int> class Launch, class... Args>
cudaError_t dispatch_d(int d, Args&&... args) {
  switch (d) {
    case 64: return Launch<2, 2>::run(d, args...);
    case 128: return Launch<4, 4>::run(d, args...);
    case 192: return Launch<6, 2>::run(d, args...);
    case 256: return Launch<8, 4>::run(d, args...);
    case 320: return Launch<10, 2>::run(d, args...);
    case 384: return Launch<12, 4>::run(d, args...);
    case 448: return Launch<14, 2>::run(d, args...);
    case 512: return Launch<16, 4>::run(d, args...);
    case 640: return Launch<20, 4>::run(d, args...);
    case 768: return Launch<24, 4>::run(d, args...);
    case 1024: return Launch<32, 4>::run(d, args...);
  }
  return cudaErrorInvalidValue;
}

template <int VPL, int VEC>
struct EmbedLaunch {
  static cudaError_t run(int d, const EmbedParams& e, const NormParams& n, int positions, cudaStream_t s) {
    const int rows = positions * e.t;
    embed_ln_kernel<VPL, VEC><<<(rows + 7) / 8, 256, 2 * d * sizeof(float), s>>>(e, n, rows, d);
    return cudaGetLastError();
  }
};

template <int VPL, int VEC>
struct NormLaunch {
  static cudaError_t run(int d, const __half* x, const NormParams& n, int rows, cudaStream_t s) {
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int blocks_needed = (rows + 7) / 8;
    const int resident = sms * ln_blocks_per_sm<VPL>();
    const int grid = blocks_needed < resident ? blocks_needed : resident;
    layernorm_kernel<VPL, VEC><<<grid, 256, 2 * d * sizeof(float), s>>>(x, n, rows, d);
    return cudaGetLastError();
  }
};

template <int VPL, int VEC>
struct HeadsLaunch {
  static cudaError_t run(int d, const HeadsParams& p, int positions, cudaStream_t s) {
    const size_t smem = p.softmax ? sizeof(float) * p.slots : 0;
    heads_kernel<VPL, VEC><<<positions, kHeadsWarps * 32, smem, s>>>(p, d);
    return cudaGetLastError();
  }
};

template <int VPL, int VEC>
struct ValueOutLaunch {
  static cudaError_t run(int d, const ValueOutParams& p, int positions, cudaStream_t s) {
    value_out_kernel<VPL, VEC><<<(positions + 7) / 8, 256, 0, s>>>(p, positions, d);
    return cudaGetLastError();
  }
};

}  // namespace

cudaError_t launch_embed_ln(const EmbedParams& e, const NormParams& n, int positions, int d, cudaStream_t s) {
  return dispatch_d<EmbedLaunch>(d, e, n, positions, s);
}

cudaError_t launch_layernorm(const __half* x, const NormParams& n, int rows, int d, cudaStream_t s) {
  return dispatch_d<NormLaunch>(d, x, n, rows, s);
}

cudaError_t launch_heads(const HeadsParams& p, int positions, int d, cudaStream_t s) {
  return dispatch_d<HeadsLaunch>(d, p, positions, s);
}

cudaError_t launch_value_out(const ValueOutParams& p, int positions, int d, cudaStream_t s) {
  return dispatch_d<ValueOutLaunch>(d, p, positions, s);
}

}  // namespace mrn
