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

  // In place: LayerNorm over the d values (biased variance, two passes, as PyTorch).
  __device__ __forceinline__ void layernorm(const float* __restrict__ g, const float* __restrict__ b, float eps,
                                            int d, int lane) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) s += v[i];
    const float mean = warp_sum(s) / static_cast<float>(d);
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) q += (v[i] - mean) * (v[i] - mean);
    const float inv = 1.0f / sqrtf(warp_sum(q) / static_cast<float>(d) + eps);
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        const int k = col(c, lane) + e;
        v[c * VEC + e] = (v[c * VEC + e] - mean) * inv * __ldg(g + k) + __ldg(b + k);
      }
    }
  }

  // The same with gamma and beta already in registers (same element layout as this row).
  __device__ __forceinline__ void layernorm_regs(const WarpRow& g, const WarpRow& b, float eps, int d) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) s += v[i];
    const float mean = warp_sum(s) / static_cast<float>(d);
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) q += (v[i] - mean) * (v[i] - mean);
    const float inv = 1.0f / sqrtf(warp_sum(q) / static_cast<float>(d) + eps);
#pragma unroll
    for (int i = 0; i < VPL; ++i) v[i] = (v[i] - mean) * inv * g.v[i] + b.v[i];
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

// ---- embedding + layer 0 norm1 (src/net/cpu.rs:59-84, src/net/cuda/kernels.cu:69-100) ----
template <int VPL, int VEC>
__global__ void __launch_bounds__(256) embed_ln_kernel(EmbedParams e, NormParams n, int rows, int d) {
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
#pragma unroll
    for (int c = 0; c < Row::kChunks; ++c)
#pragma unroll
      for (int k = 0; k < VEC; ++k) {
        const int o = Row::col(c, lane) + k;
        r.v[c * VEC + k] =
            __ldg(e.piece_embed + static_cast<size_t>(piece) * d + o) + __ldg(e.square_embed + static_cast<size_t>(s) * d + o);
      }
  } else {
#pragma unroll
    for (int k = 0; k < VPL; ++k) r.v[k] = 0.f;
  }
  // norm1 sees the f16 values the residual stream keeps
  r.round_to_half();
  r.store(e.x + static_cast<size_t>(row) * d, lane);
  r.layernorm(n.gamma, n.beta, n.eps, d, lane);
  const size_t off = static_cast<size_t>(row) * d * (n.out_type == ActType::kBf16 ? 2 : 1);
  r.store_act(static_cast<uint8_t*>(n.out) + off, n.out_type, n.inv_q, lane);
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
  // d = 32 VPL; a power of two makes 1/d exact, so the mean is the reference's sum / d
  constexpr bool kPow2 = (VPL & (VPL - 1)) == 0;
  const float inv_d = 1.f / static_cast<float>(d);
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
    const float inv = rsqrtf((kPow2 ? q * inv_d : q / static_cast<float>(d)) + n.eps);
    // y = ((v - mean) * inv) * gamma + beta, two lanes per instruction
    const float2 i2 = make_float2(inv, inv), mi2 = make_float2(-mean * inv, -mean * inv);
#pragma unroll
    for (int k = 0; k < Row::kChunks; ++k) {
      const int col = Row::col(k, lane);
#pragma unroll
      for (int e = 0; e < VEC; e += 2) {
        const float2 g = *reinterpret_cast<const float2*>(gb + col + e);
        const float2 b = *reinterpret_cast<const float2*>(gb + d + col + e);
        const float2 t = fma2(make_float2(cur.v[k * VEC + e], cur.v[k * VEC + e + 1]), i2, mi2);
        const float2 y = fma2(t, g, b);
        cur.v[k * VEC + e] = y.x, cur.v[k * VEC + e + 1] = y.y;
      }
    }
    cur.store_act(static_cast<uint8_t*>(n.out) + static_cast<size_t>(row) * d * out_bytes, n.out_type, 1.f, lane);
    row += stride;
    if (row >= rows) break;
  }
}

// ---- attention ---------------------------------------------------------------------------
// Work item = (position, head); Q, K and V of the item (t <= 80 rows, zero-padded to 80) live
// in shared memory. Warp w owns query rows 16w..16w+15: S = Q K^T for its strip stays in
// registers (mma.sync m16n8k16, f32 accumulation), the softmax runs on the accumulators with
// quad shuffles, and the probabilities feed P V straight from registers.
__device__ __forceinline__ void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], const void* p) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], const void* p) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}

__device__ __forceinline__ void ldmatrix_x2(uint32_t (&r)[2], const void* p) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(a));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

constexpr int kAttnRows = 80;
constexpr int kAttnWarps = kAttnRows / 16;
constexpr int kAttnCtasPerSm = 3;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(a), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ float ex2_approx(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// Persistent: each CTA walks (position, head) items with a stride of the grid, keeping two
// Q/K/V buffers so the next item's loads (cp.async) overlap the current item's math. Rows
// T..79 of both buffers are zeroed once and never written again. T (tokens per position) is a
// template parameter so the key masks fold to constants: key tiles entirely past T are skipped.
// Each warp writes its normalised 16-row output strip over its own (dead) Q rows in shared
// memory and stores it with 16-byte writes.
template <int HD, int T, bool E4M3>
__global__ void __launch_bounds__(kAttnWarps * 32, kAttnCtasPerSm) attention_kernel(AttentionParams p, int items) {
  constexpr int LD = HD + 8;  // bf16 elements per staged row (16-byte multiple, conflict-free)
  constexpr int CH = HD / 8;  // 16-byte chunks per row
  constexpr int MAT = kAttnRows * LD;
  constexpr int NT = (T + 7) / 8;    // key tiles of 8 holding at least one valid key
  constexpr int KS = (T + 15) / 16;  // k16 steps of P V
  constexpr int ROWS_PER_PASS = kAttnWarps * 32 / CH;
  static_assert(T <= kAttnRows && 2 * KS <= 10, "tokens per position");
  extern __shared__ __align__(16) __nv_bfloat16 smem_attn[];  // [2][3][kAttnRows][LD]

  const int d = p.d, heads = p.heads;
  const __nv_bfloat16* qkv = static_cast<const __nv_bfloat16*>(p.qkv);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tq = lane & 3;
  const int r0 = warp * 16;

  for (int i = threadIdx.x; i < 2 * 3 * (kAttnRows - T) * CH; i += blockDim.x) {
    const int per_mat = (kAttnRows - T) * CH;
    const int m = i / per_mat, rem = i - m * per_mat;
    const int row = T + rem / CH, ch = rem % CH;
    *reinterpret_cast<uint4*>(smem_attn + m * MAT + row * LD + ch * 8) = make_uint4(0, 0, 0, 0);
  }

  const int ld_ch = threadIdx.x % CH, ld_row0 = threadIdx.x / CH;
  auto load = [&](int item, int buf) {
    const int pos = item / heads, head = item - pos * heads;
    const __nv_bfloat16* base = qkv + static_cast<size_t>(pos) * T * 3 * d + head * HD + ld_ch * 8;
    __nv_bfloat16* dst = smem_attn + buf * 3 * MAT + ld_ch * 8;
#pragma unroll
    for (int m = 0; m < 3; ++m)
#pragma unroll
      for (int row = ld_row0; row < T; row += ROWS_PER_PASS)
        cp_async16(dst + m * MAT + row * LD, base + static_cast<size_t>(row) * 3 * d + m * d);
  };

  int item = blockIdx.x;
  if (item < items) load(item, 0);
  cp_async_commit();
  const float scale_log2 = rsqrtf(static_cast<float>(HD)) * 1.4426950408889634f;
  for (int it = 0; item < items; ++it, item += gridDim.x) {
    const int buf = it & 1;
    const int next = item + gridDim.x;
    if (next < items) load(next, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();

    __nv_bfloat16* sq = smem_attn + buf * 3 * MAT;
    const __nv_bfloat16* sk = sq + MAT;
    const __nv_bfloat16* sv = sk + MAT;
    const int pos = item / heads, head = item - pos * heads;
    if (r0 < T) {
      // S = Q K^T for rows r0..r0+15 against the key tiles holding valid keys.
      float s[2 * KS][4];
#pragma unroll
      for (int nt = 0; nt < 2 * KS; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
      // ldmatrix lane roles: lane l supplies the row address of 8x8 matrix l / 8, row l % 8.
      const int lm = lane >> 3, lr = lane & 7;
#pragma unroll
      for (int kk = 0; kk < HD; kk += 16) {
        // A fragment: matrices (rows r0.., k kk), (r0+8.., kk), (r0.., kk+8), (r0+8.., kk+8)
        uint32_t a[4];
        ldmatrix_x4(a, sq + (r0 + (lm & 1) * 8 + lr) * LD + kk + (lm >> 1) * 8);
        // B fragments of two key tiles per ldmatrix: (keys nt*8.., k kk), (nt*8.., kk+8),
        // (nt*8+8.., kk), (nt*8+8.., kk+8)
#pragma unroll
        for (int nt = 0; nt + 1 < NT; nt += 2) {
          uint32_t b[4];
          ldmatrix_x4(b, sk + (nt * 8 + (lm >> 1) * 8 + lr) * LD + kk + (lm & 1) * 8);
          mma_16816(s[nt], a, b[0], b[1]);
          mma_16816(s[nt + 1], a, b[2], b[3]);
        }
        if constexpr (NT % 2 == 1) {
          uint32_t b[2];
          ldmatrix_x2(b, sk + ((NT - 1) * 8 + lr) * LD + kk + (lm & 1) * 8);
          mma_16816(s[NT - 1], a, b[0], b[1]);
        }
      }
      // Softmax of rows g (values 0,1) and g+8 (values 2,3); keys >= T are masked.
      float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int j = 0; j < 2; ++j)
          if (nt * 8 + 7 < T || nt * 8 + 2 * tq + j < T) {
            m0 = fmaxf(m0, s[nt][j]);
            m1 = fmaxf(m1, s[nt][2 + j]);
          }
      m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, 1));
      m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, 2));
      m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, 1));
      m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, 2));
      const float b0 = -m0 * scale_log2, b1 = -m1 * scale_log2;
      float l0 = 0.f, l1 = 0.f;
#pragma unroll
      for (int nt = 0; nt < 2 * KS; ++nt)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          if (nt >= NT) {
            s[nt][j] = s[nt][2 + j] = 0.f;
          } else if (nt * 8 + 7 < T || nt * 8 + 2 * tq + j < T) {
            s[nt][j] = ex2_approx(fmaf(s[nt][j], scale_log2, b0));
            s[nt][2 + j] = ex2_approx(fmaf(s[nt][2 + j], scale_log2, b1));
          } else {
            s[nt][j] = s[nt][2 + j] = 0.f;
          }
          l0 += s[nt][j];
          l1 += s[nt][2 + j];
        }
      l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
      l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
      l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
      l1 += __shfl_xor_sync(0xffffffffu, l1, 2);

      // O = P V: P comes from the S accumulators (two n-tiles make one k16 A fragment).
      float o[HD / 8][4];
#pragma unroll
      for (int nt = 0; nt < HD / 8; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < KS; ++kk) {
        uint32_t a[4];
        a[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
        a[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
        a[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
        a[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
        const int key = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
        for (int nt = 0; nt < HD / 8; nt += 2) {
          uint32_t b[4];
          ldmatrix_x4_trans(b, sv + key * LD + nt * 8 + ((lane >> 4) & 1) * 8);
          mma_16816(o[nt], a, b[0], b[1]);
          mma_16816(o[nt + 1], a, b[2], b[3]);
        }
      }

      // Normalised strip -> this warp's Q rows (no longer read) -> 16-byte global stores.
      const float inv0 = 1.f / l0, inv1 = 1.f / l1;
      __syncwarp();
#pragma unroll
      for (int nt = 0; nt < HD / 8; ++nt) {
        const int col = nt * 8 + 2 * tq;
        if constexpr (E4M3) {
          uint8_t* so = reinterpret_cast<uint8_t*>(sq);
          *reinterpret_cast<__nv_fp8x2_storage_t*>(so + (r0 + g) * (LD * 2) + col) = __nv_cvt_float2_to_fp8x2(
              make_float2(o[nt][0] * inv0 * p.inv_q, o[nt][1] * inv0 * p.inv_q), __NV_SATFINITE, __NV_E4M3);
          *reinterpret_cast<__nv_fp8x2_storage_t*>(so + (r0 + g + 8) * (LD * 2) + col) = __nv_cvt_float2_to_fp8x2(
              make_float2(o[nt][2] * inv1 * p.inv_q, o[nt][3] * inv1 * p.inv_q), __NV_SATFINITE, __NV_E4M3);
        } else {
          *reinterpret_cast<__nv_bfloat162*>(sq + (r0 + g) * LD + col) = __floats2bfloat162_rn(o[nt][0] * inv0, o[nt][1] * inv0);
          *reinterpret_cast<__nv_bfloat162*>(sq + (r0 + g + 8) * LD + col) =
              __floats2bfloat162_rn(o[nt][2] * inv1, o[nt][3] * inv1);
        }
      }
      __syncwarp();
      constexpr int kRowBytes = HD * (E4M3 ? 1 : 2);
      constexpr int kChunks = kRowBytes / 16;  // 16-byte chunks per output row
      for (int i = lane; i < 16 * kChunks; i += 32) {
        const int rr = i / kChunks, c = i - rr * kChunks;
        const int row = r0 + rr;
        if (row >= T) continue;
        const uint4 v = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(sq) + row * (LD * 2) + c * 16);
        uint8_t* dst = static_cast<uint8_t*>(p.out) +
                       ((static_cast<size_t>(pos) * T + row) * d + head * HD) * (E4M3 ? 1 : 2) + c * 16;
        *reinterpret_cast<uint4*>(dst) = v;
      }
    }
    // Every warp is done with `buf` before the load two items ahead overwrites it.
    __syncthreads();
  }
  cp_async_wait<0>();
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
    r.layernorm(p.final_g, p.final_b, p.eps, d, lane);
    r.layernorm(p.value_g, p.value_b, p.eps, d, lane);
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
      r.layernorm(p.final_g, p.final_b, p.eps, d, lane);
      r.layernorm(p.policy_g, p.policy_b, p.eps, d, lane);
      const float* w = p.policy_w + static_cast<size_t>(plane) * d;
      float acc = 0.f;
#pragma unroll
      for (int c = 0; c < Row::kChunks; ++c)
#pragma unroll
        for (int e = 0; e < VEC; ++e) acc += r.v[c * VEC + e] * __ldg(w + Row::col(c, lane) + e);
      logit = warp_sum(acc) + __ldg(p.policy_bias + plane);
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
    embed_ln_kernel<VPL, VEC><<<(rows + 7) / 8, 256, 0, s>>>(e, n, rows, d);
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

namespace {
template <int HD, int T>
cudaError_t launch_attention_t(const AttentionParams& p, int grid, int items, cudaStream_t s) {
  const size_t smem = 2 * 3 * kAttnRows * (HD + 8) * sizeof(__nv_bfloat16);
  if (p.out_type == ActType::kE4m3)
    attention_kernel<HD, T, true><<<grid, kAttnWarps * 32, smem, s>>>(p, items);
  else
    attention_kernel<HD, T, false><<<grid, kAttnWarps * 32, smem, s>>>(p, items);
  return cudaGetLastError();
}

template <int HD, int T>
cudaError_t prepare_attention_t() {
  const int smem = 2 * 3 * kAttnRows * (HD + 8) * 2;
  cudaError_t e = cudaFuncSetAttribute(attention_kernel<HD, T, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(attention_kernel<HD, T, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
}
}  // namespace

// Board mode has 65 tokens (one state token, 64 squares; src/net/model.rs:17).
cudaError_t launch_attention(const AttentionParams& p, int positions, int head_dim, cudaStream_t s) {
  if (p.t != 65) return cudaErrorInvalidValue;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int items = positions * p.heads;
  const int grid = items < sms * kAttnCtasPerSm ? items : sms * kAttnCtasPerSm;
  if (head_dim == 64) return launch_attention_t<64, 65>(p, grid, items, s);
  if (head_dim == 32) return launch_attention_t<32, 65>(p, grid, items, s);
  return cudaErrorInvalidValue;
}

cudaError_t prepare_attention() {
  cudaError_t e = prepare_attention_t<64, 65>();
  if (e != cudaSuccess) return e;
  return prepare_attention_t<32, 65>();
}

cudaError_t launch_heads(const HeadsParams& p, int positions, int d, cudaStream_t s) {
  return dispatch_d<HeadsLaunch>(d, p, positions, s);
}

cudaError_t launch_value_out(const ValueOutParams& p, int positions, int d, cudaStream_t s) {
  return dispatch_d<ValueOutLaunch>(d, p, positions, s);
}

}  // namespace mrn
