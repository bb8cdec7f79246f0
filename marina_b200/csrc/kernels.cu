// The evaluator's non-GEMM kernels: token embedding (fused with layer 0's norm1), warp-per-row
// LayerNorm, per-(position, head) attention on the tensor cores, the legal-move policy head
// and the value head's output layer. See kernels.cuh for the data layout.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include <type_traits>

#include "kernels.cuh"
#include "launch.h"
#include "ptx.cuh"
#include "rows.cuh"

namespace mrn {

namespace {

constexpr int kPlanes = 73;
constexpr int kActions = 64 * kPlanes;

// ---- embedding + layer 0 norm1 (src/net/cpu.rs:59-84, src/net/cuda/kernels.cu:69-100) ----
template <int VPL, int VEC>
__global__ void __launch_bounds__(256) embed_ln_kernel(EmbedParams e, NormParams n, int rows, int d) {
  // gamma [d], beta [d], both times the output's 1/scale (1 for bf16 outputs)
  extern __shared__ __align__(16) float gb[];
  const float oq = n.out_type != ActType::kBf16 ? n.inv_q : 1.f;
  for (int k = threadIdx.x; k < d; k += blockDim.x) {
    gb[k] = n.gamma[k] * oq;
    gb[d + k] = n.beta[k] * oq;
  }
  __syncthreads();
  grid_dep_wait();
  grid_dep_launch();
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
  if (!n.out) return;  // layer 0's QKV normalises x itself
  ln_apply(r, gb, gb + d, ln_stats(r, d, n.eps), lane);
  const size_t off = static_cast<size_t>(row) * d * act_row_bytes(n.out_type);
  r.store_act(static_cast<uint8_t*>(n.out) + off, n.out_type, 1.f, lane);
}

// ---- LayerNorm, one warp per row (src/net/cpu.rs:323-343) --------------------------------
// Warps stride over rows; gamma and beta sit in shared memory and the next three rows are in
// flight (packed f16, VPL/2 registers each) while the current row is reduced. At 64 registers
// a thread (d <= 512), four 256-thread blocks fit on an SM: 32 warps x 3 rows of reads
// outstanding; wider rows get 128 registers and two blocks.
// (The two-term e4m3 store needs more registers at d = 512: three blocks of 80.)
template <int VPL, ActType OUT>
constexpr int ln_blocks_per_sm() {
  return VPL > 16 ? 2 : (VPL == 16 && OUT == ActType::kE4m3x2) ? 3 : 4;
}

// OUT (= n.out_type) is a template parameter so that each instantiation holds one store path.
template <int VPL, int VEC, ActType OUT>
__global__ void __launch_bounds__(256, ln_blocks_per_sm<VPL, OUT>()) layernorm_kernel(const __half* __restrict__ x,
                                                                                 NormParams n, int rows, int d) {
  // gamma [d], beta [d], both times the output's 1/scale (1 for bf16 outputs)
  extern __shared__ __align__(16) float gb[];
  const float oq = OUT != ActType::kBf16 ? n.inv_q : 1.f;
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    gb[i] = n.gamma[i] * oq;
    gb[d + i] = n.beta[i] * oq;
  }
  __syncthreads();
  grid_dep_wait();
  grid_dep_launch();
  const int lane = threadIdx.x & 31;
  const int stride = gridDim.x * 8;
  int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  constexpr size_t out_bytes = act_row_bytes(OUT);
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
    cur.template store_act<OUT>(static_cast<uint8_t*>(n.out) + static_cast<size_t>(row) * d * out_bytes, 1.f, lane);
    row += stride;
    if (row >= rows) break;
  }
}

// ---- heads -----------------------------------------------------------------------------
// One CTA (8 warps) per position. Each warp takes every 8th legal slot: the slot's square token
// gets the final norm and the policy norm in registers (src/net/cpu.rs:137,140-152) and its
// logit is bias[plane] + <token, W[plane]> (src/net/cuda/kernels.cu:407-444 gathers the same
// logits). Warp 0 also normalises the state token for the value head's first layer. The
// softmax over the legal slots is block-wide (src/net/cpu.rs:177-178).
constexpr int kHeadsWarps = 8;

// Two slots in flight take 2 x 2 rows of VPL values per thread. Blocks per SM for the register
// bound: the most at which the rows stay in registers (three blocks for d = 192 and d = 512,
// which then takes 80 registers; one block from d = 768).
template <int VPL>
constexpr int heads_blocks_per_sm() {
  return VPL >= 24 ? 1 : (VPL <= 8 || VPL == 16) ? 3 : 2;
}

template <int VPL, int VEC>
__global__ void __launch_bounds__(kHeadsWarps * 32, heads_blocks_per_sm<VPL>()) heads_kernel(HeadsParams p, int d) {
  extern __shared__ float logits[];  // [slots] when p.softmax
  __shared__ float red[kHeadsWarps];
  using Row = WarpRow<VPL, VEC>;
  const int pos = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t row0 = static_cast<size_t>(pos) * p.t;
  grid_dep_wait();
  grid_dep_launch();

  if (warp == 0) {
    Row r;
    r.load(p.x + row0 * d, lane);
    ln_apply(r, p.final_g, p.final_b, ln_stats(r, d, p.eps), lane);
    ln_apply(r, p.value_g, p.value_b, ln_stats(r, d, p.eps), lane);
    r.store_act(static_cast<__nv_bfloat16*>(p.value_in) + static_cast<size_t>(pos) * d, ActType::kBf16, 1.f, lane);
  }

  // Warp w owns slots w, w + 8, ...: one coalesced read gives it the actions of 32 of them
  // (lane i holds slot base + 8 i), padding and out-of-range slots get -inf at once, and the
  // legal ones are evaluated two at a time, so each warp's chain of dependent loads and
  // reductions is half as long as one slot after another.
  auto put = [&](int slot, float logit) {
    if (p.softmax)
      logits[slot] = logit;
    else
      p.priors[static_cast<size_t>(pos) * p.slots + slot] = logit;
  };
  auto logit_of = [&](int plane, Row& r, const Row& w) {
    ln_apply(r, p.final_g, p.final_b, ln_stats(r, d, p.eps), lane);
    ln_apply(r, p.policy_g, p.policy_b, ln_stats(r, d, p.eps), lane);
    float2 acc = make_float2(0.f, 0.f);
#pragma unroll
    for (int k = 0; k < VPL; k += 2)
      acc = fma2(make_float2(r.v[k], r.v[k + 1]), make_float2(w.v[k], w.v[k + 1]), acc);
    return warp_sum(acc.x + acc.y) + __ldg(p.policy_bias + plane);
  };
  for (int base = warp; base < p.slots; base += 32 * kHeadsWarps) {
    const int slot = base + kHeadsWarps * lane;
    int action = -1;
    if (slot < p.slots) action = p.legal ? p.legal[static_cast<size_t>(pos) * p.slots + slot] : slot;
    if (action >= kActions) {
      if (p.status) atomicCAS(p.status, 0, kErrBadAction);
      action = -1;
    }
    if (slot < p.slots && action < 0) put(slot, -INFINITY);
    unsigned todo = __ballot_sync(~0u, action >= 0);
    while (todo) {
      const int l1 = __ffs(todo) - 1;
      todo &= todo - 1;
      const int l2 = todo ? __ffs(todo) - 1 : l1;  // an odd last slot is computed twice
      todo &= todo - 1;
      const int a1 = __shfl_sync(~0u, action, l1), a2 = __shfl_sync(~0u, action, l2);
      Row r1, r2, w1, w2;
      r1.load(p.x + (row0 + p.square_start + a1 / kPlanes) * d, lane);
      r2.load(p.x + (row0 + p.square_start + a2 / kPlanes) * d, lane);
      w1.load(p.policy_w + static_cast<size_t>(a1 % kPlanes) * d, lane);
      w2.load(p.policy_w + static_cast<size_t>(a2 % kPlanes) * d, lane);
      const float z1 = logit_of(a1 % kPlanes, r1, w1), z2 = logit_of(a2 % kPlanes, r2, w2);
      if (lane == 0) {
        put(base + kHeadsWarps * l1, z1);
        if (l2 != l1) put(base + kHeadsWarps * l2, z2);
      }
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
  grid_dep_wait();
  grid_dep_launch();
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
    return launch_kernel(embed_ln_kernel<VPL, VEC>, dim3((rows + 7) / 8), dim3(256), 2 * d * sizeof(float), s, e, n,
                         rows, d);
  }
};

template <int VPL, int VEC>
struct NormLaunch {
  static cudaError_t run(int d, const __half* x, const NormParams& n, int rows, cudaStream_t s) {
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    switch (n.out_type) {
      case ActType::kBf16: return go<ActType::kBf16>(sms, d, x, n, rows, s);
      case ActType::kE4m3: return go<ActType::kE4m3>(sms, d, x, n, rows, s);
      case ActType::kE4m3x2: return go<ActType::kE4m3x2>(sms, d, x, n, rows, s);
    }
    return cudaErrorInvalidValue;
  }

  template <ActType OUT>
  static cudaError_t go(int sms, int d, const __half* x, const NormParams& n, int rows, cudaStream_t s) {
    const int blocks_needed = (rows + 7) / 8;
    const int resident = sms * ln_blocks_per_sm<VPL, OUT>();
    const int grid = blocks_needed < resident ? blocks_needed : resident;
    return launch_kernel(layernorm_kernel<VPL, VEC, OUT>, dim3(grid), dim3(256), 2 * d * sizeof(float), s, x, n, rows,
                         d);
  }
};

template <int VPL, int VEC>
struct HeadsLaunch {
  static cudaError_t run(int d, const HeadsParams& p, int positions, cudaStream_t s) {
    const size_t smem = p.softmax ? sizeof(float) * p.slots : 0;
    return launch_kernel(heads_kernel<VPL, VEC>, dim3(positions), dim3(kHeadsWarps * 32), smem, s, p, d);
  }
};

template <int VPL, int VEC>
struct ValueOutLaunch {
  static cudaError_t run(int d, const ValueOutParams& p, int positions, cudaStream_t s) {
    return launch_kernel(value_out_kernel<VPL, VEC>, dim3((positions + 7) / 8), dim3(256), 0, s, p, positions, d);
  }
};

// Four priors per thread: one 16-byte read, one 8-byte write.
__global__ void __launch_bounds__(256) priors_to_half_kernel(const float* __restrict__ in, __half* __restrict__ out,
                                                             int quads) {
  grid_dep_wait();
  grid_dep_launch();
  const int i = blockIdx.x * 256 + threadIdx.x;
  if (i >= quads) return;
  const float4 v = reinterpret_cast<const float4*>(in)[i];
  __half2 h[2] = {__floats2half2_rn(v.x, v.y), __floats2half2_rn(v.z, v.w)};
  reinterpret_cast<uint2*>(out)[i] = *reinterpret_cast<const uint2*>(h);
}

// Loads the kernels a network of width d launches (cudaFuncGetAttributes makes the runtime load a
// function that lazy module loading would otherwise load, and allocate device memory for, at its
// first launch).
template <int VPL, int VEC>
struct LoadKernels {
  static cudaError_t run(int) {
    cudaFuncAttributes a;
    cudaError_t e;
    if ((e = cudaFuncGetAttributes(&a, embed_ln_kernel<VPL, VEC>)) != cudaSuccess) return e;
    if ((e = cudaFuncGetAttributes(&a, layernorm_kernel<VPL, VEC, ActType::kBf16>)) != cudaSuccess) return e;
    if ((e = cudaFuncGetAttributes(&a, layernorm_kernel<VPL, VEC, ActType::kE4m3>)) != cudaSuccess) return e;
    if ((e = cudaFuncGetAttributes(&a, layernorm_kernel<VPL, VEC, ActType::kE4m3x2>)) != cudaSuccess) return e;
    if ((e = cudaFuncGetAttributes(&a, heads_kernel<VPL, VEC>)) != cudaSuccess) return e;
    if ((e = cudaFuncGetAttributes(&a, value_out_kernel<VPL, VEC>)) != cudaSuccess) return e;
    return cudaFuncGetAttributes(&a, priors_to_half_kernel);
  }
};

}  // namespace

cudaError_t load_row_kernels(int d) { return dispatch_d<LoadKernels>(d); }

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

cudaError_t launch_priors_to_half(const float* in, __half* out, int count, cudaStream_t s) {
  if (count <= 0 || count % 4 != 0) return cudaErrorInvalidValue;
  const int quads = count / 4;
  return launch_kernel(priors_to_half_kernel, dim3((quads + 255) / 256), dim3(256), 0, s, in, out, quads);
}

}  // namespace mrn
