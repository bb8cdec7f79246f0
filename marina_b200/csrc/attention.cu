// Self-attention of the encoder, one work item per (position, head): softmax(Q K^T / sqrt(hd)) V
// over the position's T = 65 tokens (src/net/cpu.rs:99-125 in the reference; its CUDA kernel
// attention_impl, src/net/cuda/kernels.cu:201-342, computes the same with WMMA).
//
// Layout: qkv is bf16 [R, 3d] (Q | K | V, head h at columns h*hd), out is bf16 or e4m3 [R, d].
//
// Persistent CTAs of 1 producer warp and kTeams teams of 5 consumer warps. CTA b takes items
// b, b + G, b + 2G, ... (G CTAs); its k-th item goes to team k % kTeams. The producer streams
// each item's Q, K and V with three TMA box loads (80 rows x one head's columns, 128- or 64-byte
// swizzled) into the team's next buffer (two per team) and signals a `full` mbarrier; the five
// warps of the team take 16 query rows each and arrive on the buffer's `empty` mbarrier when
// done. Teams never wait on one another, and nothing waits on the whole CTA.
//
// The 80-row boxes start at the position's first token; rows 65..79 belong to the next position
// (or lie past the last row, read as zeros): their keys are masked out of the softmax, their
// values meet probability 0, and their query rows are not stored.
//
// Per warp (query rows r0..r0+15): S = Q K^T with mma.sync m16n8k16 (f32 accumulation), the
// softmax on the accumulators with quad shuffles (ex2 with the 1/sqrt(hd) scale folded into the
// exponent), O = P V with P straight from the accumulators, then the normalised strip is
// written into the warp's own (dead) Q rows and stored with 16-byte writes. Every mbarrier wait
// is bounded (kWaitLimitNs); a wait that gives up records an error code and the kernel unwinds.
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include "e4m3x2.cuh"
#include "kernels.cuh"
#include "launch.h"
#include "ptx.cuh"
#include "tmap.h"

namespace mrn {

namespace {

constexpr int kAttnRows = 80;  // rows of a box: T = 65 rounded up to 16-row MMA strips
constexpr int kTeamWarps = kAttnRows / 16;
constexpr int kTeams = 3;
constexpr int kBufs = 2;  // buffers per team
constexpr int kAttnThreads = 32 * (1 + kTeams * kTeamWarps);
constexpr int kErrTimeoutAttention = 6;

__device__ __forceinline__ void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t (&r)[2], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float ex2f(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// Byte offset of 16-byte chunk `c` of row `r` in a TMA box with RB-byte rows and the matching
// swizzle (128 B: chunk ^ (row & 7); 64 B: chunk ^ ((row >> 1) & 3)).
template <int RB>
__device__ __forceinline__ uint32_t swz(int r, int c) {
  if constexpr (RB == 128) return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4));
  return static_cast<uint32_t>(r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
}

template <int HD, int T, int OUT>  // OUT: 0 bf16, 1 e4m3, 2 two-term e4m3 (hi | lo rows)
__global__ void __launch_bounds__(kAttnThreads, 1)
    attention_kernel(const __grid_constant__ CUtensorMap map_qkv, AttentionParams p, int items) {
  constexpr int RB = HD * 2;                  // bytes per staged row
  constexpr int MAT = kAttnRows * RB;         // one of Q, K, V
  constexpr int ITEM = 3 * MAT;
  constexpr int NT = (T + 7) / 8;             // key tiles of 8 holding at least one valid key
  constexpr int KS = (T + 15) / 16;           // k16 steps of P V
  static_assert(T <= kAttnRows && 2 * KS <= 10, "tokens per position");
  static_assert(MAT % 1024 == 0, "swizzle atoms");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kTeams * kBufs * ITEM);  // [team][buf]
  uint64_t* empty = full + kTeams * kBufs;                                      // [team][buf]
  volatile int* abort = reinterpret_cast<volatile int*>(empty + kTeams * kBufs);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int d = p.d, heads = p.heads;
  const int G = static_cast<int>(gridDim.x);
  if (threadIdx.x == 0) {
    for (int i = 0; i < kTeams * kBufs; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kTeamWarps);
    }
    *abort = 0;
    fence_barrier_init();
    tma_prefetch_map(&map_qkv);
  }
  __syncthreads();
  grid_dep_wait();
  grid_dep_launch();

  if (warp == 0) {
    if (lane == 0) {
      // ---- producer: Q, K, V of every item of this CTA, in order
      uint32_t issued = 0, parities = 0;  // per buffer: a load is in flight / its phase parity
      for (int k = 0; static_cast<int>(blockIdx.x) + k * G < items && !*abort; ++k) {
        const int item = static_cast<int>(blockIdx.x) + k * G;
        const int team = k % kTeams, j = k / kTeams, buf = j % kBufs, slot = team * kBufs + buf;
        const uint32_t par = (j / kBufs) & 1;
        if (!mbar_wait(&empty[slot], par ^ 1u, abort)) {
          raise_error(p.status, abort, kErrTimeoutAttention);
          break;
        }
        const int pos = item / heads, head = item - pos * heads;
        uint8_t* dst = smem + slot * ITEM;
        mbar_arrive_expect_tx(&full[slot], ITEM);
        tma_load_2d(dst, &map_qkv, &full[slot], head * HD, pos * T);
        tma_load_2d(dst + MAT, &map_qkv, &full[slot], d + head * HD, pos * T);
        tma_load_2d(dst + 2 * MAT, &map_qkv, &full[slot], 2 * d + head * HD, pos * T);
        issued |= 1u << slot;
        parities = (parities & ~(1u << slot)) | (par << slot);
      }
      if (*abort) {
        // Let the copies still in flight land before the CTA's shared memory goes away.
        for (int s = 0; s < kTeams * kBufs; ++s)
          if (issued & (1u << s)) mbar_wait_bounded(&full[s], (parities >> s) & 1u);
      }
    }
  } else {
    // ---- consumers
    const int team = (warp - 1) / kTeamWarps;
    const int r0 = ((warp - 1) % kTeamWarps) * 16;
    const int g = lane >> 2, tq = lane & 3;
    const int lm = lane >> 3, lr = lane & 7;  // ldmatrix: lane supplies row lr of matrix lm
    const float scale_log2 = rsqrtf(static_cast<float>(HD)) * 1.4426950408889634f;
    for (int k = team; static_cast<int>(blockIdx.x) + k * G < items; k += kTeams) {
      const int item = static_cast<int>(blockIdx.x) + k * G;
      const int j = k / kTeams, buf = j % kBufs, slot = team * kBufs + buf;
      if (!mbar_wait(&full[slot], (j / kBufs) & 1, abort)) {
        if (lane == 0) raise_error(p.status, abort, kErrTimeoutAttention);
        break;
      }
      __syncwarp();  // ldmatrix / mma.sync below are .aligned: the whole warp, reconverged
      uint8_t* sq = smem + slot * ITEM;
      const uint32_t aq = smem_u32(sq), ak = aq + MAT, av = aq + 2 * MAT;
      const int pos = item / heads, head = item - pos * heads;

      // S = Q K^T for rows r0..r0+15 against the key tiles holding valid keys.
      float s[2 * KS][4];
#pragma unroll
      for (int nt = 0; nt < 2 * KS; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < HD; kk += 16) {
        uint32_t a[4];  // matrices (rows r0.., k kk), (r0+8.., kk), (r0.., kk+8), (r0+8.., kk+8)
        ldsm_x4(a, aq + swz<RB>(r0 + (lm & 1) * 8 + lr, kk / 8 + (lm >> 1)));
#pragma unroll
        for (int nt = 0; nt + 1 < NT; nt += 2) {
          uint32_t b[4];  // (keys nt*8.., k kk), (nt*8.., kk+8), (nt*8+8.., kk), (nt*8+8.., kk+8)
          ldsm_x4(b, ak + swz<RB>(nt * 8 + (lm >> 1) * 8 + lr, kk / 8 + (lm & 1)));
          mma_16816(s[nt], a, b[0], b[1]);
          mma_16816(s[nt + 1], a, b[2], b[3]);
        }
        if constexpr (NT % 2 == 1) {
          uint32_t b[2];
          ldsm_x2(b, ak + swz<RB>((NT - 1) * 8 + lr, kk / 8 + (lm & 1)));
          mma_16816(s[NT - 1], a, b[0], b[1]);
        }
      }
      // Softmax of rows g (values 0,1) and g+8 (values 2,3); keys >= T are masked.
      float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e)
          if (nt * 8 + 7 < T || nt * 8 + 2 * tq + e < T) {
            m0 = fmaxf(m0, s[nt][e]);
            m1 = fmaxf(m1, s[nt][2 + e]);
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
        for (int e = 0; e < 2; ++e) {
          if (nt >= NT) {
            s[nt][e] = s[nt][2 + e] = 0.f;
          } else if (nt * 8 + 7 < T || nt * 8 + 2 * tq + e < T) {
            s[nt][e] = ex2f(fmaf(s[nt][e], scale_log2, b0));
            s[nt][2 + e] = ex2f(fmaf(s[nt][2 + e], scale_log2, b1));
          } else {
            s[nt][e] = s[nt][2 + e] = 0.f;
          }
          l0 += s[nt][e];
          l1 += s[nt][2 + e];
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
        const int key = kk * 16 + lr + (lm & 1) * 8;
#pragma unroll
        for (int nt = 0; nt < HD / 8; nt += 2) {
          uint32_t b[4];
          ldsm_x4_trans(b, av + swz<RB>(key, nt + (lm >> 1)));
          mma_16816(o[nt], a, b[0], b[1]);
          mma_16816(o[nt + 1], a, b[2], b[3]);
        }
      }

      // Normalised strip -> this warp's Q rows (no longer read; own XOR layout: chunk ^ row)
      // -> 16-byte global stores of the rows < T.
      constexpr int kOutRow = HD * (OUT == 1 ? 1 : 2);  // output bytes per row (x2: HD hi, then HD lo)
      constexpr int kChunks = kOutRow / 16;
      const float inv0 = 1.f / l0, inv1 = 1.f / l1;
      uint8_t* so = sq + r0 * RB;  // 16 rows x RB bytes
      auto at = [&](int r, int byte) {
        return so + r * RB + ((((byte >> 4) ^ (r & 7)) & (RB / 16 - 1)) << 4) + (byte & 15);
      };
#pragma unroll
      for (int nt = 0; nt < HD / 8; ++nt) {
        const int col = nt * 8 + 2 * tq;
        if constexpr (OUT == 2) {
          uint16_t hi, lo;
          split_e4m3x2(make_float2(o[nt][0] * inv0 * p.inv_q, o[nt][1] * inv0 * p.inv_q), hi, lo);
          *reinterpret_cast<uint16_t*>(at(g, col)) = hi;
          *reinterpret_cast<uint16_t*>(at(g, HD + col)) = lo;
          split_e4m3x2(make_float2(o[nt][2] * inv1 * p.inv_q, o[nt][3] * inv1 * p.inv_q), hi, lo);
          *reinterpret_cast<uint16_t*>(at(g + 8, col)) = hi;
          *reinterpret_cast<uint16_t*>(at(g + 8, HD + col)) = lo;
        } else if constexpr (OUT == 1) {
          *reinterpret_cast<__nv_fp8x2_storage_t*>(at(g, col)) = __nv_cvt_float2_to_fp8x2(
              make_float2(o[nt][0] * inv0 * p.inv_q, o[nt][1] * inv0 * p.inv_q), __NV_SATFINITE, __NV_E4M3);
          *reinterpret_cast<__nv_fp8x2_storage_t*>(at(g + 8, col)) = __nv_cvt_float2_to_fp8x2(
              make_float2(o[nt][2] * inv1 * p.inv_q, o[nt][3] * inv1 * p.inv_q), __NV_SATFINITE, __NV_E4M3);
        } else {
          *reinterpret_cast<__nv_bfloat162*>(at(g, 2 * col)) = __floats2bfloat162_rn(o[nt][0] * inv0, o[nt][1] * inv0);
          *reinterpret_cast<__nv_bfloat162*>(at(g + 8, 2 * col)) =
              __floats2bfloat162_rn(o[nt][2] * inv1, o[nt][3] * inv1);
        }
      }
      __syncwarp();
#pragma unroll
      for (int i = lane; i < 16 * kChunks; i += 32) {
        const int rr = i / kChunks, c = i - rr * kChunks;
        const int row = r0 + rr;
        if (row < T) {
          const uint4 v = *reinterpret_cast<const uint4*>(at(rr, c * 16));
          const size_t grow = static_cast<size_t>(pos) * T + row;
          uint8_t* dst;
          if constexpr (OUT == 2)  // hi chunks to the head's columns, lo chunks d bytes further on
            dst = static_cast<uint8_t*>(p.out) + grow * 2 * d + head * HD + (c * 16 < HD ? c * 16 : d + c * 16 - HD);
          else
            dst = static_cast<uint8_t*>(p.out) + (grow * d + head * HD) * (OUT == 1 ? 1 : 2) + c * 16;
          *reinterpret_cast<uint4*>(dst) = v;
        }
      }
      // This warp is done with the buffer.
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }
  }
  __syncthreads();
}

template <int HD, int T>
constexpr int attention_smem() {
  return 1024 + kTeams * kBufs * 3 * kAttnRows * HD * 2 + 2 * kTeams * kBufs * 8 + 16;
}

template <int HD, int T>
cudaError_t launch_attention_t(const AttentionParams& p, const CUtensorMap& map, int grid, int items, cudaStream_t s) {
  constexpr int smem = attention_smem<HD, T>();
  if (p.out_type == ActType::kE4m3)
    return launch_kernel(attention_kernel<HD, T, 1>, dim3(grid), dim3(kAttnThreads), smem, s, map, p, items);
  if (p.out_type == ActType::kE4m3x2)
    return launch_kernel(attention_kernel<HD, T, 2>, dim3(grid), dim3(kAttnThreads), smem, s, map, p, items);
  return launch_kernel(attention_kernel<HD, T, 0>, dim3(grid), dim3(kAttnThreads), smem, s, map, p, items);
}

template <int HD, int T>
cudaError_t prepare_attention_t() {
  constexpr int smem = attention_smem<HD, T>();
  cudaError_t e = cudaFuncSetAttribute(attention_kernel<HD, T, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(attention_kernel<HD, T, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) !=
      cudaSuccess)
    return e;
  return cudaFuncSetAttribute(attention_kernel<HD, T, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
}

// The qkv tensor as TMA sees it: [rows, 3d] bf16, boxes of 80 rows x head_dim columns with the
// swizzle of a head_dim * 2-byte row.
bool make_qkv_map(CUtensorMap* map, const void* qkv, int rows, int d, int head_dim) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn || (reinterpret_cast<uintptr_t>(qkv) & 15) != 0) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(3 * d), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(3 * d) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(head_dim), kAttnRows};
  const cuuint32_t estrides[2] = {1, 1};
  const CUtensorMapSwizzle sw = head_dim == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(qkv), dims, strides, box, estrides,
            CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

// Board mode has 65 tokens (one state token, 64 squares; src/net/model.rs:17).
cudaError_t launch_attention(const AttentionParams& p, int positions, int head_dim, cudaStream_t s) {
  if (p.t != 65 || (head_dim != 64 && head_dim != 32)) return cudaErrorInvalidValue;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  CUtensorMap map;
  if (!make_qkv_map(&map, p.qkv, positions * p.t, p.d, head_dim)) return cudaErrorInvalidValue;
  const int items = positions * p.heads;
  const int grid = items < sms ? items : sms;
  if (head_dim == 64) return launch_attention_t<64, 65>(p, map, grid, items, s);
  return launch_attention_t<32, 65>(p, map, grid, items, s);
}

cudaError_t prepare_attention() {
  cudaError_t e = prepare_attention_t<64, 65>();
  if (e != cudaSuccess) return e;
  return prepare_attention_t<32, 65>();
}

}  // namespace mrn
