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
#include <stdlib.h>

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

template <int HD, int T, bool E4M3>
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
      constexpr int kOutRow = HD * (E4M3 ? 1 : 2);  // output bytes per row
      constexpr int kChunks = kOutRow / 16;
      const float inv0 = 1.f / l0, inv1 = 1.f / l1;
      uint8_t* so = sq + r0 * RB;  // 16 rows x RB bytes
      auto at = [&](int r, int byte) {
        return so + r * RB + ((((byte >> 4) ^ (r & 7)) & (RB / 16 - 1)) << 4) + (byte & 15);
      };
#pragma unroll
      for (int nt = 0; nt < HD / 8; ++nt) {
        const int col = nt * 8 + 2 * tq;
        if constexpr (E4M3) {
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
          uint8_t* dst = static_cast<uint8_t*>(p.out) +
                         ((static_cast<size_t>(pos) * T + row) * d + head * HD) * (E4M3 ? 1 : 2) + c * 16;
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

// ---- tcgen05 attention (head_dim 64) ---------------------------------------------------
// The same (position, head) items on the fifth-generation tensor cores: per item two MMAs with
// M = 128 (the 65 query rows of the box, the rest ignored), S = Q K^T (N = 80 keys of the box,
// K = 64) into TMEM, then O = P V with P (bf16) written back into TMEM by the softmax warps as
// the MMA's A operand and V read straight from the TMA box as an N-major B operand (N = 64,
// K = 80). The tensor work per item drops from ~780k mma.sync MACs to 1.3M tcgen05 MACs issued
// by one thread, so the kernel is left to the HBM traffic of Q, K, V.
//
// Roles: warp 0 lane 0 TMA producer (Q, K, V boxes into kTcSmemSlots item buffers); warp 1 lane 0
// MMA issuer; warps 2.. in kTcGroups groups of four, one query row per thread (warp w: TMEM lanes
// 32 (w % 4)): group g runs softmax and epilogue of the items k = g mod kTcGroups, each in its own
// TMEM slot of 128 columns (S in [0, 80), then P in [0, 40) and O in [40, 104)). Per item:
// MMA1(k) | softmax(k) | MMA2(k) | epilogue(k); the groups keep kTcGroups items in flight and the
// MMA issuer polls both queues and issues whichever is ready. Every wait is bounded.
constexpr int kTcSmemSlots = 6;
constexpr int kTcGroups = 4;
constexpr int kTcTmemSlots = kTcGroups;  // one per softmax group
constexpr int kTcTmemStride = 128;
constexpr int kTcKeys = kAttnRows;  // N of S = Q K^T, K of O = P V
constexpr int kTcThreads = 32 * (2 + 4 * kTcGroups);

template <bool E4M3>
__global__ void __launch_bounds__(kTcThreads, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap map_qkv, AttentionParams p, int items) {
  constexpr int HD = 64, T = 65;
  constexpr int RB = HD * 2;
  constexpr int MAT = kAttnRows * RB;  // 10 KB: one of Q, K, V
  constexpr int ITEM = 3 * MAT;
  constexpr uint32_t kIdescS = idesc_bf16(128, kTcKeys);
  constexpr uint32_t kIdescO = idesc_bf16_bmn(128, HD);
  constexpr uint32_t kPCol = 0, kOCol = kTcKeys / 2;  // P over S's first 40 columns, O after it
  static_assert(kOCol + HD <= kTcTmemStride && kTcTmemSlots * kTcTmemStride <= 512, "TMEM columns");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kTcSmemSlots * ITEM);  // [kTcSmemSlots]
  uint64_t* sfree = full + kTcSmemSlots;                                      // [kTcSmemSlots]
  uint64_t* s_full = sfree + kTcSmemSlots;                                    // [kTcTmemSlots]
  uint64_t* p_full = s_full + kTcTmemSlots;
  uint64_t* o_full = p_full + kTcTmemSlots;
  uint64_t* t_free = o_full + kTcTmemSlots;
  uint64_t* drain = t_free + kTcTmemSlots;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int d = p.d, heads = p.heads;
  const int G = static_cast<int>(gridDim.x);
  const int mine = (items - static_cast<int>(blockIdx.x) + G - 1) / G;  // this CTA's items
  if (threadIdx.x == 0) {
    for (int i = 0; i < kTcSmemSlots; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&sfree[i], 1);
    }
    for (int i = 0; i < kTcTmemSlots; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_full[i], 1);
      mbar_init(&t_free[i], 4);
    }
    mbar_init(drain, 1);
    *abort = 0;
    fence_barrier_init();
    tma_prefetch_map(&map_qkv);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 512);
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
      // ---- producer
      uint32_t issued = 0, parities = 0;
      for (int k = 0; k < mine && !*abort; ++k) {
        const int item = static_cast<int>(blockIdx.x) + k * G;
        const int sl = k % kTcSmemSlots;
        const uint32_t par = (k / kTcSmemSlots) & 1;
        if (!mbar_wait(&sfree[sl], par ^ 1u, abort)) {
          raise_error(p.status, abort, kErrTimeoutAttention);
          break;
        }
        const int pos = item / heads, head = item - pos * heads;
        uint8_t* dst = smem + sl * ITEM;
        mbar_arrive_expect_tx(&full[sl], ITEM);
        tma_load_2d(dst, &map_qkv, &full[sl], head * HD, pos * T);
        tma_load_2d(dst + MAT, &map_qkv, &full[sl], d + head * HD, pos * T);
        tma_load_2d(dst + 2 * MAT, &map_qkv, &full[sl], 2 * d + head * HD, pos * T);
        issued |= 1u << sl;
        parities = (parities & ~(1u << sl)) | (par << sl);
      }
      if (*abort) {
        for (int sl = 0; sl < kTcSmemSlots; ++sl)
          if (issued & (1u << sl)) mbar_wait_bounded(&full[sl], (parities >> sl) & 1u);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer, event-driven: MMA1 of the next item as soon as its Q/K/V have landed and
      // its TMEM slot is free (at most kTcGroups items ahead), MMA2 of the oldest item as soon
      // as its P is in TMEM; both in item order.
      bool issued = false;
      int n1 = 0, n2 = 0;
      unsigned long long idle_since = 0;
      uint32_t spins = 0;
      while (n2 < mine) {
        bool progress = false;
        if (n1 < mine && n1 - n2 < kTcGroups) {
          const int t = n1 % kTcTmemSlots, sl = n1 % kTcSmemSlots;
          if (mbar_test(smem_u32(&full[sl]), (n1 / kTcSmemSlots) & 1u) &&
              mbar_test(smem_u32(&t_free[t]), ((n1 / kTcTmemSlots) & 1u) ^ 1u)) {
            tc_fence_after();
            const uint32_t q = smem_u32(smem + sl * ITEM), kb = q + MAT;
            // Q rows 80..127 run into the K box: garbage query rows, never read back.
#pragma unroll
            for (int kk = 0; kk < HD / 16; ++kk)
              mma_bf16(tmem + static_cast<uint32_t>(t * kTcTmemStride), desc_sw128(q + 32u * kk),
                       desc_sw128(kb + 32u * kk), kIdescS, kk != 0);
            issued = true;
            tc_commit(&s_full[t]);
            ++n1;
            progress = true;
          }
        }
        if (n2 < n1) {
          const int t = n2 % kTcTmemSlots, sl = n2 % kTcSmemSlots;
          if (mbar_test(smem_u32(&p_full[t]), (n2 / kTcTmemSlots) & 1u)) {
            tc_fence_after();
            const uint32_t base = tmem + static_cast<uint32_t>(t * kTcTmemStride);
            const uint32_t v = smem_u32(smem + sl * ITEM + 2 * MAT);
#pragma unroll
            for (int kk = 0; kk < kTcKeys / 16; ++kk)  // 16 keys = 8 P columns = 16 V rows (2048 B)
              mma_bf16_tmem_a(base + kOCol, base + kPCol + 8u * kk, desc_sw128(v + 2048u * kk), kIdescO, kk != 0);
            tc_commit(&o_full[t]);
            tc_commit(&sfree[sl]);
            ++n2;
            progress = true;
          }
        }
        if (progress) {
          spins = 0;
        } else if ((++spins & 31u) == 0) {
          const unsigned long long now = globaltimer();
          if (idle_since == 0) idle_since = now;
          if (*abort || now - idle_since > kWaitLimitNs) {
            raise_error(p.status, abort, kErrTimeoutAttention);
            break;
          }
        }
        if (progress) idle_since = 0;
      }
      if (*abort && issued) {
        tc_commit(drain);
        if (!mbar_wait_bounded(drain, 0) && p.status) atomicCAS(p.status, 0, kErrTimeoutDrain);
      }
    }
  } else {
    // ---- softmax + epilogue: one query row per thread, group g takes items g, g + kTcGroups, ...
    const int group = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const bool valid = row < T;
    const uint32_t lanes = static_cast<uint32_t>(quarter * 32) << 16;
    const float scale_log2 = 0.125f * 1.4426950408889634f;  // 1/sqrt(64) in base 2
    for (int k = group; k < mine; k += kTcGroups) {
      const int t = k % kTcTmemSlots;
      const uint32_t par = (k / kTcTmemSlots) & 1u;
      const uint32_t base = tmem + lanes + static_cast<uint32_t>(t * kTcTmemStride);
      if (!mbar_wait(&s_full[t], par, abort)) {
        if (lane == 0) raise_error(p.status, abort, kErrTimeoutAttention);
        break;
      }
      tc_fence_after();
      if (quarter == 3) {
        // Query rows 96..127 do not exist: keep in step with the group's barriers, nothing else
        // (MMA2 multiplies whatever these TMEM lanes hold into output rows that are never read).
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[t]);
        if (!mbar_wait(&o_full[t], par, abort)) {
          if (lane == 0) raise_error(p.status, abort, kErrTimeoutAttention);
          break;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&t_free[t]);
        continue;
      }
      float sv[80];
      tmem_ld32(base, *reinterpret_cast<float(*)[32]>(sv));
      tmem_ld32(base + 32, *reinterpret_cast<float(*)[32]>(sv + 32));
      tmem_ld16(base + 64, *reinterpret_cast<float(*)[16]>(sv + 64));
      // Softmax over keys 0..64 (keys 65..79 of the box belong to the next position: P = 0).
      float m = sv[0];
#pragma unroll
      for (int j = 1; j < T; ++j) m = fmaxf(m, sv[j]);
      const float bm = -m * scale_log2;
      float l = 0.f;
      uint32_t pk[40];
#pragma unroll
      for (int j = 0; j < 40; ++j) {
        const float e0 = 2 * j < T ? ex2f(fmaf(sv[2 * j], scale_log2, bm)) : 0.f;
        const float e1 = 2 * j + 1 < T ? ex2f(fmaf(sv[2 * j + 1], scale_log2, bm)) : 0.f;
        l += e0 + e1;
        pk[j] = valid ? pack_bf16(e0, e1) : 0u;
      }
#pragma unroll
      for (int j = 0; j < 40; j += 8) tmem_st8(base + kPCol + j, *reinterpret_cast<const uint32_t(*)[8]>(pk + j));
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[t]);

      // epilogue: O row * (1 / l), quantised, 64 contiguous output bytes per row
      if (!mbar_wait(&o_full[t], par, abort)) {
        if (lane == 0) raise_error(p.status, abort, kErrTimeoutAttention);
        break;
      }
      tc_fence_after();
      float o[64];
      tmem_ld32(base + kOCol, *reinterpret_cast<float(*)[32]>(o));
      tmem_ld32(base + kOCol + 32, *reinterpret_cast<float(*)[32]>(o + 32));
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&t_free[t]);
      if (valid) {
        const int item = static_cast<int>(blockIdx.x) + k * G;
        const int pos = item / heads, head = item - pos * heads;
        const float f = (E4M3 ? p.inv_q : 1.f) / l;
        uint8_t* dst = static_cast<uint8_t*>(p.out) +
                       ((static_cast<size_t>(pos) * T + row) * d + head * HD) * (E4M3 ? 1 : 2);
        if constexpr (E4M3) {
#pragma unroll
          for (int c = 0; c < 64; c += 16) {
            __nv_fp8x2_storage_t q8[8];
#pragma unroll
            for (int e = 0; e < 8; ++e)
              q8[e] = __nv_cvt_float2_to_fp8x2(make_float2(o[c + 2 * e] * f, o[c + 2 * e + 1] * f), __NV_SATFINITE,
                                               __NV_E4M3);
            *reinterpret_cast<uint4*>(dst + c) = *reinterpret_cast<const uint4*>(q8);
          }
        } else {
#pragma unroll
          for (int c = 0; c < 64; c += 8) {
            uint32_t b[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) b[e] = pack_bf16(o[c + 2 * e] * f, o[c + 2 * e + 1] * f);
            *reinterpret_cast<uint4*>(dst + 2 * c) = make_uint4(b[0], b[1], b[2], b[3]);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

constexpr int attention_tc_smem() {
  return 1024 + kTcSmemSlots * 3 * kAttnRows * 128 + (2 * kTcSmemSlots + 4 * kTcTmemSlots + 1) * 8 + 16;
}

// The tcgen05 kernel is opt-in (MRN_ATTN_TC=1): correct, but about 5% slower than the mma.sync
// kernel at batch 4096 (211 against 200 us per launch); its nine small MMAs per item are bound by
// per-instruction cost rather than by tensor throughput.
bool attention_tc_enabled() {
  static const bool on = [] {
    const char* e = getenv("MRN_ATTN_TC");
    return e && e[0] == '1';
  }();
  return on;
}

template <int HD, int T>
constexpr int attention_smem() {
  return 1024 + kTeams * kBufs * 3 * kAttnRows * HD * 2 + 2 * kTeams * kBufs * 8 + 16;
}

template <int HD, int T>
cudaError_t launch_attention_t(const AttentionParams& p, const CUtensorMap& map, int grid, int items, cudaStream_t s) {
  constexpr int smem = attention_smem<HD, T>();
  if (p.out_type == ActType::kE4m3)
    return launch_kernel(attention_kernel<HD, T, true>, dim3(grid), dim3(kAttnThreads), smem, s, map, p, items);
  return launch_kernel(attention_kernel<HD, T, false>, dim3(grid), dim3(kAttnThreads), smem, s, map, p, items);
}

template <int HD, int T>
cudaError_t prepare_attention_t() {
  constexpr int smem = attention_smem<HD, T>();
  cudaError_t e = cudaFuncSetAttribute(attention_kernel<HD, T, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(attention_kernel<HD, T, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
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
  if (head_dim == 64 && attention_tc_enabled()) {
    if (p.out_type == ActType::kE4m3)
      return launch_kernel(attention_tc_kernel<true>, dim3(grid), dim3(kTcThreads), attention_tc_smem(), s, map, p,
                           items);
    return launch_kernel(attention_tc_kernel<false>, dim3(grid), dim3(kTcThreads), attention_tc_smem(), s, map, p,
                         items);
  }
  if (head_dim == 64) return launch_attention_t<64, 65>(p, map, grid, items, s);
  return launch_attention_t<32, 65>(p, map, grid, items, s);
}

cudaError_t prepare_attention() {
  cudaError_t e = prepare_attention_t<64, 65>();
  if (e != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(attention_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                attention_tc_smem())) != cudaSuccess)
    return e;
  if ((e = cudaFuncSetAttribute(attention_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                attention_tc_smem())) != cudaSuccess)
    return e;
  return prepare_attention_t<32, 65>();
}

}  // namespace mrn
