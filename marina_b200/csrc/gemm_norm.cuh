// The CTA-pair GEMM of gemm.cuh with the LayerNorm that feeds it folded into the kernel:
//
//     D[M, N] = e4m3(LN(x) * gamma + beta) · B[N, K]^T,        x = the f16 residual stream [M, K]
//
// (QKV after norm1, FFN1 after norm2: the pre-LN block of src/net/cpu.rs:113-160). The
// normalised, quantised A never goes to global memory: each CTA of a pair normalises its
// 128 rows of the current 256-row block straight into shared memory, in the 128-byte swizzled
// K-major layout a TMA load would have produced, and keeps it there while the pair walks the
// block's N tiles. The LayerNorm kernel's launch, its h write and the GEMM's h read are gone;
// the price is reading x as f16 (2 bytes per element instead of 1).
//
// Roles (64 + 32 x (epilogue + norm warps) threads per CTA):
//   warp 0, one lane : TMA producer of B only (this CTA's 128 rows of the pair's 256-column tile).
//   warp 1, one lane : MMA issuer on the leader: M = 256, N = 256, K = 32 tcgen05.mma over both
//                      CTAs' shared memory (cta_group::2), A from the resident block.
//   epilogue warps   : as gemm_pair_kernel (at most 12).
//   norm warps       : LayerNorm of this CTA's rows of the next block into the other A buffer
//                      (two buffers: a block is normalised while the MMAs read the previous one),
//                      one warp per row with three rows of x in flight; the arithmetic is
//                      rows.cuh's, the same the LayerNorm kernel runs, so A is bit-identical.
//
// Work split: the (256-row block, 256-column tile) units in n-fastest order are cut into one
// contiguous range per pair, so a pair normalises each block it touches once and the ranges
// differ in length by at most one unit.
//
// Barriers (leader's copy used unless stated): full/empty/tmem_full/tmem_empty as
// gemm_pair_kernel; a_full[b] counts the norm warps of both CTAs (the peer's arrive remotely,
// after a proxy fence that makes their generic stores visible to the tensor core's reads);
// a_empty[b] (each CTA's own) is committed by the MMA issuer, multicast, once the last MMA
// reading buffer b has completed. Every wait is bounded.
#pragma once

#include "gemm.cuh"
#include "rows.cuh"

namespace mrn {

// The normalised A operand: x rows [M, K] (f16), per-column gamma/beta, and the e4m3 scale.
struct NormA {
  const __half* x;
  const float* gamma;
  const float* beta;
  float eps;
  float inv_q;  // 1 / e4m3 scale of the normalised rows
};

constexpr int kNormK = 512;  // K (= d) of the instantiated kernel: 16 values per lane

// Epilogue warps: the epilogue's own count, at most 12 (the GELU epilogue's 16 would leave the
// norm warps too few registers).
template <int OUT_BYTES, int EPI_WARPS>
struct NormShape {
  static constexpr int kBN = 256;
  static constexpr int kBHalf = 128;
  static constexpr int kEpiWarps = EPI_WARPS > 12 ? 12 : EPI_WARPS;
  static constexpr int kNormWarps = 8;
  static constexpr int kChunkBytes = kTileM * kStageRowBytes;       // 128 rows x 128 K bytes
  static constexpr int kABytes = (kNormK / kStageRowBytes) * kChunkBytes;
  static constexpr int kBBytes = kBHalf * kStageRowBytes;
  static constexpr int kEpiBufBytes = 32 * kEpiChunk * OUT_BYTES;
  static constexpr int kEpiBuffers = 2;
  static constexpr int kEpiBytes = kEpiBuffers * kEpiWarps * kEpiBufBytes;
  static constexpr int kGbBytes = 2 * kNormK * 4;
  static constexpr int kBarrierBytes = 256;
  static constexpr int kFit = (kMaxSmem - 1024 - kBarrierBytes - 2 * kABytes - kEpiBytes - kGbBytes) / kBBytes;
  static constexpr int kStages = kFit > 6 ? 6 : kFit;
  static_assert(kStages >= 2, "not enough shared memory for a 2-stage B ring");
  static constexpr int kSmemBytes = 1024 + 2 * kABytes + kStages * kBBytes + kEpiBytes + kGbBytes + kBarrierBytes;
  static constexpr int kThreads = 64 + 32 * (kEpiWarps + kNormWarps);
};

template <class Epi>
__global__ void __cluster_dims__(2, 1, 1)
    __launch_bounds__(NormShape<Epi::kOutBytes, Epi::kWarps>::kThreads, 1)
        gemm_norm_kernel(const __grid_constant__ CUtensorMap map_b, const __grid_constant__ CUtensorMap map_out,
                         Epi epi, NormA na, int M, int N, int* status) {
  using S = NormShape<Epi::kOutBytes, Epi::kWarps>;
  constexpr int BN = S::kBN;
  constexpr int kStages = S::kStages;
  constexpr int kEpiWarps = S::kEpiWarps;
  constexpr int kNormWarps = S::kNormWarps;
  constexpr int kEpiBufBytes = S::kEpiBufBytes;
  constexpr int kKBlocks = kNormK / kStageRowBytes;
  constexpr uint32_t kIdesc = idesc_e4m3(2 * kTileM, BN);
  constexpr int kRowBytes = kEpiChunk * Epi::kOutBytes;
  constexpr int kVpl = kNormK / 32;
  constexpr int kRowsPerWarp = kTileM / kNormWarps;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sm_a = smem;                         // [2] normalised blocks, 1024-aligned
  uint8_t* sm_b = smem + 2 * S::kABytes;        // [kStages] B ring
  uint8_t* sm_epi = sm_b + kStages * S::kBBytes;
  float* gb = reinterpret_cast<float*>(sm_epi + S::kEpiBytes);  // gamma [kNormK], beta [kNormK], x inv_q
  uint64_t* bars = reinterpret_cast<uint64_t*>(gb + 2 * kNormK);
  uint64_t* full = bars;                     // [kStages] both CTAs' B bytes -> leader's MMA
  uint64_t* empty = bars + kStages;          // [kStages] MMA -> each CTA's producer
  uint64_t* tmem_full = bars + 2 * kStages;  // [2] MMA -> each CTA's epilogue
  uint64_t* tmem_empty = tmem_full + 2;      // [2] both CTAs' epilogues -> MMA
  uint64_t* a_full = tmem_empty + 2;         // [2] both CTAs' norm warps -> MMA
  uint64_t* a_empty = a_full + 2;            // [2] MMA -> each CTA's norm warps
  uint64_t* drain = a_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1;
  const int pairs = gridDim.x >> 1;
  const int n_tiles = N / BN;
  const long long units = static_cast<long long>((M + 2 * kTileM - 1) / (2 * kTileM)) * n_tiles;
  const int begin = static_cast<int>(units * pair / pairs);
  const int end = static_cast<int>(units * (pair + 1) / pairs);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], 2 * kEpiWarps);
      mbar_init(&a_full[a], 2 * kNormWarps);
      mbar_init(&a_empty[a], 1);
    }
    mbar_init(drain, 1);
    *abort = 0;
    fence_barrier_init();
    tma_prefetch_map(&map_b);
    tma_prefetch_map(&map_out);
  }
  // The LayerNorm kernel's gamma/beta times the output's 1/scale, rounded the same way.
  for (int i = threadIdx.x; i < kNormK; i += blockDim.x) {
    gb[i] = na.gamma[i] * na.inv_q;
    gb[kNormK + i] = na.beta[i] * na.inv_q;
  }
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
      // ---- TMA producer (both CTAs): this CTA's half of B; bytes counted on the leader
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, parity_mask = 0;
      for (int u = begin; u < end && !*abort; ++u) {
        const int nb = (u % n_tiles) * BN + static_cast<int>(rank) * S::kBHalf;
        for (int kb = 0; kb < kKBlocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort)) {
            raise_error(status, abort, kErrTimeoutProducer);
            break;
          }
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * S::kBBytes);
          const uint32_t bar = map_to_rank(smem_u32(&full[stage]), 0);
          tma_load_2d_pair(sm_b + stage * S::kBBytes, &map_b, bar, kb * kStageRowBytes, nb);
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
      int blk = -1;
      int abuf = 0;
      bool issued = false;
      for (int u = begin; u < end; ++u) {
        if (u == begin || u % n_tiles == 0) {
          ++blk;
          abuf = blk & 1;
          if (!mbar_wait_cluster(&a_full[abuf], (blk >> 1) & 1u, abort)) {
            raise_error(status, abort, kErrTimeoutMma);
            break;
          }
        }
        if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1u, abort)) {
          raise_error(status, abort, kErrTimeoutMma);
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(acc * BN);
        const uint32_t a_base = smem_u32(sm_a + abuf * S::kABytes);
        bool ok = true;
        for (int kb = 0; kb < kKBlocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort)) {
            raise_error(status, abort, kErrTimeoutMma);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = a_base + static_cast<uint32_t>(kb * S::kChunkBytes);
          const uint32_t b_addr = smem_u32(sm_b + stage * S::kBBytes);
#pragma unroll
          for (int k = 0; k < kStageRowBytes / 32; ++k)
            mma_pair_e4m3(d, desc_sw128(a_addr + 32u * k), desc_sw128(b_addr + 32u * k), kIdesc, (kb | k) != 0);
          issued = true;
          tc_commit_pair(&empty[stage], 0x3);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit_pair(&tmem_full[acc], 0x3);
        // The block's last tile: its A buffer is free once these MMAs complete.
        if (u + 1 == end || (u + 1) % n_tiles == 0) tc_commit_pair(&a_empty[abuf], 0x3);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      if (*abort && issued) {
        tc_commit_pair(drain, 0x1);
        if (!mbar_wait_bounded(drain, 0) && status) atomicCAS(status, 0, kErrTimeoutDrain);
      }
    }
  } else if (warp < 2 + kEpiWarps) {
    // ---- epilogue (both CTAs): this CTA's 128 rows x 256 columns
    constexpr int kParts = kEpiWarps / 4;
    const int quarter = warp & 3;
    const int part = (warp - 2) >> 2;
    uint8_t* const sb0 = sm_epi + (warp - 2) * S::kEpiBuffers * kEpiBufBytes;
    int buf = 0;
    const uint32_t empty_addr0 = map_to_rank(smem_u32(&tmem_empty[0]), 0);
    const uint32_t empty_addr1 = map_to_rank(smem_u32(&tmem_empty[1]), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int u = begin; u < end; ++u) {
      const int m0 = (u / n_tiles) * 2 * kTileM + static_cast<int>(rank) * kTileM;
      const int n0 = (u % n_tiles) * BN;
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
        buf ^= 1;
        if (lane == 0) bulk_wait_read<S::kEpiBuffers - 1>();
        __syncwarp();
#pragma unroll
        for (int j = 0; j < Epi::kOutBytes * 2; ++j)
          *reinterpret_cast<uint4*>(sb + staged_offset<kRowBytes>(lane, j)) = out[j];
        fence_async_shared();
        __syncwarp();
        if (lane == 0) {
          if (row0 < M) tma_store_2d(&map_out, sb, n0 + c, row0);
          bulk_commit();
        }
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  } else if (begin < end) {
    // ---- norm warps (both CTAs): row r = nw + kNormWarps * j of this CTA's half of each block
    const int nw = warp - 2 - kEpiWarps;
    const int mb0 = begin / n_tiles;
    const int total = ((end - 1) / n_tiles - mb0 + 1) * kRowsPerWarp;
    using Row = WarpRow<kVpl, 4>;
    using Raw = RawRow<kVpl, 4>;
    auto row_of = [&](int q) {
      return (mb0 + q / kRowsPerWarp) * 2 * kTileM + static_cast<int>(rank) * kTileM + nw + kNormWarps * (q % kRowsPerWarp);
    };
    auto fetch = [&](Raw& r, int q) {
      if (q < total) {
        const int row = row_of(q);
        if (row < M) r.load(na.x + static_cast<size_t>(row) * kNormK, lane);
      }
    };
    Raw r0, r1, r2;
    fetch(r0, 0);
    fetch(r1, 1);
    fetch(r2, 2);
    for (int q = 0; q < total; ++q) {
      const int i = q / kRowsPerWarp;
      const int j = q % kRowsPerWarp;
      const int abuf = i & 1;
      if (j == 0 && !mbar_wait(&a_empty[abuf], ((i >> 1) & 1u) ^ 1u, abort)) {
        if (lane == 0) raise_error(status, abort, kErrTimeoutNorm);
        break;
      }
      const int row = row_of(q);
      const int r = nw + kNormWarps * j;
      Row cur;
      r0.unpack(cur);
      r0 = r1;
      r1 = r2;
      fetch(r2, q + 3);
      uint32_t packed[Row::kChunks];
      if (row < M) {
        ln_apply(cur, gb, gb + kNormK, ln_stats(cur, kNormK, na.eps), lane);
#pragma unroll
        for (int c = 0; c < Row::kChunks; ++c) {
          __nv_fp8x2_storage_t p[2] = {
              __nv_cvt_float2_to_fp8x2(make_float2(cur.v[4 * c], cur.v[4 * c + 1]), __NV_SATFINITE, __NV_E4M3),
              __nv_cvt_float2_to_fp8x2(make_float2(cur.v[4 * c + 2], cur.v[4 * c + 3]), __NV_SATFINITE, __NV_E4M3)};
          packed[c] = *reinterpret_cast<const uint32_t*>(p);
        }
      } else {
#pragma unroll
        for (int c = 0; c < Row::kChunks; ++c) packed[c] = 0u;  // rows past M: zeros (their outputs are clipped)
      }
      // Column 4 (32 c + lane) of the row: K chunk c, byte 4 lane of its 128-byte swizzle row.
      uint8_t* const dst = sm_a + abuf * S::kABytes + r * kStageRowBytes + (lane & 3) * 4;
#pragma unroll
      for (int c = 0; c < Row::kChunks; ++c)
        *reinterpret_cast<uint32_t*>(dst + c * S::kChunkBytes + (((lane >> 2) ^ (r & 7)) << 4)) = packed[c];
      if (j == kRowsPerWarp - 1) {
        fence_async_shared();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(map_to_rank(smem_u32(&a_full[abuf]), 0));
      }
    }
  }

  tc_fence_before();
  __syncwarp();
  cluster_sync();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, kTmemCols);
  }
}

}  // namespace mrn
