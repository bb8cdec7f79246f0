// The encoder's MLP block in one kernel: FFN1 -> GELU -> FFN2 -> residual add,
//
//     f = e4m3(GELU(h · W1^T · s1 + b1) · inv_q)      [M, ff]   (kept in shared memory)
//     x += f · W2^T · s2 + b2                          [M, d]    (f16 atomic adds in L2)
//
// (the feed-forward half of the pre-LN block, src/net/cpu.rs:135-160, with the reference CUDA
// backend's e4m3 activations). Unfused, f is written to and read back from HBM: 2 bytes per
// element of a [M, 4d] tensor, the largest round trip of the pass. Here it never leaves the SM.
//
// Work split: a cluster of two CTAs owns a 128-row tile at a time. CTA r computes the hidden
// chunks j = 2i + r (128 columns of f each, i < ff / 256) into TMEM, applies the GELU epilogue
// and writes the e4m3 chunk into its own shared memory in the 128-byte swizzled K-major layout
// of an MMA operand; a bulk copy sends it to the same slot of the other CTA. Both CTAs then run
// FFN2 over all ff / 128 chunks in the same (natural) order, CTA r producing output columns
// [r d/2, (r+1) d/2). No FLOP is done twice and each CTA's TMEM holds the 128 x d/2 output
// accumulator (256 columns) plus two 128-column hidden accumulators.
//
// Roles per CTA (19 warps):
//   warp 0, one lane : TMA producer: the tile's A rows (h, 4 boxes of 128 x 128 bytes, and an
//                      L2 prefetch of the next tile's), then W1 / W2 slices in MMA order through
//                      a ring of three 32 KB slots.
//   warp 1, one lane : MMA issuer (tcgen05, cta_group::1, e4m3): FFN1 chunk i = 16 MMAs
//                      (M 128, N 128, K 32) into a hidden accumulator; FFN2 chunk j = 4 MMAs
//                      (M 128, N 256, K 32) into the output accumulator. Order per tile:
//                      F1(0) F1(1) F1(2), then per i: F2(2i) F2(2i+1) F1(i+3): FFN1 runs three
//                      chunks ahead of the FFN2 that consumes them, so the GELU epilogue and the
//                      exchange of a chunk overlap about two chunks' worth of MMAs. (F1(i+3)
//                      reuses the hidden accumulator of F1(i+1), which its GELU warps drained
//                      right after F1(i+1) completed.)
//   warp 2, one lane : exchange: sends each finished own chunk to the peer CTA (cp.async.bulk
//                      shared::cta -> shared::cluster, completing on the peer's slot barrier, on
//                      which it also arrives with the expected byte count) and releases it to
//                      its own MMA issuer.
//   warps 3..18      : GELU epilogue of own chunks (warp w: TMEM lanes 32 (w % 4), 32 of the
//                      chunk's columns); at the end of a tile, warps 3..10 drain the output
//                      accumulator as the residual epilogue.
//
// Hidden-chunk slots (four, 16 KB) are shared by both CTAs' chunk streams: global chunk number
// n (tile iteration x chunks + j) uses slot n % 4 in both CTAs. f_full[s] (1 arrival plus, for
// the peer's chunks, the copy's bytes; both come from the chunk owner's exchange warp) gates the
// MMA; f_empty[s] (2 arrivals: a multicast commit from each CTA's MMA issuer) frees the slot in
// both CTAs at once, which is also what lets the owner send into the peer's slot; f_local[s] (16
// arrivals) tells the exchange warp an own chunk is complete. Every wait is bounded; a CTA that
// gives up waits (bounded) for the chunks that may still be copied into it before it exits.
#pragma once

#include "gemm.cuh"

namespace mrn {

// x[0..8) += v (8 halves) as one fire-and-forget atomic add in L2.
__device__ __forceinline__ void red_add_h8(__half* x, uint4 v) {
  asm volatile("red.relaxed.gpu.global.add.noftz.v4.f16x2 [%0], {%1, %2, %3, %4};" ::"l"(x), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

constexpr int kMlpD = 512;  // d of the instantiated kernel

struct MlpShape {
  static constexpr int kOutCols = kMlpD / 2;                    // output columns per CTA
  static constexpr int kChunk = 128;                            // hidden columns per chunk
  static constexpr int kKBlocks1 = kMlpD / kStageRowBytes;      // FFN1 K blocks of 128
  static constexpr int kBlockBytes = kTileM * kStageRowBytes;   // 128 rows x 128 bytes
  static constexpr int kABytes = kKBlocks1 * kBlockBytes;       // the tile's h rows
  static constexpr int kWBytes = kOutCols * kStageRowBytes;     // W2 slice, or two W1 K blocks
  static constexpr int kWStages = 3;
  static constexpr int kFBytes = kBlockBytes;                   // one hidden chunk
  static constexpr int kFSlots = 4;
  static constexpr int kF1Lead = 3;                             // FFN1 chunks issued ahead of FFN2
  static constexpr int kGeluWarps = 16;
  static constexpr int kOutWarps = 8;
  static constexpr int kBarrierBytes = 256;
  static constexpr int kSmemBytes = 1024 + kABytes + kWStages * kWBytes + kFSlots * kFBytes +
                                    kBarrierBytes;
  static constexpr int kThreads = 32 * (3 + kGeluWarps);
  static_assert(kWBytes == 2 * kBlockBytes, "a W slot holds one W2 slice or two W1 K blocks");
  static_assert(kSmemBytes <= kMaxSmem, "shared memory");
  // a_full/empty, w_full/empty, h_full/empty, f_full/empty/local, out_full/empty, drain; TMEM slot, abort
  static_assert((2 + 2 * kWStages + 4 + 3 * kFSlots + 3) * 8 + 8 <= kBarrierBytes, "barrier space");
};

template <class Gelu>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(MlpShape::kThreads, 1)
    gemm_mlp_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_w1,
                    const __grid_constant__ CUtensorMap map_w2, __half* __restrict__ x, Gelu gelu,
                    EpiResidual res, int M, int ff, int* status) {
  using S = MlpShape;
  constexpr uint32_t kIdesc1 = idesc_e4m3(kTileM, S::kChunk);
  constexpr uint32_t kIdesc2 = idesc_e4m3(kTileM, S::kOutCols);
  constexpr uint32_t kAccOut = 0;                    // TMEM columns [0, 256)
  constexpr uint32_t kAccH = S::kOutCols;            // [256, 384), [384, 512)

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sm_a = smem;
  uint8_t* sm_w = sm_a + S::kABytes;
  uint8_t* sm_f = sm_w + S::kWStages * S::kWBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm_f + S::kFSlots * S::kFBytes);
  uint64_t* a_full = bars;                    // TMA -> MMA (the tile's h rows)
  uint64_t* a_empty = bars + 1;               // MMA -> TMA
  uint64_t* w_full = bars + 2;                       // [kWStages]
  uint64_t* w_empty = w_full + S::kWStages;          // [kWStages]
  uint64_t* h_full = w_empty + S::kWStages;          // [2] MMA -> GELU warps
  uint64_t* h_empty = h_full + 2;             // [2] GELU warps -> MMA
  uint64_t* f_full = h_empty + 2;                    // [kFSlots] the owner's exchange warp -> MMA
  uint64_t* f_empty = f_full + S::kFSlots;           // [kFSlots] both CTAs' MMAs -> slot writers
  uint64_t* f_local = f_empty + S::kFSlots;          // [kFSlots] GELU warps -> exchange warp
  uint64_t* out_full = f_local + S::kFSlots;         // MMA -> output epilogue
  uint64_t* out_empty = out_full + 1;         // output epilogue -> MMA
  uint64_t* drain = out_empty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rank = static_cast<int>(cluster_ctarank());
  const uint32_t peer = static_cast<uint32_t>(rank ^ 1);
  const int cid = static_cast<int>(cluster_id_x());
  const int ncl = static_cast<int>(cluster_count_x());
  const int m_tiles = (M + kTileM - 1) / kTileM;
  const int chunks = ff / S::kChunk;
  const int own = chunks / 2;

  if (threadIdx.x == 0) {
    mbar_init(a_full, 1);
    mbar_init(a_empty, 1);
    for (int s = 0; s < S::kWStages; ++s) {
      mbar_init(&w_full[s], 1);
      mbar_init(&w_empty[s], 1);
    }
    for (int s = 0; s < S::kFSlots; ++s) {
      mbar_init(&f_full[s], 1);
      mbar_init(&f_empty[s], 2);
      mbar_init(&f_local[s], S::kGeluWarps);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&h_full[b], 1);
      mbar_init(&h_empty[b], S::kGeluWarps);
    }
    mbar_init(out_full, 1);
    mbar_init(out_empty, S::kOutWarps);
    mbar_init(drain, 1);
    *abort = 0;
    fence_barrier_init();
    tma_prefetch_map(&map_a);
    tma_prefetch_map(&map_w1);
    tma_prefetch_map(&map_w2);
  }
  cluster_sync();  // both CTAs' barriers exist before either signals the other's
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
      int wn = 0;
      bool ok = true;
      uint32_t w_issued = 0, w_parity = 0;
      bool a_issued = false;
      uint32_t a_parity = 0;
      auto w_slot = [&](bool& ok_) -> int {
        const int s = wn % S::kWStages;
        if (!mbar_wait(&w_empty[s], ((wn / S::kWStages) & 1) ^ 1u, abort)) {
          raise_error(status, abort, kErrTimeoutProducer);
          ok_ = false;
          return -1;
        }
        mbar_arrive_expect_tx(&w_full[s], S::kWBytes);
        w_issued |= 1u << s;
        w_parity = (w_parity & ~(1u << s)) | (((wn / S::kWStages) & 1u) << s);
        ++wn;
        return s;
      };
      auto load_f1 = [&](int i) {
        const int j = 2 * i + rank;
        for (int hf = 0; hf < 2 && ok; ++hf) {
          const int s = w_slot(ok);
          if (s < 0) return;
          uint8_t* dst = sm_w + s * S::kWBytes;
          tma_load_2d(dst, &map_w1, &w_full[s], (2 * hf) * kStageRowBytes, j * S::kChunk);
          tma_load_2d(dst + S::kBlockBytes, &map_w1, &w_full[s], (2 * hf + 1) * kStageRowBytes, j * S::kChunk);
        }
      };
      auto load_f2 = [&](int j) {
        if (!ok) return;
        const int s = w_slot(ok);
        if (s < 0) return;
        tma_load_2d(sm_w + s * S::kWBytes, &map_w2, &w_full[s], j * S::kChunk, rank * S::kOutCols);
      };
      int it = 0;
      for (int t = cid; t < m_tiles && ok && !*abort; t += ncl, ++it) {
        if (!mbar_wait(a_empty, (it & 1) ^ 1u, abort)) {
          raise_error(status, abort, kErrTimeoutProducer);
          break;
        }
        mbar_arrive_expect_tx(a_full, S::kABytes);
        for (int kb = 0; kb < S::kKBlocks1; ++kb)
          tma_load_2d(sm_a + kb * S::kBlockBytes, &map_a, a_full, kb * kStageRowBytes, t * kTileM);
        a_issued = true;
        a_parity = it & 1;
        if (t + ncl < m_tiles)
          for (int kb = 0; kb < S::kKBlocks1; ++kb) tma_prefetch_l2_2d(&map_a, kb * kStageRowBytes, (t + ncl) * kTileM);
        for (int i = 0; i < S::kF1Lead && i < own; ++i) load_f1(i);
        for (int i = 0; i < own && ok; ++i) {
          load_f2(2 * i);
          load_f2(2 * i + 1);
          if (i + S::kF1Lead < own) load_f1(i + S::kF1Lead);
        }
      }
      if (*abort) {
        // Let the copies still in flight land before the CTA's shared memory goes away.
        if (a_issued) mbar_wait_bounded(a_full, a_parity);
        for (int s = 0; s < S::kWStages; ++s)
          if (w_issued & (1u << s)) mbar_wait_bounded(&w_full[s], (w_parity >> s) & 1u);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer
      int wn = 0, f1n = 0;
      bool ok = true, issued = false;
      auto w_wait = [&]() -> int {
        const int s = wn % S::kWStages;
        if (!mbar_wait(&w_full[s], (wn / S::kWStages) & 1u, abort)) {
          raise_error(status, abort, kErrTimeoutMma);
          ok = false;
          return -1;
        }
        tc_fence_after();
        ++wn;
        return s;
      };
      auto f1 = [&](int i) {
        if (!ok) return;
        const int b = f1n & 1;
        if (!mbar_wait(&h_empty[b], ((f1n >> 1) & 1) ^ 1u, abort)) {
          raise_error(status, abort, kErrTimeoutMma);
          ok = false;
          return;
        }
        tc_fence_after();
        const uint32_t d = tmem + kAccH + static_cast<uint32_t>(b * S::kChunk);
        for (int hf = 0; hf < 2; ++hf) {
          const int s = w_wait();
          if (s < 0) return;
          const uint32_t wa = smem_u32(sm_w + s * S::kWBytes);
#pragma unroll
          for (int kb2 = 0; kb2 < 2; ++kb2) {
            const uint32_t aa = smem_u32(sm_a + (2 * hf + kb2) * S::kBlockBytes);
#pragma unroll
            for (int k = 0; k < kStageRowBytes / 32; ++k)
              mma_e4m3(d, desc_sw128(aa + 32u * k), desc_sw128(wa + kb2 * S::kBlockBytes + 32u * k), kIdesc1,
                       (hf | kb2 | k) != 0);
          }
          issued = true;
          tc_commit(&w_empty[s]);
        }
        tc_commit(&h_full[b]);
        if (i == own - 1) tc_commit(a_empty);  // the tile's h rows are no longer read
        ++f1n;
      };
      int it = 0;
      int next_n = 0;  // the next hidden chunk number to consume
      auto f2 = [&](int j) {
        if (!ok) return;
        const int n = it * chunks + j;
        const int fs = n % S::kFSlots;
        if (!mbar_wait_cluster(&f_full[fs], (n / S::kFSlots) & 1u, abort)) {
          raise_error(status, abort, kErrTimeoutMma);
          ok = false;
          return;
        }
        if (j == 0 && !mbar_wait(out_empty, (it & 1) ^ 1u, abort)) {
          raise_error(status, abort, kErrTimeoutMma);
          ok = false;
          return;
        }
        tc_fence_after();
        const int s = w_wait();
        if (s < 0) return;
        const uint32_t fa = smem_u32(sm_f + fs * S::kFBytes);
        const uint32_t wa = smem_u32(sm_w + s * S::kWBytes);
#pragma unroll
        for (int k = 0; k < kStageRowBytes / 32; ++k)
          mma_e4m3(tmem + kAccOut, desc_sw128(fa + 32u * k), desc_sw128(wa + 32u * k), kIdesc2, (j | k) != 0);
        issued = true;
        tc_commit(&w_empty[s]);
        tc_commit_mc(&f_empty[fs], 0x3);  // this CTA no longer reads the slot (both CTAs' barriers)
        next_n = n + 1;
        if (j == chunks - 1) tc_commit(out_full);
      };
      for (int t = cid; t < m_tiles && ok; t += ncl, ++it) {
        if (!mbar_wait(a_full, it & 1, abort)) {
          raise_error(status, abort, kErrTimeoutMma);
          break;
        }
        tc_fence_after();
        for (int i = 0; i < S::kF1Lead && i < own; ++i) f1(i);
        for (int i = 0; i < own && ok; ++i) {
          f2(2 * i);
          f2(2 * i + 1);
          if (i + S::kF1Lead < own) f1(i + S::kF1Lead);
        }
      }
      // The last commit through each slot (this CTA's and the peer's, which arrive here
      // asynchronously) has landed before this CTA's shared memory can go away.
      for (int s = 0; s < S::kFSlots; ++s) {
        const int uses = (next_n - s + S::kFSlots - 1) / S::kFSlots;
        if (uses > 0) mbar_wait_bounded(&f_empty[s], static_cast<uint32_t>(uses - 1) & 1u);
      }
      if (*abort) {
        if (issued) {
          tc_commit(drain);
          if (!mbar_wait_bounded(drain, 0) && status) atomicCAS(status, 0, kErrTimeoutDrain);
        }
        // The peer may still be copying a chunk into a slot whose next phase this CTA has not
        // consumed: give each such phase its bounded wait before shared memory is released.
        for (int s = 0; s < S::kFSlots; ++s) {
          const int consumed = (next_n - s + S::kFSlots - 1) / S::kFSlots;
          mbar_wait_bounded(&f_full[s], static_cast<uint32_t>(consumed) & 1u);
        }
      }
    }
  } else if (warp == 2) {
    if (lane == 0) {
      // ---- exchange: own chunks only, in order; the peer's chunks need nothing from this CTA
      uint32_t own_uses = 0;  // bit s: parity of this CTA's own chunks through slot s
      int it = 0;
      for (int t = cid; t < m_tiles && !*abort; t += ncl, ++it) {
        bool ok = true;
        for (int j = rank; j < chunks; j += 2) {
          const int fs = (it * chunks + j) % S::kFSlots;
          // The GELU warps waited for the slot to be free in both CTAs before writing it, so the
          // peer's slot is free and its barrier is in the phase this chunk completes.
          if (!mbar_wait(&f_local[fs], (own_uses >> fs) & 1u, abort)) {
            raise_error(status, abort, kErrTimeoutExchange);
            ok = false;
            break;
          }
          own_uses ^= 1u << fs;
          uint8_t* slot = sm_f + fs * S::kFBytes;
          const uint32_t peer_bar = map_to_rank(smem_u32(&f_full[fs]), peer);
          mbar_arrive_expect_tx_cluster(peer_bar, S::kFBytes);
          bulk_copy_to_peer(map_to_rank(smem_u32(slot), peer), slot, S::kFBytes, peer_bar);
          mbar_arrive(&f_full[fs]);
        }
        if (!ok) break;
      }
    }
  } else {
    // ---- GELU epilogue (16 warps) and, on warps 3..10, the output epilogue
    const int quarter = warp & 3;
    const int part = (warp - 3) >> 2;
    const int row = quarter * 32 + lane;
    int gn = 0, it = 0;
    bool ok = true;
    for (int t = cid; t < m_tiles && ok; t += ncl, ++it) {
      for (int i = 0; i < own; ++i, ++gn) {
        const int j = 2 * i + rank;
        const int n = it * chunks + j;
        const int fs = n % S::kFSlots;
        const int b = gn & 1;
        float4 bias[8];
        load_bias32(gelu.bias, j * S::kChunk + part * 32, bias);  // in flight during the wait
        if (!mbar_wait(&h_full[b], (gn >> 1) & 1u, abort)) {
          if (lane == 0) raise_error(status, abort, kErrTimeoutEpilogue);
          ok = false;
          break;
        }
        tc_fence_after();
        float v[32];
        tmem_ld32(tmem + (static_cast<uint32_t>(quarter * 32) << 16) + kAccH + static_cast<uint32_t>(b * S::kChunk + part * 32),
                  v);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&h_empty[b]);
        uint4 out[2];
        gelu.pack_with(bias, v, out);
        if (!mbar_wait(&f_empty[fs], ((n / S::kFSlots) & 1u) ^ 1u, abort)) {
          if (lane == 0) raise_error(status, abort, kErrTimeoutEpilogue);
          ok = false;
          break;
        }
        // Columns [32 part, 32 part + 32) of the chunk: 16-byte units 2 part, 2 part + 1 of the row.
        uint8_t* dst = sm_f + fs * S::kFBytes + row * kStageRowBytes;
        *reinterpret_cast<uint4*>(dst + (((2 * part) ^ (row & 7)) << 4)) = out[0];
        *reinterpret_cast<uint4*>(dst + (((2 * part + 1) ^ (row & 7)) << 4)) = out[1];
        fence_async_shared();
        __syncwarp();
        if (lane == 0) mbar_arrive(&f_local[fs]);
      }
      if (!ok || part >= 2) continue;
      // Output epilogue: columns part * 32 + 64 c of this CTA's half, c < 4.
      if (!mbar_wait(out_full, it & 1, abort)) {
        if (lane == 0) raise_error(status, abort, kErrTimeoutEpilogue);
        ok = false;
        break;
      }
      tc_fence_after();
      // Each lane owns one row: its 32 columns are 64 contiguous bytes of x, added to with four
      // vector f16 atomic adds in L2 (no read back, no staging, nothing to wait for).
      const int xrow = t * kTileM + row;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        const int col = rank * S::kOutCols + part * 32 + 64 * c;
        float v[32];
        tmem_ld32(tmem + (static_cast<uint32_t>(quarter * 32) << 16) + kAccOut + static_cast<uint32_t>(col - rank * S::kOutCols),
                  v);
        if (c == 3) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(out_empty);
        }
        uint4 o[4];
        res.pack(col, v, o);
        if (xrow < M) {
          __half* px = x + static_cast<size_t>(xrow) * kMlpD + col;
#pragma unroll
          for (int q = 0; q < 4; ++q) red_add_h8(px + 8 * q, o[q]);
        }
      }
    }
  }

  tc_fence_before();
  __syncwarp();
  cluster_sync();  // neither CTA leaves while the other may still store into it or signal it
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace mrn
