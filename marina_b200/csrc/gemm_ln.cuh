// Residual GEMM with the LayerNorm that follows it fused into the epilogue:
//
//     x[M, d] += A[M, K] · B[d, K]^T · scale + bias          (the f16 residual stream)
//     h[M, d]  = LN(x) · gamma + beta                        (bf16, or e4m3 codes of h · inv_q)
//
// It replaces "residual GEMM, then a LayerNorm pass over x" at the two places of an encoder layer
// where one follows the other: out-proj -> norm2 and FFN2 -> the next layer's norm1
// (src/net/cpu.rs:126-128 and :133-134 -> :97 in the reference; LayerNorm as layer_norm_row,
// :331-344). Fused, x is read once and written once per residual add instead of read twice and
// written once, and the LayerNorm launch goes away.
//
// A row of x is d wide; a CTA keeps two accumulators of BN columns in TMEM (so the MMAs of the
// next row block overlap the epilogue of this one), so a cluster of S = d / BN CTAs shares each
// 128-row block: CTA r of a cluster computes columns [r·BN, r·BN + BN) of every row block the
// cluster takes (its slice of B is the same for the whole launch), and the CTAs of the cluster
// combine per-row statistics through distributed shared memory.
//
// Roles (64 + 32 · 4 · BN/32 threads):
//   warp 0, one lane : TMA producer (128 x 128-byte A tile, BN x 128-byte B tile per stage).
//   warp 1, one lane : MMA issuer, M = 128, N = BN, accumulators alternating between tiles.
//   warps 2..        : epilogue, BN/32 warps per TMEM lane quarter, one 32-column chunk each.
//                      Per row block, each warp:
//       1. writes x_old of its 32 x 32 block (loaded, coalesced, while the previous block was
//          processed) into a swizzled staging block, starts loading the next block's x_old,
//          then each thread (one row) forms x_new = acc · scale + bias + x_old in f32, rounded
//          once to f16, in place, and one lane stores the block to x through TMA;
//       2. computes its 32 columns' mean and sum of squared deviations (M2, two passes over
//          the stored values) per row; the warps of the cluster merge them into the row's
//          mean and variance;
//       3. packs h = (x_new - mean) · rstd · gamma + beta into the same staging block once
//          the x_new store has read it, and stores it through TMA.
//   Steps 2-3 are pipelined across row blocks: a warp forms x_new of block t, then finishes
//   block t - 1 (whose statistics had block t's step 1 to travel), then posts block t's
//   statistics. Each warp therefore has two staging blocks, and the exchange buffers and
//   barriers come in two sets used by alternate blocks. Finishing t - 1 before posting t is
//   what makes two sets enough: a CTA can post block t + 1 (overwriting the set of t - 1 in
//   every CTA) only after finishing block t, which needs every CTA's post of block t, which
//   each CTA makes after it has read the set of t - 1.
//
// Merging (mean, M2) of equal-sized column blocks uses the pairwise update of Chan, Golub and
// LeVeque (mean = average of the means, M2 = sum of M2 + block size · sum of squared mean
// deviations): each warp writes its pair into local shared memory and arrives on the quarter's
// local barrier; the quarter's first warp merges the quarter's pairs in a fixed order, stores
// the CTA's pair into slot [rank] of every CTA of the cluster and arrives on their exchange
// barriers; every warp then merges the S slots in rank order. Every CTA merges the same values
// in the same order, so all compute bit-identical statistics; the variance is the reference's
// biased two-pass one up to rounding. Every wait is bounded (kWaitLimitNs); a wait that gives
// up records an error code and the kernel unwinds.
#pragma once

#include "gemm.cuh"

namespace mrn {

constexpr int kLnMaxCluster = 8;  // portable cluster size limit

struct LnParams {
  const float* bias;   // [d]
  const float* gamma;  // [d]
  const float* beta;   // [d]
  const __half* x;     // [M, d] residual stream before the update (read by the epilogue threads)
  float scale;         // accumulator dequantisation
  float eps;
  float inv_q;         // 1 / e4m3 scale of h (e4m3 output only)
  int d;
};

template <int BN>
struct LnShape {
  static_assert(BN % 32 == 0 && BN >= 64 && BN <= 128, "BN must be 64, 96 or 128");
  static constexpr int kQuarterWarps = BN / 32;  // epilogue warps per TMEM lane quarter
  static constexpr int kEpiWarps = 4 * kQuarterWarps;
  static constexpr int kThreads = 64 + 32 * kEpiWarps;
  static constexpr int kABytes = kTileM * kStageRowBytes;
  static constexpr int kBBytes = BN * kStageRowBytes;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kEpiBufBytes = 32 * 32 * 2;                   // one 32 x 32 f16 block
  static constexpr int kEpiBytes = 2 * kEpiWarps * kEpiBufBytes;     // two blocks per warp
  static constexpr int kLocBytes = 2 * 4 * kQuarterWarps * 32 * 8;   // [set][quarter][warp][row] pairs
  static constexpr int kXchBytes = 2 * 4 * kLnMaxCluster * 32 * 8;   // [set][quarter][rank][row] pairs
  static constexpr int kParamBytes = 3 * BN * 4;                     // bias, gamma, beta slices
  static constexpr int kBarrierBytes = 512;
  static constexpr int kFit =
      (kMaxSmem - 1024 - kEpiBytes - kLocBytes - kXchBytes - kParamBytes - kBarrierBytes) / kStageBytes;
  static constexpr int kStages = kFit > 8 ? 8 : kFit;
  static_assert(kStages >= 2, "not enough shared memory for a 2-stage pipeline");
  static constexpr int kSmemBytes =
      1024 + kStages * kStageBytes + kEpiBytes + kLocBytes + kXchBytes + kParamBytes + kBarrierBytes;
  static constexpr uint32_t kTmemCols = 2 * BN <= 128 ? 128u : 256u;  // power of two >= 2 accumulators
};

template <int BN, bool FP8, bool E4M3>
__global__ void __launch_bounds__(LnShape<BN>::kThreads, 1)
    gemm_ln_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                   const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_h,
                   const LnParams p, int M, int K, int* status) {
  using S = LnShape<BN>;
  constexpr int kStages = S::kStages;
  constexpr int kEpiWarps = S::kEpiWarps;
  constexpr int kQW = S::kQuarterWarps;
  constexpr int kElemsPerStage = FP8 ? 128 : 64;
  constexpr uint32_t kIdesc = FP8 ? idesc_e4m3(kTileM, BN) : idesc_bf16(kTileM, BN);
  constexpr int kHRowBytes = E4M3 ? 32 : 64;  // staged h bytes per row of a 32-column chunk

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sm_a = smem;
  uint8_t* sm_b = smem + kStages * S::kABytes;
  uint8_t* sm_epi = smem + kStages * S::kStageBytes;
  float2* loc = reinterpret_cast<float2*>(sm_epi + S::kEpiBytes);                 // [2][4][kQW][32]
  float2* xch = reinterpret_cast<float2*>(sm_epi + S::kEpiBytes + S::kLocBytes);  // [2][4][8][32]
  // This CTA's slices of bias, gamma and beta ([3][BN]), read by every row.
  float* prm = reinterpret_cast<float*>(sm_epi + S::kEpiBytes + S::kLocBytes + S::kXchBytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm_epi + S::kEpiBytes + S::kLocBytes + S::kXchBytes + S::kParamBytes);
  uint64_t* full = bars;                      // [kStages] TMA -> MMA
  uint64_t* empty = bars + kStages;           // [kStages] MMA -> TMA
  uint64_t* tmem_full = bars + 2 * kStages;   // [2] MMA -> epilogue
  uint64_t* tmem_empty = tmem_full + 2;       // [2] epilogue -> MMA
  uint64_t* drain = tmem_empty + 2;           // [1]
  uint64_t* lbar = drain + 1;                 // [2][4] quarter's warps -> its first warp
  uint64_t* xbar = lbar + 8;                  // [2][4] cluster's CTAs -> this CTA
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xbar + 8);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const uint32_t csize = cluster_size();
  const int cid = static_cast<int>(cluster_id_x());
  const int ncl = static_cast<int>(cluster_count_x());
  const int n0 = static_cast<int>(rank) * BN;
  const int m_tiles = (M + kTileM - 1) / kTileM;
  const int k_blocks = (K + kElemsPerStage - 1) / kElemsPerStage;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], kEpiWarps);
    }
    mbar_init(drain, 1);
    for (int i = 0; i < 8; ++i) {
      mbar_init(&lbar[i], kQW);
      mbar_init(&xbar[i], csize);
    }
    *abort = 0;
    fence_barrier_init();
    tma_prefetch_map(&map_a);
    tma_prefetch_map(&map_b);
    tma_prefetch_map(&map_x);
    tma_prefetch_map(&map_h);
  }
  for (int i = threadIdx.x; i < BN; i += blockDim.x) {
    prm[i] = p.bias[n0 + i];
    prm[BN + i] = p.gamma[n0 + i];
    prm[2 * BN + i] = p.beta[n0 + i];
  }
  // Every CTA's barriers exist before any CTA of the cluster arrives on them.
  cluster_sync();
  if (warp == 0) {
    tmem_alloc(tmem_slot, S::kTmemCols);
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
      uint32_t issued_mask = 0, parity_mask = 0;
      for (int tile = cid; tile < m_tiles && !*abort; tile += ncl) {
        const int m0 = tile * kTileM;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort)) {
            raise_error(status, abort, kErrTimeoutProducer);
            break;
          }
          mbar_arrive_expect_tx(&full[stage], S::kStageBytes);
          tma_load_2d(sm_a + stage * S::kABytes, &map_a, &full[stage], kb * kElemsPerStage, m0);
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
      for (int tile = cid; tile < m_tiles; tile += ncl) {
        if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1u, abort)) {
          raise_error(status, abort, kErrTimeoutMma);
          break;
        }
        tc_fence_after();
        const uint32_t dt = tmem + static_cast<uint32_t>(acc * BN);
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
            if constexpr (FP8)
              mma_e4m3(dt, ad, bd, kIdesc, (kb | k) != 0);
            else
              mma_bf16(dt, ad, bd, kIdesc, (kb | k) != 0);
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
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      if (*abort && issued) {
        tc_commit(drain);
        if (!mbar_wait_bounded(drain, 0) && status) atomicCAS(status, 0, kErrTimeoutDrain);
      }
    }
  } else {
    // ---- epilogue: warp w reads TMEM lane quarter w % 4, chunk `part` of this CTA's columns.
    const int quarter = warp & 3;
    const int part = (warp - 2) >> 2;
    const int col = n0 + part * 32;
    uint8_t* const sbuf = sm_epi + (warp - 2) * 2 * S::kEpiBufBytes;  // two staging blocks
    const float2 s2 = make_float2(p.scale, p.scale);
    // Coalesced x_old loads: lane l reads 16-byte chunk l % 4 of rows l / 4 + 8 i (i < 4).
    const int xr = lane >> 2, xc = lane & 3;

    // Posts this warp's (mean, M2) of row block `it` (buffer set b = it & 1): the quarter's
    // first warp merges the quarter's pairs and sends the CTA's pair to every CTA of the cluster.
    auto post = [&](int it, float mean_w, float m2_w) -> bool {
      const int q = (it & 1) * 4 + quarter;
      loc[(q * kQW + part) * 32 + lane] = make_float2(mean_w, m2_w);
      __syncwarp();
      if (lane == 0) mbar_arrive(&lbar[q]);
      if (part != 0) return true;
      if (!mbar_wait(&lbar[q], (it >> 1) & 1, abort)) return false;
      float2 w[kQW];
      float mean = 0.f, m2 = 0.f;
#pragma unroll
      for (int i = 0; i < kQW; ++i) {
        w[i] = loc[(q * kQW + i) * 32 + lane];
        mean += w[i].x;
        m2 += w[i].y;
      }
      mean *= 1.f / kQW;
      float dev = 0.f;
#pragma unroll
      for (int i = 0; i < kQW; ++i) dev += (w[i].x - mean) * (w[i].x - mean);
      m2 += 32.f * dev;
      const uint32_t slot = smem_u32(&xch[(q * kLnMaxCluster + static_cast<int>(rank)) * 32 + lane]);
      for (uint32_t r = 0; r < csize; ++r) st_cluster_f32x2(map_to_rank(slot, r), mean, m2);
      fence_acq_rel_cluster();
      __syncwarp();
      if (lane == 0) {
        const uint32_t bar = smem_u32(&xbar[q]);
        for (uint32_t r = 0; r < csize; ++r) mbar_arrive_cluster(map_to_rank(bar, r));
      }
      return true;
    };

    // Finishes row block `it` at `row0`: merges the cluster's pairs into the row's mean and
    // variance, then h = (x_new - mean) * rstd * gamma + beta from the staged x_new, stored
    // through TMA from the same staging block.
    auto finish = [&](int it, int row0) -> bool {
      const int b = it & 1;
      const int q = b * 4 + quarter;
      if (!mbar_wait_cluster(&xbar[q], (it >> 1) & 1, abort)) return false;
      float mean = 0.f, m2 = 0.f;
      for (uint32_t r = 0; r < csize; ++r) {
        const float2 c = xch[(q * kLnMaxCluster + static_cast<int>(r)) * 32 + lane];
        mean += c.x;
        m2 += c.y;
      }
      mean *= 1.f / static_cast<float>(csize);
      float dev = 0.f;
      for (uint32_t r = 0; r < csize; ++r) {
        const float c = xch[(q * kLnMaxCluster + static_cast<int>(r)) * 32 + lane].x;
        dev += (c - mean) * (c - mean);
      }
      m2 += static_cast<float>(BN) * dev;
      const float rstd = 1.0f / sqrtf(m2 / static_cast<float>(p.d) + p.eps);
      uint8_t* sb = sbuf + b * S::kEpiBufBytes;
      uint4 out[kHRowBytes / 16];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 qv = *reinterpret_cast<const uint4*>(sb + staged_offset<64>(lane, j));
        const __half2* qh = reinterpret_cast<const __half2*>(&qv);
#pragma unroll
        for (int e = 0; e < 8; e += 4) {
          const float2 f0 = __half22float2(qh[e / 2]);
          const float2 f1 = __half22float2(qh[e / 2 + 1]);
          const float4 g = *reinterpret_cast<const float4*>(prm + BN + part * 32 + 8 * j + e);
          const float4 bt = *reinterpret_cast<const float4*>(prm + 2 * BN + part * 32 + 8 * j + e);
          const float y0 = (f0.x - mean) * rstd * g.x + bt.x;
          const float y1 = (f0.y - mean) * rstd * g.y + bt.y;
          const float y2 = (f1.x - mean) * rstd * g.z + bt.z;
          const float y3 = (f1.y - mean) * rstd * g.w + bt.w;
          const int k = 2 * j + e / 4;  // 4-column group within the 32 columns
          if constexpr (E4M3) {
            __nv_fp8x2_storage_t q2[2] = {
                __nv_cvt_float2_to_fp8x2(make_float2(y0 * p.inv_q, y1 * p.inv_q), __NV_SATFINITE, __NV_E4M3),
                __nv_cvt_float2_to_fp8x2(make_float2(y2 * p.inv_q, y3 * p.inv_q), __NV_SATFINITE, __NV_E4M3)};
            reinterpret_cast<uint32_t*>(out)[k] = *reinterpret_cast<const uint32_t*>(q2);
          } else {
            __nv_bfloat162 h2[2] = {__floats2bfloat162_rn(y0, y1), __floats2bfloat162_rn(y2, y3)};
            reinterpret_cast<uint2*>(out)[k] = *reinterpret_cast<const uint2*>(h2);
          }
        }
      }
      // Every lane has read its x_new row; the x_new store of this block (older than the most
      // recent bulk group, the next block's x_new store) has read it too.
      if (lane == 0) bulk_wait_read<1>();
      __syncwarp();
#pragma unroll
      for (int j = 0; j < kHRowBytes / 16; ++j)
        *reinterpret_cast<uint4*>(sb + staged_offset<kHRowBytes>(lane, j)) = out[j];
      fence_async_shared();
      __syncwarp();
      if (lane == 0) {
        if (row0 < M) tma_store_2d(&map_h, sb, col, row0);
        bulk_commit();
      }
      return true;
    };

    uint4 xo[4];  // the next row block's x_old, rows xr + 8 i, chunk xc (8 f16 values)
    auto load_x_old = [&](int tile) {
      const int r0 = tile * kTileM + quarter * 32 + xr;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int row = r0 + 8 * i;
        xo[i] = row < M ? *reinterpret_cast<const uint4*>(p.x + static_cast<size_t>(row) * p.d + col + 8 * xc)
                        : make_uint4(0u, 0u, 0u, 0u);
      }
    };
    if (cid < m_tiles) load_x_old(cid);
    int it = 0;
    int prev_row0 = 0;
    bool ok = true;
    for (int tile = cid; tile < m_tiles; tile += ncl, ++it) {
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      const int row0 = tile * kTileM + quarter * 32;
      uint8_t* sb = sbuf + (it & 1) * S::kEpiBufBytes;
      // This staging block was last read by the stores of block it - 2.
      if (lane == 0) bulk_wait_read<0>();
      __syncwarp();
#pragma unroll
      for (int i = 0; i < 4; ++i) *reinterpret_cast<uint4*>(sb + staged_offset<64>(xr + 8 * i, xc)) = xo[i];
      __syncwarp();
      if (tile + ncl < m_tiles) load_x_old(tile + ncl);  // in flight until the next block
      if (!mbar_wait(&tmem_full[acc], acc_phase, abort)) {
        if (lane == 0) raise_error(status, abort, kErrTimeoutEpilogue);
        ok = false;
        break;
      }
      tc_fence_after();
      // x_new = acc * scale + bias + x_old in f32, rounded once to f16, in place
      const uint32_t taddr =
          tmem + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN + part * 32);
      float sum = 0.f;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float v[16];
        tmem_ld16(taddr + 16 * half, v);
        if (half == 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tmem_empty[acc]);
        }
#pragma unroll
        for (int c = 0; c < 16; c += 8) {
          uint4* at = reinterpret_cast<uint4*>(sb + staged_offset<64>(lane, (16 * half + c) / 8));
          const uint4 old = *at;
          const __half2* xh = reinterpret_cast<const __half2*>(&old);
          uint4 nw;
          __half2* nh = reinterpret_cast<__half2*>(&nw);
#pragma unroll
          for (int e = 0; e < 8; e += 2) {
            const float2 bb = *reinterpret_cast<const float2*>(prm + part * 32 + 16 * half + c + e);
            const float2 y = fma2(make_float2(v[c + e], v[c + e + 1]), s2, bb);
            const float2 xf = __half22float2(xh[e / 2]);
            nh[e / 2] = __floats2half2_rn(y.x + xf.x, y.y + xf.y);
            const float2 r = __half22float2(nh[e / 2]);  // the statistics see the stored values
            sum += r.x + r.y;
          }
          *at = nw;
        }
      }
      fence_async_shared();
      __syncwarp();
      if (lane == 0) {
        if (row0 < M) tma_store_2d(&map_x, sb, col, row0);
        bulk_commit();
      }
      // this warp's 32 columns: mean and M2 (two passes over the stored values)
      const float mean_w = sum * (1.f / 32.f);
      float m2_w = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 qv = *reinterpret_cast<const uint4*>(sb + staged_offset<64>(lane, j));
        const __half2* qh = reinterpret_cast<const __half2*>(&qv);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __half22float2(qh[e]);
          m2_w += (f.x - mean_w) * (f.x - mean_w) + (f.y - mean_w) * (f.y - mean_w);
        }
      }
      if (it > 0 && !finish(it - 1, prev_row0)) {
        if (lane == 0) raise_error(status, abort, kErrTimeoutExchange);
        ok = false;
        break;
      }
      if (!post(it, mean_w, m2_w)) {
        if (lane == 0) raise_error(status, abort, kErrTimeoutExchange);
        ok = false;
        break;
      }
      prev_row0 = row0;
    }
    if (ok && it > 0) {
      // With a single block, its x_new store is still the most recent bulk group.
      if (lane == 0) bulk_wait_read<0>();
      __syncwarp();
      if (!finish(it - 1, prev_row0) && lane == 0) raise_error(status, abort, kErrTimeoutExchange);
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  tc_fence_before();
  __syncwarp();
  // No CTA leaves while another CTA of the cluster may still write its shared memory.
  cluster_sync();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, S::kTmemCols);
  }
}

}  // namespace mrn
