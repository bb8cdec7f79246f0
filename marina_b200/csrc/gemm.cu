// Instantiations and host dispatch of the tcgen05 GEMM.
#include <stdio.h>
#include <stdlib.h>

#include "gemm.cuh"
#include "gemm.h"
#include "launch.h"
#include "tmap.h"

namespace mrn {

namespace {

template <int BN, class Epi, bool X2>
using ShapeOf = GemmShape<BN, Epi::kWarps, Epi::kOutBytes, X2 ? 2 : 1>;

template <class Epi, bool X2>
using PairShapeOf = PairShape<Epi::kOutBytes, Epi::kWarps, X2 ? 2 : 1>;

template <int BN, bool FP8, bool X2, class Epi>
cudaError_t launch_one(const GemmPlan& p, const Epi& epi, cudaStream_t stream) {
  using S = ShapeOf<BN, Epi, X2>;
  return launch_kernel(gemm_tc_kernel<BN, FP8, Epi, X2>, dim3(p.grid), dim3(S::kThreads), S::kSmemBytes, stream,
                       p.map_a, p.map_a2, p.map_b, p.map_out, epi, p.args.m, p.args.n, p.args.k, p.args.status);
}

template <bool FP8, bool X2, class Epi>
cudaError_t launch_pair(const GemmPlan& p, const Epi& epi, cudaStream_t stream) {
  using P = PairShapeOf<Epi, X2>;
  return launch_kernel(gemm_pair_kernel<FP8, Epi, X2>, dim3(p.grid), dim3(P::kThreads), P::kSmemBytes, stream,
                       p.map_a, p.map_a2, p.map_b, p.map_out, epi, p.args.m, p.args.n, p.args.k, p.args.status);
}

// The epilogue functor of `a` handed to `launch` (a single-CTA or CTA-pair launcher taking the
// functor), for the epilogues that exist for these operand types.
template <bool FP8, bool X2, class Launch>
cudaError_t with_epilogue(const GemmArgs& a, Launch launch) {
  switch (a.epi) {
    case Epilogue::kBias:
      return launch(EpiBiasBf16{a.bias, a.scale});
    case Epilogue::kResidual:
      return launch(EpiResidual{a.bias, a.scale});
    case Epilogue::kGeluBf16:
      if constexpr (!FP8) return launch(EpiGelu<false>{a.bias, a.scale, a.inv_q});
      break;
    case Epilogue::kGeluTanhBf16:
      if constexpr (!FP8) return launch(EpiGeluTanh<false>{a.bias, a.scale, a.inv_q});
      break;
    case Epilogue::kGeluE4m3:
      if constexpr (FP8 && !X2) return launch(EpiGelu<true>{a.bias, a.scale, a.inv_q});
      break;
    case Epilogue::kGeluTanhE4m3:
      if constexpr (FP8 && !X2) return launch(EpiGeluTanh<true>{a.bias, a.scale, a.inv_q});
      break;
    case Epilogue::kGeluE4m3x2:
      if constexpr (X2) return launch(EpiGeluE4m3x2<false>{a.bias, a.scale, a.inv_q, a.n});
      break;
    case Epilogue::kGeluTanhE4m3x2:
      if constexpr (X2) return launch(EpiGeluE4m3x2<true>{a.bias, a.scale, a.inv_q, a.n});
      break;
  }
  return cudaErrorInvalidValue;
}

template <bool FP8, bool X2>
cudaError_t launch_pair_epi(const GemmPlan& p, cudaStream_t stream) {
  return with_epilogue<FP8, X2>(p.args, [&](const auto& epi) { return launch_pair<FP8, X2>(p, epi, stream); });
}

template <bool FP8, bool X2, class Epi>
cudaError_t prepare_pair() {
  return cudaFuncSetAttribute(gemm_pair_kernel<FP8, Epi, X2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              PairShapeOf<Epi, X2>::kSmemBytes);
}

// MRN_GEMM_PAIR: 0 never plan CTA pairs, 1 only from K = 1024, 2 from K = 512 for every epilogue;
// unset (-1): the measured rule of use_pair.
int pair_mode() {
  static const int m = [] {
    const char* e = getenv("MRN_GEMM_PAIR");
    return e && e[0] >= '0' && e[0] <= '2' ? e[0] - '0' : -1;
  }();
  return m;
}

// Rows from which the bias epilogue (QKV) runs on CTA pairs at K = 512.
constexpr int kPairBiasMinRows = 65536;

// CTA pairs (256 x 256 tiles, each CTA loading half of B) need N a multiple of 256. They halve
// the operand bytes per FLOP and deepen the ring, which pays for long main loops (K >= 1024:
// FFN2) and, with bf16 operands, for the residual epilogue from K = 512 (out-proj: 10-20% faster
// at every batch from 256 to 4096 positions) and for the bias epilogue from K = 512 once M is
// large (QKV: level at 512 positions, 2-4% faster from 1024, 6% slower at 256). The GELU
// epilogues stay on single CTAs (FFN1 1-10% slower on pairs), and so do one-term e4m3 operands
// at K = 512 (batch 4096: QKV 246 -> 281 us, out-proj 114 -> 133 on pairs); two-term e4m3 runs
// the out-proj on pairs (159 -> 150 us) and QKV on single CTAs (350 -> 362 on pairs). Pairs also
// need a full wave of 128-row tiles (M >= 128 rows x SMs): with fewer, single CTAs on narrow tiles
// spread the GEMM over more SMs (batch 1: 0.517 -> 0.445 ms per pass, 16: 0.596 -> 0.515, 64:
// 0.763 -> 0.703; level at 256).
bool use_pair(const GemmArgs& a, int num_sms) {
  if (a.n % 256 != 0 || a.pair == 0) return false;
  if (a.pair == 1) return true;
  switch (pair_mode()) {
    case 0: return false;
    case 1: return a.k >= 1024;
    case 2: return a.k >= 512;
  }
  if (a.m < kTileM * num_sms) return false;
  if (a.k >= 1024) return true;
  if (a.k < 512) return false;
  if (a.epi == Epilogue::kResidual) return !a.fp8 || a.x2;
  return a.epi == Epilogue::kBias && !a.fp8 && a.m >= kPairBiasMinRows;
}

template <int BN, bool FP8, bool X2>
cudaError_t launch_bn(const GemmPlan& p, cudaStream_t stream) {
  return with_epilogue<FP8, X2>(p.args, [&](const auto& epi) { return launch_one<BN, FP8, X2>(p, epi, stream); });
}

template <bool FP8, bool X2>
cudaError_t launch_single(const GemmPlan& p, cudaStream_t stream) {
  switch (p.bn) {
    case 256: return launch_bn<256, FP8, X2>(p, stream);
    case 192: return launch_bn<192, FP8, X2>(p, stream);
    case 128: return launch_bn<128, FP8, X2>(p, stream);
    case 64: return launch_bn<64, FP8, X2>(p, stream);
  }
  return cudaErrorInvalidValue;
}

template <int BN, bool FP8, bool X2, class Epi>
cudaError_t prepare_one() {
  return cudaFuncSetAttribute(gemm_tc_kernel<BN, FP8, Epi, X2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              ShapeOf<BN, Epi, X2>::kSmemBytes);
}

template <int BN>
cudaError_t prepare_bn() {
  cudaError_t e;
  if ((e = prepare_one<BN, false, false, EpiBiasBf16>()) != cudaSuccess) return e;
  if ((e = prepare_one<BN, false, false, EpiResidual>()) != cudaSuccess) return e;
  if ((e = prepare_one<BN, false, false, EpiGelu<false>>()) != cudaSuccess) return e;
  if ((e = prepare_one<BN, false, false, EpiGeluTanh<false>>()) != cudaSuccess) return e;
  if ((e = prepare_one<BN, true, false, EpiGeluTanh<true>>()) != cudaSuccess) return e;
  if ((e = prepare_one<BN, true, false, EpiBiasBf16>()) != cudaSuccess) return e;
  if ((e = prepare_one<BN, true, false, EpiResidual>()) != cudaSuccess) return e;
  if ((e = prepare_one<BN, true, false, EpiGelu<true>>()) != cudaSuccess) return e;
  if ((e = prepare_one<BN, true, true, EpiBiasBf16>()) != cudaSuccess) return e;
  if ((e = prepare_one<BN, true, true, EpiResidual>()) != cudaSuccess) return e;
  if ((e = prepare_one<BN, true, true, EpiGeluE4m3x2<false>>()) != cudaSuccess) return e;
  return prepare_one<BN, true, true, EpiGeluE4m3x2<true>>();
}

}  // namespace

int gemm_pick_bn(int n) {
  for (int bn : {256, 192, 128, 64})
    if (n % bn == 0) return bn;
  return 0;
}

bool gemm_plan(GemmPlan* plan, const GemmArgs& args, int num_sms, char* err) {
  plan->args = args;
  plan->pair = false;
  plan->bn = gemm_pick_bn(args.n);
  const int eb = args.fp8 ? 1 : 2;
  if (args.m <= 0 || args.n <= 0 || args.k <= 0) {
    snprintf(err, 256, "gemm: empty shape %dx%dx%d", args.m, args.n, args.k);
    return false;
  }
  if (plan->bn == 0) {
    snprintf(err, 256, "gemm: N=%d is not a multiple of 64", args.n);
    return false;
  }
  if ((args.k * eb) % 16 != 0) {
    snprintf(err, 256, "gemm: K=%d rows are not a multiple of 16 bytes", args.k);
    return false;
  }
  const bool x2_out = args.epi == Epilogue::kGeluE4m3x2 || args.epi == Epilogue::kGeluTanhE4m3x2;
  if ((args.epi == Epilogue::kGeluE4m3 || args.epi == Epilogue::kGeluTanhE4m3) && (!args.fp8 || args.x2)) {
    snprintf(err, 256, "gemm: e4m3 GELU output is only planned for one-term FP8 operands");
    return false;
  }
  if (x2_out != args.x2 && args.epi != Epilogue::kBias && args.epi != Epilogue::kResidual) {
    snprintf(err, 256, "gemm: two-term e4m3 GELU output is planned for two-term operands only");
    return false;
  }
  if (args.x2 && (!args.fp8 || args.k % 16 != 0)) {
    snprintf(err, 256, "gemm: two-term activations need e4m3 operands and K a multiple of 16 (K=%d)", args.k);
    return false;
  }
  if ((args.epi == Epilogue::kGeluBf16 || args.epi == Epilogue::kGeluTanhBf16) && args.fp8) {
    snprintf(err, 256, "gemm: bf16 GELU output is only planned for bf16 operands");
    return false;
  }
  if (args.ldo < args.n || (reinterpret_cast<uintptr_t>(args.out) & 15) != 0 ||
      (reinterpret_cast<uintptr_t>(args.bias) & 15) != 0) {
    snprintf(err, 256, "gemm: output/bias misaligned or ldo %d < N %d", args.ldo, args.n);
    return false;
  }
  plan->pair = use_pair(args, num_sms);
  // The memory-bound residual GEMMs with a short K (out-proj) run 128-column tiles with four
  // TMEM accumulators: the reduce-add stores drain behind three tiles of MMAs.
  if (!plan->pair && args.epi == Epilogue::kResidual && args.k < 1024 && args.n % 128 == 0) plan->bn = 128;
  // Small batches: the narrowest tile (64, then 128 columns) whose tiles still fit in one wave of
  // the SMs. More SMs share the GEMM, and the narrower stages hold more of its K loop in flight
  // (batch 1: 0.585 -> 0.513 ms per pass with 64-column tiles; batch 16: 0.638 -> 0.595 with 128;
  // from batch 64 the widest tile is faster).
  if (!plan->pair) {
    const int m_tiles = (args.m + kTileM - 1) / kTileM;
    for (int bn : {64, 128})
      if (bn < plan->bn && args.n % bn == 0 && m_tiles * (args.n / bn) <= num_sms) {
        plan->bn = bn;
        break;
      }
  }
  // Two-term A: [M, 2K] with each row's K hi codes then its K lo codes, read through two maps.
  const uint64_t a_row = args.x2 ? 2 * static_cast<uint64_t>(args.k) : 0;
  if (!make_kmajor_map(&plan->map_a, args.a, eb, args.m, args.k, kTileM, a_row) ||
      !make_kmajor_map(&plan->map_a2, args.x2 ? static_cast<const uint8_t*>(args.a) + args.k : args.a, eb, args.m,
                       args.k, kTileM, a_row) ||
      !make_kmajor_map(&plan->map_b, args.b, eb, args.n, args.k, plan->pair ? 128 : plan->bn)) {
    snprintf(err, 256, "gemm: cuTensorMapEncodeTiled failed (M=%d N=%d K=%d)", args.m, args.n, args.k);
    return false;
  }
  bool out_ok = false;
  switch (args.epi) {
    case Epilogue::kBias:
    case Epilogue::kGeluBf16:
    case Epilogue::kGeluTanhBf16:
      out_ok = make_store_map(&plan->map_out, args.out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, args.m, args.n, args.ldo);
      break;
    case Epilogue::kGeluE4m3:
    case Epilogue::kGeluTanhE4m3:
      out_ok = make_store_map(&plan->map_out, args.out, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, args.m, args.n, args.ldo);
      break;
    case Epilogue::kResidual:
      out_ok = make_store_map(&plan->map_out, args.out, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, args.m, args.n, args.ldo);
      break;
    case Epilogue::kGeluE4m3x2:
    case Epilogue::kGeluTanhE4m3x2:
      // [M, 2N]: the hi block of columns [n0 + c, +32) and the lo block N columns further on
      out_ok = args.ldo >= 2 * args.n &&
               make_store_map(&plan->map_out, args.out, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, args.m, 2 * args.n, args.ldo);
      break;
  }
  if (!out_ok) {
    snprintf(err, 256, "gemm: output tensor map failed (M=%d N=%d ldo=%d)", args.m, args.n, args.ldo);
    return false;
  }
  if (plan->pair) {
    const int tiles = ((args.m + 2 * kTileM - 1) / (2 * kTileM)) * (args.n / 256);
    const int pairs = num_sms / 2;
    plan->grid = 2 * (tiles < pairs ? tiles : pairs);
  } else {
    const int tiles = ((args.m + kTileM - 1) / kTileM) * (args.n / plan->bn);
    plan->grid = tiles < num_sms ? tiles : num_sms;
  }
  return true;
}

cudaError_t gemm_prepare_device() {
  cudaError_t e;
  if ((e = prepare_pair<false, false, EpiBiasBf16>()) != cudaSuccess) return e;
  if ((e = prepare_pair<false, false, EpiResidual>()) != cudaSuccess) return e;
  if ((e = prepare_pair<false, false, EpiGelu<false>>()) != cudaSuccess) return e;
  if ((e = prepare_pair<false, false, EpiGeluTanh<false>>()) != cudaSuccess) return e;
  if ((e = prepare_pair<true, false, EpiGeluTanh<true>>()) != cudaSuccess) return e;
  if ((e = prepare_pair<true, false, EpiBiasBf16>()) != cudaSuccess) return e;
  if ((e = prepare_pair<true, false, EpiResidual>()) != cudaSuccess) return e;
  if ((e = prepare_pair<true, false, EpiGelu<true>>()) != cudaSuccess) return e;
  if ((e = prepare_pair<true, true, EpiBiasBf16>()) != cudaSuccess) return e;
  if ((e = prepare_pair<true, true, EpiResidual>()) != cudaSuccess) return e;
  if ((e = prepare_pair<true, true, EpiGeluE4m3x2<false>>()) != cudaSuccess) return e;
  if ((e = prepare_pair<true, true, EpiGeluE4m3x2<true>>()) != cudaSuccess) return e;
  if ((e = prepare_bn<256>()) != cudaSuccess) return e;
  if ((e = prepare_bn<192>()) != cudaSuccess) return e;
  if ((e = prepare_bn<128>()) != cudaSuccess) return e;
  return prepare_bn<64>();
}

#ifdef MRN_TEST_HOOKS
cudaError_t gemm_test_hooks(unsigned long long wait_limit_ns, int no_loads, cudaStream_t stream) {
  cudaError_t e = cudaMemcpyToSymbolAsync(g_wait_limit_ns, &wait_limit_ns, sizeof(wait_limit_ns), 0,
                                          cudaMemcpyHostToDevice, stream);
  if (e != cudaSuccess) return e;
  return cudaMemcpyToSymbolAsync(g_test_no_loads, &no_loads, sizeof(no_loads), 0, cudaMemcpyHostToDevice, stream);
}
#endif

cudaError_t gemm_launch(const GemmPlan& plan, cudaStream_t stream) {
  const GemmArgs& a = plan.args;
  if (plan.pair)
    return a.x2 ? launch_pair_epi<true, true>(plan, stream)
                : a.fp8 ? launch_pair_epi<true, false>(plan, stream) : launch_pair_epi<false, false>(plan, stream);
  return a.x2 ? launch_single<true, true>(plan, stream)
              : a.fp8 ? launch_single<true, false>(plan, stream) : launch_single<false, false>(plan, stream);
}

}  // namespace mrn
