// Instantiations and host dispatch of the tcgen05 GEMM.
#include <stdio.h>
#include <stdlib.h>

#include "gemm.cuh"
#include "gemm.h"
#include "launch.h"
#include "tmap.h"

namespace mrn {

namespace {

template <int BN, class Epi>
using ShapeOf = GemmShape<BN, Epi::kWarps, Epi::kOutBytes>;

template <int BN, bool FP8, class Epi>
cudaError_t launch_one(const GemmPlan& p, const Epi& epi, cudaStream_t stream) {
  return launch_kernel(gemm_tc_kernel<BN, FP8, Epi>, dim3(p.grid), dim3(ShapeOf<BN, Epi>::kThreads),
                       ShapeOf<BN, Epi>::kSmemBytes, stream, p.map_a, p.map_b, p.map_out, epi, p.args.m, p.args.n,
                       p.args.k, p.args.status);
}

template <bool FP8, class Epi>
cudaError_t launch_pair(const GemmPlan& p, const Epi& epi, cudaStream_t stream) {
  using P = PairShape<Epi::kOutBytes, Epi::kWarps>;
  return launch_kernel(gemm_pair_kernel<FP8, Epi>, dim3(p.grid), dim3(P::kThreads), P::kSmemBytes, stream, p.map_a,
                       p.map_b, p.map_out, epi, p.args.m, p.args.n, p.args.k, p.args.status);
}

template <bool FP8>
cudaError_t launch_pair_epi(const GemmPlan& p, cudaStream_t stream) {
  const GemmArgs& a = p.args;
  switch (a.epi) {
    case Epilogue::kBias:
      return launch_pair<FP8>(p, EpiBiasBf16{a.bias, a.scale}, stream);
    case Epilogue::kResidual:
      return launch_pair<FP8>(p, EpiResidual{a.bias, a.scale}, stream);
    case Epilogue::kGeluBf16:
      if constexpr (!FP8) return launch_pair<FP8>(p, EpiGelu<false>{a.bias, a.scale, a.inv_q}, stream);
      break;
    case Epilogue::kGeluE4m3:
      if constexpr (FP8) return launch_pair<FP8>(p, EpiGelu<true>{a.bias, a.scale, a.inv_q}, stream);
      break;
    case Epilogue::kGeluTanhBf16:
      if constexpr (!FP8) return launch_pair<FP8>(p, EpiGeluTanh<false>{a.bias, a.scale, a.inv_q}, stream);
      break;
    case Epilogue::kGeluTanhE4m3:
      if constexpr (FP8) return launch_pair<FP8>(p, EpiGeluTanh<true>{a.bias, a.scale, a.inv_q}, stream);
      break;
    default:
      break;
  }
  return cudaErrorInvalidValue;
}

template <bool FP8, class Epi>
cudaError_t prepare_pair() {
  return cudaFuncSetAttribute(gemm_pair_kernel<FP8, Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              PairShape<Epi::kOutBytes, Epi::kWarps>::kSmemBytes);
}

// Smallest K planned on CTA pairs (N a multiple of 256): MRN_GEMM_PAIR=0 never, =2 from K = 512,
// otherwise from K = 1024.
int pair_min_k() {
  static const int k = [] {
    const char* e = getenv("MRN_GEMM_PAIR");
    return e && e[0] == '0' ? 1 << 30 : e && e[0] == '2' ? 512 : 1024;
  }();
  return k;
}

template <int BN, bool FP8>
cudaError_t launch_bn(const GemmPlan& p, cudaStream_t stream) {
  const GemmArgs& a = p.args;
  switch (a.epi) {
    case Epilogue::kBias:
      return launch_one<BN, FP8>(p, EpiBiasBf16{a.bias, a.scale}, stream);
    case Epilogue::kResidual:
      return launch_one<BN, FP8>(p, EpiResidual{a.bias, a.scale}, stream);
    case Epilogue::kGeluBf16:
      if constexpr (!FP8) return launch_one<BN, FP8>(p, EpiGelu<false>{a.bias, a.scale, a.inv_q}, stream);
      break;
    case Epilogue::kGeluE4m3:
      if constexpr (FP8) return launch_one<BN, FP8>(p, EpiGelu<true>{a.bias, a.scale, a.inv_q}, stream);
      break;
    case Epilogue::kGeluTanhBf16:
      if constexpr (!FP8) return launch_one<BN, FP8>(p, EpiGeluTanh<false>{a.bias, a.scale, a.inv_q}, stream);
      break;
    case Epilogue::kGeluTanhE4m3:
      if constexpr (FP8) return launch_one<BN, FP8>(p, EpiGeluTanh<true>{a.bias, a.scale, a.inv_q}, stream);
      break;
    default:
      break;
  }
  return cudaErrorInvalidValue;
}

template <bool FP8>
cudaError_t launch_fp8(const GemmPlan& p, cudaStream_t stream) {
  switch (p.bn) {
    case 256: return launch_bn<256, FP8>(p, stream);
    case 192: return launch_bn<192, FP8>(p, stream);
    case 128: return launch_bn<128, FP8>(p, stream);
    case 64: return launch_bn<64, FP8>(p, stream);
  }
  return cudaErrorInvalidValue;
}

template <int BN, bool FP8, class Epi>
cudaError_t prepare_one() {
  return cudaFuncSetAttribute(gemm_tc_kernel<BN, FP8, Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              ShapeOf<BN, Epi>::kSmemBytes);
}

template <int BN>
cudaError_t prepare_bn() {
  cudaError_t e;
  if ((e = prepare_one<BN, false, EpiBiasBf16>()) != cudaSuccess) return e;
  if ((e = prepare_one<BN, false, EpiResidual>()) != cudaSuccess) return e;
  if ((e = prepare_one<BN, false, EpiGelu<false>>()) != cudaSuccess) return e;
  if ((e = prepare_one<BN, false, EpiGeluTanh<false>>()) != cudaSuccess) return e;
  if ((e = prepare_one<BN, true, EpiGeluTanh<true>>()) != cudaSuccess) return e;
  if ((e = prepare_one<BN, true, EpiBiasBf16>()) != cudaSuccess) return e;
  if ((e = prepare_one<BN, true, EpiResidual>()) != cudaSuccess) return e;
  return prepare_one<BN, true, EpiGelu<true>>();
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
  if ((args.epi == Epilogue::kGeluE4m3 || args.epi == Epilogue::kGeluTanhE4m3) && !args.fp8) {
    snprintf(err, 256, "gemm: e4m3 GELU output is only planned for FP8 operands");
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
  // CTA pairs halve the operand bytes per FLOP, which pays where the main loop is long (FFN2,
  // K = 4d); with K = d the two CTAs' coupled epilogues cost more than that saves.
  plan->pair = args.n % 256 == 0 && args.k >= pair_min_k();
  // The memory-bound residual GEMMs with a short K (out-proj) run 128-column tiles with four
  // TMEM accumulators: the reduce-add stores drain behind three tiles of MMAs.
  if (!plan->pair && args.epi == Epilogue::kResidual && args.k < 1024 && args.n % 128 == 0) plan->bn = 128;
  if (!make_kmajor_map(&plan->map_a, args.a, eb, args.m, args.k, kTileM) ||
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
  if ((e = prepare_pair<false, EpiBiasBf16>()) != cudaSuccess) return e;
  if ((e = prepare_pair<false, EpiResidual>()) != cudaSuccess) return e;
  if ((e = prepare_pair<false, EpiGelu<false>>()) != cudaSuccess) return e;
  if ((e = prepare_pair<false, EpiGeluTanh<false>>()) != cudaSuccess) return e;
  if ((e = prepare_pair<true, EpiGeluTanh<true>>()) != cudaSuccess) return e;
  if ((e = prepare_pair<true, EpiBiasBf16>()) != cudaSuccess) return e;
  if ((e = prepare_pair<true, EpiResidual>()) != cudaSuccess) return e;
  if ((e = prepare_pair<true, EpiGelu<true>>()) != cudaSuccess) return e;
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
  if (plan.pair) return plan.args.fp8 ? launch_pair_epi<true>(plan, stream) : launch_pair_epi<false>(plan, stream);
  return plan.args.fp8 ? launch_fp8<true>(plan, stream) : launch_fp8<false>(plan, stream);
}

}  // namespace mrn
