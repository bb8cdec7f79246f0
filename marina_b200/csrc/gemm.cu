// Instantiations and host dispatch of the tcgen05 GEMM.
#include <stdio.h>
#include <stdlib.h>

#include "gemm.cuh"
#include "gemm.h"
#include "gemm_ln.cuh"
#include "gemm_mlp.cuh"
#include "gemm_norm.cuh"
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

bool pair_enabled() {
  static const bool on = [] {
    const char* e = getenv("MRN_GEMM_PAIR");
    return !(e && e[0] == '0');
  }();
  return on;
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

// ---- residual GEMM + LayerNorm (gemm_ln.cuh): one cluster of n / BN CTAs per row block
// `attr` has room for two attributes: the cluster shape and, when on, programmatic launch.
cudaLaunchConfig_t ln_config(dim3 grid, int threads, int smem, int cluster, cudaStream_t stream,
                             cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1 + pdl_attribute(attr + 1);
  return cfg;
}

template <int BN, bool FP8>
cudaError_t launch_ln_bn(const GemmPlan& p, cudaStream_t stream) {
  using S = LnShape<BN>;
  const GemmArgs& a = p.args;
  const LnParams lp{a.bias, a.gamma, a.beta, static_cast<const __half*>(a.out), a.scale, a.eps, a.ln_inv_q, a.n};
  cudaLaunchAttribute attr[2];
  const cudaLaunchConfig_t cfg = ln_config(dim3(p.grid, 1, 1), S::kThreads, S::kSmemBytes, p.cluster, stream, attr);
  return cudaLaunchKernelEx(&cfg, gemm_ln_kernel<BN, FP8, FP8>, p.map_a, p.map_b, p.map_out, p.map_aux, lp, a.m, a.k,
                            a.status);
}

cudaError_t launch_ln(const GemmPlan& p, cudaStream_t stream) {
  const bool f = p.args.fp8;
  switch (p.bn) {
    case 128: return f ? launch_ln_bn<128, true>(p, stream) : launch_ln_bn<128, false>(p, stream);
    case 96: return f ? launch_ln_bn<96, true>(p, stream) : launch_ln_bn<96, false>(p, stream);
    case 64: return f ? launch_ln_bn<64, true>(p, stream) : launch_ln_bn<64, false>(p, stream);
  }
  return cudaErrorInvalidValue;
}

// Clusters of `cluster` CTAs of this instantiation that fit on the device at once (0 if none).
template <int BN, bool FP8>
int ln_max_clusters(int cluster) {
  using S = LnShape<BN>;
  cudaLaunchAttribute attr[2];
  const cudaLaunchConfig_t cfg = ln_config(dim3(cluster, 1, 1), S::kThreads, S::kSmemBytes, cluster, nullptr, attr);
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, gemm_ln_kernel<BN, FP8, FP8>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

int ln_max_clusters(int bn, bool fp8, int cluster) {
  switch (bn) {
    case 128: return fp8 ? ln_max_clusters<128, true>(cluster) : ln_max_clusters<128, false>(cluster);
    case 96: return fp8 ? ln_max_clusters<96, true>(cluster) : ln_max_clusters<96, false>(cluster);
    case 64: return fp8 ? ln_max_clusters<64, true>(cluster) : ln_max_clusters<64, false>(cluster);
  }
  return 0;
}

template <int BN>
cudaError_t prepare_ln() {
  cudaError_t e = cudaFuncSetAttribute(gemm_ln_kernel<BN, false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       LnShape<BN>::kSmemBytes);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(gemm_ln_kernel<BN, true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              LnShape<BN>::kSmemBytes);
}

// ---- GEMM with the LayerNorm of A in the kernel (gemm_norm.cuh)
template <class Epi>
cudaError_t launch_norm(const GemmPlan& p, const Epi& epi, cudaStream_t stream) {
  using S = NormShape<Epi::kOutBytes, Epi::kWarps>;
  const GemmArgs& a = p.args;
  const NormA na{static_cast<const __half*>(a.norm_x), a.gamma, a.beta, a.eps, a.ln_inv_q};
  return launch_kernel(gemm_norm_kernel<Epi>, dim3(p.grid), dim3(S::kThreads), S::kSmemBytes, stream, p.map_b,
                       p.map_out, epi, na, a.m, a.n, a.status);
}

cudaError_t launch_norm_epi(const GemmPlan& p, cudaStream_t stream) {
  const GemmArgs& a = p.args;
  switch (a.epi) {
    case Epilogue::kBias: return launch_norm(p, EpiBiasBf16{a.bias, a.scale}, stream);
    case Epilogue::kGeluE4m3: return launch_norm(p, EpiGelu<true>{a.bias, a.scale, a.inv_q}, stream);
    case Epilogue::kGeluTanhE4m3: return launch_norm(p, EpiGeluTanh<true>{a.bias, a.scale, a.inv_q}, stream);
    default: break;
  }
  return cudaErrorInvalidValue;
}

template <class Epi>
cudaError_t prepare_norm() {
  return cudaFuncSetAttribute(gemm_norm_kernel<Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              NormShape<Epi::kOutBytes, Epi::kWarps>::kSmemBytes);
}

bool plan_norm(GemmPlan* plan, const GemmArgs& args, int num_sms, char* err) {
  if (!gemm_norm_supported(args)) {
    snprintf(err, 256, "gemm+norm: needs e4m3, K=%d, N%%256==0, bias/e4m3-GELU epilogue, aligned buffers (M=%d N=%d K=%d)",
             kNormK, args.m, args.n, args.k);
    return false;
  }
  plan->norm = true;
  plan->bn = 256;
  const bool e4m3_out = args.epi != Epilogue::kBias;
  if (!make_kmajor_map(&plan->map_b, args.b, 1, args.n, args.k, 128) ||
      !make_store_map(&plan->map_out, args.out,
                      e4m3_out ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, e4m3_out ? 1 : 2,
                      args.m, args.n, args.ldo)) {
    snprintf(err, 256, "gemm+norm: cuTensorMapEncodeTiled failed (M=%d N=%d K=%d)", args.m, args.n, args.k);
    return false;
  }
  const int units = ((args.m + 2 * kTileM - 1) / (2 * kTileM)) * (args.n / 256);
  const int pairs = num_sms / 2;
  plan->grid = 2 * (units < pairs ? units : pairs);
  return true;
}

// ---- the fused MLP block (gemm_mlp.cuh)
template <class Gelu>
cudaError_t launch_mlp(const MlpPlan& p, const Gelu& gelu, cudaStream_t stream) {
  const MlpArgs& a = p.args;
  return launch_kernel(gemm_mlp_kernel<Gelu>, dim3(p.grid), dim3(MlpShape::kThreads), MlpShape::kSmemBytes, stream,
                       p.map_h, p.map_w1, p.map_w2, static_cast<__half*>(a.x), gelu, EpiResidual{a.b2, a.s2}, a.m,
                       a.ff, a.status);
}

template <class Gelu>
cudaError_t prepare_mlp() {
  return cudaFuncSetAttribute(gemm_mlp_kernel<Gelu>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              MlpShape::kSmemBytes);
}

bool plan_ln(GemmPlan* plan, const GemmArgs& args, char* err) {
  const int eb = args.fp8 ? 1 : 2;
  plan->bn = gemm_ln_pick_bn(args.n);
  if (plan->bn == 0) {
    snprintf(err, 256, "gemm+layernorm: no CTA slice of 128, 96 or 64 columns splits d=%d into <= %d CTAs", args.n,
             kLnMaxCluster);
    return false;
  }
  if (args.ldo != args.n || args.ln_e4m3 != args.fp8 || !args.gamma || !args.beta || !args.ln_out ||
      (reinterpret_cast<uintptr_t>(args.gamma) & 15) != 0 || (reinterpret_cast<uintptr_t>(args.beta) & 15) != 0 ||
      (reinterpret_cast<uintptr_t>(args.ln_out) & 15) != 0) {
    snprintf(err, 256, "gemm+layernorm: needs ldo == N, aligned gamma/beta/h, and e4m3 h exactly with e4m3 operands");
    return false;
  }
  plan->cluster = args.n / plan->bn;
  if (!make_kmajor_map(&plan->map_a, args.a, eb, args.m, args.k, kTileM) ||
      !make_kmajor_map(&plan->map_b, args.b, eb, args.n, args.k, plan->bn) ||
      !make_store_map(&plan->map_out, args.out, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, args.m, args.n, args.n) ||
      !make_store_map(&plan->map_aux, args.ln_out,
                      args.ln_e4m3 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                      args.ln_e4m3 ? 1 : 2, args.m, args.n, args.n)) {
    snprintf(err, 256, "gemm+layernorm: cuTensorMapEncodeTiled failed (M=%d N=%d K=%d)", args.m, args.n, args.k);
    return false;
  }
  const int fit = ln_max_clusters(plan->bn, args.fp8, plan->cluster);
  if (fit <= 0) {
    snprintf(err, 256, "gemm+layernorm: clusters of %d CTAs do not fit on this device", plan->cluster);
    return false;
  }
  const int tiles = (args.m + kTileM - 1) / kTileM;
  plan->grid = plan->cluster * (tiles < fit ? tiles : fit);
  return true;
}

}  // namespace

int gemm_ln_pick_bn(int n) {
  for (int bn : {128, 96, 64})
    if (n % bn == 0 && n / bn <= kLnMaxCluster) return bn;
  return 0;
}

bool gemm_norm_supported(const GemmArgs& a) {
  auto aligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  return a.fp8 && a.k == kNormK && a.m > 0 && a.n > 0 && a.n % 256 == 0 && a.ldo >= a.n && a.ldo % 16 == 0 &&
         (a.epi == Epilogue::kBias || a.epi == Epilogue::kGeluE4m3 || a.epi == Epilogue::kGeluTanhE4m3) && a.norm_x &&
         a.gamma && a.beta && a.bias && a.out && aligned(a.norm_x) && aligned(a.gamma) && aligned(a.beta) &&
         aligned(a.bias) && aligned(a.out);
}

bool mlp_supported(const MlpArgs& a) {
  auto aligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  return a.m > 0 && a.d == kMlpD && a.ff >= 512 && a.ff % 256 == 0 && a.h && a.w1 && a.w2 && a.b1 && a.b2 && a.x &&
         aligned(a.h) && aligned(a.w1) && aligned(a.w2) && aligned(a.b1) && aligned(a.b2) && aligned(a.x);
}

bool mlp_plan(MlpPlan* plan, const MlpArgs& a, int num_sms, char* err) {
  if (!mlp_supported(a)) {
    snprintf(err, 256, "mlp: needs d = %d, ff a multiple of 256 (>= 512), aligned buffers (M=%d d=%d ff=%d)", kMlpD,
             a.m, a.d, a.ff);
    return false;
  }
  plan->args = a;
  if (!make_kmajor_map(&plan->map_h, a.h, 1, a.m, a.d, kTileM) ||
      !make_kmajor_map(&plan->map_w1, a.w1, 1, a.ff, a.d, MlpShape::kChunk) ||
      !make_kmajor_map(&plan->map_w2, a.w2, 1, a.d, a.ff, MlpShape::kOutCols)) {
    snprintf(err, 256, "mlp: cuTensorMapEncodeTiled failed (M=%d d=%d ff=%d)", a.m, a.d, a.ff);
    return false;
  }
  const int tiles = (a.m + kTileM - 1) / kTileM;
  const int clusters = num_sms / 2;
  plan->grid = 2 * (tiles < clusters ? tiles : clusters);
  return true;
}

cudaError_t mlp_launch(const MlpPlan& p, cudaStream_t stream) {
  const MlpArgs& a = p.args;
  if (a.tanh_gelu) return launch_mlp(p, EpiGeluTanh<true>{a.b1, a.s1, a.inv_q}, stream);
  return launch_mlp(p, EpiGelu<true>{a.b1, a.s1, a.inv_q}, stream);
}

int gemm_pick_bn(int n) {
  for (int bn : {256, 192, 128, 64})
    if (n % bn == 0) return bn;
  return 0;
}

bool gemm_plan(GemmPlan* plan, const GemmArgs& args, int num_sms, char* err) {
  plan->args = args;
  plan->pair = false;
  plan->norm = false;
  plan->cluster = 0;
  if (args.norm_x) return plan_norm(plan, args, num_sms, err);
  if (args.epi == Epilogue::kResidualLn) {
    if (args.m <= 0 || args.k <= 0 || (args.k * (args.fp8 ? 1 : 2)) % 16 != 0 ||
        (reinterpret_cast<uintptr_t>(args.out) & 15) != 0 || (reinterpret_cast<uintptr_t>(args.bias) & 15) != 0) {
      snprintf(err, 256, "gemm+layernorm: bad shape %dx%dx%d or misaligned x/bias", args.m, args.n, args.k);
      return false;
    }
    return plan_ln(plan, args, err);
  }
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
  plan->pair = pair_enabled() && args.n % 256 == 0 && args.k >= 1024;
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
    case Epilogue::kResidualLn:
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
  if ((e = prepare_ln<128>()) != cudaSuccess) return e;
  if ((e = prepare_ln<96>()) != cudaSuccess) return e;
  if ((e = prepare_ln<64>()) != cudaSuccess) return e;
  if ((e = prepare_mlp<EpiGelu<true>>()) != cudaSuccess) return e;
  if ((e = prepare_mlp<EpiGeluTanh<true>>()) != cudaSuccess) return e;
  if ((e = prepare_norm<EpiBiasBf16>()) != cudaSuccess) return e;
  if ((e = prepare_norm<EpiGelu<true>>()) != cudaSuccess) return e;
  if ((e = prepare_norm<EpiGeluTanh<true>>()) != cudaSuccess) return e;
  return prepare_bn<64>();
}

cudaError_t gemm_launch(const GemmPlan& plan, cudaStream_t stream) {
  if (plan.norm) return launch_norm_epi(plan, stream);
  if (plan.args.epi == Epilogue::kResidualLn) return launch_ln(plan, stream);
  if (plan.pair) return plan.args.fp8 ? launch_pair_epi<true>(plan, stream) : launch_pair_epi<false>(plan, stream);
  return plan.args.fp8 ? launch_fp8<true>(plan, stream) : launch_fp8<false>(plan, stream);
}

}  // namespace mrn
