// Kernel-level entry points for the GPU test-suite: each runs one kernel of the evaluator on
// caller-owned device buffers, so every kernel can be checked on its own against a plain
// fp32 reference before the whole forward pass is compared with the CPU oracle.
#include <stdio.h>
#include <string.h>

#include "../../include/marina_b200.h"
#include "gemm.h"
#include "kernels.cuh"

namespace {
thread_local char g_test_error[512];

int fail(const char* msg) {
  snprintf(g_test_error, sizeof(g_test_error), "%s", msg);
  return MRN_ERR_ARGUMENT;
}

int num_sms() {
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

bool prepare() {
  static bool prepared = false;
  if (!prepared) {
    if (mrn::gemm_prepare_device() != cudaSuccess) return false;
    prepared = true;
  }
  return true;
}

int run(const mrn::GemmArgs& args, void* stream) {
  mrn::GemmPlan plan;
  char err[256];
  if (!mrn::gemm_plan(&plan, args, num_sms(), err)) return fail(err);
  const cudaError_t e = mrn::gemm_launch(plan, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    snprintf(g_test_error, sizeof(g_test_error), "gemm launch: %s", cudaGetErrorString(e));
    return MRN_ERR_CUDA;
  }
  return MRN_OK;
}
}  // namespace

extern "C" {

const char* mrn_test_last_error(void) { return g_test_error; }

int mrn_test_gemm(int fp8, int epilogue, const void* a, const void* b, const float* bias, void* out, int ldo, int m,
                  int n, int k, float scale, float inv_q, int* status, void* stream) {
  if (!prepare()) return fail("gemm_prepare_device failed");
  mrn::GemmArgs args;
  args.a = a;
  args.b = b;
  args.m = m;
  args.n = n;
  args.k = k;
  args.fp8 = fp8 != 0;
  args.epi = static_cast<mrn::Epilogue>(epilogue);
  args.out = out;
  args.ldo = ldo;
  args.bias = bias;
  args.scale = scale;
  args.inv_q = inv_q;
  args.status = status;
  if (args.epi == mrn::Epilogue::kResidualLn) return fail("epilogue 4 goes through mrn_test_gemm_ln");
  return run(args, stream);
}

int mrn_test_gemm_ln(int fp8, const void* a, const void* b, const float* bias, const float* gamma, const float* beta,
                     void* x, void* h, int m, int d, int k, float scale, float eps, float inv_q, int* status,
                     void* stream) {
  if (!prepare()) return fail("gemm_prepare_device failed");
  mrn::GemmArgs args;
  args.a = a;
  args.b = b;
  args.m = m;
  args.n = d;
  args.k = k;
  args.fp8 = fp8 != 0;
  args.epi = mrn::Epilogue::kResidualLn;
  args.out = x;
  args.ldo = d;
  args.bias = bias;
  args.scale = scale;
  args.status = status;
  args.gamma = gamma;
  args.beta = beta;
  args.eps = eps;
  args.ln_out = h;
  args.ln_e4m3 = fp8 != 0;
  args.ln_inv_q = inv_q;
  return run(args, stream);
}

int mrn_test_gemm_norm(int epilogue, const void* x, const float* gamma, const float* beta, float eps, float a_inv_q,
                       const void* b, const float* bias, void* out, int ldo, int m, int n, int k, float scale,
                       float inv_q, int* status, void* stream) {
  if (!prepare()) return fail("gemm_prepare_device failed");
  mrn::GemmArgs args;
  args.b = b;
  args.m = m;
  args.n = n;
  args.k = k;
  args.fp8 = true;
  args.epi = static_cast<mrn::Epilogue>(epilogue);
  args.out = out;
  args.ldo = ldo;
  args.bias = bias;
  args.scale = scale;
  args.inv_q = inv_q;
  args.status = status;
  args.norm_x = x;
  args.gamma = gamma;
  args.beta = beta;
  args.eps = eps;
  args.ln_inv_q = a_inv_q;
  return run(args, stream);
}

int mrn_test_mlp(int tanh_gelu, const void* h, const void* w1, const float* b1, const void* w2, const float* b2,
                 void* x, int m, int d, int ff, float s1, float inv_q, float s2, int* status, void* stream) {
  if (!prepare()) return fail("gemm_prepare_device failed");
  mrn::MlpArgs a;
  a.h = h, a.w1 = w1, a.w2 = w2, a.b1 = b1, a.b2 = b2, a.x = x;
  a.m = m, a.d = d, a.ff = ff, a.s1 = s1, a.s2 = s2, a.inv_q = inv_q, a.tanh_gelu = tanh_gelu != 0;
  a.status = status;
  mrn::MlpPlan plan;
  char err[256];
  if (!mrn::mlp_plan(&plan, a, num_sms(), err)) return fail(err);
  const cudaError_t e = mrn::mlp_launch(plan, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    snprintf(g_test_error, sizeof(g_test_error), "mlp launch: %s", cudaGetErrorString(e));
    return MRN_ERR_CUDA;
  }
  return MRN_OK;
}

int mrn_test_attention(const void* qkv, void* out, int positions, int d, int heads, int e4m3, float inv_q, int* status,
                       void* stream) {
  static bool prepared = false;
  if (!prepared) {
    if (mrn::prepare_attention() != cudaSuccess) return fail("prepare_attention failed");
    prepared = true;
  }
  if (heads <= 0 || d % heads != 0) return fail("attention: d must be a multiple of heads");
  const mrn::AttentionParams ap{qkv, out, e4m3 ? mrn::ActType::kE4m3 : mrn::ActType::kBf16, inv_q, 65, d, heads, status};
  const cudaError_t e = mrn::launch_attention(ap, positions, d / heads, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    snprintf(g_test_error, sizeof(g_test_error), "attention launch: %s", cudaGetErrorString(e));
    return MRN_ERR_CUDA;
  }
  return MRN_OK;
}

int mrn_test_layernorm(const void* x, const float* gamma, const float* beta, float eps, int e4m3, float inv_q,
                       void* out, int rows, int d, void* stream) {
  const mrn::NormParams np{gamma, beta, eps, out, e4m3 ? mrn::ActType::kE4m3 : mrn::ActType::kBf16, inv_q};
  const cudaError_t e = mrn::launch_layernorm(static_cast<const __half*>(x), np, rows, d, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    snprintf(g_test_error, sizeof(g_test_error), "layernorm launch: %s", cudaGetErrorString(e));
    return MRN_ERR_CUDA;
  }
  return MRN_OK;
}

}  // extern "C"
