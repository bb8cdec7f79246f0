// Kernel-level entry points for the GPU test-suite (include/marina_b200_test.h), built into their
// own library (libmarina_b200_test.so) together with the evaluator's kernels compiled with
// MRN_TEST_HOOKS: each runs one kernel on caller-owned device buffers, so every kernel can be
// checked on its own against a plain fp32 reference before the whole forward pass is compared
// with the CPU oracle, and one makes a GEMM's bounded waits run out on purpose.
#include <stdio.h>
#include <string.h>

#include "../../include/marina_b200.h"
#include "../../include/marina_b200_test.h"
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

MRN_TEST_API const char* mrn_test_last_error(void) { return g_test_error; }

MRN_TEST_API int mrn_test_gemm(int fp8, int epilogue, int pair, const void* a, const void* b, const float* bias,
                               void* out, int ldo, int m, int n, int k, float scale, float inv_q, int* status,
                               void* stream) {
  if (!prepare()) return fail("gemm_prepare_device failed");
  if (pair < -1 || pair > 1) return fail("pair must be -1 (the planning rule), 0 (single CTAs) or 1 (CTA pairs)");
  mrn::GemmArgs args;
  args.a = a;
  args.b = b;
  args.m = m;
  args.n = n;
  args.k = k;
  if (fp8 < 0 || fp8 > 2) return fail("fp8 must be 0 (bf16), 1 (e4m3) or 2 (two-term e4m3 A)");
  args.fp8 = fp8 != 0;
  args.x2 = fp8 == 2;
  args.pair = pair;
  args.epi = static_cast<mrn::Epilogue>(epilogue);
  args.out = out;
  args.ldo = ldo;
  args.bias = bias;
  args.scale = scale;
  args.inv_q = inv_q;
  args.status = status;
  return run(args, stream);
}

MRN_TEST_API int mrn_test_gemm_wait_expiry(unsigned long long wait_limit_ns, const void* a, const void* b,
                                           const float* bias, void* out, int m, int n, int k, int* status,
                                           void* stream) {
  if (!prepare()) return fail("gemm_prepare_device failed");
  if (wait_limit_ns < 1000 || wait_limit_ns > 2000000000ull) return fail("wait limit outside [1 us, 2 s]");
  mrn::GemmArgs args;
  args.a = a;
  args.b = b;
  args.m = m;
  args.n = n;
  args.k = k;
  args.epi = mrn::Epilogue::kBias;
  args.out = out;
  args.ldo = n;
  args.bias = bias;
  args.status = status;
  mrn::GemmPlan plan;
  char err[256];
  if (!mrn::gemm_plan(&plan, args, num_sms(), err)) return fail(err);
  if (plan.pair) return fail("the expiry test runs the single-CTA kernel: use K < 1024");
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = mrn::gemm_test_hooks(wait_limit_ns, 1, s);
  if (e == cudaSuccess) e = mrn::gemm_launch(plan, s);
  // Restore the defaults in stream order whatever happened to the launch.
  const cudaError_t r = mrn::gemm_test_hooks(2000000000ull, 0, s);
  if (e == cudaSuccess) e = r;
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    snprintf(g_test_error, sizeof(g_test_error), "expiry test: %s", cudaGetErrorString(e));
    return MRN_ERR_CUDA;
  }
  int word = 0;
  if ((e = cudaMemcpy(&word, status, sizeof(word), cudaMemcpyDeviceToHost)) != cudaSuccess) {
    snprintf(g_test_error, sizeof(g_test_error), "expiry test: %s", cudaGetErrorString(e));
    return MRN_ERR_CUDA;
  }
  if (word == 0) return MRN_OK;
  snprintf(g_test_error, sizeof(g_test_error), "device-side wait gave up in a GEMM (code %d)", word);
  return MRN_ERR_DEVICE_FAULT;
}

MRN_TEST_API int mrn_test_attention(const void* qkv, void* out, int positions, int d, int heads, int e4m3,
                                    float inv_q, int* status, void* stream) {
  static bool prepared = false;
  if (!prepared) {
    if (mrn::prepare_attention() != cudaSuccess) return fail("prepare_attention failed");
    prepared = true;
  }
  if (heads <= 0 || d % heads != 0) return fail("attention: d must be a multiple of heads");
  if (e4m3 < 0 || e4m3 > 2) return fail("e4m3 must be 0, 1 or 2");
  const mrn::AttentionParams ap{qkv, out, static_cast<mrn::ActType>(e4m3), inv_q, 65, d, heads, status};
  const cudaError_t e = mrn::launch_attention(ap, positions, d / heads, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    snprintf(g_test_error, sizeof(g_test_error), "attention launch: %s", cudaGetErrorString(e));
    return MRN_ERR_CUDA;
  }
  return MRN_OK;
}

MRN_TEST_API int mrn_test_layernorm(const void* x, const float* gamma, const float* beta, float eps, int e4m3,
                                    float inv_q, void* out, int rows, int d, void* stream) {
  if (e4m3 < 0 || e4m3 > 2) return fail("e4m3 must be 0, 1 or 2");
  const mrn::NormParams np{gamma, beta, eps, out, static_cast<mrn::ActType>(e4m3), inv_q};
  const cudaError_t e = mrn::launch_layernorm(static_cast<const __half*>(x), np, rows, d, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    snprintf(g_test_error, sizeof(g_test_error), "layernorm launch: %s", cudaGetErrorString(e));
    return MRN_ERR_CUDA;
  }
  return MRN_OK;
}

}  // extern "C"
