// Host interface of the tcgen05 GEMM (gemm.cuh): a plan (tensor maps + launch shape) is
// built once per (buffer, batch bucket) and launched many times, including inside CUDA
// graphs.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

namespace mrn {

enum class Epilogue : int {
  kBias = 0,       // out bf16 = acc*scale + bias                  (QKV projection)
  kGeluBf16 = 1,   // out bf16 = GELU(acc*scale + bias)            (FFN1, bf16 activations)
  kGeluE4m3 = 2,   // out e4m3 = GELU(acc*scale + bias) * inv_q    (FFN1, FP8 activations)
  kResidual = 3,   // x f16 += acc*scale + bias                    (out-proj, FFN2)
  kGeluTanhBf16 = 5,  // kGeluBf16 with the tanh-form GELU             (FFN1 of Gelu::Tanh cards)
  kGeluTanhE4m3 = 6,  // kGeluE4m3 with the tanh-form GELU
  kGeluE4m3x2 = 7,    // out [M, 2N] = two-term e4m3 of GELU(acc*scale + bias) * inv_q: hi codes, then lo codes
  kGeluTanhE4m3x2 = 8,  // kGeluE4m3x2 with the tanh-form GELU
};

struct GemmArgs {
  const void* a = nullptr;  // activations [M, K], bf16 or e4m3, row-major
  const void* b = nullptr;  // weight [N, K], same type, row-major (PyTorch Linear layout)
  int m = 0, n = 0, k = 0;
  bool fp8 = false;          // operands are e4m3 (kind::f8f6f4) instead of bf16 (kind::f16)
  bool x2 = false;           // (fp8) A is two-term e4m3 [M, 2K]: each row's K hi codes, then its K lo codes
  int pair = -1;             // CTA pairs: -1 the planning rule, 0 never, 1 whenever N % 256 == 0
  Epilogue epi = Epilogue::kBias;
  void* out = nullptr;       // bf16 / e4m3 output, or the f16 residual stream
  int ldo = 0;               // row stride of `out` in elements
  const float* bias = nullptr;  // [N]
  float scale = 1.f;         // dequantisation of the accumulator (weight scale x activation scale)
  float inv_q = 1.f;         // 1 / output quantisation scale (kGeluE4m3)
  int* status = nullptr;     // device error word (first error wins)
};

struct GemmPlan {
  CUtensorMap map_a;
  CUtensorMap map_a2;  // x2: the lo codes of A (otherwise a copy of map_a)
  CUtensorMap map_b;
  CUtensorMap map_out;
  GemmArgs args;
  int bn = 0;
  int grid = 0;
  bool pair = false;  // 256 x 256 tiles on CTA pairs (tcgen05 cta_group::2)
};

// Widest supported N tile (256, 192, 128, 64) dividing n; 0 if none. Plans for N a multiple of
// 256 and M >= 128 rows x SMs run on CTA pairs for K >= 1024, and from K = 512 for the residual
// epilogue (bf16 or two-term e4m3 operands) and for the bias epilogue with bf16 operands on
// M >= 65,536 rows (MRN_GEMM_PAIR=0: never; =1: K >= 1024 at any M; =2: from K = 512 at any M).
// Without pairs, small batches take the narrowest tile whose tiles fit in one wave.
int gemm_pick_bn(int n);

// Validate shapes and alignment and build the tensor maps. `err` (>= 256 bytes) receives a
// message on failure.
bool gemm_plan(GemmPlan* plan, const GemmArgs& args, int num_sms, char* err);

// Opt every kernel instantiation into its dynamic shared memory size (once per device).
cudaError_t gemm_prepare_device();

cudaError_t gemm_launch(const GemmPlan& plan, cudaStream_t stream);

#ifdef MRN_TEST_HOOKS
// Test builds only: set, in stream order, the bounded waits' limit of the GEMM kernels and
// whether their TMA producers issue no loads (so that the MMA and epilogue waits run out).
cudaError_t gemm_test_hooks(unsigned long long wait_limit_ns, int no_loads, cudaStream_t stream);
#endif

// Algorithmic FLOPs of one launch (2·M·N·K).
inline double gemm_flops(const GemmArgs& a) { return 2.0 * a.m * static_cast<double>(a.n) * a.k; }

}  // namespace mrn
