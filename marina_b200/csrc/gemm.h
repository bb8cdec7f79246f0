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
  kResidualLn = 4, // kResidual, then h = LN(x)*gamma + beta       (out-proj -> norm2, FFN2 -> norm1)
  kGeluTanhBf16 = 5,  // kGeluBf16 with the tanh-form GELU             (FFN1 of Gelu::Tanh cards)
  kGeluTanhE4m3 = 6,  // kGeluE4m3 with the tanh-form GELU
};

struct GemmArgs {
  const void* a = nullptr;  // activations [M, K], bf16 or e4m3, row-major
  const void* b = nullptr;  // weight [N, K], same type, row-major (PyTorch Linear layout)
  int m = 0, n = 0, k = 0;
  bool fp8 = false;          // operands are e4m3 (kind::f8f6f4) instead of bf16 (kind::f16)
  Epilogue epi = Epilogue::kBias;
  void* out = nullptr;       // bf16 / e4m3 output, or the f16 residual stream
  int ldo = 0;               // row stride of `out` in elements
  const float* bias = nullptr;  // [N]
  float scale = 1.f;         // dequantisation of the accumulator (weight scale x activation scale)
  float inv_q = 1.f;         // 1 / output quantisation scale (kGeluE4m3)
  int* status = nullptr;     // device error word (first error wins)
  // kResidualLn: the LayerNorm of the updated rows of `out` (N = d, ldo = d). With `norm_x`:
  // the LayerNorm that produces A (K = d).
  const float* gamma = nullptr;  // [N], or [K] with norm_x
  const float* beta = nullptr;   // [N], or [K] with norm_x
  float eps = 1e-5f;
  void* ln_out = nullptr;        // h [M, N], bf16 or e4m3
  bool ln_e4m3 = false;
  float ln_inv_q = 1.f;          // 1 / e4m3 scale of h (kResidualLn) or of the normalised A
  // Normalised A (e4m3 operands, K = 512, N a multiple of 256; epilogues kBias, kGeluE4m3,
  // kGeluTanhE4m3): A = e4m3((LN(norm_x) * gamma + beta) * ln_inv_q) is computed inside the
  // kernel from the f16 residual stream norm_x [M, K], and `a` is not read.
  const void* norm_x = nullptr;
};

struct GemmPlan {
  CUtensorMap map_a;
  CUtensorMap map_b;
  CUtensorMap map_out;
  GemmArgs args;
  int bn = 0;
  int grid = 0;
  bool pair = false;  // 256 x 256 tiles on CTA pairs (tcgen05 cta_group::2)
  CUtensorMap map_aux;  // kResidualLn: the h store map
  int cluster = 0;      // kResidualLn: CTAs per row block (N / bn)
  bool norm = false;    // A normalised in the kernel (gemm_norm.cuh)
};

// Widest supported N tile (256, 192, 128, 64) dividing n; 0 if none. Plans for N a multiple of
// 256 and K >= 1024 run on CTA pairs unless the environment sets MRN_GEMM_PAIR=0.
int gemm_pick_bn(int n);

// kResidualLn: the N slice of one CTA (128, 96 or 64 dividing n with n / slice <= 8); 0 if none.
int gemm_ln_pick_bn(int n);

// Whether gemm_plan accepts `norm_x` for this shape and epilogue (the kernel is instantiated for
// K = 512 only).
bool gemm_norm_supported(const GemmArgs& args);

// Validate shapes and alignment and build the tensor maps. `err` (>= 256 bytes) receives a
// message on failure.
bool gemm_plan(GemmPlan* plan, const GemmArgs& args, int num_sms, char* err);

// Opt every kernel instantiation into its dynamic shared memory size (once per device).
cudaError_t gemm_prepare_device();

cudaError_t gemm_launch(const GemmPlan& plan, cudaStream_t stream);

// The encoder's MLP block in one launch (gemm_mlp.cuh): x += e4m3(GELU(h · w1^T · s1 + b1) · inv_q)
// · w2^T · s2 + b2, e4m3 operands, d = 512, ff a multiple of 256; the [M, ff] hidden tensor stays
// on chip.
struct MlpArgs {
  const void* h = nullptr;    // [M, d] e4m3
  const void* w1 = nullptr;   // [ff, d] e4m3
  const void* w2 = nullptr;   // [d, ff] e4m3
  const float* b1 = nullptr;  // [ff]
  const float* b2 = nullptr;  // [d]
  void* x = nullptr;          // [M, d] f16 residual stream
  int m = 0, d = 0, ff = 0;
  float s1 = 1.f, s2 = 1.f, inv_q = 1.f;
  bool tanh_gelu = false;     // the card's tanh-form GELU
  int* status = nullptr;
};

struct MlpPlan {
  CUtensorMap map_h, map_w1, map_w2;
  MlpArgs args;
  int grid = 0;
};

bool mlp_supported(const MlpArgs& args);
bool mlp_plan(MlpPlan* plan, const MlpArgs& args, int num_sms, char* err);
cudaError_t mlp_launch(const MlpPlan& plan, cudaStream_t stream);

// Algorithmic FLOPs of one launch (2·M·N·K).
inline double gemm_flops(const GemmArgs& a) { return 2.0 * a.m * static_cast<double>(a.n) * a.k; }

}  // namespace mrn
