// The evaluator context (one per GPU) and its per-bucket launch plans, shared by the
// runtime's translation units.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>

#include <map>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include "gemm.h"
#include "kernels.cuh"

struct mrn_ctx;

namespace mrn {

struct DevLayer {
  float *n1g = nullptr, *n1b = nullptr, *n2g = nullptr, *n2b = nullptr;
  void *w_qkv = nullptr, *w_o = nullptr, *w_1 = nullptr, *w_2 = nullptr;
  float *b_qkv = nullptr, *b_o = nullptr, *b_1 = nullptr, *b_2 = nullptr;
  float ws[4] = {1, 1, 1, 1};  // weight dequantisation scale: qkv, out, ff1, ff2
  float as[4] = {1, 1, 1, 1};  // activation scales: norm1 out, attention out, norm2 out, GELU out
};

struct Bucket {
  int positions = 0;
  std::vector<GemmPlan> plans;  // 4 per layer, then the value head's first layer
  // Per layer: [2l] a LayerNorm launch (norm2) follows out-proj, [2l+1] one (the next layer's
  // norm1) follows FFN2. 0 where the norm runs inside a GEMM: in the consuming GEMM's A operand
  // (gemm_norm.cuh) or in the residual GEMM's epilogue (gemm_ln.cuh).
  std::vector<uint8_t> ln_launch;
  bool embed_norm = true;  // the embedding kernel writes layer 0's norm1 (its QKV does not normalise A)
  std::vector<MlpPlan> mlp;  // per layer when FFN1 + FFN2 run as one fused MLP launch (else empty)
  cudaGraphExec_t graph = nullptr;
};

// Buffers one forward pass runs on (the context's own, or the static scratch's).
struct LayerBuffers {
  void* h;
  void* qkv;
  void* attn;
  void* ff;
  __half* x;
};

// Per kernel class timing of one eager pass (mrn_profile).
struct Profiler {
  cudaStream_t stream;
  std::vector<std::pair<int, std::pair<cudaEvent_t, cudaEvent_t>>> marks;
  int pending = -1;
  cudaEvent_t start_ev = nullptr;
  void begin(int cls) {
    pending = cls;
    cudaEventCreate(&start_ev);
    cudaEventRecord(start_ev, stream);
  }
  void end() {
    cudaEvent_t e;
    cudaEventCreate(&e);
    cudaEventRecord(e, stream);
    marks.push_back({pending, {start_ev, e}});
  }
};

}  // namespace mrn

struct mrn_ctx {
  int device = 0;
  int precision = 0;
  int max_batch = 0;
  int max_bucket = 0;
  int num_sms = 0;
  int d = 0, layers = 0, heads = 0, dff = 0, t = 0, square_start = 0;
  float eps = 1e-5f;
  int gelu = 0;
  mrn::ActType act = mrn::ActType::kBf16;
  size_t act_bytes = 2;
  std::mutex mu;
  cudaStream_t stream = nullptr;
  std::vector<void*> allocations;

  // weights
  float *piece = nullptr, *square = nullptr, *state = nullptr, *cast_w = nullptr, *cast_b = nullptr, *ep = nullptr;
  std::vector<mrn::DevLayer> dl;
  float *fn_g = nullptr, *fn_b = nullptr, *pn_g = nullptr, *pn_b = nullptr, *pw = nullptr, *pb = nullptr;
  float *vn_g = nullptr, *vn_b = nullptr, *vb1 = nullptr, *vw2 = nullptr, *vb2 = nullptr;
  __nv_bfloat16* vw1 = nullptr;

  // activations and I/O
  uint8_t* boards = nullptr;
  int32_t* legal = nullptr;
  __half* x = nullptr;  // residual stream [R, d], f16
  void* h = nullptr;
  __nv_bfloat16* qkv = nullptr;
  void* attn = nullptr;
  void* ff = nullptr;
  __nv_bfloat16* vnorm = nullptr;
  __nv_bfloat16* vhid = nullptr;
  float* priors = nullptr;
  float* wdl = nullptr;
  int* status = nullptr;
  float* logits = nullptr;  // [max_bucket, 4672], allocated by the first mrn_logits
  __half* priors16 = nullptr;  // [max_bucket, 224], allocated by the first mrn_evaluate_f16
  // pinned staging
  uint8_t* h_boards = nullptr;
  int32_t* h_legal = nullptr;
  float* h_priors = nullptr;
  float* h_wdl = nullptr;
  int* h_status = nullptr;

  std::map<int, mrn::Bucket> buckets;
  std::string describe;
  std::string last_error;

  int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    last_error = buf;
    return code;
  }
};

namespace mrn {
// The four GEMMs of layer `l` over `rows` rows: QKV, out-proj, FFN1, FFN2. With `norm`, QKV and
// FFN1 compute norm1 / norm2 of x themselves where the normalised-A kernel supports the shape.
// With `fuse`, out-proj carries norm2 and FFN2 (all layers but the last) the next layer's norm1 as
// the fused residual + LayerNorm epilogue, unless the consuming GEMM normalises A itself.
// With `mlp`, FFN1 and FFN2 are planned for the fused MLP kernel (mlp_args): FFN1 reads h and FFN2
// carries no LayerNorm.
void layer_gemm_args(const mrn_ctx* c, int l, int rows, const LayerBuffers& b, bool fuse, bool norm, bool mlp,
                     GemmArgs (&g)[4]);
// The fused MLP of a layer from its FFN1 and FFN2 arguments; false where the kernel does not
// support the layer (not e4m3, d != 512, ...).
bool mlp_args(const GemmArgs& ffn1, const GemmArgs& ffn2, MlpArgs* out);
// Whether FFN1 + FFN2 run as one fused launch (environment MRN_MLP=1; off by default).
bool mlp_enabled();
// Whether the kernels after the first of a pass over `positions` positions launch with
// programmatic dependent launch (environment MRN_PDL: 1 always, 0 never; by default for small
// batches).
bool pdl_enabled(int positions);
// Whether layer l's QKV GEMM computes norm1 itself (under the same `norm` setting).
bool qkv_normalises(const mrn_ctx* c, int l, int rows, const LayerBuffers& b, bool norm);
// Whether plans use the fused residual + LayerNorm epilogue (environment MRN_GEMM_LN=1; off by default).
bool ln_fusion_enabled();
// Whether QKV and FFN1 normalise their A operand in the kernel (environment MRN_GEMM_NORM=1; off by
// default: the CTA-pair kernel it needs is slower at K = d than LayerNorm launch + single-CTA GEMM).
bool norm_a_enabled();
// The LayerNorm launch that stands in for an unfused site: norm2 of layer `l` (site 0) or norm1 of
// layer l + 1 (site 1), from x into h.
cudaError_t launch_site_layernorm(const mrn_ctx* c, int l, int site, const LayerBuffers& b, int rows,
                                  cudaStream_t s);
}  // namespace mrn
