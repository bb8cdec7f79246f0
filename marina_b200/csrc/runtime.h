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
  std::vector<GemmPlan> plans;  // 4 per layer (QKV, out-proj, FFN1, FFN2), then the value head's first layer
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

  // Ordering of the passes on this context's buffers across streams: every entry point that
  // enqueues a pass makes its stream wait for `pass_done` when the previous pass ran on another
  // stream (`pass_stream`), and records `pass_done` on its own stream after the pass.
  cudaEvent_t pass_done = nullptr;
  cudaStream_t pass_stream = nullptr;
  bool pass_recorded = false;
  // Device address of static_forward.cu's scratch array on this context's device, looked up in
  // mrn_create with the device current (nullptr, with the reason in static_error, if that failed).
  uint8_t* static_scratch = nullptr;
  std::string static_error;

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
// Before a pass on stream `s`: wait for the context's previous pass if it was enqueued on another
// stream (no-op while `s` is being captured into a graph: ordering captured work is the
// capturer's). After the pass: record its completion on `s`. Both return an mrn_status.
int begin_pass(mrn_ctx* c, cudaStream_t s);
int end_pass(mrn_ctx* c, cudaStream_t s);
// Looks up the static scratch array's device address for c (static_forward.cu); called by
// mrn_create with c's device current.
void static_scratch_setup(mrn_ctx* c);
// The four GEMMs of layer `l` over `rows` rows: QKV, out-proj, FFN1, FFN2.
void layer_gemm_args(const mrn_ctx* c, int l, int rows, const LayerBuffers& b, GemmArgs (&g)[4]);
// Whether the kernels after the first of a pass over `positions` positions launch with
// programmatic dependent launch (environment MRN_PDL: 1 always, 0 never; by default for small
// batches).
bool pdl_enabled(int positions);
// The LayerNorm after a residual GEMM: norm2 of layer `l` (site 0) or norm1 of layer l + 1
// (site 1), from x into h.
cudaError_t launch_site_layernorm(const mrn_ctx* c, int l, int site, const LayerBuffers& b, int rows,
                                  cudaStream_t s);
}  // namespace mrn
