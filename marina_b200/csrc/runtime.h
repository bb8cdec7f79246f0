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
  cudaGraphExec_t graph = nullptr;
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

