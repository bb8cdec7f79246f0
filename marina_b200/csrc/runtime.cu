// The evaluator's runtime and C ABI (include/marina_b200.h): one context per GPU holding a
// full weight replica in the precision's device layout, activation buffers sized for the
// context's largest batch, pinned staging, and one CUDA graph per batch bucket that replays
// the whole forward pass (src/net/cuda/mod.rs:612-700 captures the same per bucket).
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/marina_b200.h"
#include "gemm.h"
#include "kernels.cuh"
#include "launch.h"
#include "runtime.h"

namespace {

using mrn::ActType;
using mrn::Epilogue;
using mrn::GemmArgs;
using mrn::GemmPlan;

constexpr float kE4m3Max = 448.f;  // largest finite e4m3 (src/net/cuda/mod.rs:86-87)
constexpr float kFp8Margin = 1.25f;  // headroom over the calibration maxima (:83-85)
constexpr int kTokens = 65;  // board mode: one state token, 64 squares (src/net/model.rs:17)

thread_local std::string g_create_error;

using mrn::Bucket;
using mrn::DevLayer;
using mrn::Profiler;

}  // namespace

namespace {

// Batch sizes a context captures a pass for: powers of two up to 256, then multiples of 128 (a
// search's calls of a few thousand leaves pad by at most 128 positions).
int bucket_for(int n) {
  if (n <= 256) {
    int b = 1;
    while (b < n) b <<= 1;
    return b;
  }
  return (n + 127) / 128 * 128;
}

#define CK(call)                                                                                     \
  do {                                                                                               \
    const cudaError_t e_ = (call);                                                                   \
    if (e_ != cudaSuccess) return c->fail(MRN_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_));   \
  } while (0)

template <class T>
int dev_alloc(mrn_ctx* c, T** p, size_t bytes) {
  void* v = nullptr;
  const cudaError_t e = cudaMalloc(&v, bytes < 256 ? 256 : bytes);
  if (e != cudaSuccess) return c->fail(MRN_ERR_CUDA, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
  c->allocations.push_back(v);
  *p = static_cast<T*>(v);
  return MRN_OK;
}

int upload_f32(mrn_ctx* c, float** dst, const float* src, size_t count) {
  int rc = dev_alloc(c, dst, count * sizeof(float));
  if (rc) return rc;
  CK(cudaMemcpy(*dst, src, count * sizeof(float), cudaMemcpyHostToDevice));
  return MRN_OK;
}

// e4m3 code -> value (sign, 4-bit exponent with bias 7, 3-bit mantissa; exponent 0 is
// subnormal; 0x7f / 0xff are NaN).
float e4m3_value(uint8_t code) {
  const int sign = code >> 7, exp = (code >> 3) & 15, man = code & 7;
  float v;
  if ((code & 0x7f) == 0x7f)
    v = NAN;
  else if (exp == 0)
    v = ldexpf(static_cast<float>(man) / 8.f, -6);
  else
    v = ldexpf(1.f + static_cast<float>(man) / 8.f, exp - 7);
  return sign ? -v : v;
}

// Upload a Linear's weight [out, in] in the precision's GEMM operand format and return its
// dequantisation scale. FP8 modes quantise with one scale per matrix, amax / 448, as the
// reference's FP8 path (src/net/cuda/mod.rs:376-405): code = e4m3(w * (1 / scale)).
int upload_weight(mrn_ctx* c, void** dst, const float* w, size_t count, float* scale) {
  if (c->precision == MRN_PRECISION_BF16) {
    std::vector<__nv_bfloat16> q(count);
    for (size_t i = 0; i < count; ++i) q[i] = __float2bfloat16(w[i]);
    int rc = dev_alloc(c, dst, count * 2);
    if (rc) return rc;
    CK(cudaMemcpy(*dst, q.data(), count * 2, cudaMemcpyHostToDevice));
    *scale = 1.f;
    return MRN_OK;
  }
  float amax = 0.f;
  for (size_t i = 0; i < count; ++i) amax = fmaxf(amax, fabsf(w[i]));
  const float s = fmaxf(amax / kE4m3Max, 1.17549435e-38f);
  const float inv = 1.f / s;
  std::vector<uint8_t> codes(count);
  for (size_t i = 0; i < count; ++i)
    codes[i] = static_cast<uint8_t>(__nv_cvt_float_to_fp8(w[i] * inv, __NV_SATFINITE, __NV_E4M3));
  *scale = s;
  if (c->precision == MRN_PRECISION_FP8 || c->precision == MRN_PRECISION_FP8_X2) {
    int rc = dev_alloc(c, dst, count);
    if (rc) return rc;
    CK(cudaMemcpy(*dst, codes.data(), count, cudaMemcpyHostToDevice));
    return MRN_OK;
  }
  // MRN_PRECISION_FP8_WEIGHTS: the codes as exact bf16 values, scale applied in the epilogue.
  float lut[256];
  for (int i = 0; i < 256; ++i) lut[i] = e4m3_value(static_cast<uint8_t>(i));
  std::vector<__nv_bfloat16> q(count);
  for (size_t i = 0; i < count; ++i) q[i] = __float2bfloat16(lut[codes[i]]);
  int rc = dev_alloc(c, dst, count * 2);
  if (rc) return rc;
  CK(cudaMemcpy(*dst, q.data(), count * 2, cudaMemcpyHostToDevice));
  return MRN_OK;
}

bool finite_all(const float* p, size_t n) {
  for (size_t i = 0; i < n; ++i)
    if (!isfinite(p[i])) return false;
  return true;
}

int check_weights(mrn_ctx* c, const mrn_weights* w) {
  const size_t d = c->d, ff = c->dff;
  struct Item {
    const char* name;
    const float* p;
    size_t n;
  };
  std::vector<Item> items = {
      {"piece_embed.weight", w->piece_embed, 13 * d},
      {"square_embed.weight", w->square_embed, 64 * d},
      {"state_embed", w->state_embed, d},
      {"castling_proj.weight", w->castling_proj.weight, 4 * d},
      {"castling_proj.bias", w->castling_proj.bias, d},
      {"en_passant_embed.weight", w->en_passant_embed, 9 * d},
      {"final_norm.weight", w->final_norm.weight, d},
      {"final_norm.bias", w->final_norm.bias, d},
      {"policy_head.norm.weight", w->policy_norm.weight, d},
      {"policy_head.norm.bias", w->policy_norm.bias, d},
      {"policy_head.proj.weight", w->policy_proj.weight, 73 * d},
      {"policy_head.proj.bias", w->policy_proj.bias, 73},
      {"value_head.norm.weight", w->value_norm.weight, d},
      {"value_head.norm.bias", w->value_norm.bias, d},
      {"value_head.ff.0.weight", w->value_ff1.weight, d * d},
      {"value_head.ff.0.bias", w->value_ff1.bias, d},
      {"value_head.ff.2.weight", w->value_ff2.weight, 3 * d},
      {"value_head.ff.2.bias", w->value_ff2.bias, 3},
  };
  if (!w->layers) return c->fail(MRN_ERR_ARGUMENT, "weights: layers is NULL");
  for (int l = 0; l < c->layers; ++l) {
    const mrn_layer& L = w->layers[l];
    items.push_back({"norm1.weight", L.norm1.weight, d});
    items.push_back({"norm1.bias", L.norm1.bias, d});
    items.push_back({"self_attn.in_proj_weight", L.in_proj.weight, 3 * d * d});
    items.push_back({"self_attn.in_proj_bias", L.in_proj.bias, 3 * d});
    items.push_back({"self_attn.out_proj.weight", L.out_proj.weight, d * d});
    items.push_back({"self_attn.out_proj.bias", L.out_proj.bias, d});
    items.push_back({"norm2.weight", L.norm2.weight, d});
    items.push_back({"norm2.bias", L.norm2.bias, d});
    items.push_back({"linear1.weight", L.linear1.weight, ff * d});
    items.push_back({"linear1.bias", L.linear1.bias, ff});
    items.push_back({"linear2.weight", L.linear2.weight, d * ff});
    items.push_back({"linear2.bias", L.linear2.bias, d});
  }
  for (const Item& it : items) {
    if (!it.p) return c->fail(MRN_ERR_ARGUMENT, "weights: tensor %s is missing (NULL)", it.name);
    if (!finite_all(it.p, it.n)) return c->fail(MRN_ERR_ARGUMENT, "weights: tensor %s holds a non-finite value", it.name);
  }
  return MRN_OK;
}

int load_weights(mrn_ctx* c, const mrn_weights* w) {
  const size_t d = c->d, ff = c->dff;
  int rc;
  if ((rc = upload_f32(c, &c->piece, w->piece_embed, 13 * d)) || (rc = upload_f32(c, &c->square, w->square_embed, 64 * d)) ||
      (rc = upload_f32(c, &c->state, w->state_embed, d)) || (rc = upload_f32(c, &c->cast_w, w->castling_proj.weight, 4 * d)) ||
      (rc = upload_f32(c, &c->cast_b, w->castling_proj.bias, d)) || (rc = upload_f32(c, &c->ep, w->en_passant_embed, 9 * d)))
    return rc;
  c->dl.resize(c->layers);
  for (int l = 0; l < c->layers; ++l) {
    const mrn_layer& L = w->layers[l];
    DevLayer& D = c->dl[l];
    if ((rc = upload_f32(c, &D.n1g, L.norm1.weight, d)) || (rc = upload_f32(c, &D.n1b, L.norm1.bias, d)) ||
        (rc = upload_f32(c, &D.n2g, L.norm2.weight, d)) || (rc = upload_f32(c, &D.n2b, L.norm2.bias, d)) ||
        (rc = upload_weight(c, &D.w_qkv, L.in_proj.weight, 3 * d * d, &D.ws[0])) ||
        (rc = upload_weight(c, &D.w_o, L.out_proj.weight, d * d, &D.ws[1])) ||
        (rc = upload_weight(c, &D.w_1, L.linear1.weight, ff * d, &D.ws[2])) ||
        (rc = upload_weight(c, &D.w_2, L.linear2.weight, d * ff, &D.ws[3])) ||
        (rc = upload_f32(c, &D.b_qkv, L.in_proj.bias, 3 * d)) || (rc = upload_f32(c, &D.b_o, L.out_proj.bias, d)) ||
        (rc = upload_f32(c, &D.b_1, L.linear1.bias, ff)) || (rc = upload_f32(c, &D.b_2, L.linear2.bias, d)))
      return rc;
  }
  if ((rc = upload_f32(c, &c->fn_g, w->final_norm.weight, d)) || (rc = upload_f32(c, &c->fn_b, w->final_norm.bias, d)) ||
      (rc = upload_f32(c, &c->pn_g, w->policy_norm.weight, d)) || (rc = upload_f32(c, &c->pn_b, w->policy_norm.bias, d)) ||
      (rc = upload_f32(c, &c->pw, w->policy_proj.weight, 73 * d)) || (rc = upload_f32(c, &c->pb, w->policy_proj.bias, 73)) ||
      (rc = upload_f32(c, &c->vn_g, w->value_norm.weight, d)) || (rc = upload_f32(c, &c->vn_b, w->value_norm.bias, d)) ||
      (rc = upload_f32(c, &c->vb1, w->value_ff1.bias, d)) || (rc = upload_f32(c, &c->vw2, w->value_ff2.weight, 3 * d)) ||
      (rc = upload_f32(c, &c->vb2, w->value_ff2.bias, 3)))
    return rc;
  std::vector<__nv_bfloat16> v1(d * d);
  for (size_t i = 0; i < d * d; ++i) v1[i] = __float2bfloat16(w->value_ff1.weight[i]);
  if ((rc = dev_alloc(c, &c->vw1, d * d * 2))) return rc;
  CK(cudaMemcpy(c->vw1, v1.data(), d * d * 2, cudaMemcpyHostToDevice));
  return MRN_OK;
}

int alloc_buffers(mrn_ctx* c) {
  const size_t B = c->max_bucket, R = B * c->t, d = c->d;
  int rc;
  if ((rc = dev_alloc(c, &c->boards, B * MRN_BOARD_BYTES)) || (rc = dev_alloc(c, &c->legal, B * MRN_MAX_LEGAL * 4)) ||
      (rc = dev_alloc(c, &c->x, R * d * 2)) || (rc = dev_alloc(c, &c->h, R * d * c->act_bytes)) ||
      (rc = dev_alloc(c, &c->qkv, R * 3 * d * 2)) || (rc = dev_alloc(c, &c->attn, R * d * c->act_bytes)) ||
      (rc = dev_alloc(c, &c->ff, R * c->dff * c->act_bytes)) || (rc = dev_alloc(c, &c->vnorm, B * d * 2)) ||
      (rc = dev_alloc(c, &c->vhid, B * d * 2)) || (rc = dev_alloc(c, &c->priors, B * MRN_MAX_LEGAL * 4)) ||
      (rc = dev_alloc(c, &c->wdl, B * 3 * 4)) || (rc = dev_alloc(c, &c->status, 64)))
    return rc;
  CK(cudaMemset(c->status, 0, 64));
  CK(cudaMemset(c->boards, 0, B * MRN_BOARD_BYTES));
  CK(cudaMemset(c->legal, 0xff, B * MRN_MAX_LEGAL * 4));
  CK(cudaMallocHost(&c->h_boards, B * MRN_BOARD_BYTES));
  CK(cudaMallocHost(&c->h_legal, B * MRN_MAX_LEGAL * 4));
  CK(cudaMallocHost(&c->h_priors, B * MRN_MAX_LEGAL * 4));
  CK(cudaMallocHost(&c->h_wdl, B * 3 * 4));
  CK(cudaMallocHost(&c->h_status, 64));
  return MRN_OK;
}

}  // namespace

namespace mrn {

// Programmatic dependent launch between the kernels of a pass. MRN_PDL=1: always; MRN_PDL=0:
// never; unset: for batches of up to kPdlMaxPositions positions. Measured on B200 (small net,
// e4m3): it takes 13% off the latency of a 1-position pass (0.490 -> 0.425 ms), 8-10% at 16-64
// positions and 2% at 256, where each kernel lasts microseconds and the gaps between them
// count; from 1024 positions on the pass runs at the power cap and came out 1-3% slower with
// the gaps closed, so it stays off there.
constexpr int kPdlMaxPositions = 256;

bool pdl_enabled(int positions) {
  static const int mode = [] {
    const char* e = getenv("MRN_PDL");
    return e && e[0] == '0' ? 0 : e && e[0] == '1' ? 1 : -1;
  }();
  return mode == 1 || (mode == -1 && positions <= kPdlMaxPositions);
}

namespace {

GemmArgs base_args(const mrn_ctx* c, int rows) {
  GemmArgs a;
  a.m = rows;
  a.fp8 = c->precision == MRN_PRECISION_FP8 || c->precision == MRN_PRECISION_FP8_X2;
  a.x2 = c->precision == MRN_PRECISION_FP8_X2;
  a.status = c->status;
  return a;
}

float gemm_scale(const mrn_ctx* c, const DevLayer& D, int i) {
  return c->act != ActType::kBf16 ? D.ws[i] * D.as[i] : D.ws[i];
}

}  // namespace

void layer_gemm_args(const mrn_ctx* c, int l, int rows, const LayerBuffers& b, GemmArgs (&g)[4]) {
  const int d = c->d, ff = c->dff;
  const DevLayer& D = c->dl[l];
  for (int i = 0; i < 4; ++i) g[i] = base_args(c, rows);
  // QKV: h -> qkv (bf16)
  g[0].a = b.h, g[0].b = D.w_qkv, g[0].n = 3 * d, g[0].k = d, g[0].epi = Epilogue::kBias, g[0].out = b.qkv;
  g[0].ldo = 3 * d, g[0].bias = D.b_qkv, g[0].scale = gemm_scale(c, D, 0);
  // out-proj: attn -> x +=
  g[1].a = b.attn, g[1].b = D.w_o, g[1].n = d, g[1].k = d, g[1].epi = Epilogue::kResidual, g[1].out = b.x;
  g[1].ldo = d, g[1].bias = D.b_o, g[1].scale = gemm_scale(c, D, 1);
  // FFN1: h -> ff = GELU(.), the card's form (the value head's GELU is always the erf one)
  const bool tanh_form = c->gelu == MRN_GELU_TANH;
  g[2].a = b.h, g[2].b = D.w_1, g[2].n = ff, g[2].k = d;
  g[2].epi = c->act == ActType::kE4m3     ? (tanh_form ? Epilogue::kGeluTanhE4m3 : Epilogue::kGeluE4m3)
             : c->act == ActType::kE4m3x2 ? (tanh_form ? Epilogue::kGeluTanhE4m3x2 : Epilogue::kGeluE4m3x2)
                                          : (tanh_form ? Epilogue::kGeluTanhBf16 : Epilogue::kGeluBf16);
  g[2].out = b.ff, g[2].ldo = c->act == ActType::kE4m3x2 ? 2 * ff : ff, g[2].bias = D.b_1, g[2].scale = gemm_scale(c, D, 2), g[2].inv_q = 1.f / D.as[3];
  // FFN2: ff -> x +=
  g[3].a = b.ff, g[3].b = D.w_2, g[3].n = d, g[3].k = ff, g[3].epi = Epilogue::kResidual, g[3].out = b.x;
  g[3].ldo = d, g[3].bias = D.b_2, g[3].scale = gemm_scale(c, D, 3);
}

cudaError_t launch_site_layernorm(const mrn_ctx* c, int l, int site, const LayerBuffers& b, int rows,
                                  cudaStream_t s) {
  const DevLayer& D = c->dl[site == 0 ? l : l + 1];
  const NormParams np = site == 0 ? NormParams{D.n2g, D.n2b, c->eps, b.h, c->act, 1.f / D.as[2]}
                                  : NormParams{D.n1g, D.n1b, c->eps, b.h, c->act, 1.f / D.as[0]};
  return launch_layernorm(b.x, np, rows, c->d, s);
}

int begin_pass(mrn_ctx* c, cudaStream_t s) {
  if (!c->pass_recorded || s == c->pass_stream) return MRN_OK;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  CK(cudaStreamIsCapturing(s, &cap));
  if (cap != cudaStreamCaptureStatusNone) return MRN_OK;
  CK(cudaStreamWaitEvent(s, c->pass_done, 0));
  return MRN_OK;
}

int end_pass(mrn_ctx* c, cudaStream_t s) {
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  CK(cudaStreamIsCapturing(s, &cap));
  if (cap != cudaStreamCaptureStatusNone) return MRN_OK;
  CK(cudaEventRecord(c->pass_done, s));
  c->pass_stream = s;
  c->pass_recorded = true;
  return MRN_OK;
}

}  // namespace mrn

namespace {

// GEMM plans of one bucket: per layer QKV, out-proj, FFN1, FFN2; then value ff1.
int make_plans(mrn_ctx* c, Bucket& b) {
  const int M = b.positions * c->t, d = c->d;
  char err[256];
  const mrn::LayerBuffers bufs{c->h, c->qkv, c->attn, c->ff, c->x};
  for (int l = 0; l < c->layers; ++l) {
    GemmArgs g[4];
    mrn::layer_gemm_args(c, l, M, bufs, g);
    for (int i = 0; i < 4; ++i) {
      GemmPlan p;
      if (!mrn::gemm_plan(&p, g[i], c->num_sms, err)) return c->fail(MRN_ERR_UNSUPPORTED, "layer %d: %s", l, err);
      b.plans.push_back(p);
    }
  }
  GemmArgs v;
  v.m = b.positions, v.n = d, v.k = d, v.fp8 = false, v.status = c->status;
  v.a = c->vnorm, v.b = c->vw1, v.epi = Epilogue::kGeluBf16, v.out = c->vhid, v.ldo = d, v.bias = c->vb1;
  GemmPlan p;
  if (!mrn::gemm_plan(&p, v, c->num_sms, err)) return c->fail(MRN_ERR_UNSUPPORTED, "value head: %s", err);
  b.plans.push_back(p);
  return MRN_OK;
}

// The whole forward pass of one bucket on `s`. `logits_out`, when set, selects raw logits over
// all actions ([positions, 4672]) and raw WDL logits instead of priors and probabilities.
int enqueue(mrn_ctx* c, Bucket& b, cudaStream_t s, float* logits_out, Profiler* prof) {
  const int P = b.positions, R = P * c->t, d = c->d;
  const ActType act = c->act;
  auto mark = [&](int cls) {
    if (prof) prof->begin(cls);
  };
  auto done = [&]() {
    if (prof) prof->end();
  };
  mrn::EmbedParams e{c->boards, c->piece, c->square, c->state, c->cast_w, c->cast_b, c->ep, c->x, c->t, c->square_start};
  const DevLayer& D0 = c->dl[0];
  mark(MRN_PROFILE_EMBED);
  CK(mrn::launch_embed_ln(e, mrn::NormParams{D0.n1g, D0.n1b, c->eps, c->h, act, 1.f / D0.as[0]}, P, d, s));
  done();
  // Every later kernel follows a kernel of this pass, so its launch may overlap the end of that
  // one (the embedding follows the input copies and launches plainly). Not while profiling:
  // the per-launch events would time overlapping kernels.
  const mrn::PdlScope pdl(!prof && mrn::pdl_enabled(P));
  const mrn::LayerBuffers bufs{c->h, c->qkv, c->attn, c->ff, c->x};
  for (int l = 0; l < c->layers; ++l) {
    const DevLayer& D = c->dl[l];
    const GemmPlan* plans = &b.plans[4 * l];
    mark(MRN_PROFILE_GEMM);
    CK(mrn::gemm_launch(plans[0], s));
    done();
    mark(MRN_PROFILE_ATTENTION);
    CK(mrn::launch_attention(mrn::AttentionParams{c->qkv, c->attn, act, 1.f / D.as[1], c->t, d, c->heads, c->status}, P,
                             d / c->heads, s));
    done();
    mark(MRN_PROFILE_GEMM);
    CK(mrn::gemm_launch(plans[1], s));
    done();
    mark(MRN_PROFILE_LAYERNORM);
    CK(mrn::launch_site_layernorm(c, l, 0, bufs, R, s));
    done();
    mark(MRN_PROFILE_GEMM);
    CK(mrn::gemm_launch(plans[2], s));
    CK(mrn::gemm_launch(plans[3], s));
    done();
    if (l + 1 < c->layers) {
      mark(MRN_PROFILE_LAYERNORM);
      CK(mrn::launch_site_layernorm(c, l, 1, bufs, R, s));
      done();
    }
  }
  mrn::HeadsParams hp;
  hp.x = c->x, hp.final_g = c->fn_g, hp.final_b = c->fn_b, hp.policy_g = c->pn_g, hp.policy_b = c->pn_b;
  hp.policy_w = c->pw, hp.policy_bias = c->pb, hp.value_g = c->vn_g, hp.value_b = c->vn_b;
  hp.legal = logits_out ? nullptr : c->legal;
  hp.slots = logits_out ? MRN_ACTIONS : MRN_MAX_LEGAL;
  hp.softmax = logits_out ? 0 : 1;
  hp.priors = logits_out ? logits_out : c->priors;
  hp.value_in = c->vnorm, hp.status = c->status, hp.eps = c->eps, hp.t = c->t, hp.square_start = c->square_start;
  mark(MRN_PROFILE_HEADS);
  CK(mrn::launch_heads(hp, P, d, s));
  CK(mrn::gemm_launch(b.plans[4 * c->layers], s));
  CK(mrn::launch_value_out(mrn::ValueOutParams{c->vhid, c->vw2, c->vb2, c->wdl, logits_out ? 0 : 1}, P, d, s));
  done();
  return MRN_OK;
}

// Embedding; per layer QKV, attention, out-proj, norm2, FFN1, FFN2; norm1 of every layer but the
// first; 3 for the heads.
int launches_per_forward(const mrn_ctx* c) { return 1 + 6 * c->layers + (c->layers - 1) + 3; }

int get_bucket(mrn_ctx* c, int n, Bucket** out) {
  const int key = bucket_for(n);
  auto it = c->buckets.find(key);
  if (it != c->buckets.end()) {
    *out = &it->second;
    return MRN_OK;
  }
  Bucket b;
  b.positions = key;
  int rc = make_plans(c, b);
  if (rc) return rc;
  // Capture the forward pass into a graph (src/net/cuda/mod.rs:689-700).
  CK(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
  rc = enqueue(c, b, c->stream, nullptr, nullptr);
  cudaGraph_t graph = nullptr;
  const cudaError_t end = cudaStreamEndCapture(c->stream, &graph);
  if (rc) {
    if (graph) cudaGraphDestroy(graph);
    return rc;
  }
  if (end != cudaSuccess || !graph) return c->fail(MRN_ERR_CUDA, "graph capture failed: %s", cudaGetErrorString(end));
  const cudaError_t inst = cudaGraphInstantiate(&b.graph, graph, 0);
  cudaGraphDestroy(graph);
  if (inst != cudaSuccess) return c->fail(MRN_ERR_CUDA, "cudaGraphInstantiate: %s", cudaGetErrorString(inst));
  *out = &c->buckets.emplace(key, std::move(b)).first->second;
  return MRN_OK;
}

// Host-side input checks (the device kernels clamp as well, so bad input cannot fault).
// Branch-free scan of every token and legal slot (vectorised by the compiler); the slow loop below
// only runs to name the first offending entry.
bool inputs_in_range(int n, const uint8_t* boards, const int32_t* legal) {
  unsigned bad = 0;
  for (int p = 0; p < n; ++p) {
    const uint8_t* b = boards + static_cast<size_t>(p) * MRN_BOARD_BYTES;
    for (int s = 0; s < 64; ++s) bad |= b[s] > 12;
    bad |= (b[64] > 15) | (b[65] > 8);
  }
  if (legal) {
    const size_t slots = static_cast<size_t>(n) * MRN_MAX_LEGAL;
    for (size_t k = 0; k < slots; ++k) bad |= static_cast<uint32_t>(legal[k] + 1) > static_cast<uint32_t>(MRN_ACTIONS);
  }
  return bad == 0;
}

int validate_inputs(mrn_ctx* c, int n, const uint8_t* boards, const int32_t* legal) {
  if (inputs_in_range(n, boards, legal)) return MRN_OK;
  for (int p = 0; p < n; ++p) {
    const uint8_t* b = boards + static_cast<size_t>(p) * MRN_BOARD_BYTES;
    for (int s = 0; s < 64; ++s)
      if (b[s] > 12) return c->fail(MRN_ERR_ARGUMENT, "position %d: piece token %d on square %d (0..12)", p, b[s], s);
    if (b[64] > 15 || b[65] > 8)
      return c->fail(MRN_ERR_ARGUMENT, "position %d: castling %d / en passant %d out of range", p, b[64], b[65]);
    if (!legal) continue;
    const int32_t* a = legal + static_cast<size_t>(p) * MRN_MAX_LEGAL;
    for (int k = 0; k < MRN_MAX_LEGAL; ++k)
      if (a[k] < -1 || a[k] >= MRN_ACTIONS)
        return c->fail(MRN_ERR_ACTION, "position %d slot %d: action %d outside [0, %d)", p, k, a[k], MRN_ACTIONS);
  }
  return MRN_OK;
}

bool is_pinned(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeHost;
}

int check_status(mrn_ctx* c, int word) {
  if (word == 0) return MRN_OK;
  if (word == mrn::kErrBadAction) return c->fail(MRN_ERR_ACTION, "a legal slot held an action index >= %d", MRN_ACTIONS);
  return c->fail(MRN_ERR_DEVICE_FAULT, "device-side wait gave up in a GEMM (code %d)", word);
}

void destroy(mrn_ctx* c) {
  if (!c) return;
  cudaSetDevice(c->device);
  if (c->stream) cudaStreamSynchronize(c->stream);
  for (auto& kv : c->buckets)
    if (kv.second.graph) cudaGraphExecDestroy(kv.second.graph);
  for (void* p : c->allocations) cudaFree(p);
  if (c->h_boards) cudaFreeHost(c->h_boards);
  if (c->h_legal) cudaFreeHost(c->h_legal);
  if (c->h_priors) cudaFreeHost(c->h_priors);
  if (c->h_wdl) cudaFreeHost(c->h_wdl);
  if (c->h_status) cudaFreeHost(c->h_status);
  if (c->stream) cudaStreamDestroy(c->stream);
  if (c->pass_done) cudaEventDestroy(c->pass_done);
  delete c;
}

const char* precision_name(int p) {
  return p == MRN_PRECISION_FP8_X2    ? "fp8x2"
         : p == MRN_PRECISION_FP8       ? "fp8"
         : p == MRN_PRECISION_FP8_WEIGHTS ? "fp8-weights"
                                          : "bf16";
}

}  // namespace

extern "C" {

MRN_API int mrn_create(const mrn_arch* arch, const mrn_weights* weights, int device, int max_batch, int precision,
                       mrn_ctx** out) {
  if (!out) {
    g_create_error = "out is NULL";
    return MRN_ERR_ARGUMENT;
  }
  *out = nullptr;
  mrn_ctx* c = new mrn_ctx();
  auto bail = [&](int rc) {
    g_create_error = c->last_error;
    destroy(c);
    return rc;
  };
  if (!arch || !weights) return bail(c->fail(MRN_ERR_ARGUMENT, "arch or weights is NULL"));
  if (max_batch < 1) return bail(c->fail(MRN_ERR_ARGUMENT, "max_batch %d < 1", max_batch));
  if (precision < MRN_PRECISION_BF16 || precision > MRN_PRECISION_FP8_X2)
    return bail(c->fail(MRN_ERR_ARGUMENT, "unknown precision %d", precision));
  c->device = device, c->precision = precision, c->max_batch = max_batch, c->max_bucket = bucket_for(max_batch);
  c->d = arch->d_model, c->layers = arch->n_layers, c->heads = arch->n_heads, c->dff = arch->d_ff;
  c->t = arch->tokens, c->square_start = arch->square_token_start, c->eps = arch->layer_norm_eps, c->gelu = arch->gelu;
  if (c->d <= 0 || c->layers <= 0 || c->heads <= 0 || c->dff <= 0 || !(c->eps > 0.f))
    return bail(c->fail(MRN_ERR_ARGUMENT, "degenerate architecture (a zero dimension or eps <= 0)"));
  if (c->d % c->heads != 0) return bail(c->fail(MRN_ERR_ARGUMENT, "d_model %d not divisible by n_heads %d", c->d, c->heads));
  if (c->square_start < 1 || c->square_start + 64 != c->t)
    return bail(c->fail(MRN_ERR_ARGUMENT, "tokens %d with square_token_start %d is not board mode", c->t, c->square_start));
  const int hd = c->d / c->heads;
  if (hd != 32 && hd != 64) return bail(c->fail(MRN_ERR_UNSUPPORTED, "head dimension %d (32 or 64 supported)", hd));
  static const int kWidths[] = {64, 128, 192, 256, 320, 384, 448, 512, 640, 768, 1024};
  bool width_ok = false;
  for (int w : kWidths) width_ok |= (c->d == w);
  if (!width_ok || c->dff % 64 != 0)
    return bail(c->fail(MRN_ERR_UNSUPPORTED, "d_model %d / d_ff %d: d_model in {64..512 step 64, 640, 768, 1024}, d_ff a multiple of 64",
                        c->d, c->dff));
  if (c->t != kTokens)
    return bail(c->fail(MRN_ERR_UNSUPPORTED, "%d tokens per position (the kernels are built for %d)", c->t, kTokens));
  if (c->gelu != MRN_GELU_ERF && c->gelu != MRN_GELU_TANH)
    return bail(c->fail(MRN_ERR_ARGUMENT, "gelu must be MRN_GELU_ERF or MRN_GELU_TANH, got %d", c->gelu));
  const bool static_act = precision == MRN_PRECISION_FP8 || precision == MRN_PRECISION_FP8_X2;
  if (static_act) {
    if (!arch->fp8_amax)
      return bail(c->fail(MRN_ERR_ARGUMENT, "e4m3 activations need the calibration (encoder.fp8.activation_amax); the card has none"));
    for (int i = 0; i < 4 * c->layers; ++i)
      if (!(arch->fp8_amax[i] > 0.f) || !isfinite(arch->fp8_amax[i]))
        return bail(c->fail(MRN_ERR_ARGUMENT, "fp8_amax[%d] must be positive and finite", i));
  }
  c->act = precision == MRN_PRECISION_FP8 ? ActType::kE4m3 : precision == MRN_PRECISION_FP8_X2 ? ActType::kE4m3x2 : ActType::kBf16;
  c->act_bytes = mrn::act_row_bytes(c->act);

  int rc = check_weights(c, weights);
  if (rc) return bail(rc);
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count) {
    cudaGetLastError();
    return bail(c->fail(MRN_ERR_CUDA, "CUDA device %d not available (%d devices)", device, count));
  }
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return bail(c->fail(MRN_ERR_CUDA, "cudaGetDeviceProperties failed"));
  if (prop.major != 10)
    return bail(c->fail(MRN_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a", device, prop.major, prop.minor));
  if (cudaSetDevice(device) != cudaSuccess) return bail(c->fail(MRN_ERR_CUDA, "cudaSetDevice(%d) failed", device));
  c->num_sms = prop.multiProcessorCount;
  if (mrn::gemm_prepare_device() != cudaSuccess || mrn::prepare_attention() != cudaSuccess)
    return bail(c->fail(MRN_ERR_CUDA, "kernel shared-memory attributes"));
  if (mrn::load_row_kernels(c->d) != cudaSuccess) return bail(c->fail(MRN_ERR_CUDA, "loading the row kernels failed"));
  if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess)
    return bail(c->fail(MRN_ERR_CUDA, "cudaStreamCreate failed"));
  if (cudaEventCreateWithFlags(&c->pass_done, cudaEventDisableTiming) != cudaSuccess)
    return bail(c->fail(MRN_ERR_CUDA, "cudaEventCreate failed"));
  mrn::static_scratch_setup(c);

  if ((rc = load_weights(c, weights))) return bail(rc);
  if (static_act)
    for (int l = 0; l < c->layers; ++l)
      for (int i = 0; i < 4; ++i) c->dl[l].as[i] = arch->fp8_amax[4 * l + i] * kFp8Margin / kE4m3Max;
  if ((rc = alloc_buffers(c))) return bail(rc);
  char desc[256];
  snprintf(desc, sizeof(desc), "b200 %s on %s: %dx%d (%d heads, d_ff %d)", precision_name(precision), prop.name, c->d,
           c->layers, c->heads, c->dff);
  c->describe = desc;
  *out = c;
  return MRN_OK;
}

namespace {

// The pass on host buffers behind mrn_evaluate (f32 priors) and mrn_evaluate_f16 (`half`: the
// priors converted to f16 on the device, so the copy back moves half the bytes).
int evaluate_host(mrn_ctx* c, int n, const uint8_t* boards, const int32_t* legal, void* priors, bool half,
                  float* wdl) {
  std::lock_guard<std::mutex> lock(c->mu);
  if (n < 0) return c->fail(MRN_ERR_ARGUMENT, "n = %d", n);
  if (n > c->max_batch) return c->fail(MRN_ERR_BATCH_TOO_LARGE, "batch of %d positions exceeds max_batch %d", n, c->max_batch);
  if (n == 0) return MRN_OK;
  if (!boards || !legal || !priors || !wdl) return c->fail(MRN_ERR_ARGUMENT, "NULL buffer");
  CK(cudaSetDevice(c->device));
  Bucket* b = nullptr;
  int rc = get_bucket(c, n, &b);
  if (rc) return rc;
  if (half && !c->priors16 &&
      (rc = dev_alloc(c, &c->priors16, static_cast<size_t>(c->max_bucket) * MRN_MAX_LEGAL * 2)))
    return rc;
  const int P = b->positions;
  const size_t prior_bytes = static_cast<size_t>(n) * MRN_MAX_LEGAL * (half ? 2 : 4);
  const bool direct_in = is_pinned(boards) && is_pinned(legal);
  const bool direct_out = is_pinned(priors) && is_pinned(wdl);
  const uint8_t* src_b = boards;
  const int32_t* src_l = legal;
  if (!direct_in) {
    memcpy(c->h_boards, boards, static_cast<size_t>(n) * MRN_BOARD_BYTES);
    memcpy(c->h_legal, legal, static_cast<size_t>(n) * MRN_MAX_LEGAL * 4);
    src_b = c->h_boards, src_l = c->h_legal;
  }
  cudaStream_t s = c->stream;
  if ((rc = mrn::begin_pass(c, s))) return rc;
  CK(cudaMemcpyAsync(c->boards, src_b, static_cast<size_t>(n) * MRN_BOARD_BYTES, cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(c->legal, src_l, static_cast<size_t>(n) * MRN_MAX_LEGAL * 4, cudaMemcpyHostToDevice, s));
  if (P > n) {
    CK(cudaMemsetAsync(c->boards + static_cast<size_t>(n) * MRN_BOARD_BYTES, 0, static_cast<size_t>(P - n) * MRN_BOARD_BYTES, s));
    CK(cudaMemsetAsync(c->legal + static_cast<size_t>(n) * MRN_MAX_LEGAL, 0xff, static_cast<size_t>(P - n) * MRN_MAX_LEGAL * 4, s));
  }
  CK(cudaGraphLaunch(b->graph, s));
  if (half) CK(mrn::launch_priors_to_half(c->priors, c->priors16, n * MRN_MAX_LEGAL, s));
  void* dst_p = direct_out ? priors : static_cast<void*>(c->h_priors);
  float* dst_w = direct_out ? wdl : c->h_wdl;
  const void* src_p = half ? static_cast<const void*>(c->priors16) : static_cast<const void*>(c->priors);
  CK(cudaMemcpyAsync(dst_p, src_p, prior_bytes, cudaMemcpyDeviceToHost, s));
  CK(cudaMemcpyAsync(dst_w, c->wdl, static_cast<size_t>(n) * 3 * 4, cudaMemcpyDeviceToHost, s));
  CK(cudaMemcpyAsync(c->h_status, c->status, 4, cudaMemcpyDeviceToHost, s));
  if ((rc = mrn::end_pass(c, s))) return rc;
  // The inputs are checked while the GPU runs: the kernels clamp out-of-range tokens and flag
  // out-of-range actions themselves, so a bad batch costs one wasted pass, never a fault; its
  // outputs are discarded and the error names the first bad entry.
  const int invalid = validate_inputs(c, n, boards, legal);
  CK(cudaStreamSynchronize(s));
  const int word = *c->h_status;
  if (word) {
    CK(cudaMemsetAsync(c->status, 0, 4, s));
    CK(cudaStreamSynchronize(s));
  }
  if (invalid) return invalid;
  if (word) return check_status(c, word);
  if (!direct_out) {
    memcpy(priors, c->h_priors, prior_bytes);
    memcpy(wdl, c->h_wdl, static_cast<size_t>(n) * 3 * 4);
  }
  return MRN_OK;
}

}  // namespace

MRN_API int mrn_evaluate(mrn_ctx* c, int n, const uint8_t* boards, const int32_t* legal, float* priors, float* wdl) {
  if (!c) {
    g_create_error = "context is NULL";
    return MRN_ERR_ARGUMENT;
  }
  return evaluate_host(c, n, boards, legal, priors, false, wdl);
}

MRN_API int mrn_evaluate_f16(mrn_ctx* c, int n, const uint8_t* boards, const int32_t* legal, uint16_t* priors,
                             float* wdl) {
  if (!c) {
    g_create_error = "context is NULL";
    return MRN_ERR_ARGUMENT;
  }
  return evaluate_host(c, n, boards, legal, priors, true, wdl);
}

MRN_API int mrn_logits(mrn_ctx* c, int n, const uint8_t* boards, float* policy, float* value) {
  if (!c) return MRN_ERR_ARGUMENT;
  std::lock_guard<std::mutex> lock(c->mu);
  if (n < 0) return c->fail(MRN_ERR_ARGUMENT, "n = %d", n);
  if (n > c->max_batch) return c->fail(MRN_ERR_BATCH_TOO_LARGE, "batch of %d positions exceeds max_batch %d", n, c->max_batch);
  if (n == 0) return MRN_OK;
  if (!boards || !policy || !value) return c->fail(MRN_ERR_ARGUMENT, "NULL buffer");
  int rc = validate_inputs(c, n, boards, nullptr);
  if (rc) return rc;
  CK(cudaSetDevice(c->device));
  Bucket* b = nullptr;
  if ((rc = get_bucket(c, n, &b))) return rc;
  const int P = b->positions;
  if (!c->logits && (rc = dev_alloc(c, &c->logits, static_cast<size_t>(c->max_bucket) * MRN_ACTIONS * 4))) return rc;
  cudaStream_t s = c->stream;
  if ((rc = mrn::begin_pass(c, s))) return rc;
  CK(cudaMemcpyAsync(c->boards, boards, static_cast<size_t>(n) * MRN_BOARD_BYTES, cudaMemcpyHostToDevice, s));
  if (P > n)
    CK(cudaMemsetAsync(c->boards + static_cast<size_t>(n) * MRN_BOARD_BYTES, 0, static_cast<size_t>(P - n) * MRN_BOARD_BYTES, s));
  if ((rc = enqueue(c, *b, s, c->logits, nullptr))) return rc;
  CK(cudaMemcpyAsync(policy, c->logits, static_cast<size_t>(n) * MRN_ACTIONS * 4, cudaMemcpyDeviceToHost, s));
  CK(cudaMemcpyAsync(value, c->wdl, static_cast<size_t>(n) * 3 * 4, cudaMemcpyDeviceToHost, s));
  CK(cudaMemcpyAsync(c->h_status, c->status, 4, cudaMemcpyDeviceToHost, s));
  if ((rc = mrn::end_pass(c, s))) return rc;
  CK(cudaStreamSynchronize(s));
  const int word = *c->h_status;
  if (word) {
    CK(cudaMemsetAsync(c->status, 0, 4, s));
    CK(cudaStreamSynchronize(s));
    return check_status(c, word);
  }
  return MRN_OK;
}

MRN_API int mrn_evaluate_device(mrn_ctx* c, int n, const uint8_t* d_boards, const int32_t* d_legal, float* d_priors,
                                float* d_wdl, void* stream) {
  if (!c) return MRN_ERR_ARGUMENT;
  std::lock_guard<std::mutex> lock(c->mu);
  if (n < 0) return c->fail(MRN_ERR_ARGUMENT, "n = %d", n);
  if (n > c->max_batch) return c->fail(MRN_ERR_BATCH_TOO_LARGE, "batch of %d positions exceeds max_batch %d", n, c->max_batch);
  if (n == 0) return MRN_OK;
  if (!d_boards || !d_legal || !d_priors || !d_wdl) return c->fail(MRN_ERR_ARGUMENT, "NULL buffer");
  CK(cudaSetDevice(c->device));
  Bucket* b = nullptr;
  int rc = get_bucket(c, n, &b);
  if (rc) return rc;
  const int P = b->positions;
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c->stream;
  if ((rc = mrn::begin_pass(c, s))) return rc;
  CK(cudaMemcpyAsync(c->boards, d_boards, static_cast<size_t>(n) * MRN_BOARD_BYTES, cudaMemcpyDeviceToDevice, s));
  CK(cudaMemcpyAsync(c->legal, d_legal, static_cast<size_t>(n) * MRN_MAX_LEGAL * 4, cudaMemcpyDeviceToDevice, s));
  if (P > n) {
    CK(cudaMemsetAsync(c->boards + static_cast<size_t>(n) * MRN_BOARD_BYTES, 0, static_cast<size_t>(P - n) * MRN_BOARD_BYTES, s));
    CK(cudaMemsetAsync(c->legal + static_cast<size_t>(n) * MRN_MAX_LEGAL, 0xff, static_cast<size_t>(P - n) * MRN_MAX_LEGAL * 4, s));
  }
  CK(cudaGraphLaunch(b->graph, s));
  CK(cudaMemcpyAsync(d_priors, c->priors, static_cast<size_t>(n) * MRN_MAX_LEGAL * 4, cudaMemcpyDeviceToDevice, s));
  CK(cudaMemcpyAsync(d_wdl, c->wdl, static_cast<size_t>(n) * 3 * 4, cudaMemcpyDeviceToDevice, s));
  return mrn::end_pass(c, s);
}

MRN_API int mrn_status_word(mrn_ctx* c, int* word) {
  if (!c || !word) return MRN_ERR_ARGUMENT;
  std::lock_guard<std::mutex> lock(c->mu);
  CK(cudaSetDevice(c->device));
  CK(cudaDeviceSynchronize());
  CK(cudaMemcpy(c->h_status, c->status, 4, cudaMemcpyDeviceToHost));
  CK(cudaMemset(c->status, 0, 4));
  *word = *c->h_status;
  return MRN_OK;
}

MRN_API int mrn_profile(mrn_ctx* c, int n, const uint8_t* d_boards, const int32_t* d_legal, float* d_priors,
                        float* d_wdl, void* stream, float* times_ms, double* flops, int* launches) {
  if (!c || !times_ms || !flops || !launches) return MRN_ERR_ARGUMENT;
  std::lock_guard<std::mutex> lock(c->mu);
  if (n <= 0 || n > c->max_batch) return c->fail(MRN_ERR_BATCH_TOO_LARGE, "profile batch %d (max %d)", n, c->max_batch);
  CK(cudaSetDevice(c->device));
  Bucket* b = nullptr;
  int rc = get_bucket(c, n, &b);
  if (rc) return rc;
  const int P = b->positions;
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c->stream;
  if ((rc = mrn::begin_pass(c, s))) return rc;
  CK(cudaMemcpyAsync(c->boards, d_boards, static_cast<size_t>(n) * MRN_BOARD_BYTES, cudaMemcpyDeviceToDevice, s));
  CK(cudaMemcpyAsync(c->legal, d_legal, static_cast<size_t>(n) * MRN_MAX_LEGAL * 4, cudaMemcpyDeviceToDevice, s));
  if (P > n) {
    CK(cudaMemsetAsync(c->boards + static_cast<size_t>(n) * MRN_BOARD_BYTES, 0, static_cast<size_t>(P - n) * MRN_BOARD_BYTES, s));
    CK(cudaMemsetAsync(c->legal + static_cast<size_t>(n) * MRN_MAX_LEGAL, 0xff, static_cast<size_t>(P - n) * MRN_MAX_LEGAL * 4, s));
  }
  Profiler prof;
  prof.stream = s;
  rc = enqueue(c, *b, s, nullptr, &prof);
  CK(cudaStreamSynchronize(s));
  for (int i = 0; i < MRN_PROFILE_SLOTS; ++i) times_ms[i] = 0.f, flops[i] = 0.0, launches[i] = 0;
  for (auto& m : prof.marks) {
    float ms = 0.f;
    cudaEventElapsedTime(&ms, m.second.first, m.second.second);
    times_ms[m.first] += ms;
    cudaEventDestroy(m.second.first);
    cudaEventDestroy(m.second.second);
  }
  if (rc) return rc;
  for (size_t i = 0; i < b->plans.size(); ++i) flops[MRN_PROFILE_GEMM] += mrn::gemm_flops(b->plans[i].args);
  launches[MRN_PROFILE_GEMM] = static_cast<int>(b->plans.size());
  launches[MRN_PROFILE_EMBED] = 1;
  launches[MRN_PROFILE_ATTENTION] = c->layers;
  launches[MRN_PROFILE_LAYERNORM] = 2 * c->layers - 1;
  launches[MRN_PROFILE_HEADS] = 2;
  flops[MRN_PROFILE_ATTENTION] = 4.0 * P * static_cast<double>(c->t) * c->t * c->d * c->layers;
  CK(cudaMemcpyAsync(d_priors, c->priors, static_cast<size_t>(n) * MRN_MAX_LEGAL * 4, cudaMemcpyDeviceToDevice, s));
  CK(cudaMemcpyAsync(d_wdl, c->wdl, static_cast<size_t>(n) * 3 * 4, cudaMemcpyDeviceToDevice, s));
  if ((rc = mrn::end_pass(c, s))) return rc;
  CK(cudaStreamSynchronize(s));
  return MRN_OK;
}

MRN_API int mrn_launches_per_forward(mrn_ctx* c, int n) {
  if (!c) return -1;
  std::lock_guard<std::mutex> lock(c->mu);
  if (n < 1 || n > c->max_batch) return -1;
  Bucket* b = nullptr;
  if (cudaSetDevice(c->device) != cudaSuccess || get_bucket(c, n, &b)) return -1;
  return launches_per_forward(c);
}

MRN_API const char* mrn_describe(mrn_ctx* c) { return c ? c->describe.c_str() : ""; }

MRN_API const char* mrn_last_error(mrn_ctx* c) { return c ? c->last_error.c_str() : g_create_error.c_str(); }

MRN_API void mrn_destroy(mrn_ctx* c) { destroy(c); }

}  // extern "C"
