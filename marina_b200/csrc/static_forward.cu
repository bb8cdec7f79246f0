// A forward pass that allocates no device memory: every intermediate buffer of the pass lives in
// one statically sized device array compiled into the library.
//
// Who needs it: callers that must not call cudaMalloc once they are running -- a host process
// whose device memory belongs to another allocator (a framework's caching pool, a plugin host
// that fixes its footprint at start-up), a latency-critical thread where an allocation can stall
// on a device-wide synchronisation, or code that must keep working when the device is full.
// They can still evaluate small batches (the search's root, a handful of leaves) through
// `mrn_evaluate_device_static`, with the weights already loaded by `mrn_create`.
//
// The array holds kStaticScratchBytes (8 MiB) and is resident on every GPU on which a context has
// been created, for the life of the process. How many positions fit depends on the network: one
// position needs 65 rows of the residual stream (f16), the two GEMM inputs and the attention
// output (bf16; e4m3 for MRN_PRECISION_FP8; two e4m3 codes, as wide as bf16, for
// MRN_PRECISION_FP8_X2), Q/K/V (bf16) and the FFN hidden layer, plus two d-wide bf16 rows for
// the value head -- 0.67 MB for the `small` network in bf16 or fp8w
// (12 positions; 17 in fp8) and 0.25 MB for `nano` (33 positions; 47 in fp8). Larger batches
// are refused with MRN_ERR_BATCH_TOO_LARGE and a message naming the limit.
//
// mrn_create looks the array's device address up (cudaGetSymbolAddress, with the context's device
// current) and keeps it in the context. That first look-up loads the module holding the array, which
// is when the device memory for it is allocated, so by the time a caller needs the no-allocation
// guarantee the array is already resident; mrn_create also loads every kernel the pass launches.
//
// All calls on a device share the array. Nothing in it has to start at zero (every buffer is
// written before it is read), so nothing is cleared, but two calls whose GPU work overlaps --
// on different streams, or through different contexts on the same device -- overwrite each
// other's intermediates: serialise them. Device-side errors go to the context's status word
// (`mrn_status_word`).
#include <cuda_bf16.h>
#include <stdio.h>

#include <string>

#include "../../include/marina_b200.h"
#include "gemm.h"
#include "kernels.cuh"
#include "launch.h"
#include "runtime.h"

namespace {

constexpr size_t kStaticScratchBytes = size_t(8) << 20;

static __device__ __align__(256) uint8_t g_static_scratch[kStaticScratchBytes];

size_t align256(size_t b) { return (b + 255) & ~size_t(255); }

// Byte offsets of the pass's buffers for `n` positions inside the array.
struct Layout {
  size_t x, h, qkv, attn, ff, vnorm, vhid, end;
};

Layout layout(const mrn_ctx* c, int n) {
  const size_t R = static_cast<size_t>(n) * c->t, d = c->d, ab = c->act_bytes;
  Layout l;
  l.x = 0;
  l.h = l.x + align256(R * d * 2);
  l.qkv = l.h + align256(R * d * ab);
  l.attn = l.qkv + align256(R * 3 * d * 2);
  l.ff = l.attn + align256(R * d * ab);
  l.vnorm = l.ff + align256(R * c->dff * ab);
  l.vhid = l.vnorm + align256(static_cast<size_t>(n) * d * 2);
  l.end = l.vhid + align256(static_cast<size_t>(n) * d * 2);
  return l;
}

int max_positions(const mrn_ctx* c) {
  int n = 0;
  while (layout(c, n + 1).end <= kStaticScratchBytes) ++n;
  return n;
}

#define CKS(call)                                                                                    \
  do {                                                                                               \
    const cudaError_t e_ = (call);                                                                   \
    if (e_ != cudaSuccess) return c->fail(MRN_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_));   \
  } while (0)

// Plan one GEMM on the stack and launch it.
int gemm(mrn_ctx* c, const mrn::GemmArgs& a, cudaStream_t s) {
  mrn::GemmPlan p;
  char err[256];
  if (!mrn::gemm_plan(&p, a, c->num_sms, err)) return c->fail(MRN_ERR_UNSUPPORTED, "%s", err);
  CKS(mrn::gemm_launch(p, s));
  return MRN_OK;
}

int forward(mrn_ctx* c, int n, const uint8_t* boards, const int32_t* legal, float* priors, float* wdl, uint8_t* base,
            cudaStream_t s) {
  using mrn::ActType;
  using mrn::Epilogue;
  const Layout L = layout(c, n);
  __half* x = reinterpret_cast<__half*>(base + L.x);
  void* h = base + L.h;
  __nv_bfloat16* qkv = reinterpret_cast<__nv_bfloat16*>(base + L.qkv);
  void* attn = base + L.attn;
  void* ff = base + L.ff;
  __nv_bfloat16* vnorm = reinterpret_cast<__nv_bfloat16*>(base + L.vnorm);
  __nv_bfloat16* vhid = reinterpret_cast<__nv_bfloat16*>(base + L.vhid);
  const int R = n * c->t, d = c->d;
  const ActType act = c->act;
  int rc;

  const mrn::DevLayer& D0 = c->dl[0];
  const mrn::LayerBuffers bufs{h, qkv, attn, ff, x};
  CKS(mrn::launch_embed_ln(
      mrn::EmbedParams{boards, c->piece, c->square, c->state, c->cast_w, c->cast_b, c->ep, x, c->t, c->square_start},
      mrn::NormParams{D0.n1g, D0.n1b, c->eps, h, act, 1.f / D0.as[0]}, n, d, s));
  // The kernels after the embedding follow one of this pass: their launches may overlap.
  const mrn::PdlScope pdl(mrn::pdl_enabled(n));
  for (int l = 0; l < c->layers; ++l) {
    const mrn::DevLayer& D = c->dl[l];
    mrn::GemmArgs g[4];
    mrn::layer_gemm_args(c, l, R, bufs, g);
    if ((rc = gemm(c, g[0], s))) return rc;
    CKS(mrn::launch_attention(mrn::AttentionParams{qkv, attn, act, 1.f / D.as[1], c->t, d, c->heads, c->status}, n,
                              d / c->heads, s));
    if ((rc = gemm(c, g[1], s))) return rc;
    CKS(mrn::launch_site_layernorm(c, l, 0, bufs, R, s));
    if ((rc = gemm(c, g[2], s))) return rc;
    if ((rc = gemm(c, g[3], s))) return rc;
    if (l + 1 < c->layers) CKS(mrn::launch_site_layernorm(c, l, 1, bufs, R, s));
  }
  mrn::HeadsParams hp;
  hp.x = x, hp.final_g = c->fn_g, hp.final_b = c->fn_b, hp.policy_g = c->pn_g, hp.policy_b = c->pn_b;
  hp.policy_w = c->pw, hp.policy_bias = c->pb, hp.value_g = c->vn_g, hp.value_b = c->vn_b;
  hp.legal = legal, hp.slots = MRN_MAX_LEGAL, hp.softmax = 1, hp.priors = priors;
  hp.value_in = vnorm, hp.status = c->status, hp.eps = c->eps, hp.t = c->t, hp.square_start = c->square_start;
  CKS(mrn::launch_heads(hp, n, d, s));
  mrn::GemmArgs v;
  v.m = n, v.n = d, v.k = d, v.fp8 = false, v.status = c->status;
  v.a = vnorm, v.b = c->vw1, v.epi = Epilogue::kGeluBf16, v.out = vhid, v.ldo = d, v.bias = c->vb1;
  if ((rc = gemm(c, v, s))) return rc;
  CKS(mrn::launch_value_out(mrn::ValueOutParams{vhid, c->vw2, c->vb2, wdl, 1}, n, d, s));
  return MRN_OK;
}

}  // namespace

extern "C" MRN_API int mrn_evaluate_device_static(mrn_ctx* c, int n, const uint8_t* d_boards, const int32_t* d_legal,
                                                  float* d_priors, float* d_wdl, void* stream) {
  if (!c) return MRN_ERR_ARGUMENT;
  std::lock_guard<std::mutex> lock(c->mu);
  if (n < 0) return c->fail(MRN_ERR_ARGUMENT, "n = %d", n);
  if (n == 0) return MRN_OK;
  if (!d_boards || !d_legal || !d_priors || !d_wdl) return c->fail(MRN_ERR_ARGUMENT, "NULL buffer");
  const int limit = max_positions(c);
  if (n > limit)
    return c->fail(MRN_ERR_BATCH_TOO_LARGE,
                   "batch of %d positions exceeds the %d that fit the %zu-byte static scratch for this network", n,
                   limit, kStaticScratchBytes);
  if (!c->static_scratch)
    return c->fail(MRN_ERR_CUDA, "the static scratch array is not available on device %d: %s", c->device,
                   c->static_error.c_str());
  const cudaError_t e = cudaSetDevice(c->device);
  if (e != cudaSuccess) return c->fail(MRN_ERR_CUDA, "cudaSetDevice: %s", cudaGetErrorString(e));
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c->stream;
  int rc = mrn::begin_pass(c, s);
  if (rc) return rc;
  if ((rc = forward(c, n, d_boards, d_legal, d_priors, d_wdl, c->static_scratch, s))) return rc;
  return mrn::end_pass(c, s);
}

namespace mrn {

void static_scratch_setup(mrn_ctx* c) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
  if (e != cudaSuccess || !p) {
    cudaGetLastError();
    c->static_error = std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e);
    return;
  }
  c->static_scratch = static_cast<uint8_t*>(p);
}

}  // namespace mrn
