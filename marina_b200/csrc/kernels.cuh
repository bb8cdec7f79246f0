// Launchers of the evaluator's non-GEMM kernels (kernels.cu). Layout: a batch of B positions
// is R = B*t token rows (t = 65: the state token, then 64 squares), row r = pos*t + i.
// The residual stream x is f16 [R, d], as in the reference's CUDA backend (its residual adds
// accumulate in f32 and round once to f16); GEMM operands are bf16 or e4m3 rows.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace mrn {

// Activation storage of a GEMM operand produced by a kernel. kE4m3x2 carries each value v (scaled
// by the operand's inv_q) as two e4m3 terms, hi = e4m3(v) and lo = e4m3(v - hi): a row of width w
// is 2w bytes, the w hi codes followed by the w lo codes.
enum class ActType : int { kBf16 = 0, kE4m3 = 1, kE4m3x2 = 2 };

// Bytes per element of a row of that storage.
__host__ __device__ constexpr int act_row_bytes(ActType t) { return t == ActType::kE4m3 ? 1 : 2; }

struct EmbedParams {
  const uint8_t* boards;     // [B, 66]
  const float* piece_embed;  // [13, d]
  const float* square_embed; // [64, d]
  const float* state_embed;  // [d]
  const float* castling_w;   // [d, 4]
  const float* castling_b;   // [d]
  const float* ep_embed;     // [9, d]
  __half* x;                 // [R, d]
  int t, square_start;
};

struct NormParams {
  const float* gamma;
  const float* beta;
  float eps;
  void* out;       // bf16 or e4m3 [R, d]
  ActType out_type;
  float inv_q;     // 1 / e4m3 scale
};

// x = tokens(boards); out = LN(x) (layer 0's norm1) in one pass, or x alone when n.out is null.
cudaError_t launch_embed_ln(const EmbedParams& e, const NormParams& n, int positions, int d, cudaStream_t s);
// out = LN(x) for rows [0, rows).
cudaError_t launch_layernorm(const __half* x, const NormParams& n, int rows, int d, cudaStream_t s);

struct AttentionParams {
  const void* qkv;   // bf16 [R, 3d]: Q | K | V, head h at columns h*hd
  void* out;         // bf16 or e4m3 [R, d]
  ActType out_type;
  float inv_q;
  int t, d, heads;
  int* status;       // device error word (a bounded wait that gave up), may be null
};
// attention.cu: per (position, head) softmax attention; builds the qkv tensor map on each call.
cudaError_t launch_attention(const AttentionParams& p, int positions, int head_dim, cudaStream_t s);
// Opt the attention kernels into their dynamic shared memory (once per device).
cudaError_t prepare_attention();

struct HeadsParams {
  const __half* x;            // [R, d] residual stream after the last layer
  const float* final_g;       // final_norm
  const float* final_b;
  const float* policy_g;      // policy_head.norm
  const float* policy_b;
  const float* policy_w;      // [73, d] f32
  const float* policy_bias;   // [73]
  const float* value_g;       // value_head.norm
  const float* value_b;
  const int32_t* legal;       // [B, slots] action indices, -1 padded; NULL = every action in order
  int slots;                  // 224, or 4672 for raw logits
  int softmax;                // 1: priors (softmax over the legal slots), 0: raw logits
  float* priors;              // [B, slots]
  void* value_in;             // bf16 [B, d]: LN_value(LN_final(x[pos, 0])) for the value GEMM
  int* status;                // device error word: action index out of range
  float eps;
  int t, square_start;
};
cudaError_t launch_heads(const HeadsParams& p, int positions, int d, cudaStream_t s);

struct ValueOutParams {
  const void* hidden;   // bf16 [B, d] GELU(value_ff1)
  const float* w2;      // [3, d]
  const float* b2;      // [3]
  float* wdl;           // [B, 3]
  int softmax;          // 1: probabilities, 0: logits
};
cudaError_t launch_value_out(const ValueOutParams& p, int positions, int d, cudaStream_t s);

// out[i] = f16(in[i]) (round to nearest) for count values, count a multiple of 4, both buffers
// 16-byte aligned: the priors in half precision for the host copy.
cudaError_t launch_priors_to_half(const float* in, __half* out, int count, cudaStream_t s);

// Loads (and so allocates the code of) every kernel above for width d, so that no later launch
// does it.
cudaError_t load_row_kernels(int d);

// Device error codes raised by these kernels (the GEMM uses 1..4).
constexpr int kErrBadAction = 16;

}  // namespace mrn
