/*
 * CPU oracle for Marina's batched transformer forward -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's fp32 CPU backend, `CpuNetwork::forward` and
 * `CpuNetwork::evaluate` (src/net/cpu.rs:48-184), with its math helpers (exp_fast :239-253,
 * erf :288-302, gelu :257-259, gelu_tanh :270-276, softmax :304-313/:364-371, layer_norm
 * :323-343, linear :346-362, dot :205-219, axpy :223-234). The reference is Rust and cannot
 * be built in this environment, so this file is the checker the CUDA library is compared
 * against; it is never linked into, loaded by or called from the product.
 *
 * Pinning: the primitives are checked against the reference's own known-answer tests
 * (src/net/cpu.rs:377-420, src/net/gemm.rs:132-159); the whole forward pass is cross-checked
 * against an independent float64 PyTorch implementation of the same architecture. The
 * reference's trained-net golden vectors (vectors.npz) are downloaded at build time and are
 * not in the reference tree, so no output of the reference itself pins the full pass.
 */
#ifndef MARINA_ORACLE_H
#define MARINA_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct oracle_arch {
  int32_t d_model, n_layers, n_heads, d_ff;
  float layer_norm_eps;
  int32_t gelu; /* 0 erf, 1 tanh (the encoder FFN only; the value head is always erf) */
  int32_t tokens, square_token_start;
} oracle_arch_t;

typedef struct oracle_linear {
  const float* weight; /* [out, in] */
  const float* bias;   /* [out] */
} oracle_linear_t;

typedef struct oracle_norm {
  const float* weight;
  const float* bias;
} oracle_norm_t;

typedef struct oracle_layer {
  oracle_norm_t norm1;
  oracle_linear_t in_proj, out_proj;
  oracle_norm_t norm2;
  oracle_linear_t linear1, linear2;
} oracle_layer_t;

typedef struct oracle_weights {
  const float* piece_embed;      /* [13, d] */
  const float* square_embed;     /* [64, d] */
  const float* state_embed;      /* [d] */
  oracle_linear_t castling_proj;   /* [d, 4] */
  const float* en_passant_embed; /* [9, d] */
  const oracle_layer_t* layers;
  oracle_norm_t final_norm, policy_norm;
  oracle_linear_t policy_proj; /* [73, d] */
  oracle_norm_t value_norm;
  oracle_linear_t value_ff1, value_ff2;
} oracle_weights_t;

/* Raw policy logits [n, 4672] (action = square * 73 + plane) and WDL logits [n, 3] of `n`
 * 66-byte boards (`CpuNetwork::logits`, src/net/cpu.rs:40-46). When `amax` is not NULL it
 * receives, per layer, max |x| of the norm1 output, attention output, norm2 output and GELU
 * output ([n_layers * 4]; the calibration `model.json` carries, src/net/model.rs:87-95).
 * `threads` sizes the worker pool (the `Threads` option). Returns 0, or -1 on bad input. */
int oracle_logits(const oracle_arch_t* arch, const oracle_weights_t* w, int n, const uint8_t* boards, float* policy,
                  float* value, float* amax, int threads);

/* `Network::evaluate` of the CPU backend (src/net/cpu.rs:167-184): priors = softmax over each
 * position's legal logits (slots of `legal` [n, 224], -1 padded, 0 written on padding),
 * wdl = softmax of the value logits. */
int oracle_evaluate(const oracle_arch_t* arch, const oracle_weights_t* w, int n, const uint8_t* boards,
                    const int32_t* legal, float* priors, float* wdl, int threads);

/* Primitives, exposed for the known-answer tests. */
float oracle_exp_fast(float x);
float oracle_erf(float x);
float oracle_gelu(float x);
float oracle_gelu_tanh(float x);
void oracle_softmax(float* values, int n);
void oracle_layer_norm(const float* input, float* output, const float* gamma, const float* beta, int rows, int d,
                       float eps);
/* c[m, n] += a[m, k] . w[n, k]^T (src/net/gemm.rs:28-36). */
void oracle_sgemm_nt(int m, int k, int n, const float* a, const float* w, float* c);
/* output[rows, out] = input[rows, in] . weight^T + bias, 512 rows per GEMM call. */
void oracle_linear(const float* input, float* output, const float* weight, const float* bias, int rows, int in_f,
                   int out_f, int threads);

#ifdef __cplusplus
}
#endif

#endif /* MARINA_ORACLE_H */
