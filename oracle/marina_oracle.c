/*
 * CPU oracle for Marina's batched transformer forward -- TEST INFRASTRUCTURE ONLY.
 * A restatement of src/net/cpu.rs (see marina_oracle.h for the scope and the pins).
 * Only the tests, the smoke check and the benchmark's CPU-baseline leg load it.
 */
#include "marina_oracle.h"

#include <float.h>
#include <math.h>
#include <omp.h>
#include <stdlib.h>
#include <string.h>

#define PLANES 73
#define ACTIONS (64 * PLANES)
#define MAX_LEGAL 224
#define ROWS_PER_CALL 512 /* src/net/cpu.rs:352 */

/* ---- math helpers ------------------------------------------------------------------ */

/* src/net/cpu.rs:239-253: Cephes expf with a 2-constant range reduction. */
float oracle_exp_fast(float x) {
  const float c1 = 0.6933594f;
  const float c2 = -2.1219444e-4f;
  x = x < -87.0f ? -87.0f : (x > 88.0f ? 88.0f : x);
  const float k = roundf(x * 1.44269504088896341f); /* f32::round: half away from zero */
  const float r = x - k * c1 - k * c2;
  const float poly =
      ((((1.9875692e-4f * r + 1.3981999e-3f) * r + 8.333452e-3f) * r + 4.1665796e-2f) * r + 1.6666665e-1f) * r +
      0.5f;
  const float e = poly * r * r + r + 1.0f;
  union {
    uint32_t u;
    float f;
  } scale;
  scale.u = (uint32_t)((int32_t)k + 127) << 23;
  return e * scale.f;
}

/* src/net/cpu.rs:288-302: Abramowitz & Stegun 7.1.26. */
float oracle_erf(float x) {
  const float p = 0.3275911f;
  const float a0 = 0.2548296f, a1 = -0.28449672f, a2 = 1.4214137f, a3 = -1.453152f, a4 = 1.0614054f;
  const float sign = x < 0.0f ? -1.0f : 1.0f;
  x = fabsf(x);
  const float t = 1.0f / (1.0f + p * x);
  const float poly = ((((a4 * t + a3) * t + a2) * t + a1) * t + a0) * t;
  return sign * (1.0f - poly * oracle_exp_fast(-x * x));
}

/* src/net/cpu.rs:257-259 */
float oracle_gelu(float x) { return 0.5f * x * (1.0f + oracle_erf(x * 0.70710678118654752f)); }

/* src/net/cpu.rs:270-276 */
float oracle_gelu_tanh(float x) {
  const float sqrt_2_over_pi = 0.7978846f;
  float u = sqrt_2_over_pi * (x + 0.044715f * x * x * x);
  u = u < -20.0f ? -20.0f : (u > 20.0f ? 20.0f : u);
  const float e = oracle_exp_fast(2.0f * u);
  return 0.5f * x * (2.0f - 2.0f / (e + 1.0f));
}

/* src/net/cpu.rs:306-313: exponentiate values - max in place, return the sum. */
static float softmax_inplace(float* v, int n, float max) {
  float sum = 0.0f;
  for (int i = 0; i < n; ++i) {
    v[i] = oracle_exp_fast(v[i] - max);
    sum += v[i];
  }
  return sum;
}

/* src/net/cpu.rs:364-371 */
void oracle_softmax(float* v, int n) {
  float max = -INFINITY;
  for (int i = 0; i < n; ++i) max = v[i] > max ? v[i] : max;
  const float sum = softmax_inplace(v, n, max);
  const float inv = 1.0f / (sum > FLT_MIN ? sum : FLT_MIN);
  for (int i = 0; i < n; ++i) v[i] *= inv;
}

/* src/net/cpu.rs:205-219: eight independent accumulators, then the tail. */
static float dot(const float* a, const float* b, int n) {
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  int i = 0;
  for (; i + 8 <= n; i += 8)
    for (int j = 0; j < 8; ++j) acc[j] += a[i + j] * b[i + j];
  float sum = 0.0f;
  for (int j = 0; j < 8; ++j) sum += acc[j];
  for (; i < n; ++i) sum += a[i] * b[i];
  return sum;
}

/* src/net/cpu.rs:223-234 */
static void axpy(float a, const float* x, float* y, int n) {
  for (int i = 0; i < n; ++i) y[i] += a * x[i];
}

/* src/net/cpu.rs:330-343: biased variance, as PyTorch. */
static void layer_norm_row(const float* row, float* out, const float* g, const float* b, int d, float eps) {
  float sum = 0.0f;
  for (int i = 0; i < d; ++i) sum += row[i];
  const float mean = sum / (float)d;
  float var = 0.0f;
  for (int i = 0; i < d; ++i) var += (row[i] - mean) * (row[i] - mean);
  var /= (float)d;
  const float inv = 1.0f / sqrtf(var + eps);
  for (int i = 0; i < d; ++i) out[i] = (row[i] - mean) * inv * g[i] + b[i];
}

void oracle_layer_norm(const float* input, float* output, const float* gamma, const float* beta, int rows, int d,
                       float eps) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; ++r)
    layer_norm_row(input + (size_t)r * d, output + (size_t)r * d, gamma, beta, d, eps);
}

/* ---- GEMM ------------------------------------------------------------------------------
 * c[m, n] += a[m, k] . w[n, k]^T. The weight is packed once into k-major panels of 32 columns
 * and an outer-product micro-kernel keeps a 4 x 32 block of c in registers (the register blocking
 * of a BLIS-style sgemm, which is how matrixmultiply -- the reference's Linux sgemm -- works). */
typedef float v16 __attribute__((vector_size(64)));

__attribute__((target_clones("avx512f", "avx2", "default"))) static void kernel_4x32(int k, const float* a,
                                                                                        int lda, const float* bt,
                                                                                        int ldb, float* c, int ldc) {
  v16 acc[4][2];
  for (int i = 0; i < 4; ++i)
    for (int j = 0; j < 2; ++j) memcpy(&acc[i][j], c + (size_t)i * ldc + 16 * j, sizeof(v16));
  for (int p = 0; p < k; ++p) {
    v16 b0, b1;
    memcpy(&b0, bt + (size_t)p * ldb, sizeof(v16));
    memcpy(&b1, bt + (size_t)p * ldb + 16, sizeof(v16));
    for (int i = 0; i < 4; ++i) {
      const float ai = a[(size_t)i * lda + p];
      acc[i][0] += ai * b0;
      acc[i][1] += ai * b1;
    }
  }
  for (int i = 0; i < 4; ++i)
    for (int j = 0; j < 2; ++j) memcpy(c + (size_t)i * ldc + 16 * j, &acc[i][j], sizeof(v16));
}

/* The weight [n, k] repacked as ceil(n/32) contiguous k x 32 column panels (zero-padded), so
 * the micro-kernel streams its operand sequentially. */
static float* pack_panels(const float* w, int n, int k) {
  const int panels = (n + 31) / 32;
  float* t = (float*)calloc((size_t)panels * k * 32, sizeof(float));
  for (int j = 0; j < n; ++j)
    for (int p = 0; p < k; ++p) t[((size_t)(j / 32) * k + p) * 32 + (j % 32)] = w[(size_t)j * k + p];
  return t;
}

/* c[m, n] += a . w^T with w given as packed panels; ragged row or column blocks run the
 * kernel on a zero-padded copy. */
static void gemm_panels(int m, int k, int n, const float* a, const float* panels, float* c) {
  float tmp[4 * 32];
  float* ab = NULL;
  for (int jb = 0; jb < n; jb += 32) {
    const float* bp = panels + (size_t)(jb / 32) * k * 32;
    const int nc = n - jb < 32 ? n - jb : 32;
    int i = 0;
    if (nc == 32)
      for (; i + 4 <= m; i += 4) kernel_4x32(k, a + (size_t)i * k, k, bp, 32, c + (size_t)i * n + jb, n);
    for (; i < m; i += 4) {
      const int mr = m - i < 4 ? m - i : 4;
      memset(tmp, 0, sizeof(tmp));
      for (int r = 0; r < mr; ++r) memcpy(tmp + r * 32, c + (size_t)(i + r) * n + jb, sizeof(float) * nc);
      const float* arows = a + (size_t)i * k;
      if (mr < 4) {
        if (!ab) ab = (float*)malloc(sizeof(float) * 4 * (size_t)k);
        memset(ab, 0, sizeof(float) * 4 * (size_t)k);
        memcpy(ab, arows, sizeof(float) * (size_t)mr * k);
        arows = ab;
      }
      kernel_4x32(k, arows, k, bp, 32, tmp, 32);
      for (int r = 0; r < mr; ++r) memcpy(c + (size_t)(i + r) * n + jb, tmp + r * 32, sizeof(float) * nc);
    }
  }
  free(ab);
}

void oracle_sgemm_nt(int m, int k, int n, const float* a, const float* w, float* c) {
  if (m == 0 || n == 0) return;
  float* panels = pack_panels(w, n, k);
  gemm_panels(m, k, n, a, panels, c);
  free(panels);
}

/* src/net/cpu.rs:346-362: each 512-row slice starts from the bias and gets one GEMM call. */
void oracle_linear(const float* input, float* output, const float* weight, const float* bias, int rows, int in_f,
                   int out_f, int threads) {
  float* panels = pack_panels(weight, out_f, in_f);
  const int slices = (rows + ROWS_PER_CALL - 1) / ROWS_PER_CALL;
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads)
  for (int s = 0; s < slices; ++s) {
    const int r0 = s * ROWS_PER_CALL;
    const int m = rows - r0 < ROWS_PER_CALL ? rows - r0 : ROWS_PER_CALL;
    float* out = output + (size_t)r0 * out_f;
    for (int r = 0; r < m; ++r) memcpy(out + (size_t)r * out_f, bias, sizeof(float) * out_f);
    gemm_panels(m, in_f, out_f, input + (size_t)r0 * in_f, panels, out);
  }
  free(panels);
}

static float max_abs(const float* v, size_t n) {
  float m = 0.0f;
  for (size_t i = 0; i < n; ++i) m = fabsf(v[i]) > m ? fabsf(v[i]) : m;
  return m;
}

/* ---- the forward pass (src/net/cpu.rs:48-164) ----------------------------------------- */
int oracle_logits(const oracle_arch_t* arch, const oracle_weights_t* w, int n, const uint8_t* boards, float* policy,
                  float* value, float* amax, int threads) {
  if (n < 0 || !arch || !w) return -1;
  if (n == 0) return 0;
  const int t = arch->tokens, d = arch->d_model, ff = arch->d_ff, heads = arch->n_heads;
  if (d % heads != 0 || arch->square_token_start < 1 || arch->square_token_start + 64 != t) return -1;
  if (threads < 1) threads = 1;
  const size_t rows = (size_t)n * t;
  const int hd = d / heads;
  const float scale = 1.0f / sqrtf((float)hd);
  const float eps = arch->layer_norm_eps;

  float* x = (float*)calloc(rows * d, sizeof(float));
  float* h = (float*)calloc(rows * d, sizeof(float));
  float* qkv = (float*)calloc(rows * 3 * d, sizeof(float));
  float* attn = (float*)calloc(rows * d, sizeof(float));
  float* f = (float*)calloc(rows * ff, sizeof(float));
  float* proj = (float*)calloc(rows * d, sizeof(float));
  if (!x || !h || !qkv || !attn || !f || !proj) {
    free(x), free(h), free(qkv), free(attn), free(f), free(proj);
    return -1;
  }

  /* tokens (src/net/cpu.rs:59-84) */
#pragma omp parallel for schedule(static) num_threads(threads)
  for (int p = 0; p < n; ++p) {
    const uint8_t* b = boards + (size_t)p * 66;
    float* state = x + (size_t)p * t * d;
    memcpy(state, w->state_embed, sizeof(float) * d);
    float bits[4];
    for (int k = 0; k < 4; ++k) bits[k] = (float)((b[64] >> k) & 1);
    for (int o = 0; o < d; ++o) {
      const float* row = w->castling_proj.weight + (size_t)o * 4;
      float s = 0.0f;
      for (int k = 0; k < 4; ++k) s += row[k] * bits[k];
      state[o] += w->castling_proj.bias[o] + s;
    }
    const int ep = b[65] < 8 ? b[65] : 8;
    for (int c = 0; c < d; ++c) state[c] += w->en_passant_embed[(size_t)ep * d + c];
    float* squares = x + ((size_t)p * t + arch->square_token_start) * d;
    for (int s = 0; s < 64; ++s) {
      const int piece = b[s] < 13 ? b[s] : 0;
      float* tok = squares + (size_t)s * d;
      for (int c = 0; c < d; ++c) tok[c] = w->piece_embed[(size_t)piece * d + c] + w->square_embed[(size_t)s * d + c];
    }
  }

  /* encoder (src/net/cpu.rs:86-137) */
  for (int li = 0; li < arch->n_layers; ++li) {
    const oracle_layer_t* L = &w->layers[li];
    oracle_layer_norm(x, h, L->norm1.weight, L->norm1.bias, (int)rows, d, eps);
    if (amax) amax[li * 4 + 0] = max_abs(h, rows * d);
    oracle_linear(h, qkv, L->in_proj.weight, L->in_proj.bias, (int)rows, d, 3 * d, threads);
#pragma omp parallel for schedule(static) num_threads(threads)
    for (int p = 0; p < n; ++p) {
      const float* q0 = qkv + (size_t)p * t * 3 * d;
      float* out = attn + (size_t)p * t * d;
      float* scores = (float*)malloc(sizeof(float) * t);
      for (int head = 0; head < heads; ++head) {
        const int qo = head * hd, ko = d + head * hd, vo = 2 * d + head * hd;
        for (int i = 0; i < t; ++i) {
          const float* q = q0 + (size_t)i * 3 * d + qo;
          float max = -INFINITY;
          for (int j = 0; j < t; ++j) {
            scores[j] = dot(q, q0 + (size_t)j * 3 * d + ko, hd) * scale;
            max = scores[j] > max ? scores[j] : max;
          }
          const float inv = 1.0f / softmax_inplace(scores, t, max);
          float* o = out + (size_t)i * d + qo;
          memset(o, 0, sizeof(float) * hd);
          for (int j = 0; j < t; ++j) axpy(scores[j] * inv, q0 + (size_t)j * 3 * d + vo, o, hd);
        }
      }
      free(scores);
    }
    if (amax) amax[li * 4 + 1] = max_abs(attn, rows * d);
    oracle_linear(attn, proj, L->out_proj.weight, L->out_proj.bias, (int)rows, d, d, threads);
#pragma omp parallel for schedule(static) num_threads(threads)
    for (size_t i = 0; i < rows * d; ++i) x[i] += proj[i];
    oracle_layer_norm(x, h, L->norm2.weight, L->norm2.bias, (int)rows, d, eps);
    if (amax) amax[li * 4 + 2] = max_abs(h, rows * d);
    oracle_linear(h, f, L->linear1.weight, L->linear1.bias, (int)rows, d, ff, threads);
    if (arch->gelu == 1) {
#pragma omp parallel for schedule(static) num_threads(threads)
      for (size_t i = 0; i < rows * ff; ++i) f[i] = oracle_gelu_tanh(f[i]);
    } else {
#pragma omp parallel for schedule(static) num_threads(threads)
      for (size_t i = 0; i < rows * ff; ++i) f[i] = oracle_gelu(f[i]);
    }
    if (amax) amax[li * 4 + 3] = max_abs(f, rows * ff);
    oracle_linear(f, proj, L->linear2.weight, L->linear2.bias, (int)rows, ff, d, threads);
#pragma omp parallel for schedule(static) num_threads(threads)
    for (size_t i = 0; i < rows * d; ++i) x[i] += proj[i];
  }
  oracle_layer_norm(x, h, w->final_norm.weight, w->final_norm.bias, (int)rows, d, eps);

  /* heads (src/net/cpu.rs:139-163) */
  float* squares = (float*)malloc(sizeof(float) * (size_t)n * 64 * d);
  float* state = (float*)malloc(sizeof(float) * (size_t)n * d);
  for (int p = 0; p < n; ++p) {
    memcpy(state + (size_t)p * d, h + (size_t)p * t * d, sizeof(float) * d);
    memcpy(squares + (size_t)p * 64 * d, h + ((size_t)p * t + arch->square_token_start) * d, sizeof(float) * 64 * d);
  }
  oracle_layer_norm(squares, squares, w->policy_norm.weight, w->policy_norm.bias, n * 64, d, eps);
  oracle_linear(squares, policy, w->policy_proj.weight, w->policy_proj.bias, n * 64, d, PLANES, threads);
  float* vnorm = (float*)malloc(sizeof(float) * (size_t)n * d);
  float* hidden = (float*)malloc(sizeof(float) * (size_t)n * d);
  oracle_layer_norm(state, vnorm, w->value_norm.weight, w->value_norm.bias, n, d, eps);
  oracle_linear(vnorm, hidden, w->value_ff1.weight, w->value_ff1.bias, n, d, d, threads);
  for (size_t i = 0; i < (size_t)n * d; ++i) hidden[i] = oracle_gelu(hidden[i]); /* value head: erf always */
  oracle_linear(hidden, value, w->value_ff2.weight, w->value_ff2.bias, n, d, 3, threads);

  free(squares), free(state), free(vnorm), free(hidden);
  free(x), free(h), free(qkv), free(attn), free(f), free(proj);
  return 0;
}

int oracle_evaluate(const oracle_arch_t* arch, const oracle_weights_t* w, int n, const uint8_t* boards,
                    const int32_t* legal, float* priors, float* wdl, int threads) {
  if (n < 0) return -1;
  if (n == 0) return 0;
  float* policy = (float*)malloc(sizeof(float) * (size_t)n * ACTIONS);
  float* value = (float*)malloc(sizeof(float) * (size_t)n * 3);
  if (!policy || !value) {
    free(policy), free(value);
    return -1;
  }
  int rc = oracle_logits(arch, w, n, boards, policy, value, NULL, threads);
  for (int p = 0; rc == 0 && p < n; ++p) {
    const int32_t* slots = legal + (size_t)p * MAX_LEGAL;
    float* pr = priors + (size_t)p * MAX_LEGAL;
    int count = 0;
    while (count < MAX_LEGAL && slots[count] >= 0) {
      if (slots[count] >= ACTIONS) {
        rc = -1;
        break;
      }
      pr[count] = policy[(size_t)p * ACTIONS + slots[count]];
      ++count;
    }
    oracle_softmax(pr, count);
    for (int i = count; i < MAX_LEGAL; ++i) pr[i] = 0.0f;
    float* v = wdl + (size_t)p * 3;
    for (int k = 0; k < 3; ++k) v[k] = value[(size_t)p * 3 + k];
    oracle_softmax(v, 3);
  }
  free(policy), free(value);
  return rc;
}
