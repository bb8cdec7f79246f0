/*
 * Kernel-level entry points of libmarina_b200_test.so, the GPU test-suite's library. They are not
 * part of the evaluator's ABI (include/marina_b200.h) and the evaluator library does not export
 * them: the test library is built from the same kernel sources, compiled with MRN_TEST_HOOKS,
 * plus these wrappers. Every call takes device pointers and runs on the caller's stream.
 */
#ifndef MARINA_B200_TEST_H
#define MARINA_B200_TEST_H

#include <stddef.h>
#include <stdint.h>

#if defined(MRN_BUILD_LIBRARY) && defined(__GNUC__)
#define MRN_TEST_API __attribute__((visibility("default")))
#else
#define MRN_TEST_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* One GEMM launch: out = epilogue(a[m,k] . b[n,k]^T * scale + bias). `fp8` selects the operand
 * types: 0 bf16, 1 e4m3, 2 e4m3 weights with a two-term e4m3 `a` [m, 2k] (each row's k hi codes,
 * then its k lo codes; the product is taken as (hi + lo) . b). `epilogue` is 0 bias->bf16,
 * 1 GELU->bf16, 2 GELU->e4m3 (x inv_q), 3 residual add into f16 `out`, 5 / 6 the tanh-form GELU
 * into bf16 / e4m3, 7 / 8 the erf / tanh GELU into two-term e4m3 (x inv_q) [m, 2n] (fp8 = 2).
 * `pair`: -1 the evaluator's planning rule, 0 single-CTA tiles, 1 CTA-pair tiles (N % 256 == 0). */
MRN_TEST_API int mrn_test_gemm(int fp8, int epilogue, int pair, const void* a, const void* b, const float* bias,
                               void* out, int ldo, int m, int n, int k, float scale, float inv_q, int* status,
                               void* stream);

/* A bf16 bias GEMM (k < 1024, the single-CTA kernel) whose TMA producer issues no loads, with
 * every bounded wait limited to `wait_limit_ns`: the MMA and epilogue warps' waits run out, the
 * kernel records the error code in `status` (zeroed by the caller), frees its tensor memory and
 * returns; no copy or MMA is ever in flight. Synchronises `stream`, restores the 2 s default
 * limit and returns MRN_ERR_DEVICE_FAULT (6) with the code in the message when a wait gave up,
 * as the evaluator's entry points do. */
MRN_TEST_API int mrn_test_gemm_wait_expiry(unsigned long long wait_limit_ns, const void* a, const void* b,
                                           const float* bias, void* out, int m, int n, int k, int* status,
                                           void* stream);

/* The attention kernel on its own: per (position, head), softmax(Q K^T / sqrt(hd)) V over the
 * position's 65 tokens from bf16 qkv [positions*65, 3d] (Q | K | V, head h at columns h*hd) into
 * out [positions*65, d], bf16 (`e4m3` 0), e4m3 codes of the value * inv_q (1), or two-term e4m3
 * codes of it (2: rows of 2d bytes, the d hi codes then the d lo codes). */
MRN_TEST_API int mrn_test_attention(const void* qkv, void* out, int positions, int d, int heads, int e4m3,
                                    float inv_q, int* status, void* stream);

/* The LayerNorm kernel on its own: out[rows,d] = LN(x) * gamma + beta from f16 x, as bf16
 * (`e4m3` 0), e4m3 codes of the value * inv_q (1) or two-term e4m3 codes of it (2, as above). */
MRN_TEST_API int mrn_test_layernorm(const void* x, const float* gamma, const float* beta, float eps, int e4m3,
                                    float inv_q, void* out, int rows, int d, void* stream);

MRN_TEST_API const char* mrn_test_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* MARINA_B200_TEST_H */
