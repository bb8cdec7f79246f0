/*
 * marina_b200: a B200 (sm_100a) evaluator for Marina's leaf batches.
 *
 * C ABI of the CUDA library that replaces the reference's CUDA backend behind its
 * `Network` trait (src/net/mod.rs:290-296). A host shim implementing `Network` packs
 * each leaf batch the way the reference's CUDA backend does (src/net/cuda/mod.rs:946-967)
 * and calls `mrn_evaluate`; nothing else in the engine changes.
 *
 * Conventions
 *   - Every function that can fail returns an `mrn_status` (0 = success). The message of
 *     the last failure on a context is `mrn_last_error(ctx)`; failures of `mrn_create`
 *     (no context yet) are reported by `mrn_last_error(NULL)` on the calling thread.
 *   - The caller owns every host buffer it passes; the library owns the device memory,
 *     pinned staging buffers, streams and CUDA graphs of a context.
 *   - One context per GPU. Calls on one context may come from any thread (the device is made
 *     current on each call); the library serialises them, and the GPU work of each pass waits
 *     for the context's previous pass even when the two were enqueued on different streams
 *     (except while the caller's stream is being captured into a graph, where ordering the
 *     captured work is the caller's).
 *   - There is no CPU fallback: without a usable sm_100 device `mrn_create` fails.
 */
#ifndef MARINA_B200_H
#define MARINA_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(MRN_BUILD_LIBRARY) && defined(__GNUC__)
#define MRN_API __attribute__((visibility("default")))
#else
#define MRN_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Bytes per position of the board upload: 64 piece tokens (canonical square order, 0 empty,
 * 1-6 own, 7-12 opponent), castling bits, en-passant file + 1. Same packing as the
 * reference's BOARD_BYTES (src/net/cuda/mod.rs:51, :951-956). */
#define MRN_BOARD_BYTES 66
/* Legal-action slots per position; unused slots hold -1 (src/net/cuda/mod.rs:53-54). */
#define MRN_MAX_LEGAL 224
/* Policy planes per square and the size of the action space (src/encoding/action.rs:17-18). */
#define MRN_POLICY_PLANES 73
#define MRN_ACTIONS (64 * MRN_POLICY_PLANES)
#define MRN_WDL 3

typedef enum mrn_status {
  MRN_OK = 0,
  MRN_ERR_ARGUMENT = 1,          /* bad pointer, size or card field */
  MRN_ERR_CUDA = 2,              /* a CUDA runtime call failed */
  MRN_ERR_BATCH_TOO_LARGE = 3,   /* n > max_batch (CudaError::BatchTooLarge, src/net/cuda/mod.rs:69-70) */
  MRN_ERR_TOO_MANY_MOVES = 4,    /* a legal list longer than MRN_MAX_LEGAL (CudaError::TooManyMoves, :71-72) */
  MRN_ERR_UNSUPPORTED = 5,       /* architecture the kernels do not cover (head dim, width, tokens) */
  MRN_ERR_DEVICE_FAULT = 6,      /* a kernel reported a device-side failure (a bounded wait gave up) */
  MRN_ERR_ACTION = 7,            /* an action index outside [0, MRN_ACTIONS) */
} mrn_status;

/* Arithmetic of the linear layers. */
typedef enum mrn_precision {
  /* bf16 weights and activations on tcgen05 kind::f16, f32 accumulation. In every precision the
   * residual stream is f16 (each residual add computed in f32 and rounded to f16), as in the
   * reference's CUDA backend (src/net/cuda/mod.rs:1-2, :193). */
  MRN_PRECISION_BF16 = 0,
  /* Weights quantised to e4m3 with one scale per matrix (src/net/cuda/mod.rs:376-405),
   * activations bf16: the e4m3 codes run on kind::f16 exactly, the scale is applied in the
   * epilogue. Same weights as MRN_PRECISION_FP8, bf16 accuracy. */
  MRN_PRECISION_FP8_WEIGHTS = 1,
  /* e4m3 weights and e4m3 activations with static per-tensor scales from the card's
   * calibration (src/net/model.rs:87-95, src/net/cuda/mod.rs:454-466), tcgen05
   * kind::f8f6f4. The reference's FP8 path (src/net/cuda/mod.rs:10-18). */
  MRN_PRECISION_FP8 = 2,
  /* e4m3 weights as MRN_PRECISION_FP8; each activation v carried as two e4m3 terms with the
   * same static scale s, hi = e4m3(v / s) and lo = e4m3(v / s - hi), and every GEMM K-step issued
   * twice (hi and lo against the same weight codes) into one f32 accumulator: kind::f8f6f4 with
   * about twice e4m3's significant bits per activation. Needs the calibration, like FP8. */
  MRN_PRECISION_FP8_X2 = 3,
} mrn_precision;

typedef enum mrn_gelu {
  MRN_GELU_ERF = 0,  /* 0.5 x (1 + erf(x / sqrt 2))                     (Gelu::Erf, src/net/model.rs:61-63) */
  MRN_GELU_TANH = 1, /* 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))) (Gelu::Tanh, :64-65) */
} mrn_gelu;

/* The architecture card, as `Architecture` (src/net/model.rs:85-103). */
typedef struct mrn_arch {
  int32_t d_model;
  int32_t n_layers;
  int32_t n_heads;
  int32_t d_ff;
  float layer_norm_eps;
  int32_t gelu;               /* mrn_gelu */
  int32_t tokens;             /* 65 in board mode */
  int32_t square_token_start; /* 1 in board mode */
  /* Per layer the four activation maxima (norm1 out, attention out, norm2 out, GELU out),
   * [n_layers * 4], or NULL when the card has no calibration (then MRN_PRECISION_FP8 and
   * MRN_PRECISION_FP8_X2 are refused). */
  const float* fp8_amax;
} mrn_arch;

/* fp32 parameters in PyTorch layout, as `Weights` (src/net/weights.rs:31-89). A Linear's
 * weight is [out_features, in_features] row-major. */
typedef struct mrn_linear {
  const float* weight;
  const float* bias;
} mrn_linear;

typedef struct mrn_norm {
  const float* weight; /* gamma [d] */
  const float* bias;   /* beta [d] */
} mrn_norm;

typedef struct mrn_layer {
  mrn_norm norm1;
  mrn_linear in_proj;  /* [3d, d]: Q; K; V */
  mrn_linear out_proj; /* [d, d] */
  mrn_norm norm2;
  mrn_linear linear1;  /* [d_ff, d] */
  mrn_linear linear2;  /* [d, d_ff] */
} mrn_layer;

typedef struct mrn_weights {
  const float* piece_embed;      /* [13, d] */
  const float* square_embed;     /* [64, d] */
  const float* state_embed;      /* [d] */
  mrn_linear castling_proj;      /* [d, 4], [d] */
  const float* en_passant_embed; /* [9, d] */
  const mrn_layer* layers;       /* [n_layers] */
  mrn_norm final_norm;
  mrn_norm policy_norm;
  mrn_linear policy_proj;        /* [73, d] */
  mrn_norm value_norm;
  mrn_linear value_ff1;          /* [d, d] */
  mrn_linear value_ff2;          /* [3, d] */
} mrn_weights;

typedef struct mrn_ctx mrn_ctx;

/* Load `weights` onto CUDA device `device` and size every buffer for `max_batch` positions.
 * Replaces `CudaNetwork::new(arch, &weights, ordinal, max_batch, fp8)`
 * (src/net/cuda/mod.rs:276-493). The weights are copied; the caller may free them after the
 * call returns. */
MRN_API int mrn_create(const mrn_arch* arch, const mrn_weights* weights, int device, int max_batch, int precision,
               mrn_ctx** out);

/* Evaluate `n` positions from host memory. `boards` is n x MRN_BOARD_BYTES, `legal` is
 * n x MRN_MAX_LEGAL action indices (square * 73 + plane) padded with -1. On success
 * `priors` (n x MRN_MAX_LEGAL) holds the softmax over each position's legal actions in slot
 * order (0 on padding) and `wdl` (n x 3) the win/draw/loss probabilities.
 * Replaces `CudaNetwork::forward` (src/net/cuda/mod.rs:919-982); the `Evaluation` of leaf p
 * is priors[p*224 .. p*224 + legal_count] and wdl[p*3 .. p*3+3] (:994-999). */
MRN_API int mrn_evaluate(mrn_ctx* ctx, int n, const uint8_t* boards, const int32_t* legal, float* priors, float* wdl);

/* `mrn_evaluate` with the priors returned as IEEE half-precision bit patterns (n x MRN_MAX_LEGAL
 * uint16_t, rounded to nearest on the device), halving the bytes copied back per position from
 * 896 to 448; `wdl` stays f32. The output format the reference's `Evaluation` gets is f32
 * (src/net/mod.rs:266-271), so a caller widens the legal slots it reads; the half rounding
 * (relative 2^-11) is far inside the priors' tolerance. The first call allocates a
 * max_batch x 224 x 2-byte device buffer. */
MRN_API int mrn_evaluate_f16(mrn_ctx* ctx, int n, const uint8_t* boards, const int32_t* legal, uint16_t* priors,
                             float* wdl);

/* Raw logits over all MRN_ACTIONS actions (`policy`, n x 4672, action-index order) and the
 * WDL logits (`value`, n x 3), the analogue of `CpuNetwork::logits` (src/net/cpu.rs:40-46)
 * for parity checks. */
MRN_API int mrn_logits(mrn_ctx* ctx, int n, const uint8_t* boards, float* policy, float* value);

/* The same forward pass as `mrn_evaluate` on device-resident inputs and outputs, enqueued on
 * `stream` (a cudaStream_t; NULL = the context's own stream) without synchronising. Used by
 * callers that keep their batches on the GPU. Check `mrn_status_word` after synchronising. */
MRN_API int mrn_evaluate_device(mrn_ctx* ctx, int n, const uint8_t* d_boards, const int32_t* d_legal, float* d_priors,
                        float* d_wdl, void* stream);

/* Read and clear the device-side error word of the context (0 = no device fault since the
 * last call). Synchronises the context's stream. */
MRN_API int mrn_status_word(mrn_ctx* ctx, int* word);

/* Per kernel class, the device time of one eager forward pass of `n` device-resident
 * positions, measured with CUDA events on `stream` around every launch. `times_ms` receives
 * MRN_PROFILE_SLOTS values (see the enum), `flops` the algorithmic FLOPs of each class and
 * `launches` the number of kernel launches of each class. */
enum mrn_profile_slot {
  MRN_PROFILE_EMBED = 0,
  MRN_PROFILE_LAYERNORM = 1,
  MRN_PROFILE_GEMM = 2,
  MRN_PROFILE_ATTENTION = 3,
  MRN_PROFILE_HEADS = 4,
  MRN_PROFILE_SLOTS = 5,
};
MRN_API int mrn_profile(mrn_ctx* ctx, int n, const uint8_t* d_boards, const int32_t* d_legal, float* d_priors, float* d_wdl,
                void* stream, float* times_ms, double* flops, int* launches);

/* Kernel launches of one forward pass of `n` positions. */
MRN_API int mrn_launches_per_forward(mrn_ctx* ctx, int n);

/* One line describing the context, as `Network::describe` (src/net/mod.rs:295). Owned by
 * the context. */
MRN_API const char* mrn_describe(mrn_ctx* ctx);

/* Message of the last failure on `ctx`, or of the calling thread's last `mrn_create` when
 * `ctx` is NULL. Never NULL. */
MRN_API const char* mrn_last_error(mrn_ctx* ctx);

MRN_API void mrn_destroy(mrn_ctx* ctx);

/* ---- several GPUs: one weight replica per device, every batch sharded across them */
typedef struct mrn_group mrn_group;

/* One context per entry of `devices` (a device may be listed more than once), each sized for its
 * shard of `max_batch` (ceil(max_batch / n_devices) positions), plus one evaluator thread per
 * device after the first. The reference has no multi-GPU backend (it builds its CUDA network on
 * ordinal 0, src/net/mod.rs:171-192); this is the sharding wrapper that makes a whole box one
 * `Network`. Failures are reported by `mrn_group_last_error(NULL)` on the calling thread. */
MRN_API int mrn_group_create(const mrn_arch* arch, const mrn_weights* weights, const int* devices, int n_devices,
                             int max_batch, int precision, mrn_group** out);

/* `mrn_evaluate` over the group: the batch is cut into n_devices contiguous shards (sizes differ by
 * at most one position), evaluated at the same time, one per device, and written into `priors` /
 * `wdl` at the shard's offset, so the outputs are in input order. No data moves between GPUs.
 * A batch larger than the group's max_batch is evaluated as consecutive max_batch chunks cut the
 * same way; after the first chunk each device thread takes the next shard as soon as it is free,
 * without waiting for the others between chunks. On failure the message names the device and the
 * shard's positions, and shards not yet started are skipped (outputs of the batch are then
 * undefined). */
MRN_API int mrn_group_evaluate(mrn_group* group, int n, const uint8_t* boards, const int32_t* legal, float* priors,
                               float* wdl);
MRN_API int mrn_group_size(mrn_group* group);
/* The context of the group's i-th device (owned by the group). */
MRN_API mrn_ctx* mrn_group_context(mrn_group* group, int i);
MRN_API const char* mrn_group_describe(mrn_group* group);
/* Message of the last failure on `group`, or of the calling thread's last `mrn_group_create`
 * when `group` is NULL. Never NULL. */
MRN_API const char* mrn_group_last_error(mrn_group* group);
MRN_API void mrn_group_destroy(mrn_group* group);

/* The forward pass of `mrn_evaluate_device` for callers that cannot allocate device memory
 * once running (a host whose device memory belongs to another allocator, a thread that must
 * not stall on an allocation, a device that is already full). It allocates nothing: all
 * intermediate buffers live in one 8 MiB array compiled into the library. `mrn_create` looks
 * the array up on its device (which is when the driver allocates it) and loads every kernel
 * the pass launches, so the array stays resident on every GPU that has had a context, for the
 * life of the process. Batches are limited to what fits that array (12 positions for the
 * `small` network in bf16/fp8w, 17 in fp8; 33 / 47 for `nano`); larger ones return
 * MRN_ERR_BATCH_TOO_LARGE. Inputs and outputs are the caller's device buffers, as for
 * `mrn_evaluate_device`. Every call on a device shares the array, so calls whose GPU work
 * overlaps (through other contexts on the same device) corrupt each other's results: serialise
 * them. This entry point has no counterpart in the reference. */
MRN_API int mrn_evaluate_device_static(mrn_ctx* ctx, int n, const uint8_t* d_boards, const int32_t* d_legal,
                                       float* d_priors, float* d_wdl, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MARINA_B200_H */
