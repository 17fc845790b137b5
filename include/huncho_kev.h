/*
 * huncho_kev.h -- C ABI of the B200-native Kev scoring forward.
 *
 * One handle is one Kev scorer on one GPU: the Qwen3.5-hybrid backbone
 * (Gated DeltaNet + gated GQA), its merged LoRA and the fp32 pointer head, with
 * a CUDA stream and a device workspace of its own. The entry points replace the
 * reference's `Backend` trait implementation for Kev
 * (crates/huncho-core/src/backend.rs:211-438, implemented by
 * crates/huncho-backend/src/qwen3_5.rs:2515-3266). Calibration, answers and
 * batching stay with the caller (huncho-core), exactly as they do above the
 * reference trait.
 *
 * Plain pointers and sizes only. All calls on one handle must come from one
 * thread at a time (the reference backend is `&mut self`, used behind a Mutex:
 * crates/huncho-core/src/engine.rs:173-180); concurrency comes from replicas,
 * one handle per GPU (crates/huncho-api/src/replicas.rs:7-61).
 */
#ifndef HUNCHO_KEV_H
#define HUNCHO_KEV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Return codes. They map onto huncho_core::error::Error variants
 * (crates/huncho-core/src/error.rs:10-45). */
#define HK_OK 0
#define HK_ERR_BACKEND (-1)     /* Error::Backend: invalid request or failed inference  */
#define HK_ERR_UNSUPPORTED (-2) /* Error::Unsupported                                  */
#define HK_ERR_PACKAGE (-3)     /* Error::Package: unreadable or inconsistent model dir */
#define HK_ERR_CUDA (-4)        /* Error::Backend raised by a CUDA failure             */
#define HK_ERR_ARGUMENT (-5)    /* null pointer or bad enum at the C boundary          */

/* Model dtypes: the type every checkpoint tensor is cast to at load, as the
 * reference's `dtype` argument (qwen3_5.rs:2202-2210).
 *   HK_DTYPE_FP32   fp32 weights and activations (CUDA-core GEMMs).
 *   HK_DTYPE_BF16   bf16 weights; tensor-core operands run as fp16, into which
 *                   bf16 values convert exactly (|w| >= 2^-17), the way the
 *                   reference runs bf16 checkpoints as fp16 on CUDA.
 *   HK_DTYPE_INT8W  int8 per-output-channel symmetric projection weights
 *                   (scale = max|w| / 127, fp32 scales, applied in the GEMM
 *                   epilogue); other tensors as HK_DTYPE_BF16.
 *   HK_DTYPE_FP16   fp16 weights and tensor-core operands.
 *   HK_DTYPE_Q8_0 / HK_DTYPE_Q4_0
 *                   the reference's packed profiles "q8_0-fp32" / "q4_0-fp32"
 *                   (Qwen3_5Backend::load_quantized_kev, crates/huncho-backend/
 *                   src/qwen_quantized.rs:395-...): model_dir holds
 *                   backbone.gguf (the converter's artifact, qwen_quantized.rs:
 *                   91-193: merged backbone, projections in GGML Q8_0 / Q4_0
 *                   blocks of 32, everything else fp32) plus the pointer head
 *                   files. Projections quantize their fp32 inputs to Q8_0 and
 *                   sum per-block integer dots (int8 tensor cores); all other
 *                   math is the fp32 model's. An artifact of the other scheme
 *                   -> HK_ERR_PACKAGE.
 * In the half-precision models the residual stream, projection outputs and
 * all elementwise math stay fp32; only tensor-core operands are fp16. */
#define HK_DTYPE_FP32 0
#define HK_DTYPE_BF16 1
#define HK_DTYPE_INT8W 2
#define HK_DTYPE_FP16 3
#define HK_DTYPE_Q8_0 4
#define HK_DTYPE_Q4_0 5

/* The reference's hard limit on independent rows per native batch
 * (qwen3_5.rs:3143-3148; BatchLimits default, backend.rs:108-121). */
#define HK_MAX_ROWS 64

typedef struct hk_model hk_model;

typedef struct hk_capabilities {
    int32_t dtype;             /* HK_DTYPE_*                                         */
    int32_t device;            /* CUDA device ordinal                                */
    int32_t max_context;       /* longest accepted row (qwen3_5.rs:2700-2705)         */
    int32_t max_rows;          /* HK_MAX_ROWS                                        */
    int32_t hidden_size;
    int32_t num_layers;
    int32_t vocab_size;        /* input vocabulary: token ids must be below it       */
    int32_t pointer_dim;       /* pointer-head width d_p (kev.rs:97, default 256)     */
    float temperature;         /* the package's calibration temperature (kev.rs:86)  */
    int32_t lora_rank;         /* 0 when no adapter was merged                       */
} hk_capabilities;

/*
 * Load a Kev model directory onto `device`:
 *   config.json, base *.safetensors (any of the HF text/conditional/PEFT name
 *   prefixes), optional adapter_model.safetensors + adapter_config.json (merged
 *   in fp32 as W += (alpha/r) B A), pointer_head.safetensors + kev_head.json.
 * Replaces Qwen3_5Backend::load_kev_on_device (qwen3_5.rs:2086-2111 ->
 * load_with_head 2185-2348).
 */
int hk_create(const char *model_dir, int device, int dtype, int max_context, hk_model **out);

/* The same model on `device` (another GPU or the source's own), with fresh
 * mutable state (stream, workspace, caches, KV page setting). On the source's
 * own GPU the new handle shares the source's weights (one device copy, freed
 * with the last handle that uses it); on another GPU the package is loaded
 * again. Handles may run concurrently from different host threads. Replaces
 * Backend::replica (backend.rs:217-222; qwen3_5.rs:2515-2535). */
int hk_replica(const hk_model *src, int device, hk_model **out);

/* Replaces Backend::capabilities (qwen3_5.rs:2541-2653). */
int hk_capabilities_get(const hk_model *m, hk_capabilities *out);

/*
 * Score `n_rows` independent rows (a packed, unpadded batch).
 *   tokens       [cu_seqlens[n_rows]]   row r is tokens[cu_seqlens[r] .. cu_seqlens[r+1])
 *   cu_seqlens   [n_rows + 1]           cu_seqlens[0] == 0, non-decreasing
 *   positions    [cu_positions[n_rows]] readout positions, relative to their row
 *   cu_positions [n_rows + 1]
 *   out_logits   [cu_positions[n_rows]] raw pointer logits, in input order
 * The decision row of every row is its last token. Synchronous; all buffers
 * are caller-owned host memory. Validation follows the reference: 1..=64
 * rows, no empty row, every token below the vocabulary, every position inside
 * its row, every row within max_context (qwen3_5.rs:2669-2705, 3143-3171).
 * Replaces Backend::forward / forward_batch / forward_padded_batch
 * (qwen3_5.rs:2655-2753, 2759-2761, 2806-2816 -> 3138-3194 + readout 3196-3255);
 * right padding is not needed because rows are packed.
 */
int hk_score(hk_model *m, int n_rows, const uint32_t *tokens, const int32_t *cu_seqlens,
             const int32_t *positions, const int32_t *cu_positions, float *out_logits);

/*
 * hk_score plus calibrated answers computed on the device, one question per
 * row (the reference calibrates on the host after Backend::forward; the
 * arithmetic is its own: crates/huncho-core/src/calibration.rs:36-64
 * temperature softmax with fp32 exponentials and an fp64 sum and division,
 * 87-95 first-maximum argmax, 114-127 peak confidence, 131-147 Kev's score
 * confidence, 172-218 validation; Engine::build_answer,
 * crates/huncho-core/src/engine.rs:1448-1513).
 *   question_types [n_rows] HK_QUESTION_CHOICE, HK_QUESTION_NOUL (exactly two
 *                  options, in the order [no, yes]) or HK_QUESTION_SCORE
 *                  (options are the levels 0, 1, ...)
 *   temperature    the package temperature (finite and > 0, else
 *                  HK_ERR_ARGUMENT)
 *   out_logits     [cu_positions[n_rows]] raw pointer logits, or NULL
 *   out_probs      [cu_positions[n_rows]] calibrated probabilities
 *   out_answers    [n_rows]
 * Every question needs at least one option, else HK_ERR_ARGUMENT. A question
 * whose logits or probabilities are not finite gets status
 * HK_ANSWER_NONFINITE_LOGITS / HK_ANSWER_NONFINITE_PROBS (the reference
 * rejects such a request with a calibration error).
 */
#define HK_QUESTION_CHOICE 0
#define HK_QUESTION_NOUL 1
#define HK_QUESTION_SCORE 2
#define HK_ANSWER_OK 0
#define HK_ANSWER_NONFINITE_LOGITS 1
#define HK_ANSWER_NONFINITE_PROBS 2
typedef struct hk_answer {
    int32_t best;     /* first-maximum option index (choice: the chosen label) */
    int32_t status;   /* HK_ANSWER_* */
    float confidence; /* peak confidence; Kev's score confidence for score questions */
    float value;      /* noul: P(yes); score: sum_i i * p_i; choice: p[best] */
} hk_answer;
int hk_score_answers(hk_model *m, int n_rows, const uint32_t *tokens, const int32_t *cu_seqlens,
                     const int32_t *positions, const int32_t *cu_positions, const int32_t *question_types,
                     float temperature, float *out_logits, float *out_probs, hk_answer *out_answers);

/*
 * Cached prefixes (prefill / fork). A cache handle names the model state after
 * a token sequence: every delta layer's recurrent state and conv tail, every
 * attention layer's K/V (the reference's LayerCache, qwen3_5.rs:1111-1125),
 * held in device memory. Handles are 64-bit ids; 0 is never a handle.
 *
 * hk_score_cached scores rows that may each continue a cached prefix:
 *   parents      [n_rows] handle per row, 0 for an independent row (or NULL
 *                for none); a row's tokens are the suffix after its prefix,
 *                its positions are relative to the suffix, and its attention
 *                and RoPE positions continue at the prefix length.
 *   mode         HK_CACHE_BRANCH: rows read their parents and leave them
 *                unchanged (Backend::forward_fork_batch and
 *                forward_padded_fork_batch, qwen3_5.rs:2780-2804, across any
 *                number of parents in one call, up to HK_MAX_CACHED_ROWS rows);
 *                HK_CACHE_CONTINUE: each row's handle advances to the state
 *                after its suffix (Backend::forward with fork_from,
 *                qwen3_5.rs:2676-2751); every row needs a distinct handle;
 *                HK_CACHE_PREFILL: each row's final state becomes a new handle
 *                in handles_out[r] (a row with a parent extends it).
 *   out_logits   as hk_score. State commits only after the whole call
 *                succeeds. Errors: unknown handle or empty suffix ->
 *                HK_ERR_BACKEND; prefix + suffix beyond max_context ->
 *                HK_ERR_BACKEND.
 */
#define HK_MAX_CACHED_ROWS 256 /* rows per hk_score_cached / hk_prefill call */
#define HK_CACHE_BRANCH 0
#define HK_CACHE_CONTINUE 1
#define HK_CACHE_PREFILL 2
int hk_score_cached(hk_model *m, int n_rows, const uint64_t *parents, int mode, const uint32_t *tokens,
                    const int32_t *cu_seqlens, const int32_t *positions, const int32_t *cu_positions,
                    float *out_logits, uint64_t *handles_out);

/* Backend::prefill (qwen3_5.rs:2833-2835) for n_rows prefixes at once: one
 * new handle per row in handles_out, no readout. */
int hk_prefill(hk_model *m, int n_rows, const uint32_t *tokens, const int32_t *cu_seqlens, uint64_t *handles_out);

/* Backend::fork (qwen3_5.rs:2818-2831): a new handle for the same state. The
 * state is shared, not copied; continuing either handle leaves the other. */
int hk_fork(hk_model *m, uint64_t handle, uint64_t *out);

/* Backend::release_cache (qwen3_5.rs:2837-2846). Releasing a parent leaves its
 * forks valid. Unknown handle -> HK_ERR_BACKEND. */
int hk_release_cache(hk_model *m, uint64_t handle);

/* Tokens a handle covers and the device bytes its state occupies. */
int hk_cache_info(const hk_model *m, uint64_t handle, int *tokens, int64_t *bytes);

/*
 * The same forward with device-resident inputs and output, enqueued on
 * `stream` (a cudaStream_t; NULL = the handle's own stream) without a host
 * synchronisation. Host copies of the two offset arrays are still needed to
 * size the launches; they must equal the device copies. Device inputs are not
 * validated (hk_score validates); use it for inputs already checked.
 * No reference counterpart: it is hk_score minus the host<->device copies.
 */
int hk_score_device(hk_model *m, int n_rows, const int32_t *cu_seqlens_host,
                    const int32_t *cu_positions_host, const uint32_t *d_tokens,
                    const int32_t *d_cu_seqlens, const int32_t *d_positions,
                    float *d_out_logits, void *stream);

/*
 * Store each attention layer's keys and values in pages of `page_tokens`
 * tokens (0 = flat), placed through a per-batch block table; a nonzero
 * `shuffle_seed` permutes the pages' pool order pseudo-randomly (deterministic
 * per seed). Results equal the flat layout. Replaces
 * Qwen3_5Backend::with_kv_page_tokens (qwen3_5.rs:1773-1809; same accepted
 * values: 0 or a power of two in 16..256, else HK_ERR_ARGUMENT).
 */
int hk_set_kv_page_tokens(hk_model *m, int page_tokens, uint64_t shuffle_seed);

/* Block until the handle's queued work is done; report a device-side error flag. */
int hk_synchronize(hk_model *m);

/* Device bytes of the handle's immutable weights, and (if store_id is not
 * NULL) an identifier of the weight store: handles on the same GPU made by
 * hk_replica share one store, so they report the same identifier. No
 * reference counterpart (the reference's replicas share Arc'd weights,
 * qwen3_5.rs:2515-2535). */
uint64_t hk_weight_bytes(const hk_model *m, uint64_t *store_id);

/* Number of kernels this handle launched since creation (for launch accounting). */
uint64_t hk_kernel_launches(const hk_model *m);

/*
 * Device-time profile of the forward's launches, by class: 0 projection GEMMs,
 * 1 delta layer (fused kernel) or delta-rule recurrence, 2 attention, 3 delta
 * input stage, 4 other (conv history, SwiGLU, gated norm), 5 RMSNorm,
 * 6 attention input stage, 7 pointer readout, 8 embedding (9 classes).
 * While enabled, each launch is bracketed by CUDA events on the handle's
 * stream. hk_profile_read synchronises the stream, writes per-class summed
 * milliseconds, algorithmic FLOPs, algorithmic HBM bytes (one read of every
 * input, one write of every output) and launch counts for the first
 * n_classes classes, and clears the record. No reference counterpart (the
 * reference has no GPU profiler integration).
 */
int hk_profile_enable(hk_model *m, int enable);
int hk_profile_read(hk_model *m, double *ms, double *flops, double *bytes, int64_t *count, int n_classes);

/* The last error message on this handle (never NULL). */
const char *hk_last_error(const hk_model *m);

/* The error message of the last failed hk_create / hk_replica on this thread. */
const char *hk_create_error(void);

void hk_destroy(hk_model *m);

#ifdef __cplusplus
}
#endif

#endif /* HUNCHO_KEV_H */
