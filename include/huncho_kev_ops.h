/*
 * huncho_kev_ops.h -- kernel-level entry points of libhuncho_kev.so.
 *
 * Single kernels of the Kev forward over caller-owned DEVICE pointers,
 * enqueued on `stream` (a cudaStream_t; NULL = legacy default stream). They
 * exist so each kernel can be checked and timed in isolation; the model-level
 * API is include/huncho_kev.h. Return HK_OK or a negative HK_ERR_* code;
 * hk_op_last_error() holds the message of the calling thread's last failure.
 */
#ifndef HUNCHO_KEV_OPS_H
#define HUNCHO_KEV_OPS_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Y[M, N] (epilogue) X[M, K] W[N, K]^T. `dtype` 0: fp32 X/W (CUDA cores),
 * 1: fp16 X/W (tcgen05 tensor cores, fp32 accumulation; single CTAs or CTA
 * pairs chosen by shape, as the model runs it), 2: fp16 X/W always on CTA
 * pairs (clusters of two CTAs sharing one cta_group::2 MMA on 256 x 256
 * tiles; the same results as 1), 3: fp32 X/W on the tensor cores as three
 * tf32 products (x w + x w_lo + x_lo w with v_lo = v - tf32(v); ~2^-20
 * relative error; epilogues 1 and 3; the low parts live in stream-ordered
 * scratch for the call). `epilogue` 0: store
 * (fp16 for dtype 1), 1: fp32 residual add into out, 2: SwiGLU over 128-row
 * gate/up blocks (fp16), 3: store fp32. `scale` (nullable) multiplies output column n by scale[n].
 * Replaces one Linear::forward of the backbone (qwen3_5.rs:306-515). */
int hk_op_gemm(int dtype, int epilogue, int M, int N, int K, const void *x, int ldx, const void *w,
               int ldw, const float *scale, void *out, int ldo, void *stream);

/* The split-precision form of hk_op_gemm's fp16 tensor-core GEMM (dtype 1),
 * the one the half-precision models run for the delta layers' and the MLPs'
 * projections: x fp16 [M, ldx] is the high part of the input and x_lo
 * [M, ldx_lo bytes] its e5m2 low part (x_true - fp16(x_true)); w fp16 [N, ldw]
 * and w8 [N, ldw8 bytes] an e4m3 copy of it. out (epilogue) = x w^T + x_lo w8^T
 * with fp32 accumulation (kind::f16 then kind::f8f6f4 tcgen05 MMAs into one
 * accumulator). SwiGLU (epilogue 2) also writes the e5m2 low part of its fp16
 * output to out_lo [M, ldo_lo bytes] when out_lo is not NULL. Byte strides
 * are multiples of 16. pairs = 1 forces CTA pairs (cta_group::2); 0 lets the
 * shape choose, as the model does. No reference counterpart (the reference's
 * CUDA path runs plain fp16 projections). */
int hk_op_gemm_split(int epilogue, int M, int N, int K, const void *x, int ldx, const uint8_t *x_lo, int ldx_lo,
                     const void *w, int ldw, const uint8_t *w8, int ldw8, const float *scale, void *out, int ldo,
                     uint8_t *out_lo, int ldo_lo, int pairs, void *stream);

/* A packed projection (the reference's Projection::Packed, qwen3_5.rs:320-369):
 * x fp32 [M, K] (leading dim ldx) quantized to Q8_0 blocks of 32 (columns >= K
 * zero; x_q int8 [M, kp] and x_d (M * kp/32 floats, written block-major) are
 * caller-provided scratch, x_q 16-byte aligned), then out fp32 [M, ldo] (+=
 * when residual) = per output, over the blocks in order, sum of
 * (float(int dot) * w_d) * x_d, with w_q int8 [N, kp] block values (Q4_0 as
 * q - 8; 16-byte aligned) and w_d fp32 [N, kp/32] block scales, fp16 values as
 * GGML stores them (the kernel's exact rounding rests on it). The block dots
 * run on tcgen05 kind::i8; w_d is transposed into stream-ordered scratch for
 * the call. kp % 32 == 0, K <= kp. Device pointers. */
int hk_op_gemm_packed(int M, int N, int K, int kp, const float *x, int ldx, const int8_t *w_q, const float *w_d,
                      int8_t *x_q, float *x_d, float *out, int ldo, int residual, void *stream);

/* Per-token gated delta rule (qwen3_5.rs:950-987) over packed rows:
 * q, k [n, nk, dk]; v [n, nv, dv]; g, beta [n, nv]; out [n, nv, dv]; fp32.
 * `exact` = 1 keeps the reference's operation order (delta_cpu.rs:99-136). */
int hk_op_delta_recurrent(const float *q, const float *k, const float *v, const float *g,
                          const float *beta, const int32_t *cu_seqlens, int n_rows, int nk, int nv,
                          int dk, int dv, int exact, float *out, void *stream);

/* The chunked forms of the same rule for 128-wide heads (the WY form of the
 * chunk-reassociated recurrence, fp16 tensor-core operands with hi/lo splits
 * on the sensitive ones, fp32 state): `kernel` 0 = mma.sync, 32-token chunks;
 * 1 = tcgen05 with the state in tensor memory, 64-token chunks. With z == NULL
 * the output is o [n, nv, 128] fp32; otherwise it is the gated RMSNorm
 * rms(o) * norm_w * silu(z) (qwen3_5.rs:193-201) in fp16 at out[t * ldo +
 * h*128 + j], with z[t * ldz + h*128 + j] fp32 (the delta layer's out_proj
 * input). No reference counterpart (the reference runs the per-token rule). */
int hk_op_delta_chunked(int kernel, const float *q, const float *k, const float *v, const float *g,
                        const float *beta, const int32_t *cu_seqlens, int n_rows, int nk, int nv, const float *z,
                        int ldz, const float *norm_w, float eps, void *out, int ldo, void *stream);

/* The whole delta layer between its in-projection and its out-projection, as
 * the half-precision models run it (one warp-specialised kernel): from the
 * fp32 projection rows proj [n, ldp] = q (nk*128) | k (nk*128) | v (nv*128) |
 * z (nv*128) | b (nv) | a (nv), the causal depthwise conv over 4 taps + SiLU
 * (conv_w [conv_dim][4], conv_dim = 2*nk*128 + nv*128), l2norm of q (times
 * 1/sqrt(128)) and k, beta = sigmoid(b), g = base_g * softplus(a + dt_bias)
 * (base_g = -exp(A_log)), the chunked gated delta rule with a zero initial
 * state per row, and the gated RMSNorm rms(o) * norm_w * silu(z), written in
 * fp16 to out [n, ldo] (the out-projection input). Replaces
 * LinearAttn::forward between in_proj and out_proj (qwen3_5.rs:846-938) with
 * recurrent_gated_delta (qwen3_5.rs:950-987). ldp % 4 == 0. */
int hk_op_delta_layer(const float *proj, int ldp, const int32_t *cu_seqlens, int n_rows, int nk, int nv,
                      const float *conv_w, const float *base_g, const float *dt_bias, const float *norm_w, float eps,
                      void *out, int ldo, void *stream);

/* Causal GQA attention with the sigmoid output gate (qwen3_5.rs:669-714).
 * act 0: fp32, 1: fp16. q [n, nh, hd]; k, v [n, nkv, hd] (act type); gate read
 * from the fp32 proj[t, h*2*hd + hd + i] (row stride ldp); out [n, ldo] (act
 * type). tok_row[n] gives
 * each token's row. */
int hk_op_attention(int act, const void *q, const void *k, const void *v, const float *proj, int ldp,
                    const int32_t *cu_seqlens, const int32_t *tok_row, int n, int n_rows, int max_len,
                    int nh, int nkv, int hd, void *out, int ldo, void *stream);

/* Pointer-head readout (qwen3_5.rs:3196-3255, kev.rs:169-173) over device
 * buffers: rows idx[0..n_dec) are decision tokens and idx[n_dec..n_dec+n_opt)
 * option tokens of the fp32 residual stream x [*, hidden] (before the final
 * norm); each row is RMS-normalised with final_w (effective weight), decision
 * rows projected by wq/bq and option rows by wk/bk ([dp, hidden], [dp], fp32),
 * and logits[j] = k_j . q_{opt_dec[j]} / sqrt(dp). Scratch (caller-owned):
 * hn [n_dec + n_opt, hidden] and proj [n_dec + n_opt, dp], fp32. Index
 * contract: every idx entry is a row of x (not checked: the kernels do not
 * know x's row count); an opt_dec entry outside [0, n_dec) gives that option
 * a NaN logit without reading another row. Null pointers, negative counts,
 * or options without a decision row: HK_ERR_ARGUMENT. */
int hk_op_readout(const float *x, int hidden, const float *final_w, float eps, const int32_t *idx,
                  const int32_t *opt_dec, int n_dec, int n_opt, const float *wq, const float *bq,
                  const float *wk, const float *bk, int dp, float *hn, float *proj, float *logits,
                  void *stream);

/* hk_op_readout without scratch arguments and without allocating: for callers
 * that cannot call cudaMalloc (a host that hands this library only device
 * memory planned ahead from its own pool, or a latency-critical serving loop
 * where cudaMalloc's implicit device synchronisation would stall other GPU
 * work). Its scratch is a library-owned 16 MiB __device__ array that every GPU
 * loading the library holds until exit; limits: n_dec + n_opt <= 1024,
 * hidden <= 3584, dp <= 512 (beyond them: HK_ERR_ARGUMENT, message in
 * hk_op_last_error). The first call on each device looks up the array's
 * device address (call it before any stream capture). All calls share the
 * array, so calls that overlap on the GPU race. No counterpart in the
 * reference (its readout is a CPU/candle tensor expression). */
int hk_op_readout_noalloc(const float *x, int hidden, const float *final_w, float eps,
                          const int32_t *idx, const int32_t *opt_dec, int n_dec, int n_opt,
                          const float *wq, const float *bq, const float *wk, const float *bk,
                          int dp, float *logits, void *stream);

/* Calibration and typed answers of already-scored questions (the device half
 * of hk_score_answers) over device buffers: logits [cu_positions[n_rows]]
 * fp32, cu_positions [n_rows + 1], question_types [n_rows] (HK_QUESTION_*);
 * writes probs [cu_positions[n_rows]] and answers [n_rows] (hk_answer
 * layout: best, status, confidence, value). Follows calibration.rs:36-64,
 * 87-147 and engine.rs:1448-1513. */
int hk_op_answers(const float *logits, const int32_t *cu_positions, const int32_t *question_types, int n_rows,
                  float temperature, float *probs, void *answers, void *stream);

/* Number of SMs the GEMM grid is sized for on the current device. */
int hk_op_num_sms(void);

const char *hk_op_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* HUNCHO_KEV_OPS_H */
