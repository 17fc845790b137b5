// Host launchers for the bandwidth-bound Kev layer kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace hk {

// Activation type selector for the launchers: the fp32 model runs float
// activations; the half-precision models (bf16 / fp16 / int8-weight
// checkpoints) run fp16 tensor-core operands.
enum ActType : int { kActF32 = 0, kActF16 = 1 };

// x[t, :] = table[ids[t], :] widened to fp32 (qwen3_5.rs:1319-1323, 1537).
// The table is float (act 0) or fp16 (act 1).
void launch_embed(int act, const uint32_t *ids, int n, const void *table, int hidden, float *x,
                  cudaStream_t s);

// out[r, :] = rms_norm(x[r, :]) * w_eff (qwen3_5.rs:180-190); w_eff = 1 + w, fp32.
// fp16 outputs optionally also write the e5m2 low part of each value to
// out_lo [rows, ldo_lo bytes] (the split-precision GEMM input, GemmArgs::x_lo).
void launch_rmsnorm(int act, const float *x, int ldx, const float *w_eff, float eps, int rows,
                    int hidden, void *out, int ldo, cudaStream_t s, uint8_t *out_lo = nullptr, int ldo_lo = 0);

// Gated DeltaNet input stage for every token (qwen3_5.rs:817-925): causal
// depthwise conv (K taps, restricted to the token's own row) + SiLU on the
// q|k|v channels of proj, L2 norm of q and k per key head (q also scaled by
// 1/sqrt(dk)), beta = sigmoid(b), g = -exp(A_log) * softplus(a + dt_bias).
struct DeltaPrepArgs {
    const float *proj;  // [n, ldp] fp32: qkv (conv_dim) | z (vd) | b (nv) | a (nv)
    int ldp;
    const int32_t *pos;  // position of each token inside its row
    int n;
    const float *conv_w;  // [conv_dim, taps]
    int taps;
    const float *base_g;   // -exp(A_log) [nv]
    const float *dt_bias;  // [nv]
    int nk, nv, dk, dv;
    float *q, *k;  // [n, nk, dk] fp32
    float *v;      // [n, nv, dv] fp32
    float *g, *beta;  // [n, nv] fp32
    // Continued rows (a fork of a cached prefix): hist_in[row] is the device
    // address of the row's conv history [taps-1][conv_dim] fp32 (the prefix's
    // last pre-conv inputs, oldest first), or 0 for none (zero history).
    const int32_t *tok_row = nullptr;
    const uint64_t *hist_in = nullptr;
    // Half-precision models: fused multiply-adds in the conv, intrinsic SiLU
    // and rsqrt (their q, k, v are split into fp16 operands right after); the
    // fp32 model keeps the reference's exact operation order.
    int fast = 0;
};
void launch_delta_prep(const DeltaPrepArgs &a, cudaStream_t s);

// Conv history of each row for its output snapshot: the last taps-1 pre-conv
// inputs of [hist_in rows ; the row's own qkv projection rows] written to
// hist_out[row] (rows with hist_out 0 are skipped).
void launch_conv_history(const float *proj, int ldp, int conv_dim, int taps, const int32_t *cu_seqlens, int n_rows,
                         const uint64_t *hist_in, const uint64_t *hist_out, cudaStream_t s);

// Per-token gated delta rule with an fp32 state per (row, value head)
// (qwen3_5.rs:950-987). `exact` keeps the reference's ascending-key fp32
// operation order with no fused multiply-adds (delta_cpu.rs:99-136).
struct DeltaRecArgs {
    const float *q, *k, *v, *g, *beta;
    const int32_t *cu_seqlens;
    const int32_t *row_order = nullptr;  // CTA i processes row row_order[i] (longest first), or i
    int n_rows, nk, nv, dk, dv;
    float *out;  // [n, nv, dv]
    int exact;
    uint32_t *err = nullptr;  // device error word (bounded waits)
    // Per-row device addresses of the initial state and of where to write the
    // final state, both [nv][dk][dv] fp32 (S[h][i][j], i the key index); 0 (or
    // a null array) means a zero initial state / no write.
    const uint64_t *state_in = nullptr, *state_out = nullptr;
};
void launch_delta_recurrent(const DeltaRecArgs &a, cudaStream_t s);
// The chunked tcgen05 form behind launch_delta_recurrent (non-exact mode,
// 128-wide heads), and its variant with the gated RMSNorm fused into the
// output (z from the fp32 projection rows at column zoff + h*128).
bool delta_tc_supported(const DeltaRecArgs &r);
void launch_delta_tc(const DeltaRecArgs &r, cudaStream_t s);
void launch_delta_tc_gated(const DeltaRecArgs &r, const float *proj, int ldp, int zoff, const float *norm_w, float eps,
                           __half *mix, int ldmix, cudaStream_t s);
// The chunked mma.sync form (32-token chunks, 128-wide heads).
bool delta_chunk_supported(const DeltaRecArgs &a);
void launch_delta_chunk(const DeltaRecArgs &a, cudaStream_t s);
// The chunked mma.sync recurrence with the gated RMSNorm fused into its output
// (z read from the fp32 projection rows at column zoff + h*128); q, k, v, g,
// beta pre-computed.
void launch_delta_chunk_gated(const DeltaRecArgs &r, const float *proj, int ldp, int zoff, const float *norm_w,
                              float eps, __half *mix, int ldmix, cudaStream_t s);
// The delta layer's input stage inputs for the fused kernel below: the fp32
// in-projection rows (ldp per row: qkv | z | b | a), conv weights, gates'
// parameters and each row's prefix conv history (as in DeltaPrepArgs).
struct DeltaFusedInput {
    const float *proj = nullptr;
    int ldp = 0, conv_dim = 0;
    const float *conv_w = nullptr, *base_g = nullptr, *dt_bias = nullptr;
    const uint64_t *hist_in = nullptr;
};
// The warp-specialised form of the fused delta layer (4 warps prepare chunk
// j+1's state-independent operands while 8 warps run chunk j's state-dependent
// products); 128-wide heads, 4 taps.
bool delta_pipe_supported(const DeltaRecArgs &r, const DeltaFusedInput &in);
// mix_lo (optional): the e5m2 low part of the output [n, ldmix_lo bytes].
void launch_delta_pipe(const DeltaRecArgs &r, const DeltaFusedInput &in, const float *norm_w, float eps, __half *mix,
                       int ldmix, cudaStream_t s, uint8_t *mix_lo = nullptr, int ldmix_lo = 0);

// out[t, h*dv + j] = rms(o)[j] * w[j] * silu(z[t, h, j]) (qwen3_5.rs:193-201,
// 934-938); o and z fp32, out in the activation type (the out_proj input).
void launch_gated_norm(int act, const float *o, const float *z, int ldz, const float *w, float eps,
                       int n, int nv, int dv, void *out, int ldo, cudaStream_t s, uint8_t *out_lo = nullptr,
                       int ldo_lo = 0);

// Full-attention input stage (qwen3_5.rs:596-615): split q | gate per head,
// q_norm / k_norm (zero-centred weights, fp32), partial RoPE on the first
// rotary_dim dims at each token's in-row position.
// Where a row's keys and values live. Flat (page_tokens == 0): key j of the row
// starting at token `start` is slot start + j. Paged: slot
// block_table[cu_pages[row] + j / page_tokens] * page_tokens + j % page_tokens,
// i.e. fixed-size pages in any order (the reference's PagedKv page list,
// kv_pages.rs:19-40, as a device block table).
struct KvPages {
    const int32_t *block_table = nullptr;
    const int32_t *cu_pages = nullptr;  // [n_rows + 1] offsets into block_table
    int page_tokens = 0;
};

__device__ __forceinline__ int kv_slot(const KvPages &p, int row, int start, int j) {
    if (p.page_tokens == 0) return start + j;
    return p.block_table[p.cu_pages[row] + j / p.page_tokens] * p.page_tokens + j % p.page_tokens;
}

struct AttnPrepArgs {
    const float *proj;  // [n, ldp] fp32: per q head [q(hd) | gate(hd)], then k (nkv*hd), v (nkv*hd)
    int ldp;
    const int32_t *pos;
    const int32_t *tok_row;  // row of each token (paged K/V)
    int n, nh, nkv, hd, rd;
    const float *qn_w, *kn_w;  // effective norm weights [hd]
    const float *inv_freq;     // [rd/2]
    float eps;
    void *q, *k, *v;  // q [n, nh, hd]; k, v [slots, nkv, hd] at kv_slot()
    KvPages pages;
    const int32_t *pre_len = nullptr;  // per row: cached prefix tokens (RoPE offset), or null
};
void launch_attn_prep(int act, const AttnPrepArgs &a, cudaStream_t s);

// Causal softmax(q k^T / sqrt(hd)) v per row with GQA (qwen3_5.rs:669-714),
// multiplied by sigmoid(gate) and written token-major [n, nh*hd].
struct AttnArgs {
    const void *q, *k, *v;  // q [n, nh, hd]; k, v [slots, nkv, hd] at kv_slot()
    const float *proj;      // gate source (fp32): proj[t, h*2*hd + hd + i]
    int ldp;
    const int32_t *cu_seqlens;
    const int32_t *tok_row;  // row of each token
    int n, n_rows, max_len, nh, nkv, hd;
    void *out;
    int ldo;
    KvPages pages;
    // Continued rows: the row's first pre_len[row] keys come from its cached
    // prefix at kv_in[row] (K [P][nkv][hd] then V [P][nkv][hd], activation
    // type); its own tokens follow at absolute positions P, P+1, ...
    const int32_t *pre_len = nullptr;
    const uint64_t *kv_in = nullptr;
    uint32_t *err = nullptr;  // device error word (bounded waits of the tcgen05 kernel)
    // K / V slots the k and v buffers hold (flat: n; paged: the page pool);
    // 0 = unknown (the tcgen05 kernel then stages K / V with cp.async instead
    // of TMA).
    int kv_slots = 0;
};
void launch_attention(int act, const AttnArgs &a, cudaStream_t s);
// The tcgen05 kernel behind launch_attention for fp16 activations and
// head_dim 128 / 256 (TMEM accumulators, 128-query tiles).
bool attention_t5_supported(const AttnArgs &a);
void launch_attention_t5(const AttnArgs &a, cudaStream_t s);
// Output snapshot K/V of each row with kv_out[row] != 0: the cached prefix
// keys (from kv_in) then the row's own keys (from the workspace slots), as
// K [P+L][nkv][hd] then V [P+L][nkv][hd].
void launch_kv_store(int act, const AttnArgs &a, const uint64_t *kv_out, cudaStream_t s);
// The tensor-core (fp16) kernel behind launch_attention for head_dim 64/128/256.
bool attention_tc_supported(int hd);
void launch_attention_tc(const AttnArgs &a, cudaStream_t s);

// out[i] = (fp16) q[i] for i < n: int8 weights expanded to fp16 (exact for
// |q| <= 127) right before the projection that uses them; out8 (optional)
// receives the e4m3 rounding of the same values (split-precision low part).
void launch_expand_i8(const int8_t *q, size_t n, __half *out, uint8_t *out8, cudaStream_t s);

// out[t, j] = silu(gu[t, j]) * gu[t, F + j] (qwen3_5.rs:1020-1031); gu fp32.
void launch_swiglu(int act, const float *gu, int ldg, int n, int f, void *out, int ldo, cudaStream_t s,
                   uint8_t *out_lo = nullptr, int ldo_lo = 0);

// Pointer readout (qwen3_5.rs:3196-3255, kev.rs:169-173). idx lists the token
// rows to read: first the n_dec decision rows, then the n_opt option rows.
struct ReadoutArgs {
    const float *x;  // residual stream [n, hidden] (before the final norm)
    int hidden;
    const float *final_w;  // effective final norm weight
    float eps;
    const int32_t *idx;   // [n_dec + n_opt] token indices
    const int32_t *opt_dec;  // [n_opt] decision row of each option
    int n_dec, n_opt;
    const float *wq, *bq, *wk, *bk;  // [dp, hidden], [dp]
    int dp;
    float scale;  // 1 / sqrt(dp), rounded from double as the reference does
    float *hn;    // scratch [n_dec + n_opt, hidden]
    float *proj;  // scratch [n_dec + n_opt, dp]
    float *logits;  // [n_opt]
};
void launch_readout(const ReadoutArgs &a, cudaStream_t s);
// Argument checks shared by the readout entry points (std::invalid_argument on failure).
void check_readout_args(const float *x, int hidden, const float *final_w, const int32_t *idx, const int32_t *opt_dec,
                        int n_dec, int n_opt, const float *wq, const float *bq, const float *wk, const float *bk,
                        int dp, const float *logits);

// Calibrated probabilities and typed answers of every question of a batch
// (answers.cu). Layout of AnswerRec equals the C ABI's hk_answer.
enum : int { kQuestionChoice = 0, kQuestionNoul = 1, kQuestionScore = 2 };
enum : int { kAnswerNonfiniteLogits = 1, kAnswerNonfiniteProbs = 2 };
struct AnswerRec {
    int32_t best, status;
    float confidence, value;
};
struct AnswerArgs {
    const float *logits;          // [cu_positions[n_rows]] raw pointer logits
    const int32_t *cu_positions;  // [n_rows + 1]
    const int32_t *qtype;         // [n_rows] kQuestion*
    int n_rows;
    float temperature;
    float *probs;     // [cu_positions[n_rows]]
    AnswerRec *out;   // [n_rows]
};
void launch_answers(const AnswerArgs &a, cudaStream_t s);

}  // namespace hk
