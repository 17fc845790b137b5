// Projection GEMMs: Y = X W^T with the layer's epilogue fused.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace hk {

enum GemmEpilogue : int {
    kEpiStore = 0,   // out (fp16 on tensor cores, fp32 on CUDA cores) [M, ldo] = acc * scale
    kEpiResidual = 1,  // out fp32 [M, ldo] += acc * scale  (residual stream, in place)
    kEpiSwiGLU = 2,  // weight rows interleaved in blocks of kSwiGLUBlock (gate, up);
                     // out [M, ldo] = silu(gate) * up, N/2 columns
    kEpiStoreF32 = 3,  // out fp32 [M, ldo] = acc * scale
};

// Rows of gate and up weights alternate in blocks of this size when the MLP
// uses the fused SwiGLU epilogue (half of the tensor-core tile's N).
constexpr int kSwiGLUBlock = 128;

struct GemmArgs {
    int M = 0, N = 0, K = 0;  // Y[M, N] = X[M, K] * W[N, K]^T
    const void *x = nullptr;  // activations, row-major, leading dim ldx (elements)
    int ldx = 0;
    const void *w = nullptr;  // weights [N, K] row-major, leading dim ldw
    int ldw = 0;
    const float *scale = nullptr;  // per weight row (int8 weights), or null
    void *out = nullptr;
    int ldo = 0;
    int epilogue = kEpiStore;
    uint32_t *err = nullptr;
    // Split-precision input (tensor-core path): x holds fp16(x_true) and x_lo
    // the e5m2 rounding of x_true - fp16(x_true) [M, ldx_lo bytes]; w8 is an
    // e4m3 copy of W [N, ldw8 bytes]. The accumulator then also receives
    // x_lo * w8^T (kind::f8f6f4 MMAs), which restores ~3 more bits of the
    // input: Y = W x_hi + W8 x_lo.
    const uint8_t *x_lo = nullptr;
    int ldx_lo = 0;
    const uint8_t *w8 = nullptr;
    int ldw8 = 0;
    // SwiGLU epilogue: the e5m2 residual of the fp16 output (the next
    // projection's x_lo), [M, ldo_lo bytes]; null = not written.
    uint8_t *out_lo = nullptr;
    int ldo_lo = 0;
    // 3xTF32 (fp32 model on the tensor cores): x and w are fp32; x_lo32 =
    // x - tf32(x) and w_lo32 = w - tf32(w), where tf32() keeps the sign, the
    // exponent and the top 10 mantissa bits (what kind::tf32 reads). Y = x w^T
    // + x w_lo^T + x_lo w^T, each term on kind::tf32, fp32 accumulation: the
    // dropped x_lo w_lo^T and the operands' own truncation leave ~2^-20
    // relative error. Epilogues 1 (residual) and 3 (fp32 store) only.
    bool tf32 = false;
    const float *x_lo32 = nullptr;
    int ldx_lo32 = 0;  // elements
    const float *w_lo32 = nullptr;
    int ldw_lo32 = 0;  // elements
};

// fp16 X and W on tcgen05 tensor cores (TMA-fed, TMEM accumulators), fp32 accumulation.
void gemm_f16_tc(const GemmArgs &a, cudaStream_t s, int num_sms);
// The same on CTA pairs (clusters of two CTAs sharing one cta_group::2 MMA on
// 256 x 256 tiles; half the operand loads per MMA work of gemm_f16_tc).
void gemm_f16_tc_pair(const GemmArgs &a, cudaStream_t s, int num_sms);
// fp32 X and W on CUDA cores (the fp32 model path).
void gemm_f32_simt(const GemmArgs &a, cudaStream_t s);
// lo[r, c] = x[r, c] - tf32(x[r, c]) for the 3xTF32 GEMM's input (rows of ld /
// ldl floats).
void launch_tf32_lo(const float *x, int ldx, int rows, int cols, float *lo, int ldl, cudaStream_t s);
// Host: the same split for a weight matrix.
inline float tf32_trunc_host(float v) {
    uint32_t u;
    __builtin_memcpy(&u, &v, 4);
    u &= 0xFFFFE000u;
    float r;
    __builtin_memcpy(&r, &u, 4);
    return r;
}

// Packed projections (GGML Q8_0 / Q4_0 weights as int8 block values [N, kp]
// and fp32 block scales, block-major [kp/32, N]): the fp32 input rows
// quantized to Q8_0 (q int8 [M, kp]; d fp32 block-major [kp/32, M]; columns
// >= K are zero), then out[m, n] (+)= sum over blocks in order of
// (float(int dot) * d_w) * d_x, the block dots on tcgen05 kind::i8 (xq, wq
// 16-byte aligned).
void launch_quantize_rows(const float *x, int ldx, int M, int K, int kp, int8_t *q, float *d, cudaStream_t s);
// out[b * rows + r] = in[r * nb + b]: block scales [rows, nb] to block-major.
void launch_transpose_scales(const float *in, int rows, int nb, float *out, cudaStream_t s);
void gemm_q8(const int8_t *xq, const float *xd, const int8_t *wq, const float *wd, int M, int N, int kp, float *out,
             int ldo, bool residual, cudaStream_t s, int num_sms, uint32_t *err = nullptr);

}  // namespace hk
