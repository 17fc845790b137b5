// Packed (GGML Q8_0 / Q4_0) projections of the reference's quantized profile
// (Projection::Packed, crates/huncho-backend/src/qwen3_5.rs:320-369; the
// artifact of crates/huncho-backend/src/qwen_quantized.rs:91-193).
//
// The reference's CPU matmul quantizes each fp32 input row to Q8_0 blocks of
// 32 (d = max|x| / 127, q = roundf(x * (1/d)), d kept as fp16) and sums per
// output, over the blocks in order, (float(sum_i q_w q_x) * d_w) * d_x in
// fp32. Here:
//   * quantize_rows_kernel: one warp per (row, block), the same Q8_0 steps;
//   * gemm_q8_kernel: int8 tensor-core products (mma.sync m16n8k32, one
//     32-wide block per instruction, a fresh int32 accumulator per block),
//     then the block's scales applied in registers with round-to-nearest
//     multiplies and adds in the reference's order, so each output equals the
//     sequential block sum exactly. Weights are stored as int8 block values
//     (Q4_0 as q - 8) [N, Kp] plus fp32 block scales [N, Kp/32].
// Tile 128 (rows) x 64 (outputs) per CTA, 8 warps of 32 x 32, a three-stage
// cp.async ring of 32-wide K blocks.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>

#include "common.cuh"
#include "gemm.cuh"

namespace hk {
namespace {

__global__ void quantize_rows_kernel(const float *x, int ldx, int M, int K, int kp, int8_t *q, float *d) {
    const int nb = kp / 32;
    const long wid = (static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (wid >= static_cast<long>(M) * nb) return;
    const int m = static_cast<int>(wid / nb), b = static_cast<int>(wid % nb);
    const int col = b * 32 + lane;
    const float v = col < K ? x[static_cast<size_t>(m) * ldx + col] : 0.0f;
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float dd = __fdiv_rn(amax, 127.0f);
    const float id = dd != 0.0f ? __fdiv_rn(1.0f, dd) : 0.0f;
    const float r = roundf(__fmul_rn(v, id));
    q[static_cast<size_t>(m) * kp + col] = static_cast<int8_t>(fminf(127.0f, fmaxf(-128.0f, r)));
    if (lane == 0) d[static_cast<size_t>(m) * nb + b] = __half2float(__float2half_rn(dd));
}

constexpr int BM = 128, BN = 64, STAGES = 3;
constexpr int LDR = 48;  // bytes per staged row (32 + 16 pad: conflict-free ldmatrix)
struct Stage {
    uint8_t a[BM * LDR];
    uint8_t b[BN * LDR];
    float ad[BM];
    float bd[BN];
};

__device__ __forceinline__ uint32_t sa(const void *p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ void cp16(void *dst, const void *src, bool ok) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sa(dst)), "l"(src), "r"(ok ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp4(void *dst, const void *src, bool ok) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(sa(dst)), "l"(src), "r"(ok ? 4 : 0) : "memory");
}
__device__ __forceinline__ void ldsm4(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(sa(p)));
}
__device__ __forceinline__ void mma_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%10, %10, %10, %10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
}

template <bool RESIDUAL>
__global__ void __launch_bounds__(256) gemm_q8_kernel(const int8_t *xq, const float *xd, const int8_t *wq,
                                                      const float *wd, int M, int N, int kp, float *out, int ldo) {
    extern __shared__ __align__(16) uint8_t smem[];
    Stage *st = reinterpret_cast<Stage *>(smem);
    const int nb = kp / 32;
    const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int wm = (warp & 3) * 32, wn = (warp >> 2) * 32;  // warp tile origin
    const int g4 = lane >> 2, t4 = lane & 3;

    auto load = [&](int blk, int s) {
        Stage &S = st[s];
        // A: 128 rows x 32 bytes = 256 x 16 B; B: 64 rows x 32 bytes = 128 x 16 B.
        {
            const int r = tid >> 1, h = tid & 1;
            const bool ok = m0 + r < M;
            cp16(&S.a[r * LDR + h * 16], xq + static_cast<size_t>(ok ? m0 + r : 0) * kp + blk * 32 + h * 16, ok);
        }
        if (tid < 128) {
            const int r = tid >> 1, h = tid & 1;
            const bool ok = n0 + r < N;
            cp16(&S.b[r * LDR + h * 16], wq + static_cast<size_t>(ok ? n0 + r : 0) * kp + blk * 32 + h * 16, ok);
        }
        if (tid < BM) {
            const bool ok = m0 + tid < M;
            cp4(&S.ad[tid], xd + static_cast<size_t>(ok ? m0 + tid : 0) * nb + blk, ok);
        } else if (tid < BM + BN) {
            const int r = tid - BM;
            const bool ok = n0 + r < N;
            cp4(&S.bd[r], wd + static_cast<size_t>(ok ? n0 + r : 0) * nb + blk, ok);
        }
    };

    float acc[2][4][4];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j][0] = acc[i][j][1] = acc[i][j][2] = acc[i][j][3] = 0.f;

#pragma unroll
    for (int s = 0; s < STAGES - 1; ++s) {
        if (s < nb) load(s, s);
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    for (int blk = 0; blk < nb; ++blk) {
        asm volatile("cp.async.wait_group %0;" ::"n"(STAGES - 2) : "memory");
        __syncthreads();
        if (blk + STAGES - 1 < nb) load(blk + STAGES - 1, (blk + STAGES - 1) % STAGES);
        asm volatile("cp.async.commit_group;" ::: "memory");
        const Stage &S = st[blk % STAGES];
        // Fragments through the 16-bit view: an int8 m16 x k32 tile is an
        // m16 x k16 tile of byte pairs (row-major A, "col" B = W rows).
        uint32_t af[2][4], bf[2][4];
        const int j = lane >> 3, i = lane & 7;
#pragma unroll
        for (int mi = 0; mi < 2; ++mi)
            ldsm4(af[mi], &S.a[(wm + mi * 16 + i + (j & 1) * 8) * LDR + (j >> 1) * 16]);
#pragma unroll
        for (int np = 0; np < 2; ++np)
            ldsm4(bf[np], &S.b[(wn + np * 16 + i + (j >> 1) * 8) * LDR + (j & 1) * 16]);
        float adv[2][2];
#pragma unroll
        for (int mi = 0; mi < 2; ++mi) {
            adv[mi][0] = S.ad[wm + mi * 16 + g4];
            adv[mi][1] = S.ad[wm + mi * 16 + g4 + 8];
        }
#pragma unroll
        for (int ni = 0; ni < 4; ++ni) {
            const float w0 = S.bd[wn + ni * 8 + 2 * t4], w1 = S.bd[wn + ni * 8 + 2 * t4 + 1];
#pragma unroll
            for (int mi = 0; mi < 2; ++mi) {
                int r[4];
                mma_s8(r, af[mi], bf[ni >> 1][(ni & 1) * 2], bf[ni >> 1][(ni & 1) * 2 + 1]);
                // sumf += (float(sumi) * d_w) * d_x, per output, in block order.
                acc[mi][ni][0] = __fadd_rn(acc[mi][ni][0], __fmul_rn(__fmul_rn(__int2float_rn(r[0]), w0), adv[mi][0]));
                acc[mi][ni][1] = __fadd_rn(acc[mi][ni][1], __fmul_rn(__fmul_rn(__int2float_rn(r[1]), w1), adv[mi][0]));
                acc[mi][ni][2] = __fadd_rn(acc[mi][ni][2], __fmul_rn(__fmul_rn(__int2float_rn(r[2]), w0), adv[mi][1]));
                acc[mi][ni][3] = __fadd_rn(acc[mi][ni][3], __fmul_rn(__fmul_rn(__int2float_rn(r[3]), w1), adv[mi][1]));
            }
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
#pragma unroll
    for (int mi = 0; mi < 2; ++mi)
#pragma unroll
        for (int ni = 0; ni < 4; ++ni)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int m = m0 + wm + mi * 16 + g4 + (e >> 1) * 8, n = n0 + wn + ni * 8 + 2 * t4 + (e & 1);
                if (m < M && n < N) {
                    float *o = out + static_cast<size_t>(m) * ldo + n;
                    *o = RESIDUAL ? __fadd_rn(*o, acc[mi][ni][e]) : acc[mi][ni][e];
                }
            }
}

}  // namespace

void launch_quantize_rows(const float *x, int ldx, int M, int K, int kp, int8_t *q, float *d, cudaStream_t s) {
    if (M <= 0) return;
    const long warps = static_cast<long>(M) * (kp / 32);
    quantize_rows_kernel<<<static_cast<unsigned>((warps + 7) / 8), 256, 0, s>>>(x, ldx, M, K, kp, q, d);
    HK_LAUNCH_CHECK();
}

void gemm_q8(const int8_t *xq, const float *xd, const int8_t *wq, const float *wd, int M, int N, int kp, float *out,
             int ldo, bool residual, cudaStream_t s) {
    if (M <= 0 || N <= 0) return;
    const int smem = static_cast<int>(sizeof(Stage) * STAGES);
    dim3 grid((M + BM - 1) / BM, (N + BN - 1) / BN);
    if (residual)
        gemm_q8_kernel<true><<<grid, 256, smem, s>>>(xq, xd, wq, wd, M, N, kp, out, ldo);
    else
        gemm_q8_kernel<false><<<grid, 256, smem, s>>>(xq, xd, wq, wd, M, N, kp, out, ldo);
    HK_LAUNCH_CHECK();
}

}  // namespace hk
