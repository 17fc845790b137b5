// fp32 projection GEMM on CUDA cores, for the fp32 model dtype.
//
// The reference's fp32 path multiplies in fp32 (qwen3_5.rs:306-515 via candle's
// CPU gemm); tensor-core tf32 would not meet the 1e-4 probability gate, so the
// fp32 model runs this register-tiled SIMT kernel: a 64x64 output tile per
// 256-thread CTA, 4x4 outputs per thread, K staged through shared memory in
// slices of 16. Same epilogues as the tensor-core GEMM (fp32 output).
#include "gemm.cuh"
#include "common.cuh"

namespace hk {
namespace {

constexpr int TM = 64, TN = 64, TK = 16;

template <int EPI>
__global__ void __launch_bounds__(256) gemm_f32_kernel(int M, int N, int K, const float *__restrict__ x,
                                                       int ldx, const float *__restrict__ w, int ldw,
                                                       const float *__restrict__ scale, float *out,
                                                       int ldo) {
    __shared__ float sx[TK][TM + 4];
    __shared__ float sw[TK][TN + 4];
    const int tid = threadIdx.x;
    const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TN;
    const int ty = tid / 16, tx = tid % 16;  // 16 x 16 threads, 4 x 4 outputs each
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += TK) {
        // 64 rows x 16 k for each operand: 1024 elements, 4 per thread.
        for (int i = tid; i < TM * TK; i += 256) {
            const int r = i / TK, kk = i % TK;
            const int gm = m0 + r, gk = k0 + kk;
            sx[kk][r] = (gm < M && gk < K) ? x[static_cast<size_t>(gm) * ldx + gk] : 0.0f;
            const int gn = n0 + r;
            sw[kk][r] = (gn < N && gk < K) ? w[static_cast<size_t>(gn) * ldw + gk] : 0.0f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < TK; ++kk) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = sx[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = sw[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int gm = m0 + ty * 4 + i;
        if (gm >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int gn = n0 + tx * 4 + j;
            if (gn >= N) continue;
            float v = acc[i][j];
            if (scale) v *= scale[gn];
            float *dst = out + static_cast<size_t>(gm) * ldo + gn;
            if (EPI == kEpiResidual)
                *dst += v;
            else
                *dst = v;
        }
    }
}

// lo = x - tf32(x): the low part of a 3xTF32 input (tf32 keeps the top 10
// mantissa bits; the difference is exact in fp32). float4 per thread when the
// rows allow it.
__global__ void tf32_lo_kernel(const float *__restrict__ x, int ldx, int rows, int cols, float *__restrict__ lo,
                               int ldl, int vec) {
    const size_t per_row = vec ? cols / 4 : cols;
    const size_t total = static_cast<size_t>(rows) * per_row;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t r = i / per_row, c = i % per_row;
        if (vec) {
            const float4 v = *reinterpret_cast<const float4 *>(x + r * ldx + 4 * c);
            float4 o;
            o.x = v.x - __uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u);
            o.y = v.y - __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u);
            o.z = v.z - __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u);
            o.w = v.w - __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u);
            *reinterpret_cast<float4 *>(lo + r * ldl + 4 * c) = o;
        } else {
            const float v = x[r * ldx + c];
            lo[r * ldl + c] = v - __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
        }
    }
}

}  // namespace

void launch_tf32_lo(const float *x, int ldx, int rows, int cols, float *lo, int ldl, cudaStream_t s) {
    if (rows <= 0 || cols <= 0) return;
    const int vec = (cols % 4 == 0 && ldx % 4 == 0 && ldl % 4 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(lo) & 15) == 0)
                        ? 1
                        : 0;
    const long items = static_cast<long>(rows) * (vec ? cols / 4 : cols);
    const int grid = static_cast<int>(items / 256 + 1 < 148 * 8 ? items / 256 + 1 : 148 * 8);
    tf32_lo_kernel<<<grid, 256, 0, s>>>(x, ldx, rows, cols, lo, ldl, vec);
    HK_LAUNCH_CHECK();
}

void gemm_f32_simt(const GemmArgs &a, cudaStream_t s) {
    if (a.M <= 0 || a.N <= 0 || a.K <= 0) return;
    dim3 grid(ceil_div(a.N, TN), ceil_div(a.M, TM));
    const float *x = static_cast<const float *>(a.x);
    const float *w = static_cast<const float *>(a.w);
    float *o = static_cast<float *>(a.out);
    switch (a.epilogue) {
        case kEpiStore:
        case kEpiStoreF32:
            gemm_f32_kernel<kEpiStore><<<grid, 256, 0, s>>>(a.M, a.N, a.K, x, a.ldx, w, a.ldw, a.scale, o, a.ldo);
            break;
        case kEpiResidual:
            gemm_f32_kernel<kEpiResidual><<<grid, 256, 0, s>>>(a.M, a.N, a.K, x, a.ldx, w, a.ldw, a.scale, o,
                                                               a.ldo);
            break;
        default: throw CudaError("fp32 GEMM supports the store and residual epilogues");
    }
    HK_LAUNCH_CHECK();
}

}  // namespace hk
