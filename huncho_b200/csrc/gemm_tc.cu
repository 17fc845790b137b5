// fp16 projection GEMM on the 5th-generation tensor cores (tcgen05), sm_100a.
//
// Y[M, N] = X[M, K] * W[N, K]^T: X is the token-major activation matrix, W a
// projection weight in its checkpoint layout ([out, in], K contiguous), so
// both operands are K-major. This is every `Linear::forward` of the backbone
// (crates/huncho-backend/src/qwen3_5.rs:306-515), with the op that follows
// each projection fused into the epilogue: the residual add of
// DecoderLayer::forward (qwen3_5.rs:1083-1104) and the SiLU(gate) * up of
// Mlp::forward (qwen3_5.rs:1020-1031).
//
// Persistent, warp-specialised CTA (one per SM):
//   warp 0      TMA producer: 128x64 X tiles and 256x64 W tiles, 128-byte
//               swizzle, into a 4-stage shared-memory ring (48 KB per stage);
//   warp 1      allocates 512 TMEM columns (two 128x256 fp32 accumulators) and
//               issues tcgen05.mma (M=128, N=256, K=16) from one thread;
//   warps 2..5  epilogue: tcgen05.ld the accumulator (each warp its 32-lane
//               quarter), apply scale / residual / SwiGLU, store to global.
// The two accumulators let the epilogue of tile i overlap the MMAs of tile i+1.
// No cluster multicast is used; every CTA loads its own tiles.
#include <cuda.h>

#include <mutex>

#include "gemm.cuh"
#include "sm100.cuh"

namespace hk {
namespace {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_STAGE_BYTES = BM * BK * 2;  // 16 KB
constexpr int B_STAGE_BYTES = BN * BK * 2;  // 32 KB
constexpr int TMEM_COLS = 2 * BN;           // double-buffered accumulator
constexpr int THREADS = 192;
constexpr int SMEM_BYTES = STAGES * (A_STAGE_BYTES + B_STAGE_BYTES) + 1024 + 256;

struct TcParams {
    int M, N, K;
    int m_tiles, n_tiles, k_blocks;
    void *out;
    int ldo;
    const float *scale;
    int vec_ok;  // out pointer / ldo allow 16-byte vector stores
    uint32_t *err;
};

__device__ __forceinline__ void store_half_32(__half *dst, const float (&v)[32], int valid, bool vec) {
    if (vec && valid >= 32) {
        uint4 pk[4];
        uint32_t *w = reinterpret_cast<uint32_t *>(pk);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            __half2 h = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
            w[i] = *reinterpret_cast<uint32_t *>(&h);
        }
        uint4 *d = reinterpret_cast<uint4 *>(dst);
#pragma unroll
        for (int i = 0; i < 4; ++i) d[i] = pk[i];
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
            if (i < valid) dst[i] = __float2half_rn(v[i]);
    }
}

template <int EPI>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_f16_tc_kernel(const __grid_constant__ CUtensorMap tm_x,
                        const __grid_constant__ CUtensorMap tm_w, TcParams p) {
    using namespace sm100;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + STAGES * A_STAGE_BYTES;
    uint64_t *full = reinterpret_cast<uint64_t *>(sB + STAGES * B_STAGE_BYTES);
    uint64_t *empty = full + STAGES;
    uint64_t *tfull = empty + STAGES;
    uint64_t *tempty = tfull + 2;
    uint64_t *drain = tempty + 2;  // MMA completion on the abort path
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int num_tiles = p.m_tiles * p.n_tiles;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 4);  // one arrival per epilogue warp
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tm_x);
        tma_prefetch_desc(&tm_w);
    }
    if (warp == 1) {
        tmem_alloc(tmem_holder, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;

    if (warp == 0) {
        if (lane == 0) {
            // ------------------------------------------------ TMA producer
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued_mask = 0, issued_parity = 0;
            for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
                const int m_blk = tile % p.m_tiles, n_blk = tile / p.m_tiles;
                for (int kb = 0; kb < p.k_blocks; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1)) {
                        set_error(p.err, kErrWaitTimeout);
                        *abort_flag = 1;
                        break;
                    }
                    mbar_expect_tx(&full[stage], A_STAGE_BYTES + B_STAGE_BYTES);
                    tma_load_2d(sA + stage * A_STAGE_BYTES, &tm_x, &full[stage], kb * BK, m_blk * BM);
                    tma_load_2d(sB + stage * B_STAGE_BYTES, &tm_w, &full[stage], kb * BK, n_blk * BN);
                    issued_mask |= 1u << stage;
                    issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            if (*abort_flag) {
                // Let every copy this thread issued land before the CTA exits.
                for (int s = 0; s < STAGES; ++s)
                    if (issued_mask & (1u << s)) (void)mbar_wait(&full[s], (issued_parity >> s) & 1);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ------------------------------------------------ MMA issuer
            constexpr uint32_t idesc = idesc_f16_f32(BM, BN);
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1)) {
                    set_error(p.err, kErrWaitTimeout);
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                for (int kb = 0; kb < p.k_blocks; ++kb) {
                    if (!mbar_wait(&full[stage], phase)) {
                        set_error(p.err, kErrWaitTimeout);
                        *abort_flag = 1;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = smem_addr(sA + stage * A_STAGE_BYTES);
                    const uint32_t b0 = smem_addr(sB + stage * B_STAGE_BYTES);
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k) {
                        mma_f16(d_tmem, desc_kmajor_sw128(a0 + k * 32), desc_kmajor_sw128(b0 + k * 32),
                                 idesc, (kb | k) != 0);
                    }
                    mma_commit(&empty[stage]);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (*abort_flag) {
                    // Let the MMAs already issued finish before TMEM is freed.
                    mma_commit(drain);
                    (void)mbar_wait(drain, 0);
                    break;
                }
                mma_commit(&tfull[acc]);
                acc ^= 1;
                if (acc == 0) acc_phase ^= 1;
            }
        }
    } else {
        // ---------------------------------------------------- epilogue
        const int quarter = warp & 3;  // TMEM lanes this warp may access
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
            if (!mbar_wait(&tfull[acc], acc_phase)) {
                set_error(p.err, kErrWaitTimeout);
                *abort_flag = 1;
                break;
            }
            if (*abort_flag) break;
            tc_fence_after();
            const int m_blk = tile % p.m_tiles, n_blk = tile / p.m_tiles;
            const int row = m_blk * BM + quarter * 32 + lane;
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN;
            const bool row_ok = row < p.M;
            if (EPI == kEpiSwiGLU) {
                // Tile columns [0,128) are gate rows, [128,256) the matching up rows.
#pragma unroll 1
                for (int c = 0; c < BN / 2; c += 32) {
                    float g[32], u[32];
                    tmem_ld32(t_row + c, g);
                    tmem_ld32(t_row + BN / 2 + c, u);
                    const int wcol = n_blk * BN + c;  // weight row of g[0]
                    if (p.scale) {
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            g[i] *= __ldg(p.scale + wcol + i);
                            u[i] *= __ldg(p.scale + wcol + BN / 2 + i);
                        }
                    }
#pragma unroll
                    for (int i = 0; i < 32; ++i) g[i] = silu_f(g[i]) * u[i];
                    const int ocol = n_blk * (BN / 2) + c;
                    if (row_ok) {
                        __half *dst = reinterpret_cast<__half *>(p.out) + static_cast<size_t>(row) * p.ldo + ocol;
                        store_half_32(dst, g, p.N / 2 - ocol, p.vec_ok);
                    }
                }
            } else {
#pragma unroll 1
                for (int c = 0; c < BN; c += 32) {
                    float v[32];
                    tmem_ld32(t_row + c, v);
                    const int col = n_blk * BN + c;
                    const int valid = p.N - col;
                    if (p.scale) {
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            if (i < valid) v[i] *= __ldg(p.scale + col + i);
                    }
                    if (!row_ok || valid <= 0) continue;
                    if (EPI == kEpiStore) {
                        __half *dst = reinterpret_cast<__half *>(p.out) + static_cast<size_t>(row) * p.ldo + col;
                        store_half_32(dst, v, valid, p.vec_ok);
                    } else {
                        float *dst = reinterpret_cast<float *>(p.out) + static_cast<size_t>(row) * p.ldo + col;
                        if (p.vec_ok && valid >= 32) {
                            float4 *d4 = reinterpret_cast<float4 *>(dst);
#pragma unroll
                            for (int i = 0; i < 8; ++i) {
                                float4 o = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
                                if (EPI == kEpiResidual) {
                                    const float4 r = d4[i];
                                    o.x += r.x;
                                    o.y += r.y;
                                    o.z += r.z;
                                    o.w += r.w;
                                }
                                d4[i] = o;
                            }
                        } else {
#pragma unroll
                            for (int i = 0; i < 32; ++i)
                                if (i < valid) dst[i] = (EPI == kEpiResidual) ? dst[i] + v[i] : v[i];
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[acc]);
            acc ^= 1;
            if (acc == 0) acc_phase ^= 1;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// ------------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault,
                                             &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    });
    if (!fn) throw CudaError("cuTensorMapEncodeTiled is unavailable");
    return fn;
}

// A 2-D fp16 tensor map over rows x inner (row stride ld elements) with a
// box of box_rows x 64 elements (128 bytes, one swizzle row) and zero fill.
CUtensorMap make_map(const void *base, int rows, int inner, int ld, int box_rows) {
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (ld * 2) % 16)
        throw CudaError("tensor-core GEMM operand must be 16-byte aligned with ld % 8 == 0");
    CUtensorMap m;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(BK), static_cast<cuuint32_t>(box_rows)};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims,
                             strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw CudaError("cuTensorMapEncodeTiled failed: " + std::to_string(r));
    return m;
}

template <int EPI>
void launch(const GemmArgs &a, cudaStream_t s, int num_sms) {
    static bool attr_set[64] = {};  // the attribute is per device
    int dev = 0;
    HK_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        HK_CUDA(cudaFuncSetAttribute(gemm_f16_tc_kernel<EPI>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    CUtensorMap tx = make_map(a.x, a.M, a.K, a.ldx, BM);
    CUtensorMap tw = make_map(a.w, a.N, a.K, a.ldw, BN);
    TcParams p;
    p.M = a.M;
    p.N = a.N;
    p.K = a.K;
    p.m_tiles = ceil_div(a.M, BM);
    p.n_tiles = ceil_div(a.N, BN);
    p.k_blocks = ceil_div(a.K, BK);
    p.out = a.out;
    p.ldo = a.ldo;
    p.scale = a.scale;
    const int elem = (EPI == kEpiStore || EPI == kEpiSwiGLU) ? 2 : 4;
    p.vec_ok = ((reinterpret_cast<uintptr_t>(a.out) & 15) == 0) && ((a.ldo * elem) % 16 == 0);
    p.err = a.err;
    const int tiles = p.m_tiles * p.n_tiles;
    const int grid = tiles < num_sms ? tiles : num_sms;
    gemm_f16_tc_kernel<EPI><<<grid, THREADS, SMEM_BYTES, s>>>(tx, tw, p);
    HK_LAUNCH_CHECK();
}

}  // namespace

void gemm_f16_tc(const GemmArgs &a, cudaStream_t s, int num_sms) {
    if (a.M <= 0 || a.N <= 0 || a.K <= 0) return;
    if (a.epilogue == kEpiSwiGLU && (a.N % BN) != 0)
        throw CudaError("fused SwiGLU GEMM needs N to be a multiple of 256");
    switch (a.epilogue) {
        case kEpiStore: launch<kEpiStore>(a, s, num_sms); break;
        case kEpiResidual: launch<kEpiResidual>(a, s, num_sms); break;
        case kEpiSwiGLU: launch<kEpiSwiGLU>(a, s, num_sms); break;
        case kEpiStoreF32: launch<kEpiStoreF32>(a, s, num_sms); break;
        default: throw CudaError("unknown GEMM epilogue");
    }
}

}  // namespace hk
