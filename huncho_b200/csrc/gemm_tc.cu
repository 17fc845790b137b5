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
//               quarter), apply scale / SwiGLU, stage 32-row x 128-byte slabs
//               in 128B-swizzled shared memory (two buffers per warp) and write
//               them with TMA bulk-tensor stores -- or TMA reduce-add into the
//               fp32 residual stream -- so global writes are full lines.
// The two accumulators let the epilogue of tile i overlap the MMAs of tile i+1.
// No cluster multicast is used; every CTA loads its own tiles. A CTA-pair form
// of the same kernel (cta_group::2, 256 x 256 tiles; see gemm_f16_tc2_kernel)
// runs the launches whose MMAs wait on operand loads.
#include <cuda.h>

#include <cstring>
#include <mutex>

#include "gemm.cuh"
#include "sm100.cuh"

namespace hk {
namespace {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
enum : int { kPassF16 = 0, kPassF8 = 1, kPassTF32 = 2 };
constexpr int A_STAGE_BYTES = BM * BK * 2;  // 16 KB
constexpr int B_STAGE_BYTES = BN * BK * 2;  // 32 KB
constexpr int TMEM_COLS = 2 * BN;           // double-buffered accumulator
constexpr int THREADS = 192;
constexpr int EPI_BUF_BYTES = 32 * 128;  // one warp's 32-row x 128-byte staging slab
constexpr int EPI_BYTES = 4 * 2 * EPI_BUF_BYTES;
constexpr int SMEM_BYTES = STAGES * (A_STAGE_BYTES + B_STAGE_BYTES) + EPI_BYTES + 1024 + 256;

struct TcParams {
    int M, N, K;
    int m_tiles, n_tiles, k_blocks;
    // The K loop of a tile as up to three passes over 128-byte stage rows, each
    // with its operand maps (0: tm_x / tm_w, 1: tm_xl / tm_wl), its K elements
    // per block (64 fp16, 128 8-bit, 32 tf32) and its MMA kind (kPass*).
    int n_pass;
    int pass_kb[3], pass_kw[3], pass_a[3], pass_b[3], pass_kind[3];
    int total_kb;
    uint8_t *out_lo;  // SwiGLU: e5m2 residual of the fp16 output, or null
    int ldo_lo;
    int n_fast;  // tile order: N fastest (narrow N: the N tiles of one M tile run together, X read once)
    void *out;
    int ldo;
    const float *scale;
    int vec_ok;  // out pointer / ldo allow 16-byte vector stores
    int tma_out; // the output goes through the TMA store tensor map
    uint32_t *err;
};

// Write one thread's 128-byte row (8 chunks of 16 bytes) into a 128B-swizzled
// staging slab: chunk c of row r lands in physical chunk c ^ (r & 7).
__device__ __forceinline__ void stage_row(uint8_t *slab, int r, const uint4 (&chunks)[8]) {
#pragma unroll
    for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4 *>(slab + r * 128 + ((c ^ (r & 7)) << 4)) = chunks[c];
}

template <int EPI>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_f16_tc_kernel(const __grid_constant__ CUtensorMap tm_x,
                        const __grid_constant__ CUtensorMap tm_w,
                        const __grid_constant__ CUtensorMap tm_o,
                        const __grid_constant__ CUtensorMap tm_xl,
                        const __grid_constant__ CUtensorMap tm_wl, TcParams p) {
    using namespace sm100;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + STAGES * A_STAGE_BYTES;
    uint8_t *sE = sB + STAGES * B_STAGE_BYTES;  // epilogue staging, 1024-aligned
    uint64_t *full = reinterpret_cast<uint64_t *>(sE + EPI_BYTES);
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
                const int m_blk = p.n_fast ? tile / p.n_tiles : tile % p.m_tiles;
                const int n_blk = p.n_fast ? tile % p.n_tiles : tile / p.m_tiles;
                for (int kb = 0, ps = 0, lk = 0; kb < p.total_kb; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1)) {
                        set_error(p.err, kErrWaitTimeout);
                        *abort_flag = 1;
                        break;
                    }
                    // Every pass's block is 128 bytes per row (the same stage geometry).
                    mbar_expect_tx(&full[stage], A_STAGE_BYTES + B_STAGE_BYTES);
                    const int kx = lk * p.pass_kw[ps];
                    tma_load_2d(sA + stage * A_STAGE_BYTES, p.pass_a[ps] ? &tm_xl : &tm_x, &full[stage], kx,
                                m_blk * BM);
                    tma_load_2d(sB + stage * B_STAGE_BYTES, p.pass_b[ps] ? &tm_wl : &tm_w, &full[stage], kx,
                                n_blk * BN);
                    if (++lk == p.pass_kb[ps]) {
                        lk = 0;
                        ++ps;
                    }
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
            constexpr uint32_t idesc8 = idesc_e5m2_e4m3_f32(BM, BN);
            constexpr uint32_t idesc32 = idesc_tf32_f32(BM, BN);
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
                for (int kb = 0, ps = 0, lk = 0; kb < p.total_kb; ++kb) {
                    if (!mbar_wait(&full[stage], phase)) {
                        set_error(p.err, kErrWaitTimeout);
                        *abort_flag = 1;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = smem_addr(sA + stage * A_STAGE_BYTES);
                    const uint32_t b0 = smem_addr(sB + stage * B_STAGE_BYTES);
                    // Four MMAs per 128-byte row: K = 16 fp16, 32 8-bit or 8 tf32 each.
                    const int kind = p.pass_kind[ps];
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const uint64_t ad = desc_kmajor_sw128(a0 + k * 32), bd = desc_kmajor_sw128(b0 + k * 32);
                        const uint32_t acc = (kb | k) != 0;
                        if (kind == kPassF16)
                            mma_f16(d_tmem, ad, bd, idesc, acc);
                        else if (kind == kPassF8)
                            mma_f8(d_tmem, ad, bd, idesc8, acc);
                        else
                            mma_tf32(d_tmem, ad, bd, idesc32, acc);
                    }
                    if (++lk == p.pass_kb[ps]) {
                        lk = 0;
                        ++ps;
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
        uint8_t *const slab0 = sE + (warp - 2) * 2 * EPI_BUF_BYTES;
        int sb = 0;  // staging buffer to fill next
        auto slab = [&]() { return slab0 + sb * EPI_BUF_BYTES; };
        int acc = 0;
        uint32_t acc_phase = 0;
        // Hand a filled slab to the TMA unit (lane 0), keeping at most one older
        // store in flight on the other buffer.
        auto issue = [&](int x, int y) {
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
                if (EPI == kEpiResidual)
                    tma_reduce_add_2d(&tm_o, slab(), x, y);
                else
                    tma_store_2d(&tm_o, slab(), x, y);
                bulk_commit();
            }
            sb ^= 1;
        };
        auto reuse_wait = [&]() {
            if (lane == 0) bulk_wait_read<1>();
            __syncwarp();
        };
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
            if (!mbar_wait(&tfull[acc], acc_phase)) {
                set_error(p.err, kErrWaitTimeout);
                *abort_flag = 1;
                break;
            }
            if (*abort_flag) break;
            tc_fence_after();
            const int m_blk = p.n_fast ? tile / p.n_tiles : tile % p.m_tiles;
            const int n_blk = p.n_fast ? tile % p.n_tiles : tile / p.m_tiles;
            const int row0 = m_blk * BM + quarter * 32;
            const int row = row0 + lane;
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN;
            const bool row_ok = row < p.M;
            const bool slab_ok = row0 < p.M;
            if (EPI == kEpiSwiGLU) {
                // Tile columns [0,128) are gate rows, [128,256) the matching up rows;
                // each round produces 64 fp16 outputs per row.
#pragma unroll 1
                for (int c = 0; c < BN / 2; c += 64) {
                    uint32_t packed[32];
#pragma unroll
                    for (int hh = 0; hh < 2; ++hh) {
                        float g[32], u[32];
                        tmem_ld32(t_row + c + 32 * hh, g);
                        tmem_ld32(t_row + BN / 2 + c + 32 * hh, u);
                        const int wcol = n_blk * BN + c + 32 * hh;  // weight row of g[0]
                        if (p.scale) {
#pragma unroll
                            for (int i = 0; i < 32; ++i) {
                                g[i] *= __ldg(p.scale + wcol + i);
                                u[i] *= __ldg(p.scale + wcol + BN / 2 + i);
                            }
                        }
                        uint32_t lo[8];
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            const float y0 = silu_fast(g[2 * i]) * u[2 * i], y1 = silu_fast(g[2 * i + 1]) * u[2 * i + 1];
                            __half2 h2 = __floats2half2_rn(y0, y1);
                            packed[16 * hh + i] = *reinterpret_cast<uint32_t *>(&h2);
                            const uint32_t l2 = static_cast<uint32_t>(lo_e5m2(y0, __low2half(h2))) |
                                                (static_cast<uint32_t>(lo_e5m2(y1, __high2half(h2))) << 8);
                            if (i & 1)
                                lo[i >> 1] |= l2 << 16;
                            else
                                lo[i >> 1] = l2;
                        }
                        if (p.out_lo && row_ok) {
                            // The next projection's low part: 32 bytes of e5m2 per row and half round.
                            uint4 *dl = reinterpret_cast<uint4 *>(p.out_lo + static_cast<size_t>(row) * p.ldo_lo +
                                                                  n_blk * (BN / 2) + c + 32 * hh);
                            dl[0] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                            dl[1] = make_uint4(lo[4], lo[5], lo[6], lo[7]);
                        }
                    }
                    const int ocol = n_blk * (BN / 2) + c;
                    if (p.tma_out) {
                        if (!slab_ok || ocol >= p.N / 2) continue;
                        reuse_wait();
                        uint4 ch[8];
#pragma unroll
                        for (int i = 0; i < 8; ++i) ch[i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2], packed[4 * i + 3]);
                        stage_row(slab(), lane, ch);
                        issue(ocol, row0);
                    } else if (row_ok) {
                        __half *dst = reinterpret_cast<__half *>(p.out) + static_cast<size_t>(row) * p.ldo + ocol;
                        const __half *hv = reinterpret_cast<const __half *>(packed);
                        for (int i = 0; i < 64 && ocol + i < p.N / 2; ++i) dst[i] = hv[i];
                    }
                }
            } else if (EPI == kEpiStore) {
#pragma unroll 1
                for (int c = 0; c < BN; c += 64) {
                    const int col = n_blk * BN + c;
                    uint32_t packed[32];
#pragma unroll
                    for (int hh = 0; hh < 2; ++hh) {
                        float v[32];
                        tmem_ld32(t_row + c + 32 * hh, v);
                        if (p.scale) {
#pragma unroll
                            for (int i = 0; i < 32; ++i)
                                if (col + 32 * hh + i < p.N) v[i] *= __ldg(p.scale + col + 32 * hh + i);
                        }
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            __half2 h2 = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
                            packed[16 * hh + i] = *reinterpret_cast<uint32_t *>(&h2);
                        }
                    }
                    if (p.tma_out) {
                        if (!slab_ok || col >= p.N) continue;
                        reuse_wait();
                        uint4 ch[8];
#pragma unroll
                        for (int i = 0; i < 8; ++i) ch[i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2], packed[4 * i + 3]);
                        stage_row(slab(), lane, ch);
                        issue(col, row0);
                    } else if (row_ok) {
                        __half *dst = reinterpret_cast<__half *>(p.out) + static_cast<size_t>(row) * p.ldo + col;
                        const __half *hv = reinterpret_cast<const __half *>(packed);
                        for (int i = 0; i < 64 && col + i < p.N; ++i) dst[i] = hv[i];
                    }
                }
            } else {
                // fp32 outputs: store, or add into the residual stream.
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
                    if (p.tma_out) {
                        if (!slab_ok || valid <= 0) continue;
                        reuse_wait();
                        uint4 ch[8];
#pragma unroll
                        for (int i = 0; i < 8; ++i)
                            ch[i] = make_uint4(__float_as_uint(v[4 * i]), __float_as_uint(v[4 * i + 1]),
                                               __float_as_uint(v[4 * i + 2]), __float_as_uint(v[4 * i + 3]));
                        stage_row(slab(), lane, ch);
                        issue(col, row0);
                    } else if (row_ok && valid > 0) {
                        float *dst = reinterpret_cast<float *>(p.out) + static_cast<size_t>(row) * p.ldo + col;
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            if (i < valid) dst[i] = (EPI == kEpiResidual) ? dst[i] + v[i] : v[i];
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[acc]);
            acc ^= 1;
            if (acc == 0) acc_phase ^= 1;
        }
        if (lane == 0) bulk_wait_all();
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}


// The same GEMM on CTA pairs (cta_group::2): a cluster of two CTAs computes a
// 256 x 256 tile with one MMA stream issued by the first CTA. Each CTA loads
// 128 rows of X and 128 rows of W (its half of the tile's N) per 64-wide K
// block, so every shared-memory byte feeds twice the MMA work of the single-CTA
// kernel and six 32 KB stages fit. Both CTAs' loads complete on the first
// CTA's `full` barrier; the first CTA's commits arrive on both CTAs' `empty`
// and `tfull` barriers; the epilogue warps of both CTAs release an
// accumulator on the first CTA's `tempty`. Each CTA's TMEM holds its 128 rows
// of the tile, drained by its own epilogue as in the single-CTA kernel.
constexpr int P_STAGES = 6;
constexpr int P_A_BYTES = BM * BK * 2;  // 16 KB: this CTA's 128 rows of X
constexpr int P_B_BYTES = BM * BK * 2;  // 16 KB: this CTA's 128 rows of W
constexpr int P_SMEM_BYTES = P_STAGES * (P_A_BYTES + P_B_BYTES) + EPI_BYTES + 1024 + 256;
static_assert(P_SMEM_BYTES <= 232448, "shared memory of one CTA");

template <int EPI>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_f16_tc2_kernel(const __grid_constant__ CUtensorMap tm_x,
                         const __grid_constant__ CUtensorMap tm_w,
                         const __grid_constant__ CUtensorMap tm_o,
                         const __grid_constant__ CUtensorMap tm_xl,
                         const __grid_constant__ CUtensorMap tm_wl, TcParams p) {
    using namespace sm100;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + P_STAGES * P_A_BYTES;
    uint8_t *sE = sB + P_STAGES * P_B_BYTES;
    uint64_t *full = reinterpret_cast<uint64_t *>(sE + EPI_BYTES);
    uint64_t *empty = full + P_STAGES;
    uint64_t *tfull = empty + P_STAGES;
    uint64_t *tempty = tfull + 2;
    uint64_t *drain = tempty + 2;
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
    const int num_tiles = p.m_tiles * p.n_tiles;  // m_tiles counts 256-row tiles here

    if (threadIdx.x == 0) {
        for (int s = 0; s < P_STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 8);  // one arrival per epilogue warp of both CTAs
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
        tmem_alloc_pair(tmem_holder, TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync_all();  // both CTAs' barriers initialised, TMEM allocated
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;

    if (warp == 0) {
        if (lane == 0) {
            // ------------------------------------------------ TMA producer (both CTAs)
            int stage = 0;
            uint32_t phase = 0;
            int issued = 0;
            for (int tile = pair; tile < num_tiles && !*abort_flag; tile += n_pairs) {
                const int m_blk = p.n_fast ? tile / p.n_tiles : tile % p.m_tiles;
                const int n_blk = p.n_fast ? tile % p.n_tiles : tile / p.m_tiles;
                for (int kb = 0, ps = 0, lk = 0; kb < p.total_kb; ++kb) {
                    if (!mbar_wait_cluster(&empty[stage], phase ^ 1)) {
                        set_error(p.err, kErrWaitTimeout);
                        *abort_flag = 1;
                        break;
                    }
                    const uint32_t bar0 = mapa_shared(smem_addr(&full[stage]), 0);
                    if (rank == 0) mbar_expect_tx(&full[stage], 2 * (P_A_BYTES + P_B_BYTES));
                    const int kx = lk * p.pass_kw[ps];
                    tma_load_2d_pair(sA + stage * P_A_BYTES, p.pass_a[ps] ? &tm_xl : &tm_x, bar0, kx,
                                     m_blk * (2 * BM) + static_cast<int>(rank) * BM);
                    tma_load_2d_pair(sB + stage * P_B_BYTES, p.pass_b[ps] ? &tm_wl : &tm_w, bar0, kx,
                                     n_blk * BN + static_cast<int>(rank) * BM);
                    if (++lk == p.pass_kb[ps]) {
                        lk = 0;
                        ++ps;
                    }
                    ++issued;
                    if (++stage == P_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            // Wait until the MMAs released every stage this CTA filled (their
            // completions arrive on this CTA's `empty` barriers), so no arrival
            // is still on its way when the CTA exits.
            for (int i = 0; i < P_STAGES && issued > 0 && !*abort_flag; ++i) {
                if (!mbar_wait_cluster(&empty[stage], phase ^ 1)) {
                    set_error(p.err, kErrWaitTimeout);
                    break;
                }
                if (++stage == P_STAGES) {
                    stage = 0;
                    phase ^= 1;
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            // ------------------------------------------------ MMA issuer (first CTA)
            constexpr uint32_t idesc = idesc_f16_f32(2 * BM, BN);
            constexpr uint32_t idesc8 = idesc_e5m2_e4m3_f32(2 * BM, BN);
            constexpr uint32_t idesc32 = idesc_tf32_f32(2 * BM, BN);
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            const uint32_t peer = 1;
            for (int tile = pair; tile < num_tiles && !*abort_flag; tile += n_pairs) {
                if (!mbar_wait_cluster(&tempty[acc], acc_phase ^ 1)) {
                    set_error(p.err, kErrWaitTimeout);
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                for (int kb = 0, ps = 0, lk = 0; kb < p.total_kb; ++kb) {
                    if (!mbar_wait_cluster(&full[stage], phase)) {
                        set_error(p.err, kErrWaitTimeout);
                        *abort_flag = 1;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = smem_addr(sA + stage * P_A_BYTES);
                    const uint32_t b0 = smem_addr(sB + stage * P_B_BYTES);
                    const int kind = p.pass_kind[ps];
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const uint64_t ad = desc_kmajor_sw128(a0 + k * 32), bd = desc_kmajor_sw128(b0 + k * 32);
                        const uint32_t acc = (kb | k) != 0;
                        if (kind == kPassF16)
                            mma_f16_pair(d_tmem, ad, bd, idesc, acc);
                        else if (kind == kPassF8)
                            mma_f8_pair(d_tmem, ad, bd, idesc8, acc);
                        else
                            mma_tf32_pair(d_tmem, ad, bd, idesc32, acc);
                    }
                    if (++lk == p.pass_kb[ps]) {
                        lk = 0;
                        ++ps;
                    }
                    mma_commit_pair(smem_addr(&empty[stage]));
                    mma_commit_pair(mapa_shared(smem_addr(&empty[stage]), peer));
                    if (++stage == P_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (*abort_flag) {
                    mma_commit_pair(smem_addr(drain));
                    (void)mbar_wait(drain, 0);
                    break;
                }
                mma_commit_pair(smem_addr(&tfull[acc]));
                mma_commit_pair(mapa_shared(smem_addr(&tfull[acc]), peer));
                acc ^= 1;
                if (acc == 0) acc_phase ^= 1;
            }
        }
    } else {
        // ---------------------------------------------------- epilogue
        const int quarter = warp & 3;  // TMEM lanes this warp may access
        uint8_t *const slab0 = sE + (warp - 2) * 2 * EPI_BUF_BYTES;
        int sb = 0;  // staging buffer to fill next
        auto slab = [&]() { return slab0 + sb * EPI_BUF_BYTES; };
        int acc = 0;
        uint32_t acc_phase = 0;
        // Hand a filled slab to the TMA unit (lane 0), keeping at most one older
        // store in flight on the other buffer.
        auto issue = [&](int x, int y) {
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
                if (EPI == kEpiResidual)
                    tma_reduce_add_2d(&tm_o, slab(), x, y);
                else
                    tma_store_2d(&tm_o, slab(), x, y);
                bulk_commit();
            }
            sb ^= 1;
        };
        auto reuse_wait = [&]() {
            if (lane == 0) bulk_wait_read<1>();
            __syncwarp();
        };
        for (int tile = pair; tile < num_tiles; tile += n_pairs) {
            if (!mbar_wait_cluster(&tfull[acc], acc_phase)) {
                set_error(p.err, kErrWaitTimeout);
                *abort_flag = 1;
                break;
            }
            if (*abort_flag) break;
            tc_fence_after();
            const int m_blk = p.n_fast ? tile / p.n_tiles : tile % p.m_tiles;
            const int n_blk = p.n_fast ? tile % p.n_tiles : tile / p.m_tiles;
            const int row0 = m_blk * (2 * BM) + static_cast<int>(rank) * BM + quarter * 32;
            const int row = row0 + lane;
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN;
            const bool row_ok = row < p.M;
            const bool slab_ok = row0 < p.M;
            if (EPI == kEpiSwiGLU) {
                // Tile columns [0,128) are gate rows, [128,256) the matching up rows;
                // each round produces 64 fp16 outputs per row.
#pragma unroll 1
                for (int c = 0; c < BN / 2; c += 64) {
                    uint32_t packed[32];
#pragma unroll
                    for (int hh = 0; hh < 2; ++hh) {
                        float g[32], u[32];
                        tmem_ld32(t_row + c + 32 * hh, g);
                        tmem_ld32(t_row + BN / 2 + c + 32 * hh, u);
                        const int wcol = n_blk * BN + c + 32 * hh;  // weight row of g[0]
                        if (p.scale) {
#pragma unroll
                            for (int i = 0; i < 32; ++i) {
                                g[i] *= __ldg(p.scale + wcol + i);
                                u[i] *= __ldg(p.scale + wcol + BN / 2 + i);
                            }
                        }
                        uint32_t lo[8];
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            const float y0 = silu_fast(g[2 * i]) * u[2 * i], y1 = silu_fast(g[2 * i + 1]) * u[2 * i + 1];
                            __half2 h2 = __floats2half2_rn(y0, y1);
                            packed[16 * hh + i] = *reinterpret_cast<uint32_t *>(&h2);
                            const uint32_t l2 = static_cast<uint32_t>(lo_e5m2(y0, __low2half(h2))) |
                                                (static_cast<uint32_t>(lo_e5m2(y1, __high2half(h2))) << 8);
                            if (i & 1)
                                lo[i >> 1] |= l2 << 16;
                            else
                                lo[i >> 1] = l2;
                        }
                        if (p.out_lo && row_ok) {
                            // The next projection's low part: 32 bytes of e5m2 per row and half round.
                            uint4 *dl = reinterpret_cast<uint4 *>(p.out_lo + static_cast<size_t>(row) * p.ldo_lo +
                                                                  n_blk * (BN / 2) + c + 32 * hh);
                            dl[0] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                            dl[1] = make_uint4(lo[4], lo[5], lo[6], lo[7]);
                        }
                    }
                    const int ocol = n_blk * (BN / 2) + c;
                    if (p.tma_out) {
                        if (!slab_ok || ocol >= p.N / 2) continue;
                        reuse_wait();
                        uint4 ch[8];
#pragma unroll
                        for (int i = 0; i < 8; ++i) ch[i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2], packed[4 * i + 3]);
                        stage_row(slab(), lane, ch);
                        issue(ocol, row0);
                    } else if (row_ok) {
                        __half *dst = reinterpret_cast<__half *>(p.out) + static_cast<size_t>(row) * p.ldo + ocol;
                        const __half *hv = reinterpret_cast<const __half *>(packed);
                        for (int i = 0; i < 64 && ocol + i < p.N / 2; ++i) dst[i] = hv[i];
                    }
                }
            } else if (EPI == kEpiStore) {
#pragma unroll 1
                for (int c = 0; c < BN; c += 64) {
                    const int col = n_blk * BN + c;
                    uint32_t packed[32];
#pragma unroll
                    for (int hh = 0; hh < 2; ++hh) {
                        float v[32];
                        tmem_ld32(t_row + c + 32 * hh, v);
                        if (p.scale) {
#pragma unroll
                            for (int i = 0; i < 32; ++i)
                                if (col + 32 * hh + i < p.N) v[i] *= __ldg(p.scale + col + 32 * hh + i);
                        }
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            __half2 h2 = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
                            packed[16 * hh + i] = *reinterpret_cast<uint32_t *>(&h2);
                        }
                    }
                    if (p.tma_out) {
                        if (!slab_ok || col >= p.N) continue;
                        reuse_wait();
                        uint4 ch[8];
#pragma unroll
                        for (int i = 0; i < 8; ++i) ch[i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2], packed[4 * i + 3]);
                        stage_row(slab(), lane, ch);
                        issue(col, row0);
                    } else if (row_ok) {
                        __half *dst = reinterpret_cast<__half *>(p.out) + static_cast<size_t>(row) * p.ldo + col;
                        const __half *hv = reinterpret_cast<const __half *>(packed);
                        for (int i = 0; i < 64 && col + i < p.N; ++i) dst[i] = hv[i];
                    }
                }
            } else {
                // fp32 outputs: store, or add into the residual stream.
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
                    if (p.tma_out) {
                        if (!slab_ok || valid <= 0) continue;
                        reuse_wait();
                        uint4 ch[8];
#pragma unroll
                        for (int i = 0; i < 8; ++i)
                            ch[i] = make_uint4(__float_as_uint(v[4 * i]), __float_as_uint(v[4 * i + 1]),
                                               __float_as_uint(v[4 * i + 2]), __float_as_uint(v[4 * i + 3]));
                        stage_row(slab(), lane, ch);
                        issue(col, row0);
                    } else if (row_ok && valid > 0) {
                        float *dst = reinterpret_cast<float *>(p.out) + static_cast<size_t>(row) * p.ldo + col;
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            if (i < valid) dst[i] = (EPI == kEpiResidual) ? dst[i] + v[i] : v[i];
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_addr(&tempty[acc]), 0));
            acc ^= 1;
            if (acc == 0) acc_phase ^= 1;
        }
        if (lane == 0) bulk_wait_all();
        __syncwarp();
    }

    tc_fence_before();
    cluster_sync_all();  // no arrival into either CTA is pending; both epilogues are done
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, TMEM_COLS);
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

}  // namespace

namespace {
CUtensorMap tensor_map_2d(CUtensorMapDataType t, const void *base, uint64_t rows, uint64_t cols,
                          uint64_t row_stride_bytes, uint32_t box_cols, uint32_t box_rows) {
    if ((reinterpret_cast<uintptr_t>(base) & 15) || row_stride_bytes % 16)
        throw CudaError("tensor map base must be 16-byte aligned with a row stride % 16 == 0");
    CUtensorMap m;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride_bytes)};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode_fn()(&m, t, 2, const_cast<void *>(base), dims, strides, box, estr,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw CudaError("cuTensorMapEncodeTiled failed: " + std::to_string(r));
    return m;
}
}  // namespace

CUtensorMap tensor_map_f16(const void *base, uint64_t rows, uint64_t cols, uint64_t row_stride_bytes,
                           uint32_t box_cols, uint32_t box_rows) {
    return tensor_map_2d(CU_TENSOR_MAP_DATA_TYPE_FLOAT16, base, rows, cols, row_stride_bytes, box_cols, box_rows);
}

CUtensorMap tensor_map_f32(const void *base, uint64_t rows, uint64_t cols, uint64_t row_stride_bytes,
                           uint32_t box_cols, uint32_t box_rows) {
    return tensor_map_2d(CU_TENSOR_MAP_DATA_TYPE_FLOAT32, base, rows, cols, row_stride_bytes, box_cols, box_rows);
}

CUtensorMap tensor_map_u8(const void *base, uint64_t rows, uint64_t cols, uint64_t row_stride_bytes,
                          uint32_t box_cols, uint32_t box_rows) {
    return tensor_map_2d(CU_TENSOR_MAP_DATA_TYPE_UINT8, base, rows, cols, row_stride_bytes, box_cols, box_rows);
}

namespace {

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

// A 2-D 8-bit tensor map (the low-part operands x_lo / w8) over rows x inner
// bytes (row stride ld bytes), box of box_rows x 128 bytes, zero fill.
CUtensorMap make_map8(const void *base, int rows, int inner, int ld, int box_rows) {
    if ((reinterpret_cast<uintptr_t>(base) & 15) || ld % 16)
        throw CudaError("8-bit GEMM operand must be 16-byte aligned with a row stride % 16 == 0");
    CUtensorMap m;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld)};
    cuuint32_t box[2] = {128, static_cast<cuuint32_t>(box_rows)};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box,
                             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw CudaError("cuTensorMapEncodeTiled (8-bit) failed: " + std::to_string(r));
    return m;
}

// A 2-D fp32 tensor map (the 3xTF32 operands): box of box_rows x 32
// elements (one 128-byte swizzle row), zero fill.
CUtensorMap make_map32(const void *base, int rows, int inner, int ld, int box_rows) {
    return tensor_map_f32(base, rows, inner, static_cast<uint64_t>(ld) * 4, 32, box_rows);
}

// The operand maps and the K-pass table of a launch: fp16 (64-wide blocks),
// optionally followed by the 8-bit low part (128-wide blocks), or the three
// tf32 passes (32-wide blocks); plus the SwiGLU low output.
void set_passes(const GemmArgs &a, int w_box_rows, TcParams &p, CUtensorMap &tx, CUtensorMap &tw, CUtensorMap &txl,
                CUtensorMap &twl) {
    std::memset(&txl, 0, sizeof(txl));
    std::memset(&twl, 0, sizeof(twl));
    auto pass = [&](int kb, int kw, int as, int bs, int kind) {
        p.pass_kb[p.n_pass] = kb;
        p.pass_kw[p.n_pass] = kw;
        p.pass_a[p.n_pass] = as;
        p.pass_b[p.n_pass] = bs;
        p.pass_kind[p.n_pass] = kind;
        ++p.n_pass;
    };
    p.n_pass = 0;
    if (a.tf32) {
        if (!a.x_lo32 || !a.w_lo32) throw CudaError("a 3xTF32 GEMM needs x_lo32 and w_lo32");
        if (a.epilogue != kEpiResidual && a.epilogue != kEpiStoreF32)
            throw CudaError("the 3xTF32 GEMM stores fp32 outputs only");
        tx = make_map32(a.x, a.M, a.K, a.ldx, BM);
        tw = make_map32(a.w, a.N, a.K, a.ldw, w_box_rows);
        txl = make_map32(a.x_lo32, a.M, a.K, a.ldx_lo32, BM);
        twl = make_map32(a.w_lo32, a.N, a.K, a.ldw_lo32, w_box_rows);
        const int kb = ceil_div(a.K, 32);
        pass(kb, 32, 0, 0, kPassTF32);  // x   w
        pass(kb, 32, 0, 1, kPassTF32);  // x   w_lo
        pass(kb, 32, 1, 0, kPassTF32);  // x_lo w
    } else {
        tx = make_map(a.x, a.M, a.K, a.ldx, BM);
        tw = make_map(a.w, a.N, a.K, a.ldw, w_box_rows);
        pass(ceil_div(a.K, BK), BK, 0, 0, kPassF16);
        if (a.x_lo && a.w8) {
            txl = make_map8(a.x_lo, a.M, a.K, a.ldx_lo, BM);
            twl = make_map8(a.w8, a.N, a.K, a.ldw8, w_box_rows);
            pass(ceil_div(a.K, 128), 128, 1, 1, kPassF8);
        } else if (a.x_lo || a.w8) {
            throw CudaError("a split-precision GEMM needs both x_lo and w8");
        }
    }
    p.total_kb = 0;
    for (int i = 0; i < p.n_pass; ++i) p.total_kb += p.pass_kb[i];
    p.out_lo = a.epilogue == kEpiSwiGLU ? a.out_lo : nullptr;
    p.ldo_lo = a.ldo_lo;
    if (p.out_lo && ((reinterpret_cast<uintptr_t>(p.out_lo) & 15) || p.ldo_lo % 16))
        throw CudaError("SwiGLU low-part output must be 16-byte aligned with a row stride % 16 == 0");
}

// Output tensor map for the epilogue's TMA stores: box of 32 rows x 128 bytes
// (32 fp32 or 64 fp16 columns), 128B swizzle. Returns false when the output
// does not meet TMA's alignment rules (the epilogue then stores directly).
bool make_out_map(CUtensorMap &m, const void *base, int rows, int cols, int ld, bool f32) {
    const int esz = f32 ? 4 : 2;
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (static_cast<long>(ld) * esz) % 16) return false;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * esz};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / esz), 32};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode_fn()(&m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                             const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <int EPI>
void launch(const GemmArgs &a, cudaStream_t s, int num_sms) {
    static SmemOptIn opt_in;
    opt_in.ensure(gemm_f16_tc_kernel<EPI>, SMEM_BYTES);
    TcParams p;
    CUtensorMap tx, tw, txl, twl;
    set_passes(a, BN, p, tx, tw, txl, twl);
    p.M = a.M;
    p.N = a.N;
    p.K = a.K;
    p.m_tiles = ceil_div(a.M, BM);
    p.n_tiles = ceil_div(a.N, BN);
    p.n_fast = p.n_tiles <= 8 ? 1 : 0;

    p.out = a.out;
    p.ldo = a.ldo;
    p.scale = a.scale;
    const int elem = (EPI == kEpiStore || EPI == kEpiSwiGLU) ? 2 : 4;
    p.vec_ok = ((reinterpret_cast<uintptr_t>(a.out) & 15) == 0) && ((a.ldo * elem) % 16 == 0);
    p.err = a.err;
    CUtensorMap to;
    std::memset(&to, 0, sizeof(to));
    const bool f32 = (EPI == kEpiResidual || EPI == kEpiStoreF32);
    const int out_cols = (EPI == kEpiSwiGLU) ? a.N / 2 : a.N;
    p.tma_out = make_out_map(to, a.out, a.M, out_cols, a.ldo, f32) ? 1 : 0;
    const int tiles = p.m_tiles * p.n_tiles;
    const int grid = tiles < num_sms ? tiles : num_sms;
    gemm_f16_tc_kernel<EPI><<<grid, THREADS, SMEM_BYTES, s>>>(tx, tw, to, txl, twl, p);
    HK_LAUNCH_CHECK();
}

template <int EPI>
void launch_pair(const GemmArgs &a, cudaStream_t s, int num_sms) {
    static SmemOptIn opt_in;
    opt_in.ensure(gemm_f16_tc2_kernel<EPI>, P_SMEM_BYTES);
    TcParams p;
    CUtensorMap tx, tw, txl, twl;
    set_passes(a, BM, p, tx, tw, txl, twl);  // each CTA of a pair loads 128 rows of W
    p.M = a.M;
    p.N = a.N;
    p.K = a.K;
    p.m_tiles = ceil_div(a.M, 2 * BM);
    p.n_tiles = ceil_div(a.N, BN);
    p.n_fast = p.n_tiles <= 8 ? 1 : 0;

    p.out = a.out;
    p.ldo = a.ldo;
    p.scale = a.scale;
    const int elem = (EPI == kEpiStore || EPI == kEpiSwiGLU) ? 2 : 4;
    p.vec_ok = ((reinterpret_cast<uintptr_t>(a.out) & 15) == 0) && ((a.ldo * elem) % 16 == 0);
    p.err = a.err;
    CUtensorMap to;
    std::memset(&to, 0, sizeof(to));
    const bool f32 = (EPI == kEpiResidual || EPI == kEpiStoreF32);
    const int out_cols = (EPI == kEpiSwiGLU) ? a.N / 2 : a.N;
    p.tma_out = make_out_map(to, a.out, a.M, out_cols, a.ldo, f32) ? 1 : 0;
    const int tiles = p.m_tiles * p.n_tiles;
    const int pairs = tiles < num_sms / 2 ? tiles : num_sms / 2;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * pairs);
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = P_SMEM_BYTES;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    HK_CUDA(cudaLaunchKernelEx(&cfg, gemm_f16_tc2_kernel<EPI>, tx, tw, to, txl, twl, p));
    HK_LAUNCH_CHECK();
}

}  // namespace

void gemm_f16_tc_pair(const GemmArgs &a, cudaStream_t s, int num_sms) {
    if (a.M <= 0 || a.N <= 0 || a.K <= 0) return;
    if (a.epilogue == kEpiSwiGLU && (a.N % BN) != 0)
        throw CudaError("fused SwiGLU GEMM needs N to be a multiple of 256");
    switch (a.epilogue) {
        case kEpiStore: launch_pair<kEpiStore>(a, s, num_sms); break;
        case kEpiResidual: launch_pair<kEpiResidual>(a, s, num_sms); break;
        case kEpiSwiGLU: launch_pair<kEpiSwiGLU>(a, s, num_sms); break;
        case kEpiStoreF32: launch_pair<kEpiStoreF32>(a, s, num_sms); break;
        default: throw CudaError("unknown GEMM epilogue");
    }
}

void gemm_f16_tc(const GemmArgs &a, cudaStream_t s, int num_sms) {
    if (a.M <= 0 || a.N <= 0 || a.K <= 0) return;
    // CTA pairs where the single-CTA kernel waits on its operand loads: the
    // fp32-store projections (the widest outputs) and long-K residual ones
    // (measured on the cfg2 shapes: +7% and +1.5%; the SwiGLU and K = 2048
    // residual launches gain nothing or lose, and stay on single CTAs).
    if (a.M >= 512 && num_sms >= 2 &&
        (a.epilogue == kEpiStoreF32 || (a.epilogue == kEpiResidual && a.K >= 3072))) {
        gemm_f16_tc_pair(a, s, num_sms);
        return;
    }
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
