// Packed (GGML Q8_0 / Q4_0) projections of the reference's quantized profile
// (Projection::Packed, crates/huncho-backend/src/qwen3_5.rs:320-369; the
// artifact of crates/huncho-backend/src/qwen_quantized.rs:91-193).
//
// The reference's CPU matmul quantizes each fp32 input row to Q8_0 blocks of
// 32 (d = max|x| / 127, q = roundf(x * (1/d)), d kept as fp16) and sums per
// output, over the blocks in order, (float(sum_i q_w q_x) * d_w) * d_x in
// fp32 (qwen_quantized.rs:137-163). Weights are stored as int8 block values
// (Q4_0 as q - 8) [N, Kp] plus fp32 block scales, block-major [Kp/32, N]
// (as are the input rows' scales [Kp/32, M]), so the 32 rows or columns of a
// warp read one 128-byte line per block. Here:
//   * quantize_rows_kernel: one warp per (row, block), the same Q8_0 steps;
//   * gemm_q8_tc_kernel: the block dots on the 5th-generation tensor cores
//     (tcgen05.mma kind::i8, M = 128, N = 128, K = 32: exactly one Q8_0 block
//     per instruction, a separate int32 accumulator in tensor memory per
//     block), and the block's scales applied by the epilogue warps in
//     registers with round-to-nearest operations in the reference's order, so
//     each output equals the block-sequential sum bit for bit. Block scales
//     are fp16 values (GGML stores them so): the exactness of -C * d_w below
//     rests on it.
//
// Persistent, warp-specialised CTA (one per SM), 128 x 128 output tiles:
//   warp 0       TMA producer: 128-row x 128-byte boxes (four blocks) of the
//                quantized input and of the weights, 128-byte swizzle, into a
//                4-stage ring (32 KB per stage);
//   warp 1       allocates all 512 TMEM columns (four 128 x 128 int32 block
//                accumulators) and issues one MMA per block from one thread;
//   warps 2..17  epilogue: warp w drains the 32 TMEM lanes (rows) of quarter
//                w % 4 and 32 of the tile's columns in two 16-column loads
//                (the second in flight while the first half is scaled),
//                releases the accumulator once both have landed, and adds the
//                scaled block dots to its running fp32 sums.
// Each block dot v leaves TMEM as int32; adding the bits of C = 1.5 * 2^23
// makes the fp32 value C + v (exact), and one paired fma per two outputs,
// fma(C + v, d_w, -C d_w), gives v * d_w with a single rounding (the exact
// product less the exact -C d_w), as the reference's float(v) * d_w. The
// multiply by d_x stays scalar (__fmul_rn: a paired multiply feeding a paired
// add is fused into a paired fma by the device compiler, measured on the
// B200, which would drop a rounding); the sums take paired adds. That scale
// arithmetic (3.5 issue slots per output and block) bounds the kernel: the
// MMAs take a tenth of it. Four block accumulators let the tensor core run
// three blocks ahead, so the epilogue warps drift apart instead of waiting on
// each block together, and each warp's block scales arrive by cp.async one
// group of four blocks ahead.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>

#include <cstring>

#include "common.cuh"
#include "gemm.cuh"
#include "sm100.cuh"

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
    if (lane == 0) d[static_cast<size_t>(b) * M + m] = __half2float(__float2half_rn(dd));
}

__global__ void transpose_scales_kernel(const float *in, int rows, int nb, float *out) {
    const long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<long>(rows) * nb) return;
    const int b = static_cast<int>(i / rows), r = static_cast<int>(i % rows);
    out[i] = in[static_cast<size_t>(r) * nb + b];
}

constexpr int QBM = 128, QBN = 128, QSTAGES = 4;
constexpr int QA_BYTES = QBM * 128;  // 16 KB: 128 rows x four 32-byte blocks
constexpr int QB_BYTES = QBN * 128;  // 16 KB
constexpr int Q_EPI_WARPS = 16;
constexpr int Q_THREADS = 64 + 32 * Q_EPI_WARPS;  // 576
constexpr int Q_ACC = 4;                          // int32 block accumulators in TMEM
constexpr int Q_TMEM_COLS = Q_ACC * QBN;          // all 512 columns
// Per epilogue warp, two group slots of block scales: 4 blocks x 32 weight
// scales (block j of the group at [32 j + lane]) and 32 lanes x 4 row scales.
constexpr int Q_SCALE_FLOATS = 2 * (128 + 128);
constexpr int Q_WBUF_BYTES = Q_EPI_WARPS * Q_SCALE_FLOATS * 4;
constexpr int Q_SMEM_BYTES = QSTAGES * (QA_BYTES + QB_BYTES) + Q_WBUF_BYTES + 1024 + 256;
static_assert(Q_SMEM_BYTES <= 232448, "shared memory of one CTA");

struct Q8Params {
    int M, N, nb;  // nb = kp / 32 blocks per row
    int m_tiles, n_tiles, n_fast;
    const float *xd;  // [nb, M]
    const float *wd;  // [nb, N]
    float *out;
    int ldo;
    int vec_ok;  // out / ldo allow 16-byte vector accesses
    uint32_t *err;
};

// An int32 block dot v (|v| <= 32 * 128 * 128 = 2^19) plus the bits of
// C = 1.5 * 2^23 is the fp32 bit pattern of C + v, exactly (|v| < 2^22).
constexpr int kDotBias = 0x4B400000;
constexpr float kDotBiasF = 12582912.0f;
__device__ __forceinline__ float2 biased_pair(uint32_t r0, uint32_t r1) {
    return make_float2(__int_as_float(static_cast<int>(r0) + kDotBias), __int_as_float(static_cast<int>(r1) + kDotBias));
}

// Four-byte asynchronous copy global -> shared, zero-filled when !ok (then
// nothing is read).
__device__ __forceinline__ void cp_async4(float *dst, const float *src, bool ok) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(sm100::smem_addr(dst)), "l"(src),
                 "r"(ok ? 4 : 0)
                 : "memory");
}

// Block scales g .. g+3 (zero past nb or outside the matrix) of this lane's
// column (wd_col = wd + column, stride N per block) and this thread's row
// (xd_row = xd + row, stride M), in flight as one cp.async group: the column's
// to wg[32 j + l] (where the warp reads them as broadcasts), the row's to
// xg[4 l + j]. Each copy instruction reads one line for the warp.
__device__ __forceinline__ void prefetch_scales(float *wg, float *xg, const float *wd_col, const float *xd_row, int g,
                                                int nb, int N, int M, bool col_ok, bool row_ok, int lane) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const bool in = g + j < nb;
        cp_async4(wg + 32 * j + lane, in && col_ok ? wd_col + static_cast<size_t>(g + j) * N : wd_col, in && col_ok);
        cp_async4(xg + 4 * lane + j, in && row_ok ? xd_row + static_cast<size_t>(g + j) * M : xd_row, in && row_ok);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
}

// tcgen05.ld of 16 consecutive 32-bit columns of this thread's TMEM lane,
// without the wait: the registers are undefined until tmem_wait_ld16 on them.
__device__ __forceinline__ void tmem_ld16_async(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}
// Wait for this thread's outstanding tcgen05.ld; the registers are named as
// read and written so no use of them is scheduled before the wait.
__device__ __forceinline__ void tmem_wait_ld16(uint32_t (&r)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15])
                 :
                 : "memory");
}

// 16 outputs' block terms into the running sums: raw holds the int32 dots of
// columns c0 .. c0+15 (ws = their weight scales), xdv the row's scale.
__device__ __forceinline__ void scale_add16(float2 (&acc)[16], int c0, const uint32_t (&raw)[16], const float *ws,
                                            float xdv) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float4 w4 = *reinterpret_cast<const float4 *>(ws + c0 + 4 * i);
        const float2 wa = make_float2(w4.x, w4.y), wb = make_float2(w4.z, w4.w);
        // f = C + dot exactly, so fma(f, d_w, -C d_w) is dot * d_w rounded
        // once, as float(dot) * d_w rounds it; -C d_w is exact (d_w has at
        // most 11 significant bits).
        const float2 nc = make_float2(-kDotBiasF, -kDotBiasF);
        const float2 t0 = __ffma2_rn(biased_pair(raw[4 * i], raw[4 * i + 1]), wa, __fmul2_rn(wa, nc));
        const float2 t1 = __ffma2_rn(biased_pair(raw[4 * i + 2], raw[4 * i + 3]), wb, __fmul2_rn(wb, nc));
        // Then * d_x (scalar __fmul_rn, never fused into the add) and the
        // running sums, two per paired add.
        float2 &a0 = acc[(c0 >> 1) + 2 * i], &a1 = acc[(c0 >> 1) + 2 * i + 1];
        a0 = __fadd2_rn(a0, make_float2(__fmul_rn(t0.x, xdv), __fmul_rn(t0.y, xdv)));
        a1 = __fadd2_rn(a1, make_float2(__fmul_rn(t1.x, xdv), __fmul_rn(t1.y, xdv)));
    }
}

template <bool RESIDUAL>
__global__ void __launch_bounds__(Q_THREADS, 1)
    gemm_q8_tc_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                      Q8Params p) {
    using namespace sm100;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + QSTAGES * QA_BYTES;
    float *wbuf = reinterpret_cast<float *>(sB + QSTAGES * QB_BYTES);
    uint64_t *full = reinterpret_cast<uint64_t *>(reinterpret_cast<uint8_t *>(wbuf) + Q_WBUF_BYTES);
    uint64_t *empty = full + QSTAGES;
    uint64_t *afull = empty + QSTAGES;  // block accumulator u holds a finished dot
    uint64_t *aempty = afull + Q_ACC;   // every epilogue warp has read accumulator u
    uint64_t *drain = aempty + Q_ACC;   // MMA completion on the abort path
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int num_tiles = p.m_tiles * p.n_tiles;
    const int n_stages = (p.nb + 3) >> 2;  // stages per tile (four blocks each)

    if (threadIdx.x == 0) {
        for (int s = 0; s < QSTAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < Q_ACC; ++b) {
            mbar_init(&afull[b], 1);
            mbar_init(&aempty[b], Q_EPI_WARPS);
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
        tmem_alloc(tmem_holder, Q_TMEM_COLS);
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
                for (int st = 0; st < n_stages; ++st) {
                    if (!mbar_wait_backoff(&empty[stage], phase ^ 1, 64)) {
                        set_error(p.err, kErrWaitTimeout);
                        *abort_flag = 1;
                        break;
                    }
                    // Byte column st * 128 is a multiple of 16; columns past kp read as zero.
                    mbar_expect_tx(&full[stage], QA_BYTES + QB_BYTES);
                    tma_load_2d(sA + stage * QA_BYTES, &tm_x, &full[stage], st * 128, m_blk * QBM);
                    tma_load_2d(sB + stage * QB_BYTES, &tm_w, &full[stage], st * 128, n_blk * QBN);
                    issued_mask |= 1u << stage;
                    issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
                    if (++stage == QSTAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            if (*abort_flag) {
                // Let every copy this thread issued land before the CTA exits.
                for (int s = 0; s < QSTAGES; ++s)
                    if (issued_mask & (1u << s)) (void)mbar_wait(&full[s], (issued_parity >> s) & 1);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ------------------------------------------------ MMA issuer
            constexpr uint32_t idesc = idesc_s8_s32(QBM, QBN);
            int stage = 0;
            uint32_t phase = 0;
            uint32_t gb = 0;  // blocks issued by this CTA: accumulator gb % Q_ACC
            for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
                for (int st = 0; st < n_stages && !*abort_flag; ++st) {
                    if (!mbar_wait_backoff(&full[stage], phase, 32)) {
                        set_error(p.err, kErrWaitTimeout);
                        *abort_flag = 1;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = smem_addr(sA + stage * QA_BYTES);
                    const uint32_t b0 = smem_addr(sB + stage * QB_BYTES);
                    const int nblk = min(4, p.nb - st * 4);
                    for (int j = 0; j < nblk; ++j, ++gb) {
                        const uint32_t u = gb % Q_ACC;
                        if (!mbar_wait_backoff(&aempty[u], ((gb / Q_ACC) & 1) ^ 1, 32)) {
                            set_error(p.err, kErrWaitTimeout);
                            *abort_flag = 1;
                            break;
                        }
                        tc_fence_after();
                        mma_i8(tmem_base + u * QBN, desc_kmajor_sw128(a0 + j * 32), desc_kmajor_sw128(b0 + j * 32),
                               idesc, 0);
                        mma_commit(&afull[u]);
                    }
                    mma_commit(&empty[stage]);
                    if (++stage == QSTAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            if (*abort_flag) {
                // Let the MMAs already issued finish before TMEM is freed.
                mma_commit(drain);
                (void)mbar_wait(drain, 0);
            }
        }
    } else {
        // ---------------------------------------------------- epilogue
        const int ew = warp - 2;
        const int quarter = warp & 3;  // TMEM lanes (tile rows) this warp may access
        const int cgrp = ew >> 2;      // the warp's 32 columns of the tile
        float *const scales = wbuf + ew * Q_SCALE_FLOATS;  // two group slots: 128 d_w, then 128 d_x
        const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + cgrp * 32;
        uint32_t gb = 0;
        for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
            const int m_blk = p.n_fast ? tile / p.n_tiles : tile % p.m_tiles;
            const int n_blk = p.n_fast ? tile % p.n_tiles : tile / p.m_tiles;
            const int row = m_blk * QBM + quarter * 32 + lane;
            const int col0 = n_blk * QBN + cgrp * 32;
            const bool row_ok = row < p.M;
            const bool col_ok = col0 + lane < p.N;
            const float *xd_row = p.xd + (row_ok ? row : 0);
            const float *wd_col = p.wd + (col_ok ? col0 + lane : 0);
            float2 acc[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) acc[i] = make_float2(0.0f, 0.0f);
            __syncwarp();  // the previous tile's reads of slot 0 are done
            prefetch_scales(scales, scales + 128, wd_col, xd_row, 0, p.nb, p.N, p.M, col_ok, row_ok, lane);
            for (int g = 0, slot = 0; g < p.nb; g += 4, slot ^= 1) {
                // This group's scales landed (this thread's copies, then the warp's).
                asm volatile("cp.async.wait_group 0;" ::: "memory");
                __syncwarp();
                const float *wg = scales + slot * 256;
                const float4 xd4 = *reinterpret_cast<const float4 *>(wg + 128 + 4 * lane);
                if (g + 4 < p.nb)  // the next group's, into the other slot (read by the last group)
                    prefetch_scales(scales + (slot ^ 1) * 256, scales + (slot ^ 1) * 256 + 128, wd_col, xd_row, g + 4,
                                    p.nb, p.N, p.M, col_ok, row_ok, lane);
                const int gn = min(4, p.nb - g);
#pragma unroll 1
                for (int j = 0; j < gn; ++j, ++gb) {
                    const uint32_t u = gb % Q_ACC;
                    const float xdv = j == 0 ? xd4.x : j == 1 ? xd4.y : j == 2 ? xd4.z : xd4.w;
                    if (!mbar_wait(&afull[u], (gb / Q_ACC) & 1)) {
                        set_error(p.err, kErrWaitTimeout);
                        *abort_flag = 1;
                        break;
                    }
                    tc_fence_after();
                    // Two 16-column halves: the second half's TMEM load is in flight
                    // while the first half is scaled.
                    const uint32_t ta = t_lane + u * QBN;
                    uint32_t r0[16], r1[16];
                    tmem_ld16_async(ta, r0);
                    tmem_wait_ld16(r0);
                    tmem_ld16_async(ta + 16, r1);
                    const float *ws = wg + 32 * j;
                    scale_add16(acc, 0, r0, ws, xdv);
                    tmem_wait_ld16(r1);
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&aempty[u]);
                    scale_add16(acc, 16, r1, ws, xdv);
                }
                if (*abort_flag) break;
            }
            if (*abort_flag) break;
            if (!row_ok) continue;
            float *dst = p.out + static_cast<size_t>(row) * p.ldo + col0;
            if (p.vec_ok && col0 + 32 <= p.N) {
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    float4 o = make_float4(acc[2 * i].x, acc[2 * i].y, acc[2 * i + 1].x, acc[2 * i + 1].y);
                    if (RESIDUAL) {
                        const float4 r = *reinterpret_cast<const float4 *>(dst + 4 * i);
                        o = make_float4(__fadd_rn(r.x, o.x), __fadd_rn(r.y, o.y), __fadd_rn(r.z, o.z),
                                        __fadd_rn(r.w, o.w));
                    }
                    *reinterpret_cast<float4 *>(dst + 4 * i) = o;
                }
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    if (col0 + i < p.N) {
                        const float v = (i & 1) ? acc[i >> 1].y : acc[i >> 1].x;
                        dst[i] = RESIDUAL ? __fadd_rn(dst[i], v) : v;
                    }
                }
            }
        }
        asm volatile("cp.async.wait_all;" ::: "memory");  // no copy outlives the CTA (abort path)
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem_base, Q_TMEM_COLS);
    }
}

}  // namespace

void launch_quantize_rows(const float *x, int ldx, int M, int K, int kp, int8_t *q, float *d, cudaStream_t s) {
    if (M <= 0) return;
    const long warps = static_cast<long>(M) * (kp / 32);
    quantize_rows_kernel<<<static_cast<unsigned>((warps + 7) / 8), 256, 0, s>>>(x, ldx, M, K, kp, q, d);
    HK_LAUNCH_CHECK();
}

void launch_transpose_scales(const float *in, int rows, int nb, float *out, cudaStream_t s) {
    const long n = static_cast<long>(rows) * nb;
    if (n <= 0) return;
    transpose_scales_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(in, rows, nb, out);
    HK_LAUNCH_CHECK();
}

void gemm_q8(const int8_t *xq, const float *xd, const int8_t *wq, const float *wd, int M, int N, int kp, float *out,
             int ldo, bool residual, cudaStream_t s, int num_sms, uint32_t *err) {
    if (M <= 0 || N <= 0) return;
    if (kp <= 0 || kp % 32 != 0) throw CudaError("packed GEMM: kp must be a positive multiple of 32");
    static SmemOptIn opt_true, opt_false;
    if (residual)
        opt_true.ensure(gemm_q8_tc_kernel<true>, Q_SMEM_BYTES);
    else
        opt_false.ensure(gemm_q8_tc_kernel<false>, Q_SMEM_BYTES);
    // Row strides of kp bytes (a multiple of 32) meet TMA's 16-byte rule.
    const CUtensorMap tx = tensor_map_u8(xq, M, kp, kp, 128, QBM);
    const CUtensorMap tw = tensor_map_u8(wq, N, kp, kp, 128, QBN);
    Q8Params p;
    p.M = M;
    p.N = N;
    p.nb = kp / 32;
    p.m_tiles = (M + QBM - 1) / QBM;
    p.n_tiles = (N + QBN - 1) / QBN;
    p.n_fast = p.n_tiles <= 8 ? 1 : 0;
    p.xd = xd;
    p.wd = wd;
    p.out = out;
    p.ldo = ldo;
    p.vec_ok = ((reinterpret_cast<uintptr_t>(out) & 15) == 0) && (ldo % 4 == 0);
    p.err = err;
    const int tiles = p.m_tiles * p.n_tiles;
    const int grid = tiles < num_sms ? tiles : num_sms;
    if (residual)
        gemm_q8_tc_kernel<true><<<grid, Q_THREADS, Q_SMEM_BYTES, s>>>(tx, tw, p);
    else
        gemm_q8_tc_kernel<false><<<grid, Q_THREADS, Q_SMEM_BYTES, s>>>(tx, tw, p);
    HK_LAUNCH_CHECK();
}

}  // namespace hk
