// Chunked gated delta rule on the 5th-generation tensor cores (tcgen05), for
// 128-wide key/value heads (qwen3_5.rs:950-987, chunk-reassociated).
//
// Per chunk of C = 64 tokens (G = in-chunk inclusive cumsum of g, gam = e^G,
// S = the state entering the chunk, all identities exact):
//     A[t,s] = b_t e^{G_t-G_s} (k_t.k_s) (s<t),   T = (I + A)^-1
//     D = T diag(b) V - T diag(b gam) K S         (the chunk's delta rows)
//     O = diag(gam) Q S + Mq D,  Mq[t,s] = e^{G_t-G_s} (q_t.k_s) (s<=t)
//     S' = gam_C S + (diag(e^{G_C-G_s}) K)^T D
// Every product is computed transposed so its M dimension is the 128-wide
// head dimension: U^T = V^T (T diag b)^T, W^T = K^T (T diag(b gam))^T,
// D^T = U^T - S^T W^T, O^T = S^T Q^T + D^T Mq^T, S'^T = gam_C S^T + D^T Kdec.
// All of them are single-CTA tcgen05.mma (M=128, N=64 or 128, K=16 steps,
// fp16 operands, fp32 accumulation) issued by one thread; the state S^T and
// the D/U/W/O accumulators live in tensor memory (384 of 512 columns), so the
// fp32 state never leaves the SM.
//
// Operands are written once, by the threads that hold them, in their natural
// row-major order into 128B-swizzled shared-memory tiles; products that need
// a transposed operand read the same tile as MN-major (V, K and Kdec are
// stored [token][dim] and serve as the M or N side of U^T, W^T and S'^T).
// Operands whose fp16 rounding moves the output (q, k, v, D, Mq) are split
// into hi + lo halves and multiplied twice; S^T, W^T, T and the decayed keys
// are single fp16.
//
// T = (I + A)^-1 comes from fp32 block forward substitution on the CTA's
// threads: the four 16x16 diagonal blocks by substitution, then three levels
// T_IJ = -T_II sum_K A_IK T_KJ. T's strictly lower part is kept transposed in
// the unused upper triangle of the A buffer (T[t][s] at A[s][t]).
//
// One CTA (16 warps) per (row, value head); rows are taken longest first.
// Warp w reads TMEM lanes 32*(w%4).. and takes column slice w/4 of each
// accumulator.
// The next chunk's q/k/v/g/b are loaded into registers while the current
// chunk computes. All mbarrier waits are bounded: on a timeout the kernel
// records an error bit, lets the MMAs it issued finish, frees its tensor
// memory and returns.
#include <math.h>

#include "common.cuh"
#include "layers.cuh"
#include "sm100.cuh"

namespace hk {
namespace {

using namespace sm100;

constexpr int C = 64, D = 128, THREADS = 512;
// Tensor-memory columns.
constexpr uint32_t TM_S = 0, TM_D1 = 128, TM_O = 192, TM_U = 256, TM_W = 320, TM_COLS = 512;
// Shared-memory operand tiles (byte offsets; every tile 1024-aligned).
constexpr int XK_H = 0;       // [k rows 0..63 ; q rows 64..127] x 128 dims, hi (K-major, 2 K-tiles of 128 rows)
constexpr int XK_L = 32768;   //                                           lo
constexpr int ST = 65536;     // S^T [128 dv][128 dk] (K-major, 2 K-tiles)
constexpr int V_H = 98304;    // v [64 s][128 dv] hi (2 tiles of 64 rows); later W^T [128 dk][64 t]
constexpr int V_L = 114688;   //                  lo
constexpr int KDEC = 131072;  // e^{G_C-G_s} k [64 s][128 dk]
constexpr int TB = 147456;    // T diag(b) [64 t][64 s] (K-major)
constexpr int TBG = 155648;   // T diag(b gam)
constexpr int DT_H = 163840;  // D^T [128 dv][64 s] hi (the fp32 A/T buffer and scratch alias DT_H/DT_L first)
constexpr int DT_L = 180224;  //                     lo
constexpr int MQ_H = 196608;  // Mq [64 t][64 s] hi
constexpr int MQ_L = 204800;  //                 lo
constexpr int TILES = 212992;
constexpr int LA = 68;                     // fp32 A/T row stride (16-byte aligned rows)
constexpr int LX = 20;                     // merge scratch row stride
constexpr int SCRATCH = DT_H + C * LA * 4; // X [3][16][LX] then Td [4][16][16] fp32, inside DT_L
constexpr int SMALL = (4 * C + 4 * C + 2 * C) * 4 + 8 * 8 + 16;  // G, gam, beta, dec | red[4][64] | sg | mbarriers, tmem
constexpr int SMEM_BYTES = TILES + SMALL + 1024;
static_assert(SCRATCH + (3 * 16 * LX + 4 * 256) * 4 <= MQ_H, "merge scratch overlaps Mq");

struct TcArgs {
    const float *q, *k, *v, *g, *beta;  // q, k [n, nk, 128]; v [n, nv, 128]; g, beta [n, nv]
    const float *proj;                  // GATED: z at proj[t, zoff + h*128 + j]
    int ldp, zoff;
    const int32_t *cu_seqlens, *row_order;
    int n_rows, nk, nv;
    float *out;  // !GATED: o [n, nv, 128]
    const float *norm_w;
    float eps;
    __half *mix;  // GATED: rms(o) w silu(z) -> [n, ldmix] fp16
    int ldmix;
    uint32_t *err;
};

// Issue D (+)= A B^T over K = NK16 * 16 from descriptors of the first K-step.
// A K-major operand whose 64-wide K-tiles are KT bytes apart advances 32 bytes
// per step within a tile; an MN-major operand (KT = 0) advances 16 rows of 128
// bytes per step.
template <int NK16, int A_KT, int B_KT>
__device__ __forceinline__ void mma_chain(uint32_t d, uint64_t a0, uint64_t b0, uint32_t idesc, bool acc) {
#pragma unroll
    for (int ks = 0; ks < NK16; ++ks) {
        const uint32_t ao = A_KT ? (ks >> 2) * A_KT + (ks & 3) * 32 : ks * 2048;
        const uint32_t bo = B_KT ? (ks >> 2) * B_KT + (ks & 3) * 32 : ks * 2048;
        mma_f16(d, a0 + (ao >> 4), b0 + (bo >> 4), idesc, (acc || ks > 0) ? 1u : 0u);
    }
}

__device__ __forceinline__ uint2 pack4(float4 x) {
    const __half2 h0 = __floats2half2_rn(x.x, x.y), h1 = __floats2half2_rn(x.z, x.w);
    return make_uint2(*reinterpret_cast<const uint32_t *>(&h0), *reinterpret_cast<const uint32_t *>(&h1));
}
// 4 consecutive elements (8 bytes, within one 16-byte chunk) as hi and lo.
__device__ __forceinline__ void st4_split(uint8_t *hi, uint8_t *lo, uint32_t off, float4 x) {
    const __half2 h0 = __floats2half2_rn(x.x, x.y), h1 = __floats2half2_rn(x.z, x.w);
    const float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
    const __half2 l0 = __floats2half2_rn(x.x - f0.x, x.y - f0.y), l1 = __floats2half2_rn(x.z - f1.x, x.w - f1.y);
    *reinterpret_cast<uint2 *>(hi + off) =
        make_uint2(*reinterpret_cast<const uint32_t *>(&h0), *reinterpret_cast<const uint32_t *>(&h1));
    *reinterpret_cast<uint2 *>(lo + off) =
        make_uint2(*reinterpret_cast<const uint32_t *>(&l0), *reinterpret_cast<const uint32_t *>(&l1));
}
__device__ __forceinline__ float2 hi_lo(float v) {
    const float h = __half2float(__float2half_rn(v));
    return make_float2(h, v - h);
}
// 8 consecutive elements (one 16-byte chunk).
__device__ __forceinline__ void st8(uint8_t *base, uint32_t off, const float *v) {
    uint4 u;
    __half2 h;
    h = __floats2half2_rn(v[0], v[1]);
    u.x = *reinterpret_cast<const uint32_t *>(&h);
    h = __floats2half2_rn(v[2], v[3]);
    u.y = *reinterpret_cast<const uint32_t *>(&h);
    h = __floats2half2_rn(v[4], v[5]);
    u.z = *reinterpret_cast<const uint32_t *>(&h);
    h = __floats2half2_rn(v[6], v[7]);
    u.w = *reinterpret_cast<const uint32_t *>(&h);
    *reinterpret_cast<uint4 *>(base + off) = u;
}

template <bool GATED>
__global__ void __launch_bounds__(THREADS, 1) delta_tc_kernel(TcArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float *G = reinterpret_cast<float *>(sm + TILES);
    float *gam = G + C;
    float *beta = gam + C;
    float *dec = beta + C;
    float *red = dec + C;      // [4][64]
    float *sg = red + 4 * C;   // [2][64]: g / beta staging
    uint64_t *bars = reinterpret_cast<uint64_t *>(sg + 2 * C);
    uint64_t *bar_d1 = bars + 0, *bar_o = bars + 1, *bar_uw = bars + 2, *bar_d = bars + 3, *bar_os = bars + 4,
             *bar_drain = bars + 5;
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 8);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);
    float *sA = reinterpret_cast<float *>(sm + DT_H);    // [64][LA] fp32: A (lower), T transposed (upper)
    float *sX = reinterpret_cast<float *>(sm + SCRATCH); // [3][16][LX]
    float *sTd = sX + 3 * 16 * LX;                       // [4][16][16]

    const int row = a.row_order ? a.row_order[blockIdx.x] : blockIdx.x, h = blockIdx.y;
    const int start = a.cu_seqlens[row], end = a.cu_seqlens[row + 1];
    if (start >= end) return;
    const int kh = h / (a.nv / a.nk);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // TMEM lanes 32*quarter.. ; column slice `part` (16 of a 64-column
    // accumulator, 32 of the 128-column state).
    const int quarter = warp & 3, part = warp >> 2;
    const uint32_t s_base = smem_addr(sm);

    if (tid == 0) {
        for (int i = 0; i < 6; ++i) mbar_init(&bars[i], 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0) {
        tmem_alloc(tmem_holder, TM_COLS);
        tmem_relinquish();
    }
    for (int i = tid; i < 32768 / 16; i += THREADS) reinterpret_cast<uint4 *>(sm + ST)[i] = make_uint4(0, 0, 0, 0);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    {  // the state starts at zero
        float z[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) z[i] = 0.f;
        tmem_st32(lane_base + TM_S + part * 32, z);
    }

    // ---- register prefetch of a chunk's inputs: warp w holds rows w + 16i of
    // q, k and v (j = 4 * tensor + i), lane = 4-column group (coalesced rows).
    float4 pf[12];
    float pg = 0.f;
    float pz[16];
    const int c4 = lane * 4;
    auto load_qkvg = [&](int c0) {
        const int nn = min(C, end - c0);
#pragma unroll
        for (int j = 0; j < 12; ++j) {
            const int which = j >> 2, r = warp + 16 * (j & 3);
            float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
            if (r < nn) {
                const size_t t = static_cast<size_t>(c0 + r);
                const float *src = which == 0 ? a.q + (t * a.nk + kh) * D
                                              : which == 1 ? a.k + (t * a.nk + kh) * D : a.v + (t * a.nv + h) * D;
                x = *reinterpret_cast<const float4 *>(src + c4);
            }
            pf[j] = x;
        }
        pg = 0.f;
        if (tid < C) {
            if (tid < nn) pg = a.g[static_cast<size_t>(c0 + tid) * a.nv + h];
        } else if (tid < 2 * C) {
            if (tid - C < nn) pg = a.beta[static_cast<size_t>(c0 + tid - C) * a.nv + h];
        }
    };
    auto load_z = [&](int c0) {
        if (!GATED) return;
        const int nn = min(C, end - c0);
        const int dv = quarter * 32 + lane;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int t = part * 16 + i;
            pz[i] = t < nn ? a.proj[static_cast<size_t>(c0 + t) * a.ldp + a.zoff + h * D + dv] : 0.f;
        }
    };
    load_qkvg(start);
    load_z(start);
    const float nw = GATED ? a.norm_w[quarter * 32 + lane] : 0.f;

    auto wait = [&](uint64_t *bar, uint32_t parity) {
        if (!mbar_wait(bar, parity)) {
            set_error(a.err, kErrWaitTimeout);
            *abort_flag = 1;
        }
    };
    // 16 consecutive entries of a small per-token array (broadcast loads).
    auto ld16 = [&](const float *src, float (&dst)[16]) {
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
            const float4 x = reinterpret_cast<const float4 *>(src)[q4];
            dst[4 * q4] = x.x;
            dst[4 * q4 + 1] = x.y;
            dst[4 * q4 + 2] = x.z;
            dst[4 * q4 + 3] = x.w;
        }
    };

    uint32_t ph = 0;
    for (int c0 = start; c0 < end && !*abort_flag; c0 += C, ph ^= 1) {
        const int n = min(C, end - c0);
        // ---- L1: gates, their in-chunk cumulative sum and the end-of-chunk decays.
        if (tid < 2 * C) sg[tid] = pg;
        __syncthreads();
        if (warp == 0) {
            const float a0 = sg[2 * lane], a1 = sg[2 * lane + 1];
            float incl = a0 + a1;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float up = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += up;
            }
            const float excl = incl - (a0 + a1);
            const float g0 = excl + a0, g1 = excl + a0 + a1;
            const float gl = __shfl_sync(0xffffffffu, incl, 31);
            G[2 * lane] = g0;
            G[2 * lane + 1] = g1;
            gam[2 * lane] = expf(g0);
            gam[2 * lane + 1] = expf(g1);
            dec[2 * lane] = expf(gl - g0);
            dec[2 * lane + 1] = expf(gl - g1);
            beta[2 * lane] = sg[C + 2 * lane];
            beta[2 * lane + 1] = sg[C + 2 * lane + 1];
        }
        __syncthreads();
        // ---- L2: operands into the swizzled tiles, each row as it was loaded.
#pragma unroll
        for (int j = 0; j < 12; ++j) {
            const int which = j >> 2, r = warp + 16 * (j & 3);
            const float4 x = pf[j];
            if (which == 0) {
                st4_split(sm + XK_H, sm + XK_L, sw128_off(128, 64 + r, c4), x);
            } else if (which == 1) {
                st4_split(sm + XK_H, sm + XK_L, sw128_off(128, r, c4), x);
                const float dr = dec[r];
                *reinterpret_cast<uint2 *>(sm + KDEC + sw128_off(64, r, c4)) =
                    pack4(make_float4(dr * x.x, dr * x.y, dr * x.z, dr * x.w));
            } else {
                st4_split(sm + V_H, sm + V_L, sw128_off(64, r, c4), x);
            }
        }
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        // ---- M1: [K;Q] K^T (3 split products) -> D1;  M2: S^T Q^T (q hi + lo) -> O.
        if (tid == 0) {
            tc_fence_after();
            const uint64_t dk0 = desc_sw128(s_base, 16, 1024);
            constexpr uint32_t id64 = idesc_f16_f32(128, 64);
            mma_chain<8, 16384, 16384>(tmem + TM_D1, dk0 + (XK_H >> 4), dk0 + (XK_H >> 4), id64, false);
            mma_chain<8, 16384, 16384>(tmem + TM_D1, dk0 + (XK_H >> 4), dk0 + (XK_L >> 4), id64, true);
            mma_chain<8, 16384, 16384>(tmem + TM_D1, dk0 + (XK_L >> 4), dk0 + (XK_H >> 4), id64, true);
            mma_commit(bar_d1);
            mma_chain<8, 16384, 16384>(tmem + TM_O, dk0 + (ST >> 4), dk0 + ((XK_H + 8192) >> 4), id64, false);
            mma_chain<8, 16384, 16384>(tmem + TM_O, dk0 + (ST >> 4), dk0 + ((XK_L + 8192) >> 4), id64, true);
            mma_commit(bar_o);
        }
        // ---- E1: A (from K K^T) into fp32, Mq (from Q K^T) into split fp16 tiles.
        wait(bar_d1, ph);
        tc_fence_after();
        {
            float v[16], gs[16];
            tmem_ld16(lane_base + TM_D1 + part * 16, v);
            ld16(G + part * 16, gs);
            if (quarter < 2) {
                const int t = quarter * 32 + lane;
                const float bt = beta[t], gt = G[t];
                float4 *dst = reinterpret_cast<float4 *>(sA + t * LA + part * 16);
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    float e[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int i = 4 * c + u, s2 = part * 16 + i;
                        e[u] = s2 < t ? bt * expf(gt - gs[i]) * v[i] : 0.f;
                    }
                    dst[c] = make_float4(e[0], e[1], e[2], e[3]);
                }
            } else {
                const int t = (quarter - 2) * 32 + lane;
                const float gt = G[t];
#pragma unroll
                for (int c8 = 0; c8 < 2; ++c8) {
                    float hv[8], lv[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const int i = c8 * 8 + e, s2 = part * 16 + i;
                        const float mq = s2 <= t ? expf(gt - gs[i]) * v[i] : 0.f;
                        const float2 hl = hi_lo(mq);
                        hv[e] = hl.x;
                        lv[e] = hl.y;
                    }
                    const uint32_t off = sw128_off(64, t, part * 16 + c8 * 8);
                    st8(sm + MQ_H, off, hv);
                    st8(sm + MQ_L, off, lv);
                }
            }
        }
        tc_fence_before();
        __syncthreads();
        // ---- INV: T = (I + A)^-1. Diagonal 16x16 blocks by forward substitution
        // (thread = block, column): T_II[r][j] goes to A[16I + j][16I + r] and,
        // with zeros on and above the diagonal, to the row-major copy Td[I].
        if (tid < 64) {
            const int I = tid >> 4, j = tid & 15;
            float *Ab = sA + 16 * I * LA + 16 * I;
            float x[16];
#pragma unroll
            for (int r = 0; r < 16; ++r) {
                float acc0 = (r == j) ? 1.f : 0.f, acc1 = 0.f;
                const float4 *ar = reinterpret_cast<const float4 *>(Ab + r * LA);
#pragma unroll
                for (int q4 = 0; q4 < (r + 3) / 4; ++q4) {
                    const float4 av = ar[q4];
                    const float ae[4] = {av.x, av.y, av.z, av.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int s2 = 4 * q4 + e;
                        if (s2 < r) {
                            if (e & 1)
                                acc1 = fmaf(-ae[e], x[s2], acc1);
                            else
                                acc0 = fmaf(-ae[e], x[s2], acc0);
                        }
                    }
                }
                x[r] = acc0 + acc1;
            }
#pragma unroll
            for (int r = 0; r < 16; ++r) {
                if (r > j) Ab[j * LA + r] = x[r];
                sTd[(I * 16 + r) * 16 + j] = r > j ? x[r] : 0.f;
            }
        }
        __syncthreads();
        // Off-diagonal blocks, level I: X_IJ = sum_{K=J}^{I-1} A_IK T_KJ (kept
        // transposed, X[J][b][a]), then T_IJ = -T_II X_IJ, stored transposed at
        // A[16J + b][16I + a]. The two 8-warp groups take different J.
        {
            const int grp = tid >> 8, ra = (tid >> 4) & 15, cb = tid & 15;
#pragma unroll
            for (int I = 1; I < 4; ++I) {
#pragma unroll
                for (int J = 0; J < I; ++J) {
                    if (grp != (I == 3 ? (J == 0 ? 0 : 1) : (J & 1))) continue;
                    float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
                    for (int K = J; K < I; ++K) {
                        const float4 *arow = reinterpret_cast<const float4 *>(sA + (16 * I + ra) * LA + 16 * K);
                        const float4 *tcol = reinterpret_cast<const float4 *>(sA + (16 * J + cb) * LA + 16 * K);
#pragma unroll
                        for (int q4 = 0; q4 < 4; ++q4) {
                            const float4 av = arow[q4], tv4 = tcol[q4];
                            const float ae[4] = {av.x, av.y, av.z, av.w}, te[4] = {tv4.x, tv4.y, tv4.z, tv4.w};
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const int c = 4 * q4 + e;
                                // T_JJ is unit lower: its upper part in storage holds A_JJ.
                                const float tv = K == J ? (c == cb ? 1.f : (c > cb ? te[e] : 0.f)) : te[e];
                                if (e & 1)
                                    acc1 = fmaf(ae[e], tv, acc1);
                                else
                                    acc0 = fmaf(ae[e], tv, acc0);
                            }
                        }
                    }
                    sX[(J * 16 + cb) * LX + ra] = acc0 + acc1;
                }
                __syncthreads();
#pragma unroll
                for (int J = 0; J < I; ++J) {
                    if (grp != (I == 3 ? (J == 0 ? 0 : 1) : (J & 1))) continue;
                    const float4 *xr = reinterpret_cast<const float4 *>(sX + (J * 16 + cb) * LX);
                    const float4 *tr = reinterpret_cast<const float4 *>(sTd + (I * 16 + ra) * 16);
                    float acc0 = sX[(J * 16 + cb) * LX + ra], acc1 = 0.f;
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4) {
                        const float4 xv = xr[q4], tv = tr[q4];
                        acc0 = fmaf(tv.x, xv.x, acc0);
                        acc1 = fmaf(tv.y, xv.y, acc1);
                        acc0 = fmaf(tv.z, xv.z, acc0);
                        acc1 = fmaf(tv.w, xv.w, acc1);
                    }
                    sA[(16 * J + cb) * LA + 16 * I + ra] = -(acc0 + acc1);
                }
                __syncthreads();
            }
        }
        // T diag(b) and T diag(b gam) as fp16 K-major [t][s] tiles.
        {
            const int t = tid & 63, ch = tid >> 6;
            const float4 b0 = reinterpret_cast<const float4 *>(beta + 8 * ch)[0],
                         b1 = reinterpret_cast<const float4 *>(beta + 8 * ch)[1];
            const float4 g0 = reinterpret_cast<const float4 *>(gam + 8 * ch)[0],
                         g1 = reinterpret_cast<const float4 *>(gam + 8 * ch)[1];
            const float bs[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
            const float gs[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
            float vb[8], vg[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const int s2 = 8 * ch + e;
                const float tv = s2 < t ? sA[s2 * LA + t] : (s2 == t ? 1.f : 0.f);
                vb[e] = tv * bs[e];
                vg[e] = vb[e] * gs[e];
            }
            const uint32_t off = sw128_off(64, t, 8 * ch);
            st8(sm + TB, off, vb);
            st8(sm + TBG, off, vg);
        }
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        // ---- M3: U^T = V^T (T diag b)^T (v hi + lo), W^T = K^T (T diag(b gam))^T.
        if (tid == 0) {
            tc_fence_after();
            const uint64_t dk0 = desc_sw128(s_base, 16, 1024);
            const uint64_t dv0 = desc_sw128(s_base, 8192, 1024);    // V: 64-dim blocks 8192 bytes apart
            const uint64_t dx0 = desc_sw128(s_base, 16384, 1024);   // K inside [K;Q]: blocks 16384 apart
            constexpr uint32_t idu = idesc_f16_f32_mj(128, 64, true, false);
            mma_chain<4, 0, 16384>(tmem + TM_U, dv0 + (V_H >> 4), dk0 + (TB >> 4), idu, false);
            mma_chain<4, 0, 16384>(tmem + TM_U, dv0 + (V_L >> 4), dk0 + (TB >> 4), idu, true);
            mma_chain<4, 0, 16384>(tmem + TM_W, dx0 + (XK_H >> 4), dk0 + (TBG >> 4), idu, false);
            mma_commit(bar_uw);
        }
        if (c0 + C < end) load_qkvg(c0 + C);  // next chunk, in flight during the rest
        // ---- E2: W^T into a [dk][t] tile (over V hi); O columns scaled by gam.
        wait(bar_uw, ph);
        wait(bar_o, ph);
        tc_fence_after();
        {
            float v[16], gs[16];
            tmem_ld16(lane_base + TM_W + part * 16, v);
            const int dk = quarter * 32 + lane;
#pragma unroll
            for (int c8 = 0; c8 < 2; ++c8) st8(sm + V_H, sw128_off(128, dk, part * 16 + c8 * 8), v + c8 * 8);
            tmem_ld16(lane_base + TM_O + part * 16, v);
            ld16(gam + part * 16, gs);
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] *= gs[i];
            tmem_st16(lane_base + TM_O + part * 16, v);
        }
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        // ---- M4: D^T = U^T - S^T W^T.
        if (tid == 0) {
            tc_fence_after();
            const uint64_t dk0 = desc_sw128(s_base, 16, 1024);
            const uint64_t dw0 = desc_sw128(s_base, 16384, 1024);
            constexpr uint32_t idd = idesc_f16_f32_mj(128, 64, false, true, true);
            mma_chain<8, 16384, 0>(tmem + TM_U, dk0 + (ST >> 4), dw0 + (V_H >> 4), idd, true);
            mma_commit(bar_d);
        }
        // ---- E3: D^T into split fp16 tiles; the state scaled by gam_C.
        wait(bar_d, ph);
        tc_fence_after();
        {
            float v[16];
            tmem_ld16(lane_base + TM_U + part * 16, v);
            const int dv = quarter * 32 + lane;
#pragma unroll
            for (int c8 = 0; c8 < 2; ++c8) {
                float hv[8], lv[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const float2 hl = hi_lo(v[c8 * 8 + e]);
                    hv[e] = hl.x;
                    lv[e] = hl.y;
                }
                const uint32_t off = sw128_off(128, dv, part * 16 + c8 * 8);
                st8(sm + DT_H, off, hv);
                st8(sm + DT_L, off, lv);
            }
            const float gc = gam[C - 1];
            float w[32];
            tmem_ld32(lane_base + TM_S + part * 32, w);
#pragma unroll
            for (int i = 0; i < 32; ++i) w[i] *= gc;
            tmem_st32(lane_base + TM_S + part * 32, w);
        }
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        // ---- M5: O^T += D^T Mq^T (3 split products); S^T += D^T Kdec (D hi + lo).
        if (tid == 0) {
            tc_fence_after();
            const uint64_t dk0 = desc_sw128(s_base, 16, 1024);
            const uint64_t dv0 = desc_sw128(s_base, 8192, 1024);
            constexpr uint32_t id64 = idesc_f16_f32(128, 64);
            constexpr uint32_t ids = idesc_f16_f32_mj(128, 128, false, true);
            mma_chain<4, 16384, 8192>(tmem + TM_O, dk0 + (DT_H >> 4), dk0 + (MQ_H >> 4), id64, true);
            mma_chain<4, 16384, 8192>(tmem + TM_O, dk0 + (DT_H >> 4), dk0 + (MQ_L >> 4), id64, true);
            mma_chain<4, 16384, 8192>(tmem + TM_O, dk0 + (DT_L >> 4), dk0 + (MQ_H >> 4), id64, true);
            mma_chain<4, 16384, 0>(tmem + TM_S, dk0 + (DT_H >> 4), dv0 + (KDEC >> 4), ids, true);
            mma_chain<4, 16384, 0>(tmem + TM_S, dk0 + (DT_L >> 4), dv0 + (KDEC >> 4), ids, true);
            mma_commit(bar_os);
        }
        // ---- E4: output (o, or its gated RMSNorm) and the fp16 state copy for the next chunk.
        wait(bar_os, ph);
        tc_fence_after();
        {
            const int dv = quarter * 32 + lane;
            float v[16];
            tmem_ld16(lane_base + TM_O + part * 16, v);  // v[i] = O[t = 16*part + i][dv]
            if (GATED) {
                // Sum of squares over this quarter's 32 value columns for each of the
                // 16 rows, by a transposing butterfly (lane l ends with row l & 15).
                float sq[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) sq[i] = v[i] * v[i];
#pragma unroll
                for (int off = 8; off >= 1; off >>= 1) {
                    const bool upper = (lane & off) != 0;
#pragma unroll
                    for (int i = 0; i < off; ++i) {
                        const float send = upper ? sq[i] : sq[i + off];
                        const float got = __shfl_xor_sync(0xffffffffu, send, off);
                        sq[i] = (upper ? sq[i + off] : sq[i]) + got;
                    }
                }
                sq[0] += __shfl_xor_sync(0xffffffffu, sq[0], 16);
                if (lane < 16) red[quarter * C + part * 16 + lane] = sq[0];
                __syncthreads();
                // Lane l forms the denominator of row 16*part + (l & 15); rows are then
                // broadcast across the warp.
                const int tl = part * 16 + (lane & 15);
                const float ss = red[tl] + red[C + tl] + red[2 * C + tl] + red[3 * C + tl];
                const float denom_l = sqrtf(ss / static_cast<float>(D) + a.eps);
                __half *mrow = a.mix + static_cast<size_t>(c0 + part * 16) * a.ldmix + h * D + dv;
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float denom = __shfl_sync(0xffffffffu, denom_l, i);
                    const float y = ((v[i] / denom) * nw) * silu_f(pz[i]);
                    if (part * 16 + i < n) mrow[static_cast<size_t>(i) * a.ldmix] = __float2half_rn(y);
                }
            } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int t = part * 16 + i;
                    if (t < n) a.out[(static_cast<size_t>(c0 + t) * a.nv + h) * D + dv] = v[i];
                }
            }
            float w[32];
            tmem_ld32(lane_base + TM_S + part * 32, w);
#pragma unroll
            for (int c8 = 0; c8 < 4; ++c8) st8(sm + ST, sw128_off(128, dv, part * 32 + c8 * 8), w + c8 * 8);
        }
        if (c0 + C < end) load_z(c0 + C);
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
    }

    // ---- teardown (also the timeout path: let issued MMAs finish first)
    if (*abort_flag && tid == 0) {
        mma_commit(bar_drain);
        (void)mbar_wait(bar_drain, 0);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, TM_COLS);
    }
}

template <bool GATED>
void launch_tc(const TcArgs &a, cudaStream_t s) {
    static SmemOptIn opt_in;
    opt_in.ensure(delta_tc_kernel<GATED>, SMEM_BYTES);
    dim3 grid(a.n_rows, a.nv);
    delta_tc_kernel<GATED><<<grid, THREADS, SMEM_BYTES, s>>>(a);
    HK_LAUNCH_CHECK();
}

TcArgs from_rec(const DeltaRecArgs &r) {
    TcArgs a{};
    a.q = r.q;
    a.k = r.k;
    a.v = r.v;
    a.g = r.g;
    a.beta = r.beta;
    a.cu_seqlens = r.cu_seqlens;
    a.row_order = r.row_order;
    a.n_rows = r.n_rows;
    a.nk = r.nk;
    a.nv = r.nv;
    a.out = r.out;
    a.err = r.err;
    return a;
}

}  // namespace

bool delta_tc_supported(const DeltaRecArgs &r) { return r.dk == D && r.dv == D && (r.nv % r.nk) == 0; }

void launch_delta_tc(const DeltaRecArgs &r, cudaStream_t s) {
    if (r.n_rows <= 0) return;
    launch_tc<false>(from_rec(r), s);
}

void launch_delta_tc_gated(const DeltaRecArgs &r, const float *proj, int ldp, int zoff, const float *norm_w, float eps,
                           __half *mix, int ldmix, cudaStream_t s) {
    if (r.n_rows <= 0) return;
    TcArgs a = from_rec(r);
    a.proj = proj;
    a.ldp = ldp;
    a.zoff = zoff;
    a.norm_w = norm_w;
    a.eps = eps;
    a.mix = mix;
    a.ldmix = ldmix;
    launch_tc<true>(a, s);
}

}  // namespace hk
