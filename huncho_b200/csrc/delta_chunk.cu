// Chunked gated delta rule on tensor cores (WY form), for 128-wide heads.
//
// The per-token recurrence of qwen3_5.rs:950-987,
//     S_t = e^{g_t} S_{t-1} + k_t d_t^T,  d_t = b_t (v_t - (e^{g_t} S_{t-1})^T k_t),
//     o_t = S_t^T q_t,
// is re-associated over chunks of C tokens. With G = the in-chunk inclusive
// cumsum of g, gam_t = e^{G_t}, and S0 the state entering the chunk:
//     A[t,s] = b_t e^{G_t - G_s} (k_t . k_s)      (s < t)
//     T      = (I + A)^{-1}                       (unit lower triangular)
//     U      = T diag(b) V,   W = T diag(b gam) K
//     D      = U - W S0                           (the chunk's d_t rows)
//     O      = diag(gam) Q S0 + Mq D,  Mq[t,s] = e^{G_t - G_s} (q_t . k_s)  (s <= t)
//     S_C    = gam_C S0 + (diag(e^{G_C - G_s}) K)^T D
// which is exact algebra; only the rounding differs from the per-token loop.
//
// One CTA of 8 warps owns one (row, value head) and walks its chunks in order,
// keeping the fp32 state S (128 x 128) in registers as the accumulator of the
// state update (warp w owns key rows 16w..16w+15). Products run on tensor
// cores (mma.sync m16n8k16, fp16 operands, fp32 accumulation); the operands
// whose rounding moves the calibrated probabilities (q, k, b*v, D and Mq) are
// split into fp16 hi + lo parts so each product carries ~22 bits, while S, W,
// T and the decayed keys use single fp16. T comes from fp32 forward
// substitution. Padding rows of a short last chunk are zero (g = 0, b = 0), so
// they change neither the outputs nor the carried state.
//
// The next chunk's inputs (q, k, v rows, g, beta, and z for the gated output)
// stream into shared memory with cp.async while the current chunk computes,
// so global latency stays off the serial chunk-to-chunk path. With GATED_OUT
// the gated RMSNorm rms(o) * w * silu(z) (qwen3_5.rs:193-201, 934-938) is
// applied to each chunk's output in the kernel and written as the fp16 input
// of out_proj, so o never leaves the SM.
#include <math.h>

#include "common.cuh"
#include "layers.cuh"
#include "mma16.cuh"

namespace hk {
namespace {

constexpr int C = 32;        // chunk length
constexpr int D = 128;       // key = value head width
constexpr int LDH = D + 8;   // padded fp16 row (conflict-free ldmatrix)
constexpr int LDC = C + 8;
constexpr int THREADS = 256;  // 8 warps
constexpr int WARPS = THREADS / 32;

struct Smem {
    __half S[D][LDH];       // fp16 copy of the state (B operand)
    __half Qh[C][LDH], Ql[C][LDH];  // q hi/lo; Qh later holds the decayed keys
    __half Kh[C][LDH], Kl[C][LDH];
    __half BK[C][LDH];      // b gam k, overwritten in place by -W
    __half Vh[C][LDH], Vl[C][LDH];  // b v hi/lo, later D hi/lo
    float A[C][C + 1];
    __half T[C][LDC];
    __half Mh[C][LDC], Ml[C][LDC];
    float G[C], gam[C], beta[C];
    float red[WARPS][C];  // per-warp partial sums of squares (gated norm)
    // cp.async staging of the next chunk's fp32 inputs
    float sq[C][D], sk[C][D], sv[C][D];
    float sz[C][D];  // z rows of the chunk whose gated output is pending
    float sg[C], sb[C];
};

struct ChunkArgs {
    // Inputs: q, k [n, nk, 128], v [n, nv, 128], g, beta [n, nv] (fp32).
    const float *q, *k, *v, *g, *beta;
    // GATED_OUT: z is read from the fp32 projection rows proj[t, zoff + h*128 + j].
    const float *proj;
    int ldp, zoff;
    const int32_t *cu_seqlens;
    const int32_t *row_order;  // CTA x handles row row_order[x] (longest rows first), or x
    int n_rows, nk, nv;
    float *out;           // !GATED_OUT: o [n, nv, 128] fp32
    const float *norm_w;  // GATED_OUT: gated-norm weight [128]
    float eps;
    __half *mix;  // GATED_OUT: out_proj input [n, ldmix]
    int ldmix;
    // Per-row addresses of the initial / final state [nv][128][128] fp32, or 0.
    const uint64_t *state_in, *state_out;
};


template <bool GATED_OUT>
__global__ void __launch_bounds__(THREADS, 1) delta_chunk_kernel(ChunkArgs a) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    Smem &sm = *reinterpret_cast<Smem *>(smem_raw);
    // Rows run longest first (row_order), so the grid's last wave is made of
    // the shortest rows.
    const int row = a.row_order ? a.row_order[blockIdx.x] : blockIdx.x, h = blockIdx.y;
    const int start = a.cu_seqlens[row], end = a.cu_seqlens[row + 1];
    if (start >= end) return;
    const int kh = h / (a.nv / a.nk);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g4 = lane >> 2, t4 = lane & 3;

    // Asynchronous loads of a chunk's inputs into the staging buffers; rows
    // past the row's end are zero-filled (so they carry g = 0, beta = 0).
    auto prefetch_qkv = [&](int c0) {
        const int nn = min(C, end - c0);
        for (int i = tid; i < 3 * C * (D / 4); i += THREADS) {
            const int which = i / (C * (D / 4)), rem = i % (C * (D / 4));
            const int r = rem / (D / 4), c = (rem % (D / 4)) * 4;
            const bool ok = r < nn;
            const size_t t = static_cast<size_t>(c0 + (ok ? r : 0));
            const float *src = which == 0 ? a.q + (t * a.nk + kh) * D + c
                                          : which == 1 ? a.k + (t * a.nk + kh) * D + c : a.v + (t * a.nv + h) * D + c;
            float *dst = which == 0 ? &sm.sq[r][c] : which == 1 ? &sm.sk[r][c] : &sm.sv[r][c];
            cp16(dst, src, ok);
        }
        if (tid < 2 * C) {
            const int r = tid % C;
            const bool ok = r < nn;
            const size_t t = static_cast<size_t>(c0 + (ok ? r : 0));
            if (tid < C)
                cp4(&sm.sg[r], a.g + t * a.nv + h, ok);
            else
                cp4(&sm.sb[r], a.beta + t * a.nv + h, ok);
        }
    };
    auto prefetch_z = [&](int c0) {
        if (!GATED_OUT) return;
        const int nn = min(C, end - c0);
        for (int i = tid; i < C * (D / 4); i += THREADS) {
            const int r = i / (D / 4), c = (i % (D / 4)) * 4;
            const bool ok = r < nn;
            const size_t t = static_cast<size_t>(c0 + (ok ? r : 0));
            cp16(&sm.sz[r][c], a.proj + t * a.ldp + a.zoff + h * D + c, ok);
        }
    };

    // State accumulator: key rows 16*warp + {g4, g4+8}, value cols 8*nt + 2*t4 + {0,1}.
    float S[16][4];
    const float *st_in = reinterpret_cast<const float *>(a.state_in ? a.state_in[row] : 0);
    if (st_in) {  // a continued row starts from its cached prefix's state
        const float *sh = st_in + static_cast<size_t>(h) * D * D;
#pragma unroll
        for (int nt = 0; nt < 16; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e)
                S[nt][e] = sh[(warp * 16 + g4 + (e >> 1) * 8) * D + nt * 8 + 2 * t4 + (e & 1)];
        // The fp16 copy from the fragments just loaded (as at the end of a chunk).
#pragma unroll
        for (int nt = 0; nt < 16; ++nt)
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                const int r = warp * 16 + g4 + hf * 8, c = nt * 8 + 2 * t4;
                *reinterpret_cast<__half2 *>(&sm.S[r][c]) = __floats2half2_rn(S[nt][2 * hf], S[nt][2 * hf + 1]);
            }
    } else {
#pragma unroll
        for (int nt = 0; nt < 16; ++nt) S[nt][0] = S[nt][1] = S[nt][2] = S[nt][3] = 0.f;
        for (int i = tid; i < D * LDH; i += THREADS) (&sm.S[0][0])[i] = __float2half_rn(0.f);
    }
    prefetch_qkv(start);
    prefetch_z(start);
    cp_commit();

    // This thread's gated-norm weights (columns nb + 8 nt + 2 t4 + {0, 1}).
    const int nb = warp * 16;
    float nwr[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
    if (GATED_OUT) {
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
            nwr[nt][0] = a.norm_w[nb + nt * 8 + 2 * t4];
            nwr[nt][1] = a.norm_w[nb + nt * 8 + 2 * t4 + 1];
        }
    }
    for (int c0 = start; c0 < end; c0 += C) {
        const int n = min(C, end - c0);
        cp_wait_all();
        __syncthreads();  // this chunk's inputs are in the staging buffers
        // ---- P0: gates. Every warp scans g in registers (lane = row; padding
        // rows carry g = 0, beta = 0); warp 0 also publishes G, gam, beta for the
        // later phases, which read them after the next barrier.
        float gv = sm.sg[lane];
        const float bv = sm.sb[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float up = __shfl_up_sync(0xffffffffu, gv, o);
            if (lane >= o) gv += up;
        }
        const float gamv = expf(gv);
        if (warp == 0) {
            sm.G[lane] = gv;
            sm.gam[lane] = gamv;
            sm.beta[lane] = bv;
        }
        // ---- P0b: operands from the staging buffers; warp w fills rows w, w+8, ...
#pragma unroll
        for (int r = warp; r < C; r += WARPS) {
            const float4 q4 = *reinterpret_cast<const float4 *>(&sm.sq[r][4 * lane]);
            const float4 k4 = *reinterpret_cast<const float4 *>(&sm.sk[r][4 * lane]);
            const float4 v4 = *reinterpret_cast<const float4 *>(&sm.sv[r][4 * lane]);
            const float qv[4] = {q4.x, q4.y, q4.z, q4.w}, kv[4] = {k4.x, k4.y, k4.z, k4.w};
            const float b = __shfl_sync(0xffffffffu, bv, r), bg = b * __shfl_sync(0xffffffffu, gamv, r);
            const float bvv[4] = {b * v4.x, b * v4.y, b * v4.z, b * v4.w};
            const float bkk[4] = {bg * kv[0], bg * kv[1], bg * kv[2], bg * kv[3]};
            split_store4(&sm.Qh[r][4 * lane], &sm.Ql[r][4 * lane], qv);
            split_store4(&sm.Kh[r][4 * lane], &sm.Kl[r][4 * lane], kv);
            split_store4(&sm.Vh[r][4 * lane], &sm.Vl[r][4 * lane], bvv);
            store4(&sm.BK[r][4 * lane], bkk);
        }
        __syncthreads();
        // The staging buffers are free again: fetch the next chunk's inputs.
        if (c0 + C < end) prefetch_qkv(c0 + C);
        cp_commit();
        // ---- P1: K K^T (warps 0-3) and Q K^T (warps 4-7); 16 rows x 16 cols per warp.
        {
            const bool kk = warp < 4;
            const int mt = (warp >> 1) & 1, n0 = (warp & 1) * 16;
            float acc[2][4];
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
#pragma unroll
            for (int k0 = 0; k0 < D; k0 += 16) {
                uint32_t ah[4], al[4], bh[4], bl[4];
                frag_a<LDH>(ah, kk ? sm.Kh : sm.Qh, mt * 16, k0, lane);
                frag_a<LDH>(al, kk ? sm.Kl : sm.Ql, mt * 16, k0, lane);
                frag_b_nk<LDH>(bh, sm.Kh, k0, n0, lane);
                frag_b_nk<LDH>(bl, sm.Kl, k0, n0, lane);
                mma(acc[0], ah, bh[0], bh[1]);
                mma(acc[1], ah, bh[2], bh[3]);
                mma(acc[0], ah, bl[0], bl[1]);
                mma(acc[1], ah, bl[2], bl[3]);
                mma(acc[0], al, bh[0], bh[1]);
                mma(acc[1], al, bh[2], bh[3]);
            }
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int t = mt * 16 + g4 + (e >> 1) * 8, s = n0 + nt * 8 + 2 * t4 + (e & 1);
                    const float dec = expf(sm.G[t] - sm.G[s]);
                    if (kk) {
                        sm.A[t][s] = s < t ? sm.beta[t] * dec * acc[nt][e] : 0.f;
                    } else {
                        const float mq = s <= t ? dec * acc[nt][e] : 0.f;
                        split_store(&sm.Mh[t][s], &sm.Ml[t][s], mq);
                    }
                }
        }
        __syncthreads();
        // ---- P2: T = (I + A)^{-1} by forward substitution (warp 0, lane = column).
        if (warp == 0) {
            float col[C];
#pragma unroll
            for (int t = 0; t < C; ++t) {
                float acc0 = (t == lane) ? 1.f : 0.f, acc1 = 0.f;
#pragma unroll
                for (int s = 0; s < t; ++s) {
                    if (s & 1)
                        acc1 = fmaf(-sm.A[t][s], col[s], acc1);
                    else
                        acc0 = fmaf(-sm.A[t][s], col[s], acc0);
                }
                col[t] = acc0 + acc1;
                sm.T[t][lane] = __float2half_rn(col[t]);
            }
        }
        __syncthreads();
        // ---- P3: U = T (b v) (hi+lo), W = T (b gam k); warp w owns cols nb = 16w..16w+15.
        float u[2][2][4];
        {
            float w[2][2][4];
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) u[mt][nt][e] = w[mt][nt][e] = 0.f;
#pragma unroll
            for (int k0 = 0; k0 < C; k0 += 16) {
                uint32_t vh[4], vl[4], bk[4];
                frag_b_kn<LDH>(vh, sm.Vh, k0, nb, lane);
                frag_b_kn<LDH>(vl, sm.Vl, k0, nb, lane);
                frag_b_kn<LDH>(bk, sm.BK, k0, nb, lane);
#pragma unroll
                for (int mt = 0; mt < 2; ++mt) {
                    uint32_t at[4];
                    frag_a<LDC>(at, sm.T, mt * 16, k0, lane);
                    mma(u[mt][0], at, vh[0], vh[1]);
                    mma(u[mt][1], at, vh[2], vh[3]);
                    mma(u[mt][0], at, vl[0], vl[1]);
                    mma(u[mt][1], at, vl[2], vl[3]);
                    mma(w[mt][0], at, bk[0], bk[1]);
                    mma(w[mt][1], at, bk[2], bk[3]);
                }
            }
            __syncwarp();
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                    for (int hf = 0; hf < 2; ++hf) {
                        const int t = mt * 16 + g4 + hf * 8, c = nb + nt * 8 + 2 * t4;
                        *reinterpret_cast<__half2 *>(&sm.BK[t][c]) =
                            __floats2half2_rn(-w[mt][nt][2 * hf], -w[mt][nt][2 * hf + 1]);
                    }
        }
        __syncthreads();
        // ---- P4: D = U + (-W) S0 and O = diag(gam) Q S0 (q hi+lo); warp w owns cols 16w..
        float o[2][2][4];
        {
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) o[mt][nt][e] = 0.f;
#pragma unroll 4
            for (int k0 = 0; k0 < D; k0 += 16) {
                uint32_t sb[4];
                frag_b_kn<LDH>(sb, sm.S, k0, nb, lane);
#pragma unroll
                for (int mt = 0; mt < 2; ++mt) {
                    uint32_t aw[4], qh[4], ql[4];
                    frag_a<LDH>(aw, sm.BK, mt * 16, k0, lane);
                    frag_a<LDH>(qh, sm.Qh, mt * 16, k0, lane);
                    frag_a<LDH>(ql, sm.Ql, mt * 16, k0, lane);
                    mma(u[mt][0], aw, sb[0], sb[1]);
                    mma(u[mt][1], aw, sb[2], sb[3]);
                    mma(o[mt][0], qh, sb[0], sb[1]);
                    mma(o[mt][1], qh, sb[2], sb[3]);
                    mma(o[mt][0], ql, sb[0], sb[1]);
                    mma(o[mt][1], ql, sb[2], sb[3]);
                }
            }
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) o[mt][nt][e] *= sm.gam[mt * 16 + g4 + (e >> 1) * 8];
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int t = mt * 16 + g4 + (e >> 1) * 8, c = nb + nt * 8 + 2 * t4 + (e & 1);
                        split_store(&sm.Vh[t][c], &sm.Vl[t][c], u[mt][nt][e]);
                    }
        }
        __syncthreads();
        // ---- P5: O += Mq D (3 split products); write O (or its gated norm); decayed keys.
        {
#pragma unroll
            for (int k0 = 0; k0 < C; k0 += 16) {
                uint32_t dh[4], dl[4];
                frag_b_kn<LDH>(dh, sm.Vh, k0, nb, lane);
                frag_b_kn<LDH>(dl, sm.Vl, k0, nb, lane);
#pragma unroll
                for (int mt = 0; mt < 2; ++mt) {
                    uint32_t mh[4], ml[4];
                    frag_a<LDC>(mh, sm.Mh, mt * 16, k0, lane);
                    frag_a<LDC>(ml, sm.Ml, mt * 16, k0, lane);
                    mma(o[mt][0], mh, dh[0], dh[1]);
                    mma(o[mt][1], mh, dh[2], dh[3]);
                    mma(o[mt][0], mh, dl[0], dl[1]);
                    mma(o[mt][1], mh, dl[2], dl[3]);
                    mma(o[mt][0], ml, dh[0], dh[1]);
                    mma(o[mt][1], ml, dh[2], dh[3]);
                }
            }
            if (!GATED_OUT) {
#pragma unroll
                for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                        for (int hf = 0; hf < 2; ++hf) {
                            const int t = mt * 16 + g4 + hf * 8;
                            if (t < n) {
                                const int c = nb + nt * 8 + 2 * t4;
                                *reinterpret_cast<float2 *>(a.out + (static_cast<size_t>(c0 + t) * a.nv + h) * D + c) =
                                    make_float2(o[mt][nt][2 * hf], o[mt][nt][2 * hf + 1]);
                            }
                        }
            } else {
                // Row sums of squares: this warp's 16 columns, reduced over the 4 lanes
                // of a row group, then over the 8 warps in a fixed order.
#pragma unroll
                for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                    for (int hf = 0; hf < 2; ++hf) {
                        float ss = 0.f;
#pragma unroll
                        for (int nt = 0; nt < 2; ++nt)
                            ss += o[mt][nt][2 * hf] * o[mt][nt][2 * hf] + o[mt][nt][2 * hf + 1] * o[mt][nt][2 * hf + 1];
                        ss += __shfl_xor_sync(0xffffffffu, ss, 1);
                        ss += __shfl_xor_sync(0xffffffffu, ss, 2);
                        if (t4 == 0) sm.red[warp][mt * 16 + g4 + hf * 8] = ss;
                    }
            }
            const float gl = sm.G[C - 1];
            for (int e = tid; e < C * (D / 4); e += THREADS) {
                const int r = e / (D / 4), c = (e % (D / 4)) * 4;
                float kd[4];
                const float dec = expf(gl - sm.G[r]);
#pragma unroll
                for (int u2 = 0; u2 < 4; ++u2)
                    kd[u2] = dec * (__half2float(sm.Kh[r][c + u2]) + __half2float(sm.Kl[r][c + u2]));
                store4(&sm.Qh[r][c], kd);
            }
        }
        __syncthreads();
        if (GATED_OUT) {
            // rms(o) * w * silu(z) -> fp16 out_proj input.
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    const int t = mt * 16 + g4 + hf * 8;
                    if (t >= n) continue;
                    float ss = 0.f;
#pragma unroll
                    for (int w8 = 0; w8 < WARPS; ++w8) ss += sm.red[w8][t];
                    const float denom = sqrtf(ss / static_cast<float>(D) + a.eps);
                    const size_t tok = static_cast<size_t>(c0 + t);
                    // fp16 output: the fast division and SiLU intrinsics are exact enough.
#pragma unroll
                    for (int nt = 0; nt < 2; ++nt) {
                        const int c = nb + nt * 8 + 2 * t4;
                        const float2 zz = *reinterpret_cast<const float2 *>(&sm.sz[t][c]);
                        const float y0 = (__fdividef(o[mt][nt][2 * hf], denom) * nwr[nt][0]) * silu_fast(zz.x);
                        const float y1 = (__fdividef(o[mt][nt][2 * hf + 1], denom) * nwr[nt][1]) * silu_fast(zz.y);
                        *reinterpret_cast<__half2 *>(a.mix + tok * a.ldmix + h * D + c) = __floats2half2_rn(y0, y1);
                    }
                }
        }
        if (GATED_OUT) {
            __syncthreads();  // every thread has read sz
            if (c0 + C < end) prefetch_z(c0 + C);
            cp_commit();
        }
        // ---- P6: S = gam_C S + Kdec^T D (D hi+lo); warp w owns key rows 16w..16w+15.
        {
            const float gc = sm.gam[C - 1];
#pragma unroll
            for (int nt = 0; nt < 16; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) S[nt][e] *= gc;
#pragma unroll
            for (int k0 = 0; k0 < C; k0 += 16) {
                uint32_t ak[4];
                frag_at<LDH>(ak, sm.Qh, warp * 16, k0, lane);
#pragma unroll
                for (int n0 = 0; n0 < D; n0 += 16) {
                    uint32_t dh[4], dl[4];
                    frag_b_kn<LDH>(dh, sm.Vh, k0, n0, lane);
                    frag_b_kn<LDH>(dl, sm.Vl, k0, n0, lane);
                    mma(S[n0 / 8], ak, dh[0], dh[1]);
                    mma(S[n0 / 8 + 1], ak, dh[2], dh[3]);
                    mma(S[n0 / 8], ak, dl[0], dl[1]);
                    mma(S[n0 / 8 + 1], ak, dl[2], dl[3]);
                }
            }
#pragma unroll
            for (int nt = 0; nt < 16; ++nt)
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    const int r = warp * 16 + g4 + hf * 8, c = nt * 8 + 2 * t4;
                    *reinterpret_cast<__half2 *>(&sm.S[r][c]) = __floats2half2_rn(S[nt][2 * hf], S[nt][2 * hf + 1]);
                }
        }
        __syncthreads();
    }
    if (a.state_out && a.state_out[row]) {
        float *sh = reinterpret_cast<float *>(a.state_out[row]) + static_cast<size_t>(h) * D * D;
#pragma unroll
        for (int nt = 0; nt < 16; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) sh[(warp * 16 + g4 + (e >> 1) * 8) * D + nt * 8 + 2 * t4 + (e & 1)] = S[nt][e];
    }
}

template <bool GO>
void launch_kernel(const ChunkArgs &a, cudaStream_t s) {
    const size_t smem = sizeof(Smem);
    static SmemOptIn opt_in;
    opt_in.ensure(delta_chunk_kernel<GO>, static_cast<int>(smem));
    dim3 grid(a.n_rows, a.nv);
    delta_chunk_kernel<GO><<<grid, THREADS, smem, s>>>(a);
    HK_LAUNCH_CHECK();
}

}  // namespace

bool delta_chunk_supported(const DeltaRecArgs &a) { return a.dk == D && a.dv == D && (a.nv % a.nk) == 0; }

void launch_delta_chunk(const DeltaRecArgs &r, cudaStream_t s) {
    if (r.n_rows <= 0) return;
    ChunkArgs a{};
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
    a.state_in = r.state_in;
    a.state_out = r.state_out;
    launch_kernel<false>(a, s);
}

void launch_delta_chunk_gated(const DeltaRecArgs &r, const float *proj, int ldp, int zoff, const float *norm_w,
                              float eps, __half *mix, int ldmix, cudaStream_t s) {
    if (r.n_rows <= 0) return;
    ChunkArgs a{};
    a.q = r.q;
    a.k = r.k;
    a.v = r.v;
    a.g = r.g;
    a.beta = r.beta;
    a.proj = proj;
    a.ldp = ldp;
    a.zoff = zoff;
    a.cu_seqlens = r.cu_seqlens;
    a.row_order = r.row_order;
    a.n_rows = r.n_rows;
    a.nk = r.nk;
    a.nv = r.nv;
    a.norm_w = norm_w;
    a.eps = eps;
    a.mix = mix;
    a.ldmix = ldmix;
    a.state_in = r.state_in;
    a.state_out = r.state_out;
    launch_kernel<true>(a, s);
}


}  // namespace hk
