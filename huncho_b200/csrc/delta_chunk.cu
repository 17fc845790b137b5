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
// One CTA of 4 warps owns one (row, value head) and walks its chunks in order,
// keeping the fp32 state S (128 x 128) in registers as the accumulator of the
// state update (warp w owns key rows 32w..32w+31). Products run on tensor
// cores (mma.sync m16n8k16, fp16 operands, fp32 accumulation); the operands
// whose rounding moves the calibrated probabilities (q, k, b*v, D and Mq) are
// split into fp16 hi + lo parts so each product carries ~22 bits, while S, W,
// T and the decayed keys use single fp16. T comes from fp32 forward
// substitution. Padding rows of a short last chunk are zero (g = 0, b = 0), so
// they change neither the outputs nor the carried state.
#include <math.h>

#include "common.cuh"
#include "layers.cuh"

namespace hk {
namespace {

constexpr int C = 32;        // chunk length
constexpr int D = 128;       // key = value head width
constexpr int LDH = D + 8;   // padded fp16 row (conflict-free ldmatrix)
constexpr int LDC = C + 8;
constexpr int THREADS = 128;

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
};

__device__ __forceinline__ uint32_t sa(const void *p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(sa(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(sa(p)));
}
__device__ __forceinline__ void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// A fragment (16 x 16, row-major source [row][col]) at (r0, c0).
template <int LD>
__device__ __forceinline__ void frag_a(uint32_t (&r)[4], const __half (*m)[LD], int r0, int c0, int lane) {
    const int j = lane >> 3, i = lane & 7;
    ldsm_x4(r, &m[r0 + i + (j & 1) * 8][c0 + (j >> 1) * 8]);
}
// A fragment of the TRANSPOSE of a row-major source: A[m][k] = src[k][m], at (m0, k0).
template <int LD>
__device__ __forceinline__ void frag_at(uint32_t (&r)[4], const __half (*m)[LD], int m0, int k0, int lane) {
    const int j = lane >> 3, i = lane & 7;
    ldsm_x4_t(r, &m[k0 + i + (j >> 1) * 8][m0 + (j & 1) * 8]);
}
// Two B fragments (k16 x n8, n-tiles n0 and n0+8) with B[k][n] = src[n][k] (src row-major by n).
template <int LD>
__device__ __forceinline__ void frag_b_nk(uint32_t (&r)[4], const __half (*m)[LD], int k0, int n0, int lane) {
    const int j = lane >> 3, i = lane & 7;
    ldsm_x4(r, &m[n0 + i + (j >> 1) * 8][k0 + (j & 1) * 8]);
}
// Two B fragments with B[k][n] = src[k][n] (src row-major by k).
template <int LD>
__device__ __forceinline__ void frag_b_kn(uint32_t (&r)[4], const __half (*m)[LD], int k0, int n0, int lane) {
    const int j = lane >> 3, i = lane & 7;
    ldsm_x4_t(r, &m[k0 + i + (j & 1) * 8][n0 + (j >> 1) * 8]);
}

__device__ __forceinline__ void split_store(__half *hi, __half *lo, float v) {
    const __half h = __float2half_rn(v);
    *hi = h;
    *lo = __float2half_rn(v - __half2float(h));
}

__global__ void __launch_bounds__(THREADS, 2) delta_chunk_kernel(DeltaRecArgs a) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    Smem &sm = *reinterpret_cast<Smem *>(smem_raw);
    const int row = blockIdx.x, h = blockIdx.y;
    const int start = a.cu_seqlens[row], end = a.cu_seqlens[row + 1];
    if (start >= end) return;
    const int kh = h / (a.nv / a.nk);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g4 = lane >> 2, t4 = lane & 3;

    // State accumulator: key rows 32*warp + 16*mt + {g4, g4+8}, value cols 8*nt + 2*t4 + {0,1}.
    float S[2][16][4];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < 16; ++nt) S[mt][nt][0] = S[mt][nt][1] = S[mt][nt][2] = S[mt][nt][3] = 0.f;
    for (int i = tid; i < D * LDH; i += THREADS) (&sm.S[0][0])[i] = __float2half_rn(0.f);

    for (int c0 = start; c0 < end; c0 += C) {
        const int n = min(C, end - c0);
        // ---- P0: gates. Warp 0 scans g; padding rows get g = 0, b = 0.
        if (warp == 0) {
            const int t = c0 + lane;
            float gv = lane < n ? a.g[static_cast<size_t>(t) * a.nv + h] : 0.f;
            const float bv = lane < n ? a.beta[static_cast<size_t>(t) * a.nv + h] : 0.f;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float up = __shfl_up_sync(0xffffffffu, gv, o);
                if (lane >= o) gv += up;
            }
            sm.G[lane] = gv;
            sm.gam[lane] = expf(gv);
            sm.beta[lane] = bv;
        }
        __syncthreads();
        // ---- P0b: operands. 32 rows x 128 cols of q, k, v; 4 columns per thread step.
        for (int e = tid; e < C * (D / 4); e += THREADS) {
            const int r = e / (D / 4), c = (e % (D / 4)) * 4;
            float4 q4 = make_float4(0.f, 0.f, 0.f, 0.f), k4 = q4, v4 = q4;
            if (r < n) {
                const size_t t = static_cast<size_t>(c0 + r);
                q4 = *reinterpret_cast<const float4 *>(a.q + (t * a.nk + kh) * D + c);
                k4 = *reinterpret_cast<const float4 *>(a.k + (t * a.nk + kh) * D + c);
                v4 = *reinterpret_cast<const float4 *>(a.v + (t * a.nv + h) * D + c);
            }
            const float b = sm.beta[r], bg = sm.beta[r] * sm.gam[r];
            const float qv[4] = {q4.x, q4.y, q4.z, q4.w}, kv[4] = {k4.x, k4.y, k4.z, k4.w},
                        vv[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                split_store(&sm.Qh[r][c + u], &sm.Ql[r][c + u], qv[u]);
                split_store(&sm.Kh[r][c + u], &sm.Kl[r][c + u], kv[u]);
                split_store(&sm.Vh[r][c + u], &sm.Vl[r][c + u], b * vv[u]);
                sm.BK[r][c + u] = __float2half_rn(bg * kv[u]);
            }
        }
        __syncthreads();
        // ---- P1: K K^T (warps 0,1) and Q K^T (warps 2,3), rows 16*(warp&1).., all 32 cols.
        {
            const int mt = warp & 1;
            const bool kk = warp < 2;
            float acc[4][4];
#pragma unroll
            for (int nt = 0; nt < 4; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
#pragma unroll
            for (int k0 = 0; k0 < D; k0 += 16) {
                uint32_t ah[4], al[4];
                frag_a<LDH>(ah, kk ? sm.Kh : sm.Qh, mt * 16, k0, lane);
                frag_a<LDH>(al, kk ? sm.Kl : sm.Ql, mt * 16, k0, lane);
#pragma unroll
                for (int n0 = 0; n0 < C; n0 += 16) {
                    uint32_t bh[4], bl[4];
                    frag_b_nk<LDH>(bh, sm.Kh, k0, n0, lane);
                    frag_b_nk<LDH>(bl, sm.Kl, k0, n0, lane);
                    mma(acc[n0 / 8], ah, bh[0], bh[1]);
                    mma(acc[n0 / 8 + 1], ah, bh[2], bh[3]);
                    mma(acc[n0 / 8], ah, bl[0], bl[1]);
                    mma(acc[n0 / 8 + 1], ah, bl[2], bl[3]);
                    mma(acc[n0 / 8], al, bh[0], bh[1]);
                    mma(acc[n0 / 8 + 1], al, bh[2], bh[3]);
                }
            }
#pragma unroll
            for (int nt = 0; nt < 4; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int t = mt * 16 + g4 + (e >> 1) * 8, s = nt * 8 + 2 * t4 + (e & 1);
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
        // ---- P3: U = T (b v) (hi+lo) and W = T (b gam k); warp w owns value/key cols 32w..32w+31.
        float u[2][4][4];
        {
            const int nb = warp * 32;
            float w[2][4][4];
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int nt = 0; nt < 4; ++nt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) u[mt][nt][e] = w[mt][nt][e] = 0.f;
#pragma unroll
            for (int k0 = 0; k0 < C; k0 += 16) {
#pragma unroll
                for (int mt = 0; mt < 2; ++mt) {
                    uint32_t at[4];
                    frag_a<LDC>(at, sm.T, mt * 16, k0, lane);
#pragma unroll
                    for (int n0 = 0; n0 < 32; n0 += 16) {
                        uint32_t vh[4], vl[4], bk[4];
                        frag_b_kn<LDH>(vh, sm.Vh, k0, nb + n0, lane);
                        frag_b_kn<LDH>(vl, sm.Vl, k0, nb + n0, lane);
                        frag_b_kn<LDH>(bk, sm.BK, k0, nb + n0, lane);
                        mma(u[mt][n0 / 8], at, vh[0], vh[1]);
                        mma(u[mt][n0 / 8 + 1], at, vh[2], vh[3]);
                        mma(u[mt][n0 / 8], at, vl[0], vl[1]);
                        mma(u[mt][n0 / 8 + 1], at, vl[2], vl[3]);
                        mma(w[mt][n0 / 8], at, bk[0], bk[1]);
                        mma(w[mt][n0 / 8 + 1], at, bk[2], bk[3]);
                    }
                }
            }
            __syncwarp();
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int nt = 0; nt < 4; ++nt)
#pragma unroll
                    for (int hf = 0; hf < 2; ++hf) {
                        const int t = mt * 16 + g4 + hf * 8, c = nb + nt * 8 + 2 * t4;
                        *reinterpret_cast<__half2 *>(&sm.BK[t][c]) =
                            __floats2half2_rn(-w[mt][nt][2 * hf], -w[mt][nt][2 * hf + 1]);
                    }
        }
        __syncthreads();
        // ---- P4: D = U + (-W) S0 and O = diag(gam) Q S0 (q hi+lo); warp w owns value cols 32w..
        float o[2][4][4];
        {
            const int nb = warp * 32;
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int nt = 0; nt < 4; ++nt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) o[mt][nt][e] = 0.f;
#pragma unroll 2
            for (int k0 = 0; k0 < D; k0 += 16) {
                uint32_t sb[2][4];
                frag_b_kn<LDH>(sb[0], sm.S, k0, nb, lane);
                frag_b_kn<LDH>(sb[1], sm.S, k0, nb + 16, lane);
#pragma unroll
                for (int mt = 0; mt < 2; ++mt) {
                    uint32_t aw[4], qh[4], ql[4];
                    frag_a<LDH>(aw, sm.BK, mt * 16, k0, lane);
                    frag_a<LDH>(qh, sm.Qh, mt * 16, k0, lane);
                    frag_a<LDH>(ql, sm.Ql, mt * 16, k0, lane);
#pragma unroll
                    for (int j = 0; j < 2; ++j) {
                        mma(u[mt][2 * j], aw, sb[j][0], sb[j][1]);
                        mma(u[mt][2 * j + 1], aw, sb[j][2], sb[j][3]);
                        mma(o[mt][2 * j], qh, sb[j][0], sb[j][1]);
                        mma(o[mt][2 * j + 1], qh, sb[j][2], sb[j][3]);
                        mma(o[mt][2 * j], ql, sb[j][0], sb[j][1]);
                        mma(o[mt][2 * j + 1], ql, sb[j][2], sb[j][3]);
                    }
                }
            }
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int nt = 0; nt < 4; ++nt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int t = mt * 16 + g4 + (e >> 1) * 8;
                        o[mt][nt][e] *= sm.gam[t];
                    }
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int nt = 0; nt < 4; ++nt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int t = mt * 16 + g4 + (e >> 1) * 8, c = nb + nt * 8 + 2 * t4 + (e & 1);
                        split_store(&sm.Vh[t][c], &sm.Vl[t][c], u[mt][nt][e]);
                    }
        }
        __syncthreads();
        // ---- P5: O += Mq D (3 split products), store O; decayed keys into Qh.
        {
            const int nb = warp * 32;
#pragma unroll
            for (int k0 = 0; k0 < C; k0 += 16) {
#pragma unroll
                for (int mt = 0; mt < 2; ++mt) {
                    uint32_t mh[4], ml[4];
                    frag_a<LDC>(mh, sm.Mh, mt * 16, k0, lane);
                    frag_a<LDC>(ml, sm.Ml, mt * 16, k0, lane);
#pragma unroll
                    for (int n0 = 0; n0 < 32; n0 += 16) {
                        uint32_t dh[4], dl[4];
                        frag_b_kn<LDH>(dh, sm.Vh, k0, nb + n0, lane);
                        frag_b_kn<LDH>(dl, sm.Vl, k0, nb + n0, lane);
                        mma(o[mt][n0 / 8], mh, dh[0], dh[1]);
                        mma(o[mt][n0 / 8 + 1], mh, dh[2], dh[3]);
                        mma(o[mt][n0 / 8], mh, dl[0], dl[1]);
                        mma(o[mt][n0 / 8 + 1], mh, dl[2], dl[3]);
                        mma(o[mt][n0 / 8], ml, dh[0], dh[1]);
                        mma(o[mt][n0 / 8 + 1], ml, dh[2], dh[3]);
                    }
                }
            }
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int nt = 0; nt < 4; ++nt)
#pragma unroll
                    for (int hf = 0; hf < 2; ++hf) {
                        const int t = mt * 16 + g4 + hf * 8;
                        if (t < n) {
                            const int c = nb + nt * 8 + 2 * t4;
                            *reinterpret_cast<float2 *>(a.out + (static_cast<size_t>(c0 + t) * a.nv + h) * D + c) =
                                make_float2(o[mt][nt][2 * hf], o[mt][nt][2 * hf + 1]);
                        }
                    }
            const float gl = sm.G[C - 1];
            for (int e = tid; e < C * D; e += THREADS) {
                const int r = e / D, c = e % D;
                const float kv = __half2float(sm.Kh[r][c]) + __half2float(sm.Kl[r][c]);
                sm.Qh[r][c] = __float2half_rn(expf(gl - sm.G[r]) * kv);
            }
        }
        __syncthreads();
        // ---- P6: S = gam_C S + Kdec^T D (D hi+lo); warp w owns key rows 32w..32w+31.
        {
            const float gc = sm.gam[C - 1];
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int nt = 0; nt < 16; ++nt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) S[mt][nt][e] *= gc;
#pragma unroll
            for (int k0 = 0; k0 < C; k0 += 16) {
                uint32_t ak[2][4];
                frag_at<LDH>(ak[0], sm.Qh, warp * 32, k0, lane);
                frag_at<LDH>(ak[1], sm.Qh, warp * 32 + 16, k0, lane);
#pragma unroll
                for (int n0 = 0; n0 < D; n0 += 16) {
                    uint32_t dh[4], dl[4];
                    frag_b_kn<LDH>(dh, sm.Vh, k0, n0, lane);
                    frag_b_kn<LDH>(dl, sm.Vl, k0, n0, lane);
#pragma unroll
                    for (int mt = 0; mt < 2; ++mt) {
                        mma(S[mt][n0 / 8], ak[mt], dh[0], dh[1]);
                        mma(S[mt][n0 / 8 + 1], ak[mt], dh[2], dh[3]);
                        mma(S[mt][n0 / 8], ak[mt], dl[0], dl[1]);
                        mma(S[mt][n0 / 8 + 1], ak[mt], dl[2], dl[3]);
                    }
                }
            }
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int nt = 0; nt < 16; ++nt)
#pragma unroll
                    for (int hf = 0; hf < 2; ++hf) {
                        const int r = warp * 32 + mt * 16 + g4 + hf * 8, c = nt * 8 + 2 * t4;
                        *reinterpret_cast<__half2 *>(&sm.S[r][c]) =
                            __floats2half2_rn(S[mt][nt][2 * hf], S[mt][nt][2 * hf + 1]);
                    }
        }
        __syncthreads();
    }
}

}  // namespace

bool delta_chunk_supported(const DeltaRecArgs &a) { return a.dk == D && a.dv == D && (a.nv % a.nk) == 0; }

void launch_delta_chunk(const DeltaRecArgs &a, cudaStream_t s) {
    if (a.n_rows <= 0) return;
    const size_t smem = sizeof(Smem);
    static bool set[64] = {};
    int dev = 0;
    HK_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64 || !set[dev]) {
        HK_CUDA(cudaFuncSetAttribute(delta_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(smem)));
        if (dev >= 0 && dev < 64) set[dev] = true;
    }
    dim3 grid(a.n_rows, a.nv);
    delta_chunk_kernel<<<grid, THREADS, smem, s>>>(a);
    HK_LAUNCH_CHECK();
}

}  // namespace hk
