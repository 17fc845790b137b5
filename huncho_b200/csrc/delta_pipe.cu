// The delta layer of the half-precision models in one warp-specialised kernel:
// the input stage (causal conv + SiLU, l2norm, gates; qwen3_5.rs:817-925), the
// chunked gated delta rule (WY form; qwen3_5.rs:950-987) and the gated RMSNorm
// output (qwen3_5.rs:193-201, 934-938), for 128-wide heads.
//
// The chunk algebra is that of the 32-token chunked kernel (delta_chunk.cu):
// with G the in-chunk cumsum of g, gam = e^G and S0 the state entering a chunk,
//     A[t,s] = b_t e^{G_t - G_s} (k_t . k_s) (s < t),  T = (I + A)^{-1},
//     U = T diag(b) V,  W = T diag(b gam) K,  D = U - W S0,
//     O = diag(gam) Q S0 + Mq D,  Mq[t,s] = e^{G_t - G_s} (q_t . k_s) (s <= t),
//     S_C = gam_C S0 + (diag(e^{G_C - G_s}) K)^T D.
// Everything up to U, W, Mq and the decayed keys depends on the chunk's inputs
// only; D, O and S_C depend on the state. One CTA per (row, value head) runs
// the two halves as two warp groups, one chunk apart:
//   * 8 prep warps: staged pre-conv rows -> conv + SiLU -> q, k (l2norm) and
//     b v; K K^T and Q K^T; T by forward substitution; U, W; decayed keys.
//     They write chunk j+1's operands into one of two hand-off buffers while
//   * 8 state warps compute chunk j: D, O, the gated-norm output and the
//     state update, with the fp32 state in registers (warp w owns key rows
//     16w..16w+15) and its fp16 copy in shared memory.
// The two groups re-divide the register file (setmaxnreg): the state warps
// hold the 128 x 128 state, the prep warps need few registers.
// Hand-off uses hardware named barriers (bar.arrive by the producer, bar.sync
// by the consumer; per buffer one "full" and one "empty" barrier), which carry
// the shared-memory ordering; no flag is polled. Products run on mma.sync
// m16n8k16 with the same fp16 hi/lo splits as the 32-token kernel (q, k, b v,
// D and Mq carry ~22 bits).
//
// Input: the delta in-projection rows in fp32, [N][ldp] = qkv (conv_dim) |
// z (value_dim) | b (nv) | a (nv) (fp16 rows would cost ~1e-3 of probability:
// q and k are the operands the outputs are most sensitive to). A row's chunk
// stream is staged one chunk ahead with cp.async.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>

#include "common.cuh"
#include "layers.cuh"
#include "mma16.cuh"

namespace hk {
namespace {

constexpr int C = 32;  // chunk length
constexpr int D = 128;  // key = value head width
constexpr int LDH = D + 8;
constexpr int LDC = C + 8;
constexpr int RAWW = 3 * D;  // this head's pre-conv q | k | v channels
constexpr int SWARPS = 8, PWARPS = 8;
// Registers per thread: 128 at launch (512 threads fill the 64K file); the
// state warpgroups take 168, the prep warpgroups keep 88 (2 x 128 x 168 +
// 2 x 128 x 88 = 65536, so the increase never waits on registers that are not
// released).
constexpr int REG_STATE = 168, REG_PREP = 88;
static_assert(SWARPS * 32 * REG_STATE + PWARPS * 32 * REG_PREP <= 65536, "register split");
constexpr int STHREADS = SWARPS * 32, PTHREADS = PWARPS * 32;
constexpr int THREADS = STHREADS + PTHREADS;

// Named barrier ids (0 is __syncthreads).
constexpr int BAR_PREP = 1, BAR_STATE = 2, BAR_FULL0 = 3, BAR_EMPTY0 = 5;

struct Handoff {
    __half Qh[C][LDH], Ql[C][LDH];  // q hi / lo
    __half W[C][LDH];               // prep: b gam k; published: -W
    __half Kd[C][LDH];              // decayed keys e^{G_C - G_s} k_s
    // prep: b v hi | lo (fp16 [2C][LDH]); published: U (fp32);
    // state: D hi | lo (fp16 [2C][LDH]) once every state warp has read U.
    float U[C][LDH];
    __half Mh[C][LDC], Ml[C][LDC];  // Mq hi / lo
    float gam[C];
};

struct Smem {
    Handoff hb[2];
    // state warps
    __half S[D * D];       // fp16 copy of the state, 128B-swizzled rows (B operand of D and O)
    float red[SWARPS][C];  // gated norm: per-warp partial sums of squares
    // prep warps
    __half Kh[C][LDH], Kl[C][LDH];
    float A[C][C + 4];  // 16-byte rows (vector reads in the substitution)
    __half T[C][LDC];
    float G[C], beta[C];
    float raw[C][RAWW];      // staged pre-conv rows of the next chunk
    float hist[2][3][RAWW];  // conv history (last 3 pre-conv rows), by chunk parity
};

static_assert(sizeof(Smem) <= 232448, "shared memory of one CTA");

__device__ __forceinline__ void bar_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }
__device__ __forceinline__ void bar_arrive(int id, int n) {
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// The state copy: row r (key), column c (value) at 16-byte chunk (c / 8) ^ (r % 8)
// of the row's 256 bytes, so 8 consecutive rows of one chunk (an ldmatrix
// fetch) and the half2 stores of a warp's rows both hit 32 distinct banks.
__device__ __forceinline__ int s_off(int r, int c) { return r * D + (((c >> 3) ^ (r & 7)) << 3) + (c & 7); }
// Two B fragments (k16 x n8, n-tiles n0 and n0 + 8) with B[k][n] = S[k][n].
__device__ __forceinline__ void frag_b_state(uint32_t (&r)[4], const __half *S, int k0, int n0, int lane) {
    const int j = lane >> 3, i = lane & 7;
    ldsm_x4_t(r, S + s_off(k0 + i + (j & 1) * 8, n0 + (j >> 1) * 8));
}

struct PipeArgs {
    const float *proj;  // [n, ldp] fp32 delta in-projection rows
    int ldp;
    const int32_t *cu_seqlens;
    const int32_t *row_order;
    int nk, nv, key_dim, value_dim, conv_dim;
    const float *conv_w, *base_g, *dt_bias;  // [conv_dim][4], [nv], [nv]
    const float *norm_w;
    float eps;
    __half *mix;
    int ldmix;
    uint8_t *mix_lo;  // e5m2 low part of the output (split-precision out_proj input), or null
    int ldmix_lo;
    const uint64_t *state_in, *state_out;  // per row [nv][128][128] fp32, or 0
    const uint64_t *hist_in;               // per row [3][conv_dim] fp32, or 0
};

__global__ void __launch_bounds__(THREADS, 1) delta_pipe_kernel(PipeArgs a) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    Smem &sm = *reinterpret_cast<Smem *>(smem_raw);
    const int row = a.row_order ? a.row_order[blockIdx.x] : blockIdx.x, h = blockIdx.y;
    const int start = a.cu_seqlens[row], end = a.cu_seqlens[row + 1];
    if (start >= end) return;
    const int nch = (end - start + C - 1) / C;
    const int kh = h / (a.nv / a.nk);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g4 = lane >> 2, t4 = lane & 3;

    if (warp < SWARPS) {
        // ================= state warps =================
        // D and O: warp (mt = w & 1, cq = w >> 1) owns rows 16 mt .. and value
        // columns 32 cq ..; the state update: warp (kt = w & 3, ch = w >> 2) owns
        // key rows 32 kt .. and value columns 64 ch .. of S (registers).
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REG_STATE));
        const int mt = warp & 1, cq = warp >> 1, kt = warp & 3, ch = warp >> 2;
        const int nb = 32 * cq;  // D / O columns
        float S[2][8][4];        // S[32 kt + 16 mi + g4 (+8)][64 ch + 8 nt + 2 t4 (+1)]
        auto s_row = [&](int mi, int e) { return 32 * kt + 16 * mi + g4 + (e >> 1) * 8; };
        auto s_col = [&](int nt, int e) { return 64 * ch + 8 * nt + 2 * t4 + (e & 1); };
        const float *st_in = reinterpret_cast<const float *>(a.state_in ? a.state_in[row] : 0);
        if (st_in) {
            const float *sh = st_in + static_cast<size_t>(h) * D * D;
#pragma unroll
            for (int mi = 0; mi < 2; ++mi)
#pragma unroll
                for (int nt = 0; nt < 8; ++nt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) S[mi][nt][e] = sh[s_row(mi, e) * D + s_col(nt, e)];
        } else {
#pragma unroll
            for (int mi = 0; mi < 2; ++mi)
#pragma unroll
                for (int nt = 0; nt < 8; ++nt) S[mi][nt][0] = S[mi][nt][1] = S[mi][nt][2] = S[mi][nt][3] = 0.f;
        }
        auto store_s16 = [&]() {
#pragma unroll
            for (int mi = 0; mi < 2; ++mi)
#pragma unroll
                for (int nt = 0; nt < 8; ++nt)
#pragma unroll
                    for (int hf = 0; hf < 2; ++hf)
                        *reinterpret_cast<__half2 *>(&sm.S[s_off(s_row(mi, 2 * hf), s_col(nt, 0))]) =
                            __floats2half2_rn(S[mi][nt][2 * hf], S[mi][nt][2 * hf + 1]);
        };
        store_s16();
        float nwr[4][2];
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
            nwr[nt][0] = a.norm_w[nb + nt * 8 + 2 * t4];
            nwr[nt][1] = a.norm_w[nb + nt * 8 + 2 * t4 + 1];
        }
        const int zcol = a.conv_dim + h * D;
        bar_sync(BAR_STATE, STHREADS);  // S16 complete

        for (int j = 0; j < nch; ++j) {
            const int c0 = start + j * C, n = min(C, end - c0), b = j & 1;
            Handoff &H = sm.hb[b];
            // z of this thread's output elements (rows t < n), loaded ahead of use.
            float2 zr[2][4];
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                const int t = mt * 16 + g4 + hf * 8;
#pragma unroll
                for (int nt = 0; nt < 4; ++nt)
                    zr[hf][nt] = t < n ? *reinterpret_cast<const float2 *>(
                                             a.proj + static_cast<size_t>(c0 + t) * a.ldp + zcol + nb + nt * 8 + 2 * t4)
                                       : make_float2(0.f, 0.f);
            }
            bar_sync(BAR_FULL0 + b, THREADS);  // chunk j's operands are published
            // ---- D = U + (-W) S0, O = diag(gam) Q S0 (q hi + lo).
            float u[4][4], o[4][4];
#pragma unroll
            for (int nt = 0; nt < 4; ++nt)
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    const float2 v2 = *reinterpret_cast<const float2 *>(&H.U[mt * 16 + g4 + hf * 8][nb + nt * 8 + 2 * t4]);
                    u[nt][2 * hf] = v2.x;
                    u[nt][2 * hf + 1] = v2.y;
                    o[nt][2 * hf] = o[nt][2 * hf + 1] = 0.f;
                }
#pragma unroll 2
            for (int k0 = 0; k0 < D; k0 += 16) {
                uint32_t sb0[4], sb1[4], aw[4], qh[4], ql[4];
                frag_b_state(sb0, sm.S, k0, nb, lane);
                frag_b_state(sb1, sm.S, k0, nb + 16, lane);
                frag_a<LDH>(aw, H.W, mt * 16, k0, lane);
                frag_a<LDH>(qh, H.Qh, mt * 16, k0, lane);
                frag_a<LDH>(ql, H.Ql, mt * 16, k0, lane);
                mma(u[0], aw, sb0[0], sb0[1]);
                mma(u[1], aw, sb0[2], sb0[3]);
                mma(u[2], aw, sb1[0], sb1[1]);
                mma(u[3], aw, sb1[2], sb1[3]);
                mma(o[0], qh, sb0[0], sb0[1]);
                mma(o[1], qh, sb0[2], sb0[3]);
                mma(o[2], qh, sb1[0], sb1[1]);
                mma(o[3], qh, sb1[2], sb1[3]);
                mma(o[0], ql, sb0[0], sb0[1]);
                mma(o[1], ql, sb0[2], sb0[3]);
                mma(o[2], ql, sb1[0], sb1[1]);
                mma(o[3], ql, sb1[2], sb1[3]);
            }
            bar_sync(BAR_STATE, STHREADS);  // every state warp has read U: D may overwrite it
            __half (*Dh)[LDH] = reinterpret_cast<__half (*)[LDH]>(&H.U[0][0]);
            __half (*Dl)[LDH] = Dh + C;
            const float gm0 = H.gam[mt * 16 + g4], gm1 = H.gam[mt * 16 + g4 + 8];
#pragma unroll
            for (int nt = 0; nt < 4; ++nt)
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    const int t = mt * 16 + g4 + hf * 8, c = nb + nt * 8 + 2 * t4;
                    o[nt][2 * hf] *= hf ? gm1 : gm0;
                    o[nt][2 * hf + 1] *= hf ? gm1 : gm0;
                    split_store2(&Dh[t][c], &Dl[t][c], u[nt][2 * hf], u[nt][2 * hf + 1]);
                }
            bar_sync(BAR_STATE, STHREADS);  // every row of D written
            // ---- O += Mq D (three split products); Mq is lower triangular, so
            // rows 0-15 need keys 0-15 only.
#pragma unroll
            for (int k0 = 0; k0 < C; k0 += 16) {
                if (k0 > 16 * mt) break;
                uint32_t mh[4], ml[4], dh0[4], dh1[4], dl0[4], dl1[4];
                frag_a<LDC>(mh, H.Mh, mt * 16, k0, lane);
                frag_a<LDC>(ml, H.Ml, mt * 16, k0, lane);
                frag_b_kn<LDH>(dh0, Dh, k0, nb, lane);
                frag_b_kn<LDH>(dh1, Dh, k0, nb + 16, lane);
                frag_b_kn<LDH>(dl0, Dl, k0, nb, lane);
                frag_b_kn<LDH>(dl1, Dl, k0, nb + 16, lane);
                mma(o[0], mh, dh0[0], dh0[1]);
                mma(o[1], mh, dh0[2], dh0[3]);
                mma(o[2], mh, dh1[0], dh1[1]);
                mma(o[3], mh, dh1[2], dh1[3]);
                mma(o[0], mh, dl0[0], dl0[1]);
                mma(o[1], mh, dl0[2], dl0[3]);
                mma(o[2], mh, dl1[0], dl1[1]);
                mma(o[3], mh, dl1[2], dl1[3]);
                mma(o[0], ml, dh0[0], dh0[1]);
                mma(o[1], ml, dh0[2], dh0[3]);
                mma(o[2], ml, dh1[0], dh1[1]);
                mma(o[3], ml, dh1[2], dh1[3]);
            }
            // Row sums of squares of O over this warp's 32 columns.
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                float ss = 0.f;
#pragma unroll
                for (int nt = 0; nt < 4; ++nt) ss += o[nt][2 * hf] * o[nt][2 * hf] + o[nt][2 * hf + 1] * o[nt][2 * hf + 1];
                ss += __shfl_xor_sync(0xffffffffu, ss, 1);
                ss += __shfl_xor_sync(0xffffffffu, ss, 2);
                if (t4 == 0) sm.red[cq][mt * 16 + g4 + hf * 8] = ss;
            }
            bar_sync(BAR_STATE, STHREADS);  // every partial sum written
            // ---- rms(o) * w * silu(z) -> fp16 out_proj input (fixed quarter order).
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                const int t = mt * 16 + g4 + hf * 8;
                if (t >= n) continue;
                const float ss = (sm.red[0][t] + sm.red[1][t]) + (sm.red[2][t] + sm.red[3][t]);
                const float denom = sqrtf(ss / static_cast<float>(D) + a.eps);
                const size_t tok = static_cast<size_t>(c0 + t);
#pragma unroll
                for (int nt = 0; nt < 4; ++nt) {
                    const int c = nb + nt * 8 + 2 * t4;
                    const float2 zz = zr[hf][nt];
                    const float y0 = (__fdividef(o[nt][2 * hf], denom) * nwr[nt][0]) * silu_fast(zz.x);
                    const float y1 = (__fdividef(o[nt][2 * hf + 1], denom) * nwr[nt][1]) * silu_fast(zz.y);
                    const __half2 yh = __floats2half2_rn(y0, y1);
                    *reinterpret_cast<__half2 *>(a.mix + tok * a.ldmix + h * D + c) = yh;
                    if (a.mix_lo)
                        *reinterpret_cast<uint16_t *>(a.mix_lo + tok * a.ldmix_lo + h * D + c) =
                            static_cast<uint16_t>(lo_e5m2(y0, __low2half(yh)) | (lo_e5m2(y1, __high2half(yh)) << 8));
                }
            }
            // ---- S = gam_C S + Kd^T D (D hi + lo).
            {
                const float gc = H.gam[C - 1];
#pragma unroll
                for (int mi = 0; mi < 2; ++mi)
#pragma unroll
                    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
                        for (int e = 0; e < 4; ++e) S[mi][nt][e] *= gc;
#pragma unroll
                for (int k0 = 0; k0 < C; k0 += 16) {
                    uint32_t ak0[4], ak1[4];
                    frag_at<LDH>(ak0, H.Kd, 32 * kt, k0, lane);
                    frag_at<LDH>(ak1, H.Kd, 32 * kt + 16, k0, lane);
#pragma unroll
                    for (int np = 0; np < 4; ++np) {
                        uint32_t dh[4], dl[4];
                        frag_b_kn<LDH>(dh, Dh, k0, 64 * ch + 16 * np, lane);
                        frag_b_kn<LDH>(dl, Dl, k0, 64 * ch + 16 * np, lane);
                        mma(S[0][2 * np], ak0, dh[0], dh[1]);
                        mma(S[0][2 * np + 1], ak0, dh[2], dh[3]);
                        mma(S[0][2 * np], ak0, dl[0], dl[1]);
                        mma(S[0][2 * np + 1], ak0, dl[2], dl[3]);
                        mma(S[1][2 * np], ak1, dh[0], dh[1]);
                        mma(S[1][2 * np + 1], ak1, dh[2], dh[3]);
                        mma(S[1][2 * np], ak1, dl[0], dl[1]);
                        mma(S[1][2 * np + 1], ak1, dl[2], dl[3]);
                    }
                }
                store_s16();
            }
            // Hand-off buffer b is free for chunk j + 2 (if the row has one).
            if (j + 2 < nch) bar_arrive(BAR_EMPTY0 + b, THREADS);
            bar_sync(BAR_STATE, STHREADS);  // S16 complete; red reusable
        }
        if (a.state_out && a.state_out[row]) {
            float *sh = reinterpret_cast<float *>(a.state_out[row]) + static_cast<size_t>(h) * D * D;
#pragma unroll
            for (int mi = 0; mi < 2; ++mi)
#pragma unroll
                for (int nt = 0; nt < 8; ++nt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) sh[s_row(mi, e) * D + s_col(nt, e)] = S[mi][nt][e];
        }
        return;
    }

    // ================= prep warps =================
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_PREP));
    const int pw = warp - SWARPS, ptid = tid - STHREADS;
    const int ch_q = kh * D, ch_k = a.key_dim + kh * D, ch_v = 2 * a.key_dim + h * D;
    const int col_b = a.conv_dim + a.value_dim + h, col_a = col_b + a.nv;
    // cp.async of a chunk's pre-conv q | k | v rows (rows past the end zero):
    // thread ptid copies 16-byte pieces p = ptid % 8 + 8 i (i < 12) of row ptid / 8.
    static_assert(PTHREADS == 8 * C && RAWW == 8 * 12 * 4, "staging map");
    const int pr_row = ptid >> 3, pr_p = ptid & 7;
    auto prefetch_raw = [&](int c0) {
        const bool ok = pr_row < end - c0;
        const float *src = a.proj + static_cast<size_t>(c0 + (ok ? pr_row : 0)) * a.ldp;
#pragma unroll
        for (int i = 0; i < 12; ++i) {
            const int which = i / 4, c = (pr_p + 8 * (i % 4)) * 4;
            cp16(&sm.raw[pr_row][which * D + c], src + (which == 0 ? ch_q : which == 1 ? ch_k : ch_v) + c, ok);
        }
    };
    {
        const float *hist = reinterpret_cast<const float *>(a.hist_in ? a.hist_in[row] : 0);
        for (int i = ptid; i < 3 * RAWW; i += PTHREADS) {
            const int jr = i / RAWW, rem = i % RAWW, which = rem / D, c = rem % D;
            const int ch = (which == 0 ? ch_q : which == 1 ? ch_k : ch_v) + c;
            sm.hist[0][jr][rem] = hist ? hist[static_cast<size_t>(jr) * a.conv_dim + ch] : 0.f;
        }
    }
    prefetch_raw(start);
    cp_commit();
    const float bg_h = a.base_g[h], dt_h = a.dt_bias[h];
    // Raw b / a of row `lane` of the current chunk, loaded one chunk ahead.
    float braw = 0.f, araw = 0.f;
    if (lane < min(C, end - start)) {
        const float *pr = a.proj + static_cast<size_t>(start + lane) * a.ldp;
        braw = pr[col_b];
        araw = pr[col_a];
    }
    __half (*VH)[LDH] = nullptr;
    for (int j = 0; j < nch; ++j) {
        const int c0 = start + j * C, n = min(C, end - c0), b = j & 1;
        Handoff &H = sm.hb[b];
        VH = reinterpret_cast<__half (*)[LDH]>(&H.U[0][0]);  // b v hi rows 0..C-1, lo rows C..2C-1
        // ---- gates: every prep warp scans g in registers (lane = row).
        const bool ok = lane < n;
        const float bv = ok ? sigmoid_f(braw) : 0.f;
        float gv = ok ? bg_h * logf(expf(araw + dt_h) + 1.0f) : 0.f;
        if (j + 1 < nch && lane < min(C, end - c0 - C)) {
            const float *pr = a.proj + static_cast<size_t>(c0 + C + lane) * a.ldp;
            braw = pr[col_b];
            araw = pr[col_a];
        }
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float up = __shfl_up_sync(0xffffffffu, gv, o);
            if (lane >= o) gv += up;
        }
        const float gamv = expf(gv);
        cp_wait_all();
        bar_sync(BAR_PREP, PTHREADS);  // staged rows visible; the previous chunk's prep is done
        if (j >= 2) bar_sync(BAR_EMPTY0 + b, THREADS);  // the state warps are done with buffer b
        if (pw == 0) {
            sm.G[lane] = gv;
            sm.beta[lane] = bv;
            H.gam[lane] = gamv;
        }
        // ---- conv + SiLU over [history ; chunk], l2norm of q (x 1/sqrt(128)) and k;
        // warp pw takes rows 4 pw .. 4 pw + 3.
        const int hcur = j & 1;
        {
            const int r0 = 4 * pw;
#pragma unroll
            for (int which = 0; which < 3; ++which) {
                // Conv weights of channels 4 lane .. 4 lane + 3 (taps contiguous
                // per channel in global memory; L1-resident after the first chunk).
                float4 w4[4], x4[7];
                {
                    const float4 *cwp = reinterpret_cast<const float4 *>(a.conv_w) +
                                        (which == 0 ? ch_q : which == 1 ? ch_k : ch_v) + 4 * lane;
                    const float4 c0w = __ldg(cwp), c1w = __ldg(cwp + 1), c2w = __ldg(cwp + 2), c3w = __ldg(cwp + 3);
                    w4[0] = make_float4(c0w.x, c1w.x, c2w.x, c3w.x);
                    w4[1] = make_float4(c0w.y, c1w.y, c2w.y, c3w.y);
                    w4[2] = make_float4(c0w.z, c1w.z, c2w.z, c3w.z);
                    w4[3] = make_float4(c0w.w, c1w.w, c2w.w, c3w.w);
                }
#pragma unroll
                for (int i = 0; i < 7; ++i) {
                    const int idx = r0 - 3 + i;
                    x4[i] = idx >= 0 ? *reinterpret_cast<const float4 *>(&sm.raw[idx][which * D + 4 * lane])
                                     : *reinterpret_cast<const float4 *>(&sm.hist[hcur][3 + idx][which * D + 4 * lane]);
                }
                float y[4][4], ss[4];
#pragma unroll
                for (int rr = 0; rr < 4; ++rr) {
                    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                    for (int t = 0; t < 4; ++t) {
                        const float4 x = x4[rr + t], w = w4[t];
                        acc[0] = fmaf(w.x, x.x, acc[0]);
                        acc[1] = fmaf(w.y, x.y, acc[1]);
                        acc[2] = fmaf(w.z, x.z, acc[2]);
                        acc[3] = fmaf(w.w, x.w, acc[3]);
                    }
#pragma unroll
                    for (int c = 0; c < 4; ++c) y[rr][c] = silu_fast(acc[c]);
                    ss[rr] = y[rr][0] * y[rr][0] + y[rr][1] * y[rr][1] + y[rr][2] * y[rr][2] + y[rr][3] * y[rr][3];
                }
                if (which < 2) {
#pragma unroll
                    for (int o = 16; o >= 1; o >>= 1)
#pragma unroll
                        for (int rr = 0; rr < 4; ++rr) ss[rr] += __shfl_xor_sync(0xffffffffu, ss[rr], o);
                }
#pragma unroll
                for (int rr = 0; rr < 4; ++rr) {
                    const int r = r0 + rr;
                    const float bb = __shfl_sync(0xffffffffu, bv, r);
                    if (which == 2) {
                        const float bvv[4] = {bb * y[rr][0], bb * y[rr][1], bb * y[rr][2], bb * y[rr][3]};
                        split_store4(&VH[r][4 * lane], &VH[C + r][4 * lane], bvv);
                    } else {
                        const float inv = which == 0 ? rsqrtf(ss[rr] + 1e-6f) * rsqrtf(static_cast<float>(D))
                                                     : rsqrtf(ss[rr] + 1e-6f);
                        const float nv4[4] = {y[rr][0] * inv, y[rr][1] * inv, y[rr][2] * inv, y[rr][3] * inv};
                        if (which == 0) {
                            split_store4(&H.Qh[r][4 * lane], &H.Ql[r][4 * lane], nv4);
                        } else {
                            split_store4(&sm.Kh[r][4 * lane], &sm.Kl[r][4 * lane], nv4);
                            const float bgk = bb * __shfl_sync(0xffffffffu, gamv, r);
                            const float bkk[4] = {bgk * nv4[0], bgk * nv4[1], bgk * nv4[2], bgk * nv4[3]};
                            store4(&H.W[r][4 * lane], bkk);
                        }
                    }
                }
                if (pw == PWARPS - 1) {  // rows C-3 .. C-1: the next chunk's history
#pragma unroll
                    for (int i = 0; i < 3; ++i)
                        *reinterpret_cast<float4 *>(&sm.hist[hcur ^ 1][i][which * D + 4 * lane]) = x4[4 + i];
                }
            }
        }
        bar_sync(BAR_PREP, PTHREADS);  // operands visible; staging free
        if (j + 1 < nch) prefetch_raw(c0 + C);
        cp_commit();
        // ---- K K^T -> A (warps 0-3) and Q K^T -> Mq (warps 4-7); 16 x 16 per warp.
        {
            const bool kk = pw < 4;
            const int mt = (pw >> 1) & 1, n0 = (pw & 1) * 16;
            // hi x hi and the two cross terms in separate accumulators (four
            // independent MMA chains instead of two), summed at the end.
            float acc[2][4], acx[2][4];
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
                acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
                acx[nt][0] = acx[nt][1] = acx[nt][2] = acx[nt][3] = 0.f;
            }
#pragma unroll
            for (int k0 = 0; k0 < D; k0 += 16) {
                uint32_t ah[4], al[4], bh[4], bl[4];
                frag_a<LDH>(ah, kk ? sm.Kh : H.Qh, mt * 16, k0, lane);
                frag_a<LDH>(al, kk ? sm.Kl : H.Ql, mt * 16, k0, lane);
                frag_b_nk<LDH>(bh, sm.Kh, k0, n0, lane);
                frag_b_nk<LDH>(bl, sm.Kl, k0, n0, lane);
                mma(acc[0], ah, bh[0], bh[1]);
                mma(acc[1], ah, bh[2], bh[3]);
                mma(acx[0], ah, bl[0], bl[1]);
                mma(acx[1], ah, bl[2], bl[3]);
                mma(acx[0], al, bh[0], bh[1]);
                mma(acx[1], al, bh[2], bh[3]);
            }
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[nt][e] += acx[nt][e];
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int t = mt * 16 + g4 + (e >> 1) * 8, s = n0 + nt * 8 + 2 * t4 + (e & 1);
                    const float dec = expf(sm.G[t] - sm.G[s]);
                    if (kk)
                        sm.A[t][s] = s < t ? sm.beta[t] * dec * acc[nt][e] : 0.f;
                    else
                        split_store(&H.Mh[t][s], &H.Ml[t][s], s <= t ? dec * acc[nt][e] : 0.f);
                }
        }
        bar_sync(BAR_PREP, PTHREADS);
        if (pw == 0) {
            // ---- T = (I + A)^{-1}. Diagonal 16 x 16 blocks by forward substitution
            // (lanes 0-15: columns of T11, lanes 16-31: columns of T22), written in
            // place over A (fp32) and into T (fp16).
            const int o = lane & 16;
            float col[16];
#pragma unroll
            for (int t = 0; t < 16; ++t) {
                const float *arow = &sm.A[o + t][o];
                float acc[4] = {(t == (lane & 15)) ? 1.f : 0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int s = 0; s + 4 <= t; s += 4) {
                    const float4 a4 = *reinterpret_cast<const float4 *>(arow + s);
                    acc[0] = fmaf(-a4.x, col[s], acc[0]);
                    acc[1] = fmaf(-a4.y, col[s + 1], acc[1]);
                    acc[2] = fmaf(-a4.z, col[s + 2], acc[2]);
                    acc[3] = fmaf(-a4.w, col[s + 3], acc[3]);
                }
#pragma unroll
                for (int s = t & ~3; s < t; ++s) acc[s & 3] = fmaf(-arow[s], col[s], acc[s & 3]);
                col[t] = (acc[0] + acc[1]) + (acc[2] + acc[3]);
            }
            __syncwarp();  // every lane has read its rows of A
#pragma unroll
            for (int t = 0; t < 16; ++t) {
                sm.A[o + t][lane] = col[t];
                sm.T[o + t][lane] = __float2half_rn(col[t]);
            }
        } else {
            // ---- decayed keys e^{G_C - G_s} (k hi + lo), meanwhile.
            const float gl = sm.G[C - 1];
            for (int e = ptid - 32; e < C * (D / 4); e += PTHREADS - 32) {  // warps 1-7
                const int r = e / (D / 4), c = (e % (D / 4)) * 4;
                const float dec = expf(gl - sm.G[r]);
                const uint2 kh2 = *reinterpret_cast<const uint2 *>(&sm.Kh[r][c]);
                const uint2 kl2 = *reinterpret_cast<const uint2 *>(&sm.Kl[r][c]);
                const float2 h0 = __half22float2(*reinterpret_cast<const __half2 *>(&kh2.x));
                const float2 h1 = __half22float2(*reinterpret_cast<const __half2 *>(&kh2.y));
                const float2 l0 = __half22float2(*reinterpret_cast<const __half2 *>(&kl2.x));
                const float2 l1 = __half22float2(*reinterpret_cast<const __half2 *>(&kl2.y));
                const float kd[4] = {dec * (h0.x + l0.x), dec * (h0.y + l0.y), dec * (h1.x + l1.x), dec * (h1.y + l1.y)};
                store4(&H.Kd[r][c], kd);
            }
        }
        bar_sync(BAR_PREP, PTHREADS);
        // ---- T21 = -T22 A21 T11: X = A21 T11 into the (zero) upper-right block
        // of A, then T21 = -T22 X; thread (i, jj) of 16 x 16.
        {
            const int i = ptid >> 4, jj = ptid & 15;
            float x = 0.f;
#pragma unroll
            for (int m = 0; m < 16; ++m) x = fmaf(sm.A[16 + i][m], sm.A[m][jj], x);
            sm.A[i][16 + jj] = x;
            bar_sync(BAR_PREP, PTHREADS);
            float y = 0.f;
#pragma unroll
            for (int k = 0; k < 16; ++k) y = fmaf(sm.A[16 + i][16 + k], sm.A[k][16 + jj], y);
            sm.T[16 + i][jj] = __float2half_rn(-y);
            sm.T[i][16 + jj] = __float2half_rn(0.f);
        }
        bar_sync(BAR_PREP, PTHREADS);
        // ---- U = T (b v) (hi + lo), W = T (b gam k); warp pw owns cols 16 pw ..
        {
            const int nb = 16 * pw;
            float u[2][2][4], w[2][2][4];
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) u[mt][nt][e] = w[mt][nt][e] = 0.f;
#pragma unroll
            for (int k0 = 0; k0 < C; k0 += 16) {
                uint32_t vh[4], vl[4], bk[4];
                frag_b_kn<LDH>(vh, VH, k0, nb, lane);
                frag_b_kn<LDH>(vl, VH + C, k0, nb, lane);
                frag_b_kn<LDH>(bk, H.W, k0, nb, lane);
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
            bar_sync(BAR_PREP, PTHREADS);  // every read of b v (under U) and b gam k done
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                    for (int hf = 0; hf < 2; ++hf) {
                        const int t = mt * 16 + g4 + hf * 8, c = nb + nt * 8 + 2 * t4;
                        *reinterpret_cast<float2 *>(&H.U[t][c]) = make_float2(u[mt][nt][2 * hf], u[mt][nt][2 * hf + 1]);
                        *reinterpret_cast<__half2 *>(&H.W[t][c]) =
                            __floats2half2_rn(-w[mt][nt][2 * hf], -w[mt][nt][2 * hf + 1]);
                    }
        }
        bar_arrive(BAR_FULL0 + b, THREADS);  // chunk j published to the state warps
    }
}

}  // namespace

bool delta_pipe_supported(const DeltaRecArgs &r, const DeltaFusedInput &in) {
    return in.proj && r.dk == 128 && r.dv == 128 && r.nk > 0 && r.nv % r.nk == 0 && (in.ldp % 4) == 0 &&
           (in.conv_dim % 4) == 0;
}

void launch_delta_pipe(const DeltaRecArgs &r, const DeltaFusedInput &in, const float *norm_w, float eps, __half *mix,
                       int ldmix, cudaStream_t s, uint8_t *mix_lo, int ldmix_lo) {
    if (r.n_rows <= 0) return;
    PipeArgs a;
    a.proj = in.proj;
    a.ldp = in.ldp;
    a.cu_seqlens = r.cu_seqlens;
    a.row_order = r.row_order;
    a.nk = r.nk;
    a.nv = r.nv;
    a.key_dim = r.nk * 128;
    a.value_dim = r.nv * 128;
    a.conv_dim = in.conv_dim;
    a.conv_w = in.conv_w;
    a.base_g = in.base_g;
    a.dt_bias = in.dt_bias;
    a.norm_w = norm_w;
    a.eps = eps;
    a.mix = mix;
    a.ldmix = ldmix;
    a.mix_lo = mix_lo;
    a.ldmix_lo = ldmix_lo;
    a.state_in = r.state_in;
    a.state_out = r.state_out;
    a.hist_in = in.hist_in;
    const int smem = static_cast<int>(sizeof(Smem));
    static SmemOptIn opt_in;
    opt_in.ensure(delta_pipe_kernel, smem);
    dim3 grid(r.n_rows, r.nv);
    delta_pipe_kernel<<<grid, THREADS, smem, s>>>(a);
    HK_LAUNCH_CHECK();
}

}  // namespace hk
