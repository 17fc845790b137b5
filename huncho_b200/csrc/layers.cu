// Bandwidth-bound layer kernels of the Kev forward: embedding gather, RMSNorm,
// the Gated DeltaNet input stage and recurrence, gated RMSNorm, the attention
// input stage, SwiGLU and the pointer readout. All compute in fp32; projection
// outputs are read as fp32, and only tensors that feed a tensor-core GEMM or
// attention are stored in the activation type (float, or fp16 for the
// half-precision models). One warp or one CTA per token row, so the loads of a
// row are contiguous and coalesced.
#include <math.h>

#include "common.cuh"
#include "layers.cuh"

namespace hk {
namespace {

// ------------------------------------------------------------------ embed
template <typename TW>
__global__ void embed_kernel(const uint32_t *__restrict__ ids, int n, const TW *__restrict__ table,
                             int hidden, float *__restrict__ x) {
    const int t = blockIdx.x;
    if (t >= n) return;
    const TW *row = table + static_cast<size_t>(ids[t]) * hidden;
    float *dst = x + static_cast<size_t>(t) * hidden;
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) dst[i] = Act<TW>::to_f(row[i]);
}

// ------------------------------------------------------------------ rmsnorm
// One warp per row; division by sqrt(mean(x^2) + eps) as the reference writes it.
template <typename T>
__global__ void rmsnorm_kernel(const float *__restrict__ x, int ldx, const float *__restrict__ w,
                               float eps, int rows, int hidden, T *__restrict__ out, int ldo,
                               uint8_t *__restrict__ out_lo, int ldo_lo) {
    const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float *xr = x + static_cast<size_t>(row) * ldx;
    T *o = out + static_cast<size_t>(row) * ldo;
    float ss = 0.f;
    if ((hidden & 127) == 0) {
        for (int i = lane * 4; i < hidden; i += 128) {
            const float4 v = *reinterpret_cast<const float4 *>(xr + i);
            ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
    } else {
        for (int i = lane; i < hidden; i += 32) ss += xr[i] * xr[i];
    }
    ss = warp_sum(ss);
    const float denom = sqrtf(ss / static_cast<float>(hidden) + eps);
    for (int i = lane; i < hidden; i += 32) {
        const float y = (xr[i] / denom) * w[i];
        o[i] = Act<T>::from_f(y);
        if constexpr (sizeof(T) == 2) {
            if (out_lo) out_lo[static_cast<size_t>(row) * ldo_lo + i] = lo_e5m2(y, o[i]);
        }
    }
}

// Register-resident form for hidden = 128 * NCH: each lane holds NCH float4 of
// its row, so the row is read once; fp16 output in 8-byte stores.
template <typename T, int NCH>
__global__ void rmsnorm_reg_kernel(const float *__restrict__ x, int ldx, const float *__restrict__ w,
                                   float eps, int rows, T *__restrict__ out, int ldo, uint8_t *__restrict__ out_lo,
                                   int ldo_lo) {
    const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float *xr = x + static_cast<size_t>(row) * ldx;
    float4 v[NCH];
#pragma unroll
    for (int c = 0; c < NCH; ++c) v[c] = *reinterpret_cast<const float4 *>(xr + c * 128 + lane * 4);
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) ss += v[c].x * v[c].x + v[c].y * v[c].y + v[c].z * v[c].z + v[c].w * v[c].w;
    ss = warp_sum(ss);
    const float denom = sqrtf(ss / static_cast<float>(NCH * 128) + eps);
    T *o = out + static_cast<size_t>(row) * ldo;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
        const int i = c * 128 + lane * 4;
        const float4 wv = *reinterpret_cast<const float4 *>(w + i);
        const float y0 = (v[c].x / denom) * wv.x, y1 = (v[c].y / denom) * wv.y;
        const float y2 = (v[c].z / denom) * wv.z, y3 = (v[c].w / denom) * wv.w;
        if constexpr (sizeof(T) == 2) {
            const __half2 a = __floats2half2_rn(y0, y1), b = __floats2half2_rn(y2, y3);
            *reinterpret_cast<uint2 *>(o + i) =
                make_uint2(*reinterpret_cast<const uint32_t *>(&a), *reinterpret_cast<const uint32_t *>(&b));
            if (out_lo)
                *reinterpret_cast<uint32_t *>(out_lo + static_cast<size_t>(row) * ldo_lo + i) =
                    lo_e5m2(y0, __low2half(a)) | (lo_e5m2(y1, __high2half(a)) << 8) |
                    (lo_e5m2(y2, __low2half(b)) << 16) | (static_cast<uint32_t>(lo_e5m2(y3, __high2half(b))) << 24);
        } else {
            *reinterpret_cast<float4 *>(o + i) = make_float4(y0, y1, y2, y3);
        }
    }
}

// ------------------------------------------------------------------ delta prep
// One CTA per token. Stage 1: conv + SiLU of every q|k|v channel (fp32, taps in
// ascending order from a zero accumulator, no fused multiply-add, matching
// conv_cpu.rs:38-49). Stage 2: per key head L2 norm of q and k. Stage 3: beta
// and g. Everything stays fp32 (the half-precision reference path rounds the
// conv output to the model dtype, qwen3_5.rs:843; this path keeps fp32).
__global__ void delta_prep_kernel(DeltaPrepArgs a) {
    extern __shared__ float conv_s[];  // [conv_dim]
    const int t = blockIdx.x;
    const int key_dim = a.nk * a.dk, value_dim = a.nv * a.dv;
    const int conv_dim = 2 * key_dim + value_dim;
    const int pos = a.pos[t];
    const float *proj = a.proj;
    // Taps before the row start read the cached prefix's conv inputs (hist
    // row taps-1+q for relative index q < 0), or nothing without a cache.
    const uint64_t haddr = (a.hist_in && a.tok_row) ? a.hist_in[a.tok_row[t]] : 0;
    const float *hist = reinterpret_cast<const float *>(haddr);
    for (int c = threadIdx.x; c < conv_dim; c += blockDim.x) {
        float acc = 0.f;
        for (int tap = 0; tap < a.taps; ++tap) {
            const int shift = a.taps - 1 - tap;
            float xv;
            if (shift > pos) {
                if (!hist) continue;
                xv = hist[static_cast<size_t>(a.taps - 1 + pos - shift) * conv_dim + c];
            } else {
                xv = proj[static_cast<size_t>(t - shift) * a.ldp + c];
            }
            acc = __fadd_rn(acc, __fmul_rn(a.conv_w[c * a.taps + tap], xv));
        }
        conv_s[c] = silu_f(acc);
    }
    __syncthreads();
    const int warp = threadIdx.x / 32, lane = threadIdx.x & 31, nwarps = blockDim.x / 32;
    const float qscale = 1.0f / sqrtf(static_cast<float>(a.dk));
    for (int hh = warp; hh < 2 * a.nk; hh += nwarps) {
        const bool is_q = hh < a.nk;
        const int head = is_q ? hh : hh - a.nk;
        const float *src = conv_s + (is_q ? 0 : key_dim) + head * a.dk;
        float ss = 0.f;
        for (int i = lane; i < a.dk; i += 32) ss += src[i] * src[i];
        ss = warp_sum(ss);
        const float inv = 1.0f / sqrtf(ss + 1e-6f);
        float *dst = (is_q ? a.q : a.k) + (static_cast<size_t>(t) * a.nk + head) * a.dk;
        for (int i = lane; i < a.dk; i += 32) dst[i] = is_q ? (src[i] * inv) * qscale : src[i] * inv;
    }
    for (int i = threadIdx.x; i < value_dim; i += blockDim.x)
        a.v[static_cast<size_t>(t) * value_dim + i] = conv_s[2 * key_dim + i];
    for (int h = threadIdx.x; h < a.nv; h += blockDim.x) {
        const float b = proj[static_cast<size_t>(t) * a.ldp + conv_dim + value_dim + h];
        const float av = proj[static_cast<size_t>(t) * a.ldp + conv_dim + value_dim + a.nv + h];
        a.beta[static_cast<size_t>(t) * a.nv + h] = sigmoid_f(b);
        const float sp = logf(expf(av + a.dt_bias[h]) + 1.0f);
        a.g[static_cast<size_t>(t) * a.nv + h] = a.base_g[h] * sp;
    }
}

// Vectorised variant for 128-wide heads and 4 taps: one warp per (block of
// TB consecutive tokens, head slot); slot < nk: a q head, < 2nk: a k head,
// < 2nk + nv: a v head, == 2nk + nv: beta and g for the block. Each lane owns
// 4 channels and keeps the last 3 inputs of each in registers, so every
// projection element is read once (float4) and every output written once.
// The conv sum keeps the taps' ascending order with separately rounded
// products (conv_cpu.rs:38-49).
template <int TB, bool FAST>
__global__ void delta_prep_vec_kernel(DeltaPrepArgs a) {
    const int warps = blockDim.x / 32;
    const int wid = blockIdx.x * warps + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    const int slots = 2 * a.nk + a.nv + 1;
    const int nblk = (a.n + TB - 1) / TB;
    if (wid >= nblk * slots) return;
    const int blk = wid / slots, slot = wid % slots;
    const int t0 = blk * TB, t1 = min(a.n, t0 + TB);
    const int key_dim = a.nk * 128, value_dim = a.nv * 128;
    const int conv_dim = 2 * key_dim + value_dim;
    if (slot == 2 * a.nk + a.nv) {  // gating: lanes over value heads
        for (int t = t0; t < t1; ++t)
            for (int h = lane; h < a.nv; h += 32) {
                const float *pr = a.proj + static_cast<size_t>(t) * a.ldp + conv_dim + value_dim;
                a.beta[static_cast<size_t>(t) * a.nv + h] = sigmoid_f(pr[h]);
                const float sp = logf(expf(pr[a.nv + h] + a.dt_bias[h]) + 1.0f);
                a.g[static_cast<size_t>(t) * a.nv + h] = a.base_g[h] * sp;
            }
        return;
    }
    const bool is_q = slot < a.nk, is_k = !is_q && slot < 2 * a.nk;
    const int c0 = (is_q ? slot * 128 : is_k ? key_dim + (slot - a.nk) * 128
                                            : 2 * key_dim + (slot - 2 * a.nk) * 128) + lane * 4;
    float w[4][4];  // [channel][tap]
#pragma unroll
    for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int k = 0; k < 4; ++k) w[c][k] = a.conv_w[(c0 + c) * 4 + k];
    // History x[t-3], x[t-2], x[t-1] for the 4 channels: inside the row from
    // proj, before its start from the row's cached conv inputs (hist row 3+q
    // for relative index q), else zero.
    auto before_row = [&](int t, int q) {
        const uint64_t addr = (a.hist_in && a.tok_row) ? a.hist_in[a.tok_row[t]] : 0;
        if (!addr) return make_float4(0.f, 0.f, 0.f, 0.f);
        return *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(addr) +
                                                 static_cast<size_t>(3 + q) * conv_dim + c0);
    };
    float4 h3, h2, h1;
    {
        const int p0 = a.pos[t0];
        h3 = p0 >= 3 ? *reinterpret_cast<const float4 *>(a.proj + static_cast<size_t>(t0 - 3) * a.ldp + c0)
                     : before_row(t0, p0 - 3);
        h2 = p0 >= 2 ? *reinterpret_cast<const float4 *>(a.proj + static_cast<size_t>(t0 - 2) * a.ldp + c0)
                     : before_row(t0, p0 - 2);
        h1 = p0 >= 1 ? *reinterpret_cast<const float4 *>(a.proj + static_cast<size_t>(t0 - 1) * a.ldp + c0)
                     : before_row(t0, p0 - 1);
    }
    const float qscale = 1.0f / sqrtf(128.0f);
    for (int t = t0; t < t1; ++t) {
        if (a.pos[t] == 0 && t > t0) {  // a new row starts
            h3 = before_row(t, -3);
            h2 = before_row(t, -2);
            h1 = before_row(t, -1);
        }
        const float4 x = *reinterpret_cast<const float4 *>(a.proj + static_cast<size_t>(t) * a.ldp + c0);
        const float xs[4][4] = {{h3.x, h2.x, h1.x, x.x}, {h3.y, h2.y, h1.y, x.y},
                                {h3.z, h2.z, h1.z, x.z}, {h3.w, h2.w, h1.w, x.w}};
        float y[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            float acc = 0.f;
#pragma unroll
            for (int k = 0; k < 4; ++k)
                acc = FAST ? fmaf(w[c][k], xs[c][k], acc) : __fadd_rn(acc, __fmul_rn(w[c][k], xs[c][k]));
            y[c] = FAST ? silu_fast(acc) : silu_f(acc);
        }
        float4 out;
        if (is_q || is_k) {
            float ss = warp_sum(y[0] * y[0] + y[1] * y[1] + y[2] * y[2] + y[3] * y[3]);
            const float inv = FAST ? rsqrtf(ss + 1e-6f) : 1.0f / sqrtf(ss + 1e-6f);
            const float sc = is_q ? qscale : 1.0f;
            out = make_float4((y[0] * inv) * sc, (y[1] * inv) * sc, (y[2] * inv) * sc, (y[3] * inv) * sc);
            float *dst = (is_q ? a.q : a.k) + static_cast<size_t>(t) * key_dim + (c0 - (is_q ? 0 : key_dim));
            *reinterpret_cast<float4 *>(dst) = out;
        } else {
            out = make_float4(y[0], y[1], y[2], y[3]);
            *reinterpret_cast<float4 *>(a.v + static_cast<size_t>(t) * value_dim + (c0 - 2 * key_dim)) = out;
        }
        h3 = h2;
        h2 = h1;
        h1 = x;
    }
}

// ------------------------------------------------------------------ delta recurrence
// One CTA per (row, value head); thread j owns state column S[:, j] in
// registers, so the memory readout sum_i S[i,j] k_i and the output readout
// sum_i S[i,j] q_i are thread-local and need no cross-thread reduction.
// k_t and q_t are broadcast through double-buffered shared memory.
template <int DK, bool EXACT>
__global__ void __launch_bounds__(128) delta_recurrent_kernel(DeltaRecArgs a) {
    __shared__ float kq[2][2][DK];
    const int row = blockIdx.x, h = blockIdx.y;
    const int j = threadIdx.x;
    const int kh = h / (a.nv / a.nk);  // repeat_interleave of key heads (qwen3_5.rs:901-915)
    const int start = a.cu_seqlens[row], end = a.cu_seqlens[row + 1];
    const uint64_t sin = a.state_in ? a.state_in[row] : 0, sout = a.state_out ? a.state_out[row] : 0;
    float S[DK];
    {
        const float *st = reinterpret_cast<const float *>(sin);
#pragma unroll
        for (int i = 0; i < DK; ++i)
            S[i] = (st && j < a.dv) ? st[(static_cast<size_t>(h) * DK + i) * a.dv + j] : 0.f;
    }
    int buf = 0;
    for (int t = start; t < end; ++t) {
        for (int i = threadIdx.x; i < DK; i += blockDim.x) {
            kq[buf][0][i] = a.k[(static_cast<size_t>(t) * a.nk + kh) * DK + i];
            kq[buf][1][i] = a.q[(static_cast<size_t>(t) * a.nk + kh) * DK + i];
        }
        __syncthreads();
        if (j < a.dv) {
            const float d = expf(a.g[static_cast<size_t>(t) * a.nv + h]);
            const float b = a.beta[static_cast<size_t>(t) * a.nv + h];
            const float vj = a.v[(static_cast<size_t>(t) * a.nv + h) * a.dv + j];
            const float *ks = kq[buf][0];
            const float *qs = kq[buf][1];
            float o;
            if (EXACT) {
                float m = 0.f;
#pragma unroll
                for (int i = 0; i < DK; ++i) {
                    S[i] = __fmul_rn(S[i], d);
                    m = __fadd_rn(m, __fmul_rn(S[i], ks[i]));
                }
                const float delta = __fmul_rn(__fsub_rn(vj, m), b);
                o = 0.f;
#pragma unroll
                for (int i = 0; i < DK; ++i) {
                    S[i] = __fadd_rn(S[i], __fmul_rn(ks[i], delta));
                    o = __fadd_rn(o, __fmul_rn(S[i], qs[i]));
                }
            } else {
                float m4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int i = 0; i < DK; ++i) {
                    S[i] *= d;
                    m4[i & 3] = fmaf(S[i], ks[i], m4[i & 3]);
                }
                const float delta = (vj - ((m4[0] + m4[1]) + (m4[2] + m4[3]))) * b;
                float o4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int i = 0; i < DK; ++i) {
                    S[i] = fmaf(ks[i], delta, S[i]);
                    o4[i & 3] = fmaf(S[i], qs[i], o4[i & 3]);
                }
                o = (o4[0] + o4[1]) + (o4[2] + o4[3]);
            }
            a.out[(static_cast<size_t>(t) * a.nv + h) * a.dv + j] = o;
        }
        buf ^= 1;
    }
    if (sout && j < a.dv) {
        float *st = reinterpret_cast<float *>(sout);
#pragma unroll
        for (int i = 0; i < DK; ++i) st[(static_cast<size_t>(h) * DK + i) * a.dv + j] = S[i];
    }
}

// Split variant for DK = 128 (the reassociated, non-exact mode): SPLIT threads
// share one state column, thread `part` owning rows part, part + SPLIT, ...
// (so the threads of a column read different shared-memory banks); partial
// sums combine with shuffles (the threads of a column are adjacent lanes).
// Token inputs are prefetched PF tokens ahead into registers, so global load
// latency stays off the serial per-token chain.
template <int DK, int SPLIT, int PF>
__global__ void __launch_bounds__(128 * SPLIT) delta_recurrent_split_kernel(DeltaRecArgs a) {
    constexpr int R = DK / SPLIT;
    __shared__ float kq[2][2][DK];
    const int row = blockIdx.x, h = blockIdx.y;
    const int col = threadIdx.x / SPLIT, part = threadIdx.x % SPLIT;
    const int kh = h / (a.nv / a.nk);
    const int start = a.cu_seqlens[row], end = a.cu_seqlens[row + 1];
    if (start >= end) return;
    const bool active = col < a.dv;
    const int li = threadIdx.x;  // loader role: li < DK loads k[li], li < 2*DK loads q[li - DK]
    float S[R];
#pragma unroll
    for (int i = 0; i < R; ++i) S[i] = 0.f;
    float pkq[PF], pv[PF], pg[PF], pb[PF];
    auto fetch = [&](int u, int t) {
        if (li < DK)
            pkq[u] = a.k[(static_cast<size_t>(t) * a.nk + kh) * DK + li];
        else if (li < 2 * DK)
            pkq[u] = a.q[(static_cast<size_t>(t) * a.nk + kh) * DK + (li - DK)];
        pv[u] = active ? a.v[(static_cast<size_t>(t) * a.nv + h) * a.dv + col] : 0.f;
        pg[u] = a.g[static_cast<size_t>(t) * a.nv + h];
        pb[u] = a.beta[static_cast<size_t>(t) * a.nv + h];
    };
#pragma unroll
    for (int u = 0; u < PF; ++u)
        if (start + u < end) fetch(u, start + u);
    int buf = 0;
    for (int t0 = start; t0 < end; t0 += PF) {
#pragma unroll
        for (int u = 0; u < PF; ++u) {
            const int t = t0 + u;
            if (t >= end) break;
            if (li < 2 * DK) kq[buf][li / DK][li % DK] = pkq[u];
            const float vj = pv[u], d = expf(pg[u]), b = pb[u];
            __syncthreads();
            if (t + PF < end) fetch(u, t + PF);
            const float *ks = kq[buf][0] + part;
            const float *qs = kq[buf][1] + part;
            float m4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int i = 0; i < R; ++i) {
                S[i] *= d;
                m4[i & 3] = fmaf(S[i], ks[i * SPLIT], m4[i & 3]);
            }
            float m = (m4[0] + m4[1]) + (m4[2] + m4[3]);
#pragma unroll
            for (int o = 1; o < SPLIT; o <<= 1) m += __shfl_xor_sync(0xffffffffu, m, o);
            const float delta = (vj - m) * b;
            float o4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int i = 0; i < R; ++i) {
                S[i] = fmaf(ks[i * SPLIT], delta, S[i]);
                o4[i & 3] = fmaf(S[i], qs[i * SPLIT], o4[i & 3]);
            }
            float o = (o4[0] + o4[1]) + (o4[2] + o4[3]);
#pragma unroll
            for (int off = 1; off < SPLIT; off <<= 1) o += __shfl_xor_sync(0xffffffffu, o, off);
            if (active && part == 0) a.out[(static_cast<size_t>(t) * a.nv + h) * a.dv + col] = o;
            buf ^= 1;
        }
    }
}

// ------------------------------------------------------------------ gated norm
template <typename T>
__global__ void gated_norm_kernel(const float *__restrict__ o, const float *__restrict__ z, int ldz,
                                  const float *__restrict__ w, float eps, int n, int nv, int dv,
                                  T *__restrict__ out, int ldo, uint8_t *__restrict__ out_lo, int ldo_lo) {
    const int item = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (item >= n * nv) return;
    const int t = item / nv, h = item % nv;
    const float *src = o + static_cast<size_t>(item) * dv;
    float ss = 0.f;
    for (int i = lane; i < dv; i += 32) ss += src[i] * src[i];
    ss = warp_sum(ss);
    const float denom = sqrtf(ss / static_cast<float>(dv) + eps);
    const float *zr = z + static_cast<size_t>(t) * ldz + h * dv;
    T *dst = out + static_cast<size_t>(t) * ldo + h * dv;
    for (int i = lane; i < dv; i += 32) {
        const float y = ((src[i] / denom) * w[i]) * silu_f(zr[i]);
        dst[i] = Act<T>::from_f(y);
        if constexpr (sizeof(T) == 2) {
            if (out_lo) out_lo[static_cast<size_t>(t) * ldo_lo + h * dv + i] = lo_e5m2(y, dst[i]);
        }
    }
}

// ------------------------------------------------------------------ attention prep
// One warp per (token, head slot): slots [0, nh) are query heads, [nh, nh+nkv)
// key heads, [nh+nkv, nh+2nkv) value heads. The normalised row is staged in
// shared memory so RoPE can pair dims i and i + rd/2 for any head size.
template <typename T>
__global__ void attn_prep_kernel(AttnPrepArgs a) {
    extern __shared__ float rowbuf[];  // [warps][hd]
    const int warps = blockDim.x / 32;
    const int wid = threadIdx.x / 32, lane = threadIdx.x & 31;
    const int slots = a.nh + 2 * a.nkv;
    const int item = blockIdx.x * warps + wid;
    if (item >= a.n * slots) return;
    const int t = item / slots, slot = item % slots;
    const float *proj = a.proj + static_cast<size_t>(t) * a.ldp;
    float *buf = rowbuf + wid * a.hd;
    if (slot >= a.nh + a.nkv) {  // value head: convert
        const int h = slot - a.nh - a.nkv;
        const float *src = proj + a.nh * 2 * a.hd + a.nkv * a.hd + h * a.hd;
        const int row = a.tok_row[t];
        const int kvs = kv_slot(a.pages, row, t - a.pos[t], a.pos[t]);
        T *dst = static_cast<T *>(a.v) + (static_cast<size_t>(kvs) * a.nkv + h) * a.hd;
        for (int i = lane; i < a.hd; i += 32) dst[i] = Act<T>::from_f(src[i]);
        return;
    }
    const bool is_q = slot < a.nh;
    const int h = is_q ? slot : slot - a.nh;
    const float *src = is_q ? proj + h * 2 * a.hd : proj + a.nh * 2 * a.hd + h * a.hd;
    const float *w = is_q ? a.qn_w : a.kn_w;
    float ss = 0.f;
    for (int i = lane; i < a.hd; i += 32) ss += src[i] * src[i];
    ss = warp_sum(ss);
    const float denom = sqrtf(ss / static_cast<float>(a.hd) + a.eps);
    for (int i = lane; i < a.hd; i += 32) buf[i] = (src[i] / denom) * w[i];
    __syncwarp();
    const float p = static_cast<float>(a.pos[t] + (a.pre_len ? a.pre_len[a.tok_row[t]] : 0));
    const int half = a.rd / 2;
    const int kvs = is_q ? t : kv_slot(a.pages, a.tok_row[t], t - a.pos[t], a.pos[t]);
    T *dst = (is_q ? static_cast<T *>(a.q) + (static_cast<size_t>(t) * a.nh + h) * a.hd
                   : static_cast<T *>(a.k) + (static_cast<size_t>(kvs) * a.nkv + h) * a.hd);
    for (int i = lane; i < a.hd; i += 32) {
        float r = buf[i];
        if (i < a.rd) {
            const int fi = i < half ? i : i - half;
            const float ang = p * a.inv_freq[fi];
            float c, sn;
            sincosf(ang, &sn, &c);
            const float rot = i < half ? -buf[i + half] : buf[i - half];
            r = r * c + rot * sn;
        }
        dst[i] = Act<T>::from_f(r);
    }
}

// The same input stage with one warp per token: each lane holds 4 consecutive
// dims of every head (float4 loads, 8- or 16-byte stores), the token's rotary
// cos/sin are computed once for all heads, and the rotate-half partner dims
// come from another lane by shuffle. Per element the arithmetic is that of
// attn_prep_kernel. HD = 128 or 256; rd a multiple of 8 and <= 128.
template <typename T, int HD>
__global__ void attn_prep_vec_kernel(AttnPrepArgs a) {
    constexpr int NCH = HD / 128;  // float4 chunks per lane and head
    const long t_l = (static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (t_l >= a.n) return;
    const int t = static_cast<int>(t_l);
    const float *proj = a.proj + static_cast<size_t>(t) * a.ldp;
    const int row = a.tok_row[t];
    const int kvs = kv_slot(a.pages, row, t - a.pos[t], a.pos[t]);
    const float pos = static_cast<float>(a.pos[t] + (a.pre_len ? a.pre_len[row] : 0));
    const int half = a.rd / 2, qh = half / 4;  // lanes per rotary half
    const bool rot_lane = lane < a.rd / 4;
    const int partner = lane < qh ? lane + qh : lane - qh;
    float cs[4] = {1.f, 1.f, 1.f, 1.f}, sn[4] = {0.f, 0.f, 0.f, 0.f};
    if (rot_lane) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int i = 4 * lane + j, fi = i < half ? i : i - half;
            sincosf(pos * a.inv_freq[fi], &sn[j], &cs[j]);
        }
    }
    auto ld4 = [](const float *p) { return *reinterpret_cast<const float4 *>(p); };
    auto st4 = [](T *dst, const float (&v)[4]) {
        if constexpr (sizeof(T) == 4) {
            *reinterpret_cast<float4 *>(dst) = make_float4(v[0], v[1], v[2], v[3]);
        } else {
            const __half2 a2 = __floats2half2_rn(v[0], v[1]), b2 = __floats2half2_rn(v[2], v[3]);
            *reinterpret_cast<uint2 *>(dst) =
                make_uint2(*reinterpret_cast<const uint32_t *>(&a2), *reinterpret_cast<const uint32_t *>(&b2));
        }
    };
    float4 wq[NCH], wk[NCH];
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
        wq[c] = ld4(a.qn_w + 128 * c + 4 * lane);
        wk[c] = ld4(a.kn_w + 128 * c + 4 * lane);
    }
    auto norm_rope = [&](const float *src, const float4 (&w)[NCH], T *dst) {
        float x[NCH][4];
        float ss = 0.f;
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
            const float4 v = ld4(src + 128 * c + 4 * lane);
            x[c][0] = v.x, x[c][1] = v.y, x[c][2] = v.z, x[c][3] = v.w;
#pragma unroll
            for (int j = 0; j < 4; ++j) ss += x[c][j] * x[c][j];
        }
        ss = warp_sum(ss);
        const float denom = sqrtf(ss / static_cast<float>(HD) + a.eps);
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
            const float wv[4] = {w[c].x, w[c].y, w[c].z, w[c].w};
#pragma unroll
            for (int j = 0; j < 4; ++j) x[c][j] = (x[c][j] / denom) * wv[j];
        }
        float o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) o[j] = __shfl_sync(0xffffffffu, x[0][j], partner);
        if (rot_lane) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float rot = lane < qh ? -o[j] : o[j];
                x[0][j] = x[0][j] * cs[j] + rot * sn[j];
            }
        }
#pragma unroll
        for (int c = 0; c < NCH; ++c) st4(dst + 128 * c + 4 * lane, x[c]);
    };
    for (int h = 0; h < a.nh; ++h)
        norm_rope(proj + h * 2 * HD, wq, static_cast<T *>(a.q) + (static_cast<size_t>(t) * a.nh + h) * HD);
    const float *kp = proj + a.nh * 2 * HD, *vp = kp + a.nkv * HD;
    for (int h = 0; h < a.nkv; ++h)
        norm_rope(kp + h * HD, wk, static_cast<T *>(a.k) + (static_cast<size_t>(kvs) * a.nkv + h) * HD);
    for (int h = 0; h < a.nkv; ++h) {
        T *dst = static_cast<T *>(a.v) + (static_cast<size_t>(kvs) * a.nkv + h) * HD;
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
            const float4 v = ld4(vp + h * HD + 128 * c + 4 * lane);
            const float vv[4] = {v.x, v.y, v.z, v.w};
            st4(dst + 128 * c + 4 * lane, vv);
        }
    }
}

// ------------------------------------------------------------------ attention (SIMT)
// One warp per (query token, query head), online softmax over the keys of
// its row up to itself; used for the fp32 model and for head sizes the
// tensor-core kernel does not take.
template <typename T>
__global__ void attn_simt_kernel(AttnArgs a) {
    const int warps = blockDim.x / 32;
    const int item = blockIdx.x * warps + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (item >= a.n * a.nh) return;
    const int t = item / a.nh, h = item % a.nh;
    const int row = a.tok_row[t];
    const int start = a.cu_seqlens[row];
    const int kh = h / (a.nh / a.nkv);
    constexpr int MAXE = 8;  // hd <= 256
    float qv[MAXE], acc[MAXE];
    const T *q = static_cast<const T *>(a.q) + (static_cast<size_t>(t) * a.nh + h) * a.hd;
#pragma unroll
    for (int e = 0; e < MAXE; ++e) {
        const int i = lane + 32 * e;
        qv[e] = i < a.hd ? Act<T>::to_f(q[i]) : 0.f;
        acc[e] = 0.f;
    }
    const float scale = 1.0f / sqrtf(static_cast<float>(a.hd));
    float m = -INFINITY, l = 0.f;
    // Keys: the row's cached prefix (P tokens) then its own tokens up to t.
    const int P = a.pre_len ? a.pre_len[row] : 0;
    const T *ck = P ? reinterpret_cast<const T *>(a.kv_in[row]) : nullptr;
    const T *cv = P ? ck + static_cast<size_t>(P) * a.nkv * a.hd : nullptr;
    for (int s = start - P; s <= t; ++s) {
        const int kvs = s >= start ? kv_slot(a.pages, row, start, s - start) : 0;
        const T *k = s >= start ? static_cast<const T *>(a.k) + (static_cast<size_t>(kvs) * a.nkv + kh) * a.hd
                                : ck + (static_cast<size_t>(s - start + P) * a.nkv + kh) * a.hd;
        float dot = 0.f;
#pragma unroll
        for (int e = 0; e < MAXE; ++e) {
            const int i = lane + 32 * e;
            if (i < a.hd) dot += qv[e] * Act<T>::to_f(k[i]);
        }
        dot = warp_sum(dot) * scale;
        const float mn = fmaxf(m, dot);
        const float corr = expf(m - mn);
        const float pw = expf(dot - mn);
        l = l * corr + pw;
        const T *v = s >= start ? static_cast<const T *>(a.v) + (static_cast<size_t>(kvs) * a.nkv + kh) * a.hd
                                : cv + (static_cast<size_t>(s - start + P) * a.nkv + kh) * a.hd;
#pragma unroll
        for (int e = 0; e < MAXE; ++e) {
            const int i = lane + 32 * e;
            if (i < a.hd) acc[e] = acc[e] * corr + pw * Act<T>::to_f(v[i]);
        }
        m = mn;
    }
    const float *gate = a.proj + static_cast<size_t>(t) * a.ldp + h * 2 * a.hd + a.hd;
    T *dst = static_cast<T *>(a.out) + static_cast<size_t>(t) * a.ldo + h * a.hd;
#pragma unroll
    for (int e = 0; e < MAXE; ++e) {
        const int i = lane + 32 * e;
        if (i < a.hd) dst[i] = Act<T>::from_f((acc[e] / l) * sigmoid_f(gate[i]));
    }
}

// ------------------------------------------------------------------ swiglu
template <typename T>
__global__ void swiglu_kernel(const float *__restrict__ gu, int ldg, int n, int f, T *__restrict__ out,
                              int ldo, uint8_t *__restrict__ out_lo, int ldo_lo) {
    const size_t total = static_cast<size_t>(n) * f;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t t = i / f, j = i % f;
        const float y = silu_f(gu[t * ldg + j]) * gu[t * ldg + f + j];
        out[t * ldo + j] = Act<T>::from_f(y);
        if constexpr (sizeof(T) == 2) {
            if (out_lo) out_lo[t * ldo_lo + j] = lo_e5m2(y, out[t * ldo + j]);
        }
    }
}

// ------------------------------------------------------------------ int8 expand
// 16 int8 values per thread and iteration: one 16-byte load, two 16-byte stores.
__global__ void expand_i8_kernel(const int8_t *__restrict__ q, size_t n16, __half *__restrict__ out,
                                 uint8_t *__restrict__ out8) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n16;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const int4 v = __ldcs(reinterpret_cast<const int4 *>(q) + i);
        const int w[4] = {v.x, v.y, v.z, v.w};
        __align__(16) __half h[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) h[j] = __int2half_rn(static_cast<int8_t>(w[j >> 2] >> (8 * (j & 3))));
        uint4 *o = reinterpret_cast<uint4 *>(out) + 2 * i;
        o[0] = *reinterpret_cast<const uint4 *>(&h[0]);
        o[1] = *reinterpret_cast<const uint4 *>(&h[8]);
        if (out8) {
            __align__(16) uint8_t e[16];
#pragma unroll
            for (int j = 0; j < 16; ++j)
                e[j] = static_cast<uint8_t>(__nv_cvt_halfraw_to_fp8(h[j], __NV_SATFINITE, __NV_E4M3));
            reinterpret_cast<uint4 *>(out8)[i] = *reinterpret_cast<const uint4 *>(e);
        }
    }
}

__global__ void expand_i8_tail_kernel(const int8_t *__restrict__ q, size_t from, size_t n, __half *__restrict__ out,
                                      uint8_t *__restrict__ out8) {
    for (size_t i = from + blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        out[i] = __int2half_rn(q[i]);
        if (out8) out8[i] = static_cast<uint8_t>(__nv_cvt_halfraw_to_fp8(out[i], __NV_SATFINITE, __NV_E4M3));
    }
}

// ------------------------------------------------------------------ readout
__global__ void readout_norm_kernel(const float *__restrict__ x, int hidden, const float *__restrict__ w,
                                    float eps, const int32_t *__restrict__ idx, int rows,
                                    float *__restrict__ out) {
    const int r = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (r >= rows) return;
    const float *xr = x + static_cast<size_t>(idx[r]) * hidden;
    float ss = 0.f;
    for (int i = lane; i < hidden; i += 32) ss += xr[i] * xr[i];
    ss = warp_sum(ss);
    const float denom = sqrtf(ss / static_cast<float>(hidden) + eps);
    for (int i = lane; i < hidden; i += 32) out[static_cast<size_t>(r) * hidden + i] = (xr[i] / denom) * w[i];
}

// y[r, j] = W[j, :] . h[r, :] + b[j]; one warp per output element (coalesced W rows).
__global__ void readout_proj_kernel(const float *__restrict__ h, int hidden, const float *__restrict__ W,
                                    const float *__restrict__ bias, int dp, int rows,
                                    float *__restrict__ y) {
    const int warps = blockDim.x / 32;
    const int j = blockIdx.x * warps + threadIdx.x / 32;
    const int r = blockIdx.y;
    const int lane = threadIdx.x & 31;
    if (j >= dp || r >= rows) return;
    const float *hr = h + static_cast<size_t>(r) * hidden;
    const float *wr = W + static_cast<size_t>(j) * hidden;
    float s = 0.f;
    for (int i = lane; i < hidden; i += 32) s += wr[i] * hr[i];
    s = warp_sum(s);
    if (lane == 0) y[static_cast<size_t>(r) * dp + j] = s + bias[j];
}

__global__ void pointer_logits_kernel(const float *__restrict__ proj, int dp, int n_dec,
                                      const int32_t *__restrict__ opt_dec, int n_opt, float scale,
                                      float *__restrict__ logits) {
    const int o = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (o >= n_opt) return;
    const int d = opt_dec[o];
    if (d < 0 || d >= n_dec) {  // no decision row to pair with: a NaN logit, no read
        if (lane == 0) logits[o] = __int_as_float(0x7fc00000);
        return;
    }
    const float *k = proj + static_cast<size_t>(n_dec + o) * dp;
    const float *q = proj + static_cast<size_t>(d) * dp;
    float s = 0.f;
    for (int i = lane; i < dp; i += 32) s += k[i] * q[i];
    s = warp_sum(s);
    if (lane == 0) logits[o] = s * scale;
}

}  // namespace

// ====================================================================== launchers
void launch_embed(int act, const uint32_t *ids, int n, const void *table, int hidden, float *x,
                  cudaStream_t s) {
    if (n <= 0) return;
    if (act == kActF32)
        embed_kernel<float><<<n, 256, 0, s>>>(ids, n, static_cast<const float *>(table), hidden, x);
    else
        embed_kernel<__half><<<n, 256, 0, s>>>(ids, n, static_cast<const __half *>(table), hidden, x);
    HK_LAUNCH_CHECK();
}

void launch_rmsnorm(int act, const float *x, int ldx, const float *w_eff, float eps, int rows,
                    int hidden, void *out, int ldo, cudaStream_t s, uint8_t *out_lo, int ldo_lo) {
    if (rows <= 0) return;
    if (act == kActF32) out_lo = nullptr;
    const int grid = ceil_div(rows, 8);
    const bool vec = (ldx % 4) == 0 && (ldo % 4) == 0 && (hidden % 128) == 0;
#define HK_RMS_REG(NCH)                                                                                          \
    if (vec && hidden == 128 * (NCH)) {                                                                          \
        if (act == kActF32)                                                                                      \
            rmsnorm_reg_kernel<float, NCH><<<grid, 256, 0, s>>>(x, ldx, w_eff, eps, rows, static_cast<float *>(out), \
                                                                ldo, nullptr, 0);                                \
        else                                                                                                     \
            rmsnorm_reg_kernel<__half, NCH><<<grid, 256, 0, s>>>(x, ldx, w_eff, eps, rows,                        \
                                                                 static_cast<__half *>(out), ldo, out_lo, ldo_lo); \
        HK_LAUNCH_CHECK();                                                                                       \
        return;                                                                                                  \
    }
    HK_RMS_REG(8)
    HK_RMS_REG(16)
    HK_RMS_REG(20)
    HK_RMS_REG(24)
    HK_RMS_REG(32)
#undef HK_RMS_REG
    if (act == kActF32)
        rmsnorm_kernel<float><<<grid, 256, 0, s>>>(x, ldx, w_eff, eps, rows, hidden, static_cast<float *>(out), ldo,
                                                   nullptr, 0);
    else
        rmsnorm_kernel<__half><<<grid, 256, 0, s>>>(x, ldx, w_eff, eps, rows, hidden, static_cast<__half *>(out),
                                                    ldo, out_lo, ldo_lo);
    HK_LAUNCH_CHECK();
}

// ------------------------------------------------------------------ snapshots
// Conv history for a row's output snapshot: the last H = taps-1 entries of
// [hist_in (H rows) ; own qkv rows (L)], i.e. concat index L + hrow.
__global__ void conv_history_kernel(const float *proj, int ldp, int conv_dim, int taps, const int32_t *cu,
                                    const uint64_t *hist_in, const uint64_t *hist_out) {
    const int r = blockIdx.x;
    const uint64_t oaddr = hist_out[r];
    if (!oaddr) return;
    const int start = cu[r], L = cu[r + 1] - start, H = taps - 1;
    const float *in = reinterpret_cast<const float *>(hist_in ? hist_in[r] : 0);
    float *out = reinterpret_cast<float *>(oaddr);
    for (int i = blockIdx.y * blockDim.x + threadIdx.x; i < H * conv_dim; i += gridDim.y * blockDim.x) {
        const int hrow = i / conv_dim, c = i % conv_dim, q = L + hrow;
        out[i] = q < H ? (in ? in[static_cast<size_t>(q) * conv_dim + c] : 0.f)
                       : proj[static_cast<size_t>(start + q - H) * ldp + c];
    }
}

// K/V of a row's output snapshot: prefix keys from kv_in, then own keys from
// the workspace slots; one CTA per (row, block of key positions).
template <typename T>
__global__ void kv_store_kernel(AttnArgs a, const uint64_t *kv_out) {
    const int r = blockIdx.x;
    const uint64_t oaddr = kv_out[r];
    if (!oaddr) return;
    const int start = a.cu_seqlens[r], L = a.cu_seqlens[r + 1] - start;
    const int P = a.pre_len ? a.pre_len[r] : 0, total = P + L;
    const size_t unit = static_cast<size_t>(a.nkv) * a.hd;
    const T *ck = P ? reinterpret_cast<const T *>(a.kv_in[r]) : nullptr;
    T *ok = reinterpret_cast<T *>(oaddr), *ov = ok + static_cast<size_t>(total) * unit;
    for (size_t i = blockIdx.y * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total * unit;
         i += static_cast<size_t>(gridDim.y) * blockDim.x) {
        const int j = static_cast<int>(i / unit);
        const size_t e = i % unit;
        T kx, vx;
        if (j < P) {
            kx = ck[static_cast<size_t>(j) * unit + e];
            vx = ck[static_cast<size_t>(P + j) * unit + e];
        } else {
            const size_t slot = static_cast<size_t>(kv_slot(a.pages, r, start, j - P));
            kx = static_cast<const T *>(a.k)[slot * unit + e];
            vx = static_cast<const T *>(a.v)[slot * unit + e];
        }
        ok[i] = kx;
        ov[i] = vx;
    }
}

void launch_conv_history(const float *proj, int ldp, int conv_dim, int taps, const int32_t *cu_seqlens, int n_rows,
                         const uint64_t *hist_in, const uint64_t *hist_out, cudaStream_t s) {
    if (n_rows <= 0 || !hist_out || taps <= 1) return;
    dim3 grid(n_rows, ceil_div((taps - 1) * conv_dim, 256 * 4));
    conv_history_kernel<<<grid, 256, 0, s>>>(proj, ldp, conv_dim, taps, cu_seqlens, hist_in, hist_out);
    HK_LAUNCH_CHECK();
}

void launch_kv_store(int act, const AttnArgs &a, const uint64_t *kv_out, cudaStream_t s) {
    if (a.n_rows <= 0 || !kv_out) return;
    dim3 grid(a.n_rows, 64);
    if (act == kActF32)
        kv_store_kernel<float><<<grid, 256, 0, s>>>(a, kv_out);
    else
        kv_store_kernel<__half><<<grid, 256, 0, s>>>(a, kv_out);
    HK_LAUNCH_CHECK();
}

void launch_delta_prep(const DeltaPrepArgs &a, cudaStream_t s) {
    if (a.n <= 0) return;
    if (a.dk == 128 && a.dv == 128 && a.taps == 4 && a.nv <= 32 && (a.ldp % 4) == 0) {
        constexpr int TB = 16;
        const long warps = static_cast<long>((a.n + TB - 1) / TB) * (2 * a.nk + a.nv + 1);
        if (a.fast)
            delta_prep_vec_kernel<TB, true><<<ceil_div(warps, 8), 256, 0, s>>>(a);
        else
            delta_prep_vec_kernel<TB, false><<<ceil_div(warps, 8), 256, 0, s>>>(a);
        HK_LAUNCH_CHECK();
        return;
    }
    const size_t smem = sizeof(float) * (2 * a.nk * a.dk + a.nv * a.dv);
    HK_CUDA(cudaFuncSetAttribute(delta_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem)));
    delta_prep_kernel<<<a.n, 256, smem, s>>>(a);
    HK_LAUNCH_CHECK();
}

template <int DK>
static void launch_rec_dk(const DeltaRecArgs &a, cudaStream_t s) {
    if (DK == 128 && !a.exact && a.dv <= 128 && !a.state_in && !a.state_out) {
        dim3 grid(a.n_rows, a.nv);
        delta_recurrent_split_kernel<128, 4, 4><<<grid, 512, 0, s>>>(a);
        return;
    }
    const int threads = a.dv <= 32 ? 32 : (a.dv <= 64 ? 64 : 128);
    dim3 grid(a.n_rows, a.nv);
    if (a.exact)
        delta_recurrent_kernel<DK, true><<<grid, threads, 0, s>>>(a);
    else
        delta_recurrent_kernel<DK, false><<<grid, threads, 0, s>>>(a);
}

void launch_delta_recurrent(const DeltaRecArgs &a, cudaStream_t s) {
    if (a.n_rows <= 0) return;
    if (!a.exact && !a.state_in && !a.state_out && delta_tc_supported(a)) {
        launch_delta_tc(a, s);
        return;
    }
    if (a.dv > 128) throw CudaError("delta recurrence supports value heads up to 128 wide");
    switch (a.dk) {
        case 4: launch_rec_dk<4>(a, s); break;
        case 8: launch_rec_dk<8>(a, s); break;
        case 16: launch_rec_dk<16>(a, s); break;
        case 32: launch_rec_dk<32>(a, s); break;
        case 64: launch_rec_dk<64>(a, s); break;
        case 128: launch_rec_dk<128>(a, s); break;
        default: throw CudaError("delta recurrence supports key heads of 4..128 (powers of two)");
    }
    HK_LAUNCH_CHECK();
}

void launch_gated_norm(int act, const float *o, const float *z, int ldz, const float *w, float eps,
                       int n, int nv, int dv, void *out, int ldo, cudaStream_t s, uint8_t *out_lo, int ldo_lo) {
    if (n <= 0) return;
    const int grid = ceil_div(static_cast<long>(n) * nv, 8);
    if (act == kActF32)
        gated_norm_kernel<float><<<grid, 256, 0, s>>>(o, z, ldz, w, eps, n, nv, dv, static_cast<float *>(out), ldo,
                                                      nullptr, 0);
    else
        gated_norm_kernel<__half><<<grid, 256, 0, s>>>(o, z, ldz, w, eps, n, nv, dv, static_cast<__half *>(out), ldo,
                                                       out_lo, ldo_lo);
    HK_LAUNCH_CHECK();
}

void launch_attn_prep(int act, const AttnPrepArgs &a, cudaStream_t s) {
    if (a.n <= 0) return;
    if ((a.hd == 128 || a.hd == 256) && a.rd % 8 == 0 && a.rd >= 8 && a.rd <= 128 && a.ldp % 4 == 0) {
        const int grid = ceil_div(static_cast<long>(a.n), 8);
        if (act == kActF32) {
            if (a.hd == 256)
                attn_prep_vec_kernel<float, 256><<<grid, 256, 0, s>>>(a);
            else
                attn_prep_vec_kernel<float, 128><<<grid, 256, 0, s>>>(a);
        } else {
            if (a.hd == 256)
                attn_prep_vec_kernel<__half, 256><<<grid, 256, 0, s>>>(a);
            else
                attn_prep_vec_kernel<__half, 128><<<grid, 256, 0, s>>>(a);
        }
        HK_LAUNCH_CHECK();
        return;
    }
    const int slots = a.nh + 2 * a.nkv;
    const int grid = ceil_div(static_cast<long>(a.n) * slots, 8);
    const size_t smem = sizeof(float) * 8 * a.hd;
    if (act == kActF32)
        attn_prep_kernel<float><<<grid, 256, smem, s>>>(a);
    else
        attn_prep_kernel<__half><<<grid, 256, smem, s>>>(a);
    HK_LAUNCH_CHECK();
}

void launch_attention(int act, const AttnArgs &a, cudaStream_t s) {
    if (a.n <= 0) return;
    if (a.hd > 256) throw CudaError("attention supports head_dim up to 256");
    if (act == kActF16 && attention_t5_supported(a)) {
        launch_attention_t5(a, s);
        return;
    }
    if (act == kActF16 && attention_tc_supported(a.hd)) {
        launch_attention_tc(a, s);
        return;
    }
    const int grid = ceil_div(static_cast<long>(a.n) * a.nh, 8);
    if (act == kActF32)
        attn_simt_kernel<float><<<grid, 256, 0, s>>>(a);
    else
        attn_simt_kernel<__half><<<grid, 256, 0, s>>>(a);
    HK_LAUNCH_CHECK();
}

void launch_expand_i8(const int8_t *q, size_t n, __half *out, uint8_t *out8, cudaStream_t s) {
    if (n == 0) return;
    const bool aligned = (reinterpret_cast<uintptr_t>(q) % 16) == 0 && (reinterpret_cast<uintptr_t>(out) % 16) == 0 &&
                         (reinterpret_cast<uintptr_t>(out8) % 16) == 0;
    const size_t n16 = aligned ? n / 16 : 0;
    if (n16) {
        const size_t blocks = (n16 + 255) / 256;
        expand_i8_kernel<<<static_cast<int>(blocks < 148 * 8 ? blocks : 148 * 8), 256, 0, s>>>(q, n16, out, out8);
        HK_LAUNCH_CHECK();
    }
    if (n16 * 16 < n) {  // the last n % 16 values, or all of them when unaligned
        const size_t rest = n - n16 * 16, blocks = (rest + 255) / 256;
        expand_i8_tail_kernel<<<static_cast<int>(blocks < 148 * 8 ? blocks : 148 * 8), 256, 0, s>>>(q, n16 * 16, n,
                                                                                                  out, out8);
        HK_LAUNCH_CHECK();
    }
}

void launch_swiglu(int act, const float *gu, int ldg, int n, int f, void *out, int ldo, cudaStream_t s,
                   uint8_t *out_lo, int ldo_lo) {
    if (n <= 0) return;
    const long total = static_cast<long>(n) * f;
    const int grid = static_cast<int>(total / 256 + 1 < 148 * 16 ? total / 256 + 1 : 148 * 16);
    if (act == kActF32)
        swiglu_kernel<float><<<grid, 256, 0, s>>>(gu, ldg, n, f, static_cast<float *>(out), ldo, nullptr, 0);
    else
        swiglu_kernel<__half><<<grid, 256, 0, s>>>(gu, ldg, n, f, static_cast<__half *>(out), ldo, out_lo, ldo_lo);
    HK_LAUNCH_CHECK();
}

void launch_readout(const ReadoutArgs &a, cudaStream_t s) {
    const int rows = a.n_dec + a.n_opt;
    if (a.n_opt <= 0) return;
    readout_norm_kernel<<<ceil_div(rows, 8), 256, 0, s>>>(a.x, a.hidden, a.final_w, a.eps, a.idx, rows, a.hn);
    HK_LAUNCH_CHECK();
    dim3 gq(ceil_div(a.dp, 8), a.n_dec);
    readout_proj_kernel<<<gq, 256, 0, s>>>(a.hn, a.hidden, a.wq, a.bq, a.dp, a.n_dec, a.proj);
    HK_LAUNCH_CHECK();
    dim3 gk(ceil_div(a.dp, 8), a.n_opt);
    readout_proj_kernel<<<gk, 256, 0, s>>>(a.hn + static_cast<size_t>(a.n_dec) * a.hidden, a.hidden, a.wk,
                                           a.bk, a.dp, a.n_opt,
                                           a.proj + static_cast<size_t>(a.n_dec) * a.dp);
    HK_LAUNCH_CHECK();
    pointer_logits_kernel<<<ceil_div(a.n_opt, 8), 256, 0, s>>>(a.proj, a.dp, a.n_dec, a.opt_dec, a.n_opt,
                                                              a.scale, a.logits);
    HK_LAUNCH_CHECK();
}

}  // namespace hk
