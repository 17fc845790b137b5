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
                               float eps, int rows, int hidden, T *__restrict__ out, int ldo) {
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
    for (int i = lane; i < hidden; i += 32) o[i] = Act<T>::from_f((xr[i] / denom) * w[i]);
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
    for (int c = threadIdx.x; c < conv_dim; c += blockDim.x) {
        float acc = 0.f;
        for (int tap = 0; tap < a.taps; ++tap) {
            const int shift = a.taps - 1 - tap;
            if (shift > pos) continue;
            const float xv = proj[static_cast<size_t>(t - shift) * a.ldp + c];
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
    float S[DK];
#pragma unroll
    for (int i = 0; i < DK; ++i) S[i] = 0.f;
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
}

// ------------------------------------------------------------------ gated norm
template <typename T>
__global__ void gated_norm_kernel(const float *__restrict__ o, const float *__restrict__ z, int ldz,
                                  const float *__restrict__ w, float eps, int n, int nv, int dv,
                                  T *__restrict__ out, int ldo) {
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
    for (int i = lane; i < dv; i += 32) dst[i] = Act<T>::from_f(((src[i] / denom) * w[i]) * silu_f(zr[i]));
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
        T *dst = static_cast<T *>(a.v) + (static_cast<size_t>(t) * a.nkv + h) * a.hd;
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
    const float p = static_cast<float>(a.pos[t]);
    const int half = a.rd / 2;
    T *dst = (is_q ? static_cast<T *>(a.q) + (static_cast<size_t>(t) * a.nh + h) * a.hd
                   : static_cast<T *>(a.k) + (static_cast<size_t>(t) * a.nkv + h) * a.hd);
    for (int i = lane; i < a.hd; i += 32) {
        float r = buf[i];
        if (i < a.rd) {
            const int fi = i < half ? i : i - half;
            const float ang = p * a.inv_freq[fi];
            const float c = cosf(ang), sn = sinf(ang);
            const float rot = i < half ? -buf[i + half] : buf[i - half];
            r = r * c + rot * sn;
        }
        dst[i] = Act<T>::from_f(r);
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
    for (int s = start; s <= t; ++s) {
        const T *k = static_cast<const T *>(a.k) + (static_cast<size_t>(s) * a.nkv + kh) * a.hd;
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
        const T *v = static_cast<const T *>(a.v) + (static_cast<size_t>(s) * a.nkv + kh) * a.hd;
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
                              int ldo) {
    const size_t total = static_cast<size_t>(n) * f;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t t = i / f, j = i % f;
        out[t * ldo + j] = Act<T>::from_f(silu_f(gu[t * ldg + j]) * gu[t * ldg + f + j]);
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
    const float *k = proj + static_cast<size_t>(n_dec + o) * dp;
    const float *q = proj + static_cast<size_t>(opt_dec[o]) * dp;
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
                    int hidden, void *out, int ldo, cudaStream_t s) {
    if (rows <= 0) return;
    const int grid = ceil_div(rows, 8);
    if (act == kActF32)
        rmsnorm_kernel<float><<<grid, 256, 0, s>>>(x, ldx, w_eff, eps, rows, hidden, static_cast<float *>(out), ldo);
    else
        rmsnorm_kernel<__half><<<grid, 256, 0, s>>>(x, ldx, w_eff, eps, rows, hidden, static_cast<__half *>(out),
                                                    ldo);
    HK_LAUNCH_CHECK();
}

void launch_delta_prep(const DeltaPrepArgs &a, cudaStream_t s) {
    if (a.n <= 0) return;
    const size_t smem = sizeof(float) * (2 * a.nk * a.dk + a.nv * a.dv);
    HK_CUDA(cudaFuncSetAttribute(delta_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem)));
    delta_prep_kernel<<<a.n, 256, smem, s>>>(a);
    HK_LAUNCH_CHECK();
}

template <int DK>
static void launch_rec_dk(const DeltaRecArgs &a, cudaStream_t s) {
    const int threads = a.dv <= 32 ? 32 : (a.dv <= 64 ? 64 : 128);
    dim3 grid(a.n_rows, a.nv);
    if (a.exact)
        delta_recurrent_kernel<DK, true><<<grid, threads, 0, s>>>(a);
    else
        delta_recurrent_kernel<DK, false><<<grid, threads, 0, s>>>(a);
}

void launch_delta_recurrent(const DeltaRecArgs &a, cudaStream_t s) {
    if (a.n_rows <= 0) return;
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
                       int n, int nv, int dv, void *out, int ldo, cudaStream_t s) {
    if (n <= 0) return;
    const int grid = ceil_div(static_cast<long>(n) * nv, 8);
    if (act == kActF32)
        gated_norm_kernel<float><<<grid, 256, 0, s>>>(o, z, ldz, w, eps, n, nv, dv, static_cast<float *>(out), ldo);
    else
        gated_norm_kernel<__half><<<grid, 256, 0, s>>>(o, z, ldz, w, eps, n, nv, dv, static_cast<__half *>(out), ldo);
    HK_LAUNCH_CHECK();
}

void launch_attn_prep(int act, const AttnPrepArgs &a, cudaStream_t s) {
    if (a.n <= 0) return;
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
    const int grid = ceil_div(static_cast<long>(a.n) * a.nh, 8);
    if (act == kActF32)
        attn_simt_kernel<float><<<grid, 256, 0, s>>>(a);
    else
        attn_simt_kernel<__half><<<grid, 256, 0, s>>>(a);
    HK_LAUNCH_CHECK();
}

void launch_swiglu(int act, const float *gu, int ldg, int n, int f, void *out, int ldo, cudaStream_t s) {
    if (n <= 0) return;
    const long total = static_cast<long>(n) * f;
    const int grid = static_cast<int>(total / 256 + 1 < 148 * 16 ? total / 256 + 1 : 148 * 16);
    if (act == kActF32)
        swiglu_kernel<float><<<grid, 256, 0, s>>>(gu, ldg, n, f, static_cast<float *>(out), ldo);
    else
        swiglu_kernel<__half><<<grid, 256, 0, s>>>(gu, ldg, n, f, static_cast<__half *>(out), ldo);
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
