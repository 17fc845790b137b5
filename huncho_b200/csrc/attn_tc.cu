// Causal varlen GQA attention with the Qwen3.5 output gate, on tensor cores
// (mma.sync m16n8k16, fp16 operands, fp32 accumulation), flash-style.
//
// Computes softmax(q k^T / sqrt(hd) + causal mask) v per row and query head,
// with query head h reading kv head h / (nh / nkv) (qwen3_5.rs:669-702), then
// multiplies by sigmoid(gate) (qwen3_5.rs:711-714) and stores the fp16 input of
// o_proj. One CTA handles 64 queries of one (row, query head): 4 warps x 16
// query rows; key/value tiles of 64 keys stream through shared memory with
// cp.async; scores, online softmax state and the output accumulator stay in
// registers. Rows are packed (cu_seqlens), so no padding is ever computed.
// Keys and values are read through kv_slot(): flat, or fixed-size pages in
// block-table order (the same math, kv_pages.rs:36-103).
#include <math.h>

#include "common.cuh"
#include "layers.cuh"

namespace hk {
namespace {

constexpr int BQ = 64, BKV = 64, THREADS = 128;

__device__ __forceinline__ uint32_t saddr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src, bool valid) {
    const int n = valid ? 16 : 0;  // zero-fill rows outside the sequence
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(saddr(dst)), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3, const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(saddr(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3, const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(saddr(p)));
}

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
}

template <int HD>
__global__ void __launch_bounds__(THREADS, 2) attn_tc_kernel(AttnArgs a) {
    constexpr int LD = HD + 8;  // padded row (halfs): conflict-free ldmatrix
    constexpr int NT = HD / 8;  // output n-tiles per warp
    extern __shared__ __align__(16) __half smem[];
    __half *sQ = smem;
    __half *sK = sQ + BQ * LD;
    __half *sV = sK + BKV * LD;

    const int row = blockIdx.z, h = blockIdx.y, q0 = blockIdx.x * BQ;
    const int start = a.cu_seqlens[row];
    const int len = a.cu_seqlens[row + 1] - start;
    if (q0 >= len) return;
    const int kh = h / (a.nh / a.nkv);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t4 = lane & 3;

    const __half *Q = static_cast<const __half *>(a.q);
    const __half *K = static_cast<const __half *>(a.k);
    const __half *V = static_cast<const __half *>(a.v);
    // A continued row's first P keys are its cached prefix; key indices below
    // are absolute (prefix first), queries are the row's own tokens.
    const int P = a.pre_len ? a.pre_len[row] : 0;
    const __half *CK = P ? reinterpret_cast<const __half *>(a.kv_in[row]) : nullptr;
    const __half *CV = P ? CK + static_cast<size_t>(P) * a.nkv * HD : nullptr;
    constexpr int CH = HD / 8;  // 16-byte chunks per row

    // Q tile.
    for (int i = tid; i < BQ * CH; i += THREADS) {
        const int r = i / CH, c = i % CH;
        const int qi = q0 + r;
        const bool ok = qi < len;
        const __half *src = Q + (static_cast<size_t>(start + (ok ? qi : 0)) * a.nh + h) * HD + c * 8;
        cp_async16(sQ + r * LD + c * 8, src, ok);
    }

    float o[NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
    const float sl2 = 1.4426950408889634f / sqrtf(static_cast<float>(HD));  // log2(e) / sqrt(hd)
    const int qrow0 = q0 + warp * 16 + g;  // this thread's rows: qrow0, qrow0 + 8
    const int kv_end = P + min(len, q0 + BQ);  // causal: keys below the last query of the tile

    for (int kv0 = 0; kv0 < kv_end; kv0 += BKV) {
        __syncthreads();  // previous tile fully consumed
        for (int i = tid; i < BKV * CH; i += THREADS) {
            const int r = i / CH, c = i % CH;
            const int ki = kv0 + r;
            const bool ok = ki < P + len;
            if (ki < P) {
                const size_t off = (static_cast<size_t>(ki) * a.nkv + kh) * HD + c * 8;
                cp_async16(sK + r * LD + c * 8, CK + off, true);
                cp_async16(sV + r * LD + c * 8, CV + off, true);
            } else {
                const int kvs = kv_slot(a.pages, row, start, ok ? ki - P : 0);
                const size_t off = (static_cast<size_t>(kvs) * a.nkv + kh) * HD + c * 8;
                cp_async16(sK + r * LD + c * 8, K + off, ok);
                cp_async16(sV + r * LD + c * 8, V + off, ok);
            }
        }
        cp_async_wait_all();
        __syncthreads();

        // S = Q K^T for this warp's 16 rows x 64 keys.
        float s[BKV / 8][4];
#pragma unroll
        for (int n = 0; n < BKV / 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
        for (int k0 = 0; k0 < HD; k0 += 16) {
            uint32_t a0, a1, a2, a3;
            {
                const int m = lane >> 3, i = lane & 7;
                ldsm_x4(a0, a1, a2, a3, sQ + (warp * 16 + i + (m & 1) * 8) * LD + k0 + (m >> 1) * 8);
            }
#pragma unroll
            for (int n0 = 0; n0 < BKV; n0 += 16) {
                uint32_t b0, b1, b2, b3;
                const int m = lane >> 3, i = lane & 7;
                ldsm_x4(b0, b1, b2, b3, sK + (n0 + i + (m >> 1) * 8) * LD + k0 + (m & 1) * 8);
                mma16816(s[n0 / 8], a0, a1, a2, a3, b0, b1);
                mma16816(s[n0 / 8 + 1], a0, a1, a2, a3, b2, b3);
            }
        }

        // Mask (causal and row end), online softmax in base 2.
        const bool diag = kv0 + BKV > P + q0;
        float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int n = 0; n < BKV / 8; ++n)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int key = kv0 + n * 8 + 2 * t4 + (e & 1);
                const int q = qrow0 + (e >> 1) * 8;
                float v = s[n][e] * sl2;
                if (key >= P + len || (diag && key > P + q)) v = -INFINITY;
                s[n][e] = v;
                mx[e >> 1] = fmaxf(mx[e >> 1], v);
            }
        float corr[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
            const float mn = fmaxf(m_r[r], mx[r]);
            corr[r] = (m_r[r] == -INFINITY) ? 0.f : exp2f(m_r[r] - mn);
            m_r[r] = mn;
        }
        float rs[2] = {0.f, 0.f};
#pragma unroll
        for (int n = 0; n < BKV / 8; ++n)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float mref = m_r[e >> 1] == -INFINITY ? 0.f : m_r[e >> 1];
                const float p = exp2f(s[n][e] - mref);
                s[n][e] = p;
                rs[e >> 1] += p;
            }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
            rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
            l_r[r] = l_r[r] * corr[r] + rs[r];
        }
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            o[n][0] *= corr[0];
            o[n][1] *= corr[0];
            o[n][2] *= corr[1];
            o[n][3] *= corr[1];
        }

        // O += P V.
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk) {
            const uint32_t a0 = pack_half2(s[2 * kk][0], s[2 * kk][1]);
            const uint32_t a1 = pack_half2(s[2 * kk][2], s[2 * kk][3]);
            const uint32_t a2 = pack_half2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
            const uint32_t a3 = pack_half2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
            for (int n0 = 0; n0 < HD; n0 += 16) {
                uint32_t b0, b1, b2, b3;
                const int m = lane >> 3, i = lane & 7;
                ldsm_x4_t(b0, b1, b2, b3, sV + (kk * 16 + i + (m & 1) * 8) * LD + n0 + (m >> 1) * 8);
                mma16816(o[n0 / 8], a0, a1, a2, a3, b0, b1);
                mma16816(o[n0 / 8 + 1], a0, a1, a2, a3, b2, b3);
            }
        }
    }

    // Normalise, gate, store fp16.
    __half *out = static_cast<__half *>(a.out);
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int qi = qrow0 + r * 8;
        if (qi >= len) continue;
        const size_t t = static_cast<size_t>(start + qi);
        const float inv = 1.0f / l_r[r];
        const float *gate = a.proj + t * a.ldp + h * 2 * HD + HD;
        __half *dst = out + t * a.ldo + h * HD;
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            const int d = n * 8 + 2 * t4;
            const float v0 = o[n][2 * r] * inv * sigmoid_f(gate[d]);
            const float v1 = o[n][2 * r + 1] * inv * sigmoid_f(gate[d + 1]);
            *reinterpret_cast<__half2 *>(dst + d) = __floats2half2_rn(v0, v1);
        }
    }
}

template <int HD>
void launch_hd(const AttnArgs &a, cudaStream_t s) {
    constexpr size_t smem = sizeof(__half) * (BQ + 2 * BKV) * (HD + 8);
    static SmemOptIn opt_in;
    opt_in.ensure(attn_tc_kernel<HD>, static_cast<int>(smem));
    dim3 grid(ceil_div(a.max_len, BQ), a.nh, a.n_rows);
    attn_tc_kernel<HD><<<grid, THREADS, smem, s>>>(a);
    HK_LAUNCH_CHECK();
}

}  // namespace

bool attention_tc_supported(int hd) { return hd == 64 || hd == 128 || hd == 256; }

void launch_attention_tc(const AttnArgs &a, cudaStream_t s) {
    switch (a.hd) {
        case 64: launch_hd<64>(a, s); break;
        case 128: launch_hd<128>(a, s); break;
        case 256: launch_hd<256>(a, s); break;
        default: throw CudaError("tensor-core attention supports head_dim 64, 128 or 256");
    }
}

}  // namespace hk
