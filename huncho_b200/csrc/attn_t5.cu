// Causal varlen GQA attention with the Qwen3.5 output gate (qwen3_5.rs:669-714)
// on the 5th-generation tensor cores: tcgen05.mma with the accumulators in
// tensor memory, for head_dim 128 and 256, fp16 operands.
//
// Two kernels share the algebra below. attn_ws_kernel (rows without a cached
// prefix: the model's path) is warp-specialised, with TMA loads through the
// page table; it is described where it is defined. attn_t5_kernel (rows that
// continue a cached prefix) runs it in one group of 4 warps.
//
// One CTA = 128 queries of one (row, query head); in attn_t5_kernel, thread =
// query row = TMEM lane; CTAs are dispatched longest (last query tile) first.
// Per tile of 64 keys:
//   S = Q K^T   (M=128, N=64, K=HD) into one of two TMEM S buffers;
//   the row softmax in registers (tcgen05.ld), P = exp2(...) as fp16 into
//   shared memory;
//   O += P V    (M=128, N=HD, K=64; V read MN-major) into the TMEM O columns.
// S of tile i+1 is issued before the softmax of tile i, so the tensor core and
// the threads overlap. The online softmax rescales lazily: a row's reference
// max (and with it the row of O) only moves when a tile's max exceeds it by
// more than 8 in log2 units, so exponents stay below 2^8 (safe in fp16) and
// O / l at the end is unchanged.
//
// Q, K, V and P live in shared memory as 128B-swizzled K-major tiles (V's
// tile is the same bytes read MN-major); K and V tiles are double-buffered and
// stream in (cp.async here, TMA in attn_ws_kernel) while earlier tiles are
// used. Keys are read through
// kv_slot() (flat or paged) and, for a row that continues a cached prefix,
// from the prefix's K/V first. Every mbarrier wait is bounded: on a timeout
// the kernel records an error bit, lets the MMAs it issued finish, frees its
// tensor memory and returns.
#include <cuda_bf16.h>
#include <math.h>

#include <cstring>

#include "common.cuh"
#include "layers.cuh"
#include "sm100.cuh"

namespace hk {
namespace {

using namespace sm100;

constexpr int BM = 128, BKV = 64, THREADS = 128;
constexpr uint32_t TM_S = 0, TM_O = 256, TM_COLS = 512;  // S buffers at columns 0 and 64; O at 256

template <int HD>
struct Tiles {
    static constexpr int Q_BYTES = BM * HD * 2;
    static constexpr int KV_BYTES = BKV * HD * 2;
    static constexpr int P_BYTES = BM * BKV * 2;
    static constexpr int Q = 0;
    static constexpr int K0 = Q + Q_BYTES;           // K buffers 0, 1
    static constexpr int V0 = K0 + 2 * KV_BYTES;     // V buffers 0, 1
    static constexpr int P0 = V0 + 2 * KV_BYTES;     // P buffers 0, 1
    static constexpr int RED = P0 + 2 * P_BYTES;     // row max (bf16, 2 tiles x 2 halves) / row sum (fp32, 2 halves)
    static constexpr int RED_BYTES = 1024;
    static constexpr int END = RED + RED_BYTES;
    static constexpr int SMEM = END + 256 + 1024;    // barriers + alignment slack
};
static_assert(Tiles<256>::SMEM <= 232448, "attention tiles exceed shared memory");

__device__ __forceinline__ void cpa16(void *dst, const void *src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src),
                 "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cpa_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cpa_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 8 consecutive fp32 values as one 16-byte fp16 store.
__device__ __forceinline__ void st8h(uint8_t *p, const float *v) {
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
    *reinterpret_cast<uint4 *>(p) = u;
}

// TMA = true: Q, K and V tiles come by TMA (one thread issues them; K / V per
// page or 64-key box through the block table), completing on mbarriers; rows
// without a cached prefix only. TMA = false: every thread stages its 16-byte
// chunks with cp.async (any row).
template <int HD, bool TMA>
__global__ void __launch_bounds__(THREADS, 1)
    attn_t5_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, AttnArgs a) {
    using L = Tiles<HD>;
    constexpr int CH = HD / 8;  // 16-byte chunks per row
    extern __shared__ uint8_t smem_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + L::END);
    uint64_t *bar_s = bars, *bar_pv = bars + 2, *bar_drain = bars + 3;
    uint64_t *bar_q = bars + 4, *bar_k = bars + 5, *bar_v = bars + 7;  // TMA completions (K, V: per buffer)
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 9);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);

    // Query tiles are the slowest grid dimension, last tile first: under the
    // causal mask a tile's work grows with its position, so the longest CTAs
    // start first and the short ones fill the tail.
    const int row = blockIdx.y, h = blockIdx.x, q0 = (gridDim.z - 1 - blockIdx.z) * BM;
    const int start = a.cu_seqlens[row];
    const int len = a.cu_seqlens[row + 1] - start;
    if (q0 >= len) return;
    const int kh = h / (a.nh / a.nkv);
    const int tid = threadIdx.x, warp = tid >> 5;
    // A continued row's first P keys are its cached prefix; key indices are
    // absolute (prefix first), queries are the row's own tokens.
    const int P = a.pre_len ? a.pre_len[row] : 0;
    const __half *CK = P ? reinterpret_cast<const __half *>(a.kv_in[row]) : nullptr;
    const __half *CV = P ? CK + static_cast<size_t>(P) * a.nkv * HD : nullptr;
    const __half *Qg = static_cast<const __half *>(a.q);
    const __half *Kg = static_cast<const __half *>(a.k);
    const __half *Vg = static_cast<const __half *>(a.v);
    const uint32_t s_base = smem_addr(sm);

    if (tid == 0) {
        for (int i = 0; i < 9; ++i) mbar_init(&bars[i], 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0) {
        tmem_alloc(tmem_holder, TM_COLS);
        tmem_relinquish();
    }

    // Chunk (row r, column group c) of a tile goes to thread r * CH + c mod 128:
    // a thread's column group is fixed and its rows step by THREADS / CH.
    constexpr int RSTEP = THREADS / CH;
    const int c_own = tid % CH, r_own = tid / CH;
    auto load_q = [&]() {
#pragma unroll 4
        for (int r = r_own; r < BM; r += RSTEP) {
            const int qi = q0 + r;
            const bool ok = qi < len;
            const __half *src = Qg + (static_cast<size_t>(start + (ok ? qi : 0)) * a.nh + h) * HD + c_own * 8;
            cpa16(sm + L::Q + sw128_off(BM, r, c_own * 8), src, ok);
        }
    };
    // The row's own keys: slot start + j (flat) or through its block table
    // (page sizes are powers of two: shift and mask).
    const int pt = a.pages.page_tokens;
    const int pshift = pt ? __ffs(pt) - 1 : 0;
    const int32_t *ptab = pt ? a.pages.block_table + a.pages.cu_pages[row] : nullptr;
    const size_t kv_stride = static_cast<size_t>(a.nkv) * HD;  // elements between slots
    auto load_kv = [&](bool is_v, int kv0, int b) {
        uint8_t *dst = sm + (is_v ? L::V0 : L::K0) + b * L::KV_BYTES;
        const __half *own = (is_v ? Vg : Kg) + static_cast<size_t>(kh) * HD + c_own * 8;
        const __half *pre = P ? (is_v ? CV : CK) + static_cast<size_t>(kh) * HD + c_own * 8 : nullptr;
#pragma unroll 4
        for (int r = r_own; r < BKV; r += RSTEP) {
            const int ki = kv0 + r;
            const bool ok = ki < P + len;
            const __half *src;
            if (ki < P) {
                src = pre + static_cast<size_t>(ki) * kv_stride;
            } else {
                const int j = ok ? ki - P : 0;
                const int slot = pt ? (ptab[j >> pshift] << pshift) + (j & (pt - 1)) : start + j;
                src = own + static_cast<size_t>(slot) * kv_stride;
            }
            cpa16(dst + sw128_off(BKV, r, c_own * 8), src, ok);
        }
    };
    // TMA form (warp 0, every lane): a K or V tile of 64 keys as boxes of
    // R = min(page, 64) rows x 64 columns (one 128-byte swizzle row) per
    // 64-column block of the head, one box per lane (at most 16), so the page
    // table lookups run in parallel; pages past the row's last one read that
    // last page instead (its values are finite; those keys are masked and
    // their V rows zeroed).
    const int R = pt ? (pt < BKV ? pt : BKV) : BKV;
    const int last_page = pt ? (len - 1) >> pshift : 0;
    const int lane = tid & 31;
    uint32_t kv_pend = 0;  // bit b: K buffer b, bit 2 + b: V buffer b has a load in flight
    constexpr int KT = HD / 64;
    const int nbox = (BKV / R) * KT;
    // K and V tiles are each loaded in order (tiles 0, 1, 2, ...): this lane's
    // page-table entry for the next tile of each stream is read one call
    // ahead, so the lookup's latency is off the issue path.
    auto page_of = [&](int j) { return ptab[(j >> pshift) < last_page ? (j >> pshift) : last_page]; };
    int pg_k = 0, pg_v = 0;
    if (TMA && pt && warp == 0 && lane < nbox) pg_k = pg_v = page_of((lane / KT) * R);
    auto tma_kv = [&](bool is_v, int kv0, int b) {
        uint8_t *dst = sm + (is_v ? L::V0 : L::K0) + b * L::KV_BYTES;
        uint64_t *bar = is_v ? &bar_v[b] : &bar_k[b];
        if (lane == 0) mbar_expect_tx(bar, L::KV_BYTES);
        __syncwarp();
        const CUtensorMap *m = is_v ? &tm_v : &tm_k;
        if (lane < nbox) {
            const int r0 = (lane / KT) * R, kt = lane % KT, j = kv0 + r0;
            int &pg = is_v ? pg_v : pg_k;
            const int slot = pt ? (pg << pshift) + (j & (pt - 1)) : start + j;
            tma_load_2d(dst + kt * BKV * 128 + r0 * 128, m, bar, kh * HD + kt * 64, slot);
            if (pt) pg = page_of(j + BKV);
        }
        kv_pend |= 1u << (is_v ? 2 + b : b);
    };
    // S = Q K^T into S buffer sb from K buffer kb (thread 0).
    auto issue_s = [&](int kb, int sb, uint32_t tmem) {
        const uint64_t d0 = desc_sw128(s_base, 16, 1024);
        const uint64_t qa = d0 + (L::Q >> 4), kb0 = d0 + ((L::K0 + kb * L::KV_BYTES) >> 4);
        constexpr uint32_t id = idesc_f16_f32(BM, BKV);
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks) {
            const uint32_t ao = (ks >> 2) * (BM * 128) + (ks & 3) * 32;
            const uint32_t bo = (ks >> 2) * (BKV * 128) + (ks & 3) * 32;
            mma_f16(tmem + TM_S + sb * BKV, qa + (ao >> 4), kb0 + (bo >> 4), id, ks > 0 ? 1u : 0u);
        }
    };
    // O (+)= P V from P buffer and V buffer b (thread 0); V read MN-major
    // (64-column blocks of the head dim 64 * 128 bytes apart, 8-key groups 1024).
    auto issue_pv = [&](int b, bool acc, uint32_t tmem) {
        const uint64_t pa = desc_sw128(s_base + L::P0 + b * L::P_BYTES, 16, 1024);
        const uint64_t vb = desc_sw128(s_base + L::V0 + b * L::KV_BYTES, BKV * 128, 1024);
        constexpr uint32_t id = idesc_f16_f32_mj(BM, HD, false, true);
#pragma unroll
        for (int ks = 0; ks < BKV / 16; ++ks)
            mma_f16(tmem + TM_O, pa + ((ks * 32) >> 4), vb + ((ks * 2048) >> 4), id, (acc || ks > 0) ? 1u : 0u);
    };
    auto wait = [&](uint64_t *bar, uint32_t parity) -> bool {
        if (!mbar_wait(bar, parity)) {
            set_error(a.err, kErrWaitTimeout);
            *abort_flag = 1;
            return false;
        }
        return true;
    };

    const int kv_end = P + min(len, q0 + BM);  // causal: keys up to the last query of the tile
    const int n_tiles = (kv_end + BKV - 1) / BKV;
    // cp.async groups per thread: {Q, K0, V0}, {K1}, then per tile i {K(i+2)}, {V(i+1)}.
    uint32_t kph = 0, vph = 0;  // TMA: bit b = parity of the next wait on K / V buffer b
    if constexpr (TMA) {
        __syncthreads();  // barriers initialised
        if (tid == 0) {
            mbar_expect_tx(bar_q, L::Q_BYTES);
#pragma unroll
            for (int kt = 0; kt < HD / 64; ++kt)
                tma_load_2d(sm + L::Q + kt * BM * 128, &tm_q, bar_q, h * HD + kt * 64, start + q0);
        }
        if (warp == 0) {
            tma_kv(false, 0, 0);
            tma_kv(true, 0, 0);
            if (n_tiles > 1) tma_kv(false, BKV, 1);
        }
    } else {
        load_q();
        load_kv(false, 0, 0);
        load_kv(true, 0, 0);
        cpa_commit();
        if (n_tiles > 1) load_kv(false, BKV, 1);
        cpa_commit();
        cpa_wait<1>();
        fence_async_smem();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    if (tid == 0) {
        if constexpr (TMA) {
            wait(bar_q, 0);
            if (wait(&bar_k[0], 0)) kv_pend &= ~1u;
            tc_fence_after();
        }
        issue_s(0, 0, tmem);
        mma_commit(&bar_s[0]);
    }
    if constexpr (TMA) kph ^= 1u;

    const int qi = q0 + tid;  // this thread's query (own index) and its absolute key limit
    const bool q_ok = qi < len;
    const int key_lim = min(P + qi, P + len - 1);
    const float sl2 = 1.4426950408889634f / sqrtf(static_cast<float>(HD));
    float m_ref = -INFINITY, l_sum = 0.f;
    uint32_t ph_s = 0u, ph_pv = 0u;  // bit b: parity of S buffer b

    for (int it = 0; it < n_tiles && !*abort_flag; ++it) {
        const int b = it & 1, kv0 = it * BKV;
        // 1. S of the next tile, once its keys have landed.
        if (it + 1 < n_tiles) {
            const int nb = (it + 1) & 1;
            if constexpr (TMA) {
                if (tid == 0) {
                    if (wait(&bar_k[nb], (kph >> nb) & 1u)) kv_pend &= ~(1u << nb);
                    tc_fence_after();
                    issue_s(nb, nb, tmem);
                    mma_commit(&bar_s[nb]);
                }
                kph ^= 1u << nb;
            } else {
                if (it == 0)
                    cpa_wait<0>();
                else
                    cpa_wait<1>();
                fence_async_smem();
                tc_fence_before();
                __syncthreads();
                if (tid == 0) {
                    tc_fence_after();
                    issue_s(nb, nb, tmem);
                    mma_commit(&bar_s[nb]);
                }
            }
        }
        // 2. This tile's scores; its K buffer is then free for tile it+2.
        wait(&bar_s[b], (ph_s >> b) & 1u);
        ph_s ^= 1u << b;
        tc_fence_after();
        if constexpr (TMA) {
            if (it + 2 < n_tiles && warp == 0) tma_kv(false, kv0 + 2 * BKV, b);
        } else {
            if (it + 2 < n_tiles) load_kv(false, kv0 + 2 * BKV, b);
            cpa_commit();
        }
        float sv[BKV];
        {
            float t32[32];
            tmem_ld32(lane_base + TM_S + b * BKV, t32);
#pragma unroll
            for (int j = 0; j < 32; ++j) sv[j] = t32[j];
            tmem_ld32(lane_base + TM_S + b * BKV + 32, t32);
#pragma unroll
            for (int j = 0; j < 32; ++j) sv[32 + j] = t32[j];
        }
        // 3. Mask (causal, row end, padding queries), tile max, lazy reference max.
        float mt = -INFINITY;
#pragma unroll
        for (int j = 0; j < BKV; ++j) {
            const bool valid = q_ok && kv0 + j <= key_lim;
            sv[j] = valid ? sv[j] * sl2 : -INFINITY;
            mt = fmaxf(mt, sv[j]);
        }
        float corr = 1.f;
        bool resc = false;
        if (mt > m_ref + 8.f) {
            resc = m_ref != -INFINITY;
            corr = resc ? exp2f(m_ref - mt) : 0.f;
            m_ref = mt;
        }
        // P is stored in fp16: the hardware base-2 exponential is exact enough
        // (its argument is <= 8 here, and -inf maps to 0).
        float psum = 0.f;
#pragma unroll
        for (int j = 0; j < BKV; ++j) {
            sv[j] = ex2_approx(sv[j] - m_ref);
            psum += sv[j];
        }
        l_sum = l_sum * corr + psum;
        // 4. The previous tile's O += P V is done: O is stable, its P and V
        // buffers are free; V of the next tile streams into that V buffer.
        if (it > 0) {
            wait(bar_pv, ph_pv);
            ph_pv ^= 1u;
            tc_fence_after();
        }
        if constexpr (TMA) {
            if (it + 1 < n_tiles && warp == 0) tma_kv(true, kv0 + BKV, (it + 1) & 1);
        } else {
            if (it + 1 < n_tiles) load_kv(true, kv0 + BKV, (it + 1) & 1);
            cpa_commit();
        }
        if (__any_sync(0xffffffffu, resc)) {
            const float f = resc ? corr : 1.f;
#pragma unroll 1
            for (int c = 0; c < HD; c += 32) {
                float o[32];
                tmem_ld32(lane_base + TM_O + c, o);
#pragma unroll
                for (int j = 0; j < 32; ++j) o[j] *= f;
                tmem_st32(lane_base + TM_O + c, o);
            }
        }
        // 5. P (this row's 64 probabilities, fp16) into P buffer b.
        uint8_t *pb = sm + L::P0 + b * L::P_BYTES;
#pragma unroll
        for (int c8 = 0; c8 < BKV / 8; ++c8) st8h(pb + sw128_off(BM, tid, c8 * 8), sv + c8 * 8);
        // 6. O += P V once this tile's V has landed.
        if constexpr (TMA) {
            // A paged tile that reaches past the row's end holds keys of the
            // row's last page beyond its tokens (never written in this batch):
            // their probabilities are 0, and their V rows are zeroed so that no
            // stale non-finite value reaches the product.
            const int valid = P + len - kv0;
            const bool tail = pt && valid < BKV;
            bool v_done = false;
            if (tail) {
                v_done = wait(&bar_v[b], (vph >> b) & 1u);
                constexpr int CPR = HD / 8;  // 16-byte chunks per key row
                uint8_t *vb = sm + L::V0 + b * L::KV_BYTES;
                for (int i = tid; i < (BKV - valid) * CPR; i += THREADS) {
                    const int r = valid + i / CPR, c = i % CPR;
                    *reinterpret_cast<uint4 *>(vb + (c >> 3) * BKV * 128 + r * 128 + (c & 7) * 16) =
                        make_uint4(0u, 0u, 0u, 0u);
                }
            }
            fence_async_smem();
            tc_fence_before();
            __syncthreads();
            if (tid == 0) {
                if (!tail) v_done = wait(&bar_v[b], (vph >> b) & 1u);
                if (v_done) kv_pend &= ~(1u << (2 + b));
                tc_fence_after();
                issue_pv(b, it > 0, tmem);
                mma_commit(bar_pv);
            }
            vph ^= 1u << b;
        } else {
            if (it > 0) cpa_wait<2>();
            fence_async_smem();
            tc_fence_before();
            __syncthreads();
            if (tid == 0) {
                tc_fence_after();
                issue_pv(b, it > 0, tmem);
                mma_commit(bar_pv);
            }
        }
    }
    if (!*abort_flag) {
        wait(bar_pv, ph_pv);
        tc_fence_after();
    }
    if constexpr (TMA) {
        // After an aborted wait: let this CTA's own loads land before it exits.
        if (tid == 0) {
            for (int b2 = 0; b2 < 2; ++b2) {
                if (kv_pend & (1u << b2)) (void)mbar_wait(&bar_k[b2], (kph >> b2) & 1u);
                if (kv_pend & (1u << (2 + b2))) (void)mbar_wait(&bar_v[b2], (vph >> b2) & 1u);
            }
            (void)mbar_wait(bar_q, 0);
        }
    } else {
        cpa_wait<0>();
    }
    __syncthreads();

    if (!*abort_flag) {
        // Normalise, gate, store fp16 (qwen3_5.rs:711-714).
        const size_t t = static_cast<size_t>(start + (q_ok ? qi : 0));
        const float inv = q_ok && l_sum > 0.f ? 1.0f / l_sum : 0.f;
        const float *gate = a.proj + t * a.ldp + h * 2 * HD + HD;
        __half *dst = static_cast<__half *>(a.out) + t * a.ldo + h * HD;
        const bool g4 = (a.ldp % 4) == 0;
#pragma unroll 1
        for (int c = 0; c < HD; c += 32) {
            float o[32];
            tmem_ld32(lane_base + TM_O + c, o);
            if (q_ok) {
                float gv[32];
                if (g4) {
#pragma unroll
                    for (int j = 0; j < 32; j += 4) {
                        const float4 x = *reinterpret_cast<const float4 *>(gate + c + j);
                        gv[j] = x.x;
                        gv[j + 1] = x.y;
                        gv[j + 2] = x.z;
                        gv[j + 3] = x.w;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) gv[j] = gate[c + j];
                }
                // fp16 output: the fast exponential and division are exact enough.
#pragma unroll
                for (int j = 0; j < 32; ++j) o[j] = o[j] * inv * __fdividef(1.0f, 1.0f + __expf(-gv[j]));
#pragma unroll
                for (int c8 = 0; c8 < 4; ++c8) st8h(reinterpret_cast<uint8_t *>(dst + c + c8 * 8), o + c8 * 8);
            }
        }
    } else if (tid == 0) {
        mma_commit(bar_drain);  // let every issued MMA finish before freeing TMEM
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

// The TMA form, warp-specialised: 8 softmax warps, two threads per query row
// (TMEM lane; each owns 32 of a tile's 64 keys and half of the output
// columns), one TMA warp and one MMA warp. The two threads of a row agree on
// the row's reference max through shared memory (the halves' maxima rounded
// to bf16, so both compute the same value; a reference max below the true one
// by a rounding step only raises the exponents, which the lazy rescale allows
// up to 8). All hand-offs are mbarriers: K / V tile i landed (TMA), S(i)
// ready (MMA commit; also frees K buffer i % 2), P(i) written (an arrival from
// every softmax thread), PV(i) done (MMA commit to bar_pv and to the V
// buffer's own barrier). Issuing a tcgen05.mma takes its thread ~70 cycles and
// a K / V tile's TMA boxes ~400, so the two issue streams run on separate
// warps and the softmax warps never issue either. Tile i's completions are
// the (i / 2)-th phase of its buffer's barriers (parity (i >> 1) & 1) and the
// i-th of bar_pv (parity i & 1); no waiter can fall two phases behind, since
// each barrier's next phase needs the waiter's own next step. Rows without a
// cached prefix only.
constexpr int WS_SOFT = 256, WS_TMA_WARP = WS_SOFT / 32, WS_MMA_WARP = WS_TMA_WARP + 1, WS_THREADS = WS_SOFT + 64;

// Barrier 1 over the WS_SOFT softmax threads (the TMA and MMA warps do not
// take part); returns whether any of them passed `v` true.
__device__ __forceinline__ bool soft_bar_or(bool v) {
    uint32_t r;
    asm volatile(
        "{\n.reg .pred p, q;\nsetp.ne.u32 p, %1, 0;\nbarrier.red.or.pred q, 1, %2, p;\nselp.u32 %0, 1, 0, q;\n}"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(v)), "n"(WS_SOFT)
        : "memory");
    return r != 0;
}

template <int HD>
__global__ void __launch_bounds__(WS_THREADS, 1)
    attn_ws_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, AttnArgs a) {
    using L = Tiles<HD>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + L::END);
    uint64_t *bar_q = bars, *bar_k = bars + 1, *bar_v = bars + 3, *bar_s = bars + 5, *bar_p = bars + 7;
    uint64_t *bar_pv = bars + 9, *bar_vfree = bars + 10, *bar_drain = bars + 12;
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 13);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);

    // Query tiles are the slowest grid dimension, last tile first (longest first).
    const int row = blockIdx.y, h = blockIdx.x, q0 = (gridDim.z - 1 - blockIdx.z) * BM;
    const int start = a.cu_seqlens[row];
    const int len = a.cu_seqlens[row + 1] - start;
    if (q0 >= len) return;
    const int kh = h / (a.nh / a.nkv);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t s_base = smem_addr(sm);

    if (tid == 0) {
        for (int i = 0; i < 13; ++i) mbar_init(&bars[i], (i == 7 || i == 8) ? WS_SOFT : 1);
        static_assert(L::RED_BYTES >= 2 * 2 * BM * 2 && L::RED_BYTES >= 2 * BM * 4, "row exchange area");
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == WS_MMA_WARP) {
        tmem_alloc(tmem_holder, TM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    const int kv_end = min(len, q0 + BM);  // causal: keys up to the last query of the tile
    const int n_tiles = (kv_end + BKV - 1) / BKV;
    const int pt = a.pages.page_tokens;
    const int pshift = pt ? __ffs(pt) - 1 : 0;
    const int32_t *ptab = pt ? a.pages.block_table + a.pages.cu_pages[row] : nullptr;
    auto wait = [&](uint64_t *bar, uint32_t parity) -> bool {
        if (!mbar_wait(bar, parity)) {
            set_error(a.err, kErrWaitTimeout);
            *abort_flag = 1;
            return false;
        }
        return true;
    };

    if (warp == WS_TMA_WARP) {
        // ---------------------------------------------------- TMA warp
        // K / V tiles as boxes of R = min(page, 64) rows x 64 columns, one box
        // per lane; each lane's page-table entry for the next tile of each
        // stream is read one call ahead. Pages past the row's last read that
        // last page instead (those keys are masked, their V rows zeroed).
        const int R = pt ? (pt < BKV ? pt : BKV) : BKV;
        const int last_page = pt ? (len - 1) >> pshift : 0;
        constexpr int KT = HD / 64;
        const int nbox = (BKV / R) * KT;
        auto page_of = [&](int j) { return ptab[(j >> pshift) < last_page ? (j >> pshift) : last_page]; };
        int pg_k = 0, pg_v = 0;
        if (pt && lane < nbox) pg_k = pg_v = page_of((lane / KT) * R);
        auto tma_kv = [&](bool is_v, int t) {
            const int b = t & 1;
            uint8_t *dst = sm + (is_v ? L::V0 : L::K0) + b * L::KV_BYTES;
            uint64_t *bar = is_v ? &bar_v[b] : &bar_k[b];
            if (lane == 0) mbar_expect_tx(bar, L::KV_BYTES);
            __syncwarp();
            if (lane < nbox) {
                const int r0 = (lane / KT) * R, kt = lane % KT, j = t * BKV + r0;
                int &pg = is_v ? pg_v : pg_k;
                const int slot = pt ? (pg << pshift) + (j & (pt - 1)) : start + j;
                tma_load_2d(dst + kt * BKV * 128 + r0 * 128, is_v ? &tm_v : &tm_k, bar, kh * HD + kt * 64, slot);
                if (pt) pg = page_of(j + BKV);
            }
        };
        if (lane == 0) {
            mbar_expect_tx(bar_q, L::Q_BYTES);
#pragma unroll
            for (int kt = 0; kt < HD / 64; ++kt)
                tma_load_2d(sm + L::Q + kt * BM * 128, &tm_q, bar_q, h * HD + kt * 64, start + q0);
        }
        int issued = 0;  // tiles whose K and V loads were issued
        for (int t = 0; t < n_tiles; ++t) {
            if (__any_sync(0xffffffffu, *abort_flag)) break;
            // K buffer t % 2 held K(t-2): free once S(t-2) completed; V buffer
            // t % 2 held V(t-2): free once PV(t-2) completed.
            bool f = true;
            if (t >= 2 && lane == 0) f = wait(&bar_s[t & 1], ((t - 2) >> 1) & 1);
            if (!__shfl_sync(0xffffffffu, f, 0)) break;
            tma_kv(false, t);
            if (t >= 2 && lane == 0) f = wait(&bar_vfree[t & 1], ((t - 2) >> 1) & 1);
            if (!__shfl_sync(0xffffffffu, f, 0)) {
                issued = -(t + 1);  // K(t) issued, V(t) not
                break;
            }
            tma_kv(true, t);
            issued = t + 1;
        }
        if (lane == 0) {
            // Every load issued here has landed before the CTA exits (the MMA
            // warp has waited for each one on the normal path).
            (void)mbar_wait(bar_q, 0);
            const int nk = issued < 0 ? -issued : issued, nv = issued < 0 ? -issued - 1 : issued;
            for (int t = (nk > 2 ? nk - 2 : 0); t < nk; ++t) (void)mbar_wait(&bar_k[t & 1], (t >> 1) & 1);
            for (int t = (nv > 2 ? nv - 2 : 0); t < nv; ++t) (void)mbar_wait(&bar_v[t & 1], (t >> 1) & 1);
        }
    } else if (warp == WS_MMA_WARP) {
        // ---------------------------------------------------- MMA warp (one thread)
        // S = Q K^T into S buffer b from K buffer b.
        auto issue_s = [&](int b) {
            const uint64_t d0 = desc_sw128(s_base, 16, 1024);
            const uint64_t qa = d0 + (L::Q >> 4), kb0 = d0 + ((L::K0 + b * L::KV_BYTES) >> 4);
            constexpr uint32_t id = idesc_f16_f32(BM, BKV);
#pragma unroll
            for (int ks = 0; ks < HD / 16; ++ks) {
                const uint32_t ao = (ks >> 2) * (BM * 128) + (ks & 3) * 32;
                const uint32_t bo = (ks >> 2) * (BKV * 128) + (ks & 3) * 32;
                mma_f16(tmem + TM_S + b * BKV, qa + (ao >> 4), kb0 + (bo >> 4), id, ks > 0 ? 1u : 0u);
            }
        };
        // O (+)= P V from P buffer and V buffer b; V read MN-major.
        auto issue_pv = [&](int b, bool acc) {
            const uint64_t pa = desc_sw128(s_base + L::P0 + b * L::P_BYTES, 16, 1024);
            const uint64_t vb = desc_sw128(s_base + L::V0 + b * L::KV_BYTES, BKV * 128, 1024);
            constexpr uint32_t id = idesc_f16_f32_mj(BM, HD, false, true);
#pragma unroll
            for (int ks = 0; ks < BKV / 16; ++ks)
                mma_f16(tmem + TM_O, pa + ((ks * 32) >> 4), vb + ((ks * 2048) >> 4), id, (acc || ks > 0) ? 1u : 0u);
        };
        if (lane == 0) {
            if (wait(bar_q, 0) && wait(&bar_k[0], 0)) {
                tc_fence_after();
                issue_s(0);
                mma_commit(&bar_s[0]);
            }
            for (int i = 0; i < n_tiles && !*abort_flag; ++i) {
                const int b = i & 1;
                // S(i+1): its S buffer held S(i-1), whose scores were read
                // before P(i-1) arrived (waited for PV(i-1) last iteration).
                if (i + 1 < n_tiles) {
                    if (!wait(&bar_k[b ^ 1], ((i + 1) >> 1) & 1)) break;
                    tc_fence_after();
                    issue_s(b ^ 1);
                    mma_commit(&bar_s[b ^ 1]);
                }
                // PV(i) once P(i) is written (S(i) read, O rescaled) and V(i) landed.
                if (!wait(&bar_p[b], (i >> 1) & 1) || !wait(&bar_v[b], (i >> 1) & 1)) break;
                tc_fence_after();
                issue_pv(b, i > 0);
                mma_commit(bar_pv);
                mma_commit(&bar_vfree[b]);
            }
            // Every MMA issued here has finished before TMEM is freed.
            mma_commit(bar_drain);
            (void)mbar_wait(bar_drain, 0);
        }
        __syncwarp();
    } else {
        // ---------------------------------------------------- softmax warps
        const int rq = tid & (BM - 1), half = tid >> 7;  // row (TMEM lane) and key / column half
        const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
        __nv_bfloat16 *xmax = reinterpret_cast<__nv_bfloat16 *>(sm + L::RED);  // [tile parity][half][BM]
        const int qi = q0 + rq;  // this thread's query and its key limit
        const bool q_ok = qi < len;
        const int key_lim = min(qi, len - 1);
        const float sl2 = 1.4426950408889634f / sqrtf(static_cast<float>(HD));
        float m_ref = -INFINITY, l_sum = 0.f;  // l_sum: this thread's half of the row sum
        for (int i = 0; i < n_tiles; ++i) {
            const int b = i & 1, kv0 = i * BKV + half * 32;
            wait(&bar_s[b], (i >> 1) & 1);
            tc_fence_after();
            float sv[32];
            tmem_ld32(lane_base + TM_S + b * BKV + half * 32, sv);
            // Mask (causal, row end, padding queries), the halves' tile max.
            float mt = -INFINITY;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const bool valid = q_ok && kv0 + j <= key_lim;
                sv[j] = valid ? sv[j] * sl2 : -INFINITY;
                mt = fmaxf(mt, sv[j]);
            }
            const __nv_bfloat16 mine = __float2bfloat16_rn(mt);
            xmax[(b * 2 + half) * BM + rq] = mine;
            // Every softmax thread passes this barrier once per tile; an abort
            // seen by any of them ends the loop for all.
            if (soft_bar_or(*abort_flag)) break;
            mt = fmaxf(__bfloat162float(mine), __bfloat162float(xmax[(b * 2 + (half ^ 1)) * BM + rq]));
            float corr = 1.f;
            bool resc = false;
            if (mt > m_ref + 8.f) {
                resc = m_ref != -INFINITY;
                corr = resc ? exp2f(m_ref - mt) : 0.f;
                m_ref = mt;
            }
            float psum = 0.f;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                sv[j] = ex2_approx(sv[j] - m_ref);
                psum += sv[j];
            }
            l_sum = l_sum * corr + psum;
            // PV(i-1) done: O is stable and P buffer b (read by PV(i-2)) is free.
            if (i > 0) {
                wait(bar_pv, (i - 1) & 1);
                tc_fence_after();
            }
            if (__any_sync(0xffffffffu, resc)) {
                const float f = resc ? corr : 1.f;
#pragma unroll 1
                for (int c = half * (HD / 2); c < (half + 1) * (HD / 2); c += 32) {
                    float o[32];
                    tmem_ld32(lane_base + TM_O + c, o);
#pragma unroll
                    for (int j = 0; j < 32; ++j) o[j] *= f;
                    tmem_st32(lane_base + TM_O + c, o);
                }
            }
            uint8_t *pb = sm + L::P0 + b * L::P_BYTES;
#pragma unroll
            for (int c8 = 0; c8 < 4; ++c8) st8h(pb + sw128_off(BM, rq, half * 32 + c8 * 8), sv + c8 * 8);
            // A paged tile that reaches past the row's end holds keys of the
            // row's last page beyond its tokens: their probabilities are 0, and
            // their V rows are zeroed so no stale non-finite value reaches P V.
            const int valid = len - i * BKV;
            if (pt && valid < BKV && wait(&bar_v[b], (i >> 1) & 1)) {
                constexpr int CPR = HD / 8;  // 16-byte chunks per key row
                uint8_t *vbuf = sm + L::V0 + b * L::KV_BYTES;
                for (int k = tid; k < (BKV - valid) * CPR; k += WS_SOFT) {
                    const int r = valid + k / CPR, c = k % CPR;
                    *reinterpret_cast<uint4 *>(vbuf + (c >> 3) * BKV * 128 + r * 128 + (c & 7) * 16) =
                        make_uint4(0u, 0u, 0u, 0u);
                }
            }
            fence_async_smem();
            tc_fence_before();
            mbar_arrive(&bar_p[b]);
        }
        const bool done = !*abort_flag && wait(bar_pv, (n_tiles - 1) & 1);
        tc_fence_after();
        // The row sum is the two halves' sum (the max exchange area, reused
        // once every thread is past its last read of it).
        float *xsum = reinterpret_cast<float *>(sm + L::RED);
        const bool stop = soft_bar_or(!done);
        xsum[half * BM + rq] = l_sum;
        soft_bar_or(false);
        if (!stop) {
            // Normalise, gate, store fp16 (qwen3_5.rs:711-714): this thread's
            // half of the row's output columns.
            const float l_row = l_sum + xsum[(half ^ 1) * BM + rq];
            const size_t t = static_cast<size_t>(start + (q_ok ? qi : 0));
            const float inv = q_ok && l_row > 0.f ? 1.0f / l_row : 0.f;
            const float *gate = a.proj + t * a.ldp + h * 2 * HD + HD;
            __half *dst = static_cast<__half *>(a.out) + t * a.ldo + h * HD;
            const bool g4 = (a.ldp % 4) == 0;
#pragma unroll 1
            for (int c = half * (HD / 2); c < (half + 1) * (HD / 2); c += 32) {
                float o[32];
                tmem_ld32(lane_base + TM_O + c, o);
                if (q_ok) {
                    float gv[32];
                    if (g4) {
#pragma unroll
                        for (int j = 0; j < 32; j += 4) {
                            const float4 x = *reinterpret_cast<const float4 *>(gate + c + j);
                            gv[j] = x.x;
                            gv[j + 1] = x.y;
                            gv[j + 2] = x.z;
                            gv[j + 3] = x.w;
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j) gv[j] = gate[c + j];
                    }
#pragma unroll
                    for (int j = 0; j < 32; ++j) o[j] = o[j] * inv * __fdividef(1.0f, 1.0f + __expf(-gv[j]));
#pragma unroll
                    for (int c8 = 0; c8 < 4; ++c8) st8h(reinterpret_cast<uint8_t *>(dst + c + c8 * 8), o + c8 * 8);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == WS_MMA_WARP) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, TM_COLS);
    }
}

template <int HD>
void launch_t5(const AttnArgs &a, cudaStream_t s) {
    dim3 grid(a.nh, a.n_rows, ceil_div(a.max_len, BM));
    const auto aligned = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    // TMA staging for rows without cached prefixes (their keys live in the
    // k / v buffers only) when the slot count is known.
    if (!a.pre_len && a.kv_slots > 0 && aligned(a.q) && aligned(a.k) && aligned(a.v)) {
        static SmemOptIn opt_in;
        opt_in.ensure(attn_ws_kernel<HD>, Tiles<HD>::SMEM);
        const int pt = a.pages.page_tokens;
        const uint32_t rows = pt ? (pt < BKV ? pt : BKV) : BKV;
        const CUtensorMap tq = tensor_map_f16(a.q, a.n, static_cast<uint64_t>(a.nh) * HD,
                                              static_cast<uint64_t>(a.nh) * HD * 2, 64, BM);
        const CUtensorMap tk = tensor_map_f16(a.k, a.kv_slots, static_cast<uint64_t>(a.nkv) * HD,
                                              static_cast<uint64_t>(a.nkv) * HD * 2, 64, rows);
        const CUtensorMap tv = tensor_map_f16(a.v, a.kv_slots, static_cast<uint64_t>(a.nkv) * HD,
                                              static_cast<uint64_t>(a.nkv) * HD * 2, 64, rows);
        attn_ws_kernel<HD><<<grid, WS_THREADS, Tiles<HD>::SMEM, s>>>(tq, tk, tv, a);
    } else {
        static SmemOptIn opt_in;
        opt_in.ensure(attn_t5_kernel<HD, false>, Tiles<HD>::SMEM);
        CUtensorMap z;
        std::memset(&z, 0, sizeof(z));
        attn_t5_kernel<HD, false><<<grid, THREADS, Tiles<HD>::SMEM, s>>>(z, z, z, a);
    }
    HK_LAUNCH_CHECK();
}

}  // namespace

bool attention_t5_supported(const AttnArgs &a) {
    return (a.hd == 128 || a.hd == 256) && a.nkv > 0 && a.nh % a.nkv == 0 && (a.ldo % 8) == 0;
}

void launch_attention_t5(const AttnArgs &a, cudaStream_t s) {
    if (a.hd == 256)
        launch_t5<256>(a, s);
    else if (a.hd == 128)
        launch_t5<128>(a, s);
    else
        throw CudaError("tcgen05 attention supports head_dim 128 or 256");
}

}  // namespace hk
