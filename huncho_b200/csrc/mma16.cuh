// mma.sync (m16n8k16, fp16 operands, fp32 accumulation) building blocks for
// the chunked delta-rule kernels: ldmatrix fragment loaders over padded
// row-major shared-memory tiles, cp.async staging, fp16 hi/lo splits.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace hk {
namespace {

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

__device__ __forceinline__ void cp16(void *dst, const void *src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sa(dst)), "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp4(void *dst, const void *src, bool valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(sa(dst)), "l"(src), "r"(valid ? 4 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void split_store(__half *hi, __half *lo, float v) {
    const __half h = __float2half_rn(v);
    *hi = h;
    *lo = __float2half_rn(v - __half2float(h));
}

// Two consecutive fp16 values (hi and lo parts of v0, v1) as 4-byte stores.
__device__ __forceinline__ void split_store2(__half *hi, __half *lo, float v0, float v1) {
    const __half2 h = __floats2half2_rn(v0, v1);
    const float2 f = __half22float2(h);
    *reinterpret_cast<__half2 *>(hi) = h;
    *reinterpret_cast<__half2 *>(lo) = __floats2half2_rn(v0 - f.x, v1 - f.y);
}

// Four consecutive fp16 values as one 8-byte store (hi and lo parts of v).
__device__ __forceinline__ void split_store4(__half *hi, __half *lo, const float (&v)[4]) {
    __half2 h0 = __floats2half2_rn(v[0], v[1]), h1 = __floats2half2_rn(v[2], v[3]);
    const float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
    __half2 l0 = __floats2half2_rn(v[0] - f0.x, v[1] - f0.y), l1 = __floats2half2_rn(v[2] - f1.x, v[3] - f1.y);
    *reinterpret_cast<uint2 *>(hi) = make_uint2(*reinterpret_cast<uint32_t *>(&h0), *reinterpret_cast<uint32_t *>(&h1));
    *reinterpret_cast<uint2 *>(lo) = make_uint2(*reinterpret_cast<uint32_t *>(&l0), *reinterpret_cast<uint32_t *>(&l1));
}
__device__ __forceinline__ void store4(__half *dst, const float (&v)[4]) {
    __half2 h0 = __floats2half2_rn(v[0], v[1]), h1 = __floats2half2_rn(v[2], v[3]);
    *reinterpret_cast<uint2 *>(dst) = make_uint2(*reinterpret_cast<uint32_t *>(&h0), *reinterpret_cast<uint32_t *>(&h1));
}

}  // namespace
}  // namespace hk
