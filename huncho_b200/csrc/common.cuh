// Shared helpers for the Kev sm_100a kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdio>
#include <stdexcept>
#include <string>

namespace hk {

// A CUDA failure on the host side becomes a C++ exception that the C ABI turns
// into HK_ERR_CUDA with the message.
struct CudaError : std::runtime_error {
    explicit CudaError(const std::string &s) : std::runtime_error(s) {}
};

#define HK_CUDA(expr)                                                                  \
    do {                                                                               \
        cudaError_t _e = (expr);                                                       \
        if (_e != cudaSuccess)                                                         \
            throw ::hk::CudaError(std::string(#expr) + ": " + cudaGetErrorString(_e)); \
    } while (0)

// Kernels launched by the calling thread (launch accounting for the C ABI).
extern thread_local uint64_t tl_launches;

#define HK_LAUNCH_CHECK()              \
    do {                               \
        ++::hk::tl_launches;           \
        HK_CUDA(cudaGetLastError());   \
    } while (0)

// Device-side error word bits. Kernels never trap: a bounded wait that gives
// up, or an index that fails a guard, sets a bit and the kernel returns.
enum : uint32_t {
    kErrWaitTimeout = 1u << 0,   // an mbarrier wait exceeded its iteration limit
    kErrBadIndex = 1u << 1,      // an index guard failed
};

__device__ __forceinline__ void set_error(uint32_t *err, uint32_t bit) {
    if (err) atomicOr(err, bit);
}

// Activation element types: float (fp32 model) or __half (the half-precision
// models: tensor-core operands are fp16, the type the reference's CUDA path
// runs half-precision checkpoints in).
template <typename T> struct Act;
template <> struct Act<float> {
    static __device__ __forceinline__ float load(const float *p) { return *p; }
    static __device__ __forceinline__ float to_f(float v) { return v; }
    static __device__ __forceinline__ float from_f(float v) { return v; }
    // Round a float to the storage type and back (the reference's casts to the
    // model dtype between ops).
    static __device__ __forceinline__ float round(float v) { return v; }
};
template <> struct Act<__half> {
    static __device__ __forceinline__ float load(const __half *p) { return __half2float(*p); }
    static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
    static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
    static __device__ __forceinline__ float round(float v) { return __half2float(__float2half_rn(v)); }
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// SiLU and sigmoid as the reference writes them: x / (1 + exp(-x)), 1 / (1 + exp(-x)).
__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }
// SiLU with the fast exponential and division intrinsics, for values rounded
// to fp16 right after (relative error ~1e-6, far below fp16's 5e-4); for
// x -> -inf the denominator overflows and the result is 0, as silu's limit.
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }
__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }

// The low part of a split-precision tensor-core input: the e5m2 rounding of
// v - float(h), where h = fp16(v) is the high part (GemmArgs::x_lo).
__device__ __forceinline__ uint8_t lo_e5m2(float v, __half h) {
    return static_cast<uint8_t>(__nv_cvt_float_to_fp8(v - __half2float(h), __NV_SATFINITE, __NV_E5M2));
}

inline int ceil_div(long a, long b) { return (int)((a + b - 1) / b); }

// Raises a kernel's dynamic shared-memory limit once per device. Handles on
// several host threads launch concurrently, so the per-device flags are
// atomics (a lost race only repeats the idempotent attribute call).
struct SmemOptIn {
    static constexpr int kMaxDevices = 64;
    std::atomic<bool> done[kMaxDevices] = {};
    template <typename Kernel>
    void ensure(Kernel *kernel, int bytes) {
        int dev = 0;
        HK_CUDA(cudaGetDevice(&dev));
        const bool tracked = dev >= 0 && dev < kMaxDevices;
        if (tracked && done[dev].load(std::memory_order_acquire)) return;
        HK_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
        if (tracked) done[dev].store(true, std::memory_order_release);
    }
};

// Sets the message hk_op_last_error() returns on the calling thread.
void set_op_error(const std::string &msg);

}  // namespace hk
