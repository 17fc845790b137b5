// The pointer-head readout with its scratch in a fixed, library-owned device
// array, for callers that cannot allocate device memory.
//
// hk_op_readout needs two scratch buffers next to its inputs and outputs (the
// normalised rows and their projections). Some callers cannot call
// cudaMalloc: a host that gives this library only device memory planned ahead
// from its own pool (for example a service embedding it behind a fixed memory
// budget), or a latency-critical serving loop where cudaMalloc's implicit
// device synchronisation would stall the other work on the GPU. For them,
// hk_op_readout_noalloc computes the same readout with its scratch in
// `g_readout_scratch`, a file-scope __device__ array of kNoAllocScratchFloats
// floats (16 MiB) that every GPU which loads the library holds until the
// process exits. It calls no cudaMalloc, cudaFree or allocating library
// routine.
//
// Limits: decision + option rows <= 1024, hidden <= 3584, pointer width <= 512.
// All calls share the one array and it keeps the last call's contents; nothing
// in it needs to start at zero (every scratch element a call reads it has
// written first). Calls that overlap on the GPU -- on two streams, or from two
// threads -- race on the array and must be serialised by the caller. Errors
// (sizes beyond the limits: HK_ERR_ARGUMENT) leave their message in
// hk_op_last_error().
//
// In host code `g_readout_scratch` names a host-side stand-in, not a device
// address. The device address comes from cudaGetSymbolAddress, once per device
// with that device current; the first call on each device does this set-up
// (so that first call should come before any stream capture).
#include <cmath>
#include <mutex>
#include <string>

#include "../../include/huncho_kev.h"
#include "../../include/huncho_kev_ops.h"
#include "common.cuh"
#include "layers.cuh"

namespace {

constexpr int kNoAllocMaxRows = 1024;
constexpr int kNoAllocMaxHidden = 3584;
constexpr int kNoAllocMaxDp = 512;
constexpr size_t kNoAllocScratchFloats = static_cast<size_t>(kNoAllocMaxRows) * (kNoAllocMaxHidden + kNoAllocMaxDp);

static __device__ __align__(256) float g_readout_scratch[kNoAllocScratchFloats];

constexpr int kMaxDevices = 64;
float *g_scratch_addr[kMaxDevices] = {};
std::mutex g_scratch_mu;

// The device address of g_readout_scratch on the current device (set-up on
// first use per device).
cudaError_t scratch_address(float **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_addr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_readout_scratch);
        if (e != cudaSuccess) return e;
        g_scratch_addr[dev] = static_cast<float *>(p);
    }
    *out = g_scratch_addr[dev];
    return cudaSuccess;
}

}  // namespace

extern "C" int hk_op_readout_noalloc(const float *x, int hidden, const float *final_w, float eps, const int32_t *idx,
                                     const int32_t *opt_dec, int n_dec, int n_opt, const float *wq, const float *bq,
                                     const float *wk, const float *bk, int dp, float *logits, void *stream) {
    const int rows = n_dec + n_opt;
    if (n_dec < 0 || n_opt < 0 || rows > kNoAllocMaxRows || hidden <= 0 || hidden > kNoAllocMaxHidden || dp <= 0 ||
        dp > kNoAllocMaxDp) {
        hk::set_op_error("hk_op_readout_noalloc: sizes exceed the fixed scratch (rows <= " +
                         std::to_string(kNoAllocMaxRows) + ", hidden <= " + std::to_string(kNoAllocMaxHidden) +
                         ", pointer width <= " + std::to_string(kNoAllocMaxDp) + ")");
        return HK_ERR_ARGUMENT;
    }
    try {
        hk::check_readout_args(x, hidden, final_w, idx, opt_dec, n_dec, n_opt, wq, bq, wk, bk, dp, logits);
    } catch (const std::exception &ex) {
        hk::set_op_error(std::string("hk_op_readout_noalloc: ") + ex.what());
        return HK_ERR_ARGUMENT;
    }
    float *scratch = nullptr;
    const cudaError_t e = scratch_address(&scratch);
    if (e != cudaSuccess) {
        hk::set_op_error(std::string("hk_op_readout_noalloc: cudaGetSymbolAddress failed: ") + cudaGetErrorString(e));
        return HK_ERR_CUDA;
    }
    try {
        hk::ReadoutArgs a;
        a.x = x;
        a.hidden = hidden;
        a.final_w = final_w;
        a.eps = eps;
        a.idx = idx;
        a.opt_dec = opt_dec;
        a.n_dec = n_dec;
        a.n_opt = n_opt;
        a.wq = wq;
        a.bq = bq;
        a.wk = wk;
        a.bk = bk;
        a.dp = dp;
        a.scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(dp)));
        a.hn = scratch;                                            // [rows, hidden]
        a.proj = scratch + static_cast<size_t>(rows) * hidden;     // [rows, dp]
        a.logits = logits;
        hk::launch_readout(a, static_cast<cudaStream_t>(stream));
    } catch (const std::exception &ex) {
        hk::set_op_error(ex.what());
        return HK_ERR_CUDA;
    }
    return HK_OK;
}
