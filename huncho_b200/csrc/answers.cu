// On-device calibration and answers for a whole scored batch.
//
// Per question (= row): the temperature softmax of its option logits with the
// reference's mixed precision (crates/huncho-core/src/calibration.rs:36-64:
// (l - max) * (1/T) and its exponential in fp32, the sum and the division in
// fp64 in option order, each probability rounded to fp32), the validation of
// calibration.rs:198-218 (finite logits, finite probabilities), and the typed
// answer fields of Engine::build_answer (crates/huncho-core/src/engine.rs:
// 1448-1513): first-maximum argmax (calibration.rs:87-95), the peak
// confidence (114-127) or Kev's score confidence (131-147), P(yes) of a noul
// question (options [no, yes]) and the expected score sum_i i p_i.
//
// Every fp32 step is written with round-to-nearest intrinsics so no multiply
// and add fuse: the results equal the host implementation's step for step.
// The fp32 exponential is the fp64 exponential rounded to fp32.
#include <cuda_runtime.h>
#include <math.h>

#include "common.cuh"
#include "layers.cuh"

namespace hk {
namespace {

__device__ __forceinline__ float clamp01(float v) { return v < 0.f ? 0.f : (v > 1.f ? 1.f : v); }

__global__ void answers_kernel(AnswerArgs a) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= a.n_rows) return;
    const int o0 = a.cu_positions[r], n = a.cu_positions[r + 1] - o0;
    const float *l = a.logits + o0;
    float *p = a.probs + o0;
    AnswerRec out{0, 0, 0.f, 0.f};
    bool finite = true;
    for (int i = 0; i < n; ++i) finite = finite && isfinite(l[i]);
    if (!finite || n == 0) {
        out.status = finite ? 0 : kAnswerNonfiniteLogits;
        for (int i = 0; i < n; ++i) p[i] = 0.f;
        a.out[r] = out;
        return;
    }
    const float inv_t = __fdiv_rn(1.0f, a.temperature);
    float mx = l[0];
    for (int i = 1; i < n; ++i) mx = fmaxf(mx, l[i]);
    double s = 0.0;
    for (int i = 0; i < n; ++i) {
        const float e = static_cast<float>(exp(static_cast<double>(__fmul_rn(__fsub_rn(l[i], mx), inv_t))));
        p[i] = e;
        s += static_cast<double>(e);
    }
    for (int i = 0; i < n; ++i) {
        p[i] = static_cast<float>(static_cast<double>(p[i]) / s);
        finite = finite && isfinite(p[i]);
    }
    if (!finite) {
        out.status = kAnswerNonfiniteProbs;
        a.out[r] = out;
        return;
    }
    int best = 0;
    for (int i = 1; i < n; ++i)
        if (p[i] > p[best]) best = i;
    out.best = best;
    const int qt = a.qtype[r];
    if (qt == kQuestionScore) {
        // Kev's score confidence: 1 - (sum_i p_i |i - mode|) / mean_i |i - center|.
        float conf = 1.f;
        if (n > 1) {
            const float center = __fdiv_rn(static_cast<float>(n - 1), 2.0f);
            float dev_u = 0.f;
            for (int i = 0; i < n; ++i) dev_u = __fadd_rn(dev_u, fabsf(__fsub_rn(static_cast<float>(i), center)));
            const float uniform_dev = __fdiv_rn(dev_u, static_cast<float>(n));
            const float mode = static_cast<float>(best);
            float dev = 0.f;
            for (int i = 0; i < n; ++i)
                dev = __fadd_rn(dev, __fmul_rn(p[i], fabsf(__fsub_rn(static_cast<float>(i), mode))));
            conf = clamp01(__fsub_rn(1.0f, __fdiv_rn(dev, uniform_dev)));
        }
        out.confidence = conf;
        float score = 0.f;
        for (int i = 0; i < n; ++i) score = __fadd_rn(score, __fmul_rn(static_cast<float>(i), p[i]));
        out.value = score;
    } else {
        // Peak confidence: (p_max - 1/n) / (1 - 1/n), clamped.
        float conf;
        if (n <= 1) {
            conf = clamp01(p[0]);
        } else {
            const float uniform = __fdiv_rn(1.0f, static_cast<float>(n));
            const float denom = __fsub_rn(1.0f, uniform);
            conf = denom <= 0.f ? 1.f : clamp01(__fdiv_rn(__fsub_rn(p[best], uniform), denom));
        }
        out.confidence = conf;
        out.value = qt == kQuestionNoul ? p[1] : p[best];
    }
    a.out[r] = out;
}

}  // namespace

void launch_answers(const AnswerArgs &a, cudaStream_t s) {
    if (a.n_rows <= 0) return;
    answers_kernel<<<(a.n_rows + 127) / 128, 128, 0, s>>>(a);
    HK_LAUNCH_CHECK();
}

}  // namespace hk
