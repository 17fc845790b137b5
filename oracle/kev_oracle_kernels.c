/*
 * CPU oracle kernels for the Kev scoring forward: TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load
 * this library; the product path (huncho_b200) never links or calls it.
 *
 * The loops restate the reference's buffered CPU kernels in their exact fp32
 * operation order (compiled with -ffp-contract=off, so no product is fused
 * into an FMA and no sum is re-associated):
 *   - kev_oracle_delta_recurrent: crates/huncho-backend/src/delta_cpu.rs:99-136
 *     (decay and memory readout fused, ascending key index; then the rank-1
 *     update and the output readout in one pass), equal to the tensor loop
 *     qwen3_5.rs:950-987.
 *   - kev_oracle_causal_conv: crates/huncho-backend/src/conv_cpu.rs:38-49
 *     (taps accumulated in ascending order into a zero-initialised row), equal
 *     to the shifted-broadcast form qwen3_5.rs:817-844.
 * Heads (recurrence) and channels (convolution) are independent, so they are
 * split over POSIX threads; the arithmetic inside each one is unchanged.
 */
#include <pthread.h>
#include <stddef.h>
#include <stdlib.h>

static int g_threads = 1;

void kev_oracle_set_threads(int n) { g_threads = n < 1 ? 1 : (n > 256 ? 256 : n); }

typedef struct {
    const float *q, *k, *v, *decay, *beta;
    int heads, seq, dk, dv;
    float *state, *out;
    int begin, end;
} delta_job;

static void delta_heads(const delta_job *a) {
    float *delta = (float *)malloc(sizeof(float) * (size_t)a->dv);
    for (int h = a->begin; h < a->end; ++h) {
        float *s = a->state + (size_t)h * a->dk * a->dv;
        for (int t = 0; t < a->seq; ++t) {
            const float *qt = a->q + ((size_t)h * a->seq + t) * a->dk;
            const float *kt = a->k + ((size_t)h * a->seq + t) * a->dk;
            const float *vt = a->v + ((size_t)h * a->seq + t) * a->dv;
            const float d = a->decay[(size_t)h * a->seq + t];
            const float b = a->beta[(size_t)h * a->seq + t];
            float *o = a->out + ((size_t)h * a->seq + t) * a->dv;
            for (int j = 0; j < a->dv; ++j) delta[j] = 0.0f;
            for (int i = 0; i < a->dk; ++i) {
                const float ki = kt[i];
                float *row = s + (size_t)i * a->dv;
                for (int j = 0; j < a->dv; ++j) {
                    row[j] *= d;
                    delta[j] += row[j] * ki;
                }
            }
            for (int j = 0; j < a->dv; ++j) delta[j] = (vt[j] - delta[j]) * b;
            for (int j = 0; j < a->dv; ++j) o[j] = 0.0f;
            for (int i = 0; i < a->dk; ++i) {
                const float ki = kt[i];
                const float qi = qt[i];
                float *row = s + (size_t)i * a->dv;
                for (int j = 0; j < a->dv; ++j) {
                    row[j] += ki * delta[j];
                    o[j] += row[j] * qi;
                }
            }
        }
    }
    free(delta);
}

static void *delta_thread(void *p) {
    delta_heads((const delta_job *)p);
    return NULL;
}

/*
 * q, k: [heads, seq, dk]; v: [heads, seq, dv]; decay (= exp(g)), beta: [heads, seq];
 * state: [heads, dk, dv] (in: initial state, out: final state); out: [heads, seq, dv].
 */
void kev_oracle_delta_recurrent(const float *q, const float *k, const float *v,
                                const float *decay, const float *beta,
                                int heads, int seq, int dk, int dv,
                                float *state, float *out) {
    int n = g_threads < heads ? g_threads : heads;
    if (n < 1) n = 1;
    delta_job jobs[256];
    pthread_t tids[256];
    for (int i = 0; i < n; ++i) {
        delta_job j = {q, k, v, decay, beta, heads, seq, dk, dv, state, out,
                       heads * i / n, heads * (i + 1) / n};
        jobs[i] = j;
    }
    for (int i = 1; i < n; ++i) pthread_create(&tids[i], NULL, delta_thread, &jobs[i]);
    delta_heads(&jobs[0]);
    for (int i = 1; i < n; ++i) pthread_join(tids[i], NULL);
}

/* x: [channels, seq]; w: [channels, taps]; out: [channels, seq] (pre-activation). */
void kev_oracle_causal_conv(const float *x, const float *w, int channels, int seq,
                            int taps, float *out) {
    for (int c = 0; c < channels; ++c) {
        float *row = out + (size_t)c * seq;
        const float *xr = x + (size_t)c * seq;
        for (int t = 0; t < seq; ++t) row[t] = 0.0f;
        for (int tap = 0; tap < taps; ++tap) {
            const int shift = taps - 1 - tap;
            if (shift >= seq) continue;
            const float wt = w[(size_t)c * taps + tap];
            for (int t = shift; t < seq; ++t) row[t] += wt * xr[t - shift];
        }
    }
}
