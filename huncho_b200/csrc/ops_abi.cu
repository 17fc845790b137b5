// Kernel-level C entry points (include/huncho_kev_ops.h) for per-kernel
// parity tests and timing.
#include <algorithm>
#include <cmath>
#include <exception>
#include <string>

#include "../../include/huncho_kev.h"
#include "../../include/huncho_kev_ops.h"
#include "common.cuh"
#include "gemm.cuh"
#include "layers.cuh"

namespace {
thread_local std::string tl_op_error;

template <typename F>
int op_guard(F &&f) {
    try {
        f();
        return HK_OK;
    } catch (const hk::CudaError &e) {
        tl_op_error = e.what();
        return HK_ERR_CUDA;
    } catch (const std::exception &e) {
        tl_op_error = e.what();
        return HK_ERR_ARGUMENT;
    }
}

int current_sms() {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}
}  // namespace

namespace hk {
// Record the calling thread's kernel-level entry-point error (hk_op_last_error).
void set_op_error(const std::string &msg) { tl_op_error = msg; }

void check_readout_args(const float *x, int hidden, const float *final_w, const int32_t *idx, const int32_t *opt_dec,
                        int n_dec, int n_opt, const float *wq, const float *bq, const float *wk, const float *bk,
                        int dp, const float *logits) {
    if (n_dec < 0 || n_opt < 0 || hidden <= 0 || dp <= 0)
        throw std::invalid_argument("readout: row counts must be >= 0, hidden and pointer width > 0");
    if (n_opt > 0 && n_dec == 0) throw std::invalid_argument("readout: options need at least one decision row");
    if (n_opt > 0 && (!x || !final_w || !idx || !opt_dec || !wq || !bq || !wk || !bk || !logits))
        throw std::invalid_argument("readout: null pointer");
}
}  // namespace hk

extern "C" {

int hk_op_gemm(int dtype, int epilogue, int M, int N, int K, const void *x, int ldx, const void *w, int ldw,
               const float *scale, void *out, int ldo, void *stream) {
    return op_guard([&] {
        hk::GemmArgs a;
        a.M = M;
        a.N = N;
        a.K = K;
        a.x = x;
        a.ldx = ldx;
        a.w = w;
        a.ldw = ldw;
        a.scale = scale;
        a.out = out;
        a.ldo = ldo;
        a.epilogue = epilogue;
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        if (dtype == 0)
            hk::gemm_f32_simt(a, s);
        else if (dtype == 1)
            hk::gemm_f16_tc(a, s, current_sms());
        else if (dtype == 2)
            hk::gemm_f16_tc_pair(a, s, current_sms());
        else if (dtype == 3) {
            // 3xTF32: the low parts of x and w in stream-ordered scratch.
            if (!x || !w || (ldx % 4) || (ldw % 4)) throw std::invalid_argument("hk_op_gemm: bad fp32 operands");
            const int ldl = (K + 3) / 4 * 4;
            float *xl = nullptr, *wl = nullptr;
            HK_CUDA(cudaMallocAsync(reinterpret_cast<void **>(&xl), static_cast<size_t>(std::max(M, 1)) * ldl * 4, s));
            HK_CUDA(cudaMallocAsync(reinterpret_cast<void **>(&wl), static_cast<size_t>(std::max(N, 1)) * ldl * 4, s));
            hk::launch_tf32_lo(static_cast<const float *>(x), ldx, M, K, xl, ldl, s);
            hk::launch_tf32_lo(static_cast<const float *>(w), ldw, N, K, wl, ldl, s);
            a.tf32 = true;
            a.x_lo32 = xl;
            a.ldx_lo32 = ldl;
            a.w_lo32 = wl;
            a.ldw_lo32 = ldl;
            std::exception_ptr err;
            try {
                hk::gemm_f16_tc(a, s, current_sms());
            } catch (...) {
                err = std::current_exception();
            }
            cudaFreeAsync(xl, s);
            cudaFreeAsync(wl, s);
            if (err) std::rethrow_exception(err);
        } else
            throw std::runtime_error(
                "hk_op_gemm: dtype must be 0 (fp32), 1 (fp16), 2 (fp16, CTA pairs) or 3 (fp32 as 3xTF32)");
    });
}

int hk_op_gemm_split(int epilogue, int M, int N, int K, const void *x, int ldx, const uint8_t *x_lo, int ldx_lo,
                     const void *w, int ldw, const uint8_t *w8, int ldw8, const float *scale, void *out, int ldo,
                     uint8_t *out_lo, int ldo_lo, int pairs, void *stream) {
    return op_guard([&] {
        if (!x || !x_lo || !w || !w8 || !out) throw std::invalid_argument("hk_op_gemm_split: null pointer");
        hk::GemmArgs a;
        a.M = M;
        a.N = N;
        a.K = K;
        a.x = x;
        a.ldx = ldx;
        a.x_lo = x_lo;
        a.ldx_lo = ldx_lo;
        a.w = w;
        a.ldw = ldw;
        a.w8 = w8;
        a.ldw8 = ldw8;
        a.scale = scale;
        a.out = out;
        a.ldo = ldo;
        a.out_lo = out_lo;
        a.ldo_lo = ldo_lo;
        a.epilogue = epilogue;
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        if (pairs)
            hk::gemm_f16_tc_pair(a, s, current_sms());
        else
            hk::gemm_f16_tc(a, s, current_sms());
    });
}

int hk_op_gemm_packed(int M, int N, int K, int kp, const float *x, int ldx, const int8_t *w_q, const float *w_d,
                      int8_t *x_q, float *x_d, float *out, int ldo, int residual, void *stream) {
    return op_guard([&] {
        if (M < 0 || N < 0 || K < 0 || kp <= 0 || kp % 32 != 0 || K > kp || ldx < K || ldo < N)
            throw std::runtime_error("hk_op_gemm_packed: bad shape");
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        if (M == 0 || N == 0) return;
        // The kernel reads block scales block-major: w_d [N, kp/32] transposed
        // into stream-ordered scratch; x_d is written block-major [kp/32, M].
        const int nb = kp / 32;
        float *wdt = nullptr;
        HK_CUDA(cudaMallocAsync(reinterpret_cast<void **>(&wdt), static_cast<size_t>(N) * nb * 4, s));
        std::exception_ptr err;
        try {
            hk::launch_transpose_scales(w_d, N, nb, wdt, s);
            hk::launch_quantize_rows(x, ldx, M, K, kp, x_q, x_d, s);
            hk::gemm_q8(x_q, x_d, w_q, wdt, M, N, kp, out, ldo, residual != 0, s, current_sms());
        } catch (...) {
            err = std::current_exception();
        }
        cudaFreeAsync(wdt, s);
        if (err) std::rethrow_exception(err);
    });
}

int hk_op_delta_recurrent(const float *q, const float *k, const float *v, const float *g, const float *beta,
                          const int32_t *cu_seqlens, int n_rows, int nk, int nv, int dk, int dv, int exact,
                          float *out, void *stream) {
    return op_guard([&] {
        hk::DeltaRecArgs a;
        a.q = q;
        a.k = k;
        a.v = v;
        a.g = g;
        a.beta = beta;
        a.cu_seqlens = cu_seqlens;
        a.n_rows = n_rows;
        a.nk = nk;
        a.nv = nv;
        a.dk = dk;
        a.dv = dv;
        a.out = out;
        a.exact = exact;
        hk::launch_delta_recurrent(a, static_cast<cudaStream_t>(stream));
    });
}

int hk_op_delta_chunked(int kernel, const float *q, const float *k, const float *v, const float *g, const float *beta,
                        const int32_t *cu_seqlens, int n_rows, int nk, int nv, const float *z, int ldz,
                        const float *norm_w, float eps, void *out, int ldo, void *stream) {
    return op_guard([&] {
        if (kernel != 0 && kernel != 1) throw std::invalid_argument("kernel must be 0 (mma.sync) or 1 (tcgen05)");
        if (nk <= 0 || nv <= 0 || nv % nk != 0) throw std::invalid_argument("value heads must be a multiple of key heads");
        if (z && (!norm_w || ldo < nv * 128 || ldz < nv * 128)) throw std::invalid_argument("bad gated-output layout");
        hk::DeltaRecArgs a;
        a.q = q;
        a.k = k;
        a.v = v;
        a.g = g;
        a.beta = beta;
        a.cu_seqlens = cu_seqlens;
        a.n_rows = n_rows;
        a.nk = nk;
        a.nv = nv;
        a.dk = 128;
        a.dv = 128;
        a.exact = 0;
        auto s = static_cast<cudaStream_t>(stream);
        if (!z) {
            a.out = static_cast<float *>(out);
            if (kernel == 0)
                hk::launch_delta_chunk(a, s);
            else
                hk::launch_delta_tc(a, s);
        } else {
            a.out = nullptr;
            __half *mix = static_cast<__half *>(out);
            if (kernel == 0)
                hk::launch_delta_chunk_gated(a, z, ldz, 0, norm_w, eps, mix, ldo, s);
            else
                hk::launch_delta_tc_gated(a, z, ldz, 0, norm_w, eps, mix, ldo, s);
        }
    });
}

int hk_op_delta_layer(const float *proj, int ldp, const int32_t *cu_seqlens, int n_rows, int nk, int nv,
                      const float *conv_w, const float *base_g, const float *dt_bias, const float *norm_w, float eps,
                      void *out, int ldo, void *stream) {
    return op_guard([&] {
        if (!proj || !cu_seqlens || !conv_w || !base_g || !dt_bias || !norm_w || !out)
            throw std::invalid_argument("hk_op_delta_layer: null pointer");
        if (n_rows < 0 || nk <= 0 || nv <= 0 || nv % nk != 0)
            throw std::invalid_argument("hk_op_delta_layer: value heads must be a positive multiple of key heads");
        const int conv_dim = 2 * nk * 128 + nv * 128;
        if (ldp < conv_dim + nv * 128 + 2 * nv || ldo < nv * 128)
            throw std::invalid_argument("hk_op_delta_layer: row strides too small for the heads");
        hk::DeltaRecArgs r;
        r.cu_seqlens = cu_seqlens;
        r.n_rows = n_rows;
        r.nk = nk;
        r.nv = nv;
        r.dk = 128;
        r.dv = 128;
        r.exact = 0;
        hk::DeltaFusedInput in;
        in.proj = proj;
        in.ldp = ldp;
        in.conv_dim = conv_dim;
        in.conv_w = conv_w;
        in.base_g = base_g;
        in.dt_bias = dt_bias;
        if (!hk::delta_pipe_supported(r, in))
            throw std::invalid_argument("hk_op_delta_layer: ldp must be a multiple of 4 floats");
        hk::launch_delta_pipe(r, in, norm_w, eps, static_cast<__half *>(out), ldo, static_cast<cudaStream_t>(stream));
    });
}

int hk_op_attention(int act, const void *q, const void *k, const void *v, const float *proj, int ldp,
                    const int32_t *cu_seqlens, const int32_t *tok_row, int n, int n_rows, int max_len, int nh,
                    int nkv, int hd, void *out, int ldo, void *stream) {
    return op_guard([&] {
        hk::AttnArgs a;
        a.q = q;
        a.k = k;
        a.v = v;
        a.proj = proj;
        a.ldp = ldp;
        a.cu_seqlens = cu_seqlens;
        a.tok_row = tok_row;
        a.n = n;
        a.n_rows = n_rows;
        a.max_len = max_len;
        a.nh = nh;
        a.nkv = nkv;
        a.hd = hd;
        a.out = out;
        a.ldo = ldo;
        a.kv_slots = n;  // flat K / V: one slot per token
        hk::launch_attention(act, a, static_cast<cudaStream_t>(stream));
    });
}

int hk_op_readout(const float *x, int hidden, const float *final_w, float eps, const int32_t *idx,
                  const int32_t *opt_dec, int n_dec, int n_opt, const float *wq, const float *bq, const float *wk,
                  const float *bk, int dp, float *hn, float *proj, float *logits, void *stream) {
    return op_guard([&] {
        hk::check_readout_args(x, hidden, final_w, idx, opt_dec, n_dec, n_opt, wq, bq, wk, bk, dp, logits);
        if (!hn || !proj) throw std::invalid_argument("hk_op_readout: null scratch pointer");
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
        a.hn = hn;
        a.proj = proj;
        a.logits = logits;
        hk::launch_readout(a, static_cast<cudaStream_t>(stream));
    });
}

int hk_op_answers(const float *logits, const int32_t *cu_positions, const int32_t *question_types, int n_rows,
                  float temperature, float *probs, void *answers, void *stream) {
    return op_guard([&] {
        if (n_rows < 0) throw std::invalid_argument("hk_op_answers: negative row count");
        if (n_rows > 0 && (!logits || !cu_positions || !question_types || !probs || !answers))
            throw std::invalid_argument("hk_op_answers: null pointer");
        if (!(temperature > 0.f) || !std::isfinite(temperature))
            throw std::invalid_argument("hk_op_answers: temperature must be positive and finite");
        hk::AnswerArgs a;
        a.logits = logits;
        a.cu_positions = cu_positions;
        a.qtype = question_types;
        a.n_rows = n_rows;
        a.temperature = temperature;
        a.probs = probs;
        a.out = static_cast<hk::AnswerRec *>(answers);
        hk::launch_answers(a, static_cast<cudaStream_t>(stream));
    });
}

int hk_op_num_sms(void) { return current_sms(); }

const char *hk_op_last_error(void) { return tl_op_error.c_str(); }

}  // extern "C"
