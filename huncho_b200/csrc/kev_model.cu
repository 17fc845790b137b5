// Kev scorer runtime: model-directory loading, device weight layout, the
// packed-batch forward and the C ABI declared in include/huncho_kev.h.
//
// The forward restates Model::forward_inner (crates/huncho-backend/src/
// qwen3_5.rs:1533-1553) for a packed batch of independent rows:
//   embed -> 24 x [RMSNorm -> mixer (Gated DeltaNet or gated GQA) -> +residual
//                  -> RMSNorm -> SwiGLU MLP -> +residual] -> pointer readout.
// Rows are packed without padding (cu_seqlens), which is what the reference's
// right padding amounts to for causal rows (qwen3_5.rs:3172-3177). The final
// RMSNorm is applied only at the readout rows (decision + option tokens),
// the only rows Qwen3_5Backend::readout reads (qwen3_5.rs:3196-3255).
#include <dirent.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <fstream>
#include <memory>
#include <sstream>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/huncho_kev.h"
#include "common.cuh"
#include "gemm.cuh"
#include "json.hpp"
#include "layers.cuh"
#include "safetensors.hpp"
#include "gguf.hpp"

namespace hk {

thread_local uint64_t tl_launches = 0;

namespace {

struct ApiError : std::runtime_error {
    int code;
    ApiError(int c, const std::string &m) : std::runtime_error(m), code(c) {}
};

std::string read_file(const std::string &p) {
    std::ifstream f(p, std::ios::binary);
    if (!f) throw ApiError(HK_ERR_PACKAGE, "cannot read " + p);
    std::stringstream ss;
    ss << f.rdbuf();
    return ss.str();
}

// ----------------------------------------------------------------- config
// Config::from_value (qwen3_5.rs:77-164), defaults included.
struct KevConfig {
    int hidden = 4096, layers = 32, nh = 16, nkv = 4, hd = 0, ffn = 12288, vocab = 248320;
    float eps = 1e-6f;
    std::vector<int> full;  // 1 = full attention layer
    int taps = 4, dk = 128, nk = 16, nv = 32, dv = 128;
    double theta = 10000.0, prf = 1.0;

    int rotary_dim() const {
        int d = static_cast<int>(std::llround(hd * prf));
        return std::max(d, 2) & ~1;
    }
    int key_dim() const { return nk * dk; }
    int value_dim() const { return nv * dv; }
    int conv_dim() const { return 2 * key_dim() + value_dim(); }

    static KevConfig from_json(const json::Value &root) {
        const json::Value *tc = root.get("text_config");
        const json::Value &t = tc ? *tc : root;
        auto num = [&](const char *k, double d) {
            const json::Value *v = t.get(k);
            return (v && v->is_num()) ? v->num : d;
        };
        KevConfig c;
        c.hidden = static_cast<int>(num("hidden_size", 4096));
        c.layers = static_cast<int>(num("num_hidden_layers", 32));
        c.nh = static_cast<int>(num("num_attention_heads", 16));
        c.nkv = static_cast<int>(num("num_key_value_heads", 4));
        c.hd = static_cast<int>(num("head_dim", c.hidden / std::max(c.nh, 1)));
        c.ffn = static_cast<int>(num("intermediate_size", 12288));
        c.vocab = static_cast<int>(num("vocab_size", 248320));
        c.eps = static_cast<float>(num("rms_norm_eps", 1e-6));
        const json::Value *lt = t.get("layer_types");
        if (lt && lt->kind == json::Value::Array) {
            for (auto &s : lt->arr) {
                if (s.str.find("full_attention") != std::string::npos)
                    c.full.push_back(1);
                else if (s.str.find("linear_attention") != std::string::npos)
                    c.full.push_back(0);
                else
                    throw ApiError(HK_ERR_PACKAGE, "unknown layer type `" + s.str + "`");
            }
        } else {
            int interval = std::max(1, static_cast<int>(num("full_attention_interval", 4)));
            for (int i = 0; i < c.layers; ++i) c.full.push_back((i + 1) % interval == 0);
        }
        c.taps = static_cast<int>(num("linear_conv_kernel_dim", 4));
        c.dk = static_cast<int>(num("linear_key_head_dim", 128));
        c.nk = static_cast<int>(num("linear_num_key_heads", 16));
        c.nv = static_cast<int>(num("linear_num_value_heads", 32));
        c.dv = static_cast<int>(num("linear_value_head_dim", 128));
        const json::Value *rp = t.get("rope_parameters");
        const json::Value *th = rp ? rp->get("rope_theta") : nullptr;
        if (!th || !th->is_num()) th = t.get("rope_theta");
        c.theta = (th && th->is_num()) ? th->num : 10000.0;
        const json::Value *pr = rp ? rp->get("partial_rotary_factor") : nullptr;
        if (!pr || !pr->is_num()) pr = t.get("partial_rotary_factor");
        c.prf = (pr && pr->is_num()) ? pr->num : 1.0;
        if (static_cast<int>(c.full.size()) < c.layers) c.full.resize(c.layers, 0);
        return c;
    }
};

// qwen3_5.rs:2496-2512.
bool canonical_weight_name(const std::string &name, std::string &out) {
    auto starts = [](const std::string &s, const char *p) { return s.rfind(p, 0) == 0; };
    if (starts(name, "model.language_model.") || starts(name, "lm_head.")) {
        out = name;
        return true;
    }
    std::string text = name;
    if (starts(name, "language_model."))
        text = name.substr(15);
    else if (starts(name, "model."))
        text = name.substr(6);
    if (starts(text, "layers.") || starts(text, "embed_tokens.") || starts(text, "norm.")) {
        out = "model.language_model." + text;
        return true;
    }
    return false;
}

uint16_t f32_to_bf16_bits(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x7FFFFFu)) return 0x7FC0;
    const uint32_t lsb = (u >> 16) & 1u;
    u += 0x7FFFu + lsb;
    return static_cast<uint16_t>(u >> 16);
}
float bf16_round(float f) {
    uint32_t u = static_cast<uint32_t>(f32_to_bf16_bits(f)) << 16;
    float r;
    std::memcpy(&r, &u, 4);
    return r;
}

// IEEE binary16 with round-to-nearest-even (overflow to inf, subnormals kept).
uint16_t f32_to_f16_bits(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) return static_cast<uint16_t>(sign | (ax > 0x7F800000u ? 0x7E00u : 0x7C00u));
    if (ax >= 0x477FF000u) return static_cast<uint16_t>(sign | 0x7C00u);  // rounds to >= 65520
    if (ax < 0x38800000u) {  // below 2^-14: subnormal (multiples of 2^-24) or zero
        float v;
        std::memcpy(&v, &ax, 4);
        return static_cast<uint16_t>(sign | static_cast<uint32_t>(std::nearbyint(v * 16777216.0f)));
    }
    uint32_t h = (((ax >> 23) - 112u) << 10) | ((ax & 0x7FFFFFu) >> 13);
    const uint32_t rem = ax & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
    return static_cast<uint16_t>(sign | h);
}
float f16_bits_to_f32(uint16_t h) {
    const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu, u;
    if (e == 0) {
        float v = static_cast<float>(m) * (1.0f / 16777216.0f);
        std::memcpy(&u, &v, 4);
        u |= sign;
    } else if (e == 31) {
        u = sign | 0x7F800000u | (m << 13);
    } else {
        u = sign | ((e + 112u) << 23) | (m << 13);
    }
    float r;
    std::memcpy(&r, &u, 4);
    return r;
}

// All base tensors of a model dir plus the adapter (merged on access), or the
// tensors of a packed package's backbone.gguf (merged at conversion).
class WeightSource {
  public:
    struct Packed {};
    WeightSource(const std::string &dir, Packed) : dir_(dir) {
        try {
            gguf_.reset(new GgufFile(dir + "/backbone.gguf"));
        } catch (const std::exception &e) {
            throw ApiError(HK_ERR_PACKAGE, std::string("packed Kev backbone: ") + e.what());
        }
        for (auto &kv : gguf_->tensors()) {
            std::string k;
            if (!canonical_weight_name(kv.first, k) || k.rfind("lm_head.", 0) == 0) continue;
            if (kv.second.type == kGgufF32) {
                views_.emplace_back(new TensorView);
                TensorView &v = *views_.back();
                v.dtype = "F32";
                v.shape = kv.second.shape;
                v.data = kv.second.data;
                v.nbytes = kv.second.nbytes;
                base_[k] = &v;
            } else {
                packed_[k] = &kv.second;
            }
        }
    }
    const GgufFile *gguf() const { return gguf_.get(); }
    const GgufTensor *packed(const std::string &k) const {
        auto it = packed_.find(k);
        return it == packed_.end() ? nullptr : it->second;
    }
    WeightSource(const std::string &dir) : dir_(dir) {
        DIR *d = opendir(dir.c_str());
        if (!d) throw ApiError(HK_ERR_PACKAGE, "cannot open model directory " + dir);
        std::vector<std::string> files;
        while (dirent *e = readdir(d)) {
            std::string n = e->d_name;
            if (n.size() > 12 && n.compare(n.size() - 12, 12, ".safetensors") == 0 &&
                n != "adapter_model.safetensors" && n != "pointer_head.safetensors" &&
                n != "joint_head.safetensors")
                files.push_back(n);
        }
        closedir(d);
        std::sort(files.begin(), files.end());
        if (files.empty())
            throw ApiError(HK_ERR_BACKEND, "no base-weight `*.safetensors` found in `" + dir + "`");
        for (auto &f : files) {
            shards_.emplace_back(new SafeTensors(dir + "/" + f));
            for (auto &kv : shards_.back()->tensors()) {
                std::string k;
                if (!canonical_weight_name(kv.first, k) || k.rfind("lm_head.", 0) == 0) continue;
                if (base_.count(k)) throw ApiError(HK_ERR_PACKAGE, "duplicate canonical base tensor `" + k + "`");
                base_[k] = &kv.second;
            }
        }
        std::ifstream probe(dir + "/adapter_model.safetensors");
        if (probe.good()) {
            adapter_.reset(new SafeTensors(dir + "/adapter_model.safetensors"));
            json::Value ac = json::parse(read_file(dir + "/adapter_config.json"));
            const json::Value *r = ac.get("r");
            const json::Value *al = ac.get("lora_alpha");
            rank_ = r && r->is_num() ? static_cast<int>(r->num) : 0;
            const float alpha = al && al->is_num() ? static_cast<float>(al->num) : static_cast<float>(rank_);
            lora_scale_ = rank_ > 0 ? alpha / static_cast<float>(rank_) : 1.0f;
            const std::string pre = "base_model.model.", suf = ".lora_A.weight";
            for (auto &kv : adapter_->tensors()) {
                const std::string &n = kv.first;
                if (n.rfind(pre, 0) != 0 || n.size() < pre.size() + suf.size() ||
                    n.compare(n.size() - suf.size(), suf.size(), suf) != 0)
                    continue;
                const std::string target = n.substr(pre.size(), n.size() - pre.size() - suf.size());
                auto bit = adapter_->tensors().find(pre + target + ".lora_B.weight");
                if (bit == adapter_->tensors().end())
                    throw ApiError(HK_ERR_BACKEND, "missing LoRA weight `" + pre + target + ".lora_B.weight`");
                std::string base;
                if (!canonical_weight_name(target + ".weight", base))
                    throw ApiError(HK_ERR_BACKEND, "unsupported LoRA target `" + target + "`");
                if (!base_.count(base))
                    throw ApiError(HK_ERR_BACKEND, "missing base weight `" + base + "` required for LoRA merge");
                lora_[base] = {&kv.second, &bit->second};
            }
        }
    }

    int lora_rank() const { return adapter_ ? rank_ : 0; }

    // fp32 copy of a base tensor with its LoRA delta merged in fp32:
    // W += (alpha / r) * (B @ A), the rank sum in ascending order
    // (qwen3_5.rs:1597-1640).
    std::vector<float> get(const std::string &k, const std::vector<int64_t> &shape) const {
        auto it = base_.find(k);
        if (it == base_.end()) throw ApiError(HK_ERR_PACKAGE, "missing tensor `" + k + "`");
        const TensorView &t = *it->second;
        int64_t want = 1;
        for (auto d : shape) want *= d;
        if (t.numel() != want) {
            std::ostringstream os;
            os << "tensor `" << k << "` has " << t.numel() << " elements, expected " << want;
            throw ApiError(HK_ERR_PACKAGE, os.str());
        }
        std::vector<float> w = to_f32(t);
        auto lit = lora_.find(k);
        if (lit != lora_.end()) {
            std::vector<float> a = to_f32(*lit->second.first), b = to_f32(*lit->second.second);
            const int64_t r = lit->second.first->shape.at(0), in = lit->second.first->shape.at(1);
            const int64_t out = lit->second.second->shape.at(0);
            if (shape.size() != 2 || shape[0] != out || shape[1] != in || lit->second.second->shape.at(1) != r)
                throw ApiError(HK_ERR_BACKEND, "LoRA shape mismatch for `" + k + "`");
            for (int64_t o = 0; o < out; ++o)
                for (int64_t i = 0; i < in; ++i) {
                    float d = 0.0f;
                    for (int64_t j = 0; j < r; ++j) d = d + b[o * r + j] * a[j * in + i];
                    w[o * in + i] = w[o * in + i] + d * lora_scale_;
                }
        }
        return w;
    }

  private:
    std::string dir_;
    std::unique_ptr<GgufFile> gguf_;
    std::vector<std::unique_ptr<TensorView>> views_;
    std::unordered_map<std::string, const GgufTensor *> packed_;
    std::vector<std::unique_ptr<SafeTensors>> shards_;
    std::unordered_map<std::string, const TensorView *> base_;
    std::unique_ptr<SafeTensors> adapter_;
    std::unordered_map<std::string, std::pair<const TensorView *, const TensorView *>> lora_;
    int rank_ = 0;
    float lora_scale_ = 1.0f;
};

// ----------------------------------------------------------------- device weights
struct Mat {
    void *w = nullptr;
    float *scale = nullptr;  // int8-weight models: per row
    int rows = 0, cols = 0, ld = 0;
    // int8-weight models: the int8 values [rows, ld] (w stays null); each
    // projection expands them to fp16 in the handle's scratch right before its
    // GEMM, and the per-row scale is applied in the GEMM epilogue.
    int8_t *q8 = nullptr;
    // Split-precision projections (the delta layers' and the MLPs' in the
    // half-precision models): an e4m3 copy of the weight values [rows, ld8
    // bytes] for the low part of the input (GemmArgs::w8); for int8 weights,
    // of the int8 values (the row scale applies to both parts).
    uint8_t *w8 = nullptr;
    int ld8 = 0;
    // fp32 model: w - tf32(w) [rows, ld] for the 3xTF32 tensor-core GEMM.
    float *w_lo = nullptr;
    // Packed profiles: int8 block values [rows, kp] and fp32 block scales,
    // block-major [kp / 32, rows] (a warp's 32 rows read one line per block).
    int8_t *q = nullptr;
    float *qd = nullptr;
    int kp = 0;
};

struct Layer {
    bool full = false;
    float *in_norm = nullptr, *post_norm = nullptr;
    Mat mix_in, mix_out, gu, down;
    float *conv_w = nullptr, *base_g = nullptr, *dt_bias = nullptr, *gnorm_w = nullptr;
    float *qn_w = nullptr, *kn_w = nullptr;
};

int round_up(int v, int m) { return (v + m - 1) / m * m; }

}  // namespace

// The device memory of a loaded package's immutable tensors (projections,
// embedding table, norms, conv and gate parameters, pointer head). Handles on
// the same GPU share one store (the reference's replicas share their weights
// through Arc clones, qwen3_5.rs:2515-2535); the last handle frees it.
struct WeightStore {
    int device = 0;
    std::vector<void *> allocs;
    size_t bytes = 0;
    ~WeightStore() {
        if (allocs.empty()) return;
        cudaSetDevice(device);
        for (void *p : allocs) cudaFree(p);
    }
};

struct Model {
    std::string dir;
    int device = 0;
    int dtype = HK_DTYPE_BF16;
    int max_context = 0;
    int num_sms = 148;
    KevConfig cfg;
    bool fused_swiglu = false;
    int lora_rank = 0;
    float temperature = 1.0f;
    int dp = 256;
    cudaStream_t stream = nullptr;
    std::shared_ptr<WeightStore> wstore = std::make_shared<WeightStore>();
    std::vector<void *> allocs;  // this handle's own small buffers (error word, cache table)
    void *embed = nullptr;
    float *final_norm = nullptr;
    float *inv_freq = nullptr;
    float *wq = nullptr, *bq = nullptr, *wk = nullptr, *bk = nullptr;
    std::vector<Layer> layers;

    // workspace
    int cap_tokens = 0, cap_rows = 0, cap_readouts = 0;
    std::vector<void *> ws;
    float *x = nullptr;
    void *xn = nullptr, *mix = nullptr, *ffn = nullptr;
    // e5m2 low parts of xn / mix / ffn for split-precision projections (rows of
    // ld_xl / ld_mixl / ld_fl bytes), or null.
    uint8_t *xn_lo = nullptr, *mix_lo = nullptr, *ffn_lo = nullptr;
    int ld_xl = 0, ld_mixl = 0, ld_fl = 0;
    float *x_lo32 = nullptr;  // fp32 model: x - tf32(x) of the projection input in flight
    int ld_lo32 = 0;
    float *proj = nullptr;  // projection outputs, always fp32
    float *dq = nullptr, *dkk = nullptr, *dvv = nullptr, *dg = nullptr, *db = nullptr, *dout = nullptr;
    void *aq = nullptr, *ak = nullptr, *av = nullptr;
    float *hn = nullptr, *rproj = nullptr, *logits = nullptr;
    // Packed profiles: Q8_0 activation rows for the projection in flight.
    int8_t *xq = nullptr;
    float *xd = nullptr;
    int max_kp = 0;
    std::map<std::string, int> packed_widths;  // huncho.input_widths
    float *probs = nullptr;           // calibrated probabilities (hk_score_answers)
    AnswerRec *answers = nullptr;     // [cap_rows]
    int32_t *qtype_dev = nullptr;     // [cap_rows]
    uint32_t *err = nullptr;
    __half *wdq = nullptr;  // int8-weight models: the projection in flight, expanded to fp16
    uint8_t *wdq8 = nullptr;  // ... and to e4m3 (the split-precision low part's weights)
    // device batch description (see build_meta_kernel)
    int32_t *meta = nullptr;
    size_t meta_cap = 0;
    // pinned staging for hk_score
    void *pinned = nullptr;
    size_t pinned_cap = 0;
    int ld_xn = 0, ldp = 0, ldmix = 0, ldf = 0;
    // KV pages (0 = flat K/V) and the page-order shuffle seed (0 = in order).
    int kv_page_tokens = 0;
    uint64_t kv_shuffle_seed = 0;
    int kv_slot_cap = 0;  // K/V slots the ak/av buffers hold
    std::vector<int32_t> row_order;  // host copy of the last batch's row order
    // Pinned host staging for the small per-batch uploads of the device-input
    // path (a ring, so a buffer is reused only after its copy has completed).
    struct HostStage {
        uint8_t *p = nullptr;
        size_t cap = 0;
        cudaEvent_t done = nullptr;
    };
    HostStage stages[4];
    int stage_next = 0;
    HostStage &stage_acquire(size_t bytes) {
        HostStage &st = stages[stage_next];
        stage_next = (stage_next + 1) % 4;
        if (st.done) HK_CUDA(cudaEventSynchronize(st.done));
        if (bytes > st.cap) {
            if (st.p) cudaFreeHost(st.p);
            st.p = nullptr;
            st.cap = 0;
            HK_CUDA(cudaHostAlloc(reinterpret_cast<void **>(&st.p), bytes * 2, cudaHostAllocDefault));
            st.cap = bytes * 2;
        }
        if (!st.done) HK_CUDA(cudaEventCreateWithFlags(&st.done, cudaEventDisableTiming));
        return st;
    }
    uint64_t launches = 0;
    std::string last_error;

    // ------------------------------------------------------------ prefix caches
    // A cached prefix (the reference's LayerCache / ModelCache behind prefill
    // and fork, qwen3_5.rs:1111-1125): the model state after `tokens` tokens,
    // in one device buffer. Per delta layer, in layer order: the recurrent
    // state [nv][dk][dv] fp32, then the conv inputs of the last taps-1 tokens
    // [taps-1][conv_dim] fp32 (oldest first, zero before the sequence start).
    // Then per attention layer: K then V [tokens][nkv][hd] in the activation
    // type. A snapshot is immutable once written and handles share it, so a
    // fork is a reference; a continued branch gets a new snapshot.
    struct Snapshot {
        int tokens = 0;
        void *buf = nullptr;
        int device = 0;
        cudaStream_t stream = nullptr;
        ~Snapshot() {
            if (buf) {
                cudaSetDevice(device);
                cudaFreeAsync(buf, stream);
            }
        }
    };
    std::unordered_map<uint64_t, std::shared_ptr<Snapshot>> caches;
    // Handle ids come from one process-wide counter, so a handle is never
    // valid in another loaded model (the reference's next_cache_handle).
    static uint64_t next_cache_id() {
        static std::atomic<uint64_t> next{1};
        return next.fetch_add(1);
    }
    std::vector<int> layer_slot;  // index among the delta layers, or among the attention layers
    int n_delta = 0, n_attn = 0;
    // Device table of a cached batch: 4 x [layers][rows] addresses (in
    // state|K, in conv history, out state|K, out conv history), then the
    // per-row prefix lengths.
    uint64_t *cache_meta = nullptr;

    static size_t r256(size_t v) { return (v + 255) / 256 * 256; }
    size_t delta_state_bytes() const { return static_cast<size_t>(cfg.nv) * cfg.dk * cfg.dv * 4; }
    size_t delta_block() const {
        return r256(delta_state_bytes() + static_cast<size_t>(cfg.taps - 1) * cfg.conv_dim() * 4);
    }
    size_t kv_block(int tokens) const { return r256(2 * static_cast<size_t>(tokens) * cfg.nkv * cfg.hd * esz()); }
    size_t snapshot_bytes(int tokens) const { return n_delta * delta_block() + n_attn * kv_block(tokens); }
    // Layer li's piece of a snapshot: delta state (conv history right after
    // it), or attention K (V right after it).
    uint64_t piece(const Snapshot &sn, int li) const {
        const uint64_t b = reinterpret_cast<uint64_t>(sn.buf);
        if (!layers[li].full) return b + layer_slot[li] * delta_block();
        return b + n_delta * delta_block() + layer_slot[li] * kv_block(sn.tokens);
    }
    // Snapshots come from the model's own stream-ordered pool, which keeps
    // freed memory for reuse instead of returning it at every synchronisation.
    cudaMemPool_t pool = nullptr;
    std::shared_ptr<Snapshot> new_snapshot(int tokens) {
        if (!pool) {
            cudaMemPoolProps props = {};
            props.allocType = cudaMemAllocationTypePinned;
            props.location.type = cudaMemLocationTypeDevice;
            props.location.id = device;
            HK_CUDA(cudaMemPoolCreate(&pool, &props));
            uint64_t keep = UINT64_MAX;
            HK_CUDA(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep));
        }
        auto sn = std::make_shared<Snapshot>();
        sn->tokens = tokens;
        sn->device = device;
        sn->stream = stream;
        HK_CUDA(cudaMallocFromPoolAsync(&sn->buf, std::max<size_t>(snapshot_bytes(tokens), 256), pool, stream));
        return sn;
    }

    // Optional per-class device timing of the forward's launches (CUDA events
    // on the handle's stream), with each launch's algorithmic FLOPs and HBM
    // bytes (one read of every input, one write of every output): 0 GEMM,
    // 1 delta layer / recurrence, 2 attention, 3 delta input stage, 4 other
    // (conv history, SwiGLU, gated norm), 5 RMSNorm, 6 attention input stage,
    // 7 readout, 8 embedding.
    static constexpr int kProfClasses = 9;
    bool prof = false;
    double attn_pairs = 0.0;  // sum over the batch's rows of T (T + 1) / 2 (causal query-key pairs)
    struct ProfRec {
        cudaEvent_t a, b;
        int cls;
        double flops, bytes;
    };
    std::vector<ProfRec> prof_recs;
    std::vector<cudaEvent_t> prof_pool;
    cudaEvent_t prof_event() {
        if (!prof_pool.empty()) {
            cudaEvent_t e = prof_pool.back();
            prof_pool.pop_back();
            return e;
        }
        cudaEvent_t e;
        HK_CUDA(cudaEventCreate(&e));
        return e;
    }
    cudaEvent_t prof_begin() {
        if (!prof) return nullptr;
        cudaEvent_t e = prof_event();
        HK_CUDA(cudaEventRecord(e, stream));
        return e;
    }
    void prof_end(cudaEvent_t a, int cls, double flops, double bytes = 0.0) {
        if (!prof || !a) return;
        cudaEvent_t b = prof_event();
        HK_CUDA(cudaEventRecord(b, stream));
        prof_recs.push_back({a, b, cls, flops, bytes});
    }

    bool packed() const { return dtype == HK_DTYPE_Q8_0 || dtype == HK_DTYPE_Q4_0; }
    // Half-precision models run the delta layers' and the MLPs' projections
    // with split-precision inputs (fp16 high part + e5m2 low part, see
    // GemmArgs::x_lo): fp16 rounding of those inputs alone moves calibrated
    // probabilities of the 0.8B / 4B models by up to 2-4e-3 against the fp32
    // reference; the low part brings it under 3e-4. The attention layers'
    // projections are insensitive (< 3e-5) and stay fp16.
    bool split_inputs() const { return dtype == HK_DTYPE_BF16 || dtype == HK_DTYPE_FP16 || dtype == HK_DTYPE_INT8W; }
    // The fp32 model path: fp32 weights, or the packed profiles (fp32 activations).
    bool f32_model() const { return dtype == HK_DTYPE_FP32 || packed(); }
    int act() const { return f32_model() ? kActF32 : kActF16; }
    size_t esz() const { return f32_model() ? 4 : 2; }
    // The checkpoint value in the model dtype (the reference casts every
    // tensor to it at load): bf16 for the bf16 and int8-weight models.
    float model_round(float v) const {
        if (dtype == HK_DTYPE_BF16 || dtype == HK_DTYPE_INT8W) return bf16_round(v);
        if (dtype == HK_DTYPE_FP16) return f16_bits_to_f32(f32_to_f16_bits(v));
        return v;
    }

    ~Model() {
        if (device >= 0) cudaSetDevice(device);
        caches.clear();
        if (stream) cudaStreamSynchronize(stream);
        if (pool) cudaMemPoolDestroy(pool);
        for (auto &r : prof_recs) {
            cudaEventDestroy(r.a);
            cudaEventDestroy(r.b);
        }
        for (auto e : prof_pool) cudaEventDestroy(e);
        for (auto &st : stages) {
            if (st.p) cudaFreeHost(st.p);
            if (st.done) cudaEventDestroy(st.done);
        }
        for (void *p : ws) cudaFree(p);
        for (void *p : allocs) cudaFree(p);
        wstore.reset();
        if (pinned) cudaFreeHost(pinned);
        if (stream) cudaStreamDestroy(stream);
    }

    template <typename T>
    T *dev_alloc(size_t count, std::vector<void *> &owner) {
        void *p = nullptr;
        const size_t bytes = std::max<size_t>(count, 1) * sizeof(T);
        HK_CUDA(cudaMalloc(&p, bytes));
        owner.push_back(p);
        if (&owner == &wstore->allocs) wstore->bytes += bytes;
        return static_cast<T *>(p);
    }
    std::vector<void *> &walloc() { return wstore->allocs; }
    float *upload_f32(const std::vector<float> &v) {
        float *p = dev_alloc<float>(v.size(), walloc());
        HK_CUDA(cudaMemcpy(p, v.data(), v.size() * sizeof(float), cudaMemcpyHostToDevice));
        return p;
    }

    // Pack row blocks [(tensor, rows)] into one [R, K] matrix in the model's
    // weight format. `order` optionally permutes output rows (SwiGLU interleave).
    // The e4m3 copy of a projection for split-precision inputs: vals [R][K]
    // (row-major, the values the fp16 operand holds), rows padded to 16 bytes.
    void make_w8(Mat &m, const std::vector<float> &vals, int R, int K) {
        m.ld8 = round_up(K, 16);
        std::vector<uint8_t> h(static_cast<size_t>(R) * m.ld8, 0);
        for (int r = 0; r < R; ++r)
            for (int i = 0; i < K; ++i)
                h[static_cast<size_t>(r) * m.ld8 + i] = static_cast<uint8_t>(
                    __nv_cvt_float_to_fp8(vals[static_cast<size_t>(r) * K + i], __NV_SATFINITE, __NV_E4M3));
        m.w8 = dev_alloc<uint8_t>(h.size(), walloc());
        HK_CUDA(cudaMemcpy(m.w8, h.data(), h.size(), cudaMemcpyHostToDevice));
    }

    Mat pack(const WeightSource &src, const std::vector<std::pair<std::string, int>> &parts, int K,
             const std::vector<int> *order = nullptr, bool split = false) {
        if (packed()) return pack_blocks(src, parts, K);
        int R = 0;
        for (auto &p : parts) R += p.second;
        std::vector<float> full(static_cast<size_t>(R) * K);
        int r0 = 0;
        for (auto &p : parts) {
            std::vector<float> w = src.get(p.first, {p.second, K});
            std::memcpy(full.data() + static_cast<size_t>(r0) * K, w.data(), w.size() * sizeof(float));
            r0 += p.second;
        }
        Mat m;
        m.rows = R;
        m.cols = K;
        m.ld = round_up(K, 8);
        auto src_row = [&](int r) { return order ? (*order)[r] : r; };
        if (dtype == HK_DTYPE_FP32) {
            std::vector<float> h(static_cast<size_t>(R) * m.ld, 0.0f);
            for (int r = 0; r < R; ++r)
                std::memcpy(&h[static_cast<size_t>(r) * m.ld], &full[static_cast<size_t>(src_row(r)) * K], K * 4);
            float *d = dev_alloc<float>(h.size(), walloc());
            HK_CUDA(cudaMemcpy(d, h.data(), h.size() * 4, cudaMemcpyHostToDevice));
            m.w = d;
            // The low part of each weight for the 3xTF32 GEMM.
            for (auto &v : h) v -= tf32_trunc_host(v);
            m.w_lo = dev_alloc<float>(h.size(), walloc());
            HK_CUDA(cudaMemcpy(m.w_lo, h.data(), h.size() * 4, cudaMemcpyHostToDevice));
        } else if (dtype == HK_DTYPE_INT8W) {
            m.ld = round_up(K, 16);  // the int8 rows double as the e4m3 rows' layout
            // Symmetric per-output-channel int8: scale = max|w| / 127,
            // q = rint(w / scale) clamped to [-127, 127]; zero rows get scale 1.
            std::vector<int8_t> h(static_cast<size_t>(R) * m.ld, 0);
            std::vector<float> sc(R);
            for (int r = 0; r < R; ++r) {
                const float *row = &full[static_cast<size_t>(src_row(r)) * K];
                int8_t *dst = &h[static_cast<size_t>(r) * m.ld];
                float amax = 0.0f;
                for (int i = 0; i < K; ++i) amax = std::max(amax, std::fabs(row[i]));
                float s = amax / 127.0f;
                if (s == 0.0f) s = 1.0f;
                sc[r] = s;
                for (int i = 0; i < K; ++i) {
                    float q = std::nearbyint(row[i] / s);
                    dst[i] = static_cast<int8_t>(std::min(127.0f, std::max(-127.0f, q)));
                }
            }
            m.q8 = dev_alloc<int8_t>(h.size(), walloc());
            HK_CUDA(cudaMemcpy(m.q8, h.data(), h.size(), cudaMemcpyHostToDevice));
            m.scale = upload_f32(sc);
            // The e4m3 copy for split-precision inputs is expanded per
            // projection with the fp16 values, so device memory holds int8 only.
            if (split) m.ld8 = m.ld;
        } else {
            std::vector<uint16_t> h(static_cast<size_t>(R) * m.ld, 0);
            for (int r = 0; r < R; ++r) {
                const float *row = &full[static_cast<size_t>(src_row(r)) * K];
                uint16_t *dst = &h[static_cast<size_t>(r) * m.ld];
                // bf16 checkpoint values convert to fp16 exactly unless |w| < 2^-17.
                for (int i = 0; i < K; ++i) dst[i] = f32_to_f16_bits(model_round(row[i]));
            }
            uint16_t *d = dev_alloc<uint16_t>(h.size(), walloc());
            HK_CUDA(cudaMemcpy(d, h.data(), h.size() * 2, cudaMemcpyHostToDevice));
            m.w = d;
            if (split) {
                std::vector<float> vals(static_cast<size_t>(R) * K);
                for (int r = 0; r < R; ++r)
                    for (int i = 0; i < K; ++i)
                        vals[static_cast<size_t>(r) * K + i] = f16_bits_to_f32(h[static_cast<size_t>(r) * m.ld + i]);
                make_w8(m, vals, R, K);
            }
        }
        return m;
    }

    // Packed projections: the artifact's Q8_0 / Q4_0 blocks of each part,
    // rows concatenated, as int8 values (Q4_0 as q - 8) and fp32 scales
    // (block-major).
    Mat pack_blocks(const WeightSource &src, const std::vector<std::pair<std::string, int>> &parts, int K) {
        const uint32_t want = dtype == HK_DTYPE_Q8_0 ? kGgufQ8_0 : kGgufQ4_0;
        const int kp = round_up(K, 32), nb = kp / 32;
        int R = 0;
        for (auto &p : parts) R += p.second;
        std::vector<int8_t> q(static_cast<size_t>(R) * kp);
        std::vector<float> d(static_cast<size_t>(R) * nb);
        int r0 = 0;
        for (auto &p : parts) {
            const GgufTensor *t = src.packed(p.first);
            if (!t) throw ApiError(HK_ERR_PACKAGE, "packed projection `" + p.first + "` missing");
            if (t->type != want)
                throw ApiError(HK_ERR_PACKAGE, "packed projection `" + p.first + "` has another block type");
            auto wit = packed_widths.find(p.first);
            if (t->shape.size() != 2 || t->shape[0] != p.second || t->shape[1] != kp || wit == packed_widths.end() ||
                wit->second != K)
                throw ApiError(HK_ERR_PACKAGE, "packed projection `" + p.first + "` shape mismatch");
            const int per = want == kGgufQ8_0 ? 34 : 18;
            for (int r = 0; r < p.second; ++r)
                for (int b = 0; b < nb; ++b) {
                    const uint8_t *blk = t->data + (static_cast<size_t>(r) * nb + b) * per;
                    uint16_t h;
                    std::memcpy(&h, blk, 2);
                    d[static_cast<size_t>(b) * R + r0 + r] = f16_bits_to_f32(h);
                    int8_t *dst = &q[static_cast<size_t>(r0 + r) * kp + b * 32];
                    if (want == kGgufQ8_0) {
                        std::memcpy(dst, blk + 2, 32);
                    } else {
                        for (int j = 0; j < 16; ++j) {
                            dst[j] = static_cast<int8_t>((blk[2 + j] & 0x0F) - 8);
                            dst[16 + j] = static_cast<int8_t>((blk[2 + j] >> 4) - 8);
                        }
                    }
                }
            r0 += p.second;
        }
        Mat m;
        m.rows = R;
        m.cols = K;
        m.ld = kp;
        m.kp = kp;
        m.q = dev_alloc<int8_t>(q.size(), walloc());
        HK_CUDA(cudaMemcpy(m.q, q.data(), q.size(), cudaMemcpyHostToDevice));
        m.qd = upload_f32(d);
        max_kp = std::max(max_kp, kp);
        return m;
    }

    // A small fp32 tensor, rounded to the model dtype first (the reference
    // loader casts every tensor to it) and kept in fp32 on the device.
    std::vector<float> small(const WeightSource &src, const std::string &k, std::vector<int64_t> shape) {
        std::vector<float> v = src.get(k, shape);
        for (auto &x : v) x = model_round(x);
        return v;
    }
    float *norm_eff(const WeightSource &src, const std::string &k, int n) {
        std::vector<float> v = small(src, k, {n});
        for (auto &x : v) x = x * 1.0f + 1.0f;  // effective_norm_weight, qwen3_5.rs:180-182
        return upload_f32(v);
    }

    void load(const std::string &model_dir) {
        dir = model_dir;
        wstore->device = device;
        std::unique_ptr<WeightSource> srcp(packed() ? new WeightSource(model_dir, WeightSource::Packed{})
                                                    : new WeightSource(model_dir));
        const WeightSource &src = *srcp;
        if (packed()) {
            // The artifact's profile must be the requested one (load_quantized_kev).
            const GgufFile &g = *src.gguf();
            const char *profile = dtype == HK_DTYPE_Q8_0 ? "kev-projections-q8_0-fp32-v1" : "kev-projections-q4_0-fp32-v1";
            auto q = g.strings().find("huncho.quantization");
            if (q == g.strings().end() || q->second != profile)
                throw ApiError(HK_ERR_PACKAGE, std::string("packed Kev artifact is not ") + profile);
            auto cj = g.strings().find("huncho.config_json");
            auto wj = g.strings().find("huncho.input_widths");
            if (cj == g.strings().end() || wj == g.strings().end())
                throw ApiError(HK_ERR_PACKAGE, "packed Kev artifact lacks its config or input widths");
            cfg = KevConfig::from_json(json::parse(cj->second));
            json::Value widths = json::parse(wj->second);
            for (auto &kv : widths.obj) packed_widths[kv.first] = static_cast<int>(kv.second.num);
        } else {
            cfg = KevConfig::from_json(json::parse(read_file(model_dir + "/config.json")));
        }
        const KevConfig &c = cfg;
        if (c.nv % c.nk != 0) throw ApiError(HK_ERR_UNSUPPORTED, "value heads must be a multiple of key heads");
        if (c.nh % c.nkv != 0) throw ApiError(HK_ERR_UNSUPPORTED, "query heads must be a multiple of kv heads");
        lora_rank = src.lora_rank();
        // Pointer head (kev.rs:118-165): fp32, shapes [dp, hidden] and [dp].
        json::Value meta = json::parse(read_file(model_dir + "/kev_head.json"));
        const json::Value *tv = meta.get("temperature");
        temperature = tv && tv->is_num() ? static_cast<float>(tv->num) : 1.0f;
        if (!std::isfinite(temperature) || temperature <= 0.0f)
            throw ApiError(HK_ERR_PACKAGE, "invalid Kev head: temperature must be finite and positive");
        const json::Value *hdv = meta.get("head_dim");
        dp = hdv && hdv->is_num() ? static_cast<int>(hdv->num) : 256;
        {
            SafeTensors head(model_dir + "/pointer_head.safetensors");
            auto get = [&](const std::string &n, std::vector<int64_t> shape) {
                auto it = head.tensors().find(n);
                if (it == head.tensors().end()) throw ApiError(HK_ERR_PACKAGE, "invalid Kev head: missing `" + n + "`");
                if (it->second.shape != shape) {
                    std::ostringstream os;
                    os << "invalid Kev head: `" << n << "` shape mismatch, expected [";
                    for (size_t i = 0; i < shape.size(); ++i) os << (i ? ", " : "") << shape[i];
                    os << "]";
                    throw ApiError(HK_ERR_PACKAGE, os.str());
                }
                std::vector<float> v = to_f32(it->second);
                for (float f : v)
                    if (!std::isfinite(f)) throw ApiError(HK_ERR_PACKAGE, "invalid Kev head: `" + n + "` contains non-finite weights");
                return upload_f32(v);
            };
            wq = get("q.weight", {dp, c.hidden});
            bq = get("q.bias", {dp});
            wk = get("k.weight", {dp, c.hidden});
            bk = get("k.bias", {dp});
        }
        // Embedding table in the model dtype.
        {
            std::vector<float> e = src.get("model.language_model.embed_tokens.weight",
                                           {static_cast<int64_t>(c.vocab), c.hidden});
            if (f32_model()) {
                float *d = dev_alloc<float>(e.size(), walloc());
                HK_CUDA(cudaMemcpy(d, e.data(), e.size() * 4, cudaMemcpyHostToDevice));
                embed = d;
            } else {
                std::vector<uint16_t> h(e.size());
                for (size_t i = 0; i < e.size(); ++i) h[i] = f32_to_f16_bits(model_round(e[i]));
                uint16_t *d = dev_alloc<uint16_t>(h.size(), walloc());
                HK_CUDA(cudaMemcpy(d, h.data(), h.size() * 2, cudaMemcpyHostToDevice));
                embed = d;
            }
        }
        final_norm = norm_eff(src, "model.language_model.norm.weight", c.hidden);
        // RoPE inverse frequencies in fp32 (qwen3_5.rs:225-232).
        {
            const int rd = c.rotary_dim(), half = rd / 2;
            std::vector<float> inv(std::max(half, 1));
            for (int i = 0; i < half; ++i)
                inv[i] = std::pow(static_cast<float>(c.theta), -(2.0f * static_cast<float>(i)) / static_cast<float>(rd));
            inv_freq = upload_f32(inv);
        }
        fused_swiglu = !f32_model() && (c.ffn % kSwiGLUBlock) == 0;
        std::vector<int> gu_order;
        if (fused_swiglu) {
            for (int b = 0; b < c.ffn / kSwiGLUBlock; ++b) {
                for (int i = 0; i < kSwiGLUBlock; ++i) gu_order.push_back(b * kSwiGLUBlock + i);
                for (int i = 0; i < kSwiGLUBlock; ++i) gu_order.push_back(c.ffn + b * kSwiGLUBlock + i);
            }
        }
        for (int i = 0; i < c.layers; ++i) {
            const std::string p = "model.language_model.layers." + std::to_string(i);
            Layer L;
            L.full = c.full[i] != 0;
            L.in_norm = norm_eff(src, p + ".input_layernorm.weight", c.hidden);
            L.post_norm = norm_eff(src, p + ".post_attention_layernorm.weight", c.hidden);
            if (!L.full) {
                const std::string a = p + ".linear_attn";
                L.mix_in = pack(src, {{a + ".in_proj_qkv.weight", c.conv_dim()}, {a + ".in_proj_z.weight", c.value_dim()},
                                      {a + ".in_proj_b.weight", c.nv}, {a + ".in_proj_a.weight", c.nv}},
                                c.hidden, nullptr, split_inputs());
                L.mix_out = pack(src, {{a + ".out_proj.weight", c.hidden}}, c.value_dim(), nullptr, split_inputs());
                L.conv_w = upload_f32(small(src, a + ".conv1d.weight", {c.conv_dim(), 1, c.taps}));
                std::vector<float> alog = small(src, a + ".A_log", {c.nv});
                for (auto &v : alog) v = -std::exp(v);  // base_g = -exp(A_log), qwen3_5.rs:800
                L.base_g = upload_f32(alog);
                L.dt_bias = upload_f32(small(src, a + ".dt_bias", {c.nv}));
                L.gnorm_w = upload_f32(small(src, a + ".norm.weight", {c.dv}));
            } else {
                const std::string a = p + ".self_attn";
                L.mix_in = pack(src, {{a + ".q_proj.weight", c.nh * c.hd * 2}, {a + ".k_proj.weight", c.nkv * c.hd},
                                      {a + ".v_proj.weight", c.nkv * c.hd}},
                                c.hidden);
                L.mix_out = pack(src, {{a + ".o_proj.weight", c.hidden}}, c.nh * c.hd);
                L.qn_w = norm_eff(src, a + ".q_norm.weight", c.hd);
                L.kn_w = norm_eff(src, a + ".k_norm.weight", c.hd);
            }
            const std::string m = p + ".mlp";
            L.gu = pack(src, {{m + ".gate_proj.weight", c.ffn}, {m + ".up_proj.weight", c.ffn}}, c.hidden,
                        fused_swiglu ? &gu_order : nullptr, split_inputs());
            L.down = pack(src, {{m + ".down_proj.weight", c.hidden}}, c.ffn, nullptr, split_inputs());
            layers.push_back(L);
        }
        ld_xn = round_up(c.hidden, 8);
        const int pd = c.conv_dim() + c.value_dim() + 2 * c.nv;
        const int pa = c.nh * c.hd * 2 + 2 * c.nkv * c.hd;
        ldp = round_up(std::max(std::max(pd, pa), fused_swiglu ? 0 : 2 * c.ffn), 8);
        ldmix = round_up(std::max(c.value_dim(), c.nh * c.hd), 8);
        ldf = round_up(c.ffn, 8);
        for (const Layer &L : layers) layer_slot.push_back(L.full ? n_attn++ : n_delta++);
        alloc_handle_state();
    }

    // The per-handle device state next to the weights: the error word and the
    // cached-batch address table.
    void alloc_handle_state() {
        if (dtype == HK_DTYPE_INT8W) {
            size_t most = 0;
            for (const Layer &L : layers)
                for (const Mat *m : {&L.mix_in, &L.mix_out, &L.gu, &L.down})
                    most = std::max(most, static_cast<size_t>(m->rows) * m->ld);
            wdq = dev_alloc<__half>(most, allocs);
            wdq8 = dev_alloc<uint8_t>(most, allocs);
        }
        err = dev_alloc<uint32_t>(1, allocs);
        HK_CUDA(cudaMemset(err, 0, 4));
        cache_meta = dev_alloc<uint64_t>(4 * layers.size() * HK_MAX_CACHED_ROWS + HK_MAX_CACHED_ROWS, allocs);
    }

    // A replica on the source's GPU: the same immutable weights (shared, not
    // copied), its own stream, workspace, error word, caches and settings.
    void share_weights(const Model &src) {
        dir = src.dir;
        cfg = src.cfg;
        fused_swiglu = src.fused_swiglu;
        lora_rank = src.lora_rank;
        temperature = src.temperature;
        dp = src.dp;
        wstore = src.wstore;
        embed = src.embed;
        final_norm = src.final_norm;
        inv_freq = src.inv_freq;
        wq = src.wq;
        bq = src.bq;
        wk = src.wk;
        bk = src.bk;
        layers = src.layers;
        max_kp = src.max_kp;
        packed_widths = src.packed_widths;
        ld_xn = src.ld_xn;
        ldp = src.ldp;
        ldmix = src.ldmix;
        ldf = src.ldf;
        layer_slot = src.layer_slot;
        n_delta = src.n_delta;
        n_attn = src.n_attn;
        alloc_handle_state();
    }

    void ensure_workspace(int tokens, int rows, int readouts) {
        if (tokens <= cap_tokens && rows <= cap_rows && readouts <= cap_readouts) return;
        for (void *p : ws) cudaFree(p);
        ws.clear();
        cap_tokens = std::max(tokens, cap_tokens);
        cap_tokens = round_up(std::max(cap_tokens, 256), 256);
        cap_rows = std::max(std::max(rows, cap_rows), HK_MAX_ROWS);
        cap_readouts = round_up(std::max(std::max(readouts, cap_readouts), 1024), 256);
        const KevConfig &c = cfg;
        const size_t N = cap_tokens, R = cap_readouts + cap_rows, e = esz();
        x = dev_alloc<float>(N * c.hidden, ws);
        xn = dev_alloc<uint8_t>(N * ld_xn * e, ws);
        proj = dev_alloc<float>(N * ldp, ws);
        mix = dev_alloc<uint8_t>(N * ldmix * e, ws);
        ffn = dev_alloc<uint8_t>(N * ldf * e, ws);
        if (dtype == HK_DTYPE_FP32) {
            ld_lo32 = round_up(std::max(std::max(ld_xn, ldmix), std::max(ldf, ldp)), 4);
            x_lo32 = dev_alloc<float>(N * ld_lo32, ws);
        }
        if (split_inputs()) {
            ld_xl = round_up(c.hidden, 16);
            ld_mixl = round_up(ldmix, 16);
            ld_fl = round_up(ldf, 16);
            xn_lo = dev_alloc<uint8_t>(N * ld_xl, ws);
            mix_lo = dev_alloc<uint8_t>(N * ld_mixl, ws);
            ffn_lo = dev_alloc<uint8_t>(N * ld_fl, ws);
        }
        HK_CUDA(cudaMemset(xn, 0, N * ld_xn * e));
        HK_CUDA(cudaMemset(mix, 0, N * ldmix * e));
        HK_CUDA(cudaMemset(ffn, 0, N * ldf * e));
        dq = dev_alloc<float>(N * c.key_dim(), ws);
        dkk = dev_alloc<float>(N * c.key_dim(), ws);
        dvv = dev_alloc<float>(N * c.value_dim(), ws);
        dg = dev_alloc<float>(N * c.nv, ws);
        db = dev_alloc<float>(N * c.nv, ws);
        dout = dev_alloc<float>(N * c.value_dim(), ws);
        aq = dev_alloc<uint8_t>(N * c.nh * c.hd * e, ws);
        // Paged K/V needs up to page_tokens - 1 padding slots per row.
        kv_slot_cap = static_cast<int>(N) + cap_rows * std::max(kv_page_tokens, 1);
        ak = dev_alloc<uint8_t>(static_cast<size_t>(kv_slot_cap) * c.nkv * c.hd * e, ws);
        av = dev_alloc<uint8_t>(static_cast<size_t>(kv_slot_cap) * c.nkv * c.hd * e, ws);
        hn = dev_alloc<float>(R * c.hidden, ws);
        rproj = dev_alloc<float>(R * dp, ws);
        logits = dev_alloc<float>(R, ws);
        if (max_kp > 0) {
            xq = dev_alloc<int8_t>(N * max_kp, ws);
            xd = dev_alloc<float>(N * (max_kp / 32), ws);
        }
        probs = dev_alloc<float>(R, ws);
        answers = dev_alloc<AnswerRec>(cap_rows, ws);
        qtype_dev = dev_alloc<int32_t>(cap_rows, ws);
        meta_cap = 4 * N + 6 * static_cast<size_t>(cap_rows) + 4 * R + 64 + N;  // + block table
        meta = dev_alloc<int32_t>(meta_cap, ws);
    }

    // xlo (with the weight's e4m3 copy) adds the low part of a split-precision
    // input; out_lo receives a SwiGLU output's low part.
    void gemm(const Mat &W, const void *xin, int ldx, int M, void *out, int ldo, int epi,
              const uint8_t *xlo = nullptr, int ldxl = 0, uint8_t *out_lo = nullptr, int ldol = 0) {
        GemmArgs a;
        a.M = M;
        a.N = W.rows;
        a.K = W.cols;
        a.x = xin;
        a.ldx = ldx;
        a.w = W.w;
        a.ldw = W.ld;
        a.scale = W.scale;
        if (W.w8 && xlo) {
            a.x_lo = xlo;
            a.ldx_lo = ldxl;
            a.w8 = W.w8;
            a.ldw8 = W.ld8;
        }
        a.out_lo = out_lo;
        a.ldo_lo = ldol;
        if (W.q8) {
            cudaEvent_t dq = prof_begin();
            const size_t n = static_cast<size_t>(W.rows) * W.ld;
            const bool lo = W.ld8 && xlo;
            launch_expand_i8(W.q8, n, wdq, lo ? wdq8 : nullptr, stream);
            prof_end(dq, 4, 0.0, (lo ? 4.0 : 3.0) * n);
            a.w = wdq;
            if (lo) {
                a.x_lo = xlo;
                a.ldx_lo = ldxl;
                a.w8 = wdq8;
                a.ldw8 = W.ld8;
            }
        }
        a.out = out;
        a.ldo = ldo;
        a.epilogue = epi;
        a.err = err;
        cudaEvent_t ev = prof_begin();
        if (W.q) {
            if (epi != kEpiStoreF32 && epi != kEpiResidual)
                throw ApiError(HK_ERR_UNSUPPORTED, "packed projections store fp32 outputs only");
            launch_quantize_rows(static_cast<const float *>(xin), ldx, M, W.cols, W.kp, xq, xd, stream);
            gemm_q8(xq, xd, W.q, W.qd, M, W.rows, W.kp, static_cast<float *>(out), ldo, epi == kEpiResidual, stream,
                    num_sms, err);
        } else if (W.w_lo) {
            // fp32 model: 3xTF32 on the tensor cores.
            launch_tf32_lo(static_cast<const float *>(xin), ldx, M, W.cols, x_lo32, ld_lo32, stream);
            a.tf32 = true;
            a.x_lo32 = x_lo32;
            a.ldx_lo32 = ld_lo32;
            a.w_lo32 = W.w_lo;
            a.ldw_lo32 = W.ld;
            gemm_f16_tc(a, stream, num_sms);
        } else if (f32_model()) {
            gemm_f32_simt(a, stream);
        } else {
            gemm_f16_tc(a, stream, num_sms);
        }
        // Algorithmic bytes: the weights, the input rows and the output rows once
        // (a residual output is read and written; SwiGLU writes half the columns).
        const double wb = (W.q ? (W.kp / 32.0) * (32.0 + 4.0) : static_cast<double>(W.cols) * (W.q8 ? 2 : esz())) +
                          (a.w8 ? static_cast<double>(W.cols) : 0.0);
        const double ob = epi == kEpiResidual ? 8.0 : epi == kEpiStoreF32 ? 4.0 : epi == kEpiSwiGLU ? esz() / 2.0
                                                                                                        : esz();
        prof_end(ev, 0, 2.0 * M * W.rows * W.cols,
                 W.rows * wb + static_cast<double>(M) * W.cols * (esz() + (a.x_lo ? 1 : 0)) +
                     static_cast<double>(M) * W.rows * ob);
    }

    // Algorithmic FLOPs of the chunked delta rule (chunk 32) for n tokens of one layer.
    static double delta_chunk_flops(int n, const KevConfig &c) {
        const double C = 32.0;
        return static_cast<double>(c.nv) * n * (2.0 * C * (c.dk + c.dv) + 6.0 * c.dk * c.dv);
    }

    // The forward over a packed batch whose description is already on the
    // device in `meta` (layout: see MetaLayout).
    // Device view of a cached batch: per-row prefix lengths and, per layer,
    // per-row snapshot addresses (see cache_meta); null arrays when unused.
    struct CacheRefs {
        const int32_t *pre_len = nullptr;
        const uint64_t *in_a = nullptr, *in_b = nullptr, *out_a = nullptr, *out_b = nullptr;
    };

    void forward(int n_rows, int n_tok, int max_len, int n_opt, const uint32_t *ids,
                 const int32_t *cu_seqlens, const int32_t *pos, const int32_t *tok_row,
                 const int32_t *ridx, const int32_t *opt_dec, float *out_logits, const KvPages &pages,
                 const int32_t *row_order, const CacheRefs *cr = nullptr) {
        const KevConfig &c = cfg;
        const int A = act();
        const size_t e = esz();
        cudaEvent_t ev = prof_begin();
        launch_embed(A, ids, n_tok, embed, c.hidden, x, stream);
        prof_end(ev, 8, 0.0, static_cast<double>(n_tok) * c.hidden * (e + 4.0));
        // One RMSNorm: the fp32 residual rows in, the normalised rows out (activation type).
        const double norm_bytes = static_cast<double>(n_tok) * c.hidden * (4.0 + e) + 4.0 * c.hidden;
        auto at_layer = [&](const uint64_t *arr, int li) -> const uint64_t * {
            return arr ? arr + static_cast<size_t>(li) * n_rows : nullptr;
        };
        for (size_t li = 0; li < layers.size(); ++li) {
            const Layer &L = layers[li];
            const uint64_t *in_a = cr ? at_layer(cr->in_a, li) : nullptr, *in_b = cr ? at_layer(cr->in_b, li) : nullptr;
            const uint64_t *out_a = cr ? at_layer(cr->out_a, li) : nullptr;
            const uint64_t *out_b = cr ? at_layer(cr->out_b, li) : nullptr;
            ev = prof_begin();
            launch_rmsnorm(A, x, c.hidden, L.in_norm, c.eps, n_tok, c.hidden, xn, ld_xn, stream,
                           L.full ? nullptr : xn_lo, ld_xl);
            prof_end(ev, 5, 0.0, norm_bytes);
            // Half-precision models: the warp-specialised delta layer kernel.
            const bool pipe = !L.full && !f32_model() && c.dk == 128 && c.dv == 128 && c.taps == 4 &&
                              c.nk > 0 && c.nv % c.nk == 0 && (ldp % 4) == 0 && (c.conv_dim() % 4) == 0;
            gemm(L.mix_in, xn, ld_xn, n_tok, proj, ldp, kEpiStoreF32, L.full ? nullptr : xn_lo, ld_xl);
            if (pipe) {
                if (out_b)
                    launch_conv_history(proj, ldp, c.conv_dim(), c.taps, cu_seqlens, n_rows, in_b, out_b, stream);
                DeltaRecArgs r;
                r.cu_seqlens = cu_seqlens;
                r.row_order = row_order;
                r.n_rows = n_rows;
                r.nk = c.nk;
                r.nv = c.nv;
                r.dk = c.dk;
                r.dv = c.dv;
                r.exact = 0;
                r.state_in = in_a;
                r.state_out = out_a;
                r.err = err;
                DeltaFusedInput in;
                in.proj = proj;
                in.ldp = ldp;
                in.conv_dim = c.conv_dim();
                in.conv_w = L.conv_w;
                in.base_g = L.base_g;
                in.dt_bias = L.dt_bias;
                in.hist_in = in_b;
                ev = prof_begin();
                launch_delta_pipe(r, in, L.gnorm_w, c.eps, static_cast<__half *>(mix), ldmix, stream, mix_lo, ld_mixl);
                // Reads each token's q | k | v | z | b | a projection row (fp32), writes its
                // gated-norm output (fp16).
                prof_end(ev, 1, delta_chunk_flops(n_tok, c),
                         static_cast<double>(n_tok) * ((c.conv_dim() + c.value_dim() + 2.0 * c.nv) * 4.0 +
                                                       c.value_dim() * 2.0));
            } else if (!L.full) {
                DeltaPrepArgs d;
                d.proj = proj;
                d.ldp = ldp;
                d.pos = pos;
                d.n = n_tok;
                d.conv_w = L.conv_w;
                d.taps = c.taps;
                d.base_g = L.base_g;
                d.dt_bias = L.dt_bias;
                d.nk = c.nk;
                d.nv = c.nv;
                d.dk = c.dk;
                d.dv = c.dv;
                d.q = dq;
                d.k = dkk;
                d.v = dvv;
                d.g = dg;
                d.beta = db;
                d.tok_row = tok_row;
                d.hist_in = in_b;
                d.fast = !f32_model();
                if (out_b)
                    launch_conv_history(proj, ldp, c.conv_dim(), c.taps, cu_seqlens, n_rows, in_b, out_b, stream);
                ev = prof_begin();
                launch_delta_prep(d, stream);
                prof_end(ev, 3, 0.0,
                         static_cast<double>(n_tok) * ((c.conv_dim() + 2.0 * c.nv) * 4.0 +
                                                       (c.conv_dim() + 2.0 * c.nv) * 4.0));
                DeltaRecArgs r;
                r.q = dq;
                r.k = dkk;
                r.v = dvv;
                r.g = dg;
                r.beta = db;
                r.cu_seqlens = cu_seqlens;
                r.row_order = row_order;
                r.n_rows = n_rows;
                r.nk = c.nk;
                r.nv = c.nv;
                r.dk = c.dk;
                r.dv = c.dv;
                r.out = dout;
                r.exact = f32_model();
                r.state_in = in_a;
                r.state_out = out_a;
                ev = prof_begin();
                launch_delta_recurrent(r, stream);
                prof_end(ev, 1, 4.0 * n_tok * c.nv * c.dk * c.dv,
                         static_cast<double>(n_tok) * (c.conv_dim() + 2.0 * c.nv + c.value_dim()) * 4.0);
                ev = prof_begin();
                launch_gated_norm(A, dout, proj + c.conv_dim(), ldp, L.gnorm_w, c.eps, n_tok, c.nv, c.dv, mix, ldmix,
                                  stream, mix_lo, ld_mixl);
                prof_end(ev, 4, 0.0, static_cast<double>(n_tok) * c.value_dim() * (8.0 + e));
            } else {
                AttnPrepArgs p;
                p.proj = proj;
                p.ldp = ldp;
                p.pos = pos;
                p.tok_row = tok_row;
                p.pages = pages;
                p.n = n_tok;
                p.nh = c.nh;
                p.nkv = c.nkv;
                p.hd = c.hd;
                p.rd = c.rotary_dim();
                p.qn_w = L.qn_w;
                p.kn_w = L.kn_w;
                p.inv_freq = inv_freq;
                p.eps = c.eps;
                p.q = aq;
                p.k = ak;
                p.v = av;
                p.pre_len = cr ? cr->pre_len : nullptr;
                ev = prof_begin();
                launch_attn_prep(A, p, stream);
                // Reads q, k, v of the projection row (fp32; the gate stays for the
                // attention kernel), writes q, k, v in the activation type.
                prof_end(ev, 6, 0.0,
                         static_cast<double>(n_tok) * (c.nh + 2.0 * c.nkv) * c.hd * (4.0 + e));
                AttnArgs at;
                at.q = aq;
                at.k = ak;
                at.v = av;
                at.proj = proj;
                at.ldp = ldp;
                at.cu_seqlens = cu_seqlens;
                at.tok_row = tok_row;
                at.n = n_tok;
                at.n_rows = n_rows;
                at.max_len = max_len;
                at.nh = c.nh;
                at.nkv = c.nkv;
                at.hd = c.hd;
                at.out = mix;
                at.ldo = ldmix;
                at.pages = pages;
                at.pre_len = cr ? cr->pre_len : nullptr;
                at.kv_in = in_a;
                at.err = err;
                at.kv_slots = pages.page_tokens ? kv_slot_cap : n_tok;
                if (out_a) launch_kv_store(A, at, out_a, stream);
                ev = prof_begin();
                launch_attention(A, at, stream);
                // QK^T and PV over the causal query-key pairs of every head.
                prof_end(ev, 2, 4.0 * c.hd * c.nh * attn_pairs,
                         static_cast<double>(n_tok) * ((c.nh + 2.0 * c.nkv) * c.hd * e + c.nh * c.hd * (4.0 + e)));
            }
            gemm(L.mix_out, mix, ldmix, n_tok, x, c.hidden, kEpiResidual, L.full ? nullptr : mix_lo, ld_mixl);
            ev = prof_begin();
            launch_rmsnorm(A, x, c.hidden, L.post_norm, c.eps, n_tok, c.hidden, xn, ld_xn, stream, xn_lo, ld_xl);
            prof_end(ev, 5, 0.0, norm_bytes);
            if (fused_swiglu) {
                gemm(L.gu, xn, ld_xn, n_tok, ffn, ldf, kEpiSwiGLU, xn_lo, ld_xl, ffn_lo, ld_fl);
            } else {
                gemm(L.gu, xn, ld_xn, n_tok, proj, ldp, kEpiStoreF32, xn_lo, ld_xl);
                ev = prof_begin();
                launch_swiglu(A, proj, ldp, n_tok, c.ffn, ffn, ldf, stream, ffn_lo, ld_fl);
                prof_end(ev, 4, 0.0, static_cast<double>(n_tok) * c.ffn * (8.0 + e));
            }
            gemm(L.down, ffn, ldf, n_tok, x, c.hidden, kEpiResidual, ffn_lo, ld_fl);
        }
        ReadoutArgs ro;
        ro.x = x;
        ro.hidden = c.hidden;
        ro.final_w = final_norm;
        ro.eps = c.eps;
        ro.idx = ridx;
        ro.opt_dec = opt_dec;
        ro.n_dec = n_rows;
        ro.n_opt = n_opt;
        ro.wq = wq;
        ro.bq = bq;
        ro.wk = wk;
        ro.bk = bk;
        ro.dp = dp;
        ro.scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(dp)));
        ro.hn = hn;
        ro.proj = rproj;
        ro.logits = out_logits;
        ev = prof_begin();
        launch_readout(ro, stream);
        // The decision and option rows of the residual stream, both pointer
        // projections (fp32) and the logits.
        prof_end(ev, 7, 2.0 * (n_rows + n_opt) * c.hidden * dp,
                 (static_cast<double>(n_rows) + n_opt) * c.hidden * 4.0 + 2.0 * dp * (c.hidden + 1.0) * 4.0 +
                     n_opt * 4.0);
    }
};

// ----------------------------------------------------------------- batch meta
// Device layout of one batch in Model::meta (int32 words):
//   ids[N] | cu_seqlens[R+1] | positions[P] | cu_positions[R+1]     (inputs)
//   pos[N] | tok_row[N] | ridx[R + P] | opt_dec[P]                  (derived)
// ridx lists the decision token of every row, then every option token.
struct MetaLayout {
    size_t ids, cu, positions, cu_pos, pos, tok_row, ridx, opt_dec, row_order, cu_pages, table, total;
    MetaLayout(int rows, int n, int p, int n_pages = 0) {
        ids = 0;
        cu = ids + n;
        positions = cu + rows + 1;
        cu_pos = positions + p;
        pos = cu_pos + rows + 1;
        tok_row = pos + n;
        ridx = tok_row + n;
        opt_dec = ridx + rows + p;
        row_order = opt_dec + p;
        cu_pages = row_order + rows;
        table = cu_pages + rows + 1;
        total = table + n_pages;
    }
};

// Host-side page plan for a batch: per-row page offsets and a block table that
// places every page of every row in a distinct pool page. With a nonzero
// seed the pool order is a deterministic pseudo-random permutation (the
// shuffled block table of the long-context stress configuration).
struct PagePlan {
    std::vector<int32_t> cu_pages, table;
};
PagePlan plan_pages(const int32_t *cu_h, int n_rows, int page_tokens, uint64_t seed) {
    PagePlan pp;
    pp.cu_pages.assign(n_rows + 1, 0);
    for (int r = 0; r < n_rows; ++r) {
        const int len = cu_h[r + 1] - cu_h[r];
        pp.cu_pages[r + 1] = pp.cu_pages[r] + (len + page_tokens - 1) / page_tokens;
    }
    const int n = pp.cu_pages[n_rows];
    pp.table.resize(n);
    for (int i = 0; i < n; ++i) pp.table[i] = i;
    if (seed) {
        uint64_t x = seed * 0x9E3779B97F4A7C15ull + 1;
        for (int i = n - 1; i > 0; --i) {
            x ^= x << 13;
            x ^= x >> 7;
            x ^= x << 17;
            const int j = static_cast<int>(x % static_cast<uint64_t>(i + 1));
            std::swap(pp.table[i], pp.table[j]);
        }
    }
    return pp;
}

namespace {

__device__ int find_row(const int32_t *cu, int rows, int v) {
    int lo = 0, hi = rows - 1;  // largest r with cu[r] <= v
    while (lo < hi) {
        const int mid = (lo + hi + 1) / 2;
        if (cu[mid] <= v)
            lo = mid;
        else
            hi = mid - 1;
    }
    return lo;
}

__global__ void build_meta_kernel(int32_t *meta, int rows, int n, int p, MetaLayout L) {
    const int32_t *cu = meta + L.cu;
    const int32_t *cup = meta + L.cu_pos;
    const int32_t *positions = meta + L.positions;
    const int total = n + rows + p;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        if (i < n) {
            const int r = find_row(cu, rows, i);
            meta[L.tok_row + i] = r;
            meta[L.pos + i] = i - cu[r];
        } else if (i < n + rows) {
            const int r = i - n;
            meta[L.ridx + r] = cu[r + 1] - 1;
        } else {
            const int j = i - n - rows;
            const int r = find_row(cup, rows, j);
            meta[L.opt_dec + j] = r;
            meta[L.ridx + rows + j] = cu[r] + positions[j];
        }
    }
}

}  // namespace

}  // namespace hk

// =================================================================== C ABI
struct hk_model {
    std::unique_ptr<hk::Model> m;
};

namespace {

thread_local std::string tl_create_error;

int fail(hk_model *h, int code, const std::string &msg) {
    if (h && h->m) h->m->last_error = msg;
    return code;
}

template <typename F>
int guarded(hk_model *h, F &&f) {
    try {
        return f();
    } catch (const hk::ApiError &e) {
        return fail(h, e.code, e.what());
    } catch (const hk::CudaError &e) {
        return fail(h, HK_ERR_CUDA, e.what());
    } catch (const std::exception &e) {
        return fail(h, HK_ERR_PACKAGE, e.what());
    }
}

int create_impl(const std::string &dir, int device, int dtype, int max_context, hk_model **out,
                const hk::Model *share = nullptr) {
    *out = nullptr;
    if (dtype != HK_DTYPE_FP32 && dtype != HK_DTYPE_BF16 && dtype != HK_DTYPE_INT8W && dtype != HK_DTYPE_FP16 &&
        dtype != HK_DTYPE_Q8_0 && dtype != HK_DTYPE_Q4_0) {
        tl_create_error = "unsupported dtype";
        return HK_ERR_UNSUPPORTED;
    }
    std::unique_ptr<hk_model> h(new hk_model);
    h->m.reset(new hk::Model);
    hk::Model &m = *h->m;
    try {
        int ndev = 0;
        HK_CUDA(cudaGetDeviceCount(&ndev));
        if (device < 0 || device >= ndev) throw hk::ApiError(HK_ERR_BACKEND, "no CUDA device " + std::to_string(device));
        m.device = device;
        HK_CUDA(cudaSetDevice(device));
        int major = 0;
        HK_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device));
        if (major != 10)
            throw hk::ApiError(HK_ERR_UNSUPPORTED, "this build targets sm_100a (B200); device is sm_" +
                                                       std::to_string(major) + "x");
        HK_CUDA(cudaDeviceGetAttribute(&m.num_sms, cudaDevAttrMultiProcessorCount, device));
        HK_CUDA(cudaStreamCreateWithFlags(&m.stream, cudaStreamNonBlocking));
        m.dtype = dtype;
        m.max_context = max_context;
        if (share)
            m.share_weights(*share);
        else
            m.load(dir);
        HK_CUDA(cudaDeviceSynchronize());
    } catch (const hk::ApiError &e) {
        tl_create_error = e.what();
        return e.code;
    } catch (const hk::CudaError &e) {
        tl_create_error = e.what();
        return HK_ERR_CUDA;
    } catch (const std::exception &e) {
        tl_create_error = std::string("invalid Kev package: ") + e.what();
        return HK_ERR_PACKAGE;
    }
    *out = h.release();
    return HK_OK;
}

}  // namespace

extern "C" {

int hk_create(const char *model_dir, int device, int dtype, int max_context, hk_model **out) {
    if (!model_dir || !out) return HK_ERR_ARGUMENT;
    if (max_context <= 0) {
        tl_create_error = "max_context must be positive";
        return HK_ERR_ARGUMENT;
    }
    return create_impl(model_dir, device, dtype, max_context, out);
}

int hk_replica(const hk_model *src, int device, hk_model **out) {
    if (!src || !out || !src->m) return HK_ERR_ARGUMENT;
    const hk::Model &s = *src->m;
    return create_impl(s.dir, device, s.dtype, s.max_context, out, device == s.device ? &s : nullptr);
}

uint64_t hk_weight_bytes(const hk_model *h, uint64_t *store_id) {
    if (!h || !h->m || !h->m->wstore) return 0;
    if (store_id) *store_id = reinterpret_cast<uint64_t>(h->m->wstore.get());
    return h->m->wstore->bytes;
}

int hk_capabilities_get(const hk_model *h, hk_capabilities *out) {
    if (!h || !out || !h->m) return HK_ERR_ARGUMENT;
    const hk::Model &m = *h->m;
    out->dtype = m.dtype;
    out->device = m.device;
    out->max_context = m.max_context;
    out->max_rows = HK_MAX_ROWS;
    out->hidden_size = m.cfg.hidden;
    out->num_layers = m.cfg.layers;
    out->vocab_size = m.cfg.vocab;
    out->pointer_dim = m.dp;
    out->temperature = m.temperature;
    out->lora_rank = m.lora_rank;
    return HK_OK;
}

static int score_device_impl(hk::Model &m, int n_rows, const int32_t *cu_h, const int32_t *cup_h,
                             cudaStream_t stream, const hk::Model::CacheRefs *cr = nullptr) {
    (void)stream;
    const int n = cu_h[n_rows], p = cup_h[n_rows];
    int max_len = 0;
    for (int r = 0; r < n_rows; ++r) max_len = std::max(max_len, cu_h[r + 1] - cu_h[r]);
    hk::KvPages pages;
    hk::PagePlan plan;
    if (m.kv_page_tokens > 0) plan = hk::plan_pages(cu_h, n_rows, m.kv_page_tokens, m.kv_shuffle_seed);
    const int n_pages = static_cast<int>(plan.table.size());
    hk::MetaLayout L(n_rows, n, p, n_pages);
    if (m.kv_page_tokens > 0) {
        if (static_cast<long>(n_pages) * m.kv_page_tokens > m.kv_slot_cap)
            throw hk::ApiError(HK_ERR_BACKEND, "paged K/V pool too small for the batch");
        pages.block_table = m.meta + L.table;
        pages.cu_pages = m.meta + L.cu_pages;
        pages.page_tokens = m.kv_page_tokens;
    }
    // Longest rows first for the per-row recurrence kernels.
    m.row_order.resize(n_rows);
    for (int r = 0; r < n_rows; ++r) m.row_order[r] = r;
    std::stable_sort(m.row_order.begin(), m.row_order.end(),
                     [&](int a, int b) { return cu_h[a + 1] - cu_h[a] > cu_h[b + 1] - cu_h[b]; });
    // Host-built parts of the batch description, through pinned staging:
    // cu_positions, then the contiguous row order | cu_pages | block table.
    {
        const size_t w_cup = static_cast<size_t>(n_rows) + 1;
        const size_t w_tail = L.total - L.row_order;
        hk::Model::HostStage &st = m.stage_acquire((w_cup + w_tail) * 4);
        int32_t *h = reinterpret_cast<int32_t *>(st.p);
        std::memcpy(h, cup_h, w_cup * 4);
        int32_t *t = h + w_cup;
        std::memcpy(t, m.row_order.data(), static_cast<size_t>(n_rows) * 4);
        if (n_pages) {
            std::memcpy(t + n_rows, plan.cu_pages.data(), plan.cu_pages.size() * 4);
            std::memcpy(t + n_rows + n_rows + 1, plan.table.data(), plan.table.size() * 4);
        }
        HK_CUDA(cudaMemcpyAsync(m.meta + L.cu_pos, h, w_cup * 4, cudaMemcpyHostToDevice, m.stream));
        HK_CUDA(cudaMemcpyAsync(m.meta + L.row_order, t, (n_pages ? w_tail : static_cast<size_t>(n_rows)) * 4,
                                cudaMemcpyHostToDevice, m.stream));
        HK_CUDA(cudaEventRecord(st.done, m.stream));
    }
    m.attn_pairs = 0.0;
    for (int r = 0; r < n_rows; ++r) {
        const double t = cu_h[r + 1] - cu_h[r];
        m.attn_pairs += t * (t + 1.0) / 2.0;
    }
    const uint64_t before = hk::tl_launches;
    hk::build_meta_kernel<<<std::min(hk::ceil_div(L.total, 256), 1024), 256, 0, m.stream>>>(m.meta, n_rows, n, p, L);
    HK_LAUNCH_CHECK();
    m.forward(n_rows, n, max_len, p, reinterpret_cast<const uint32_t *>(m.meta + L.ids), m.meta + L.cu,
              m.meta + L.pos, m.meta + L.tok_row, m.meta + L.ridx, m.meta + L.opt_dec, m.logits, pages,
              m.meta + L.row_order, cr);

    m.launches += hk::tl_launches - before;
    return HK_OK;
}

}  // extern "C"

static_assert(sizeof(hk_answer) == sizeof(hk::AnswerRec), "hk_answer and AnswerRec share one layout");

// Calibrated answers requested with a scoring call (hk_score_answers).
struct AnswerReq {
    const int32_t *qtypes;
    float temperature;
    float *probs;
    hk_answer *answers;
};

// The host-buffer scoring path shared by hk_score, hk_score_cached and
// hk_score_answers. pre[r] is row r's cached prefix length (0 without a
// cache); cr the device table; aq the answers to compute on the device.
static void score_host(hk::Model &m, int n_rows, const uint32_t *tokens, const int32_t *cu_seqlens,
                       const int32_t *positions, const int32_t *cu_positions, float *out_logits,
                       const std::vector<int> *pre, const hk::Model::CacheRefs *cr,
                       const AnswerReq *aq = nullptr) {
    // Validation mirrors forward_independent_batch (qwen3_5.rs:3143-3171)
    // and Backend::forward (qwen3_5.rs:2669-2705).
    if (n_rows < 1 || n_rows > (pre ? HK_MAX_CACHED_ROWS : HK_MAX_ROWS))
        throw hk::ApiError(HK_ERR_BACKEND, pre ? "cached batches take 1..=256 rows"
                                               : "Qwen3.5 batch must contain 1..=64 independent rows");
    if (cu_seqlens[0] != 0 || cu_positions[0] != 0)
        throw hk::ApiError(HK_ERR_ARGUMENT, "cu_seqlens[0] and cu_positions[0] must be 0");
    for (int r = 0; r < n_rows; ++r) {
        const int len = cu_seqlens[r + 1] - cu_seqlens[r];
        const int np = cu_positions[r + 1] - cu_positions[r];
        const int P = pre ? (*pre)[r] : 0;
        if (len <= 0)
            throw hk::ApiError(HK_ERR_BACKEND, P ? "cached continuation requires nonempty suffix tokens"
                                                 : "Qwen3.5 batches require valid independent rows without cache handles");
        if (np < 0) throw hk::ApiError(HK_ERR_ARGUMENT, "cu_positions must be non-decreasing");
        if (P + len > m.max_context)
            throw hk::ApiError(HK_ERR_BACKEND, "sequence length " + std::to_string(P + len) +
                                                   " exceeds max_context " + std::to_string(m.max_context));
        for (int i = cu_seqlens[r]; i < cu_seqlens[r + 1]; ++i)
            if (tokens[i] >= static_cast<uint32_t>(m.cfg.vocab))
                throw hk::ApiError(HK_ERR_BACKEND, "Qwen3.5 token ID is outside the vocabulary");
        for (int j = cu_positions[r]; j < cu_positions[r + 1]; ++j)
            if (positions[j] < 0 || positions[j] >= len)
                throw hk::ApiError(HK_ERR_BACKEND, "Qwen3.5 readout position is outside the token sequence");
    }
    if (aq) {  // calibration.rs:198-218 (temperature), one question per row
        if (!std::isfinite(aq->temperature) || !(aq->temperature > 0.f))
            throw hk::ApiError(HK_ERR_ARGUMENT, "temperature must be positive and finite");
        for (int r = 0; r < n_rows; ++r) {
            const int np = cu_positions[r + 1] - cu_positions[r], qt = aq->qtypes[r];
            if (qt != HK_QUESTION_CHOICE && qt != HK_QUESTION_NOUL && qt != HK_QUESTION_SCORE)
                throw hk::ApiError(HK_ERR_ARGUMENT, "unknown question type");
            if (np < 1 || (qt == HK_QUESTION_NOUL && np != 2))
                throw hk::ApiError(HK_ERR_ARGUMENT, "a question needs one readout position per option "
                                                    "(noul: exactly two, [no, yes])");
        }
    }
    const int n = cu_seqlens[n_rows], p = cu_positions[n_rows];
    HK_CUDA(cudaSetDevice(m.device));
    m.ensure_workspace(n, n_rows, p);
    hk::MetaLayout L(n_rows, n, p);
    const size_t in_words = L.pos;  // ids | cu | positions | cu_pos
    // pinned: inputs | logits | error word | question types | probabilities | answers
    const size_t bytes = in_words * 4 + static_cast<size_t>(p) * 4 + 64 +
                         (aq ? static_cast<size_t>(n_rows) * 4 + static_cast<size_t>(p) * 4 +
                                   static_cast<size_t>(n_rows) * sizeof(hk_answer) + 64
                             : 0);
    if (bytes > m.pinned_cap) {
        if (m.pinned) cudaFreeHost(m.pinned);
        m.pinned = nullptr;
        m.pinned_cap = 0;
        HK_CUDA(cudaHostAlloc(&m.pinned, bytes * 2, cudaHostAllocDefault));
        m.pinned_cap = bytes * 2;
    }
    int32_t *st = static_cast<int32_t *>(m.pinned);
    std::memcpy(st + L.ids, tokens, static_cast<size_t>(n) * 4);
    std::memcpy(st + L.cu, cu_seqlens, static_cast<size_t>(n_rows + 1) * 4);
    if (p) std::memcpy(st + L.positions, positions, static_cast<size_t>(p) * 4);
    std::memcpy(st + L.cu_pos, cu_positions, static_cast<size_t>(n_rows + 1) * 4);
    HK_CUDA(cudaMemcpyAsync(m.meta, st, in_words * 4, cudaMemcpyHostToDevice, m.stream));
    score_device_impl(m, n_rows, cu_seqlens, cu_positions, m.stream, cr);
    float *res = reinterpret_cast<float *>(st + in_words);
    uint32_t *errw = reinterpret_cast<uint32_t *>(res + p);
    int32_t *qt_h = reinterpret_cast<int32_t *>(errw + 16);
    float *pr_h = reinterpret_cast<float *>(qt_h + n_rows);
    hk_answer *ans_h = reinterpret_cast<hk_answer *>(pr_h + p + 8);
    if (aq) {
        std::memcpy(qt_h, aq->qtypes, static_cast<size_t>(n_rows) * 4);
        HK_CUDA(cudaMemcpyAsync(m.qtype_dev, qt_h, static_cast<size_t>(n_rows) * 4, cudaMemcpyHostToDevice, m.stream));
        hk::AnswerArgs a;
        a.logits = m.logits;
        a.cu_positions = m.meta + L.cu_pos;
        a.qtype = m.qtype_dev;
        a.n_rows = n_rows;
        a.temperature = aq->temperature;
        a.probs = m.probs;
        a.out = m.answers;
        hk::launch_answers(a, m.stream);
        HK_CUDA(cudaMemcpyAsync(pr_h, m.probs, static_cast<size_t>(p) * 4, cudaMemcpyDeviceToHost, m.stream));
        HK_CUDA(cudaMemcpyAsync(ans_h, m.answers, static_cast<size_t>(n_rows) * sizeof(hk_answer),
                                cudaMemcpyDeviceToHost, m.stream));
    }
    if (p && out_logits)
        HK_CUDA(cudaMemcpyAsync(res, m.logits, static_cast<size_t>(p) * 4, cudaMemcpyDeviceToHost, m.stream));
    HK_CUDA(cudaMemcpyAsync(errw, m.err, 4, cudaMemcpyDeviceToHost, m.stream));
    HK_CUDA(cudaStreamSynchronize(m.stream));
    if (*errw) {
        HK_CUDA(cudaMemsetAsync(m.err, 0, 4, m.stream));
        HK_CUDA(cudaStreamSynchronize(m.stream));
        throw hk::ApiError(HK_ERR_CUDA, "device error flag " + std::to_string(*errw) + " set during the forward");
    }
    if (p && out_logits) std::memcpy(out_logits, res, static_cast<size_t>(p) * 4);
    if (aq) {
        std::memcpy(aq->probs, pr_h, static_cast<size_t>(p) * 4);
        std::memcpy(aq->answers, ans_h, static_cast<size_t>(n_rows) * sizeof(hk_answer));
    }
}

extern "C" {

int hk_score(hk_model *h, int n_rows, const uint32_t *tokens, const int32_t *cu_seqlens,
             const int32_t *positions, const int32_t *cu_positions, float *out_logits) {
    if (!h || !h->m || !cu_seqlens || !cu_positions) return HK_ERR_ARGUMENT;
    hk::Model &m = *h->m;
    return guarded(h, [&]() -> int {
        score_host(m, n_rows, tokens, cu_seqlens, positions, cu_positions, out_logits, nullptr, nullptr);
        return HK_OK;
    });
}

int hk_score_answers(hk_model *h, int n_rows, const uint32_t *tokens, const int32_t *cu_seqlens,
                     const int32_t *positions, const int32_t *cu_positions, const int32_t *question_types,
                     float temperature, float *out_logits, float *out_probs, hk_answer *out_answers) {
    if (!h || !h->m || !cu_seqlens || !cu_positions || !question_types || !out_probs || !out_answers)
        return HK_ERR_ARGUMENT;
    hk::Model &m = *h->m;
    return guarded(h, [&]() -> int {
        const AnswerReq aq{question_types, temperature, out_probs, out_answers};
        score_host(m, n_rows, tokens, cu_seqlens, positions, cu_positions, out_logits, nullptr, nullptr, &aq);
        return HK_OK;
    });
}

int hk_score_cached(hk_model *h, int n_rows, const uint64_t *parents, int mode, const uint32_t *tokens,
                    const int32_t *cu_seqlens, const int32_t *positions, const int32_t *cu_positions,
                    float *out_logits, uint64_t *handles_out) {
    if (!h || !h->m || !cu_seqlens || !cu_positions) return HK_ERR_ARGUMENT;
    if (mode != HK_CACHE_BRANCH && mode != HK_CACHE_CONTINUE && mode != HK_CACHE_PREFILL) return HK_ERR_ARGUMENT;
    if (mode == HK_CACHE_PREFILL && !handles_out) return HK_ERR_ARGUMENT;
    hk::Model &m = *h->m;
    return guarded(h, [&]() -> int {
        using Snap = hk::Model::Snapshot;
        if (n_rows < 1 || n_rows > HK_MAX_CACHED_ROWS)
            throw hk::ApiError(HK_ERR_BACKEND, "cached batches take 1..=256 rows");
        HK_CUDA(cudaSetDevice(m.device));
        std::vector<std::shared_ptr<Snap>> in(n_rows), out(n_rows);
        std::vector<int> pre(n_rows, 0);
        for (int r = 0; r < n_rows; ++r) {
            const uint64_t id = parents ? parents[r] : 0;
            if (id) {
                auto it = m.caches.find(id);
                if (it == m.caches.end()) throw hk::ApiError(HK_ERR_BACKEND, "unknown Qwen3.5 cache handle");
                in[r] = it->second;
                pre[r] = in[r]->tokens;
            } else if (mode == HK_CACHE_CONTINUE) {
                throw hk::ApiError(HK_ERR_ARGUMENT, "every continued row needs a cache handle");
            }
            if (mode == HK_CACHE_CONTINUE)
                for (int q = 0; q < r; ++q)
                    if (parents[q] == id)
                        throw hk::ApiError(HK_ERR_ARGUMENT, "a cache handle can be continued by one row per call");
        }
        const int NL = static_cast<int>(m.layers.size());
        for (int r = 0; r < n_rows; ++r) {
            const int len = cu_seqlens[r + 1] - cu_seqlens[r];
            if (mode != HK_CACHE_BRANCH && len > 0 && pre[r] + len <= m.max_context) out[r] = m.new_snapshot(pre[r] + len);
        }
        bool any_in = false, any_out = mode != HK_CACHE_BRANCH;
        for (auto &sp : in) any_in = any_in || sp;
        // Per-layer, per-row snapshot addresses and the prefix lengths.
        const size_t LR = static_cast<size_t>(NL) * n_rows;
        std::vector<uint64_t> tab(4 * LR + (n_rows + 1) / 2, 0);
        for (int li = 0; li < NL; ++li)
            for (int r = 0; r < n_rows; ++r) {
                const size_t k = static_cast<size_t>(li) * n_rows + r;
                const bool delta = !m.layers[li].full;
                if (in[r]) {
                    tab[k] = m.piece(*in[r], li);
                    if (delta) tab[LR + k] = tab[k] + m.delta_state_bytes();
                }
                if (out[r]) {
                    tab[2 * LR + k] = m.piece(*out[r], li);
                    if (delta) tab[3 * LR + k] = tab[2 * LR + k] + m.delta_state_bytes();
                }
            }
        std::memcpy(reinterpret_cast<int32_t *>(tab.data() + 4 * LR), pre.data(), static_cast<size_t>(n_rows) * 4);
        {
            hk::Model::HostStage &stg = m.stage_acquire(tab.size() * 8);
            std::memcpy(stg.p, tab.data(), tab.size() * 8);
            HK_CUDA(cudaMemcpyAsync(m.cache_meta, stg.p, tab.size() * 8, cudaMemcpyHostToDevice, m.stream));
            HK_CUDA(cudaEventRecord(stg.done, m.stream));
        }
        hk::Model::CacheRefs cr;
        cr.pre_len = reinterpret_cast<const int32_t *>(m.cache_meta + 4 * LR);
        if (any_in) {
            cr.in_a = m.cache_meta;
            cr.in_b = m.cache_meta + LR;
        }
        if (any_out) {
            cr.out_a = m.cache_meta + 2 * LR;
            cr.out_b = m.cache_meta + 3 * LR;
        }
        score_host(m, n_rows, tokens, cu_seqlens, positions, cu_positions, out_logits, &pre, &cr);
        // Commit only after the whole forward succeeded (qwen3_5.rs:2745-2751).
        for (int r = 0; r < n_rows; ++r) {
            if (mode == HK_CACHE_CONTINUE) {
                m.caches[parents[r]] = out[r];
            } else if (mode == HK_CACHE_PREFILL) {
                const uint64_t id = hk::Model::next_cache_id();
                m.caches[id] = out[r];
                handles_out[r] = id;
            }
        }
        return HK_OK;
    });
}

int hk_prefill(hk_model *h, int n_rows, const uint32_t *tokens, const int32_t *cu_seqlens, uint64_t *handles_out) {
    if (!h || !h->m || !cu_seqlens || !handles_out || n_rows < 1 || n_rows > HK_MAX_CACHED_ROWS) return HK_ERR_ARGUMENT;
    std::vector<int32_t> cup(static_cast<size_t>(n_rows) + 1, 0);
    return hk_score_cached(h, n_rows, nullptr, HK_CACHE_PREFILL, tokens, cu_seqlens, nullptr, cup.data(), nullptr,
                           handles_out);
}

int hk_fork(hk_model *h, uint64_t handle, uint64_t *out) {
    if (!h || !h->m || !out) return HK_ERR_ARGUMENT;
    hk::Model &m = *h->m;
    auto it = m.caches.find(handle);
    if (it == m.caches.end()) return fail(h, HK_ERR_BACKEND, "unknown Qwen3.5 cache handle");
    const uint64_t id = hk::Model::next_cache_id();
    m.caches[id] = it->second;
    *out = id;
    return HK_OK;
}

int hk_release_cache(hk_model *h, uint64_t handle) {
    if (!h || !h->m) return HK_ERR_ARGUMENT;
    hk::Model &m = *h->m;
    return guarded(h, [&]() -> int {
        HK_CUDA(cudaSetDevice(m.device));
        if (!m.caches.erase(handle)) throw hk::ApiError(HK_ERR_BACKEND, "unknown Qwen3.5 cache handle");
        return HK_OK;
    });
}

int hk_cache_info(const hk_model *h, uint64_t handle, int *tokens, int64_t *bytes) {
    if (!h || !h->m || !tokens || !bytes) return HK_ERR_ARGUMENT;
    const hk::Model &m = *h->m;
    auto it = m.caches.find(handle);
    if (it == m.caches.end()) return HK_ERR_BACKEND;
    *tokens = it->second->tokens;
    *bytes = static_cast<int64_t>(m.snapshot_bytes(it->second->tokens));
    return HK_OK;
}

int hk_score_device(hk_model *h, int n_rows, const int32_t *cu_seqlens_host, const int32_t *cu_positions_host,
                    const uint32_t *d_tokens, const int32_t *d_cu_seqlens, const int32_t *d_positions,
                    float *d_out_logits, void *stream) {
    if (!h || !h->m || !cu_seqlens_host || !cu_positions_host || !d_tokens || !d_cu_seqlens) return HK_ERR_ARGUMENT;
    hk::Model &m = *h->m;
    return guarded(h, [&]() -> int {
        if (n_rows < 1 || n_rows > HK_MAX_ROWS)
            throw hk::ApiError(HK_ERR_BACKEND, "Qwen3.5 batch must contain 1..=64 independent rows");
        const int n = cu_seqlens_host[n_rows], p = cu_positions_host[n_rows];
        HK_CUDA(cudaSetDevice(m.device));
        m.ensure_workspace(n, n_rows, p);
        cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : m.stream;
        cudaStream_t own = m.stream;
        m.stream = s;
        hk::MetaLayout L(n_rows, n, p);
        HK_CUDA(cudaMemcpyAsync(m.meta + L.ids, d_tokens, static_cast<size_t>(n) * 4, cudaMemcpyDeviceToDevice, s));
        HK_CUDA(cudaMemcpyAsync(m.meta + L.cu, d_cu_seqlens, static_cast<size_t>(n_rows + 1) * 4,
                                cudaMemcpyDeviceToDevice, s));
        if (p)
            HK_CUDA(cudaMemcpyAsync(m.meta + L.positions, d_positions, static_cast<size_t>(p) * 4,
                                    cudaMemcpyDeviceToDevice, s));
        int rc;
        try {
            rc = score_device_impl(m, n_rows, cu_seqlens_host, cu_positions_host, s);
            if (p)
                HK_CUDA(cudaMemcpyAsync(d_out_logits, m.logits, static_cast<size_t>(p) * 4, cudaMemcpyDeviceToDevice, s));
        } catch (...) {
            m.stream = own;
            throw;
        }
        m.stream = own;
        return rc;
    });
}

int hk_synchronize(hk_model *h) {
    if (!h || !h->m) return HK_ERR_ARGUMENT;
    hk::Model &m = *h->m;
    return guarded(h, [&]() -> int {
        HK_CUDA(cudaSetDevice(m.device));
        HK_CUDA(cudaDeviceSynchronize());
        uint32_t e = 0;
        HK_CUDA(cudaMemcpy(&e, m.err, 4, cudaMemcpyDeviceToHost));
        if (e) {
            HK_CUDA(cudaMemset(m.err, 0, 4));
            throw hk::ApiError(HK_ERR_CUDA, "device error flag " + std::to_string(e) + " set during the forward");
        }
        return HK_OK;
    });
}

uint64_t hk_kernel_launches(const hk_model *h) { return (h && h->m) ? h->m->launches : 0; }

int hk_set_kv_page_tokens(hk_model *h, int page_tokens, uint64_t shuffle_seed) {
    if (!h || !h->m) return HK_ERR_ARGUMENT;
    hk::Model &m = *h->m;
    if (page_tokens != 0 && (page_tokens < 16 || page_tokens > 256 || (page_tokens & (page_tokens - 1)) != 0))
        return fail(h, HK_ERR_ARGUMENT, "KV page tokens must be 0 or a power of two in 16..256");
    if (page_tokens != m.kv_page_tokens) {
        m.kv_page_tokens = page_tokens;
        m.cap_tokens = m.cap_rows = m.cap_readouts = 0;  // re-size the K/V pool on the next call
    }
    m.kv_shuffle_seed = shuffle_seed;
    return HK_OK;
}

int hk_profile_enable(hk_model *h, int enable) {
    if (!h || !h->m) return HK_ERR_ARGUMENT;
    h->m->prof = enable != 0;
    return HK_OK;
}

int hk_profile_read(hk_model *h, double *ms, double *flops, double *bytes, int64_t *count, int n_classes) {
    if (!h || !h->m || !ms || !flops || !bytes || !count) return HK_ERR_ARGUMENT;
    hk::Model &m = *h->m;
    return guarded(h, [&]() -> int {
        HK_CUDA(cudaSetDevice(m.device));
        HK_CUDA(cudaDeviceSynchronize());  // events may sit on a caller's stream
        for (int i = 0; i < n_classes; ++i) {
            ms[i] = 0.0;
            flops[i] = 0.0;
            bytes[i] = 0.0;
            count[i] = 0;
        }
        for (auto &r : m.prof_recs) {
            float t = 0.f;
            HK_CUDA(cudaEventElapsedTime(&t, r.a, r.b));
            if (r.cls < n_classes) {
                ms[r.cls] += t;
                flops[r.cls] += r.flops;
                bytes[r.cls] += r.bytes;
                count[r.cls] += 1;
            }
            m.prof_pool.push_back(r.a);
            m.prof_pool.push_back(r.b);
        }
        m.prof_recs.clear();
        return HK_OK;
    });
}

const char *hk_last_error(const hk_model *h) {
    if (!h || !h->m) return "null handle";
    return h->m->last_error.c_str();
}

const char *hk_create_error(void) { return tl_create_error.c_str(); }

void hk_destroy(hk_model *h) { delete h; }

}  // extern "C"
