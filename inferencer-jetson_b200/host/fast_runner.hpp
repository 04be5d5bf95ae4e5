// C++ shim with the reference runner's class names, constructor and method
// signatures over the C ABI (include/ijb200.h).
//
// The reference's host code (GGUF reader, tokenizer, generate loop in
// inferencer.cu) constructs FastRunner from its GGUF (inferencer.cu:1196-1198),
// calls FastRunner::forward (:1424-1426), FastRunner::prefill (:1279-1283),
// FastRunner::reset (:1264) and FastGPU::matvec (:1156), reads runner.layers /
// dim / vocab / context and the device pointers gpu.x and gpu.logits
// (:1727-1754), and brackets steps with gpu.start_timer / stop_timer,
// accumulating gpu.gpu_seconds and gpu.calls (:1857-1889).  This header keeps
// those names, members and argument meanings, so that code compiles against it
// unchanged once it includes this header instead of defining its own
// FastRunner (namespace ijb_host; `using ijb_host::FastRunner;`).  A non-zero
// status from the library is rethrown as std::runtime_error, the reference's
// error convention (cuda_check, :126-128).
//
// Header-only; link libijb200.so.  The GGUF type is a template parameter so
// the header does not depend on the reference's source: anything with the
// reference GGUF's members (param(), params, tensors with dims / type / gpu)
// works.
#pragma once

#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/ijb200.h"

namespace ijb_host {

inline void check(int rc, const ijb_engine *e, const char *where) {
    if (rc != IJB_OK) throw std::runtime_error(std::string(where) + ": " + ijb_last_error(e));
}

// The members of FastGPU the reference's callers touch (inferencer.cu:1101-1180).
struct FastGPU {
    float *x = nullptr;       // residual stream of the last token (device)
    float *logits = nullptr;  // logits of the last token (device)
    unsigned long long calls = 0;
    double gpu_seconds = 0;

    // FastGPU::matvec(const Tensor &, const float *in, float *out, cols, rows):
    // y = W x on the engine's quantised activation path; `t` is the reference
    // GGUF's Tensor (or anything with its dims and type); the weight must be one
    // the engine was built with, found by device pointer.
    template <class TensorT>
    void matvec(const TensorT &t, const float *input, float *output, int expected_cols, int expected_rows) {
        if (static_cast<int>(t.dims[0]) != expected_cols || static_cast<int>(t.dims[1]) != expected_rows ||
            (t.type != IJB_TYPE_Q4_K && t.type != IJB_TYPE_Q6_K))
            throw std::runtime_error("Unexpected quantized matrix shape");
        int idx = -1;
        for (size_t i = 0; i < names_.size() && idx < 0; ++i)
            if (ptrs_[i] == static_cast<const void *>(t.gpu)) idx = ijb_tensor_index(e_, names_[i].c_str());
        if (idx < 0) throw std::runtime_error("matvec: tensor not registered with the engine");
        check(ijb_matvec(e_, idx, input, output, expected_cols, expected_rows, 1, nullptr), e_, "matvec");
        ++calls;
    }
    // FastGPU::start_timer / stop_timer (:1172-1179): device time (CUDA events on
    // the engine's stream) of the steps run in between, added to gpu_seconds.
    void start_timer() { timed_ = 0.0; }
    void stop_timer() { gpu_seconds += timed_; }

   private:
    friend class FastRunner;
    void step_done() {
        timed_ += ijb_last_step_ms(e_) / 1000.0;
        const int n = ijb_last_step_size(e_);
        if (n > 0) {
            x = const_cast<float *>(ijb_residual_dev(e_)) + static_cast<long>(n - 1) * dim_;
            logits = const_cast<float *>(ijb_logits_dev(e_)) + static_cast<long>(n - 1) * vocab_;
        }
    }
    ijb_engine *e_ = nullptr;
    int dim_ = 0, vocab_ = 0;
    double timed_ = 0.0;
    std::vector<std::string> names_;
    std::vector<const void *> ptrs_;
};

class FastRunner {
   public:
    // FastRunner(GGUF &, max_context, use_dp4a, use_q6_dp4a, norm_quant,
    // rope_cache, gate_launch_warps, q6_launch_warps, prefill_capacity)
    // (inferencer.cu:1196-1198).  The fusion switches and launch widths select
    // kernel variants of the reference; this build always runs its fused
    // kernels, so they are accepted and ignored.  prefill_capacity becomes the
    // engine's packed-step size (at least 1).  Any Llama shape the engine
    // supports is accepted, not only the 3B one.
    template <class GGUFT>
    FastRunner(GGUFT &model, int max_context, bool use_dp4a, bool use_q6_dp4a, bool norm_quant = false,
               bool rope_cache = false, int gate_launch_warps = 4, int q6_launch_warps = 4,
               int prefill_capacity = 1, int device = 0, bool kv_f32 = false)
        : context(max_context) {
        (void)norm_quant;
        (void)rope_cache;
        (void)gate_launch_warps;
        (void)q6_launch_warps;
        dim = model.param("llama.embedding_length");
        layers = model.param("llama.block_count");
        heads = model.param("llama.attention.head_count");
        kv_heads = model.param("llama.attention.head_count_kv");
        hidden = model.param("llama.feed_forward_length");
        vocab = model.param("llama.vocab_size");
        head_dim = dim / heads;
        kv_dim = head_dim * kv_heads;
        eps = static_cast<float>(model.params.at("llama.attention.layer_norm_rms_epsilon"));
        ijb_model_desc d{};
        d.dim = dim;
        d.layers = layers;
        d.heads = heads;
        d.kv_heads = kv_heads;
        d.hidden = hidden;
        d.vocab = vocab;
        d.eps = eps;
        d.rope_base = static_cast<float>(model.params.at("llama.rope.freq_base"));
        d.context = max_context;
        d.max_batch = prefill_capacity > 1 ? prefill_capacity : 1;
        d.max_seqs = 2;
        d.page_size = 16;
        d.use_dp4a = use_dp4a;
        d.use_q6_dp4a = use_q6_dp4a;
        d.kv_f32 = kv_f32;
        d.device = device;
        std::vector<ijb_tensor_view> views;
        views.reserve(model.tensors.size());
        for (const auto &kv : model.tensors) {
            ijb_tensor_view v{};
            v.name = kv.first.c_str();
            v.type = static_cast<int>(kv.second.type);
            v.n_dims = static_cast<int>(kv.second.dims.size());
            for (size_t i = 0; i < kv.second.dims.size() && i < 4; ++i)
                v.dims[i] = static_cast<int64_t>(kv.second.dims[i]);
            v.data_dev = kv.second.gpu;
            views.push_back(v);
            gpu.names_.push_back(kv.first);
            gpu.ptrs_.push_back(kv.second.gpu);
        }
        check(ijb_create(&d, views.data(), static_cast<int>(views.size()), &e_), nullptr, "engine create");
        gpu.e_ = e_;
        gpu.dim_ = dim;
        gpu.vocab_ = vocab;
        gpu.x = const_cast<float *>(ijb_residual_dev(e_));
        gpu.logits = const_cast<float *>(ijb_logits_dev(e_));
    }
    ~FastRunner() { ijb_destroy(e_); }
    FastRunner(const FastRunner &) = delete;
    FastRunner &operator=(const FastRunner &) = delete;

    void reset() { check(ijb_reset(e_), e_, "reset"); }

    // FastRunner::forward (:1424-1426): the argmax, or -1 without logits.  The
    // traces, when given, receive what the reference records: layer_trace one
    // vector of dim residuals per layer; quant_trace the int8 activations
    // quantised in each layer (attention input, attention output, feed-forward
    // input: dim each; down-projection input: hidden).
    int forward(int token, int pos, bool need_logits, std::vector<std::vector<float>> *layer_trace = nullptr,
                std::vector<std::vector<int8_t>> *quant_trace = nullptr) {
        int next = -1;
        if (!layer_trace && !quant_trace) {
            check(ijb_forward(e_, token, pos, need_logits ? 1 : 0, &next), e_, "forward");
        } else {
            std::vector<float> lt(layer_trace ? static_cast<size_t>(layers) * dim : 0);
            std::vector<int8_t> qt(quant_trace ? static_cast<size_t>(layers) * qwidth() : 0);
            check(ijb_forward_traced(e_, token, pos, need_logits ? 1 : 0, &next, layer_trace ? lt.data() : nullptr,
                                     quant_trace ? qt.data() : nullptr),
                  e_, "forward");
            if (layer_trace) append_layers(lt.data(), *layer_trace);
            if (quant_trace) append_quant(qt.data(), *quant_trace);
        }
        gpu.step_done();
        gpu.calls += 7ull * layers + (need_logits ? 1 : 0);
        return next;
    }

    // FastRunner::prefill (:1279-1283): the argmax after the last token.
    // layer_trace: the last token's residual per layer; quant_trace: its
    // quantised activations; all_layer_trace: input.size() * layers vectors,
    // token-major; first_quant_trace: the first token's quantised activations.
    int prefill(const std::vector<int> &input, std::vector<std::vector<float>> *layer_trace = nullptr,
                std::vector<std::vector<int8_t>> *quant_trace = nullptr,
                std::vector<std::vector<float>> *all_layer_trace = nullptr,
                std::vector<std::vector<int8_t>> *first_quant_trace = nullptr) {
        int next = -1;
        const int n = static_cast<int>(input.size());
        if (!layer_trace && !quant_trace && !all_layer_trace && !first_quant_trace) {
            check(ijb_prefill(e_, input.data(), n, &next), e_, "prefill");
        } else {
            std::vector<float> all(static_cast<size_t>(n) * layers * dim);
            std::vector<int8_t> first(static_cast<size_t>(layers) * qwidth()), last(first.size());
            check(ijb_prefill_traced(e_, input.data(), n, &next, all.data(), first.data(), last.data()), e_,
                  "prefill");
            if (all_layer_trace) {
                all_layer_trace->resize(static_cast<size_t>(n) * layers);
                for (size_t i = 0; i < all_layer_trace->size(); ++i)
                    (*all_layer_trace)[i].assign(all.begin() + i * dim, all.begin() + (i + 1) * dim);
            }
            if (layer_trace) append_layers(all.data() + static_cast<size_t>(n - 1) * layers * dim, *layer_trace);
            if (quant_trace) append_quant(last.data(), *quant_trace);
            if (first_quant_trace) append_quant(first.data(), *first_quant_trace);
        }
        gpu.step_done();
        gpu.calls += (7ull * layers) * static_cast<unsigned long long>(n) + 1;
        return next;
    }

    ijb_engine *engine() { return e_; }

    int dim = 0, layers = 0, heads = 0, kv_heads = 0, head_dim = 0, kv_dim = 0, hidden = 0, vocab = 0, context = 0;
    float eps = 0.f;
    FastGPU gpu;

   private:
    size_t qwidth() const { return 3u * dim + hidden; }
    void append_layers(const float *src, std::vector<std::vector<float>> &out) const {
        for (int l = 0; l < layers; ++l) out.emplace_back(src + static_cast<size_t>(l) * dim, src + (l + 1) * dim);
    }
    void append_quant(const int8_t *src, std::vector<std::vector<int8_t>> &out) const {
        for (int l = 0; l < layers; ++l) {
            const int8_t *q = src + static_cast<size_t>(l) * qwidth();
            out.emplace_back(q, q + dim);
            out.emplace_back(q + dim, q + 2 * dim);
            out.emplace_back(q + 2 * dim, q + 3 * dim);
            out.emplace_back(q + 3 * dim, q + 3 * dim + hidden);
        }
    }
    ijb_engine *e_ = nullptr;
};

}  // namespace ijb_host
