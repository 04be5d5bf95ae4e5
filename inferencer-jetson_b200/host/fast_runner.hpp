// C++ shim with the reference runner's method signatures over the C ABI.
//
// The reference's host code (GGUF reader, tokenizer, generate loop in
// inferencer.cu) calls FastGPU::matvec (inferencer.cu:1156), FastRunner::forward
// (:1424), FastRunner::prefill (:1279) and FastRunner::reset (:1264), reads
// runner.layers / dim / vocab / gpu.x / gpu.logits, and brackets steps with
// gpu.start_timer / stop_timer (:1172-1179).  This header keeps those names and
// argument meanings and maps them onto include/ijb200.h; a non-zero status is
// rethrown as std::runtime_error, the reference's error convention
// (cuda_check, :126-128).  Header-only: link libijb200.so.
#pragma once

#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/ijb200.h"

namespace ijb_host {

inline void check(int rc, const ijb_engine *e, const char *where) {
    if (rc != IJB_OK) throw std::runtime_error(std::string(where) + ": " + ijb_last_error(e));
}

// One tensor as the reference's GGUF reader describes it (Tensor,
// inferencer.cu:178-186): GGUF dims, GGML type id and the device pointer into
// the uploaded blob.
struct TensorRef {
    std::string name;
    std::vector<uint64_t> dims;
    uint32_t type;
    const void *gpu;
};

struct ModelParams {
    int dim, layers, heads, kv_heads, hidden, vocab;
    float eps, rope_base;
};

// The parts of FastGPU the reference's callers touch.
class FastGPU {
   public:
    explicit FastGPU(ijb_engine *e) : e_(e) {}
    // FastGPU::matvec(const Tensor &, const float *in, float *out, cols, rows)
    void matvec(const TensorRef &t, const float *input, float *output, int expected_cols, int expected_rows) {
        int idx = ijb_tensor_index(e_, t.name.c_str());
        if (idx < 0 || (t.type != IJB_TYPE_Q4_K && t.type != IJB_TYPE_Q6_K))
            throw std::runtime_error("Unexpected quantized matrix shape");
        check(ijb_matvec(e_, idx, input, output, expected_cols, expected_rows, 1, nullptr), e_, "matvec");
        ++calls;
    }
    // FastGPU::start_timer / stop_timer: device time of the steps in between
    void start_timer() {}
    void stop_timer() { gpu_seconds += ijb_last_step_ms(e_) / 1000.0; }
    const float *logits() const { return ijb_logits_dev(e_); }
    const float *x() const { return ijb_residual_dev(e_); }
    unsigned long long calls = 0;
    double gpu_seconds = 0;

   private:
    ijb_engine *e_;
};

// FastRunner over the engine.  The constructor takes what FastRunner's
// constructor reads from the GGUF (hyper-parameters, :1205-1214, and the
// tensor table) plus the --context / INT8-path flags of the CLI.
class FastRunner {
   public:
    FastRunner(const ModelParams &mp, const std::vector<TensorRef> &tensors, int max_context, bool use_dp4a,
               bool use_q6_dp4a, int device = 0, int max_batch = 32, bool kv_f32 = false)
        : dim(mp.dim), layers(mp.layers), vocab(mp.vocab), context(max_context), gpu(nullptr) {
        ijb_model_desc d{};
        d.dim = mp.dim;
        d.layers = mp.layers;
        d.heads = mp.heads;
        d.kv_heads = mp.kv_heads;
        d.hidden = mp.hidden;
        d.vocab = mp.vocab;
        d.eps = mp.eps;
        d.rope_base = mp.rope_base;
        d.context = max_context;
        d.max_batch = max_batch;
        d.max_seqs = 2;
        d.page_size = 16;
        d.use_dp4a = use_dp4a;
        d.use_q6_dp4a = use_q6_dp4a;
        d.kv_f32 = kv_f32;
        d.device = device;
        std::vector<ijb_tensor_view> views;
        views.reserve(tensors.size());
        for (const auto &t : tensors) {
            ijb_tensor_view v{};
            v.name = t.name.c_str();
            v.type = static_cast<int>(t.type);
            v.n_dims = static_cast<int>(t.dims.size());
            for (size_t i = 0; i < t.dims.size() && i < 4; ++i) v.dims[i] = static_cast<int64_t>(t.dims[i]);
            v.data_dev = t.gpu;
            views.push_back(v);
        }
        check(ijb_create(&d, views.data(), static_cast<int>(views.size()), &e_), nullptr, "engine create");
        gpu = FastGPU(e_);
    }
    ~FastRunner() { ijb_destroy(e_); }
    FastRunner(const FastRunner &) = delete;
    FastRunner &operator=(const FastRunner &) = delete;

    void reset() { check(ijb_reset(e_), e_, "reset"); }

    // FastRunner::forward(token, pos, need_logits) -> argmax or -1
    int forward(int token, int pos, bool need_logits) {
        int next = -1;
        check(ijb_forward(e_, token, pos, need_logits ? 1 : 0, &next), e_, "forward");
        return next;
    }

    // FastRunner::prefill(input) -> argmax after the last token
    int prefill(const std::vector<int> &input) {
        int next = -1;
        check(ijb_prefill(e_, input.data(), static_cast<int>(input.size()), &next), e_, "prefill");
        return next;
    }

    ijb_engine *engine() { return e_; }

    int dim, layers, vocab, context;
    FastGPU gpu;

   private:
    ijb_engine *e_ = nullptr;
};

}  // namespace ijb_host
