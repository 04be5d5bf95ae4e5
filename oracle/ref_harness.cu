// Harness around the reference's own CUDA implementation (test infrastructure).
//
// The reference ships no library and no tests; its hot path lives in one
// file.  This harness #includes that file unmodified (the build passes
// -I<reference dir> and -Dmain=reference_main, see oracle/Makefile.ref) and
// exposes a few extern "C" entry points that run the reference's stock kernels
// and runner classes on caller data.  It is built into oracle/_ref/ (never
// committed) and used only to capture golden outputs of the reference on a
// B200 (tests/golden/make_ref_golden.py), to time the reference's kernels, and
// to run the reference's tokenizer on the host for the tokenizer goldens
// (tests/golden/make_tokenizer_golden.py).
#include "inferencer.cu"

namespace {
thread_local std::string g_err;

int fail(const std::exception &e) {
    g_err = e.what();
    return -1;
}

template <class T>
struct DevBuf {
    T *p = nullptr;
    size_t n = 0;
    explicit DevBuf(size_t count, size_t pad_bytes = 256) : n(count) {
        cuda_check(cudaMalloc(&p, count * sizeof(T) + pad_bytes), "harness alloc");
        cuda_check(cudaMemset(p, 0, count * sizeof(T) + pad_bytes), "harness memset");
    }
    ~DevBuf() { cudaFree(p); }
    void up(const T *h) { cuda_check(cudaMemcpy(p, h, n * sizeof(T), cudaMemcpyHostToDevice), "harness H2D"); }
    void down(T *h) const { cuda_check(cudaMemcpy(h, p, n * sizeof(T), cudaMemcpyDeviceToHost), "harness D2H"); }
};

__global__ void ref_dequant_kernel(const u8 *blocks, long nblocks, int type, float *out) {
    long idx = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (idx >= nblocks * 256) return;
    long b = idx / 256;
    int i = (int)(idx % 256);
    out[idx] = type == 12 ? q4_value(blocks + b * 144, i) : q6_value(blocks + b * 210, i);
}
}  // namespace

extern "C" {

const char *ref_last_error() { return g_err.c_str(); }

// q4_value / q6_value (inferencer.cu:454-487) over every weight of nblocks.
int ref_dequant(int type, const uint8_t *blocks, long nblocks, float *out) {
    try {
        if (type != 12 && type != 14) throw std::runtime_error("bad type");
        size_t bpb = type == 12 ? 144 : 210;
        DevBuf<u8> w(nblocks * bpb);
        DevBuf<float> y(nblocks * 256);
        w.up(blocks);
        long total = nblocks * 256;
        ref_dequant_kernel<<<(unsigned)((total + 255) / 256), 256>>>(w.p, nblocks, type, y.p);
        cuda_check(cudaGetLastError(), "dequant launch");
        y.down(out);
        return 0;
    } catch (const std::exception &e) { return fail(e); }
}

// FastGPU::matvec (inferencer.cu:1156-1171) on a caller matrix: the stock
// dispatch (quantize_x32_cuda + gemv_q4_dp4a / gemv_q6_dp4a, or gemv_quant<T>).
// Also returns the quantised activation when the INT8 path ran.
int ref_matvec(int type, const uint8_t *w_host, int cols, int rows, const float *x_host, float *y_host,
               int use_dp4a, int use_q6_dp4a, int q6_warps, int8_t *xq_out, float *xscale_out) {
    try {
        if (cols > 8192 || cols % 256) throw std::runtime_error("cols must be a multiple of 256, <= 8192");
        size_t bytes = (size_t)rows * (cols / 256) * (type == 12 ? 144 : 210);
        FastGPU gpu(1, 128, 1024, use_dp4a != 0, use_q6_dp4a != 0, q6_warps);
        DevBuf<u8> w(bytes);
        DevBuf<float> x(cols), y(rows);
        w.up(w_host);
        x.up(x_host);
        Tensor t;
        t.dims = {(u64)cols, (u64)rows};
        t.type = (u32)type;
        t.offset = 0;
        t.gpu = w.p;
        gpu.matvec(t, x.p, y.p, cols, rows);
        cuda_check(cudaDeviceSynchronize(), "matvec sync");
        y.down(y_host);
        if (xq_out) cuda_check(cudaMemcpy(xq_out, gpu.xq, cols, cudaMemcpyDeviceToHost), "xq D2H");
        if (xscale_out)
            cuda_check(cudaMemcpy(xscale_out, gpu.xscale, (cols / 32) * sizeof(float), cudaMemcpyDeviceToHost),
                       "xscale D2H");
        return 0;
    } catch (const std::exception &e) { return fail(e); }
}

// Times FastGPU::matvec on `copies` rotated device copies of one matrix with
// CUDA events; returns the mean milliseconds per call in *ms.
int ref_time_matvec(int type, const uint8_t *w_host, int cols, int rows, const float *x_host, int use_dp4a,
                    int use_q6_dp4a, int q6_warps, int copies, int iters, float *ms) {
    try {
        size_t bytes = (size_t)rows * (cols / 256) * (type == 12 ? 144 : 210);
        FastGPU gpu(1, 128, 1024, use_dp4a != 0, use_q6_dp4a != 0, q6_warps);
        std::vector<std::unique_ptr<DevBuf<u8>>> ws;
        for (int c = 0; c < copies; ++c) {
            ws.emplace_back(new DevBuf<u8>(bytes));
            ws.back()->up(w_host);
        }
        DevBuf<float> x(cols), y(rows);
        x.up(x_host);
        Tensor t;
        t.dims = {(u64)cols, (u64)rows};
        t.type = (u32)type;
        t.offset = 0;
        for (int i = 0; i < 3 * copies; ++i) {
            t.gpu = ws[i % copies]->p;
            gpu.matvec(t, x.p, y.p, cols, rows);
        }
        cudaEvent_t a, b;
        cuda_check(cudaEventCreate(&a), "event");
        cuda_check(cudaEventCreate(&b), "event");
        cuda_check(cudaEventRecord(a), "record");
        for (int i = 0; i < iters; ++i) {
            t.gpu = ws[i % copies]->p;
            gpu.matvec(t, x.p, y.p, cols, rows);
        }
        cuda_check(cudaEventRecord(b), "record");
        cuda_check(cudaEventSynchronize(b), "sync");
        float total = 0;
        cuda_check(cudaEventElapsedTime(&total, a, b), "elapsed");
        *ms = total / iters;
        cudaEventDestroy(a);
        cudaEventDestroy(b);
        return 0;
    } catch (const std::exception &e) { return fail(e); }
}

// rmsnorm_cuda (inferencer.cu:821-834), one CTA of 256 threads.
int ref_rmsnorm(const float *x_host, const float *w_host, float *out_host, int n, float eps) {
    try {
        DevBuf<float> x(n), w(n), o(n);
        x.up(x_host);
        w.up(w_host);
        rmsnorm_cuda<<<1, 256>>>(x.p, w.p, o.p, n, eps);
        cuda_check(cudaGetLastError(), "rmsnorm launch");
        o.down(out_host);
        return 0;
    } catch (const std::exception &e) { return fail(e); }
}

// attention_cuda (inferencer.cu:982-1009): head_dim is fixed at 128 by the
// kernel.  Caches are [ctx][kv_dim] fp32 for one layer.
int ref_attention(const float *q_host, const float *k_host, const float *v_host, float *out_host, int heads,
                  int kv_heads, int pos, int context) {
    try {
        int kv_dim = kv_heads * 128;
        if (pos >= context) throw std::runtime_error("pos >= context");
        DevBuf<float> q(heads * 128), k((size_t)context * kv_dim), v((size_t)context * kv_dim), o(heads * 128);
        q.up(q_host);
        k.up(k_host);
        v.up(v_host);
        attention_cuda<<<heads, 128>>>(q.p, k.p, v.p, o.p, 0, pos, context, kv_dim, heads / kv_heads);
        cuda_check(cudaGetLastError(), "attention launch");
        o.down(out_host);
        return 0;
    } catch (const std::exception &e) { return fail(e); }
}

// argmax_blocks_cuda + argmax_final_cuda (inferencer.cu:1063-1099).
int ref_argmax(const float *values_host, int n, int *index) {
    try {
        int blocks = (n + 255) / 256;
        if (blocks > 512) throw std::runtime_error("n too large");
        DevBuf<float> v(n), bv(512);
        DevBuf<int> bi(512), out(1);
        v.up(values_host);
        argmax_blocks_cuda<<<blocks, 256>>>(v.p, bv.p, bi.p, n);
        argmax_final_cuda<<<1, 512>>>(bv.p, bi.p, out.p, blocks);
        cuda_check(cudaGetLastError(), "argmax launch");
        out.down(index);
        return 0;
    } catch (const std::exception &e) { return fail(e); }
}

// GGUF + FastRunner (inferencer.cu:204-340, :1182-1531) on a GGUF file: feeds
// `n` tokens at positions 0..n-1 through FastRunner::forward (need_logits on
// every step) and copies each step's argmax and logits out.  The runner only
// accepts the Llama-3.2-3B shape (inferencer.cu:1215-1217).
int ref_run_gguf(const char *path, int context, const int *tokens, int n, int use_dp4a, int use_q6_dp4a,
                 int fused, int *next_out, float *logits_out, int vocab) {
    try {
        GGUF model(path);
        model.upload();
        FastRunner runner(model, context, use_dp4a != 0, use_q6_dp4a != 0, fused != 0, fused != 0, 4, 4, 1);
        if (runner.vocab != vocab) throw std::runtime_error("vocab mismatch");
        for (int i = 0; i < n; ++i) {
            next_out[i] = runner.forward(tokens[i], i, true);
            if (logits_out)
                cuda_check(cudaMemcpy(logits_out + (size_t)i * vocab, runner.gpu.logits, vocab * sizeof(float),
                                      cudaMemcpyDeviceToHost),
                           "logits D2H");
        }
        return 0;
    } catch (const std::exception &e) { return fail(e); }
}

// Steady decode timing of the reference runner (inferencer.cu:1870-1883):
// forward() over `prompt` tokens, then `steps` greedy steps each ending in
// the runner's own D2H sync; returns wall seconds of the decode steps.
int ref_time_decode(const char *path, int context, const int *prompt, int n_prompt, int steps, int fused,
                    double *decode_seconds) {
    try {
        GGUF model(path);
        model.upload();
        FastRunner runner(model, context, true, true, fused != 0, fused != 0, 4, 4, 1);
        int next = 0;
        for (int i = 0; i < n_prompt; ++i) next = runner.forward(prompt[i], i, i + 1 == n_prompt);
        auto t0 = Clock::now();
        for (int i = 0; i < steps; ++i) next = runner.forward(next, n_prompt + i, true);
        *decode_seconds = seconds(t0, Clock::now());
        return 0;
    } catch (const std::exception &e) { return fail(e); }
}

}  // extern "C"

// ---------------------------------------------------------------- tokenizer --
// The reference's Tokenizer (inferencer.cu:361-451) on the tokenizer arrays of
// a GGUF file (host only; no GPU involved).  The GGUF and Tokenizer of the
// last path are kept between calls.
namespace {
struct RefTok {
    std::string path;
    std::unique_ptr<GGUF> model;
    std::unique_ptr<Tokenizer> tok;
};
RefTok &ref_tok(const char *path) {
    static RefTok t;
    if (!t.tok || t.path != path) {
        t.tok.reset();
        t.model.reset(new GGUF(path));
        t.tok.reset(new Tokenizer(*t.model));
        t.path = path;
    }
    return t;
}
}  // namespace

extern "C" {

// Tokenizer::encode of len bytes; writes min(cap, *n) ids and the count to *n.
int ref_tokenize(const char *gguf_path, const char *text, long len, int *ids, long cap, long *n) {
    try {
        const std::vector<int> out = ref_tok(gguf_path).tok->encode(std::string(text, static_cast<size_t>(len)));
        *n = static_cast<long>(out.size());
        for (long i = 0; i < *n && i < cap; ++i) ids[i] = out[i];
        return 0;
    } catch (const std::exception &e) { return fail(e); }
}

// Tokenizer::decode of one id; writes min(cap, *len) bytes and the length to *len.
int ref_detokenize(const char *gguf_path, int id, char *bytes, int cap, int *len) {
    try {
        const std::string s = ref_tok(gguf_path).tok->decode(id);
        *len = static_cast<int>(s.size());
        for (int i = 0; i < *len && i < cap; ++i) bytes[i] = s[i];
        return 0;
    } catch (const std::exception &e) { return fail(e); }
}

// chat_prompt (inferencer.cu:1534-1551) of len bytes of prompt.
int ref_chat_prompt(const char *gguf_path, const char *prompt, long len, int *ids, long cap, long *n) {
    try {
        const std::vector<int> out = chat_prompt(*ref_tok(gguf_path).tok, std::string(prompt, static_cast<size_t>(len)));
        *n = static_cast<long>(out.size());
        for (long i = 0; i < *n && i < cap; ++i) ids[i] = out[i];
        return 0;
    } catch (const std::exception &e) { return fail(e); }
}

// Tokenizer::special.
int ref_special_token(const char *gguf_path, const char *name, int *id) {
    try {
        *id = ref_tok(gguf_path).tok->special(name);
        return 0;
    } catch (const std::exception &e) { return fail(e); }
}

}  // extern "C"
