// The C-ABI engine (include/ijb200.h): weight registry and load-time repack,
// paged fp16 KV pool, sequence table, packed decode steps captured into CUDA
// graphs with programmatic dependent launch between kernels.
//
// It takes the place of FastGPU (inferencer.cu:1101-1180) and FastRunner
// (:1182-1532).  Per layer a step on the CUDA-core GEMV (1-2 tokens, or any
// step of an engine with max_batch < 16) launches five kernels where the
// reference launches 13-17 (QKV + RoPE + KV write, attention, O + residual,
// gate/up + SiLU, down + residual), plus the streaming attention's finish
// kernel for an fp16, head_dim-64 cache; tensor-core steps (3 or more tokens)
// add an activation-prep launch before each projection.  The whole step is one
// CUDA graph.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>
#include <atomic>

#include "../../include/ijb200.h"
#include "attention.cuh"
#include "common.cuh"
#include "gemv.cuh"
#include "misc.cuh"
#include "mma_gemm.cuh"

namespace ijb {

static std::atomic<uint64_t> g_launches{0};

struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string &m) : std::runtime_error(m), code(c) {}
};

static void ck(cudaError_t e, const char *where) {
    if (e != cudaSuccess) throw Error(IJB_ERR_CUDA, std::string(where) + ": " + cudaGetErrorString(e));
}

static void require(bool ok, const std::string &msg, int code = IJB_ERR_INVALID) {
    if (!ok) throw Error(code, msg);
}

template <class T>
static T *dev_alloc(size_t count, const char *what) {
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, count * sizeof(T) + 16);
    if (e != cudaSuccess) throw Error(IJB_ERR_NOMEM, std::string("cudaMalloc ") + what + ": " + cudaGetErrorString(e));
    return static_cast<T *>(p);
}

struct Weight {
    std::string name;
    int type = 0;
    int rows = 0, cols = 0;
    const uint8_t *data = nullptr;  // usable layout (Q4_K GGUF, Q6_K unit layout, F32)
    int row_bytes = 0;
    void *owned = nullptr;
    bool has_mma = false;  // chunked copy for the tensor-core path
    MmaWeight mma;
    void *mma_owned = nullptr;
};

struct StepGraph {
    cudaGraphExec_t exec = nullptr;
    bool need_logits = true;
    uint64_t launches = 0;  // kernels in the graph
};

}  // namespace ijb

using namespace ijb;

struct ijb_engine {
    ijb_model_desc d{};
    int head_dim = 0, kv_dim = 0;
    int num_sms = 0;
    cudaStream_t stream = nullptr;
    std::vector<Weight> w;
    std::unordered_map<std::string, int> by_name;
    struct Layer {
        int attn_norm, ffn_norm, q, k, v, o, gate, up, down;
    };
    std::vector<Layer> layers;
    int token_embd = -1, output = -1, output_norm = -1;

    // KV pool: per layer, num_pages pages of [K: kv_heads x page x hd][V: same]
    // elements, fp16 (default) or fp32
    void *kv = nullptr;
    int kv_f32 = 0;
    int kv_elem = 2;
    long page_stride = 0;
    long num_pages = 0;
    std::vector<int> free_pages;
    int max_pages_per_seq = 0;
    int *page_table_dev = nullptr;
    std::vector<CUtensorMap> kv_maps;  // per layer, for the streaming attention (fp16 cache, head_dim 64)
    int *page_table_host = nullptr;  // pinned mirror [max_seqs][max_pages_per_seq]
    std::vector<std::vector<int>> seq_pages;
    std::vector<int> seq_len;
    std::vector<char> seq_used;

    // RoPE tables [context][head_dim/2]
    float *rope_cos = nullptr, *rope_sin = nullptr;

    // activations for max_batch tokens
    float *x = nullptr, *q = nullptr, *attn = nullptr, *h = nullptr, *logits = nullptr;
    unsigned long long *keys = nullptr;
    int *next_dev = nullptr;
    int *meta_dev = nullptr;   // [4][max_batch]: token, seq, pos, slot
    int *meta_host = nullptr;  // pinned
    int *next_host = nullptr;  // pinned
    float *attn_partial = nullptr;
    int *attn_counters = nullptr;
    uint8_t *x16 = nullptr;  // fp16 activation tiles of the tensor-core path, one per 64-token chunk
    float *x_inv = nullptr;
    // steps wider than one tensor-core chunk run their chunks' launches on
    // parallel branches: chunk c > 0 on side[(c - 1) % nside]
    static constexpr int kMaxSide = 7;
    int nside = 0;
    cudaStream_t side[kMaxSide] = {};
    cudaEvent_t ev_fork = nullptr, ev_join[kMaxSide] = {};
    int mma_max_split = 8, mma_split_cost = 1;
    bool mma_wide = true;
    int mma_bulk_out = 0;  // thread stores measured faster than per-row bulk copies
    int mma_min_batch = kMmaMinBatch;
    int attn_split_len = 64, attn_max_splits = 1;
    int attn_stream_min = 1;  // smallest step that uses the streaming attention
    uint32_t *status = nullptr;
    unsigned long long *scratch_key = nullptr;

    std::unordered_map<int, StepGraph> graphs;  // key: (n * 2 + need_logits) * 2 + traced
    // device-side greedy loop (ijb_generate): its step graph, state, outputs, stop ids
    StepGraph gen_graph;
    GenState *gen_state = nullptr;
    int *gen_out = nullptr;
    int *gen_stop = nullptr;
    // debug traces of traced steps (allocated on first use): the residual after
    // every layer [max_batch][layers][dim] and the four int8 activations the
    // INT8 path quantises per layer [max_batch][layers][trace_q_stride]
    float *trace_x = nullptr;
    int8_t *trace_q = nullptr;
    long trace_q_stride = 0;
    cudaEvent_t ev_start = nullptr, ev_end = nullptr;
    bool pdl = false;      // programmatic dependent launch between the step's kernels
    bool mma_pdl = true;   // the same for the tensor-core path's prep and GEMM launches
    bool attn_pdl = false;   // the same for the attention launches of tensor-core steps
    bool small_attn_pdl = true;  // the same for the QKV, attention and O launches of CUDA-core steps
    bool attn_prep = false;  // the attention finish kernel builds the O projection's activation tile
    float last_step_ms = 0.f;
    std::string err;
    int last_n = 0;
};

namespace {
thread_local std::string t_create_err;
}  // namespace

namespace ijb {
void set_thread_error(const std::string &msg) { t_create_err = msg; }
void count_launches(uint64_t n) { g_launches += n; }
}  // namespace ijb

namespace {

int fail(ijb_engine *e, const std::exception &ex) {
    const Error *er = dynamic_cast<const Error *>(&ex);
    int code = er ? er->code : IJB_ERR_INVALID;
    if (e) e->err = ex.what();
    else t_create_err = ex.what();
    return code;
}

cudaStream_t pick(ijb_engine *e, void *s) { return s ? static_cast<cudaStream_t>(s) : e->stream; }

constexpr int kGenMaxStop = 16;  // stop ids of ijb_generate
constexpr int kGenRound = 8;     // ijb_generate steps queued per host check

// Bytes of one chunk's fp16 activation tile (up to kMmaMaxNWide tokens of the
// widest row, kMaxCols).
constexpr size_t kX16ChunkBytes = static_cast<size_t>(kMaxCols / 128) * kMmaMaxNWide * 256;

// ------------------------------------------------------------ GEMV params --

void add_seg(GemvParams &p, const Weight &w, const Weight *w2, int epi, float *out, long out_stride, int row_offset,
             const ijb_model_desc &d) {
    require(p.nseg < kMaxSegs, "too many GEMV segments");
    GemvSeg &s = p.seg[p.nseg++];
    s.w0 = w.data;
    s.w1 = w2 ? w2->data : nullptr;
    s.type = w.type;
    s.dp4a = w.type == kQ4K ? d.use_dp4a : d.use_q6_dp4a;
    s.rows = w.rows;
    s.row_bytes = w.row_bytes;
    // a work item is a gate/up pair or a RoPE row pair, else one row
    s.item_rows = (w2 != nullptr || epi == kEpiRopeQ || epi == kEpiRopeKCache) ? 2 : 1;
    s.item0 = p.total_items;
    s.nitems = w2 ? w.rows : w.rows / s.item_rows;
    s.epi = epi;
    s.out = out;
    s.out_stride = out_stride;
    s.row_offset = row_offset;
    p.total_items += s.nitems;
    if (!s.dp4a) p.need_f = 1;
    else if (s.type == kQ4K) p.need_q4 = 1;
    else p.need_q6 = 1;
}

GemvParams base_params(ijb_engine *e, int cols, int batch, const float *x, long x_stride, const float *norm_w) {
    GemvParams p;
    std::memset(&p, 0, sizeof(p));
    p.cols = cols;
    p.batch = batch;
    p.x = x;
    p.x_stride = x_stride;
    p.norm_w = norm_w;
    p.eps = e->d.eps;
    p.rope_cos = e->rope_cos;
    p.rope_sin = e->rope_sin;
    p.half_head = e->head_dim / 2;
    p.kv_heads = e->d.kv_heads;
    p.head_dim = e->head_dim;
    p.page_size = e->d.page_size;
    p.page_stride = e->page_stride;
    p.kv_f32 = e->kv_f32;
    p.argmax_keys = e->keys;
    p.status = e->status;
    return p;
}

void launch_gemv(ijb_engine *e, const GemvParams &p, cudaStream_t s, bool pdl, bool force_pdl = false) {
    ck(gemv_launch(p, e->num_sms, s, (pdl && e->pdl) || force_pdl), "GEMV launch");
    ++g_launches;
}

// One projection (the segments of `seg_fn`) over tokens [g0, g0+gn): the
// tensor-core GEMM for 16..64 tokens, the CUDA-core GEMV in groups of 8 below.
struct ProjSeg {
    int w0, w1, epi;
    float *out;
    long out_stride;
};

// Whether a projection of gn tokens over `segs` runs on the tensor cores, and
// the activation path (*dp: 1 = the reference's int8 quantisation) it uses.
bool proj_uses_mma(const ijb_engine *e, int gn, const ProjSeg *segs, int nsegs, int *dp_out) {
    const ijb_model_desc &d = e->d;
    bool mma_ok = gn >= e->mma_min_batch;
    int dp = -1;
    for (int i = 0; i < nsegs && mma_ok; ++i) {
        const Weight &w = e->w[segs[i].w0];
        const int sdp = w.type == kQ4K ? d.use_dp4a : d.use_q6_dp4a;
        if (dp < 0) dp = sdp;
        mma_ok = w.has_mma && sdp == dp && (segs[i].w1 < 0 || e->w[segs[i].w1].has_mma);
    }
    if (dp_out) *dp_out = dp;
    return mma_ok;
}

// x16_ready: the activation tile of the (single, <= kMmaMaxN-token) tensor-core
// chunk has already been built by the previous kernel.
// gemv_pdl: the CUDA-core launch uses programmatic dependent launch even when
// the engine's IJB_PDL is off.
void launch_projection(ijb_engine *e, cudaStream_t s, int g0, int gn, const float *x, long x_stride,
                       const float *norm_w, const ProjSeg *segs, int nsegs, char *kbase, long v_off,
                       bool x16_ready = false, bool gemv_pdl = false) {
    const ijb_model_desc &d = e->d;
    const int *tpos = e->meta_dev + 2 * d.max_batch;
    const int *tslot = e->meta_dev + 3 * d.max_batch;
    int dp = -1;
    const bool mma_ok = proj_uses_mma(e, gn, segs, nsegs, &dp);
    require(!x16_ready || (mma_ok && gn <= kMmaMaxN), "prepared activation without a single tensor-core chunk");
    const int cols = e->w[segs[0].w0].cols;
    if (mma_ok) {
        // the projection's tiles and K split (the same for every chunk); a launch
        // whose CTAs each hold one tile takes up to kMmaMaxNWide tokens
        int tiles = 0;
        for (int i = 0; i < nsegs; ++i) {
            const int rows = e->w[segs[i].w0].rows;
            tiles += segs[i].w1 >= 0 ? (rows + 63) / 64 : (rows + kMmaTileM - 1) / kMmaTileM;
        }
        int bps = 0;
        const int ksplit = mma_choose_split(tiles, cols / 256, e->mma_max_split, e->mma_split_cost, &bps);
        const int chunk = e->mma_wide && gn > kMmaMaxN && mma_wide_ok(tiles, ksplit) ? kMmaMaxNWide : kMmaMaxN;
        // the chunks are independent (their own tokens, activation tile and outputs)
        // and read the same weights, so they run side by side and the later reads
        // of each weight tile hit L2
        const int nchunks = (gn + chunk - 1) / chunk;
        const int nbranch = std::min(nchunks - 1, e->nside);
        if (nbranch > 0) {
            ck(cudaEventRecord(e->ev_fork, s), "chunk fork");
            for (int i = 0; i < nbranch; ++i) ck(cudaStreamWaitEvent(e->side[i], e->ev_fork, 0), "chunk fork");
        }
        for (int t0 = 0; t0 < gn; t0 += chunk) {
            const int tn = std::min(chunk, gn - t0);
            const int n_pad = (tn + 15) / 16 * 16;
            const int c = t0 / chunk;
            cudaStream_t cs = c == 0 || nbranch == 0 ? s : e->side[(c - 1) % nbranch];
            uint8_t *x16 = e->x16 + static_cast<size_t>(c) * kX16ChunkBytes;
            float *x_inv = e->x_inv + c * kMmaMaxNWide;
            if (!x16_ready) {
                ck(mma_prep_launch(x + static_cast<long>(t0) * x_stride, x_stride, norm_w, d.eps, cols, tn, n_pad, dp,
                                   x16, x_inv, cs, e->mma_pdl),
                   "activation prep launch");
                ++g_launches;
            }
            MmaParams m;
            std::memset(&m, 0, sizeof(m));
            for (int i = 0; i < nsegs; ++i) {
                const Weight &w0 = e->w[segs[i].w0];
                MmaSeg &sg = m.seg[m.nseg];
                m.w[2 * i] = w0.mma;
                sg.w0 = 2 * i;
                sg.w1 = -1;
                if (segs[i].w1 >= 0) {
                    m.w[2 * i + 1] = e->w[segs[i].w1].mma;
                    sg.w1 = 2 * i + 1;
                }
                sg.type = w0.type;
                sg.rows = w0.rows;
                sg.tile0 = m.total_tiles;
                sg.ntiles = sg.w1 >= 0 ? (w0.rows + 63) / 64 : (w0.rows + kMmaTileM - 1) / kMmaTileM;
                sg.epi = segs[i].epi;
                sg.out = segs[i].out ? segs[i].out + static_cast<long>(g0 + t0) * segs[i].out_stride : nullptr;
                sg.out_stride = segs[i].out_stride;
                sg.row_offset = 0;
                m.total_tiles += sg.ntiles;
                ++m.nseg;
            }
            m.cols = cols;
            m.batch = tn;
            m.n_pad = n_pad;
            m.x16 = x16;
            m.x_inv = x_inv;
            m.rope_cos = e->rope_cos;
            m.rope_sin = e->rope_sin;
            m.half_head = e->head_dim / 2;
            m.tok_pos = tpos + g0 + t0;
            m.tok_slot = tslot + g0 + t0;
            m.k_cache = kbase;
            m.v_cache = kbase ? kbase + v_off * e->kv_elem : nullptr;
            m.kv_f32 = e->kv_f32;
            m.kv_heads = d.kv_heads;
            m.head_dim = e->head_dim;
            m.page_size = d.page_size;
            m.page_stride = e->page_stride;
            m.argmax_keys = e->keys + g0 + t0;
            m.status = e->status;
            require(m.total_tiles == tiles, "projection tile count");
            m.ksplit = ksplit;
            m.bps = bps;
            m.bulk_out = e->mma_bulk_out;
            ck(mma_gemm_launch(m, cs, e->mma_pdl), "tensor-core GEMM launch");
            ++g_launches;
        }
        for (int i = 0; i < nbranch; ++i) {
            ck(cudaEventRecord(e->ev_join[i], e->side[i]), "chunk join");
            ck(cudaStreamWaitEvent(s, e->ev_join[i], 0), "chunk join");
        }
        return;
    }
    for (int q0 = 0; q0 < gn; q0 += kMaxBatch) {
        const int qn = std::min(kMaxBatch, gn - q0);
        GemvParams p = base_params(e, cols, qn, x + static_cast<long>(q0) * x_stride, x_stride, norm_w);
        p.tok_pos = tpos + g0 + q0;
        p.tok_slot = tslot + g0 + q0;
        p.k_cache = kbase;
        p.v_cache = kbase ? kbase + v_off * e->kv_elem : nullptr;
        p.argmax_keys = e->keys + g0 + q0;
        for (int i = 0; i < nsegs; ++i)
            add_seg(p, e->w[segs[i].w0], segs[i].w1 >= 0 ? &e->w[segs[i].w1] : nullptr, segs[i].epi,
                    segs[i].out ? segs[i].out + static_cast<long>(g0 + q0) * segs[i].out_stride : nullptr,
                    segs[i].out_stride, 0, d);
        launch_gemv(e, p, s, true, gemv_pdl);
    }
}

// Every kernel of one packed step over n tokens (meta already on the device).
void enqueue_trace_quant(ijb_engine *e, int n, const float *x, long x_stride, const float *norm_w, int cols, int l,
                         long offset, cudaStream_t s) {
    const long row = static_cast<long>(e->d.layers) * e->trace_q_stride;
    ck(trace_quant_launch(x, x_stride, norm_w, e->d.eps, cols, n, e->trace_q + l * e->trace_q_stride + offset, row, s),
       "trace launch");
    ++g_launches;
}

// The four projection launches of layer l for a packed step of n tokens (the
// step's meta already on the device).
void enqueue_qkv(ijb_engine *e, int l, int n, cudaStream_t s) {
    const ijb_model_desc &d = e->d;
    const auto &L = e->layers[l];
    char *kbase = static_cast<char *>(e->kv) + l * e->num_pages * e->page_stride * e->kv_elem;
    const long v_off = static_cast<long>(d.kv_heads) * d.page_size * e->head_dim;
    const ProjSeg segs[3] = {{L.q, -1, kEpiRopeQ, e->q, d.dim},
                             {L.k, -1, kEpiRopeKCache, nullptr, 0},
                             {L.v, -1, kEpiVCache, nullptr, 0}};
    launch_projection(e, s, 0, n, e->x, d.dim, reinterpret_cast<const float *>(e->w[L.attn_norm].data), segs, 3,
                      kbase, v_off, false, n < e->mma_min_batch && e->small_attn_pdl);
}
void enqueue_o(ijb_engine *e, int l, int n, cudaStream_t s, bool x16_ready = false) {
    const ProjSeg o_segs[1] = {{e->layers[l].o, -1, kEpiAdd, e->x, e->d.dim}};
    launch_projection(e, s, 0, n, e->attn, e->d.dim, nullptr, o_segs, 1, nullptr, 0, x16_ready,
                      n < e->mma_min_batch && e->small_attn_pdl);
}
void enqueue_gateup(ijb_engine *e, int l, int n, cudaStream_t s) {
    const auto &L = e->layers[l];
    const ProjSeg segs[1] = {{L.gate, L.up, kEpiSiluPair, e->h, e->d.hidden}};
    launch_projection(e, s, 0, n, e->x, e->d.dim, reinterpret_cast<const float *>(e->w[L.ffn_norm].data), segs, 1,
                      nullptr, 0);
}
void enqueue_down(ijb_engine *e, int l, int n, cudaStream_t s) {
    const ProjSeg segs[1] = {{e->layers[l].down, -1, kEpiAdd, e->x, e->d.dim}};
    launch_projection(e, s, 0, n, e->h, e->d.hidden, nullptr, segs, 1, nullptr, 0);
}

// Layer l's attention over the n tokens of the step metadata (meta_dev): the
// split kernel, or the streaming kernel where the cache has TMA maps.
AttnParams attn_params(ijb_engine *e, int l, int n) {
    const ijb_model_desc &d = e->d;
    const long layer_pool = e->num_pages * e->page_stride;
    const long v_off = static_cast<long>(d.kv_heads) * d.page_size * e->head_dim;
    char *kbase = static_cast<char *>(e->kv) + l * layer_pool * e->kv_elem;
    const int *tseq = e->meta_dev + d.max_batch;
    const int *tpos = e->meta_dev + 2 * d.max_batch;
    AttnParams a;
    std::memset(&a, 0, sizeof(a));
    a.q = e->q;
    a.q_stride = d.dim;
    a.out = e->attn;
    a.out_stride = d.dim;
    a.k_cache = kbase;
    a.v_cache = kbase + v_off * e->kv_elem;
    a.kv_f32 = e->kv_f32;
    a.page_stride = e->page_stride;
    a.page_size = d.page_size;
    a.page_table = e->page_table_dev;
    a.max_pages_per_seq = e->max_pages_per_seq;
    a.tok_seq = tseq;
    a.tok_pos = tpos;
    a.batch = n;
    a.heads = d.heads;
    a.kv_heads = d.kv_heads;
    a.head_dim = e->head_dim;
    a.scale = 1.0f / std::sqrt(static_cast<float>(e->head_dim));
    // steps below attn_stream_min (batch 1) take the split kernel with short
    // splits: more CTAs for one sequence's few positions
    a.split_len = n < e->attn_stream_min ? attention_split_len_min() : e->attn_split_len;
    a.max_splits = e->attn_max_splits;
    a.partial = e->attn_partial;
    a.counters = e->attn_counters;
    a.work = e->attn_counters + d.max_batch * d.kv_heads;
    a.num_ctas = e->num_sms;
    a.status = e->status;
    if (!e->kv_maps.empty() && n >= e->attn_stream_min) {
        a.kv_map = e->kv_maps[l];
        a.has_map = 1;
    }
    return a;
}

void enqueue_step(ijb_engine *e, int n, bool need_logits, cudaStream_t s, bool traced = false) {
    const ijb_model_desc &d = e->d;
    const int *tok = e->meta_dev;
    const Weight &emb = e->w[e->token_embd];
    ck(embed_launch(emb.data, emb.row_bytes, d.dim, tok, n, e->x, d.dim, e->keys, s, e->pdl), "embedding launch");
    ++g_launches;
    for (int l = 0; l < d.layers; ++l) {
        const auto &L = e->layers[l];
        if (traced)
            enqueue_trace_quant(e, n, e->x, d.dim, reinterpret_cast<const float *>(e->w[L.attn_norm].data), d.dim, l, 0,
                                s);
        enqueue_qkv(e, l, n, s);
        AttnParams a = attn_params(e, l, n);
        // the streaming attention's finish kernel also builds the O projection's
        // activation tile when that projection is one tensor-core chunk
        const ProjSeg o_segs[1] = {{L.o, -1, kEpiAdd, e->x, d.dim}};
        int o_dp = 0;
        const bool o_fused =
            e->attn_prep && attention_kernels(a) == 2 && n <= kMmaMaxN && proj_uses_mma(e, n, o_segs, 1, &o_dp);
        if (o_fused) {
            a.x16 = e->x16;
            a.x_inv = e->x_inv;
            a.n_pad = (n + 15) / 16 * 16;
            a.use_dp4a = o_dp;
        }
        // tensor-core steps chain their launches with programmatic dependent launch
        ck(attention_launch(a, s, e->pdl || (n >= e->mma_min_batch ? e->attn_pdl : e->small_attn_pdl)),
           "attention launch");
        g_launches += attention_kernels(a);
        if (traced) enqueue_trace_quant(e, n, e->attn, d.dim, nullptr, d.dim, l, d.dim, s);
        enqueue_o(e, l, n, s, o_fused && !traced);
        if (traced)
            enqueue_trace_quant(e, n, e->x, d.dim, reinterpret_cast<const float *>(e->w[L.ffn_norm].data), d.dim, l,
                                2L * d.dim, s);
        enqueue_gateup(e, l, n, s);
        if (traced) enqueue_trace_quant(e, n, e->h, d.hidden, nullptr, d.hidden, l, 3L * d.dim, s);
        enqueue_down(e, l, n, s);
        if (traced)  // residual after the layer -> trace_x[token][l]
            ck(cudaMemcpy2DAsync(e->trace_x + static_cast<long>(l) * d.dim, static_cast<size_t>(d.layers) * d.dim * 4,
                                 e->x, static_cast<size_t>(d.dim) * 4, static_cast<size_t>(d.dim) * 4, n,
                                 cudaMemcpyDeviceToDevice, s),
               "layer trace copy");
    }
    if (!need_logits) return;
    {
        const ProjSeg segs[1] = {{e->output >= 0 ? e->output : e->token_embd, -1, kEpiLogitsArgmax, e->logits, d.vocab}};
        launch_projection(e, s, 0, n, e->x, d.dim, reinterpret_cast<const float *>(e->w[e->output_norm].data), segs, 1,
                          nullptr, 0);
    }
    ck(keys_to_tokens_launch(e->keys, n, e->next_dev, s, e->pdl), "argmax decode launch");
    ++g_launches;
}

// The engine's device status word, read after the stream has synchronised: a
// kernel that gave up a bounded wait, or failed a bounds check, left a non-zero
// code there.  The word is cleared and the call fails with IJB_ERR_DEVICE; the
// engine stays usable (nothing faulted).
void check_status_word(ijb_engine *e, uint32_t st) {
    if (st) {
        ck(cudaMemset(e->status, 0, sizeof(uint32_t)), "status clear");
        std::string what;
        if (st & kDevErrWaitTimeout) what += " (a bounded wait expired)";
        if (st & kDevErrBadIndex) what += " (an index failed its bounds check)";
        throw Error(IJB_ERR_DEVICE, "kernel reported device error code " + std::to_string(st) + what);
    }
}

// The same, reading the word from the device.
void check_device_status(ijb_engine *e) {
    uint32_t st = 0;
    ck(cudaMemcpy(&st, e->status, sizeof(st), cudaMemcpyDeviceToHost), "status read");
    check_status_word(e, st);
}

// Captures (once per n / need_logits) and replays the whole step: H2D of the
// step's metadata, every kernel, D2H of the next tokens.
void run_step(ijb_engine *e, int n, bool need_logits, bool traced = false) {
    const int key = (n * 2 + (need_logits ? 1 : 0)) * 2 + (traced ? 1 : 0);
    auto it = e->graphs.find(key);
    if (it == e->graphs.end()) {
        cudaGraph_t graph;
        const uint64_t before = g_launches.load();
        ck(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal), "begin capture");
        try {
            ck(cudaMemcpyAsync(e->meta_dev, e->meta_host, 4 * e->d.max_batch * sizeof(int), cudaMemcpyHostToDevice,
                               e->stream),
               "meta H2D");
            enqueue_step(e, n, need_logits, e->stream, traced);
            // the next tokens with the status word behind them, or the status word alone
            const int B = e->d.max_batch;
            if (need_logits)
                ck(cudaMemcpyAsync(e->next_host, e->next_dev, (B + 1) * sizeof(int), cudaMemcpyDeviceToHost, e->stream),
                   "next D2H");
            else
                ck(cudaMemcpyAsync(e->next_host + B, e->next_dev + B, sizeof(int), cudaMemcpyDeviceToHost, e->stream),
                   "status D2H");
        } catch (...) {
            cudaStreamEndCapture(e->stream, &graph);
            throw;
        }
        ck(cudaStreamEndCapture(e->stream, &graph), "end capture");
        StepGraph sg;
        sg.launches = g_launches.load() - before;
        g_launches.store(before);  // counted at each replay instead
        cudaError_t ie = cudaGraphInstantiate(&sg.exec, graph, 0);
        cudaGraphDestroy(graph);
        ck(ie, "graph instantiate");
        it = e->graphs.emplace(key, sg).first;
    }
    // launches inside the graph count as launches of this library (counted
    // once per replay, as many as the capture enqueued)
    g_launches += it->second.launches;
    ck(cudaEventRecord(e->ev_start, e->stream), "step timer start");
    ck(cudaGraphLaunch(it->second.exec, e->stream), "graph launch");
    ck(cudaEventRecord(e->ev_end, e->stream), "step timer end");
    ck(cudaStreamSynchronize(e->stream), "step synchronize");
    ck(cudaEventElapsedTime(&e->last_step_ms, e->ev_start, e->ev_end), "step timer");
    check_status_word(e, static_cast<uint32_t>(e->next_host[e->d.max_batch]));
    e->last_n = n;
}

// Makes sure `seq` owns pages for positions [0, upto]; returns the slot of `pos`.
int slot_for(ijb_engine *e, int seq, int pos) {
    const int ps = e->d.page_size;
    auto &pages = e->seq_pages[seq];
    bool changed = false;
    while (static_cast<int>(pages.size()) * ps <= pos) {
        require(!e->free_pages.empty(), "KV page pool exhausted", IJB_ERR_CAPACITY);
        require(static_cast<int>(pages.size()) < e->max_pages_per_seq, "sequence exceeds context", IJB_ERR_CAPACITY);
        pages.push_back(e->free_pages.back());
        e->free_pages.pop_back();
        e->page_table_host[static_cast<long>(seq) * e->max_pages_per_seq + pages.size() - 1] = pages.back();
        changed = true;
    }
    if (changed)
        ck(cudaMemcpyAsync(e->page_table_dev + static_cast<long>(seq) * e->max_pages_per_seq,
                           e->page_table_host + static_cast<long>(seq) * e->max_pages_per_seq,
                           pages.size() * sizeof(int), cudaMemcpyHostToDevice, e->stream),
           "page table H2D");
    return pages[pos / ps] * ps + pos % ps;
}

// Fills meta for entries (seq, token) at explicit positions and runs a step.
void packed_step(ijb_engine *e, int n, const int *seqs, const int *tokens, const int *positions, bool need_logits,
                 bool traced = false) {
    const ijb_model_desc &d = e->d;
    require(n >= 1 && n <= d.max_batch, "step size must be 1..max_batch", IJB_ERR_CAPACITY);
    int *mt = e->meta_host;
    // the previous step synchronised, so the pinned staging buffer is free
    for (int i = 0; i < n; ++i) {
        const int sq = seqs[i], pos = positions[i], tk = tokens[i];
        require(sq >= 0 && sq < d.max_seqs && e->seq_used[sq], "unknown sequence id");
        require(pos >= 0 && pos < d.context && tk >= 0 && tk < d.vocab, "Token or position outside model context");
        mt[i] = tk;
        mt[d.max_batch + i] = sq;
        mt[2 * d.max_batch + i] = pos;
        mt[3 * d.max_batch + i] = slot_for(e, sq, pos);
    }
    for (int i = n; i < d.max_batch; ++i) mt[i] = mt[d.max_batch + i] = mt[2 * d.max_batch + i] = mt[3 * d.max_batch + i] = 0;
    run_step(e, n, need_logits, traced);
}

void ensure_trace_buffers(ijb_engine *e) {
    if (e->trace_x) return;
    const ijb_model_desc &d = e->d;
    e->trace_q_stride = (3L * d.dim + d.hidden + 15) / 16 * 16;
    e->trace_x = dev_alloc<float>(static_cast<size_t>(d.max_batch) * d.layers * d.dim, "layer trace");
    e->trace_q = dev_alloc<int8_t>(static_cast<size_t>(d.max_batch) * d.layers * e->trace_q_stride, "quant trace");
}

// Copies token i of the last traced step: its residuals [layers][dim] and its
// quantised activations [layers][3*dim + hidden] (either pointer may be null).
void download_trace(ijb_engine *e, int i, float *layer_trace, int8_t *quant_trace) {
    const ijb_model_desc &d = e->d;
    if (layer_trace)
        ck(cudaMemcpy(layer_trace, e->trace_x + static_cast<long>(i) * d.layers * d.dim,
                      static_cast<size_t>(d.layers) * d.dim * 4, cudaMemcpyDeviceToHost),
           "layer trace download");
    if (quant_trace) {
        const long width = 3L * d.dim + d.hidden;
        ck(cudaMemcpy2D(quant_trace, width, e->trace_q + static_cast<long>(i) * d.layers * e->trace_q_stride,
                        e->trace_q_stride, width, d.layers, cudaMemcpyDeviceToHost),
           "quant trace download");
    }
}

void validate_weight(const Weight &w, int type_a, int type_b, int rows, int cols) {
    require(w.type == type_a || w.type == type_b, "Unexpected quantization for " + w.name);
    require(w.rows == rows && w.cols == cols, "Unexpected quantized matrix shape for " + w.name);
}

}  // namespace

// =================================================================== C ABI ==

extern "C" {

int ijb_create(const ijb_model_desc *desc, const ijb_tensor_view *tensors, int n_tensors, ijb_engine **out) {
    std::unique_ptr<ijb_engine> e(new ijb_engine());
    try {
        require(desc && out && tensors, "null argument");
        e->d = *desc;
        ijb_model_desc &d = e->d;
        if (d.page_size <= 0) d.page_size = 16;
        require(d.dim > 0 && d.dim % 256 == 0 && d.dim <= kMaxCols, "dim must be a multiple of 256, <= 8192");
        require(d.hidden > 0 && d.hidden % 256 == 0 && d.hidden <= kMaxCols, "hidden must be a multiple of 256, <= 8192");
        require(d.heads > 0 && d.kv_heads > 0 && d.heads % d.kv_heads == 0 && d.dim % d.heads == 0, "bad head counts");
        e->head_dim = d.dim / d.heads;
        e->kv_dim = e->head_dim * d.kv_heads;
        const int G = d.heads / d.kv_heads;
        require(e->head_dim == 64 || e->head_dim == 128, "head_dim must be 64 or 128");
        require(G == 1 || G == 2 || G == 3 || G == 4 || G == 6 || G == 8,
                "heads / kv_heads must be 1, 2, 3, 4, 6 or 8");
        require(d.vocab > 0 && d.vocab <= 512 * 256, "vocab must be <= 131072 (the reference's two-pass argmax)");
        require(d.layers > 0 && d.context > 0 && d.max_batch > 0 && d.max_seqs > 0, "bad limits");
        require(d.page_size == 16 || d.page_size == 32 || d.page_size == 8, "page_size must be 8, 16 or 32");
        ck(cudaSetDevice(d.device), "cudaSetDevice");
        ck(cudaDeviceGetAttribute(&e->num_sms, cudaDevAttrMultiProcessorCount, d.device), "SM count");
        ck(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking), "stream");
        ck(gemv_prepare(), "GEMV attributes");
        {
            // IJB_PDL=1 launches the step's kernels with programmatic dependent
            // launch.  Off by default: measured on B200, a decode step of
            // the 1B model took 0.98 ms with it and 0.79 ms without.
            const char *env = std::getenv("IJB_PDL");
            e->pdl = env && env[0] == '1';
            // IJB_MMA_PDL=0 turns it off for the tensor-core path, where the next
            // GEMM's weight loads and dequantisation overlap the previous kernel
            const char *env2 = std::getenv("IJB_MMA_PDL");
            e->mma_pdl = !(env2 && env2[0] == '0');
            // IJB_ATTN_PDL=1: programmatic dependent launch for the attention
            // launches of tensor-core steps; IJB_ATTN_PREP=1: the attention finish
            // kernel builds the O projection's activation tile instead of its prep
            // launch.  Both off by default: measured on B200 (same box, ragged64
            // step) 1.666 ms with neither, 1.684 with the fused prep, 1.687 with
            // PDL, 1.710 with both.
            env2 = std::getenv("IJB_ATTN_PDL");
            e->attn_pdl = env2 && env2[0] == '1';
            env2 = std::getenv("IJB_ATTN_PREP");
            e->attn_prep = env2 && env2[0] == '1';
            // IJB_SMALL_ATTN_PDL=0: CUDA-core steps launch their QKV projection,
            // attention and O projection without PDL (with it, measured on B200: a 1B
            // batch-1 step 0.830 -> 0.786 ms; PDL on the gate/up or down launch as well
            // makes it slower, 0.821 / 0.831 ms, and on every kernel 0.89 ms)
            env2 = std::getenv("IJB_SMALL_ATTN_PDL");
            e->small_attn_pdl = !(env2 && env2[0] == '0');
            // IJB_ATTN_STREAM_MIN: steps of fewer tokens use the CUDA-core split
            // kernel with 128-position splits.  Off by default: a 1B batch-1 step
            // measured 0.767 ms that way against 0.781 ms with the streaming
            // kernel, but a sequence's tokens would then depend on whether it is
            // decoded alone or in a batch (the two kernels round differently)
            env2 = std::getenv("IJB_ATTN_STREAM_MIN");
            if (env2) e->attn_stream_min = std::max(1, std::atoi(env2));
        }
        ck(attention_prepare(), "attention attributes");
        ck(cudaEventCreate(&e->ev_start), "event");
        ck(cudaEventCreate(&e->ev_end), "event");

        for (int i = 0; i < n_tensors; ++i) {
            const ijb_tensor_view &t = tensors[i];
            require(t.name != nullptr, "tensor without name");
            Weight w;
            w.name = t.name;
            w.type = t.type;
            require(t.n_dims >= 1 && t.n_dims <= 4, "Invalid tensor dimensions: " + w.name);
            w.cols = static_cast<int>(t.dims[0]);
            w.rows = t.n_dims >= 2 ? static_cast<int>(t.dims[1]) : 1;
            require(t.data_dev != nullptr, "tensor without data: " + w.name);
            if (t.type == IJB_TYPE_Q4_K || t.type == IJB_TYPE_Q6_K) {
                // power-of-two scale of the tensor-core path, from the GGUF blocks
                require(w.cols % 256 == 0, "Invalid quantized tensor shape: " + w.name);
                int *bits = dev_alloc<int>(1, "scale scan");
                cudaError_t se = mma_scale_scan_launch(t.type, static_cast<const uint8_t *>(t.data_dev),
                                                       static_cast<long>(w.rows) * (w.cols / 256), bits, e->stream);
                unsigned int hb = 0;
                if (se == cudaSuccess) se = cudaMemcpyAsync(&hb, bits, 4, cudaMemcpyDeviceToHost, e->stream);
                if (se == cudaSuccess) se = cudaStreamSynchronize(e->stream);
                cudaFree(bits);
                ck(se, "weight scale scan");
                float maxw;
                std::memcpy(&maxw, &hb, 4);
                int ex = 0;
                if (maxw > 0.f) std::frexp(maxw, &ex);
                w.mma.scale_exp = maxw > 0.f ? std::max(-60, std::min(60, 15 - ex)) : 0;
            }
            if (t.type == IJB_TYPE_Q4_K) {
                w.row_bytes = w.cols / 256 * kQ4Bytes;
                if (reinterpret_cast<uintptr_t>(t.data_dev) % 16 == 0) {
                    w.data = static_cast<const uint8_t *>(t.data_dev);
                } else {
                    uint8_t *c = dev_alloc<uint8_t>(static_cast<size_t>(w.rows) * w.row_bytes, "Q4_K copy");
                    ck(cudaMemcpy(c, t.data_dev, static_cast<size_t>(w.rows) * w.row_bytes, cudaMemcpyDeviceToDevice),
                       "Q4_K copy");
                    w.data = c;
                    w.owned = c;
                }
            } else if (t.type == IJB_TYPE_Q6_K) {
                require(w.cols % 256 == 0, "Invalid quantized tensor shape: " + w.name);
                w.row_bytes = static_cast<int>(q6_planar_row_bytes(w.cols));
                uint8_t *c = dev_alloc<uint8_t>(static_cast<size_t>(w.rows) * w.row_bytes, "Q6_K repack");
                ck(repack_q6_launch(t.data_dev, c, w.rows, w.cols, e->stream), "Q6_K repack");
                w.data = c;
                w.owned = c;
            } else if (t.type == IJB_TYPE_F32) {
                w.row_bytes = w.cols * 4;
                w.data = static_cast<const uint8_t *>(t.data_dev);
            } else {
                throw Error(IJB_ERR_INVALID, "Unsupported tensor storage type: " + w.name);
            }
            e->by_name[w.name] = static_cast<int>(e->w.size());
            e->w.push_back(w);
        }
        auto find = [&](const std::string &n) {
            auto it = e->by_name.find(n);
            require(it != e->by_name.end(), "Missing tensor: " + n);
            return it->second;
        };
        e->token_embd = find("token_embd.weight");
        require(e->w[e->token_embd].type == IJB_TYPE_Q6_K, "Expected Q6_K token embedding");
        validate_weight(e->w[e->token_embd], kQ6K, kQ6K, d.vocab, d.dim);
        e->output_norm = find("output_norm.weight");
        if (e->by_name.count("output.weight")) {
            e->output = e->by_name["output.weight"];
            validate_weight(e->w[e->output], kQ4K, kQ6K, d.vocab, d.dim);
        }
        for (int l = 0; l < d.layers; ++l) {
            const std::string p = "blk." + std::to_string(l) + ".";
            ijb_engine::Layer L;
            L.attn_norm = find(p + "attn_norm.weight");
            L.ffn_norm = find(p + "ffn_norm.weight");
            L.q = find(p + "attn_q.weight");
            L.k = find(p + "attn_k.weight");
            L.v = find(p + "attn_v.weight");
            L.o = find(p + "attn_output.weight");
            L.gate = find(p + "ffn_gate.weight");
            L.up = find(p + "ffn_up.weight");
            L.down = find(p + "ffn_down.weight");
            validate_weight(e->w[L.q], kQ4K, kQ4K, d.dim, d.dim);
            validate_weight(e->w[L.k], kQ4K, kQ4K, e->kv_dim, d.dim);
            validate_weight(e->w[L.v], kQ4K, kQ6K, e->kv_dim, d.dim);
            validate_weight(e->w[L.o], kQ4K, kQ4K, d.dim, d.dim);
            validate_weight(e->w[L.gate], kQ4K, kQ4K, d.hidden, d.dim);
            validate_weight(e->w[L.up], kQ4K, kQ4K, d.hidden, d.dim);
            validate_weight(e->w[L.down], kQ4K, kQ6K, d.dim, d.hidden);
            require(e->w[L.attn_norm].type == IJB_TYPE_F32 && e->w[L.attn_norm].cols == d.dim, "bad attn_norm");
            require(e->w[L.ffn_norm].type == IJB_TYPE_F32 && e->w[L.ffn_norm].cols == d.dim, "bad ffn_norm");
            e->layers.push_back(L);
        }
        require(e->w[e->output_norm].type == IJB_TYPE_F32 && e->w[e->output_norm].cols == d.dim, "bad output_norm");

        // chunked weight copies of the tensor-core path ([64-row group][block
        // column] chunks, so that each stage of a tile is a few plain bulk copies)
        if (d.max_batch >= kMmaEngineMinBatch) {
            ck(mma_prepare(), "tensor-core GEMM attributes");
            for (size_t i = 0; i < e->w.size(); ++i) {
                Weight &w = e->w[i];
                if (w.type != kQ4K && w.type != kQ6K) continue;
                uint8_t *c = dev_alloc<uint8_t>(static_cast<size_t>(mma_tile_bytes(w.type, w.rows, w.cols)),
                                                "tensor-core weight copy");
                ck(mma_tile_repack_launch(w.type, w.data, w.row_bytes, w.rows, w.cols, c, e->stream),
                   "tensor-core weight copy");
                w.mma.chunks = c;
                w.mma.nblocks = w.cols / 256;
                w.mma_owned = c;
                w.has_mma = true;
            }
            ck(cudaStreamSynchronize(e->stream), "tensor-core weight copy");
            const int nchunks = (d.max_batch + kMmaMaxN - 1) / kMmaMaxN;
            e->x16 = dev_alloc<uint8_t>(static_cast<size_t>(nchunks) * kX16ChunkBytes, "fp16 activation");
            ck(cudaMemset(e->x16, 0, static_cast<size_t>(nchunks) * kX16ChunkBytes), "fp16 activation clear");
            e->x_inv = dev_alloc<float>(static_cast<size_t>(nchunks) * kMmaMaxNWide, "activation scales");
            e->nside = std::min(nchunks - 1, ijb_engine::kMaxSide);
            if (e->nside > 0) ck(cudaEventCreateWithFlags(&e->ev_fork, cudaEventDisableTiming), "event");
            for (int i = 0; i < e->nside; ++i) {
                ck(cudaStreamCreateWithFlags(&e->side[i], cudaStreamNonBlocking), "stream");
                ck(cudaEventCreateWithFlags(&e->ev_join[i], cudaEventDisableTiming), "event");
            }
            const char *env = std::getenv("IJB_MMA_MIN_BATCH");  // diagnostic: path switch-over point
            if (env) e->mma_min_batch = std::max(1, std::atoi(env));
            // split-K tuning: most parts per tile, and the exchange's cost in block columns
            if ((env = std::getenv("IJB_MMA_MAX_SPLIT"))) e->mma_max_split = std::max(1, std::atoi(env));
            if ((env = std::getenv("IJB_MMA_SPLIT_COST"))) e->mma_split_cost = std::max(0, std::atoi(env));
            if ((env = std::getenv("IJB_MMA_BULK_OUT"))) e->mma_bulk_out = std::atoi(env) != 0;
            // 128-token chunks where every CTA of the launch holds one tile
            if ((env = std::getenv("IJB_MMA_WIDE"))) e->mma_wide = std::atoi(env) != 0;
        }

        // RoPE tables, computed on the host the way FastRunner's constructor
        // does (inferencer.cu:1218-1230): float pow, angle = pos * freq, cos/sin.
        const int half = e->head_dim / 2;
        std::vector<float> cs(static_cast<size_t>(d.context) * half), sn(cs.size()), freq(half);
        for (int i = 0; i < half; ++i) freq[i] = std::pow(d.rope_base, -2.f * i / e->head_dim);
        for (int pos = 0; pos < d.context; ++pos)
            for (int i = 0; i < half; ++i) {
                float angle = pos * freq[i];
                cs[static_cast<size_t>(pos) * half + i] = std::cos(angle);
                sn[static_cast<size_t>(pos) * half + i] = std::sin(angle);
            }
        e->rope_cos = dev_alloc<float>(cs.size(), "RoPE cos");
        e->rope_sin = dev_alloc<float>(sn.size(), "RoPE sin");
        ck(cudaMemcpy(e->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice), "RoPE upload");
        ck(cudaMemcpy(e->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice), "RoPE upload");

        // KV pool
        e->max_pages_per_seq = (d.context + d.page_size - 1) / d.page_size;
        e->num_pages = d.num_pages > 0 ? d.num_pages : static_cast<long>(d.max_seqs) * e->max_pages_per_seq;
        e->page_stride = 2L * d.kv_heads * d.page_size * e->head_dim;
        e->kv_f32 = d.kv_f32 ? 1 : 0;
        e->kv_elem = e->kv_f32 ? 4 : 2;
        const size_t kv_bytes = static_cast<size_t>(d.layers) * e->num_pages * e->page_stride * e->kv_elem;
        e->kv = dev_alloc<char>(kv_bytes, "KV pool");
        ck(cudaMemset(e->kv, 0, kv_bytes), "KV clear");
        if (!e->kv_f32 && (e->head_dim == 64 || e->head_dim == 128)) {
            const long layer_pool = e->num_pages * e->page_stride;
            e->kv_maps.resize(d.layers);
            for (int l = 0; l < d.layers && !e->kv_maps.empty(); ++l)
                if (attention_make_kv_map(&e->kv_maps[l], static_cast<char *>(e->kv) + l * layer_pool * e->kv_elem,
                                          e->head_dim, d.kv_heads, d.page_size, e->page_stride, e->num_pages) != 0)
                    e->kv_maps.clear();  // the CUDA-core attention serves every layer then
        }
        for (long p = e->num_pages - 1; p >= 0; --p) e->free_pages.push_back(static_cast<int>(p));
        const size_t pt = static_cast<size_t>(d.max_seqs) * e->max_pages_per_seq;
        e->page_table_dev = dev_alloc<int>(pt, "page table");
        ck(cudaMemset(e->page_table_dev, 0, pt * sizeof(int)), "page table clear");
        ck(cudaMallocHost(&e->page_table_host, pt * sizeof(int)), "page table mirror");
        std::memset(e->page_table_host, 0, pt * sizeof(int));
        e->seq_pages.resize(d.max_seqs);
        e->seq_len.assign(d.max_seqs, 0);
        e->seq_used.assign(d.max_seqs, 0);
        e->seq_used[0] = 1;  // sequence 0 backs ijb_forward / ijb_prefill

        // activations
        const size_t B = d.max_batch;
        e->x = dev_alloc<float>(B * d.dim, "residual");
        e->q = dev_alloc<float>(B * d.dim, "query");
        e->attn = dev_alloc<float>(B * d.dim, "attention out");
        e->h = dev_alloc<float>(B * d.hidden, "ffn hidden");
        e->logits = dev_alloc<float>(B * d.vocab, "logits");
        e->keys = dev_alloc<unsigned long long>(B, "argmax keys");
        // the next tokens, then the device status word: one copy brings both back
        e->next_dev = dev_alloc<int>(B + 1, "next tokens");
        e->meta_dev = dev_alloc<int>(4 * B, "step meta");
        ck(cudaMemset(e->meta_dev, 0, 4 * B * sizeof(int)), "meta clear");
        ck(cudaMallocHost(&e->meta_host, 4 * B * sizeof(int)), "meta staging");
        ck(cudaMallocHost(&e->next_host, (B + 1) * sizeof(int)), "next staging");
        std::memset(e->meta_host, 0, 4 * B * sizeof(int));
        // attention: partial softmax records per (token, head) at work-item granularity
        e->attn_split_len = attention_split_len();
        e->attn_max_splits = (d.context + attention_item_len() - 1) / attention_item_len();
        e->attn_partial = dev_alloc<float>(B * d.heads * e->attn_max_splits * (e->head_dim + 2), "attention partials");
        e->attn_counters = dev_alloc<int>(B * d.kv_heads + 2, "attention counters");
        ck(cudaMemset(e->attn_counters, 0, (B * d.kv_heads + 2) * sizeof(int)), "counters clear");
        e->status = reinterpret_cast<uint32_t *>(e->next_dev + B);
        ck(cudaMemset(e->status, 0, sizeof(uint32_t)), "status clear");
        e->scratch_key = dev_alloc<unsigned long long>(1, "argmax scratch");
        ck(cudaStreamSynchronize(e->stream), "create synchronize");
        *out = e.release();
        return IJB_OK;
    } catch (const std::exception &ex) {
        int code = fail(nullptr, ex);
        ijb_destroy(e.release());
        return code;
    }
}

void ijb_destroy(ijb_engine *e) {
    if (!e) return;
    if (e->d.device >= 0) cudaSetDevice(e->d.device);
    if (e->stream) cudaStreamSynchronize(e->stream);
    for (auto &kv : e->graphs)
        if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
    if (e->gen_graph.exec) cudaGraphExecDestroy(e->gen_graph.exec);
    cudaFree(e->gen_state);
    cudaFree(e->gen_out);
    cudaFree(e->gen_stop);
    for (auto &w : e->w) {
        if (w.owned) cudaFree(w.owned);
        if (w.mma_owned) cudaFree(w.mma_owned);
    }
    cudaFree(e->kv);
    cudaFree(e->page_table_dev);
    if (e->page_table_host) cudaFreeHost(e->page_table_host);
    cudaFree(e->rope_cos);
    cudaFree(e->rope_sin);
    cudaFree(e->x);
    cudaFree(e->q);
    cudaFree(e->attn);
    cudaFree(e->h);
    cudaFree(e->logits);
    cudaFree(e->keys);
    cudaFree(e->next_dev);
    cudaFree(e->meta_dev);
    if (e->meta_host) cudaFreeHost(e->meta_host);
    if (e->next_host) cudaFreeHost(e->next_host);
    cudaFree(e->x16);
    cudaFree(e->x_inv);
    cudaFree(e->attn_partial);
    cudaFree(e->attn_counters);
    cudaFree(e->scratch_key);
    cudaFree(e->trace_x);
    cudaFree(e->trace_q);
    if (e->ev_start) cudaEventDestroy(e->ev_start);
    if (e->ev_end) cudaEventDestroy(e->ev_end);
    if (e->ev_fork) cudaEventDestroy(e->ev_fork);
    for (int i = 0; i < e->nside; ++i) {
        if (e->ev_join[i]) cudaEventDestroy(e->ev_join[i]);
        if (e->side[i]) cudaStreamDestroy(e->side[i]);
    }
    if (e->stream) cudaStreamDestroy(e->stream);
    delete e;
}

const char *ijb_last_error(const ijb_engine *e) { return e ? e->err.c_str() : t_create_err.c_str(); }

int ijb_tensor_index(const ijb_engine *e, const char *name) {
    if (!e || !name) return -1;
    auto it = e->by_name.find(name);
    return it == e->by_name.end() ? -1 : it->second;
}

int ijb_matvec(ijb_engine *e, int ti, const float *x, float *y, int cols, int rows, int batch, void *stream) {
    try {
        require(e != nullptr, "null engine");
        require(ti >= 0 && ti < static_cast<int>(e->w.size()), "bad tensor index");
        const Weight &w = e->w[ti];
        require((w.type == kQ4K || w.type == kQ6K) && w.cols == cols && w.rows == rows,
                "Unexpected quantized matrix shape");
        require(batch >= 1 && cols <= kMaxCols, "bad batch or cols");
        cudaStream_t s = pick(e, stream);
        const ProjSeg segs[1] = {{ti, -1, kEpiStore, y, rows}};
        launch_projection(e, s, 0, batch, x, cols, nullptr, segs, 1, nullptr, 0);
        return IJB_OK;
    } catch (const std::exception &ex) {
        return fail(e, ex);
    }
}

int ijb_forward(ijb_engine *e, int token, int pos, int need_logits, int *next_token) {
    try {
        require(e != nullptr, "null engine");
        require(pos >= 0 && pos < e->d.context && token >= 0 && token < e->d.vocab,
                "Token or position outside model context");
        require(pos <= e->seq_len[0], "position beyond the cached length of the sequence");
        const int seq = 0;
        packed_step(e, 1, &seq, &token, &pos, need_logits != 0);
        e->seq_len[0] = pos + 1;
        if (next_token) *next_token = need_logits ? e->next_host[0] : -1;
        return IJB_OK;
    } catch (const std::exception &ex) {
        return fail(e, ex);
    }
}

int ijb_forward_traced(ijb_engine *e, int token, int pos, int need_logits, int *next_token, float *layer_trace,
                       int8_t *quant_trace) {
    try {
        require(e != nullptr, "null engine");
        require(pos >= 0 && pos < e->d.context && token >= 0 && token < e->d.vocab,
                "Token or position outside model context");
        require(pos <= e->seq_len[0], "position beyond the cached length of the sequence");
        ensure_trace_buffers(e);
        const int seq = 0;
        packed_step(e, 1, &seq, &token, &pos, need_logits != 0, true);
        e->seq_len[0] = pos + 1;
        if (next_token) *next_token = need_logits ? e->next_host[0] : -1;
        download_trace(e, 0, layer_trace, quant_trace);
        return IJB_OK;
    } catch (const std::exception &ex) {
        return fail(e, ex);
    }
}

int ijb_prefill_traced(ijb_engine *e, const int *tokens, int n, int *next_token, float *all_layer_trace,
                       int8_t *first_quant_trace, int8_t *last_quant_trace) {
    try {
        require(e != nullptr && tokens != nullptr && n >= 1, "bad arguments");
        require(n <= e->d.context, "prompt exceeds context", IJB_ERR_CAPACITY);
        ensure_trace_buffers(e);
        e->seq_len[0] = 0;
        const ijb_model_desc &d = e->d;
        std::vector<int> seqs(d.max_batch, 0), pos(d.max_batch);
        for (int c = 0; c < n; c += d.max_batch) {
            const int cn = std::min(d.max_batch, n - c);
            for (int i = 0; i < cn; ++i) pos[i] = c + i;
            const bool last = c + cn == n;
            packed_step(e, cn, seqs.data(), tokens + c, pos.data(), last, true);
            e->seq_len[0] = c + cn;
            for (int i = 0; i < cn && all_layer_trace; ++i)
                download_trace(e, i, all_layer_trace + static_cast<long>(c + i) * d.layers * d.dim, nullptr);
            if (c == 0) download_trace(e, 0, nullptr, first_quant_trace);
            if (last) {
                download_trace(e, cn - 1, nullptr, last_quant_trace);
                if (next_token) *next_token = e->next_host[cn - 1];
            }
        }
        return IJB_OK;
    } catch (const std::exception &ex) {
        return fail(e, ex);
    }
}

int ijb_last_step_size(const ijb_engine *e) { return e ? e->last_n : -1; }

int ijb_time_layer_projections(ijb_engine *e, int n, int reps, float *ms_per_layer) {
    try {
        require(e != nullptr && ms_per_layer != nullptr, "bad arguments");
        require(n >= 1 && n <= e->d.max_batch && n <= e->d.context, "n must be 1..max_batch");
        require(reps >= 1 && reps <= 1000, "reps must be 1..1000");
        require(e->seq_len[0] == 0 && e->seq_pages[0].empty(),
                "sequence 0 must be empty (its KV pages receive the timed K/V writes)");
        ck(cudaSetDevice(e->d.device), "cudaSetDevice");
        // tokens 0..n-1 of sequence 0 at positions 0..n-1 (their K/V slots are sequence 0's pages)
        const ijb_model_desc &d = e->d;
        int *mt = e->meta_host;
        for (int i = 0; i < n; ++i) {
            mt[i] = i % d.vocab;
            mt[d.max_batch + i] = 0;
            mt[2 * d.max_batch + i] = i;
            mt[3 * d.max_batch + i] = slot_for(e, 0, i);
        }
        ck(cudaMemcpyAsync(e->meta_dev, e->meta_host, 4 * d.max_batch * sizeof(int), cudaMemcpyHostToDevice, e->stream),
           "meta H2D");
        cudaGraph_t graph;
        cudaGraphExec_t exec = nullptr;
        const uint64_t before = g_launches.load();
        ck(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal), "begin capture");
        try {
            for (int r = 0; r < reps; ++r) {
                enqueue_qkv(e, 0, n, e->stream);
                enqueue_o(e, 0, n, e->stream);
                enqueue_gateup(e, 0, n, e->stream);
                enqueue_down(e, 0, n, e->stream);
            }
        } catch (...) {
            cudaStreamEndCapture(e->stream, &graph);
            throw;
        }
        ck(cudaStreamEndCapture(e->stream, &graph), "end capture");
        const uint64_t launches = g_launches.load() - before;
        cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        ck(ie, "graph instantiate");
        float ms = 0.f;
        cudaError_t le = cudaGraphLaunch(exec, e->stream);  // warm-up
        if (le == cudaSuccess) le = cudaEventRecord(e->ev_start, e->stream);
        if (le == cudaSuccess) le = cudaGraphLaunch(exec, e->stream);
        if (le == cudaSuccess) le = cudaEventRecord(e->ev_end, e->stream);
        if (le == cudaSuccess) le = cudaStreamSynchronize(e->stream);
        if (le == cudaSuccess) le = cudaEventElapsedTime(&ms, e->ev_start, e->ev_end);
        cudaGraphExecDestroy(exec);
        ck(le, "layer timing");
        g_launches += launches;  // the second replay (the capture counted the first)
        check_device_status(e);
        // the timed K/V writes leave sequence 0 holding n positions of no meaning
        for (int p : e->seq_pages[0]) e->free_pages.push_back(p);
        e->seq_pages[0].clear();
        *ms_per_layer = ms / reps;
        return IJB_OK;
    } catch (const std::exception &ex) {
        return fail(e, ex);
    }
}

int ijb_time_layer_attention(ijb_engine *e, int n, const int *seq_ids, int reps, float *ms_per_layer,
                              long long *kv_bytes) {
    try {
        require(e != nullptr && seq_ids != nullptr && ms_per_layer != nullptr && kv_bytes != nullptr, "bad arguments");
        const ijb_model_desc &d = e->d;
        require(n >= 1 && n <= d.max_batch, "n must be 1..max_batch");
        require(reps >= 1 && reps <= 1000, "reps must be 1..1000");
        ck(cudaSetDevice(d.device), "cudaSetDevice");
        // one query token per sequence at its newest position: the launch reads
        // the sequence's whole cached context, as the next decode step would
        int *mt = e->meta_host;
        long long positions = 0;
        for (int i = 0; i < n; ++i) {
            const int sq = seq_ids[i];
            require(sq >= 0 && sq < d.max_seqs && e->seq_used[sq], "unknown sequence id");
            const int len = e->seq_len[sq];
            require(len >= 1, "sequence holds no positions");
            mt[i] = 0;
            mt[d.max_batch + i] = sq;
            mt[2 * d.max_batch + i] = len - 1;
            mt[3 * d.max_batch + i] = slot_for(e, sq, len - 1);  // an existing slot: no page is taken
            positions += len;
        }
        ck(cudaMemcpyAsync(e->meta_dev, e->meta_host, 4 * d.max_batch * sizeof(int), cudaMemcpyHostToDevice, e->stream),
           "meta H2D");
        const AttnParams a = attn_params(e, 0, n);
        const bool pdl = e->pdl || (n >= e->mma_min_batch ? e->attn_pdl : e->small_attn_pdl);
        cudaGraph_t graph;
        cudaGraphExec_t exec = nullptr;
        ck(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal), "begin capture");
        cudaError_t ce = cudaSuccess;
        for (int r = 0; r < reps && ce == cudaSuccess; ++r) ce = attention_launch(a, e->stream, pdl);
        const cudaError_t ee = cudaStreamEndCapture(e->stream, &graph);
        if (ee == cudaSuccess && ce != cudaSuccess) cudaGraphDestroy(graph);
        ck(ce, "attention launch");
        ck(ee, "end capture");
        cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        ck(ie, "graph instantiate");
        float ms = 0.f;
        cudaError_t le = cudaGraphLaunch(exec, e->stream);  // warm-up
        if (le == cudaSuccess) le = cudaEventRecord(e->ev_start, e->stream);
        if (le == cudaSuccess) le = cudaGraphLaunch(exec, e->stream);
        if (le == cudaSuccess) le = cudaEventRecord(e->ev_end, e->stream);
        if (le == cudaSuccess) le = cudaStreamSynchronize(e->stream);
        if (le == cudaSuccess) le = cudaEventElapsedTime(&ms, e->ev_start, e->ev_end);
        cudaGraphExecDestroy(exec);
        ck(le, "attention timing");
        g_launches += 2ull * reps * attention_kernels(a);
        check_device_status(e);
        *ms_per_layer = ms / reps;
        *kv_bytes = positions * d.kv_heads * 2LL * e->head_dim * e->kv_elem;
        return IJB_OK;
    } catch (const std::exception &ex) {
        return fail(e, ex);
    }
}

int ijb_seq_prefill(ijb_engine *e, int seq, const int *tokens, int n, int *next_token) {
    try {
        require(e != nullptr && tokens != nullptr && n >= 1, "bad arguments");
        require(seq >= 0 && seq < e->d.max_seqs && e->seq_used[seq], "unknown sequence id");
        const int start = e->seq_len[seq];
        require(start + n <= e->d.context, "prompt exceeds context", IJB_ERR_CAPACITY);
        std::vector<int> seqs(e->d.max_batch, seq), pos(e->d.max_batch);
        for (int c = 0; c < n; c += e->d.max_batch) {
            const int cn = std::min(e->d.max_batch, n - c);
            for (int i = 0; i < cn; ++i) pos[i] = start + c + i;
            const bool last = c + cn == n;
            packed_step(e, cn, seqs.data(), tokens + c, pos.data(), last);
            e->seq_len[seq] = start + c + cn;
            if (last && next_token) *next_token = e->next_host[cn - 1];
        }
        return IJB_OK;
    } catch (const std::exception &ex) {
        return fail(e, ex);
    }
}

int ijb_prefill(ijb_engine *e, const int *tokens, int n, int *next_token) {
    if (!e) return IJB_ERR_INVALID;
    e->seq_len[0] = 0;
    return ijb_seq_prefill(e, 0, tokens, n, next_token);
}

int ijb_reset(ijb_engine *e) {
    if (!e) return IJB_ERR_INVALID;
    e->seq_len[0] = 0;
    return IJB_OK;
}

const float *ijb_logits_dev(const ijb_engine *e) { return e ? e->logits : nullptr; }
const float *ijb_residual_dev(const ijb_engine *e) { return e ? e->x : nullptr; }

int ijb_seq_open(ijb_engine *e, int *seq_id) {
    try {
        require(e != nullptr && seq_id != nullptr, "bad arguments");
        for (int s = 1; s < e->d.max_seqs; ++s)
            if (!e->seq_used[s]) {
                e->seq_used[s] = 1;
                e->seq_len[s] = 0;
                *seq_id = s;
                return IJB_OK;
            }
        throw Error(IJB_ERR_CAPACITY, "sequence table full");
    } catch (const std::exception &ex) {
        return fail(e, ex);
    }
}

int ijb_seq_close(ijb_engine *e, int seq) {
    try {
        require(e != nullptr && seq > 0 && seq < e->d.max_seqs && e->seq_used[seq], "unknown sequence id");
        for (int p : e->seq_pages[seq]) e->free_pages.push_back(p);
        e->seq_pages[seq].clear();
        e->seq_len[seq] = 0;
        e->seq_used[seq] = 0;
        return IJB_OK;
    } catch (const std::exception &ex) {
        return fail(e, ex);
    }
}

int ijb_seq_length(const ijb_engine *e, int seq) {
    if (!e || seq < 0 || seq >= e->d.max_seqs || !e->seq_used[seq]) return -1;
    return e->seq_len[seq];
}

int ijb_generate(ijb_engine *e, int seq, int first_token, int max_tokens, const int *stop_ids, int n_stop,
                 int *out_tokens, int *n_out) {
    try {
        require(e != nullptr && out_tokens != nullptr && n_out != nullptr, "bad arguments");
        const ijb_model_desc &d = e->d;
        require(seq >= 0 && seq < d.max_seqs && e->seq_used[seq], "unknown sequence id");
        require(first_token >= 0 && first_token < d.vocab, "Token or position outside model context");
        require(max_tokens >= 0 && n_stop >= 0 && n_stop <= kGenMaxStop && (n_stop == 0 || stop_ids),
                "bad generate limits (stop ids: at most 16)");
        *n_out = 0;
        const int pos0 = e->seq_len[seq];
        // the reference loop's first iteration, on the host: `next` from the prefill
        for (int i = 0; i < n_stop; ++i)
            if (first_token == stop_ids[i]) return IJB_OK;
        if (max_tokens == 0) return IJB_OK;
        out_tokens[0] = first_token;
        *n_out = 1;
        if (max_tokens == 1 || pos0 >= d.context) return IJB_OK;
        // at most this many steps feed a new position; their pages are allocated now
        const int steps = std::min(max_tokens - 1, d.context - pos0);
        int *mt = e->meta_host;
        std::memset(mt, 0, 4 * d.max_batch * sizeof(int));
        for (int k = steps - 1; k >= 0; --k) slot_for(e, seq, pos0 + k);
        mt[0] = first_token;
        mt[d.max_batch] = seq;
        mt[2 * d.max_batch] = pos0;
        mt[3 * d.max_batch] = slot_for(e, seq, pos0);
        if (!e->gen_state) {
            e->gen_state = dev_alloc<GenState>(1, "generate state");
            e->gen_out = dev_alloc<int>(d.context + 1, "generate output");
            e->gen_stop = dev_alloc<int>(kGenMaxStop, "generate stop ids");
        }
        GenState g{};
        g.count = 1;
        g.max_tokens = max_tokens;
        g.context = d.context;
        g.n_stop = n_stop;
        g.seq = seq;
        g.page_size = d.page_size;
        g.max_pages_per_seq = e->max_pages_per_seq;
        cudaStream_t s = e->stream;
        ck(cudaMemcpyAsync(e->meta_dev, mt, 4 * d.max_batch * sizeof(int), cudaMemcpyHostToDevice, s), "meta H2D");
        ck(cudaMemcpyAsync(e->gen_state, &g, sizeof(g), cudaMemcpyHostToDevice, s), "generate state H2D");
        if (n_stop) ck(cudaMemcpyAsync(e->gen_stop, stop_ids, n_stop * sizeof(int), cudaMemcpyHostToDevice, s), "stop H2D");
        ck(cudaStreamSynchronize(s), "generate setup");  // the host buffers above are stack / staging memory
        if (!e->gen_graph.exec) {
            // one batch-1 step reading its inputs from meta_dev, then the advance kernel
            cudaGraph_t graph;
            const uint64_t before = g_launches.load();
            ck(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal), "begin capture");
            try {
                enqueue_step(e, 1, true, s, false);
                ck(gen_advance_launch(e->gen_state, e->next_dev, e->meta_dev, d.max_batch, e->page_table_dev,
                                      e->gen_stop, e->gen_out, s),
                   "generate advance launch");
                ++g_launches;
            } catch (...) {
                cudaStreamEndCapture(s, &graph);
                throw;
            }
            ck(cudaStreamEndCapture(s, &graph), "end capture");
            e->gen_graph.launches = g_launches.load() - before;
            g_launches.store(before);
            cudaError_t ie = cudaGraphInstantiate(&e->gen_graph.exec, graph, 0);
            cudaGraphDestroy(graph);
            ck(ie, "graph instantiate");
        }
        // steps are queued in rounds without waiting for their tokens; the host
        // reads the state once per round (steps queued past the end recompute the
        // last position, see the advance kernel)
        ck(cudaEventRecord(e->ev_start, s), "generate timer start");
        int queued = 0;
        while (queued < steps) {
            const int round = std::min(kGenRound, steps - queued);
            for (int k = 0; k < round; ++k) ck(cudaGraphLaunch(e->gen_graph.exec, s), "graph launch");
            g_launches += e->gen_graph.launches * round;
            queued += round;
            ck(cudaMemcpyAsync(&g, e->gen_state, sizeof(g), cudaMemcpyDeviceToHost, s), "generate state D2H");
            ck(cudaStreamSynchronize(s), "generate synchronize");
            if (g.done) break;
        }
        ck(cudaEventRecord(e->ev_end, s), "generate timer end");
        ck(cudaMemcpyAsync(out_tokens + 1, e->gen_out + 1, (g.count - 1) * sizeof(int), cudaMemcpyDeviceToHost, s),
           "generate output D2H");
        ck(cudaStreamSynchronize(s), "generate synchronize");
        float ms = 0.f;
        ck(cudaEventElapsedTime(&ms, e->ev_start, e->ev_end), "generate timer");
        e->last_step_ms = ms / static_cast<float>(queued);
        e->last_n = 1;
        check_device_status(e);
        *n_out = g.count;
        e->seq_len[seq] = pos0 + g.processed;
        // pages allocated for positions the loop did not reach go back to the pool
        auto &pages = e->seq_pages[seq];
        const size_t keep = (e->seq_len[seq] + d.page_size - 1) / d.page_size;
        while (pages.size() > keep) {
            e->free_pages.push_back(pages.back());
            pages.pop_back();
        }
        return IJB_OK;
    } catch (const std::exception &ex) {
        return fail(e, ex);
    }
}

int ijb_decode_step(ijb_engine *e, int n, const int *seq_ids, const int *tokens, int *next_tokens) {
    try {
        require(e != nullptr && seq_ids != nullptr && tokens != nullptr, "bad arguments");
        require(n >= 1 && n <= e->d.max_batch, "step size must be 1..max_batch", IJB_ERR_CAPACITY);
        std::vector<int> pos(n);
        std::unordered_map<int, int> next_pos;
        for (int i = 0; i < n; ++i) {
            const int s = seq_ids[i];
            require(s >= 0 && s < e->d.max_seqs && e->seq_used[s], "unknown sequence id");
            auto it = next_pos.find(s);
            pos[i] = it == next_pos.end() ? e->seq_len[s] : it->second;
            next_pos[s] = pos[i] + 1;
        }
        packed_step(e, n, seq_ids, tokens, pos.data(), true);
        for (auto &kv : next_pos) e->seq_len[kv.first] = kv.second;
        if (next_tokens) std::memcpy(next_tokens, e->next_host, n * sizeof(int));
        return IJB_OK;
    } catch (const std::exception &ex) {
        return fail(e, ex);
    }
}

int ijb_argmax(const float *values, int n, int *index, void *stream) {
    try {
        require(values && index && n >= 1 && n <= 512 * 256, "bad argmax arguments");
        static unsigned long long *scratch[64] = {nullptr};
        static std::mutex mu;
        int dev = 0;
        ck(cudaGetDevice(&dev), "cudaGetDevice");
        require(dev >= 0 && dev < 64, "device ordinal");
        {
            std::lock_guard<std::mutex> lock(mu);
            if (!scratch[dev]) scratch[dev] = dev_alloc<unsigned long long>(1, "argmax scratch");
        }
        ck(argmax_launch(values, n, scratch[dev], index, static_cast<cudaStream_t>(stream)), "argmax launch");
        g_launches += 2;
        return IJB_OK;
    } catch (const std::exception &ex) {
        return fail(nullptr, ex);
    }
}

int ijb_dequant(int type, const void *blocks, long n_blocks, float *out, void *stream) {
    try {
        require(type == IJB_TYPE_Q4_K || type == IJB_TYPE_Q6_K, "type must be Q4_K or Q6_K");
        require(blocks && out && n_blocks >= 0, "bad dequant arguments");
        ck(dequant_launch(type, blocks, n_blocks, out, static_cast<cudaStream_t>(stream)), "dequant launch");
        ++g_launches;
        return IJB_OK;
    } catch (const std::exception &ex) {
        return fail(nullptr, ex);
    }
}

long ijb_q6k_planar_row_bytes(int cols) { return cols > 0 && cols % 256 == 0 ? q6_planar_row_bytes(cols) : -1; }

int ijb_repack_q6k(const void *src, void *dst, int rows, int cols, void *stream) {
    try {
        require(src && dst && rows >= 0 && cols > 0 && cols % 256 == 0, "bad repack arguments");
        ck(repack_q6_launch(src, dst, rows, cols, static_cast<cudaStream_t>(stream)), "repack launch");
        ++g_launches;
        return IJB_OK;
    } catch (const std::exception &ex) {
        return fail(nullptr, ex);
    }
}

int ijb_gemv(int type, const void *w, const float *x, float *y, int cols, int rows, int batch, int use_dp4a,
             void *stream) {
    try {
        require(type == IJB_TYPE_Q4_K || type == IJB_TYPE_Q6_K, "type must be Q4_K or Q6_K");
        require(w && x && y && rows >= 1 && cols > 0 && cols % 256 == 0 && cols <= kMaxCols, "bad GEMV arguments");
        require(batch >= 1 && batch <= kMaxBatch, "batch must be 1..8");
        require(reinterpret_cast<uintptr_t>(w) % 16 == 0, "weights must be 16-byte aligned");
        int dev = 0, sms = 0;
        ck(cudaGetDevice(&dev), "cudaGetDevice");
        ck(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "SM count");
        Weight wt;
        wt.type = type;
        wt.rows = rows;
        wt.cols = cols;
        wt.data = static_cast<const uint8_t *>(w);
        wt.row_bytes = type == IJB_TYPE_Q4_K ? cols / 256 * kQ4Bytes : static_cast<int>(q6_planar_row_bytes(cols));
        ijb_model_desc d{};
        d.use_dp4a = use_dp4a & 1;
        d.use_q6_dp4a = use_dp4a & 1;
        GemvParams p;
        std::memset(&p, 0, sizeof(p));
        p.cols = cols;
        p.batch = batch;
        p.x = x;
        p.x_stride = cols;
        add_seg(p, wt, nullptr, kEpiStore, y, rows, 0, d);
        ck(gemv_launch(p, sms, static_cast<cudaStream_t>(stream), (use_dp4a & IJB_GEMV_PDL) != 0), "GEMV launch");
        ++g_launches;
        return IJB_OK;
    } catch (const std::exception &ex) {
        return fail(nullptr, ex);
    }
}

int ijb_probe_wait_timeout(ijb_engine *e, uint64_t limit_ns) {
    try {
        require(e != nullptr, "null engine");
        require(limit_ns >= 1000 && limit_ns <= 100000000ull, "limit_ns must be 1 us .. 100 ms");
        ck(cudaSetDevice(e->d.device), "cudaSetDevice");
        ck(wait_probe_launch(e->status, limit_ns, e->stream), "wait probe launch");
        ++g_launches;
        ck(cudaStreamSynchronize(e->stream), "wait probe synchronize");
        check_device_status(e);
        return IJB_OK;
    } catch (const std::exception &ex) {
        return fail(e, ex);
    }
}

}  // extern "C"

struct ijb_weight {
    int type = 0, rows = 0, cols = 0, device = 0;
    MmaWeight mma{};
    uint8_t *x16 = nullptr;
    float *x_inv = nullptr;
    uint32_t *status = nullptr;
};

extern "C" {

int ijb_weight_create(int type, const void *w_dev, int rows, int cols, int device, ijb_weight **out) {
    std::unique_ptr<ijb_weight> w(new ijb_weight());
    uint8_t *unit = nullptr;
    try {
        require(out != nullptr && w_dev != nullptr, "null argument");
        require(type == IJB_TYPE_Q4_K || type == IJB_TYPE_Q6_K, "type must be Q4_K or Q6_K");
        require(rows >= 1 && cols > 0 && cols % 256 == 0 && cols <= kMaxCols, "bad matrix shape");
        require(reinterpret_cast<uintptr_t>(w_dev) % 16 == 0, "weights must be 16-byte aligned");
        ck(cudaSetDevice(device), "cudaSetDevice");
        ck(mma_prepare(), "tensor-core GEMM attributes");
        w->type = type;
        w->rows = rows;
        w->cols = cols;
        w->device = device;
        // power-of-two scale from the GGUF blocks, as ijb_create does
        int *bits = dev_alloc<int>(1, "scale scan");
        cudaError_t se = mma_scale_scan_launch(type, static_cast<const uint8_t *>(w_dev),
                                               static_cast<long>(rows) * (cols / 256), bits, nullptr);
        unsigned int hb = 0;
        if (se == cudaSuccess) se = cudaMemcpy(&hb, bits, 4, cudaMemcpyDeviceToHost);
        cudaFree(bits);
        ck(se, "weight scale scan");
        float maxw;
        std::memcpy(&maxw, &hb, 4);
        int ex = 0;
        if (maxw > 0.f) std::frexp(maxw, &ex);
        w->mma.scale_exp = maxw > 0.f ? std::max(-60, std::min(60, 15 - ex)) : 0;
        w->mma.nblocks = cols / 256;
        const uint8_t *src = static_cast<const uint8_t *>(w_dev);
        long row_bytes = cols / 256 * kQ4Bytes;
        if (type == IJB_TYPE_Q6_K) {  // the chunked copy reads the Q6_K unit layout
            row_bytes = q6_planar_row_bytes(cols);
            unit = dev_alloc<uint8_t>(static_cast<size_t>(rows) * row_bytes, "Q6_K unit layout");
            ck(repack_q6_launch(w_dev, unit, rows, cols, nullptr), "Q6_K repack");
            src = unit;
        }
        uint8_t *c = dev_alloc<uint8_t>(static_cast<size_t>(mma_tile_bytes(type, rows, cols)), "tensor-core weight copy");
        w->mma.chunks = c;
        ck(mma_tile_repack_launch(type, src, row_bytes, rows, cols, c, nullptr), "tensor-core weight copy");
        ck(cudaDeviceSynchronize(), "weight prepare");
        cudaFree(unit);
        unit = nullptr;
        w->x16 = dev_alloc<uint8_t>(static_cast<size_t>(kMaxCols / 128) * kMmaMaxN * 256, "fp16 activation");
        ck(cudaMemset(w->x16, 0, static_cast<size_t>(kMaxCols / 128) * kMmaMaxN * 256), "fp16 activation clear");
        w->x_inv = dev_alloc<float>(kMmaMaxN, "activation scales");
        w->status = dev_alloc<uint32_t>(1, "status");
        ck(cudaMemset(w->status, 0, 4), "status clear");
        g_launches += 3 + (type == IJB_TYPE_Q6_K ? 1 : 0);
        *out = w.release();
        return IJB_OK;
    } catch (const std::exception &ex) {
        cudaFree(unit);
        ijb_weight_destroy(w.release());
        return fail(nullptr, ex);
    }
}

void ijb_weight_destroy(ijb_weight *w) {
    if (!w) return;
    cudaSetDevice(w->device);
    cudaFree(const_cast<uint8_t *>(w->mma.chunks));
    cudaFree(w->x16);
    cudaFree(w->x_inv);
    cudaFree(w->status);
    delete w;
}

int ijb_weight_matmul(ijb_weight *w, const float *x_dev, int n, const float *norm_w_dev, float eps, int use_dp4a,
                      float *y_dev, long y_stride, int key_offset, unsigned long long *keys_dev, void *stream) {
    try {
        require(w != nullptr && x_dev != nullptr && y_dev != nullptr, "null argument");
        require(n >= 1 && y_stride >= w->rows && key_offset >= 0, "bad matmul arguments");
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        if (keys_dev) ck(cudaMemsetAsync(keys_dev, 0, static_cast<size_t>(n) * 8, s), "keys clear");
        const int nb = w->cols / 256;
        for (int t0 = 0; t0 < n; t0 += kMmaMaxN) {
            const int tn = std::min(kMmaMaxN, n - t0);
            const int n_pad = (tn + 15) / 16 * 16;
            ck(mma_prep_launch(x_dev + static_cast<long>(t0) * w->cols, w->cols, norm_w_dev, eps, w->cols, tn, n_pad,
                               use_dp4a ? 1 : 0, w->x16, w->x_inv, s, false),
               "activation prep launch");
            MmaParams m;
            std::memset(&m, 0, sizeof(m));
            m.w[0] = w->mma;
            MmaSeg &sg = m.seg[0];
            sg.w0 = 0;
            sg.w1 = -1;
            sg.type = w->type;
            sg.rows = w->rows;
            sg.tile0 = 0;
            sg.ntiles = (w->rows + kMmaTileM - 1) / kMmaTileM;
            sg.epi = keys_dev ? kEpiLogitsArgmax : kEpiStore;
            sg.out = y_dev + static_cast<long>(t0) * y_stride;
            sg.out_stride = y_stride;
            sg.key_offset = key_offset;
            m.nseg = 1;
            m.total_tiles = sg.ntiles;
            m.cols = w->cols;
            m.batch = tn;
            m.n_pad = n_pad;
            m.x16 = w->x16;
            m.x_inv = w->x_inv;
            m.argmax_keys = keys_dev ? keys_dev + t0 : nullptr;
            m.status = w->status;
            m.ksplit = mma_choose_split(m.total_tiles, nb, 8, 1, &m.bps);
            ck(mma_gemm_launch(m, s, false), "tensor-core GEMM launch");
            g_launches += 2;
        }
        return IJB_OK;
    } catch (const std::exception &ex) {
        return fail(nullptr, ex);
    }
}

int ijb_weight_status(ijb_weight *w) {
    if (!w) return IJB_ERR_INVALID;
    uint32_t st = 0;
    if (cudaMemcpy(&st, w->status, 4, cudaMemcpyDeviceToHost) != cudaSuccess) return IJB_ERR_CUDA;
    if (st) {
        cudaMemset(w->status, 0, 4);
        set_thread_error("kernel reported device error code " + std::to_string(st));
        return IJB_ERR_DEVICE;
    }
    return IJB_OK;
}

int ijb_keys_to_tokens(const unsigned long long *keys_dev, int n, int *tokens_dev, void *stream) {
    try {
        require(keys_dev && tokens_dev && n >= 1, "bad arguments");
        ck(keys_to_tokens_launch(keys_dev, n, tokens_dev, static_cast<cudaStream_t>(stream), false),
           "argmax decode launch");
        ++g_launches;
        return IJB_OK;
    } catch (const std::exception &ex) {
        return fail(nullptr, ex);
    }
}

uint64_t ijb_kernel_launches(void) { return g_launches.load(); }

float ijb_last_step_ms(const ijb_engine *e) { return e ? e->last_step_ms : -1.f; }

}  // extern "C"
