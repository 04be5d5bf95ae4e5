/*
 * ijb200 — C ABI of the B200 (sm_100a) decode hot path for inferencer-jetson
 * style Llama-3.2 GGUF models (Q4_K / Q6_K weights).
 *
 * This is the drop-in boundary for the reference's C++ runner classes in
 * inferencer.cu: FastGPU (:1101-1180) and FastRunner (:1182-1532).  A thin C++
 * shim with the reference's method signatures sits on top of it
 * (inferencer-jetson_b200/host/fast_runner.hpp).
 *
 * Conventions
 *   - Every call returns an int status: IJB_OK (0) or an IJB_ERR_* code.  The
 *     message of the last failure is available from ijb_last_error().  No C++
 *     exception crosses this boundary (the reference throws
 *     std::runtime_error from cuda_check, inferencer.cu:126-128, and from its
 *     shape checks; the shim turns a non-zero status back into that).
 *   - Pointers named *_dev are device pointers on the engine's device; all
 *     other pointers are host pointers.  `stream` is a cudaStream_t passed as
 *     void* (NULL = the engine's own stream).
 *   - Tensor dims follow GGUF: dims[0] is the row length (cols), dims[1] the
 *     row count (Tensor::cols()/rows(), inferencer.cu:184-185).
 *   - Type ids are GGML's: 0 F32, 1 F16, 12 Q4_K, 14 Q6_K (inferencer.cu:194-201).
 */
#ifndef IJB200_H
#define IJB200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define IJB_OK 0
#define IJB_ERR_INVALID 1   /* bad argument, shape, type or range */
#define IJB_ERR_CUDA 2      /* a CUDA runtime call failed */
#define IJB_ERR_NOMEM 3     /* device or host allocation failed */
#define IJB_ERR_CAPACITY 4  /* KV page pool, sequence table or batch limit exhausted */
#define IJB_ERR_DEVICE 5    /* a kernel reported an error (bounded wait expired, bad index) */

#define IJB_TYPE_F32 0
#define IJB_TYPE_F16 1
#define IJB_TYPE_Q4_K 12
#define IJB_TYPE_Q6_K 14

typedef struct ijb_engine ijb_engine;

/* Model hyper-parameters (the GGUF keys FastRunner reads, inferencer.cu:1205-1214)
 * plus serving limits.  The reference accepts only the 3B shape
 * (:1215-1217); this build takes any Llama shape with dim, hidden a multiple
 * of 256 and <= 8192, head_dim 64 or 128, and vocab <= 131072. */
typedef struct {
    int dim;             /* llama.embedding_length */
    int layers;          /* llama.block_count */
    int heads;           /* llama.attention.head_count */
    int kv_heads;        /* llama.attention.head_count_kv */
    int hidden;          /* llama.feed_forward_length */
    int vocab;           /* llama.vocab_size */
    float eps;           /* llama.attention.layer_norm_rms_epsilon */
    float rope_base;     /* llama.rope.freq_base */
    int context;         /* max positions per sequence (FastRunner --context) */
    int max_batch;       /* max tokens in one packed step */
    int max_seqs;        /* max open sequences */
    int page_size;       /* tokens per KV page; 0 = 16 */
    long num_pages;      /* KV page pool size; 0 = max_seqs * ceil(context/page_size) */
    int use_dp4a;        /* Q4_K on the INT8 activation path (reference default; --float-gemv clears) */
    int use_q6_dp4a;     /* Q6_K on the INT8 activation path (reference default; --float-q6 clears) */
    int kv_f32;          /* 1: cache K/V as fp32 like the reference (inferencer.cu:1132); 0: fp16 (half the bytes) */
    int device;          /* CUDA device ordinal */
} ijb_model_desc;

/* A view of one GGUF tensor already on the device (Tensor, inferencer.cu:178-186;
 * Tensor::gpu points into the blob GGUF::upload copied, :321-339). */
typedef struct {
    const char *name;      /* GGUF tensor name, e.g. "blk.0.attn_q.weight" */
    int type;              /* IJB_TYPE_* */
    int n_dims;
    int64_t dims[4];
    const void *data_dev;  /* device pointer, 16-byte aligned for quantised types */
} ijb_tensor_view;

/* Builds an engine over the given tensors: validates names, types and shapes,
 * takes engine-owned copies (Q6_K rows are repacked into a 16-byte aligned
 * plane layout), allocates activations, the paged fp16 KV pool and the RoPE
 * tables (computed on the host exactly as FastRunner's constructor does,
 * inferencer.cu:1218-1230).  Replaces FastGPU::FastGPU + FastRunner::FastRunner. */
int ijb_create(const ijb_model_desc *desc, const ijb_tensor_view *tensors, int n_tensors, ijb_engine **out);

/* Frees everything the engine owns (FastGPU::~FastGPU, inferencer.cu:1141-1150). */
void ijb_destroy(ijb_engine *engine);

/* Message of the last failed call on `engine` (or of the last failed
 * ijb_create in this thread when engine is NULL).  Never NULL. */
const char *ijb_last_error(const ijb_engine *engine);

/* Index of a tensor passed to ijb_create, by GGUF name; -1 if absent. */
int ijb_tensor_index(const ijb_engine *engine, const char *name);

/* y[b] = W x[b] for `batch` activations (x_dev [batch][cols] fp32, y_dev
 * [batch][rows] fp32), with the quantised activation path the engine was
 * created with.  Drop-in for FastGPU::matvec (inferencer.cu:1156-1171; batch
 * > 1 replaces FastRunner::batch_matvec, :1265-1278). */
int ijb_matvec(ijb_engine *engine, int tensor_index, const float *x_dev, float *y_dev, int cols, int rows,
               int batch, void *stream);

/* One decode token of the single-sequence runner (sequence 0): embeds
 * `token` at position `pos`, runs every layer, and when need_logits is set,
 * the final norm, lm_head and greedy argmax; *next_token receives the argmax
 * (or -1 without logits).  Requires 0 <= pos < context, 0 <= token < vocab,
 * and pos <= current length of sequence 0.  Drop-in for FastRunner::forward
 * (inferencer.cu:1424-1531). */
int ijb_forward(ijb_engine *engine, int token, int pos, int need_logits, int *next_token);

/* Prefill of the single-sequence runner from position 0: the tokens run
 * through packed steps of up to max_batch tokens; *next_token is the argmax
 * after the last one.  Drop-in for FastRunner::prefill (inferencer.cu:1279-1423). */
int ijb_prefill(ijb_engine *engine, const int *tokens, int n, int *next_token);

/* FastRunner::forward with its debug traces (inferencer.cu:1424-1426): as
 * ijb_forward; when non-NULL, layer_trace [layers][dim] receives the residual
 * stream after every layer, and quant_trace [layers][3*dim + hidden] the int8
 * activations the reference's INT8 path quantises in each layer (the
 * attention input, the attention output, the feed-forward input, the
 * down-projection input), computed with the reference's RMSNorm and per-32
 * quantiser.  Slower than ijb_forward (a separate step graph with trace
 * copies). */
int ijb_forward_traced(ijb_engine *engine, int token, int pos, int need_logits, int *next_token, float *layer_trace,
                       int8_t *quant_trace);

/* FastRunner::prefill with its debug traces (inferencer.cu:1279-1283): as
 * ijb_prefill; all_layer_trace [n][layers][dim] receives every token's
 * residual after every layer, first_quant_trace / last_quant_trace
 * [layers][3*dim + hidden] the first and last token's quantised activations.
 * Any trace pointer may be NULL. */
int ijb_prefill_traced(ijb_engine *engine, const int *tokens, int n, int *next_token, float *all_layer_trace,
                       int8_t *first_quant_trace, int8_t *last_quant_trace);

/* Entries in the last step run (1 after ijb_forward; the last chunk's size
 * after a prefill): row (size - 1) of ijb_logits_dev / ijb_residual_dev is the
 * last token's, which FastGPU::logits / FastGPU::x hold in the reference. */
int ijb_last_step_size(const ijb_engine *engine);

/* Forgets sequence 0's cached positions (FastRunner::reset, inferencer.cu:1264). */
int ijb_reset(ijb_engine *engine);

/* Device pointers to the last step's fp32 logits [n][vocab] and residual
 * stream [n][dim] (FastGPU::logits and FastGPU::x, inferencer.cu:1101-1103). */
const float *ijb_logits_dev(const ijb_engine *engine);
const float *ijb_residual_dev(const ijb_engine *engine);

/* Ragged continuous batching (new; the reference runs one sequence). */
int ijb_seq_open(ijb_engine *engine, int *seq_id);
int ijb_seq_close(ijb_engine *engine, int seq_id);
int ijb_seq_length(const ijb_engine *engine, int seq_id);

/* One packed step over n entries: entry i appends tokens[i] to sequence
 * seq_ids[i] at that sequence's next position.  Entries may repeat a
 * sequence with consecutive tokens (chunked prefill) or name distinct
 * sequences (decode).  With next_tokens non-NULL, each entry's greedy argmax is
 * copied to the host; the call returns after the step completed. */
int ijb_decode_step(ijb_engine *engine, int n, const int *seq_ids, const int *tokens, int *next_tokens);

/* Greedy generation of one sequence with the token feedback on the device:
 * the reference's decode loop (main, inferencer.cu:1870-1883) from `next`
 * (first_token, the prefill's argmax) at the sequence's next position.  A
 * token equal to one of stop_ids (n_stop <= 16) ends the loop and is not
 * emitted; otherwise it is emitted, and the loop ends after max_tokens
 * emitted tokens or when the position to feed it at reaches the context.
 * out_tokens (room for max_tokens) receives the emitted tokens, *n_out their
 * count; the sequence's cached length grows by the positions fed.  Each step
 * is the batch-1 step graph followed by a one-thread kernel that turns its
 * argmax into the next step's token, position and KV slot, so steps are
 * queued without a host round trip (the host checks the state once per 8
 * steps; steps queued past the end recompute the last position). */
int ijb_generate(ijb_engine *engine, int seq_id, int first_token, int max_tokens, const int *stop_ids, int n_stop,
                 int *out_tokens, int *n_out);

/* Prefill one sequence with n tokens (chunks of max_batch); *next_token is
 * the argmax after the last token. */
int ijb_seq_prefill(ijb_engine *engine, int seq_id, const int *tokens, int n, int *next_token);

/* ---- standalone kernels (no engine) ---- */

/* Greedy argmax with the reference's tie rule (argmax_blocks_cuda +
 * argmax_final_cuda, inferencer.cu:1063-1099); n <= 131072. */
int ijb_argmax(const float *values_dev, int n, int *index_dev, void *stream);

/* Dequantise n_blocks super-blocks to fp32, bit-identical to q4_value /
 * q6_value (inferencer.cu:454-487).  `blocks_dev` is GGUF layout. */
int ijb_dequant(int type, const void *blocks_dev, long n_blocks, float *out_dev, void *stream);

/* Bytes per row of the repacked Q6_K plane layout for `cols` columns
 * (ql | qh | scales | d, padded to 16 bytes). */
long ijb_q6k_planar_row_bytes(int cols);

/* GGUF Q6_K rows -> plane layout (the load-time repack GGUF::upload feeds). */
int ijb_repack_q6k(const void *src_dev, void *dst_dev, int rows, int cols, void *stream);

/* Standalone GEMV over one matrix: w_dev is GGUF layout for Q4_K, plane
 * layout (ijb_repack_q6k) for Q6_K; bit 0 of use_dp4a selects the INT8
 * activation path (quantize_x32_cuda + gemv_q4_dp4a / gemv_q6_dp4a) or the
 * FP32 path (gemv_quant<T>), inferencer.cu:544-674.  With IJB_GEMV_PDL also
 * set, the kernel is launched with programmatic dependent launch: in a stream
 * or graph of consecutive GEMVs each one's weight prefetch overlaps the tail of
 * the one before (its activation is read only after that one completed).
 * batch <= 8. */
#define IJB_GEMV_PDL 2
int ijb_gemv(int type, const void *w_dev, const float *x_dev, float *y_dev, int cols, int rows, int batch,
             int use_dp4a, void *stream);

/* The same argmax as ijb_argmax, for callers that cannot allocate device
 * memory: code running while a CUDA graph is captured (allocation is not
 * allowed there), host loops that cannot take the device synchronisation an
 * allocation may cause, frameworks that own all device memory through their
 * own allocator.  ijb_argmax allocates an 8-byte scratch key on its first
 * call on a device; this entry point allocates nothing.  It computes one
 * winner per 256 values into a fixed 512-slot array in device memory that the
 * library holds on every GPU that loads it (4 KB), then the winner of those:
 * n must be 1..131072 (512 x 256), larger n is rejected with IJB_ERR_INVALID.
 * Its first call on a device looks up that array's device address (no
 * allocation); make that first call before any stream capture.  Every call
 * writes the slots it reads, so nothing carries over between calls, but all
 * calls share the one array: calls that overlap on the GPU (other streams,
 * other host threads) race and must be serialised by the caller.  Asynchronous
 * on `stream`.  No counterpart in the reference. */
int ijb_argmax_noalloc(const float *values_dev, int n, int *index_dev, void *stream);

/* Exercises the engine's failure path without a fault: launches, on the
 * engine's stream, one kernel whose bounded wait on a barrier that nothing
 * signals gives up after limit_ns (1 us .. 100 ms), records the timeout in
 * the engine's device status word and returns.  The call then fails the way a
 * step whose kernel gave up a wait fails: IJB_ERR_DEVICE, with the status word
 * cleared and the engine usable for the next step.  Every device-side wait of
 * the library is bounded the same way (2 s in the step kernels).  No
 * counterpart in the reference, whose device work has no waits of its own
 * (its errors surface through cuda_check, inferencer.cu:126-128). */
int ijb_probe_wait_timeout(ijb_engine *engine, uint64_t limit_ns);

/* Timing helper: replays layer 0's four projection launches exactly as a
 * packed step of n tokens issues them (QKV with RoPE and the K/V cache write,
 * O with the residual add, gate/up with SiLU, down with the residual add, each
 * with its activation preparation; no attention), `reps` times in one CUDA
 * graph, and writes the mean device time of one layer's chain in
 * milliseconds (CUDA events on the engine's stream).  Sequence 0 must be
 * empty; its pages take the timed K/V writes and are released afterwards.
 * The engine's activations are overwritten.  No counterpart in the reference
 * (a measurement aid for the dominant kernel). */
int ijb_time_layer_projections(ijb_engine *engine, int n, int reps, float *ms_per_layer);

/* Timing helper: layer 0's decode attention for one query token of each of
 * the n listed open sequences at its newest position (so each launch reads
 * every cached K/V row of those sequences, as the next decode step would),
 * launched as a packed step of n tokens launches it (streaming kernel and
 * merge, or the split kernel), `reps` times in one CUDA graph.  Writes the
 * mean device time of one layer's attention in milliseconds (CUDA events on
 * the engine's stream) and the K/V bytes one launch reads.  The engine's
 * attention output is overwritten; the cache is only read.  No counterpart
 * in the reference (a measurement aid; the reference's decode attention is
 * attention_cuda, inferencer.cu:981-1009). */
int ijb_time_layer_attention(ijb_engine *engine, int n, const int *seq_ids, int reps, float *ms_per_layer,
                             long long *kv_bytes);

/* ---- one quantised matrix on the tensor cores, outside an engine ----
 * For callers that hold one matrix or a slice of one, e.g. each rank's
 * row slice of a row-split lm_head (the reference's lm_head GEMV,
 * inferencer.cu:1519-1526, with its argmax, :1063-1099). */
typedef struct ijb_weight ijb_weight;

/* Prepares rows x cols of GGUF-layout Q4_K / Q6_K blocks at w_dev (16-byte
 * aligned, on `device`) for ijb_weight_matmul: the same chunked copy and
 * power-of-two scale ijb_create makes for packed steps (the source may be
 * freed afterwards). */
int ijb_weight_create(int type, const void *w_dev, int rows, int cols, int device, ijb_weight **out);
void ijb_weight_destroy(ijb_weight *weight);

/* y[t][r] = W norm(x[t]) for n tokens (x_dev [n][cols] fp32; y_dev rows
 * t*y_stride .. +rows), on the INT8 (use_dp4a, the reference's per-32
 * activation quantisation) or FP32 activation path; with norm_w_dev non-NULL
 * an RMSNorm with those weights and eps comes first.  With keys_dev non-NULL
 * it also receives, per token, the packed argmax key of (logit, key_offset +
 * row) over this matrix's rows with the reference's tie rule: keys of several
 * row slices combine by taking their maximum, and ijb_keys_to_tokens turns a
 * key into the token index.  Asynchronous on `stream`; calls on one weight
 * must not overlap (they share its activation buffer). */
int ijb_weight_matmul(ijb_weight *weight, const float *x_dev, int n, const float *norm_w_dev, float eps, int use_dp4a,
                      float *y_dev, long y_stride, int key_offset, unsigned long long *keys_dev, void *stream);

/* IJB_ERR_DEVICE (and clears it) if a kernel of this weight reported a
 * device error (a bounded wait expired); call after synchronising. */
int ijb_weight_status(ijb_weight *weight);

/* Packed argmax keys -> token indices (n keys, device memory). */
int ijb_keys_to_tokens(const unsigned long long *keys_dev, int n, int *tokens_dev, void *stream);

/* Number of kernels the library launched since load (for launch accounting). */
uint64_t ijb_kernel_launches(void);

/* Device time (CUDA events on the engine's stream) of the last step run by
 * ijb_forward / ijb_prefill / ijb_decode_step, in milliseconds: the
 * counterpart of FastGPU's event timer (start_timer/stop_timer, inferencer.cu:1172-1179). */
float ijb_last_step_ms(const ijb_engine *engine);

/* ---- tokenizer (host only; no GPU involved) ----
 * Llama-3 byte-level BPE over a GGUF vocabulary, replacing the reference's
 * Tokenizer (inferencer.cu:361-451) with the same results: its pre-tokenizer
 * pattern (followed by a scanner over PCRE2's own character classes, or
 * matched by PCRE2 itself for text that is not valid UTF-8; the runtime
 * library libpcre2-8.so.0 is loaded on first use), its byte-symbol map,
 * merges applied lowest rank first and leftmost first, and its error
 * messages.  Thread-safe after creation; each thread keeps a piece cache of
 * up to 65,536 pieces for the tokenizer it used last. */
typedef struct ijb_tokenizer ijb_tokenizer;

/* Builds a tokenizer from tokenizer.ggml.tokens (exactly 128256 strings, as
 * the reference requires: "Expected Llama 3 tokenizer") and
 * tokenizer.ggml.merges ("left right" strings, rank = index); on failure the
 * message is available from ijb_tokenizer_last_error(NULL) in this thread.
 * Replaces Tokenizer::Tokenizer (inferencer.cu:368-390). */
int ijb_tokenizer_create(const char *const *tokens, int n_tokens, const char *const *merges, int n_merges,
                         ijb_tokenizer **out);
void ijb_tokenizer_destroy(ijb_tokenizer *tokenizer);
/* Message of the last failed call on `tokenizer` (NULL: of the last failed
 * ijb_tokenizer_create in this thread).  Never NULL. */
const char *ijb_tokenizer_last_error(const ijb_tokenizer *tokenizer);
/* Token ids of len bytes of text (Tokenizer::encode, :415-431): writes the
 * first min(cap, *n) ids to ids and the full count to *n (call again with a
 * larger buffer when *n > cap). */
int ijb_tokenizer_encode(ijb_tokenizer *tokenizer, const char *text, long len, int *ids, long cap, long *n);
/* ijb_tokenizer_encode of n_texts texts on `threads` host threads (0: all the
 * hardware has): the ids of text i go to ids[offsets[i] .. offsets[i + 1]),
 * offsets having n_texts + 1 entries.  When the ids exceed cap, offsets is
 * still filled (offsets[n_texts] = the count needed) and the call returns
 * IJB_ERR_CAPACITY without writing ids. */
int ijb_tokenizer_encode_batch(ijb_tokenizer *tokenizer, const char *const *texts, const long *lens, int n_texts,
                               int *ids, long cap, long *offsets, int threads);
/* The bytes token id stands for (Tokenizer::decode, :432-445): writes the
 * first min(cap, *len) bytes and the full length to *len. */
int ijb_tokenizer_decode(ijb_tokenizer *tokenizer, int id, char *bytes, int cap, int *len);
/* Id of a token by its exact string, e.g. "<|eot_id|>" (Tokenizer::special, :446-450). */
int ijb_tokenizer_special(ijb_tokenizer *tokenizer, const char *name, int *id);
/* The chat layout of one user turn (chat_prompt, inferencer.cu:1534-1551):
 * <|begin_of_text|> <|start_header_id|> "user" <|end_header_id|> "\n\n" + prompt
 * <|eot_id|> <|start_header_id|> "assistant" <|end_header_id|> "\n\n"; ids and
 * *n as in ijb_tokenizer_encode. */
int ijb_tokenizer_chat_prompt(ijb_tokenizer *tokenizer, const char *prompt, long len, int *ids, long cap, long *n);

#ifdef __cplusplus
}
#endif

#endif /* IJB200_H */
