// Launchers of the small kernels (misc.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace ijb {

long q6_planar_row_bytes(int cols);
cudaError_t repack_q6_launch(const void *src, void *dst, int rows, int cols, cudaStream_t stream);
cudaError_t embed_launch(const uint8_t *emb, long row_bytes, int dim, const int *tokens, int n, float *x,
                         long x_stride, unsigned long long *keys, cudaStream_t stream, bool pdl);
cudaError_t dequant_launch(int type, const void *blocks, long nblocks, float *out, cudaStream_t stream);
cudaError_t argmax_launch(const float *v, int n, unsigned long long *key_scratch, int *index, cudaStream_t stream);
// Error message of the last failed engine-less call on this thread
// (ijb_last_error(NULL)), and the library's kernel launch counter.
void set_thread_error(const std::string &msg);
void count_launches(uint64_t n);

// Debug trace: per token, optional RMSNorm then the per-32 int8 codes of x
// (row stride x_stride) into out (row stride out_stride).
cudaError_t trace_quant_launch(const float *x, long x_stride, const float *norm_w, float eps, int cols, int n,
                               int8_t *out, long out_stride, cudaStream_t stream);

// One kernel whose bounded wait (limit_ns) on a barrier that nothing signals
// expires and records kDevErrWaitTimeout in *status.
cudaError_t wait_probe_launch(uint32_t *status, uint64_t limit_ns, cudaStream_t stream);

cudaError_t keys_to_tokens_launch(const unsigned long long *keys, int n, int *tokens, cudaStream_t stream, bool pdl);

// State of the device-side greedy loop of one sequence (ijb_generate).
struct GenState {
    int done;       // the loop has ended (stop id, max_tokens or context)
    int count;      // tokens emitted so far
    int processed;  // positions fed to the model by the loop's steps
    int max_tokens, context, n_stop, seq, page_size, max_pages_per_seq;
};
// One thread: consumes the step's next token and sets up the next step's meta
// (token, position, KV slot) in place, or ends the loop.
cudaError_t gen_advance_launch(GenState *g, const int *next, int *meta, int max_batch, const int *page_table,
                               const int *stop_ids, int *out, cudaStream_t stream);

}  // namespace ijb
