// Host-visible parameters of the paged decode-attention launch.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ijb {

struct AttnParams {
    // fp16 cache with head_dim 64 or 128: 3-D TMA map over this layer's pool, box =
    // one (page, kv head) run of page_size rows, 128-byte swizzled (see
    // attention_make_kv_map); the tensor-core kernel is used when has_map
    CUtensorMap kv_map;
    int has_map;
    const float *q;        // [batch][q_stride], RoPE already applied
    long q_stride;
    float *out;            // [batch][out_stride]
    long out_stride;
    const void *k_cache;   // this layer's pool base (K part of page 0)
    const void *v_cache;   // this layer's pool base (V part of page 0)
    int kv_f32;            // cache elements are fp32 (else fp16)
    long page_stride;      // elements per page
    int page_size;
    const int *page_table; // [max_seqs][max_pages_per_seq]
    int max_pages_per_seq;
    const int *tok_seq;    // [batch]
    const int *tok_pos;    // [batch]: attends to positions 0..pos
    int batch, heads, kv_heads, head_dim;
    float scale;           // 1/sqrt(head_dim)
    int split_len;         // positions per split of the split kernel (attention_split_len_min()..attention_split_len())
    int max_splits;        // partial records per (token, head); >= ceil(context / attention_item_len())
    float *partial;        // [batch][heads][max_splits][head_dim + 2] scratch
    int *counters;         // [batch][kv_heads], zero between launches
    int *work;             // [2] streaming kernel's item counter and finished-CTA counter, zero between launches
    int num_ctas;          // streaming kernel grid (one CTA per SM)
    // optional: the O projection's fp16 activation tile (mma_prep_launch layout),
    // built by the streaming path's finish kernel instead of a separate prep
    uint8_t *x16;
    float *x_inv;
    int n_pad;
    int use_dp4a;
    uint32_t *status;      // device error word (bounded waits)
};

cudaError_t attention_launch(const AttnParams &p, cudaStream_t stream, bool pdl);
int attention_kernels(const AttnParams &p);  // kernels attention_launch launches for p
// Encodes the TMA map of one layer's fp16 KV pool for the tensor-core
// kernel: dims {head_dim, 2 * kv_heads * page_size rows, num_pages}; returns
// 0 on success, -1 where the tensor-core kernel does not apply (head_dim not 64 or 128).
int attention_make_kv_map(CUtensorMap *map, const void *layer_base, int head_dim, int kv_heads, int page_size,
                          long page_stride_elems, long num_pages);
int attention_split_len();      // longest split of the split kernel (positions)
int attention_split_len_min();  // shortest split of the split kernel (positions)
int attention_item_len();   // positions per work item of the streaming kernel (finest split)
cudaError_t attention_prepare();  // once per device, before any launch

}  // namespace ijb
