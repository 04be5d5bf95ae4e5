// Host-visible description of one fused quantised-GEMV launch.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace ijb {

// What happens to each output row once its dot product is known.
enum Epilogue : int {
    kEpiStore = 0,         // out[b][row] = y
    kEpiAdd = 1,           // out[b][row] += y (residual add, add_cuda inferencer.cu:1043)
    kEpiRopeQ = 2,         // rotate the row pair, store (rope_cuda :906)
    kEpiRopeKCache = 3,    // rotate the row pair into the paged K cache (rope_cache_cuda :930)
    kEpiVCache = 4,        // store into the paged V cache (cache_cuda :919)
    kEpiSiluPair = 5,      // out[b][i] = silu(gate_i) * up_i (silu_cuda :1053)
    kEpiLogitsArgmax = 6,  // out[b][row] = y and a packed argmax key per token (:1063-1099)
};

constexpr int kMaxSegs = 4;
constexpr int kMaxBatch = 8;    // tokens per CUDA-core GEMV launch
constexpr int kMaxCols = 8192;  // activation length the prologue stages
constexpr int kUnitBlocks = 8;  // super-blocks per streamed unit (2048 weights)

// Q6_K "unit" layout (repack_q6 in misc.cu): each row is a sequence of units
// of up to 8 super-blocks.  A unit of n blocks holds n 208-byte block bodies,
// then the n fp16 block scales d, padded to 16 bytes (1680 bytes for n = 8).
// A block body is laid out for the 4 lanes that read it, lane j = 2*g + h
// (g: the block's 128-weight half, h: positions 16h..16h+15 of each 32-wide
// part):
//   [0, 64)    ql[g*64 + 16h .. +16]       per lane, 16 bytes each
//   [64, 128)  ql[g*64 + 32 + 16h .. +16]
//   [128, 192) qh[g*32 + 16h .. +16]
//   [192, 208) scales[g*8 + 2*part + h] for part 0..3 (4 bytes per lane)
// Bodies start on 16-byte boundaries (the tensor-core path's chunked copy takes
// them from here unchanged).  Only bytes move, so every weight is unchanged.
// Q4_K rows keep the GGUF layout (144-byte blocks are already 16-byte aligned).
__host__ __device__ inline int q6_unit_bytes(int nblocks) { return (nblocks * 210 + 15) / 16 * 16; }
__host__ __device__ inline long q6_unit_row_bytes(int cols) {
    const int nb = cols / 256, full = nb / kUnitBlocks, rest = nb % kUnitBlocks;
    return static_cast<long>(full) * q6_unit_bytes(kUnitBlocks) + (rest ? q6_unit_bytes(rest) : 0);
}

struct GemvSeg {
    const uint8_t *w0;  // rows [0, rows)
    const uint8_t *w1;  // second matrix of a gate/up pair (kEpiSiluPair) or null
    int type;           // 12 = Q4_K (GGUF layout), 14 = Q6_K (unit layout)
    int dp4a;           // 1: INT8 activations (DP4A path), 0: FP32 activations
    int rows;           // rows of w0 (and of w1)
    int row_bytes;      // bytes between consecutive rows
    int item_rows;      // rows per work item: 1, or 2 (RoPE pair / gate-up pair)
    int item0;          // first global item index of this segment
    int nitems;
    int epi;
    float *out;         // fp32 output base, token b at out + b * out_stride
    long out_stride;
    int row_offset;     // index of this segment's row 0 within its output vector
};

struct GemvParams {
    GemvSeg seg[kMaxSegs];
    int nseg;
    int total_items;
    int cols;  // K
    int batch; // tokens
    // prologue
    const float *x;  // [batch][x_stride]
    long x_stride;
    const float *norm_w;  // RMSNorm weight or null (no norm)
    float eps;
    int need_q4;  // build int8 activations in the Q4_K lane order
    int need_q6;  // build int8 activations in the Q6_K lane order
    int need_f;   // keep fp32 activations
    // epilogue extras
    const float *rope_cos;  // [ctx][half_head]
    const float *rope_sin;
    int half_head;
    const int *tok_pos;   // [batch] position of each token
    const int *tok_slot;  // [batch] KV slot = page * page_size + offset
    void *k_cache;        // this layer's K pool base
    void *v_cache;        // this layer's V pool base
    int kv_f32;           // cache elements are fp32 (else fp16)
    int kv_heads;
    int head_dim;
    int page_size;
    long page_stride;                 // elements per page (K and V of every kv head)
    unsigned long long *argmax_keys;  // [batch]
    uint32_t *status;                 // device error word
};

cudaError_t gemv_launch(const GemvParams &p, int num_sms, cudaStream_t stream, bool pdl);
int gemv_max_batch(int cols, int need_q4, int need_q6, int need_f);
cudaError_t gemv_prepare();

}  // namespace ijb
