// Host-visible description of the tensor-core (tcgen05) quantised GEMM used
// for packed steps of 3..128 tokens per launch.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "gemv.cuh"

namespace ijb {

constexpr int kMmaTileM = 128;    // weight rows per tile (TMEM lanes)
constexpr int kMmaMaxN = 64;      // tokens per launch (MMA N, padded to 16)
// Tokens per launch when every CTA of the launch holds one tile
// (mma_wide_ok): the activation stages double and the output tile reuses the
// raw weight stages, so each weight tile is dequantised once for 128 tokens.
constexpr int kMmaMaxNWide = 128;
// Engines with max_batch >= kMmaEngineMinBatch hold the tensor-core weight copy
// and run steps of kMmaMinBatch or more tokens on it (measured on B200, 1B decode
// steps: 2 tokens 1.01 ms on CUDA cores / 1.20 ms on the tensor cores; 3 tokens
// 1.37 / 1.23; 8 tokens 3.03 / 1.26; 12 tokens 4.38 / 1.27); smaller engines
// run every step on the CUDA-core GEMV.
constexpr int kMmaMinBatch = 3;
constexpr int kMmaEngineMinBatch = 16;

// Row groups of the tensor-core path's weight layout.
constexpr int kMmaRowGroup = 64;
// Bytes of one (row group, block column) chunk: Q4_K 64 GGUF blocks of 144
// bytes; Q6_K 64 block bodies of 208 bytes (unit layout order) then their 64
// fp16 d values.
constexpr int kMmaChunkQ4 = kMmaRowGroup * 144;
constexpr int kMmaChunkQ6Body = kMmaRowGroup * 208;
constexpr int kMmaChunkQ6 = kMmaChunkQ6Body + kMmaRowGroup * 2;

// One weight matrix as the tensor-core path reads it: chunks [row group][block
// column] of contiguous bytes (mma_tile_repack_launch), so that a stage of a
// 128-row tile is two or four plain bulk copies, and a power-of-two scale
// 2^scale_exp that keeps every dequantised weight in fp16's normal range.
struct MmaWeight {
    const uint8_t *chunks;
    int scale_exp;
    int nblocks;  // block columns (cols / 256)
};

// Bytes of the chunked copy of a rows x cols matrix (row groups rounded up to
// an even count, so that any 128-row tile reads inside the buffer).
long mma_tile_bytes(int type, int rows, int cols);
// Writes the chunked copy: src is the Q4_K GGUF layout or the Q6_K unit
// layout (row_bytes per row); rows past `rows` are zero.
cudaError_t mma_tile_repack_launch(int type, const uint8_t *src, long row_bytes, int rows, int cols, uint8_t *dst,
                                   cudaStream_t stream);

struct MmaSeg {
    int w0, w1;        // indexes into MmaParams::w (w1 < 0 unless a gate/up pair)
    int type;          // 12 / 14
    int rows;          // rows of w0 (and w1)
    int tile0, ntiles; // global tile range of this segment
    int epi;           // Epilogue (gemv.cuh)
    float *out;
    long out_stride;
    int row_offset;
    int key_offset;    // added to the row index of the argmax keys (a row slice of a larger matrix)
};

struct MmaParams {
    MmaWeight w[2 * kMaxSegs];
    MmaSeg seg[kMaxSegs];
    int nseg;
    int total_tiles;
    // split K: each tile's K range is cut into ksplit parts of bps block
    // columns, run by the ksplit CTAs of one cluster (mma_choose_split); the
    // parts exchange fp32 partial sums through the cluster's shared memory
    int ksplit;
    int bps;
    int bulk_out;  // finished token rows leave as bulk (TMA engine) copies, else as coalesced thread stores
    int cols;             // K
    int batch;            // tokens in this launch (<= kMmaMaxN, or kMmaMaxNWide when mma_wide_ok)
    int n_pad;            // MMA N: batch rounded up to 16
    const uint8_t *x16;   // prepared activation (mma_prep_launch), [cols/128][n_pad/8][16][8][16 B]
    const float *x_inv;   // [n_pad] 2^-kx of each token
    // fused epilogue parameters (same meaning as GemvParams)
    const float *rope_cos;
    const float *rope_sin;
    int half_head;
    const int *tok_pos;
    const int *tok_slot;
    void *k_cache;
    void *v_cache;
    int kv_f32;
    int kv_heads;
    int head_dim;
    int page_size;
    long page_stride;
    unsigned long long *argmax_keys;
    uint32_t *status;
};

// Builds the fp16 activation tile of `batch` tokens: optional RMSNorm, the
// reference's per-32 int8 quantisation then dequantisation (use_dp4a) or the
// plain fp32 values, times a per-token power of two, in the tensor cores'
// K-major layout.  Padding tokens up to n_pad are zero.
cudaError_t mma_prep_launch(const float *x, long x_stride, const float *norm_w, float eps, int cols, int batch,
                            int n_pad, int use_dp4a, uint8_t *x16, float *x_inv, cudaStream_t stream, bool pdl);
// The same for token n alone, by the 256 threads of the calling CTA (all of
// them call it; it synchronises the block).
__device__ void mma_prep_token(const float *x, long x_stride, const float *norm_w, float eps, int cols, int batch, int n,
                               int n_pad, int use_dp4a, uint8_t *x16, float *x_inv);

// Exponent e with max|w| * 2^e <= 2^15 for a quantised matrix (one reduction
// over its block scales); written to *out_exp on the device.
cudaError_t mma_scale_scan_launch(int type, const uint8_t *w, long nblocks_gguf_layout, int *out_max_bits,
                                  cudaStream_t stream);

// pdl: launch with programmatic stream serialisation; the kernel loads and
// dequantises weights before waiting for the previous kernel, and reads the
// activation and writes outputs only after the wait.
cudaError_t mma_gemm_launch(const MmaParams &p, cudaStream_t stream, bool pdl);
// Parts per tile (the cluster size) for a launch of `tiles` tiles of
// `nblocks` 256-wide block columns, from how many clusters of each size fit
// on the GPU at once (at most max_split parts; a split costs split_cost block
// columns of time); *bps receives block columns per part.  Needs
// mma_prepare() first.
int mma_choose_split(int tiles, int nblocks, int max_split, int split_cost, int *bps);
// Whether a launch of `tiles` tiles in clusters of `ksplit` parts gives every
// CTA a single tile (all clusters resident at once), which launches of more
// than kMmaMaxN tokens require.  Needs mma_prepare() first.
bool mma_wide_ok(int tiles, int ksplit);
// Sets the kernel's shared-memory limit and measures cluster occupancy for
// the current device.
cudaError_t mma_prepare();
int mma_smem_bytes();

}  // namespace ijb
