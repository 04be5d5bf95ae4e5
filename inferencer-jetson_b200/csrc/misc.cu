// Small kernels around the GEMVs: Q6_K load-time repack, embedding lookup,
// bit-exact dequantisation, the stand-alone argmax and the argmax-key decode.
#include <mutex>
#include <string>

#include "../../include/ijb200.h"
#include "common.cuh"
#include "gemv.cuh"
#include "misc.cuh"

namespace ijb {

long q6_planar_row_bytes(int cols) { return q6_unit_row_bytes(cols); }

// GGUF Q6_K row (nb blocks of ql[128] qh[64] scales[16] d[2]) -> the unit
// layout described in gemv.cuh.  Bytes are only moved.
__global__ void ijb_repack_q6_kernel(const uint8_t *src, uint8_t *dst, int rows, int nb, long dst_row_bytes) {
    const long row = blockIdx.x;
    if (row >= rows) return;
    const uint8_t *s = src + row * nb * 210;
    uint8_t *d = dst + row * dst_row_bytes;
    for (long i = threadIdx.x; i < dst_row_bytes; i += blockDim.x) d[i] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < nb * 210; i += blockDim.x) {
        const int blk = i / 210, o = i % 210;
        const int u = blk / kUnitBlocks, lb = blk % kUnitBlocks;
        const int n = min(kUnitBlocks, nb - u * kUnitBlocks);
        const long body = static_cast<long>(u) * q6_unit_bytes(kUnitBlocks) + lb * 208;
        long to;
        if (o < 128) {  // ql[g*64 + half*32 + 16h + j]
            const int g = o / 64, half = (o % 64) / 32, h = (o % 32) / 16;
            to = body + half * 64 + (2 * g + h) * 16 + (o % 16);
        } else if (o < 192) {  // qh[g*32 + 16h + j]
            const int q = o - 128, g = q / 32, h = (q % 32) / 16;
            to = body + 128 + (2 * g + h) * 16 + (q % 16);
        } else if (o < 208) {  // scales[g*8 + 2*part + h]
            const int q = o - 192, g = q / 8, part = (q % 8) / 2, h = q % 2;
            to = body + 192 + (2 * g + h) * 4 + part;
        } else {  // d after the unit's bodies
            to = static_cast<long>(u) * q6_unit_bytes(kUnitBlocks) + n * 208 + lb * 2 + (o - 208);
        }
        d[to] = s[i];
    }
}

// Weight i of block blk of a unit-layout Q6_K row, exactly q6_value
// (inferencer.cu:473-487): d * scale * q with both products exact in fp32.
__device__ __forceinline__ float q6_planar_value(const uint8_t *row, int nb, int blk, int i) {
    const int u = blk / kUnitBlocks, lb = blk % kUnitBlocks;
    const int n = min(kUnitBlocks, nb - u * kUnitBlocks);
    const uint8_t *unit = row + static_cast<long>(u) * q6_unit_bytes(kUnitBlocks);
    const uint8_t *body = unit + lb * 208;
    const int g = i / 128, p = i % 128, part = p / 32, l = p % 32, h = l / 16, j = l % 16;
    const int lane = 2 * g + h;
    int low = body[(part & 1) * 64 + lane * 16 + j];
    low = part < 2 ? (low & 15) : (low >> 4);
    const int high = (body[128 + lane * 16 + j] >> (part * 2)) & 3;
    const int q = (low | (high << 4)) - 32;
    const int sc = static_cast<int8_t>(body[192 + lane * 4 + part]);
    const float d = half_bits_to_float(*reinterpret_cast<const uint16_t *>(unit + n * 208 + lb * 2));
    return __fmul_rn(__fmul_rn(d, static_cast<float>(sc)), static_cast<float>(q));
}

// embedding_cuda / embedding_batch_cuda (inferencer.cu:806-819) over the
// planar token_embd; also clears the per-token argmax keys of the step.
__global__ void ijb_embed_kernel(const uint8_t *emb, long row_bytes, int dim, const int *tokens, int n, float *x,
                             long x_stride, unsigned long long *keys) {
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.y;
    if (b >= n) return;
    const int tok = tokens[b];
    const int nb = dim / 256;
    const uint8_t *row = emb + static_cast<long>(tok) * row_bytes;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x)
        x[b * x_stride + i] = q6_planar_value(row, nb, i / 256, i % 256);
    if (keys && blockIdx.x == 0 && threadIdx.x == 0) keys[b] = 0ull;
}

// q4_value (inferencer.cu:454-471): d*sc*q - dmin*m.  d*sc and (d*sc)*q are
// exact in fp32 (at most 11+6+4 significant bits), so the only rounding is
// the final subtraction, with or without a fused multiply-add.
__global__ void ijb_dequant_kernel(int type, const uint8_t *blocks, long nblocks, float *out) {
    const long idx = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x;
    if (idx >= nblocks * 256) return;
    const long blk = idx / 256;
    const int i = static_cast<int>(idx % 256);
    if (type == kQ4K) {
        const uint8_t *b = blocks + blk * 144;
        const float d = half_bits_to_float(*reinterpret_cast<const uint16_t *>(b));
        const float dmin = half_bits_to_float(*reinterpret_cast<const uint16_t *>(b + 2));
        const uint8_t *s = b + 4, *qs = b + 16;
        const int sub = i / 32, qi = (i / 64) * 32 + (i % 32);
        const int q = (i % 64) < 32 ? (qs[qi] & 15) : (qs[qi] >> 4);
        int sc, m;
        if (sub < 4) {
            sc = s[sub] & 63;
            m = s[sub + 4] & 63;
        } else {
            sc = (s[sub + 4] & 15) | ((s[sub - 4] >> 6) << 4);
            m = (s[sub + 4] >> 4) | ((s[sub] >> 6) << 4);
        }
        out[idx] = __fsub_rn(__fmul_rn(__fmul_rn(d, static_cast<float>(sc)), static_cast<float>(q)),
                             __fmul_rn(dmin, static_cast<float>(m)));
    } else {
        const uint8_t *b = blocks + blk * 210;
        const int group = i / 128, p = i % 128, lane = p % 32, part = p / 32;
        int low = b[group * 64 + (part % 2) * 32 + lane];
        low = part < 2 ? (low & 15) : (low >> 4);
        const int high = (b[128 + group * 32 + lane] >> (part * 2)) & 3;
        const int q = (low | (high << 4)) - 32;
        const int sc = static_cast<int8_t>(b[192 + group * 8 + part * 2 + lane / 16]);
        const float d = half_bits_to_float(*reinterpret_cast<const uint16_t *>(b + 208));
        out[idx] = __fmul_rn(__fmul_rn(d, static_cast<float>(sc)), static_cast<float>(q));
    }
}

// Stand-alone argmax with the reference's tie rule (see argmax_key): one
// pass of atomicMax over packed keys, then a one-thread decode.
__global__ void ijb_argmax_keys_kernel(const float *v, int n, unsigned long long *key) {
    unsigned long long best = 0ull;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const unsigned long long k = argmax_key(v[i], i);
        best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
    }
    if ((threadIdx.x & 31) == 0 && best) atomicMax(key, best);
}

// keys[b] -> tokens[b].  A key is zero only when no value reached it (no
// token was scanned); such keys decode to -1.  NaN values get keys above zero
// but below every non-NaN value, so NaN never wins against a number, and an
// all-NaN row decodes to index 0 (the smallest rank), which is also what the
// reference's trees return for it.
__global__ void ijb_keys_to_tokens_kernel(const unsigned long long *keys, int n, int *tokens) {
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < n) tokens[b] = keys[b] ? argmax_key_index(keys[b]) : -1;
}

static cudaLaunchConfig_t pdl_config(dim3 grid, dim3 block, cudaStream_t stream, bool pdl,
                                     cudaLaunchAttribute *attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = stream;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cfg;
}

cudaError_t repack_q6_launch(const void *src, void *dst, int rows, int cols, cudaStream_t stream) {
    if (rows <= 0) return cudaSuccess;
    ijb_repack_q6_kernel<<<rows, 256, 0, stream>>>(static_cast<const uint8_t *>(src), static_cast<uint8_t *>(dst), rows,
                                               cols / 256, q6_planar_row_bytes(cols));
    return cudaGetLastError();
}

cudaError_t embed_launch(const uint8_t *emb, long row_bytes, int dim, const int *tokens, int n, float *x,
                         long x_stride, unsigned long long *keys, cudaStream_t stream, bool pdl) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_config(dim3((dim + 255) / 256, n), dim3(256), stream, pdl, attr);
    return cudaLaunchKernelEx(&cfg, ijb_embed_kernel, emb, row_bytes, dim, tokens, n, x, x_stride, keys);
}

cudaError_t dequant_launch(int type, const void *blocks, long nblocks, float *out, cudaStream_t stream) {
    const long total = nblocks * 256;
    if (total <= 0) return cudaSuccess;
    ijb_dequant_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, stream>>>(
        type, static_cast<const uint8_t *>(blocks), nblocks, out);
    return cudaGetLastError();
}

cudaError_t argmax_launch(const float *v, int n, unsigned long long *key_scratch, int *index, cudaStream_t stream) {
    cudaError_t e = cudaMemsetAsync(key_scratch, 0, sizeof(unsigned long long), stream);
    if (e != cudaSuccess) return e;
    int blocks = (n + 255) / 256;
    if (blocks > 1024) blocks = 1024;
    ijb_argmax_keys_kernel<<<blocks, 256, 0, stream>>>(v, n, key_scratch);
    ijb_keys_to_tokens_kernel<<<1, 32, 0, stream>>>(key_scratch, 1, index);
    return cudaGetLastError();
}

// Debug trace of an activation the INT8 path quantises (what the reference
// records in FastRunner::forward's quant_trace, inferencer.cu:1447-1452,
// :1471-1476, :1490-1495, :1503-1508): per token (one CTA of 256 threads) an
// optional RMSNorm with rmsnorm_cuda's 256 strided partial sums and tree
// (:821-834), then quantize_x32_cuda's per-32 int8 codes (:544-556).
__global__ void __launch_bounds__(256) ijb_trace_quant_kernel(const float *x, long x_stride, const float *norm_w,
                                                              float eps, int cols, int8_t *out, long out_stride) {
    __shared__ float partial[256];
    const float *xr = x + blockIdx.x * x_stride;
    int8_t *o = out + blockIdx.x * out_stride;
    float r = 1.f;
    if (norm_w) {
        float sum = 0.f;
        for (int i = threadIdx.x; i < cols; i += 256) sum = fmaf(xr[i], xr[i], sum);
        partial[threadIdx.x] = sum;
        __syncthreads();
        for (int stride = 128; stride > 0; stride /= 2) {
            if (static_cast<int>(threadIdx.x) < stride) partial[threadIdx.x] += partial[threadIdx.x + stride];
            __syncthreads();
        }
        r = rsqrtf(partial[0] / cols + eps);
    }
    const int lane = threadIdx.x & 31;
    for (int g = threadIdx.x >> 5; g < cols / 32; g += 8) {
        const int i = g * 32 + lane;
        float v = xr[i];
        if (norm_w) v = __fmul_rn(__fmul_rn(v, r), norm_w[i]);
        float amax = fabsf(v);
        for (int o2 = 16; o2 > 0; o2 >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o2));
        const float scale = amax > 0.f ? amax / 127.f : 1.f;
        o[i] = static_cast<int8_t>(max(-127, min(127, __float2int_rn(v / scale))));
    }
}

cudaError_t trace_quant_launch(const float *x, long x_stride, const float *norm_w, float eps, int cols, int n,
                               int8_t *out, long out_stride, cudaStream_t stream) {
    ijb_trace_quant_kernel<<<n, 256, 0, stream>>>(x, x_stride, norm_w, eps, cols, out, out_stride);
    return cudaGetLastError();
}

// Failure-path probe: one thread waits on a shared-memory barrier that
// nothing signals, with the given limit, so the wait expires, records
// kDevErrWaitTimeout in *status and returns; nothing faults or hangs.
__global__ void ijb_wait_probe_kernel(uint32_t *status, uint64_t limit_ns) {
    __shared__ uint64_t bar;
    __shared__ uint32_t abort_flag;
    if (threadIdx.x == 0) {
        abort_flag = 0u;
        mbar_init(&bar, 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) mbar_wait_bounded(&bar, 0, status, &abort_flag, limit_ns);
}

cudaError_t wait_probe_launch(uint32_t *status, uint64_t limit_ns, cudaStream_t stream) {
    ijb_wait_probe_kernel<<<1, 32, 0, stream>>>(status, limit_ns);
    return cudaGetLastError();
}

// ---------------------------------------------------- device-side greedy loop --

// After one batch-1 step of ijb_generate: the step's next token (next[0]) is
// the reference generate loop's `next` (inferencer.cu:1870-1883): a stop id
// ends the loop unemitted; otherwise it is emitted, and the loop ends after
// max_tokens emitted tokens or when the position to feed it at reaches the
// context; otherwise it becomes the next step's input at the next position,
// whose KV slot comes from the sequence's page table (pages allocated by the
// host beforehand).  Once done, the step's inputs stay as they are, so any
// step already queued recomputes the last position: the same K/V, written to
// the same slot.
__global__ void ijb_gen_advance_kernel(GenState *g, const int *next, int *meta, int max_batch, const int *page_table,
                                       const int *stop_ids, int *out) {
    if (threadIdx.x != 0 || g->done) return;
    const int t = next[0];
    ++g->processed;  // the token in meta was fed at its position
    for (int i = 0; i < g->n_stop; ++i)
        if (t == stop_ids[i]) {
            g->done = 1;
            return;
        }
    out[g->count++] = t;
    const int pos = meta[2 * max_batch] + 1;
    if (g->count >= g->max_tokens || pos >= g->context) {
        g->done = 1;
        return;
    }
    const int ps = g->page_size;
    meta[0] = t;
    meta[2 * max_batch] = pos;
    meta[3 * max_batch] = page_table[static_cast<long>(g->seq) * g->max_pages_per_seq + pos / ps] * ps + pos % ps;
}

cudaError_t gen_advance_launch(GenState *g, const int *next, int *meta, int max_batch, const int *page_table,
                               const int *stop_ids, int *out, cudaStream_t stream) {
    ijb_gen_advance_kernel<<<1, 32, 0, stream>>>(g, next, meta, max_batch, page_table, stop_ids, out);
    return cudaGetLastError();
}

cudaError_t keys_to_tokens_launch(const unsigned long long *keys, int n, int *tokens, cudaStream_t stream,
                                  bool pdl) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_config(dim3((n + 127) / 128), dim3(128), stream, pdl, attr);
    return cudaLaunchKernelEx(&cfg, ijb_keys_to_tokens_kernel, keys, n, tokens);
}

// ------------------------------------------- argmax without allocation --
//
// Some callers cannot call cudaMalloc: code that runs while a CUDA graph is
// being captured (allocation is not allowed inside a capture), host loops
// that cannot afford the device synchronisation an allocation may cause, and
// frameworks whose device memory is owned by their own allocator.
// ijb_argmax allocates its 8-byte scratch key the first time it runs on a
// device; ijb_argmax_noalloc below allocates nothing.  It keeps the
// reference's two-pass structure (argmax_blocks_cuda, argmax_final_cuda,
// inferencer.cu:1063-1099): one winner per 256 values, then one over the
// winners, with the winners in a fixed array in device memory that the
// library holds on every GPU that loads it.

constexpr int kNoAllocArgmaxSlots = 512;  // 512 winners x 256 values = the reference's 131072 limit
static __device__ __align__(256) unsigned long long g_argmax_slots[kNoAllocArgmaxSlots];

// Pass 1: CTA b writes the best packed key of values [256b, 256b + 256).
__global__ void ijb_argmax_slots_kernel(const float *v, int n, unsigned long long *slots) {
    __shared__ unsigned long long warp_best[8];
    const int i = blockIdx.x * 256 + threadIdx.x;
    unsigned long long best = i < n ? argmax_key(v[i], i) : 0ull;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
    }
    if ((threadIdx.x & 31) == 0) warp_best[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long b = 0ull;
        for (int w = 0; w < 8; ++w) b = warp_best[w] > b ? warp_best[w] : b;
        slots[blockIdx.x] = b;
    }
}

// Pass 2: one CTA reduces the winners and writes the index.  NaN values lose
// to every number; an all-NaN input gives index 0, as the reference's trees
// do (every key is non-zero for n >= 1, so the -1 branch is never taken).
__global__ void ijb_argmax_slots_final_kernel(const unsigned long long *slots, int nslots, int *index) {
    __shared__ unsigned long long warp_best[kNoAllocArgmaxSlots / 32];
    unsigned long long best = static_cast<int>(threadIdx.x) < nslots ? slots[threadIdx.x] : 0ull;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
    }
    if ((threadIdx.x & 31) == 0) warp_best[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long b = 0ull;
        for (int w = 0; w < kNoAllocArgmaxSlots / 32; ++w) b = warp_best[w] > b ? warp_best[w] : b;
        *index = b ? argmax_key_index(b) : -1;
    }
}

// Device address of g_argmax_slots on each device, looked up once per device
// with that device current (host code must not use the symbol's name as a
// device pointer).
static unsigned long long *g_slots_addr[64] = {nullptr};
static std::mutex g_slots_mu;

static cudaError_t slots_address(unsigned long long **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_slots_mu);
    if (!g_slots_addr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_argmax_slots);
        if (e != cudaSuccess) return e;
        g_slots_addr[dev] = static_cast<unsigned long long *>(p);
    }
    *out = g_slots_addr[dev];
    return cudaSuccess;
}

}  // namespace ijb

extern "C" int ijb_argmax_noalloc(const float *values_dev, int n, int *index_dev, void *stream) {
    using namespace ijb;
    if (!values_dev || !index_dev) {
        set_thread_error("ijb_argmax_noalloc: null pointer");
        return IJB_ERR_INVALID;
    }
    if (n < 1 || n > kNoAllocArgmaxSlots * 256) {
        set_thread_error("ijb_argmax_noalloc: n = " + std::to_string(n) + " is outside 1.." +
                         std::to_string(kNoAllocArgmaxSlots * 256) + " (the static scratch holds " +
                         std::to_string(kNoAllocArgmaxSlots) + " partial winners of 256 values)");
        return IJB_ERR_INVALID;
    }
    unsigned long long *slots = nullptr;
    cudaError_t e = slots_address(&slots);
    if (e == cudaSuccess) {
        const int nslots = (n + 255) / 256;
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        ijb_argmax_slots_kernel<<<nslots, 256, 0, s>>>(values_dev, n, slots);
        ijb_argmax_slots_final_kernel<<<1, kNoAllocArgmaxSlots, 0, s>>>(slots, nslots, index_dev);
        e = cudaGetLastError();
        count_launches(2);
    }
    if (e != cudaSuccess) {
        set_thread_error(std::string("ijb_argmax_noalloc: ") + cudaGetErrorString(e));
        return IJB_ERR_CUDA;
    }
    return IJB_OK;
}
