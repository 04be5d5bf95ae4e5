// GQA decode attention over the paged fp16 KV cache (split-KV, sm_100a).
//
// Replaces attention_cuda / attention_batch_cuda (inferencer.cu:982-1041): the
// reference runs one 128-thread CTA per query head and walks positions 0..pos
// serially with two block barriers per position over an fp32 [layer][ctx][kv]
// cache.  Here one CTA handles one (token, kv head, split of positions): the
// group's query heads share every K/V row it loads, lanes own positions while
// scoring and head-dim elements while accumulating V, and each split keeps an
// online-softmax state (max, sum, unnormalised output).  The last CTA of a
// (token, kv head) to finish merges the splits (no device-wide wait: it is
// elected with an atomic counter that it resets for the next launch).
//
// Softmax: score = (q . k) * scale, p = exp(score - max), out = sum(p v)/sum(p),
// with __expf as in the reference.  K/V are read as fp16 or fp32 (the
// engine's cache format).
#include "attention.cuh"
#include "common.cuh"

namespace ijb {

constexpr int kAttnWarps = 4;
constexpr int kAttnThreads = kAttnWarps * 32;
constexpr int kAttnChunk = 32;   // positions a warp scores at once (one per lane)
constexpr int kAttnSplit = 512;  // positions per CTA: each warp walks every 4th chunk of 32

// K/V tile stages per warp: two (the next chunk loads while this one is used)
// when a 32-row K+V tile pair is at most 8 KB, else one.
template <int HD, typename KT>
__host__ __device__ constexpr int attn_stages() { return HD * static_cast<int>(sizeof(KT)) <= 128 ? 2 : 1; }
template <int HD, typename KT>
__host__ __device__ constexpr int attn_smem() {
    return kAttnWarps * attn_stages<HD, KT>() * 2 * kAttnChunk * HD * static_cast<int>(sizeof(KT));
}

// Loads of cached K/V elements as fp32 from either storage format.
__device__ __forceinline__ void load8(const __half *p, float (&f)[8]) {
    const uint4 raw = *reinterpret_cast<const uint4 *>(p);
    const __half2 *h2 = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float2 v = __half22float2(h2[j]);
        f[2 * j] = v.x;
        f[2 * j + 1] = v.y;
    }
}
__device__ __forceinline__ void load8(const float *p, float (&f)[8]) {
    const float4 a = *reinterpret_cast<const float4 *>(p), b = *reinterpret_cast<const float4 *>(p + 4);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}
template <int N>
__device__ __forceinline__ void loadn(const __half *p, float (&f)[N]) {
    if constexpr (N == 2) {
        const float2 v = __half22float2(*reinterpret_cast<const __half2 *>(p));
        f[0] = v.x;
        f[1] = v.y;
    } else {
        const uint2 raw = *reinterpret_cast<const uint2 *>(p);
        const float2 v0 = __half22float2(*reinterpret_cast<const __half2 *>(&raw.x));
        const float2 v1 = __half22float2(*reinterpret_cast<const __half2 *>(&raw.y));
        f[0] = v0.x; f[1] = v0.y; f[2] = v1.x; f[3] = v1.y;
    }
}
template <int N>
__device__ __forceinline__ void loadn(const float *p, float (&f)[N]) {
    if constexpr (N == 2) {
        const float2 v = *reinterpret_cast<const float2 *>(p);
        f[0] = v.x;
        f[1] = v.y;
    } else {
        const float4 v = *reinterpret_cast<const float4 *>(p);
        f[0] = v.x; f[1] = v.y; f[2] = v.z; f[3] = v.w;
    }
}

// One CTA = one (token, kv head, split of up to kAttnSplit positions).  Warp
// w takes chunks w, w+4, w+8, ... of 32 positions: lane 0 copies the K and V
// page rows of a chunk into one of the warp's tile stages with cp.async.bulk
// (the next chunk loads while this one is used), lanes score one position
// each (rows read in a lane-rotated chunk order, so the 128-bit shared loads do
// not collide in banks), and the warp keeps an online-softmax state per query
// head across its chunks, accumulating V with lanes owning head-dim elements.
template <int HD, int G, typename KT>
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const __grid_constant__ AttnParams p) {
    constexpr int DPL = HD / 32;  // head-dim elements per lane in the V phase
    constexpr int CH = HD / 8;    // 8-element chunks per row
    constexpr int ST = attn_stages<HD, KT>();
    const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    extern __shared__ __align__(128) uint8_t smem[];
    KT *tiles = reinterpret_cast<KT *>(smem) + warp * ST * 2 * kAttnChunk * HD;  // [ST][K, V][32][HD]
    __shared__ __align__(16) float qs[G][HD];
    __shared__ float wm[kAttnWarps][G], wl[kAttnWarps][G];
    __shared__ __align__(16) float wo[kAttnWarps][G][HD];
    __shared__ __align__(8) uint64_t bar[kAttnWarps][ST];
    __shared__ int is_last;
    __shared__ uint32_t cta_abort;

    pdl_trigger();
    pdl_wait();

    const int pos = p.tok_pos[b];
    const int seq = p.tok_seq[b];
    const int n_pos = pos + 1;
    const int p0 = split * p.split_len;
    const int nsplit = (n_pos + p.split_len - 1) / p.split_len;
    if (p0 >= n_pos) return;  // this token has fewer splits (uniform across the CTA)
    const int p1 = min(n_pos, p0 + p.split_len);
    const int nchunks = (p1 - p0 + kAttnChunk - 1) / kAttnChunk;
    const int mine = warp < nchunks ? (nchunks - warp + kAttnWarps - 1) / kAttnWarps : 0;
    const int *pages = p.page_table + static_cast<long>(seq) * p.max_pages_per_seq;
    const long head_off = static_cast<long>(kvh) * p.page_size * HD;

    if (threadIdx.x == 0) cta_abort = 0u;  // read only after the __syncthreads below
    if (lane == 0) {
        for (int st = 0; st < ST; ++st) mbar_init(&bar[warp][st], 1);
        fence_barrier_init();
    }
    __syncwarp();
    // chunk k of this warp -> stage k % ST: the pages holding its valid rows
    auto issue = [&](int k) {
        const int t0 = p0 + (warp + kAttnWarps * k) * kAttnChunk;
        const int cnt = min(kAttnChunk, p1 - t0);
        const int npg = (cnt + p.page_size - 1) / p.page_size;
        const uint32_t row_bytes = HD * sizeof(KT);
        KT *kt = tiles + (k % ST) * 2 * kAttnChunk * HD, *vt = kt + kAttnChunk * HD;
        uint64_t *bb = &bar[warp][k % ST];
        mbar_arrive_expect_tx(bb, 2u * npg * p.page_size * row_bytes);
        for (int j = 0; j < npg; ++j) {
            const long page = pages[(t0 + j * p.page_size) / p.page_size];
            const KT *ks = static_cast<const KT *>(p.k_cache) + page * p.page_stride + head_off;
            const KT *vs = static_cast<const KT *>(p.v_cache) + page * p.page_stride + head_off;
            bulk_g2s(kt + j * p.page_size * HD, ks, p.page_size * row_bytes, bb);
            bulk_g2s(vt + j * p.page_size * HD, vs, p.page_size * row_bytes, bb);
        }
    };
    if (lane == 0)
        for (int k = 0; k < ST && k < mine; ++k) issue(k);
    const float *q = p.q + static_cast<long>(b) * p.q_stride + static_cast<long>(kvh) * G * HD;
    for (int i = threadIdx.x; i < G * HD; i += kAttnThreads) qs[i / HD][i % HD] = q[i];
    __syncthreads();

    float m[G], l[G], o[G][DPL];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int j = 0; j < DPL; ++j) o[g][j] = 0.f;
    }
    for (int k = 0; k < mine; ++k) {
        mbar_wait_bounded(&bar[warp][k % ST], (k / ST) & 1, p.status, &cta_abort);
        const KT *ktile = tiles + (k % ST) * 2 * kAttnChunk * HD, *vtile = ktile + kAttnChunk * HD;
        const int t0 = p0 + (warp + kAttnWarps * k) * kAttnChunk;
        const int cnt = min(kAttnChunk, p1 - t0);
        // ---- scores: lane -> position t0 + lane
        float s[G];
#pragma unroll
        for (int g = 0; g < G; ++g) s[g] = 0.f;
        const KT *krow = ktile + lane * HD;
#pragma unroll
        for (int c = 0; c < CH; ++c) {
            const int cc = (c + lane) % CH;
            float kf[8];
            load8(krow + cc * 8, kf);
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float4 qa = *reinterpret_cast<const float4 *>(&qs[g][cc * 8]);
                const float4 qb = *reinterpret_cast<const float4 *>(&qs[g][cc * 8 + 4]);
                s[g] = fmaf(qa.x, kf[0], s[g]);
                s[g] = fmaf(qa.y, kf[1], s[g]);
                s[g] = fmaf(qa.z, kf[2], s[g]);
                s[g] = fmaf(qa.w, kf[3], s[g]);
                s[g] = fmaf(qb.x, kf[4], s[g]);
                s[g] = fmaf(qb.y, kf[5], s[g]);
                s[g] = fmaf(qb.z, kf[6], s[g]);
                s[g] = fmaf(qb.w, kf[7], s[g]);
            }
        }
        // ---- online softmax: rescale the running state to the new maximum
        float pr[G];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float sg = lane < cnt ? s[g] * p.scale : -INFINITY;
            const float mn = fmaxf(m[g], warp_max(sg));
            const float alpha = m[g] == -INFINITY ? 0.f : __expf(m[g] - mn);
            pr[g] = lane < cnt ? __expf(sg - mn) : 0.f;
            l[g] = fmaf(l[g], alpha, warp_sum(pr[g]));
#pragma unroll
            for (int j = 0; j < DPL; ++j) o[g][j] *= alpha;
            m[g] = mn;
        }
        // ---- V: lane -> head-dim elements [lane*DPL, lane*DPL+DPL)
#pragma unroll 4
        for (int tt = 0; tt < cnt; ++tt) {
            float vf[DPL];
            loadn<DPL>(vtile + tt * HD + lane * DPL, vf);
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float pg = __shfl_sync(0xffffffffu, pr[g], tt);
#pragma unroll
                for (int j = 0; j < DPL; ++j) o[g][j] = fmaf(pg, vf[j], o[g][j]);
            }
        }
        __syncwarp();  // every lane is done with this stage
        if (lane == 0 && k + ST < mine) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue(k + ST);
        }
    }

    // ---- merge the warps of this CTA
#pragma unroll
    for (int g = 0; g < G; ++g) {
        if (lane == 0) {
            wm[warp][g] = m[g];
            wl[warp][g] = l[g];
        }
#pragma unroll
        for (int j = 0; j < DPL; ++j) wo[warp][g][lane * DPL + j] = o[g][j];
    }
    __syncthreads();
    if (nsplit == 1) {  // the only split: normalise and write
        for (int i = threadIdx.x; i < G * HD; i += kAttnThreads) {
            const int g = i / HD, d = i % HD;
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, wm[w][g]);
            float L = 0.f, O = 0.f;
#pragma unroll
            for (int w = 0; w < kAttnWarps; ++w) {
                const float f = wm[w][g] == -INFINITY ? 0.f : __expf(wm[w][g] - M);
                L = fmaf(wl[w][g], f, L);
                O = fmaf(wo[w][g][d], f, O);
            }
            p.out[static_cast<long>(b) * p.out_stride + (static_cast<long>(kvh) * G + g) * HD + d] = O / L;
        }
        return;
    }
    float *part = p.partial + ((static_cast<long>(b) * p.heads + kvh * G) * p.max_splits) * (HD + 2);
    for (int i = threadIdx.x; i < G * HD; i += kAttnThreads) {
        const int g = i / HD, d = i % HD;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, wm[w][g]);
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w) {
            const float f = wm[w][g] == -INFINITY ? 0.f : __expf(wm[w][g] - M);
            L = fmaf(wl[w][g], f, L);
            O = fmaf(wo[w][g][d], f, O);
        }
        float *rec = part + (static_cast<long>(g) * p.max_splits + split) * (HD + 2);
        rec[2 + d] = O;
        if (d == 0) {
            rec[0] = M;
            rec[1] = L;
        }
    }

    // ---- the last split to finish for this (token, kv head) merges them
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        int *ctr = p.counters + b * p.kv_heads + kvh;
        const int prev = atomicAdd(ctr, 1);
        is_last = (prev == nsplit - 1);
        if (is_last) *ctr = 0;  // ready for the next launch
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    for (int i = threadIdx.x; i < G * HD; i += kAttnThreads) {
        const int g = i / HD, d = i % HD;
        const volatile float *recs = part + static_cast<long>(g) * p.max_splits * (HD + 2);
        float M = -INFINITY;
        for (int sp = 0; sp < nsplit; ++sp) M = fmaxf(M, recs[sp * (HD + 2)]);
        float L = 0.f, O = 0.f;
        for (int sp = 0; sp < nsplit; ++sp) {
            const float f = __expf(recs[sp * (HD + 2)] - M);
            L = fmaf(recs[sp * (HD + 2) + 1], f, L);
            O = fmaf(recs[sp * (HD + 2) + 2 + d], f, O);
        }
        p.out[static_cast<long>(b) * p.out_stride + (static_cast<long>(kvh) * G + g) * HD + d] = O / L;
    }
}

template <int HD, int G, typename KT>
static cudaError_t launch_attn(const AttnParams &p, dim3 grid, cudaStream_t stream, bool pdl) {
    const int smem = attn_smem<HD, KT>();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, attention_kernel<HD, G, KT>, p);
}

template <typename KT>
static cudaError_t attention_launch_t(const AttnParams &p, dim3 grid, cudaStream_t stream, bool pdl) {
    const int G = p.heads / p.kv_heads;
    if (p.head_dim == 64) {
        if (G == 4) return launch_attn<64, 4, KT>(p, grid, stream, pdl);
        if (G == 8) return launch_attn<64, 8, KT>(p, grid, stream, pdl);
        if (G == 2) return launch_attn<64, 2, KT>(p, grid, stream, pdl);
        if (G == 1) return launch_attn<64, 1, KT>(p, grid, stream, pdl);
    } else if (p.head_dim == 128) {
        if (G == 4) return launch_attn<128, 4, KT>(p, grid, stream, pdl);
        if (G == 8) return launch_attn<128, 8, KT>(p, grid, stream, pdl);
        if (G == 2) return launch_attn<128, 2, KT>(p, grid, stream, pdl);
        if (G == 1) return launch_attn<128, 1, KT>(p, grid, stream, pdl);
    }
    return cudaErrorInvalidValue;
}

int attention_split_len() { return kAttnSplit; }

// Opts every instance in to its K/V tile shared memory on the current device
// (done once per device at engine creation, outside any graph capture).
template <int HD, int G, typename KT>
static cudaError_t set_attr() {
    const int smem = attn_smem<HD, KT>();
    return cudaFuncSetAttribute(attention_kernel<HD, G, KT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
}

template <typename KT>
static cudaError_t set_attrs_t() {
    cudaError_t e;
    if ((e = set_attr<64, 1, KT>()) || (e = set_attr<64, 2, KT>()) || (e = set_attr<64, 4, KT>()) ||
        (e = set_attr<64, 8, KT>()) || (e = set_attr<128, 1, KT>()) || (e = set_attr<128, 2, KT>()) ||
        (e = set_attr<128, 4, KT>()) || (e = set_attr<128, 8, KT>()))
        return e;
    return cudaSuccess;
}

cudaError_t attention_prepare() {
    cudaError_t e = set_attrs_t<__half>();
    return e != cudaSuccess ? e : set_attrs_t<float>();
}

cudaError_t attention_launch(const AttnParams &p, cudaStream_t stream, bool pdl) {
    if (p.split_len != kAttnSplit || p.page_size > 32 || 32 % p.page_size) return cudaErrorInvalidValue;
    dim3 grid(p.max_splits, p.kv_heads, p.batch);
    return p.kv_f32 ? attention_launch_t<float>(p, grid, stream, pdl) : attention_launch_t<__half>(p, grid, stream, pdl);
}

}  // namespace ijb
