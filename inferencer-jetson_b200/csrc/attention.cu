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
    __shared__ int pg_s[kAttnSplit / 8];  // this split's page ids (page_size >= 8)

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
    {
        const int *pt = p.page_table + static_cast<long>(seq) * p.max_pages_per_seq + p0 / p.page_size;
        for (int i = threadIdx.x; i < (p1 - p0 + p.page_size - 1) / p.page_size; i += kAttnThreads) pg_s[i] = pt[i];
        __syncthreads();
    }
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
            const long page = pg_s[(t0 - p0) / p.page_size + j];
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

// ------------------------------------------------ tensor-core variant --
//
// fp16 cache, head_dim 64: the same CTA/warp/chunk schedule as above, but
// scores and P·V run on mma.sync.m16n8k16 (fp16 in, fp32 accumulate).  The
// query heads of the KV group are the M rows (G of 16, the rest zero), a
// chunk's 32 positions the N (scores) or K (P·V) extent.  K/V page runs arrive
// through a 3-D TMA map with 128-byte swizzle, so the ldmatrix reads of both
// tiles are free of bank conflicts; the P fragment is built in registers from
// the score accumulators.  The query and the probabilities enter the MMAs as
// fp16 hi + lo pairs (two MMAs each), so only the cache's own fp16 rounding
// remains; softmax stays fp32 with __expf as above.

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr)
                 : "memory");
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr)
                 : "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *map, int x, int y, int z, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
            "r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}
// Byte offset of 16-byte chunk `c` of row `r` in a 128-byte-swizzled tile
// (1024-byte aligned): the chunk index is XORed with the row's low 3 bits.
__device__ __forceinline__ uint32_t swz(int r, int c) { return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4)); }

constexpr int kMmaAttnStages = 2;
constexpr int kMmaAttnTile = kAttnChunk * 128;  // one K or V tile: 32 rows of 64 fp16
constexpr int kMmaAttnSmem = kAttnWarps * kMmaAttnStages * 2 * kMmaAttnTile + 1024;  // + alignment slack

template <int G>
__global__ void __launch_bounds__(kAttnThreads) attention_mma_kernel(const __grid_constant__ AttnParams p) {
    constexpr int HD = 64, ST = kMmaAttnStages;
    const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;

    extern __shared__ uint8_t smem_raw[];
    const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;  // swizzled TMA tiles need 1024-byte alignment
    const uint32_t wtiles = base + static_cast<uint32_t>(warp * ST * 2 * kMmaAttnTile);  // [ST][K, V]
    __shared__ float wm[kAttnWarps][G], wl[kAttnWarps][G];
    __shared__ __align__(16) float wo[kAttnWarps][G][HD];
    __shared__ __align__(8) uint64_t bar[kAttnWarps][ST];
    __shared__ int is_last;
    __shared__ uint32_t cta_abort;
    __shared__ int pg_s[kAttnSplit / 8];  // this split's page ids (page_size >= 8)

    pdl_trigger();
    pdl_wait();

    const int pos = p.tok_pos[b];
    const int seq = p.tok_seq[b];
    const int n_pos = pos + 1;
    const int p0 = split * p.split_len;
    const int nsplit = (n_pos + p.split_len - 1) / p.split_len;
    if (p0 >= n_pos) return;
    const int p1 = min(n_pos, p0 + p.split_len);
    const int nchunks = (p1 - p0 + kAttnChunk - 1) / kAttnChunk;
    const int mine = warp < nchunks ? (nchunks - warp + kAttnWarps - 1) / kAttnWarps : 0;
    {
        const int *pt = p.page_table + static_cast<long>(seq) * p.max_pages_per_seq + p0 / p.page_size;
        for (int i = threadIdx.x; i < (p1 - p0 + p.page_size - 1) / p.page_size; i += kAttnThreads) pg_s[i] = pt[i];
        __syncthreads();
    }
    const int ps = p.page_size;

    if (threadIdx.x == 0) cta_abort = 0u;
    if (lane == 0) {
        for (int st = 0; st < ST; ++st) mbar_init(&bar[warp][st], 1);
        fence_barrier_init();
    }
    __syncwarp();
    auto issue = [&](int k) {
        const int t0 = p0 + (warp + kAttnWarps * k) * kAttnChunk;
        const int cnt = min(kAttnChunk, p1 - t0);
        const int npg = (cnt + ps - 1) / ps;
        const uint32_t kt = wtiles + static_cast<uint32_t>((k % ST) * 2 * kMmaAttnTile), vt = kt + kMmaAttnTile;
        uint64_t *bb = &bar[warp][k % ST];
        mbar_arrive_expect_tx(bb, 2u * npg * ps * 128u);
        for (int j = 0; j < npg; ++j) {
            const int page = pg_s[(t0 - p0) / ps + j];
            tma_load_3d(kt + j * ps * 128, &p.kv_map, 0, kvh * ps, page, bb);
            tma_load_3d(vt + j * ps * 128, &p.kv_map, 0, (p.kv_heads + kvh) * ps, page, bb);
        }
    };
    if (lane == 0)
        for (int k = 0; k < ST && k < mine; ++k) issue(k);

    // query fragments (rows = the group's heads, 16 wide: rows >= G are zero),
    // [k-step][hi, lo][a0, a2]
    uint32_t qa[4][2][2];
    {
        const float *q = p.q + static_cast<long>(b) * p.q_stride + static_cast<long>(kvh) * G * HD;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            if (gid < G) {
                const float2 v0 = *reinterpret_cast<const float2 *>(q + gid * HD + 16 * kk + 2 * tig);
                const float2 v1 = *reinterpret_cast<const float2 *>(q + gid * HD + 16 * kk + 8 + 2 * tig);
                const __half2 h0 = __floats2half2_rn(v0.x, v0.y), h1 = __floats2half2_rn(v1.x, v1.y);
                const float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
                qa[kk][0][0] = *reinterpret_cast<const uint32_t *>(&h0);
                qa[kk][0][1] = *reinterpret_cast<const uint32_t *>(&h1);
                qa[kk][1][0] = pack_h2(v0.x - f0.x, v0.y - f0.y);
                qa[kk][1][1] = pack_h2(v1.x - f1.x, v1.y - f1.y);
            } else {
                qa[kk][0][0] = qa[kk][0][1] = qa[kk][1][0] = qa[kk][1][1] = 0u;
            }
        }
    }
    __syncthreads();  // barriers initialised, cta_abort cleared

    float o[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
    float m = -INFINITY, l = 0.f;  // this lane's head row gid
    for (int k = 0; k < mine; ++k) {
        mbar_wait_bounded(&bar[warp][k % ST], (k / ST) & 1, p.status, &cta_abort);
        const uint32_t kt = wtiles + static_cast<uint32_t>((k % ST) * 2 * kMmaAttnTile), vt = kt + kMmaAttnTile;
        const int t0 = p0 + (warp + kAttnWarps * k) * kAttnChunk;
        const int cnt = min(kAttnChunk, p1 - t0);
        if (cnt < kAttnChunk) {  // V rows past the last position: zero (their weights are zero, keep them finite)
            for (int r = cnt + (lane >> 3); r < kAttnChunk; r += 4)
                asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(vt + r * 128 + (lane & 7) * 16), "r"(0u)
                             : "memory");
            __syncwarp();
        }
        // ---- scores S[head][position] = Q . K^T, 4 tiles of 8 positions
        float sc[4][4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
            for (int kk2 = 0; kk2 < 2; ++kk2) {
                uint32_t kb[4];
                ldsm_x4(kt + swz(8 * j + (lane & 7), 4 * kk2 + (lane >> 3)), kb);
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    mma16816(sc[j], qa[2 * kk2][h][0], qa[2 * kk2][h][1], kb[0], kb[1]);
                    mma16816(sc[j], qa[2 * kk2 + 1][h][0], qa[2 * kk2 + 1][h][1], kb[2], kb[3]);
                }
            }
        }
        // ---- online softmax for row gid (the lane quad holds its 32 positions)
        float mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const float v = 8 * j + 2 * tig + e < cnt ? sc[j][e] * p.scale : -INFINITY;
                sc[j][e] = v;
                mx = fmaxf(mx, v);
            }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float mn = fmaxf(m, mx);
        const float alpha = m == -INFINITY ? 0.f : __expf(m - mn);
        float rs = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const float pr = sc[j][e] == -INFINITY ? 0.f : __expf(sc[j][e] - mn);
                sc[j][e] = pr;
                rs += pr;
            }
        rs += __shfl_xor_sync(0xffffffffu, rs, 1);
        rs += __shfl_xor_sync(0xffffffffu, rs, 2);
        l = fmaf(l, alpha, rs);
        m = mn;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
            o[nt][0] *= alpha;
            o[nt][1] *= alpha;
        }
        // ---- O += P V: P from the score registers, V tiles through ldmatrix.trans
#pragma unroll
        for (int kp = 0; kp < 2; ++kp) {
            const __half2 h0 = __floats2half2_rn(sc[2 * kp][0], sc[2 * kp][1]);
            const __half2 h2 = __floats2half2_rn(sc[2 * kp + 1][0], sc[2 * kp + 1][1]);
            const float2 f0 = __half22float2(h0), f2 = __half22float2(h2);
            const uint32_t pa0 = *reinterpret_cast<const uint32_t *>(&h0), pa2 = *reinterpret_cast<const uint32_t *>(&h2);
            const uint32_t pl0 = pack_h2(sc[2 * kp][0] - f0.x, sc[2 * kp][1] - f0.y);
            const uint32_t pl2 = pack_h2(sc[2 * kp + 1][0] - f2.x, sc[2 * kp + 1][1] - f2.y);
#pragma unroll
            for (int nt2 = 0; nt2 < 4; ++nt2) {
                uint32_t vb[4];
                const int mi = lane >> 3;
                ldsm_x4_t(vt + swz(16 * kp + (mi & 1) * 8 + (lane & 7), 2 * nt2 + (mi >> 1)), vb);
                mma16816(o[2 * nt2], pa0, pa2, vb[0], vb[1]);
                mma16816(o[2 * nt2 + 1], pa0, pa2, vb[2], vb[3]);
                mma16816(o[2 * nt2], pl0, pl2, vb[0], vb[1]);
                mma16816(o[2 * nt2 + 1], pl0, pl2, vb[2], vb[3]);
            }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // this stage's generic accesses before TMA refills it
        __syncwarp();
        if (lane == 0 && k + ST < mine) issue(k + ST);
    }

    // ---- merge the warps of this CTA, then the splits (as in attention_kernel)
    if (gid < G) {
        if (tig == 0) {
            wm[warp][gid] = m;
            wl[warp][gid] = l;
        }
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
            wo[warp][gid][8 * nt + 2 * tig] = o[nt][0];
            wo[warp][gid][8 * nt + 2 * tig + 1] = o[nt][1];
        }
    }
    __syncthreads();
    if (nsplit == 1) {
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
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        int *ctr = p.counters + b * p.kv_heads + kvh;
        const int prev = atomicAdd(ctr, 1);
        is_last = (prev == nsplit - 1);
        if (is_last) *ctr = 0;
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

template <int G>
static cudaError_t launch_attn_mma(const AttnParams &p, dim3 grid, cudaStream_t stream, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = kMmaAttnSmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, attention_mma_kernel<G>, p);
}

typedef CUresult (*EncodeTiledFnA)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int attention_make_kv_map(CUtensorMap *map, const void *layer_base, int head_dim, int kv_heads, int page_size,
                          long page_stride_elems, long num_pages) {
    if (head_dim != 64 || (reinterpret_cast<uintptr_t>(layer_base) & 15)) return -1;
    static EncodeTiledFnA fn = nullptr;
    if (!fn) {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return -1;
        fn = reinterpret_cast<EncodeTiledFnA>(ptr);
    }
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(head_dim), static_cast<cuuint64_t>(2 * kv_heads * page_size),
                          static_cast<cuuint64_t>(num_pages)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(head_dim * 2), static_cast<cuuint64_t>(page_stride_elems * 2)};
    cuuint32_t box[3] = {static_cast<cuuint32_t>(head_dim), static_cast<cuuint32_t>(page_size), 1};
    cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void *>(layer_base), dims, strides, box,
                          estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : -1;
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
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(attention_mma_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMmaAttnSmem)) ||
        (e = cudaFuncSetAttribute(attention_mma_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMmaAttnSmem)) ||
        (e = cudaFuncSetAttribute(attention_mma_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMmaAttnSmem)) ||
        (e = cudaFuncSetAttribute(attention_mma_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMmaAttnSmem)))
        return e;
    e = set_attrs_t<__half>();
    return e != cudaSuccess ? e : set_attrs_t<float>();
}

cudaError_t attention_launch(const AttnParams &p, cudaStream_t stream, bool pdl) {
    if (p.split_len != kAttnSplit || p.page_size < 8 || p.page_size > 32 || 32 % p.page_size)
        return cudaErrorInvalidValue;
    dim3 grid(p.max_splits, p.kv_heads, p.batch);
    if (p.has_map && p.head_dim == 64 && !p.kv_f32) {
        const int G = p.heads / p.kv_heads;
        if (G == 4) return launch_attn_mma<4>(p, grid, stream, pdl);
        if (G == 8) return launch_attn_mma<8>(p, grid, stream, pdl);
        if (G == 2) return launch_attn_mma<2>(p, grid, stream, pdl);
        if (G == 1) return launch_attn_mma<1>(p, grid, stream, pdl);
    }
    return p.kv_f32 ? attention_launch_t<float>(p, grid, stream, pdl) : attention_launch_t<__half>(p, grid, stream, pdl);
}

}  // namespace ijb
