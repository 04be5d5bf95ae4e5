// GQA decode attention over the paged fp16 KV cache (split-KV, sm_100a).
//
// Replaces attention_cuda / attention_batch_cuda (inferencer.cu:982-1041): the
// reference runs one 128-thread CTA per query head and walks positions 0..pos
// serially with two block barriers per position over an fp32 [layer][ctx][kv]
// cache.  Two kernels here, both splitting a sequence's positions and keeping
// an online-softmax state (max, sum, unnormalised output) per split, the KV
// group's query heads sharing every K/V row loaded:
//  * ijb_attention_stream_kernel (fp16 cache, head_dim 64 or 128): persistent, one CTA of
//    streaming warps per SM, 128-position work items, tensor-core chunks; the
//    splits are merged by ijb_attention_finish_kernel (one CTA per token);
//  * ijb_attention_kernel (fp32 cache, and beyond the streaming kernel's
//    limits): one CTA per (token, kv head, split of up to 512 positions) on
//    CUDA cores, lanes owning positions while scoring and head-dim elements
//    while accumulating V; the last CTA of a (token, kv head) to finish merges
//    the splits (elected with an atomic counter that it resets for the next
//    launch).
//
// Softmax: score = (q . k) * scale, p = exp(score - max), out = sum(p v)/sum(p),
// with __expf as in the reference.  K/V are read as fp16 or fp32 (the
// engine's cache format).
#include "attention.cuh"
#include "common.cuh"
#include "mma_gemm.cuh"

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
__global__ void __launch_bounds__(kAttnThreads) ijb_attention_kernel(const __grid_constant__ AttnParams p) {
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
// fp16 cache, head_dim 64 or 128 (HD / 64 swizzled 128-byte halves per row):
// scores and P·V run on mma.sync.m16n8k16 (fp16 in, fp32 accumulate).  The
// chunk's positions (scores) or the head dims (P·V) are the M rows, the KV
// group's query heads the 8 columns (attn_chunk_t below).  K/V page runs arrive
// through a 3-D TMA map with 128-byte swizzle, so the ldmatrix reads of both
// tiles are free of bank conflicts; the P fragment is built in registers from
// the score accumulators.  The query and the probabilities enter the MMAs as
// fp16 hi + lo pairs (two MMAs each), so only the cache's own fp16 rounding
// remains; softmax stays fp32 with __expf as above.

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
// The same in a tile of CH rows whose rows are wider than the 128-byte swizzle
// span (head_dim 128: 256 bytes): it is stored as consecutive 128-byte-wide
// halves [half][CH rows][128 B], chunk c of a row in half c / 8.
template <int CH>
__device__ __forceinline__ uint32_t swz_wide(int r, int c) {
    return static_cast<uint32_t>((c >> 3) * CH * 128) + swz(r, c & 7);
}
// mma.m16n8k16 with all four A registers (rows 8-15 in use).
__device__ __forceinline__ void mma16816_a4(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// Transpose of the 8x8 fp16 matrix whose fragment (row lane/4, columns
// 2(lane%4) and +1) this warp holds.
__device__ __forceinline__ uint32_t movm_t(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}


// One chunk of up to 16*MT positions on the tensor cores with positions as
// the MMA rows and the group's query heads as its 8 columns (G <= 8):
//   S^T[pos][head] = K[pos][:] . Q^T           (MT tiles of 16 positions)
//   O^T[dim][head] += V^T[dim][pos] . P^T      (HD/16 tiles of 16 dims)
// The lane holds heads 2(lane%4) and 2(lane%4)+1: its online-softmax state
// m[2], l[2]; the max and sum run over the 8 lanes of equal lane%4.  P^T
// comes from the score accumulators through movmatrix transposes.  Q and P
// enter as fp16 hi + lo pairs (two MMAs each), so only the cache's own fp16
// rounding remains; softmax is fp32 with __expf.  kt / vt: the chunk's
// 128-byte-swizzled K and V tiles (V rows past cnt are zeroed here).
template <int HD, int MT>
__device__ __forceinline__ void attn_chunk_t(uint32_t kt, uint32_t vt, int cnt, float scale,
                                             const uint32_t (&qb)[HD / 16][2][2], float (&o)[HD / 16][4],
                                             float (&m)[2], float (&l)[2], int lane) {
    constexpr int CH = 16 * MT;   // positions of the chunk
    constexpr int KS = HD / 16;   // k-steps of the scores, dim tiles of the output
    const int gid = lane >> 2, mi = lane >> 3;
    if (cnt < CH) {  // V rows past the last position: zero (their weights are zero, keep them finite)
        for (int r = cnt + (lane >> 3); r < CH; r += 4)
#pragma unroll
            for (int hf = 0; hf < HD / 64; ++hf)
                asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(vt + hf * CH * 128 + r * 128 +
                                                                            (lane & 7) * 16),
                             "r"(0u)
                             : "memory");
        __syncwarp();
    }
    // ---- scores: sc[mt] = S^T rows 16mt + gid (+8), heads 2(lane%4) (+1)
    float sc[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
        sc[mt][0] = sc[mt][1] = sc[mt][2] = sc[mt][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
            uint32_t ka[4];
            ldsm_x4(kt + swz_wide<CH>(16 * mt + 8 * (mi & 1) + (lane & 7), 2 * kk + (mi >> 1)), ka);
            mma16816_a4(sc[mt], ka, qb[kk][0][0], qb[kk][0][1]);
            mma16816_a4(sc[mt], ka, qb[kk][1][0], qb[kk][1][1]);
        }
    }
    // ---- online softmax per head
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float v = 16 * mt + gid + 8 * (i >> 1) < cnt ? sc[mt][i] * scale : -INFINITY;
            sc[mt][i] = v;
            mx[i & 1] = fmaxf(mx[i & 1], v);
        }
    float alpha[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
        mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], 4));
        mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], 8));
        mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], 16));
        const float mn = fmaxf(m[e], mx[e]);
        alpha[e] = m[e] == -INFINITY ? 0.f : __expf(m[e] - mn);
        m[e] = mn;
    }
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float pr = sc[mt][i] == -INFINITY ? 0.f : __expf(sc[mt][i] - m[i & 1]);
            sc[mt][i] = pr;
            rs[i & 1] += pr;
        }
#pragma unroll
    for (int e = 0; e < 2; ++e) {
        rs[e] += __shfl_xor_sync(0xffffffffu, rs[e], 4);
        rs[e] += __shfl_xor_sync(0xffffffffu, rs[e], 8);
        rs[e] += __shfl_xor_sync(0xffffffffu, rs[e], 16);
        l[e] = fmaf(l[e], alpha[e], rs[e]);
    }
#pragma unroll
    for (int md = 0; md < KS; ++md) {
        o[md][0] *= alpha[0];
        o[md][1] *= alpha[1];
        o[md][2] *= alpha[0];
        o[md][3] *= alpha[1];
    }
    // ---- O^T += V^T P^T, 16 positions per k-step
#pragma unroll
    for (int kp = 0; kp < MT; ++kp) {
        const __half2 ht = __floats2half2_rn(sc[kp][0], sc[kp][1]), hb = __floats2half2_rn(sc[kp][2], sc[kp][3]);
        const float2 ft = __half22float2(ht), fb = __half22float2(hb);
        const uint32_t bt = movm_t(*reinterpret_cast<const uint32_t *>(&ht));
        const uint32_t bb = movm_t(*reinterpret_cast<const uint32_t *>(&hb));
        const uint32_t lt = movm_t(pack_h2(sc[kp][0] - ft.x, sc[kp][1] - ft.y));
        const uint32_t lb = movm_t(pack_h2(sc[kp][2] - fb.x, sc[kp][3] - fb.y));
#pragma unroll
        for (int md = 0; md < KS; ++md) {
            uint32_t va[4];
            ldsm_x4_t(vt + swz_wide<CH>(16 * kp + 8 * (mi >> 1) + (lane & 7), 2 * md + (mi & 1)), va);
            mma16816_a4(o[md], va, bt, bb);
            mma16816_a4(o[md], va, lt, lb);
        }
    }
}

// ------------------------------------------------ streaming variant --
//
// fp16 cache, head_dim 64 or 128, tensor-core chunks as above, as a persistent
// kernel: one CTA of stream_warps<HD>() independent warps per SM.  The work is cut
// into items of up to kAttnItem positions of one (token, kv head): a warp's
// first item is fixed by its index, the next ones come from a device-wide
// counter (the request for the following item is in flight while the current
// one is set up).  Each warp keeps kStreamStages chunks of K/V in flight
// through the 3-D TMA map, across item boundaries (a warp's queue holds the
// items its in-flight chunks belong to), refilling a stage as soon as it is
// used, so a warp's copies never drain between items and no CTA waits for
// another wave.  A finished item leaves its softmax state (max, sum,
// unnormalised output) per head for ijb_attention_finish_kernel, or the output
// itself when it covers the whole sequence.  The last CTA to finish resets the
// item counter.

// Build-time shape of the streaming kernel (warps per CTA, chunks in flight per
// warp, positions per chunk).  Measured on B200 (ragged64 step, same box):
// 8 x 2 x 32 1.641 ms; 8 x 3 x 32 1.657; 6 x 2 x 64 1.673; 4 x 3 x 64 1.703;
// 8 x 3 or 4 x 16 1.740; 10 x 2 x 32 and 12 x 2 x 32 slower than 8 x 3 x 32.
#ifndef IJB_STREAM_WARPS
#define IJB_STREAM_WARPS 8
#endif
#ifndef IJB_STREAM_STAGES
#define IJB_STREAM_STAGES 2
#endif
#ifndef IJB_STREAM_CHUNK
#define IJB_STREAM_CHUNK 32
#endif
constexpr int kStreamWarps = IJB_STREAM_WARPS;
constexpr int kStreamStages = IJB_STREAM_STAGES;
constexpr int kStreamChunk = IJB_STREAM_CHUNK;          // positions per chunk (per stage)
// head_dim 128: a stage's K and V tiles take twice the bytes, so six warps
// fit the shared memory at two stages each
constexpr int kStreamWarps128 = 6;
template <int HD>
__host__ __device__ constexpr int stream_warps() { return HD == 64 ? kStreamWarps : kStreamWarps128; }
// one K or V tile: kStreamChunk rows of HD fp16, as HD / 64 swizzled 128-byte-wide halves
template <int HD>
__host__ __device__ constexpr int stream_tile() { return kStreamChunk * HD * 2; }
template <int HD>
__host__ __device__ constexpr int stream_smem() {
    return stream_warps<HD>() * IJB_STREAM_STAGES * 2 * stream_tile<HD>() + 1024;  // + alignment slack
}
static_assert(stream_smem<128>() + 8 * 1024 <= 227 * 1024, "head_dim-128 streaming attention shared memory");
constexpr int kStreamQueue = kStreamStages + 1;  // items a warp's in-flight chunks can span, plus the one in use
#ifndef IJB_ATTN_ITEM
#define IJB_ATTN_ITEM 128
#endif
constexpr int kAttnItem = IJB_ATTN_ITEM;         // positions per work item
constexpr int kItemPages = kAttnItem / 8;        // page ids of an item (page_size >= 8)
static_assert(kStreamChunk % 16 == 0 && kStreamChunk <= 64 && kAttnItem % kStreamChunk == 0 && kAttnItem <= 256,
              "streaming attention shape");
constexpr int kStreamMaxBatch = 256;

struct StreamItem {
    int b, h, j, p0, p1, nch, pad0, pad1;
    int pg[kItemPages];
};

template <int HD, int G>
__global__ void __launch_bounds__(stream_warps<HD>() * 32, 1)
    ijb_attention_stream_kernel(const __grid_constant__ AttnParams p) {
    constexpr int ST = kStreamStages, QN = kStreamQueue, SW = stream_warps<HD>(), TILE = stream_tile<HD>();
    constexpr int KS = HD / 16, NH = HD / 64;  // k-steps / dim tiles; 128-byte halves of a row
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;

    extern __shared__ uint8_t smem_raw[];
    const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;  // swizzled TMA tiles need 1024-byte alignment
    const uint32_t wtiles = base + static_cast<uint32_t>(warp * ST * 2 * TILE);  // [ST][K, V]
    __shared__ int first_s[kStreamMaxBatch + 1];  // first work item of each token (prefix sums)
    __shared__ int nj_s[kStreamMaxBatch];         // items per kv head of each token
    __shared__ int seq_s[kStreamMaxBatch];
    __shared__ int npos_s[kStreamMaxBatch];
    __shared__ StreamItem q_s[SW][QN];
    __shared__ __align__(8) uint64_t bar[SW][ST];
    __shared__ uint32_t cta_abort;

    if (threadIdx.x == 0) cta_abort = 0u;
    if (lane == 0) {
        for (int st = 0; st < ST; ++st) mbar_init(&bar[warp][st], 1);
        fence_barrier_init();
    }
    pdl_trigger();
    // work items from the step's token metadata (written before the step's first
    // kernel), then wait for the previous kernel (Q and the newest K/V rows)
    if (warp == 0) {
        int run = 0;
        for (int b0 = 0; b0 < p.batch; b0 += 32) {
            const int b = b0 + lane;
            int nj = 0;
            if (b < p.batch) {
                const int n_pos = p.tok_pos[b] + 1;
                nj = (n_pos + kAttnItem - 1) / kAttnItem;
                nj_s[b] = nj;
                npos_s[b] = n_pos;
                seq_s[b] = p.tok_seq[b];
            }
            int v = nj * p.kv_heads;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int n = __shfl_up_sync(0xffffffffu, v, o);
                if (lane >= o) v += n;
            }
            if (b < p.batch) first_s[b + 1] = run + v;
            run += __shfl_sync(0xffffffffu, v, 31);
        }
        if (lane == 0) first_s[0] = 0;
    }
    __syncthreads();
    pdl_wait();
    const int total = first_s[p.batch];
    const int ps = p.page_size;

    // this warp's next item into queue slot `slot` (warp-uniform)
    const int nwarps = static_cast<int>(gridDim.x) * SW;
    bool first = true;
    int pending = 0;  // lane 0: the counter value for the following item (request in flight)
    auto grab = [&](int slot) -> bool {
        int id;
        if (first) {
            id = static_cast<int>(blockIdx.x) * SW + warp;
            first = false;
        } else {
            id = __shfl_sync(0xffffffffu, pending, 0) + nwarps;
        }
        if (id >= total) return false;
        if (lane == 0) pending = atomicAdd(p.work, 1);
        int lo = 0, hi = p.batch - 1;  // last token whose first item is <= id
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (first_s[mid] <= id) lo = mid;
            else hi = mid - 1;
        }
        const int b = lo, r = id - first_s[b], nj = nj_s[b];
        const int p0 = (r % nj) * kAttnItem, p1 = min(npos_s[b], p0 + kAttnItem);
        StreamItem &it = q_s[warp][slot];
        if (lane < (p1 - p0 + ps - 1) / ps)
            it.pg[lane] = p.page_table[static_cast<long>(seq_s[b]) * p.max_pages_per_seq + p0 / ps + lane];
        if (lane == 0) {
            it.b = b;
            it.h = r / nj;
            it.j = r % nj;
            it.p0 = p0;
            it.p1 = p1;
            it.nch = (p1 - p0 + kStreamChunk - 1) / kStreamChunk;
        }
        __syncwarp();
        return true;
    };
    // chunk c of item `it` into stage `stage` (warp-uniform)
    auto issue = [&](const StreamItem &it, int c, int stage) {
        const int t0 = it.p0 + c * kStreamChunk;
        const int npg = (min(kStreamChunk, it.p1 - t0) + ps - 1) / ps;
        const uint32_t kt = wtiles + static_cast<uint32_t>(stage * 2 * TILE), vt = kt + TILE;
        uint64_t *bb = &bar[warp][stage];
        if (lane == 0) mbar_arrive_expect_tx(bb, 2u * npg * ps * 128u * NH);
        __syncwarp();
        if (lane < 2 * npg * NH) {
            // one copy per lane: the 128-byte-wide half lane % NH of page (lane / NH) / 2,
            // K (even (lane / NH)) or V (odd)
            const int hf = lane % NH, kv = (lane / NH) & 1, j = lane / (2 * NH);
            const int page = it.pg[(t0 - it.p0) / ps + j];
            const uint32_t dst = (kv ? vt : kt) + static_cast<uint32_t>(hf * kStreamChunk * 128 + j * ps * 128);
            tma_load_3d(dst, &p.kv_map, 64 * hf, (kv ? p.kv_heads + it.h : it.h) * ps, page, bb);
        }
    };

    int q_head = 0, q_tail = 0;  // queue: items in use / grabbed (running counts)
    int is_item = 0, is_ch = 0;  // issue cursor
    int issued = 0, done = 0, cc = 0;
    bool exhausted = false;
    uint32_t qa[KS][2][2];
    float o[KS][4];  // O^T: dims 16md + gid (+8), heads 2tig (+1)
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
    // keep ST chunks of the warp's stream in flight (warp-uniform)
    auto refill = [&]() {
        while (issued - done < ST) {
            if (is_item == q_tail) {
                if (exhausted) break;
                if (!grab(q_tail % QN)) {
                    exhausted = true;
                    break;
                }
                ++q_tail;
            }
            const StreamItem &it = q_s[warp][is_item % QN];
            if (is_ch == it.nch) {
                ++is_item;
                is_ch = 0;
                continue;
            }
            issue(it, is_ch, issued % ST);
            ++is_ch;
            ++issued;
        }
    };
    // the query of queued item k, raw (the MMA fragments are built when it starts)
    float qv[KS][4];
    int qv_item = -1;
    auto load_q = [&](int k) {
        const StreamItem &it = q_s[warp][k % QN];
        const float *q = p.q + static_cast<long>(it.b) * p.q_stride + static_cast<long>(it.h) * G * HD;
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
            float2 v0 = make_float2(0.f, 0.f), v1 = v0;
            if (gid < G) {
                v0 = *reinterpret_cast<const float2 *>(q + gid * HD + 16 * kk + 2 * tig);
                v1 = *reinterpret_cast<const float2 *>(q + gid * HD + 16 * kk + 8 + 2 * tig);
            }
            qv[kk][0] = v0.x;
            qv[kk][1] = v0.y;
            qv[kk][2] = v1.x;
            qv[kk][3] = v1.y;
        }
        qv_item = k;
    };
    refill();
    while (done < issued) {
        const StreamItem &it = q_s[warp][q_head % QN];
        if (cc == 0) {
            // query fragments of the item's (token, kv head), the MMA's B operand:
            // column gid = head gid (zero for gid >= G), [k-step][hi, lo][b0, b1]
            if (qv_item != q_head) load_q(q_head);
#pragma unroll
            for (int kk = 0; kk < KS; ++kk) {
                const __half2 h0 = __floats2half2_rn(qv[kk][0], qv[kk][1]), h1 = __floats2half2_rn(qv[kk][2], qv[kk][3]);
                const float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
                qa[kk][0][0] = *reinterpret_cast<const uint32_t *>(&h0);
                qa[kk][0][1] = *reinterpret_cast<const uint32_t *>(&h1);
                qa[kk][1][0] = pack_h2(qv[kk][0] - f0.x, qv[kk][1] - f0.y);
                qa[kk][1][1] = pack_h2(qv[kk][2] - f1.x, qv[kk][3] - f1.y);
            }
#pragma unroll
            for (int md = 0; md < KS; ++md) o[md][0] = o[md][1] = o[md][2] = o[md][3] = 0.f;
            m[0] = m[1] = -INFINITY;
            l[0] = l[1] = 0.f;
        }
        const int stage = done % ST;
        mbar_wait_bounded(&bar[warp][stage], (done / ST) & 1, p.status, &cta_abort);
        const uint32_t kt = wtiles + static_cast<uint32_t>(stage * 2 * TILE), vt = kt + TILE;
        const int t0 = it.p0 + cc * kStreamChunk;
        attn_chunk_t<HD, kStreamChunk / 16>(kt, vt, min(kStreamChunk, it.p1 - t0), p.scale, qa, o, m, l, lane);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic accesses before TMA refills the stage
        __syncwarp();
        ++done;
        refill();  // the used stage goes back into flight before anything else
        if (++cc < it.nch) continue;

        // ---- the item is finished: output, or its state for the merge
        cc = 0;
        const int b = it.b, h = it.h, j = it.j, nsplit = nj_s[b];
        ++q_head;
        if (q_head < q_tail) load_q(q_head);  // the next item's query loads during what follows
        if (nsplit == 1) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                if (2 * tig + e >= G) continue;
                float *out = p.out + static_cast<long>(b) * p.out_stride + (static_cast<long>(h) * G + 2 * tig + e) * HD;
                const float inv = 1.f / l[e];
#pragma unroll
                for (int md = 0; md < KS; ++md) {
                    out[16 * md + gid] = o[md][e] * inv;
                    out[16 * md + gid + 8] = o[md][2 + e] * inv;
                }
            }
            continue;
        }
        float *part = p.partial + ((static_cast<long>(b) * p.heads + h * G) * p.max_splits) * (HD + 2);
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            if (2 * tig + e >= G) continue;
            float *rec = part + (static_cast<long>(2 * tig + e) * p.max_splits + j) * (HD + 2);
            if (gid == 0) {
                rec[0] = m[e];
                rec[1] = l[e];
            }
#pragma unroll
            for (int md = 0; md < KS; ++md) {
                rec[2 + 16 * md + gid] = o[md][e];
                rec[2 + 16 * md + gid + 8] = o[md][2 + e];
            }
        }
    }
    // every warp of the grid has taken its last item once all CTAs get here:
    // the last CTA resets the item counter for the next launch
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(p.work + 1, 1) == static_cast<int>(gridDim.x) - 1) {
            p.work[0] = 0;
            p.work[1] = 0;
            __threadfence();
        }
    }
}

// One CTA per token.  Each warp merges the items of one kv head of a token
// whose sequence spans more than one item: lane s holds the max and sum of
// items s and s + 32 (at most 64 items), the weights exp(m_s - M) come from a warp max, then each
// lane sums two output dims over the items, KB items of every head per round
// of loads.  When the O projection runs on the tensor cores (x16 set), the CTA
// then builds the token's fp16 activation row for it (mma_prep_token), which
// takes the place of the projection's own prep launch.
template <int HD, int G>
__global__ void __launch_bounds__(256) ijb_attention_finish_kernel(const __grid_constant__ AttnParams p) {
    constexpr int KB = G * HD >= 512 ? 4 : 8, NH = HD / 64;  // items per round of loads; dim pairs per lane
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int b = blockIdx.x;
    const int nsplit = b < p.batch ? (p.tok_pos[b] + kAttnItem) / kAttnItem : 0;
    for (int h = warp; nsplit > 1 && h < p.kv_heads; h += 8) {
        const float *part = p.partial + ((static_cast<long>(b) * p.heads + h * G) * p.max_splits) * (HD + 2);
        // lane s holds items s and s + 32 (up to 64 items)
        float fg[G], fg2[G], Lg[G];
        float2 O[G][NH];  // dims 2 lane + 64 hf (+1)
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float *recs = part + static_cast<long>(g) * p.max_splits * (HD + 2);
            const float ms = lane < nsplit ? recs[lane * (HD + 2)] : -INFINITY;
            const float ls = lane < nsplit ? recs[lane * (HD + 2) + 1] : 0.f;
            const float ms2 = lane + 32 < nsplit ? recs[(lane + 32) * (HD + 2)] : -INFINITY;
            const float ls2 = lane + 32 < nsplit ? recs[(lane + 32) * (HD + 2) + 1] : 0.f;
            const float M = warp_max(fmaxf(ms, ms2));
            fg[g] = lane < nsplit ? __expf(ms - M) : 0.f;
            fg2[g] = lane + 32 < nsplit ? __expf(ms2 - M) : 0.f;
            Lg[g] = warp_sum(fg[g] * ls + fg2[g] * ls2);
#pragma unroll
            for (int hf = 0; hf < NH; ++hf) O[g][hf] = make_float2(0.f, 0.f);
        }
        for (int k0 = 0; k0 < nsplit; k0 += KB) {
            float2 v[G][KB][NH];
#pragma unroll
            for (int g = 0; g < G; ++g)
#pragma unroll
                for (int k = 0; k < KB; ++k)
#pragma unroll
                    for (int hf = 0; hf < NH; ++hf)
                        v[g][k][hf] = k0 + k < nsplit
                                          ? reinterpret_cast<const float2 *>(
                                                part + (static_cast<long>(g) * p.max_splits + k0 + k) * (HD + 2) + 2)
                                                [lane + 32 * hf]
                                          : make_float2(0.f, 0.f);
#pragma unroll
            for (int g = 0; g < G; ++g)
#pragma unroll
                for (int k = 0; k < KB; ++k) {
                    const float fk = __shfl_sync(0xffffffffu, k0 + k < 32 ? fg[g] : fg2[g], (k0 + k) & 31);
#pragma unroll
                    for (int hf = 0; hf < NH; ++hf) {
                        O[g][hf].x = fmaf(v[g][k][hf].x, fk, O[g][hf].x);
                        O[g][hf].y = fmaf(v[g][k][hf].y, fk, O[g][hf].y);
                    }
                }
        }
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float *out = p.out + static_cast<long>(b) * p.out_stride + (static_cast<long>(h) * G + g) * HD;
#pragma unroll
            for (int hf = 0; hf < NH; ++hf)
                *reinterpret_cast<float2 *>(out + 2 * lane + 64 * hf) =
                    make_float2(O[g][hf].x / Lg[g], O[g][hf].y / Lg[g]);
        }
    }
    if (p.x16) {
        __syncthreads();  // the merged rows are read back below
        mma_prep_token(p.out, p.out_stride, nullptr, 0.f, p.heads * HD, p.batch, b, p.n_pad, p.use_dp4a, p.x16, p.x_inv);
    }
}

template <int HD, int G>
static cudaError_t launch_attn_stream(const AttnParams &p, cudaStream_t stream, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.num_ctas);
    cfg.blockDim = dim3(stream_warps<HD>() * 32);
    cfg.dynamicSmemBytes = stream_smem<HD>();
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, ijb_attention_stream_kernel<HD, G>, p);
    if (e != cudaSuccess) return e;
    cfg.gridDim = dim3(p.x16 ? p.n_pad : p.batch);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = 0;
    return cudaLaunchKernelEx(&cfg, ijb_attention_finish_kernel<HD, G>, p);
}

typedef CUresult (*EncodeTiledFnA)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int attention_make_kv_map(CUtensorMap *map, const void *layer_base, int head_dim, int kv_heads, int page_size,
                          long page_stride_elems, long num_pages) {
    if ((head_dim != 64 && head_dim != 128) || (reinterpret_cast<uintptr_t>(layer_base) & 15)) return -1;
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
    // one 128-byte-wide box (64 fp16) per copy: the 128-byte swizzle span; a
    // head_dim-128 row is fetched as two boxes at x = 0 and x = 64
    cuuint32_t box[3] = {64, static_cast<cuuint32_t>(page_size), 1};
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
    return cudaLaunchKernelEx(&cfg, ijb_attention_kernel<HD, G, KT>, p);
}

template <typename KT>
static cudaError_t attention_launch_t(const AttnParams &p, dim3 grid, cudaStream_t stream, bool pdl) {
    const int G = p.heads / p.kv_heads;
    if (p.head_dim == 64) {
        if (G == 4) return launch_attn<64, 4, KT>(p, grid, stream, pdl);
        if (G == 8) return launch_attn<64, 8, KT>(p, grid, stream, pdl);
        if (G == 2) return launch_attn<64, 2, KT>(p, grid, stream, pdl);
        if (G == 1) return launch_attn<64, 1, KT>(p, grid, stream, pdl);
        if (G == 3) return launch_attn<64, 3, KT>(p, grid, stream, pdl);
        if (G == 6) return launch_attn<64, 6, KT>(p, grid, stream, pdl);
    } else if (p.head_dim == 128) {
        if (G == 4) return launch_attn<128, 4, KT>(p, grid, stream, pdl);
        if (G == 8) return launch_attn<128, 8, KT>(p, grid, stream, pdl);
        if (G == 2) return launch_attn<128, 2, KT>(p, grid, stream, pdl);
        if (G == 1) return launch_attn<128, 1, KT>(p, grid, stream, pdl);
        if (G == 3) return launch_attn<128, 3, KT>(p, grid, stream, pdl);
        if (G == 6) return launch_attn<128, 6, KT>(p, grid, stream, pdl);
    }
    return cudaErrorInvalidValue;
}

// The streaming kernel serves fp16 caches with head_dim 64 or 128 up to 64 work items
// (8192 positions) per sequence and kStreamMaxBatch tokens; anything else, or a
// G it is not built for, goes to the CUDA-core split kernel.
static bool stream_path(const AttnParams &p) {
    const int G = p.kv_heads > 0 ? p.heads / p.kv_heads : 0;
    return p.has_map && (p.head_dim == 64 || p.head_dim == 128) && !p.kv_f32 && p.work && p.num_ctas >= 1 && p.batch <= kStreamMaxBatch &&
           p.max_splits <= 64 && (G == 1 || G == 2 || G == 3 || G == 4 || G == 6 || G == 8) && G * p.kv_heads == p.heads &&
           p.page_size <= kStreamChunk && kStreamChunk % p.page_size == 0;  // a chunk is whole pages
}

int attention_split_len() { return kAttnSplit; }
int attention_split_len_min() { return kAttnItem; }
int attention_kernels(const AttnParams &p) { return stream_path(p) ? 2 : 1; }
int attention_item_len() { return kAttnItem; }

// Opts every instance in to its K/V tile shared memory on the current device
// (done once per device at engine creation, outside any graph capture).
template <int HD, int G, typename KT>
static cudaError_t set_attr() {
    const int smem = attn_smem<HD, KT>();
    return cudaFuncSetAttribute(ijb_attention_kernel<HD, G, KT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
}

template <typename KT>
static cudaError_t set_attrs_t() {
    cudaError_t e;
    if ((e = set_attr<64, 1, KT>()) || (e = set_attr<64, 2, KT>()) || (e = set_attr<64, 4, KT>()) ||
        (e = set_attr<64, 8, KT>()) || (e = set_attr<128, 1, KT>()) || (e = set_attr<128, 2, KT>()) ||
        (e = set_attr<128, 4, KT>()) || (e = set_attr<128, 8, KT>()) || (e = set_attr<64, 3, KT>()) ||
        (e = set_attr<64, 6, KT>()) || (e = set_attr<128, 3, KT>()) || (e = set_attr<128, 6, KT>()))
        return e;
    return cudaSuccess;
}

template <int HD>
static cudaError_t set_stream_attrs() {
    cudaError_t e;
    const int smem = stream_smem<HD>();
    if ((e = cudaFuncSetAttribute(ijb_attention_stream_kernel<HD, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) ||
        (e = cudaFuncSetAttribute(ijb_attention_stream_kernel<HD, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) ||
        (e = cudaFuncSetAttribute(ijb_attention_stream_kernel<HD, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) ||
        (e = cudaFuncSetAttribute(ijb_attention_stream_kernel<HD, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) ||
        (e = cudaFuncSetAttribute(ijb_attention_stream_kernel<HD, 6>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) ||
        (e = cudaFuncSetAttribute(ijb_attention_stream_kernel<HD, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)))
        return e;
    return cudaSuccess;
}

cudaError_t attention_prepare() {
    cudaError_t e;
    if ((e = set_stream_attrs<64>()) || (e = set_stream_attrs<128>())) return e;
    e = set_attrs_t<__half>();
    return e != cudaSuccess ? e : set_attrs_t<float>();
}

cudaError_t attention_launch(const AttnParams &p, cudaStream_t stream, bool pdl) {
    // the split kernel's split length: kAttnItem..kAttnSplit positions, whole chunks and
    // pages, so that split indexes stay below max_splits (counted in kAttnItem items)
    if (p.split_len < kAttnItem || p.split_len > kAttnSplit || p.split_len % kAttnChunk || p.page_size < 8 ||
        p.page_size > 32 || 32 % p.page_size || p.split_len % p.page_size)
        return cudaErrorInvalidValue;
    if (p.max_splits * kAttnItem < 1) return cudaErrorInvalidValue;
    if (stream_path(p)) {
        if (p.x16 && (p.n_pad < p.batch || p.n_pad > kMmaMaxN || p.n_pad % 16 || p.heads * p.head_dim > kMaxCols))
            return cudaErrorInvalidValue;
        const int G = p.heads / p.kv_heads;
        if (p.head_dim == 64) {
            if (G == 4) return launch_attn_stream<64, 4>(p, stream, pdl);
            if (G == 8) return launch_attn_stream<64, 8>(p, stream, pdl);
            if (G == 2) return launch_attn_stream<64, 2>(p, stream, pdl);
            if (G == 1) return launch_attn_stream<64, 1>(p, stream, pdl);
            if (G == 3) return launch_attn_stream<64, 3>(p, stream, pdl);
            if (G == 6) return launch_attn_stream<64, 6>(p, stream, pdl);
        } else {
            if (G == 3) return launch_attn_stream<128, 3>(p, stream, pdl);
            if (G == 4) return launch_attn_stream<128, 4>(p, stream, pdl);
            if (G == 8) return launch_attn_stream<128, 8>(p, stream, pdl);
            if (G == 2) return launch_attn_stream<128, 2>(p, stream, pdl);
            if (G == 1) return launch_attn_stream<128, 1>(p, stream, pdl);
            if (G == 6) return launch_attn_stream<128, 6>(p, stream, pdl);
        }
    }
    // one CTA per split of kAttnSplit positions (the partial records are kept
    // at kAttnItem granularity, so max_splits counts items)
    dim3 grid((p.max_splits * kAttnItem + p.split_len - 1) / p.split_len, p.kv_heads, p.batch);
    return p.kv_f32 ? attention_launch_t<float>(p, grid, stream, pdl) : attention_launch_t<__half>(p, grid, stream, pdl);
}

}  // namespace ijb
