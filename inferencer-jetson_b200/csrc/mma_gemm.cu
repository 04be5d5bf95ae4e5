// Tensor-core (tcgen05) quantised GEMM for packed steps of 16..64 tokens.
//
// Replaces, for a ragged batch, what the reference does one token at a time
// (gemv_batch_dp4a, qkv_batch_cuda, gate_up_batch_cuda, inferencer.cu:678-751):
// every weight is read from HBM once per step instead of once per token.
//
// One persistent CTA per SM walks 128-row tiles of the launch's matrices
// (a gate/up tile is 64 gate rows + the same 64 up rows).  Warp roles:
//   * warp 0, lane 0: TMA producer.  Per 256-wide block column of a tile it
//     loads the raw quantised bytes as 2-D TMA boxes (Q4_K: [128 rows][144 B];
//     Q6_K: the 208-byte block bodies and the unit's 16 bytes of d) into a
//     3-stage ring, and per 128-wide half the prepared fp16 activation chunk
//     into the fp16 stage the MMA will read.
//   * warps 6..13: dequantise a raw block column into two fp16 K-major
//     tiles [128 rows][128 K] in the UMMA canonical no-swizzle layout.  The
//     fp32 weight is computed as the reference does (q4_value / q6_value,
//     inferencer.cu:454-487, exact products, one rounding for Q4_K), times the
//     matrix's power-of-two scale, then rounded to fp16.
//   * warp 1, lane 0: issues tcgen05.mma (kind::f16, M=128, N = tokens
//     rounded up to 16, K=16) into an fp32 accumulator in TMEM, double
//     buffered across tiles; tcgen05.commit releases fp16 stages and signals
//     finished accumulators.
//   * warps 2..5 (one per TMEM lane quadrant): read the accumulator with
//     tcgen05.ld, undo the two power-of-two scales and apply the fused
//     epilogue of the GEMV (store, residual add, RoPE + paged K write, V write,
//     SiLU * up, logits + argmax key).
// All waits are bounded; TMEM is always released before the CTA exits.
#include <cmath>
#include <cstdio>
#include <cstring>

#include "common.cuh"
#include "mma_gemm.cuh"

namespace ijb {

constexpr int kKChunk = 128;  // K per fp16 stage (half a super-block)
constexpr int kRawStages = 3;
constexpr int kF16Stages = 2;  // dequantised weight stages
constexpr int kXStages = 3;    // activation stages
constexpr int kRawStageBytes = 128 * 208 + 128 * 16;  // Q6_K bodies + d (Q4_K uses 128 * 144)
constexpr int kQ6DOff = 128 * 208;                    // d box within a Q6_K raw stage
constexpr int kW16Bytes = kMmaTileM * kKChunk * 2;    // 32 KB
constexpr int kX16Bytes = kMmaMaxN * kKChunk * 2;     // 16 KB
constexpr int kExchStride = kMmaMaxN + 1;             // floats per row of the SiLU exchange buffer
constexpr int kProducerWarp = 0, kMmaWarp = 1, kEpiWarp0 = 2, kConvWarp0 = 6, kConvWarps = 8;
constexpr int kMmaThreads = (kConvWarp0 + kConvWarps) * 32;

struct MmaSmem {
    int raw, w16, x16, exch, bars, tmem, total;
};

__host__ __device__ constexpr MmaSmem mma_smem() {
    MmaSmem L{};
    int off = 0;
    L.raw = off;
    off += kRawStages * kRawStageBytes;
    L.w16 = off;
    off += kF16Stages * kW16Bytes;
    L.x16 = off;
    off += kXStages * kX16Bytes;
    L.exch = off;
    off += 64 * kExchStride * 4;
    off = (off + 7) / 8 * 8;
    L.bars = off;
    off += 20 * 8;
    L.tmem = off;
    off += 16;
    L.total = (off + 127) / 128 * 128;
    return L;
}

int mma_smem_bytes() { return mma_smem().total; }

// ------------------------------------------------------------ PTX helpers --

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// UMMA shared-memory descriptor, K-major, no swizzle: core matrices of 8
// rows x 16 bytes; LBO = byte distance between the two core matrices of one
// K=16 step, SBO = byte distance between 8-row groups.
__device__ __forceinline__ uint64_t umma_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((addr & 0x3FFFFu) >> 4);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
    d |= 1ull << 46;  // descriptor version for sm_100
    return d;         // base offset 0, legacy LBO mode, layout type 0 (no swizzle)
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// ------------------------------------------------------------ tile helpers --

__device__ __forceinline__ int mma_seg_of_tile(const MmaParams &p, int t) {
    int s = 0;
#pragma unroll
    for (int i = 1; i < kMaxSegs; ++i)
        if (i < p.nseg && t >= p.seg[i].tile0) s = i;
    return s;
}

// Segment row held by tile lane r (0..127), and whether it exists.
__device__ __forceinline__ int tile_row(const MmaSeg &s, int lt, int r, bool &valid) {
    int row;
    if (s.w1 >= 0) row = lt * 64 + (r & 63);
    else row = lt * 128 + r;
    valid = row < s.rows;
    return row;
}

// ------------------------------------------------------------- dequantise --

// Q4_K half h of a raw block column -> fp16 K-major tile.  Thread (row, q)
// covers sub-blocks 2(2h+q) (low nibbles) and 2(2h+q)+1 (high nibbles).
__device__ __forceinline__ void convert_q4(const uint8_t *raw, uint8_t *w16, int row, int q, int h, float scale) {
    const uint8_t *bp = raw + row * 144;
    const uint4 hdr = *reinterpret_cast<const uint4 *>(bp);
    const int gq = 2 * h + q;
    const uint4 qa = *reinterpret_cast<const uint4 *>(bp + 16 + gq * 32);
    const uint4 qb = *reinterpret_cast<const uint4 *>(bp + 32 + gq * 32);
    const float d = half_bits_to_float(hdr.x & 0xffff), dmin = half_bits_to_float(hdr.x >> 16);
    auto byte = [&](int k) -> int {
        const uint32_t w = k < 4 ? hdr.y : (k < 8 ? hdr.z : hdr.w);
        return (w >> ((k & 3) * 8)) & 255;
    };
    int sc[2], m[2];
#pragma unroll
    for (int t = 0; t < 2; ++t) {
        const int j = 2 * gq + t;
        if (j < 4) {
            sc[t] = byte(j) & 63;
            m[t] = byte(j + 4) & 63;
        } else {
            sc[t] = (byte(j + 4) & 15) | ((byte(j - 4) >> 6) << 4);
            m[t] = (byte(j + 4) >> 4) | ((byte(j) >> 6) << 4);
        }
    }
    // w = (d*sc)*q - dmin*m: d*sc and its product with q are exact, so one
    // fused multiply-add rounds exactly like the reference; the power-of-two
    // scale is exact too.
    const float s1[2] = {d * static_cast<float>(sc[0]) * scale, d * static_cast<float>(sc[1]) * scale};
    const float s2[2] = {dmin * static_cast<float>(m[0]) * scale, dmin * static_cast<float>(m[1]) * scale};
    const uint32_t words[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    uint8_t *dst = w16 + (row >> 3) * 2048 + (row & 7) * 16;
#pragma unroll
    for (int j = 0; j < 8; ++j) {  // k-core q*8 + j: positions 8j..8j+7 of the 64
        const int t = j >> 2;      // 0: low nibbles (sub 2gq), 1: high nibbles (sub 2gq+1)
        const uint32_t w0 = words[(j & 3) * 2], w1 = words[(j & 3) * 2 + 1];
        const uint32_t n0 = t ? (w0 >> 4) & 0x0F0F0F0Fu : w0 & 0x0F0F0F0Fu;
        const uint32_t n1 = t ? (w1 >> 4) & 0x0F0F0F0Fu : w1 & 0x0F0F0F0Fu;
        float f[8];
        f[0] = fmaf(byte_to_float(n0, 0x7440), s1[t], -s2[t]);
        f[1] = fmaf(byte_to_float(n0, 0x7441), s1[t], -s2[t]);
        f[2] = fmaf(byte_to_float(n0, 0x7442), s1[t], -s2[t]);
        f[3] = fmaf(byte_to_float(n0, 0x7443), s1[t], -s2[t]);
        f[4] = fmaf(byte_to_float(n1, 0x7440), s1[t], -s2[t]);
        f[5] = fmaf(byte_to_float(n1, 0x7441), s1[t], -s2[t]);
        f[6] = fmaf(byte_to_float(n1, 0x7442), s1[t], -s2[t]);
        f[7] = fmaf(byte_to_float(n1, 0x7443), s1[t], -s2[t]);
        const uint4 o = make_uint4(pack_half2(f[0], f[1]), pack_half2(f[2], f[3]), pack_half2(f[4], f[5]),
                                   pack_half2(f[6], f[7]));
        *reinterpret_cast<uint4 *>(dst + (q * 8 + j) * 128) = o;
    }
}

// Q6_K half h (= the block's 128-weight group g) of a raw block column ->
// fp16 K-major tile.  Thread (row, q) is the block-body lane j = 2h + q:
// positions part*32 + 16q + 0..15 of the group's four parts.
__device__ __forceinline__ void convert_q6(const uint8_t *raw, uint8_t *w16, int row, int q, int h, int lb,
                                           float scale) {
    const uint8_t *body = raw + row * 208;
    const int j = 2 * h + q;
    const uint4 la = reinterpret_cast<const uint4 *>(body)[j];
    const uint4 lbq = reinterpret_cast<const uint4 *>(body + 64)[j];
    const uint4 hh = reinterpret_cast<const uint4 *>(body + 128)[j];
    const uint32_t sc4 = reinterpret_cast<const uint32_t *>(body + 192)[j];
    const float d = half_bits_to_float(*reinterpret_cast<const uint16_t *>(raw + kQ6DOff + row * 16 + lb * 2));
    const uint32_t A[4] = {la.x, la.y, la.z, la.w}, Bw[4] = {lbq.x, lbq.y, lbq.z, lbq.w};
    const uint32_t H[4] = {hh.x, hh.y, hh.z, hh.w};
    uint8_t *dst = w16 + (row >> 3) * 2048 + (row & 7) * 16;
#pragma unroll
    for (int pt = 0; pt < 4; ++pt) {
        // d * scale is exact in fp32 (11 + 8 bits), and so is its product with q
        const float s = d * static_cast<float>(static_cast<int8_t>((sc4 >> (8 * pt)) & 255)) * scale;
#pragma unroll
        for (int half = 0; half < 2; ++half) {  // k-core pt*4 + 2q + half: 8 positions
            uint32_t qw[2];
#pragma unroll
            for (int w = 0; w < 2; ++w) {
                const int wi = half * 2 + w;
                const uint32_t lo = (pt & 1) ? Bw[wi] : A[wi];
                const uint32_t low = pt < 2 ? (lo & 0x0F0F0F0Fu) : ((lo >> 4) & 0x0F0F0F0Fu);
                qw[w] = low | (((H[wi] >> (2 * pt)) & 0x03030303u) << 4);  // codes 0..63
            }
            float f[8];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                f[e] = (__int_as_float(__byte_perm(qw[0], 0x4B000000u, 0x7440 + e)) - 8388640.0f) * s;
                f[4 + e] = (__int_as_float(__byte_perm(qw[1], 0x4B000000u, 0x7440 + e)) - 8388640.0f) * s;
            }
            const uint4 o = make_uint4(pack_half2(f[0], f[1]), pack_half2(f[2], f[3]), pack_half2(f[4], f[5]),
                                       pack_half2(f[6], f[7]));
            *reinterpret_cast<uint4 *>(dst + (pt * 4 + 2 * q + half) * 128) = o;
        }
    }
}

// --------------------------------------------------------------- epilogue --

__device__ void mma_epilogue_value(const MmaParams &p, const MmaSeg &s, int row, bool valid, int n, float y,
                                   float partner) {
    switch (s.epi) {
        case kEpiStore:
            if (valid) s.out[n * s.out_stride + s.row_offset + row] = y;
            break;
        case kEpiAdd:
            if (valid) s.out[n * s.out_stride + s.row_offset + row] += y;
            break;
        case kEpiRopeQ:
        case kEpiRopeKCache: {
            if (!valid) break;
            // pair (2j, 2j+1) rotated with frequency j % (head_dim/2) (rope_cuda, inferencer.cu:906-917)
            const int j = row >> 1, f = j % p.half_head;
            const int pos = p.tok_pos[n];
            const float c = p.rope_cos[pos * p.half_head + f], sn = p.rope_sin[pos * p.half_head + f];
            const bool even = (row & 1) == 0;
            const float a = even ? y : partner, b = even ? partner : y;
            const float r = even ? a * c - b * sn : a * sn + b * c;
            if (s.epi == kEpiRopeQ) {
                s.out[n * s.out_stride + s.row_offset + row] = r;
            } else {
                const int slot = p.tok_slot[n];
                const int page = slot / p.page_size, t = slot % p.page_size;
                const int head = row / p.head_dim, dd = row % p.head_dim;
                const long off = static_cast<long>(page) * p.page_stride +
                                 (static_cast<long>(head) * p.page_size + t) * p.head_dim + dd;
                if (p.kv_f32) static_cast<float *>(p.k_cache)[off] = r;
                else static_cast<__half *>(p.k_cache)[off] = __float2half_rn(r);
            }
            break;
        }
        case kEpiVCache: {
            if (!valid) break;
            const int slot = p.tok_slot[n];
            const int page = slot / p.page_size, t = slot % p.page_size;
            const int head = row / p.head_dim, dd = row % p.head_dim;
            const long off = static_cast<long>(page) * p.page_stride +
                             (static_cast<long>(head) * p.page_size + t) * p.head_dim + dd;
            if (p.kv_f32) static_cast<float *>(p.v_cache)[off] = y;
            else static_cast<__half *>(p.v_cache)[off] = __float2half_rn(y);
            break;
        }
        default:
            break;
    }
}

// ----------------------------------------------------------------- kernel --

// Applies a tile row's epilogue from the split-K partials of its tile, summed
// in part order (so the result does not depend on which part finished last).
// Eight tokens at a time, so each part contributes 8 (or 16) independent loads.
__device__ void mma_reduced_epilogue(const MmaParams &p, const MmaSeg &sg, const float *tile_part, int r, int row,
                                     bool valid, int lane) {
    const long part_stride = static_cast<long>(p.n_pad) * 128;
    const bool silu = sg.epi == kEpiSiluPair;
    const bool pairs = sg.epi == kEpiRopeQ || sg.epi == kEpiRopeKCache;
    const int rz = silu ? (r + 64) & 127 : (r ^ 1);  // the row whose sum the epilogue also needs
    for (int n0 = 0; n0 < p.batch; n0 += 8) {
        float y[8], z[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) y[k] = z[k] = 0.f;
#pragma unroll 4
        for (int s = 0; s < p.ksplit; ++s) {
            const float *src = tile_part + s * part_stride + n0 * 128;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                y[k] += __ldcg(src + k * 128 + r);
                if (silu || pairs) z[k] += __ldcg(src + k * 128 + rz);
            }
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int n = n0 + k;
            if (silu) {
                if (r < 64 && valid && n < p.batch)
                    sg.out[n * sg.out_stride + sg.row_offset + row] = y[k] / (1.f + __expf(-y[k])) * z[k];
            } else if (sg.epi == kEpiLogitsArgmax) {
                const bool ok = valid && n < p.batch;
                if (ok) sg.out[n * sg.out_stride + sg.row_offset + row] = y[k];
                unsigned long long key = ok ? argmax_key(y[k], sg.row_offset + row) : 0ull;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
                    key = other > key ? other : key;
                }
                if (lane == 0 && key) atomicMax(p.argmax_keys + n, key);
            } else if (n < p.batch) {
                mma_epilogue_value(p, sg, row, valid, n, y[k], z[k]);
            }
        }
    }
}

__global__ void __launch_bounds__(kMmaThreads, 1) mma_gemm_kernel(const __grid_constant__ MmaParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    constexpr MmaSmem L = mma_smem();
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bars);
    uint64_t *full_raw = bars, *empty_raw = bars + 3, *full_w16 = bars + 6, *empty_w16 = bars + 8;
    uint64_t *full_x = bars + 10, *empty_x = bars + 13, *acc_full = bars + 16, *acc_empty = bars + 18;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L.tmem);
    uint32_t *cta_abort = tmem_slot + 1;
    int *last_flag = reinterpret_cast<int *>(tmem_slot + 2);
    float *exch = reinterpret_cast<float *>(smem + L.exch);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb = p.cols / 256;
    const int n_pad = p.n_pad;
    const int total_units = p.total_tiles * p.ksplit;
    const uint32_t tmem_cols = n_pad * 2 <= 32 ? 32 : (n_pad * 2 <= 64 ? 64 : 128);

    if (threadIdx.x == 0) {
        *cta_abort = 0u;
        for (int i = 0; i < kRawStages; ++i) {
            mbar_init(full_raw + i, 1);
            mbar_init(empty_raw + i, kConvWarps);
        }
        for (int i = 0; i < kF16Stages; ++i) {
            mbar_init(full_w16 + i, kConvWarps);
            mbar_init(empty_w16 + i, 1);
        }
        for (int i = 0; i < kXStages; ++i) {
            mbar_init(full_x + i, 1);
            mbar_init(empty_x + i, 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(acc_full + i, 1);
            mbar_init(acc_empty + i, 4);
        }
        fence_barrier_init();
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(tmem_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_trigger();

    if (warp == kProducerWarp) {
        if (lane == 0) {
            uint32_t rc = 0, xc = 0;
            const uint32_t xbytes = static_cast<uint32_t>(n_pad) * kKChunk * 2;
            bool waited = false;
            for (int u = blockIdx.x; u < total_units; u += gridDim.x) {
                const int t = u / p.ksplit, sp = u % p.ksplit;
                const MmaSeg &sg = p.seg[mma_seg_of_tile(p, t)];
                const int lt = t - sg.tile0;
                const bool pair = sg.w1 >= 0;
                const int y0 = pair ? lt * 64 : lt * 128;
                const int b0 = sp * p.bps, b1 = min(nb, b0 + p.bps);
                for (int b = b0; b < b1; ++b) {
                    const int r = rc % kRawStages;
                    if (rc >= kRawStages)
                        mbar_wait_bounded(empty_raw + r, ((rc / kRawStages) - 1) & 1, p.status, cta_abort);
                    uint8_t *dst = smem + L.raw + r * kRawStageBytes;
                    if (sg.type == kQ4K) {
                        mbar_arrive_expect_tx(full_raw + r, 128 * 144);
                        tma_load_2d(dst, &p.w[sg.w0].body, b * 144, y0, full_raw + r);
                        if (pair) tma_load_2d(dst + 64 * 144, &p.w[sg.w1].body, b * 144, y0, full_raw + r);
                    } else {
                        const int uu = b / kUnitBlocks, lb = b % kUnitBlocks;
                        const int n_u = min(kUnitBlocks, nb - uu * kUnitBlocks);
                        const int xb = uu * q6_unit_bytes(kUnitBlocks) + lb * 208;
                        const int xd = uu * q6_unit_bytes(kUnitBlocks) + n_u * 208;
                        mbar_arrive_expect_tx(full_raw + r, kRawStageBytes);
                        tma_load_2d(dst, &p.w[sg.w0].body, xb, y0, full_raw + r);
                        tma_load_2d(dst + kQ6DOff, &p.w[sg.w0].dvec, xd, y0, full_raw + r);
                        if (pair) {
                            tma_load_2d(dst + 64 * 208, &p.w[sg.w1].body, xb, y0, full_raw + r);
                            tma_load_2d(dst + kQ6DOff + 64 * 16, &p.w[sg.w1].dvec, xd, y0, full_raw + r);
                        }
                    }
                    ++rc;
                    if (!waited) {  // the activation is written by the previous kernel
                        pdl_wait();
                        waited = true;
                    }
                    for (int h = 0; h < 2; ++h) {
                        const int xs = xc % kXStages;
                        if (xc >= kXStages) mbar_wait_bounded(empty_x + xs, ((xc / kXStages) - 1) & 1, p.status, cta_abort);
                        mbar_arrive_expect_tx(full_x + xs, xbytes);
                        bulk_g2s(smem + L.x16 + xs * kX16Bytes, p.x16 + static_cast<long>(2 * b + h) * xbytes, xbytes,
                                 full_x + xs);
                        ++xc;
                    }
                }
            }
            if (!waited) pdl_wait();
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            // D (fp32) [128 x n_pad] = A (fp16, K-major) * B (fp16, K-major)^T
            const uint32_t idesc = (1u << 4) | (static_cast<uint32_t>(n_pad >> 3) << 17) | (8u << 24);
            uint32_t fc = 0, xc = 0, i = 0;
            for (int u = blockIdx.x; u < total_units; u += gridDim.x, ++i) {
                const int sp = u % p.ksplit;
                const int b0 = sp * p.bps, b1 = min(nb, b0 + p.bps);
                const int a = i & 1;
                if (i >= 2) mbar_wait_bounded(acc_empty + a, ((i >> 1) - 1) & 1, p.status, cta_abort);
                tc_fence_after();
                const uint32_t dcol = tmem_base + static_cast<uint32_t>(a * n_pad);
                for (int b = b0; b < b1; ++b) {
                    for (int h = 0; h < 2; ++h) {
                        const int f = fc % kF16Stages, xs = xc % kXStages;
                        mbar_wait_bounded(full_w16 + f, (fc / kF16Stages) & 1, p.status, cta_abort);
                        mbar_wait_bounded(full_x + xs, (xc / kXStages) & 1, p.status, cta_abort);
                        tc_fence_after();
                        const uint32_t wa = smem_u32(smem + L.w16 + f * kW16Bytes);
                        const uint32_t xa = smem_u32(smem + L.x16 + xs * kX16Bytes);
#pragma unroll
                        for (int kk = 0; kk < kKChunk / 16; ++kk) {
                            umma_f16(dcol, umma_desc(wa + kk * 256, 128, 2048), umma_desc(xa + kk * 256, 128, 2048),
                                     idesc, (b != b0 || h || kk) ? 1u : 0u);
                        }
                        umma_commit(empty_w16 + f);
                        umma_commit(empty_x + xs);
                        ++fc;
                        ++xc;
                    }
                }
                umma_commit(acc_full + a);
            }
        }
    } else if (warp < kConvWarp0) {
        // ---------------------------------------------------------- epilogue
        const int quad = warp & 3;  // TMEM lanes [32*quad, 32*quad + 32)
        const int r = quad * 32 + lane;
        pdl_wait();
        uint32_t i = 0;
        for (int u = blockIdx.x; u < total_units; u += gridDim.x, ++i) {
            const int t = u / p.ksplit, sp = u % p.ksplit;
            const MmaSeg &sg = p.seg[mma_seg_of_tile(p, t)];
            const int lt = t - sg.tile0;
            const int a = i & 1;
            mbar_wait_bounded(acc_full + a, (i >> 1) & 1, p.status, cta_abort);
            tc_fence_after();
            bool valid;
            const int row = tile_row(sg, lt, r, valid);
            const float wscale = ldexpf(1.0f, -p.w[r >= 64 && sg.w1 >= 0 ? sg.w1 : sg.w0].scale_exp);
            const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + a * n_pad;
            if (p.ksplit > 1) {
                // write this part's values; the last part of the tile reduces
                float *mine = p.partial + (static_cast<long>(t) * p.ksplit + sp) * n_pad * 128;
                for (int c0 = 0; c0 < n_pad; c0 += 16) {
                    float v[16];
                    tmem_ld16(taddr + c0, v);
#pragma unroll
                    for (int k = 0; k < 16; ++k) __stcg(mine + (c0 + k) * 128 + r, v[k] * wscale * p.x_inv[c0 + k]);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(acc_empty + a);
                __threadfence();
                named_bar_sync(1, 128);
                if (threadIdx.x == kEpiWarp0 * 32) {
                    const int prev = atomicAdd(p.counters + t, 1);
                    *last_flag = prev == p.ksplit - 1;
                    if (prev == p.ksplit - 1) p.counters[t] = 0;  // ready for the next launch
                }
                named_bar_sync(1, 128);
                if (*last_flag) {
                    __threadfence();
                    mma_reduced_epilogue(p, sg, p.partial + static_cast<long>(t) * p.ksplit * n_pad * 128, r, row,
                                         valid, lane);
                }
                named_bar_sync(1, 128);  // last_flag is rewritten by the next unit
                continue;
            }
            for (int c0 = 0; c0 < n_pad; c0 += 16) {
                float v[16];
                tmem_ld16(taddr + c0, v);
#pragma unroll
                for (int k = 0; k < 16; ++k) v[k] *= wscale * p.x_inv[c0 + k];
                if (sg.epi == kEpiSiluPair) {
                    // up rows live in quadrants 2 and 3: hand them to the gate rows
                    if (quad >= 2)
                        for (int k = 0; k < 16; ++k) exch[(r - 64) * kExchStride + c0 + k] = v[k];
                    named_bar_sync(1, 128);
                    if (quad < 2 && valid) {
                        for (int k = 0; k < 16 && c0 + k < p.batch; ++k) {
                            const float g = v[k], uu = exch[r * kExchStride + c0 + k];
                            sg.out[(c0 + k) * sg.out_stride + sg.row_offset + row] = g / (1.f + __expf(-g)) * uu;
                        }
                    }
                    named_bar_sync(1, 128);
                } else if (sg.epi == kEpiLogitsArgmax) {
                    for (int k = 0; k < 16 && c0 + k < p.batch; ++k) {
                        const int n = c0 + k;
                        if (valid) sg.out[n * sg.out_stride + sg.row_offset + row] = v[k];
                        unsigned long long key = valid ? argmax_key(v[k], sg.row_offset + row) : 0ull;
#pragma unroll
                        for (int o = 16; o > 0; o >>= 1) {
                            const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
                            key = other > key ? other : key;
                        }
                        if (lane == 0 && key) atomicMax(p.argmax_keys + n, key);
                    }
                } else {
                    for (int k = 0; k < 16; ++k) {
                        const float partner = __shfl_xor_sync(0xffffffffu, v[k], 1);
                        if (c0 + k < p.batch) mma_epilogue_value(p, sg, row, valid, c0 + k, v[k], partner);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty + a);
        }
    } else {
        // ---------------------------------------------------------- dequant
        const int ct = threadIdx.x - kConvWarp0 * 32;  // 0..255
        const int row = ct & 127, q = ct >> 7;
        uint32_t rc = 0, fc = 0;
        for (int u = blockIdx.x; u < total_units; u += gridDim.x) {
            const int t = u / p.ksplit, sp = u % p.ksplit;
            const MmaSeg &sg = p.seg[mma_seg_of_tile(p, t)];
            const float scale = ldexpf(1.0f, p.w[row >= 64 && sg.w1 >= 0 ? sg.w1 : sg.w0].scale_exp);
            const int b0 = sp * p.bps, b1 = min(nb, b0 + p.bps);
            for (int b = b0; b < b1; ++b) {
                const int r = rc % kRawStages;
                mbar_wait_bounded(full_raw + r, (rc / kRawStages) & 1, p.status, cta_abort);
                const uint8_t *raw = smem + L.raw + r * kRawStageBytes;
                for (int h = 0; h < 2; ++h) {
                    const int f = fc % kF16Stages;
                    if (fc >= kF16Stages) mbar_wait_bounded(empty_w16 + f, ((fc / kF16Stages) - 1) & 1, p.status, cta_abort);
                    uint8_t *w16 = smem + L.w16 + f * kW16Bytes;
                    if (sg.type == kQ4K) convert_q4(raw, w16, row, q, h, scale);
                    else convert_q6(raw, w16, row, q, h, b % kUnitBlocks, scale);
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    __syncwarp();
                    if (lane == 0) mbar_arrive(full_w16 + f);
                    ++fc;
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(empty_raw + r);
                ++rc;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kMmaWarp)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(tmem_cols)
                     : "memory");
}

// --------------------------------------------------------- activation prep --

// One CTA per token: the GEMV prologue's arithmetic (RMSNorm in the
// reference's reduction order, per-32 int8 quantisation) then x^ = q * scale
// (DP4A semantics) or x (FP32 semantics), times 2^kx so that max|x^| lies in
// [2^14, 2^15), rounded to fp16 into the MMA layout.
__global__ void mma_prep_kernel(const float *x, long x_stride, const float *norm_w, float eps, int cols, int batch,
                                int n_pad, int use_dp4a, uint8_t *x16, float *x_inv) {
    pdl_trigger();
    pdl_wait();
    const int n = blockIdx.x, tid = threadIdx.x;
    __shared__ float red[256];
    __shared__ float amax_s[8];
    const long chunk_bytes = static_cast<long>(n_pad) * kKChunk * 2;
    auto dst_of = [&](int k) -> uint8_t * {  // 16 bytes holding positions k..k+7 of token n
        const int c = k / kKChunk, kc = (k % kKChunk) / 8;
        return x16 + c * chunk_bytes + (n >> 3) * 2048 + kc * 128 + (n & 7) * 16;
    };
    if (n >= batch) {
        for (int k = tid * 8; k < cols; k += 256 * 8) *reinterpret_cast<uint4 *>(dst_of(k)) = make_uint4(0, 0, 0, 0);
        if (tid == 0) x_inv[n] = 0.f;
        return;
    }
    const float *xr = x + n * x_stride;
    float r = 1.f;
    if (norm_w) {
        float s = 0.f;
        for (int i = tid; i < cols; i += 256) s = fmaf(xr[i], xr[i], s);
        red[tid] = s;
        __syncthreads();
        for (int st = 128; st > 0; st >>= 1) {
            if (tid < st) red[tid] += red[tid + st];
            __syncthreads();
        }
        r = rsqrtf(red[0] / static_cast<float>(cols) + eps);
    }
    // pass 1: values and the token's max |x^|
    float local_max = 0.f;
    const int chunks = cols / 8;
    float vals[kMaxCols / (256 * 8)][8];
    for (int j = 0; j < kMaxCols / (256 * 8); ++j) {
        const int c = tid + 256 * j;
        if (c >= chunks) continue;
        float v[8];
        const float4 a = *reinterpret_cast<const float4 *>(xr + c * 8);
        const float4 b = *reinterpret_cast<const float4 *>(xr + c * 8 + 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        if (norm_w) {
            const float4 wa = *reinterpret_cast<const float4 *>(norm_w + c * 8);
            const float4 wb = *reinterpret_cast<const float4 *>(norm_w + c * 8 + 4);
            const float w8[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
            for (int e = 0; e < 8; ++e) v[e] = __fmul_rn(__fmul_rn(v[e], r), w8[e]);
        }
        if (use_dp4a) {
            // quantize_x32_cuda (inferencer.cu:544-556) over the 32-value group = 4 lanes
            float am = 0.f;
#pragma unroll
            for (int e = 0; e < 8; ++e) am = fmaxf(am, fabsf(v[e]));
            am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
            am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
            const float scale = am > 0.f ? am / 127.f : 1.f;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                int q = __float2int_rn(v[e] / scale);
                q = max(-127, min(127, q));
                v[e] = static_cast<float>(q) * scale;
            }
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            vals[j][e] = v[e];
            local_max = fmaxf(local_max, fabsf(v[e]));
        }
    }
    local_max = warp_max(local_max);
    if ((tid & 31) == 0) amax_s[tid >> 5] = local_max;
    __syncthreads();
    float amax = 0.f;
    for (int w = 0; w < 8; ++w) amax = fmaxf(amax, amax_s[w]);
    int e2 = 0;
    if (amax > 0.f) frexpf(amax, &e2);
    const int kx = amax > 0.f ? 15 - e2 : 0;  // amax * 2^kx in [2^14, 2^15)
    const float up = ldexpf(1.0f, kx);
    for (int j = 0; j < kMaxCols / (256 * 8); ++j) {
        const int c = tid + 256 * j;
        if (c >= chunks) continue;
        const uint4 o = make_uint4(pack_half2(vals[j][0] * up, vals[j][1] * up), pack_half2(vals[j][2] * up, vals[j][3] * up),
                                   pack_half2(vals[j][4] * up, vals[j][5] * up), pack_half2(vals[j][6] * up, vals[j][7] * up));
        *reinterpret_cast<uint4 *>(dst_of(c * 8)) = o;
    }
    if (tid == 0) x_inv[n] = ldexpf(1.0f, -kx);
}

// Bound of max|w| over GGUF blocks: Q4_K |d|*63*15 + |dmin|*63, Q6_K
// |d|*128*32; atomicMax on the float's bits (non-negative floats order as
// integers).
__global__ void mma_scale_scan_kernel(int type, const uint8_t *w, long nblocks, unsigned int *out) {
    float best = 0.f;
    for (long b = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; b < nblocks;
         b += static_cast<long>(gridDim.x) * blockDim.x) {
        float bound;
        if (type == kQ4K) {
            const uint8_t *bp = w + b * 144;
            const float d = fabsf(half_bits_to_float(*reinterpret_cast<const uint16_t *>(bp)));
            const float dm = fabsf(half_bits_to_float(*reinterpret_cast<const uint16_t *>(bp + 2)));
            bound = d * 945.f + dm * 63.f;
        } else {
            const uint8_t *bp = w + b * 210;
            bound = fabsf(half_bits_to_float(*reinterpret_cast<const uint16_t *>(bp + 208))) * 4096.f;
        }
        if (!(bound <= 3.0e38f)) bound = 3.0e38f;  // inf / NaN scales
        best = fmaxf(best, bound);
    }
    best = warp_max(best);
    if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(best));
}

// ------------------------------------------------------------------- host --

cudaError_t mma_prep_launch(const float *x, long x_stride, const float *norm_w, float eps, int cols, int batch,
                            int n_pad, int use_dp4a, uint8_t *x16, float *x_inv, cudaStream_t stream) {
    if (cols % 256 || cols > kMaxCols || batch < 1 || n_pad > kMmaMaxN || n_pad % 16) return cudaErrorInvalidValue;
    mma_prep_kernel<<<n_pad, 256, 0, stream>>>(x, x_stride, norm_w, eps, cols, batch, n_pad, use_dp4a, x16, x_inv);
    return cudaGetLastError();
}

cudaError_t mma_scale_scan_launch(int type, const uint8_t *w, long nblocks, int *out_max_bits, cudaStream_t stream) {
    cudaError_t e = cudaMemsetAsync(out_max_bits, 0, sizeof(int), stream);
    if (e != cudaSuccess) return e;
    mma_scale_scan_kernel<<<256, 256, 0, stream>>>(type, w, nblocks, reinterpret_cast<unsigned int *>(out_max_bits));
    return cudaGetLastError();
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

static int encode_box(CUtensorMap *m, const void *data, int rows, long row_bytes, int box_bytes, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return -1;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_bytes), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(box_bytes), static_cast<cuuint32_t>(box_rows)};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(data), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : static_cast<int>(r);
}

int mma_make_weight(int type, const void *data, int rows, long row_bytes, int rows_per_box, MmaWeight *out, char *err,
                    int err_len) {
    std::memset(out, 0, sizeof(*out));
    if ((reinterpret_cast<uintptr_t>(data) & 15) || (row_bytes & 15)) {
        std::snprintf(err, err_len, "tensor-core path needs 16-byte aligned rows");
        return -1;
    }
    const int body = type == kQ4K ? 144 : 208;
    out->rows_per_box = rows_per_box;
    int r = encode_box(&out->body, data, rows, row_bytes, body, rows_per_box);
    if (r == 0 && type == kQ6K) r = encode_box(&out->dvec, data, rows, row_bytes, 16, rows_per_box);
    if (r != 0) std::snprintf(err, err_len, "cuTensorMapEncodeTiled failed (%d)", r);
    return r;
}

cudaError_t mma_prepare() {
    return cudaFuncSetAttribute(mma_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, mma_smem().total);
}

int mma_choose_split(int tiles, int nblocks, int num_sms, int *bps) {
    int ks = (num_sms + tiles - 1) / tiles;
    if (ks > nblocks) ks = nblocks;
    if (ks < 1) ks = 1;
    *bps = (nblocks + ks - 1) / ks;
    return (nblocks + *bps - 1) / *bps;
}

cudaError_t mma_gemm_launch(const MmaParams &p, int num_sms, cudaStream_t stream) {
    if (p.n_pad < 16 || p.n_pad > kMmaMaxN || p.n_pad % 16 || p.cols % 256 || p.total_tiles < 1 || p.ksplit < 1 ||
        p.bps < 1 || (p.ksplit > 1 && (!p.partial || !p.counters)))
        return cudaErrorInvalidValue;
    const int units = p.total_tiles * p.ksplit;
    const int grid = num_sms < units ? num_sms : units;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kMmaThreads);
    cfg.dynamicSmemBytes = mma_smem().total;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, mma_gemm_kernel, p);
}

}  // namespace ijb
