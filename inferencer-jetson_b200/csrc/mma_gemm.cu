// Tensor-core (tcgen05) quantised GEMM for packed steps: up to 64 tokens per
// launch, or up to 128 when every CTA of the launch holds one tile.
//
// Replaces, for a ragged batch, what the reference does one token at a time
// (gemv_batch_dp4a, qkv_batch_cuda, gate_up_batch_cuda, inferencer.cu:678-751):
// every weight is read from HBM once per step instead of once per token.
//
// Work is cut into 128-row tiles of the launch's matrices (a gate/up tile is
// 64 gate rows + the same 64 up rows) and, when there are too few tiles to
// fill the GPU, each tile's K range into `ksplit` parts run by the CTAs of one
// thread-block cluster.  Warp roles of a CTA:
//   * warp 0, lane 0: weight producer.  Per 256-wide block column of a tile it
//     copies the raw quantised bytes of the tile's two 64-row groups, each a
//     contiguous chunk of the weight's chunked copy (Q4_K: [64 rows][144 B];
//     Q6_K: [64][208 B] block bodies and [64] fp16 d), with plain bulk copies
//     into a 4-stage ring (3 stages in 128-token launches, whose activation
//     stages are twice as large).
//   * warp 6, lane 0: activation producer: per 64-wide K stage, one bulk copy
//     of the prepared fp16 activation chunk into an 8-stage ring (two block
//     columns in flight).
//   * warps 7..22: dequantise, four groups of four warps; group g converts
//     64-wide group g of every block column, each warp the 32 rows of its TMEM
//     lane quadrant, one thread per row, straight into TMEM with tcgen05.st
//     (the MMA's A operand).  Nibbles become fp16 through exponent-bias
//     patterns (0x6400 | q is 1024 + q) and one fp16 FMA applies the sub-block
//     scale and offset; the K order inside each 8-wide core is permuted so that
//     this needs no byte shuffles, and the activation tile is written in the
//     same order.
//   * warps 1 and 23, lane 0: MMA issue, tcgen05.mma (kind::f16, M=128, N =
//     tokens rounded up to 16, K=16) into two fp32 accumulator chains in TMEM
//     (warp 1: even 64-wide groups, columns from 0; warp 23: odd groups, from
//     384; up to 128 columns each beside the 256 columns of weight stages);
//     tcgen05.commit releases stages and signals finished accumulators.  Every
//     launch width sums a token's products in this order.  CTAs with several
//     tiles double-buffer the chains across tiles.
//   * warps 2..5 (one per TMEM lane quadrant), joined by the converter warps
//     when the CTA has a single tile: read and add the two chains with
//     tcgen05.ld, undo the two power-of-two scales and apply the fused
//     epilogue of the GEMV (store, residual add, RoPE + paged K write, V write,
//     SiLU * up, logits + argmax key) through a [token][row] shared-memory
//     tile, storing with coalesced thread stores.  With split K the parts
//     first stage their partial sums in shared memory; each part then sums a
//     slice of the tokens over the cluster's shared memory (DSMEM) in part
//     order, so the result does not depend on timing.
// All waits are bounded; TMEM is always released before the CTA exits.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "mma_gemm.cuh"

namespace ijb {

constexpr int kKChunk = 64;  // K per fp16 stage: one Q4_K group of 64 weights
constexpr int kGroups = 4;   // 64-wide groups of a 256-wide block column
constexpr int kStages = 8;   // fp16 weight + activation stages: two block columns in flight
constexpr int kRawStages = 4;
constexpr int kRawStageBytes = 128 * 208 + 128 * 2;  // Q6_K bodies + d (Q4_K uses 128 * 144)
constexpr int kQ6DOff = 128 * 208;                    // d box within a Q6_K raw stage
constexpr uint32_t kTmemCols = 512;  // accumulator chain 0 [0, 128), fp16 weight stages [128, 384), chain 1 [384, 512)
constexpr uint32_t kTmemA = 128;     // first column of the weight stages (32 per stage)
constexpr uint32_t kTmemAcc1 = 384;  // chain 1 of the accumulators
constexpr int kRawStagesWide = kRawStages - 1;       // raw stages of a launch wider than kMmaMaxN tokens
constexpr int kCoreStride = 128;                      // bytes between 8-wide K cores
constexpr int kGroupStride = (kKChunk / 8) * 128;     // bytes between 8-row groups (1 KB)
constexpr int kMaxCluster = 8;
// the epilogue's output tile, [token][kStage] floats (a token's 128 rows contiguous,
// 16-byte aligned rows for bulk stores)
constexpr int kStage = kMmaTileM + 4;
constexpr int kProducerWarp = 0, kMmaWarp = 1, kEpiWarp0 = 2, kXWarp = 6, kConvWarp0 = 7, kConvWarps = 16;
constexpr int kMma2Warp = kConvWarp0 + kConvWarps;  // second MMA issuer of CTAs with several tiles
constexpr int kMmaThreads = (kMma2Warp + 1) * 32;
constexpr int kEpiThreadsSingle = (4 + kConvWarps) * 32;  // epilogue + converter warps of a one-tile CTA
constexpr int kNumBars = 2 * kRawStages + 2 * kStages + 4 + 2;

// Two layouts share the block.  Launches of up to kMmaMaxN tokens: kRawStages
// raw weight stages, the activation stages, then the output tile.  Wider
// launches (one tile per CTA): kRawStagesWide raw stages and activation stages
// twice as large; their output tile reuses the raw stages, which are idle once
// the tile's last MMA has committed.
struct MmaSmem {
    int raw, x16, red, x16w, redw, tok, segs, bars, tmem, total;
};

__host__ __device__ constexpr MmaSmem mma_smem() {
    MmaSmem L{};
    L.raw = 0;
    L.x16 = kRawStages * kRawStageBytes;
    L.red = L.x16 + kStages * kMmaMaxN * kKChunk * 2;
    const int narrow_end = L.red + kMmaMaxN * kStage * 4;
    L.x16w = kRawStagesWide * kRawStageBytes;
    L.redw = 0;
    const int wide_end = L.x16w + kStages * kMmaMaxNWide * kKChunk * 2;
    int off = narrow_end > wide_end ? narrow_end : wide_end;
    L.tok = off;  // x_inv, positions and KV slots of the launch's tokens, then argmax keys
    off += 3 * kMmaMaxNWide * 4 + kMmaMaxNWide * 8;
    L.segs = off;  // the launch's segments and weight scale exponents
    off += kMaxSegs * static_cast<int>(sizeof(MmaSeg)) + 2 * kMaxSegs * 4;
    off = (off + 7) / 8 * 8;
    L.bars = off;
    off += kNumBars * 8;
    L.tmem = off;
    off += 16;
    L.total = (off + 127) / 128 * 128;
    return L;
}
static_assert(mma_smem().total <= 227 * 1024, "shared memory of the tensor-core GEMM");
static_assert(mma_smem().redw + kMmaMaxNWide * kStage * 4 <= mma_smem().x16w, "wide output tile within the raw stages");
static_assert(mma_smem().x16 % 128 == 0 && mma_smem().x16w % 128 == 0, "activation stages aligned");
static_assert((kStage * 4) % 16 == 0, "bulk-store rows");

// Tokens per part's epilogue slice (a multiple of 4).
__host__ __device__ constexpr int split_per(int batch, int parts) { return ((batch + parts - 1) / parts + 3) / 4 * 4; }

int mma_smem_bytes() { return mma_smem().total; }

// ------------------------------------------------------------ PTX helpers --


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

// Same with A (M x K fp16, rows in TMEM lanes, two K elements per column) in TMEM.
__device__ __forceinline__ void umma_f16_ta(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 16 columns without waiting; tmem_wait16 completes every earlier load and
// makes the 16 values it is given depend on the wait.
__device__ __forceinline__ void tmem_ld16_nw(uint32_t taddr, uint32_t *r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait16(uint32_t *r) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
                 :
                 : "memory");
}
// 8 columns without waiting, and the matching wait (see tmem_ld16_nw).
__device__ __forceinline__ void tmem_ld8_nw(uint32_t taddr, uint32_t *r) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait8(uint32_t *r) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7])
                 :
                 : "memory");
}
// Lane (warp quadrant + lane) of TMEM gets 8 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
                 "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
}

// Bulk (TMA engine) stores of shared-memory rows: plain copy or fp32 add into
// global memory; bytes and both addresses multiples of 16.
__device__ __forceinline__ void bulk_s2g(void *gdst, const void *ssrc, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(smem_u32(ssrc)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_s2g_add(void *gdst, const void *ssrc, uint32_t bytes) {
    asm volatile("cp.reduce.async.bulk.global.shared::cta.bulk_group.add.f32 [%0], [%1], %2;" ::"l"(gdst),
                 "r"(smem_u32(ssrc)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

__device__ __forceinline__ __half2 bits_h2(uint32_t u) { return *reinterpret_cast<const __half2 *>(&u); }
__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<const uint32_t *>(&h); }

// ------------------------------------------------------- cluster helpers --

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_id() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_count() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
    return r;
}
// All threads of all CTAs of the cluster (a plain CTA barrier without one).
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Shared-memory address of the same variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t dsmem_addr(uint32_t local, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
    return r;
}
__device__ __forceinline__ float4 dsmem_ld4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr)
                 : "memory");
    return v;
}
// Arrives on the mbarrier at `bar` in CTA `rank`, releasing this thread's
// earlier writes (and those it has synchronised with) at cluster scope.
__device__ __forceinline__ void mbar_arrive_remote(uint64_t *bar, uint32_t rank) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(dsmem_addr(smem_u32(bar), rank))
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
        : "memory");
    return ok != 0;
}
static __device__ __noinline__ bool mbar_wait_cluster_slow(uint64_t *bar, uint32_t parity, uint32_t *status,
                                                           volatile uint32_t *cta_abort) {
    if (*cta_abort) return false;
    uint64_t start = 0;
    for (uint32_t n = 1;; ++n) {
        if (mbar_try_wait_cluster(bar, parity)) return true;
        if ((n & 15u) == 0) {
            if (*cta_abort) return false;
            const uint64_t now = global_timer_ns();
            if (start == 0) {
                start = now;
            } else if (now - start > kWaitLimitNs) {
                *cta_abort = 1u;
                if (status) atomicOr(status, kDevErrWaitTimeout);
                return false;
            }
        }
    }
}
// mbar_wait_bounded with acquire at cluster scope (for arrivals from peers).
__device__ __forceinline__ bool mbar_wait_cluster_bounded(uint64_t *bar, uint32_t parity, uint32_t *status,
                                                          volatile uint32_t *cta_abort) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    return mbar_wait_cluster_slow(bar, parity, status, cta_abort);
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
//
// K order of a stage.  Stage g (0..3) of a block column holds the block's
// weights 64g .. 64g+63 as 8 cores of 8; core j holds, in this order,
//   64g + 4j + {0, 2, 1, 3}   and   64g + 32 + 4j + {0, 2, 1, 3}.
// For Q4_K these are the low nibbles (sub-block 2g) and high nibbles
// (sub-block 2g+1) of the 32-bit word j of the group's 32 bytes, so a mask
// of 0x000F000F / 0x00F000F0 on the word and on the word >> 8 yields the four
// fp16 pairs.  ijb_mma_prep_kernel writes the activation in the same order.

// Q4_K group g of a raw block column -> fp16 stage.  The weight is
// (d*sc)*q - dmin*m as in q4_value (inferencer.cu:454-471), with the scale
// products rounded to fp16 and one fp16 rounding of the result; q comes out
// exact (1024 + q minus 1024, or (1024 + 16q) / 16 - 64).
__device__ __forceinline__ void convert_q4(const uint8_t *raw, uint32_t tmem_row, int row, int g, float scale) {
    const uint8_t *bp = raw + row * 144;
    const uint4 hdr = *reinterpret_cast<const uint4 *>(bp);
    const uint4 qa = *reinterpret_cast<const uint4 *>(bp + 16 + g * 32);
    const uint4 qb = *reinterpret_cast<const uint4 *>(bp + 32 + g * 32);
    const float d = half_bits_to_float(hdr.x & 0xffff), dmin = half_bits_to_float(hdr.x >> 16);
    auto byte = [&](int k) -> int {
        const uint32_t w = k < 4 ? hdr.y : (k < 8 ? hdr.z : hdr.w);
        return (w >> ((k & 3) * 8)) & 255;
    };
    int sc[2], m[2];
#pragma unroll
    for (int t = 0; t < 2; ++t) {
        const int j = 2 * g + t;
        if (j < 4) {
            sc[t] = byte(j) & 63;
            m[t] = byte(j + 4) & 63;
        } else {
            sc[t] = (byte(j + 4) & 15) | ((byte(j - 4) >> 6) << 4);
            m[t] = (byte(j + 4) >> 4) | ((byte(j) >> 6) << 4);
        }
    }
    const __half2 s1a = __float2half2_rn(d * static_cast<float>(sc[0]) * scale);
    const __half2 s1b = __float2half2_rn(d * static_cast<float>(sc[1]) * scale);
    const __half2 n2a = __float2half2_rn(-(dmin * static_cast<float>(m[0]) * scale));
    const __half2 n2b = __float2half2_rn(-(dmin * static_cast<float>(m[1]) * scale));
    const __half2 k1024 = __float2half2_rn(1024.f), k16th = __float2half2_rn(0.0625f), km64 = __float2half2_rn(-64.f);
    const uint32_t words[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
    for (int j2 = 0; j2 < 8; j2 += 2) {  // two 8-wide cores = 8 TMEM columns per store
        uint32_t o[8];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t w = words[j2 + h], w8 = w >> 8;
            const __half2 qa02 = __hsub2(bits_h2((w & 0x000F000Fu) | 0x64006400u), k1024);
            const __half2 qa13 = __hsub2(bits_h2((w8 & 0x000F000Fu) | 0x64006400u), k1024);
            const __half2 qb02 = __hfma2(bits_h2((w & 0x00F000F0u) | 0x64006400u), k16th, km64);
            const __half2 qb13 = __hfma2(bits_h2((w8 & 0x00F000F0u) | 0x64006400u), k16th, km64);
            o[4 * h + 0] = h2_bits(__hfma2(qa02, s1a, n2a));
            o[4 * h + 1] = h2_bits(__hfma2(qa13, s1a, n2a));
            o[4 * h + 2] = h2_bits(__hfma2(qb02, s1b, n2b));
            o[4 * h + 3] = h2_bits(__hfma2(qb13, s1b, n2b));
        }
        tmem_st8(tmem_row + static_cast<uint32_t>(j2 * 4), o);
    }
}

// Q6_K group g of a raw block column (unit layout body, gemv.cuh) -> fp16 stage.
// Weights 64g .. 64g+63 are, in Q6_K terms, parts 2(g&1) and 2(g&1)+1 of the
// 128-half g>>1, positions l = 0..31 (lanes 2(g>>1) and 2(g>>1)+1 of the
// unit layout).  The 6-bit code is assembled in an fp16 mantissa (1024 + q,
// or 1024 + 16q for the high nibbles), q - 32 is exact, and one fp16 multiply
// by d*scale (rounded to fp16) gives the weight of q6_value
// (inferencer.cu:473-487) with two roundings.
__device__ __forceinline__ void convert_q6(const uint8_t *raw, uint32_t tmem_row, int row, int g, float scale) {
    const uint8_t *body = raw + row * 208;
    const int h = g >> 1, hi = g & 1;
    const uint4 *A = reinterpret_cast<const uint4 *>(body) + 2 * h;
    const uint4 *B = reinterpret_cast<const uint4 *>(body + 64) + 2 * h;
    const uint4 *H = reinterpret_cast<const uint4 *>(body + 128) + 2 * h;
    const uint2 scw = *reinterpret_cast<const uint2 *>(body + 192 + 8 * h);
    const float d = half_bits_to_float(*reinterpret_cast<const uint16_t *>(raw + kQ6DOff + row * 2)) * scale;
    const __half2 k1056 = __float2half2_rn(1056.f), k16th = __float2half2_rn(0.0625f), km96 = __float2half2_rn(-96.f);
#pragma unroll 1
    for (int l2 = 0; l2 < 2; ++l2) {
        const uint32_t s4 = l2 ? scw.y : scw.x;
        const __half2 sa = __float2half2_rn(d * static_cast<float>(static_cast<int8_t>((s4 >> (16 * hi)) & 255)));
        const __half2 sb = __float2half2_rn(d * static_cast<float>(static_cast<int8_t>((s4 >> (16 * hi + 8)) & 255)));
        const uint4 a4 = A[l2], b4 = B[l2], h4 = H[l2];
        const uint32_t aw[4] = {a4.x, a4.y, a4.z, a4.w}, bw[4] = {b4.x, b4.y, b4.z, b4.w};
        const uint32_t hw[4] = {h4.x, h4.y, h4.z, h4.w};
        uint32_t o[8];
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
            const uint32_t a = aw[jj], b = bw[jj], q = hw[jj];
            const uint32_t a8 = a >> 8, b8 = b >> 8;
            const uint32_t qp4 = q << 4, qm4 = q >> 4, qp2 = q << 2, qm6 = q >> 6;
            __half2 v02a, v13a, v02b, v13b;
            if (!hi) {  // low nibbles, high bits 0-1 (part 0) and 2-3 (part 1)
                v02a = __hsub2(bits_h2((a & 0x000F000Fu) | (qp4 & 0x00300030u) | 0x64006400u), k1056);
                v13a = __hsub2(bits_h2((a8 & 0x000F000Fu) | (qm4 & 0x00300030u) | 0x64006400u), k1056);
                v02b = __hsub2(bits_h2((b & 0x000F000Fu) | (qp2 & 0x00300030u) | 0x64006400u), k1056);
                v13b = __hsub2(bits_h2((b8 & 0x000F000Fu) | (qm6 & 0x00300030u) | 0x64006400u), k1056);
            } else {    // high nibbles, high bits 4-5 (part 2) and 6-7 (part 3), scaled by 16
                v02a = __hfma2(bits_h2((a & 0x00F000F0u) | (qp4 & 0x03000300u) | 0x64006400u), k16th, km96);
                v13a = __hfma2(bits_h2((a8 & 0x00F000F0u) | (qm4 & 0x03000300u) | 0x64006400u), k16th, km96);
                v02b = __hfma2(bits_h2((b & 0x00F000F0u) | (qp2 & 0x03000300u) | 0x64006400u), k16th, km96);
                v13b = __hfma2(bits_h2((b8 & 0x00F000F0u) | (qm6 & 0x03000300u) | 0x64006400u), k16th, km96);
            }
            o[4 * (jj & 1) + 0] = h2_bits(__hmul2(v02a, sa));
            o[4 * (jj & 1) + 1] = h2_bits(__hmul2(v13a, sa));
            o[4 * (jj & 1) + 2] = h2_bits(__hmul2(v02b, sb));
            o[4 * (jj & 1) + 3] = h2_bits(__hmul2(v13b, sb));
            if (jj & 1) tmem_st8(tmem_row + static_cast<uint32_t>((4 * l2 + jj - 1) * 4), o);
        }
    }
}

// --------------------------------------------------------------- epilogue --
//
// The epilogue runs once per tile, so its code is kept compact (it is cold in
// the instruction cache every time): the accumulator is first moved to shared
// memory, then one rolled loop per token applies the fused operation.  Token
// positions, KV slots and activation scales are staged in shared memory at
// kernel start; the residual add is a fire-and-forget red.global.add (one
// writer per element, so the result is the plain fp32 sum).

struct EpiTok {
    const float *x_inv;         // [n_pad]
    const int *pos;             // [n_pad]
    const int *slot;            // [n_pad]
    unsigned long long *keys;   // [n_pad] this CTA's best logits key per token (shared memory)
};

// Per tile row: output pointer for token 0 and everything the operation needs.
struct EpiRow {
    float *out;       // segment output + row offset + row; token n at out[n * stride]
    float *out_pair;  // gate/up tiles: the output of gate row (lane & 63)
    long stride;
    int epi, f, head, dd, row;
    bool valid, even, valid_pair;
};

__device__ __forceinline__ EpiRow make_epi_row(const MmaParams &p, const MmaSeg &sg, int row, bool valid) {
    EpiRow e;
    e.out = sg.out + sg.row_offset + row;
    e.out_pair = e.out;
    e.valid_pair = valid;
    e.stride = sg.out_stride;
    e.epi = sg.epi;
    e.row = sg.row_offset + row;
    e.valid = valid;
    e.even = (row & 1) == 0;
    e.f = p.half_head > 0 ? (row >> 1) % p.half_head : 0;  // RoPE frequency of the pair (2j, 2j+1)
    e.head = p.head_dim > 0 ? row / p.head_dim : 0;
    e.dd = p.head_dim > 0 ? row % p.head_dim : 0;
    return e;
}

// KV cache element of (token n, tile row) for a K or V write.
__device__ __forceinline__ long kv_offset(const MmaParams &p, const EpiRow &e, const EpiTok &tk, int n) {
    const int slot = tk.slot[n];
    return static_cast<long>(slot / p.page_size) * p.page_stride +
           (static_cast<long>(e.head) * p.page_size + slot % p.page_size) * p.head_dim + e.dd;
}

// Phase B of the epilogue: stage[n][r] holds the finished GEMM value of tile
// lane r for the tokens of this part's slice (below t_hi); apply the row
// operation in place (SiLU pairs, RoPE), write the KV cache, or (no bulk path)
// store the outputs directly.  The calling thread handles row r for tokens
// n0, n0 + step, ... (step = threads / 128); per-token loops are warp-uniform.
__device__ void epi_rows(const MmaParams &p, const EpiRow &e, const EpiTok &tk, float *stage, int r, int n0, int step,
                         int t_hi, bool bulk) {
    float *col = stage + r;  // token n at col[n * kStage]
    switch (e.epi) {
        case kEpiSiluPair: {
            // gate row r & 63 of every other token of the thread's phase (both halves
            // of each 128 work); silu(g) * u with the fast division (2 ulp)
            float *gcol = stage + (r & 63);
            const bool valid = r < 64 ? e.valid : e.valid_pair;
            float *out = r < 64 ? e.out : e.out_pair;
#pragma unroll 4
            for (int n = n0 + step * (r >> 6); n < t_hi; n += 2 * step) {
                const float g = gcol[n * kStage], u = gcol[n * kStage + 64];
                const float v = __fdividef(g, 1.f + __expf(-g)) * u;
                if (bulk) gcol[n * kStage] = v;
                else if (valid) out[n * e.stride] = v;
            }
            break;
        }
        case kEpiRopeQ:
        case kEpiRopeKCache: {
            // rope_cuda (inferencer.cu:906-917); the partner row r ^ 1 is the neighbouring lane
            const float *pc = p.rope_cos + e.f, *ps = p.rope_sin + e.f;
            for (int nb = n0; nb < t_hi; nb += 8 * step) {
                float y[8], z[8], c[8], sn[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const int n = min(nb + k * step, t_hi - 1);
                    y[k] = col[n * kStage];
                    z[k] = stage[n * kStage + (r ^ 1)];
                    const int pos = tk.pos[n] * p.half_head;
                    c[k] = __ldg(pc + pos);
                    sn[k] = __ldg(ps + pos);
                }
                __syncwarp();
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const int n = nb + k * step;
                    if (n >= t_hi) break;
                    const float a = e.even ? y[k] : z[k], b = e.even ? z[k] : y[k];
                    const float v = e.even ? a * c[k] - b * sn[k] : a * sn[k] + b * c[k];
                    if (e.epi == kEpiRopeQ) {
                        if (bulk) col[n * kStage] = v;
                        else if (e.valid) e.out[n * e.stride] = v;
                    } else if (e.valid) {
                        const long off = kv_offset(p, e, tk, n);
                        if (p.kv_f32) static_cast<float *>(p.k_cache)[off] = v;
                        else static_cast<__half *>(p.k_cache)[off] = __float2half_rn(v);
                    }
                }
                __syncwarp();
            }
            break;
        }
        case kEpiVCache:
            if (e.valid)
                for (int n = n0; n < t_hi; n += step) {
                    const long off = kv_offset(p, e, tk, n);
                    if (p.kv_f32) static_cast<float *>(p.v_cache)[off] = col[n * kStage];
                    else static_cast<__half *>(p.v_cache)[off] = __float2half_rn(col[n * kStage]);
                }
            break;
        case kEpiStore:
        case kEpiLogitsArgmax:
            if (!bulk && e.valid)
                for (int n = n0; n < t_hi; n += step) e.out[n * e.stride] = col[n * kStage];
            break;
        case kEpiAdd:
            if (!bulk && e.valid)
                for (int n = n0; n < t_hi; n += step)
                    asm volatile("red.global.add.f32 [%0], %1;" ::"l"(e.out + n * e.stride), "f"(col[n * kStage])
                                 : "memory");
            break;
        default:
            break;
    }
}

// Logits: the best (value, row) key of each token over the tile's `count`
// rows, two threads per token scanning 64 rows each; kept in the CTA's
// shared key array (flushed to global once at the end of the kernel).
__device__ void epi_argmax(const float *stage, const EpiTok &tk, int row_base, int count, int t_lo, int t_hi) {
    const int tid = threadIdx.x - kEpiWarp0 * 32;  // 0..127
    for (int n0 = t_lo; n0 < t_hi; n0 += 64) {
        const int n = n0 + (tid >> 1), h = tid & 1;
        unsigned long long best = 0ull;
        if (n < t_hi) {
            const float *v = stage + n * kStage;
            unsigned long long b8[8] = {0ull, 0ull, 0ull, 0ull, 0ull, 0ull, 0ull, 0ull};
            for (int i = 0; i < 64; i += 8) {
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int rr = h * 64 + ((i + u + n) & 63);  // staggered so the pair's lanes hit different banks
                    const unsigned long long key = rr < count ? argmax_key(v[rr], row_base + rr) : 0ull;
                    b8[u] = key > b8[u] ? key : b8[u];
                }
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) best = b8[u] > best ? b8[u] : best;
        }
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, 1);
        best = other > best ? other : best;
        if (h == 0 && n < t_hi && best) atomicMax(tk.keys + n, best);
    }
}

// ----------------------------------------------------------------- kernel --

// The kernel declares no static shared memory: with a static block in front of
// the dynamic one, results came out wrong on B200 (cause not identified), so
// every shared buffer is carved from the dynamic block (mma_smem).
__global__ void __launch_bounds__(kMmaThreads, 1) ijb_mma_gemm_kernel(const __grid_constant__ MmaParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    constexpr MmaSmem L = mma_smem();
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bars);
    uint64_t *full_raw = bars, *empty_raw = full_raw + kRawStages;
    uint64_t *full = empty_raw + kRawStages, *empty = full + kStages;  // fp16 weight + activation stage
    uint64_t *acc_full = empty + kStages, *acc_empty = acc_full + 2;
    uint64_t *part_ready = acc_empty + 2, *part_free = part_ready + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L.tmem);
    uint32_t *cta_abort = tmem_slot + 1;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb = p.cols / 256;
    const int n_pad = p.n_pad;
    // more than kMmaMaxN tokens: the wide layout (one tile per CTA, checked below)
    const bool wide = n_pad > kMmaMaxN;
    const int nraw = wide ? kRawStagesWide : kRawStages;
    uint8_t *const x16_s = smem + (wide ? L.x16w : L.x16);
    const uint32_t xstage = static_cast<uint32_t>(n_pad) * kKChunk * 2;  // bytes of one activation stage
    float *red = reinterpret_cast<float *>(smem + (wide ? L.redw : L.red));
    const int ksplit = p.ksplit;
    const int rank = static_cast<int>(cluster_rank());
    const int tile_first = static_cast<int>(cluster_id()), tile_step = static_cast<int>(cluster_count());
    const int b0 = rank * p.bps, b1 = min(nb, b0 + p.bps);  // this part's block columns
    const uint32_t tmem_cols = kTmemCols;
    const bool single = tile_first + tile_step >= p.total_tiles;  // this CTA has one tile
    if (wide && !single) {  // the host only launches wide tiles one per CTA (mma_wide_ok)
        if (threadIdx.x == 0) atomicOr(p.status, kDevErrBadIndex);
        return;  // the whole cluster leaves before any barrier or TMEM allocation
    }

    MmaSeg *seg_s = reinterpret_cast<MmaSeg *>(smem + L.segs);
    int *wexp_s = reinterpret_cast<int *>(seg_s + kMaxSegs);
    if (warp == kProducerWarp) {
        // the launch's segments into shared memory
        if (lane < p.nseg) {
            const MmaSeg sg = p.seg[lane];
            seg_s[lane] = sg;
            for (int h = 0; h < 2; ++h) {
                const int wi = h ? sg.w1 : sg.w0;
                if (wi >= 0) wexp_s[wi] = p.w[wi].scale_exp;
            }
        }
    }
    if (threadIdx.x == 0) {
        *cta_abort = 0u;
        for (int i = 0; i < kRawStages; ++i) {
            mbar_init(full_raw + i, 1);
            mbar_init(empty_raw + i, kConvWarps);
        }
        for (int i = 0; i < kStages; ++i) {
            mbar_init(full + i, kConvWarps / kGroups + 1);  // the group's warps + the activation copy
            mbar_init(empty + i, 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(acc_full + i, 2);  // a commit from each issuing thread
            mbar_init(acc_empty + i, 4);
        }
        mbar_init(part_ready, ksplit);
        mbar_init(part_free, ksplit);
        fence_barrier_init();
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(tmem_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    cluster_sync_all();  // barriers of every CTA of the cluster are initialised
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_trigger();

    // MMA issue for the 64-wide groups in `mask` of every block column: D (fp32)
    // [128 x n_pad] = A (fp16 weights in TMEM) * B (fp16 activation, K-major)^T,
    // into one accumulator chain per issuing thread (summed by the epilogue).
    // A thread issues a tcgen05.mma only every ~130 cycles whatever N, while two
    // threads issuing into separate accumulators share the tensor core (~69
    // cycles per MMA): warps 1 (even groups, TMEM columns from 0) and 23 (odd
    // groups, from 384) issue, for every CTA, so every launch sums a token's
    // products in the same order whatever its width (chains of up to 128
    // columns beside the 256 columns of weight stages); CTAs with several tiles
    // double-buffer the chains across tiles.
    auto mma_loop = [&](uint32_t mask, uint32_t chain_col) {
        const uint32_t idesc = (1u << 4) | (static_cast<uint32_t>(n_pad >> 3) << 17) | (8u << 24);
        const uint64_t b_desc0 = umma_desc(smem_u32(x16_s), kCoreStride, kGroupStride);
        uint32_t blk = 0, i = 0;
        for (int t = tile_first; t < p.total_tiles; t += tile_step, ++i) {
            const int a = i & 1;
            if (i >= 2) mbar_wait_bounded(acc_empty + a, ((i >> 1) - 1) & 1, p.status, cta_abort);
            tc_fence_after();
            const uint32_t dcol = tmem_base + chain_col + static_cast<uint32_t>(single ? 0 : a * n_pad);
            uint32_t acc = 0;
            for (int b = b0; b < b1; ++b, ++blk) {
                const uint32_t ph = (blk >> 1) & 1;
#pragma unroll
                for (int g = 0; g < kGroups; ++g) {
                    if (!((mask >> g) & 1u)) continue;
                    const int st = (blk & 1) * kGroups + g;
                    mbar_wait_bounded(full + st, ph, p.status, cta_abort);
                    tc_fence_after();
                    // A: stage st's 32 TMEM columns, 8 per K=16 step; B: the descriptor's
                    // address field advances by 16 B units (stage, then 256 B per K=16 step)
                    const uint32_t ta = tmem_base + kTmemA + static_cast<uint32_t>(st * 32);
                    const uint64_t bd = b_desc0 + static_cast<uint64_t>(st * (xstage >> 4));
#pragma unroll
                    for (int kk = 0; kk < kKChunk / 16; ++kk) {
                        umma_f16_ta(dcol, ta + kk * 8, bd + kk * 16, idesc, acc);
                        acc = 1u;
                    }
                    umma_commit(empty + st);
                }
            }
            umma_commit(acc_full + a);
        }
    };

    if (warp == kProducerWarp) {
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();  // weights are read once per step
            uint32_t rc = 0;
            int r = 0;
            for (int t = tile_first; t < p.total_tiles; t += tile_step) {
                const MmaSeg sg = seg_s[mma_seg_of_tile(p, t)];
                const int lt = t - sg.tile0;
                const bool pair = sg.w1 >= 0;
                // the tile's two row groups: rows 0-63 and 64-127 of a plain tile, or
                // row group lt of the gate and of the up matrix
                const MmaWeight &wa = p.w[sg.w0], &wb = pair ? p.w[sg.w1] : p.w[sg.w0];
                const long ga = pair ? lt : 2L * lt, gb = pair ? lt : 2L * lt + 1;
                for (int b = b0; b < b1; ++b, ++rc) {
                    if (rc >= static_cast<uint32_t>(nraw))
                        mbar_wait_bounded(empty_raw + r, ((rc / nraw) - 1) & 1, p.status, cta_abort);
                    uint8_t *dst = smem + L.raw + r * kRawStageBytes;
                    if (sg.type == kQ4K) {
                        mbar_arrive_expect_tx(full_raw + r, 2 * kMmaChunkQ4);
                        bulk_g2s_evict_first(dst, wa.chunks + (ga * nb + b) * kMmaChunkQ4, kMmaChunkQ4, full_raw + r, pol);
                        bulk_g2s_evict_first(dst + kMmaChunkQ4, wb.chunks + (gb * nb + b) * kMmaChunkQ4, kMmaChunkQ4, full_raw + r, pol);
                    } else {
                        const uint8_t *ca = wa.chunks + (ga * nb + b) * kMmaChunkQ6;
                        const uint8_t *cb = wb.chunks + (gb * nb + b) * kMmaChunkQ6;
                        mbar_arrive_expect_tx(full_raw + r, 2 * kMmaChunkQ6);
                        bulk_g2s_evict_first(dst, ca, kMmaChunkQ6Body, full_raw + r, pol);
                        bulk_g2s_evict_first(dst + kMmaChunkQ6Body, cb, kMmaChunkQ6Body, full_raw + r, pol);
                        bulk_g2s_evict_first(dst + kQ6DOff, ca + kMmaChunkQ6Body, kMmaRowGroup * 2, full_raw + r, pol);
                        bulk_g2s_evict_first(dst + kQ6DOff + kMmaRowGroup * 2, cb + kMmaChunkQ6Body, kMmaRowGroup * 2, full_raw + r, pol);
                    }
                    if (++r == nraw) r = 0;
                }
            }
        }
    } else if (warp == kXWarp) {
        if (lane == 0) {
            pdl_wait();  // the activation is written by the previous kernel
            // block column B (counted over this CTA's work) uses stages (B & 1) * 4 + g,
            // each for the (B >> 1)-th time
            uint32_t blk = 0;
            const uint32_t xbytes = static_cast<uint32_t>(n_pad) * kKChunk * 2;
            for (int t = tile_first; t < p.total_tiles; t += tile_step) {
                for (int b = b0; b < b1; ++b, ++blk) {
                    const uint32_t use = blk >> 1;
                    for (int g = 0; g < kGroups; ++g) {
                        const int st = (blk & 1) * kGroups + g;
                        if (use) mbar_wait_bounded(empty + st, (use - 1) & 1, p.status, cta_abort);
                        mbar_arrive_expect_tx(full + st, xbytes);
                        bulk_g2s(x16_s + st * xstage, p.x16 + static_cast<long>(b * kGroups + g) * xbytes,
                                 xbytes, full + st);
                    }
                }
            }
        }
    } else if (warp == kMmaWarp || warp == kMma2Warp) {
        if (lane == 0) mma_loop(warp == kMmaWarp ? 0x5u : 0xAu, warp == kMmaWarp ? 0u : kTmemAcc1);
    } else {
        const bool conv = warp >= kConvWarp0;
        if (conv) {
            // ---------------------------------------------------------- dequant
            // four groups of four warps; group g converts group g of every block
            // column, warp w covers the rows of TMEM lane quadrant w % 4
            const int g = (warp - kConvWarp0) / 4;
            const int row = (warp & 3) * 32 + lane;
            const uint32_t tmem_lane = tmem_base + (static_cast<uint32_t>((warp & 3) * 32) << 16) + kTmemA;
            uint32_t blk = 0;
            int r = 0;
            for (int t = tile_first; t < p.total_tiles; t += tile_step) {
                const MmaSeg sg = seg_s[mma_seg_of_tile(p, t)];
                const float scale = ldexpf(1.0f, wexp_s[row >= 64 && sg.w1 >= 0 ? sg.w1 : sg.w0]);
                for (int b = b0; b < b1; ++b, ++blk) {
                    const int st = (blk & 1) * kGroups + g;
                    const uint32_t use = blk >> 1;
                    const uint32_t tmem_row = tmem_lane + static_cast<uint32_t>(st * 32);
                    mbar_wait_bounded(full_raw + r, (blk / nraw) & 1, p.status, cta_abort);
                    if (use) mbar_wait_bounded(empty + st, (use - 1) & 1, p.status, cta_abort);
                    tc_fence_after();
                    const uint8_t *raw = smem + L.raw + r * kRawStageBytes;
                    if (sg.type == kQ4K) convert_q4(raw, tmem_row, row, g, scale);
                    else convert_q6(raw, tmem_row, row, g, scale);
                    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(full + st);
                        mbar_arrive(empty_raw + r);
                    }
                    if (++r == nraw) r = 0;
                }
            }
        }
        if (!conv || single) {
            // ---------------------------------------------------------- epilogue
            // Run by the four epilogue warps, joined by the sixteen converter warps
            // (then idle) when the CTA has a single tile: E threads, e = 0..E-1.
            const int E = single ? kEpiThreadsSingle : 128;
            const int bar_id = single ? 2 : 1;
            const int e = conv ? (4 + warp - kConvWarp0) * 32 + lane : (warp - kEpiWarp0) * 32 + lane;
            const int quad = warp & 3;  // TMEM lanes [32*quad, 32*quad + 32)
            const int dr = quad * 32 + lane;  // the tile row this thread drains from TMEM
            // drain: 16-column blocks of the accumulators; with one tile the four
            // converter warps of a quadrant take one block each, else the epilogue
            // warp of the quadrant takes all
            const int jq = conv ? (warp - kConvWarp0) / 4 : -1;
            const int cb_first = single ? jq : 0, cb_step = single ? 4 : 1;
            if (!conv) pdl_wait();
            float *xinv_s = reinterpret_cast<float *>(smem + L.tok);
            int *pos_s = reinterpret_cast<int *>(xinv_s + kMmaMaxNWide), *slot_s = pos_s + kMmaMaxNWide;
            unsigned long long *keys_s = reinterpret_cast<unsigned long long *>(slot_s + kMmaMaxNWide);
            if (!conv && dr < n_pad) {
                xinv_s[dr] = p.x_inv[dr];
                pos_s[dr] = p.tok_pos && dr < p.batch ? p.tok_pos[dr] : 0;
                slot_s[dr] = p.tok_slot && dr < p.batch ? p.tok_slot[dr] : 0;
                keys_s[dr] = 0ull;
            }
            named_bar_sync(bar_id, E);
            const EpiTok tk{xinv_s, pos_s, slot_s, keys_s};
            bool any_logits = false;
            const int per = split_per(p.batch, ksplit);  // tokens of each part's epilogue slice
            const int r = e & 127, ph = e >> 7, nph = E >> 7;  // row and token phase of the row work
            uint32_t i = 0;
            for (int t = tile_first; t < p.total_tiles; t += tile_step, ++i) {
                const MmaSeg sg = seg_s[mma_seg_of_tile(p, t)];
                const int lt = t - sg.tile0;
                const int a = i & 1;
                // the tile's row bookkeeping, done while its accumulator is still being summed
                bool valid;
                const int row = tile_row(sg, lt, r, valid);
                EpiRow er = make_epi_row(p, sg, row, valid);
                if (sg.w1 >= 0 && r >= 64) {  // up-row threads also finish gate row r - 64 (SiLU pass)
                    bool v2;
                    const int row2 = tile_row(sg, lt, r - 64, v2);
                    er.out_pair = sg.out + sg.row_offset + row2;
                    er.valid_pair = v2;
                }
                any_logits |= sg.epi == kEpiLogitsArgmax;
                const float wscale = ldexpf(1.0f, -wexp_s[dr >= 64 && sg.w1 >= 0 ? sg.w1 : sg.w0]);
                const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
                // the bulk stores of the previous tile have finished reading the staging tile
                if (i > 0) {
                    if (warp == kEpiWarp0) bulk_wait_read();
                    named_bar_sync(bar_id, E);
                }
                // ... and (split K) every part has read its slice of this CTA's previous tile
                if (ksplit > 1 && i > 0) mbar_wait_cluster_bounded(part_free, (i - 1) & 1, p.status, cta_abort);
                mbar_wait_bounded(acc_full + a, (i >> 1) & 1, p.status, cta_abort);
                tc_fence_after();
                // accumulator chains -> stage[token][row], summed in a fixed order and scaled
                float *stage = red;
                if (cb_first >= 0) {
                    // 8 columns at a time: chain 0 + chain 1
                    for (int c0 = cb_first * 16; c0 < n_pad; c0 += cb_step * 16) {
#pragma unroll 1
                        for (int h = 0; h < 16; h += 8) {
                            const int c = c0 + h;
                            uint32_t v[8], w[8];
                            float sum[8];
                            tmem_ld8_nw(taddr + a * n_pad + c, v);
                            tmem_ld8_nw(taddr + kTmemAcc1 + a * n_pad + c, w);
                            tmem_wait8(v);
                            tmem_wait8(w);
#pragma unroll
                            for (int k = 0; k < 8; ++k) sum[k] = __uint_as_float(v[k]) + __uint_as_float(w[k]);
#pragma unroll
                            for (int k = 0; k < 8; ++k) stage[(c + k) * kStage + dr] = sum[k] * wscale * xinv_s[c + k];
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (!single && lane == 0) mbar_arrive(acc_empty + a);
                int t_lo = 0, t_hi = p.batch;
                if (ksplit > 1) {
                    // the parts signal each other that their partial tiles are staged, then
                    // part s sums its token slice of every part's tile over the cluster's
                    // shared memory (DSMEM), in part order, so the result does not depend on
                    // timing; the sums overwrite the slice in this CTA's own tile
                    named_bar_sync(bar_id, E);
                    if (warp == kEpiWarp0 && lane < ksplit) {
                        asm volatile("fence.acq_rel.cluster;" ::: "memory");
                        mbar_arrive_remote(part_ready, lane);
                    }
                    const bool ok = mbar_wait_cluster_bounded(part_ready, i & 1, p.status, cta_abort);
                    t_lo = min(p.batch, rank * per);
                    t_hi = ok ? min(p.batch, t_lo + per) : t_lo;
                    // items of four rows x one token, a warp covering one token's 128 rows
                    const int items = (t_hi - t_lo) * 32;
                    const uint32_t base = smem_u32(stage);
                    for (int it = e; it < items; it += E) {
                        const uint32_t off = static_cast<uint32_t>(((t_lo + (it >> 5)) * kStage + (it & 31) * 4) * 4);
                        float4 y = make_float4(0.f, 0.f, 0.f, 0.f);
                        for (int q0 = 0; q0 < ksplit; q0 += 4) {  // four loads in flight, summed in part order
                            float4 v[4];
#pragma unroll
                            for (int q = 0; q < 4; ++q)
                                if (q0 + q < ksplit) v[q] = dsmem_ld4(dsmem_addr(base + off, q0 + q));
#pragma unroll
                            for (int q = 0; q < 4; ++q) {
                                if (q0 + q < ksplit) {
                                    y.x += v[q].x; y.y += v[q].y; y.z += v[q].z; y.w += v[q].w;
                                }
                            }
                        }
                        *reinterpret_cast<float4 *>(reinterpret_cast<uint8_t *>(stage) + off) = y;
                    }
                    // the peers may refill their tiles once every part has read its slice
                    if (t + tile_step < p.total_tiles) {
                        named_bar_sync(bar_id, E);
                        if (warp == kEpiWarp0 && lane < ksplit) {
                            asm volatile("fence.acq_rel.cluster;" ::: "memory");
                            mbar_arrive_remote(part_free, lane);
                        }
                    }
                }
                named_bar_sync(bar_id, E);
                // rows this tile writes and whether whole token rows can go out as bulk stores
                const int row0 = sg.w1 >= 0 ? lt * 64 : lt * 128;
                const int count = min(sg.w1 >= 0 ? 64 : 128, sg.rows - row0);
                float *gbase = sg.out + sg.row_offset + row0;
                const bool bulk_kind = sg.epi == kEpiStore || sg.epi == kEpiAdd || sg.epi == kEpiSiluPair ||
                                       sg.epi == kEpiRopeQ || sg.epi == kEpiLogitsArgmax;
                const bool bulk = p.bulk_out && bulk_kind && count > 0 && (count & 3) == 0 &&
                                  (sg.out_stride & 3) == 0 && (reinterpret_cast<uintptr_t>(gbase) & 15) == 0;
                epi_rows(p, er, tk, stage, r, t_lo + ph, nph, t_hi, bulk);
                if (sg.epi == kEpiLogitsArgmax) {
                    named_bar_sync(bar_id, E);
                    if (!conv) epi_argmax(stage, tk, sg.key_offset + sg.row_offset + row0, count, t_lo, t_hi);
                }
                if (bulk) {
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    named_bar_sync(bar_id, E);
                    if (warp == kEpiWarp0) {  // one token row per lane at a time
                        for (int n = t_lo + lane; n < t_hi; n += 32) {
                            if (sg.epi == kEpiAdd) bulk_s2g_add(gbase + n * sg.out_stride, stage + n * kStage, count * 4);
                            else bulk_s2g(gbase + n * sg.out_stride, stage + n * kStage, count * 4);
                        }
                        bulk_commit();
                    }
                }
            }
            if (warp == kEpiWarp0) bulk_wait_read();  // the writes complete with the grid
            if (any_logits && !conv) {  // this CTA's best key per token, one global atomic each
                named_bar_sync(1, 128);
                if (dr < p.batch && keys_s[dr]) atomicMax(p.argmax_keys + dr, keys_s[dr]);
            }
        }
    }

    tc_fence_before();
    __syncwarp();
    cluster_sync_all();  // no CTA leaves while a peer may still read its shared memory
    tc_fence_after();
    if (warp == kMmaWarp)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(tmem_cols)
                     : "memory");
}

// --------------------------------------------------------- activation prep --

// One token by NT threads (tid 0..NT-1, synchronising on named barrier bar_id;
// part_s/amax_s: 2 * NT/32 floats of shared memory each, double-buffered by
// `parity` so that consecutive tokens need no extra barrier): the GEMV
// prologue's arithmetic (RMSNorm, the reference's per-32 int8 quantisation)
// then x^ = q * scale (DP4A semantics) or x (FP32 semantics), times 2^kx so
// that max|x^| lies in [2^14, 2^15), rounded to fp16 into the MMA layout:
// chunk c (64 wide) is [n/8][core j][n%8][8 values] with core j holding
// 64c + 4j + {0,2,1,3} and 64c + 32 + 4j + {0,2,1,3}.  Each thread owns cores;
// the 8 cores of a chunk sit on 8 adjacent lanes, so a 32-wide quantisation
// group is an 8-lane shuffle reduction.  With wait_pdl the norm weights are
// read before griddepcontrol.wait (they do not depend on the previous kernel)
// and everything else after it.
template <int NT>
__device__ void mma_prep_token_t(const float *x, long x_stride, const float *norm_w, float eps, int cols, int batch,
                                 int n, int n_pad, int use_dp4a, uint8_t *x16, float *x_inv, int tid, int bar_id,
                                 float *part_s, float *amax_s, int parity, bool wait_pdl) {
    constexpr int W = NT / 32;
    constexpr int kPer = kMaxCols / (NT * 8);
    const int lane = tid & 31, warp = tid >> 5;
    part_s += parity * W;
    amax_s += parity * W;
    const long chunk_bytes = static_cast<long>(n_pad) * kKChunk * 2;
    const int cores = cols / 8;
    auto dst_of = [&](int core) -> uint8_t * {
        return x16 + (core >> 3) * chunk_bytes + (n >> 3) * kGroupStride + (core & 7) * kCoreStride + (n & 7) * 16;
    };
    // the norm weight of every value this thread owns
    float wv[kPer][8];
    if (norm_w && n < batch) {
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            const int core = tid + NT * j;
            if (core >= cores) continue;
            const int k0 = (core >> 3) * 64 + (core & 7) * 4;
            const float4 wa = __ldg(reinterpret_cast<const float4 *>(norm_w + k0));
            const float4 wb = __ldg(reinterpret_cast<const float4 *>(norm_w + k0 + 32));
            wv[j][0] = wa.x; wv[j][1] = wa.y; wv[j][2] = wa.z; wv[j][3] = wa.w;
            wv[j][4] = wb.x; wv[j][5] = wb.y; wv[j][6] = wb.z; wv[j][7] = wb.w;
        }
    }
    if (wait_pdl) pdl_wait();
    if (n >= batch) {
        for (int c = tid; c < cores; c += NT) *reinterpret_cast<uint4 *>(dst_of(c)) = make_uint4(0, 0, 0, 0);
        if (tid == 0) x_inv[n] = 0.f;
        return;
    }
    const float *xr = x + n * x_stride;
    float vals[kPer][8];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
        const int core = tid + NT * j;
        if (core >= cores) continue;
        const int k0 = (core >> 3) * 64 + (core & 7) * 4;  // first of the low four; +32 for the high four
        const float4 a = *reinterpret_cast<const float4 *>(xr + k0);
        const float4 b = *reinterpret_cast<const float4 *>(xr + k0 + 32);
        vals[j][0] = a.x; vals[j][1] = a.y; vals[j][2] = a.z; vals[j][3] = a.w;
        vals[j][4] = b.x; vals[j][5] = b.y; vals[j][6] = b.z; vals[j][7] = b.w;
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = fmaf(vals[j][e], vals[j][e], ss);
    }
    float r = 1.f;
    if (norm_w) {  // RMSNorm: warp sums, then the warp partials in a fixed order
        ss = warp_sum(ss);
        if (lane == 0) part_s[warp] = ss;
        named_bar_sync(bar_id, NT);
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < W; ++w) tot += part_s[w];
        r = rsqrtf(tot / static_cast<float>(cols) + eps);
    }
    float local_max = 0.f;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
        const int core = tid + NT * j;
        if (core >= cores) continue;  // warp-uniform: cores is a multiple of 32
        float *v = vals[j];
        if (norm_w) {
#pragma unroll
            for (int e = 0; e < 8; ++e) v[e] = __fmul_rn(__fmul_rn(v[e], r), wv[j][e]);
        }
        if (use_dp4a) {
            // quantize_x32_cuda (inferencer.cu:544-556): groups 64c..64c+31 (v[0..3] of
            // the chunk's 8 lanes) and 64c+32..64c+63 (v[4..7])
            float am0 = 0.f, am1 = 0.f;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                am0 = fmaxf(am0, fabsf(v[e]));
                am1 = fmaxf(am1, fabsf(v[4 + e]));
            }
#pragma unroll
            for (int o = 1; o < 8; o <<= 1) {
                am0 = fmaxf(am0, __shfl_xor_sync(0xffffffffu, am0, o));
                am1 = fmaxf(am1, __shfl_xor_sync(0xffffffffu, am1, o));
            }
            const float sc0 = am0 > 0.f ? am0 / 127.f : 1.f, sc1 = am1 > 0.f ? am1 / 127.f : 1.f;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const float scale = e < 4 ? sc0 : sc1;
                int q = __float2int_rn(v[e] / scale);
                q = max(-127, min(127, q));
                v[e] = static_cast<float>(q) * scale;
            }
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) local_max = fmaxf(local_max, fabsf(v[e]));
    }
    local_max = warp_max(local_max);
    if (lane == 0) amax_s[warp] = local_max;
    named_bar_sync(bar_id, NT);
    float amax = 0.f;
#pragma unroll
    for (int w = 0; w < W; ++w) amax = fmaxf(amax, amax_s[w]);
    int e2 = 0;
    if (amax > 0.f) frexpf(amax, &e2);
    const int kx = amax > 0.f ? 15 - e2 : 0;  // amax * 2^kx in [2^14, 2^15)
    const float up = ldexpf(1.0f, kx);
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
        const int core = tid + NT * j;
        if (core >= cores) continue;
        const float *v = vals[j];
        const uint4 o = make_uint4(pack_half2(v[0] * up, v[2] * up), pack_half2(v[1] * up, v[3] * up),
                                   pack_half2(v[4] * up, v[6] * up), pack_half2(v[5] * up, v[7] * up));
        *reinterpret_cast<uint4 *>(dst_of(core)) = o;
    }
    if (tid == 0) x_inv[n] = ldexpf(1.0f, -kx);
}

__device__ void mma_prep_token(const float *x, long x_stride, const float *norm_w, float eps, int cols, int batch, int n,
                               int n_pad, int use_dp4a, uint8_t *x16, float *x_inv) {
    __shared__ float part_s[16], amax_s[16];
    mma_prep_token_t<256>(x, x_stride, norm_w, eps, cols, batch, n, n_pad, use_dp4a, x16, x_inv,
                          static_cast<int>(threadIdx.x), 0, part_s, amax_s, 0, false);
}

// One CTA of NT threads per token.  256 for every row width: wider CTAs for
// the 8192-wide input of the down projection shorten the prep alone but make the
// step slower (measured on B200, ragged64: 1.794 ms with 1024 threads for it,
// 1.784 ms with 256), presumably because they hold whole SMs that the next
// GEMM's CTAs wait for.
template <int NT>
__global__ void __launch_bounds__(NT) ijb_mma_prep_kernel(const float *x, long x_stride, const float *norm_w, float eps,
                                                          int cols, int batch, int n_pad, int use_dp4a, uint8_t *x16,
                                                          float *x_inv) {
    __shared__ float part_s[2 * (NT / 32)], amax_s[2 * (NT / 32)];
    pdl_trigger();
    mma_prep_token_t<NT>(x, x_stride, norm_w, eps, cols, batch, static_cast<int>(blockIdx.x), n_pad, use_dp4a, x16,
                         x_inv, static_cast<int>(threadIdx.x), 0, part_s, amax_s, 0, true);
}

// Bound of max|w| over GGUF blocks: Q4_K |d|*63*15 + |dmin|*63, Q6_K
// |d|*128*32; atomicMax on the float's bits (non-negative floats order as
// integers).
__global__ void ijb_mma_scale_scan_kernel(int type, const uint8_t *w, long nblocks, unsigned int *out) {
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
        if (bound != bound) bound = 0.f;                // a NaN scale makes only its own block NaN
        else if (!(bound <= 3.0e38f)) bound = 3.0e38f;  // inf scales
        best = fmaxf(best, bound);
    }
    best = warp_max(best);
    if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(best));
}

// ------------------------------------------------------------------- host --

cudaError_t mma_prep_launch(const float *x, long x_stride, const float *norm_w, float eps, int cols, int batch,
                            int n_pad, int use_dp4a, uint8_t *x16, float *x_inv, cudaStream_t stream, bool pdl) {
    if (cols % 256 || cols > kMaxCols || batch < 1 || n_pad > kMmaMaxNWide || n_pad % 16) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(n_pad);
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, ijb_mma_prep_kernel<256>, x, x_stride, norm_w, eps, cols, batch, n_pad, use_dp4a, x16,
                              x_inv);
}

cudaError_t mma_scale_scan_launch(int type, const uint8_t *w, long nblocks, int *out_max_bits, cudaStream_t stream) {
    cudaError_t e = cudaMemsetAsync(out_max_bits, 0, sizeof(int), stream);
    if (e != cudaSuccess) return e;
    ijb_mma_scale_scan_kernel<<<256, 256, 0, stream>>>(type, w, nblocks, reinterpret_cast<unsigned int *>(out_max_bits));
    return cudaGetLastError();
}

// ------------------------------------------------------- chunked weights --

long mma_tile_bytes(int type, int rows, int cols) {
    const long groups = ((rows + kMmaRowGroup - 1) / kMmaRowGroup + 1) / 2 * 2;
    return groups * (cols / 256) * (type == kQ4K ? kMmaChunkQ4 : kMmaChunkQ6);
}

// One CTA per (row group, block column), one thread per row of the group.
__global__ void ijb_mma_tile_repack_kernel(int type, const uint8_t *src, long row_bytes, int rows, int nb, uint8_t *dst) {
    const long g = blockIdx.x / nb;
    const int b = blockIdx.x % nb, i = threadIdx.x;
    const long row = g * kMmaRowGroup + i;
    uint8_t *chunk = dst + static_cast<long>(blockIdx.x) * (type == kQ4K ? kMmaChunkQ4 : kMmaChunkQ6);
    if (type == kQ4K) {
        uint4 *o = reinterpret_cast<uint4 *>(chunk + i * 144);
        const uint4 *in = reinterpret_cast<const uint4 *>(src + row * row_bytes + b * 144L);
        for (int k = 0; k < 9; ++k) o[k] = row < rows ? in[k] : make_uint4(0, 0, 0, 0);
    } else {
        // unit layout (gemv.cuh): unit u of kUnitBlocks blocks holds their bodies, then their d values
        const int u = b / kUnitBlocks, lb = b % kUnitBlocks, n_u = min(kUnitBlocks, nb - u * kUnitBlocks);
        const uint8_t *unit = src + row * row_bytes + static_cast<long>(u) * q6_unit_bytes(kUnitBlocks);
        uint4 *o = reinterpret_cast<uint4 *>(chunk + i * 208);
        const uint4 *in = reinterpret_cast<const uint4 *>(unit + lb * 208);
        for (int k = 0; k < 13; ++k) o[k] = row < rows ? in[k] : make_uint4(0, 0, 0, 0);
        reinterpret_cast<uint16_t *>(chunk + kMmaChunkQ6Body)[i] =
            row < rows ? *reinterpret_cast<const uint16_t *>(unit + n_u * 208 + lb * 2) : 0;
    }
}

cudaError_t mma_tile_repack_launch(int type, const uint8_t *src, long row_bytes, int rows, int cols, uint8_t *dst,
                                   cudaStream_t stream) {
    if ((type != kQ4K && type != kQ6K) || cols % 256 || rows < 1 || (row_bytes & 15) ||
        (reinterpret_cast<uintptr_t>(src) & 15) || (reinterpret_cast<uintptr_t>(dst) & 15))
        return cudaErrorInvalidValue;
    const int nb = cols / 256;
    const long groups = mma_tile_bytes(type, rows, cols) / (static_cast<long>(nb) * (type == kQ4K ? kMmaChunkQ4 : kMmaChunkQ6));
    ijb_mma_tile_repack_kernel<<<static_cast<unsigned>(groups * nb), kMmaRowGroup, 0, stream>>>(type, src, row_bytes, rows,
                                                                                            nb, dst);
    return cudaGetLastError();
}

// Clusters of k CTAs (one CTA per SM) that can be resident at once, k = 1..8.
static int g_cluster_cap[kMaxCluster + 1];
static std::mutex g_cap_mu;

cudaError_t mma_prepare() {
    cudaError_t e =
        cudaFuncSetAttribute(ijb_mma_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, mma_smem().total);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(g_cap_mu);
    int dev = 0, sms = 0;
    e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    g_cluster_cap[1] = sms;
    for (int k = 2; k <= kMaxCluster; ++k) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(k);
        cfg.blockDim = dim3(kMmaThreads);
        cfg.dynamicSmemBytes = mma_smem().total;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = k;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, ijb_mma_gemm_kernel, &cfg) != cudaSuccess) {
            cudaGetLastError();
            n = 0;
        }
        g_cluster_cap[k] = n;
    }
    return cudaSuccess;
}

int mma_choose_split(int tiles, int nblocks, int max_split, int split_cost, int *bps) {
    // cost ~ waves of clusters x block columns per part, plus split_cost block
    // columns' time for the exchange of partial sums when the K range is split
    int best_k = 1, best_cost = 0;
    for (int k = 1; k <= kMaxCluster && k <= nblocks && k <= max_split; ++k) {
        const int per = (nblocks + k - 1) / k;
        if ((nblocks + per - 1) / per != k) continue;  // every part non-empty
        const int cap = g_cluster_cap[k];
        if (cap < 1) continue;
        const int waves = (tiles + cap - 1) / cap;
        const int cost = waves * per + (k > 1 ? split_cost : 0);
        if (k == 1 || cost < best_cost) {
            best_k = k;
            best_cost = cost;
        }
    }
    *bps = (nblocks + best_k - 1) / best_k;
    return best_k;
}

bool mma_wide_ok(int tiles, int ksplit) {
    return ksplit >= 1 && ksplit <= kMaxCluster && tiles >= 1 && g_cluster_cap[ksplit] >= tiles;
}

cudaError_t mma_gemm_launch(const MmaParams &p, cudaStream_t stream, bool pdl) {
    if (p.n_pad > kMmaMaxN && !mma_wide_ok(p.total_tiles, p.ksplit)) return cudaErrorInvalidValue;
    if (p.n_pad < 16 || p.n_pad > kMmaMaxNWide || p.n_pad % 16 || p.cols % 256 || p.total_tiles < 1 || p.ksplit < 1 ||
        p.ksplit > kMaxCluster || p.bps < 1 || (p.ksplit - 1) * p.bps >= p.cols / 256 ||
        p.ksplit * p.bps < p.cols / 256 || g_cluster_cap[p.ksplit] < 1)
        return cudaErrorInvalidValue;
    const int clusters = p.total_tiles < g_cluster_cap[p.ksplit] ? p.total_tiles : g_cluster_cap[p.ksplit];
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(clusters * p.ksplit);
    cfg.blockDim = dim3(kMmaThreads);
    cfg.dynamicSmemBytes = mma_smem().total;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = p.ksplit;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, ijb_mma_gemm_kernel, p);
}

}  // namespace ijb
