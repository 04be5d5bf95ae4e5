// Fused Q4_K / Q6_K GEMV and skinny GEMM (1..8 tokens) on CUDA cores, sm_100a.
//
// Replaces the reference's one-warp-per-row kernels gemv_q4_dp4a,
// gemv_q6_dp4a, gemv_quant<T>, qkv_cuda, gate_up_cuda and gemv_batch_dp4a
// (inferencer.cu:558-804) together with the small kernels that run around them
// (rmsnorm_quantize_cuda :839, quantize_x32_cuda :544, rope_cache_cuda :930,
// cache_cuda :919, add_cuda :1043, silu_cuda :1053, argmax :1063-1099).
//
// One launch is a persistent grid of 8-warp CTAs: two per SM (four for a long
// one-token stream such as the lm_head); two leave room on the SM for the next
// kernel's CTAs.  Every warp works
// on its own list of rows (or row pairs) and streams them through a private
// ring of shared-memory slots with cp.async.bulk (the TMA engine's 1-D copy),
// completing on one mbarrier per slot; lane 0 keeps kDepth units of 2048
// weights in flight.  The first copies are issued before griddepcontrol.wait,
// so a kernel's weights stream in while the previous kernel finishes.  After
// the wait, all warps build the activation in shared memory once (optional
// RMSNorm, then the reference's per-32 int8 quantisation for the DP4A path,
// fp32 for the FP32 path); from then on warps never synchronise with each
// other.  Each lane covers 64 weights of a unit (one 32-weight sub-block pair
// of Q4_K or one 16-position column of a Q6_K 128-weight group), so block
// scales are decoded once per 64 weights.  A row's lane sums are reduced with
// shuffles when its last unit is done, and the warp writes the fused
// epilogue: store, residual add, RoPE on a row pair into q or the paged K
// cache, V store, SiLU * up on a gate/up pair, or logits with an argmax key.
#include "common.cuh"
#include "gemv.cuh"

namespace ijb {

constexpr int kWarps = 8;          // 2 CTAs fit per SM, so the next kernel's CTA prefetches alongside
constexpr int kThreads = kWarps * 32;
#ifndef IJB_GEMV_DEPTH
#define IJB_GEMV_DEPTH 3
#endif
constexpr int kDepth = IJB_GEMV_DEPTH;  // units in flight per warp
constexpr int kSlotBytes = 1680;   // largest unit: 8 Q6_K blocks (8 Q4_K blocks: 1152)
constexpr int kNormThreads = 256;  // the reference's RMSNorm reduction width

// Shared memory: per-warp slot rings, their mbarriers, the RMSNorm partials,
// then the activation of every token.  The int8 activation is stored in the
// order lanes read it, separately for each weight format in the launch, so
// every 128-bit shared load of the dot products is free of bank conflicts:
//   q6: [b][unit][part 0..3][lane 0..31] 16 bytes, plus per lane an int4 of
//       its four 16-value code sums and a float4 of its four group scales;
//   q4: [b][unit][chunk 0..3][lane 0..31] 16 bytes (chunks: low-nibble
//       sub-block positions 0-15, 16-31, then high-nibble ones), an int4 of
//       the chunks' code sums and a float2 of the two sub-blocks' scales.
struct SmemLayout {
    int ring, bars, red, q6x, q6s, q6f, q4x, q4s, q4f, xf, xsumf, total;
};

__host__ __device__ inline int align_up(int v, int a) { return (v + a - 1) / a * a; }

__host__ __device__ inline SmemLayout smem_layout(int cols, int batch, int need_q4, int need_q6, int need_f) {
    SmemLayout L;
    const int U = (cols / 256 + kUnitBlocks - 1) / kUnitBlocks;  // units per row
    int off = 0;
    L.ring = off;
    off += kWarps * kDepth * kSlotBytes;
    off = align_up(off, 8);
    L.bars = off;
    off += kWarps * kDepth * 8;
    L.red = off;
    off += kNormThreads * 4;
    off = align_up(off, 16);
    L.q6x = off;
    if (need_q6) off += batch * U * 2048;
    L.q6s = off;
    if (need_q6) off += batch * U * 32 * 16;
    L.q6f = off;
    if (need_q6) off += batch * U * 32 * 16;
    L.q4x = off;
    if (need_q4) off += batch * U * 2048;
    L.q4s = off;
    if (need_q4) off += batch * U * 32 * 16;
    L.q4f = off;
    if (need_q4) off += batch * U * 32 * 8;
    off = align_up(off, 16);
    L.xf = off;
    if (need_f) off += batch * cols * 4;
    L.xsumf = off;
    if (need_f) off += batch * (cols / 16) * 4;
    L.total = align_up(off, 128);
    return L;
}

// Lane of quarter j (0..3) of block blk (0..7) of a Q6_K unit, and back: blocks
// b and b + 4 share each 8-lane phase of a warp's 16-byte shared-memory loads,
// and as the unit's block bodies are 208 bytes apart their 64-byte pieces fall
// in opposite halves of the banks (blocks b and b + 1 would overlap in 4 banks).
__device__ __forceinline__ int q6_lane(int blk, int j) { return 8 * (blk & 3) + 4 * (blk >> 2) + j; }
__device__ __forceinline__ int q6_blk(int lane) { return ((lane >> 3) & 3) + 4 * ((lane >> 2) & 1); }

// ---------------------------------------------------------------- prologue --

// Builds the activation of every token in shared memory.  RMSNorm follows
// rmsnorm_cuda (inferencer.cu:821-834) including its reduction order: 256
// strided partial sums of x*x, a shared-memory tree, rsqrtf(sum/n + eps),
// out = x * scale * w.  The int8 path follows quantize_x32_cuda (:544-556):
// per 32 values scale = amax > 0 ? amax / 127 : 1 and
// q = clamp(rn(v / scale), -127, 127).  Per-16 sums of q (and of v for the FP32
// path) feed the Q4_K min term and the Q6_K zero point.
__device__ void build_activation(const GemvParams &p, const SmemLayout &L, uint8_t *smem) {
    const int tid = threadIdx.x;
    const int K = p.cols;
    float *red = reinterpret_cast<float *>(smem + L.red);
    float *xf = reinterpret_cast<float *>(smem + L.xf);
    float *xsumf = reinterpret_cast<float *>(smem + L.xsumf);
    const int U = (K / 256 + kUnitBlocks - 1) / kUnitBlocks;
    const int chunks = (K / 8 + kThreads - 1) / kThreads;  // 8-element chunks per thread
    for (int b = 0; b < p.batch; ++b) {
        const float *x = p.x + b * p.x_stride;
        float r = 1.f;
        if (p.norm_w) {
            if (tid < kNormThreads) {
                float s = 0.f;
#pragma unroll 4
                for (int i = tid; i < K; i += kNormThreads) s = fmaf(x[i], x[i], s);
                red[tid] = s;
            }
            __syncthreads();
            for (int stride = kNormThreads / 2; stride > 0; stride >>= 1) {
                if (tid < stride) red[tid] += red[tid + stride];
                __syncthreads();
            }
            r = rsqrtf(red[0] / static_cast<float>(K) + p.eps);
            __syncthreads();  // red[] is reused for the next token
        }
        // thread t owns chunks c = t + 256*j of 8 consecutive elements: a 32-value
        // group lives in 4 consecutive lanes
        for (int j = 0; j < chunks; ++j) {
            const int c = tid + kThreads * j;
            const bool in = c * 8 < K;  // uniform per group of 4 lanes (K % 32 == 0)
            float v[8];
            if (in) {
                const float4 a = *reinterpret_cast<const float4 *>(x + c * 8);
                const float4 bb = *reinterpret_cast<const float4 *>(x + c * 8 + 4);
                v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
                v[4] = bb.x; v[5] = bb.y; v[6] = bb.z; v[7] = bb.w;
                if (p.norm_w) {
                    const float4 wa = *reinterpret_cast<const float4 *>(p.norm_w + c * 8);
                    const float4 wb = *reinterpret_cast<const float4 *>(p.norm_w + c * 8 + 4);
                    const float w8[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
                    for (int e = 0; e < 8; ++e) v[e] = __fmul_rn(__fmul_rn(v[e], r), w8[e]);
                }
            }
            if (p.need_f) {
                float h = 0.f;
                if (in) {
#pragma unroll
                    for (int e = 0; e < 8; ++e) h += v[e];
                    float4 *dst = reinterpret_cast<float4 *>(xf + b * K + c * 8);
                    dst[0] = make_float4(v[0], v[1], v[2], v[3]);
                    dst[1] = make_float4(v[4], v[5], v[6], v[7]);
                }
                h += __shfl_xor_sync(0xffffffffu, h, 1);  // 16 values = 2 lanes
                if (in && (tid & 1) == 0) xsumf[b * (K / 16) + c / 2] = h;
            }
            if (p.need_q4 | p.need_q6) {
                float amax = 0.f;
                if (in) {
#pragma unroll
                    for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(v[e]));
                }
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));  // 32 values = 4 lanes
                const float scale = amax > 0.f ? amax / 127.f : 1.f;
                int hs = 0;
                uint32_t packed[2] = {0u, 0u};
                if (in) {
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        int q = __float2int_rn(v[e] / scale);
                        q = max(-127, min(127, q));
                        hs += q;
                        packed[e >> 2] |= (static_cast<uint32_t>(q) & 255u) << ((e & 3) * 8);
                    }
                }
                hs += __shfl_xor_sync(0xffffffffu, hs, 1);  // 16 values = 2 lanes
                if (in) {
                    const int p0 = c * 8;
                    const int u = p0 / 2048, q = p0 % 2048, blk = q / 256, i = q % 256;
                    const int bu = b * U + u;
                    if (p.need_q6) {
                        const int g = i / 128, pt = (i % 128) / 32, l = i % 32, h = l / 16;
                        const int lane = q6_lane(blk, 2 * g + h);
                        *reinterpret_cast<uint2 *>(smem + L.q6x + ((bu * 4 + pt) * 32 + lane) * 16 + (l % 16)) =
                            make_uint2(packed[0], packed[1]);
                        if ((l % 16) == 0) reinterpret_cast<int *>(smem + L.q6s)[(bu * 32 + lane) * 4 + pt] = hs;
                        if (l == 0) {  // both lanes of this 32-value group use its scale
                            reinterpret_cast<float *>(smem + L.q6f)[(bu * 32 + lane) * 4 + pt] = scale;
                            reinterpret_cast<float *>(smem + L.q6f)[(bu * 32 + lane + 1) * 4 + pt] = scale;
                        }
                    }
                    if (p.need_q4) {
                        const int g = i / 64, hi = (i % 64) / 32, jj = i % 32, ch = hi * 2 + jj / 16;
                        const int lane = 4 * blk + g;
                        *reinterpret_cast<uint2 *>(smem + L.q4x + ((bu * 4 + ch) * 32 + lane) * 16 + (jj % 16)) =
                            make_uint2(packed[0], packed[1]);
                        if ((jj % 16) == 0) reinterpret_cast<int *>(smem + L.q4s)[(bu * 32 + lane) * 4 + ch] = hs;
                        if (jj == 0) reinterpret_cast<float *>(smem + L.q4f)[(bu * 32 + lane) * 2 + hi] = scale;
                    }
                }
            }
        }
    }
}

// ------------------------------------------------------------ dot products --

// Scale / min of Q4_K sub-block j from the 12 packed bytes (q4_scale_min,
// inferencer.cu:489-497).
__device__ __forceinline__ void q4_sm(uint32_t s0, uint32_t s1, uint32_t s2, int j, int &sc, int &m) {
    auto byte = [&](int k) -> int {
        const uint32_t w = k < 4 ? s0 : (k < 8 ? s1 : s2);
        return (w >> ((k & 3) * 8)) & 255;
    };
    if (j < 4) {
        sc = byte(j) & 63;
        m = byte(j + 4) & 63;
    } else {
        sc = (byte(j + 4) & 15) | ((byte(j - 4) >> 6) << 4);
        m = (byte(j + 4) >> 4) | ((byte(j) >> 6) << 4);
    }
}

__device__ __forceinline__ int dp4a(uint32_t a, uint32_t b, int c) {
    return __dp4a(static_cast<int>(a), static_cast<int>(b), c);
}

// One Q4_K unit (up to 8 GGUF blocks, inferencer.cu:453-471) held in shared
// memory.  Lane -> block lane/4 and group g = lane%4: the 32 bytes
// qs[g*32 .. g*32+32] hold sub-block 2g (low nibbles) and 2g+1 (high nibbles).
template <int B>
__device__ __forceinline__ void q4_unit(const uint8_t *unit, int nb_u, int u, int lane, const GemvParams &p,
                                        const SmemLayout &L, const uint8_t *smem, int use_dp4a, float (&acc)[B]) {
    const int gblk0 = u * kUnitBlocks;
    const int blk = lane >> 2, g = lane & 3;
    if (blk >= nb_u) return;
    const uint8_t *bp = unit + blk * 144;
    const uint4 hdr = *reinterpret_cast<const uint4 *>(bp);
    const uint4 q0 = *reinterpret_cast<const uint4 *>(bp + 16 + g * 32);
    const uint4 q1 = *reinterpret_cast<const uint4 *>(bp + 32 + g * 32);
    const float d = half_bits_to_float(hdr.x & 0xffff), dmin = half_bits_to_float(hdr.x >> 16);
    int sc_lo, m_lo, sc_hi, m_hi;
    q4_sm(hdr.y, hdr.z, hdr.w, 2 * g, sc_lo, m_lo);
    q4_sm(hdr.y, hdr.z, hdr.w, 2 * g + 1, sc_hi, m_hi);
    const float a_lo = d * static_cast<float>(sc_lo), b_lo = dmin * static_cast<float>(m_lo);
    const float a_hi = d * static_cast<float>(sc_hi), b_hi = dmin * static_cast<float>(m_hi);
    const int K = p.cols;
    const int base = (gblk0 + blk) * 256 + g * 64;  // first low-nibble position
    const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    if (use_dp4a) {
        uint32_t lo[8], hi[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            lo[j] = w[j] & 0x0F0F0F0Fu;
            hi[j] = (w[j] >> 4) & 0x0F0F0F0Fu;
        }
        const int U = (K / 256 + kUnitBlocks - 1) / kUnitBlocks;
#pragma unroll
        for (int b = 0; b < B; ++b) {
            const int bu = b * U + u;
            const uint4 *xl = reinterpret_cast<const uint4 *>(smem + L.q4x) + bu * 128 + lane;
            const uint4 l0 = xl[0], l1 = xl[32], h0 = xl[64], h1 = xl[96];
            // four independent chains of four (integer sums: the order is free)
            int dl = dp4a(lo[0], l0.x, 0), dl2 = dp4a(lo[4], l1.x, 0);
            int dh = dp4a(hi[0], h0.x, 0), dh2 = dp4a(hi[4], h1.x, 0);
            dl = dp4a(lo[1], l0.y, dl);
            dl2 = dp4a(lo[5], l1.y, dl2);
            dh = dp4a(hi[1], h0.y, dh);
            dh2 = dp4a(hi[5], h1.y, dh2);
            dl = dp4a(lo[2], l0.z, dl);
            dl2 = dp4a(lo[6], l1.z, dl2);
            dh = dp4a(hi[2], h0.z, dh);
            dh2 = dp4a(hi[6], h1.z, dh2);
            dl = dp4a(lo[3], l0.w, dl);
            dl2 = dp4a(lo[7], l1.w, dl2);
            dh = dp4a(hi[3], h0.w, dh);
            dh2 = dp4a(hi[7], h1.w, dh2);
            dl += dl2;
            dh += dh2;
            const int4 s4 = reinterpret_cast<const int4 *>(smem + L.q4s)[bu * 32 + lane];
            const float2 sx = reinterpret_cast<const float2 *>(smem + L.q4f)[bu * 32 + lane];
            float t = fmaf(a_lo, static_cast<float>(dl), -b_lo * static_cast<float>(s4.x + s4.y)) * sx.x;
            t = fmaf(fmaf(a_hi, static_cast<float>(dh), -b_hi * static_cast<float>(s4.z + s4.w)), sx.y, t);
            acc[b] += t;
        }
    } else {
        const float *xf = reinterpret_cast<const float *>(smem + L.xf);
        const float *xsumf = reinterpret_cast<const float *>(smem + L.xsumf);
#pragma unroll
        for (int b = 0; b < B; ++b) {
            const float *xl = xf + b * K + base;
            float sl = 0.f, sh = 0.f;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint32_t lo = w[j] & 0x0F0F0F0Fu, hi = (w[j] >> 4) & 0x0F0F0F0Fu;
                const float4 a = *reinterpret_cast<const float4 *>(xl + 4 * j);
                const float4 h = *reinterpret_cast<const float4 *>(xl + 32 + 4 * j);
                sl = fmaf(byte_to_float(lo, 0x7440), a.x, sl);
                sl = fmaf(byte_to_float(lo, 0x7441), a.y, sl);
                sl = fmaf(byte_to_float(lo, 0x7442), a.z, sl);
                sl = fmaf(byte_to_float(lo, 0x7443), a.w, sl);
                sh = fmaf(byte_to_float(hi, 0x7440), h.x, sh);
                sh = fmaf(byte_to_float(hi, 0x7441), h.y, sh);
                sh = fmaf(byte_to_float(hi, 0x7442), h.z, sh);
                sh = fmaf(byte_to_float(hi, 0x7443), h.w, sh);
            }
            const float4 f4 = *reinterpret_cast<const float4 *>(xsumf + b * (K / 16) + base / 16);
            float t = fmaf(a_lo, sl, -b_lo * (f4.x + f4.y));
            t = fmaf(a_hi, sh, fmaf(-b_hi, f4.z + f4.w, t));
            acc[b] += t;
        }
    }
}

// One Q6_K unit in the unit layout (gemv.cuh).  Lane -> block q6_blk(lane),
// 128-weight group g = (lane/2)%2 and 16 positions l0 = (lane%2)*16: 64
// weights, one scale per part.  Weight (g, part, l) is
// d * scale[g*8+part*2+l/16] * (q - 32), q assembled as in q6_value
// (inferencer.cu:473-487).
template <int B>
__device__ __forceinline__ void q6_unit(const uint8_t *unit, int nb_u, int u, int lane, const GemvParams &p,
                                        const SmemLayout &L, const uint8_t *smem, int use_dp4a, float (&acc)[B]) {
    const int blk = q6_blk(lane);
    if (blk >= nb_u) return;
    const int gblk0 = u * kUnitBlocks;
    const int g = (lane >> 1) & 1, l0 = (lane & 1) * 16;
    const uint8_t *body = unit + blk * 208;  // this lane's block; lane within the block = lane & 3
    const int j = lane & 3;
    const uint4 la = reinterpret_cast<const uint4 *>(body)[j];
    const uint4 lb = reinterpret_cast<const uint4 *>(body + 64)[j];
    const uint4 hh = reinterpret_cast<const uint4 *>(body + 128)[j];
    const uint32_t sc4 = reinterpret_cast<const uint32_t *>(body + 192)[j];
    const float d = half_bits_to_float(*reinterpret_cast<const uint16_t *>(unit + nb_u * 208 + blk * 2));
    int sc[4];
#pragma unroll
    for (int pt = 0; pt < 4; ++pt) sc[pt] = static_cast<int>(static_cast<int8_t>((sc4 >> (8 * pt)) & 255));
    const uint32_t A[4] = {la.x, la.y, la.z, la.w}, Bw[4] = {lb.x, lb.y, lb.z, lb.w};
    const uint32_t H[4] = {hh.x, hh.y, hh.z, hh.w};
    uint32_t q[4][4];  // [part][word], codes 0..63
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        q[0][j] = (A[j] & 0x0F0F0F0Fu) | ((H[j] << 4) & 0x30303030u);
        q[1][j] = (Bw[j] & 0x0F0F0F0Fu) | ((H[j] << 2) & 0x30303030u);
        q[2][j] = ((A[j] >> 4) & 0x0F0F0F0Fu) | (H[j] & 0x30303030u);
        q[3][j] = ((Bw[j] >> 4) & 0x0F0F0F0Fu) | ((H[j] >> 2) & 0x30303030u);
    }
    const int K = p.cols;
    const int base = (gblk0 + blk) * 256 + g * 128 + l0;  // position of part 0
    if (use_dp4a) {
        const int U = (K / 256 + kUnitBlocks - 1) / kUnitBlocks;
#pragma unroll
        for (int b = 0; b < B; ++b) {
            const int bu = b * U + u;
            const uint4 *xv4 = reinterpret_cast<const uint4 *>(smem + L.q6x) + bu * 128 + lane;
            const int4 s4 = reinterpret_cast<const int4 *>(smem + L.q6s)[bu * 32 + lane];
            const float4 f4 = reinterpret_cast<const float4 *>(smem + L.q6f)[bu * 32 + lane];
            const int sums[4] = {s4.x, s4.y, s4.z, s4.w};
            const float scl[4] = {f4.x, f4.y, f4.z, f4.w};
            float t = 0.f;
#pragma unroll
            for (int pt = 0; pt < 4; ++pt) {
                const uint4 xv = xv4[pt * 32];
                int dt = dp4a(q[pt][0], xv.x, 0);
                dt = dp4a(q[pt][1], xv.y, dt);
                dt = dp4a(q[pt][2], xv.z, dt);
                dt = dp4a(q[pt][3], xv.w, dt);
                dt -= 32 * sums[pt];  // codes carry a zero point of 32
                t = fmaf(static_cast<float>(sc[pt] * dt), scl[pt], t);
            }
            acc[b] = fmaf(d, t, acc[b]);
        }
    } else {
        const float *xf = reinterpret_cast<const float *>(smem + L.xf);
#pragma unroll
        for (int b = 0; b < B; ++b) {
            float t = 0.f;
#pragma unroll
            for (int pt = 0; pt < 4; ++pt) {
                const float *xv = xf + b * K + base + pt * 32;
                float s = 0.f;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float4 a = *reinterpret_cast<const float4 *>(xv + 4 * j);
                    // 0x4B0000qq - (2^23 + 32) = q - 32 exactly
                    s = fmaf(__int_as_float(__byte_perm(q[pt][j], 0x4B000000u, 0x7440)) - 8388640.0f, a.x, s);
                    s = fmaf(__int_as_float(__byte_perm(q[pt][j], 0x4B000000u, 0x7441)) - 8388640.0f, a.y, s);
                    s = fmaf(__int_as_float(__byte_perm(q[pt][j], 0x4B000000u, 0x7442)) - 8388640.0f, a.z, s);
                    s = fmaf(__int_as_float(__byte_perm(q[pt][j], 0x4B000000u, 0x7443)) - 8388640.0f, a.w, s);
                }
                t = fmaf(static_cast<float>(sc[pt]), s, t);
            }
            acc[b] = fmaf(d, t, acc[b]);
        }
    }
}

// ------------------------------------------------------------ work items --

// Position in a warp's stream of units: item -> row of the item -> unit.
struct Cursor {
    int item, r, u, seg;
};

__device__ __forceinline__ int seg_of_item(const GemvParams &p, int item) {
    int s = 0;
#pragma unroll
    for (int i = 1; i < kMaxSegs; ++i)
        if (i < p.nseg && item >= p.seg[i].item0) s = i;
    return s;
}

__device__ __forceinline__ void cursor_start(const GemvParams &p, int item, Cursor &c) {
    c.item = item;
    c.r = 0;
    c.u = 0;
    c.seg = item < p.total_items ? seg_of_item(p, item) : 0;
}

__device__ __forceinline__ void cursor_next(const GemvParams &p, int stride, int units_per_row, Cursor &c) {
    if (++c.u < units_per_row) return;
    c.u = 0;
    if (++c.r < p.seg[c.seg].item_rows) return;
    c.r = 0;
    c.item += stride;
    // items only grow, so the segment index only moves forward
    while (c.seg + 1 < p.nseg && c.item >= p.seg[c.seg + 1].item0) ++c.seg;
}

// Global address and byte count of the cursor's unit.
__device__ __forceinline__ const uint8_t *unit_src(const GemvParams &p, const Cursor &c, int nb, uint32_t &bytes) {
    const GemvSeg &s = p.seg[c.seg];
    const int li = c.item - s.item0;
    const uint8_t *base;
    int row;
    if (s.w1) {
        base = c.r ? s.w1 : s.w0;
        row = li;
    } else {
        base = s.w0;
        row = li * s.item_rows + c.r;
    }
    const int nb_u = min(kUnitBlocks, nb - c.u * kUnitBlocks);
    if (s.type == kQ4K) {
        bytes = static_cast<uint32_t>(nb_u) * kQ4Bytes;
        return base + static_cast<long>(row) * s.row_bytes + c.u * kUnitBlocks * kQ4Bytes;
    }
    bytes = static_cast<uint32_t>(q6_unit_bytes(nb_u));
    return base + static_cast<long>(row) * s.row_bytes + c.u * q6_unit_bytes(kUnitBlocks);
}

// A segment's fields that the main loop needs per unit, held in registers:
// what the prefetching cursor needs to address a unit ...
struct FetchSeg {
    const uint8_t *w0, *w1;
    long row_bytes;
    int item0, item_end, item_rows;
    uint32_t unit_bytes, last_bytes;
    __device__ __forceinline__ void load(const GemvParams &p, int si, int last_nb) {
        const GemvSeg &s = p.seg[si];
        w0 = s.w0;
        w1 = s.w1;
        row_bytes = s.row_bytes;
        item0 = s.item0;
        item_end = s.item0 + s.nitems;
        item_rows = s.item_rows;
        unit_bytes = static_cast<uint32_t>(s.type == kQ4K ? kUnitBlocks * kQ4Bytes : q6_unit_bytes(kUnitBlocks));
        last_bytes = static_cast<uint32_t>(s.type == kQ4K ? last_nb * kQ4Bytes : q6_unit_bytes(last_nb));
    }
    // Row r of item `item` (a pair's second row is the same row of w1, else the next row).
    __device__ __forceinline__ const uint8_t *row_ptr(int item, int r) const {
        const int li = item - item0;
        if (w1) return (r ? w1 : w0) + static_cast<long>(li) * row_bytes;
        return w0 + static_cast<long>(li * item_rows + r) * row_bytes;
    }
};
// ... and what the consuming cursor needs to compute and finish it.
struct UseSeg {
    int item0, item_end, item_rows, type, dp4a;
    __device__ __forceinline__ void load(const GemvParams &p, int si) {
        const GemvSeg &s = p.seg[si];
        item0 = s.item0;
        item_end = s.item0 + s.nitems;
        item_rows = s.item_rows;
        type = s.type;
        dp4a = s.dp4a;
    }
};

// ----------------------------------------------------------- epilogue --

// Writes one finished item (1 or 2 rows) for token b; y0/y1 are the rows' dots.
__device__ void epilogue(const GemvParams &p, const GemvSeg &s, int li, int b, float y0, float y1,
                         unsigned long long &best) {
    switch (s.epi) {
        case kEpiStore:
        case kEpiAdd: {
            const int row = li * s.item_rows;
            float *o = s.out + b * s.out_stride + s.row_offset + row;
            if (s.epi == kEpiAdd) {
                o[0] += y0;
                if (s.item_rows == 2) o[1] += y1;
            } else {
                o[0] = y0;
                if (s.item_rows == 2) o[1] = y1;
            }
            break;
        }
        case kEpiLogitsArgmax: {
            const int row = s.row_offset + li;
            s.out[b * s.out_stride + row] = y0;
            const unsigned long long k = argmax_key(y0, row);
            best = k > best ? k : best;
            break;
        }
        case kEpiSiluPair:
            // gate / (1 + exp(-gate)) * up (silu_cuda, inferencer.cu:1053-1056)
            s.out[b * s.out_stride + s.row_offset + li] = y0 / (1.f + __expf(-y0)) * y1;
            break;
        case kEpiRopeQ:
        case kEpiRopeKCache: {
            // pair (2j, 2j+1), frequency j % (head_dim/2) (rope_cuda :906-917)
            const int row = 2 * li, f = li % p.half_head;
            const int pos = p.tok_pos[b];
            const float c = p.rope_cos[pos * p.half_head + f], sn = p.rope_sin[pos * p.half_head + f];
            const float r0 = y0 * c - y1 * sn, r1 = y0 * sn + y1 * c;
            if (s.epi == kEpiRopeQ) {
                float *o = s.out + b * s.out_stride + s.row_offset + row;
                o[0] = r0;
                o[1] = r1;
            } else {
                const int slot = p.tok_slot[b];
                const int page = slot / p.page_size, t = slot % p.page_size;
                const int head = row / p.head_dim, dd = row % p.head_dim;
                const long off = static_cast<long>(page) * p.page_stride +
                                 (static_cast<long>(head) * p.page_size + t) * p.head_dim + dd;
                if (p.kv_f32)
                    *reinterpret_cast<float2 *>(static_cast<float *>(p.k_cache) + off) = make_float2(r0, r1);
                else
                    *reinterpret_cast<__half2 *>(static_cast<__half *>(p.k_cache) + off) = __floats2half2_rn(r0, r1);
            }
            break;
        }
        case kEpiVCache: {
            const int row = li * s.item_rows;
            const int slot = p.tok_slot[b];
            const int page = slot / p.page_size, t = slot % p.page_size;
            for (int r = 0; r < s.item_rows; ++r) {
                const int rr = row + r;
                const int head = rr / p.head_dim, dd = rr % p.head_dim;
                const long off = static_cast<long>(page) * p.page_stride +
                                 (static_cast<long>(head) * p.page_size + t) * p.head_dim + dd;
                const float v = r ? y1 : y0;
                if (p.kv_f32) static_cast<float *>(p.v_cache)[off] = v;
                else static_cast<__half *>(p.v_cache)[off] = __float2half_rn(v);
            }
            break;
        }
    }
}

// ----------------------------------------------------------------- kernel --

// kLean: the launch is one segment of single-row items whose epilogue is a
// store, a residual add or logits + argmax key (the lm_head, O and down
// projections, standalone GEMVs); its loop keeps the segment's constants in
// registers and steps its cursors without the general bookkeeping (item rows,
// segment changes, pair epilogues), which otherwise costs more instructions per
// unit than the dot products.
template <int B, bool kLean>
__global__ void __launch_bounds__(kThreads, (B == 1 ? 4 : 2)) ijb_gemv_kernel(const __grid_constant__ GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint32_t cta_abort;
    const SmemLayout L = smem_layout(p.cols, B, p.need_q4, p.need_q6, p.need_f);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bars) + warp * kDepth;
    uint8_t *ring = smem + L.ring + warp * kDepth * kSlotBytes;
    const int nb = p.cols / 256;
    const int upr = (nb + kUnitBlocks - 1) / kUnitBlocks;  // units per row
    const int gw = blockIdx.x * kWarps + warp, GW = gridDim.x * kWarps;

    // prefetch this warp's first units (weights only: no dependency on the
    // previous kernel, so this runs before griddepcontrol.wait)
    Cursor pf;
    cursor_start(p, gw, pf);
    if (threadIdx.x == 0) cta_abort = 0u;  // read only after the __syncthreads below
    if (lane == 0) {
        for (int s = 0; s < kDepth; ++s) mbar_init(bars + s, 1);
        fence_barrier_init();
    }
    for (int s = 0; s < kDepth && pf.item < p.total_items; ++s) {
        if (lane == 0) {
            uint32_t bytes;
            const uint8_t *src = unit_src(p, pf, nb, bytes);
            mbar_arrive_expect_tx(bars + s, bytes);
            bulk_g2s(ring + s * kSlotBytes, src, bytes, bars + s);
        }
        cursor_next(p, GW, upr, pf);
    }
    __syncwarp();
    pdl_trigger();
    pdl_wait();
    build_activation(p, L, smem);
    __syncthreads();

    if constexpr (kLean) {
        const GemvSeg &s0 = p.seg[0];
        const int type = s0.type, dp4a = s0.dp4a, epi = s0.epi, rows = p.total_items;
        const uint8_t *w0 = s0.w0;
        const long row_bytes = s0.row_bytes, out_stride = s0.out_stride;
        float *out = s0.out + s0.row_offset;
        const int unit_full = type == kQ4K ? kUnitBlocks * kQ4Bytes : q6_unit_bytes(kUnitBlocks);
        const int last_nb = nb - (upr - 1) * kUnitBlocks;
        const uint32_t last_bytes = static_cast<uint32_t>(type == kQ4K ? last_nb * kQ4Bytes : q6_unit_bytes(last_nb));
        int prow = pf.item, pu = pf.u;  // the next unit to fetch (the prologue fetched kDepth)
        float acc[B];
#pragma unroll
        for (int b = 0; b < B; ++b) acc[b] = 0.f;
        unsigned long long best = 0ull;  // lane b: best argmax key of token b
        int slot = 0, u = 0;
        uint32_t phase = 0;
        for (int row = gw; row < rows;) {
            mbar_wait_bounded(bars + slot, phase, p.status, &cta_abort);
            const uint8_t *unit = ring + slot * kSlotBytes;
            const int nb_u = u == upr - 1 ? last_nb : kUnitBlocks;
            if (type == kQ4K)
                q4_unit<B>(unit, nb_u, u, lane, p, L, smem, dp4a, acc);
            else
                q6_unit<B>(unit, nb_u, u, lane, p, L, smem, dp4a, acc);
            __syncwarp();
            if (prow < rows) {  // refill this slot with the unit kDepth ahead
                if (lane == 0) {
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    const uint32_t bytes = pu == upr - 1 ? last_bytes : static_cast<uint32_t>(unit_full);
                    mbar_arrive_expect_tx(bars + slot, bytes);
                    bulk_g2s(ring + slot * kSlotBytes, w0 + prow * row_bytes + static_cast<long>(pu) * unit_full, bytes,
                             bars + slot);
                }
                if (++pu == upr) {
                    pu = 0;
                    prow += GW;
                }
            }
            if (++u == upr) {  // last unit of the row: reduce and write it
#pragma unroll
                for (int b = 0; b < B; ++b) {
                    const float y = warp_sum(acc[b]);
                    acc[b] = 0.f;
                    if (lane == b && b < p.batch) {
                        float *o = out + b * out_stride + row;
                        if (epi == kEpiAdd) {
                            *o += y;
                        } else {
                            *o = y;
                            if (epi == kEpiLogitsArgmax) {
                                const unsigned long long key = argmax_key(y, s0.row_offset + row);
                                best = key > best ? key : best;
                            }
                        }
                    }
                }
                u = 0;
                row += GW;
            }
            if (++slot == kDepth) {
                slot = 0;
                phase ^= 1u;
            }
        }
        if (best && p.argmax_keys && lane < p.batch) atomicMax(p.argmax_keys + lane, best);
        return;
    }

    // General loop: several segments, two-row items (RoPE pairs, gate/up
    // pairs).  Each cursor keeps its segment's fields in registers and reloads
    // them only when it crosses into the next segment.
    const int last_nb = nb - (upr - 1) * kUnitBlocks;
    UseSeg cs;    // the consuming cursor's segment
    FetchSeg ps;  // the prefetching cursor's segment
    int cseg = seg_of_item(p, gw), item = gw, r = 0, u = 0;
    cs.load(p, cseg);
    int pseg = pf.seg, pitem = pf.item, pr = pf.r, pu = pf.u;
    ps.load(p, pseg, last_nb);
    float acc[B];
    float res0[B];
#pragma unroll
    for (int b = 0; b < B; ++b) acc[b] = res0[b] = 0.f;
    unsigned long long best = 0ull;  // lane b: best argmax key of token b
    const int total = p.total_items;
    int slot = 0;
    uint32_t phase = 0;
    while (item < total) {
        mbar_wait_bounded(bars + slot, phase, p.status, &cta_abort);
        const int nb_u = u == upr - 1 ? last_nb : kUnitBlocks;
        const uint8_t *unit = ring + slot * kSlotBytes;
        if (cs.type == kQ4K)
            q4_unit<B>(unit, nb_u, u, lane, p, L, smem, cs.dp4a, acc);
        else
            q6_unit<B>(unit, nb_u, u, lane, p, L, smem, cs.dp4a, acc);
        __syncwarp();
        // refill this slot with the unit kDepth ahead
        if (pitem < total) {
            if (lane == 0) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                const uint32_t bytes = pu == upr - 1 ? ps.last_bytes : ps.unit_bytes;
                const uint8_t *src = ps.row_ptr(pitem, pr) + static_cast<long>(pu) * ps.unit_bytes;
                mbar_arrive_expect_tx(bars + slot, bytes);
                bulk_g2s(ring + slot * kSlotBytes, src, bytes, bars + slot);
            }
            if (++pu == upr) {
                pu = 0;
                if (++pr == ps.item_rows) {
                    pr = 0;
                    pitem += GW;
                    if (pitem >= ps.item_end && pitem < total) {  // items only grow
                        while (pseg + 1 < p.nseg && pitem >= p.seg[pseg + 1].item0) ++pseg;
                        ps.load(p, pseg, last_nb);
                    }
                }
            }
        }
        if (++u == upr) {  // last unit of a row: reduce it
            u = 0;
            float y[B];
#pragma unroll
            for (int b = 0; b < B; ++b) {
                y[b] = warp_sum(acc[b]);
                acc[b] = 0.f;
            }
            if (r + 1 < cs.item_rows) {
#pragma unroll
                for (int b = 0; b < B; ++b) res0[b] = y[b];
                ++r;
            } else {
                const GemvSeg &sg = p.seg[cseg];
                const int li = item - cs.item0;
#pragma unroll
                for (int b = 0; b < B; ++b)
                    if (lane == b && b < p.batch) {
                        if (cs.item_rows == 2) epilogue(p, sg, li, b, res0[b], y[b], best);
                        else epilogue(p, sg, li, b, y[b], 0.f, best);
                    }
                r = 0;
                item += GW;
                if (item >= cs.item_end && item < total) {
                    while (cseg + 1 < p.nseg && item >= p.seg[cseg + 1].item0) ++cseg;
                    cs.load(p, cseg);
                }
            }
        }
        if (++slot == kDepth) {
            slot = 0;
            phase ^= 1u;
        }
    }
    if (best && p.argmax_keys && lane < p.batch) atomicMax(p.argmax_keys + lane, best);
}

// ------------------------------------------------------------------- host --

static int g_dyn_limit[64] = {0};

// Opt every kernel instance in to the largest dynamic shared memory the
// device allows next to its static shared memory, once per device (kept out
// of the launch path so launches can be captured into graphs).
static cudaError_t prepare_attributes() {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (g_dyn_limit[dev]) return cudaSuccess;
    int optin = 0;
    e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return e;
    const void *fns[8] = {(const void *)ijb_gemv_kernel<1, false>, (const void *)ijb_gemv_kernel<2, false>,
                          (const void *)ijb_gemv_kernel<4, false>, (const void *)ijb_gemv_kernel<8, false>,
                          (const void *)ijb_gemv_kernel<1, true>,  (const void *)ijb_gemv_kernel<2, true>,
                          (const void *)ijb_gemv_kernel<4, true>,  (const void *)ijb_gemv_kernel<8, true>};
    int limit = optin;
    for (int i = 0; i < 8; ++i) {
        cudaFuncAttributes fa;
        e = cudaFuncGetAttributes(&fa, fns[i]);
        if (e != cudaSuccess) return e;
        const int lim = optin - static_cast<int>(fa.sharedSizeBytes);
        limit = lim < limit ? lim : limit;
    }
    limit &= ~127;
    for (int i = 0; i < 8; ++i) {
        e = cudaFuncSetAttribute(fns[i], cudaFuncAttributeMaxDynamicSharedMemorySize, limit);
        if (e != cudaSuccess) return e;
    }
    g_dyn_limit[dev] = limit;
    return cudaSuccess;
}

cudaError_t gemv_prepare() { return prepare_attributes(); }

// The lean loop's conditions (see ijb_gemv_kernel).
static bool lean_launch(const GemvParams &p) {
    const GemvSeg &s = p.seg[0];
    return p.nseg == 1 && s.item0 == 0 && s.item_rows == 1 && s.w1 == nullptr &&
           (s.epi == kEpiStore || s.epi == kEpiAdd || s.epi == kEpiLogitsArgmax);
}

template <int B>
static cudaError_t launch_b(const GemvParams &p, int grid, int smem, cudaStream_t stream, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (lean_launch(p)) return cudaLaunchKernelEx(&cfg, ijb_gemv_kernel<B, true>, p);
    return cudaLaunchKernelEx(&cfg, ijb_gemv_kernel<B, false>, p);
}

// Tokens the kernel instance is compiled for: the smallest of 1, 2, 4, 8
// that holds `batch` (extra slots are computed and never stored).
static int batch_instance(int batch) { return batch <= 1 ? 1 : batch <= 2 ? 2 : batch <= 4 ? 4 : 8; }

static cudaError_t launch_group(const GemvParams &p, int num_sms, cudaStream_t stream, bool pdl) {
    const int inst = batch_instance(p.batch);
    const int smem = smem_layout(p.cols, inst, p.need_q4, p.need_q6, p.need_f).total;
    if (p.total_items < 1) return cudaSuccess;
    switch (inst) {
        case 1: {
            // two CTAs per SM leave room for the next kernel's CTAs; a long
            // stream (>= 32 units per warp at two per SM, e.g. the lm_head) runs
            // four, whose extra copies in flight lift it from ~0.61 to ~0.70 of
            // HBM bandwidth on B200 (short ones lose to the extra prologues)
            const long units = static_cast<long>(p.total_items) * p.seg[0].item_rows * ((p.cols / 256 + kUnitBlocks - 1) / kUnitBlocks);
            const int per_sm = units >= 32L * 2 * num_sms * kWarps ? 4 : 2;
            return launch_b<1>(p, per_sm * num_sms, smem, stream, pdl);
        }
        // 2-8 tokens: two CTAs per SM, as many as their registers allow (one per SM
        // measured 1.45x slower on the Q6_K lm_head at 8 tokens: 260 against 181 us)
        case 2: return launch_b<2>(p, 2 * num_sms, smem, stream, pdl);
        case 4: return launch_b<4>(p, 2 * num_sms, smem, stream, pdl);
        default: return launch_b<8>(p, 2 * num_sms, smem, stream, pdl);
    }
}

// Largest token count (1, 2, 4 or 8) whose activations fit in shared memory.
int gemv_max_batch(int cols, int need_q4, int need_q6, int need_f) {
    int dev = 0;
    if (prepare_attributes() != cudaSuccess || cudaGetDevice(&dev) != cudaSuccess) return 0;
    for (int b = kMaxBatch; b >= 1; b /= 2)
        if (smem_layout(cols, b, need_q4, need_q6, need_f).total <= g_dyn_limit[dev]) return b;
    return 0;
}

// Launches the GEMV, in several token groups when the batch's activations do
// not fit one CTA's shared memory (every per-token pointer is offset).
cudaError_t gemv_launch(const GemvParams &p, int num_sms, cudaStream_t stream, bool pdl) {
    if (p.batch < 1 || p.batch > kMaxBatch || p.cols % 256 || p.cols > kMaxCols) return cudaErrorInvalidValue;
    cudaError_t e = prepare_attributes();
    if (e != cudaSuccess) return e;
    const int group = gemv_max_batch(p.cols, p.need_q4, p.need_q6, p.need_f);
    if (group < 1) return cudaErrorInvalidValue;
    for (int g0 = 0; g0 < p.batch; g0 += group) {
        GemvParams q = p;
        q.batch = p.batch - g0 < group ? p.batch - g0 : group;
        q.x = p.x + g0 * p.x_stride;
        for (int s = 0; s < p.nseg; ++s)
            if (q.seg[s].out) q.seg[s].out = p.seg[s].out + g0 * p.seg[s].out_stride;
        if (p.tok_pos) q.tok_pos = p.tok_pos + g0;
        if (p.tok_slot) q.tok_slot = p.tok_slot + g0;
        if (p.argmax_keys) q.argmax_keys = p.argmax_keys + g0;
        e = launch_group(q, num_sms, stream, pdl);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace ijb
