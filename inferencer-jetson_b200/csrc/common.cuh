// Shared device helpers for the sm_100a kernels: mbarrier + 1-D bulk copies
// (cp.async.bulk, the TMA engine's untiled form), programmatic dependent
// launch, bounded waits, and the GGUF block constants.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ijb {

constexpr int kQ4K = 12;
constexpr int kQ6K = 14;
constexpr int kQ4Bytes = 144;  // GGUF Q4_K super-block (inferencer.cu:258)
constexpr int kQ6Bytes = 210;  // GGUF Q6_K super-block

// Error codes a kernel can leave in the engine's device status word.
constexpr uint32_t kDevErrWaitTimeout = 1u;  // a bounded mbarrier/flag wait expired
constexpr uint32_t kDevErrBadIndex = 2u;     // an index failed its bounds check

// Wall-clock limit for any device-side wait (nanoseconds, %globaltimer).
// Every wait of the library's kernels uses it; ijb_probe_wait_timeout passes
// a shorter one to exercise the failure path.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Tests the phase; if it is not complete the thread is suspended until it
// completes or the hint (in ns) elapses, so waiting warps do not spin.
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
        : "memory");
    return ok != 0;
}

// Slow path of mbar_wait_bounded, kept out of line so that the many wait
// sites of a kernel stay small in the instruction cache.
static __device__ __noinline__ bool mbar_wait_slow(uint64_t *bar, uint32_t parity, uint32_t *status,
                                                   volatile uint32_t *cta_abort, uint64_t limit_ns) {
    if (*cta_abort) return false;
    uint64_t start = 0;
    for (uint32_t n = 1;; ++n) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((n & 15u) == 0) {
            if (*cta_abort) return false;
            const uint64_t now = global_timer_ns();
            if (start == 0) {
                start = now;
            } else if (now - start > limit_ns) {
                *cta_abort = 1u;
                if (status) atomicOr(status, kDevErrWaitTimeout);
                return false;
            }
        }
    }
}

// Waits for the barrier phase with the given parity.  Gives up after
// limit_ns (kWaitLimitNs unless given): records kDevErrWaitTimeout in the launch's device status word
// and raises `cta_abort` (a flag in the CTA's shared memory, zeroed at kernel
// start), after which every later wait of the CTA returns at once, so a CTA
// that lost one wait ends within one time limit.  Each poll suspends the
// thread for up to 1 ms; the clock and the flag are read every 16 polls.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, uint32_t *status,
                                                  volatile uint32_t *cta_abort, uint64_t limit_ns = kWaitLimitNs) {
    if (mbar_try_wait(bar, parity)) return true;
    return mbar_wait_slow(bar, parity, status, cta_abort, limit_ns);
}

// 1-D bulk copy global -> shared, completing on `bar` (transaction bytes).
// dst, src and bytes must all be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Same, with an L2 evict-first hint: streamed weights are read once per step.
__device__ __forceinline__ void bulk_g2s_evict_first(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                                     uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
        "%4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Programmatic dependent launch (the kernel is launched with
// cudaLaunchAttributeProgrammaticStreamSerialization).  `pdl_wait` blocks
// until every prerequisite grid has completed and its writes are visible;
// `pdl_trigger` lets the next kernel in the stream be scheduled early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float half_bits_to_float(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// Exact int -> float for small non-negative byte values: 0x4B0000xx is the
// float 2^23 + xx, so subtracting 2^23 gives xx with no rounding.
__device__ __forceinline__ float byte_to_float(uint32_t word, uint32_t selector) {
    return __int_as_float(__byte_perm(word, 0x4B000000u, selector)) - 8388608.0f;
}

// Key for the reference's argmax tournament (argmax_blocks_cuda +
// argmax_final_cuda, inferencer.cu:1063-1099): a left-biased 256-wide tree per
// block, then a 512-wide tree over blocks.  Among equal maxima it keeps the
// index whose block number, then in-block position, is smallest in
// bit-reversed order.  Packing (value, that rank) into 64 bits makes the
// winner the unsigned maximum key, so atomicMax reproduces the tournament.
__device__ __forceinline__ unsigned long long argmax_key(float v, int index) {
    if (v == 0.0f) v = 0.0f;  // -0 and +0 compare equal in the reference's `>`
    uint32_t b = __float_as_uint(v);
    uint32_t ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    if (v != v) ord = 0u;  // NaN never wins
    uint32_t blk = static_cast<uint32_t>(index) >> 8, pos = static_cast<uint32_t>(index) & 255u;
    uint32_t rank = ((__brev(blk) >> 23) << 8) | (__brev(pos) >> 24);
    return (static_cast<unsigned long long>(ord) << 32) | (0xFFFFFFFFu - rank);
}

__device__ __forceinline__ int argmax_key_index(unsigned long long key) {
    uint32_t rank = 0xFFFFFFFFu - static_cast<uint32_t>(key & 0xFFFFFFFFull);
    uint32_t blk = __brev(rank >> 8) >> 23, pos = __brev(rank & 255u) >> 24;
    return static_cast<int>((blk << 8) | pos);
}

}  // namespace ijb
