// Shared device helpers for libatlas_cuda (sm_100a only).
//
// PTX wrappers for the Blackwell async machinery the kernels use: mbarriers,
// 1-D bulk copies (TMA, cp.async.bulk) global -> shared, acquire/release
// counters for cross-CTA phase ordering. Every spin-wait here is bounded: it
// gives up after kWaitLimitNs of wall-clock time, records a status code in the
// caller's error word and returns false, so a stuck dependency ends the kernel
// with an error the host reads back instead of hanging the device.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "libatlas_cuda is built for sm_100a only"
#endif

namespace atlas {

// Device status codes written to the error word (host maps them to ATLAS_E*).
enum : uint32_t {
    kStatusOk = 0,
    kStatusBarrierTimeout = 1,   // grid phase barrier never completed
    kStatusStageTimeout = 2,     // an mbarrier (bulk-copy stage) never completed
    kStatusBadArgument = 3,      // device-side argument check failed
    kStatusCombineTimeout = 4,   // attention split combine never saw all splits
    kStatusPeerTimeout = 5,      // a tensor-parallel peer's arrivals never came
};

// Wall-clock bound of one wait (globaltimer, ns): far above any legitimate
// wait (a whole decode step is < 1 ms) and far below a hang.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint64_t global_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void *p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier --

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;"
                 ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

// Raise the transaction count of the current phase by `bytes` (no arrival).
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes)
{
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n"
        " mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Non-blocking test of phase `parity` of `bar`.
__device__ __forceinline__ bool mbar_test(uint64_t *bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n"
        " mbarrier.test_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for phase `parity` of `bar`. Returns false (and sets *err) when
// kWaitLimitNs passes, or early if another thread already recorded an error.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile uint32_t *err,
                                          uint32_t code = kStatusStageTimeout)
{
    uint64_t t0 = 0;
    for (uint32_t i = 0;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 31u) == 31u) {
            if (*err != kStatusOk) return false;
            const uint64_t now = global_ns();
            if (!t0) t0 = now;
            else if (now - t0 > kWaitLimitNs) break;
        }
    }
    atomicCAS(const_cast<uint32_t *>(err), kStatusOk, code);
    return false;
}

// ------------------------------------------------------------ bulk copies --

// 1-D bulk copy global -> this CTA's shared memory, completing on `bar`.
// Requires 16-byte aligned src/dst and a size that is a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// Same, with an L2 eviction-priority hint (weights are streamed once per step).
__device__ __forceinline__ void bulk_g2s_hint(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                              uint64_t policy)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
        ::"r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first()
{
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// ------------------------------------------------- cross-CTA ordering ------

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t *p)
{
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_release_add(uint32_t *p, uint32_t v)
{
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t atom_acq_rel_add(uint32_t *p, uint32_t v)
{
    uint32_t old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// System scope (another GPU writes the counter over NVLink).
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p)
{
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_release_sys_add(uint32_t *p, uint32_t v)
{
    asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded wait until *ctr >= target (mod 2^32), acquire at system scope.
__device__ __forceinline__ bool wait_counter_sys(const uint32_t *ctr, uint32_t target, volatile uint32_t *err)
{
    uint64_t t0 = 0;
    for (uint32_t i = 0;; ++i) {
        if ((int32_t)(ld_acquire_sys(ctr) - target) >= 0) return true;
        if (*err != kStatusOk) return false;
        if (i > 32) {
            __nanosleep(32);
            const uint64_t now = global_ns();
            if (!t0) t0 = now;
            else if (now - t0 > kWaitLimitNs) break;
        }
    }
    atomicCAS(const_cast<uint32_t *>(err), kStatusOk, kStatusPeerTimeout);
    return false;
}

// Bounded wait until *ctr >= target (acquire). False on timeout / prior error.
__device__ __forceinline__ bool wait_counter(const uint32_t *ctr, uint32_t target, volatile uint32_t *err,
                                             uint32_t code)
{
    uint64_t t0 = 0;
    for (uint32_t i = 0;; ++i) {
        if ((int32_t)(ld_acquire(ctr) - target) >= 0) return true;
        if (*err != kStatusOk) return false;
        if (i > 32) {
            __nanosleep(32);
            const uint64_t now = global_ns();
            if (!t0) t0 = now;
            else if (now - t0 > kWaitLimitNs) break;
        }
    }
    atomicCAS(const_cast<uint32_t *>(err), kStatusOk, code);
    return false;
}

// ------------------------------------------------------------ numerics -----

// Exact binary16 -> binary32 (the hardware conversion is exact for every
// finite value and keeps NaN payloads in the high mantissa bits).
__device__ __forceinline__ float h2f(uint16_t bits)
{
    return __half2float(__ushort_as_half(bits));
}

// Small integers to float without the conversion unit: 2^23 + v read as a
// float is exact for v < 2^23, and subtracting 2^23 leaves v exactly.
__device__ __forceinline__ float u2f_small(uint32_t v) { return __uint_as_float(0x4B000000u | v) - 8388608.0f; }
// The int8 in the low byte of `byte`: offset to 0..255 by flipping the sign bit.
__device__ __forceinline__ float s8f(uint32_t byte)
{
    return __uint_as_float(0x4B000000u | ((byte ^ 0x80u) & 0xffu)) - 8388736.0f;
}

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace atlas
