// Batched prefill kernels (sm_100a): the dense contraction on tcgen05 tensor
// cores with Q4_K / Q6_K weights dequantized into shared memory, the
// activation split/tiling pass that feeds it, the embedding gather and the
// causal GQA attention over the KV cache.
//
// Contraction kernel: clusters of two CTAs (one per SM) drive the 2-SM MMA
// (tcgen05.mma.cta_group::2, M = 256 tokens, N = 256 weight rows, K = 16).
// Each SM of a pair holds 128 of the tokens and 128 of the weight rows of
// every operand tile, and a 128-token x 256-row fp32 accumulator in tensor
// memory. A pair is persistent over work units (row tile, 256-token tile,
// K range). Per CTA:
//   warp 0      bulk-copies the pre-split activation tile of each 64-wide
//               K block (hi + lo binary16, already in the 128-byte swizzled
//               K-major layout) into the 3-stage ring;
//   warps 6-21  dequantize this CTA's 128 weight rows x 64 K values straight
//               from the raw super-blocks in global memory (bit-exact with
//               src/brain_runtime.c:960-1083; two groups of 8 warps take
//               alternate stages, two threads per row, a group's next
//               stage's bytes loaded while the current one converts),
//               scale them by 2^wexp, split them into binary16 hi/lo and
//               store them swizzled next to the activations;
//   warp 1      allocates 512 TMEM columns (two accumulators). In the even
//               CTA one thread issues the MMAs of every product term once
//               both SMs' stages are full, and multicasts the stage release
//               and the finished accumulator to both CTAs; in the odd CTA it
//               waits for its own activation copy and dequant warps and
//               relays one arrival per stage to the even CTA;
//   warps 2-5   read this CTA's accumulator with tcgen05.ld (lane = token),
//               undo the power-of-two scales and apply the fused epilogue:
//               bias, RoPE and the KV-cache store for Q/K/V, residual add
//               for O / down, SwiGLU for gate+up (a tile's 256 rows are 128
//               gate rows - dequantized by the even CTA - and the same 128 up
//               rows - by the odd one - so every accumulator row holds both).
//               With split-K each unit stores its partial tile and the last
//               unit of a tile to arrive sums the partials in K order.
// Every wait is bounded (2 s of globaltimer); on a timeout the CTA records a
// status, drains its outstanding copies and MMAs, and both CTAs of the pair
// meet at a final cluster barrier before freeing TMEM and exiting.
#include <cfloat>
#include <cmath>
#include "common.cuh"
#include "quant.cuh"
#include "prefill.h"

namespace atlas {
namespace pf {

// ------------------------------------------------ cluster / tcgen05 PTX ----

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ uint32_t cluster_rank()
{
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// All threads of both CTAs of the pair.
__device__ __forceinline__ void cluster_sync()
{
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Arrive on the barrier at the same shared-memory offset in CTA `cta` of the cluster.
__device__ __forceinline__ void mbar_arrive_cta(uint64_t *bar, uint32_t cta)
{
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_addr(bar)), "r"(cta));
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t *bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n"
        " mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait with cluster-scope acquire (arrivals come from both CTAs).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t *bar, uint32_t parity, volatile uint32_t *err)
{
    uint64_t t0 = 0;
    for (uint32_t i = 0;; ++i) {
        if (mbar_try_wait_cluster(bar, parity)) return true;
        if ((i & 31u) == 31u) {
            if (*err != kStatusOk) return false;
            const uint64_t now = global_ns();
            if (!t0) t0 = now;
            else if (now - t0 > kWaitLimitNs) break;
        }
    }
    atomicCAS(const_cast<uint32_t *>(err), kStatusOk, (uint32_t)kStatusStageTimeout);
    return false;
}

// Teardown wait: bounded, ignores the error word (lets in-flight copies and
// MMAs finish before the CTA frees its resources).
__device__ __forceinline__ bool mbar_drain(uint64_t *bar, uint32_t parity)
{
    const uint64_t t0 = global_ns();
    while (!mbar_try_wait_cluster(bar, parity))
        if (global_ns() - t0 > kWaitLimitNs) return false;
    return true;
}

// Warp-uniform bounded wait: every lane polls, the warp agrees on the outcome.
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity, volatile uint32_t *err)
{
    const bool ok = mbar_wait_cluster(bar, parity, err);
    return __all_sync(0xffffffffu, ok);
}

// Prefetch [p, p + bytes) into L2 (16-byte aligned address, size a multiple of 16).
__device__ __forceinline__ void prefetch_l2(const void *p, uint32_t bytes)
{
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// 2-SM tensor memory: the same warp of both CTAs allocates / frees.
__device__ __forceinline__ void tmem_alloc2(uint32_t *slot, uint32_t ncols)
{
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)), "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc2(uint32_t taddr, uint32_t ncols)
{
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[tmem] (+)= A[smem] . B[smem]^T over the CTA pair, both operands K-major binary16.
__device__ __forceinline__ void umma2_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accum)
{
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n"
        ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum)
        : "memory");
}

// Arrive on `bar` in both CTAs of the pair once every MMA this thread issued is done.
__device__ __forceinline__ void umma2_commit_both(uint64_t *bar)
{
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
                 ::"r"(smem_addr(bar)), "h"((uint16_t)3u)
                 : "memory");
}

__device__ __forceinline__ void umma2_commit(uint64_t *bar)
{
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8])
{
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory operand descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (stride byte offset), leading byte offset 16 (unused by
// this layout), descriptor version 1, base offset 0 (1024-byte aligned tiles).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr)
{
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)(1024u >> 4) << 32) |
           ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}

// Instruction descriptor: fp32 accumulator, A = B = binary16, both K-major,
// N = 256, M = 256 (the pair).
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(kRowTile >> 3) << 17) | ((uint32_t)(kPairTokens >> 4) << 24);

// Byte offset of 16-byte chunk `chunk` (K elements 8*chunk..8*chunk+7) of
// operand row `row` in a 128-byte-swizzled K-major tile.
__host__ __device__ constexpr uint32_t sw128_off(uint32_t row, uint32_t chunk)
{
    return (row >> 3) * 1024u + (row & 7u) * 128u + ((chunk ^ (row & 7u)) << 4);
}

// --------------------------------------------------------- shared layout --

struct Bars {
    uint64_t xfull[kStages];   // this CTA's activation copy landed (tx count)
    uint64_t full[kStages];    // even CTA: its dequant group (8 warps) + the odd CTA's relay
    uint64_t wfull[kStages];   // odd CTA: its dequant group (8 warps), relayed to the even CTA
    uint64_t empty[kStages];   // both: the MMAs reading the stage completed
    uint64_t acc_full[2];      // both: accumulator complete
    uint64_t acc_empty[2];     // even CTA: the pair's 8 epilogue warps are done reading
    uint64_t fin;              // even CTA: teardown, all MMAs completed
    uint32_t tmem;
    uint32_t status;
};

constexpr size_t kGemmSmem = (size_t)kStages * kStageBytes + 1024 + sizeof(Bars);

struct Unit {
    uint32_t tile, tt, ks, kb0, kb1;   // tt: 256-token tile
};

__device__ __forceinline__ Unit unit_of(const GemmArgs &a, uint32_t u)
{
    Unit x;
    x.ks = u % a.ksplit;
    const uint32_t r = u / a.ksplit;
    x.tt = r % a.tok_pairs;
    x.tile = r / a.tok_pairs;
    x.kb0 = (uint32_t)((uint64_t)a.kblocks * x.ks / a.ksplit);
    x.kb1 = (uint32_t)((uint64_t)a.kblocks * (x.ks + 1) / a.ksplit);
    return x;
}

__device__ __forceinline__ uint32_t seg_of_tile(const GemmArgs &a, uint32_t tile)
{
    uint32_t s = 0;
    while (s + 1 < a.n_seg && tile >= a.seg[s + 1].tile0) ++s;
    return s;
}

// -------------------------------------------------------------- dequant ----

// Float 2^23 + b for a byte b of v (k = byte index): exact small-integer
// conversion without I2F.
__device__ __forceinline__ float byte_f23(uint32_t v, int k)
{
    return __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7440u | (uint32_t)k));
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b)
{
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// Store 8 scaled weights as binary16 hi (and lo) at a swizzled chunk. With
// the lo term, hi is w with its 13 low mantissa bits cleared (exact in
// binary16 within the scaled range) and lo = w - hi rounded to binary16, so
// hi + lo keeps 21+ significant bits without converting hi back to fp32.
template <int TERMS>
__device__ __forceinline__ void store_chunk(uint8_t *bhi, uint32_t off, const float (&w)[8])
{
    if (TERMS >= 3) {
        float hm[8], lo[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            hm[i] = __uint_as_float(__float_as_uint(w[i]) & 0xffffe000u);
            lo[i] = w[i] - hm[i];
        }
        *reinterpret_cast<uint4 *>(bhi + off) =
            make_uint4(pack_h2(hm[0], hm[1]), pack_h2(hm[2], hm[3]), pack_h2(hm[4], hm[5]), pack_h2(hm[6], hm[7]));
        *reinterpret_cast<uint4 *>(bhi + kBTermBytes + off) =
            make_uint4(pack_h2(lo[0], lo[1]), pack_h2(lo[2], lo[3]), pack_h2(lo[4], lo[5]), pack_h2(lo[6], lo[7]));
    } else {
        *reinterpret_cast<uint4 *>(bhi + off) =
            make_uint4(pack_h2(w[0], w[1]), pack_h2(w[2], w[3]), pack_h2(w[4], w[5]), pack_h2(w[6], w[7]));
    }
}

// Raw bytes one dequant thread needs for its half (32 values) of one 64-value
// K block of one row.
struct Raw {
    uint32_t w[20];
    uint32_t sh;   // Q6_K: funnel shift (0 or 16) of the 4-byte aligned words
};

// Half `hf` (values 32hf..32hf+31) of 64-value chunk kq of super-block `blk`.
__device__ __forceinline__ void load_raw(uint32_t type, const uint8_t *blk, uint32_t kq, uint32_t hf, Raw &r)
{
    if (type == 12u) {
        // header (d, dmin, 12 scale bytes) + the chunk's 32 quant bytes (low
        // nibbles: first half, high nibbles: second); 16-byte aligned
        const uint4 h = __ldg(reinterpret_cast<const uint4 *>(blk));
        const uint4 q0 = __ldg(reinterpret_cast<const uint4 *>(blk + 16 + 32 * kq));
        const uint4 q1 = __ldg(reinterpret_cast<const uint4 *>(blk + 32 + 32 * kq));
        r.w[0] = h.x; r.w[1] = h.y; r.w[2] = h.z; r.w[3] = h.w;
        r.w[4] = q0.x; r.w[5] = q0.y; r.w[6] = q0.z; r.w[7] = q0.w;
        r.w[8] = q1.x; r.w[9] = q1.y; r.w[10] = q1.z; r.w[11] = q1.w;
    } else {
        // Q6_K (2-byte aligned blocks), values 128n + 32j + l with n = kq / 2,
        // j = 2(kq & 1) + hf: ql[64n + 32hf + l], qh[32n + l], scales
        // [8n + 2j, 8n + 2j + 1] (l / 16 picks one), d
        const uint32_t n = kq >> 1;
        const uintptr_t b = reinterpret_cast<uintptr_t>(blk);
        r.sh = (uint32_t)(b & 2u) * 8u;
        const uint32_t *ql = reinterpret_cast<const uint32_t *>((b + 64 * n + 32 * hf) & ~(uintptr_t)3);
        const uint32_t *qh = reinterpret_cast<const uint32_t *>((b + 128 + 32 * n) & ~(uintptr_t)3);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            r.w[i] = __ldg(ql + i);
            r.w[9 + i] = __ldg(qh + i);
        }
        r.w[8] = r.sh ? __ldg(ql + 8) : 0u;
        r.w[17] = r.sh ? __ldg(qh + 8) : 0u;
        const uint32_t j = 2u * (kq & 1u) + hf;
        const unsigned short *sc = reinterpret_cast<const unsigned short *>(blk + 192 + 8 * n + 2 * j);
        r.w[18] = (uint32_t)__ldg(sc);
        r.w[19] = (uint32_t)__ldg(reinterpret_cast<const unsigned short *>(blk + 208));
    }
}

// Dequantize the 32 values held in `r` (half hf of chunk kq), scaled by
// p2 = 2^wexp, into swizzled chunks 4hf..4hf+3 of tile row `row`.
template <int TERMS>
__device__ __forceinline__ void dequant_half(uint32_t type, const Raw &r, uint32_t kq, uint32_t hf, float p2,
                                             uint8_t *bhi, uint32_t row)
{
    const uint32_t rbase = (row >> 3) * 1024u + (row & 7u) * 128u, r7 = row & 7u;
    if (type == 12u) {
        // src/brain_runtime.c:960-1015: y = (d*sc) * q - dmin*m per 32-value
        // sub-block j = 2kq + hf; get_scale_min_k4 (:939-958) on the header
        // words: bytes 4-7 (scales 0-3), 8-11 (4-7), 12-15 (8-11)
        const float d = h2f((uint16_t)(r.w[0] & 0xffffu)), dmin = h2f((uint16_t)(r.w[0] >> 16));
        const uint32_t j = 2u * kq + hf, t = (j & 3u) * 8u;
        const uint32_t y = (r.w[1] >> t) & 255u, z = (r.w[2] >> t) & 255u, x = (r.w[3] >> t) & 255u;
        const bool low = j < 4u;
        const uint32_t sc = low ? (y & 63u) : ((x & 15u) | ((y >> 6) << 4));
        const uint32_t mn = low ? (z & 63u) : ((x >> 4) | ((z >> 6) << 4));
        const float a = __fmul_rn(__fmul_rn(d, (float)sc), p2);   // exact: 2^wexp scaling
        const float bm = __fmul_rn(__fmul_rn(dmin, (float)mn), p2);
        const uint32_t sh = 4u * hf;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            float w[8];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint32_t v = (r.w[4 + 2 * c + h] >> sh) & 0x0f0f0f0fu;
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float q = byte_f23(v, k) - 8388608.0f;
                    w[4 * h + k] = fmaf(a, q, -bm);   // == fl(fl(a*q) - b): a*q is exact
                }
            }
            store_chunk<TERMS>(bhi, rbase + (((4u * hf + (uint32_t)c) ^ r7) << 4), w);
        }
    } else {
        // src/brain_runtime.c:1049-1083: y = (d * sc) * (q - 32)
        const float d = h2f((uint16_t)r.w[19]);
        const uint32_t s4 = 4u * (kq & 1u), s2 = s4 + 2u * hf;
        const float ds0 = __fmul_rn(__fmul_rn(d, (float)(int)(int8_t)(r.w[18] & 0xffu)), p2);
        const float ds1 = __fmul_rn(__fmul_rn(d, (float)(int)(int8_t)(r.w[18] >> 8)), p2);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const float sc = c < 2 ? ds0 : ds1;   // l / 16
            float w[8];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int wi = 2 * c + h;
                const uint32_t lw = __funnelshift_r(r.w[wi], r.w[wi + 1], r.sh);
                const uint32_t hw = __funnelshift_r(r.w[9 + wi], r.w[10 + wi], r.sh);
                const uint32_t q = ((lw >> s4) & 0x0f0f0f0fu) | (((hw >> s2) & 0x03030303u) << 4);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float qf = byte_f23(q, k) - 8388640.0f;   // q - 32, exact
                    w[4 * h + k] = __fmul_rn(sc, qf);
                }
            }
            store_chunk<TERMS>(bhi, rbase + (((4u * hf + (uint32_t)c) ^ r7) << 4), w);
        }
    }
}

// ------------------------------------------------------------- epilogue ----

__device__ __forceinline__ float silu_mul(float z, float u)
{
    return (z / (1.0f + expf(-z))) * u;   // src/brain_runtime.c:1755-1758
}

__device__ __forceinline__ void add4(float (&v)[8], int j, float4 f)
{
    v[4 * j] += f.x;
    v[4 * j + 1] += f.y;
    v[4 * j + 2] += f.z;
    v[4 * j + 3] += f.w;
}

// 8 consecutive output floats (n of them valid); vector accesses when the
// segment's layout keeps every 8-float group 16-byte aligned.
__device__ __forceinline__ void store8(float *p, const float (&y)[8], uint32_t n, bool vec)
{
    if (vec && n == 8u) {
        reinterpret_cast<float4 *>(p)[0] = make_float4(y[0], y[1], y[2], y[3]);
        reinterpret_cast<float4 *>(p)[1] = make_float4(y[4], y[5], y[6], y[7]);
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if ((uint32_t)j < n) p[j] = y[j];
    }
}

__device__ __forceinline__ void load8(const float *p, float (&y)[8], uint32_t n, bool vec)
{
    if (vec && n == 8u) {
        const float4 f0 = reinterpret_cast<const float4 *>(p)[0], f1 = reinterpret_cast<const float4 *>(p)[1];
        y[0] = f0.x; y[1] = f0.y; y[2] = f0.z; y[3] = f0.w;
        y[4] = f1.x; y[5] = f1.y; y[6] = f1.z; y[7] = f1.w;
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) y[j] = (uint32_t)j < n ? p[j] : 0.f;
    }
}

__device__ __forceinline__ float4 h4_to_f4(uint2 u)
{
    const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
}

// Store n of 8 values at element e of a segment's output (fp32, or binary16
// for an fp16 KV cache).
__device__ __forceinline__ void put8(const GemmSeg &g, size_t e, const float (&y)[8], uint32_t n)
{
    if (!g.f16) {
        store8(g.out + e, y, n, g.vec4 != 0);
        return;
    }
    __half *p = reinterpret_cast<__half *>(g.out) + e;
    if (g.vec4 && n == 8u) {
        uint4 u;
        u.x = pack_h2(y[0], y[1]);
        u.y = pack_h2(y[2], y[3]);
        u.z = pack_h2(y[4], y[5]);
        u.w = pack_h2(y[6], y[7]);
        *reinterpret_cast<uint4 *>(p) = u;
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if ((uint32_t)j < n) p[j] = __float2half_rn(y[j]);
    }
}

__device__ __forceinline__ void put1(const GemmSeg &g, size_t e, float y)
{
    if (g.f16) reinterpret_cast<__half *>(g.out)[e] = __float2half_rn(y);
    else g.out[e] = y;
}

// --------------------------------------------------------------- kernel ----

template <int TERMS>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ GemmArgs a)
{
    extern __shared__ uint8_t smem_raw[];
    const uint32_t base_addr = smem_addr(smem_raw);
    uint8_t *smem = smem_raw + (((base_addr + 1023u) & ~1023u) - base_addr);
    Bars *bars = reinterpret_cast<Bars *>(smem + (size_t)kStages * kStageBytes);
    volatile uint32_t *err = &bars->status;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t rank = cluster_rank(), pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
    const uint32_t n_units = a.n_tiles * a.tok_pairs * a.ksplit;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&bars->xfull[s], 1);
            mbar_init(&bars->full[s], kDequantWarps / 2 + 1);   // one group of 8 warps + the relay
            mbar_init(&bars->wfull[s], kDequantWarps / 2);
            mbar_init(&bars->empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bars->acc_full[b], 1);
            mbar_init(&bars->acc_empty[b], 8);
        }
        mbar_init(&bars->fin, 1);
        bars->status = kStatusOk;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc2(&bars->tmem, 512);
    tc_fence_before();
    cluster_sync();   // barriers of both CTAs initialised, TMEM allocated
    tc_fence_after();
    const uint32_t tmem = bars->tmem;

    if (warp == 0) {
        // ---------------------------------------------- activation copies --
        if (lane == 0) {
            const uint32_t xbytes = TERMS == 1 ? kATermBytes : 2 * kATermBytes;
            uint32_t it = 0;
            for (uint32_t u = pair; u < n_units; u += n_pairs) {
                const Unit un = unit_of(a, u);
                const uint32_t tok_tile = 2u * un.tt + rank;
                bool ok = true;
                for (uint32_t kb = un.kb0; kb < un.kb1; ++kb, ++it) {
                    const uint32_t s = it % kStages, ph = (it / kStages) & 1u;
                    if (!mbar_wait_cluster(&bars->empty[s], ph ^ 1u, err)) { ok = false; break; }
                    mbar_arrive_expect_tx(&bars->xfull[s], xbytes);
                    bulk_g2s(smem + (size_t)s * kStageBytes,
                             a.xt + ((size_t)tok_tile * a.kblocks + kb) * kXTileBytes, xbytes, &bars->xfull[s]);
                }
                if (!ok) break;
            }
            // drain: every issued copy lands before the CTA may exit
            for (uint32_t i = 0; i < (uint32_t)kStages && i < it; ++i) {
                const uint32_t idx = it - 1 - i;
                mbar_drain(&bars->xfull[idx % kStages], (idx / kStages) & 1u);
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            // ---------------------------------------------- MMA issue --
            uint32_t it = 0, lu = 0;
            for (uint32_t u = pair; u < n_units; u += n_pairs, ++lu) {
                const Unit un = unit_of(a, u);
                const uint32_t buf = lu & 1u, ap = (lu >> 1) & 1u;
                if (!mbar_wait_cluster(&bars->acc_empty[buf], ap ^ 1u, err)) break;
                tc_fence_after();
                const uint32_t d = tmem + buf * (uint32_t)kRowTile;
                bool ok = true;
                for (uint32_t kb = un.kb0; kb < un.kb1; ++kb, ++it) {
                    const uint32_t s = it % kStages, ph = (it / kStages) & 1u;
                    if (!mbar_wait_cluster(&bars->xfull[s], ph, err) || !mbar_wait_cluster(&bars->full[s], ph, err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t st = smem_addr(smem + (size_t)s * kStageBytes);
#pragma unroll
                    for (uint32_t k4 = 0; k4 < 4; ++k4) {
                        const uint64_t ah = sw128_desc(st + 32u * k4);
                        const uint64_t bh = sw128_desc(st + 2u * kATermBytes + 32u * k4);
                        umma2_f16(d, ah, bh, kIdesc, (kb != un.kb0 || k4 != 0u) ? 1u : 0u);
                        if (TERMS >= 2) umma2_f16(d, sw128_desc(st + kATermBytes + 32u * k4), bh, kIdesc, 1u);
                        if (TERMS >= 3)
                            umma2_f16(d, ah, sw128_desc(st + 2u * kATermBytes + kBTermBytes + 32u * k4), kIdesc, 1u);
                    }
                    umma2_commit_both(&bars->empty[s]);
                }
                if (!ok) break;
                umma2_commit_both(&bars->acc_full[buf]);
            }
            // drain: all MMAs issued by this thread complete before TMEM is freed
            umma2_commit(&bars->fin);
            mbar_drain(&bars->fin, 0);
        } else if (lane == 0) {
            // ------------------------------------- odd CTA: copy relay --
            uint32_t it = 0;
            for (uint32_t u = pair; u < n_units; u += n_pairs) {
                const Unit un = unit_of(a, u);
                bool ok = true;
                for (uint32_t kb = un.kb0; kb < un.kb1; ++kb, ++it) {
                    const uint32_t s = it % kStages, ph = (it / kStages) & 1u;
                    if (!mbar_wait_cluster(&bars->xfull[s], ph, err) || !mbar_wait_cluster(&bars->wfull[s], ph, err)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_cta(&bars->full[s], 0);
                }
                if (!ok) break;
            }
        }
        __syncwarp();
    } else if (warp >= 6) {
        // ------------------------------------------------------ dequant --
        // Two groups of 8 warps take alternate stages (group g the stages
        // it with it % 2 == g), two threads per weight row (halves of the
        // 64-value K block). A group has two stage periods per stage it
        // converts; the raw bytes of its next stage are loaded (into the
        // other of two register buffers) before the current one converts.
        const uint32_t grp = (warp - 6u) >> 3;
        const uint32_t dt = ((warp - 6u) & 7u) * 32u + lane, row = dt >> 1, hf = dt & 1u;
        struct Src {
            const uint8_t *wrow;
            uint32_t type, bb, kb0, kb1;
            float p2;
            bool valid;
        };
        auto src_of = [&](uint32_t u) {
            const Unit un = unit_of(a, u);
            const GemmSeg *sg;
            uint32_t grow;
            if (a.epi == GEPI_SWIGLU) {
                sg = &a.seg[rank];                   // even CTA: gate rows, odd CTA: up rows
                grow = un.tile * 128u + row;
            } else {
                sg = &a.seg[seg_of_tile(a, un.tile)];
                grow = (un.tile - sg->tile0) * (uint32_t)kRowTile + rank * 128u + row;
            }
            Src s;
            s.valid = grow < sg->rows;
            s.type = sg->type;
            s.bb = s.type == 12u ? 144u : 210u;
            s.p2 = ldexpf(1.0f, sg->wexp);
            s.wrow = sg->w + (size_t)(s.valid ? grow : 0u) * sg->row_bytes;
            s.kb0 = un.kb0;
            s.kb1 = un.kb1;
            return s;
        };
        // One thread per row (group 0) pulls the row's K range of a unit
        // into L2 with a bulk prefetch a whole unit ahead, so the register
        // loads wait for L2, not HBM.
        auto prefetch_unit = [&](const Src &s) {
            if (grp || hf || !s.valid) return;
            const uintptr_t b0 = reinterpret_cast<uintptr_t>(s.wrow + (size_t)(s.kb0 >> 2) * s.bb) & ~(uintptr_t)15;
            const uintptr_t b1 = reinterpret_cast<uintptr_t>(s.wrow + (size_t)((s.kb1 + 3u) >> 2) * s.bb) & ~(uintptr_t)15;
            if (b1 > b0) prefetch_l2(reinterpret_cast<const void *>(b0), (uint32_t)(b1 - b0));
        };
        struct Pos {
            uint32_t u, kb, it;
            Src s;
            bool live;
        };
        auto advance = [&](Pos &p) {   // the next stage of the pair's sequence
            ++p.it;
            if (++p.kb < p.s.kb1) return;
            p.u += n_pairs;
            p.live = p.u < n_units;
            if (!p.live) return;
            p.s = src_of(p.u);
            p.kb = p.s.kb0;
            if (p.u + n_pairs < n_units) prefetch_unit(src_of(p.u + n_pairs));
        };
        Pos cur;
        cur.u = pair;
        cur.it = 0;
        cur.live = pair < n_units;
        if (cur.live) {
            cur.s = src_of(pair);
            cur.kb = cur.s.kb0;
            prefetch_unit(cur.s);
            if (pair + n_pairs < n_units) prefetch_unit(src_of(pair + n_pairs));
            if (grp) advance(cur);
        }
        if (cur.live) {
            Raw ra, rb;
            if (cur.s.valid) load_raw(cur.s.type, cur.s.wrow + (size_t)(cur.kb >> 2) * cur.s.bb, cur.kb & 3u, hf, ra);
            // one stage of this group: load its next stage into `nxt`, convert
            // `cur_raw`; false when the group's work is done or a wait failed
            auto stage = [&](const Raw &cur_raw, Raw &nxt) -> bool {
                Pos q = cur;
                advance(q);
                if (q.live) advance(q);
                if (q.live && q.s.valid) load_raw(q.s.type, q.s.wrow + (size_t)(q.kb >> 2) * q.s.bb, q.kb & 3u, hf, nxt);
                const uint32_t s = cur.it % kStages, ph = (cur.it / kStages) & 1u;
                if (!warp_wait(&bars->empty[s], ph ^ 1u, err)) return false;
                uint8_t *bhi = smem + (size_t)s * kStageBytes + 2u * kATermBytes;
                if (cur.s.valid) {
                    dequant_half<TERMS>(cur.s.type, cur_raw, cur.kb & 3u, hf, cur.s.p2, bhi, row);
                } else {
                    const uint32_t rbase = (row >> 3) * 1024u + (row & 7u) * 128u;
#pragma unroll
                    for (uint32_t c = 0; c < 4; ++c) {
                        const uint32_t off = rbase + (((4u * hf + c) ^ (row & 7u)) << 4);
                        *reinterpret_cast<uint4 *>(bhi + off) = make_uint4(0, 0, 0, 0);
                        if (TERMS >= 3) *reinterpret_cast<uint4 *>(bhi + kBTermBytes + off) = make_uint4(0, 0, 0, 0);
                    }
                }
                fence_proxy_async();
                __syncwarp();
                if (lane == 0) mbar_arrive(rank == 0 ? &bars->full[s] : &bars->wfull[s]);
                cur = q;
                return cur.live;
            };
            while (stage(ra, rb) && stage(rb, ra)) {
            }
        }
    } else {
        // ----------------------------------------------------- epilogue --
        // Each warp owns 32 token rows (its TMEM lane quarter) and handles them
        // independently, split-K arrivals included (one counter per quarter).
        const uint32_t quarter = warp & 3u, trow = quarter * 32u + lane;
        uint32_t lu = 0;
        for (uint32_t u = pair; u < n_units; u += n_pairs, ++lu) {
            const Unit un = unit_of(a, u);
            const uint32_t buf = lu & 1u, ap = (lu >> 1) & 1u;
            if (!warp_wait(&bars->acc_full[buf], ap, err)) break;
            tc_fence_after();
            const uint32_t tbase = tmem + ((quarter * 32u) << 16) + buf * (uint32_t)kRowTile;
            const uint32_t t = (2u * un.tt + rank) * (uint32_t)kTokTile + trow;
            const bool tvalid = t < a.tokens;
            const uint32_t tile_id = (un.tile * a.tok_pairs + un.tt) * 2u + rank;
            if (a.ksplit > 1) {
                // store this K range's partial tile; the split-K reduction
                // kernel sums the partials in K order and applies the epilogue
                float *dst = a.ws + ((size_t)(tile_id * a.ksplit + un.ks) * kTokTile + trow) * kRowTile;
                for (uint32_t c = 0; c < (uint32_t)kRowTile; c += 16) {
                    uint32_t r[16];
                    tmem_ld16(tbase + c, r);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; j += 4)
                        __stcg(reinterpret_cast<float4 *>(dst + c + j),
                               make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]), __uint_as_float(r[j + 2]),
                                           __uint_as_float(r[j + 3])));
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    if (rank == 0) mbar_arrive(&bars->acc_empty[buf]);
                    else mbar_arrive_cta(&bars->acc_empty[buf], 0);
                }
                continue;
            }
            // values of columns [c, c+8) of this thread's token row (accumulator scale)
            auto fetch = [&](uint32_t c, float (&v)[8]) {
                uint32_t r[8];
                tmem_ld8(tbase + c, r);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 8; ++j) v[j] = __uint_as_float(r[j]);
            };
            const float xs = tvalid ? __ldg(a.xscale + t) : 0.f;
            if (a.epi == GEPI_SWIGLU) {
                const GemmSeg &g = a.seg[0];
                const float sg = xs * ldexpf(1.0f, -g.wexp), su = xs * ldexpf(1.0f, -a.seg[1].wexp);
                float *o = g.out + (size_t)(t + g.tok_off) * g.tok_stride;
                for (uint32_t c = 0; c < 128u; c += 8) {
                    float vg[8], vu[8];
                    fetch(c, vg);
                    fetch(128u + c, vu);
                    const uint32_t r0 = un.tile * 128u + c;
#pragma unroll
                    for (int j = 0; j < 8; ++j) vg[j] = silu_mul(vg[j] * sg, vu[j] * su);
                    if (tvalid && r0 < g.rows)
                        store8(o + (r0 >> 7) * g.head_stride + (r0 & 127u), vg, min(8u, g.rows - r0), g.vec4 != 0);
                }
            } else {
                const GemmSeg &g = a.seg[seg_of_tile(a, un.tile)];
                const float s = xs * ldexpf(1.0f, -g.wexp);
                const uint32_t row0 = (un.tile - g.tile0) * (uint32_t)kRowTile;
                float *o = g.out + (size_t)(t + g.tok_off) * g.tok_stride;
                if (g.rope) {
                    // RoPE pairs (i, i + 64) of each 128-row head (src/brain_runtime.c:1391-1398)
                    const float2 *cs = reinterpret_cast<const float2 *>(a.rope) + (size_t)(a.pos0 + t) * 64u;
                    for (uint32_t hh = 0; hh < 2u; ++hh)
                        for (uint32_t c = 0; c < 64u; c += 8) {
                            float va[8], vb[8];
                            fetch(hh * 128u + c, va);
                            fetch(hh * 128u + 64u + c, vb);
                            const uint32_t ra = row0 + hh * 128u + c, rb = ra + 64u;
                            if (!tvalid || rb >= g.rows) continue;
                            const uint32_t na = min(8u, g.rows - ra), nb = min(8u, g.rows - rb);
#pragma unroll
                            for (int j = 0; j < 8; ++j) {
                                const float2 r = __ldg(cs + c + (uint32_t)j);
                                const float x0 = va[j] * s + ((g.bias && (uint32_t)j < na) ? __ldg(g.bias + ra + j) : 0.f);
                                const float x1 = vb[j] * s + ((g.bias && (uint32_t)j < nb) ? __ldg(g.bias + rb + j) : 0.f);
                                va[j] = __fsub_rn(__fmul_rn(x0, r.x), __fmul_rn(x1, r.y));
                                vb[j] = __fadd_rn(__fmul_rn(x0, r.y), __fmul_rn(x1, r.x));
                            }
                            const size_t et = (size_t)(t + g.tok_off) * g.tok_stride;
                            put8(g, et + (ra >> 7) * g.head_stride + (ra & 127u), va, na);
                            put8(g, et + (rb >> 7) * g.head_stride + (rb & 127u), vb, nb);
                        }
                } else {
                    for (uint32_t c = 0; c < (uint32_t)kRowTile; c += 8) {
                        float v[8];
                        fetch(c, v);
                        const uint32_t r0 = row0 + c;
                        if (!tvalid || r0 >= g.rows) continue;
                        const uint32_t n = min(8u, g.rows - r0);
                        float *p = o + (r0 >> 7) * g.head_stride + (r0 & 127u);
                        if (a.epi == GEPI_RESID) {
                            float x[8];
                            load8(p, x, n, g.vec4 != 0);   // residual stream, src/brain_runtime.c:1745, :1762
#pragma unroll
                            for (int j = 0; j < 8; ++j) v[j] = x[j] + v[j] * s;
                            store8(p, v, n, g.vec4 != 0);
                        } else {
#pragma unroll
                            for (int j = 0; j < 8; ++j)
                                v[j] = v[j] * s + ((g.bias && (uint32_t)j < n) ? __ldg(g.bias + r0 + j) : 0.f);
                            put8(g, (size_t)(t + g.tok_off) * g.tok_stride + (r0 >> 7) * g.head_stride + (r0 & 127u), v, n);
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if (rank == 0) mbar_arrive(&bars->acc_empty[buf]);
                else mbar_arrive_cta(&bars->acc_empty[buf], 0);
            }
        }
    }

    // Both CTAs stay resident until the pair is done: the even CTA's MMAs read
    // the odd CTA's shared memory and the odd CTA arrives on the even one's
    // barriers.
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    tc_fence_after();
    if (warp == 1) tmem_dealloc2(tmem, 512);
    if (threadIdx.x == 0 && bars->status != kStatusOk) atomicCAS(a.status, kStatusOk, bars->status);
}


// ------------------------------------------------------ split-K reduce ----

// Sums the K ranges' partial tiles of a split contraction in K order and
// applies its epilogue. One thread per (tile, token row, 4 columns):
// consecutive threads read consecutive 16-byte pieces of a partial row.
// RoPE tiles take the column pairs (c, c + 64) of each head in one thread,
// SwiGLU tiles the gate / up pairs (c, c + 128).
__global__ void __launch_bounds__(256) splitk_kernel(const __grid_constant__ GemmArgs a)
{
    const uint64_t total = (uint64_t)a.n_tiles * a.tok_pairs * 2u * kTokTile * 64u;
    const size_t kstride = (size_t)kTokTile * kRowTile;
    for (uint64_t item = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; item < total;
         item += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t c = 4u * (uint32_t)(item & 63u), trow = (uint32_t)((item >> 6) % kTokTile);
        const uint32_t tile_id = (uint32_t)(item / (64u * kTokTile));
        const uint32_t rank = tile_id & 1u, rest = tile_id >> 1, tt = rest % a.tok_pairs, tile = rest / a.tok_pairs;
        const uint32_t t = (2u * tt + rank) * (uint32_t)kTokTile + trow;
        if (t >= a.tokens) continue;
        const bool swiglu = a.epi == GEPI_SWIGLU;
        const GemmSeg &g = a.seg[swiglu ? 0u : seg_of_tile(a, tile)];
        const bool paired = swiglu || g.rope;
        const uint32_t off2 = swiglu ? 128u : 64u;
        if (paired && (c & (2u * off2 - 1u)) >= off2) continue;   // the second column of a pair
        const float *base = a.ws + ((size_t)tile_id * a.ksplit * kTokTile + trow) * kRowTile + c;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f), w = v;
        for (uint32_t k = 0; k < a.ksplit; ++k) {
            const float4 p = __ldcg(reinterpret_cast<const float4 *>(base + k * kstride));
            v.x += p.x; v.y += p.y; v.z += p.z; v.w += p.w;
            if (paired) {
                const float4 q = __ldcg(reinterpret_cast<const float4 *>(base + k * kstride + off2));
                w.x += q.x; w.y += q.y; w.z += q.z; w.w += q.w;
            }
        }
        const float xs = __ldg(a.xscale + t);
        const float va[4] = {v.x, v.y, v.z, v.w}, vb[4] = {w.x, w.y, w.z, w.w};
        if (swiglu) {
            const float sg = xs * ldexpf(1.0f, -g.wexp), su = xs * ldexpf(1.0f, -a.seg[1].wexp);
            float *o = g.out + (size_t)(t + g.tok_off) * g.tok_stride;
            for (int j = 0; j < 4; ++j) {
                const uint32_t r = tile * 128u + c + (uint32_t)j;
                if (r < g.rows) o[(r >> 7) * g.head_stride + (r & 127u)] = silu_mul(va[j] * sg, vb[j] * su);
            }
            continue;
        }
        const float s = xs * ldexpf(1.0f, -g.wexp);
        const uint32_t row0 = (tile - g.tile0) * (uint32_t)kRowTile;
        float *o = g.out + (size_t)(t + g.tok_off) * g.tok_stride;
        if (g.rope) {
            // src/brain_runtime.c:1391-1398
            const float2 *cs = reinterpret_cast<const float2 *>(a.rope) + (size_t)(a.pos0 + t) * 64u;
            for (int j = 0; j < 4; ++j) {
                const uint32_t ra = row0 + c + (uint32_t)j, rb = ra + 64u;
                if (rb >= g.rows) continue;
                const float2 r = __ldg(cs + ((c + (uint32_t)j) & 63u));
                const float x0 = va[j] * s + (g.bias ? __ldg(g.bias + ra) : 0.f);
                const float x1 = vb[j] * s + (g.bias ? __ldg(g.bias + rb) : 0.f);
                const size_t et = (size_t)(t + g.tok_off) * g.tok_stride;
                put1(g, et + (ra >> 7) * g.head_stride + (ra & 127u), __fsub_rn(__fmul_rn(x0, r.x), __fmul_rn(x1, r.y)));
                put1(g, et + (rb >> 7) * g.head_stride + (rb & 127u), __fadd_rn(__fmul_rn(x0, r.y), __fmul_rn(x1, r.x)));
            }
            continue;
        }
        float prev[4] = {0.f, 0.f, 0.f, 0.f};
        if (a.epi == GEPI_RESID)
            for (int j = 0; j < 4; ++j) {
                const uint32_t r = row0 + c + (uint32_t)j;
                if (r < g.rows) prev[j] = o[(r >> 7) * g.head_stride + (r & 127u)];
            }
        for (int j = 0; j < 4; ++j) {
            const uint32_t r = row0 + c + (uint32_t)j;
            if (r >= g.rows) continue;
            float y = va[j] * s;
            if (a.epi == GEPI_RESID) y = prev[j] + y;   // src/brain_runtime.c:1745, :1762
            else if (g.bias) y += __ldg(g.bias + r);
            put1(g, (size_t)(t + g.tok_off) * g.tok_stride + (r >> 7) * g.head_stride + (r & 127u), y);
        }
    }
}

// ---------------------------------------------------- activation split ----

// One CTA per token row (padding rows of the last token tile included):
// optional rms_norm (src/brain_runtime.c:1338-1371: double sum of squares,
// out = x * inv * w), power-of-two scaling of the row into [2^14, 2^15),
// binary16 hi/lo split, stored as 128-byte-swizzled K-major tiles
// [token tile][K block][hi, lo][128 rows x 64]. The row is read from global
// memory once (into shared memory, cols floats of dynamic shared memory).
__global__ void __launch_bounds__(256) split_kernel(const float *x, uint32_t ldx, uint32_t cols, uint32_t tokens,
                                                    const float *norm_w, float eps, uint8_t *xt, float *xscale)
{
    extern __shared__ float rowbuf[];
    __shared__ double dred[8];
    __shared__ float fred[8];
    const uint32_t t = blockIdx.x, tl = t % kTokTile, tt = t / kTokTile, kbn = cols / kKBlock;
    const uint32_t nch = cols / 8;
    uint8_t *tile0 = xt + (size_t)tt * kbn * kXTileBytes;
    if (t >= tokens) {
        for (uint32_t ch = threadIdx.x; ch < nch; ch += blockDim.x) {
            uint8_t *p = tile0 + (size_t)(ch >> 3) * kXTileBytes + sw128_off(tl, ch & 7u);
            *reinterpret_cast<uint4 *>(p) = make_uint4(0, 0, 0, 0);
            *reinterpret_cast<uint4 *>(p + kATermBytes) = make_uint4(0, 0, 0, 0);
        }
        if (threadIdx.x == 0) xscale[t] = 0.f;
        return;
    }
    const float *xr = x + (size_t)t * ldx;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const bool vec = ((reinterpret_cast<uintptr_t>(xr) & 15u) == 0);
    // pass 1: the row into shared memory, with the sum of squares (RMSNorm)
    // or, without a norm, the largest magnitude
    double ss = 0.0;
    float amax = 0.f;
    const bool norm = norm_w != nullptr;
    if (vec) {
        for (uint32_t i = threadIdx.x; i < cols / 4; i += blockDim.x) {
            const float4 v = __ldcg(reinterpret_cast<const float4 *>(xr) + i);
            reinterpret_cast<float4 *>(rowbuf)[i] = v;
            if (norm) ss += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
            else amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
    } else {
        for (uint32_t i = threadIdx.x; i < cols; i += blockDim.x) {
            const float v = __ldcg(xr + i);
            rowbuf[i] = v;
            if (norm) ss += (double)v * v;
            else amax = fmaxf(amax, fabsf(v));
        }
    }
    if (norm) {
        // pass 2: normalise in place, then the largest magnitude
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) dred[warp] = ss;
        __syncthreads();
        double tot = 0.0;
        for (int i = 0; i < 8; ++i) tot += dred[i];
        const float inv = 1.0f / sqrtf((float)(tot / (double)cols) + eps);
        for (uint32_t i = threadIdx.x; i < cols; i += blockDim.x) {
            const float v = __fmul_rn(__fmul_rn(rowbuf[i], inv), __ldg(norm_w + i));
            rowbuf[i] = v;
            amax = fmaxf(amax, fabsf(v));
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0) fred[warp] = amax;
    __syncthreads();
    amax = 0.f;
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fred[i]);
    int e = 0;
    if (amax > 0.f && amax <= FLT_MAX) frexpf(amax, &e);
    // exponent kept in [-126, 126] so that 2^sx and 2^-sx stay finite normal
    // numbers: a row of tiny values (a SwiGLU output of all-negative gates
    // can sit near the fp32 underflow limit) then contributes ~0, as in fp32
    const int sx = amax > 0.f ? max(-126, min(126, 15 - e)) : 0;
    const float p2 = ldexpf(1.0f, sx);
    for (uint32_t ch = threadIdx.x; ch < nch; ch += blockDim.x) {
        const float4 a0 = reinterpret_cast<const float4 *>(rowbuf)[2 * ch];
        const float4 a1 = reinterpret_cast<const float4 *>(rowbuf)[2 * ch + 1];
        const float v[8] = {a0.x * p2, a0.y * p2, a0.z * p2, a0.w * p2, a1.x * p2, a1.y * p2, a1.z * p2, a1.w * p2};
        uint32_t h[4], l[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            h[j] = pack_h2(v[2 * j], v[2 * j + 1]);
            const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&h[j]));
            l[j] = pack_h2(v[2 * j] - f.x, v[2 * j + 1] - f.y);
        }
        uint8_t *p = tile0 + (size_t)(ch >> 3) * kXTileBytes + sw128_off(tl, ch & 7u);
        *reinterpret_cast<uint4 *>(p) = make_uint4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<uint4 *>(p + kATermBytes) = make_uint4(l[0], l[1], l[2], l[3]);
    }
    if (threadIdx.x == 0) xscale[t] = ldexpf(1.0f, -sx);
}

// ------------------------------------------------------------ embedding ----

// x[t] = token_embd row ids[t] (load_embedding_row, src/brain_runtime.c:1311-1332).
__global__ void embed_kernel(const uint32_t *ids, uint32_t tokens, const uint8_t *embd, uint32_t type,
                             uint64_t row_bytes, uint32_t hidden, float *x)
{
    const uint32_t t = blockIdx.x;
    if (t >= tokens) return;
    const uint8_t *row = embd + (size_t)ids[t] * row_bytes;
    const uint32_t be = block_elems(type), bb = block_bytes(type);
    for (uint32_t i = threadIdx.x; i < hidden; i += blockDim.x)
        x[(size_t)t * hidden + i] = deq_elem(type, row + (size_t)(i / be) * bb, (int)(i % be));
}

// Prompt attention: prefill_attn.cu (tensor cores).

// ------------------------------------------------- weight scale bound ------

// Upper bound of |w| over a Q4_K / Q6_K tensor from its block headers, as
// float bits (non-negative floats order like unsigned integers).
__global__ void wbound_kernel(uint32_t type, const uint8_t *blocks, uint64_t nblocks, uint32_t *out_bits)
{
    float mx = 0.f;
    for (uint64_t b = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; b < nblocks; b += (uint64_t)gridDim.x * blockDim.x) {
        const uint8_t *p = blocks + b * (type == 12u ? 144u : 210u);
        float v;
        if (type == 12u) {
            const float d = fabsf(h2f_exact(ld_u16(p))), dm = fabsf(h2f_exact(ld_u16(p + 2)));
            v = d * 63.f * 15.f + dm * 63.f;
        } else {
            v = fabsf(h2f_exact(ld_u16(p + 208))) * 128.f * 32.f;
        }
        if (!(v <= FLT_MAX)) v = FLT_MAX;   // NaN / inf headers: clamp
        mx = fmaxf(mx, v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31u) == 0) atomicMax(out_bits, __float_as_uint(mx));
}

}  // namespace pf
}  // namespace atlas

using namespace atlas;
using namespace atlas::pf;

extern "C" size_t atlas_prefill_gemm_smem() { return kGemmSmem; }

namespace {

using GemmFn = void (*)(GemmArgs);

GemmFn gemm_fn(uint32_t terms)
{
    return terms == 1 ? gemm_kernel<1> : terms == 2 ? gemm_kernel<2> : gemm_kernel<3>;
}

cudaError_t gemm_prepare(uint32_t terms)
{
    static bool attr_set[3] = {false, false, false};
    if (terms < 1 || terms > 3) return cudaErrorInvalidValue;
    if (!attr_set[terms - 1]) {
        cudaError_t e = cudaFuncSetAttribute(gemm_fn(terms), cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemmSmem);
        if (e != cudaSuccess) return e;
        attr_set[terms - 1] = true;
    }
    return cudaSuccess;
}

}  // namespace

// CTA pairs of the contraction kernel that fit on the device at once.
extern "C" cudaError_t atlas_prefill_gemm_pairs(int *pairs)
{
    cudaError_t e = gemm_prepare(3);
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(sms & ~1));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kGemmSmem;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, gemm_fn(3), &cfg);
    if (e != cudaSuccess) return e;
    *pairs = n;
    return cudaSuccess;
}

// grid = 2 x the number of CTA pairs (clusters of two are compiled in).
extern "C" cudaError_t atlas_launch_prefill_gemm(const GemmArgs *a, int grid, cudaStream_t stream)
{
    cudaError_t e = gemm_prepare(a->terms);
    if (e != cudaSuccess) return e;
    if (grid < 2 || (grid & 1)) return cudaErrorInvalidValue;
    gemm_fn(a->terms)<<<grid, kThreads, kGemmSmem, stream>>>(*a);
    e = cudaGetLastError();
    if (e != cudaSuccess || a->ksplit <= 1) return e;
    int sms = 0, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    splitk_kernel<<<4 * sms, 256, 0, stream>>>(*a);
    return cudaGetLastError();
}

// qwen3 per-head q/k RMSNorm then RoPE over a prompt chunk
// (src/brain_runtime.c:1727-1737, rms_norm :1338-1371, rope :1377-1401): one
// CTA of 64 threads per (token, head); thread p holds the RoPE pair (p, p + 64).
// Query heads are normalized in place in q [tokens][q_heads * 128]; key heads
// are read from kin [tokens][kv_heads * 128] and written into the KV cache at
// positions pos0 + t (binary16 when kv_f16).
__global__ void __launch_bounds__(64) qk_norm_rope_kernel(float *q, uint32_t q_heads, const float *kin, void *kcache,
                                                          uint32_t kv_heads, uint32_t max_context, uint32_t pos0,
                                                          const float *qn, const float *kn, const float2 *rope,
                                                          float eps, uint32_t kv_f16)
{
    __shared__ double red[2];
    const uint32_t t = blockIdx.x, hh = blockIdx.y, p = threadIdx.x;
    const bool isq = hh < q_heads;
    const float *src = isq ? q + ((size_t)t * q_heads + hh) * 128u : kin + ((size_t)t * kv_heads + (hh - q_heads)) * 128u;
    const float *w = isq ? qn : kn;
    const float a = src[p], b = src[p + 64u];
    double ss = (double)a * a + (double)b * b;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((p & 31u) == 0u) red[p >> 5] = ss;
    __syncthreads();
    const float inv = 1.0f / sqrtf((float)((red[0] + red[1]) / 128.0) + eps);
    const float x0 = __fmul_rn(__fmul_rn(a, inv), w[p]), x1 = __fmul_rn(__fmul_rn(b, inv), w[p + 64u]);
    const float2 r = rope[(size_t)(pos0 + t) * 64u + p];
    const float y0 = __fsub_rn(__fmul_rn(x0, r.x), __fmul_rn(x1, r.y));
    const float y1 = __fadd_rn(__fmul_rn(x0, r.y), __fmul_rn(x1, r.x));
    if (isq) {
        float *dst = q + ((size_t)t * q_heads + hh) * 128u;
        dst[p] = y0;
        dst[p + 64u] = y1;
        return;
    }
    const size_t off = ((size_t)(hh - q_heads) * max_context + pos0 + t) * 128u;
    if (kv_f16) {
        reinterpret_cast<__half *>(kcache)[off + p] = __float2half_rn(y0);
        reinterpret_cast<__half *>(kcache)[off + p + 64u] = __float2half_rn(y1);
    } else {
        reinterpret_cast<float *>(kcache)[off + p] = y0;
        reinterpret_cast<float *>(kcache)[off + p + 64u] = y1;
    }
}

extern "C" cudaError_t atlas_launch_prefill_qknorm(float *q, uint32_t q_heads, const float *kin, void *kcache,
                                                   uint32_t kv_heads, uint32_t max_context, uint32_t pos0,
                                                   uint32_t tokens, const float *qn, const float *kn,
                                                   const float2 *rope, float eps, uint32_t kv_f16,
                                                   cudaStream_t stream)
{
    qk_norm_rope_kernel<<<dim3(tokens, q_heads + kv_heads), 64, 0, stream>>>(q, q_heads, kin, kcache, kv_heads,
                                                                            max_context, pos0, qn, kn, rope, eps,
                                                                            kv_f16);
    return cudaGetLastError();
}

extern "C" cudaError_t atlas_launch_prefill_split(const float *x, uint32_t ldx, uint32_t cols, uint32_t tokens,
                                                  uint32_t tok_pad, const float *norm_w, float eps, uint8_t *xt,
                                                  float *xscale, cudaStream_t stream)
{
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)(kSplitMaxCols * 4));
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    if (cols > kSplitMaxCols || cols % kKBlock) return cudaErrorInvalidValue;
    split_kernel<<<tok_pad, 256, cols * 4, stream>>>(x, ldx, cols, tokens, norm_w, eps, xt, xscale);
    return cudaGetLastError();
}

extern "C" cudaError_t atlas_launch_prefill_embed(const uint32_t *ids, uint32_t tokens, const uint8_t *embd,
                                                  uint32_t type, uint64_t row_bytes, uint32_t hidden, float *x,
                                                  cudaStream_t stream)
{
    embed_kernel<<<tokens, 256, 0, stream>>>(ids, tokens, embd, type, row_bytes, hidden, x);
    return cudaGetLastError();
}

extern "C" cudaError_t atlas_launch_wbound(uint32_t type, const uint8_t *blocks, uint64_t nblocks, uint32_t *out_bits,
                                           cudaStream_t stream)
{
    wbound_kernel<<<148, 256, 0, stream>>>(type, blocks, nblocks, out_bits);
    return cudaGetLastError();
}
