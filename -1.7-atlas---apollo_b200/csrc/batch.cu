// Batched decode step kernels (sm_100a): see batch.h.
//
// mvb_kernel: y_s = W x_s for up to 8 sequences s at once. A task is 16 weight
// rows x one 256-element block (Q4_K 144 bytes, Q6_K 210 bytes per row), as in
// the single-sequence GEMV, and every task now feeds all 8 sequences: the
// MMA's B operand holds one sequence per column (mma.sync m16n8k16, binary16
// hi and lo parts of x as two MMAs), so the weights' dequantization, the
// copies and the instruction stream are shared by the 8 tokens.
//
// Each CTA owns whole 16-row tiles of one segment within one K slice of at
// most kSplitMax blocks, stages that slice of the 8 inputs in shared memory
// (x * norm weight, a power-of-two scale per sequence and CTA, binary16 hi/lo,
// 16-element sums), streams its tasks through per-warp cp.async rings and
// writes the slice's partial rows. Tiles shared by several warps are added in
// warp order; slices are added in slice order by the consumer.
#include <algorithm>
#include <cfloat>
#include <cmath>
#include "common.cuh"
#include "quant.cuh"
#include "tc_tiles.cuh"
#include "batch.h"

namespace atlas {
namespace bt {
namespace {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ void cpa16(uint32_t dst, const void *src, uint64_t policy)
{
    asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "l"(policy)
                 : "memory");
}
__device__ __forceinline__ void cpa_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cpa_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
__device__ __forceinline__ void bsync() { asm volatile("bar.sync 1, %0;" ::"n"(kBThreads) : "memory"); }

// 4 bytes at a 2-byte-aligned shared-memory address.
__device__ __forceinline__ uint32_t ldw2(const uint8_t *p)
{
    const uintptr_t ad = reinterpret_cast<uintptr_t>(p);
    const uint32_t *q = reinterpret_cast<const uint32_t *>(ad & ~uintptr_t(3));
    return __funnelshift_r(q[0], q[1], (uint32_t)(ad & 3u) * 8u);
}

constexpr uint32_t kQ4Row = 144u, kQ6Row = 240u;   // slot row strides (odd multiples of 16 bytes)

struct __align__(16) BHdr {
    uint32_t wstart[kBWarps];   // first task of each warp
    uint32_t cnt[kBWarps];      // arrivals at a shared tile, indexed by its first warp
    uint32_t smax[kMaxSeq];     // max |x| of each sequence's slice (float bits)
    float sinv[kMaxSeq];        // 1 / the sequence's power-of-two scale
    uint2 cp[8][32];            // per (copy i, lane): source offset in the block's rows, slot offset
};
__host__ __device__ constexpr uint32_t a128(uint32_t v) { return (v + 127u) & ~127u; }
__host__ __device__ constexpr uint32_t hdr_bytes() { return a128((uint32_t)sizeof(BHdr)); }
// partial rows of shared tiles: [warp][first / last tile][16 rows][8 sequences]
constexpr uint32_t kPartBytes = kBWarps * 2u * 128u * 4u;
// staged x: quads [split_blocks * 64][8 sequences] of (hi 01, hi 23, lo 01, lo 23), then the
// 16-element sums [split_blocks * 16][8]
__host__ __device__ constexpr uint32_t xq_bytes(uint32_t sb) { return sb * 64u * kMaxSeq * 16u; }
__host__ __device__ constexpr uint32_t xs_bytes(uint32_t sb) { return a128(sb * 16u * kMaxSeq * 4u); }
// 32-element sums for the Q4_K min term: [split_blocks][8 sequences][4] of (hi pair, lo pair)
__host__ __device__ constexpr uint32_t xm_bytes(uint32_t sb) { return a128(sb * 32u * 8u); }
__host__ __device__ constexpr uint32_t smem_total(uint32_t sb, uint32_t nslot, uint32_t slot)
{
    return hdr_bytes() + kPartBytes + xq_bytes(sb) + xs_bytes(sb) + xm_bytes(sb) + kBWarps * nslot * slot;
}

// ------------------------------------------------------------- staging ----
//
// Quad e4 of sequence s sits at x unit e4 * 8 + col(e4, s): a 16-byte load is
// served 8 lanes at a time, and the 8 lanes of a phase - rows g = 2p, 2p + 1,
// k positions t = 0..3 - must fall in 8 distinct 16-byte bank groups. Their
// quads are e4 = base + 2t (Q4_K words) or base + t (Q6_K words), so the
// column is the sequence XOR twice a 2-bit function of e4 that runs over all 4
// values as t does.
__device__ __forceinline__ uint32_t xcol(uint32_t e4, uint32_t s, bool q4)
{
    return s ^ ((q4 ? ((e4 >> 1) & 3u) : (e4 & 3u)) << 1);
}

// The CTA's K slice (blocks b0 .. b0 + nbs - 1) of every sequence's input:
// pass 1 stores x (times the norm weight) as floats in the quad slots and
// takes each sequence's max |x|; pass 2 scales by a power of two putting the
// max in [2^13, 2^14), splits into binary16 hi + lo in place and writes the
// 16-element sums. Sequences >= nseq are zeros.
__device__ void stage_x(const BArgs &a, BHdr *h, uint4 *xq, float *xs, uint2 *xm, uint32_t b0, uint32_t nbs, bool q4)
{
    const uint32_t nq = nbs * 64u, total = nq * kMaxSeq;
    const uint32_t lane = threadIdx.x & 31u;
    float4 *xf = reinterpret_cast<float4 *>(xq);
    for (uint32_t i = threadIdx.x; i < total; i += kBThreads) {
        const uint32_t s = i / nq, e4 = i - s * nq;   // a warp's 32 items share s (nq is a multiple of 64)
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (s < a.nseq) {
            const uint32_t k = b0 * 256u + 4u * e4;
            v = __ldcg(reinterpret_cast<const float4 *>(a.x + (size_t)s * a.xstride + k));
            if (a.norm_w) {
                const float4 w = __ldg(reinterpret_cast<const float4 *>(a.norm_w + k));
                v.x *= w.x; v.y *= w.y; v.z *= w.z; v.w *= w.w;
            }
        }
        xf[e4 * kMaxSeq + xcol(e4, s, q4)] = v;
        float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0 && m > 0.f) atomicMax(&h->smax[s], __float_as_uint(m));   // max: order-independent
    }
    bsync();
    if (threadIdx.x < kMaxSeq) {
        const float m = __uint_as_float(h->smax[threadIdx.x]);
        // exponent capped at 126: tiny slices keep a finite scale (cf. the single-sequence staging)
        const int e = (m > 0.f && isfinite(m)) ? min(13 - ilogbf(m), 126) : 0;
        h->sinv[threadIdx.x] = exp2f((float)-e);
        h->smax[threadIdx.x] = __float_as_uint(exp2f((float)e));   // now the scale itself
    }
    bsync();
    // item i: quad e4 = 4 (i / 32) + i % 4 of sequence (i / 4) % 8, so the 4
    // quads of a 16-element group sit in adjacent lanes
    for (uint32_t i = threadIdx.x; i < total; i += kBThreads) {
        const uint32_t s = (i >> 2) & 7u, e4 = (i >> 5) * 4u + (i & 3u);
        const float sc = __uint_as_float(h->smax[s]);
        const float4 v = xf[e4 * kMaxSeq + xcol(e4, s, q4)];
        const float e0 = v.x * sc, e1 = v.y * sc, e2 = v.z * sc, e3 = v.w * sc;
        const __half2 h01 = __floats2half2_rn(e0, e1), h23 = __floats2half2_rn(e2, e3);
        const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
        const __half2 l01 = __floats2half2_rn(e0 - f01.x, e1 - f01.y), l23 = __floats2half2_rn(e2 - f23.x, e3 - f23.y);
        uint4 pk;
        pk.x = *reinterpret_cast<const uint32_t *>(&h01);
        pk.y = *reinterpret_cast<const uint32_t *>(&h23);
        pk.z = *reinterpret_cast<const uint32_t *>(&l01);
        pk.w = *reinterpret_cast<const uint32_t *>(&l23);
        xq[e4 * kMaxSeq + xcol(e4, s, q4)] = pk;   // in place: the slot is this item's only
        float sum = (e0 + e1) + (e2 + e3);
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        if ((i & 3u) == 0u) xs[(e4 >> 2) * kMaxSeq + s] = sum;
    }
    bsync();
    if (q4) {
        // the 32-element sums of sub-blocks 2t, 2t + 1 of sequence g (entry g * 4 + t of
        // each block) as binary16 hi / lo pairs, scaled by 2^-6 (|sum| < 2^19 -> < 2^13)
        for (uint32_t i = threadIdx.x; i < nbs * 32u; i += kBThreads) {
            const uint32_t b = i >> 5, g = (i >> 2) & 7u, t = i & 3u;
            const float *x16 = xs + (b * 16u + 4u * t) * kMaxSeq + g;
            const float v0 = (x16[0] + x16[kMaxSeq]) * 0.015625f;
            const float v1 = (x16[2u * kMaxSeq] + x16[3u * kMaxSeq]) * 0.015625f;
            const __half2 hi = __floats2half2_rn(v0, v1);
            const float2 fh = __half22float2(hi);
            const __half2 lo = __floats2half2_rn(v0 - fh.x, v1 - fh.y);
            xm[i] = make_uint2(*reinterpret_cast<const uint32_t *>(&hi), *reinterpret_cast<const uint32_t *>(&lo));
        }
        bsync();
    }
}

// ----------------------------------------------------------- tile math ----
//
// Lane (g, t) of the MMA: A rows g and g + 8 are weight rows, B column g is
// sequence g, and the lane's four k slots (2t, 2t + 1, 2t + 8, 2t + 9) carry
// four consecutive elements of the block - the four bytes of one quant word
// it reads - so B lane (g, t) holds quad e4 of sequence g, hi part for one MMA
// and lo part for the other. Accumulator lane (g, t) ends with rows g, g + 8
// x sequences 2t, 2t + 1.

__device__ __forceinline__ uint32_t hfma2u(uint32_t a, uint32_t b, uint32_t c)
{
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ uint32_t hmul2u(uint32_t a, uint32_t b)
{
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t hsub2u(uint32_t a, uint32_t b)
{
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ void mma1688(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t b, const float (&c)[4])
{
    asm("mma.sync.aligned.m16n8k8.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%8,%9,%10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(b), "f"(c[0]), "f"(c[1]), "f"(c[2]), "f"(c[3]));
}

// Q4_K (dequant_q4_k, src/brain_runtime.c:960-1015): chunk c of 64 elements is
// 32 quant bytes; lane t reads bytes 8t .. 8t + 7 (word s: elements
// 64c + 32 hn + 8t + 4s + 0..3, hn = low / high nibble). A holds sc_j q: the
// quant byte under an exponent byte is the binary16 1024 + q (low nibble) or
// 1024 + 16 q (high nibble in place), and one fused multiply-add per pair,
// (1024 + q) sc - 1024 sc or (1024 + 16 q) sc / 16 - 64 sc, gives q sc exactly
// (q sc <= 945). So the 16 k steps of the task sum into one accumulator
// (hi and lo parts of x: two), scaled once by d; the min term
// dmin sum_j m_j sum(x over sub-block j) is one m16n8k8 MMA pair of the m_j
// (binary16 subnormals) against the staged 32-element sums.
__device__ __forceinline__ void q4k_task8(const uint8_t *r0, const uint8_t *r1, const uint4 *xq, const uint2 *xm,
                                          uint32_t lane, float (&acc)[4])
{
    const uint32_t g = lane >> 2, t = lane & 3u;
    const uint4 h0 = *reinterpret_cast<const uint4 *>(r0), h1 = *reinterpret_cast<const uint4 *>(r1);
    // get_scale_min_k4 (src/brain_runtime.c:939-958) for the 8 sub-blocks, four per word
    const uint32_t sl0 = h0.y & 0x3f3f3f3fu, ml0 = h0.z & 0x3f3f3f3fu;
    const uint32_t sh0 = (h0.w & 0x0f0f0f0fu) | ((h0.y >> 2) & 0x30303030u);
    const uint32_t mh0 = ((h0.w >> 4) & 0x0f0f0f0fu) | ((h0.z >> 2) & 0x30303030u);
    const uint32_t sl1 = h1.y & 0x3f3f3f3fu, ml1 = h1.z & 0x3f3f3f3fu;
    const uint32_t sh1 = (h1.w & 0x0f0f0f0fu) | ((h1.y >> 2) & 0x30303030u);
    const uint32_t mh1 = ((h1.w >> 4) & 0x0f0f0f0fu) | ((h1.z >> 2) & 0x30303030u);
    float ca[4] = {0.f, 0.f, 0.f, 0.f}, cb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (uint32_t c = 0; c < 4u; ++c) {
        const uint2 w0 = *reinterpret_cast<const uint2 *>(r0 + 16u + 32u * c + 8u * t);
        const uint2 w1 = *reinterpret_cast<const uint2 *>(r1 + 16u + 32u * c + 8u * t);
#pragma unroll
        for (uint32_t hn = 0; hn < 2u; ++hn) {
            const uint32_t j = 2u * c + hn, jb = j & 3u;
            const uint32_t sel = jb | 0x40u | (jb << 8) | 0x4000u;   // (byte jb, 0x64) twice
            // (sc, sc) in binary16: (1024 + sc) - 1024
            const uint32_t s0 = hsub2u(__byte_perm(j < 4u ? sl0 : sh0, 0x64u, sel), 0x64006400u);
            const uint32_t s1 = hsub2u(__byte_perm(j < 4u ? sl1 : sh1, 0x64u, sel), 0x64006400u);
            const uint32_t mul0 = hn ? hmul2u(s0, 0x2c002c00u) : s0, mul1 = hn ? hmul2u(s1, 0x2c002c00u) : s1;
            const uint32_t add0 = hmul2u(s0, hn ? 0xd400d400u : 0xe400e400u);   // -64 sc or -1024 sc
            const uint32_t add1 = hmul2u(s1, hn ? 0xd400d400u : 0xe400e400u);
#pragma unroll
            for (uint32_t s = 0; s < 2u; ++s) {
                const uint32_t m = hn ? 0xf0f0f0f0u : 0x0f0f0f0fu;
                const uint32_t v0 = (s ? w0.y : w0.x) & m, v1 = (s ? w1.y : w1.x) & m;
                const uint32_t e4 = 16u * c + 8u * hn + 2u * t + s;
                const uint4 xv = xq[e4 * kMaxSeq + xcol(e4, g, true)];
                const uint32_t a0 = hfma2u(__byte_perm(v0, 0x64u, 0x4140), mul0, add0);
                const uint32_t a1 = hfma2u(__byte_perm(v1, 0x64u, 0x4140), mul1, add1);
                const uint32_t a2 = hfma2u(__byte_perm(v0, 0x64u, 0x4342), mul0, add0);
                const uint32_t a3 = hfma2u(__byte_perm(v1, 0x64u, 0x4342), mul1, add1);
                const float pa[4] = {ca[0], ca[1], ca[2], ca[3]}, pb[4] = {cb[0], cb[1], cb[2], cb[3]};
                mma16816(ca, a0, a1, a2, a3, make_uint2(xv.x, xv.y), pa);
                mma16816(cb, a0, a1, a2, a3, make_uint2(xv.z, xv.w), pb);
            }
        }
    }
    // min term: A = m_{2t}, m_{2t+1} of rows g, g + 8 as binary16 subnormals m 2^-24
    const uint32_t msel = (t & 1u) ? 0x4342u : 0x4140u;
    const uint32_t am0 = __byte_perm(t < 2u ? ml0 : mh0, 0u, msel), am1 = __byte_perm(t < 2u ? ml1 : mh1, 0u, msel);
    const uint2 xb = xm[g * 4u + t];
    const float zero[4] = {0.f, 0.f, 0.f, 0.f};
    float cm[4], cm2[4];
    mma1688(cm, am0, am1, xb.x, zero);
    mma1688(cm2, am0, am1, xb.y, cm);
    const float d0 = h2f((uint16_t)(h0.x & 0xffffu)), dm0 = h2f((uint16_t)(h0.x >> 16)) * 1073741824.0f;
    const float d1 = h2f((uint16_t)(h1.x & 0xffffu)), dm1 = h2f((uint16_t)(h1.x >> 16)) * 1073741824.0f;
    acc[0] = fmaf(-dm0, cm2[0], fmaf(d0, ca[0] + cb[0], acc[0]));
    acc[1] = fmaf(-dm0, cm2[1], fmaf(d0, ca[1] + cb[1], acc[1]));
    acc[2] = fmaf(-dm1, cm2[2], fmaf(d1, ca[2] + cb[2], acc[2]));
    acc[3] = fmaf(-dm1, cm2[3], fmaf(d1, ca[3] + cb[3], acc[3]));
}

// Q6_K (dequant_q6_k, src/brain_runtime.c:1049-1083), the block at a 2-byte
// aligned address: element 128h + 32k + l has ql[64h + 32(k & 1) + l] (nibble
// k >> 1), qh[32h + l] bits 2k..2k+1 and scale 8h + 2k + l / 16. The k step
// (h, l16, k) is one 16-element scale group; lane t takes l = 16 l16 + 4t ..
// + 3, one word of ql and one of qh. q - 32 is applied through the group's
// sum of x.
__device__ __forceinline__ void q6k_task8(const uint8_t *r0, const uint8_t *r1, const uint4 *xq, const float *xs,
                                          uint32_t lane, float (&acc)[4])
{
    const uint32_t g = lane >> 2, t = lane & 3u;
    const float d0 = h2f(*reinterpret_cast<const uint16_t *>(r0 + 208)) * kTwo24;
    const float d1 = h2f(*reinterpret_cast<const uint16_t *>(r1 + 208)) * kTwo24;
#pragma unroll
    for (uint32_t h = 0; h < 2u; ++h) {
#pragma unroll
        for (uint32_t l16 = 0; l16 < 2u; ++l16) {
            const uint32_t ol = 64u * h + 16u * l16 + 4u * t, oh = 128u + 32u * h + 16u * l16 + 4u * t;
            const uint32_t qa0 = ldw2(r0 + ol), qb0 = ldw2(r0 + ol + 32u), qh0 = ldw2(r0 + oh);
            const uint32_t qa1 = ldw2(r1 + ol), qb1 = ldw2(r1 + ol + 32u), qh1 = ldw2(r1 + oh);
#pragma unroll
            for (uint32_t k = 0; k < 4u; ++k) {
                const uint32_t lo0 = (k & 1u) ? qb0 : qa0, lo1 = (k & 1u) ? qb1 : qa1;
                const uint32_t ns = 4u * (k >> 1);
                const uint32_t v0 = ((lo0 >> ns) & 0x0f0f0f0fu) | (((qh0 >> (2u * k)) & 0x03030303u) << 4);
                const uint32_t v1 = ((lo1 >> ns) & 0x0f0f0f0fu) | (((qh1 >> (2u * k)) & 0x03030303u) << 4);
                const uint32_t e4 = 32u * h + 8u * k + 4u * l16 + t;
                const uint4 xv = xq[e4 * kMaxSeq + xcol(e4, g, false)];
                const uint32_t a0 = sub2(v0, 0x4140), a1 = sub2(v1, 0x4140), a2 = sub2(v0, 0x4342), a3 = sub2(v1, 0x4342);
                const float zero[4] = {0.f, 0.f, 0.f, 0.f};
                float cp[4], cs[4];   // x hi, then + x lo in the same accumulator
                mma16816(cp, a0, a1, a2, a3, make_uint2(xv.x, xv.y), zero);
                mma16816(cs, a0, a1, a2, a3, make_uint2(xv.z, xv.w), cp);
                const uint32_t G = 8u * h + 2u * k + l16;
                const float S0 = d0 * s8f(r0[192u + G]), S1 = d1 * s8f(r1[192u + G]);
                const float2 x2 = *reinterpret_cast<const float2 *>(xs + G * kMaxSeq + 2u * t);
                const float o0 = 32.0f * x2.x * (1.0f / kTwo24), o1 = 32.0f * x2.y * (1.0f / kTwo24);
                acc[0] = fmaf(S0, cs[0] - o0, acc[0]);
                acc[1] = fmaf(S0, cs[1] - o1, acc[1]);
                acc[2] = fmaf(S1, cs[2] - o0, acc[2]);
                acc[3] = fmaf(S1, cs[3] - o1, acc[3]);
            }
        }
    }
}

// ------------------------------------------------------- copies, flush ----

// One task's copies into a slot (16 rows x one block): Q4_K rows as their
// 144-byte blocks (9 chunks of 16 bytes per row, 5 per lane), Q6_K rows as the
// 224-byte window from the 16-byte boundary at or below the 2-byte-aligned
// block (14 chunks, 7 per lane). Offsets come from the CTA's table.
template <bool Q4>
__device__ __forceinline__ void issue(const uint8_t *base, const BHdr *h, uint32_t slot, uint32_t lane, uint64_t policy)
{
#pragma unroll
    for (uint32_t i = 0; i < (Q4 ? 5u : 7u); ++i) {
        const uint2 e = h->cp[i][lane];
        if (Q4) {
            if (i < 4u || lane < 16u) cpa16(slot + e.y, base + e.x, policy);
        } else {
            const uint8_t *win = reinterpret_cast<const uint8_t *>(reinterpret_cast<uintptr_t>(base + e.x) & ~uintptr_t(15));
            cpa16(slot + e.y, win + e.y % kQ6Row, policy);
        }
    }
}

// Tile t (16 rows) finished by this warp's tasks: alone, or as one of warps
// wa..wb (partials in shared memory, the last to arrive adds them in warp
// order). acc: rows g, g + 8 x sequences 2t, 2t + 1, already unscaled.
__device__ __forceinline__ void flush(const BArgs &a, const BCta &c, BHdr *h, float *pslot, uint32_t t, uint32_t tj0,
                                      uint32_t wa, uint32_t wb, uint32_t my0, const float (&acc)[4])
{
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u, g = lane >> 2, q = lane & 3u;
    const uint32_t r[4] = {g, g, g + 8u, g + 8u}, s[4] = {2u * q, 2u * q + 1u, 2u * q, 2u * q + 1u};
    float v[4] = {acc[0], acc[1], acc[2], acc[3]};
    if (wa != wb) {
        const uint32_t which = my0 >= tj0 ? 0u : 1u;
        float *pp = pslot + (warp * 2u + which) * 128u;
#pragma unroll
        for (int i = 0; i < 4; ++i) pp[r[i] * kMaxSeq + s[i]] = v[i];
        __syncwarp();
        uint32_t last = 0;
        if (lane == 0) {
            __threadfence_block();
            last = (atomicAdd(&h->cnt[wa], 1u) + 1u == wb - wa + 1u) ? 1u : 0u;
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (!last) return;
        __threadfence_block();
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = 0.f;
        for (uint32_t w = wa; w <= wb; ++w) {
            const uint32_t ww = (w > wa || h->wstart[wa] >= tj0) ? 0u : 1u;
            const volatile float *qq = pslot + (w * 2u + ww) * 128u;
#pragma unroll
            for (int i = 0; i < 4; ++i) v[i] += qq[r[i] * kMaxSeq + s[i]];
        }
    }
    const BSeg &sg = a.seg[c.seg];
#pragma unroll
    for (int i = 0; i < 4; ++i)
        if (s[i] < a.nseq)
            a.part[((size_t)c.split * a.nseq + s[i]) * a.prows + sg.prow0 + 16u * t + r[i]] = v[i];
}

template <int NS, bool Q4>
__device__ void consume(const BArgs &a, const BCta &c, BHdr *h, float *pslot, uint4 *xq, float *xs, uint2 *xm,
                        uint8_t *ring)
{
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u, g = lane >> 2, q = lane & 3u;
    const BSeg &sg = a.seg[c.seg];
    const uint32_t b0 = c.split * a.split_blocks, nbs = min(a.split_blocks, a.nb - b0);
    const uint32_t L = (c.t1 - c.t0) * nbs, weff = min(kBWarps, L);
    const bool active = warp < weff;
    const uint32_t my0 = active ? h->wstart[warp] : 0u;
    const uint32_t my1 = active ? (warp + 1u < weff ? h->wstart[warp + 1u] : L) : 0u;
    const uint32_t n = my1 - my0;
    const uint32_t rb = (uint32_t)sg.row_bytes, bb = Q4 ? 144u : 210u;
    // task j of the CTA: tile t0 + j / nbs, block b0 + j % nbs
    uint32_t it = my0 / nbs, ib = my0 - it * nbs;   // issue cursor
    uint32_t ct = it, cb = ib;                      // consume cursor
    const uint64_t policy = policy_evict_first();
    const uint32_t ring_w = smem_addr(ring) + warp * (uint32_t)NS * a.slot_bytes;
    auto blk = [&](uint32_t tt, uint32_t b) {
        return sg.w + (uint64_t)(16u * (c.t0 + tt)) * rb + (uint64_t)(b0 + b) * bb;
    };
#pragma unroll
    for (uint32_t k = 0; k + 1u < (uint32_t)NS; ++k) {
        if (k < n) {
            issue<Q4>(blk(it, ib), h, ring_w + k * a.slot_bytes, lane, policy);
            if (++ib == nbs) { ib = 0u; ++it; }
        }
        cpa_commit();
    }
    if (a.pdl) pdl_wait();
    stage_x(a, h, xq, xs, xm, b0, nbs, Q4);
    if (!active) return;
    auto warp_of = [&](uint32_t j) { return ((j + 1u) * weff + L - 1u) / L - 1u; };
    const uint32_t first = my0 / nbs, lastt = (my1 - 1u) / nbs;
    const uint32_t fa = warp_of(first * nbs), fb = warp_of(first * nbs + nbs - 1u);
    const uint32_t la = warp_of(lastt * nbs), lb = warp_of(lastt * nbs + nbs - 1u);
    const uint8_t *ringp = ring + (size_t)warp * NS * a.slot_bytes;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    uint32_t si = 0, sn = (uint32_t)NS - 1u;
    for (uint32_t k = 0; k < n; ++k) {
        if (k + (uint32_t)NS - 1u < n) {
            issue<Q4>(blk(it, ib), h, ring_w + sn * a.slot_bytes, lane, policy);
            if (++ib == nbs) { ib = 0u; ++it; }
        }
        cpa_commit();
        if (++sn == (uint32_t)NS) sn = 0u;
        cpa_wait<NS - 1>();
        __syncwarp();
        const uint8_t *slot = ringp + si * a.slot_bytes;
        if (++si == (uint32_t)NS) si = 0u;
        const uint4 *xqb = xq + (size_t)cb * 64u * kMaxSeq;
        const float *xsb = xs + cb * 16u * kMaxSeq;
        if (Q4) {
            q4k_task8(slot + g * kQ4Row, slot + (g + 8u) * kQ4Row, xqb, xm + cb * 32u, lane, acc);
        } else {
            // the block's offset inside its 16-byte-aligned window, per row
            const uintptr_t blk0 = reinterpret_cast<uintptr_t>(blk(ct, cb));
            q6k_task8(slot + g * kQ6Row + ((blk0 + g * rb) & 15u), slot + (g + 8u) * kQ6Row + ((blk0 + (g + 8u) * rb) & 15u),
                      xqb, xsb, lane, acc);
        }
        __syncwarp();   // the slot is refilled by a later iteration's copies
        const uint32_t t = ct;
        if (++cb == nbs) { cb = 0u; ++ct; }
        if (ct != t || k + 1u == n) {
            const uint32_t wa = t == first ? fa : (t == lastt ? la : warp);
            const uint32_t wb = t == first ? fb : (t == lastt ? lb : warp);
            float v[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) v[i] = acc[i] * h->sinv[2u * q + (uint32_t)(i & 1)];
            flush(a, c, h, pslot, c.t0 + t, t * nbs, wa, wb, my0, v);
            acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
        }
    }
}

template <int NS>
__global__ void __launch_bounds__(kBThreads, 1) mvb_kernel(const __grid_constant__ BArgs a)
{
    extern __shared__ __align__(128) uint8_t smem[];
    BHdr *h = reinterpret_cast<BHdr *>(smem);
    float *pslot = reinterpret_cast<float *>(smem + hdr_bytes());
    const uint32_t sb = a.split_blocks;
    uint4 *xq = reinterpret_cast<uint4 *>(smem + hdr_bytes() + kPartBytes);
    float *xs = reinterpret_cast<float *>(smem + hdr_bytes() + kPartBytes + xq_bytes(sb));
    uint2 *xm = reinterpret_cast<uint2 *>(smem + hdr_bytes() + kPartBytes + xq_bytes(sb) + xs_bytes(sb));
    uint8_t *ring = smem + hdr_bytes() + kPartBytes + xq_bytes(sb) + xs_bytes(sb) + xm_bytes(sb);
    const BCta c = a.cta[blockIdx.x];
    const BSeg &sg = a.seg[c.seg];
    const bool q4 = sg.type == 12u;
    {
        const uint32_t b0 = c.split * a.split_blocks, nbs = min(a.split_blocks, a.nb - b0);
        const uint32_t L = (c.t1 - c.t0) * nbs, weff = min(kBWarps, L);
        if (threadIdx.x < kBWarps) {
            h->cnt[threadIdx.x] = 0u;
            h->wstart[threadIdx.x] = threadIdx.x < weff ? threadIdx.x * L / weff : 0xffffffffu;
        }
        if (threadIdx.x < kMaxSeq) h->smax[threadIdx.x] = 0u;
        const uint32_t rb = (uint32_t)sg.row_bytes;
        for (uint32_t e = threadIdx.x; e < 8u * 32u; e += blockDim.x) {
            const uint32_t i = e >> 5, l = e & 31u, idx = l + 32u * i;
            uint2 v = make_uint2(0u, 0u);
            if (q4 && idx < 144u) {
                const uint32_t r = idx / 9u, p = idx - 9u * r;
                v = make_uint2(r * rb + 16u * p, r * kQ4Row + 16u * p);
            } else if (!q4 && idx < 224u) {
                const uint32_t r = idx / 14u, p = idx - 14u * r;
                v = make_uint2(r * rb, r * kQ6Row + 16u * p);
            }
            h->cp[i][l] = v;
        }
    }
    __syncthreads();
    pdl_launch();
    if (q4) consume<NS, true>(a, c, h, pslot, xq, xs, xm, ring);
    else consume<NS, false>(a, c, h, pslot, xq, xs, xm, ring);
    cpa_wait<0>();   // no copy may still target this CTA's shared memory when it exits
}

// ------------------------------------------------------ reduce kernels ----

// Sum of squares of the 256 values v of a CTA (one per thread), in double, by
// a fixed tree.
__device__ __forceinline__ double block_ssq(float v, double *red)
{
    double ss = (double)v * (double)v;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31u) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    double t = 0.0;
    if (threadIdx.x == 0)
        for (int w = 0; w < 8; ++w) t += red[w];
    return t;
}

__device__ __forceinline__ float rms_factor(const double *ssq, uint32_t n, uint32_t s, uint32_t hidden, float eps)
{
    if (!ssq) return 1.0f;
    double t = 0.0;
    for (uint32_t i = 0; i < n; ++i) t += ssq[s * n + i];
    return 1.0f / sqrtf((float)(t / (double)hidden) + eps);
}

// Partial rows -> outputs: thread = (row, sequence blockIdx.y); slices are
// added in slice order.
__global__ void __launch_bounds__(256) reduce_kernel(const __grid_constant__ BReduce a)
{
    __shared__ float bv[8];
    __shared__ uint32_t bi[8];
    pdl_launch();
    if (a.pdl) pdl_wait();
    const uint32_t s = blockIdx.y, r = blockIdx.x * kRowChunk + threadIdx.x;
    const float inv = rms_factor(a.ssq, a.nssq, s, a.hidden, a.eps);
    float v = -FLT_MAX;
    if (r < a.rows) {
        float x = 0.f, u = 0.f;
        for (uint32_t k = 0; k < a.nsplit; ++k) {
            const float *p = a.part + ((size_t)k * a.nseq + s) * a.prows;
            x += __ldcg(p + r);
            if (a.mode == BRED_SWIGLU) u += __ldcg(p + a.rows + r);
        }
        x *= inv;
        if (a.mode == BRED_SWIGLU) {
            u *= inv;
            x = (x / (1.0f + expf(-x))) * u;   // src/brain_runtime.c:1755-1758
        } else if (a.bias) {
            x += a.bias[r];
        }
        a.out[(size_t)s * a.ostride + r] = x;
        v = x;
    }
    if (a.mode != BRED_LOGITS) return;
    float best = v;
    uint32_t idx = r < a.rows ? r : 0xffffffffu;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (ov > best || (ov == best && oi < idx)) { best = ov; idx = oi; }
    }
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    if (lane == 0) { bv[warp] = best; bi[warp] = idx; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < 8; ++w)
            if (bv[w] > best || (bv[w] == best && bi[w] < idx)) { best = bv[w]; idx = bi[w]; }
        a.pmax[s * gridDim.x + blockIdx.x] = best;
        a.pidx[s * gridDim.x + blockIdx.x] = idx;
    }
}

// Residual add (src/brain_runtime.c:1745, :1762): thread = (row, sequence
// blockIdx.y); the chunk's sum of squares for the next rms_norm.
__global__ void __launch_bounds__(256) resid_kernel(const __grid_constant__ BResid a)
{
    __shared__ double red[8];
    pdl_launch();
    if (a.pdl) pdl_wait();
    const uint32_t s = blockIdx.y, r = blockIdx.x * kRowChunk + threadIdx.x;
    float v = 0.f;
    if (r < a.hidden) {
        float *x = a.x + (size_t)s * a.hidden;
        v = x[r];
        for (uint32_t k = 0; k < a.nsplit; ++k) v += __ldcg(a.part + ((size_t)k * a.nseq + s) * a.prows + r);
        x[r] = v;
    }
    const double t = block_ssq(v, red);
    if (threadIdx.x == 0) a.ssq[s * gridDim.x + blockIdx.x] = t;
}

// Token rows of every sequence (bit-exact dequantization): thread = (element,
// sequence blockIdx.y), and the chunk's sum of squares.
__global__ void __launch_bounds__(256) embedb_kernel(const uint8_t *embd, uint64_t row_bytes, uint32_t type,
                                                     uint32_t hidden, uint32_t vocab, float *x, double *ssq,
                                                     d2::DecState *st)
{
    __shared__ double red[8];
    pdl_launch();
    const uint32_t s = blockIdx.y, i = blockIdx.x * kRowChunk + threadIdx.x;
    const uint32_t token = *reinterpret_cast<volatile const uint32_t *>(&st[s].token);
    if (token >= vocab) {
        if (blockIdx.x == 0 && threadIdx.x == 0) atomicCAS(&st[s].status, kStatusOk, kStatusBadArgument);
        return;
    }
    const uint32_t be = block_elems(type), bbytes = block_bytes(type);
    float v = 0.f;
    if (i < hidden) {
        v = deq_elem(type, embd + (uint64_t)token * row_bytes + (i / be) * bbytes, (int)(i % be));
        x[(size_t)s * hidden + i] = v;
    }
    const double t = block_ssq(v, red);
    if (threadIdx.x == 0) ssq[s * gridDim.x + blockIdx.x] = t;
}

// Greedy pick of sequence blockIdx.x over the reduce's per-CTA (max, row)
// pairs (lowest row among equal maxima, atlas_sample_token's greedy branch,
// src/brain_runtime.c:1783); then the sequence's state advances.
__global__ void __launch_bounds__(256) argmaxb_kernel(const float *pmax, const uint32_t *pidx, uint32_t n,
                                                      d2::DecState *st)
{
    __shared__ float bv[8];
    __shared__ uint32_t bi[8];
    pdl_launch();
    pdl_wait();
    const uint32_t s = blockIdx.x;
    float best = -FLT_MAX;
    uint32_t idx = 0xffffffffu;
    for (uint32_t i = threadIdx.x; i < n; i += 256u) {
        const float v = __ldcg(pmax + s * n + i);
        const uint32_t k = __ldcg(pidx + s * n + i);
        if (v > best || (v == best && k < idx)) { best = v; idx = k; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (ov > best || (ov == best && oi < idx)) { best = ov; idx = oi; }
    }
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    if (lane == 0) { bv[warp] = best; bi[warp] = idx; }
    __syncthreads();
    if (threadIdx.x != 0) return;
    for (int w = 1; w < 8; ++w)
        if (bv[w] > best || (bv[w] == best && bi[w] < idx)) { best = bv[w]; idx = bi[w]; }
    d2::DecState &d = st[s];
    d.next_token = idx;
    d.next_logit = best;
    if (d.out_ids && d.step < d.max_steps) d.out_ids[d.step] = idx;
    if (d.advance) {
        d.token = idx;
        d.pos = d.pos + 1u;
        d.step = d.step + 1u;
    }
    d.epoch = d.epoch + 1u;
}

cudaError_t launch_ex(const void *fn, void **args, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

const void *mvb_fn(uint32_t nslot)
{
    switch (nslot) {
    case 2: return (const void *)mvb_kernel<2>;
    case 3: return (const void *)mvb_kernel<3>;
    case 4: return (const void *)mvb_kernel<4>;
    default: return nullptr;
    }
}

}  // namespace

size_t mvb_smem(uint32_t split_blocks, uint32_t nslot, uint32_t slot_bytes)
{
    return smem_total(split_blocks, nslot, slot_bytes);
}

}  // namespace bt
}  // namespace atlas

using namespace atlas;
using namespace atlas::bt;

extern "C" cudaError_t atlas_bt_setup(size_t smem)
{
    for (uint32_t ns = 2; ns <= kBMaxSlots; ++ns) {
        const cudaError_t e = cudaFuncSetAttribute(mvb_fn(ns), cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

extern "C" cudaError_t atlas_bt_launch_mv(const BArgs *a, uint32_t grid, cudaStream_t stream)
{
    const void *fn = mvb_fn(a->nslot);
    if (!fn || a->nseq == 0u || a->nseq > kMaxSeq) return cudaErrorInvalidValue;
    BArgs copy = *a;
    void *args[] = {&copy};
    return launch_ex(fn, args, dim3(grid), dim3(kBThreads), a->smem_bytes, stream, a->pdl != 0u);
}

// grid: row chunks of kRowChunk (BRED_LOGITS: the pmax / pidx columns per sequence)
extern "C" cudaError_t atlas_bt_launch_reduce(const BReduce *a, uint32_t grid, cudaStream_t stream)
{
    if (grid * kRowChunk < a->rows) return cudaErrorInvalidValue;
    BReduce copy = *a;
    void *args[] = {&copy};
    return launch_ex((const void *)reduce_kernel, args, dim3(grid, a->nseq), dim3(kRowChunk), 0, stream,
                     a->pdl != 0u);
}

extern "C" cudaError_t atlas_bt_launch_resid(const BResid *a, cudaStream_t stream)
{
    BResid copy = *a;
    void *args[] = {&copy};
    return launch_ex((const void *)resid_kernel, args, dim3((a->hidden + kRowChunk - 1u) / kRowChunk, a->nseq),
                     dim3(kRowChunk), 0, stream, a->pdl != 0u);
}

extern "C" cudaError_t atlas_bt_launch_embed(const uint8_t *embd, uint64_t row_bytes, uint32_t type, uint32_t hidden,
                                             uint32_t vocab, float *x, double *ssq, d2::DecState *st, uint32_t nseq,
                                             cudaStream_t stream)
{
    void *args[] = {&embd, &row_bytes, &type, &hidden, &vocab, &x, &ssq, &st};
    return launch_ex((const void *)embedb_kernel, args, dim3((hidden + kRowChunk - 1u) / kRowChunk, nseq),
                     dim3(kRowChunk), 0, stream, false);
}

extern "C" cudaError_t atlas_bt_launch_argmax(const float *pmax, const uint32_t *pidx, uint32_t n, d2::DecState *st,
                                              uint32_t nseq, cudaStream_t stream)
{
    void *args[] = {&pmax, &pidx, &n, &st};
    return launch_ex((const void *)argmaxb_kernel, args, dim3(nseq), dim3(256), 0, stream, true);
}
