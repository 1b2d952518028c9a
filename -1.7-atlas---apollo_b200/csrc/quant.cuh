// Q4_K / Q6_K (and the reference's other block types) on the device.
//
// Two families of functions:
//  * deq_*_elem: bit-exact dequantization of one element, the reference's
//    arithmetic (src/brain_runtime.c:960-1121) with every product and
//    difference rounded separately (__fmul_rn / __fsub_rn: no FMA contraction).
//  * *_slice_dot: the decode GEMV inner loop over one 32-element "slice" of a
//    super-block, operating on raw bytes already staged in shared memory.
//
// GEMV slice geometry (shared by Q4_K and Q6_K so that one set of x registers
// serves both): slice s of a row = 8*b + 2*c + hf covers, inside block b,
//   lo group: elements 64c + 16hf + l,       l = 0..15
//   hi group: elements 64c + 32 + 16hf + l,  l = 0..15
// Q4_K (src/brain_runtime.c:960-1015): qs bytes 32c + 16hf + l give the lo
//   (low nibble, scale/min pair 2c) and hi (high nibble, pair 2c+1) values.
// Q6_K (src/brain_runtime.c:1049-1083) with half h = c/2, kk = c%2: element
//   128h + 32k + l' comes from ql[64h + l'] (k = 0, 2) / ql[64h + 32 + l']
//   (k = 1, 3) and qh[32h + l'] bits 2k..2k+1; with l' = 16hf + l the lo group
//   is k = 2kk and the hi group k = 2kk + 1, scale index 8h + hf + 2k.
//
// Values are turned into floats without an int->float conversion: a byte q
// (0..63) placed in bits 16..23 under exponent byte 0x43 is the float 128 + q.
// So a group's dot is  sum (128 + q) x - C * sum x  with C = 128 (Q4_K) or 160
// (Q6_K, folding the -32 offset); sum x per group is precomputed with x.
// The products accumulate in fp32 pairs (FFMA2) and the result stays within a
// few fp32 ulps of the reference's sum of fp32(w) * x.
#pragma once
#include "common.cuh"

namespace atlas {

// ------------------------------------------------------- bit-exact dequant --

// binary16 -> binary32 with integer operations only (NaN payloads and signed
// zeros exactly as the reference's half_to_float, src/brain_runtime.c:203-247).
__device__ __forceinline__ float h2f_exact(uint32_t h)
{
    const uint32_t sign = (h & 0x8000u) << 16, e = (h >> 10) & 31u;
    uint32_t m = h & 1023u, bits;
    if (e == 31u) {
        bits = sign | 0x7f800000u | (m << 13);
    } else if (e != 0u) {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    } else if (m == 0u) {
        bits = sign;
    } else {
        const uint32_t shift = (uint32_t)__clz((int)m) - 21u;  // bring bit 10 up
        m <<= shift;
        bits = sign | ((113u - shift) << 23) | ((m & 1023u) << 13);
    }
    return __uint_as_float(bits);
}

__device__ __forceinline__ uint32_t ld_u16(const uint8_t *p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8); }

// get_scale_min_k4 (src/brain_runtime.c:939-958) over the 12 packed bytes.
__device__ __forceinline__ void k4_scale_min(int j, const uint8_t *p, uint32_t &sc, uint32_t &mn)
{
    if (j < 4) {
        sc = p[j] & 63u;
        mn = p[j + 4] & 63u;
    } else {
        sc = (p[j + 4] & 15u) | ((uint32_t)(p[j - 4] >> 6) << 4);
        mn = (p[j + 4] >> 4) | ((uint32_t)(p[j] >> 6) << 4);
    }
}

__device__ __forceinline__ float deq_q4k_elem(const uint8_t *b, int i)
{
    const int c = i >> 6, within = i & 63, hi = within >> 5, l = within & 31;
    uint32_t sc, mn;
    k4_scale_min(2 * c + hi, b + 4, sc, mn);
    const float d = h2f_exact(ld_u16(b)), dmin = h2f_exact(ld_u16(b + 2));
    const uint32_t byte = b[16 + 32 * c + l];
    const uint32_t q = hi ? (byte >> 4) : (byte & 15u);
    const float scale = __fmul_rn(d, (float)sc), minv = __fmul_rn(dmin, (float)mn);
    return __fsub_rn(__fmul_rn(scale, (float)q), minv);
}

// Q5_K as the reference decodes it (src/brain_runtime.c:1017-1043), including
// its qh pointer advancing 8 bytes per 64-value chunk.
__device__ __forceinline__ float deq_q5k_elem(const uint8_t *b, int i)
{
    const int c = i >> 6, within = i & 63, hi = within >> 5, l = within & 31;
    uint32_t sc, mn;
    k4_scale_min(2 * c + hi, b + 4, sc, mn);
    const float d = h2f_exact(ld_u16(b)), dmin = h2f_exact(ld_u16(b + 2));
    const uint32_t qb = b[48 + 32 * c + l], hb = b[16 + 8 * c + l];
    const uint32_t q = (hi ? (qb >> 4) : (qb & 15u)) + ((hb >> (2 * c + hi)) & 1u ? 16u : 0u);
    const float scale = __fmul_rn(d, (float)sc), minv = __fmul_rn(dmin, (float)mn);
    return __fsub_rn(__fmul_rn(scale, (float)q), minv);
}

__device__ __forceinline__ float deq_q6k_elem(const uint8_t *b, int i)
{
    const int h = i >> 7, p = i & 127, k = p >> 5, l = p & 31;
    const uint32_t lo = b[64 * h + 32 * (k & 1) + l];
    const uint32_t hb = b[128 + 32 * h + l];
    const uint32_t q = ((k & 2) ? (lo >> 4) : (lo & 15u)) | (((hb >> (2 * k)) & 3u) << 4);
    const int sc = (int)(int8_t)b[192 + 8 * h + (l >> 4) + 2 * k];
    const float d = h2f_exact(ld_u16(b + 208));
    return __fmul_rn(__fmul_rn(d, (float)sc), (float)((int)q - 32));
}

// dequant_block's 32-element types and F16 (src/brain_runtime.c:1085-1121).
__device__ __forceinline__ float deq_small_elem(uint32_t type, const uint8_t *b, int i)
{
    const float d = h2f_exact(ld_u16(b));
    if (type == 1u) return d;                                        // F16
    if (type == 8u) return __fmul_rn(d, (float)(int8_t)b[2 + i]);    // Q8_0
    const bool q50 = type == 6u;
    const uint8_t *hp = b + (q50 ? 2 : 4), *nib = b + (q50 ? 6 : 8);
    const uint32_t high = (uint32_t)hp[0] | ((uint32_t)hp[1] << 8) | ((uint32_t)hp[2] << 16) | ((uint32_t)hp[3] << 24);
    uint32_t q = i < 16 ? (nib[i & 15] & 15u) : (nib[i & 15] >> 4);
    q |= ((high >> i) & 1u) << 4;
    if (q50) return __fmul_rn(d, __fsub_rn((float)q, 16.0f));
    return __fadd_rn(__fmul_rn(d, (float)q), h2f_exact(ld_u16(b + 2)));   // Q5_1
}

__host__ __device__ constexpr uint32_t block_bytes(uint32_t type)
{
    return type == 1u ? 2u : type == 6u ? 22u : type == 7u ? 24u : type == 8u ? 34u :
           type == 12u ? 144u : type == 13u ? 176u : type == 14u ? 210u : 0u;
}

__host__ __device__ constexpr uint32_t block_elems(uint32_t type)
{
    return type == 1u ? 1u : (type == 6u || type == 7u || type == 8u) ? 32u :
           (type == 12u || type == 13u || type == 14u) ? 256u : 0u;
}

__device__ __forceinline__ float deq_elem(uint32_t type, const uint8_t *b, int i)
{
    switch (type) {
    case 12u: return deq_q4k_elem(b, i);
    case 13u: return deq_q5k_elem(b, i);
    case 14u: return deq_q6k_elem(b, i);
    default: return deq_small_elem(type, b, i);
    }
}

// --------------------------------------------------------- GEMV slices -----

// float(128 + byte k of v) for bytes 0..63: byte k moved to bits 16..23, 0x43
// into bits 24..31, zeros below.
__device__ __forceinline__ float byte_as_float_128(uint32_t v, int k)
{
    return __uint_as_float(__byte_perm(v, 0x43u, 0x4055u | ((uint32_t)k << 8)));
}

// acc += (128 + q) * x for the 4 bytes of v against x pair values xa, xb.
__device__ __forceinline__ void fma_word(uint32_t v, float2 xa, float2 xb, float2 &acc)
{
    const float2 w0 = make_float2(byte_as_float_128(v, 0), byte_as_float_128(v, 1));
    const float2 w1 = make_float2(byte_as_float_128(v, 2), byte_as_float_128(v, 3));
    acc = __ffma2_rn(w0, xa, acc);
    acc = __ffma2_rn(w1, xb, acc);
}

struct SliceX {
    float2 lo[8], hi[8];  // x for the lo / hi group, consecutive pairs
    float slo, shi;       // sum of the lo / hi group
};

// One Q4_K slice (block bytes at `blk`, 16-byte aligned in shared memory).
__device__ __forceinline__ float q4k_slice_dot(const uint8_t *blk, int c, int hf, const SliceX &x)
{
    const uint4 hdr = *reinterpret_cast<const uint4 *>(blk);
    const uint4 qv = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * c + 16 * hf);
    const float d = h2f((uint16_t)(hdr.x & 0xffffu)), dmin = h2f((uint16_t)(hdr.x >> 16));
    // scale/min pairs j0 = 2c (lo), j1 = 2c + 1 (hi); bytes 0-3 in y, 4-7 in z, 8-11 in w
    uint32_t sc0, mn0, sc1, mn1;
    {
        const int j0 = 2 * c, j1 = 2 * c + 1;
        const uint32_t t0 = (uint32_t)(j0 & 3) * 8u, t1 = (uint32_t)(j1 & 3) * 8u;
        const uint32_t y0 = (hdr.y >> t0) & 255u, z0 = (hdr.z >> t0) & 255u, w0 = (hdr.w >> t0) & 255u;
        const uint32_t y1 = (hdr.y >> t1) & 255u, z1 = (hdr.z >> t1) & 255u, w1 = (hdr.w >> t1) & 255u;
        const bool low = c < 2;
        sc0 = low ? (y0 & 63u) : ((w0 & 15u) | ((y0 >> 6) << 4));
        mn0 = low ? (z0 & 63u) : ((w0 >> 4) | ((z0 >> 6) << 4));
        sc1 = low ? (y1 & 63u) : ((w1 & 15u) | ((y1 >> 6) << 4));
        mn1 = low ? (z1 & 63u) : ((w1 >> 4) | ((z1 >> 6) << 4));
    }
    float2 al = make_float2(0.f, 0.f), ah = make_float2(0.f, 0.f);
    const uint32_t q[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        const uint32_t lo = q[w] & 0x0f0f0f0fu, hi = (q[w] >> 4) & 0x0f0f0f0fu;
        fma_word(lo, x.lo[2 * w], x.lo[2 * w + 1], al);
        fma_word(hi, x.hi[2 * w], x.hi[2 * w + 1], ah);
    }
    const float s_lo = al.x + al.y, s_hi = ah.x + ah.y;
    const float d0 = d * (float)sc0, d1 = d * (float)sc1;
    const float m0 = dmin * (float)mn0, m1 = dmin * (float)mn1;
    return fmaf(d0, s_lo, -fmaf(128.0f, d0, m0) * x.slo) + fmaf(d1, s_hi, -fmaf(128.0f, d1, m1) * x.shi);
}

// 16 bytes starting at an even (possibly not 4-aligned) shared-memory address.
__device__ __forceinline__ void ld16_unaligned(const uint8_t *p, uint32_t (&o)[4])
{
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t *w = reinterpret_cast<const uint32_t *>(a & ~uintptr_t(3));
    const uint32_t sh = (uint32_t)(a & 3u) * 8u;
    const uint32_t w0 = w[0], w1 = w[1], w2 = w[2], w3 = w[3], w4 = w[4];
    o[0] = __funnelshift_r(w0, w1, sh);
    o[1] = __funnelshift_r(w1, w2, sh);
    o[2] = __funnelshift_r(w2, w3, sh);
    o[3] = __funnelshift_r(w3, w4, sh);
}

// One Q6_K slice (block at an even shared-memory address).
__device__ __forceinline__ float q6k_slice_dot(const uint8_t *blk, int c, int hf, const SliceX &x)
{
    const int h = c >> 1, kk = c & 1;
    uint32_t A[4], B[4], Q[4];
    ld16_unaligned(blk + 64 * h + 16 * hf, A);
    ld16_unaligned(blk + 64 * h + 32 + 16 * hf, B);
    ld16_unaligned(blk + 128 + 32 * h + 16 * hf, Q);
    const float d = h2f((uint16_t)ld_u16(blk + 208));
    const int sbase = 192 + 8 * h + hf + 4 * kk;
    const float s_lo_scale = d * (float)(int8_t)blk[sbase];
    const float s_hi_scale = d * (float)(int8_t)blk[sbase + 2];
    const uint32_t sa = 4u * (uint32_t)kk;
    float2 al = make_float2(0.f, 0.f), ah = make_float2(0.f, 0.f);
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        const uint32_t qs = Q[w] >> sa;
        const uint32_t lo = ((A[w] >> sa) & 0x0f0f0f0fu) | ((qs << 4) & 0x30303030u);
        const uint32_t hi = ((B[w] >> sa) & 0x0f0f0f0fu) | ((qs << 2) & 0x30303030u);
        fma_word(lo, x.lo[2 * w], x.lo[2 * w + 1], al);
        fma_word(hi, x.hi[2 * w], x.hi[2 * w + 1], ah);
    }
    const float s_lo = al.x + al.y, s_hi = ah.x + ah.y;
    return fmaf(s_lo_scale, s_lo, -160.0f * s_lo_scale * x.slo) + fmaf(s_hi_scale, s_hi, -160.0f * s_hi_scale * x.shi);
}

}  // namespace atlas
