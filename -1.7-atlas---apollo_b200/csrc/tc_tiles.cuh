// Tensor-core tiles of the decode GEMVs (mma.sync m16n8k16, fp32 accumulate),
// fp32-accurate: matvec_rows (src/brain_runtime.c:1133-1185) with the Q4_K /
// Q6_K block decoders (:960-1083) folded into the A operand.
//
//   A = weights. A 4- or 6-bit quant q, zero-extended into a 16-bit lane, is
//     the fp16 subnormal q * 2^-24 - exactly; one byte permute builds two A
//     values straight from the raw super-block bytes.
//   B = input x split as x = hi + lo, both fp16 (hi = fp16(x), lo =
//     fp16(x - hi)), after scaling x by a power of two so max|x| sits near
//     2^13: 22 significant bits. Even B columns hold hi, odd columns lo, so the
//     fragment of every lane receives sum(q*hi) and sum(q*lo) for its rows.
//   k order: inside each 16-wide k step, lane t's four k slots map to the four
//     consecutive elements 4t..4t+3, so each A fragment register is built from
//     one 32-bit word of the block and B is stored to match: the staged x of a
//     256-element block column is 64 groups of 16 bytes (4 hi + 4 lo halves of
//     elements 4i..4i+3), followed elsewhere by one sum per 16 elements.
//   Scales: per 32-element sub-block (Q4_K: d*sc, dmin*m) or 16-element group
//     (Q6_K: d*sc, with the -32 offset folded via the group's sum of x); lane
//     t applies the groups j with j % 4 == t, and the 4 lanes of a row group
//     are summed by the caller.
#pragma once
#include <cstdint>
#include "common.cuh"
#include "quant.cuh"

namespace atlas {
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint2 b,
                                         const float (&c)[4])
{
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b.x), "r"(b.y), "f"(c[0]), "f"(c[1]), "f"(c[2]), "f"(c[3]));
}

// bytes 0,1 (sel 0x4140) or 2,3 (sel 0x4342) of v as two zero-extended 16-bit
// lanes: the fp16 subnormals q0 * 2^-24, q1 * 2^-24
__device__ __forceinline__ uint32_t sub2(uint32_t v, uint32_t sel) { return __byte_perm(v, 0u, sel); }

__device__ __forceinline__ uint32_t ld32u(const uint8_t *p)
{
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t *w = reinterpret_cast<const uint32_t *>(a & ~uintptr_t(3));
    return __funnelshift_r(w[0], w[1], (uint32_t)(a & 3u) * 8u);
}

constexpr float kTwo24 = 16777216.0f;

// NT independent 16-row x 256-element Q4_K tiles (NT = 1 or 2, interleaved
// for instruction-level parallelism). Tile n: rows (g, g+8) of this lane at
// r0[n] / r1[n] (nullptr: row absent), the block column's staged x groups
// xb[n] and 16-element sums xs[n]. Adds this lane's sub-blocks (j = t, t + 4).
template <int NT, bool FULL>
__device__ __forceinline__ void q4k_tiles(const uint8_t *const (&r0)[NT], const uint8_t *const (&r1)[NT],
                                          const uint8_t *const (&xb)[NT], const float *const (&xs)[NT], int g, int t,
                                          float (&o0)[NT], float (&o1)[NT])
{
    float dsc[NT][2][2], dmn[NT][2][2];
#pragma unroll
    for (int n = 0; n < NT; ++n) {
        const uint8_t *rows[2] = {r0[n], r1[n]};
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            dsc[n][r][0] = dsc[n][r][1] = dmn[n][r][0] = dmn[n][r][1] = 0.f;
            if (!FULL && !rows[r]) continue;
            const uint4 hd = *reinterpret_cast<const uint4 *>(rows[r]);
            const float d = h2f((uint16_t)(hd.x & 0xffffu)), dm = h2f((uint16_t)(hd.x >> 16));
            const uint32_t sh = 8u * (uint32_t)t;
            const uint32_t y = (hd.y >> sh) & 255u, z = (hd.z >> sh) & 255u, w = (hd.w >> sh) & 255u;
            dsc[n][r][0] = d * u2f_small(y & 63u);                        // j = t
            dmn[n][r][0] = dm * u2f_small(z & 63u);
            dsc[n][r][1] = d * u2f_small((w & 15u) | ((y >> 6) << 4));    // j = t + 4
            dmn[n][r][1] = dm * u2f_small((w >> 4) | ((z >> 6) << 4));
        }
    }
    const float zero[4] = {0.f, 0.f, 0.f, 0.f};
    const uint32_t podd = (uint32_t)(g & 1) * 8u;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        float dlo[NT][4], dhi[NT][4];
#pragma unroll
        for (int hp = 0; hp < 2; ++hp) {
            const uint32_t off = 16u + 32u * c + 16u * hp + 4u * t;
#pragma unroll
            for (int n = 0; n < NT; ++n) {
                const uint32_t w0 = (FULL || r0[n]) ? *reinterpret_cast<const uint32_t *>(r0[n] + off) : 0u;
                const uint32_t w1 = (FULL || r1[n]) ? *reinterpret_cast<const uint32_t *>(r1[n] + off) : 0u;
                const uint32_t l0 = w0 & 0x0f0f0f0fu, h0 = (w0 >> 4) & 0x0f0f0f0fu;
                const uint32_t l1 = w1 & 0x0f0f0f0fu, h1 = (w1 >> 4) & 0x0f0f0f0fu;
                const uint2 blo = *reinterpret_cast<const uint2 *>(xb[n] + (16u * c + 4u * hp + (uint32_t)t) * 16u + podd);
                const uint2 bhi = *reinterpret_cast<const uint2 *>(xb[n] + (16u * c + 8u + 4u * hp + (uint32_t)t) * 16u + podd);
                if (hp == 0) {
                    mma16816(dlo[n], sub2(l0, 0x4140), sub2(l1, 0x4140), sub2(l0, 0x4342), sub2(l1, 0x4342), blo, zero);
                    mma16816(dhi[n], sub2(h0, 0x4140), sub2(h1, 0x4140), sub2(h0, 0x4342), sub2(h1, 0x4342), bhi, zero);
                } else {
                    const float clo[4] = {dlo[n][0], dlo[n][1], dlo[n][2], dlo[n][3]};
                    const float chi[4] = {dhi[n][0], dhi[n][1], dhi[n][2], dhi[n][3]};
                    mma16816(dlo[n], sub2(l0, 0x4140), sub2(l1, 0x4140), sub2(l0, 0x4342), sub2(l1, 0x4342), blo, clo);
                    mma16816(dhi[n], sub2(h0, 0x4140), sub2(h1, 0x4140), sub2(h0, 0x4342), sub2(h1, 0x4342), bhi, chi);
                }
            }
        }
        // this lane's sub-block in chunk c, if any: j = 2c + (t & 1) with (c & 1) == (t >> 1)
        if ((c & 1) == (t >> 1)) {
            const int slot = c >> 1, j = 2 * c + (t & 1);
#pragma unroll
            for (int n = 0; n < NT; ++n) {
                const float *D = (t & 1) ? dhi[n] : dlo[n];
                const float sx = xs[n][2 * j] + xs[n][2 * j + 1];
                o0[n] += dsc[n][0][slot] * ((D[0] + D[1]) * kTwo24) - dmn[n][0][slot] * sx;
                o1[n] += dsc[n][1][slot] * ((D[2] + D[3]) * kTwo24) - dmn[n][1][slot] * sx;
            }
        }
    }
}

// NT independent 16-row x 256-element Q6_K tiles (blocks at even, not
// necessarily 4-aligned addresses). Lane t keeps the 16-element groups with
// k == t: one scale per (h, hp) and row, selected outside the k loop.
// SAME_X: all NT tiles use the block column of xb[0] / xs[0] (row tiles of
// one block column), so the B fragments are loaded once.
template <int NT, bool FULL, bool SAME_X = false>
__device__ __forceinline__ void q6k_tiles(const uint8_t *const (&r0)[NT], const uint8_t *const (&r1)[NT],
                                          const uint8_t *const (&xb)[NT], const float *const (&xs)[NT], int g, int t,
                                          float (&o0)[NT], float (&o1)[NT])
{
    float d0[NT], d1[NT];
#pragma unroll
    for (int n = 0; n < NT; ++n) {
        d0[n] = (FULL || r0[n]) ? h2f((uint16_t)ld_u16(r0[n] + 208)) : 0.f;
        d1[n] = (FULL || r1[n]) ? h2f((uint16_t)ld_u16(r1[n] + 208)) : 0.f;
    }
    const float zero[4] = {0.f, 0.f, 0.f, 0.f};
    const uint32_t podd = (uint32_t)(g & 1) * 8u;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int hp = 0; hp < 2; ++hp) {
            const uint32_t oa = 64u * h + 16u * hp + 4u * t, ob = oa + 32u, oq = 128u + 32u * h + 16u * hp + 4u * t;
            const uint32_t si = 192u + 8u * h + hp + 2u * (uint32_t)t;   // scale of group k == t
            uint32_t A0[NT], B0[NT], Q0[NT], A1[NT], B1[NT], Q1[NT];
            float s0[NT], s1[NT], keep[NT][4];
#pragma unroll
            for (int n = 0; n < NT; ++n) {
                const bool h0 = FULL || r0[n], h1 = FULL || r1[n];
                A0[n] = h0 ? ld32u(r0[n] + oa) : 0u; B0[n] = h0 ? ld32u(r0[n] + ob) : 0u;
                Q0[n] = h0 ? ld32u(r0[n] + oq) : 0u;
                A1[n] = h1 ? ld32u(r1[n] + oa) : 0u; B1[n] = h1 ? ld32u(r1[n] + ob) : 0u;
                Q1[n] = h1 ? ld32u(r1[n] + oq) : 0u;
                s0[n] = h0 ? d0[n] * s8f(r0[n][si]) : 0.f;
                s1[n] = h1 ? d1[n] * s8f(r1[n][si]) : 0.f;
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint32_t sa = (k & 2) ? 4u : 0u;
                const uint32_t e0 = 128u * h + 32u * k + 16u * hp;  // first element of the 16-group
#pragma unroll
                for (int n = 0; n < NT; ++n) {
                    uint32_t v0, v1;
                    if (k == 3) {
                        v0 = ((B0[n] >> 4) & 0x0f0f0f0fu) | ((Q0[n] >> 2) & 0x30303030u);
                        v1 = ((B1[n] >> 4) & 0x0f0f0f0fu) | ((Q1[n] >> 2) & 0x30303030u);
                    } else {
                        const uint32_t qs = (k == 0) ? 4u : (k == 1) ? 2u : 0u;
                        const uint32_t x0 = (k & 1) ? B0[n] : A0[n], x1 = (k & 1) ? B1[n] : A1[n];
                        v0 = ((x0 >> sa) & 0x0f0f0f0fu) | ((Q0[n] << qs) & 0x30303030u);
                        v1 = ((x1 >> sa) & 0x0f0f0f0fu) | ((Q1[n] << qs) & 0x30303030u);
                    }
                    const uint2 b = *reinterpret_cast<const uint2 *>(xb[SAME_X ? 0 : n] + (e0 / 4u + (uint32_t)t) * 16u + podd);
                    float dd[4];
                    mma16816(dd, sub2(v0, 0x4140), sub2(v1, 0x4140), sub2(v0, 0x4342), sub2(v1, 0x4342), b, zero);
                    const bool mine = k == t;
#pragma unroll
                    for (int e = 0; e < 4; ++e) keep[n][e] = mine ? dd[e] : (k == 0 ? 0.f : keep[n][e]);
                }
            }
#pragma unroll
            for (int n = 0; n < NT; ++n) {
                const float sx = 32.0f * xs[SAME_X ? 0 : n][8u * h + 2u * (uint32_t)t + hp];
                o0[n] += s0[n] * ((keep[n][0] + keep[n][1]) * kTwo24 - sx);
                o1[n] += s1[n] * ((keep[n][2] + keep[n][3]) * kTwo24 - sx);
            }
        }
    }
}

}  // namespace atlas
