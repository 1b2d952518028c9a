// Prompt attention on tensor cores (sm_100a): causal GQA attention for the
// prompt tokens of a prefill chunk (gqa_single_token per token,
// src/brain_runtime.c:1407-1528), with fp32-level accuracy.
//
// A unit is (KV head g, tile of qt query tokens, span of cached positions),
// 128 query rows r = token * group + head (qt = 128 / group). Each of the 8
// warps owns one 16-row MMA tile and walks the span 64 keys at a time:
//   S = Q K^T   mma.sync m16n8k16 (f16 in, f32 accumulate), K by ldmatrix
//   online softmax of S in registers (scale 1/sqrt(128), causal mask)
//   O += P V    P straight from the S registers, V by ldmatrix.trans
// Every product uses the binary16 split x = hi + lo of both operands and adds
// hi*hi + lo*hi + hi*lo (22 significant bits per product, fp32 accumulation),
// as the prefill contractions do: a single binary16 product would move the
// large scores of random-weight models enough to change the softmax.
// A (g, tile) whose keys fit one span writes its output directly; otherwise
// each span stores (acc, max, sum) per row and the last span to finish merges
// them (the same records as before: acc[128], max, sum).
#include <cfloat>
#include <cmath>
#include <cuda_fp16.h>
#include "common.cuh"
#include "prefill.h"

namespace atlas {
namespace pf {
namespace {

constexpr uint32_t kTcRows = 128, kTcKeys = 64, kTcStride = 136;   // halves per staged row (272 B)
constexpr uint32_t kTcRec = 132;

struct TcSmem {
    __half khi[kTcKeys][kTcStride], klo[kTcKeys][kTcStride];
    __half vhi[kTcKeys][kTcStride], vlo[kTcKeys][kTcStride];
    uint32_t flag;
};

__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(const void *p, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(smem_addr(p)));
}

__device__ __forceinline__ void ldsm_x4_t(const void *p, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(smem_addr(p)));
}

// (a, b) -> binary16 hi pair and lo pair (lo = x - hi, rounded)
__device__ __forceinline__ void split2(float a, float b, uint32_t &hi, uint32_t &lo)
{
    const __half2 h = __floats2half2_rn(a, b);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(a - hf.x, b - hf.y);
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = *reinterpret_cast<const uint32_t *>(&l);
}

__device__ __forceinline__ float4 ld_row4(const void *cache, size_t off, uint32_t d4, bool f16)
{
    if (!f16) return __ldcg(reinterpret_cast<const float4 *>(static_cast<const float *>(cache) + off) + d4);
    const uint2 u = __ldcg(reinterpret_cast<const uint2 *>(static_cast<const __half *>(cache) + off) + d4);
    const float2 x = __half22float2(*reinterpret_cast<const __half2 *>(&u.x));
    const float2 y = __half22float2(*reinterpret_cast<const __half2 *>(&u.y));
    return make_float4(x.x, x.y, y.x, y.y);
}

}  // namespace

__global__ void __launch_bounds__(256, 1) attn_tc_kernel(const __grid_constant__ AttnArgs a)
{
    extern __shared__ __align__(16) uint8_t smem_raw[];
    TcSmem &sm = *reinterpret_cast<TcSmem *>(smem_raw);
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u, g8 = lane >> 2, t4 = lane & 3u;
    const uint32_t group = a.q_heads / a.kv_heads, qdim = a.q_heads * 128u, qt_n = a.q_tokens;
    const uint32_t ostride = a.out_stride ? a.out_stride : qdim;
    const bool f16 = a.kv_f16 != 0u;
    const float scale = 1.0f / sqrtf(128.0f);
    for (uint32_t u = blockIdx.x; u < a.n_units; u += gridDim.x) {
        const uint32_t code = a.unit_tab[u];
        const uint32_t g = code & 0xffu, qt = (code >> 8) & 0xfffu, part = code >> 20;
        const uint32_t t0 = qt * qt_n, t1 = min(t0 + qt_n, a.tokens);
        const uint32_t kend = a.pos0 + t1;                       // keys [0, kend) for this tile
        const uint32_t nparts = (kend + a.span - 1) / a.span;
        const uint32_t k0 = part * a.span, k1 = min(k0 + a.span, kend);
        // this lane's two rows of the warp's tile: rr[0] = 16 warp + g8, rr[1] = rr[0] + 8
        uint32_t qpos[2];
        bool rv[2];
        const float *qrow[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const uint32_t r = 16u * warp + g8 + 8u * (uint32_t)i, qi = r / group, h = r % group;
            rv[i] = qi < qt_n && t0 + qi < t1;
            qpos[i] = a.pos0 + t0 + qi;
            qrow[i] = a.q + (size_t)(t0 + qi) * qdim + (size_t)(g * group + h) * 128u;
        }
        // Q fragments (A operand, rows g8 / g8 + 8, dims 16 kk + 2 t4 (+ 8)), split hi / lo
        uint32_t qh[8][4], ql[8][4];
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int i = j & 1;                                  // a0, a2: row g8; a1, a3: row g8 + 8
                const uint32_t d = 16u * (uint32_t)kk + 2u * t4 + ((j & 2) ? 8u : 0u);
                float2 v = make_float2(0.f, 0.f);
                if (rv[i]) v = __ldcg(reinterpret_cast<const float2 *>(qrow[i] + d));
                split2(v.x, v.y, qh[kk][j], ql[kk][j]);
            }
        }
        float m[2] = {-FLT_MAX, -FLT_MAX}, l[2] = {0.f, 0.f};
        float o[16][4];
#pragma unroll
        for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
        for (uint32_t p0 = k0; p0 < k1; p0 += kTcKeys) {
            __syncthreads();   // previous chunk (or unit) done with the staged K / V
            for (uint32_t i = tid; i < kTcKeys * 32u; i += 256u) {
                const uint32_t j = i >> 5, d4 = i & 31u, pos = p0 + j;
                float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
                if (pos < k1) {
                    const size_t off = ((size_t)g * a.max_context + pos) * 128u;
                    kv = ld_row4(a.k_cache, off, d4, f16);
                    vv = ld_row4(a.v_cache, off, d4, f16);
                }
                uint32_t h0, l0, h1, l1;
                split2(kv.x, kv.y, h0, l0);
                split2(kv.z, kv.w, h1, l1);
                *reinterpret_cast<uint2 *>(&sm.khi[j][4 * d4]) = make_uint2(h0, h1);
                *reinterpret_cast<uint2 *>(&sm.klo[j][4 * d4]) = make_uint2(l0, l1);
                split2(vv.x, vv.y, h0, l0);
                split2(vv.z, vv.w, h1, l1);
                *reinterpret_cast<uint2 *>(&sm.vhi[j][4 * d4]) = make_uint2(h0, h1);
                *reinterpret_cast<uint2 *>(&sm.vlo[j][4 * d4]) = make_uint2(l0, l1);
            }
            __syncthreads();
            // S = Q K^T: 8 key tiles of 8, 8 dim steps of 16
            float s[8][4];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
                // lane address: key 8 j + (lane & 7), dims 8 (lane >> 3) of each 32-dim pair of steps
                const uint32_t key = 8u * (uint32_t)j + (lane & 7u), dsub = 8u * (lane >> 3);
#pragma unroll
                for (int kk = 0; kk < 8; kk += 2) {
                    uint32_t bh[4], bl[4];
                    ldsm_x4(&sm.khi[key][16u * kk + dsub], bh[0], bh[1], bh[2], bh[3]);
                    ldsm_x4(&sm.klo[key][16u * kk + dsub], bl[0], bl[1], bl[2], bl[3]);
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const int k2 = kk + e;
                        mma_f16(s[j], qh[k2][0], qh[k2][1], qh[k2][2], qh[k2][3], bh[2 * e], bh[2 * e + 1]);
                        mma_f16(s[j], ql[k2][0], ql[k2][1], ql[k2][2], ql[k2][3], bh[2 * e], bh[2 * e + 1]);
                        mma_f16(s[j], qh[k2][0], qh[k2][1], qh[k2][2], qh[k2][3], bl[2 * e], bl[2 * e + 1]);
                    }
                }
            }
            // online softmax per row (src/brain_runtime.c:1430-1476 computes the
            // same weights in one pass): lane holds keys 8 j + 2 t4 (+1) of rows g8, g8 + 8
            uint32_t ph[4][4], pl[4][4];   // P as A fragments of 4 key steps of 16
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                float mx = m[i];
#pragma unroll
                for (int j = 0; j < 8; ++j)
#pragma unroll
                    for (int c = 0; c < 2; ++c) {
                        const uint32_t key = p0 + 8u * (uint32_t)j + 2u * t4 + (uint32_t)c;
                        const bool ok = rv[i] && key <= qpos[i] && key < k1;
                        float &v = s[j][2 * i + c];
                        v = ok ? v * scale : -INFINITY;
                        mx = fmaxf(mx, v);
                    }
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
                const float corr = expf(m[i] - mx);
                float sum = 0.f;
#pragma unroll
                for (int j = 0; j < 8; ++j)
#pragma unroll
                    for (int c = 0; c < 2; ++c) {
                        float &v = s[j][2 * i + c];
                        v = v == -INFINITY ? 0.f : expf(v - mx);
                        sum += v;
                    }
                sum += __shfl_xor_sync(0xffffffffu, sum, 1);
                sum += __shfl_xor_sync(0xffffffffu, sum, 2);
                m[i] = mx;
                l[i] = fmaf(l[i], corr, sum);
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    o[j][2 * i] *= corr;
                    o[j][2 * i + 1] *= corr;
                }
            }
#pragma unroll
            for (int kp = 0; kp < 4; ++kp) {
                split2(s[2 * kp][0], s[2 * kp][1], ph[kp][0], pl[kp][0]);
                split2(s[2 * kp][2], s[2 * kp][3], ph[kp][1], pl[kp][1]);
                split2(s[2 * kp + 1][0], s[2 * kp + 1][1], ph[kp][2], pl[kp][2]);
                split2(s[2 * kp + 1][2], s[2 * kp + 1][3], ph[kp][3], pl[kp][3]);
            }
            // O += P V: 16 dim tiles of 8, 4 key steps of 16; V^T fragments by ldmatrix.trans
#pragma unroll
            for (int kp = 0; kp < 4; ++kp) {
                // matrix i: keys 16 kp + 8 (i & 1) + (lane & 7), dims 8 (jd + (i >> 1))
                const uint32_t mi = lane >> 3, key = 16u * kp + 8u * (mi & 1u) + (lane & 7u);
#pragma unroll
                for (int jd = 0; jd < 16; jd += 2) {
                    uint32_t vh[4], vl[4];
                    ldsm_x4_t(&sm.vhi[key][8u * (jd + (mi >> 1))], vh[0], vh[1], vh[2], vh[3]);
                    ldsm_x4_t(&sm.vlo[key][8u * (jd + (mi >> 1))], vl[0], vl[1], vl[2], vl[3]);
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        float(&acc)[4] = o[jd + e];
                        mma_f16(acc, ph[kp][0], ph[kp][1], ph[kp][2], ph[kp][3], vh[2 * e], vh[2 * e + 1]);
                        mma_f16(acc, pl[kp][0], pl[kp][1], pl[kp][2], pl[kp][3], vh[2 * e], vh[2 * e + 1]);
                        mma_f16(acc, ph[kp][0], ph[kp][1], ph[kp][2], ph[kp][3], vl[2 * e], vl[2 * e + 1]);
                    }
                }
            }
        }   // key chunks of the span
        if (nparts == 1) {
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                if (!rv[i]) continue;
                const uint32_t r = 16u * warp + g8 + 8u * (uint32_t)i, qi = r / group, h = r % group;
                float *dst = a.out + (size_t)(t0 + qi) * ostride + (size_t)(g * group + h) * 128u;
                const float inv = l[i] > 0.f ? 1.0f / l[i] : 0.f;
#pragma unroll
                for (int jd = 0; jd < 16; ++jd)
                    *reinterpret_cast<float2 *>(dst + 8u * jd + 2u * t4) =
                        make_float2(o[jd][2 * i] * inv, o[jd][2 * i + 1] * inv);
            }
            continue;
        }
        // partial record of this span: acc[128], max, sum per row
        const uint32_t u0 = u - part;   // the tile's spans are consecutive units
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const uint32_t r = 16u * warp + g8 + 8u * (uint32_t)i;
            float *rec = a.part + ((size_t)u * kTcRows + r) * kTcRec;
#pragma unroll
            for (int jd = 0; jd < 16; ++jd)
                __stcg(reinterpret_cast<float2 *>(rec + 8u * jd + 2u * t4), make_float2(o[jd][2 * i], o[jd][2 * i + 1]));
            if (t4 == 0) { __stcg(rec + 128, m[i]); __stcg(rec + 129, l[i]); }
        }
        __threadfence();
        __syncthreads();
        if (tid == 0) {
            const uint32_t old = atom_acq_rel_add(a.ctr + g * a.q_tiles + qt, 1u);
            sm.flag = (old == nparts - 1u) ? 1u : 0u;
        }
        __syncthreads();
        if (!sm.flag) continue;
        __threadfence();
        // merge: thread = (row, 64-dim half); the records come from L2
        for (uint32_t i = tid; i < kTcRows * 2u; i += 256u) {
            const uint32_t r = i >> 1, half = i & 1u, qi = r / group, h = r % group;
            if (qi >= qt_n || t0 + qi >= t1) continue;
            float M = -FLT_MAX;
            for (uint32_t c = 0; c < nparts; ++c) M = fmaxf(M, __ldcg(a.part + ((size_t)(u0 + c) * kTcRows + r) * kTcRec + 128));
            float L = 0.f;
            float4 acc[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
            for (uint32_t c = 0; c < nparts; ++c) {
                const float *rec = a.part + ((size_t)(u0 + c) * kTcRows + r) * kTcRec;
                const float mc = __ldcg(rec + 128);
                const float f = mc == -FLT_MAX ? 0.f : expf(mc - M);
                L = fmaf(f, __ldcg(rec + 129), L);
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const float4 v = __ldcg(reinterpret_cast<const float4 *>(rec + 64u * half) + j);
                    acc[j].x = fmaf(f, v.x, acc[j].x);
                    acc[j].y = fmaf(f, v.y, acc[j].y);
                    acc[j].z = fmaf(f, v.z, acc[j].z);
                    acc[j].w = fmaf(f, v.w, acc[j].w);
                }
            }
            const float inv = L > 0.f ? 1.0f / L : 0.f;
            float *dst = a.out + (size_t)(t0 + qi) * ostride + (size_t)(g * group + h) * 128u + 64u * half;
#pragma unroll
            for (int j = 0; j < 16; ++j)
                reinterpret_cast<float4 *>(dst)[j] =
                    make_float4(acc[j].x * inv, acc[j].y * inv, acc[j].z * inv, acc[j].w * inv);
        }
        if (tid == 0) a.ctr[g * a.q_tiles + qt] = 0;
    }
}

}  // namespace pf
}  // namespace atlas

extern "C" cudaError_t atlas_launch_prefill_attn_tc(const atlas::pf::AttnArgs *a, int grid, cudaStream_t stream)
{
    using atlas::pf::attn_tc_kernel;
    static bool attr_set = false;
    const int bytes = (int)sizeof(atlas::pf::TcSmem);
    if (!attr_set) {
        const cudaError_t e = cudaFuncSetAttribute(attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    attn_tc_kernel<<<grid, 256, bytes, stream>>>(*a);
    return cudaGetLastError();
}
