// Graph decode step (sm_100a): the reference's forward_token
// (src/brain_runtime.c:1698-1772) and greedy pick (:1783) as a chain of
// kernels - embed, per layer {mv qkv, attention, mv o, mv gate/up, mv down},
// mv head, argmax - launched with programmatic dependent launch and replayed
// from one CUDA graph per token.
//
// Every kernel first lets its successor launch (griddepcontrol.launch_dependents)
// and only then waits for its predecessor (griddepcontrol.wait). A kernel is
// sized to take at most half of an SM, so the successor's CTAs become resident
// while the current kernel runs and their producer warps stream the next
// weights into shared memory ahead of time: weights never depend on the
// activations, so HBM keeps streaming across kernel boundaries.
//
// mv kernel (dequant-GEMV, one CTA per SM): a producer warp copies the raw
// Q4_K / Q6_K rows of the CTA's task range into a shared-memory ring with 1-D
// bulk copies, one copy per row piece, rows placed at an odd multiple of 16
// bytes apart so that the 8 row groups of a warp hit distinct banks. Eight
// consumer warps stage the input (rms_norm'ed, split into fp16 hi/lo), then run
// the tensor-core tiles of tc_tiles.cuh on their tasks (16 rows x 256
// elements each) and reduce the tiles' row sums in a fixed order: inside the
// CTA through shared memory, across neighbouring CTAs through a small global
// buffer and a per-tile arrival counter (the last CTA to arrive finishes the
// tile). No thread ever waits for another CTA.
#include <algorithm>
#include <cfloat>
#include <cmath>
#include "common.cuh"
#include "quant.cuh"
#include "tc_tiles.cuh"
#include "decode2.h"

namespace atlas {
namespace d2 {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// consumer warps only (the producer warp never joins)
__device__ __forceinline__ void mv_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kMvWarps * 32) : "memory"); }

__host__ __device__ constexpr uint32_t align128(uint32_t v) { return (v + 127u) & ~127u; }

// smallest odd multiple of 16 that is >= v
__host__ __device__ constexpr uint32_t odd16(uint32_t v)
{
    const uint32_t m = (v + 15u) / 16u;
    return 16u * (m | 1u);
}

// Dynamic shared memory of an mv CTA:
//   MvHdr | tile area: tcnt[tslots], tpart[tslots][2][kMvWarps][16] | x area | ring
struct __align__(16) MvHdr {
    uint64_t full[kMvMaxSlots];
    uint64_t empty[kMvMaxSlots];
    double dred[kMvWarps];
    float fred[kMvWarps];
    float amax[kMvWarps];
    uint32_t aidx[kMvWarps];
    uint32_t *tcnt;    // arrivals per open tile slot
    float *tpart;      // per-warp row sums of open tiles
};

__host__ __device__ constexpr uint32_t mv_hdr_bytes() { return align128((uint32_t)sizeof(MvHdr)); }
__host__ __device__ constexpr uint32_t mv_tcnt_bytes(uint32_t tslots) { return (tslots * 4u + 15u) & ~15u; }
__host__ __device__ constexpr uint32_t mv_tile_bytes(uint32_t tslots)
{
    return align128(mv_tcnt_bytes(tslots) + tslots * 2u * kMvWarps * 16u * 4u);
}
__host__ __device__ constexpr uint32_t mv_x_bytes(uint32_t cols) { return align128(cols * 4u + cols / 16u * 4u); }

__device__ __forceinline__ float *tpart_at(const MvHdr *h, uint32_t ts, uint32_t s, uint32_t w)
{
    return h->tpart + ((ts * 2u + s) * kMvWarps + w) * 16u;
}

// One (tile, segment) run of block columns inside a ring slot; its 16 rows sit
// at off + i * stride (+ the row piece's misalignment `lead`).
struct Portion {
    uint32_t t, s, b0, n, off, stride, j;   // j: first task of the run
};

__device__ __forceinline__ uint32_t mv_bb(uint32_t type) { return type == 12u ? 144u : 210u; }

// Runs of the slot holding tasks [js, je) of segment `segi` (or of the pair).
__device__ __forceinline__ uint32_t slot_portions(const MvArgs &a, uint32_t segi, uint32_t js, uint32_t je,
                                                  Portion (&pr)[kMvMaxPortions])
{
    const uint32_t P = a.paired ? 2u : 1u, TP = a.nb * P;
    uint32_t j = js, off = 0, np = 0;
#pragma unroll
    for (int q = 0; q < kMvMaxPortions; ++q) {
        if (j >= je) break;
        const uint32_t t = j / TP, r = j % TP;
        const uint32_t s = a.paired ? r / a.nb : segi;
        const uint32_t b0 = r % a.nb, n = min(a.nb - b0, je - j);
        const uint32_t stride = odd16(n * mv_bb(a.seg[s].type) + 15u);
        pr[q] = Portion{t, s, b0, n, off, stride, j};
        off += 16u * stride;
        j += n;
        ++np;
    }
    return np;
}

// Global address of row i of a run (the bulk copy starts at it rounded down to 16 bytes).
__device__ __forceinline__ const uint8_t *run_row(const MvArgs &a, const Portion &p, uint32_t i)
{
    const MvSeg &sg = a.seg[p.s];
    return sg.w + (uint64_t)(16u * p.t + i) * sg.row_bytes + (uint64_t)p.b0 * mv_bb(sg.type);
}

// ----------------------------------------------------------- producer ----

__device__ void mv_producer(const MvArgs &a, MvHdr *h, uint8_t *ring, const MvCta &c, volatile uint32_t *err)
{
    const uint32_t lane = threadIdx.x & 31u;
    const uint64_t policy = policy_evict_first();
    const uint32_t nslots = (c.j1 - c.j0 + a.st - 1u) / a.st;
    for (uint32_t k = 0; k < nslots; ++k) {
        const uint32_t ri = k % a.nslot;
        if (k >= a.nslot) {
            uint32_t ok = 1u;
            if (lane == 0) ok = mbar_wait(&h->empty[ri], ((k / a.nslot) & 1u) ^ 1u, err) ? 1u : 0u;
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
        }
        const uint32_t js = c.j0 + k * a.st, je = min(c.j1, js + a.st);
        Portion pr[kMvMaxPortions];
        const uint32_t np = slot_portions(a, c.seg, js, je, pr);
        uint8_t *slot = ring + (size_t)ri * a.slot_bytes;
        // lane L copies rows L and L + 32 of the slot's runs (16 rows per run)
        const uint8_t *src[2];
        uint8_t *dst[2];
        uint32_t nbytes[2] = {0u, 0u};
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const uint32_t idx = lane + 32u * (uint32_t)u, p = idx / 16u, i = idx % 16u;
            if (p >= np) continue;
            Portion q = pr[0];
#pragma unroll
            for (int v = 1; v < kMvMaxPortions; ++v)
                if ((uint32_t)v == p) q = pr[v];
            const uint8_t *g = run_row(a, q, i);
            const uint32_t lead = (uint32_t)(reinterpret_cast<uintptr_t>(g) & 15u);
            src[u] = g - lead;
            dst[u] = slot + q.off + i * q.stride;
            nbytes[u] = (lead + q.n * mv_bb(a.seg[q.s].type) + 15u) & ~15u;
        }
        uint32_t total = nbytes[0] + nbytes[1];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
        if (lane == 0) mbar_arrive_expect_tx(&h->full[ri], total);
        __syncwarp();
#pragma unroll
        for (int u = 0; u < 2; ++u)
            if (nbytes[u]) bulk_g2s_hint(dst[u], src[u], nbytes[u], &h->full[ri], policy);
    }
    // every issued copy lands before the CTA may exit
    if (lane == 0) {
        const uint32_t first = nslots > a.nslot ? nslots - a.nslot : 0u;
        for (uint32_t k = first; k < nslots; ++k)
            if (!mbar_wait(&h->full[k % a.nslot], (k / a.nslot) & 1u, err)) break;
    }
}

// ------------------------------------------------------ input staging ----

// Stage x (times norm_w when normalizing) in shared memory as fp16 (hi, lo)
// groups plus one sum per 16 elements, in units of x * xscale, xscale a power
// of two putting max|x| in [2^13, 2^14). The rms_norm factor is a scalar, so
// it is applied to the row sums instead: W (x w inv) = inv * W (x w), with
// the sum of squares in double as src/brain_runtime.c:1345-1360. Returns the
// factor for the row sums: inv_rms / xscale.
__device__ float mv_stage_x(const MvArgs &a, MvHdr *h, uint8_t *xarea)
{
    const uint32_t n = a.cols;
    const bool norm = a.norm_w != nullptr;
    float4 *xf = reinterpret_cast<float4 *>(xarea);
    float mx = 0.f;
    double ss = 0.0;
    constexpr uint32_t kStride = kMvWarps * 32;
    for (uint32_t i0 = threadIdx.x; i0 < n / 4u; i0 += 4u * kStride) {
        float4 v[4], w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t i = i0 + (uint32_t)j * kStride;
            if (i < n / 4u) {
                v[j] = __ldcg(reinterpret_cast<const float4 *>(a.x) + i);
                if (norm) w[j] = __ldg(reinterpret_cast<const float4 *>(a.norm_w) + i);
            }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t i = i0 + (uint32_t)j * kStride;
            if (i >= n / 4u) continue;
            float4 x = v[j];
            if (norm) {
                ss += (double)x.x * (double)x.x;
                ss += (double)x.y * (double)x.y;
                ss += (double)x.z * (double)x.z;
                ss += (double)x.w * (double)x.w;
                x.x *= w[j].x; x.y *= w[j].y; x.z *= w[j].z; x.w *= w[j].w;
            }
            xf[i] = x;
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w))));
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        ss += __shfl_xor_sync(0xffffffffu, ss, o);
    }
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    if (lane == 0) { h->fred[warp] = mx; h->dred[warp] = ss; }
    mv_sync();
    float m = 0.f;
    double t = 0.0;
#pragma unroll
    for (int w = 0; w < kMvWarps; ++w) { m = fmaxf(m, h->fred[w]); t += h->dred[w]; }
    // exponent capped at 126: rows of tiny values (a SwiGLU output of
    // all-negative gates) keep a finite scale and contribute ~0, as in fp32
    const float s = (m > 0.f && isfinite(m)) ? exp2f((float)min(13 - ilogbf(m), 126)) : 1.0f;
    const float inv_rms = norm ? 1.0f / sqrtf((float)(t / (double)n) + a.eps) : 1.0f;
    float *xs16 = reinterpret_cast<float *>(xarea + (size_t)n * 4u);
    for (uint32_t u = threadIdx.x; u < n / 16u; u += kStride) {
        float sum = 0.f;
        uint4 pk[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float4 v = xf[4 * u + q];
            const float e[4] = {v.x * s, v.y * s, v.z * s, v.w * s};
            __half hi[4], lo[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                hi[i] = __float2half_rn(e[i]);
                lo[i] = __float2half_rn(e[i] - __half2float(hi[i]));
                sum += e[i];
            }
            pk[q].x = (uint32_t)__half_as_ushort(hi[0]) | ((uint32_t)__half_as_ushort(hi[1]) << 16);
            pk[q].y = (uint32_t)__half_as_ushort(hi[2]) | ((uint32_t)__half_as_ushort(hi[3]) << 16);
            pk[q].z = (uint32_t)__half_as_ushort(lo[0]) | ((uint32_t)__half_as_ushort(lo[1]) << 16);
            pk[q].w = (uint32_t)__half_as_ushort(lo[2]) | ((uint32_t)__half_as_ushort(lo[3]) << 16);
        }
        // in place: unit u's 64 bytes are only read by this thread
#pragma unroll
        for (int q = 0; q < 4; ++q) reinterpret_cast<uint4 *>(xarea)[4 * u + q] = pk[q];
        xs16[u] = sum;
    }
    mv_sync();
    return inv_rms / s;
}

// ---------------------------------------------------------- consumers ----

struct MvBest {
    float v;
    uint32_t i;
};

// largest CTA of segment `segi` whose range starts at or before task j
__device__ __forceinline__ uint32_t cta_of(const MvArgs &a, uint32_t segi, uint32_t j)
{
    uint32_t lo = a.seg_cta0[segi], hi = a.seg_cta0[segi + 1] - 1u;
    while (lo < hi) {
        const uint32_t mid = (lo + hi + 1u) / 2u;
        if (__ldg(&a.cta[mid].j0) <= j) lo = mid;
        else hi = mid - 1u;
    }
    return lo;
}

// Epilogue of tile t. Lane i < 16 holds row i (paired: the gate sum; lane
// 16 + i the up sum of the same row).
__device__ __forceinline__ void mv_finish(const MvArgs &a, uint32_t segi, uint32_t t, float v, uint32_t lane,
                                          MvBest &best)
{
    const uint32_t row = 16u * t + (lane & 15u);
    if (a.epi == MV_SWIGLU) {
        const float up = __shfl_down_sync(0xffffffffu, v, 16);
        if (lane < 16u) a.seg[0].out[row] = (v / (1.0f + expf(-v))) * up;   // src/brain_runtime.c:1755-1758
        return;
    }
    if (lane >= 16u) return;
    const MvSeg &sg = a.seg[segi];
    if (a.epi == MV_RESID) {
        sg.out[row] = __ldcg(sg.out + row) + v;   // src/brain_runtime.c:1745, :1762
        return;
    }
    const float r = sg.bias ? v + __ldg(sg.bias + row) : v;
    sg.out[row] = r;
    if (a.epi == MV_LOGITS && (r > best.v || (r == best.v && row < best.i))) { best.v = r; best.i = row; }
}

// The warp's row sums of tile t are complete. Publish them; the last of the
// CTA's warps with tasks in the tile adds them up in warp order and finishes
// the tile - or, for a tile shared with neighbouring CTAs, publishes the
// CTA's sums and the last CTA to arrive adds those up in CTA order.
__device__ void mv_flush(const MvArgs &a, MvHdr *h, const MvCta &c, uint32_t t, const float (&acc)[2][2],
                         float out_scale, MvBest &best)
{
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u, g = lane >> 2;
    const uint32_t P = a.paired ? 2u : 1u, TP = a.nb * P, ts = t % a.tslots;
#pragma unroll
    for (uint32_t s = 0; s < 2; ++s) {
        if (s >= P) break;
        float v0 = acc[s][0], v1 = acc[s][1];
        v0 += __shfl_xor_sync(0xffffffffu, v0, 1);
        v0 += __shfl_xor_sync(0xffffffffu, v0, 2);
        v1 += __shfl_xor_sync(0xffffffffu, v1, 1);
        v1 += __shfl_xor_sync(0xffffffffu, v1, 2);
        if ((lane & 3u) == 0u) {
            float *tp = tpart_at(h, ts, s, warp);
            tp[g] = v0;
            tp[g + 8u] = v1;
        }
    }
    const uint32_t a0 = max(c.j0, t * TP), a1 = min(c.j1, (t + 1u) * TP), n = a1 - a0;
    const uint32_t expect = min(n, (uint32_t)kMvWarps);
    __syncwarp();
    uint32_t last = 0;
    if (lane == 0) {
        __threadfence_block();
        last = (atomicAdd(&h->tcnt[ts], 1u) + 1u == expect) ? 1u : 0u;
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) return;
    __threadfence_block();
    const uint32_t i = lane & 15u, s = lane >> 4;
    float v = 0.f;
    if (s < P) {
        const uint32_t w0 = (a0 - c.j0) % kMvWarps;
        const volatile float *tp = tpart_at(h, ts, s, 0) + i;
#pragma unroll
        for (uint32_t w = 0; w < (uint32_t)kMvWarps; ++w)
            if (n >= (uint32_t)kMvWarps || ((w + kMvWarps - w0) % kMvWarps) < n) v += tp[w * 16u];
        v *= out_scale;
    }
    __syncwarp();
    if (lane == 0) h->tcnt[ts] = 0u;
    if (t * TP >= c.j0 && (t + 1u) * TP <= c.j1) {
        mv_finish(a, c.seg, t, v, lane, best);
        return;
    }
    // tile shared with neighbouring CTAs
    const uint32_t side = (t == c.j0 / TP) ? 0u : 1u;
    if (s < P) a.bpart[((size_t)blockIdx.x * 2u + side) * 32u + s * 16u + i] = v;
    __threadfence();
    __syncwarp();
    const uint32_t cf = cta_of(a, c.seg, t * TP), cl = cta_of(a, c.seg, (t + 1u) * TP - 1u);
    uint32_t *ctr = a.tctr + a.seg_tile0[c.seg] + t;
    uint32_t done = 0;
    if (lane == 0) done = (atom_acq_rel_add(ctr, 1u) == cl - cf) ? 1u : 0u;
    done = __shfl_sync(0xffffffffu, done, 0);
    if (!done) return;
    __syncwarp();
    __threadfence();
    float tot = 0.f;
    if (s < P)
        for (uint32_t cc = cf; cc <= cl; ++cc) {
            const uint32_t sd = (t == __ldg(&a.cta[cc].j0) / TP) ? 0u : 1u;
            tot += __ldcg(a.bpart + ((size_t)cc * 2u + sd) * 32u + s * 16u + i);
        }
    if (lane == 0) *ctr = 0u;
    mv_finish(a, c.seg, t, tot, lane, best);
}

// Consumer warp: tasks c.j0 + warp + 8m, each one 16-row x 256-element tile
// of the staged slot. Returns false after a failed wait (status recorded).
__device__ bool mv_consumer(const MvArgs &a, MvHdr *h, uint8_t *xarea, const uint8_t *ring, const MvCta &c,
                            volatile uint32_t *err, MvBest &best)
{
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const int g = (int)(lane >> 2), t4 = (int)(lane & 3u);
    if (a.pdl) pdl_wait();
    const float out_scale = mv_stage_x(a, h, xarea);
    const float *xs16 = reinterpret_cast<const float *>(xarea + (size_t)a.cols * 4u);
    float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
    uint32_t cur = 0xffffffffu;
    for (uint32_t j = c.j0 + warp; j < c.j1; j += kMvWarps) {
        const uint32_t k = (j - c.j0) / a.st, ri = k % a.nslot;
        uint32_t ok = 1u;
        if (lane == 0) ok = mbar_wait(&h->full[ri], (k / a.nslot) & 1u, err) ? 1u : 0u;
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) return false;
        const uint32_t js = c.j0 + k * a.st, je = min(c.j1, js + a.st);
        Portion pr[kMvMaxPortions];
        const uint32_t np = slot_portions(a, c.seg, js, je, pr);
        Portion q = pr[0];
#pragma unroll
        for (int u = 1; u < kMvMaxPortions; ++u)
            if ((uint32_t)u < np && j >= pr[u].j) q = pr[u];
        const uint32_t b = q.b0 + (j - q.j);
        if (q.t != cur) {
            if (cur != 0xffffffffu) mv_flush(a, h, c, cur, acc, out_scale, best);
            cur = q.t;
            acc[0][0] = acc[0][1] = acc[1][0] = acc[1][1] = 0.f;
        }
        const MvSeg &sg = a.seg[q.s];
        const uint32_t bb = mv_bb(sg.type);
        const uint8_t *slot = ring + (size_t)ri * a.slot_bytes + q.off + (b - q.b0) * bb;
        const uint32_t l0 = (uint32_t)(reinterpret_cast<uintptr_t>(run_row(a, q, (uint32_t)g)) & 15u);
        const uint32_t l1 = (uint32_t)(reinterpret_cast<uintptr_t>(run_row(a, q, (uint32_t)g + 8u)) & 15u);
        const uint8_t *r0[1] = {slot + (uint32_t)g * q.stride + l0};
        const uint8_t *r1[1] = {slot + ((uint32_t)g + 8u) * q.stride + l1};
        const uint8_t *xb[1] = {xarea + (size_t)b * 1024u};
        const float *xs[1] = {xs16 + (size_t)b * 16u};
        float o0[1] = {0.f}, o1[1] = {0.f};
        if (sg.type == 12u) q4k_tiles<1, true>(r0, r1, xb, xs, g, t4, o0, o1);
        else q6k_tiles<1, true>(r0, r1, xb, xs, g, t4, o0, o1);
        __syncwarp();
        if (lane == 0) mbar_arrive(&h->empty[ri]);
        if (a.paired && (q.s & 1u)) {
            acc[1][0] += o0[0];
            acc[1][1] += o1[0];
        } else {
            acc[0][0] += o0[0];
            acc[0][1] += o1[0];
        }
    }
    if (cur != 0xffffffffu) mv_flush(a, h, c, cur, acc, out_scale, best);
    return true;
}

__global__ void __launch_bounds__(kMvThreads, 2) mv_kernel(const __grid_constant__ MvArgs a)
{
    extern __shared__ __align__(128) uint8_t smem[];
    MvHdr *h = reinterpret_cast<MvHdr *>(smem);
    uint8_t *tiles = smem + mv_hdr_bytes();
    uint8_t *xarea = tiles + mv_tile_bytes(a.tslots);
    uint8_t *ring = xarea + mv_x_bytes(a.cols);
    const MvCta c = a.cta[blockIdx.x];
    volatile uint32_t *err = a.status;
    if (threadIdx.x == 0) {
        h->tcnt = reinterpret_cast<uint32_t *>(tiles);
        h->tpart = reinterpret_cast<float *>(tiles + mv_tcnt_bytes(a.tslots));
        for (uint32_t i = 0; i < a.nslot; ++i) {
            mbar_init(&h->full[i], 1u);
            mbar_init(&h->empty[i], a.st);
        }
        for (uint32_t i = 0; i < a.tslots; ++i) h->tcnt[i] = 0u;
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch();
    if (threadIdx.x >= (uint32_t)kMvWarps * 32u) {
        mv_producer(a, h, ring, c, err);
        return;
    }
    MvBest best{-FLT_MAX, 0xffffffffu};
    mv_consumer(a, h, xarea, ring, c, err, best);
    if (a.epi != MV_LOGITS) return;
    // one (max, row) per CTA; the argmax kernel reduces them
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best.v, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, best.i, o);
        if (ov > best.v || (ov == best.v && oi < best.i)) { best.v = ov; best.i = oi; }
    }
    if (lane == 0) { h->amax[warp] = best.v; h->aidx[warp] = best.i; }
    mv_sync();
    if (threadIdx.x == 0) {
        for (int w = 1; w < kMvWarps; ++w)
            if (h->amax[w] > best.v || (h->amax[w] == best.v && h->aidx[w] < best.i)) { best.v = h->amax[w]; best.i = h->aidx[w]; }
        a.pmax[blockIdx.x] = best.v;
        a.pidx[blockIdx.x] = best.i;
    }
}

// ---------------------------------------------------------- attention ----

struct __align__(16) AttnSmem {
    float4 q[kAttnMaxGroup][32];   // RoPE'd queries of the group (128 dims)
    float4 k[kAttnTile][32];       // staged K rows
    float4 v[kAttnTile][32];       // staged V rows
    float4 knew[32], vnew[32];     // the current token's RoPE'd k and its v
    float cden[kAttnMaxGroup];
    uint32_t flag;
};
// followed by the combine weights cw[splits][kAttnMaxGroup]

__device__ __forceinline__ float4 kv_load4(const void *cache, size_t row, uint32_t c4, bool f16)
{
    if (!f16) return __ldcg(reinterpret_cast<const float4 *>(cache) + row * 32u + c4);
    const uint2 hb = __ldcg(reinterpret_cast<const uint2 *>(cache) + row * 32u + c4);
    const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&hb.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&hb.y));
    return make_float4(a.x, a.y, b.x, b.y);
}

__device__ __forceinline__ float warp_maxf(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Split-K flash-decode over the KV cache (gqa_single_token,
// src/brain_runtime.c:1482-1528), one CTA per (KV head, split). The splits in
// use grow with the context (at least kAttnMinSpan positions each); every
// warp takes one query head of the group: scores one position per lane (q . k
// over 128 dims read in a lane-rotated order, conflict-free), online softmax,
// P.V with lane = 4 output dims. The split holding the current position
// applies RoPE to the fresh k and appends k and v to the cache
// (src/brain_runtime.c:1496-1500). The last split of a KV head to finish
// combines all splits' (max, sum, acc) records.
__global__ void __launch_bounds__(kAttnThreads) attn_kernel(const __grid_constant__ AttnArgs a)
{
    extern __shared__ __align__(16) uint8_t smem_a[];
    AttnSmem &sm = *reinterpret_cast<AttnSmem *>(smem_a);
    float *cw = reinterpret_cast<float *>(smem_a + sizeof(AttnSmem));
    pdl_launch();
    pdl_wait();
    const uint32_t pos = *reinterpret_cast<volatile const uint32_t *>(&a.st->pos);
    if (pos >= a.max_context) {
        if (blockIdx.x == 0 && threadIdx.x == 0) atomicCAS(&a.st->status, kStatusOk, kStatusBadArgument);
        return;
    }
    const uint32_t n = pos + 1u;
    const uint32_t ns = min(a.splits, (n + kAttnMinSpan - 1u) / kAttnMinSpan);
    const uint32_t span = (n + ns - 1u) / ns;
    const uint32_t kvh = blockIdx.x / a.splits, s = blockIdx.x % a.splits;
    if (s >= ns) return;
    const uint32_t group = a.q_heads / a.kv_heads;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t t0 = min(s * span, n), t1 = min(n, t0 + span);
    const bool has_pos = t0 <= pos && pos < t1;
    const bool f16 = a.kv_fp16 != 0u;
    const float scale = 1.0f / sqrtf(128.0f);
    float *qf = reinterpret_cast<float *>(sm.q);
    for (uint32_t i = threadIdx.x; i < group * 64u; i += kAttnThreads) {
        const uint32_t hq = i >> 6, p = i & 63u;
        const float *qh = a.q + (size_t)(kvh * group + hq) * 128u;
        const float qa = __ldcg(qh + p), qb = __ldcg(qh + p + 64u);
        const float2 cs = __ldg(a.rope + (size_t)pos * 64u + p);
        qf[hq * 128u + p] = qa * cs.x - qb * cs.y;   // src/brain_runtime.c:1391-1393
        qf[hq * 128u + p + 64u] = qa * cs.y + qb * cs.x;
    }
    if (has_pos) {
        float *kn = reinterpret_cast<float *>(sm.knew), *vn = reinterpret_cast<float *>(sm.vnew);
        const float *kh = a.k + (size_t)kvh * 128u;
        for (uint32_t p = threadIdx.x; p < 64u; p += kAttnThreads) {
            const float ka = __ldcg(kh + p), kb = __ldcg(kh + p + 64u);
            const float2 cs = __ldg(a.rope + (size_t)pos * 64u + p);
            kn[p] = ka * cs.x - kb * cs.y;
            kn[p + 64u] = ka * cs.y + kb * cs.x;
        }
        for (uint32_t i = threadIdx.x; i < 128u; i += kAttnThreads) vn[i] = __ldcg(a.v + (size_t)kvh * 128u + i);
    }
    __syncthreads();
    if (has_pos && threadIdx.x < 128u) {
        const size_t off = ((size_t)kvh * a.max_context + pos) * 128u + threadIdx.x;
        const float kv = reinterpret_cast<const float *>(sm.knew)[threadIdx.x];
        const float vv = reinterpret_cast<const float *>(sm.vnew)[threadIdx.x];
        if (f16) {
            reinterpret_cast<__half *>(a.k_cache)[off] = __float2half_rn(kv);
            reinterpret_cast<__half *>(a.v_cache)[off] = __float2half_rn(vv);
        } else {
            reinterpret_cast<float *>(a.k_cache)[off] = kv;
            reinterpret_cast<float *>(a.v_cache)[off] = vv;
        }
    }
    float m = -FLT_MAX, l = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    const size_t head_row0 = (size_t)kvh * a.max_context;
    for (uint32_t tb = t0; tb < t1; tb += kAttnTile) {
        const uint32_t te = min(tb + kAttnTile, t1), ce = max(tb, min(te, pos));
        for (uint32_t idx = threadIdx.x; idx < (ce - tb) * 32u; idx += kAttnThreads) {
            const uint32_t r = idx >> 5, c4 = idx & 31u;
            sm.k[r][c4] = kv_load4(a.k_cache, head_row0 + tb + r, c4, f16);
            sm.v[r][c4] = kv_load4(a.v_cache, head_row0 + tb + r, c4, f16);
        }
        if (pos >= tb && pos < te && threadIdx.x < 32u) {
            sm.k[pos - tb][threadIdx.x] = sm.knew[threadIdx.x];
            sm.v[pos - tb][threadIdx.x] = sm.vnew[threadIdx.x];
        }
        __syncthreads();
        if (warp < group) {
            for (uint32_t sb = tb; sb < te; sb += 32u) {
                const uint32_t p = sb + lane;
                const bool valid = p < te;
                float sc = -FLT_MAX;
                if (valid) {
                    float dot = 0.f;
#pragma unroll 8
                    for (uint32_t i = 0; i < 32u; ++i) {
                        const uint32_t d4 = (i + lane) & 31u;
                        const float4 qv = sm.q[warp][d4];
                        const float4 kv = sm.k[p - tb][d4];
                        dot = fmaf(qv.x, kv.x, dot);
                        dot = fmaf(qv.y, kv.y, dot);
                        dot = fmaf(qv.z, kv.z, dot);
                        dot = fmaf(qv.w, kv.w, dot);
                    }
                    sc = dot * scale;
                }
                const float mn = fmaxf(m, warp_maxf(sc));
                const float corr = expf(m - mn);
                const float w = valid ? expf(sc - mn) : 0.f;
                l = l * corr + warp_sum(w);
                acc.x *= corr; acc.y *= corr; acc.z *= corr; acc.w *= corr;
                const uint32_t np = min(32u, te - sb);
                for (uint32_t jj = 0; jj < np; ++jj) {
                    const float wj = __shfl_sync(0xffffffffu, w, (int)jj);
                    const float4 vv = sm.v[sb + jj - tb][lane];
                    acc.x = fmaf(wj, vv.x, acc.x);
                    acc.y = fmaf(wj, vv.y, acc.y);
                    acc.z = fmaf(wj, vv.z, acc.z);
                    acc.w = fmaf(wj, vv.w, acc.w);
                }
                m = mn;
            }
        }
        __syncthreads();
    }
    if (warp < group) {
        float *dst = a.part + (((size_t)kvh * a.splits + s) * group + warp) * kRec;
        reinterpret_cast<float4 *>(dst)[lane] = acc;
        if (lane == 0) { dst[128] = m; dst[129] = l; }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const uint32_t old = atom_acq_rel_add(a.ctr + kvh, 1u);
        sm.flag = (old == ns - 1u) ? 1u : 0u;
        if (sm.flag) a.ctr[kvh] = 0u;
    }
    __syncthreads();
    if (!sm.flag) return;
    __threadfence();
    // combine: weights exp(m_s - M) per split and head, then the weighted sums
    for (uint32_t hq = warp; hq < group; hq += kAttnThreads / 32u) {
        float M = -FLT_MAX;
        for (uint32_t q = lane; q < ns; q += 32u)
            M = fmaxf(M, __ldcg(a.part + (((size_t)kvh * a.splits + q) * group + hq) * kRec + 128u));
        M = warp_maxf(M);
        float den = 0.f;
        for (uint32_t q = lane; q < ns; q += 32u) {
            const float2 ml = __ldcg(reinterpret_cast<const float2 *>(
                a.part + (((size_t)kvh * a.splits + q) * group + hq) * kRec + 128u));
            const float w = expf(ml.x - M);
            cw[q * kAttnMaxGroup + hq] = w;
            den += w * ml.y;
        }
        den = warp_sum(den);
        if (lane == 0) sm.cden[hq] = den;
    }
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < group * 32u; i += kAttnThreads) {
        const uint32_t hq = i >> 5, d4 = i & 31u;
        float4 num = make_float4(0.f, 0.f, 0.f, 0.f);
        for (uint32_t q0 = 0; q0 < ns; q0 += 8u) {
            float4 v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (q0 + j < ns)
                    v[j] = __ldcg(reinterpret_cast<const float4 *>(
                        a.part + (((size_t)kvh * a.splits + q0 + j) * group + hq) * kRec) + d4);
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (q0 + j < ns) {
                    const float w = cw[(q0 + j) * kAttnMaxGroup + hq];
                    num.x = fmaf(w, v[j].x, num.x);
                    num.y = fmaf(w, v[j].y, num.y);
                    num.z = fmaf(w, v[j].z, num.z);
                    num.w = fmaf(w, v[j].w, num.w);
                }
        }
        const float den = sm.cden[hq];
        const float inv = den > 0.f ? 1.0f / den : 0.f;
        reinterpret_cast<float4 *>(a.att + (size_t)(kvh * group + hq) * 128u)[d4] =
            make_float4(num.x * inv, num.y * inv, num.z * inv, num.w * inv);
    }
}

// --------------------------------------------------------- embed, argmax --

// token_embd row of the current token -> x, bit-exact (load_embedding_row,
// src/brain_runtime.c:1311-1332). First kernel of a step: ordinary stream order.
__global__ void __launch_bounds__(256) embed_kernel(const uint8_t *embd, uint64_t row_bytes, uint32_t type,
                                                    uint32_t hidden, uint32_t vocab, float *x, DecState *st)
{
    pdl_launch();
    const uint32_t token = *reinterpret_cast<volatile const uint32_t *>(&st->token);
    if (token >= vocab) {
        if (blockIdx.x == 0 && threadIdx.x == 0) atomicCAS(&st->status, kStatusOk, kStatusBadArgument);
        return;
    }
    const uint32_t be = block_elems(type), bb = block_bytes(type);
    const uint8_t *row = embd + (uint64_t)token * row_bytes;
    const uint32_t i = blockIdx.x * 256u + threadIdx.x;
    if (i < hidden) x[i] = deq_elem(type, row + (i / be) * bb, (int)(i % be));
}

// Greedy pick over the head's per-CTA (max, row) partials, lowest row among
// equal maxima (atlas_sample_token's greedy branch, src/brain_runtime.c:1783);
// then advance the step state.
__global__ void __launch_bounds__(256) argmax_kernel(const float *pmax, const uint32_t *pidx, uint32_t n,
                                                     DecState *st)
{
    __shared__ float bv[8];
    __shared__ uint32_t bi[8];
    pdl_launch();
    pdl_wait();
    float best = -FLT_MAX;
    uint32_t idx = 0xffffffffu;
    for (uint32_t i = threadIdx.x; i < n; i += 256u) {
        const float v = __ldcg(pmax + i);
        const uint32_t k = __ldcg(pidx + i);
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
    st->next_token = idx;
    st->next_logit = best;
    if (st->out_ids && st->step < st->max_steps) st->out_ids[st->step] = idx;
    if (st->advance) {
        st->token = idx;
        st->pos = st->pos + 1u;
        st->step = st->step + 1u;
    }
}

}  // namespace d2
}  // namespace atlas

// ------------------------------------------------------------ launchers ----

using namespace atlas::d2;

namespace {

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

}  // namespace

extern "C" size_t atlas_d2_mv_smem(uint32_t cols, uint32_t nslot, uint32_t slot_bytes, uint32_t tslots)
{
    return (size_t)mv_hdr_bytes() + mv_tile_bytes(tslots) + mv_x_bytes(cols) + (size_t)nslot * slot_bytes;
}

extern "C" size_t atlas_d2_attn_smem(uint32_t splits)
{
    return sizeof(AttnSmem) + (size_t)splits * kAttnMaxGroup * sizeof(float);
}

// Raise the kernels' dynamic shared-memory limits (call before any capture).
extern "C" cudaError_t atlas_d2_setup(size_t mv_smem, size_t attn_smem)
{
    cudaError_t e = cudaFuncSetAttribute(mv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)mv_smem);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)attn_smem);
}

extern "C" cudaError_t atlas_d2_launch_mv(const MvArgs *a, uint32_t grid, cudaStream_t stream)
{
    MvArgs copy = *a;
    void *args[] = {&copy};
    return launch_ex((const void *)mv_kernel, args, dim3(grid), dim3(kMvThreads), a->smem_bytes, stream, a->pdl != 0u);
}

extern "C" cudaError_t atlas_d2_launch_attn(const AttnArgs *a, uint32_t grid, cudaStream_t stream)
{
    AttnArgs copy = *a;
    void *args[] = {&copy};
    return launch_ex((const void *)attn_kernel, args, dim3(grid), dim3(kAttnThreads), atlas_d2_attn_smem(a->splits),
                     stream, true);
}

extern "C" cudaError_t atlas_d2_launch_embed(const uint8_t *embd, uint64_t row_bytes, uint32_t type, uint32_t hidden,
                                             uint32_t vocab, float *x, DecState *st, cudaStream_t stream)
{
    void *args[] = {&embd, &row_bytes, &type, &hidden, &vocab, &x, &st};
    return launch_ex((const void *)embed_kernel, args, dim3((hidden + 255u) / 256u), dim3(256), 0, stream, false);
}

extern "C" cudaError_t atlas_d2_launch_argmax(const float *pmax, const uint32_t *pidx, uint32_t n, DecState *st,
                                              cudaStream_t stream)
{
    void *args[] = {&pmax, &pidx, &n, &st};
    return launch_ex((const void *)argmax_kernel, args, dim3(1), dim3(256), 0, stream, true);
}
