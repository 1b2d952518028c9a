// Graph decode step (sm_100a): the reference's forward_token
// (src/brain_runtime.c:1698-1772) and greedy pick (:1783) as a chain of
// kernels - embed, per layer {mv qkv, attention, mv o, mv gate/up, mv down},
// mv head, argmax - launched with programmatic dependent launch and replayed
// from one CUDA graph per token.
//
// Every kernel first lets its successor launch (griddepcontrol.launch_dependents)
// and only then waits for its predecessor (griddepcontrol.wait). A successor
// CTA becomes resident on an SM as soon as resources there allow - for two
// mv kernels, when the predecessor's CTA on that SM exits (at 128 registers
// per thread the register banks hold one 9-warp mv CTA per SM) - and its
// producer warp starts streaming weights at once: weights never depend on
// the activations, so HBM keeps streaming while other SMs finish the
// predecessor. (A 96-register build that fits two mv CTAs per SM ran the 3B
// step 16 % slower: co-resident CTAs compete for issue slots; caps of 128
// and 168 registers ran it 1.3 % and 1.0 % faster than 112.)
//
// mv kernel (dequant-GEMV, one CTA per SM): a producer warp copies the raw
// Q4_K / Q6_K rows of the CTA's task range into a shared-memory ring with
// 1-D bulk copies of row pairs, placed an odd multiple of 16 bytes apart so
// that the 8 row groups of a warp hit distinct banks. Eight
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

// Loads the step's trace pointer (lane 0 of each warp, early, so that the
// load is long done when the warp records its stamps at the end).
__device__ __forceinline__ uint64_t *trace_ptr(const DecState *st)
{
    if (!st || (threadIdx.x & 31u)) return nullptr;
    return *reinterpret_cast<uint64_t *const volatile *>(&st->trace);
}
// Warp w's stamps into launch `slot`'s record of this CTA (lane 0 only).
__device__ __forceinline__ void trace_done(uint64_t *tr, uint32_t slot, uint64_t t_start, uint64_t t_ready,
                                           uint64_t t_wait = 0, uint64_t t_peers = 0)
{
    if (!tr || blockIdx.x >= kTraceCtas) return;
    const uint32_t warp = threadIdx.x >> 5;
    uint64_t *rec = tr + ((size_t)slot * kTraceCtas + blockIdx.x) * kTraceWords;
    if (warp == 0) {
        rec[0] = t_start;
        rec[1] = t_ready;
        rec[kTraceWords - 2] = t_peers;
        rec[kTraceWords - 1] = t_wait;
    }
    if (warp + 4u < kTraceWords) rec[2 + warp] = global_ns();
}

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
//   MvHdr | tile area: tcnt[tslots], tpart[tslots][2][kMvWarps][kMvRows]
//         | slot descriptors | x area | ring
struct __align__(16) MvHdr {
    uint64_t full[kMvMaxSlots];
    uint64_t empty[kMvMaxSlots];
    double dred[kMvWarps];
    float fred[kMvWarps];
    float amax[kMvWarps];
    uint32_t aidx[kMvWarps];
    uint32_t *tcnt;    // arrivals per open tile slot
    float *tpart;      // per-warp row sums of open tiles
    uint4 *desc;       // [nslot][8] task descriptors
    uint8_t *lead;     // [nslot][kMvMaxPortions][16] copy misalignments
};

__host__ __device__ constexpr uint32_t mv_hdr_bytes() { return align128((uint32_t)sizeof(MvHdr)); }
__host__ __device__ constexpr uint32_t mv_tcnt_bytes(uint32_t tslots) { return (tslots * 4u + 15u) & ~15u; }
// per-warp partial rows of an open tile, rows kTpRow floats apart so that the
// cooperative finish (lane = (warp k, row, segment)) reads distinct banks
constexpr uint32_t kTpRow = kMvRows + 1u;
__host__ __device__ constexpr uint32_t mv_tile_bytes(uint32_t tslots)
{
    return align128(mv_tcnt_bytes(tslots) + tslots * 2u * kMvWarps * kTpRow * 4u);
}
// Per ring slot: one descriptor per task - ring offset of the task's block in
// the run's first copy, copy stride | row stride << 16, tile, segment | run
// << 4 | log2 copies << 8 | block << 16 - and the copies' misalignments.
__host__ __device__ constexpr uint32_t mv_desc_bytes(uint32_t nslot)
{
    return align128(nslot * (kMvMaxSt * 16u + kMvMaxPortions * 16u));
}
// staged input: binary16 hi / lo per element, the 16-element sums, and (mv4_kernel) one 1 / scale per 256-element block
__host__ __device__ constexpr uint32_t mv_x_bytes(uint32_t cols) { return align128(cols * 4u + cols / 16u * 4u + cols / 256u * 4u); }

__device__ __forceinline__ float *tpart_at(const MvHdr *h, uint32_t ts, uint32_t s, uint32_t w)
{
    return h->tpart + ((ts * 2u + s) * kMvWarps + w) * kTpRow;
}

// One (tile, segment) run of n block columns inside a ring slot. A run of
// whole rows (n == nb) is copied as C = seg.copies bulk copies of R = 16 / C
// adjacent rows (the rows are adjacent in memory), a partial run row by row
// (C = 16, R = 1). Copy q sits at off + q * cstride, cstride an odd multiple
// of 16 bytes, its rows rstride (= row_bytes) apart after the copy's
// misalignment lead_q. MMA row m of the tile is row (m % C) * R + m / C: the
// 8 rows an MMA row group reads come from different copies (distinct banks),
// or - where the host saw that rows of one copy already fall in distinct
// banks - from one copy.
struct Portion {
    uint32_t t, s, b0, n, off, cstride, rstride, c, j;   // c = log2 C, j: first task of the run
};

__device__ __forceinline__ uint32_t mv_bb(uint32_t type) { return type == 12u ? 144u : 210u; }

__host__ __device__ constexpr uint32_t ceil16(uint32_t v) { return (v + 15u) & ~15u; }

__device__ __forceinline__ uint32_t log2u(uint32_t v) { return 31u - (uint32_t)__clz(v); }

__device__ __forceinline__ Portion pick(const Portion (&pr)[kMvMaxPortions], uint32_t p)
{
    Portion q = pr[0];
#pragma unroll
    for (int v = 1; v < kMvMaxPortions; ++v)
        if ((uint32_t)v == p) q = pr[v];
    return q;
}

// ----------------------------------------------------------- producer ----

// One pass per ring slot: wait until the slot is free, lay out its runs from
// a (tile, segment, block) cursor (no divisions), write the descriptors of its
// tasks and the copies' misalignments, then every copying lane announces its
// own bytes and issues its bulk copy; lane 0's arrival publishes the
// descriptors. A bulk copy costs tens of nanoseconds of the SM's copy engine
// whatever its size, so whole-row runs go in few large copies.
__device__ void mv_producer(const MvArgs &a, MvHdr *h, uint8_t *ring, const MvCta &c, volatile uint32_t *err)
{
    const uint32_t lane = threadIdx.x & 31u;
    const uint64_t policy = policy_evict_first();
    const uint32_t P = a.paired ? 2u : 1u, TP = a.nb * P;
    const uint32_t L = c.j1 - c.j0, nslots = (L + a.st - 1u) / a.st;
    uint32_t ct = c.j0 / TP, cs = a.paired ? 0u : c.seg, cb = 0u;   // ranges start on a tile
    uint32_t j = 0;                                                 // task position in the range
    for (uint32_t k = 0; k < nslots; ++k) {
        const uint32_t ri = k % a.nslot;
        if (k >= a.nslot) {
            uint32_t ok = 1u;
            if (lane == 0) ok = mbar_wait(&h->empty[ri], ((k / a.nslot) & 1u) ^ 1u, err) ? 1u : 0u;
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
        }
        const uint32_t js = j, je = min(L, js + a.st);
        Portion pr[kMvMaxPortions];
        uint32_t np = 0, off = 0;
#pragma unroll
        for (int q = 0; q < kMvMaxPortions; ++q) {
            if (j >= je) break;
            const MvSeg &sg = a.seg[cs];
            const uint32_t n = min(a.nb - cb, je - j);
            const bool whole = n == a.nb;
            const uint32_t C = whole ? sg.copies : 16u;
            const uint32_t rstride = (uint32_t)sg.row_bytes;
            const uint32_t cstride = whole ? odd16((16u / C) * rstride + 15u) : odd16(n * mv_bb(sg.type) + 15u);
            pr[q] = Portion{ct, cs, cb, n, off, cstride, rstride, log2u(C), j};
            off += C * cstride;
            j += n;
            ++np;
            cb += n;
            if (cb == a.nb) {
                cb = 0u;
                if (a.paired && cs == 0u) {
                    cs = 1u;
                } else {
                    if (a.paired) cs = 0u;
                    ++ct;
                }
            }
        }
        uint8_t *slot = ring + (size_t)ri * a.slot_bytes;
        if (lane < je - js) {
            const uint32_t jt = js + lane;
            uint32_t p = 0;
#pragma unroll
            for (int v = 1; v < kMvMaxPortions; ++v)
                if ((uint32_t)v < np && jt >= pr[v].j) p = (uint32_t)v;
            const Portion q = pick(pr, p);
            const uint32_t b = q.b0 + (jt - q.j);
            const uint32_t base = ri * a.slot_bytes + q.off + (b - q.b0) * mv_bb(a.seg[q.s].type);
            h->desc[ri * kMvMaxSt + lane] =
                make_uint4(base, q.cstride | (q.rstride << 16), q.t, q.s | (p << 4) | (q.c << 8) | (b << 16));
        }
        // lane L: copy L % 16 of runs L / 16 and L / 16 + 2
#pragma unroll
        for (uint32_t u = 0; u < 2; ++u) {
            const uint32_t p = lane / 16u + 2u * u, i = lane % 16u;
            if (p >= np) continue;
            const Portion q = pick(pr, p);
            const uint32_t C = 1u << q.c, R = 16u / C;
            if (i >= C) continue;
            const MvSeg &sg = a.seg[q.s];
            const uint8_t *g = sg.w + (uint64_t)((uint32_t)kMvRows * q.t + i * R) * sg.row_bytes +
                               (uint64_t)q.b0 * mv_bb(sg.type);
            const uint32_t lead = (uint32_t)(reinterpret_cast<uintptr_t>(g) & 15u);
            const uint32_t nbytes = ceil16(lead + (C == 16u ? q.n * mv_bb(sg.type) : R * q.rstride));
            h->lead[(ri * (uint32_t)kMvMaxPortions + p) * 16u + i] = (uint8_t)lead;
            mbar_expect_tx(&h->full[ri], nbytes);
            bulk_g2s_hint(slot + q.off + i * q.cstride, g - lead, nbytes, &h->full[ri], policy);
        }
        __syncwarp();   // descriptors and leads of all lanes before lane 0's release
        if (lane == 0) mbar_arrive(&h->full[ri]);
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
// factor for the row sums: inv_rms / xscale. Pass 1 keeps eight 16-byte loads
// per thread in flight (x comes from L2); pass 2 converts one 4-element group
// per thread and step, the 16-element sums reduced across 4 adjacent lanes.
// q4_order: the CTA's tasks are Q4_K - each 4-element group is stored as
// (x0, x2, x1, x3), the order in which q4k_task pairs the nibbles of a quant
// word (bytes 0 and 2, bytes 1 and 3) without byte permutes.
// W: the staging warps (threads 0 .. 32 W - 1, synchronised on named barrier 1);
// dred / fred: W slots each for the block reductions.
// The partial rows the input staging adds to x, after the wait for the
// preceding kernel: tensor parallel, the preceding row-split projection's
// slots from every rank (once their counter has seen this occurrence), x =
// a.x + slot 0 + slot 1 + ... in rank order; one GPU, the K parts of the
// preceding launch in part order. own0 .. own1: this CTA's share of the sum
// (float4 indices) to write back to xout.
template <int W>
__device__ __forceinline__ void stage_partials(const MvArgs &a, uint32_t n4, uint64_t *t_wait, const float4 *&red,
                                               uint32_t &nred, uint32_t &own0, uint32_t &own1)
{
    if (a.in_part) {
        red = reinterpret_cast<const float4 *>(a.in_part);
        nred = a.in_nparts;
    } else if (a.in_red) {
        if (threadIdx.x == 0) {
            const uint32_t epoch = *reinterpret_cast<volatile const uint32_t *>(&a.dstate->epoch);
            const uint32_t k = epoch * a.seq_mul + a.seq_add;
            wait_counter_sys(reinterpret_cast<const uint32_t *>(a.peer[a.rank] + a.in_cnt), k * a.in_arrivals,
                             a.status);
            if (t_wait) t_wait[1] = global_ns();   // the peers' partial rows have all arrived
        }
        asm volatile("bar.sync 1, %0;" ::"n"(W * 32) : "memory");
        red = reinterpret_cast<const float4 *>(a.peer[a.rank] + a.in_red);
        nred = a.tp;
    } else {
        return;
    }
    own0 = (uint32_t)((uint64_t)n4 * blockIdx.x / gridDim.x);
    own1 = (uint32_t)((uint64_t)n4 * (blockIdx.x + 1u) / gridDim.x);
}

template <int W>
__device__ float mv_stage_x(const MvArgs &a, double *dred, float *fred, uint8_t *xarea, bool q4_order,
                           uint64_t *t_wait = nullptr, uint32_t x_off = 0u)
{
    const uint32_t n4 = a.cols / 4u;
    const bool norm = a.norm_w != nullptr;
    const float4 *xin = reinterpret_cast<const float4 *>(a.x + x_off);
    const float4 *nw = norm ? reinterpret_cast<const float4 *>(a.norm_w + x_off) : nullptr;
    float4 *xf = reinterpret_cast<float4 *>(xarea);
    float mx = 0.f;
    double ss = 0.0;
    constexpr uint32_t kStride = W * 32;
    constexpr int kDepth = 8;
    // the norm weights of the first round do not depend on the preceding
    // kernel: load them before waiting for it
    float4 w[kDepth];
    if (norm) {
#pragma unroll
        for (int j = 0; j < kDepth; ++j) {
            const uint32_t i = threadIdx.x + (uint32_t)j * kStride;
            if (i < n4) w[j] = __ldg(nw + i);
        }
    }
    if (a.pdl) pdl_wait();
    if (t_wait) t_wait[0] = global_ns();
    const float4 *red = nullptr;
    uint32_t nred = 0, own0 = 0, own1 = 0;
    stage_partials<W>(a, n4, t_wait, red, nred, own0, own1);
    for (uint32_t i0 = threadIdx.x; i0 < n4; i0 += kDepth * kStride) {
        float4 v[kDepth];
#pragma unroll
        for (int j = 0; j < kDepth; ++j) {
            const uint32_t i = i0 + (uint32_t)j * kStride;
            if (i < n4) {
                v[j] = __ldcg(xin + i);
                if (norm && i0 != threadIdx.x) w[j] = __ldg(nw + i);
            }
        }
        if (red) {
            for (uint32_t r = 0; r < nred; ++r) {
#pragma unroll
                for (int j = 0; j < kDepth; ++j) {
                    const uint32_t i = i0 + (uint32_t)j * kStride;
                    if (i < n4) {
                        const float4 p = __ldcg(red + (size_t)r * n4 + i);
                        v[j].x += p.x; v[j].y += p.y; v[j].z += p.z; v[j].w += p.w;
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < kDepth; ++j) {
                const uint32_t i = i0 + (uint32_t)j * kStride;
                if (i >= own0 && i < own1 && a.xout) reinterpret_cast<float4 *>(a.xout)[i] = v[j];
            }
        }
        if (a.x_hi) {
            // the rank's slice of the attention output inside its o blocks
#pragma unroll
            for (int j = 0; j < kDepth; ++j) {
                const uint32_t e = 4u * (i0 + (uint32_t)j * kStride);
                if (e + 0u < a.x_lo || e + 0u >= a.x_hi) v[j].x = 0.f;
                if (e + 1u < a.x_lo || e + 1u >= a.x_hi) v[j].y = 0.f;
                if (e + 2u < a.x_lo || e + 2u >= a.x_hi) v[j].z = 0.f;
                if (e + 3u < a.x_lo || e + 3u >= a.x_hi) v[j].w = 0.f;
            }
        }
#pragma unroll
        for (int j = 0; j < kDepth; ++j) {
            const uint32_t i = i0 + (uint32_t)j * kStride;
            if (i >= n4) continue;
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
        if (norm) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    }
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    if (lane == 0) { fred[warp] = mx; dred[warp] = ss; }
    asm volatile("bar.sync 1, %0;" ::"n"(W * 32) : "memory");
    // warp 0 reduces the warps' partials and derives the two scalars once
    if (warp == 0) {
        float m = lane < (uint32_t)W ? fred[lane] : 0.f;
        double t = lane < (uint32_t)W ? dred[lane] : 0.0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            if (norm) t += __shfl_xor_sync(0xffffffffu, t, o);
        }
        __syncwarp();
        if (lane == 0) {
            // exponent capped at 126: rows of tiny values (a SwiGLU output of
            // all-negative gates) keep a finite scale and contribute ~0, as in fp32
            fred[0] = (m > 0.f && isfinite(m)) ? exp2f((float)min(13 - ilogbf(m), 126)) : 1.0f;
            fred[1] = norm ? 1.0f / sqrtf((float)(t / (double)a.cols) + a.eps) : 1.0f;
        }
    }
    asm volatile("bar.sync 1, %0;" ::"n"(W * 32) : "memory");
    const float s = fred[0], inv_rms = fred[1];
    float *xs16 = reinterpret_cast<float *>(xarea + (size_t)a.cols * 4u);
    // n4 is a multiple of 4 (cols % 256 == 0) and the stride of 256 keeps the
    // four groups of a 16-element sum in lanes 4k..4k+3 of one warp
    for (uint32_t i = threadIdx.x; i < n4; i += kStride) {
        const float4 v = xf[i];
        const float e0 = v.x * s, e1 = v.y * s, e2 = v.z * s, e3 = v.w * s;
        float sum = e0 + e1 + e2 + e3;
        // hi = fp16(e), lo = fp16(e - hi), two per conversion; Q4_K CTAs keep
        // the order (x0, x2, x1, x3) of the quant words' nibble pairs
        const float a0 = e0, a1 = q4_order ? e2 : e1, a2 = q4_order ? e1 : e2, a3 = e3;
        const __half2 h01 = __floats2half2_rn(a0, a1), h23 = __floats2half2_rn(a2, a3);
        const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
        const __half2 l01 = __floats2half2_rn(a0 - f01.x, a1 - f01.y), l23 = __floats2half2_rn(a2 - f23.x, a3 - f23.y);
        uint4 pk;
        pk.x = *reinterpret_cast<const uint32_t *>(&h01);
        pk.y = *reinterpret_cast<const uint32_t *>(&h23);
        pk.z = *reinterpret_cast<const uint32_t *>(&l01);
        pk.w = *reinterpret_cast<const uint32_t *>(&l23);
        reinterpret_cast<uint4 *>(xarea)[i] = pk;   // in place: group i is only touched by this thread
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        if ((lane & 3u) == 0u) xs16[i / 4u] = sum;
    }
    asm volatile("bar.sync 1, %0;" ::"n"(W * 32) : "memory");
    return inv_rms / s;
}

// Input staging of mv4_kernel, in 256-element blocks: warp w stages blocks
// w, w + W, ... (lane l holds float4s l and 32 + l of a block): x plus the
// preceding launch's partial rows (stage_partials), times the rms_norm
// weight, scaled by a power of two of the block's own (its largest |x| near
// 2^13), split into binary16 hi / lo, with the 16-element sums. The block
// scales need no CTA-wide maximum: the tasks multiply their block sums by
// isb[b] = 1 / scale, and the rms factor (returned; 1 without a norm) is
// applied when a tile finishes. One CTA barrier, after which every warp
// reduces the warps' sums of squares itself.
// I8 (the Q4_K / Q6_K tasks): instead of binary16 pairs, three int8 planes
// per element, e = x 2^k ~ hi + mid / 128 + lo / 16384 with max|e| of the
// block in [63.75, 127.5) (hi in -127..127, mid and lo in -64..64: the
// residual is below 2^-21 of the block's largest |x|, under the rounding of
// an fp32 dot product of these lengths). A block's 1024 bytes hold 32 chunks
// of 8 elements, each [hi x8][mid x8][lo x8][zero x8]: the integer MMAs'
// B operands are 8-byte loads from one plane (or the zero slice) of a chunk,
// conflict-free per half warp. The 16-element sums are those of e.
template <int W, bool I8 = false>
__device__ float m4_stage_x(const MvArgs &a, double *dred, uint8_t *xarea, bool q4_order, uint64_t *t_wait,
                            uint32_t x_off)
{
    constexpr int kB = 4;   // blocks of a warp per round: 8 float4 loads in flight per lane
    const uint32_t nblk = a.cols / 256u, n4 = a.cols / 4u;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const bool norm = a.norm_w != nullptr;
    const float4 *xin = reinterpret_cast<const float4 *>(a.x + x_off);
    const float4 *nw = norm ? reinterpret_cast<const float4 *>(a.norm_w + x_off) : nullptr;
    float *xs16 = reinterpret_cast<float *>(xarea + (size_t)a.cols * 4u);
    float *isb = xs16 + a.cols / 16u;
    uint4 *xq = reinterpret_cast<uint4 *>(xarea);
    // the norm weights of the first round do not depend on the preceding kernel
    float4 w[kB][2];
    if (norm) {
#pragma unroll
        for (int j = 0; j < kB; ++j) {
            const uint32_t b = warp + (uint32_t)j * W;
            if (b < nblk) {
                w[j][0] = __ldg(nw + 64u * b + lane);
                w[j][1] = __ldg(nw + 64u * b + 32u + lane);
            }
        }
    }
    if (a.pdl) pdl_wait();
    if (t_wait) t_wait[0] = global_ns();
    const float4 *red = nullptr;
    uint32_t nred = 0, own0 = 0, own1 = 0;
    stage_partials<W>(a, n4, t_wait, red, nred, own0, own1);
    double ss = 0.0;
    for (uint32_t b0 = warp; b0 < nblk; b0 += (uint32_t)kB * W) {
        float4 v[kB][2];
#pragma unroll
        for (int j = 0; j < kB; ++j) {
            const uint32_t b = b0 + (uint32_t)j * W;
#pragma unroll
            for (uint32_t hh = 0; hh < 2u; ++hh) {
                const uint32_t i = 64u * b + 32u * hh + lane;
                if (b < nblk) {
                    v[j][hh] = __ldcg(xin + i);
                    if (norm && b0 != warp) w[j][hh] = __ldg(nw + i);
                }
            }
        }
        if (red) {
            for (uint32_t r = 0; r < nred; ++r) {
#pragma unroll
                for (int j = 0; j < kB; ++j) {
                    const uint32_t b = b0 + (uint32_t)j * W;
#pragma unroll
                    for (uint32_t hh = 0; hh < 2u; ++hh) {
                        if (b < nblk) {
                            const float4 p = __ldcg(red + (size_t)r * n4 + 64u * b + 32u * hh + lane);
                            v[j][hh].x += p.x; v[j][hh].y += p.y; v[j][hh].z += p.z; v[j][hh].w += p.w;
                        }
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < kB; ++j) {
                const uint32_t b = b0 + (uint32_t)j * W;
#pragma unroll
                for (uint32_t hh = 0; hh < 2u; ++hh) {
                    const uint32_t i = 64u * b + 32u * hh + lane;
                    if (b < nblk && i >= own0 && i < own1 && a.xout) reinterpret_cast<float4 *>(a.xout)[i] = v[j][hh];
                }
            }
        }
#pragma unroll
        for (int j = 0; j < kB; ++j) {
            const uint32_t b = b0 + (uint32_t)j * W;
            if (b >= nblk) break;   // warp-uniform
            float m = 0.f;
#pragma unroll
            for (uint32_t hh = 0; hh < 2u; ++hh) {
                float4 x = v[j][hh];
                if (a.x_hi) {
                    // the rank's slice of the attention output inside its o blocks
                    const uint32_t e = 4u * (64u * b + 32u * hh + lane);
                    if (e + 0u < a.x_lo || e + 0u >= a.x_hi) x.x = 0.f;
                    if (e + 1u < a.x_lo || e + 1u >= a.x_hi) x.y = 0.f;
                    if (e + 2u < a.x_lo || e + 2u >= a.x_hi) x.z = 0.f;
                    if (e + 3u < a.x_lo || e + 3u >= a.x_hi) x.w = 0.f;
                }
                if (norm) {
                    ss += (double)x.x * (double)x.x;
                    ss += (double)x.y * (double)x.y;
                    ss += (double)x.z * (double)x.z;
                    ss += (double)x.w * (double)x.w;
                    x.x *= w[j][hh].x; x.y *= w[j][hh].y; x.z *= w[j][hh].z; x.w *= w[j][hh].w;
                }
                v[j][hh] = x;
                m = fmaxf(m, fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w))));
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            if constexpr (I8) {
                int k = 0;
                if (m > 0.f && isfinite(m)) {
                    k = 6 - ilogbf(m);   // m 2^k in [64, 128)
                    if (k > 126) k = 126;
                    else if (m * __int_as_float((127 + k) << 23) >= 127.5f) --k;
                }
                const float sc = __int_as_float((127 + k) << 23);
                // A NaN or inf element cannot be carried by the int8 planes (the
                // conversion makes NaN 0 and saturates inf): the block's factor
                // becomes NaN instead, so every row sum over it is NaN, as the
                // fp32 products of the reference are.
                bool nonfinite = false;
#pragma unroll
                for (uint32_t hh = 0; hh < 2u; ++hh) {
                    const float4 x = v[j][hh];
                    nonfinite |= !isfinite(x.x) || !isfinite(x.y) || !isfinite(x.z) || !isfinite(x.w);
                }
                nonfinite = __any_sync(0xffffffffu, nonfinite);
                if (lane == 0) isb[b] = nonfinite ? __int_as_float(0x7fc00000) : __int_as_float((127 - k) << 23);
                uint8_t *xblk = xarea + (size_t)b * 1024u;
#pragma unroll
                for (uint32_t hh = 0; hh < 2u; ++hh) {
                    const uint32_t i = 64u * b + 32u * hh + lane;
                    const float4 x = v[j][hh];
                    const float e[4] = {x.x * sc, x.y * sc, x.z * sc, x.w * sc};
                    int q[3][4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const float h1 = rintf(e[u]);
                        const float r1 = (e[u] - h1) * 128.0f;
                        const float m1 = rintf(r1);
                        const float l1 = rintf((r1 - m1) * 128.0f);
                        q[0][u] = (int)h1;
                        q[1][u] = (int)m1;
                        q[2][u] = (int)l1;
                    }
                    uint32_t pw[3];
#pragma unroll
                    for (int p = 0; p < 3; ++p)
                        pw[p] = __byte_perm(__byte_perm((uint32_t)q[p][0], (uint32_t)q[p][1], 0x0040u),
                                            __byte_perm((uint32_t)q[p][2], (uint32_t)q[p][3], 0x0040u), 0x5410u);
                    // lane pairs (2c, 2c + 1) hold elements 0-3 and 4-7 of chunk
                    // 16 hh + c: the even lane stores the chunk's hi and mid
                    // slices, the odd one lo and zero (one 16-byte store each)
                    const uint32_t o0 = __shfl_xor_sync(0xffffffffu, pw[0], 1);
                    const uint32_t o1 = __shfl_xor_sync(0xffffffffu, pw[1], 1);
                    const uint32_t o2 = __shfl_xor_sync(0xffffffffu, pw[2], 1);
                    const bool odd = lane & 1u;
                    const uint4 st = odd ? make_uint4(o2, pw[2], 0u, 0u) : make_uint4(pw[0], o0, pw[1], o1);
                    *reinterpret_cast<uint4 *>(xblk + (16u * hh + (lane >> 1)) * 32u + 16u * (lane & 1u)) = st;
                    float sum = (e[0] + e[1]) + (e[2] + e[3]);
                    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
                    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
                    if ((lane & 3u) == 0u) xs16[i / 4u] = sum;
                }
                continue;
            }
            // scale 2^k: exponent capped at 126, so that rows of tiny values
            // (a SwiGLU output of all-negative gates) keep a finite scale
            const int k = (m > 0.f && isfinite(m)) ? min(13 - ilogbf(m), 126) : 0;
            const float sc = __int_as_float((127 + k) << 23);
            if (lane == 0) isb[b] = __int_as_float((127 - k) << 23);
#pragma unroll
            for (uint32_t hh = 0; hh < 2u; ++hh) {
                const uint32_t i = 64u * b + 32u * hh + lane;
                const float4 x = v[j][hh];
                const float e0 = x.x * sc, e1 = x.y * sc, e2 = x.z * sc, e3 = x.w * sc;
                float sum = e0 + e1 + e2 + e3;
                // hi = fp16(e), lo = fp16(e - hi); Q4_K CTAs keep the order
                // (x0, x2, x1, x3) of the quant words' nibble pairs
                const float a0 = e0, a1 = q4_order ? e2 : e1, a2 = q4_order ? e1 : e2, a3 = e3;
                const __half2 h01 = __floats2half2_rn(a0, a1), h23 = __floats2half2_rn(a2, a3);
                const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
                const __half2 l01 = __floats2half2_rn(a0 - f01.x, a1 - f01.y), l23 = __floats2half2_rn(a2 - f23.x, a3 - f23.y);
                uint4 pk;
                pk.x = *reinterpret_cast<const uint32_t *>(&h01);
                pk.y = *reinterpret_cast<const uint32_t *>(&h23);
                pk.z = *reinterpret_cast<const uint32_t *>(&l01);
                pk.w = *reinterpret_cast<const uint32_t *>(&l23);
                xq[i] = pk;
                sum += __shfl_xor_sync(0xffffffffu, sum, 1);
                sum += __shfl_xor_sync(0xffffffffu, sum, 2);
                if ((lane & 3u) == 0u) xs16[i / 4u] = sum;
            }
        }
    }
    if (norm) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) dred[warp] = ss;
    }
    asm volatile("bar.sync 1, %0;" ::"n"(W * 32) : "memory");
    if (!norm) return 1.0f;
    double t = lane < (uint32_t)W ? dred[lane] : 0.0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    return 1.0f / sqrtf((float)(t / (double)a.cols) + a.eps);
}

// ---------------------------------------------------------- consumers ----

struct MvBest {
    float v;
    uint32_t i;
};

// Epilogue of tile t: lane i < 16 holds row i (v0; paired: v0 = gate, v1 =
// up); `pre` is the row's bias (store) or residual (residual add), loaded
// when the warp started the tile.
__device__ __forceinline__ void mv_finish(const MvArgs &a, uint32_t segi, uint32_t t, float v0, float v1, float pre,
                                          uint32_t lane, MvBest &best)
{
    const uint32_t row = (uint32_t)kMvRows * t + lane;
    if (a.epi == MV_SWIGLU) {
        a.seg[0].out[row] = (v0 / (1.0f + expf(-v0))) * v1;   // src/brain_runtime.c:1755-1758
        return;
    }
    const MvSeg &sg = a.seg[segi];
    if (a.epi == MV_RESID) {
        sg.out[row] = pre + v0;   // src/brain_runtime.c:1745, :1762
        return;
    }
    if (a.epi == MV_PART) {
        // this rank's partial row into its slot at every rank (the residual
        // is added by the consumer's staging)
        for (uint32_t p = 0; p < a.tp; ++p)
            reinterpret_cast<float *>(a.peer[p] + a.out_red)[(size_t)a.rank * sg.rows + row] = v0;
        return;
    }
    const float r = sg.bias ? v0 + pre : v0;
    sg.out[row] = r;
    if (a.epi == MV_LOGITS && (r > best.v || (r == best.v && row < best.i))) { best.v = r; best.i = row; }
}

// Epilogue operand of row lane of tile t (lanes < 16), read early.
__device__ __forceinline__ float mv_pre(const MvArgs &a, uint32_t segi, uint32_t t, uint32_t lane)
{
    if (lane >= 16u) return 0.f;
    const MvSeg &sg = a.seg[segi];
    const uint32_t row = (uint32_t)kMvRows * t + lane;
    if (a.epi == MV_RESID) return __ldcg(sg.out + row);
    if (a.epi == MV_STORE && sg.bias) return __ldg(sg.bias + row);
    return 0.f;
}

// Weight row (within the tile) of MMA row m when the run's rows come in
// 1 << c copies: copy m % C, row m / C of the copy.
__device__ __forceinline__ uint32_t mv_wrow(uint32_t m, uint32_t c)
{
    return (m & ((1u << c) - 1u)) * (16u >> c) + (m >> c);
}

// The warp's row sums of tile t are complete (acc[s][0]: MMA row g, acc[s][1]:
// MMA row g + 8 of segment s, this lane's share; lc[s]: the copy layout of
// segment s in this tile - one whole-row run, or partial runs only). Publish them; the last of
// the CTA's warps with tasks in the tile adds them up in warp order and
// finishes the tile.
__device__ void mv_flush(const MvArgs &a, MvHdr *h, const MvCta &c, uint32_t t, const uint32_t (&lc)[2],
                         const float (&acc)[2][2], float out_scale, float pre, MvBest &best)
{
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u, g = lane >> 2;
    const uint32_t P = a.paired ? 2u : 1u, TP = a.nb * P;
    const uint32_t ts = (t - c.j0 / TP) % a.tslots;   // tiles are opened in order
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
            tp[mv_wrow(g, lc[s])] = v0;
            tp[mv_wrow(g + 8u, lc[s])] = v1;
        }
    }
    const uint32_t expect = min(TP, (uint32_t)kMvWarps);
    __syncwarp();
    uint32_t last = 0;
    if (lane == 0) {
        __threadfence_block();
        last = (atomicAdd(&h->tcnt[ts], 1u) + 1u == expect) ? 1u : 0u;
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) return;
    __threadfence_block();
    const uint32_t i = lane & 15u;
    float v[2] = {0.f, 0.f};
    const uint32_t w0 = (t * TP - c.j0) % kMvWarps;
#pragma unroll
    for (uint32_t s = 0; s < 2; ++s) {
        if (s >= P) break;
        const volatile float *tp = tpart_at(h, ts, s, 0) + i;
#pragma unroll
        for (uint32_t w = 0; w < (uint32_t)kMvWarps; ++w)
            if (TP >= (uint32_t)kMvWarps || ((w + kMvWarps - w0) % kMvWarps) < TP) v[s] += tp[w * kTpRow];
        v[s] *= out_scale;
    }
    __syncwarp();
    if (lane == 0) h->tcnt[ts] = 0u;
    if (lane < 16u) mv_finish(a, c.seg, t, v[0], v[1], pre, lane, best);
}

__device__ __forceinline__ void ldmatrix_x4(const void *p, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(smem_addr(p)));
}

// Address of MMA row m of a run's block: copy m % C at cstride, row m / C
// of the copy at rstride (Q4_K rows are 16-byte aligned: no misalignment).
__device__ __forceinline__ const uint8_t *q4_row(const uint8_t *blk, uint32_t m, uint32_t lc, uint32_t cstride,
                                                 uint32_t rstride)
{
    return blk + (m & ((1u << lc) - 1u)) * cstride + (m >> lc) * rstride;
}

// One Q4_K task (16 rows x 256 elements) for lane (g, t): MMA rows g and
// g + 8 (q4_row). The arithmetic of q4k_tiles (tc_tiles.cuh); the 128 quant
// bytes of the rows come in with four ldmatrix.x4 (a matrix = 8 rows x 16
// bytes), which hand lane (g, t) word t of each 16-byte chunk of its rows:
// exactly the A-fragment word.
__device__ __forceinline__ void q4k_task(const uint8_t *blk, uint32_t lc, uint32_t cstride, uint32_t rstride,
                                         const uint8_t *xb, const float *xs, uint32_t lane, float &o0, float &o1)
{
    const uint32_t g = lane >> 2, t = lane & 3u;
    uint32_t W[8][2];
    {
        // lane i addresses row i & 7 of matrix i >> 3 = (row half, chunk pair)
        const uint32_t m = lane >> 3;
        const uint8_t *rb = q4_row(blk, (lane & 7u) + 8u * (m & 1u), lc, cstride, rstride) + 16u + 16u * (m >> 1);
#pragma unroll
        for (int q = 0; q < 4; ++q)
            ldmatrix_x4(rb + 32u * (uint32_t)q, W[2 * q][0], W[2 * q][1], W[2 * q + 1][0], W[2 * q + 1][1]);
    }
    float dsc[2][2], dmn[2][2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const uint4 hd = *reinterpret_cast<const uint4 *>(q4_row(blk, g + 8u * (uint32_t)r, lc, cstride, rstride));
        const float d = h2f((uint16_t)(hd.x & 0xffffu)), dm = h2f((uint16_t)(hd.x >> 16));
        const uint32_t sh = 8u * t;
        const uint32_t y = (hd.y >> sh) & 255u, z = (hd.z >> sh) & 255u, w = (hd.w >> sh) & 255u;
        dsc[r][0] = d * u2f_small(y & 63u);                        // sub-block j = t
        dmn[r][0] = dm * u2f_small(z & 63u);
        dsc[r][1] = d * u2f_small((w & 15u) | ((y >> 6) << 4));    // j = t + 4
        dmn[r][1] = dm * u2f_small((w >> 4) | ((z >> 6) << 4));
    }
    const float zero[4] = {0.f, 0.f, 0.f, 0.f};
    const uint32_t podd = (g & 1u) * 8u;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        float dlo[4], dhi[4];
#pragma unroll
        for (int hp = 0; hp < 2; ++hp) {
            // 16-bit lanes straight from the quant words: bytes (0, 2) and
            // (1, 3) of each word (the x groups are staged in that order);
            // low nibbles as subnormals q 2^-24, high nibbles in place as
            // 16 q 2^-24 (exact; the 16 is taken out with the scale)
            const uint32_t w0 = W[2 * c + hp][0], w1 = W[2 * c + hp][1];
            const uint32_t v0 = w0 >> 8, v1 = w1 >> 8;
            const uint2 blo = *reinterpret_cast<const uint2 *>(xb + (16u * c + 4u * hp + t) * 16u + podd);
            const uint2 bhi = *reinterpret_cast<const uint2 *>(xb + (16u * c + 8u + 4u * hp + t) * 16u + podd);
            const uint32_t kl = 0x000f000fu, kh = 0x00f000f0u;
            if (hp == 0) {
                mma16816(dlo, w0 & kl, w1 & kl, v0 & kl, v1 & kl, blo, zero);
                mma16816(dhi, w0 & kh, w1 & kh, v0 & kh, v1 & kh, bhi, zero);
            } else {
                const float clo[4] = {dlo[0], dlo[1], dlo[2], dlo[3]};
                const float chi[4] = {dhi[0], dhi[1], dhi[2], dhi[3]};
                mma16816(dlo, w0 & kl, w1 & kl, v0 & kl, v1 & kl, blo, clo);
                mma16816(dhi, w0 & kh, w1 & kh, v0 & kh, v1 & kh, bhi, chi);
            }
        }
        // this lane's sub-block in chunk c, if any: j = 2c + (t & 1) with (c & 1) == (t >> 1)
        if ((uint32_t)(c & 1) == (t >> 1)) {
            const int slot = c >> 1, j = 2 * c + (int)(t & 1u);
            const float *D = (t & 1u) ? dhi : dlo;
            const float unit = (t & 1u) ? kTwo24 * 0.0625f : kTwo24;   // high nibbles came as 16 q
            const float sx = xs[2 * j] + xs[2 * j + 1];
            o0 += dsc[0][slot] * ((D[0] + D[1]) * unit) - dmn[0][slot] * sx;
            o1 += dsc[1][slot] * ((D[2] + D[3]) * unit) - dmn[1][slot] * sx;
        }
    }
}

// Consumer warp w: positions w + 8m of the CTA's task order - task u = w % st
// of every (8 / st)-th slot starting at slot w / st when st <= 8, tasks w and
// w + 8 of every slot when st = 16; the producer's descriptor gives the
// task's tile, block and place in the ring.
// Returns false after a failed wait (status recorded).
__device__ bool mv_consumer(const MvArgs &a, MvHdr *h, uint8_t *xarea, const uint8_t *ring, const MvCta &c,
                            volatile uint32_t *err, MvBest &best)
{
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const int g = (int)(lane >> 2), t4 = (int)(lane & 3u);
    // waits for the preceding kernel; a CTA's tasks are all of its segment's type
    const float out_scale = mv_stage_x<kMvWarps>(a, h->dred, h->fred, xarea, a.seg[c.seg].type == 12u, nullptr, a.seg[c.seg].x_off);
    const float *xs16 = reinterpret_cast<const float *>(xarea + (size_t)a.cols * 4u);
    const uint32_t per = a.st > (uint32_t)kMvWarps ? a.st / kMvWarps : 1u;    // tasks per slot visit
    const uint32_t step = a.st > (uint32_t)kMvWarps ? 1u : kMvWarps / a.st, u = warp % a.st;
    uint32_t ri = warp / a.st, ph = 0, qi = 0;
    while (ri >= a.nslot) { ri -= a.nslot; ph ^= 1u; }
    float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
    uint32_t cur = 0xffffffffu, cur_lc[2] = {0u, 0u};
    float pre = 0.f;
    uint32_t ready = 0u;        // lane 0: this slot's copies were already seen complete
    const uint32_t L = c.j1 - c.j0;
    for (uint32_t i = warp; i < L; i += kMvWarps) {   // task positions w + 8m
        uint32_t ok = 1u;
        if (qi == 0u && lane == 0 && !ready) ok = mbar_wait(&h->full[ri], ph, err) ? 1u : 0u;
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) return false;
        const uint4 dsc = h->desc[ri * kMvMaxSt + u + (uint32_t)kMvWarps * qi];
        const uint32_t t = dsc.z, s = dsc.w & 15u, run = (dsc.w >> 4) & 15u, lc = (dsc.w >> 8) & 15u, b = dsc.w >> 16;
        const uint32_t cstride = dsc.y & 0xffffu, rstride = dsc.y >> 16;
        // probe the next slot now; the answer is used one task later
        uint32_t rn = ri + step, pn = ph;
        while (rn >= a.nslot) {
            rn -= a.nslot;
            pn ^= 1u;
        }
        // a warp's last task of this slot visit releases the slot
        const bool last = qi + 1u == per || i + kMvWarps >= L;
        if (qi == 0u) {
            ready = 0u;
            if (lane == 0 && i + per * kMvWarps < L) ready = mbar_test(&h->full[rn], pn) ? 1u : 0u;
        }
        if (t != cur) {
            if (cur != 0xffffffffu) mv_flush(a, h, c, cur, cur_lc, acc, out_scale, pre, best);
            cur = t;
            acc[0][0] = acc[0][1] = acc[1][0] = acc[1][1] = 0.f;
            pre = mv_pre(a, c.seg, t, lane);
        }
        // a segment of a tile comes as one whole run or as partial runs only
        if (a.paired && (s & 1u)) cur_lc[1] = lc;
        else cur_lc[0] = lc;
        const uint8_t *blk = ring + dsc.x;
        const uint8_t *xb = xarea + (size_t)b * 1024u;
        const float *xs = xs16 + (size_t)b * 16u;
        float o0 = 0.f, o1 = 0.f;
        if (a.seg[s].type == 12u) {
            q4k_task(blk, lc, cstride, rstride, xb, xs, lane, o0, o1);
        } else {
            const uint8_t *ld = h->lead + (ri * (uint32_t)kMvMaxPortions + run) * 16u;
            const uint32_t m0 = (uint32_t)g, m1 = (uint32_t)g + 8u, cm = (1u << lc) - 1u;
            const uint8_t *r0[1] = {blk + (m0 & cm) * cstride + ld[m0 & cm] + (m0 >> lc) * rstride};
            const uint8_t *r1[1] = {blk + (m1 & cm) * cstride + ld[m1 & cm] + (m1 >> lc) * rstride};
            const uint8_t *xbs[1] = {xb};
            const float *xss[1] = {xs};
            float p0[1] = {0.f}, p1[1] = {0.f};
            q6k_tiles<1, true>(r0, r1, xbs, xss, g, t4, p0, p1);
            o0 = p0[0];
            o1 = p1[0];
        }
        __syncwarp();
        if (last && lane == 0) mbar_arrive(&h->empty[ri]);
        if (a.paired && (s & 1u)) {
            acc[1][0] += o0;
            acc[1][1] += o1;
        } else {
            acc[0][0] += o0;
            acc[0][1] += o1;
        }
        if (last) {
            ri = rn;
            ph = pn;
            qi = 0u;
        } else {
            ++qi;
        }
    }
    if (cur != 0xffffffffu) mv_flush(a, h, c, cur, cur_lc, acc, out_scale, pre, best);
    return true;
}

__global__ void __maxnreg__(128) mv_kernel(const __grid_constant__ MvArgs a)
{
    extern __shared__ __align__(128) uint8_t smem[];
    MvHdr *h = reinterpret_cast<MvHdr *>(smem);
    uint8_t *tiles = smem + mv_hdr_bytes();
    uint8_t *descs = tiles + mv_tile_bytes(a.tslots);
    uint8_t *xarea = descs + mv_desc_bytes(a.nslot);
    uint8_t *ring = xarea + mv_x_bytes(a.cols);
    const MvCta c = a.cta[blockIdx.x];
    volatile uint32_t *err = a.status;
    // a consumer waits for a slot kMvWarps / st slots after its previous one:
    // with fewer ring entries its parity wait would alias an older phase
    if (a.st == 0u || a.st > kMvMaxSt || a.nslot > (uint32_t)kMvMaxSlots || a.nslot * a.st < (uint32_t)kMvWarps) {
        if (threadIdx.x == 0) atomicCAS(a.status, kStatusOk, kStatusBadArgument);
        return;
    }
    if (threadIdx.x == 0) {
        h->tcnt = reinterpret_cast<uint32_t *>(tiles);
        h->tpart = reinterpret_cast<float *>(tiles + mv_tcnt_bytes(a.tslots));
        h->desc = reinterpret_cast<uint4 *>(descs);
        h->lead = descs + a.nslot * kMvMaxSt * 16u;
        for (uint32_t i = 0; i < a.nslot; ++i) {
            mbar_init(&h->full[i], 1u);
            mbar_init(&h->empty[i], min(a.st, (uint32_t)kMvWarps));   // one arrival per warp with tasks in it
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
    if (a.epi == MV_PART) {
        // every pushing thread orders its own remote stores, then one arrival
        // per CTA at every rank (lane p of warp 0 at rank p)
        __threadfence_system();
        mv_sync();
        if (threadIdx.x < a.tp) red_release_sys_add(reinterpret_cast<uint32_t *>(a.peer[threadIdx.x] + a.out_cnt), 1u);
        return;
    }
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
    if (warp != 0u) return;
    for (int w = 1; w < kMvWarps; ++w)
        if (h->amax[w] > best.v || (h->amax[w] == best.v && h->aidx[w] < best.i)) { best.v = h->amax[w]; best.i = h->aidx[w]; }
    if (a.tp > 1u) {
        // (max, global row) into this rank's slot at every rank: lane p
        // stores at rank p and releases there
        if (lane < a.tp) {
            reinterpret_cast<float *>(a.peer[lane] + a.out_red)[a.rank * kTpPStride + blockIdx.x] = best.v;
            reinterpret_cast<uint32_t *>(a.peer[lane] + a.out_red + a.tp * kTpPStride * 4u)[a.rank * kTpPStride +
                                                                                           blockIdx.x] =
                a.row_base + best.i;
            red_release_sys_add(reinterpret_cast<uint32_t *>(a.peer[lane] + a.out_cnt), 1u);
        }
    } else if (lane == 0) {
        a.pmax[blockIdx.x] = best.v;
        a.pidx[blockIdx.x] = best.i;
    }
}

// ------------------------------------------------------------ mv4 kernel ----
//
// Every warp owns the tasks [start(w), start(w + 1)) of the CTA's range,
// start(w) = j0 + floor(w L / W): consecutive blocks of the same row tile, so
// a warp sums a tile's blocks in registers and finishes it alone unless its
// range begins or ends inside the tile. A tile shared by warps wa..wb is
// finished by the last of them to arrive, which adds the warps' partial rows
// in warp order (a fixed order: the result does not depend on timing).
//
// Copies: each warp keeps nslot - 1 tasks in flight in its own ring; the
// first nslot - 1 are issued before the wait for the preceding kernel (the
// weights never depend on it), so they stream while x is staged. Task
// cursors advance incrementally and every lane's copy offsets come from a
// table built once per CTA, so the loop has no divisions.

struct __align__(16) M4Hdr {
    double dred[kM4Warps];
    float fred[kM4Warps];
    float amax[kM4Warps];
    uint32_t aidx[kM4Warps];
    uint32_t cnt[kM4Warps];     // arrivals at a shared tile, indexed by its first warp
    uint32_t wstart[kM4Warps];  // first task of each warp
    uint2 cp[8][32];            // per (copy i, lane): source offset in the block's rows, slot offset
};
// partial rows of shared tiles: [warp][first / last tile][segment][16]
constexpr uint32_t kM4PartBytes = kM4Warps * 2u * 2u * 16u * 4u;

__host__ __device__ constexpr uint32_t m4_hdr_bytes() { return align128((uint32_t)sizeof(M4Hdr)); }
__host__ __device__ constexpr uint32_t m4_smem_bytes(uint32_t cols, uint32_t warps, uint32_t nslot, uint32_t slot_bytes)
{
    return m4_hdr_bytes() + kM4PartBytes + mv_x_bytes(cols) + warps * nslot * slot_bytes;
}

template <int W>
__device__ __forceinline__ void m4_sync() { asm volatile("bar.sync 1, %0;" ::"n"(W * 32) : "memory"); }

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, uint64_t policy)
{
    asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "l"(policy)
                 : "memory");
}
__device__ __forceinline__ void cp_async16_plain(uint32_t dst, const void *src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void m4_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// First task of warp w of weff (w = weff gives the range's end).
// (32-bit arithmetic: a CTA holds far fewer than 2^27 tasks.)
__device__ __forceinline__ uint32_t m4_start(uint32_t j0, uint32_t L, uint32_t weff, uint32_t w)
{
    return j0 + w * L / weff;
}
// The warp whose range holds task j.
__device__ __forceinline__ uint32_t m4_warp_of(uint32_t j0, uint32_t L, uint32_t weff, uint32_t j)
{
    return ((j - j0 + 1u) * weff + L - 1u) / L - 1u;
}

// Task cursor: row tile t, segment s (0 / 1 of a pair), block column b.
struct M4Cur {
    uint32_t t, s, b;
};
__device__ __forceinline__ void m4_next(M4Cur &c, uint32_t nb, bool paired)
{
    if (++c.b == nb) {
        c.b = 0u;
        if (paired && c.s == 0u) {
            c.s = 1u;
        } else {
            c.s = 0u;
            ++c.t;
        }
    }
}

// The CTA's operands of one kind: all its tasks share the type and row length.
struct M4Seg {
    const uint8_t *w0, *w1;     // segment (pair: gate, up) row 0
    uint32_t rb, bb, q4;        // row bytes, block bytes, Q4_K?
    uint32_t ncp;               // copies per lane per task
};

__device__ __forceinline__ const uint8_t *m4_block(const M4Seg &g, const M4Cur &c)
{
    return (c.s ? g.w1 : g.w0) + (uint64_t)(16u * c.t) * g.rb + c.b * g.bb;
}

// Slot row of MMA row m of a Q4_K task: rows 1 <-> 2 of every 4 swapped, so
// that the two rows (2i, 2i + 1) a quarter warp reads with its 16-byte quant
// loads sit two rows (288 bytes, two 16-byte bank groups) apart: with rows
// 144 bytes apart in order, rows one apart put a lane pair's adjacent bank
// groups onto the next row's and the loads conflicted 2-way.
__host__ __device__ constexpr uint32_t q4_slot_row(uint32_t m) { return ((m + 1u) & 2u) ? m ^ 3u : m; }

// Issue the copies of one task (16 rows x one block) into a slot: Q4_K 144
// chunks (5 per lane, the last by lanes 0-15), Q6_K 224 (7 per lane).
template <bool Q4>
__device__ __forceinline__ void m4_issue(const M4Seg &g, const M4Hdr *h, const M4Cur &c, uint32_t slot, uint32_t lane,
                                         uint64_t policy)
{
    const uint8_t *base = m4_block(g, c);
#pragma unroll
    for (uint32_t i = 0; i < (Q4 ? 5u : 7u); ++i) {
        const uint2 e = h->cp[i][lane];
        if (Q4) {
            if (i < 4u || lane < 16u) cp_async16(slot + e.y, base + e.x, policy);
        } else {
            // the 16-byte boundary at or below the row's block, plus the chunk's offset
            const uint8_t *win =
                reinterpret_cast<const uint8_t *>(reinterpret_cast<uintptr_t>(base + e.x) & ~uintptr_t(15));
            cp_async16(slot + (e.y & 0xffffu), win + (e.y >> 16), policy);
        }
    }
}

// Rows g and g + 8 of a tile's partial sums (this lane's share, summed over
// the 4 lanes of a row) -> lane i < 16 holds row i.
__device__ __forceinline__ float m4_rows(float v0, float v1, uint32_t lane)
{
    v0 += __shfl_xor_sync(0xffffffffu, v0, 1);
    v0 += __shfl_xor_sync(0xffffffffu, v0, 2);
    v1 += __shfl_xor_sync(0xffffffffu, v1, 1);
    v1 += __shfl_xor_sync(0xffffffffu, v1, 2);
    const uint32_t src = 4u * (lane & 7u);
    const float a0 = __shfl_sync(0xffffffffu, v0, src), a1 = __shfl_sync(0xffffffffu, v1, src);
    return (lane & 8u) ? a1 : a0;
}

// Finish tile t after this warp's last task in it: alone (wa == wb), or as
// one of the warps wa..wb sharing it (partials in shared memory; the last to
// arrive adds them in warp order). A tile that other CTAs hold tasks of too
// (the CTA's range starts or ends inside it) is then finished by the last of
// those CTAs to arrive, which adds their partial rows in CTA order.
__device__ __forceinline__ void m4_flush_body(const MvArgs &a, M4Hdr *h, float *part, const MvCta &c, uint32_t t,
                                              uint32_t tj0, uint32_t wa, uint32_t wb, uint32_t my0, float a00,
                                              float a01, float a10, float a11, float out_scale, MvBest &best)
{
    const uint32_t seg = c.seg;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    float r0 = m4_rows(a00, a01, lane);
    float r1 = a.paired ? m4_rows(a10, a11, lane) : 0.f;
    if (wa != wb) {
        // slot 0: the tile where this warp's range starts; slot 1: where it ends
        const uint32_t which = my0 >= tj0 ? 0u : 1u;
        float *pp = part + (warp * 2u + which) * 32u;
        if (lane < 16u) {
            pp[lane] = r0;
            pp[16u + lane] = r1;
        }
        __syncwarp();
        uint32_t last = 0;
        if (lane == 0) {
            __threadfence_block();
            last = (atomicAdd(&h->cnt[wa], 1u) + 1u == wb - wa + 1u) ? 1u : 0u;
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (!last) return;
        __threadfence_block();
        r0 = r1 = 0.f;
        const uint32_t i = lane & 15u;
        for (uint32_t w = wa; w <= wb; ++w) {
            const uint32_t ww = (w > wa || h->wstart[wa] >= tj0) ? 0u : 1u;
            const volatile float *q = part + (w * 2u + ww) * 32u;
            r0 += q[i];
            r1 += q[16u + i];
        }
    }
    r0 *= out_scale;
    r1 *= out_scale;
    const uint32_t TPn = a.nb * (a.paired ? 2u : 1u);
    if (tj0 < c.j0 || tj0 + TPn > c.j1) {
        // t is this CTA's first tile when its range starts inside t (then
        // slot 0; also when the range lies inside t), else its last (slot 1)
        const bool first = tj0 <= c.j0, last = tj0 + TPn >= c.j1;
        const uint32_t ca = first ? c.ca : blockIdx.x, cb = last ? c.cb : blockIdx.x;
        float *gp = a.xpart + ((size_t)blockIdx.x * 2u + (first ? 0u : 1u)) * 32u;
        if (lane < 16u) {
            __stcg(gp + lane, r0);
            __stcg(gp + 16u + lane, r1);
            __threadfence();
        }
        __syncwarp();
        uint32_t fin = 0;
        if (lane == 0) fin = atomicAdd(a.xcnt + ca, 1u) + 1u == cb - ca + 1u ? 1u : 0u;
        fin = __shfl_sync(0xffffffffu, fin, 0);
        if (!fin) return;
        __threadfence();
        r0 = r1 = 0.f;
        const uint32_t i = lane & 15u;
        for (uint32_t k = ca; k <= cb; ++k) {
            // t is CTA k's first tile exactly when k's range starts inside it
            const float *q = a.xpart + ((size_t)k * 2u + (a.cta[k].j0 >= tj0 ? 0u : 1u)) * 32u;
            r0 += __ldcg(q + i);
            r1 += __ldcg(q + 16u + i);
        }
        // back to zero for the next launch, whose CTAs arrive only after this grid is complete
        if (lane == 0) a.xcnt[ca] = 0u;
    }
    const float pre = mv_pre(a, seg, t, lane);
    if (lane < 16u) mv_finish(a, seg, t, r0, r1, pre, lane, best);
}

// Out of line for the Q4_K / Q6_K kernels (code size); the other types'
// kernels inline the body.
__device__ __noinline__ void m4_flush(const MvArgs &a, M4Hdr *h, float *part, const MvCta &c, uint32_t t, uint32_t tj0,
                                      uint32_t wa, uint32_t wb, uint32_t my0, float a00, float a01, float a10,
                                      float a11, float out_scale, MvBest &best)
{
    m4_flush_body(a, h, part, c, t, tj0, wa, wb, my0, a00, a01, a10, a11, out_scale, best);
}

// 16 bytes at a 2-byte-aligned shared-memory address, as four words: five
// aligned loads and a funnel shift by the misalignment (0 or 16 bits).
__device__ __forceinline__ void ld16_u2(const uint8_t *p, uint32_t (&w)[4])
{
    const uintptr_t ad = reinterpret_cast<uintptr_t>(p);
    const uint32_t *q = reinterpret_cast<const uint32_t *>(ad & ~uintptr_t(3));
    const uint32_t sh = (uint32_t)(ad & 3u) * 8u;
    uint32_t v[5];
#pragma unroll
    for (int i = 0; i < 5; ++i) v[i] = q[i];
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = __funnelshift_r(v[i], v[i + 1], sh);
}

// 8 / 16 bytes at byte offset `off` (2-byte aligned) of a 4-byte-aligned
// shared-memory base: three / five aligned word loads and funnel shifts by
// the misalignment (0 or 16 bits). The offset is applied to the pointer, so
// the loads stay shared-memory loads with 32-bit addresses.
__device__ __forceinline__ uint2 ld8_at(const uint8_t *base, uint32_t off)
{
    const uint32_t *q = reinterpret_cast<const uint32_t *>(base + (off & ~3u));
    const uint32_t sh = (off & 3u) * 8u;
    const uint32_t v0 = q[0], v1 = q[1], v2 = q[2];
    return make_uint2(__funnelshift_r(v0, v1, sh), __funnelshift_r(v1, v2, sh));
}
__device__ __forceinline__ void ld16_at(const uint8_t *base, uint32_t off, uint32_t (&w)[4])
{
    const uint32_t *q = reinterpret_cast<const uint32_t *>(base + (off & ~3u));
    const uint32_t sh = (off & 3u) * 8u;
    uint32_t v[5];
#pragma unroll
    for (int i = 0; i < 5; ++i) v[i] = q[i];
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = __funnelshift_r(v[i], v[i + 1], sh);
}

// d += A (16 x 32, u8, row) * B (32 x 8, s8, col), s32 accumulators
// (lane (g, t): a0 = A[g][4t..4t+3], a1 = A[g+8][4t..], a2 = A[g][16+4t..],
// a3 = A[g+8][16+4t..]; b.x = B[4t..4t+3][g], b.y = B[16+4t..][g];
// d = D[g][2t], D[g][2t+1], D[g+8][2t], D[g+8][2t+1]).
__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint2 b)
{
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b.x), "r"(b.y));
}

// Integer-MMA tasks (16 rows x one 256-element block) over the int8 planes of
// m4_stage_x<W, true>. In one MMA, lanes t = 0, 1 of a row group carry the
// k slots of one scale group and lanes t = 2, 3 those of another; B column
// n holds plane n & 3 (hi, mid, lo, zero) of group n >> 2's elements and
// zero elsewhere, so accumulator columns 2t, 2t + 1 of lane t end as exact
// integer sums of its own group: (hi, mid) for even t, (lo, -) for odd t.
// The group scales are applied in integers (exact: |sums| < 2^31), the block
// scale d, the plane units and the offsets in fp32 once per task. xl: this
// lane's B base in the staged block, m4_bsel; the caller multiplies the
// results by the block's 1 / 2^k.
//
// B base of lane (g, t): plane g & 3 of the chunk when the lane's column
// belongs to the group its k slots carry ((g >> 2) == (t >> 1)), else a
// zero slice. q6: Q6_K chunk layout (lane t's elements 8t + 32c + 128q),
// else Q4_K (64 (t >> 1) + 16 (t & 1) + 32 nu + 64 pi, halves of 8), whose
// zero lanes of a half warp all read one slice (a broadcast: distinct zero
// slices there would share banks with each other).
__device__ __forceinline__ uint32_t m4_bsel(uint32_t lane, bool q6)
{
    const uint32_t g = lane >> 2, t = lane & 3u;
    const bool act = (g >> 2) == (t >> 1) && (g & 3u) < 3u;
    if (q6) return 32u * t + 8u * (act ? (g & 3u) : 3u);
    return act ? 512u * (t >> 1) + 64u * (t & 1u) + 8u * (g & 3u) : 512u * (g >> 2) + 24u;
}

// Q4_K (dequant_q4_k, src/brain_runtime.c:960-1003): y = d sc_j q x - dmin
// m_j x per 32-element sub-block j. Lane t reads the 16 quant bytes
// 16 (t & 1) .. of chunk pi + 2 (t >> 1) (pi = 0, 1) of rows g and g + 8;
// low nibbles (nu = 0) are sub-block 2 (pi + 2 (t >> 1)), high nibbles
// (nu = 1, masked in place: 16 q) the next one. Two MMAs (8 bytes each) per
// (pi, nu); the sums are 16 q x for nu = 1, so 16 sc multiplies the nu = 0
// sums and the total is divided by 16 at the end. The min term uses the
// staged 16-element sums of e, once per (row, sub-block), by the even lanes.
__device__ __forceinline__ void q4k_task8(const uint8_t *r0, const uint8_t *r1, const uint8_t *xl, const float *xs,
                                          uint32_t t, float &o0, float &o1)
{
    const uint4 H0 = *reinterpret_cast<const uint4 *>(r0), H1 = *reinterpret_cast<const uint4 *>(r1);
    const bool upper = t >= 2u;   // sub-blocks 4..7 (the 6-bit scales packed across bytes)
    uint32_t SC[2], MN[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const uint4 H = r ? H1 : H0;
        const uint32_t sc03 = H.y & 0x3f3f3f3fu, m03 = H.z & 0x3f3f3f3fu;
        const uint32_t sc47 = (H.w & 0x0f0f0f0fu) | ((H.y >> 2) & 0x30303030u);
        const uint32_t m47 = ((H.w >> 4) & 0x0f0f0f0fu) | ((H.z >> 2) & 0x30303030u);
        SC[r] = upper ? sc47 : sc03;
        MN[r] = upper ? m47 : m03;
    }
    int T[4] = {0, 0, 0, 0};
    float M0 = 0.f, M1 = 0.f;
    const uint32_t off = 16u + 64u * (t >> 1) + 16u * (t & 1u);
#pragma unroll
    for (uint32_t pi = 0; pi < 2u; ++pi) {
        const uint4 W0 = *reinterpret_cast<const uint4 *>(r0 + off + 32u * pi);
        const uint4 W1 = *reinterpret_cast<const uint4 *>(r1 + off + 32u * pi);
#pragma unroll
        for (uint32_t nu = 0; nu < 2u; ++nu) {
            const uint32_t k = nu ? 0xf0f0f0f0u : 0x0f0f0f0fu;
            const uint8_t *xp = xl + 256u * pi + 128u * nu;
            int D[4] = {0, 0, 0, 0};
            mma_u8s8(D, W0.x & k, W1.x & k, W0.y & k, W1.y & k, *reinterpret_cast<const uint2 *>(xp));
            mma_u8s8(D, W0.z & k, W1.z & k, W0.w & k, W1.w & k, *reinterpret_cast<const uint2 *>(xp + 32));
            const uint32_t sh = 8u * (2u * pi + nu);
            const int s0 = (int)(((SC[0] >> sh) & 63u) << (nu ? 0u : 4u));
            const int s1 = (int)(((SC[1] >> sh) & 63u) << (nu ? 0u : 4u));
            T[0] += s0 * D[0];
            T[1] += s0 * D[1];
            T[2] += s1 * D[2];
            T[3] += s1 * D[3];
            const uint32_t j = 2u * pi + 4u * (t >> 1) + nu;
            const float xj = xs[2u * j] + xs[2u * j + 1u];
            M0 += u2f_small((MN[0] >> sh) & 63u) * xj;
            M1 += u2f_small((MN[1] >> sh) & 63u) * xj;
        }
    }
    const bool odd = t & 1u;
    const float u0 = odd ? 1.0f / (16384.0f * 16.0f) : 1.0f / 16.0f, u1 = odd ? 0.f : 1.0f / (128.0f * 16.0f);
    const float mo = odd ? 0.f : 1.f;
    o0 += h2f((uint16_t)(H0.x & 0xffffu)) * ((float)T[0] * u0 + (float)T[1] * u1) - h2f((uint16_t)(H0.x >> 16)) * (mo * M0);
    o1 += h2f((uint16_t)(H1.x & 0xffffu)) * ((float)T[2] * u0 + (float)T[3] * u1) - h2f((uint16_t)(H1.x >> 16)) * (mo * M1);
}

// A 6-bit quant of group c (0..3) from the ql / qh words of 4 consecutive
// l: low or high nibbles of ql, qh bit pair c moved to bits 4-5 of each byte
// (m02 = qh & 0x33.., m13 = qh & 0xcc..: no bits cross a byte).
__device__ __forceinline__ uint32_t q6_quant(uint32_t c, uint32_t ql_lo, uint32_t ql_hi, uint32_t m02, uint32_t m13)
{
    const uint32_t lowm = 0x0f0f0f0fu;
    switch (c) {
    case 0: return (ql_lo & lowm) | ((m02 << 4) & 0xf0f0f0f0u);
    case 1: return (ql_hi & lowm) | ((m13 << 2) & 0xf0f0f0f0u);
    case 2: return ((ql_lo >> 4) & lowm) | (m02 & 0xf0f0f0f0u);
    default: return ((ql_hi >> 4) & lowm) | ((m13 >> 2) & 0xf0f0f0f0u);
    }
}

// prmt.b32 in its default mode: a selector nibble with bit 3 set replicates
// the sign bit of the byte its low bits select (a sign-extended int8 when
// the four nibbles are k, k | 8, k | 8, k | 8).
__device__ __forceinline__ uint32_t prmt_sx(uint32_t x, uint32_t sel)
{
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(x), "r"(0u), "r"(sel));
    return r;
}
__host__ __device__ constexpr uint32_t sx_sel(uint32_t k) { return k | ((k | 8u) * 0x1110u); }

// Q6_K (dequant_q6_k, src/brain_runtime.c:1049-1083): y = d sc_G (q - 32) x
// per 16-element group G. Lane t reads ql bytes 8t.. and 32 + 8t.. of half
// q (64 q ..) and qh bytes 8t.. (128 + 32 q ..) of rows g and g + 8; MMA
// (q, c) takes group c's quants of those 8 l, group 8q + 2c + (t >> 1). The
// -32 offset is applied with the staged 16-element sums of e, once per (row,
// group), by the even lanes. sel0 / sel1: byte_perm selectors of scale byte
// (t >> 1) / 2 + (t >> 1) of a word, sign-extended.
__device__ __forceinline__ void q6k_task8(const uint8_t *w0, uint32_t b0, const uint8_t *w1, uint32_t b1,
                                          const uint8_t *xl, const float *xs, uint32_t t, uint32_t sel0, uint32_t sel1,
                                          float &o0, float &o1)
{
    // w0 / w1: the 16-byte-aligned windows of rows g / g + 8, b0 / b1: the
    // blocks' (even) offsets in them
    uint32_t S0[4], S1[4];
    ld16_at(w0, b0 + 192u, S0);
    ld16_at(w1, b1 + 192u, S1);
    int T[4] = {0, 0, 0, 0};
    float F0 = 0.f, F1 = 0.f;
#pragma unroll
    for (uint32_t q = 0; q < 2u; ++q) {
        const uint32_t ql = 64u * q + 8u * t, qh = 128u + 32u * q + 8u * t;
        const uint2 l0 = ld8_at(w0, b0 + ql), h0 = ld8_at(w0, b0 + ql + 32u);
        const uint2 l1 = ld8_at(w1, b1 + ql), h1 = ld8_at(w1, b1 + ql + 32u);
        const uint2 e0 = ld8_at(w0, b0 + qh), e1 = ld8_at(w1, b1 + qh);
        const uint32_t m02[4] = {e0.x & 0x33333333u, e0.y & 0x33333333u, e1.x & 0x33333333u, e1.y & 0x33333333u};
        const uint32_t m13[4] = {e0.x & 0xccccccccu, e0.y & 0xccccccccu, e1.x & 0xccccccccu, e1.y & 0xccccccccu};
#pragma unroll
        for (uint32_t c = 0; c < 4u; ++c) {
            int D[4] = {0, 0, 0, 0};
            mma_u8s8(D, q6_quant(c, l0.x, h0.x, m02[0], m13[0]), q6_quant(c, l1.x, h1.x, m02[2], m13[2]),
                     q6_quant(c, l0.y, h0.y, m02[1], m13[1]), q6_quant(c, l1.y, h1.y, m02[3], m13[3]),
                     *reinterpret_cast<const uint2 *>(xl + 512u * q + 128u * c));
            const uint32_t sel = (c & 1u) ? sel1 : sel0;
            const int s0 = (int)prmt_sx(S0[2u * q + (c >> 1)], sel);
            const int s1 = (int)prmt_sx(S1[2u * q + (c >> 1)], sel);
            T[0] += s0 * D[0];
            T[1] += s0 * D[1];
            T[2] += s1 * D[2];
            T[3] += s1 * D[3];
            const float xg = xs[8u * q + 2u * c + (t >> 1)];
            F0 += (float)s0 * xg;
            F1 += (float)s1 * xg;
        }
    }
    const bool odd = t & 1u;
    const float u0 = odd ? 1.0f / 16384.0f : 1.0f, u1 = odd ? 0.f : 1.0f / 128.0f, fo = odd ? 0.f : 32.0f;
    const float d0 = h2f(*reinterpret_cast<const uint16_t *>(w0 + b0 + 208u));
    const float d1 = h2f(*reinterpret_cast<const uint16_t *>(w1 + b1 + 208u));
    o0 += d0 * ((float)T[0] * u0 + (float)T[1] * u1 - fo * F0);
    o1 += d1 * ((float)T[2] * u0 + (float)T[3] * u1 - fo * F1);
}

// ------------------------------------------------ other block types ----
//
// A task of type TY (F16, Q5_0, Q5_1, Q8_0, Q5_K) reads every weight of a
// 16-element group G as  w = S q + M,  with q a small unsigned integer and
// S, M per row and group (dequant_block, src/brain_runtime.c:1017-1121):
//   Q5_0  q = nibble | high bit << 4   S = d        M = -16 d
//   Q5_1  q = nibble | high bit << 4   S = d        M = m
//   Q8_0  q = int8 + 128               S = d        M = -128 d
//   Q5_K  q = nibble | high bit << 4   S = d sc_j   M = -dmin m_j   (j = G / 2)
//   F16   the binary16 weight itself   S = 1        M = 0
// so a row's dot over G is  S sum(q x) + M sum(x).  q enters the MMA as a
// zero-extended 16-bit lane (the fp16 subnormal q 2^-24 exactly). The four
// lanes of a row group share each MMA: in round `it`, lane t of a row
// group supplies the k slots of group G = 4 it + t, four elements per MMA, and
// B holds x only in the column pair (hi, lo) of the group its lane carries,
// so accumulator columns 2t, 2t + 1 end as group G's sums for rows g, g + 8.

// The group's 4-byte words of quant values (bytes zero-extended later), and
// the group's (S, M) for one row of a task chunk at `r` (shared memory).
template <uint32_t TY>
__device__ __forceinline__ void gen_group(const uint8_t *r, uint32_t it, uint32_t t, uint32_t (&q)[4], float &s,
                                          float &m)
{
    if (TY == 8u) {   // Q8_0: 34-byte blocks of 32 (d, int8[32])
        const uint8_t *b = r + 34u * (2u * it + (t >> 1));
        ld16_u2(b + 2u + 16u * (t & 1u), q);
#pragma unroll
        for (int i = 0; i < 4; ++i) q[i] ^= 0x80808080u;
        s = h2f(*reinterpret_cast<const uint16_t *>(b));
        m = -128.0f * s;
    } else if (TY == 6u) {   // Q5_0: 22-byte blocks (d, qh u32, qs[16])
        const uint8_t *b = r + 22u * (2u * it + (t >> 1));
        const uint32_t half = t & 1u;
        ld16_u2(b + 6u, q);
        const uint32_t qh = *reinterpret_cast<const uint16_t *>(b + 2u + 2u * half);
#pragma unroll
        for (uint32_t i = 0; i < 4u; ++i) {
            // bits 4i..4i+3 of the group's 16 high bits -> bit 4 of bytes 0..3
            const uint32_t h4 = (qh >> (4u * i)) & 15u;
            q[i] = ((q[i] >> (4u * half)) & 0x0f0f0f0fu) | (((h4 * 0x00204081u) & 0x01010101u) << 4);
        }
        s = h2f(*reinterpret_cast<const uint16_t *>(b));
        m = -16.0f * s;
    } else if (TY == 7u) {   // Q5_1: 24-byte blocks (d, m, qh u32, qs[16])
        const uint8_t *b = r + 24u * (2u * it + (t >> 1));
        const uint32_t half = t & 1u;
        const uint2 w0 = *reinterpret_cast<const uint2 *>(b + 8u), w1 = *reinterpret_cast<const uint2 *>(b + 16u);
        const uint32_t hd = *reinterpret_cast<const uint32_t *>(b);
        const uint32_t qh = *reinterpret_cast<const uint32_t *>(b + 4u) >> (16u * half);
        const uint32_t raw[4] = {w0.x, w0.y, w1.x, w1.y};
#pragma unroll
        for (uint32_t i = 0; i < 4u; ++i) {
            const uint32_t h4 = (qh >> (4u * i)) & 15u;
            q[i] = ((raw[i] >> (4u * half)) & 0x0f0f0f0fu) | (((h4 * 0x00204081u) & 0x01010101u) << 4);
        }
        s = h2f((uint16_t)(hd & 0xffffu));
        m = h2f((uint16_t)(hd >> 16));
    } else {   // Q5_K: the 176-byte super-block (d, dmin, scales[12], qh[32], ql[128])
        const uint32_t hi = t >> 1, half = t & 1u, sh = 2u * it + hi;
        const uint4 ql = *reinterpret_cast<const uint4 *>(r + 48u + 32u * it + 16u * half);
        // the reference's qh bytes 16 + 8 c + l for chunk c = it (its pointer
        // advances 8 bytes per 64 values), bit 2 c + hi
        const uint2 h0 = *reinterpret_cast<const uint2 *>(r + 16u + 8u * it + 16u * half);
        const uint2 h1 = *reinterpret_cast<const uint2 *>(r + 24u + 8u * it + 16u * half);
        const uint32_t lw[4] = {ql.x, ql.y, ql.z, ql.w}, hw[4] = {h0.x, h0.y, h1.x, h1.y};
        const uint32_t rot = (4u - sh) & 31u;   // bit sh of every byte -> bit 4
#pragma unroll
        for (uint32_t i = 0; i < 4u; ++i)
            q[i] = ((lw[i] >> (4u * hi)) & 0x0f0f0f0fu) | (__funnelshift_l(hw[i], hw[i], rot) & 0x10101010u);
        const uint32_t hd = *reinterpret_cast<const uint32_t *>(r);
        uint32_t sc, mn;
        k4_scale_min((int)sh, r + 4, sc, mn);
        s = h2f((uint16_t)(hd & 0xffffu)) * u2f_small(sc);
        m = -(h2f((uint16_t)(hd >> 16)) * u2f_small(mn));
    }
}

// One task (16 rows x 256 elements) of type TY for lane (g, t): rows g (r0)
// and g + 8 (r1) of the slot; xb / xs: the block column's staged x groups
// (natural element order) and 16-element sums.
template <uint32_t TY>
__device__ __forceinline__ void gen_task(const uint8_t *r0, const uint8_t *r1, const uint8_t *xb, const float *xs,
                                         uint32_t lane, float &o0, float &o1)
{
    const uint32_t g = lane >> 2, t = lane & 3u;
    const uint32_t podd = (g & 1u) * 8u;
    const bool bmine = (g >> 1) == t;
    const float zero[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (uint32_t it = 0; it < 4u; ++it) {
        const uint32_t G = 4u * it + t;
        float c[4] = {0.f, 0.f, 0.f, 0.f};
        if (TY == 1u) {
            // F16: the group's 32 bytes; elements 4i, 4i + 1 in word 2i, 4i + 2, 4i + 3 in word 2i + 1
            const uint4 u0 = *reinterpret_cast<const uint4 *>(r0 + 32u * G),
                        u1 = *reinterpret_cast<const uint4 *>(r0 + 32u * G + 16u);
            const uint4 v0 = *reinterpret_cast<const uint4 *>(r1 + 32u * G),
                        v1 = *reinterpret_cast<const uint4 *>(r1 + 32u * G + 16u);
            const uint32_t w0[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};   // row g
            const uint32_t w1[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};   // row g + 8
#pragma unroll
            for (uint32_t i = 0; i < 4u; ++i) {
                uint2 b = make_uint2(0u, 0u);
                if (bmine) b = *reinterpret_cast<const uint2 *>(xb + (4u * G + i) * 16u + podd);
                const float cc[4] = {c[0], c[1], c[2], c[3]};
                mma16816(c, w0[2 * i], w1[2 * i], w0[2 * i + 1], w1[2 * i + 1], b, i == 0u ? zero : cc);
            }
            o0 += c[0] + c[1];
            o1 += c[2] + c[3];
        } else {
            uint32_t q0[4], q1[4];
            float s0, m0, s1, m1;
            gen_group<TY>(r0, it, t, q0, s0, m0);
            gen_group<TY>(r1, it, t, q1, s1, m1);
#pragma unroll
            for (uint32_t i = 0; i < 4u; ++i) {
                uint2 b = make_uint2(0u, 0u);
                if (bmine) b = *reinterpret_cast<const uint2 *>(xb + (4u * G + i) * 16u + podd);
                const float cc[4] = {c[0], c[1], c[2], c[3]};
                mma16816(c, sub2(q0[i], 0x4140), sub2(q1[i], 0x4140), sub2(q0[i], 0x4342), sub2(q1[i], 0x4342), b,
                         i == 0u ? zero : cc);
            }
            const float sx = xs[G];
            o0 += fmaf(s0, (c[0] + c[1]) * kTwo24, m0 * sx);
            o1 += fmaf(s1, (c[2] + c[3]) * kTwo24, m1 * sx);
        }
    }
}

// Copies of one task of type TY: lane L copies row L % 16's 16-byte chunks
// L / 16, L / 16 + 2, ...
template <uint32_t TY>
__device__ __forceinline__ void m4_issue_gen(const uint8_t *base, uint32_t rb, uint32_t slot, uint32_t lane)
{
    constexpr uint32_t NP = m4_chunk_bytes(TY) / 16u, RS = m4_gen_row(TY);
    const uint32_t r = lane & 15u, p0 = lane >> 4;
    const uint8_t *src = base + r * rb + 16u * p0;
    const uint32_t dst = slot + r * RS + 16u * p0;
#pragma unroll
    for (uint32_t i = 0; i < (NP + 1u) / 2u; ++i)
        if (p0 + 2u * i < NP) cp_async16_plain(dst + 32u * i, src + 32u * i);
}

template <int NS, uint32_t TY, int W>
__device__ void m4_consume(const MvArgs &a, M4Hdr *h, float *part, uint8_t *xarea, uint8_t *ring, const MvCta &c,
                           MvBest &best, uint64_t &t_ready, uint64_t *t_wait)
{
    constexpr bool Q4 = TY == 12u, Q6 = TY == 14u;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t g = lane >> 2;
    const uint32_t L = c.j1 - c.j0, weff = min((uint32_t)W, L);
    const bool active = warp < weff;
    const bool paired = a.paired != 0u;
    const uint32_t nb = a.nb, TP = nb * (paired ? 2u : 1u);
    const uint32_t my0 = active ? h->wstart[warp] : 0u;
    const uint32_t my1 = active ? (warp + 1u < weff ? h->wstart[warp + 1u] : c.j1) : 0u;
    const uint32_t n = my1 - my0;
    M4Seg sg;
    {
        const MvSeg &s0 = a.seg[c.seg];
        sg.w0 = s0.w;
        sg.w1 = paired ? a.seg[1].w : s0.w;
        sg.rb = (uint32_t)s0.row_bytes;
        sg.q4 = Q4 ? 1u : 0u;
        sg.bb = m4_chunk_bytes(TY);
        sg.ncp = Q4 ? 5u : 7u;
    }
    M4Cur ci{}, cc{};
    uint32_t first_tile = 0, last_tile = 0;
    if (active) {
        first_tile = my0 / TP;
        last_tile = (my1 - 1u) / TP;
        const uint32_t r = my0 - first_tile * TP;
        ci.t = first_tile;
        ci.s = paired && r >= nb ? 1u : 0u;
        ci.b = r - ci.s * nb;
        cc = ci;
    }
    const uint64_t policy = policy_evict_first();
    const uint32_t ring_w = smem_addr(ring) + warp * (uint32_t)NS * a.slot_bytes;
    // prologue: the first NS - 1 tasks, at most kPre of them before the wait
    // for the preceding kernel and the input staging, the rest after. Issuing
    // copies stalls a warp once the memory pipe's queue is full (16 warps x
    // 4 tasks of gate/up is 22 MB in flight), which delays its wait and
    // staging; 3 before and the rest after measured best (7B 2.533 -> 2.514
    // ms/token against all 4 before, 14B 4.82 -> 4.79).
    constexpr uint32_t kPre = 3u;
#pragma unroll
    for (uint32_t k = 0; k + 1u < (uint32_t)NS && k < kPre; ++k) {
        if (k < n) {
            if constexpr (Q4 || Q6) m4_issue<Q4>(sg, h, ci, ring_w + k * a.slot_bytes, lane, policy);
            else m4_issue_gen<TY>(m4_block(sg, ci), sg.rb, ring_w + k * a.slot_bytes, lane);
            m4_next(ci, nb, paired);
        }
        m4_commit();
    }
    const float out_scale = m4_stage_x<W, Q4 || Q6>(a, h->dred, xarea, Q4, t_wait, a.seg[c.seg].x_off);
#pragma unroll
    for (uint32_t k = kPre; k + 1u < (uint32_t)NS; ++k) {
        if (k < n) {
            if constexpr (Q4 || Q6) m4_issue<Q4>(sg, h, ci, ring_w + k * a.slot_bytes, lane, policy);
            else m4_issue_gen<TY>(m4_block(sg, ci), sg.rb, ring_w + k * a.slot_bytes, lane);
            m4_next(ci, nb, paired);
        }
        m4_commit();
    }
    t_ready = global_ns();
    if (!active) return;
    // sharing of the first and last tiles with neighbouring warps
    // (the CTA's range may start and end inside a tile: clamp to it)
    const uint32_t fa = m4_warp_of(c.j0, L, weff, max(first_tile * TP, c.j0)),
                   fb = m4_warp_of(c.j0, L, weff, min(first_tile * TP + TP, c.j1) - 1u);
    const uint32_t la = m4_warp_of(c.j0, L, weff, max(last_tile * TP, c.j0)),
                   lb = m4_warp_of(c.j0, L, weff, min(last_tile * TP + TP, c.j1) - 1u);
    const float *xs16 = reinterpret_cast<const float *>(xarea + (size_t)a.cols * 4u);
    const float *isb = xs16 + a.cols / 16u;
    const uint8_t *ringp = ring + (size_t)warp * NS * a.slot_bytes;
    const uint32_t wlow = (uint32_t)reinterpret_cast<uintptr_t>(sg.w0), wlow1 = (uint32_t)reinterpret_cast<uintptr_t>(sg.w1);
    const uint32_t bsel = m4_bsel(lane, Q6), t4 = lane & 3u;
    const uint32_t sel0 = sx_sel(t4 >> 1), sel1 = sx_sel(2u + (t4 >> 1));
    float a00 = 0.f, a01 = 0.f, a10 = 0.f, a11 = 0.f;
    uint32_t si = 0, sn = (uint32_t)NS - 1u;   // slots of the consumed and of the next issued task
    for (uint32_t k = 0; k < n; ++k) {
        if (k + (uint32_t)NS - 1u < n) {
            if constexpr (Q4 || Q6) m4_issue<Q4>(sg, h, ci, ring_w + sn * a.slot_bytes, lane, policy);
            else m4_issue_gen<TY>(m4_block(sg, ci), sg.rb, ring_w + sn * a.slot_bytes, lane);
            m4_next(ci, nb, paired);
        }
        m4_commit();
        if (++sn == (uint32_t)NS) sn = 0u;
        cp_async_wait<NS - 1>();
        __syncwarp();
        const uint8_t *slot = ringp + si * a.slot_bytes;
        if (++si == (uint32_t)NS) si = 0u;
        const uint8_t *xb = xarea + cc.b * 1024u;
        const float *xs = xs16 + cc.b * 16u;
        float o0 = 0.f, o1 = 0.f;
        if constexpr (Q4) {
            q4k_task8(slot + q4_slot_row(g) * kM4Q4Row, slot + q4_slot_row(g + 8u) * kM4Q4Row, xb + bsel, xs, t4, o0,
                      o1);
        } else if constexpr (Q6) {
            // the block's offset inside its 16-byte-aligned window, per row
            const uint32_t lb0 = (cc.s ? wlow1 : wlow) + 16u * cc.t * sg.rb + cc.b * 210u;
            q6k_task8(slot + g * kM4Q6Row, (lb0 + g * sg.rb) & 15u, slot + (g + 8u) * kM4Q6Row,
                      (lb0 + (g + 8u) * sg.rb) & 15u, xb + bsel, xs, t4, sel0, sel1, o0, o1);
        } else {
            gen_task<TY>(slot + g * m4_gen_row(TY), slot + (g + 8u) * m4_gen_row(TY), xb, xs, lane, o0, o1);
        }
        __syncwarp();   // the slot is re-filled by a later iteration's copies
        const float sb = isb[cc.b];
        o0 *= sb;
        o1 *= sb;
        if (cc.s) {
            a10 += o0;
            a11 += o1;
        } else {
            a00 += o0;
            a01 += o1;
        }
        const uint32_t t = cc.t;
        m4_next(cc, nb, paired);
        if (cc.t != t || k + 1u == n) {
            const uint32_t wa = t == first_tile ? fa : (t == last_tile ? la : warp);
            const uint32_t wb = t == first_tile ? fb : (t == last_tile ? lb : warp);
            if constexpr (Q4 || Q6) m4_flush(a, h, part, c, t, t * TP, wa, wb, my0, a00, a01, a10, a11, out_scale, best);
            else m4_flush_body(a, h, part, c, t, t * TP, wa, wb, my0, a00, a01, a10, a11, out_scale, best);
            a00 = a01 = a10 = a11 = 0.f;
        }
    }
}

// W = 16: one CTA per SM; W = 8: two CTAs fit on an SM (registers), so that
// the next launch's CTAs become resident, and stream their first weights,
// while this launch still runs.
// GT = 0: Q4_K and Q6_K segments (each CTA takes its segment's type); GT = one
// of the other block types (F16, Q5_0, Q5_1, Q8_0, Q5_K): every segment has it.
template <int NS, int W, uint32_t GT>
__global__ void __launch_bounds__(W * 32, W == 8 ? 2 : 1) mv4_kernel(const __grid_constant__ MvArgs a)
{
    extern __shared__ __align__(128) uint8_t smem[];
    M4Hdr *h = reinterpret_cast<M4Hdr *>(smem);
    float *part = reinterpret_cast<float *>(smem + m4_hdr_bytes());
    uint8_t *xarea = smem + m4_hdr_bytes() + kM4PartBytes;
    uint8_t *ring = xarea + mv_x_bytes(a.cols);
    const uint64_t t_start = global_ns();
    uint64_t *const tr = trace_ptr(a.dstate);
    uint64_t t_ready = 0, t_wait[2] = {0, 0};
    const MvCta c = a.cta[blockIdx.x];
    {
        const uint32_t L = c.j1 - c.j0, weff = min((uint32_t)W, L);
        if (threadIdx.x < (uint32_t)W) {
            h->cnt[threadIdx.x] = 0u;
            h->wstart[threadIdx.x] = threadIdx.x < weff ? m4_start(c.j0, L, weff, threadIdx.x) : 0xffffffffu;
        }
        // copy table: Q4_K 16 rows x 9 chunks of 16 bytes (5 per lane); Q6_K
        // 16 rows x 14 chunks (a 224-byte window holds the 210-byte block at
        // any 2-byte offset), 7 per lane
        const bool q4 = a.seg[c.seg].type == 12u;
        const uint32_t rb = (uint32_t)a.seg[c.seg].row_bytes;
        for (uint32_t e = threadIdx.x; e < 8u * 32u; e += blockDim.x) {
            const uint32_t i = e >> 5, l = e & 31u, idx = l + 32u * i;
            uint2 v = make_uint2(0u, 0xffffffffu);
            if (q4 && idx < 144u) {
                const uint32_t r = idx / 9u, p = idx - 9u * r;
                v = make_uint2(r * rb + 16u * p, q4_slot_row(r) * kM4Q4Row + 16u * p);
            } else if (!q4 && idx < 224u) {
                // slot offset in the low half, the chunk's offset in the window in the high half
                const uint32_t r = idx / 14u, p = idx - 14u * r;
                v = make_uint2(r * rb, (r * kM4Q6Row + 16u * p) | (16u * p) << 16);
            }
            h->cp[i][l] = v;
        }
    }
    __syncthreads();
    pdl_launch();
    MvBest best{-FLT_MAX, 0xffffffffu};
    if constexpr (GT != 0u) {
        m4_consume<NS, GT, W>(a, h, part, xarea, ring, c, best, t_ready, t_wait);
    } else {
        if (a.seg[c.seg].type == 12u) m4_consume<NS, 12u, W>(a, h, part, xarea, ring, c, best, t_ready, t_wait);
        else m4_consume<NS, 14u, W>(a, h, part, xarea, ring, c, best, t_ready, t_wait);
    }
    cp_async_wait<0>();   // no copy may still target this CTA's shared memory when it exits
    if (a.epi == MV_PART) {
        // The barrier orders every thread's partial-row stores to the peers
        // before the system-scope releases, which are cumulative: a rank that
        // acquires the counter sees all of them. Lane p of warp 0 signals rank
        // p, so the ranks' releases are one warp instruction, not tp in turn.
        m4_sync<W>();
        if (threadIdx.x < a.tp) red_release_sys_add(reinterpret_cast<uint32_t *>(a.peer[threadIdx.x] + a.out_cnt), 1u);
        trace_done(tr, a.trace_slot, t_start, t_ready, t_wait[0], t_wait[1]);
        return;
    }
    trace_done(tr, a.trace_slot, t_start, t_ready, t_wait[0], t_wait[1]);
    if (a.epi != MV_LOGITS) return;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best.v, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, best.i, o);
        if (ov > best.v || (ov == best.v && oi < best.i)) { best.v = ov; best.i = oi; }
    }
    if (lane == 0) { h->amax[warp] = best.v; h->aidx[warp] = best.i; }
    m4_sync<W>();
    if (warp != 0u) return;
    // every lane of warp 0 reduces the warps' pairs (the same order, so the
    // same result in every lane)
    for (int w = 1; w < W; ++w)
        if (h->amax[w] > best.v || (h->amax[w] == best.v && h->aidx[w] < best.i)) { best.v = h->amax[w]; best.i = h->aidx[w]; }
    if (a.tp > 1u) {
        // lane p stores (max, global row) into this rank's slot at rank p,
        // then releases it there (its own stores, in program order)
        if (lane < a.tp) {
            reinterpret_cast<float *>(a.peer[lane] + a.out_red)[a.rank * kTpPStride + blockIdx.x] = best.v;
            reinterpret_cast<uint32_t *>(a.peer[lane] + a.out_red + a.tp * kTpPStride * 4u)[a.rank * kTpPStride +
                                                                                           blockIdx.x] =
                a.row_base + best.i;
            red_release_sys_add(reinterpret_cast<uint32_t *>(a.peer[lane] + a.out_cnt), 1u);
        }
    } else if (lane == 0) {
        a.pmax[blockIdx.x] = best.v;
        a.pidx[blockIdx.x] = best.i;
    }
}

// ---------------------------------------------------------- attention ----

constexpr uint32_t kAttnWarps = kAttnThreads / 32u;
constexpr uint32_t kAttnPer = kAttnTile / kAttnWarps;   // positions of a tile per warp

struct AttnTiles {
    uint8_t k[2][kAttnTile * 512];      // staged K rows, as stored in the cache (fp32 or fp16), two tiles
    uint8_t v[2][kAttnTile * 512];      // staged V rows
};

// attn_tc16_kernel: tiles of 64 fp16 rows, padded to 272 bytes
constexpr uint32_t kTcTile = 64, kTcRowH = 136;
struct AttnTcTiles {
    __half k[2][kTcTile][kTcRowH];
    __half v[2][kTcTile][kTcRowH];
};

struct __align__(16) AttnSmem {
    float4 q[kAttnMaxGroup][32];        // RoPE'd queries of the group (128 dims)
    union {
        AttnTiles tl;
        AttnTcTiles tc;
        float wrec[kAttnWarps][kAttnMaxGroup][kRec];   // after the last tile: every warp's (acc, max, sum) per head
    } u;
    float4 knew[32], vnew[32];          // the current token's RoPE'd k and its v
    float rec[kAttnMaxGroup][kRec];     // this split's (acc[128], max, sum) per query head, read by the cluster
    float cw[32];                       // last merge: weight of each cluster record
    float qinv[kAttnMaxGroup + 1];      // qwen3: 1 / rms of each query head and (last) of the new k
    float cden;
    uint64_t bar[2];                    // tile arrival, per buffer
    uint32_t flag;
};

// 4 elements d4 of a staged cache row (fp32 or fp16 rows)
__device__ __forceinline__ float4 kv_row4(const uint8_t *row, uint32_t d4, bool f16)
{
    if (!f16) return reinterpret_cast<const float4 *>(row)[d4];
    const uint2 hb = reinterpret_cast<const uint2 *>(row)[d4];
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

__device__ __forceinline__ uint32_t cluster_ctarank()
{
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Every thread of every CTA of the cluster; shared-memory writes before it
// are visible to the cluster's reads after it.
__device__ __forceinline__ void cluster_sync_all()
{
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// The float at the same shared-memory offset as p in CTA `cta` of the cluster.
__device__ __forceinline__ float ld_cluster(const float *p, uint32_t cta)
{
    uint32_t r;
    float v;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr(p)), "r"(cta));
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(r) : "memory");
    return v;
}

// Sums over the warp of GP values at once. Slot i of lane l holds the lane's
// part of head i ^ (l >> (5 - log2 GP)); each of the first log2 GP levels
// keeps half of the slots and adds the partner lane's matching slot, the
// remaining levels are plain. Lane l ends with the sum of head
// l >> (5 - log2 GP); every addition is own + partner of a butterfly over
// lane distances 16, 8, 4, 2, 1, as in warp_sum.
template <int GP>
__device__ __forceinline__ float head_sums(float (&p)[GP])
{
    int lev = 0;
#pragma unroll
    for (int n = GP; n > 1; n >>= 1, ++lev) {
#pragma unroll
        for (int i = 0; i < n / 2; ++i) p[i] += __shfl_xor_sync(0xffffffffu, p[i + n / 2], 16 >> lev);
    }
    float v = p[0];
#pragma unroll
    for (int o = 16 >> lev; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Split-K flash-decode over the KV cache (gqa_single_token,
// src/brain_runtime.c:1482-1528). One CTA per (KV head, split); the splits in
// use grow with the context (at least kAttnMinSpan positions each) and come
// in clusters of kAttnCluster consecutive splits of one KV head. A split's
// cached K and V rows are contiguous in the cache, so each tile of up to
// kAttnTile positions arrives as two bulk copies into one of two buffers: the
// tile after the current one is always in flight, and the first two are
// issued before waiting for the preceding kernel (cached rows and the step's
// position were written by earlier steps). The split holding the current
// position applies RoPE to the fresh k and appends k and v to the cache
// (src/brain_runtime.c:1496-1500).
//
// Warp w takes kAttnPer positions of every tile and all GP (>= group) query
// heads of the KV head: lane = 4 of the 128 dimensions for the scores (one
// K row read serves every head; head_sums reduces all heads' dot products in
// one pass), then lane = (head, j) for the online softmax and P.V, holding
// float4s j, j + 32 / GP, ... of its head (the head's lanes read adjacent
// float4s of a V row: no bank conflicts). The warps' states merge into the
// split's record per head; the cluster's CTA r merges head r over the
// cluster's records (distributed
// shared memory). With one cluster that is the output; otherwise the cluster
// record goes to global memory and the last cluster to finish a head merges
// all clusters' records of that head.
// After the predecessor wait: the group's queries (qwen3 norm, RoPE) into
// shared memory, and in the split that owns the current position the new k
// (norm, RoPE) and v, appended to the cache. All threads.
__device__ __forceinline__ void attn_stage_qkv(const AttnArgs &a, AttnSmem &sm, uint32_t kvh, uint32_t group,
                                               uint32_t pos, bool has_pos, bool f16, size_t head_row0)
{
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const bool qkn = a.q_norm != nullptr;
    if (qkn) {
        // qwen3 per-head RMSNorm before RoPE (src/brain_runtime.c:1727-1737,
        // rms_norm :1338-1371): warp w takes query head w, and the new k
        // (index group) where this split appends it
        for (uint32_t hh = warp; hh <= group; hh += kAttnWarps) {
            if (hh == group && !has_pos) break;
            const float *src = hh < group ? a.q + (size_t)(kvh * group + hh) * 128u : a.k + (size_t)kvh * 128u;
            const float4 v = __ldcg(reinterpret_cast<const float4 *>(src) + lane);
            double ss = (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            if (lane == 0) sm.qinv[hh] = 1.0f / sqrtf((float)(ss / 128.0) + a.eps);
        }
        __syncthreads();
    }
    float *qf = reinterpret_cast<float *>(sm.q);
    for (uint32_t i = threadIdx.x; i < group * 64u; i += kAttnThreads) {
        const uint32_t hq = i >> 6, p = i & 63u;
        const float *qh = a.q + (size_t)(kvh * group + hq) * 128u;
        float qa = __ldcg(qh + p), qb = __ldcg(qh + p + 64u);
        if (qkn) {
            const float inv = sm.qinv[hq];
            qa = __fmul_rn(__fmul_rn(qa, inv), __ldg(a.q_norm + p));
            qb = __fmul_rn(__fmul_rn(qb, inv), __ldg(a.q_norm + p + 64u));
        }
        const float2 cs = __ldg(a.rope + (size_t)pos * 64u + p);
        qf[hq * 128u + p] = qa * cs.x - qb * cs.y;   // src/brain_runtime.c:1391-1393
        qf[hq * 128u + p + 64u] = qa * cs.y + qb * cs.x;
    }
    if (has_pos) {
        float *kn = reinterpret_cast<float *>(sm.knew), *vn = reinterpret_cast<float *>(sm.vnew);
        const float *kh = a.k + (size_t)kvh * 128u;
        for (uint32_t p = threadIdx.x; p < 64u; p += kAttnThreads) {
            float ka = __ldcg(kh + p), kb = __ldcg(kh + p + 64u);
            if (qkn) {
                const float inv = sm.qinv[group];
                ka = __fmul_rn(__fmul_rn(ka, inv), __ldg(a.k_norm + p));
                kb = __fmul_rn(__fmul_rn(kb, inv), __ldg(a.k_norm + p + 64u));
            }
            const float2 cs = __ldg(a.rope + (size_t)pos * 64u + p);
            kn[p] = ka * cs.x - kb * cs.y;
            kn[p + 64u] = ka * cs.y + kb * cs.x;
        }
        for (uint32_t i = threadIdx.x; i < 128u; i += kAttnThreads) vn[i] = __ldcg(a.v + (size_t)kvh * 128u + i);
    }
    __syncthreads();
    if (has_pos && threadIdx.x < 128u) {
        const size_t off = (head_row0 + pos) * 128u + threadIdx.x;
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
}

// The warps' (acc, max, sum) records of every head are in sm.u.wrec: merge
// them into the split's record, then over the cluster (CTA r takes head r)
// and, with several clusters, over the clusters of the KV head (the last
// cluster to finish a head). All threads of every CTA of the cluster.
__device__ __forceinline__ void attn_merge(const AttnArgs &a, AttnSmem &sm, uint32_t kvh, uint32_t group,
                                           uint32_t cl, uint32_t ncl)
{
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    __syncthreads();
    {
        const uint32_t hh = threadIdx.x >> 5, d4 = lane;   // 8 heads x 32 float4
        if (hh < group) {
            float M = -FLT_MAX;
#pragma unroll
            for (uint32_t w = 0; w < kAttnWarps; ++w) M = fmaxf(M, sm.u.wrec[w][hh][128]);
            float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
            float L = 0.f;
#pragma unroll
            for (uint32_t w = 0; w < kAttnWarps; ++w) {
                const float e = expf(sm.u.wrec[w][hh][128] - M);
                const float4 v = reinterpret_cast<const float4 *>(sm.u.wrec[w][hh])[d4];
                L = fmaf(e, sm.u.wrec[w][hh][129], L);
                o.x = fmaf(e, v.x, o.x);
                o.y = fmaf(e, v.y, o.y);
                o.z = fmaf(e, v.z, o.z);
                o.w = fmaf(e, v.w, o.w);
            }
            reinterpret_cast<float4 *>(sm.rec[hh])[d4] = o;
            if (d4 == 0u) {
                sm.rec[hh][128] = M;
                sm.rec[hh][129] = L;
            }
        }
    }
    cluster_sync_all();
    // CTA r of the cluster merges head r over the cluster's records; thread = dimension
    const uint32_t hh = cluster_ctarank();
    const bool merges = hh < group;
    float o = 0.f, L = 0.f, M = -FLT_MAX;
    if (merges && threadIdx.x < 128u) {
        float mc[kAttnCluster];
#pragma unroll
        for (uint32_t c = 0; c < kAttnCluster; ++c) {
            mc[c] = ld_cluster(&sm.rec[hh][128], c);
            M = fmaxf(M, mc[c]);
        }
#pragma unroll
        for (uint32_t c = 0; c < kAttnCluster; ++c) {
            const float e = expf(mc[c] - M);
            L = fmaf(e, ld_cluster(&sm.rec[hh][129], c), L);
            o = fmaf(e, ld_cluster(&sm.rec[hh][threadIdx.x], c), o);
        }
    }
    cluster_sync_all();   // no CTA leaves while the cluster may still read its records
    if (!merges) return;
    float *out = a.att + (size_t)(kvh * group + hh) * 128u;
    if (ncl == 1u) {
        if (threadIdx.x < 128u) out[threadIdx.x] = o * (L > 0.f ? 1.0f / L : 0.f);
        return;
    }
    float *crec = a.part + (((size_t)kvh * (a.splits / kAttnCluster) + cl) * group + hh) * kRec;
    if (threadIdx.x < 128u) crec[threadIdx.x] = o;
    if (threadIdx.x == 0) {
        crec[128] = M;
        crec[129] = L;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        uint32_t *ctr = a.ctr + kvh * group + hh;
        const uint32_t old = atom_acq_rel_add(ctr, 1u);
        sm.flag = (old == ncl - 1u) ? 1u : 0u;
        if (sm.flag) *ctr = 0u;
    }
    __syncthreads();
    if (!sm.flag) return;
    __threadfence();
    // the last cluster of head hh merges every cluster's record of it
    const float *rec0 = a.part + ((size_t)kvh * (a.splits / kAttnCluster) * group + hh) * kRec;
    const size_t cstride = (size_t)group * kRec;
    if (warp == 0) {
        const float mcl = lane < ncl ? __ldcg(rec0 + lane * cstride + 128u) : -FLT_MAX;
        const float Mx = warp_maxf(mcl);
        const float e = lane < ncl ? expf(mcl - Mx) : 0.f;
        const float den = warp_sum(lane < ncl ? e * __ldcg(rec0 + lane * cstride + 129u) : 0.f);
        sm.cw[lane] = e;
        if (lane == 0) sm.cden = den;
    }
    __syncthreads();
    if (threadIdx.x < 128u) {
        float num = 0.f;
        for (uint32_t c = 0; c < ncl; ++c) num = fmaf(sm.cw[c], __ldcg(rec0 + c * cstride + threadIdx.x), num);
        const float den = sm.cden;
        out[threadIdx.x] = num * (den > 0.f ? 1.0f / den : 0.f);
    }
}

template <int GP>
__device__ __forceinline__ void attn_body(const AttnArgs &a)
{
    extern __shared__ __align__(16) uint8_t smem_a[];
    AttnSmem &sm = *reinterpret_cast<AttnSmem *>(smem_a);
    const uint64_t t_start = global_ns();
    uint64_t *const tr = trace_ptr(a.st);
    pdl_launch();
    const uint32_t pos = *reinterpret_cast<volatile const uint32_t *>(&a.st->pos);
    if (pos >= a.max_context) {
        if (blockIdx.x == 0 && threadIdx.x == 0) atomicCAS(&a.st->status, kStatusOk, kStatusBadArgument);
        return;
    }
    const uint32_t n = pos + 1u;
    const uint32_t ms = a.min_span ? a.min_span : kAttnMinSpan;
    // splits in use: whole clusters (a.splits is a multiple of the cluster size)
    const uint32_t ns = min(a.splits, ((n + ms - 1u) / ms + kAttnCluster - 1u) / kAttnCluster * kAttnCluster);
    const uint32_t span = (n + ns - 1u) / ns;
    const uint32_t kvh = blockIdx.x / a.splits, s = blockIdx.x % a.splits;
    if (s >= ns) return;   // the whole cluster leaves
    const uint32_t ncl = ns / kAttnCluster, cl = s / kAttnCluster;
    const uint32_t group = a.q_heads / a.kv_heads;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t t0 = min(s * span, n), t1 = min(n, t0 + span);
    const bool has_pos = t0 <= pos && pos < t1;
    const bool f16 = a.kv_fp16 != 0u;
    const uint32_t rowb = f16 ? 256u : 512u;
    const float scale = 1.0f / sqrtf(128.0f);
    volatile uint32_t *err = &a.st->status;
    const size_t head_row0 = (size_t)kvh * a.max_context;
    // tile [tb, tb + kAttnTile) of the split into buffer b: cached rows
    // [tb, min(te, pos)) by bulk copies; two tiles are in flight
    auto issue = [&](uint32_t tb, uint32_t b) {
        const uint32_t te = min(tb + kAttnTile, t1), ce = max(tb, min(te, pos));
        const uint32_t bytes = (ce - tb) * rowb;
        mbar_arrive_expect_tx(&sm.bar[b], 2u * bytes);
        if (bytes) {
            bulk_g2s(sm.u.tl.k[b], reinterpret_cast<const uint8_t *>(a.k_cache) + (head_row0 + tb) * rowb, bytes,
                     &sm.bar[b]);
            bulk_g2s(sm.u.tl.v[b], reinterpret_cast<const uint8_t *>(a.v_cache) + (head_row0 + tb) * rowb, bytes,
                     &sm.bar[b]);
        }
    };
    if (threadIdx.x == 0) {
        mbar_init(&sm.bar[0], 1u);
        mbar_init(&sm.bar[1], 1u);
        fence_mbar_init();
        if (t0 < t1) issue(t0, 0u);
        if (t0 + kAttnTile < t1) issue(t0 + kAttnTile, 1u);
    }
    __syncthreads();
    pdl_wait();
    const uint64_t t_ready = global_ns();
    attn_stage_qkv(a, sm, kvh, group, pos, has_pos, f16, head_row0);
    constexpr uint32_t kL = GP == 8 ? 3u : GP == 4 ? 2u : GP == 2 ? 1u : 0u;
    const uint32_t hm = lane >> (5u - kL);                       // this lane's head after head_sums
    constexpr uint32_t kHs = 32u >> kL;                          // lanes per head
    const uint32_t hl = lane & (kHs - 1u);                       // its place among them: float4s hl + kHs i
    float4 qr[GP];
#pragma unroll
    for (int i = 0; i < GP; ++i) {
        const uint32_t hh = (uint32_t)i ^ hm;
        qr[i] = hh < group ? sm.q[hh][lane] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float m = -FLT_MAX, l = 0.f;
    float4 acc[GP];
#pragma unroll
    for (int i = 0; i < GP; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    uint32_t it = 0;
    for (uint32_t tb = t0; tb < t1; tb += kAttnTile, ++it) {
        const uint32_t te = min(tb + kAttnTile, t1), b = it & 1u;
        const uint8_t *kt = sm.u.tl.k[b], *vt = sm.u.tl.v[b];
        mbar_wait(&sm.bar[b], (it >> 1) & 1u, err);
        const uint32_t p0 = tb + kAttnPer * warp;   // this warp's positions p0 .. p0 + kAttnPer - 1
        float sc[kAttnPer];
#pragma unroll
        for (uint32_t j = 0; j < kAttnPer; ++j) {
            const uint32_t p = p0 + j;
            sc[j] = -FLT_MAX;
            if (p < te) {
                const float4 kv = p == pos ? sm.knew[lane] : kv_row4(kt + (size_t)(p - tb) * rowb, lane, f16);
                float d[GP];
#pragma unroll
                for (int i = 0; i < GP; ++i)
                    d[i] = fmaf(qr[i].x, kv.x, qr[i].y * kv.y) + fmaf(qr[i].z, kv.z, qr[i].w * kv.w);
                sc[j] = head_sums<GP>(d) * scale;
            }
        }
        float mc = sc[0];
#pragma unroll
        for (uint32_t j = 1; j < kAttnPer; ++j) mc = fmaxf(mc, sc[j]);
        const float mn = fmaxf(m, mc);
        const float corr = expf(m - mn);
        float w[kAttnPer], ws = 0.f;
#pragma unroll
        for (uint32_t j = 0; j < kAttnPer; ++j) {
            w[j] = p0 + j < te ? expf(sc[j] - mn) : 0.f;
            ws += w[j];
        }
        l = l * corr + ws;
#pragma unroll
        for (int i = 0; i < GP; ++i) {
            acc[i].x *= corr;
            acc[i].y *= corr;
            acc[i].z *= corr;
            acc[i].w *= corr;
        }
#pragma unroll
        for (uint32_t j = 0; j < kAttnPer; ++j) {
            const uint32_t p = p0 + j;
            if (p < te) {
                const uint8_t *vr = vt + (size_t)(p - tb) * rowb;
#pragma unroll
                for (int i = 0; i < GP; ++i) {
                    const uint32_t d4 = hl + kHs * (uint32_t)i;   // the head's lanes read adjacent float4s
                    const float4 vv = p == pos ? sm.vnew[d4] : kv_row4(vr, d4, f16);
                    acc[i].x = fmaf(w[j], vv.x, acc[i].x);
                    acc[i].y = fmaf(w[j], vv.y, acc[i].y);
                    acc[i].z = fmaf(w[j], vv.z, acc[i].z);
                    acc[i].w = fmaf(w[j], vv.w, acc[i].w);
                }
            }
        }
        m = mn;
        __syncthreads();   // tile consumed: its buffer takes the tile after next
        if (threadIdx.x == 0 && tb + 2u * kAttnTile < t1) issue(tb + 2u * kAttnTile, b);
    }
    // every copy was consumed: the tile buffers hold the warps' states now
    if (hm < group) {
        float *dst = sm.u.wrec[warp][hm];
#pragma unroll
        for (int i = 0; i < GP; ++i) reinterpret_cast<float4 *>(dst)[hl + kHs * (uint32_t)i] = acc[i];
        if (hl == 0u) {
            dst[128] = m;
            dst[129] = l;
        }
    }
    attn_merge(a, sm, kvh, group, cl, ncl);
    trace_done(tr, a.trace_slot, t_start, t_ready);
}

// Sequence s's view of a batched step's arguments.
__device__ __forceinline__ AttnArgs seq_view(const AttnArgs &a, uint32_t s)
{
    AttnArgs v = a;
    v.q = a.q + (size_t)s * a.qkv_stride;
    v.k = a.k + (size_t)s * a.qkv_stride;
    v.v = a.v + (size_t)s * a.qkv_stride;
    v.k_cache = static_cast<uint8_t *>(a.k_cache) + s * a.cache_seq_bytes;
    v.v_cache = static_cast<uint8_t *>(a.v_cache) + s * a.cache_seq_bytes;
    v.att = a.att + (size_t)s * a.att_stride;
    v.part = a.part + (size_t)s * a.part_seq;
    v.ctr = a.ctr + (size_t)s * a.ctr_seq;
    v.st = a.st + s;
    return v;
}

template <int GP>
__global__ void __launch_bounds__(kAttnThreads, 2) attn_kernel(const __grid_constant__ AttnArgs a)
{
    attn_body<GP>(a);
}

template <int GP>
__global__ void __launch_bounds__(kAttnThreads, 2) attn_kernel_b(const __grid_constant__ AttnArgs a)
{
    const AttnArgs v = seq_view(a, blockIdx.y);
    attn_body<GP>(v);
}

// ------------------------------------------- attention, fp16 cache, MMA ----

__device__ __forceinline__ void cp_async16(void *dst, const void *src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void ldmatrix_x4_t(const void *p, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(smem_addr(p)));
}

// d += A (16 x 16) B (16 x 8), binary16 in, fp32 accumulate
__device__ __forceinline__ void mma_k16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// d += A (16 x 8) B (8 x 8)
__device__ __forceinline__ void mma_k8(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0)
{
    asm volatile("mma.sync.aligned.m16n8k8.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a0), "r"(a1), "r"(b0));
}

// (x, y) -> binary16 pair hi and the rounded remainder lo (x = hi + lo to ~22 bits)
__device__ __forceinline__ void split_h2(float x, float y, uint32_t &hi, uint32_t &lo)
{
    const __half2 h = __floats2half2_rn(x, y);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(x - hf.x, y - hf.y);
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = *reinterpret_cast<const uint32_t *>(&l);
}

// Decode attention over an fp16 KV cache on tensor cores: the same splits,
// clusters, staging of q / k / v and merges as attn_kernel, with the tile
// loop as two MMAs. The cached K and V rows are binary16 already (exact MMA
// operands); q and the softmax weights P are split into binary16 pairs
// hi + lo, stacked as MMA rows 0-7 (hi) and 8-15 (lo) of one A operand, so
// each product term is one MMA and row h plus row h + 8 is the head's sum:
//   S = [q_hi; q_lo] K^T   m16n8k16, K by ldmatrix (8 positions per warp)
//   O += [P_hi; P_lo] V    m16n8k8,  V by ldmatrix.trans (16 tiles of 8 dims)
// Tiles of 64 positions arrive by per-thread 16-byte cp.async into rows of
// 272 bytes (the 8 rows an ldmatrix reads fall in distinct banks), two tiles
// in flight, the first two issued before the predecessor wait. Warp w takes
// positions 8w .. 8w + 7 of a tile; lane (g, t) holds head g's scores of
// positions 2t, 2t + 1 and its outputs of dimensions 8j + 2t, 8j + 2t + 1.
__device__ __forceinline__ void attn_tc16_body(const AttnArgs &a)
{
    extern __shared__ __align__(16) uint8_t smem_a[];
    AttnSmem &sm = *reinterpret_cast<AttnSmem *>(smem_a);
    const uint64_t t_start = global_ns();
    uint64_t *const tr = trace_ptr(a.st);
    pdl_launch();
    const uint32_t pos = *reinterpret_cast<volatile const uint32_t *>(&a.st->pos);
    if (pos >= a.max_context) {
        if (blockIdx.x == 0 && threadIdx.x == 0) atomicCAS(&a.st->status, kStatusOk, kStatusBadArgument);
        return;
    }
    const uint32_t n = pos + 1u;
    const uint32_t ms = a.min_span ? a.min_span : kAttnMinSpan;
    const uint32_t ns = min(a.splits, ((n + ms - 1u) / ms + kAttnCluster - 1u) / kAttnCluster * kAttnCluster);
    const uint32_t span = (n + ns - 1u) / ns;
    const uint32_t kvh = blockIdx.x / a.splits, s = blockIdx.x % a.splits;
    if (s >= ns) return;   // the whole cluster leaves
    const uint32_t ncl = ns / kAttnCluster, cl = s / kAttnCluster;
    const uint32_t group = a.q_heads / a.kv_heads;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u, g = lane >> 2, t = lane & 3u;
    const uint32_t t0 = min(s * span, n), t1 = min(n, t0 + span);
    const bool has_pos = t0 <= pos && pos < t1;
    const float scale = 1.0f / sqrtf(128.0f);
    const size_t head_row0 = (size_t)kvh * a.max_context;
    const uint8_t *kc = reinterpret_cast<const uint8_t *>(a.k_cache) + head_row0 * 256u;
    const uint8_t *vc = reinterpret_cast<const uint8_t *>(a.v_cache) + head_row0 * 256u;
    // cached rows [tb, min(te, pos)) of tile tb into buffer b, one group per
    // call (an empty one past the split's end)
    auto issue = [&](uint32_t tb, uint32_t b) {
        if (tb < t1) {
            const uint32_t te = min(tb + kTcTile, t1), ce = max(tb, min(te, pos));
            const uint32_t chunks = (ce - tb) * 16u;   // 16-byte pieces of 256-byte rows
            for (uint32_t i = threadIdx.x; i < chunks; i += kAttnThreads) {
                const uint32_t r = i >> 4, c = i & 15u;
                cp_async16(&sm.u.tc.k[b][r][8u * c], kc + (size_t)(tb + r) * 256u + 16u * c);
                cp_async16(&sm.u.tc.v[b][r][8u * c], vc + (size_t)(tb + r) * 256u + 16u * c);
            }
        }
        cp_async_commit();
    };
    issue(t0, 0u);
    issue(t0 + kTcTile, 1u);
    pdl_wait();
    const uint64_t t_ready = global_ns();
    attn_stage_qkv(a, sm, kvh, group, pos, has_pos, true, head_row0);
    // A operands of q: rows g (hi) and g + 8 (lo) of head g, 8 steps of 16 dimensions
    uint32_t qa[8][4];
    {
        const float *qg = reinterpret_cast<const float *>(sm.q[g < group ? g : 0u]);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            if (g < group) {
                split_h2(qg[16 * k + 2 * (int)t], qg[16 * k + 2 * (int)t + 1], qa[k][0], qa[k][1]);
                split_h2(qg[16 * k + 2 * (int)t + 8], qg[16 * k + 2 * (int)t + 9], qa[k][2], qa[k][3]);
            } else {
                qa[k][0] = qa[k][1] = qa[k][2] = qa[k][3] = 0u;
            }
        }
    }
    float m = -FLT_MAX, l = 0.f;
    float o[16][4];
#pragma unroll
    for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    const float *knew = reinterpret_cast<const float *>(sm.knew), *vnew = reinterpret_cast<const float *>(sm.vnew);
    uint32_t it = 0;
    for (uint32_t tb = t0; tb < t1; tb += kTcTile, ++it) {
        const uint32_t te = min(tb + kTcTile, t1), b = it & 1u;
        const uint32_t nrow = max(tb, min(te, pos)) - tb;   // rows the copies filled
        cp_async_wait1();   // this tile's group; the next tile's may still be in flight
        __syncthreads();
        // the other rows: the current position (the new k and v, rounded as the
        // cache keeps them) and zeros past the split's end (a weight of 0 times
        // stale shared memory could be NaN)
        if (nrow < kTcTile) {   // CTA-uniform: full tiles of cached rows skip the fill and its barrier
            for (uint32_t i = threadIdx.x; i < (kTcTile - nrow) * 128u; i += kAttnThreads) {
                const uint32_t r = nrow + (i >> 7), d = i & 127u;
                const bool cur = has_pos && tb + r == pos;   // only the owning split has the new k, v
                sm.u.tc.k[b][r][d] = __float2half_rn(cur ? knew[d] : 0.f);
                sm.u.tc.v[b][r][d] = __float2half_rn(cur ? vnew[d] : 0.f);
            }
            __syncthreads();
        }
        const uint32_t pw = tb + 8u * warp;   // this warp's positions pw .. pw + 7
        if (pw < te) {
            const __half *krow = &sm.u.tc.k[b][8u * warp + (lane & 7u)][0];
            const __half *vrow = &sm.u.tc.v[b][8u * warp + (lane & 7u)][0];
            float sacc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int k = 0; k < 8; k += 2) {
                // matrices: dims 16k + 8 (lane >> 3) .. + 7 of the warp's 8 rows
                uint32_t b4[4];
                ldmatrix_x4(krow + 16u * (uint32_t)k + 8u * (lane >> 3), b4[0], b4[1], b4[2], b4[3]);
                mma_k16(sacc, qa[k], b4[0], b4[1]);
                mma_k16(sacc, qa[k + 1], b4[2], b4[3]);
            }
            const uint32_t p0 = pw + 2u * t;
            const float s0 = p0 < te ? (sacc[0] + sacc[2]) * scale : -FLT_MAX;
            const float s1 = p0 + 1u < te ? (sacc[1] + sacc[3]) * scale : -FLT_MAX;
            float mx = fmaxf(s0, s1);
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            const float mn = fmaxf(m, mx);
            const float corr = expf(m - mn);
            const float w0 = p0 < te ? expf(s0 - mn) : 0.f;
            const float w1 = p0 + 1u < te ? expf(s1 - mn) : 0.f;
            float ws = w0 + w1;
            ws += __shfl_xor_sync(0xffffffffu, ws, 1);
            ws += __shfl_xor_sync(0xffffffffu, ws, 2);
            l = l * corr + ws;
            m = mn;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                o[j][0] *= corr;
                o[j][1] *= corr;
                o[j][2] *= corr;
                o[j][3] *= corr;
            }
            uint32_t ph, pl;
            split_h2(w0, w1, ph, pl);
#pragma unroll
            for (int jd = 0; jd < 16; jd += 4) {
                // matrices: dims 8 (jd + (lane >> 3)) .. + 7 of the warp's 8 rows, transposed
                uint32_t v4[4];
                ldmatrix_x4_t(vrow + 8u * ((uint32_t)jd + (lane >> 3)), v4[0], v4[1], v4[2], v4[3]);
#pragma unroll
                for (int e = 0; e < 4; ++e) mma_k8(o[jd + e], ph, pl, v4[e]);
            }
        }
        __syncthreads();   // tile consumed: its buffer takes the tile after next
        issue(tb + 2u * kTcTile, b);
    }
    cp_async_wait0();
    if (g < group) {
        float *dst = sm.u.wrec[warp][g];
#pragma unroll
        for (int j = 0; j < 16; ++j)
            *reinterpret_cast<float2 *>(dst + 8 * j + 2 * (int)t) = make_float2(o[j][0] + o[j][2], o[j][1] + o[j][3]);
        if (t == 0u) {
            dst[128] = m;
            dst[129] = l;
        }
    }
    attn_merge(a, sm, kvh, group, cl, ncl);
    trace_done(tr, a.trace_slot, t_start, t_ready);
}

__global__ void __launch_bounds__(kAttnThreads, 2) attn_tc16_kernel(const __grid_constant__ AttnArgs a)
{
    attn_tc16_body(a);
}

__global__ void __launch_bounds__(kAttnThreads, 2) attn_tc16_kernel_b(const __grid_constant__ AttnArgs a)
{
    const AttnArgs v = seq_view(a, blockIdx.y);
    attn_tc16_body(v);
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
// then advance the step state. Tensor parallel: the partials of every rank,
// once the head counter `cnt` has seen this step's `arrivals`.
__global__ void __launch_bounds__(256) argmax_kernel(const float *pmax, const uint32_t *pidx, uint32_t n,
                                                     DecState *st, const uint32_t *cnt, uint32_t arrivals)
{
    __shared__ float bv[8];
    __shared__ uint32_t bi[8];
    pdl_launch();
    pdl_wait();
    if (cnt) {
        if (threadIdx.x == 0) {
            const uint32_t epoch = *reinterpret_cast<volatile const uint32_t *>(&st->epoch);
            wait_counter_sys(cnt, (epoch + 1u) * arrivals, &st->status);
        }
        __syncthreads();
    }
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
        // prompt mode: the next prompt token instead of the pick
        st->token = (st->in_ids && st->step + 1u < st->n_in) ? st->in_ids[st->step + 1u] : idx;
        st->pos = st->pos + 1u;
        st->step = st->step + 1u;
    }
    st->epoch = st->epoch + 1u;
}

// ------------------------------------------- prefill all-reduce (TP) ----

// Reduce-scatter + all-gather of a prefill chunk's partial rows over peer
// memory, one cooperative launch (all CTAs resident: they wait on counters
// that this GPU's CTAs also feed). Every rank takes an equal slice of the
// float4 elements, adds the ranks' partials in rank order to its residual
// and stores the sums into every rank's residual; the ready counter (one
// arrival per rank) says every partial is written, the done counter (one
// arrival per CTA of every rank) says every slice has landed and nobody
// reads this rank's partials any more.
__global__ void __launch_bounds__(256) tp_allreduce_kernel(const __grid_constant__ TpReduceArgs a)
{
    uint8_t *own = a.peer[a.rank];
    if (blockIdx.x == 0 && threadIdx.x < a.tp) {
        __threadfence_system();
        red_release_sys_add(reinterpret_cast<uint32_t *>(a.peer[threadIdx.x] + kTpCntReady), 1u);
    }
    if (threadIdx.x == 0)
        wait_counter_sys(reinterpret_cast<const uint32_t *>(own + kTpCntReady), a.seq * a.tp, a.status);
    __syncthreads();
    const uint32_t s0 = (uint32_t)((uint64_t)a.n4 * a.rank / a.tp), s1 = (uint32_t)((uint64_t)a.n4 * (a.rank + 1u) / a.tp);
    const float4 *xr = reinterpret_cast<const float4 *>(own + a.px);
    for (uint32_t e = s0 + blockIdx.x * blockDim.x + threadIdx.x; e < s1; e += gridDim.x * blockDim.x) {
        float4 v = __ldcg(xr + e);
        for (uint32_t q = 0; q < a.tp; ++q) {
            const float4 *pq = reinterpret_cast<const float4 *>(a.peer[q] + a.part) + e;
            const float4 w = q == a.rank ? __ldcg(pq) : __ldcv(pq);
            v.x += w.x; v.y += w.y; v.z += w.z; v.w += w.w;
        }
        for (uint32_t p = 0; p < a.tp; ++p) reinterpret_cast<float4 *>(a.peer[p] + a.px)[e] = v;
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x < a.tp) red_release_sys_add(reinterpret_cast<uint32_t *>(a.peer[threadIdx.x] + kTpCntDone), 1u);
    if (threadIdx.x == 0)
        wait_counter_sys(reinterpret_cast<const uint32_t *>(own + kTpCntDone), a.seq * a.tp * gridDim.x, a.status);
    __syncthreads();
}

}  // namespace d2
}  // namespace atlas

// ------------------------------------------------------------ launchers ----

using namespace atlas::d2;

namespace {

// cluster > 1: clusters of that many consecutive CTAs (grid.x a multiple of it)
cudaError_t launch_ex(const void *fn, void **args, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl,
                      uint32_t cluster = 1)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    if (cluster > 1) {
        at[1].id = cudaLaunchAttributeClusterDimension;
        at[1].val.clusterDim.x = cluster;
        at[1].val.clusterDim.y = 1;
        at[1].val.clusterDim.z = 1;
        cfg.numAttrs = 2;
    }
    return cudaLaunchKernelExC(&cfg, fn, args);
}

// attention instance for `group` query heads per KV head (rounded up to a
// power of two); tc: the tensor-core kernel of fp16 caches
const void *attn_fn(uint32_t group, bool tc = false, bool batch = false)
{
    if (batch) {
        if (tc) return (const void *)attn_tc16_kernel_b;
        if (group <= 1u) return (const void *)attn_kernel_b<1>;
        if (group <= 2u) return (const void *)attn_kernel_b<2>;
        if (group <= 4u) return (const void *)attn_kernel_b<4>;
        return (const void *)attn_kernel_b<8>;
    }
    if (tc) return (const void *)attn_tc16_kernel;
    if (group <= 1u) return (const void *)attn_kernel<1>;
    if (group <= 2u) return (const void *)attn_kernel<2>;
    if (group <= 4u) return (const void *)attn_kernel<4>;
    return (const void *)attn_kernel<8>;
}

}  // namespace

namespace {
template <uint32_t GT>
const void *mv4_gen_fn(uint32_t nslot, uint32_t warps)
{
    if (warps == 16u) {
        switch (nslot) {
        case 2: return (const void *)mv4_kernel<2, 16, GT>;
        case 3: return (const void *)mv4_kernel<3, 16, GT>;
        case 4: return (const void *)mv4_kernel<4, 16, GT>;
        default: return nullptr;
        }
    }
    if (warps == 8u) {
        switch (nslot) {
        case 2: return (const void *)mv4_kernel<2, 8, GT>;
        case 3: return (const void *)mv4_kernel<3, 8, GT>;
        default: return nullptr;
        }
    }
    return nullptr;
}

const void *mv4_fn(uint32_t nslot, uint32_t warps, uint32_t gen_type = 0u)
{
    switch (gen_type) {
    case 0u: break;
    case 1u: return mv4_gen_fn<1u>(nslot, warps);
    case 6u: return mv4_gen_fn<6u>(nslot, warps);
    case 7u: return mv4_gen_fn<7u>(nslot, warps);
    case 8u: return mv4_gen_fn<8u>(nslot, warps);
    case 13u: return mv4_gen_fn<13u>(nslot, warps);
    default: return nullptr;
    }
    if (warps == 16u) {
        switch (nslot) {
        case 2: return (const void *)mv4_kernel<2, 16, 0u>;
        case 3: return (const void *)mv4_kernel<3, 16, 0u>;
        case 4: return (const void *)mv4_kernel<4, 16, 0u>;
        case 5: return (const void *)mv4_kernel<5, 16, 0u>;
        case 6: return (const void *)mv4_kernel<6, 16, 0u>;
        default: return nullptr;
        }
    }
    if (warps == 8u) {
        switch (nslot) {
        case 2: return (const void *)mv4_kernel<2, 8, 0u>;
        case 3: return (const void *)mv4_kernel<3, 8, 0u>;
        case 4: return (const void *)mv4_kernel<4, 8, 0u>;
        case 5: return (const void *)mv4_kernel<5, 8, 0u>;
        case 6: return (const void *)mv4_kernel<6, 8, 0u>;
        default: return nullptr;
        }
    }
    return nullptr;
}
}  // namespace

extern "C" size_t atlas_d2_mv_smem(uint32_t cols, uint32_t nslot, uint32_t slot_bytes, uint32_t tslots)
{
    return (size_t)mv_hdr_bytes() + mv_tile_bytes(tslots) + mv_desc_bytes(nslot) + mv_x_bytes(cols) +
           (size_t)nslot * slot_bytes;
}

// Clusters of the attention launch (kAttnCluster CTAs each) that fit on the
// device at once, for `group` query heads per KV head; 0 on error.
extern "C" int atlas_d2_attn_max_clusters(uint32_t group, uint32_t tc)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kAttnCluster * 64u);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = sizeof(AttnSmem);
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = kAttnCluster;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaFuncSetAttribute(attn_fn(group, tc != 0u), cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)sizeof(AttnSmem)) != cudaSuccess ||
        cudaOccupancyMaxActiveClusters(&n, attn_fn(group, tc != 0u), &cfg) != cudaSuccess)
        return 0;
    return n;
}

extern "C" size_t atlas_d2_attn_smem(uint32_t splits)
{
    (void)splits;
    return sizeof(AttnSmem);
}

// Raise the kernels' dynamic shared-memory limits (call before any capture).
extern "C" cudaError_t atlas_d2_setup(size_t mv_smem, size_t attn_smem)
{
    cudaError_t e = cudaFuncSetAttribute(mv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)mv_smem);
    if (e != cudaSuccess) return e;
    for (uint32_t w : {8u, 16u})
        for (uint32_t ns = 2; ns <= kM4MaxSlots; ++ns)
            for (uint32_t gt : {0u, 1u, 6u, 7u, 8u, 13u}) {
                const void *fn = mv4_fn(ns, w, gt);
                if (fn && (e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)mv_smem)) !=
                              cudaSuccess)
                    return e;
            }
    for (bool b : {false, true}) {
        for (uint32_t g = 1; g <= kAttnMaxGroup; g *= 2u)
            if ((e = cudaFuncSetAttribute(attn_fn(g, false, b), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)attn_smem)) != cudaSuccess)
                return e;
        if ((e = cudaFuncSetAttribute(attn_fn(1, true, b), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)attn_smem)) != cudaSuccess)
            return e;
    }
    return cudaSuccess;
}

extern "C" size_t atlas_d2_mv4_smem(uint32_t cols, uint32_t warps, uint32_t nslot, uint32_t slot_bytes)
{
    return m4_smem_bytes(cols, warps, nslot, slot_bytes);
}

extern "C" cudaError_t atlas_d2_launch_mv(const MvArgs *a, uint32_t grid, cudaStream_t stream)
{
    MvArgs copy = *a;
    void *args[] = {&copy};
    if (a->engine == 1u) {
        const void *fn = mv4_fn(a->nslot, a->warps, a->gen_type);
        if (!fn) return cudaErrorInvalidValue;
        return launch_ex(fn, args, dim3(grid), dim3(32u * a->warps), a->smem_bytes, stream, a->pdl != 0u);
    }
    return launch_ex((const void *)mv_kernel, args, dim3(grid), dim3(kMvThreads), a->smem_bytes, stream, a->pdl != 0u);
}

// A batched step's attention: grid.y = nseq sequences.
extern "C" cudaError_t atlas_d2_launch_attn_b(const AttnArgs *a, uint32_t grid, uint32_t nseq, cudaStream_t stream)
{
    AttnArgs copy = *a;
    void *args[] = {&copy};
    const uint32_t group = a->q_heads / a->kv_heads;
    if (group == 0u || group > kAttnMaxGroup || a->splits % kAttnCluster != 0u || a->splits / kAttnCluster > 32u ||
        grid != a->kv_heads * a->splits || nseq == 0u)
        return cudaErrorInvalidValue;
    if (a->tc && !a->kv_fp16) return cudaErrorInvalidValue;
    return launch_ex(attn_fn(group, a->tc != 0u, true), args, dim3(grid, nseq), dim3(kAttnThreads),
                     atlas_d2_attn_smem(a->splits), stream, true, kAttnCluster);
}

extern "C" cudaError_t atlas_d2_launch_attn(const AttnArgs *a, uint32_t grid, cudaStream_t stream)
{
    AttnArgs copy = *a;
    void *args[] = {&copy};
    const uint32_t group = a->q_heads / a->kv_heads;
    if (group == 0u || group > kAttnMaxGroup || a->splits % kAttnCluster != 0u || a->splits / kAttnCluster > 32u ||
        grid != a->kv_heads * a->splits)
        return cudaErrorInvalidValue;
    if (a->tc && !a->kv_fp16) return cudaErrorInvalidValue;
    return launch_ex(attn_fn(group, a->tc != 0u), args, dim3(grid), dim3(kAttnThreads), atlas_d2_attn_smem(a->splits),
                     stream, true, kAttnCluster);
}

extern "C" cudaError_t atlas_d2_launch_embed(const uint8_t *embd, uint64_t row_bytes, uint32_t type, uint32_t hidden,
                                             uint32_t vocab, float *x, DecState *st, cudaStream_t stream)
{
    void *args[] = {&embd, &row_bytes, &type, &hidden, &vocab, &x, &st};
    return launch_ex((const void *)embed_kernel, args, dim3((hidden + 255u) / 256u), dim3(256), 0, stream, false);
}

extern "C" cudaError_t atlas_d2_launch_argmax(const float *pmax, const uint32_t *pidx, uint32_t n, DecState *st,
                                              const uint32_t *cnt, uint32_t arrivals, cudaStream_t stream)
{
    void *args[] = {&pmax, &pidx, &n, &st, &cnt, &arrivals};
    return launch_ex((const void *)argmax_kernel, args, dim3(1), dim3(256), 0, stream, true);
}

// grid: CTAs of the cooperative launch (the same on every rank)
extern "C" cudaError_t atlas_tp_allreduce(const TpReduceArgs *a, uint32_t grid, cudaStream_t stream)
{
    TpReduceArgs copy = *a;
    void *args[] = {&copy};
    return cudaLaunchCooperativeKernel((const void *)tp_allreduce_kernel, dim3(grid), dim3(256), args, 0, stream);
}
