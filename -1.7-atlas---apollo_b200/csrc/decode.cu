// Persistent decode kernel: one CTA per SM runs a whole decode step (the
// reference's forward_token, src/brain_runtime.c:1698-1772, plus the greedy
// pick of atlas_sample_token :1783) as a program of phases (engine.h).
//
// Warp roles per CTA
//   warp 8 (producer): one lane walks the CTA's work items of every phase in
//     order and issues 1-D bulk copies (cp.async.bulk) of their raw weight
//     rows / KV-cache tiles into an n_stages-deep shared-memory ring, limited
//     only by free ring slots - never by activations - so weight streaming
//     continues across phase boundaries;
//   warps 0-7 (consumers): wait for the previous phase's counter (acquire),
//     stage the phase's input vector in shared memory, consume the staged
//     bytes and release the phase counter.
//
// GEMV on tensor cores (mma.sync m16n8k16, fp32 accumulate), fp32-accurate:
//   A = weights. A 4- or 6-bit quant q, zero-extended into a 16-bit lane, is
//     the fp16 subnormal q * 2^-24 - exactly; one byte permute builds two A
//     values straight from the raw super-block bytes.
//   B = input x split as x = hi + lo, both fp16 (hi = fp16(x), lo =
//     fp16(x - hi)), after scaling x by a power of two so max|x| sits near
//     2^13: 22 significant bits. Even B columns hold hi, odd columns lo, so the
//     fragment of every lane receives sum(q*hi) and sum(q*lo) for its rows.
//   k order: inside each 16-wide k step, lane t's four k slots map to the four
//     consecutive elements 4t..4t+3, so each A fragment register is built from
//     one 32-bit word of the block and B is stored to match.
//   Scales: per 32-element sub-block (Q4_K: d*sc, dmin*m) or 16-element group
//     (Q6_K: d*sc, with the -32 offset folded via the group's sum of x); lane
//     t applies the groups j with j % 4 == t, and the 4 lanes of a row group
//     are summed at the end of an item.
#include <algorithm>
#include <cfloat>
#include "common.cuh"
#include "engine.h"
#include "quant.cuh"
#include "tc_tiles.cuh"

namespace atlas {

struct Chunk {
    const uint8_t *src;     // contiguous chunk: 16-byte aligned source
    uint32_t bytes;         // bytes delivered by the chunk's copies
    uint32_t lead;          // contiguous chunk: offset of the first row in the stage
    uint32_t seg, r0, r1;   // segment, segment-local rows [r0, r1) (ATTN: K/V and positions)
    uint32_t b0, b1;        // block columns [b0, b1)
    uint32_t rel0;          // item-relative row of r0
};

struct __align__(16) SmemHdr {
    uint64_t full[kMaxStages];
    uint64_t empty[kMaxStages];
    Phase ph;
    float wres[2][kConsumerWarps][2][kMaxItemRows];  // per-warp row partials, double-buffered by item
    double dred[kConsumerWarps];
    float fred[kConsumerWarps];
    float inv_rms, xscale;
    float amax[kConsumerWarps];
    uint32_t aidx[kConsumerWarps];
    uint32_t flag;
};

// Attention buffers; they live in the x staging area, which only GEMV phases use.
struct __align__(16) AttnSmem {
    float4 q[kMaxGroup][kHeadDim / 4];  // RoPE'd queries of the item's group
    float4 knew[kHeadDim / 4], vnew[kHeadDim / 4];
    float cw[kMaxSplits][kMaxGroup];    // combine weights exp(m_s - M)
    float cden[kMaxGroup];
};

constexpr uint32_t kHdrBytes = (sizeof(SmemHdr) + 127u) & ~127u;

// View of the dynamic shared memory: header, x staging area, stage ring.
struct Smem {
    SmemHdr *h;
    AttnSmem *a;        // overlays xarea
    uint8_t *xarea;     // GEMV input: groups of 4 elements as 4 hi + 4 lo halves, then one sum per 16 elements
    uint8_t *ring;
    uint32_t n_stages, stage_bytes;
    uint32_t phase_index;   // current phase (diagnostic stamps)
    __device__ __forceinline__ uint8_t *stage(uint32_t k) const { return ring + (size_t)(k % n_stages) * stage_bytes; }
    __device__ __forceinline__ uint64_t *full(uint32_t k) const { return &h->full[k % n_stages]; }
    __device__ __forceinline__ uint64_t *empty(uint32_t k) const { return &h->empty[k % n_stages]; }
    __device__ __forceinline__ uint32_t par(uint32_t k) const { return (k / n_stages) & 1u; }
};

// ------------------------------------------------------ chunk enumeration --

__device__ __forceinline__ void align_range(const uint8_t *p, uint64_t bytes, const uint8_t *&lo, uint32_t &n, uint32_t &lead)
{
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uintptr_t l = a & ~uintptr_t(15), e = (a + bytes + 15) & ~uintptr_t(15);
    lo = reinterpret_cast<const uint8_t *>(l);
    n = (uint32_t)(e - l);
    lead = (uint32_t)(a - l);
}

// Segment portions of GEMV item `it`: (segment, local rows, item-relative row).
__device__ __forceinline__ int gemv_portions(const Phase &ph, uint32_t it, uint32_t (&sg)[2], uint32_t (&la)[2],
                                             uint32_t (&lb)[2], uint32_t (&rel)[2], uint32_t &np)
{
    const uint32_t r0 = it * ph.item_rows;
    np = 0;
    if (ph.paired) {
        const uint32_t r1 = min(r0 + ph.item_rows, ph.seg[0].rows);
        for (uint32_t s = 0; s < ph.n_seg && s < 2; ++s) { sg[np] = s; la[np] = r0; lb[np] = r1; rel[np] = 0; ++np; }
        return (int)np;
    }
    const uint32_t r1 = min(r0 + ph.item_rows, ph.seg_start[ph.n_seg]);
    for (uint32_t s = 0; s < ph.n_seg && np < 2; ++s) {
        const uint32_t a = max(r0, ph.seg_start[s]), b = min(r1, ph.seg_start[s + 1]);
        if (a >= b) continue;
        sg[np] = s; la[np] = a - ph.seg_start[s]; lb[np] = b - ph.seg_start[s]; rel[np] = a - r0; ++np;
    }
    return (int)np;
}

__device__ __forceinline__ uint32_t gemv_colchunks(const Phase &ph)
{
    const uint32_t nb = ph.cols / 256u;
    return (nb + ph.chunk_blocks - 1u) / ph.chunk_blocks;
}

// Chunks of an item: for each segment portion, its rows in runs of
// chunk_rows, each run in column chunks of chunk_blocks.
__device__ __forceinline__ uint32_t gemv_item_chunks(const Phase &ph, uint32_t it)
{
    uint32_t sg[2], la[2], lb[2], rel[2], np;
    gemv_portions(ph, it, sg, la, lb, rel, np);
    uint32_t n = 0;
    for (uint32_t p = 0; p < np; ++p) n += (lb[p] - la[p] + ph.chunk_rows - 1) / ph.chunk_rows;
    return n * gemv_colchunks(ph);
}

__device__ __forceinline__ Chunk gemv_item_chunk(const Phase &ph, uint32_t it, uint32_t ci, bool need_bytes = true)
{
    uint32_t sg[2], la[2], lb[2], rel[2], np;
    gemv_portions(ph, it, sg, la, lb, rel, np);
    const uint32_t ncc = gemv_colchunks(ph), nb = ph.cols / 256u;
    uint32_t run = ci / ncc;
    const uint32_t cb = ci % ncc;
    uint32_t p = 0;
    for (; p + 1 < np; ++p) {
        const uint32_t runs = (lb[p] - la[p] + ph.chunk_rows - 1) / ph.chunk_rows;
        if (run < runs) break;
        run -= runs;
    }
    Chunk c;
    c.seg = sg[p];
    c.r0 = la[p] + run * ph.chunk_rows;
    c.r1 = min(c.r0 + ph.chunk_rows, lb[p]);
    c.rel0 = rel[p] + run * ph.chunk_rows;
    c.b0 = cb * ph.chunk_blocks;
    c.b1 = min(c.b0 + ph.chunk_blocks, nb);
    const Seg &s = ph.seg[c.seg];
    if (ph.seg_stride == 0) {
        align_range(s.w + (uint64_t)c.r0 * s.row_bytes, (uint64_t)(c.r1 - c.r0) * s.row_bytes, c.src, c.bytes, c.lead);
    } else {
        const uint32_t bb = block_bytes(s.type);
        uint32_t total = 0;
        for (uint32_t r = c.r0; need_bytes && r < c.r1; ++r) {
            const uint8_t *lo;
            uint32_t n, lead;
            align_range(s.w + (uint64_t)r * s.row_bytes + (uint64_t)c.b0 * bb, (uint64_t)(c.b1 - c.b0) * bb, lo, n, lead);
            total += n;
        }
        c.src = nullptr;
        c.bytes = total;
        c.lead = 0;
    }
    return c;
}

// Positions per attention item: a multiple of kAttnChunk, grown with the
// context so that kv_heads * splits stays near one item per CTA (and at most
// kMaxSplits splits per KV head).
__device__ __forceinline__ uint32_t attn_split_len(const Program &pg, uint32_t pos)
{
    uint32_t target = gridDim.x / pg.kv_heads;
    if (target < 1u) target = 1u;
    if (target > (uint32_t)kMaxSplits) target = kMaxSplits;
    const uint32_t n = pos + 1u;
    const uint32_t chunks = (n + (uint32_t)kAttnChunk * target - 1u) / ((uint32_t)kAttnChunk * target);
    return (uint32_t)kAttnChunk * (chunks ? chunks : 1u);
}

__device__ __forceinline__ uint32_t attn_items(const Program &pg, uint32_t pos)
{
    const uint32_t L = attn_split_len(pg, pos);
    return pg.kv_heads * ((pos + L) / L);
}

// ATTN item (kv head g, split s) covers positions [p0, min(p0 + L, pos + 1));
// its cached part [p0, min(p0 + L, pos)) is staged as (K, V) chunk pairs of up
// to kAttnChunk positions; position pos comes from the fresh projections.
__device__ __forceinline__ uint32_t attn_item_pairs(const Program &pg, uint32_t item, uint32_t pos)
{
    const uint32_t L = attn_split_len(pg, pos), nsplit = (pos + L) / L;
    const uint32_t s = item % nsplit, p0 = s * L, p1 = min(p0 + L, pos);
    return p1 > p0 ? (p1 - p0 + kAttnChunk - 1) / kAttnChunk : 0u;
}

__device__ __forceinline__ Chunk attn_chunk(const Program &pg, const Phase &ph, uint32_t item, uint32_t pos,
                                            uint32_t pair, uint32_t kv)
{
    const uint32_t L = attn_split_len(pg, pos), nsplit = (pos + L) / L;
    const uint32_t g = item / nsplit, s = item % nsplit;
    const uint32_t t0 = s * L + pair * kAttnChunk, t1 = min(t0 + (uint32_t)kAttnChunk, min(s * L + L, pos));
    const uint32_t esz = pg.kv_fp16 ? 2u : 4u, row = pg.head_dim * esz;
    const uint64_t head_off = (uint64_t)g * pg.max_context * row;
    const uint8_t *base = reinterpret_cast<const uint8_t *>(kv ? ph.v_cache : ph.k_cache);
    Chunk c;
    align_range(base + head_off + (uint64_t)t0 * row, (uint64_t)(t1 - t0) * row, c.src, c.bytes, c.lead);
    c.seg = kv; c.r0 = t0; c.r1 = t1; c.b0 = c.b1 = 0; c.rel0 = 0;
    return c;
}

__device__ __forceinline__ uint32_t phase_items(const Program &pg, const Phase &ph, uint32_t pos)
{
    switch (ph.kind) {
    case PH_GEMV: return ph.n_items;
    case PH_ATTN: return attn_items(pg, pos);
    case PH_EMBED: return (pg.hidden + 255u) / 256u;
    case PH_ARGMAX: return 1u;
    default: return 0u;
    }
}

// --------------------------------------------------------------- producer --

__device__ void producer(const Program &pg, const Smem &sm, uint32_t pos, volatile uint32_t *err)
{
    const uint64_t policy = policy_evict_first();
    uint32_t k = 0;
    for (uint32_t p = 0; p < pg.n_phases; ++p) {
        const Phase &ph = pg.phases[p];
        const uint32_t n = phase_items(pg, ph, pos);
        for (uint32_t it = blockIdx.x; it < n; it += gridDim.x) {
            const uint32_t nc = ph.kind == PH_GEMV ? gemv_item_chunks(ph, it)
                              : ph.kind == PH_ATTN ? 2u * attn_item_pairs(pg, it, pos) : 0u;
            for (uint32_t ci = 0; ci < nc; ++ci, ++k) {
                if (k >= sm.n_stages && !mbar_wait(sm.empty(k), sm.par(k) ^ 1u, err)) return;
                uint8_t *dst = sm.stage(k);
                if (ph.kind == PH_ATTN) {
                    const Chunk c = attn_chunk(pg, ph, it, pos, ci >> 1, ci & 1u);
                    mbar_arrive_expect_tx(sm.full(k), c.bytes);
                    bulk_g2s(dst, c.src, c.bytes, sm.full(k));
                    continue;
                }
                const Chunk c = gemv_item_chunk(ph, it, ci);
                mbar_arrive_expect_tx(sm.full(k), c.bytes);
                if (ph.seg_stride == 0) {
                    bulk_g2s_hint(dst, c.src, c.bytes, sm.full(k), policy);
                } else {
                    const Seg &s = ph.seg[c.seg];
                    const uint32_t bb = block_bytes(s.type);
                    for (uint32_t r = c.r0; r < c.r1; ++r) {
                        const uint8_t *lo;
                        uint32_t nbytes, lead;
                        align_range(s.w + (uint64_t)r * s.row_bytes + (uint64_t)c.b0 * bb, (uint64_t)(c.b1 - c.b0) * bb,
                                    lo, nbytes, lead);
                        bulk_g2s_hint(dst + (size_t)(r - c.r0) * ph.seg_stride, lo, nbytes, sm.full(k), policy);
                    }
                }
            }
        }
        if (pg.trace) pg.trace[((size_t)blockIdx.x * pg.n_phases + p) * 4 + 3] = global_ns();
    }
    // Drain: every issued copy has landed before the CTA may exit.
    for (uint32_t j = (k > sm.n_stages ? k - sm.n_stages : 0); j < k; ++j)
        if (!mbar_wait(sm.full(j), sm.par(j), err)) return;
}

// ------------------------------------------------------------- consumers --

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory"); }

__device__ __forceinline__ bool stage_wait(const Smem &sm, uint32_t k, volatile uint32_t *err)
{
    return mbar_wait(sm.full(k), sm.par(k), err);
}

__device__ __forceinline__ void stage_release(const Smem &sm, uint32_t k)
{
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(sm.empty(k));
}

// Wait (one thread) for every CTA to have finished phase p, then make the
// results visible to all consumer threads.
__device__ __forceinline__ bool wait_phase(const Program &pg, uint32_t p, uint32_t epoch, volatile uint32_t *err)
{
    __shared__ uint32_t ok_flag;
    if (threadIdx.x == 0) {
        // the acquire load orders this CTA's later reads (all from L2) after the
        // producers' release arrivals; the barrier below extends it to the CTA
        const bool ok = wait_counter(pg.phase_ctr + 8u * p, (epoch + 1u) * gridDim.x, err, kStatusBarrierTimeout);
        ok_flag = ok ? 1u : 0u;
    }
    consumer_sync();
    return ok_flag != 0;
}

__device__ __forceinline__ void arrive_phase(const Program &pg, uint32_t p)
{
    consumer_sync();
    if (threadIdx.x == 0) {
        __threadfence();
        red_release_add(pg.phase_ctr + 8u * p, 1u);
    }
}

// Stage the phase input in shared memory as fp16 (hi, lo) groups plus one sum
// per 16 elements, in units of (x * norm_w) * xscale, xscale a power of two.
// One pass over x from L2: the RMSNorm factor is a scalar, so it is applied
// to the GEMV results instead (W (x w inv) = inv * W (x w)); the sum of
// squares (in double, src/brain_runtime.c:1345-1351) and max|x w| come out of
// the same pass and one block reduction. Returns the factor the epilogue
// applies: inv_rms / xscale (1 / xscale for un-normalized inputs).
__device__ float stage_x(const Program &pg, const Phase &ph, const Smem &sm)
{
    const uint32_t n = ph.cols;
    const bool norm = ph.input_mode == IN_RMSNORM;
    float4 *xf = reinterpret_cast<float4 *>(sm.xarea);
    float mx = 0.f;
    double ss = 0.0;
    // four independent loads in flight per thread (x comes from L2)
    constexpr uint32_t kStride = kConsumerWarps * 32;
    for (uint32_t i0 = threadIdx.x; i0 < n / 4u; i0 += 4u * kStride) {
        float4 v[4], w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t i = i0 + (uint32_t)j * kStride;
            if (i < n / 4u) {
                v[j] = __ldcg(reinterpret_cast<const float4 *>(ph.in) + i);
                if (norm) w[j] = __ldg(reinterpret_cast<const float4 *>(ph.norm_w) + i);
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
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) { sm.h->fred[warp] = mx; sm.h->dred[warp] = ss; }
    consumer_sync();
    float m = 0.f;
    double t = 0.0;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) { m = fmaxf(m, sm.h->fred[w]); t += sm.h->dred[w]; }
    // scale so that max|x| lands in [2^13, 2^14): far from fp16 overflow, and
    // the lo parts of small elements stay normal. The exponent is capped at
    // 126 so that the scale stays finite for rows of tiny values (a SwiGLU
    // output of all-negative gates can sit near the fp32 underflow limit);
    // such rows then contribute ~0, as they do in fp32.
    const float s = (m > 0.f && isfinite(m)) ? exp2f((float)min(13 - ilogbf(m), 126)) : 1.0f;
    const float inv_rms = norm ? 1.0f / sqrtf((float)(t / (double)n) + pg.rms_eps) : 1.0f;
    float *xs16 = reinterpret_cast<float *>(sm.xarea + (size_t)n * 4u);
    for (uint32_t u = threadIdx.x; u < n / 16u; u += kConsumerWarps * 32) {
        float sum = 0.f;
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
            uint4 pk;
            pk.x = (uint32_t)__half_as_ushort(hi[0]) | ((uint32_t)__half_as_ushort(hi[1]) << 16);
            pk.y = (uint32_t)__half_as_ushort(hi[2]) | ((uint32_t)__half_as_ushort(hi[3]) << 16);
            pk.z = (uint32_t)__half_as_ushort(lo[0]) | ((uint32_t)__half_as_ushort(lo[1]) << 16);
            pk.w = (uint32_t)__half_as_ushort(lo[2]) | ((uint32_t)__half_as_ushort(lo[3]) << 16);
            reinterpret_cast<uint4 *>(sm.xarea)[4 * u + q] = pk;
        }
        xs16[u] = sum;
    }
    consumer_sync();
    return inv_rms / s;
}

__device__ bool run_gemv_phase(const Program &pg, const Phase &gph, const Smem &sm, uint32_t &k, volatile uint32_t *err)
{
    for (uint32_t i = threadIdx.x; i < sizeof(Phase) / 4; i += kConsumerWarps * 32)
        reinterpret_cast<uint32_t *>(&sm.h->ph)[i] = reinterpret_cast<const uint32_t *>(&gph)[i];
    consumer_sync();
    const Phase &ph = sm.h->ph;
    const float out_scale = stage_x(pg, ph, sm);
    if (pg.trace_ext && threadIdx.x == 0) pg.trace_ext[((size_t)blockIdx.x * pg.n_phases + sm.phase_index) * 8 + 0] = global_ns();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const float *xs16 = reinterpret_cast<const float *>(sm.xarea + (size_t)ph.cols * 4u);
    float best = -FLT_MAX;
    uint32_t best_i = 0xffffffffu;
    uint32_t buf = 0;
    for (uint32_t it = blockIdx.x; it < ph.n_items; it += gridDim.x, buf ^= 1u) {
        float acc[2][kMaxItemRows / 16][2];
#pragma unroll
        for (int a = 0; a < 2; ++a)
#pragma unroll
            for (int b = 0; b < kMaxItemRows / 16; ++b) { acc[a][b][0] = 0.f; acc[a][b][1] = 0.f; }
        const uint32_t nc = gemv_item_chunks(ph, it);
        uint32_t task = 0;
        for (uint32_t ci = 0; ci < nc; ++ci, ++k) {
            const Chunk c = gemv_item_chunk(ph, it, ci, false);
            if (!stage_wait(sm, k, err)) return false;
            const Seg &sg = ph.seg[c.seg];
            const uint32_t bb = block_bytes(sg.type);
            const uint32_t nrows = c.r1 - c.r0, nrt = (nrows + 15u) / 16u, ncol = c.b1 - c.b0;
            const uint32_t slot = ph.paired ? c.seg : 0u;
            const uint8_t *st = sm.stage(k);
            const uint32_t ntasks = nrt * ncol;
            // tasks of this chunk handled by this warp: (task + i) % 8 == warp
            const uint32_t first = (uint32_t)(warp - (int)(task % kConsumerWarps) + kConsumerWarps) % kConsumerWarps;
            const uint64_t coff = (uint64_t)c.b0 * bb;
            // row pointers of task ti for this lane's rows (nullptr: row absent)
            auto rows_of = [&](uint32_t ti, const uint8_t *&p0, const uint8_t *&p1, uint32_t &bcol, uint32_t &irt) {
                const uint32_t rt = ti / ncol, bl = ti % ncol;
                const uint32_t i0 = rt * 16u + (uint32_t)g, i1 = i0 + 8u;
                p0 = p1 = nullptr;
                if (ph.seg_stride == 0) {
                    const uint8_t *base = st + c.lead + (uint64_t)(c.b0 + bl) * bb;
                    if (i0 < nrows) p0 = base + (uint64_t)i0 * sg.row_bytes;
                    if (i1 < nrows) p1 = base + (uint64_t)i1 * sg.row_bytes;
                } else {
                    const uintptr_t w = reinterpret_cast<uintptr_t>(sg.w);
                    if (i0 < nrows) p0 = st + (size_t)i0 * ph.seg_stride + ((w + (uint64_t)(c.r0 + i0) * sg.row_bytes + coff) & 15u) + (uint64_t)bl * bb;
                    if (i1 < nrows) p1 = st + (size_t)i1 * ph.seg_stride + ((w + (uint64_t)(c.r0 + i1) * sg.row_bytes + coff) & 15u) + (uint64_t)bl * bb;
                }
                bcol = c.b0 + bl;
                irt = (c.rel0 / 16u) + rt;   // item row tile
            };
            auto add = [&](uint32_t irt, float o0, float o1) {
#pragma unroll
                for (int q = 0; q < kMaxItemRows / 16; ++q) {
                    if ((uint32_t)q != irt) continue;
                    if (slot == 0u) { acc[0][q][0] += o0; acc[0][q][1] += o1; }
                    else { acc[1][q][0] += o0; acc[1][q][1] += o1; }
                }
            };
            const bool full = (nrows % 16u) == 0u;   // every row tile of the chunk has its 16 rows
            uint32_t ti = first;
            for (; ti + kConsumerWarps < ntasks; ti += 2u * kConsumerWarps) {
                const uint8_t *p0[2], *p1[2], *xb[2];
                const float *xs[2];
                uint32_t bcol[2], irt[2];
                rows_of(ti, p0[0], p1[0], bcol[0], irt[0]);
                rows_of(ti + kConsumerWarps, p0[1], p1[1], bcol[1], irt[1]);
#pragma unroll
                for (int n = 0; n < 2; ++n) { xb[n] = sm.xarea + (size_t)bcol[n] * 1024u; xs[n] = xs16 + (size_t)bcol[n] * 16u; }
                float o0[2] = {0.f, 0.f}, o1[2] = {0.f, 0.f};
                if (full) {
                    if (sg.type == 12u) q4k_tiles<2, true>(p0, p1, xb, xs, g, t, o0, o1);
                    else q6k_tiles<2, true>(p0, p1, xb, xs, g, t, o0, o1);
                } else {
                    if (sg.type == 12u) q4k_tiles<2, false>(p0, p1, xb, xs, g, t, o0, o1);
                    else q6k_tiles<2, false>(p0, p1, xb, xs, g, t, o0, o1);
                }
                add(irt[0], o0[0], o1[0]);
                add(irt[1], o0[1], o1[1]);
            }
            if (ti < ntasks) {
                const uint8_t *p0[1], *p1[1], *xb[1];
                const float *xs[1];
                uint32_t bcol, irt;
                rows_of(ti, p0[0], p1[0], bcol, irt);
                xb[0] = sm.xarea + (size_t)bcol * 1024u;
                xs[0] = xs16 + (size_t)bcol * 16u;
                float o0[1] = {0.f}, o1[1] = {0.f};
                if (sg.type == 12u) q4k_tiles<1, false>(p0, p1, xb, xs, g, t, o0, o1);
                else q6k_tiles<1, false>(p0, p1, xb, xs, g, t, o0, o1);
                add(irt, o0[0], o1[0]);
            }
            task += ntasks;
            stage_release(sm, k);
        }
        // per-warp partials: sum the 4 lanes of each row group, stage them, one barrier
        const uint32_t item_r0 = it * ph.item_rows;
        const uint32_t total = ph.paired ? ph.seg[0].rows : ph.seg_start[ph.n_seg];
        const uint32_t nr = min(ph.item_rows, total - item_r0);
        const uint32_t nslots = ph.paired ? ph.n_seg : 1u;
#pragma unroll
        for (int a = 0; a < 2; ++a)
#pragma unroll
            for (int q = 0; q < kMaxItemRows / 16; ++q)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    float v = acc[a][q][e];
                    v += __shfl_xor_sync(0xffffffffu, v, 1);
                    v += __shfl_xor_sync(0xffffffffu, v, 2);
                    const uint32_t r = (uint32_t)q * 16u + (uint32_t)g + 8u * (uint32_t)e;
                    if (t == 0 && (uint32_t)a < nslots && r < (uint32_t)kMaxItemRows) sm.h->wres[buf][warp][a][r] = v;
                }
        consumer_sync();
        for (uint32_t r = threadIdx.x; r < nr; r += kConsumerWarps * 32) {
            float v0 = 0.f, v1 = 0.f;
#pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) {
                v0 += sm.h->wres[buf][w][0][r];
                v1 += sm.h->wres[buf][w][1][r];
            }
            v0 *= out_scale;
            v1 *= out_scale;
            const uint32_t row = item_r0 + r;
            if (ph.epilogue == EPI_SWIGLU) {
                ph.seg[0].out[row] = (v0 / (1.0f + expf(-v0))) * v1;   // src/brain_runtime.c:1755-1758
            } else {
                uint32_t sgi = 0;
                while (sgi + 1 < ph.n_seg && row >= ph.seg_start[sgi + 1]) ++sgi;
                const uint32_t lr = row - ph.seg_start[sgi];
                float *out = ph.seg[sgi].out;
                if (ph.epilogue == EPI_RESID_ADD) {
                    out[lr] = __ldcg(out + lr) + v0;
                } else {
                    const float *bias = ph.seg[sgi].bias;
                    out[lr] = bias ? v0 + __ldg(bias + lr) : v0;
                    if (v0 > best || (v0 == best && lr < best_i)) { best = v0; best_i = lr; }
                }
            }
        }
    }
    if (ph.epilogue == EPI_LOGITS) {
        // one (max, argmax) per CTA; the greedy pick reduces them
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, best, o);
            const uint32_t oi = __shfl_xor_sync(0xffffffffu, best_i, o);
            if (ob > best || (ob == best && oi < best_i)) { best = ob; best_i = oi; }
        }
        if (lane == 0) { sm.h->amax[warp] = best; sm.h->aidx[warp] = best_i; }
        consumer_sync();
        if (threadIdx.x == 0) {
            for (int w = 1; w < kConsumerWarps; ++w)
                if (sm.h->amax[w] > best || (sm.h->amax[w] == best && sm.h->aidx[w] < best_i)) { best = sm.h->amax[w]; best_i = sm.h->aidx[w]; }
            ph.partial_max[blockIdx.x] = best;
            ph.partial_idx[blockIdx.x] = best_i;
        }
    }
    consumer_sync();
    return true;
}

// RoPE angle for pair p at position pos from the host-built table (the
// reference's powf/cosf/sinf values, src/brain_runtime.c:1383-1387).
__device__ __forceinline__ void rope_pair(const Program &pg, uint32_t pos, int p, float a, float b, float &oa, float &ob)
{
    const float2 cs = __ldg(pg.rope + (size_t)pos * (pg.head_dim / 2) + p);
    oa = a * cs.x - b * cs.y;   // src/brain_runtime.c:1391-1393
    ob = a * cs.y + b * cs.x;
}

__device__ __forceinline__ float4 kv_row4(const uint8_t *row, uint32_t i4, bool f16)
{
    if (!f16) return reinterpret_cast<const float4 *>(row)[i4];
    const uint2 h = reinterpret_cast<const uint2 *>(row)[i4];
    const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&h.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&h.y));
    return make_float4(a.x, a.y, b.x, b.y);
}

__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Split-K flash-decode (gqa_single_token, src/brain_runtime.c:1482-1528): for
// each (kv head g, split s) item, every warp takes one query head of the group
// and walks the split's positions 32 at a time, one position per lane (score
// = q . k over 128 dims read in a lane-rotated order, conflict-free), with an
// online softmax; P.V accumulates with lane = 4 output dims. The last split of
// a head to finish combines all splits' (max, sum, acc) partials; a partial is
// stored as acc[head_dim], max, sum, 2 pad floats (16-byte aligned records).
__device__ bool run_attn_phase(const Program &pg, const Phase &ph, const Smem &sm, uint32_t &k, uint32_t pos,
                               volatile uint32_t *err)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t hd = pg.head_dim, group = pg.q_heads / pg.kv_heads;
    const uint32_t L = attn_split_len(pg, pos), nsplit = (pos + L) / L;
    const uint32_t n = pg.kv_heads * nsplit;
    const float scale = 1.0f / sqrtf((float)hd);
    const bool f16 = pg.kv_fp16 != 0;
    const uint32_t row_bytes = hd * (f16 ? 2u : 4u);
    for (uint32_t it = blockIdx.x; it < n; it += gridDim.x) {
        const uint32_t g = it / nsplit, s = it % nsplit;
        const uint32_t p0 = s * L, p1 = min(p0 + L, pos + 1);
        const bool last_split = (p1 == pos + 1);
        // RoPE'd queries of the group; the fresh k (RoPE'd) and v in the last split
        float *qf = reinterpret_cast<float *>(sm.a->q);
        {
            // group * 64 pairs over 256 threads: at most 2 per thread, loads first
            constexpr uint32_t kStride = kConsumerWarps * 32;
            float qa[2], qb[2];
            float2 cs[2];
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const uint32_t i = threadIdx.x + (uint32_t)j * kStride;
                if (i < group * (hd / 2)) {
                    const uint32_t h = i / (hd / 2), p = i % (hd / 2);
                    const float *qh = ph.q + (size_t)(g * group + h) * hd;
                    qa[j] = __ldcg(qh + p);
                    qb[j] = __ldcg(qh + p + hd / 2);
                    cs[j] = __ldg(pg.rope + (size_t)pos * (hd / 2) + p);
                }
            }
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const uint32_t i = threadIdx.x + (uint32_t)j * kStride;
                if (i < group * (hd / 2)) {
                    const uint32_t h = i / (hd / 2), p = i % (hd / 2);
                    qf[h * hd + p] = qa[j] * cs[j].x - qb[j] * cs[j].y;       // src/brain_runtime.c:1391-1393
                    qf[h * hd + p + hd / 2] = qa[j] * cs[j].y + qb[j] * cs[j].x;
                }
            }
        }
        if (last_split) {
            float *kn = reinterpret_cast<float *>(sm.a->knew), *vn = reinterpret_cast<float *>(sm.a->vnew);
            for (uint32_t p = threadIdx.x; p < hd / 2; p += kConsumerWarps * 32) {
                const float *kh = ph.k + (size_t)g * hd;
                float a, b;
                rope_pair(pg, pos, (int)p, __ldcg(kh + p), __ldcg(kh + p + hd / 2), a, b);
                kn[p] = a;
                kn[p + hd / 2] = b;
            }
            for (uint32_t i = threadIdx.x; i < hd; i += kConsumerWarps * 32) vn[i] = __ldcg(ph.v + (size_t)g * hd + i);
        }
        consumer_sync();
        if (pg.trace_ext && threadIdx.x == 0 && it == blockIdx.x) pg.trace_ext[((size_t)blockIdx.x * pg.n_phases + sm.phase_index) * 8 + 0] = global_ns();
        if (last_split) {
            // KV append at pos (src/brain_runtime.c:1496-1500); read by the next steps.
            const float *kn = reinterpret_cast<const float *>(sm.a->knew), *vn = reinterpret_cast<const float *>(sm.a->vnew);
            const size_t off = ((size_t)g * pg.max_context + pos) * hd;
            for (uint32_t i = threadIdx.x; i < hd; i += kConsumerWarps * 32) {
                if (f16) {
                    reinterpret_cast<__half *>(ph.k_cache)[off + i] = __float2half_rn(kn[i]);
                    reinterpret_cast<__half *>(ph.v_cache)[off + i] = __float2half_rn(vn[i]);
                } else {
                    reinterpret_cast<float *>(ph.k_cache)[off + i] = kn[i];
                    reinterpret_cast<float *>(ph.v_cache)[off + i] = vn[i];
                }
            }
        }
        // per-warp state for its query head (group <= 8 = one head per warp)
        float m[1] = {-FLT_MAX}, l[1] = {0.f};
        float4 acc[1] = {make_float4(0.f, 0.f, 0.f, 0.f)};
        const uint32_t cached_end = min(p1, pos);
        for (uint32_t t0 = p0; t0 < p1; t0 += kAttnChunk) {
            const bool staged = t0 < cached_end;
            const uint8_t *kst = nullptr, *vst = nullptr;
            if (staged) {
                if (!stage_wait(sm, k, err)) return false;
                if (!stage_wait(sm, k + 1, err)) return false;
                if (pg.trace_ext && threadIdx.x == 0 && it == blockIdx.x && t0 == p0)
                    pg.trace_ext[((size_t)blockIdx.x * pg.n_phases + sm.phase_index) * 8 + 3] = global_ns();
                const uint32_t esz = f16 ? 2u : 4u;
                const uintptr_t ka = reinterpret_cast<uintptr_t>(ph.k_cache) + ((size_t)g * pg.max_context + t0) * hd * esz;
                const uintptr_t va = reinterpret_cast<uintptr_t>(ph.v_cache) + ((size_t)g * pg.max_context + t0) * hd * esz;
                kst = sm.stage(k) + (ka & 15u);
                vst = sm.stage(k + 1) + (va & 15u);
            }
            const uint32_t t_end = min(t0 + (uint32_t)kAttnChunk, p1);
            for (uint32_t sb = t0; sb < t_end; sb += 32) {
                const uint32_t p = sb + (uint32_t)lane;
                const bool valid = p < t_end;
                const bool fresh = p == pos;
                const uint8_t *krow = fresh ? reinterpret_cast<const uint8_t *>(sm.a->knew)
                                            : (staged ? kst + (size_t)(p - t0) * row_bytes : nullptr);
                const bool krow_f16 = f16 && !fresh;
#pragma unroll
                for (int hi = 0; hi < 1; ++hi) {
                    const uint32_t h = (uint32_t)warp + (uint32_t)hi * kConsumerWarps;
                    if (h >= group) break;
                    float sc = -FLT_MAX;
                    if (valid) {
                        float dot = 0.f;
#pragma unroll 8
                        for (uint32_t i = 0; i < 32; ++i) {
                            const uint32_t d4 = (i + (uint32_t)lane) & 31u;
                            const float4 qv = sm.a->q[h][d4];
                            const float4 kv = kv_row4(krow, d4, krow_f16);
                            dot = fmaf(qv.x, kv.x, dot);
                            dot = fmaf(qv.y, kv.y, dot);
                            dot = fmaf(qv.z, kv.z, dot);
                            dot = fmaf(qv.w, kv.w, dot);
                        }
                        sc = dot * scale;
                    }
                    const float mn = fmaxf(m[hi], warp_max(sc));
                    const float corr = expf(m[hi] - mn);
                    const float w = valid ? expf(sc - mn) : 0.f;
                    l[hi] = l[hi] * corr + warp_sum(w);
                    float4 a = acc[hi];
                    a.x *= corr; a.y *= corr; a.z *= corr; a.w *= corr;
                    const uint32_t np = min(32u, t_end - sb);
                    for (uint32_t j = 0; j < np; ++j) {
                        const float wj = __shfl_sync(0xffffffffu, w, (int)j);
                        const uint32_t pj = sb + j;
                        const float4 vv = pj == pos ? sm.a->vnew[lane]
                                                    : kv_row4(vst + (size_t)(pj - t0) * row_bytes, (uint32_t)lane, f16);
                        a.x = fmaf(wj, vv.x, a.x);
                        a.y = fmaf(wj, vv.y, a.y);
                        a.z = fmaf(wj, vv.z, a.z);
                        a.w = fmaf(wj, vv.w, a.w);
                    }
                    acc[hi] = a;
                    m[hi] = mn;
                }
            }
            if (pg.trace_ext && threadIdx.x == 0 && it == blockIdx.x && t0 == p0)
                pg.trace_ext[((size_t)blockIdx.x * pg.n_phases + sm.phase_index) * 8 + 4] = global_ns();
            if (staged) {
                stage_release(sm, k);
                stage_release(sm, k + 1);
                k += 2;
            }
        }
        for (int hi = 0; hi < 1; ++hi) {
            const uint32_t h = (uint32_t)warp + (uint32_t)hi * kConsumerWarps;
            if (h >= group) break;
            float *dst = ph.part + (((size_t)g * nsplit + s) * group + h) * (hd + 4);
            reinterpret_cast<float4 *>(dst)[lane] = acc[hi];
            if (lane == 0) { dst[hd] = m[hi]; dst[hd + 1] = l[hi]; }
        }
        // Last split of head g to arrive combines all splits.
        consumer_sync();
        if (pg.trace_ext && threadIdx.x == 0 && it == blockIdx.x) pg.trace_ext[((size_t)blockIdx.x * pg.n_phases + sm.phase_index) * 8 + 1] = global_ns();
        if (threadIdx.x == 0) {
            __threadfence();
            const uint32_t old = atom_acq_rel_add(ph.split_ctr + g, 1u);
            sm.h->flag = (old == nsplit - 1u) ? 1u : 0u;
            if (sm.h->flag) { ph.split_ctr[g] = 0u; __threadfence(); }
        }
        consumer_sync();
        if (pg.trace_ext && threadIdx.x == 0 && it == blockIdx.x) pg.trace_ext[((size_t)blockIdx.x * pg.n_phases + sm.phase_index) * 8 + 2] = global_ns();
        if (sm.h->flag) {
            for (uint32_t h = (uint32_t)warp; h < group; h += kConsumerWarps) {
                // one pass over the splits' (max, sum): lane q holds splits q, q + 32
                float ms[2] = {-FLT_MAX, -FLT_MAX}, ls[2] = {0.f, 0.f};
#pragma unroll
                for (int r = 0; r < 2; ++r) {
                    const uint32_t q = (uint32_t)lane + 32u * r;
                    if (q < nsplit) {
                        const float2 ml = __ldcg(reinterpret_cast<const float2 *>(
                            ph.part + (((size_t)g * nsplit + q) * group + h) * (hd + 4) + hd));
                        ms[r] = ml.x;
                        ls[r] = ml.y;
                    }
                }
                const float M = warp_max(fmaxf(ms[0], ms[1]));
                float den = 0.f;
#pragma unroll
                for (int r = 0; r < 2; ++r) {
                    const uint32_t q = (uint32_t)lane + 32u * r;
                    if (q < nsplit) {
                        const float w = expf(ms[r] - M);
                        sm.a->cw[q][h] = w;
                        den += w * ls[r];
                    }
                }
                den = warp_sum(den);
                if (lane == 0) sm.a->cden[h] = den;
            }
            consumer_sync();
            for (uint32_t i = threadIdx.x; i < group * (hd / 4); i += kConsumerWarps * 32) {
                const uint32_t h = i / (hd / 4), d4 = i % (hd / 4);
                float4 num = make_float4(0.f, 0.f, 0.f, 0.f);
                // eight partial loads in flight at a time (they come from L2)
                for (uint32_t q0 = 0; q0 < nsplit; q0 += 8) {
                    float4 v[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        if (q0 + j < nsplit)
                            v[j] = __ldcg(reinterpret_cast<const float4 *>(
                                ph.part + (((size_t)g * nsplit + q0 + j) * group + h) * (hd + 4)) + d4);
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        if (q0 + j < nsplit) {
                            const float w = sm.a->cw[q0 + j][h];
                            num.x = fmaf(w, v[j].x, num.x);
                            num.y = fmaf(w, v[j].y, num.y);
                            num.z = fmaf(w, v[j].z, num.z);
                            num.w = fmaf(w, v[j].w, num.w);
                        }
                }
                const float den = sm.a->cden[h];
                const float inv = den > 0.f ? 1.0f / den : 0.f;
                float4 o = make_float4(num.x * inv, num.y * inv, num.z * inv, num.w * inv);
                reinterpret_cast<float4 *>(ph.att + (size_t)(g * group + h) * hd)[d4] = o;
            }
        }
        consumer_sync();
    }
    return true;
}

// token_embd row of the current token -> x, bit-exact (load_embedding_row,
// src/brain_runtime.c:1311-1332); item i covers elements [256 i, 256 i + 256).
__device__ void run_embed_phase(const Program &pg, const Phase &ph, uint32_t token)
{
    const uint32_t be = block_elems(ph.embd_type), bb = block_bytes(ph.embd_type);
    const uint8_t *row = ph.embd + (uint64_t)token * ph.embd_row_bytes;
    for (uint32_t it = blockIdx.x; it * 256u < pg.hidden; it += gridDim.x) {
        const uint32_t i = it * 256u + threadIdx.x;
        if (i < pg.hidden) ph.x[i] = deq_elem(ph.embd_type, row + (i / be) * bb, (int)(i % be));
    }
}

// Greedy pick over the head items' partials (lowest index among equal maxima).
__device__ void run_argmax_phase(const Program &pg, const Phase &ph, const Smem &sm)
{
    if (blockIdx.x != 0) return;
    const Phase &head = pg.phases[ph.layer];  // index of the logits phase
    float best = -FLT_MAX;
    uint32_t bi = 0xffffffffu;
    const uint32_t nparts = min(ph.argmax_items, gridDim.x);  // one partial per CTA with head items
    for (uint32_t i = threadIdx.x; i < nparts; i += kConsumerWarps * 32) {
        const float v = __ldcg(head.partial_max + i);
        const uint32_t idx = __ldcg(head.partial_idx + i);
        if (v > best || (v == best && idx < bi)) { best = v; bi = idx; }
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
    }
    if (lane == 0) { sm.h->amax[warp] = best; sm.h->aidx[warp] = bi; }
    consumer_sync();
    if (threadIdx.x == 0) {
        for (int w = 1; w < kConsumerWarps; ++w)
            if (sm.h->amax[w] > best || (sm.h->amax[w] == best && sm.h->aidx[w] < bi)) { best = sm.h->amax[w]; bi = sm.h->aidx[w]; }
        StepState *st = pg.state;
        st->next_token = bi;
        st->next_logit = best;
        if (st->out_ids && st->step < st->max_steps) st->out_ids[st->step] = bi;
    }
}


__device__ bool consumer(const Program &pg, Smem sm, uint32_t pos, uint32_t token, uint32_t epoch,
                         volatile uint32_t *err)
{
    uint32_t k = 0;
    uint64_t *tr = pg.trace ? pg.trace + (size_t)blockIdx.x * pg.n_phases * 4 : nullptr;
    for (uint32_t p = 0; p < pg.n_phases; ++p) {
        const Phase &ph = pg.phases[p];
        const uint32_t n = phase_items(pg, ph, pos);
        const bool mine = blockIdx.x < n;
        sm.phase_index = p;
        if (tr && threadIdx.x == 0) tr[p * 4 + 0] = global_ns();
        if (mine && p > 0 && !wait_phase(pg, p - 1, epoch, err)) return false;
        if (tr && threadIdx.x == 0) tr[p * 4 + 1] = global_ns();
        if (mine) {
            bool ok = true;
            switch (ph.kind) {
            case PH_GEMV: ok = run_gemv_phase(pg, ph, sm, k, err); break;
            case PH_ATTN: ok = run_attn_phase(pg, ph, sm, k, pos, err); break;
            case PH_EMBED: run_embed_phase(pg, ph, token); break;
            case PH_ARGMAX: run_argmax_phase(pg, ph, sm); break;
            default: break;
            }
            if (!ok) return false;
        }
        arrive_phase(pg, p);
        if (tr && threadIdx.x == 0) tr[p * 4 + 2] = global_ns();
    }
    return true;
}

__global__ void __launch_bounds__(kThreads, 1) decode_kernel(Program pg)
{
    extern __shared__ __align__(128) uint8_t smem_raw[];
    Smem sm;
    sm.h = reinterpret_cast<SmemHdr *>(smem_raw);
    sm.xarea = smem_raw + kHdrBytes;
    sm.a = reinterpret_cast<AttnSmem *>(sm.xarea);
    sm.ring = sm.xarea + max(x_area_bytes(pg.max_cols), (uint32_t)((sizeof(AttnSmem) + 127u) & ~127u));
    sm.n_stages = pg.n_stages;
    sm.stage_bytes = pg.stage_bytes;
    StepState *st = pg.state;
    volatile uint32_t *err = &st->status;
    const uint32_t pos = st->pos, token = st->token, epoch = st->epoch;
    const int warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < sm.n_stages; ++s) {
            mbar_init(&sm.h->full[s], 1);
            mbar_init(&sm.h->empty[s], kConsumerWarps);
        }
        fence_mbar_init();
    }
    __syncthreads();
    if (warp == kConsumerWarps) {
        if ((threadIdx.x & 31) == 0) producer(pg, sm, pos, err);
    } else {
        consumer(pg, sm, pos, token, epoch, err);
    }
    __syncthreads();
    // The last CTA out advances the step state for the next launch.
    if (threadIdx.x == 0) {
        __threadfence();
        const uint32_t old = atom_acq_rel_add(&st->exit_ctr, 1u);
        if (old == (epoch + 1u) * gridDim.x - 1u) {
            if (pg.advance && st->status == kStatusOk) {
                st->token = st->next_token;
                st->pos = pos + 1u;
                st->step = st->step + 1u;
            }
            __threadfence();
            st->epoch = epoch + 1u;
        }
    }
}

}  // namespace atlas

extern "C" size_t atlas_decode_hdr_bytes() { return atlas::kHdrBytes; }
extern "C" size_t atlas_decode_attn_bytes() { return (sizeof(atlas::AttnSmem) + 127u) & ~size_t(127); }

// Host-side launcher (used by model.cu). smem = header + x area + ring.
extern "C" cudaError_t atlas_launch_decode(const atlas::Program *pg, int grid, cudaStream_t stream)
{
    const size_t xa = std::max<size_t>(atlas::x_area_bytes(pg->max_cols), (sizeof(atlas::AttnSmem) + 127u) & ~size_t(127));
    const size_t smem = atlas::kHdrBytes + xa + (size_t)pg->n_stages * pg->stage_bytes;
    static size_t configured[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (configured[dev] < smem) {
        e = cudaFuncSetAttribute(atlas::decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        configured[dev] = smem;
    }
    void *args[] = {const_cast<atlas::Program *>(pg)};
    return cudaLaunchCooperativeKernel((const void *)atlas::decode_kernel, dim3(grid), dim3(atlas::kThreads), args, smem,
                                       stream);
}
