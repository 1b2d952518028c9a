// Persistent decode kernel: one CTA per SM runs a whole decode step (the
// reference's forward_token, src/brain_runtime.c:1698-1772, plus the greedy
// pick of atlas_sample_token :1783) as a program of phases (engine.h).
//
// Per CTA (8 warps)
//   * the pump (thread 0, called between its own work and inside every wait
//     loop): walks the CTA's work items of every phase in order and issues 1-D
//     bulk copies (cp.async.bulk, TMA) of their raw weight rows / KV-cache tiles
//     into a kStages-deep shared-memory ring, limited only by free ring slots -
//     never by activations - so weight streaming continues across phase
//     boundaries;
//   * all warps: wait for the previous phase's counter (acquire), load this
//     phase's activation vector into registers, and consume the staged bytes:
//     Q4_K/Q6_K decode + fp32 FMA + warp-shuffle row reductions, or
//     flash-decode attention; then release the phase counter.
#include <cfloat>
#include "common.cuh"
#include "engine.h"
#include "quant.cuh"

namespace atlas {

struct Chunk {
    const uint8_t *src;   // 16-byte aligned source
    uint32_t bytes;       // multiple of 16
    uint32_t lead;        // offset of the first useful byte inside the stage
    uint32_t seg, r0, r1; // GEMV: segment and its local rows; ATTN: 0=K / 1=V and positions
};

struct __align__(128) Smem {
    uint8_t stage[kStages][kStageBytes];
    uint64_t full[kStages];
    uint64_t empty[kStages];
    float rowres[kMaxSeg][kMaxItemRows];
    float red[kConsumerWarps], red2[kConsumerWarps];
    double dred[kConsumerWarps];
    Phase ph;                           // current GEMV phase descriptor
    float inv_rms;
    float amax[kConsumerWarps];
    uint32_t aidx[kConsumerWarps];
    uint32_t flag;
    // attention
    float4 q[kMaxGroup][kHeadDim / 4];  // RoPE'd queries of the item's group
    float4 knew[kHeadDim / 4], vnew[kHeadDim / 4];
    float cw[kMaxSplits][kMaxGroup];    // combine weights exp(m_s - M)
    float cden[kMaxGroup];
    // pump (thread 0): position of the next chunk to issue
    uint32_t pump_p, pump_it, pump_c, pump_nc, pump_issued, pump_done;
    Chunk pump_ch[kMaxSeg];
};


// ------------------------------------------------------ chunk enumeration --

__device__ __forceinline__ Chunk make_chunk(const uint8_t *base, uint64_t start, uint64_t bytes)
{
    const uintptr_t a = reinterpret_cast<uintptr_t>(base) + start;
    const uintptr_t lo = a & ~uintptr_t(15), hi = (a + bytes + 15) & ~uintptr_t(15);
    Chunk c;
    c.src = reinterpret_cast<const uint8_t *>(lo);
    c.bytes = (uint32_t)(hi - lo);
    c.lead = (uint32_t)(a - lo);
    return c;
}

// GEMV item -> up to kMaxSeg chunks (one per segment touched).
__device__ __forceinline__ int gemv_chunks(const Phase &ph, uint32_t item, Chunk (&out)[kMaxSeg])
{
    int n = 0;
    const uint32_t r0 = item * ph.item_rows;
    if (ph.paired) {
        const uint32_t r1 = min(r0 + ph.item_rows, ph.seg[0].rows);
        for (uint32_t s = 0; s < ph.n_seg; ++s) {
            Chunk c = make_chunk(ph.seg[s].w, (uint64_t)r0 * ph.seg[s].row_bytes,
                                 (uint64_t)(r1 - r0) * ph.seg[s].row_bytes);
            c.seg = s; c.r0 = r0; c.r1 = r1;
            out[n++] = c;
        }
        return n;
    }
    const uint32_t r1 = min(r0 + ph.item_rows, ph.seg_start[ph.n_seg]);
    for (uint32_t s = 0; s < ph.n_seg; ++s) {
        const uint32_t a = max(r0, ph.seg_start[s]), b = min(r1, ph.seg_start[s + 1]);
        if (a >= b) continue;
        const uint32_t la = a - ph.seg_start[s], lb = b - ph.seg_start[s];
        Chunk c = make_chunk(ph.seg[s].w, (uint64_t)la * ph.seg[s].row_bytes,
                             (uint64_t)(lb - la) * ph.seg[s].row_bytes);
        c.seg = s; c.r0 = la; c.r1 = lb;
        out[n++] = c;
    }
    return n;
}

// Positions per attention item: a multiple of kAttnChunk, grown with the
// context so that kv_heads * splits stays near one item per CTA (and at most
// kMaxSplits splits per KV head).
__device__ __forceinline__ uint32_t attn_split_len(const Program &pg, uint32_t pos)
{
    uint32_t target = gridDim.x / pg.kv_heads;
    if (target < 1u) target = 1u;
    if (target > (uint32_t)kMaxSplits / 2u) target = kMaxSplits / 2u;
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
__device__ __forceinline__ int attn_chunks(const Program &pg, const Phase &ph, uint32_t item, uint32_t pos,
                                           Chunk (&out)[kMaxSeg])
{
    (void)out;
    return 0;  // attention items are enumerated chunk-pair by chunk-pair (attn_chunk_pair)
}

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
    Chunk c = make_chunk(base, head_off + (uint64_t)t0 * row, (uint64_t)(t1 - t0) * row);
    c.seg = kv; c.r0 = t0; c.r1 = t1;
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

// Number of staged chunks of an item, and chunk i of it (GEMV chunks are
// precomputed into `buf` by item_chunk_count).
__device__ __forceinline__ uint32_t item_chunk_count(const Program &pg, const Phase &ph, uint32_t item, uint32_t pos,
                                                     Chunk (&buf)[kMaxSeg])
{
    if (ph.kind == PH_GEMV) return (uint32_t)gemv_chunks(ph, item, buf);
    if (ph.kind == PH_ATTN) return 2u * attn_item_pairs(pg, item, pos);
    return 0u;
}

__device__ __forceinline__ Chunk item_chunk(const Program &pg, const Phase &ph, uint32_t item, uint32_t pos, uint32_t i,
                                            const Chunk (&buf)[kMaxSeg])
{
    if (ph.kind == PH_ATTN) return attn_chunk(pg, ph, item, pos, i >> 1, i & 1u);
    return buf[i];
}

// ------------------------------------------------------------------ pump --

// Thread 0 only. Issues bulk copies for upcoming chunks while ring slots are
// free (a slot is free once all 8 warps released the chunk kStages earlier);
// never blocks.
__device__ void pump(const Program &pg, Smem &sm, uint32_t pos)
{
    while (!sm.pump_done) {
        const uint32_t k = sm.pump_issued, s = k % kStages, round = k / kStages;
        if (round > 0 && !mbar_test(&sm.empty[s], (round - 1) & 1u)) return;
        // find the next chunk
        while (sm.pump_c >= sm.pump_nc) {
            // advance to the next item of this CTA (or the next phase)
            const Phase &ph = pg.phases[sm.pump_p];
            uint32_t it = sm.pump_it + gridDim.x;
            if (sm.pump_nc == 0xffffffffu) it = blockIdx.x;  // first item of phase pump_p
            if (it < phase_items(pg, ph, pos)) {
                sm.pump_it = it;
                sm.pump_nc = item_chunk_count(pg, ph, it, pos, sm.pump_ch);
                sm.pump_c = 0;
            } else {
                if (++sm.pump_p >= pg.n_phases) { sm.pump_done = 1; return; }
                sm.pump_nc = 0xffffffffu;
                sm.pump_c = 0xffffffffu;
            }
        }
        const Chunk c = item_chunk(pg, pg.phases[sm.pump_p], sm.pump_it, pos, sm.pump_c++, sm.pump_ch);
        mbar_arrive_expect_tx(&sm.full[s], c.bytes);
        if (pg.phases[sm.pump_p].kind == PH_GEMV) bulk_g2s_hint(sm.stage[s], c.src, c.bytes, &sm.full[s], policy_evict_first());
        else bulk_g2s(sm.stage[s], c.src, c.bytes, &sm.full[s]);
        sm.pump_issued = k + 1;
        if (pg.trace && sm.pump_done == 0) pg.trace[((size_t)blockIdx.x * pg.n_phases + sm.pump_p) * 4 + 3] = global_ns();
    }
}

// Wait for chunk k's bytes (all threads); thread 0 keeps pumping meanwhile.
__device__ __forceinline__ bool stage_wait(const Program &pg, Smem &sm, uint32_t k, uint32_t pos,
                                           volatile uint32_t *err)
{
    const uint32_t s = k % kStages, par = (k / kStages) & 1u;
    if (threadIdx.x != 0) return mbar_wait(&sm.full[s], par, err);
    uint64_t t0 = 0;
    for (uint32_t i = 0;; ++i) {
        pump(pg, sm, pos);
        if (mbar_test(&sm.full[s], par)) return true;
        if ((i & 15u) == 15u) {
            if (*err != kStatusOk) return false;
            const uint64_t now = global_ns();
            if (!t0) t0 = now;
            else if (now - t0 > kWaitLimitNs) break;
        }
    }
    atomicCAS(const_cast<uint32_t *>(err), kStatusOk, kStatusStageTimeout);
    return false;
}

// Release chunk k's stage (one arrival per warp); thread 0 refills the ring.
__device__ __forceinline__ void stage_release(const Program &pg, Smem &sm, uint32_t k, uint32_t pos)
{
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(&sm.empty[k % kStages]);
    if (threadIdx.x == 0) pump(pg, sm, pos);
}

// ------------------------------------------------------------- consumers --

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory"); }

__device__ __forceinline__ void group_sync(int id, int nthreads)
{
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Wait (one thread) for every CTA to have finished phase p, then make the
// results visible to all consumer threads.
__device__ __forceinline__ bool wait_phase(const Program &pg, Smem &sm, uint32_t p, uint32_t epoch, uint32_t pos,
                                           volatile uint32_t *err)
{
    __shared__ uint32_t ok_flag;
    if (threadIdx.x == 0) {
        const uint32_t *ctr = pg.phase_ctr + 8u * p;
        const uint32_t target = (epoch + 1u) * gridDim.x;
        bool ok = false;
        uint64_t t0 = 0;
        for (uint32_t i = 0;; ++i) {
            if ((int32_t)(ld_acquire(ctr) - target) >= 0) { ok = true; break; }
            if (*err != kStatusOk) break;
            pump(pg, sm, pos);
            if ((i & 15u) == 15u) {
                const uint64_t now = global_ns();
                if (!t0) t0 = now;
                else if (now - t0 > kWaitLimitNs) {
                    atomicCAS(const_cast<uint32_t *>(err), kStatusOk, kStatusBarrierTimeout);
                    break;
                }
            }
        }
        __threadfence();
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

// Per-CTA RMSNorm scale over the hidden vector (sum of squares in double as
// src/brain_runtime.c:1345-1351; 1/sqrtf(float(mean)+eps) as :1353-1358).
__device__ float cta_inv_rms(const float *x, uint32_t n, float eps, Smem &sm)
{
    double ss = 0.0;
    for (uint32_t i = threadIdx.x * 4u; i < n; i += kConsumerWarps * 32 * 4) {
        const float4 v = __ldcg(reinterpret_cast<const float4 *>(x + i));
        ss += (double)v.x * (double)v.x;
        ss += (double)v.y * (double)v.y;
        ss += (double)v.z * (double)v.z;
        ss += (double)v.w * (double)v.w;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) sm.dred[warp] = ss;
    consumer_sync();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int w = 0; w < kConsumerWarps; ++w) t += sm.dred[w];
        sm.inv_rms = 1.0f / sqrtf((float)(t / (double)n) + eps);
    }
    consumer_sync();
    return sm.inv_rms;
}

// Rows of one staged chunk, for the NS slices this lane owns. Two rows are in
// flight per warp for instruction-level parallelism.
template <int NS, bool Q6>
__device__ __forceinline__ void chunk_rows(const uint8_t *base, uint64_t rb, uint32_t nrows, uint32_t NG, int gi,
                                           const uint32_t (&boff)[NS], const int (&cc)[NS], const int (&hf)[NS],
                                           const bool (&valid)[NS], const SliceX (&x)[NS], float *res, uint32_t W,
                                           int wi, int warp, int lane, Smem &sm)
{
    for (uint32_t r = (uint32_t)gi; r < nrows; r += 2u * NG) {
        const uint8_t *p0 = base + (uint64_t)r * rb;
        const bool two = r + NG < nrows;
        const uint8_t *p1 = two ? p0 + (uint64_t)NG * rb : p0;
        float a0 = 0.f, a1 = 0.f;
#pragma unroll
        for (int j = 0; j < NS; ++j) {
            if (valid[j]) {
                if (Q6) {
                    a0 += q6k_slice_dot(p0 + boff[j], cc[j], hf[j], x[j]);
                    a1 += q6k_slice_dot(p1 + boff[j], cc[j], hf[j], x[j]);
                } else {
                    a0 += q4k_slice_dot(p0 + boff[j], cc[j], hf[j], x[j]);
                    a1 += q4k_slice_dot(p1 + boff[j], cc[j], hf[j], x[j]);
                }
            }
        }
        a0 = warp_sum(a0);
        a1 = warp_sum(a1);
        if (W == 1u) {
            if (lane == 0) {
                res[r] = a0;
                if (two) res[r + NG] = a1;
            }
        } else {
            if (lane == 0) { sm.red[warp] = a0; sm.red2[warp] = a1; }
            group_sync(2 + gi, (int)W * 32);
            if (wi == 0 && lane == 0) {
                float t0 = 0.f, t1 = 0.f;
                for (uint32_t q = 0; q < W; ++q) { t0 += sm.red[gi * W + q]; t1 += sm.red2[gi * W + q]; }
                res[r] = t0;
                if (two) res[r + NG] = t1;
            }
            group_sync(2 + gi, (int)W * 32);
        }
    }
}

template <int NS>
__device__ bool run_gemv_phase(const Program &pg, const Phase &gph, Smem &sm, uint32_t &k, uint32_t pos,
                               volatile uint32_t *err)
{
    // The descriptor is read throughout the phase: keep a copy in shared memory.
    for (uint32_t i = threadIdx.x; i < sizeof(Phase) / 4; i += kConsumerWarps * 32)
        reinterpret_cast<uint32_t *>(&sm.ph)[i] = reinterpret_cast<const uint32_t *>(&gph)[i];
    consumer_sync();
    const Phase &ph = sm.ph;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t W = ph.warps_per_row, NG = kConsumerWarps / W;
    const int gi = warp / (int)W, wi = warp % (int)W;
    const uint32_t S = ph.cols / 32u;
    const float *in = ph.in;
    float inv = 1.f;
    const bool norm = ph.input_mode == IN_RMSNORM;
    if (norm) inv = cta_inv_rms(in, ph.cols, pg.rms_eps, sm);
    // This lane's slices of the (normalized) input, and their positions.
    SliceX x[NS];
    uint32_t blk[NS];
    int cc[NS], hf[NS];
    bool valid[NS];
#pragma unroll
    for (int j = 0; j < NS; ++j) {
        const uint32_t s = (uint32_t)(wi * 32 + lane) + (uint32_t)j * 32u * W;
        valid[j] = s < S;
        const uint32_t ss = valid[j] ? s : 0u;
        blk[j] = ss >> 3;
        cc[j] = (int)((ss & 7u) >> 1);
        hf[j] = (int)(ss & 1u);
        const uint32_t base = 256u * blk[j] + 64u * (uint32_t)cc[j] + 16u * (uint32_t)hf[j];
        float lo[16], hi[16];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            float4 a = __ldcg(reinterpret_cast<const float4 *>(in + base + 4 * q));
            float4 b = __ldcg(reinterpret_cast<const float4 *>(in + base + 32 + 4 * q));
            if (norm) {
                const float4 wa = __ldg(reinterpret_cast<const float4 *>(ph.norm_w + base + 4 * q));
                const float4 wb = __ldg(reinterpret_cast<const float4 *>(ph.norm_w + base + 32 + 4 * q));
                a.x = a.x * inv * wa.x; a.y = a.y * inv * wa.y; a.z = a.z * inv * wa.z; a.w = a.w * inv * wa.w;
                b.x = b.x * inv * wb.x; b.y = b.y * inv * wb.y; b.z = b.z * inv * wb.z; b.w = b.w * inv * wb.w;
            }
            lo[4 * q] = a.x; lo[4 * q + 1] = a.y; lo[4 * q + 2] = a.z; lo[4 * q + 3] = a.w;
            hi[4 * q] = b.x; hi[4 * q + 1] = b.y; hi[4 * q + 2] = b.z; hi[4 * q + 3] = b.w;
        }
        float sl = 0.f, sh = 0.f;
#pragma unroll
        for (int e = 0; e < 16; ++e) {
            if (!valid[j]) { lo[e] = 0.f; hi[e] = 0.f; }
            sl += lo[e];
            sh += hi[e];
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            x[j].lo[e] = make_float2(lo[2 * e], lo[2 * e + 1]);
            x[j].hi[e] = make_float2(hi[2 * e], hi[2 * e + 1]);
        }
        x[j].slo = sl;
        x[j].shi = sh;
    }
    float best = -FLT_MAX;
    uint32_t best_i = 0xffffffffu;
    for (uint32_t it = blockIdx.x; it < ph.n_items; it += gridDim.x) {
        Chunk ch[kMaxSeg];
        const int nc = gemv_chunks(ph, it, ch);
        const uint32_t item_r0 = it * ph.item_rows;
        for (int c = 0; c < nc; ++c, ++k) {
            const uint32_t s = k % kStages;
            if (!stage_wait(pg, sm, k, pos, err)) return false;
            const uint32_t sg = ch[c].seg;
            const uint64_t rb = ph.seg[sg].row_bytes;
            const uint8_t *base = sm.stage[s] + ch[c].lead;
            const uint32_t nrows = ch[c].r1 - ch[c].r0;
            const uint32_t rel0 = ph.paired ? 0u : (ch[c].r0 + ph.seg_start[sg] - item_r0);
            float *res = &sm.rowres[sg][rel0];
            if (ph.seg[sg].type == 14u) {
                uint32_t boff[NS];
#pragma unroll
                for (int j = 0; j < NS; ++j) boff[j] = 210u * blk[j];
                chunk_rows<NS, true>(base, rb, nrows, NG, gi, boff, cc, hf, valid, x, res, W, wi, warp, lane, sm);
            } else {
                uint32_t boff[NS];
#pragma unroll
                for (int j = 0; j < NS; ++j) boff[j] = 144u * blk[j];
                chunk_rows<NS, false>(base, rb, nrows, NG, gi, boff, cc, hf, valid, x, res, W, wi, warp, lane, sm);
            }
            stage_release(pg, sm, k, pos);
        }
        consumer_sync();
        // epilogue over the item's rows
        const uint32_t total = ph.paired ? ph.seg[0].rows : ph.seg_start[ph.n_seg];
        const uint32_t nr = min(ph.item_rows, total - item_r0);
        for (uint32_t r = threadIdx.x; r < nr; r += kConsumerWarps * 32) {
            const uint32_t row = item_r0 + r;
            if (ph.epilogue == EPI_SWIGLU) {
                const float z = sm.rowres[0][r], up = sm.rowres[1][r];
                ph.seg[0].out[row] = (z / (1.0f + expf(-z))) * up;   // src/brain_runtime.c:1755-1758
            } else {
                uint32_t sgi = 0;
                while (sgi + 1 < ph.n_seg && row >= ph.seg_start[sgi + 1]) ++sgi;
                const uint32_t lr = row - ph.seg_start[sgi];
                const float v = sm.rowres[sgi][r];
                float *out = ph.seg[sgi].out;
                if (ph.epilogue == EPI_RESID_ADD) {
                    out[lr] = __ldcg(out + lr) + v;
                } else {
                    const float *bias = ph.seg[sgi].bias;
                    out[lr] = bias ? v + __ldg(bias + lr) : v;
                    if (v > best || (v == best && lr < best_i)) { best = v; best_i = lr; }
                }
            }
        }
        consumer_sync();
    }
    if (ph.epilogue == EPI_LOGITS) {
        // one (max, argmax) per CTA; the greedy pick reduces gridDim.x of them
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, best, o);
            const uint32_t oi = __shfl_xor_sync(0xffffffffu, best_i, o);
            if (ob > best || (ob == best && oi < best_i)) { best = ob; best_i = oi; }
        }
        if (lane == 0) { sm.amax[warp] = best; sm.aidx[warp] = best_i; }
        consumer_sync();
        if (threadIdx.x == 0) {
            for (int w = 1; w < kConsumerWarps; ++w)
                if (sm.amax[w] > best || (sm.amax[w] == best && sm.aidx[w] < best_i)) { best = sm.amax[w]; best_i = sm.aidx[w]; }
            ph.partial_max[blockIdx.x] = best;
            ph.partial_idx[blockIdx.x] = best_i;
        }
    }
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
__device__ bool run_attn_phase(const Program &pg, const Phase &ph, Smem &sm, uint32_t &k, uint32_t pos,
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
        float *qf = reinterpret_cast<float *>(sm.q);
        for (uint32_t i = threadIdx.x; i < group * (hd / 2); i += kConsumerWarps * 32) {
            const uint32_t h = i / (hd / 2), p = i % (hd / 2);
            const float *qh = ph.q + (size_t)(g * group + h) * hd;
            float a, b;
            rope_pair(pg, pos, (int)p, __ldcg(qh + p), __ldcg(qh + p + hd / 2), a, b);
            qf[h * hd + p] = a;
            qf[h * hd + p + hd / 2] = b;
        }
        if (last_split) {
            float *kn = reinterpret_cast<float *>(sm.knew), *vn = reinterpret_cast<float *>(sm.vnew);
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
        if (last_split) {
            // KV append at pos (src/brain_runtime.c:1496-1500); read by the next steps.
            const float *kn = reinterpret_cast<const float *>(sm.knew), *vn = reinterpret_cast<const float *>(sm.vnew);
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
        // per-warp state for up to two query heads (group <= 16 over 8 warps)
        float m[2] = {-FLT_MAX, -FLT_MAX}, l[2] = {0.f, 0.f};
        float4 acc[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
        const uint32_t cached_end = min(p1, pos);
        for (uint32_t t0 = p0; t0 < p1; t0 += kAttnChunk) {
            const bool staged = t0 < cached_end;
            const uint8_t *kst = nullptr, *vst = nullptr;
            if (staged) {
                if (!stage_wait(pg, sm, k, pos, err)) return false;
                if (!stage_wait(pg, sm, k + 1, pos, err)) return false;
                const uint32_t esz = f16 ? 2u : 4u;
                const uintptr_t ka = reinterpret_cast<uintptr_t>(ph.k_cache) + ((size_t)g * pg.max_context + t0) * hd * esz;
                const uintptr_t va = reinterpret_cast<uintptr_t>(ph.v_cache) + ((size_t)g * pg.max_context + t0) * hd * esz;
                kst = sm.stage[k % kStages] + (ka & 15u);
                vst = sm.stage[(k + 1) % kStages] + (va & 15u);
            }
            const uint32_t t_end = min(t0 + (uint32_t)kAttnChunk, p1);
            for (uint32_t sb = t0; sb < t_end; sb += 32) {
                const uint32_t p = sb + (uint32_t)lane;
                const bool valid = p < t_end;
                const bool fresh = p == pos;
                const uint8_t *krow = fresh ? reinterpret_cast<const uint8_t *>(sm.knew)
                                            : (staged ? kst + (size_t)(p - t0) * row_bytes : nullptr);
                const bool krow_f16 = f16 && !fresh;
#pragma unroll
                for (int hi = 0; hi < 2; ++hi) {
                    const uint32_t h = (uint32_t)warp + (uint32_t)hi * kConsumerWarps;
                    if (h >= group) break;
                    float sc = -FLT_MAX;
                    if (valid) {
                        float dot = 0.f;
#pragma unroll 8
                        for (uint32_t i = 0; i < 32; ++i) {
                            const uint32_t d4 = (i + (uint32_t)lane) & 31u;
                            const float4 qv = sm.q[h][d4];
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
                        const float4 vv = pj == pos ? sm.vnew[lane]
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
            if (staged) {
                stage_release(pg, sm, k, pos);
                stage_release(pg, sm, k + 1, pos);
                k += 2;
            }
        }
        for (int hi = 0; hi < 2; ++hi) {
            const uint32_t h = (uint32_t)warp + (uint32_t)hi * kConsumerWarps;
            if (h >= group) break;
            float *dst = ph.part + (((size_t)g * nsplit + s) * group + h) * (hd + 4);
            reinterpret_cast<float4 *>(dst)[lane] = acc[hi];
            if (lane == 0) { dst[hd] = m[hi]; dst[hd + 1] = l[hi]; }
        }
        // Last split of head g to arrive combines all splits.
        consumer_sync();
        if (threadIdx.x == 0) {
            __threadfence();
            const uint32_t old = atom_acq_rel_add(ph.split_ctr + g, 1u);
            sm.flag = (old == nsplit - 1u) ? 1u : 0u;
            if (sm.flag) { ph.split_ctr[g] = 0u; __threadfence(); }
        }
        consumer_sync();
        if (sm.flag) {
            for (uint32_t h = (uint32_t)warp; h < group; h += kConsumerWarps) {
                float M = -FLT_MAX;
                for (uint32_t q = (uint32_t)lane; q < nsplit; q += 32)
                    M = fmaxf(M, __ldcg(ph.part + (((size_t)g * nsplit + q) * group + h) * (hd + 4) + hd));
                M = warp_max(M);
                float den = 0.f;
                for (uint32_t q = (uint32_t)lane; q < nsplit; q += 32) {
                    const float *src = ph.part + (((size_t)g * nsplit + q) * group + h) * (hd + 4);
                    const float w = expf(__ldcg(src + hd) - M);
                    sm.cw[q][h] = w;
                    den += w * __ldcg(src + hd + 1);
                }
                den = warp_sum(den);
                if (lane == 0) sm.cden[h] = den;
            }
            consumer_sync();
            for (uint32_t i = threadIdx.x; i < group * (hd / 4); i += kConsumerWarps * 32) {
                const uint32_t h = i / (hd / 4), d4 = i % (hd / 4);
                float4 num = make_float4(0.f, 0.f, 0.f, 0.f);
                for (uint32_t q = 0; q < nsplit; ++q) {
                    const float w = sm.cw[q][h];
                    const float4 v = __ldcg(reinterpret_cast<const float4 *>(
                        ph.part + (((size_t)g * nsplit + q) * group + h) * (hd + 4)) + d4);
                    num.x = fmaf(w, v.x, num.x);
                    num.y = fmaf(w, v.y, num.y);
                    num.z = fmaf(w, v.z, num.z);
                    num.w = fmaf(w, v.w, num.w);
                }
                const float den = sm.cden[h];
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
__device__ void run_argmax_phase(const Program &pg, const Phase &ph, Smem &sm)
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
    if (lane == 0) { sm.amax[warp] = best; sm.aidx[warp] = bi; }
    consumer_sync();
    if (threadIdx.x == 0) {
        for (int w = 1; w < kConsumerWarps; ++w)
            if (sm.amax[w] > best || (sm.amax[w] == best && sm.aidx[w] < bi)) { best = sm.amax[w]; bi = sm.aidx[w]; }
        StepState *st = pg.state;
        st->next_token = bi;
        st->next_logit = best;
        if (st->out_ids && st->step < st->max_steps) st->out_ids[st->step] = bi;
    }
}

template <int NS>
__device__ bool dispatch_gemv(const Program &pg, const Phase &ph, Smem &sm, uint32_t &k, volatile uint32_t *err);

__device__ bool consumer(const Program &pg, Smem &sm, uint32_t pos, uint32_t token, uint32_t epoch,
                         volatile uint32_t *err)
{
    uint32_t k = 0;
    uint64_t *tr = pg.trace ? pg.trace + (size_t)blockIdx.x * pg.n_phases * 4 : nullptr;
    for (uint32_t p = 0; p < pg.n_phases; ++p) {
        const Phase &ph = pg.phases[p];
        const uint32_t n = phase_items(pg, ph, pos);
        const bool mine = blockIdx.x < n;
        if (tr && threadIdx.x == 0) tr[p * 4 + 0] = global_ns();
        if (mine && p > 0 && !wait_phase(pg, sm, p - 1, epoch, pos, err)) return false;
        if (tr && threadIdx.x == 0) tr[p * 4 + 1] = global_ns();
        if (mine) {
            bool ok = true;
            switch (ph.kind) {
            case PH_GEMV:
                switch (ph.n_slices) {
                case 1: ok = run_gemv_phase<1>(pg, ph, sm, k, pos, err); break;
                case 2: ok = run_gemv_phase<2>(pg, ph, sm, k, pos, err); break;
                case 3: ok = run_gemv_phase<(kMaxSlices >= 3 ? 3 : 1)>(pg, ph, sm, k, pos, err); break;
                default: ok = run_gemv_phase<kMaxSlices>(pg, ph, sm, k, pos, err); break;
                }
                break;
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
    Smem &sm = *reinterpret_cast<Smem *>(smem_raw);
    StepState *st = pg.state;
    volatile uint32_t *err = &st->status;
    const uint32_t pos = st->pos, token = st->token, epoch = st->epoch;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], kConsumerWarps);
        }
        fence_mbar_init();
        sm.pump_p = 0;
        sm.pump_it = 0;
        sm.pump_c = 0xffffffffu;
        sm.pump_nc = 0xffffffffu;
        sm.pump_issued = 0;
        sm.pump_done = pg.n_phases == 0;
    }
    __syncthreads();
    if (threadIdx.x == 0) pump(pg, sm, pos);
    consumer(pg, sm, pos, token, epoch, err);
    __syncthreads();
    if (threadIdx.x == 0) {
        // Every issued copy must have landed before the CTA exits (they all
        // have on the normal path; after an error some may still be in flight).
        for (uint32_t j = 0; j < sm.pump_issued; ++j) {
            if (j + kStages < sm.pump_issued) continue;
            uint64_t t0 = global_ns();
            while (!mbar_test(&sm.full[j % kStages], (j / kStages) & 1u) && global_ns() - t0 < kWaitLimitNs) {}
        }
        // The last CTA out advances the step state for the next launch.
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

// Host-side launcher (used by model.cu).
extern "C" cudaError_t atlas_launch_decode(const atlas::Program *pg, int grid, cudaStream_t stream)
{
    const size_t smem = sizeof(atlas::Smem);
    static bool configured[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!configured[dev]) {
        e = cudaFuncSetAttribute(atlas::decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    void *args[] = {const_cast<atlas::Program *>(pg)};
    return cudaLaunchCooperativeKernel((const void *)atlas::decode_kernel, dim3(grid), dim3(atlas::kThreads), args, smem,
                                       stream);
}

extern "C" size_t atlas_decode_smem_bytes() { return sizeof(atlas::Smem); }
