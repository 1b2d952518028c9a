// Persistent decode kernel: one CTA per SM runs a whole decode step (the
// reference's forward_token, src/brain_runtime.c:1698-1772, plus the greedy
// pick of atlas_sample_token :1783) as a program of phases (engine.h).
//
// Warp roles per CTA
//   warp 8 (producer): one elected lane walks the CTA's work items of every
//     phase in order and issues 1-D bulk copies (cp.async.bulk, TMA) of their
//     raw weight rows / KV-cache tiles into a kStages-deep shared-memory ring,
//     limited only by free ring slots - never by activations - so weight
//     streaming continues across phase boundaries.
//   warps 0-7 (consumers): wait for the previous phase's counter (acquire),
//     load this phase's activation vector into registers, and consume the
//     staged bytes: Q4_K/Q6_K decode + fp32 FMA + warp-shuffle row reductions,
//     or flash-decode attention; then release the phase counter.
#include <cfloat>
#include "common.cuh"
#include "engine.h"
#include "quant.cuh"

namespace atlas {

struct __align__(128) Smem {
    uint8_t stage[kStages][kStageBytes];
    uint64_t full[kStages];
    uint64_t empty[kStages];
    float rowres[kMaxSeg][kMaxItemRows];
    float red[kConsumerWarps];
    double dred[kConsumerWarps];
    float inv_rms;
    float amax[kConsumerWarps];
    uint32_t aidx[kConsumerWarps];
    uint32_t flag;
    // attention
    float q[kMaxGroup][kHeadDim];       // RoPE'd queries of the item's group
    float knew[kHeadDim], vnew[kHeadDim];
    float ml[kMaxGroup][2];
};

struct Chunk {
    const uint8_t *src;   // 16-byte aligned source
    uint32_t bytes;       // multiple of 16
    uint32_t lead;        // offset of the first useful byte inside the stage
    uint32_t seg, r0, r1; // GEMV: segment and its local rows; ATTN: 0=K / 1=V and positions
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

__device__ __forceinline__ uint32_t attn_split_len(const Program &pg)
{
    return kStageBytes / (pg.head_dim * (pg.kv_fp16 ? 2u : 4u));
}

__device__ __forceinline__ uint32_t attn_items(const Program &pg, uint32_t pos)
{
    return pg.kv_heads * ((pos + attn_split_len(pg)) / attn_split_len(pg));
}

// ATTN item (kv head g, split s): cached positions [p0, min(p1, pos)) as a K
// chunk and a V chunk; the current position comes from the fresh projections.
__device__ __forceinline__ int attn_chunks(const Program &pg, const Phase &ph, uint32_t item, uint32_t pos,
                                           Chunk (&out)[kMaxSeg])
{
    const uint32_t L = attn_split_len(pg), nsplit = (pos + L) / L;
    const uint32_t g = item / nsplit, s = item % nsplit;
    const uint32_t p0 = s * L, p1 = min(p0 + L, pos);
    if (p1 <= p0) return 0;
    const uint32_t esz = pg.kv_fp16 ? 2u : 4u, row = pg.head_dim * esz;
    const uint64_t head_off = (uint64_t)g * pg.max_context * row;
    int n = 0;
    for (uint32_t kv = 0; kv < 2; ++kv) {
        const uint8_t *base = reinterpret_cast<const uint8_t *>(kv ? ph.v_cache : ph.k_cache);
        Chunk c = make_chunk(base, head_off + (uint64_t)p0 * row, (uint64_t)(p1 - p0) * row);
        c.seg = kv; c.r0 = p0; c.r1 = p1;
        out[n++] = c;
    }
    return n;
}

__device__ __forceinline__ uint32_t phase_items(const Program &pg, const Phase &ph, uint32_t pos)
{
    switch (ph.kind) {
    case PH_GEMV: return ph.n_items;
    case PH_ATTN: return attn_items(pg, pos);
    case PH_EMBED: return 1u;
    case PH_ARGMAX: return 1u;
    default: return 0u;
    }
}

__device__ __forceinline__ int item_chunks(const Program &pg, const Phase &ph, uint32_t item, uint32_t pos,
                                           Chunk (&out)[kMaxSeg])
{
    if (ph.kind == PH_GEMV) return gemv_chunks(ph, item, out);
    if (ph.kind == PH_ATTN) return attn_chunks(pg, ph, item, pos, out);
    return 0;
}

// --------------------------------------------------------------- producer --

__device__ void producer(const Program &pg, Smem &sm, uint32_t pos, volatile uint32_t *err)
{
    const uint64_t policy = policy_evict_first();
    uint32_t k = 0;
    for (uint32_t p = 0; p < pg.n_phases; ++p) {
        const Phase &ph = pg.phases[p];
        const uint32_t n = phase_items(pg, ph, pos);
        for (uint32_t it = blockIdx.x; it < n; it += gridDim.x) {
            Chunk ch[kMaxSeg];
            const int nc = item_chunks(pg, ph, it, pos, ch);
            for (int c = 0; c < nc; ++c, ++k) {
                const uint32_t s = k % kStages, round = k / kStages;
                if (round > 0 && !mbar_wait(&sm.empty[s], (round - 1) & 1u, err)) return;
                mbar_arrive_expect_tx(&sm.full[s], ch[c].bytes);
                if (ph.kind == PH_GEMV) bulk_g2s_hint(sm.stage[s], ch[c].src, ch[c].bytes, &sm.full[s], policy);
                else bulk_g2s(sm.stage[s], ch[c].src, ch[c].bytes, &sm.full[s]);
            }
        }
        if (pg.trace) pg.trace[((size_t)blockIdx.x * pg.n_phases + p) * 4 + 3] = global_ns();
    }
    // Drain: every issued copy must have landed before the CTA can exit
    // (waiting on the copies themselves, not on the consumers, so an aborted
    // consumer cannot stall this).
    for (uint32_t j = (k > kStages ? k - kStages : 0); j < k; ++j) {
        const uint32_t s = j % kStages;
        if (!mbar_wait(&sm.full[s], (j / kStages) & 1u, err, kStatusStageTimeout)) return;
    }
}

// ------------------------------------------------------------- consumers --

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory"); }

__device__ __forceinline__ void group_sync(int id, int nthreads)
{
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Wait (one thread) for every CTA to have finished phase p, then make the
// results visible to all consumer threads.
__device__ __forceinline__ bool wait_phase(const Program &pg, uint32_t p, uint32_t epoch, volatile uint32_t *err)
{
    __shared__ uint32_t ok_flag;
    if (threadIdx.x == 0) {
        const bool ok = wait_counter(pg.phase_ctr + 8u * p, (epoch + 1u) * gridDim.x, err, kStatusBarrierTimeout);
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
    for (uint32_t i = threadIdx.x; i < n; i += kConsumerWarps * 32) {
        const double v = (double)__ldcg(x + i);
        ss += v * v;
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

template <int NS>
struct XRegs {
    SliceX sl[NS];
};

// Load this lane's slices of the (optionally normalized) input vector.
template <int NS>
__device__ __forceinline__ void load_x(const Phase &ph, float inv, int wi, int lane, XRegs<NS> &xr)
{
    const uint32_t S = ph.cols / 32u, W = ph.warps_per_row;
#pragma unroll
    for (int j = 0; j < NS; ++j) {
        const uint32_t s = (uint32_t)(wi * 32 + lane) + (uint32_t)j * 32u * W;
        SliceX &x = xr.sl[j];
        x.slo = 0.f; x.shi = 0.f;
        if (s >= S) {
#pragma unroll
            for (int e = 0; e < 8; ++e) { x.lo[e] = make_float2(0.f, 0.f); x.hi[e] = make_float2(0.f, 0.f); }
            continue;
        }
        const uint32_t b = s >> 3, c = (s & 7u) >> 1, hf = s & 1u;
        const uint32_t base = 256u * b + 64u * c + 16u * hf;
        float v[32];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
            const uint32_t i0 = base + e, i1 = base + 32u + e;
            float a = __ldcg(ph.in + i0), bb = __ldcg(ph.in + i1);
            if (ph.input_mode == IN_RMSNORM) {
                a = a * inv * __ldg(ph.norm_w + i0);
                bb = bb * inv * __ldg(ph.norm_w + i1);
            }
            v[e] = a; v[16 + e] = bb;
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            x.lo[e] = make_float2(v[2 * e], v[2 * e + 1]);
            x.hi[e] = make_float2(v[16 + 2 * e], v[16 + 2 * e + 1]);
        }
        float sl = 0.f, sh = 0.f;
#pragma unroll
        for (int e = 0; e < 16; ++e) { sl += v[e]; sh += v[16 + e]; }
        x.slo = sl; x.shi = sh;
    }
}

template <int NS>
__device__ __forceinline__ float row_dot(const uint8_t *row, uint32_t type, uint32_t S, uint32_t W, int wi, int lane,
                                         const XRegs<NS> &xr)
{
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < NS; ++j) {
        const uint32_t s = (uint32_t)(wi * 32 + lane) + (uint32_t)j * 32u * W;
        if (s < S) {
            const uint32_t b = s >> 3, c = (s & 7u) >> 1, hf = s & 1u;
            if (type == 12u) acc += q4k_slice_dot(row + 144u * b, (int)c, (int)hf, xr.sl[j]);
            else acc += q6k_slice_dot(row + 210u * b, (int)c, (int)hf, xr.sl[j]);
        }
    }
    return acc;
}

template <int NS>
__device__ bool run_gemv_phase(const Program &pg, const Phase &ph, Smem &sm, uint32_t &k, volatile uint32_t *err)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t W = ph.warps_per_row, NG = kConsumerWarps / W;
    const int gi = warp / (int)W, wi = warp % (int)W;
    const uint32_t S = ph.cols / 32u;
    float inv = 1.f;
    if (ph.input_mode == IN_RMSNORM) inv = cta_inv_rms(ph.in, ph.cols, pg.rms_eps, sm);
    XRegs<NS> xr;
    load_x<NS>(ph, inv, wi, lane, xr);
    for (uint32_t it = blockIdx.x; it < ph.n_items; it += gridDim.x) {
        Chunk ch[kMaxSeg];
        const int nc = gemv_chunks(ph, it, ch);
        const uint32_t item_r0 = it * ph.item_rows;
        for (int c = 0; c < nc; ++c, ++k) {
            const uint32_t s = k % kStages;
            if (!mbar_wait(&sm.full[s], (k / kStages) & 1u, err)) return false;
            const Seg &sg = ph.seg[ch[c].seg];
            const uint8_t *base = sm.stage[s] + ch[c].lead;
            const uint32_t nrows = ch[c].r1 - ch[c].r0;
            // item-relative row index of this chunk's first row
            const uint32_t rel0 = ph.paired ? 0u : (ch[c].r0 + ph.seg_start[ch[c].seg] - item_r0);
            for (uint32_t r = (uint32_t)gi; r < nrows; r += NG) {
                float v = warp_sum(row_dot<NS>(base + (uint64_t)r * sg.row_bytes, sg.type, S, W, wi, lane, xr));
                if (W == 1u) {
                    if (lane == 0) sm.rowres[ch[c].seg][rel0 + r] = v;
                } else {
                    if (lane == 0) sm.red[warp] = v;
                    group_sync(2 + gi, (int)W * 32);
                    if (wi == 0 && lane == 0) {
                        float t = 0.f;
                        for (uint32_t q = 0; q < W; ++q) t += sm.red[gi * W + q];
                        sm.rowres[ch[c].seg][rel0 + r] = t;
                    }
                    group_sync(2 + gi, (int)W * 32);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.empty[s]);
        }
        consumer_sync();
        // epilogue over the item's rows
        const uint32_t total = ph.paired ? ph.seg[0].rows : ph.seg_start[ph.n_seg];
        const uint32_t nr = min(ph.item_rows, total - item_r0);
        float best = -FLT_MAX;
        uint32_t best_i = 0xffffffffu;
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
                const Seg &sg = ph.seg[sgi];
                if (ph.epilogue == EPI_RESID_ADD) {
                    sg.out[lr] = __ldcg(sg.out + lr) + v;
                } else {
                    sg.out[lr] = sg.bias ? v + __ldg(sg.bias + lr) : v;
                    if (ph.epilogue == EPI_LOGITS && (v > best || (v == best && lr < best_i))) { best = v; best_i = lr; }
                }
            }
        }
        if (ph.epilogue == EPI_LOGITS) {
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
                ph.partial_max[it] = best;
                ph.partial_idx[it] = best_i;
            }
        }
        consumer_sync();
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

__device__ __forceinline__ float kv_load(const void *base, bool fp16, size_t i)
{
    return fp16 ? __half2float(reinterpret_cast<const __half *>(base)[i]) : reinterpret_cast<const float *>(base)[i];
}

// Split-K flash-decode for one (kv head, split) item, then the combine by the
// last split to arrive (gqa_single_token, src/brain_runtime.c:1482-1528).
__device__ bool run_attn_phase(const Program &pg, const Phase &ph, Smem &sm, uint32_t &k, uint32_t pos,
                               volatile uint32_t *err)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t hd = pg.head_dim, group = pg.q_heads / pg.kv_heads;
    const uint32_t L = attn_split_len(pg), nsplit = (pos + L) / L;
    const uint32_t n = pg.kv_heads * nsplit;
    const float scale = 1.0f / sqrtf((float)hd);
    const bool f16 = pg.kv_fp16 != 0;
    for (uint32_t it = blockIdx.x; it < n; it += gridDim.x) {
        const uint32_t g = it / nsplit, s = it % nsplit;
        const uint32_t p0 = s * L, p1 = min(p0 + L, pos + 1);  // includes pos in the last split
        const bool last_split = (p1 == pos + 1);
        // RoPE'd queries of the group (and the fresh k, v in the last split)
        for (uint32_t i = threadIdx.x; i < group * (hd / 2); i += kConsumerWarps * 32) {
            const uint32_t h = i / (hd / 2), p = i % (hd / 2);
            const float *qh = ph.q + (size_t)(g * group + h) * hd;
            float a, b;
            rope_pair(pg, pos, (int)p, __ldcg(qh + p), __ldcg(qh + p + hd / 2), a, b);
            sm.q[h][p] = a;
            sm.q[h][p + hd / 2] = b;
        }
        if (last_split) {
            for (uint32_t p = threadIdx.x; p < hd / 2; p += kConsumerWarps * 32) {
                const float *kh = ph.k + (size_t)g * hd;
                float a, b;
                rope_pair(pg, pos, (int)p, __ldcg(kh + p), __ldcg(kh + p + hd / 2), a, b);
                sm.knew[p] = a;
                sm.knew[p + hd / 2] = b;
            }
            for (uint32_t i = threadIdx.x; i < hd; i += kConsumerWarps * 32) sm.vnew[i] = __ldcg(ph.v + (size_t)g * hd + i);
        }
        consumer_sync();
        if (last_split) {
            // KV append at pos (src/brain_runtime.c:1496-1500); read back next step.
            const size_t off = ((size_t)g * pg.max_context + pos) * hd;
            for (uint32_t i = threadIdx.x; i < hd; i += kConsumerWarps * 32) {
                if (f16) {
                    reinterpret_cast<__half *>(ph.k_cache)[off + i] = __float2half_rn(sm.knew[i]);
                    reinterpret_cast<__half *>(ph.v_cache)[off + i] = __float2half_rn(sm.vnew[i]);
                } else {
                    reinterpret_cast<float *>(ph.k_cache)[off + i] = sm.knew[i];
                    reinterpret_cast<float *>(ph.v_cache)[off + i] = sm.vnew[i];
                }
            }
        }
        // Cached positions come from the staged K and V chunks.
        const uint32_t cached_end = min(p1, pos);
        const bool has_chunks = cached_end > p0;
        const uint8_t *kst = nullptr, *vst = nullptr;
        uint32_t sk = 0, sv = 0;
        if (has_chunks) {
            sk = k % kStages;
            if (!mbar_wait(&sm.full[sk], (k / kStages) & 1u, err)) return false;
            sv = (k + 1) % kStages;
            if (!mbar_wait(&sm.full[sv], ((k + 1) / kStages) & 1u, err)) return false;
            const uint32_t esz = f16 ? 2u : 4u, row = hd * esz;
            const size_t head_off = (size_t)g * pg.max_context * row;
            const uintptr_t ka = reinterpret_cast<uintptr_t>(ph.k_cache) + head_off + (size_t)p0 * row;
            const uintptr_t va = reinterpret_cast<uintptr_t>(ph.v_cache) + head_off + (size_t)p0 * row;
            kst = sm.stage[sk] + (ka & 15u);
            vst = sm.stage[sv] + (va & 15u);
        }
        // One warp per query head of the group; lane owns dims [4*lane, 4*lane+4).
        for (uint32_t h = (uint32_t)warp; h < group; h += kConsumerWarps) {
            float qv[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) qv[e] = sm.q[h][4 * lane + e];
            float m = -FLT_MAX, l = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
            const uint32_t np = p1 - p0;
            for (uint32_t t = 0; t < np; ++t) {
                const uint32_t p = p0 + t;
                float kv4[4], vv4[4];
                if (p == pos) {
#pragma unroll
                    for (int e = 0; e < 4; ++e) { kv4[e] = sm.knew[4 * lane + e]; vv4[e] = sm.vnew[4 * lane + e]; }
                } else {
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        kv4[e] = kv_load(kst, f16, (size_t)t * hd + 4 * lane + e);
                        vv4[e] = kv_load(vst, f16, (size_t)t * hd + 4 * lane + e);
                    }
                }
                float part = qv[0] * kv4[0] + qv[1] * kv4[1] + qv[2] * kv4[2] + qv[3] * kv4[3];
                const float sc = warp_sum(part) * scale;
                const float mn = fmaxf(m, sc);
                const float corr = expf(m - mn), w = expf(sc - mn);
                l = l * corr + w;
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[e] = acc[e] * corr + w * vv4[e];
                m = mn;
            }
            float *dst = ph.part + (((size_t)g * nsplit + s) * group + h) * (hd + 2);
#pragma unroll
            for (int e = 0; e < 4; ++e) dst[4 * lane + e] = acc[e];
            if (lane == 0) { dst[hd] = m; dst[hd + 1] = l; }
        }
        if (has_chunks) {
            __syncwarp();
            if (lane == 0) { mbar_arrive(&sm.empty[sk]); mbar_arrive(&sm.empty[sv]); }
            k += 2;
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
            for (uint32_t i = threadIdx.x; i < group * hd; i += kConsumerWarps * 32) {
                const uint32_t h = i / hd, d = i % hd;
                float M = -FLT_MAX;
                for (uint32_t q = 0; q < nsplit; ++q)
                    M = fmaxf(M, __ldcg(ph.part + (((size_t)g * nsplit + q) * group + h) * (hd + 2) + hd));
                float num = 0.f, den = 0.f;
                for (uint32_t q = 0; q < nsplit; ++q) {
                    const float *src = ph.part + (((size_t)g * nsplit + q) * group + h) * (hd + 2);
                    const float w = expf(__ldcg(src + hd) - M);
                    num += w * __ldcg(src + d);
                    den += w * __ldcg(src + hd + 1);
                }
                ph.att[(size_t)(g * group + h) * hd + d] = den > 0.f ? num / den : 0.f;
            }
        }
        consumer_sync();
    }
    return true;
}

// token_embd row of the current token -> x, bit-exact (load_embedding_row,
// src/brain_runtime.c:1311-1332).
__device__ void run_embed_phase(const Program &pg, const Phase &ph, uint32_t token)
{
    if (blockIdx.x != 0) return;
    const uint32_t be = block_elems(ph.embd_type), bb = block_bytes(ph.embd_type);
    const uint8_t *row = ph.embd + (uint64_t)token * ph.embd_row_bytes;
    for (uint32_t i = threadIdx.x; i < pg.hidden; i += kConsumerWarps * 32)
        ph.x[i] = deq_elem(ph.embd_type, row + (i / be) * bb, (int)(i % be));
}

// Greedy pick over the head items' partials (lowest index among equal maxima).
__device__ void run_argmax_phase(const Program &pg, const Phase &ph, Smem &sm)
{
    if (blockIdx.x != 0) return;
    const Phase &head = pg.phases[ph.layer];  // index of the logits phase
    float best = -FLT_MAX;
    uint32_t bi = 0xffffffffu;
    for (uint32_t i = threadIdx.x; i < ph.argmax_items; i += kConsumerWarps * 32) {
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
        if (mine && p > 0 && !wait_phase(pg, p - 1, epoch, err)) return false;
        if (tr && threadIdx.x == 0) tr[p * 4 + 1] = global_ns();
        if (mine) {
            bool ok = true;
            switch (ph.kind) {
            case PH_GEMV:
                switch (ph.n_slices) {
                case 1: ok = run_gemv_phase<1>(pg, ph, sm, k, err); break;
                case 2: ok = run_gemv_phase<2>(pg, ph, sm, k, err); break;
                case 3: ok = run_gemv_phase<3>(pg, ph, sm, k, err); break;
                default: ok = run_gemv_phase<4>(pg, ph, sm, k, err); break;
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
    const int warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], kConsumerWarps);
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
