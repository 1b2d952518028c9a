// Host/device description of the graph decode step (decode2.cu): one kernel
// per operation of forward_token (src/brain_runtime.c:1698-1772), chained with
// programmatic dependent launch and replayed as one CUDA graph per token.
//
//   embed -> [ mv q,k,v (rms_norm, +bias) -> attention (RoPE, KV append)
//              -> mv o (+residual) -> mv gate,up (rms_norm, SwiGLU)
//              -> mv down (+residual) ] x layers
//   -> mv head (rms_norm, logits, per-CTA max) -> argmax (next token)
//
// The token, its position and the step index live in device memory
// (DecState); the argmax kernel advances them, so consecutive replays
// generate consecutive tokens without the host.
#pragma once
#include <cstdint>

namespace atlas {
namespace d2 {

struct DecState {
    uint32_t pos;          // position of the token being processed
    uint32_t token;        // token being processed; the argmax writes the next one
    uint32_t step;         // index into out_ids
    uint32_t status;       // first error (kStatus*), 0 = ok
    uint32_t next_token;   // greedy pick of the last step
    float next_logit;      // its logit
    uint32_t max_steps;    // capacity of out_ids
    uint32_t advance;      // 1: after the pick, token = pick, pos += 1, step += 1
    uint32_t *out_ids;     // optional device array of picks
    const uint32_t *in_ids;  // prompt mode: the token after step s is in_ids[s + 1] while s + 1 < n_in
    uint32_t n_in;
    uint32_t epoch;        // steps completed since creation (tensor-parallel exchange sequence)
    uint64_t *trace;       // null, or the trace records of the next step (kernels record globaltimer stamps)
};

// Trace record of launch `slot` of the step, CTA c: kTraceWords stamps at
// trace + (slot * kTraceCtas + c) * kTraceWords - [0] the CTA started, [1] its
// inputs were ready (after the wait for the preceding kernel, the input
// staging and any tensor-parallel exchange), [2 + w] warp w finished (w < 16),
// [kTraceWords - 2] the peers' partial rows had all arrived (tensor-parallel
// GEMV launches), [kTraceWords - 1] the wait for the preceding kernel returned
// (GEMV launches).
constexpr uint32_t kTraceCtas = 512, kTraceWords = 20;

// ------------------------------------------------ tensor-parallel exchange --
//
// Every rank owns one exchange area in device memory, mapped into the other
// ranks' processes. Row-split projections (o, down) push their partial rows
// into every rank's area, at the slot of the pushing rank, and count one
// arrival per CTA at every rank; the next kernel's input staging waits for
// all arrivals of that occurrence and sums the slots in rank order, so every
// rank computes the same x. The head pushes its per-CTA (max, row) pairs the
// same way for the argmax. Counters only grow: occurrence k of a stage is
// complete when the counter reaches k * arrivals (mod 2^32).
constexpr uint32_t kTpMax = 8;
constexpr uint32_t kTpPStride = 256;    // per-rank (max, row) slots, >= CTAs of the head launch
constexpr uint32_t kTpCntO = 0, kTpCntDn = 4, kTpCntHead = 8;   // counter byte offsets (decode)
constexpr uint32_t kTpCntReady = 12, kTpCntDone = 16;            // prefill exchange counters

// Decode slots, then the prefill regions: the rank's partial rows of a
// row-split contraction [tmax][hidden] and the residual stream [tmax][hidden]
// (peers write their reduced slices into it).
struct TpLayout {
    uint32_t red_o, red_dn, pmax, pidx;
    uint64_t part, px, bytes;   // byte offsets / total size
};

__host__ __device__ inline TpLayout tp_layout(uint32_t tp, uint32_t hidden, uint32_t tmax = 0)
{
    TpLayout l{};
    l.red_o = 128u;
    l.red_dn = l.red_o + ((tp * hidden * 4u + 127u) & ~127u);
    l.pmax = l.red_dn + ((tp * hidden * 4u + 127u) & ~127u);
    l.pidx = l.pmax + tp * kTpPStride * 4u;
    l.part = (l.pidx + tp * kTpPStride * 4u + 255u) & ~255u;
    l.px = l.part + (((uint64_t)tmax * hidden * 4u + 255u) & ~uint64_t(255));
    l.bytes = l.px + (uint64_t)tmax * hidden * 4u;
    return l;
}

// One all-reduce of a prefill chunk's partial rows (tokens x hidden floats):
// every rank adds all ranks' partials, in rank order, to its residual slice
// and writes the sums into every rank's residual.
struct TpReduceArgs {
    uint8_t *peer[kTpMax];
    uint32_t tp, rank;
    uint64_t part, px;          // region offsets (TpLayout)
    uint32_t n4;                // float4 elements (tokens * hidden / 4)
    uint32_t seq;               // occurrence number of this all-reduce (1, 2, ...)
    uint32_t *status;
};

// ------------------------------------------------------------ mv kernel ----
//
// Work is counted in tasks: one task = 16 rows x one 256-element block column.
// Task j of a segment covers tile t = j / nb (rows 16t..16t+15), block j % nb;
// a paired (SwiGLU) kernel interleaves the gate and up segments per tile:
// t = j / (2 nb), segment (j / nb) & 1. Every CTA owns a contiguous range of
// whole tiles of one segment (or of the pair), so every tile is finished
// inside one CTA, in shared memory.
constexpr int kMvRows = 16;                       // rows per tile (one MMA row tile)
constexpr int kMvWarps = 8;                       // consumer warps; warp w takes tasks j0 + w + 8m
constexpr int kMvThreads = (kMvWarps + 1) * 32;   // + one producer warp
constexpr int kMvMaxSlots = 8;
constexpr int kMvMaxTileSlots = 128;              // open tiles tracked in shared memory, at most
constexpr int kMvMaxPortions = 4;                 // (tile, segment) runs in one slot
constexpr uint32_t kMvMaxSt = 16;                 // tasks per ring slot, at most (16: two per warp)

// MV_PART: partial rows of a row-split projection, pushed to every rank
enum MvEpi : uint32_t { MV_STORE = 0, MV_RESID = 1, MV_SWIGLU = 2, MV_LOGITS = 3, MV_PART = 4 };

// K parts of one launch (segments of one matrix, each over a slice of the columns)
constexpr uint32_t kMvMaxKParts = 3u;

struct MvSeg {
    const uint8_t *w;      // row 0 of the raw GGUF tensor
    uint64_t row_bytes;
    uint32_t type;         // 12 = Q4_K, 14 = Q6_K; mv4_kernel: also 1, 6, 7, 8, 13
    uint32_t rows;         // multiple of kMvRows
    const float *bias;     // optional (MV_STORE)
    float *out;
    uint32_t copies;       // bulk copies per whole-row run of 16 rows: 1, 2, 4 or 8
    uint32_t x_off;        // mv4_kernel: the segment's input starts at x + x_off (a K part of a longer row;
                           // such launches carry no rms_norm, whose factor needs the whole row)
};

struct MvCta {
    uint32_t seg;          // segment (0 when paired)
    uint32_t j0, j1;       // task range (mv_kernel: whole tiles; mv4_kernel: any tasks of the segment)
    uint32_t pad_;
    // mv4_kernel, a range that starts or ends inside a row tile: the first
    // CTA whose range holds part of this CTA's first tile, and the last CTA
    // whose range holds part of its last tile
    uint32_t ca, cb;
    uint32_t pad2_[2];
};

struct MvArgs {
    MvSeg seg[3];
    uint32_t n_seg, paired, nb, cols;
    uint32_t epi;
    uint32_t st;           // tasks per ring slot (1, 2, 4, 8 or 16)
    uint32_t nslot;        // ring depth
    uint32_t slot_bytes;
    uint32_t tslots;       // open-tile slots: > (nslot + 1) * st / tasks per tile + 1
    uint32_t smem_bytes;   // dynamic shared memory of the launch
    const MvCta *cta;      // [gridDim.x]
    const float *x;        // input vector (cols floats)
    const float *norm_w;   // rms_norm weight, or null
    float eps;
    float *pmax;           // MV_LOGITS: per-CTA maximum and its row
    uint32_t *pidx;
    uint32_t *status;
    uint32_t pdl;          // launched as a programmatic dependent
    // tensor parallel (tp > 1)
    uint8_t *peer[kTpMax];   // exchange areas of the ranks, as mapped in this process
    uint32_t tp, rank;
    const DecState *dstate;  // epoch of the current step
    // input staging: x = a.x + sum over ranks of the receive slots at in_red,
    // once in_cnt has seen occurrence epoch * seq_mul + seq_add; the sum is
    // written back to xout (each CTA its share). in_red == 0: no exchange.
    uint32_t in_red, in_cnt, in_arrivals, seq_mul, seq_add;
    float *xout;
    // one GPU: x = a.x + the in_nparts K-part partial rows at in_part (rows
    // [r * cols, (r + 1) * cols) for part r, added in part order), written back
    // to xout (each CTA its share); the preceding launch (PDL) wrote them
    const float *in_part;
    uint32_t in_nparts;
    // mv4_kernel, row tiles shared by CTAs: partial rows [cta][first / last
    // tile][32] and arrival counters [first CTA of the tile], zero between launches
    float *xpart;
    uint32_t *xcnt;
    uint32_t x_lo, x_hi;     // x_hi > 0: staged elements outside [x_lo, x_hi) are zero
    // MV_PART / MV_LOGITS pushes: receive offset and counter at every rank
    uint32_t out_red, out_cnt;
    uint32_t row_base;       // MV_LOGITS: global index of row 0
    uint32_t engine;         // 0: mv_kernel (producer warp + shared ring); 1: mv4_kernel (per-warp rings)
    uint32_t trace_slot;     // this launch's index in the step (trace records)
    uint32_t warps;          // mv4_kernel: 8 (two CTAs per SM) or 16 warps per CTA
    uint32_t gen_type;       // mv4_kernel: 0 (Q4_K / Q6_K segments), or the other block type of every segment
};

// ------------------------------------------------------------ mv4 kernel ----
//
// The same launches (MvArgs, task ranges, epilogues) on a kernel without a
// producer warp: 8 or 16 warps, each with a contiguous range of the CTA's tasks
// and its own ring of nslot task slots filled by cp.async (16-byte copies
// issued by its own lanes). A slot holds the 16 rows of one task: Q4_K rows
// 144 bytes apart (the block itself), Q6_K rows as 224-byte windows from the
// 16-byte boundary at or below the block (the 2-byte-aligned 210-byte block
// lies inside at any offset), kM4Q6Row apart (rows in distinct banks).
constexpr int kM4Warps = 16;
constexpr int kM4Threads = kM4Warps * 32;
constexpr uint32_t kM4Q4Row = 144u, kM4Q6Row = 240u;
constexpr uint32_t kM4MaxSlots = 6u;
// bytes past the end of a Q6_K tensor that a 224-byte window may read (14), rounded up
constexpr uint32_t kM4Q6Overread = 48u;

// The reference's other block types (F16 = 1, Q5_0 = 6, Q5_1 = 7, Q8_0 = 8,
// Q5_K = 13) run on the same kernel: a task copies the row's whole chunk of
// 256 elements - 512, 176, 192, 272, 176 bytes, multiples of 16 - rows
// m4_gen_row bytes apart (an odd multiple of 16), with 16 bytes of slack
// after the last row for the 20-byte reads of 2-byte-aligned fields.
__host__ __device__ constexpr uint32_t m4_chunk_bytes(uint32_t type)
{
    return type == 12u ? 144u : type == 14u ? 210u : type == 6u ? 176u : type == 7u ? 192u : type == 8u ? 272u :
           type == 13u ? 176u : type == 1u ? 512u : 0u;
}
__host__ __device__ constexpr bool m4_other_type(uint32_t type)
{
    return type == 1u || type == 6u || type == 7u || type == 8u || type == 13u;
}
__host__ __device__ constexpr uint32_t m4_gen_row(uint32_t type)
{
    return (m4_chunk_bytes(type) / 16u) & 1u ? m4_chunk_bytes(type) : m4_chunk_bytes(type) + 16u;
}
__host__ __device__ constexpr uint32_t m4_slot_bytes(uint32_t type)
{
    return type == 12u ? 16u * kM4Q4Row : type == 14u ? 16u * kM4Q6Row : 16u * m4_gen_row(type) + 16u;
}
// ring depths of the kernels of the other types (16 warps: 2..4, 8 warps: 2..3)
constexpr uint32_t kM4GenSlots16 = 4u, kM4GenSlots8 = 3u;

// ------------------------------------------------------ attention kernel ----

constexpr uint32_t kAttnThreads = 256;
constexpr uint32_t kAttnTile = 32;      // cached positions staged per tile (two tiles in flight)
constexpr uint32_t kAttnMinSpan = 16;   // positions per split, at least
constexpr uint32_t kAttnCluster = 8;    // consecutive splits of a KV head merged in one thread-block cluster
constexpr uint32_t kAttnMaxGroup = 8;   // query heads per KV head (one warp each)
constexpr uint32_t kRec = 132;          // partial record: acc[128], max, sum, 2 pad

struct AttnArgs {
    const float *q, *k, *v;     // projections of the current token (+bias, no RoPE)
    void *k_cache, *v_cache;    // this layer's [kv_heads][max_context][128]
    float *att;                 // [q_heads][128]
    float *part;                // cluster records [kv_heads][splits / kAttnCluster][group][kRec]
    uint32_t *ctr;              // per query head, zero between launches
    const float2 *rope;         // (cos, sin) [position][64]
    DecState *st;
    uint32_t q_heads, kv_heads, max_context, splits, kv_fp16;
    uint32_t min_span;          // cached positions per split, at least (0: kAttnMinSpan)
    const float *q_norm, *k_norm;   // qwen3: per-head RMSNorm weights [128] of q and k, or null
    float eps;
    uint32_t tc;                // fp16 cache: tensor-core kernel (attn_tc16_kernel)
    uint32_t trace_slot;        // this launch's index in the step (trace records)
    // batched step (attn_kernel_b: blockIdx.y = sequence s): q, k, v at + s *
    // qkv_stride, the caches at + s * cache_seq_bytes, att at + s * att_stride,
    // part at + s * part_seq, ctr at + s * ctr_seq, st at + s
    uint32_t qkv_stride, att_stride, part_seq, ctr_seq;
    uint64_t cache_seq_bytes;
};

}  // namespace d2
}  // namespace atlas
