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

enum MvEpi : uint32_t { MV_STORE = 0, MV_RESID = 1, MV_SWIGLU = 2, MV_LOGITS = 3 };

struct MvSeg {
    const uint8_t *w;      // row 0 of the raw GGUF tensor
    uint64_t row_bytes;
    uint32_t type;         // 12 = Q4_K, 14 = Q6_K
    uint32_t rows;         // multiple of kMvRows
    const float *bias;     // optional (MV_STORE)
    float *out;
    uint32_t copies;       // bulk copies per whole-row run of 16 rows: 1, 2, 4 or 8
    uint32_t pad_;
};

struct MvCta {
    uint32_t seg;          // segment (0 when paired)
    uint32_t j0, j1;       // task range (whole tiles)
    uint32_t pad_;
};

struct MvArgs {
    MvSeg seg[3];
    uint32_t n_seg, paired, nb, cols;
    uint32_t epi;
    uint32_t st;           // tasks per ring slot (1, 2, 4 or 8)
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
};

// ------------------------------------------------------ attention kernel ----

constexpr uint32_t kAttnThreads = 256;
constexpr uint32_t kAttnTile = 64;      // cached positions staged per tile
constexpr uint32_t kAttnMinSpan = 16;   // positions per split, at least
constexpr uint32_t kAttnMaxGroup = 8;   // query heads per KV head (one warp each)
constexpr uint32_t kRec = 132;          // partial record: acc[128], max, sum, 2 pad

struct AttnArgs {
    const float *q, *k, *v;     // projections of the current token (+bias, no RoPE)
    void *k_cache, *v_cache;    // this layer's [kv_heads][max_context][128]
    float *att;                 // [q_heads][128]
    float *part;                // [kv_heads][splits][group][kRec]
    uint32_t *ctr;              // per KV head, zero between launches
    const float2 *rope;         // (cos, sin) [position][64]
    DecState *st;
    uint32_t q_heads, kv_heads, max_context, splits, kv_fp16;
};

}  // namespace d2
}  // namespace atlas
