// Host/device description of a decode "program" run by the persistent decode
// kernel (decode.cu).
//
// A program is an ordered list of phases. Every CTA (one per SM) walks the
// same list: for each phase it processes the work items i with
// i % gridDim.x == blockIdx.x, then arrives on that phase's counter; before its
// first item of a phase it waits until every CTA has arrived on the previous
// phase's counter. Each item's weight (or KV-cache) bytes are streamed into a
// shared-memory ring with 1-D bulk copies issued ahead of use - across phase
// boundaries too, because weights never depend on activations - so the warps
// wait only for the activations.
#pragma once
#include <cstdint>

namespace atlas {

// 8 consumer warps + 1 producer warp per CTA, one CTA per SM.
constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kMaxStages = 8;
constexpr int kMaxItemRows = 64;     // rows of one segment in one GEMV item (multiple of 16)
constexpr int kMaxSeg = 3;
constexpr int kHeadDim = 128;
constexpr int kAttnChunk = 64;       // cached positions per staged K (or V) chunk
constexpr int kMaxSplits = 64;       // attention splits per KV head
constexpr int kMaxGroup = 8;         // query heads per KV head (one warp each)

enum PhaseKind : uint32_t {
    PH_EMBED = 0,   // x = dequant(token_embd row of the current token)
    PH_GEMV = 1,    // segmented GEMV with a fused prologue / epilogue
    PH_ATTN = 2,    // RoPE + KV append + split-K flash-decode + split combine
    PH_ARGMAX = 3,  // reduce the head items' (max, index) partials -> next token
};

enum InputMode : uint32_t {
    IN_RAW = 0,      // x as stored
    IN_RMSNORM = 1,  // rms_norm(x, norm_w) computed per CTA (src/brain_runtime.c:1338)
};

enum Epilogue : uint32_t {
    EPI_STORE = 0,       // out[r] = dot (+ bias[r])
    EPI_RESID_ADD = 1,   // out[r] += dot      (residual stream)
    EPI_SWIGLU = 2,      // out[r] = silu(dot0) * dot1   (segments 0 = gate, 1 = up)
    EPI_LOGITS = 3,      // out[r] = dot and (max, argmax) per item
};

struct Seg {
    const uint8_t *w;     // row 0 of the raw GGUF tensor
    uint64_t row_bytes;
    uint32_t type;        // 12 = Q4_K, 14 = Q6_K
    uint32_t rows;
    const float *bias;    // optional, EPI_STORE only
    float *out;
};

struct Phase {
    uint32_t kind;
    uint32_t layer;
    // ---- PH_GEMV ----
    // An item is item_rows rows of every segment it touches (paired: the same
    // rows of each segment; otherwise a range of the concatenated row space).
    // Its bytes are staged in chunks of item_rows rows x chunk_blocks block
    // columns: contiguous rows when chunk_blocks covers the row (seg_stride 0),
    // else one copy per row segment, row i at stage + i * seg_stride.
    uint32_t n_items;
    uint32_t item_rows;
    uint32_t paired;
    uint32_t n_seg;
    uint32_t cols;          // input length (multiple of 256)
    uint32_t chunk_rows;    // rows per chunk (16 or 32; divides item_rows)
    uint32_t chunk_blocks;  // block columns per chunk
    uint32_t seg_stride;    // bytes per row segment in a segmented chunk (0: contiguous)
    uint32_t input_mode;
    uint32_t epilogue;
    uint32_t seg_start[kMaxSeg + 1];  // cumulative row offsets (concatenated row space)
    Seg seg[kMaxSeg];
    const float *in;        // input vector (cols floats)
    const float *norm_w;    // IN_RMSNORM weight
    float *partial_max;     // EPI_LOGITS: per-CTA max
    uint32_t *partial_idx;  // EPI_LOGITS: per-CTA argmax
    // ---- PH_ATTN ----
    const float *q, *k, *v; // fresh projections (bias added, RoPE not yet applied)
    void *k_cache, *v_cache;// this layer's cache, [kv_head][position][head_dim]
    float *att;             // output, q_dim floats
    float *part;            // split partials: [kv_head][split][group][head_dim + 4]
    uint32_t *split_ctr;    // per KV head arrival counters (reset by the combiner)
    // ---- PH_EMBED ----
    const uint8_t *embd;    // token_embd raw rows
    uint64_t embd_row_bytes;
    uint32_t embd_type;
    float *x;
    // ---- PH_ARGMAX ----
    uint32_t argmax_items;  // number of CTAs holding head partials
};

// Mutable per-launch state in device memory. The first two fields are owned
// by the device (they only ever grow); the host rewrites the rest before a
// call (from `pos` on).
struct StepState {
    uint32_t epoch;        // launches completed (phase counters are epoch-relative)
    uint32_t exit_ctr;     // CTAs that finished, epoch-relative
    uint32_t pos;          // position of the token being processed
    uint32_t token;        // token id being processed
    uint32_t status;       // first error recorded (kStatus*), 0 = ok
    uint32_t next_token;   // greedy pick of this step
    float next_logit;
    uint32_t step;         // index into out_ids for multi-step generation
    uint32_t max_steps;
    uint32_t pad_;
    uint32_t *out_ids;     // optional device array of picks, or null
};

struct Program {
    const Phase *phases;   // device array
    uint32_t n_phases;
    uint32_t *phase_ctr;   // device array [n_phases], epoch-relative arrival counts (stride 8)
    StepState *state;
    // model constants needed by PH_ATTN / PH_EMBED
    uint32_t q_heads, kv_heads, head_dim, kv_fp16;
    uint32_t hidden;
    float rms_eps;
    const float2 *rope;    // [max_context][head_dim/2] (cos, sin)
    uint32_t max_context;
    uint32_t advance;      // 1: after the step, token = next_token and pos += 1
    uint64_t *trace;       // optional: [cta][phase][4] globaltimer stamps (diagnostics)
    uint64_t *trace_ext;   // optional: [cta][phase][8] stamps inside a phase (diagnostics)
    // shared-memory plan (host-chosen per model)
    uint32_t n_stages;     // bulk-copy ring depth
    uint32_t stage_bytes;  // bytes per stage (multiple of 128)
    uint32_t max_cols;     // largest GEMV input length (x staging area)
};

// Dynamic shared memory: [SmemHdr][x staging: max_cols * 4.25 B][stages]
constexpr uint32_t x_area_bytes(uint32_t max_cols) { return ((max_cols * 4u + max_cols / 4u) + 127u) & ~127u; }

}  // namespace atlas
