// Host/device description of the batched-prefill kernels (prefill.cu).
//
// Prefill runs the decoder over T prompt tokens at once
// (forward_prefill_batch, src/brain_runtime_batch.c:1644-1718): every linear
// layer becomes a dense contraction Y[T][rows] = X[T][cols] . W[rows][cols]^T
// on the 5th-generation tensor cores (tcgen05.mma, fp32 accumulators in
// tensor memory), with the Q4_K / Q6_K weights dequantized tile by tile into
// shared memory.
//
// Numerics. The reference multiplies fp32 activations by fp32 dequantized
// weights. Both operands are split into binary16 pairs, v = hi + lo with
// hi = fp16(v) and lo = fp16(v - hi), after exact power-of-two scaling into the
// binary16 range (activations per token, weights per tensor); the contraction
// sums hi.hi + lo.hi + hi.lo in fp32. Each product then carries ~22
// significant bits, the level of fp32 rounding, which these models need: their
// attention logits are large enough that a binary16-rounded key or query
// already moves the softmax (a single-term bf16/fp16 product would not meet
// the logit tolerance). `terms` selects 1, 2 or 3 products for measurements.
#pragma once
#include <cstdint>

namespace atlas {
namespace pf {

constexpr int kTokTile = 128;          // tokens per CTA (TMEM lanes)
constexpr int kPairTokens = 256;       // MMA M over the CTA pair
constexpr int kRowTile = 256;          // MMA N: weight rows per tile (TMEM columns); 128 per CTA
constexpr int kKBlock = 64;            // K elements per stage: one 128-byte swizzle row
constexpr int kStages = 3;
constexpr uint32_t kATermBytes = kTokTile * 128;        // one operand term of a CTA's tokens (16 KB)
constexpr uint32_t kBTermBytes = (kRowTile / 2) * 128;  // one operand term of a CTA's weight rows (16 KB)
constexpr uint32_t kStageBytes = 2 * kATermBytes + 2 * kBTermBytes;
constexpr int kWarps = 22;             // 0 copy, 1 MMA, 2-5 epilogue, 6-21 dequant
constexpr int kDequantWarps = kWarps - 6;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxSeg = 3;
constexpr uint32_t kXTileBytes = 2 * kATermBytes;  // hi + lo of one (token tile, K block)
constexpr uint32_t kSplitMaxCols = 57344;          // longest input row the split pass stages

enum GemmEpilogue : uint32_t {
    GEPI_STORE = 0,   // out = acc + bias (optionally RoPE'd)
    GEPI_RESID = 1,   // out += acc          (residual stream)
    GEPI_SWIGLU = 2,  // out = silu(gate) * up; tile = 128 gate rows + the same 128 up rows
};

// One weight tensor of a (possibly concatenated) contraction. Output element
// (token t, row r) is written at
//   out + (r / 128) * head_stride + (t + tok_off) * tok_stride + r % 128
// which covers plain row-major outputs (head_stride 128, tok_stride = ld) and
// the head-major KV cache (head_stride = max_context * 128, tok_stride 128).
struct GemmSeg {
    const uint8_t *w;      // row 0 of the raw GGUF tensor
    uint64_t row_bytes;
    uint32_t type;         // 12 = Q4_K, 14 = Q6_K
    uint32_t rows;
    int32_t wexp;          // weights are scaled by 2^wexp before the split
    uint32_t rope;         // apply RoPE to each 128-row head (position pos0 + t)
    const float *bias;     // per row, optional
    float *out;
    uint64_t head_stride;
    uint64_t tok_stride;
    uint32_t tok_off;
    uint32_t tile0;        // first row tile of this segment
    uint32_t vec4;         // out, head_stride and tok_stride keep 16-float groups 16-byte aligned
    uint32_t f16;          // out holds binary16 (an fp16 KV cache); offsets count elements
};

struct GemmArgs {
    GemmSeg seg[kMaxSeg];
    uint32_t n_seg;
    uint32_t epi;
    uint32_t n_tiles;      // row tiles over all segments (paired: tiles of 128 + 128 rows)
    uint32_t tok_pairs;    // 256-token tiles (one per CTA pair)
    uint32_t ksplit;       // K ranges per tile (split-K; a reduction kernel sums them)
    uint32_t kblocks;      // cols / 64
    uint32_t tokens;
    uint32_t pos0;         // position of token 0 (RoPE)
    uint32_t terms;        // 1: hi.hi, 2: + lo.hi, 3: + hi.lo
    const uint8_t *xt;     // activation tiles written by the split kernel
    const float *xscale;   // per token 2^-sx
    const float *rope;     // (cos, sin) table [position][64]
    float *ws;             // split-K partials [tile][K range][128 tokens][256 rows]
    uint32_t *status;
};

// Causal GQA attention over the KV cache for a block of prompt tokens.
struct AttnArgs {
    const float *q;        // [T][q_dim], RoPE applied
    const float *k_cache;  // [kv_heads][max_context][128]
    const float *v_cache;
    float *out;            // [T][q_dim]
    float *part;           // per (unit) partial records
    uint32_t *ctr;         // per (kv head, query tile) arrival counters
    uint32_t *status;
    uint32_t tokens, pos0, q_heads, kv_heads, max_context;
    uint32_t q_tiles;      // ceil(T / q_tokens)
    uint32_t span;         // cached positions per unit (multiple of 64)
    uint32_t n_units;
    const uint32_t *unit_tab;   // per unit: g | query tile << 8 | span index << 20;
                                // the spans of one (g, tile) are consecutive
    uint32_t out_stride;        // floats between tokens of out (0: q_heads * 128)
    uint32_t kv_f16;            // the KV cache holds binary16
    uint32_t q_tokens;          // query tokens per unit (128 / group: 128 query rows)
};

}  // namespace pf
}  // namespace atlas
