// Host/device description of the streaming GEMV kernel (gemv.cu): one kernel
// per matrix-vector product of the decode step, fp32 FMAs on CUDA cores.
//
// y[r] = sum_k w[r][k] * x[k] over the raw Q4_K / Q6_K rows of up to three
// concatenated tensors (Q/K/V, gate/up), with the input optionally
// rms_norm'ed (src/brain_runtime.c:1338-1371) and a fused epilogue. Each CTA
// owns a block of rows; each warp takes 4 rows at a time and each lane a set
// of 64-value slices of those rows, so one x slice in registers serves 4
// rows; per-slice partial dots are reduced across the warp.
#pragma once
#include <cstdint>

namespace atlas {
namespace gv {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kRowsPerPass = 4;        // rows a warp works on together
constexpr int kMaxSeg = 3;

enum GemvEpilogue : uint32_t {
    GV_STORE = 0,    // out[r] = y (+ bias[r])
    GV_RESID = 1,    // out[r] += y
    GV_SWIGLU = 2,   // out[r] = silu(y_gate) * y_up; rows interleaved gate/up per pass
    GV_LOGITS = 3,   // out[r] = y, and one (max, argmax) per CTA
};

struct GemvSeg {
    const uint8_t *w;      // row 0 of the raw GGUF tensor
    uint64_t row_bytes;
    uint32_t type;         // 12 = Q4_K, 14 = Q6_K
    uint32_t rows;
    const float *bias;     // optional (GV_STORE)
    float *out;
};

struct GemvArgs {
    GemvSeg seg[kMaxSeg];
    uint32_t n_seg;
    uint32_t seg_start[kMaxSeg + 1];   // cumulative rows (paired: seg 0 and 1 share rows)
    uint32_t cols;                     // K (multiple of 256)
    uint32_t rows_per_cta;             // multiple of kRowsPerPass * kWarps / (paired ? 2 : 1)
    uint32_t total_rows;               // output rows (paired: the gate rows)
    const float *x;
    const float *norm_w;               // rms_norm weights, or null for the raw input
    float eps;
    uint32_t epi;
    float *pmax;                       // GV_LOGITS: per-CTA maximum and its row
    uint32_t *pidx;
    uint32_t pdl;                      // wait for the preceding kernel (programmatic launch)
};

}  // namespace gv
}  // namespace atlas
