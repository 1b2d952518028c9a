// Batched decode step (batch.cu): one token for each of up to 8 independent
// sequences per step, every weight read once per step. forward_token
// (src/brain_runtime.c:1698-1772) runs once per sequence in the reference
// (one sequence per process); here the 8 sequences are the 8 columns of the
// same tensor-core tiles.
//
//   embed (all sequences, rms factor) -> [ mvb q,k,v -> reduce (bias) ->
//   attention (per sequence) -> mvb o -> residual (+rms factor) -> mvb gate,up
//   -> reduce (SwiGLU) -> mvb down -> residual (+rms factor) ] x layers ->
//   mvb head -> reduce (logits, per-CTA maxima) -> argmax (per sequence)
//
// mvb (the batched dequant-GEMV) splits K: a CTA stages the 8 inputs of one
// K slice (at most kSplitMax 256-element blocks) in shared memory and writes
// the slice's partial rows; the reduce and residual kernels add the slices
// in slice order (a fixed order: results do not depend on timing).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include "decode2.h"

namespace atlas {
namespace bt {

constexpr uint32_t kMaxSeq = 8;       // sequences per step (the MMA's 8 columns)
constexpr uint32_t kSplitMax = 8;     // 256-element blocks of x staged per CTA
constexpr uint32_t kBWarps = 16;
constexpr uint32_t kBThreads = kBWarps * 32;
constexpr uint32_t kBMaxSlots = 4;

struct BSeg {
    const uint8_t *w;      // row 0 of the raw GGUF tensor (Q4_K or Q6_K)
    uint64_t row_bytes;
    uint32_t type, rows;   // rows: multiple of 16
    uint32_t prow0;        // first row of the segment among the launch's partial rows
    uint32_t pad_;
};

// A CTA: tiles [t0, t1) of segment seg, K slice `split`.
struct BCta {
    uint32_t seg, t0, t1, split;
};

struct BArgs {
    BSeg seg[3];
    uint32_t n_seg, nb, cols, nseq;
    uint32_t nsplit, split_blocks;   // K slices, 256-element blocks per slice (the last may be shorter)
    uint32_t prows;                  // partial rows of the launch (all segments)
    uint32_t nslot, slot_bytes, smem_bytes;
    const BCta *cta;                 // [gridDim.x]
    const float *x;                  // input of sequence s at x + s * xstride
    uint32_t xstride;
    const float *norm_w;             // rms_norm weight, or null (the 1/rms factor is the consumer's)
    float *part;                     // partial rows [nsplit][nseq][prows]
    uint32_t pdl;
    uint32_t *status;
};

// Partial rows -> outputs (one launch, every sequence).
enum BRedMode : uint32_t {
    BRED_STORE = 0,    // out = inv * sum + bias
    BRED_SWIGLU = 1,   // out[r] = silu(inv * sum[r]) * (inv * sum[rows + r]), r < rows
    BRED_LOGITS = 2,   // out = inv * sum, and per-CTA per-sequence (max, row)
};

// Grid (row chunks of 256, nseq). The rms factor of sequence s is
// 1 / sqrt(sum(ssq[s][0..nssq)) / hidden + eps) (src/brain_runtime.c:1345-1360,
// the sum of squares in double), or 1 without ssq.
struct BReduce {
    const float *part;
    uint32_t nsplit, nseq, prows;
    uint32_t mode, rows;
    const float *bias;     // [rows] or null
    const double *ssq;     // [nseq][nssq] partial sums of squares of the normed input, or null
    uint32_t nssq, hidden;
    float eps;
    float *out;            // out[s * ostride + r]
    uint32_t ostride;
    float *pmax;           // BRED_LOGITS: [nseq][gridDim.x]
    uint32_t *pidx;
    uint32_t pdl;
};

// Grid (row chunks of 256, nseq): x[s] += the sum of the partial rows, and
// chunk c's sum of squares of the new x[s] into ssq[s * gridDim.x + c].
struct BResid {
    const float *part;
    uint32_t nsplit, nseq, prows;
    float *x;
    uint32_t hidden;
    double *ssq;
    uint32_t pdl;
};
constexpr uint32_t kRowChunk = 256;

// Dynamic shared memory of an mvb CTA.
size_t mvb_smem(uint32_t split_blocks, uint32_t nslot, uint32_t slot_bytes);

}  // namespace bt
}  // namespace atlas

extern "C" {
cudaError_t atlas_bt_setup(size_t smem);
cudaError_t atlas_bt_launch_mv(const atlas::bt::BArgs *a, uint32_t grid, cudaStream_t stream);
cudaError_t atlas_bt_launch_reduce(const atlas::bt::BReduce *a, uint32_t grid, cudaStream_t stream);
cudaError_t atlas_bt_launch_resid(const atlas::bt::BResid *a, cudaStream_t stream);
cudaError_t atlas_bt_launch_embed(const uint8_t *embd, uint64_t row_bytes, uint32_t type, uint32_t hidden,
                                  uint32_t vocab, float *x, double *ssq, atlas::d2::DecState *st, uint32_t nseq,
                                  cudaStream_t stream);
cudaError_t atlas_bt_launch_argmax(const float *pmax, const uint32_t *pidx, uint32_t n, atlas::d2::DecState *st,
                                   uint32_t nseq, cudaStream_t stream);
}
