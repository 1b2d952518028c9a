/*
 * libatlas_cuda: B200 (sm_100a) inference library for Qwen2-family models with
 * raw GGUF Q4_K / Q6_K weights. Plain C ABI: pointers and sizes only.
 *
 * This is the wider device boundary under the reference's model/forward API
 * (src/brain_runtime.c:1698 forward_token; src/brain_runtime_batch.c:1644
 * forward_prefill_batch). The reference's own narrow device plugin
 * (src/gpu_matvec.h:13-17) is provided unchanged in include/gpu_matvec.h.
 *
 * Conventions
 *  - Every int-returning function returns ATLAS_OK (0) on success and a
 *    negative ATLAS_E* code on failure; atlas_cuda_last_error() gives the text.
 *    Nothing exits the process, nothing traps, and there is no CPU fallback:
 *    without a usable sm_100 device every call fails with ATLAS_ENODEV.
 *  - A handle is used by one host thread at a time. Host buffers passed in are
 *    only read during the call; output buffers are written before return.
 *  - Weight bytes are uploaded unchanged (144-byte Q4_K and 210-byte Q6_K
 *    super-blocks, rows in file order).
 */
#ifndef ATLAS_CUDA_H
#define ATLAS_CUDA_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    ATLAS_OK = 0,
    ATLAS_EINVAL = -1,   /* bad argument or unsupported shape / tensor type */
    ATLAS_ENODEV = -2,   /* no sm_100 CUDA device */
    ATLAS_ENOMEM = -3,   /* device or host allocation failed */
    ATLAS_ECUDA = -4,    /* a CUDA runtime call failed */
    ATLAS_ETIMEOUT = -5, /* a bounded device-side wait ran out (status read back, context intact) */
    ATLAS_ENCCL = -6,    /* a tensor-parallel exchange failed (a peer never arrived) */
    ATLAS_ERANGE = -7    /* position / token / size beyond what the handle was created for */
};

/* ggml tensor type ids as used by the reference (src/brain_runtime.c:79-86). */
enum {
    ATLAS_TYPE_F32 = 0,
    ATLAS_TYPE_F16 = 1,
    ATLAS_TYPE_Q5_0 = 6,
    ATLAS_TYPE_Q5_1 = 7,
    ATLAS_TYPE_Q8_0 = 8,
    ATLAS_TYPE_Q4_K = 12,
    ATLAS_TYPE_Q5_K = 13,
    ATLAS_TYPE_Q6_K = 14
};

typedef struct AtlasCuda AtlasCuda;

/* One GGUF tensor as the host loader found it (TensorInfo, src/brain_runtime.c:138-144).
   dims[0] is the inner (column) extent, dims[1] the rows. `data` points at the
   tensor's bytes in host memory (for example into an mmap of the file). */
typedef struct {
    const char *name;
    uint32_t type;
    uint32_t n_dims;
    uint64_t dims[4];
    const void *data;
} AtlasTensorDesc;

/* Model shape (ModelShape, src/brain_runtime.c:93-99) plus placement. */
typedef struct {
    uint32_t hidden, q_dim, kv_dim, q_heads, kv_heads, head_dim, ffn, layers, vocab;
    uint32_t max_context;  /* KV-cache positions to allocate (no 8192 cap) */
    uint32_t max_prefill;  /* largest prefill call, in tokens (0: 512) */
    float rope_base;       /* rope.freq_base, default 1e6 */
    float rms_eps;         /* 1e-6 in the reference (src/brain_runtime.c:115) */
    int32_t has_qk_norm;   /* qwen3 per-head q/k RMSNorm (src/brain_runtime.c:1727-1737) */
    int32_t kv_fp16;       /* 0: fp32 KV cache (default), 1: fp16 KV cache (see below) */
    int32_t device;        /* CUDA device ordinal */
    int32_t tp_rank;       /* tensor-parallel rank, 0..tp_size-1 (one process per GPU) */
    int32_t tp_size;       /* 1, or 2 / 4 / 8 when kv_heads % tp_size == 0 (see atlas_cuda_tp_*) */
    uint32_t max_batch;    /* sequences with a KV cache of their own (0 or 1: one); see atlas_cuda_generate_batch */
} AtlasModelDesc;

/* KV-cache precision: the reference keeps K and V in fp32 (src/brain_runtime.c:2019-2020).
   fp16 halves the cache traffic, but on models whose attention logits are large
   (the synthetic random-weight models reach |score| ~ 100s) its 2^-11 rounding of
   K moves scores by ~0.1 and can change a peaked softmax, so fp32 is the default.

   Uploads the tensors named by the reference's forward_token and builds the
   decode program. Tied models may omit output.weight (token_embd is used). */
int atlas_cuda_create(const AtlasModelDesc *desc, const AtlasTensorDesc *tensors,
                      uint32_t n_tensors, AtlasCuda **out);
void atlas_cuda_destroy(AtlasCuda *h);
const char *atlas_cuda_last_error(const AtlasCuda *h);

/* Batched prefill of ids[0..n) at positions pos0..pos0+n-1 (as consecutive
   forward_token calls would, src/brain_runtime.c:2025-2028). Optionally returns
   the last token's logits (vocab floats, host) and its greedy pick. */
int atlas_cuda_prefill(AtlasCuda *h, const uint32_t *ids, uint32_t n, uint32_t pos0,
                       float *last_logits, uint32_t *argmax);

/* One decode step: forward_token(id, pos) then the greedy pick of
   atlas_sample_token (src/brain_runtime.c:1783, greedy branch). logits may be NULL. */
int atlas_cuda_decode(AtlasCuda *h, uint32_t id, uint32_t pos, float *logits, uint32_t *argmax);

/* Greedy generation loop kept on the device: starting from token `first` at
   position pos0, runs `steps` forward passes; out_ids[i] is the greedy pick after
   step i (the reference's decode loop, src/brain_runtime.c:2036-2048, without
   the stop-token test). */
int atlas_cuda_generate(AtlasCuda *h, uint32_t first, uint32_t pos0, uint32_t steps,
                        uint32_t *out_ids);

/* Per-phase device time of the last decode/generate call and kernel launch
   counts since creation (diagnostics for the benchmark). */
/* Several independent sequences (no counterpart in the reference, which runs one
   sequence per process, src/brain_runtime.c:1698 and :2036-2048; the per-sequence
   arithmetic is forward_token's). Sequence s (s < desc.max_batch) has its own KV
   cache; sequence 0's is the one atlas_cuda_prefill / decode / generate use.
   Q4_K / Q6_K files, one GPU.
   atlas_cuda_prefill_seq: atlas_cuda_prefill into sequence seq's cache.
   atlas_cuda_generate_batch: `steps` greedy steps of nseq <= 8 sequences at once,
     sequence s starting from token first[s] at position pos0[s]; out_ids[s * steps + i]
     is the pick after step i (every weight is read once per step for all sequences).
   atlas_cuda_decode_batch: one step: token ids[s] at position pos[s] for each
     sequence; logits [nseq][vocab] (or NULL) and the greedy picks argmax[nseq]. */
int atlas_cuda_prefill_seq(AtlasCuda *h, uint32_t seq, const uint32_t *ids, uint32_t n, uint32_t pos0,
                           float *last_logits, uint32_t *argmax);
int atlas_cuda_generate_batch(AtlasCuda *h, uint32_t nseq, const uint32_t *first, const uint32_t *pos0,
                              uint32_t steps, uint32_t *out_ids);
int atlas_cuda_decode_batch(AtlasCuda *h, uint32_t nseq, const uint32_t *ids, const uint32_t *pos, float *logits,
                            uint32_t *argmax);

int atlas_cuda_stats(const AtlasCuda *h, uint64_t *kernel_launches, double *last_ms);

/* Device time (CUDA events on the handle's stream) summed over every decode /
   generate / prefill call since creation. */
int atlas_cuda_device_ms(const AtlasCuda *h, double *total_ms);

/* Diagnostics: runs one decode step of (id, pos) with device-side timestamps
   (globaltimer, ns). out_ns (host, cap uint64 slots) receives n_ctas * n_phases
   * 4 values [wait start, wait end, phase end, producer done] per CTA and phase,
   followed by n_ctas * n_phases * 8 stamps taken inside the phases (0 = none).
   n_ctas / n_phases / phase_kinds (kind * 16 + epilogue) describe the layout. */
int atlas_cuda_trace_step(AtlasCuda *h, uint32_t id, uint32_t pos, uint64_t *out_ns, size_t cap,
                          uint32_t *n_ctas, uint32_t *n_phases, uint32_t *phase_kinds);

/* One decode step of the graph engine (forward_token + greedy pick at `pos`)
   with device timestamps: every mv / attention launch records, per CTA, the
   globaltimer (ns) when it started, when its inputs were ready (after the
   wait for the preceding kernel, the input staging and, under tensor
   parallelism, the wait for the peers' partial rows), and when each warp
   finished. out receives n_launches x n_ctas x n_words stamps (0 = not
   recorded; launch 0 is the embedding, then 5 per layer - q/k/v, attention,
   o, gate/up, down - then the head and the argmax). With out == NULL only
   the three sizes are returned. Diagnostics; no counterpart in the
   reference. */
int atlas_cuda_trace_graph(AtlasCuda *h, uint32_t id, uint32_t pos, uint64_t *out, size_t cap,
                           uint32_t *n_launches, uint32_t *n_ctas, uint32_t *n_words);

/* ---- tensor parallelism (one process per GPU, tp_size ranks) ----

   The layout of the reference's forward_token across ranks: query heads with
   their KV heads (and the KV cache) split by KV head; attn_q/k/v, ffn_gate/up
   and the output head split by rows; attn_output and ffn_down split by their
   256-column blocks, each rank summing its partial rows; every partial sum
   is exchanged over peer memory (NVLink) inside the decode kernels and added
   in rank order, so all ranks hold the same residual stream and pick the
   same token. Create the handle with desc.tp_rank / tp_size, export its
   exchange area with atlas_cuda_tp_handle, give every rank all ranks'
   handles (rank order) through atlas_cuda_tp_connect, then call
   prefill / decode / generate on every rank with the same arguments.
   Logits outputs receive only the rank's vocab slice (vocab_row0 ..
   vocab_row0 + vocab_rows - 1; other entries are left untouched). Prompts
   run batched on every rank's shards (the partial rows of attn_output and
   ffn_down all-reduced over peer memory), their last token through the
   decode step. A failed step (ATLAS_ENCCL /
   ATLAS_ETIMEOUT) leaves the ranks out of step: destroy and recreate all.
   Destroy the handles only after every rank finished its last call. */

typedef struct {
    uint32_t q_head0, q_heads;        /* query heads of the rank */
    uint32_t kv_head0, kv_heads;      /* KV heads (and their cache) */
    uint32_t o_block0, o_blocks;      /* 256-column blocks of attn_output.weight the rank reads */
    uint32_t o_lo, o_hi;              /* the rank's attention-output elements inside those blocks */
    uint32_t ffn_row0, ffn_rows;      /* ffn_gate / ffn_up rows, = ffn_down columns (256-multiples) */
    uint32_t vocab_row0, vocab_rows;  /* output.weight rows: the rank's logits */
} AtlasTpSlice;

#define ATLAS_TP_HANDLE_BYTES 64

/* The slice of rank `rank` of `size` for a model shape (no device needed). */
int atlas_cuda_tp_slice(const AtlasModelDesc *desc, int rank, int size, AtlasTpSlice *out);
/* The handle's exchange area as ATLAS_TP_HANDLE_BYTES bytes to give the other ranks. */
int atlas_cuda_tp_handle(AtlasCuda *h, void *out);
/* handles: tp_size * ATLAS_TP_HANDLE_BYTES bytes in rank order (this rank's own
   entry included). Maps the peers' exchange areas and builds the decode step. */
int atlas_cuda_tp_connect(AtlasCuda *h, const void *handles);

/* ---- stateless kernels over caller-owned DEVICE memory (parity tests) ---- */

/* Bit-exact dequantization of nblocks super-blocks (the reference's
   dequant_q4_k / dequant_q6_k, src/brain_runtime.c:960 / :1049).
   stream is a cudaStream_t or NULL for the default stream. */
int atlas_cuda_dequant(uint32_t type, const void *d_blocks, uint64_t nblocks, float *d_out,
                       void *stream);

/* y[rows] = W[rows x cols] x[cols] for a Q4_K / Q6_K tensor in device memory
   (matvec_rows, src/brain_runtime.c:1133) on the streaming GEMV kernel: fp32
   FMAs over the exactly dequantized quants, one launch, no scratch memory.
   d_weights: 16-byte aligned for Q4_K, 2-byte for Q6_K; cols a multiple of 256,
   at most 49152; d_x 16-byte aligned, d_y 4-byte aligned. */
int atlas_cuda_gemv(uint32_t type, const void *d_weights, uint64_t rows, uint64_t cols,
                    const float *d_x, float *d_y, void *stream);

/* A GEMV for callers that cannot allocate device memory: a host that owns all
   of HBM and hands plugins no allocator, or a path that cannot absorb
   cudaMalloc's device synchronisation. No counterpart in the reference.
   Same arguments and result as atlas_cuda_gemv (y = W x, within 1e-4 max|y|
   of the oracle), computed by the persistent decode kernel, which needs
   launch scratch (kernel descriptor, phase counters, step state). That
   scratch is a 4 KB static device array in this library, held by every GPU
   that loads it until the process exits; the call makes no cudaMalloc or
   cudaFree. Its first call on a device looks up the array's device address
   (cudaGetSymbolAddress) and keeps it, so that first call should come before
   any stream capture, and the kept address does not survive cudaDeviceReset.
   All calls share the one array: calls that overlap on the GPU (other streams,
   other host threads) race and give wrong results. The call waits for the
   stream and reads the kernel's status word back: it returns ATLAS_ETIMEOUT
   if a bounded device wait ran out, and y is complete when it returns
   ATLAS_OK. Input lengths beyond what the kernel stages in shared memory
   (about 49,000 columns on B200) are rejected with ATLAS_EINVAL. */
int atlas_cuda_gemv_noalloc(uint32_t type, const void *d_weights, uint64_t rows, uint64_t cols,
                            const float *d_x, float *d_y, void *stream);

/* Y[tokens x rows] = X[tokens x cols] W^T (all fp32, row-major, device
   pointers) through the prefill contraction kernel (batch_matvec_rows,
   src/brain_runtime_batch.c:1525): 2-SM tcgen05 MMA over binary16 hi/lo
   splits of X and of the dequantized weights (three products, fp32
   accumulation: fp32-level accuracy). type: ATLAS_TYPE_Q4_K (16-byte aligned
   weights) or ATLAS_TYPE_Q6_K (2-byte aligned); cols a multiple of 256 and at
   most 57344. Scratch is allocated per call and the call synchronizes
   `stream`. ATLAS_EINVAL for bad arguments, ATLAS_ETIMEOUT if a bounded
   device wait gave up. */
int atlas_cuda_gemm(uint32_t type, const void *d_weights, uint64_t rows, uint64_t cols,
                    const float *d_x, uint64_t tokens, float *d_y, void *stream);

/* Number of SMs / compute capability of `device`, or a negative code. */
int atlas_cuda_device_info(int device, int *sm_count, int *cc_major, int *cc_minor);

#ifdef __cplusplus
}
#endif
#endif
