// libatlas_cuda C ABI: model upload, decode-program construction, decode /
// generate / prefill entry points and the stateless test kernels.
//
// Device memory layout of a model (one arena per tensor class, 256-byte
// aligned tensors): raw GGUF weight bytes exactly as in the file; norm weights
// and biases as fp32 vectors; the KV cache [layer][kv_head][position][128] in
// fp16 (or fp32); activations x, q, k, v, att, ffn (fp32), logits (fp32);
// attention split partials; a RoPE (cos, sin) table built on the host with the
// reference's own powf / cosf / sinf (src/brain_runtime.c:1383-1387).
#include <algorithm>
#include <cfloat>
#include <cmath>
#include <cstddef>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <array>
#include <vector>
#include "../../include/atlas_cuda.h"
#include "engine.h"
#include "quant.cuh"

#include "prefill.h"
#include "gemv.h"
#include "decode2.h"
#include "batch.h"

extern "C" cudaError_t atlas_launch_decode(const atlas::Program *pg, int grid, cudaStream_t stream);
extern "C" size_t atlas_decode_hdr_bytes();
extern "C" size_t atlas_decode_attn_bytes();
extern "C" cudaError_t atlas_launch_prefill_gemm(const atlas::pf::GemmArgs *a, int grid, cudaStream_t stream);
extern "C" cudaError_t atlas_prefill_gemm_pairs(int *pairs);
extern "C" cudaError_t atlas_launch_gemv2(const atlas::gv::GemvArgs *a, cudaStream_t stream);
extern "C" cudaError_t atlas_launch_prefill_split(const float *x, uint32_t ldx, uint32_t cols, uint32_t tokens,
                                                  uint32_t tok_pad, const float *norm_w, float eps, uint8_t *xt,
                                                  float *xscale, cudaStream_t stream);
extern "C" cudaError_t atlas_launch_prefill_embed(const uint32_t *ids, uint32_t tokens, const uint8_t *embd,
                                                  uint32_t type, uint64_t row_bytes, uint32_t hidden, float *x,
                                                  cudaStream_t stream);
extern "C" cudaError_t atlas_launch_prefill_attn_tc(const atlas::pf::AttnArgs *a, int grid, cudaStream_t stream);
extern "C" size_t atlas_d2_mv_smem(uint32_t cols, uint32_t nslot, uint32_t slot_bytes, uint32_t tslots);
extern "C" size_t atlas_d2_mv4_smem(uint32_t cols, uint32_t warps, uint32_t nslot, uint32_t slot_bytes);
extern "C" size_t atlas_d2_attn_smem(uint32_t splits);
extern "C" int atlas_d2_attn_max_clusters(uint32_t group, uint32_t tc);
extern "C" cudaError_t atlas_d2_setup(size_t mv_smem, size_t attn_smem);
extern "C" cudaError_t atlas_d2_launch_mv(const atlas::d2::MvArgs *a, uint32_t grid, cudaStream_t stream);
extern "C" cudaError_t atlas_d2_launch_attn(const atlas::d2::AttnArgs *a, uint32_t grid, cudaStream_t stream);
extern "C" cudaError_t atlas_d2_launch_attn_b(const atlas::d2::AttnArgs *a, uint32_t grid, uint32_t nseq,
                                              cudaStream_t stream);
extern "C" cudaError_t atlas_d2_launch_embed(const uint8_t *embd, uint64_t row_bytes, uint32_t type, uint32_t hidden,
                                             uint32_t vocab, float *x, atlas::d2::DecState *st, cudaStream_t stream);
extern "C" cudaError_t atlas_d2_launch_argmax(const float *pmax, const uint32_t *pidx, uint32_t n,
                                              atlas::d2::DecState *st, const uint32_t *cnt, uint32_t arrivals,
                                              cudaStream_t stream);
extern "C" cudaError_t atlas_launch_prefill_qknorm(float *q, uint32_t q_heads, const float *kin, void *kcache,
                                                   uint32_t kv_heads, uint32_t max_context, uint32_t pos0,
                                                   uint32_t tokens, const float *qn, const float *kn,
                                                   const float2 *rope, float eps, uint32_t kv_f16,
                                                   cudaStream_t stream);
extern "C" cudaError_t atlas_tp_allreduce(const atlas::d2::TpReduceArgs *a, uint32_t grid, cudaStream_t stream);
extern "C" cudaError_t atlas_launch_wbound(uint32_t type, const uint8_t *blocks, uint64_t nblocks, uint32_t *out_bits,
                                           cudaStream_t stream);


using namespace atlas;

namespace {

thread_local char g_tls_error[512];

struct DevBuf {
    void *p = nullptr;
    size_t n = 0;
};

struct ProgramBuffers {
    Program pg{};
    Phase *d_phases = nullptr;
    uint32_t *d_ctr = nullptr;
    StepState *d_state = nullptr;
    std::vector<Phase> phases;
};

}  // namespace

struct AtlasCuda {
    AtlasModelDesc desc{};
    int sm_count = 0;
    cudaStream_t stream = nullptr;
    std::string err;
    std::vector<void *> allocs;
    // Pinned staging of the weight upload (creation only): host threads fill
    // one buffer while the copy engine drains the other.
    struct Staging {
        uint8_t *buf[2] = {nullptr, nullptr};
        cudaEvent_t done[2] = {nullptr, nullptr};
        size_t cap = 0;
        int next = 0;
    } stg;
    // weights
    struct W {
        const uint8_t *q = nullptr, *k = nullptr, *v = nullptr, *o = nullptr, *gate = nullptr, *up = nullptr, *down = nullptr;
        uint32_t tq = 0, tk = 0, tv = 0, to = 0, tg = 0, tu = 0, td = 0;
        const float *attn_norm = nullptr, *ffn_norm = nullptr, *bq = nullptr, *bk = nullptr, *bv = nullptr;
        const float *qn = nullptr, *kn = nullptr;   // qwen3 per-head q / k RMSNorm weights [head_dim]
        void *kc = nullptr, *vc = nullptr;
        // prefill: power-of-two exponents that bring each tensor's weights into
        // [2^14, 2^15) before the binary16 split
        int eq = 0, ek = 0, ev = 0, eo = 0, eg = 0, eu = 0, ed = 0;
    };
    // Batched prefill buffers, sized for desc.max_prefill tokens per chunk.
    struct Prefill {
        uint32_t cap = 0, tok_pad = 0, terms = 3, max_units = 0, pairs = 0;
        float *x = nullptr, *q = nullptr, *att = nullptr, *ffn = nullptr, *xscale = nullptr, *ws = nullptr;
        float *apart = nullptr;
        float *kq = nullptr;   // qwen3: the chunk's keys before their norm and RoPE
        uint8_t *xt = nullptr;
        uint32_t *actr = nullptr, *units = nullptr, *ids = nullptr, *status = nullptr;
        ProgramBuffers tail;   // final rms_norm + head GEMV + argmax of the last token
    } pf;
    std::vector<W> layers;
    const uint8_t *embd = nullptr, *head = nullptr;
    uint32_t t_embd = 0, t_head = 0;
    const float *out_norm = nullptr;
    float *x = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *att = nullptr, *ffn = nullptr, *logits = nullptr;
    float *part = nullptr;
    uint32_t *split_ctr = nullptr;
    float *pmax = nullptr;
    uint32_t *pidx = nullptr;
    float2 *rope = nullptr;
    uint32_t *d_out_ids = nullptr;
    uint32_t out_ids_cap = 0;
    ProgramBuffers decode;
    // Graph decode step (decode2.cu): one CUDA graph of PDL-chained kernels.
    struct Graph2 {
        bool on = false;
        d2::DecState *st = nullptr;
        float *apart = nullptr;
        uint32_t *actr = nullptr, *status = nullptr;
        uint32_t splits = 0, kernels = 0;
        bool attn_tc = false;   // fp16 cache: the tensor-core decode attention
        uint64_t *trace = nullptr;   // trace records of atlas_cuda_trace_graph (allocated on first use)
        cudaGraph_t graph = nullptr;
        cudaGraphExec_t exec = nullptr;
    } g2;
    uint64_t launches = 0;
    double last_ms = 0.0;
    double total_ms = 0.0;
    uint32_t n_stages = 0, stage_bytes = 0, max_cols = 0;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    // Tensor parallel: this rank's slice, the exchange areas (own and the
    // peers' mappings), the second residual buffer, prompt ids for prompt mode.
    int tp = 1, rank = 0;
    AtlasTpSlice sl{};
    uint8_t *xchg = nullptr;
    uint8_t *peer[d2::kTpMax] = {};
    bool peer_mapped[d2::kTpMax] = {};
    float *x2 = nullptr;
    // one GPU: the down projection in K parts (partial rows [part][hidden]),
    // added to the residual by the next launch's input staging
    float *kpart = nullptr;
    uint32_t kparts = 1;
    // mv4_kernel: partial rows and counters of row tiles cut between CTAs
    float *xpart = nullptr;
    uint32_t *xcnt = nullptr;
    uint32_t *d_in_ids = nullptr;
    uint32_t in_cap = 0;
    // Several sequences (batch.cu): each has a KV-cache region of kv_seq_bytes
    // in every layer's cache; kv_off selects the region the batched prefill
    // writes. gb: the batched step of nseq sequences as one CUDA graph.
    uint32_t max_batch = 1;
    uint64_t kv_seq_bytes = 0, kv_off = 0;
    struct GraphB {
        bool on = false;
        uint32_t nseq = 0, kernels = 0, out_cap = 0, red_logits = 0;
        size_t part_cap = 0;   // floats
        d2::DecState *st = nullptr;
        float *x = nullptr, *qkv = nullptr, *att = nullptr, *ffn = nullptr, *logits = nullptr;
        double *ssq = nullptr;   // [sequence][row chunk] sums of squares of the residual stream
        float *part = nullptr, *apart = nullptr, *pmax = nullptr;
        uint32_t *actr = nullptr, *pidx = nullptr, *out_ids = nullptr;
        std::vector<float *> qkv_bias;   // per layer: q, k, v biases back to back (null: none)
        cudaGraph_t graph = nullptr;
        cudaGraphExec_t exec = nullptr;
    } gb;
    // Matrices of the reference's other block types (F16, Q5_0, Q5_1, Q8_0,
    // Q5_K): the graph decode step only, prompts replayed through it token by
    // token (prompt mode); the batched prefill's tensor-core contractions take
    // Q4_K / Q6_K.
    bool other_types = false;
    uint32_t pf_seq = 0;   // prefill all-reduces run so far (their exchange occurrence numbers)
    bool broken = false;   // a failed tensor-parallel step left the ranks out of step
};

namespace {

int fail(AtlasCuda *h, int code, const char *fmt, ...)
{
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    if (h) h->err = buf;
    snprintf(g_tls_error, sizeof(g_tls_error), "%s", buf);
    return code;
}

#define CU(h, call)                                                                          \
    do {                                                                                     \
        cudaError_t e_ = (call);                                                             \
        if (e_ != cudaSuccess)                                                               \
            return fail((h), ATLAS_ECUDA, "%s failed: %s", #call, cudaGetErrorString(e_));   \
    } while (0)

// Device check with a per-device cache (cudaGetDeviceProperties costs
// milliseconds; the attribute queries are cheap and asked once).
int device_ok(int device, int *sms)
{
    static int cached_sms[64];
    static int cached_major[64];
    if (device < 0 || device >= 64) return ATLAS_ENODEV;
    if (!cached_major[device]) {
        int n = 0;
        if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0 || device >= n) return ATLAS_ENODEV;
        int major = 0, count = 0;
        if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess ||
            cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
            return ATLAS_ENODEV;
        cached_sms[device] = count;
        cached_major[device] = major;
    }
    if (cached_major[device] != 10) return ATLAS_ENODEV;
    if (sms) *sms = cached_sms[device];
    return ATLAS_OK;
}

template <typename T>
int dalloc(AtlasCuda *h, T **out, size_t bytes)
{
    void *p = nullptr;
    const size_t n = (bytes + 255) & ~size_t(255);
    cudaError_t e = cudaMalloc(&p, n ? n : 256);
    if (e != cudaSuccess) return fail(h, ATLAS_ENOMEM, "cudaMalloc(%zu) failed: %s", n, cudaGetErrorString(e));
    h->allocs.push_back(p);
    *out = reinterpret_cast<T *>(p);
    return ATLAS_OK;
}

// Host bytes -> device. Large copies go through the pinned staging buffers in
// chunks: host threads copy chunk i into one buffer while chunk i - 1's
// transfer runs from the other (a pageable cudaMemcpy stages through the
// driver's own small buffers one at a time).
int upload(AtlasCuda *h, void *dst, const void *src, size_t bytes)
{
    AtlasCuda::Staging &st = h->stg;
    if (!st.cap || bytes < (size_t(4) << 20)) {
        CU(h, cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice));
        return ATLAS_OK;
    }
    const unsigned nt = std::max(1u, std::min(8u, std::thread::hardware_concurrency()));
    for (size_t off = 0; off < bytes; off += st.cap) {
        const size_t n = std::min(st.cap, bytes - off);
        const int i = st.next;
        st.next ^= 1;
        CU(h, cudaEventSynchronize(st.done[i]));   // the buffer's previous transfer has finished
        const uint8_t *s0 = static_cast<const uint8_t *>(src) + off;
        std::vector<std::thread> pool;
        const size_t per = (n / nt + 4095) & ~size_t(4095);
        for (unsigned t = 0; t < nt; ++t) {
            const size_t a = std::min(n, t * per), b = std::min(n, a + per);
            if (a < b) pool.emplace_back([&st, i, s0, a, b] { memcpy(st.buf[i] + a, s0 + a, b - a); });
        }
        for (std::thread &th : pool) th.join();
        CU(h, cudaMemcpyAsync(static_cast<uint8_t *>(dst) + off, st.buf[i], n, cudaMemcpyHostToDevice, h->stream));
        CU(h, cudaEventRecord(st.done[i], h->stream));
    }
    return ATLAS_OK;
}

void staging_open(AtlasCuda *h)
{
    AtlasCuda::Staging &st = h->stg;
    const size_t cap = size_t(64) << 20;
    for (int i = 0; i < 2; ++i) {
        if (cudaHostAlloc(reinterpret_cast<void **>(&st.buf[i]), cap, cudaHostAllocDefault) != cudaSuccess ||
            cudaEventCreateWithFlags(&st.done[i], cudaEventDisableTiming) != cudaSuccess) {
            cudaGetLastError();
            return;   // plain pageable copies (cap stays 0)
        }
    }
    st.cap = cap;
}

void staging_close(AtlasCuda *h)
{
    AtlasCuda::Staging &st = h->stg;
    if (st.cap) cudaStreamSynchronize(h->stream);
    for (int i = 0; i < 2; ++i) {
        if (st.buf[i]) cudaFreeHost(st.buf[i]);
        if (st.done[i]) cudaEventDestroy(st.done[i]);
        st.buf[i] = nullptr;
        st.done[i] = nullptr;
    }
    st.cap = 0;
}

const AtlasTensorDesc *find(const AtlasTensorDesc *t, uint32_t n, const char *name)
{
    for (uint32_t i = 0; i < n; ++i)
        if (t[i].name && !strcmp(t[i].name, name)) return &t[i];
    return nullptr;
}

uint64_t elems(const AtlasTensorDesc *t)
{
    uint64_t e = 1;
    for (uint32_t d = 0; d < t->n_dims; ++d) e *= t->dims[d];
    return e;
}

// Tensor-parallel slice of rank `rank` of `size`: KV heads (with their query
// heads) split evenly; attn_output columns = the rank's attention-output
// elements, widened to whole 256-blocks (a block shared by two ranks is read
// by both, each zeroing the other's elements); FFN rows in whole 256-blocks
// (ffn_down's columns follow them); output-head rows in whole 16-row tiles.
// Returns a static reason string, or nullptr when the shape splits.
const char *tp_slice_of(const AtlasModelDesc &d, int rank, int size, AtlasTpSlice &s)
{
    s = AtlasTpSlice{};
    if (size != 1 && size != 2 && size != 4 && size != 8) return "tp_size must be 1, 2, 4 or 8";
    if (rank < 0 || rank >= size) return "tp_rank out of range";
    if (!d.kv_heads || d.kv_heads % (uint32_t)size) return "kv_heads is not a multiple of tp_size";
    if (!d.q_heads || d.q_heads % d.kv_heads) return "q_heads is not a multiple of kv_heads";
    const uint32_t nbf = d.ffn / 256u, tiles = d.vocab / 16u;
    if (d.ffn % 256u || nbf < (uint32_t)size) return "ffn is too small to split";
    if (d.vocab % 16u || tiles < (uint32_t)size) return "vocab is not a multiple of 16 rows per rank";
    const uint32_t r = (uint32_t)rank, n = (uint32_t)size, group = d.q_heads / d.kv_heads;
    s.kv_heads = d.kv_heads / n;
    s.kv_head0 = r * s.kv_heads;
    s.q_heads = s.kv_heads * group;
    s.q_head0 = s.kv_head0 * group;
    const uint32_t q0 = s.q_head0 * 128u, q1 = q0 + s.q_heads * 128u;
    s.o_block0 = q0 / 256u;
    s.o_blocks = (q1 + 255u) / 256u - s.o_block0;
    s.o_lo = q0 - 256u * s.o_block0;
    s.o_hi = q1 - 256u * s.o_block0;
    const uint32_t f0 = (uint32_t)((uint64_t)nbf * r / n), f1 = (uint32_t)((uint64_t)nbf * (r + 1u) / n);
    s.ffn_row0 = 256u * f0;
    s.ffn_rows = 256u * (f1 - f0);
    const uint32_t v0 = (uint32_t)((uint64_t)tiles * r / n), v1 = (uint32_t)((uint64_t)tiles * (r + 1u) / n);
    s.vocab_row0 = 16u * v0;
    s.vocab_rows = 16u * (v1 - v0);
    return nullptr;
}

// Rows [row0, row0 + nrows) and 256-column chunks [b0, b0 + nblk) of a matrix
// tensor [rows x cols] of a GEMV type (Q4_K, Q6_K; F16, Q5_0, Q5_1, Q8_0,
// Q5_K). The blocks are uploaded unchanged; a chunk-column slice (a
// tensor-parallel rank's share of a row-split projection) is packed row after
// row.
int upload_matrix_part(AtlasCuda *h, const AtlasTensorDesc *t, uint64_t cols, uint64_t rows, uint64_t row0,
                       uint64_t nrows, uint64_t b0, uint64_t nblk, const uint8_t **dev, uint32_t *type)
{
    if (!t) return fail(h, ATLAS_EINVAL, "missing matrix tensor");
    if (t->type != ATLAS_TYPE_Q4_K && t->type != ATLAS_TYPE_Q6_K && !d2::m4_other_type(t->type))
        return fail(h, ATLAS_EINVAL,
                    "%s: tensor type %u is not supported by the decode engine (F16, Q5_0, Q5_1, Q8_0, Q4_K, Q5_K, "
                    "Q6_K)",
                    t->name, t->type);
    if (t->n_dims != 2 || t->dims[0] != cols || t->dims[1] != rows || cols % 256)
        return fail(h, ATLAS_EINVAL, "%s: dims %llu x %llu, expected %llu x %llu", t->name,
                    (unsigned long long)t->dims[0], (unsigned long long)t->dims[1], (unsigned long long)cols,
                    (unsigned long long)rows);
    // bb: bytes of one row's 256 elements
    const uint64_t nb = cols / 256, bb = 256u / block_elems(t->type) * block_bytes(t->type), rb = nb * bb;
    if (row0 + nrows > rows || b0 + nblk > nb || !nrows || !nblk) return fail(h, ATLAS_EINVAL, "%s: bad slice", t->name);
    const uint64_t bytes = nrows * nblk * bb;
    uint8_t *d = nullptr;
    // slack past the end: the decode GEMV reads a Q6_K block as a 256-byte
    // window from the 16-byte boundary below it
    int rc = dalloc(h, &d, bytes + d2::kM4Q6Overread);
    if (rc) return rc;
    const uint8_t *src = static_cast<const uint8_t *>(t->data) + row0 * rb;
    if (nblk == nb) {
        if ((rc = upload(h, d, src, bytes))) return rc;
    } else {
        std::vector<uint8_t> tmp(bytes);
        for (uint64_t r = 0; r < nrows; ++r) memcpy(&tmp[r * nblk * bb], src + r * rb + b0 * bb, nblk * bb);
        if ((rc = upload(h, d, tmp.data(), bytes))) return rc;
    }
    *dev = d;
    *type = t->type;
    return ATLAS_OK;
}

// Matrix tensor [rows x cols] of a supported GEMV type, uploaded unchanged.
int upload_matrix(AtlasCuda *h, const AtlasTensorDesc *t, uint64_t cols, uint64_t rows, const uint8_t **dev,
                  uint32_t *type)
{
    return upload_matrix_part(h, t, cols, rows, 0, rows, 0, cols / 256, dev, type);
}

// F32 or F16 vector of n elements -> fp32 on the device (load_f32_vector,
// src/brain_runtime.c:1280-1309).
int upload_vector(AtlasCuda *h, const AtlasTensorDesc *t, uint64_t n, const float **dev, uint64_t off = 0,
                  uint64_t count = 0)
{
    if (!count) count = n;
    if (!t || elems(t) != n) return fail(h, ATLAS_EINVAL, "%s: vector of %llu elements expected", t ? t->name : "?",
                                         (unsigned long long)n);
    std::vector<float> tmp(n);
    if (t->type == ATLAS_TYPE_F32) {
        memcpy(tmp.data(), t->data, n * 4);
    } else if (t->type == ATLAS_TYPE_F16) {
        const uint16_t *s = static_cast<const uint16_t *>(t->data);
        for (uint64_t i = 0; i < n; ++i) {
            const uint32_t hb = s[i], sign = (hb & 0x8000u) << 16, e = (hb >> 10) & 31u;
            uint32_t m = hb & 1023u, bits;
            if (e == 31u) bits = sign | 0x7f800000u | (m << 13);
            else if (e) bits = sign | ((e + 112u) << 23) | (m << 13);
            else if (!m) bits = sign;
            else {
                uint32_t sh = 0;
                while (!(m & 0x400u)) { m <<= 1; ++sh; }
                bits = sign | ((113u - sh) << 23) | ((m & 1023u) << 13);
            }
            memcpy(&tmp[i], &bits, 4);
        }
    } else {
        return fail(h, ATLAS_EINVAL, "%s: vector type %u unsupported", t->name, t->type);
    }
    if (off + count > n) return fail(h, ATLAS_EINVAL, "%s: bad vector slice", t->name);
    float *d = nullptr;
    int rc = dalloc(h, &d, count * 4);
    if (rc) return rc;
    CU(h, cudaMemcpy(d, tmp.data() + off, count * 4, cudaMemcpyHostToDevice));
    *dev = d;
    return ATLAS_OK;
}

// GEMV geometry. Items are 16, 32 or 64 rows (MMA row tiles of 16; powers of
// two so item boundaries line up with segment boundaries, which are multiples
// of 128). Chunks are whole rows when 16 rows fit a stage, otherwise 16-row x
// chunk_blocks-column tiles staged one row segment at a time.
void plan_gemv(Phase &ph, uint32_t total_rows, uint32_t grid, uint32_t stage_bytes)
{
    const uint32_t nb = ph.cols / 256u;
    uint32_t bb_max = 0;
    for (uint32_t s = 0; s < ph.n_seg; ++s) bb_max = std::max(bb_max, block_bytes(ph.seg[s].type));
    const uint64_t row_max = (uint64_t)nb * bb_max;
    if (16u * row_max + 32u <= stage_bytes) {
        ph.chunk_blocks = nb;
        ph.seg_stride = 0;
        ph.chunk_rows = (32u * row_max + 32u <= stage_bytes) ? 32u : 16u;
        // item size minimising the busiest CTA's work: rows it streams plus a
        // per-item cost of about 8 rows (partials, barrier, epilogue)
        ph.item_rows = 16;
        uint64_t best = ~0ull;
        for (uint32_t r : {16u, 32u, 64u}) {
            const uint64_t items = (total_rows + r - 1) / r, waves = (items + grid - 1) / grid;
            const uint64_t cost = waves * (r + 8u);
            if (cost <= best) { best = cost; ph.item_rows = r; }
        }
        if (ph.chunk_rows > ph.item_rows) ph.chunk_rows = ph.item_rows;
    } else {
        // 16 row segments of B blocks each, every segment padded by <= 45 bytes
        uint32_t B = (stage_bytes - 16u * 48u) / (16u * bb_max);
        if (B < 1) B = 1;
        const uint32_t nch = (nb + B - 1) / B;
        B = (nb + nch - 1) / nch;  // even out the column chunks
        ph.chunk_blocks = B;
        ph.seg_stride = (B * bb_max + 30u + 15u) & ~15u;
        ph.chunk_rows = 16;
        ph.item_rows = 16;
    }
    ph.n_items = (total_rows + ph.item_rows - 1) / ph.item_rows;
}

Phase gemv_phase(uint32_t cols, uint32_t grid, uint32_t stage_bytes, bool paired, std::initializer_list<Seg> segs,
                 const float *in, uint32_t input_mode, const float *norm_w, uint32_t epi)
{
    Phase ph{};
    ph.kind = PH_GEMV;
    ph.cols = cols;
    ph.paired = paired ? 1u : 0u;
    ph.n_seg = 0;
    for (const Seg &s : segs) {
        ph.seg_start[ph.n_seg + 1] = ph.seg_start[ph.n_seg] + s.rows;
        ph.seg[ph.n_seg++] = s;
    }
    const uint32_t total = paired ? ph.seg[0].rows : ph.seg_start[ph.n_seg];
    plan_gemv(ph, total, grid, stage_bytes);
    ph.in = in;
    ph.input_mode = input_mode;
    ph.norm_w = norm_w;
    ph.epilogue = epi;
    return ph;
}

// Shared-memory plan: header + x staging for the longest GEMV input + as many
// 56 KB stages as fit (2..kMaxStages).
constexpr uint32_t kStageBytesDefault = 57344;

int plan_smem(int device, uint32_t max_cols, uint32_t &n_stages, uint32_t &stage_bytes)
{
    int optin = 0;
    if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device) != cudaSuccess) return ATLAS_ECUDA;
    const size_t xa = std::max<size_t>(x_area_bytes(max_cols), atlas_decode_attn_bytes());
    const size_t fixed = atlas_decode_hdr_bytes() + xa + 1024;  // + static shared margin
    if ((size_t)optin <= fixed) return ATLAS_EINVAL;
    const size_t avail = (size_t)optin - fixed;
    // at least 3 stages; a stage must hold one 64-position fp32 K (or V) tile
    size_t sb = std::min<size_t>(kStageBytesDefault, (avail / 3) & ~size_t(127));
    if (sb < 33792) return ATLAS_EINVAL;
    stage_bytes = (uint32_t)sb;
    n_stages = (uint32_t)std::min<size_t>(kMaxStages, avail / sb);
    return ATLAS_OK;
}

Seg seg_of(const uint8_t *w, uint32_t type, uint32_t rows, uint32_t cols, const float *bias, float *out)
{
    Seg s{};
    s.w = w;
    s.type = type;
    s.rows = rows;
    s.row_bytes = (uint64_t)(cols / 256) * block_bytes(type);
    s.bias = bias;
    s.out = out;
    return s;
}

int finalize_program(AtlasCuda *h, ProgramBuffers &pb, const AtlasCuda *m)
{
    const size_t n = pb.phases.size();
    int rc = dalloc(h, &pb.d_phases, n * sizeof(Phase));
    if (rc) return rc;
    CU(h, cudaMemcpy(pb.d_phases, pb.phases.data(), n * sizeof(Phase), cudaMemcpyHostToDevice));
    if ((rc = dalloc(h, &pb.d_ctr, n * 8 * sizeof(uint32_t)))) return rc;
    CU(h, cudaMemset(pb.d_ctr, 0, n * 8 * sizeof(uint32_t)));
    if ((rc = dalloc(h, &pb.d_state, sizeof(StepState)))) return rc;
    CU(h, cudaMemset(pb.d_state, 0, sizeof(StepState)));
    pb.pg.phases = pb.d_phases;
    if (m) {
        pb.pg.n_stages = m->n_stages;
        pb.pg.stage_bytes = m->stage_bytes;
        pb.pg.max_cols = m->max_cols;
    }
    pb.pg.n_phases = (uint32_t)n;
    pb.pg.phase_ctr = pb.d_ctr;
    pb.pg.state = pb.d_state;
    if (m) {
        pb.pg.q_heads = m->desc.q_heads;
        pb.pg.kv_heads = m->desc.kv_heads;
        pb.pg.head_dim = m->desc.head_dim;
        pb.pg.kv_fp16 = m->desc.kv_fp16 ? 1u : 0u;
        pb.pg.hidden = m->desc.hidden;
        pb.pg.rms_eps = m->desc.rms_eps;
        pb.pg.rope = m->rope;
        pb.pg.max_context = m->desc.max_context;
    }
    return ATLAS_OK;
}

// Host-side copy of the step state fields the API reads back.
struct StateHost {
    StepState s;
};

int reset_program(AtlasCuda *h, ProgramBuffers &pb)
{
    CU(h, cudaMemsetAsync(pb.d_ctr, 0, pb.phases.size() * 8 * sizeof(uint32_t), h->stream));
    CU(h, cudaMemsetAsync(pb.d_state, 0, sizeof(StepState), h->stream));
    return ATLAS_OK;
}

int status_to_code(AtlasCuda *h, uint32_t st)
{
    if (st == kStatusOk) return ATLAS_OK;
    if (st == kStatusBarrierTimeout) return fail(h, ATLAS_ETIMEOUT, "device phase barrier timed out (status %u)", st);
    if (st == kStatusStageTimeout) return fail(h, ATLAS_ETIMEOUT, "device copy stage timed out (status %u)", st);
    if (st == kStatusCombineTimeout) return fail(h, ATLAS_ETIMEOUT, "attention split combine timed out (status %u)", st);
    if (st == kStatusPeerTimeout) return fail(h, ATLAS_ENCCL, "a tensor-parallel peer did not arrive (status %u)", st);
    return fail(h, ATLAS_ECUDA, "device reported status %u", st);
}

// Run `steps` launches of a decode-kernel program starting from (token, pos).
// `timed`: record the launches' device time as this call's (last_ms) - off
// when the program is one part of a larger timed call.
int run_program(AtlasCuda *h, ProgramBuffers &pb, uint32_t token, uint32_t pos, uint32_t steps, uint32_t *out_ids_dev,
                uint32_t *last_token, float *last_logit, bool timed = true)
{
    StepState init{};
    init.pos = pos;
    init.token = token;
    init.out_ids = out_ids_dev;
    init.max_steps = steps;
    // epoch / exit_ctr continue from the device values: only the host-owned
    // tail of the state (from pos on) is written.
    const size_t off = offsetof(StepState, pos);
    CU(h, cudaMemcpyAsync(reinterpret_cast<uint8_t *>(pb.d_state) + off, reinterpret_cast<const uint8_t *>(&init) + off,
                          sizeof(StepState) - off, cudaMemcpyHostToDevice, h->stream));
    if (timed) CU(h, cudaEventRecord(h->ev0, h->stream));
    for (uint32_t i = 0; i < steps; ++i) {
        CU(h, atlas_launch_decode(&pb.pg, h->sm_count, h->stream));
        ++h->launches;
    }
    if (timed) CU(h, cudaEventRecord(h->ev1, h->stream));
    StepState out{};
    CU(h, cudaMemcpyAsync(&out, pb.d_state, sizeof(StepState), cudaMemcpyDeviceToHost, h->stream));
    CU(h, cudaStreamSynchronize(h->stream));
    if (timed) {
        float ms = 0.f;
        cudaEventElapsedTime(&ms, h->ev0, h->ev1);
        h->last_ms = ms;
        h->total_ms += ms;
    }
    if (out.status != kStatusOk) {
        const int rc = status_to_code(h, out.status);
        reset_program(h, pb);
        cudaStreamSynchronize(h->stream);
        return rc;
    }
    if (last_token) *last_token = out.next_token;
    if (last_logit) *last_logit = out.next_logit;
    return ATLAS_OK;
}

// ------------------------------------------------ graph decode step ------

// Shared memory a kernel may take so that two CTAs (this kernel's and its
// successor's) fit on one SM: (228 KB - 2 x 1 KB reserved) / 2.
constexpr uint32_t kHalfSmBytes = 115712;

// Decode GEMV kernel of the graph step: 1 = mv4_kernel (per-warp rings),
// 0 = mv_kernel (producer warp and a ring shared by the CTA).
constexpr uint32_t kMvEngine = 1u;

struct MvPlan {
    d2::MvArgs a{};
    uint32_t grid = 0;
};

d2::MvSeg mvseg(const uint8_t *w, uint32_t type, uint32_t rows, uint32_t cols, const float *bias, float *out)
{
    d2::MvSeg s{};
    s.w = w;
    s.type = type;
    s.rows = rows;
    s.row_bytes = (uint64_t)(cols / block_elems(type)) * block_bytes(type);
    s.bias = bias;
    s.out = out;
    return s;
}

// Bulk copies per whole-row run of 16 rows (decode2.cu): the fewest of 1, 2,
// 4, 8 whose layout puts the 8 rows of an MMA row group (rows m = 0..7 or
// 8..15 -> copy m % C, row m / C of the copy) in shared-memory bank groups
// that collide at most twice.
uint32_t mv_copies(uint64_t row_bytes)
{
    auto odd16 = [](uint64_t v) { return 16u * (((v + 15u) / 16u) | 1u); };
    for (uint32_t C : {1u, 2u, 4u, 8u}) {
        const uint64_t R = 16u / C, cst = odd16(R * row_bytes + 15u);
        uint32_t worst = 0;
        for (uint32_t half = 0; half < 2; ++half) {
            uint32_t hits[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            for (uint32_t m = 8 * half; m < 8 * half + 8; ++m) {
                const uint64_t addr = (m % C) * cst + (m / C) * row_bytes;
                worst = std::max(worst, ++hits[(addr / 16u) % 8u]);
            }
        }
        if (worst <= 2u) return C;
    }
    return 8u;
}

// Task ranges and ring plan of one mv launch shape. Segments get CTAs in
// proportion to their bytes; inside a segment (or the gate/up pair) every CTA
// takes an equal share (+-1) of whole 16-row tiles, so no tile spans two CTAs.
// The ring slot holds `st` tasks; `st` and the ring depth are the largest
// that keep the launch within half an SM's shared memory with at least 3
// slots.
int plan_mv(AtlasCuda *h, MvPlan &p, uint32_t cols, bool paired, const std::vector<d2::MvSeg> &segs, uint32_t epi)
{
    d2::MvArgs &a = p.a;
    a = d2::MvArgs{};
    a.cols = cols;
    a.nb = cols / 256u;
    a.paired = paired ? 1u : 0u;
    a.epi = epi;
    bool other = false;   // a segment of another block type: mv4_kernel's all-types variant
    for (const d2::MvSeg &sg : segs) {
        if (a.n_seg == 3) return fail(h, ATLAS_EINVAL, "mv: too many segments");
        const bool ok_type = sg.type == 12u || sg.type == 14u || d2::m4_other_type(sg.type);
        if (!ok_type || sg.rows % (uint32_t)d2::kMvRows || !sg.rows)
            return fail(h, ATLAS_EINVAL, "mv: segment type %u rows %u unsupported", sg.type, sg.rows);
        if (sg.type != 14u && (reinterpret_cast<uintptr_t>(sg.w) & 15u))
            return fail(h, ATLAS_EINVAL, "mv: type %u tensor not 16-byte aligned", sg.type);
        other = other || d2::m4_other_type(sg.type);
        a.seg[a.n_seg] = sg;
        a.seg[a.n_seg].copies = mv_copies(sg.row_bytes);
        ++a.n_seg;
    }
    if (!cols || cols % 256u || (paired && (a.n_seg != 2 || a.seg[0].rows != a.seg[1].rows)))
        return fail(h, ATLAS_EINVAL, "mv: bad shape");
    if (paired && a.seg[0].type != a.seg[1].type)
        return fail(h, ATLAS_EINVAL, "mv: gate and up of types %u and %u (one type per pair)", a.seg[0].type,
                    a.seg[1].type);
    const uint32_t G = (uint32_t)h->sm_count;
    const uint32_t P = paired ? 2u : 1u, TP = a.nb * P;
    std::vector<uint32_t> cta_n, tiles;
    if (paired) {
        tiles.push_back(a.seg[0].rows / (uint32_t)d2::kMvRows);
        cta_n.push_back(std::min(G, tiles[0]));
    } else {
        // CTAs per segment: the SMs go one at a time to the segment whose
        // warps carry the largest load, a warp's load being its tasks times
        // the cost of one task of the segment's type (a Q6_K task issues about
        // 1.9x the instructions of a Q4_K one: 898 against 475 at the 7B
        // shape). Shares by bytes gave the 7B q/k/v launch's v segment 2 Q6_K
        // tasks per warp while q and k ran 2 Q4_K ones.
        auto cost = [](uint32_t type) { return type == 14u ? 1.9 : type == 12u ? 1.0 : 1.5; };
        auto load = [&](uint32_t s, uint32_t n) {
            const uint64_t per_cta = ((uint64_t)tiles[s] * a.nb + n - 1u) / n;
            return (double)((per_cta + d2::kM4Warps - 1u) / d2::kM4Warps) * cost(a.seg[s].type);
        };
        for (uint32_t s = 0; s < a.n_seg; ++s) {
            tiles.push_back(a.seg[s].rows / (uint32_t)d2::kMvRows);
            cta_n.push_back(1u);
        }
        if (a.n_seg > G) return fail(h, ATLAS_EINVAL, "mv: more segments than SMs");
        for (uint32_t used = a.n_seg; used < G; ++used) {
            uint32_t best = a.n_seg;
            double bl = -1.0;
            for (uint32_t s = 0; s < a.n_seg; ++s) {
                const double l = load(s, cta_n[s]);
                if (cta_n[s] < tiles[s] && l > bl) {
                    bl = l;
                    best = s;
                }
            }
            if (best == a.n_seg) break;
            ++cta_n[best];
        }
    }
    std::vector<d2::MvCta> ctas;
    for (size_t s = 0; s < cta_n.size(); ++s)
        for (uint32_t c = 0; c < cta_n[s]; ++c) {
            d2::MvCta e{};
            e.seg = (uint32_t)s;
            e.j0 = (uint32_t)((uint64_t)tiles[s] * c / cta_n[s]) * TP;
            e.j1 = (uint32_t)((uint64_t)tiles[s] * (c + 1) / cta_n[s]) * TP;
            ctas.push_back(e);
        }
    p.grid = (uint32_t)ctas.size();
    // ring plan
    auto odd16 = [](uint32_t v) { return 16u * (((v + 15u) / 16u) | 1u); };
    // bytes of a run of n blocks (decode2.cu mv_producer), largest over the segments
    auto run_bytes = [&](uint32_t n) {
        uint32_t m = 0;
        for (uint32_t s = 0; s < a.n_seg; ++s) {
            const d2::MvSeg &sg = a.seg[s];
            const uint32_t bb = block_bytes(sg.type), rb = (uint32_t)sg.row_bytes;
            m = std::max(m, n == a.nb ? sg.copies * odd16((16u / sg.copies) * rb + 15u) : 16u * odd16(n * bb + 15u));
        }
        return m;
    };
    // A warp runs at most (nslot + 1) * st tasks ahead of the slowest warp,
    // so tslots > (nslot + 1) * st / TP + 1 open-tile slots never collide.
    auto tslots_of = [&](uint32_t nslot, uint32_t st) { return (nslot + 1u) * st / TP + 2u; };
    // Rows longer than 8 blocks are staged in K-slices, one bulk copy per row
    // piece: such launches take the whole SM so that the pieces can be 8
    // blocks long (a bulk copy costs the copy engine tens of nanoseconds
    // whatever its size), giving up co-residency with their neighbours.
    const uint32_t budgets[2] = {a.nb > 8u ? 227u * 1024u : kHalfSmBytes, 227u * 1024u};
    bool ok = other;   // mv_kernel takes Q4_K and Q6_K only: no plan of its own then
    // The largest slot wins (per-slot costs - descriptors, copy issue,
    // barrier round trips - dominate small slots), on the whole SM if it
    // must: mv CTAs do not share an SM anyway (registers)
    for (uint32_t st : {16u, 8u, 4u, 2u, 1u}) {
        for (uint32_t budget : budgets) {
            // runs in a slot: a partial first run, whole rows, a partial last one
            const uint32_t npmax = std::min(st, (st - 1u) / a.nb + 2u);
            if (npmax > (uint32_t)d2::kMvMaxPortions) continue;
            uint32_t worst = 0;   // over where the slot's first run starts
            for (uint32_t r1 = 1; r1 <= std::min(st, a.nb); ++r1) {
                uint32_t sum = run_bytes(r1), left = st - r1;
                while (left) {
                    const uint32_t n = std::min(a.nb, left);
                    sum += run_bytes(n);
                    left -= n;
                }
                worst = std::max(worst, sum);
            }
            const uint32_t slot = (worst + 127u) & ~127u;
            uint32_t nslot = d2::kMvMaxSlots;
            while (nslot && (tslots_of(nslot, st) > (uint32_t)d2::kMvMaxTileSlots ||
                             atlas_d2_mv_smem(cols, nslot, slot, tslots_of(nslot, st)) > budget))
                --nslot;
            // a warp's next slot is kMvWarps / st slots on; it may be at most
            // one ring round ahead of the slots still in use (mbarrier parity)
            if (nslot >= std::max(3u, (uint32_t)d2::kMvWarps / st)) {
                a.st = st;
                a.nslot = nslot;
                a.slot_bytes = slot;
                a.tslots = tslots_of(nslot, st);
                ok = true;
                break;
            }
        }
        if (ok) break;
    }
    if (!ok) return fail(h, ATLAS_EINVAL, "mv: no shared-memory plan for %u columns", cols);
    if (!other) a.smem_bytes = (uint32_t)atlas_d2_mv_smem(cols, a.nslot, a.slot_bytes, a.tslots);
    if (other) {
        // the kernel of that one type: 16 warps with up to 4 slots, else 8
        // warps with up to 3 (F16 tasks take 8 KB a slot)
        for (uint32_t s = 1; s < a.n_seg; ++s)
            if (a.seg[s].type != a.seg[0].type)
                return fail(h, ATLAS_EINVAL, "mv: a launch of type %u with a segment of type %u", a.seg[0].type,
                            a.seg[s].type);
        const uint32_t slot = d2::m4_slot_bytes(a.seg[0].type);
        a.engine = 0u;
        for (const uint32_t warps : {16u, 8u}) {
            const uint32_t top = warps == 16u ? d2::kM4GenSlots16 : d2::kM4GenSlots8;
            for (uint32_t ns = top; ns >= 2u && !a.engine; --ns)
                if (atlas_d2_mv4_smem(cols, warps, ns, slot) <= 227u * 1024u) {
                    a.engine = 1u;
                    a.gen_type = a.seg[0].type;
                    a.warps = warps;
                    a.nslot = ns;
                    a.slot_bytes = slot;
                    a.smem_bytes = (uint32_t)atlas_d2_mv4_smem(cols, warps, ns, slot);
                }
            if (a.engine) break;
        }
        if (!a.engine) return fail(h, ATLAS_EINVAL, "mv: no shared-memory plan for %u columns", cols);
    } else if (kMvEngine == 1u) {
        // per-warp rings (mv4_kernel): 16 warps with the deepest ring the SM
        // holds (at least 2 slots). The kernel is bound by instruction issue,
        // so all 16 warps stay busy: 8-warp CTAs that let the next launch's
        // CTAs start early measured 32 % slower on the 7B step (3.41 against
        // 2.59 ms), and 8 warps with deeper rings slower on the down
        // projection too. Inputs too long for two slots stay on mv_kernel.
        uint32_t slot = 0;
        for (uint32_t s = 0; s < a.n_seg; ++s)
            slot = std::max(slot, a.seg[s].type == 12u ? 16u * d2::kM4Q4Row : 16u * d2::kM4Q6Row);
        auto deepest = [&](uint32_t warps, uint32_t budget) {
            for (uint32_t ns = d2::kM4MaxSlots; ns >= 2u; --ns)
                if (atlas_d2_mv4_smem(cols, warps, ns, slot) <= budget) return ns;
            return 0u;
        };
        const struct { uint32_t warps, budget, min_ns; } choices[] = {{16u, 227u * 1024u, 2u}};
        for (const auto &ch : choices) {
            const uint32_t ns = deepest(ch.warps, ch.budget);
            if (ns >= ch.min_ns) {
                a.engine = 1u;
                a.warps = ch.warps;
                a.nslot = ns;
                a.slot_bytes = slot;
                a.smem_bytes = (uint32_t)atlas_d2_mv4_smem(cols, ch.warps, ns, slot);
                break;
            }
        }
    }
    // mv4_kernel: every CTA of a segment takes an equal share of its tasks,
    // not whole row tiles (224 tiles of 74 blocks on 148 SMs give some CTAs
    // twice the tiles of others), when that lowers the most tasks any warp
    // runs: a tile cut between CTAs is finished by the last of them to arrive
    // (a fence, an atomic and a read-back of the partial rows at the end of
    // the launch), which costs more than it saves when the busiest warps keep
    // their task count. ATLAS_MV_TILE_RANGES=1 / 0 forces whole tiles / shares.
    const char *tr = getenv("ATLAS_MV_TILE_RANGES");
    bool shares = false;
    if (a.engine == 1u) {
        uint32_t worst_tiles = 0, worst_shares = 0;
        for (size_t s = 0; s < cta_n.size(); ++s) {
            const uint32_t per_tile = (tiles[s] + cta_n[s] - 1u) / cta_n[s] * TP;
            const uint32_t per_share = (uint32_t)(((uint64_t)tiles[s] * TP + cta_n[s] - 1u) / cta_n[s]);
            worst_tiles = std::max(worst_tiles, (per_tile + a.warps - 1u) / a.warps);
            worst_shares = std::max(worst_shares, (per_share + a.warps - 1u) / a.warps);
        }
        shares = tr ? atoi(tr) == 0 : worst_shares < worst_tiles;
    }
    if (shares) {
        ctas.clear();
        for (size_t s = 0; s < cta_n.size(); ++s) {
            const uint64_t n = (uint64_t)tiles[s] * TP;
            for (uint32_t c = 0; c < cta_n[s]; ++c) {
                d2::MvCta e{};
                e.seg = (uint32_t)s;
                e.j0 = (uint32_t)(n * c / cta_n[s]);
                e.j1 = (uint32_t)(n * (c + 1) / cta_n[s]);
                ctas.push_back(e);
            }
        }
        if (!h->xpart) {
            int rc = dalloc(h, &h->xpart, (size_t)G * 2u * 32u * sizeof(float));
            if (!rc) rc = dalloc(h, &h->xcnt, (size_t)G * sizeof(uint32_t));
            if (rc) return rc;
            CU(h, cudaMemset(h->xcnt, 0, (size_t)G * sizeof(uint32_t)));
        }
        a.xpart = h->xpart;
        a.xcnt = h->xcnt;
    }
    // neighbours holding parts of each CTA's first and last tiles
    for (size_t k = 0; k < ctas.size(); ++k) {
        const uint32_t f0 = ctas[k].j0 / TP * TP, l1 = ((ctas[k].j1 - 1u) / TP + 1u) * TP;
        size_t ca = k, cb = k;
        while (ca > 0 && ctas[ca - 1].seg == ctas[k].seg && ctas[ca - 1].j1 > f0) --ca;
        while (cb + 1 < ctas.size() && ctas[cb + 1].seg == ctas[k].seg && ctas[cb + 1].j0 < l1) ++cb;
        ctas[k].ca = (uint32_t)ca;
        ctas[k].cb = (uint32_t)cb;
    }
    d2::MvCta *dc = nullptr;
    int rc = dalloc(h, &dc, ctas.size() * sizeof(d2::MvCta));
    if (rc) return rc;
    CU(h, cudaMemcpy(dc, ctas.data(), ctas.size() * sizeof(d2::MvCta), cudaMemcpyHostToDevice));
    a.cta = dc;
    a.eps = h->desc.rms_eps;
    a.pmax = h->pmax;
    a.pidx = h->pidx;
    a.status = h->g2.status;
    a.pdl = 1u;
    return ATLAS_OK;
}

// Layer l's launch of a planned shape: the layer-0 plan with the layer's
// weight pointers when its matrices have layer 0's types, else the plan of
// the layer's own types (a Q4_K_M file mixes Q4_K and Q6_K across layers)
// with the launch's other fields kept. Plans of a type combination are made
// once (cache).
int layer_plan(AtlasCuda *h, const MvPlan &p0, bool paired, const std::vector<d2::MvSeg> &segs, MvPlan &out,
               std::vector<std::pair<std::vector<uint32_t>, MvPlan>> &cache)
{
    out = p0;
    std::vector<uint32_t> key{p0.a.cols, p0.a.epi, paired ? 1u : 0u};
    bool same = true;
    uint32_t i = 0;
    for (const d2::MvSeg &sg : segs) {
        out.a.seg[i].w = sg.w;
        out.a.seg[i].bias = sg.bias;
        same = same && sg.type == p0.a.seg[i].type;
        key.push_back(sg.type);
        key.push_back(sg.rows);
        ++i;
    }
    if (same) return ATLAS_OK;
    const MvPlan *fresh = nullptr;
    for (const auto &e : cache)
        if (e.first == key) fresh = &e.second;
    if (!fresh) {
        MvPlan p;
        const int rc = plan_mv(h, p, p0.a.cols, paired, segs, p0.a.epi);
        if (rc) return rc;
        cache.emplace_back(key, p);
        fresh = &cache.back().second;
    }
    if (p0.a.epi == d2::MV_PART && fresh->grid != p0.grid)
        return fail(h, ATLAS_EINVAL, "tensor parallel: layer types change the grid of a row-split launch");
    for (uint32_t s = 0; s < p0.a.n_seg; ++s) {
        out.a.seg[s].type = fresh->a.seg[s].type;
        out.a.seg[s].row_bytes = fresh->a.seg[s].row_bytes;
        out.a.seg[s].copies = fresh->a.seg[s].copies;
    }
    out.a.st = fresh->a.st;
    out.a.nslot = fresh->a.nslot;
    out.a.slot_bytes = fresh->a.slot_bytes;
    out.a.tslots = fresh->a.tslots;
    out.a.smem_bytes = fresh->a.smem_bytes;
    out.a.cta = fresh->a.cta;
    out.a.xpart = fresh->a.xpart;
    out.a.xcnt = fresh->a.xcnt;
    out.a.engine = fresh->a.engine;
    out.a.warps = fresh->a.warps;
    out.a.gen_type = fresh->a.gen_type;
    out.grid = fresh->grid;
    return ATLAS_OK;
}

// Kernel family of a block type: Q4_K and Q6_K share mv4_kernel's dispatch,
// every other type has a kernel of its own.
uint32_t mv_family(uint32_t type) { return d2::m4_other_type(type) ? type : 0u; }

// Layer l's q/k/v projections as one launch per kernel family among the
// three matrices (a file may keep attn_q in Q8_0 and attn_k / attn_v in
// Q4_K / Q6_K); x and the step state are the decode step's.
int split_qkv(AtlasCuda *h, const d2::MvSeg (&sg)[3], std::vector<MvPlan> &out,
              std::vector<std::pair<std::vector<uint32_t>, MvPlan>> &cache)
{
    out.clear();
    bool done[3] = {false, false, false};
    for (uint32_t i = 0; i < 3; ++i) {
        if (done[i]) continue;
        std::vector<d2::MvSeg> grp;
        std::vector<uint32_t> key{h->desc.hidden, (uint32_t)d2::MV_STORE, 0u};
        for (uint32_t j = i; j < 3; ++j)
            if (!done[j] && mv_family(sg[j].type) == mv_family(sg[i].type)) {
                grp.push_back(sg[j]);
                key.push_back(sg[j].type);
                key.push_back(sg[j].rows);
                done[j] = true;
            }
        const MvPlan *fresh = nullptr;
        for (const auto &e : cache)
            if (e.first == key) fresh = &e.second;
        if (!fresh) {
            MvPlan p;
            int rc = ATLAS_OK;
            rc = plan_mv(h, p, h->desc.hidden, false, grp, d2::MV_STORE);
            if (rc) return rc;
            cache.emplace_back(key, p);
            fresh = &cache.back().second;
        }
        MvPlan p = *fresh;
        for (size_t k = 0; k < grp.size(); ++k) {
            p.a.seg[k].w = grp[k].w;
            p.a.seg[k].bias = grp[k].bias;
            p.a.seg[k].out = grp[k].out;
        }
        p.a.x = h->x;
        p.a.dstate = h->g2.st;
        out.push_back(p);
    }
    return ATLAS_OK;
}

// K parts of the one-GPU down projection: one when the whole row's staged
// input leaves shared memory for a 3-slot ring of Q6_K tasks in every one of
// 16 warps, else the most parts (up to kMvMaxKParts, dividing the row's
// blocks) that do. With FFN 18944 (7B) the whole row leaves room for 2 slots;
// shorter parts also shorten every CTA's input staging (14B: 4.91 ms/token
// with 2 parts, 4.83 with 3). ATLAS_DOWN_KPARTS=n sets the count.
uint32_t down_kparts(const AtlasCuda *h)
{
    if (h->tp > 1 || h->other_types) return 1u;
    const uint32_t nb = h->sl.ffn_rows / 256u, slot = 16u * d2::kM4Q6Row;
    if (const char *e = getenv("ATLAS_DOWN_KPARTS")) {
        const uint32_t n = (uint32_t)std::max(1, atoi(e));
        return n <= d2::kMvMaxKParts && nb % n == 0 ? n : 1u;
    }
    if (atlas_d2_mv4_smem(nb * 256u, 16u, 3u, slot) <= 227u * 1024u) return 1u;
    for (uint32_t n = d2::kMvMaxKParts; n >= 2u; --n)
        if (nb % n == 0 && atlas_d2_mv4_smem(nb / n * 256u, 16u, 3u, slot) <= 227u * 1024u) return n;
    return 1u;
}

// The down projection's segments: one per K part, each over its slice of the
// columns (weights from the part's first block, input from x + x_off) and
// storing its partial rows into h->kpart; one part: the residual add.
std::vector<d2::MvSeg> down_segs(AtlasCuda *h, const uint8_t *w, uint32_t type, uint32_t parts)
{
    const AtlasModelDesc &d = h->desc;
    const uint32_t cols = h->sl.ffn_rows;
    if (parts <= 1u) return {mvseg(w, type, d.hidden, cols, nullptr, h->x)};
    std::vector<d2::MvSeg> v;
    const uint32_t pc = cols / parts;
    for (uint32_t p = 0; p < parts; ++p) {
        d2::MvSeg s = mvseg(w + (uint64_t)p * (pc / 256u) * block_bytes(type), type, d.hidden, cols, nullptr,
                            h->kpart + (size_t)p * d.hidden);
        s.x_off = p * pc;
        v.push_back(s);
    }
    return v;
}

// Capture one decode step as a CUDA graph of PDL-chained kernels. With
// tensor parallelism the shapes are the rank's slice; o and down push partial
// rows (MV_PART) that the next kernel's staging sums in rank order, with the
// residual kept in two buffers: qkv stages x2 + down partials into x,
// gate/up stages x + o partials into x2.
int build_graph2(AtlasCuda *h)
{
    const AtlasModelDesc &d = h->desc;
    const AtlasTpSlice &sl = h->sl;
    AtlasCuda::Graph2 &g = h->g2;
    const uint32_t G = (uint32_t)h->sm_count, group = d.q_heads / d.kv_heads, tp = (uint32_t)h->tp;
    const uint32_t lq = sl.q_heads * 128u, lkv = sl.kv_heads * 128u;
    if (group > d2::kAttnMaxGroup) return fail(h, ATLAS_EINVAL, "graph decode: more than 8 query heads per KV head");
    int rc = dalloc(h, &g.st, sizeof(d2::DecState));
    if (rc) return rc;
    CU(h, cudaMemset(g.st, 0, sizeof(d2::DecState)));
    g.status = &g.st->status;
    // two attention CTAs fit on an SM: up to two splits per SM and KV head,
    // in whole clusters, and at most 3/4 of the clusters the device holds at
    // once (a second wave doubles the launch at long contexts; a full first
    // wave waits for the last free SMs of a GPC as the preceding kernel drains)
    const uint32_t C = d2::kAttnCluster;
    g.splits = std::max(C, std::min(2u * G / sl.kv_heads, 160u) / C * C);
    // fp16 cache: the tensor-core kernel unless ATLAS_ATTN_TC=0
    const char *tce = getenv("ATLAS_ATTN_TC");
    g.attn_tc = d.kv_fp16 && !(tce && atoi(tce) == 0);
    const int max_cl = atlas_d2_attn_max_clusters(group, g.attn_tc ? 1u : 0u);
    if (max_cl > 0) g.splits = std::max(C, std::min(g.splits, (uint32_t)max_cl * 3u / 4u / sl.kv_heads * C));
    if ((rc = dalloc(h, &g.apart, (size_t)sl.kv_heads * (g.splits / C) * group * d2::kRec * sizeof(float)))) return rc;
    if ((rc = dalloc(h, &g.actr, (size_t)sl.q_heads * 4u))) return rc;
    CU(h, cudaMemset(g.actr, 0, (size_t)sl.q_heads * 4u));

    const AtlasCuda::W &w0 = h->layers[0];
    const uint32_t o_cols = sl.o_blocks * 256u;
    const uint32_t part = tp > 1 ? (uint32_t)d2::MV_PART : (uint32_t)d2::MV_RESID;
    MvPlan qkv, o, gu, dn, hd;
    // q, k and v in one launch when one kernel takes all three (always under
    // tensor parallelism: Q4_K / Q6_K files only)
    const bool qkv_one0 = mv_family(w0.tq) == mv_family(w0.tk) && mv_family(w0.tk) == mv_family(w0.tv);
    if (qkv_one0 &&
        (rc = plan_mv(h, qkv, d.hidden, false,
                      {mvseg(w0.q, w0.tq, lq, d.hidden, w0.bq, h->q), mvseg(w0.k, w0.tk, lkv, d.hidden, w0.bk, h->k),
                       mvseg(w0.v, w0.tv, lkv, d.hidden, w0.bv, h->v)},
                      d2::MV_STORE)))
        return rc;
    if ((rc = plan_mv(h, o, o_cols, false, {mvseg(w0.o, w0.to, d.hidden, o_cols, nullptr, h->x)}, part))) return rc;
    if ((rc = plan_mv(h, gu, d.hidden, true,
                      {mvseg(w0.gate, w0.tg, sl.ffn_rows, d.hidden, nullptr, h->ffn),
                       mvseg(w0.up, w0.tu, sl.ffn_rows, d.hidden, nullptr, nullptr)},
                      d2::MV_SWIGLU)))
        return rc;
    // one GPU, long FFN rows: down in K parts whose partial rows the next
    // launch adds, with the residual alternating between x (even layers) and
    // x2 (odd layers) - qkv of layer l + 1 stages R(l) + parts into R(l + 1)
    h->kparts = down_kparts(h);
    const uint32_t KP = h->kparts;
    if ((rc = plan_mv(h, dn, sl.ffn_rows / KP, false, down_segs(h, w0.down, w0.td, KP), KP > 1 ? (uint32_t)d2::MV_STORE : part)))
        return rc;
    if (KP > 1 && dn.a.engine != 1u) return fail(h, ATLAS_EINVAL, "graph decode: K parts need the mv4 kernel");
    // (down has no rms_norm: a K part's staging sees only its slice of the row)
    auto resid = [&](uint32_t l) { return KP > 1 && (l & 1u) ? h->x2 : h->x; };
    if ((rc = plan_mv(h, hd, d.hidden, false, {mvseg(h->head, h->t_head, sl.vocab_rows, d.hidden, nullptr, h->logits)},
                      d2::MV_LOGITS)))
        return rc;
    qkv.a.x = h->x;
    o.a.x = h->att + (size_t)sl.o_block0 * 256u;
    gu.a.x = h->x;
    dn.a.x = h->ffn;
    hd.a.x = h->x;
    hd.a.norm_w = h->out_norm;
    if (KP > 1) {
        hd.a.x = resid(d.layers - 1u);
        hd.a.in_part = h->kpart;
        hd.a.in_nparts = KP;
    }
    uint32_t arr_o = 0, arr_dn = 0, arr_hd = 0;
    if (tp > 1) {
        // arrivals per occurrence: one per CTA of every rank; o and down have
        // the same rows (hidden) on every rank, head grids follow the slices
        if (o.grid != std::min(G, d.hidden / 16u) || dn.grid != o.grid)
            return fail(h, ATLAS_EINVAL, "tensor parallel: unexpected o / down grid");
        arr_o = tp * o.grid;
        arr_dn = tp * dn.grid;
        for (uint32_t r = 0; r < tp; ++r) {
            AtlasTpSlice rs{};
            tp_slice_of(d, (int)r, (int)tp, rs);
            arr_hd += std::min(G, rs.vocab_rows / 16u);
        }
        if (hd.grid != std::min(G, sl.vocab_rows / 16u) || hd.grid > d2::kTpPStride)
            return fail(h, ATLAS_EINVAL, "tensor parallel: unexpected head grid");
        const d2::TpLayout xl = d2::tp_layout(tp, d.hidden);
        for (MvPlan *p : {&qkv, &o, &gu, &dn, &hd}) {
            for (uint32_t r = 0; r < tp; ++r) p->a.peer[r] = h->peer[r];
            p->a.tp = tp;
            p->a.rank = (uint32_t)h->rank;
            p->a.dstate = g.st;
            p->a.seq_mul = d.layers;
        }
        o.a.x_lo = sl.o_lo;
        o.a.x_hi = sl.o_hi;
        o.a.out_red = xl.red_o;
        o.a.out_cnt = d2::kTpCntO;
        dn.a.out_red = xl.red_dn;
        dn.a.out_cnt = d2::kTpCntDn;
        gu.a.in_red = xl.red_o;
        gu.a.in_cnt = d2::kTpCntO;
        gu.a.in_arrivals = arr_o;
        gu.a.xout = h->x2;
        hd.a.x = h->x2;
        hd.a.in_red = xl.red_dn;
        hd.a.in_cnt = d2::kTpCntDn;
        hd.a.in_arrivals = arr_dn;
        hd.a.seq_add = d.layers;
        hd.a.out_red = xl.pmax;
        hd.a.out_cnt = d2::kTpCntHead;
        hd.a.row_base = sl.vocab_row0;
    }
    size_t mv_smem = 0;
    for (MvPlan *p : {&qkv, &o, &gu, &dn, &hd}) {
        mv_smem = std::max<size_t>(mv_smem, p->a.smem_bytes);
        p->a.dstate = g.st;   // the step's state (tensor-parallel epoch, trace pointer)
    }
    // every layer's launches: q/k/v (one per kernel family), o, gate/up, down
    std::vector<std::array<MvPlan, 4>> lp(d.layers);
    std::vector<std::vector<MvPlan>> lqkv(d.layers);
    {
        std::vector<std::pair<std::vector<uint32_t>, MvPlan>> cache;
        for (uint32_t l = 0; l < d.layers; ++l) {
            const AtlasCuda::W &w = h->layers[l];
            const d2::MvSeg qs[3] = {mvseg(w.q, w.tq, lq, d.hidden, w.bq, h->q), mvseg(w.k, w.tk, lkv, d.hidden, w.bk, h->k),
                                     mvseg(w.v, w.tv, lkv, d.hidden, w.bv, h->v)};
            const bool one = mv_family(w.tq) == mv_family(w.tk) && mv_family(w.tk) == mv_family(w.tv);
            if (one && qkv_one0) {
                MvPlan p;
                if ((rc = layer_plan(h, qkv, false, {qs[0], qs[1], qs[2]}, p, cache))) return rc;
                lqkv[l].push_back(p);
            } else {
                if (tp > 1) return fail(h, ATLAS_EINVAL, "tensor parallel: q, k, v of one kernel family only");
                if ((rc = split_qkv(h, qs, lqkv[l], cache))) return rc;
            }
            for (const MvPlan &p : lqkv[l]) mv_smem = std::max<size_t>(mv_smem, p.a.smem_bytes);
            if ((rc = layer_plan(h, o, false, {mvseg(w.o, w.to, d.hidden, o_cols, nullptr, h->x)}, lp[l][1], cache)) ||
                (rc = layer_plan(h, gu, true,
                                 {mvseg(w.gate, w.tg, sl.ffn_rows, d.hidden, nullptr, h->ffn),
                                  mvseg(w.up, w.tu, sl.ffn_rows, d.hidden, nullptr, nullptr)},
                                 lp[l][2], cache)) ||
                (rc = layer_plan(h, dn, false, down_segs(h, w.down, w.td, KP), lp[l][3], cache)))
                return rc;
            if (KP > 1) {
                if (lp[l][3].a.engine != 1u) return fail(h, ATLAS_EINVAL, "graph decode: K parts need the mv4 kernel");
                lp[l][1].a.seg[0].out = resid(l);   // o adds into the layer's residual buffer
            }
            for (const MvPlan &p : lp[l]) mv_smem = std::max<size_t>(mv_smem, p.a.smem_bytes);
        }
    }
    CU(h, atlas_d2_setup(mv_smem, atlas_d2_attn_smem(g.splits)));

    d2::AttnArgs at{};
    at.q = h->q;
    at.k = h->k;
    at.v = h->v;
    at.att = h->att + (size_t)sl.q_head0 * 128u;
    at.part = g.apart;
    at.ctr = g.actr;
    at.rope = h->rope;
    at.st = g.st;
    at.q_heads = sl.q_heads;
    at.kv_heads = sl.kv_heads;
    at.max_context = d.max_context;
    at.splits = g.splits;
    at.tc = g.attn_tc ? 1u : 0u;
    at.kv_fp16 = d.kv_fp16 ? 1u : 0u;
    at.eps = d.rms_eps;
    if (const char *e = getenv("ATLAS_ATTN_MIN_SPAN")) at.min_span = (uint32_t)std::max(1, atoi(e));

    const uint64_t embd_row = (uint64_t)(d.hidden / block_elems(h->t_embd)) * block_bytes(h->t_embd);
    CU(h, cudaStreamBeginCapture(h->stream, cudaStreamCaptureModeThreadLocal));
    uint32_t kernels = 0;
    cudaError_t e = atlas_d2_launch_embed(h->embd, embd_row, h->t_embd, d.hidden, d.vocab, h->x, g.st, h->stream);
    ++kernels;
    for (uint32_t l = 0; l < d.layers && e == cudaSuccess; ++l) {
        const AtlasCuda::W &w = h->layers[l];
        d2::MvArgs a{};
        for (const MvPlan &p : lqkv[l]) {
            a = p.a;
            a.norm_w = w.attn_norm;
            if (tp > 1 && l > 0) {
                // x = x2 + the down partials of layer l - 1 (occurrence epoch * L + l)
                const d2::TpLayout xl = d2::tp_layout(tp, d.hidden);
                a.x = h->x2;
                a.in_red = xl.red_dn;
                a.in_cnt = d2::kTpCntDn;
                a.in_arrivals = arr_dn;
                a.seq_add = l;
                a.xout = h->x;
            } else if (KP > 1 && l > 0) {
                // x = R(l - 1) + the down parts of layer l - 1, kept as R(l)
                a.x = resid(l - 1u);
                a.in_part = h->kpart;
                a.in_nparts = KP;
                a.xout = resid(l);
            }
            a.trace_slot = kernels++;
            if ((e = atlas_d2_launch_mv(&a, p.grid, h->stream)) != cudaSuccess) break;
        }
        if (e != cudaSuccess) break;
        at.k_cache = w.kc;
        at.v_cache = w.vc;
        at.q_norm = w.qn;
        at.k_norm = w.kn;
        at.trace_slot = kernels++;
        if ((e = atlas_d2_launch_attn(&at, sl.kv_heads * g.splits, h->stream)) != cudaSuccess) break;
        a = lp[l][1].a;
        a.trace_slot = kernels++;
        if ((e = atlas_d2_launch_mv(&a, lp[l][1].grid, h->stream)) != cudaSuccess) break;
        a = lp[l][2].a;
        a.norm_w = w.ffn_norm;
        a.seq_add = l + 1u;
        if (KP > 1) a.x = resid(l);
        a.trace_slot = kernels++;
        if ((e = atlas_d2_launch_mv(&a, lp[l][2].grid, h->stream)) != cudaSuccess) break;
        a = lp[l][3].a;
        a.trace_slot = kernels++;
        if ((e = atlas_d2_launch_mv(&a, lp[l][3].grid, h->stream)) != cudaSuccess) break;
    }
    if (e == cudaSuccess) {
        hd.a.trace_slot = kernels;
        e = atlas_d2_launch_mv(&hd.a, hd.grid, h->stream);
        ++kernels;
    }
    if (e == cudaSuccess) {
        if (tp > 1) {
            const d2::TpLayout xl = d2::tp_layout(tp, d.hidden);
            e = atlas_d2_launch_argmax(reinterpret_cast<const float *>(h->xchg + xl.pmax),
                                       reinterpret_cast<const uint32_t *>(h->xchg + xl.pidx), tp * d2::kTpPStride, g.st,
                                       reinterpret_cast<const uint32_t *>(h->xchg + d2::kTpCntHead), arr_hd, h->stream);
        } else {
            e = atlas_d2_launch_argmax(h->pmax, h->pidx, hd.grid, g.st, nullptr, 0u, h->stream);
        }
        ++kernels;
    }
    cudaGraph_t graph = nullptr;
    const cudaError_t e2 = cudaStreamEndCapture(h->stream, &graph);
    if (e != cudaSuccess || e2 != cudaSuccess) {
        if (graph) cudaGraphDestroy(graph);
        return fail(h, ATLAS_ECUDA, "graph capture failed: %s", cudaGetErrorString(e != cudaSuccess ? e : e2));
    }
    g.graph = graph;
    CU(h, cudaGraphInstantiate(&g.exec, graph, 0));
    g.kernels = kernels;
    g.on = true;
    return ATLAS_OK;
}

// `steps` replays of the step graph from (token, pos); out_ids_dev receives
// the picks when set (advance mode), else one step's pick is returned. With
// in_ids_dev (prompt mode) the token after step s is in_ids_dev[s + 1] while
// there is one. The state's epoch (the exchange sequence) is never rewritten.
int run_graph2(AtlasCuda *h, uint32_t token, uint32_t pos, uint32_t steps, uint32_t *out_ids_dev, uint32_t *last_token,
               float *last_logit, const uint32_t *in_ids_dev = nullptr, uint32_t n_in = 0)
{
    AtlasCuda::Graph2 &g = h->g2;
    if (h->broken)
        return fail(h, ATLAS_ENCCL, "an earlier tensor-parallel step failed; recreate the handles of all ranks");
    if (!g.on) return fail(h, ATLAS_EINVAL, "the decode step is not built (tensor parallel: call atlas_cuda_tp_connect)");
    d2::DecState init{};
    init.pos = pos;
    init.token = token;
    init.max_steps = out_ids_dev ? steps : 0u;
    init.advance = 1u;
    init.out_ids = out_ids_dev;
    init.in_ids = in_ids_dev;
    init.n_in = n_in;
    CU(h, cudaMemcpyAsync(g.st, &init, offsetof(d2::DecState, epoch), cudaMemcpyHostToDevice, h->stream));
    CU(h, cudaEventRecord(h->ev0, h->stream));
    for (uint32_t i = 0; i < steps; ++i) CU(h, cudaGraphLaunch(g.exec, h->stream));
    CU(h, cudaEventRecord(h->ev1, h->stream));
    h->launches += (uint64_t)steps * g.kernels;
    d2::DecState out{};
    CU(h, cudaMemcpyAsync(&out, g.st, sizeof(out), cudaMemcpyDeviceToHost, h->stream));
    CU(h, cudaStreamSynchronize(h->stream));
    float ms = 0.f;
    cudaEventElapsedTime(&ms, h->ev0, h->ev1);
    h->last_ms = ms;
    h->total_ms += ms;
    if (out.status != kStatusOk) {
        if (h->tp > 1) {
            // the ranks' exchange counters no longer agree
            h->broken = true;
            if (out.status == kStatusPeerTimeout)
                return fail(h, ATLAS_ENCCL, "a tensor-parallel peer did not arrive (status %u)", out.status);
            return status_to_code(h, out.status);
        }
        const int rc = status_to_code(h, out.status);
        // clear what a failed step may have left behind
        cudaMemsetAsync(g.actr, 0, (size_t)h->sl.q_heads * 4u, h->stream);
        cudaMemsetAsync(g.st, 0, sizeof(d2::DecState), h->stream);
        cudaStreamSynchronize(h->stream);
        return rc;
    }
    if (last_token) *last_token = out.next_token;
    if (last_logit) *last_logit = out.next_logit;
    return ATLAS_OK;
}

int run_decode(AtlasCuda *h, uint32_t token, uint32_t pos, uint32_t steps, uint32_t *out_ids_dev, uint32_t *last_token,
               float *last_logit)
{
    if (h->g2.on || h->tp > 1) return run_graph2(h, token, pos, steps, out_ids_dev, last_token, last_logit);
    return run_program(h, h->decode, token, pos, steps, out_ids_dev, last_token, last_logit);
}

int build_decode_program(AtlasCuda *h)
{
    const AtlasModelDesc &d = h->desc;
    const uint32_t G = (uint32_t)h->sm_count;
    h->max_cols = std::max(d.hidden, std::max(d.q_dim, d.ffn));
    if (plan_smem(d.device, h->max_cols, h->n_stages, h->stage_bytes) != ATLAS_OK)
        return fail(h, ATLAS_EINVAL, "model too large for the shared-memory plan (input length %u)", h->max_cols);
    const uint32_t SB = h->stage_bytes;
    std::vector<Phase> &P = h->decode.phases;
    Phase e{};
    e.kind = PH_EMBED;
    e.embd = h->embd;
    e.embd_type = h->t_embd;
    e.embd_row_bytes = (uint64_t)(d.hidden / block_elems(h->t_embd)) * block_bytes(h->t_embd);
    e.x = h->x;
    P.push_back(e);
    for (uint32_t l = 0; l < d.layers; ++l) {
        const AtlasCuda::W &w = h->layers[l];
        Phase qkv = gemv_phase(d.hidden, G, SB, false,
                               {seg_of(w.q, w.tq, d.q_dim, d.hidden, w.bq, h->q),
                                seg_of(w.k, w.tk, d.kv_dim, d.hidden, w.bk, h->k),
                                seg_of(w.v, w.tv, d.kv_dim, d.hidden, w.bv, h->v)},
                               h->x, IN_RMSNORM, w.attn_norm, EPI_STORE);
        qkv.layer = l;
        P.push_back(qkv);
        Phase at{};
        at.kind = PH_ATTN;
        at.layer = l;
        at.q = h->q; at.k = h->k; at.v = h->v;
        at.k_cache = w.kc; at.v_cache = w.vc;
        at.att = h->att;
        at.part = h->part;
        at.split_ctr = h->split_ctr;
        P.push_back(at);
        Phase o = gemv_phase(d.q_dim, G, SB, false, {seg_of(w.o, w.to, d.hidden, d.q_dim, nullptr, h->x)}, h->att, IN_RAW,
                             nullptr, EPI_RESID_ADD);
        o.layer = l;
        P.push_back(o);
        Phase gu = gemv_phase(d.hidden, G, SB, true,
                              {seg_of(w.gate, w.tg, d.ffn, d.hidden, nullptr, h->ffn),
                               seg_of(w.up, w.tu, d.ffn, d.hidden, nullptr, nullptr)},
                              h->x, IN_RMSNORM, w.ffn_norm, EPI_SWIGLU);
        gu.layer = l;
        P.push_back(gu);
        Phase dn = gemv_phase(d.ffn, G, SB, false, {seg_of(w.down, w.td, d.hidden, d.ffn, nullptr, h->x)}, h->ffn, IN_RAW,
                              nullptr, EPI_RESID_ADD);
        dn.layer = l;
        P.push_back(dn);
    }
    Phase hd = gemv_phase(d.hidden, G, SB, false, {seg_of(h->head, h->t_head, d.vocab, d.hidden, nullptr, h->logits)}, h->x,
                          IN_RMSNORM, h->out_norm, EPI_LOGITS);
    // one (max, argmax) partial per CTA that holds head items (allocated at creation)
    int rc = ATLAS_OK;
    hd.partial_max = h->pmax;
    hd.partial_idx = h->pidx;
    const uint32_t head_index = (uint32_t)P.size();
    P.push_back(hd);
    Phase am{};
    am.kind = PH_ARGMAX;
    am.layer = head_index;
    am.argmax_items = std::min(hd.n_items, G);
    P.push_back(am);
    rc = finalize_program(h, h->decode, h);
    if (rc) return rc;
    h->decode.pg.advance = 1;
    return ATLAS_OK;
}

// Rows per CTA of the streaming GEMV: a multiple of 32 (8 warps x 4 rows)
// giving about two CTAs per SM.
uint32_t gemv_rows_per_cta(uint32_t rows, uint32_t sms)
{
    uint32_t r = (rows + 2 * sms - 1) / (2 * sms);
    r = (r + 31u) & ~31u;
    return std::min(256u, std::max(32u, r));
}

// ------------------------------------------------------------------ prefill --

// Exponent e with bound * 2^e in [2^14, 2^15): weights scaled by 2^e keep
// their binary16 hi/lo split inside the normal range.
int weight_exponent(float bound)
{
    if (!(bound > 0.f) || !(bound <= 3.0e38f)) return 0;
    int e = 0;
    frexpf(bound, &e);
    return 15 - e;
}

int compute_weight_exponents(AtlasCuda *h)
{
    const AtlasModelDesc &d = h->desc;
    const size_t n = (size_t)d.layers * 7;
    uint32_t *bits = nullptr;
    int rc = dalloc(h, &bits, n * 4);
    if (rc) return rc;
    CU(h, cudaMemsetAsync(bits, 0, n * 4, h->stream));
    for (uint32_t l = 0; l < d.layers; ++l) {
        const AtlasCuda::W &w = h->layers[l];
        const AtlasTpSlice &sl = h->sl;
        const uint64_t lq = sl.q_heads * 128ull, lkv = sl.kv_heads * 128ull;
        const struct { const uint8_t *p; uint32_t t; uint64_t elems; } m[7] = {
            {w.q, w.tq, lq * d.hidden},   {w.k, w.tk, lkv * d.hidden},
            {w.v, w.tv, lkv * d.hidden},  {w.o, w.to, (uint64_t)d.hidden * sl.o_blocks * 256u},
            {w.gate, w.tg, (uint64_t)sl.ffn_rows * d.hidden}, {w.up, w.tu, (uint64_t)sl.ffn_rows * d.hidden},
            {w.down, w.td, (uint64_t)d.hidden * sl.ffn_rows}};
        for (int i = 0; i < 7; ++i)
            CU(h, atlas_launch_wbound(m[i].t, m[i].p, m[i].elems / 256, bits + l * 7 + i, h->stream));
    }
    std::vector<uint32_t> hb(n);
    CU(h, cudaMemcpyAsync(hb.data(), bits, n * 4, cudaMemcpyDeviceToHost, h->stream));
    CU(h, cudaStreamSynchronize(h->stream));
    for (uint32_t l = 0; l < d.layers; ++l) {
        AtlasCuda::W &w = h->layers[l];
        int *e[7] = {&w.eq, &w.ek, &w.ev, &w.eo, &w.eg, &w.eu, &w.ed};
        for (int i = 0; i < 7; ++i) {
            float f;
            memcpy(&f, &hb[l * 7 + i], 4);
            *e[i] = weight_exponent(f);
        }
    }
    return ATLAS_OK;
}

uint32_t prefill_max_units(const AtlasCuda *h)
{
    return 3u * (uint32_t)h->sm_count + ((h->pf.cap + 7) / 8) * h->desc.kv_heads + 16u;
}

int alloc_prefill(AtlasCuda *h)
{
    const AtlasModelDesc &d = h->desc;
    AtlasCuda::Prefill &p = h->pf;
    p.cap = d.max_prefill;
    p.tok_pad = (p.cap + pf::kPairTokens - 1) / pf::kPairTokens * pf::kPairTokens;
    if (const char *t = getenv("ATLAS_PREFILL_TERMS")) {
        const int v = atoi(t);
        if (v >= 1 && v <= 3) p.terms = (uint32_t)v;
    }
    const uint32_t G = (uint32_t)h->sm_count, tok_tiles = p.tok_pad / pf::kTokTile;
    const uint32_t max_cols = std::max(d.hidden, std::max(d.q_dim, d.ffn));
    const AtlasTpSlice &sl = h->sl;
    int rc;
    if (h->tp > 1) {
        // the residual stream lives in the exchange area: peers write their reduced slices into it
        const d2::TpLayout xl = d2::tp_layout((uint32_t)h->tp, d.hidden, d.max_prefill);
        p.x = reinterpret_cast<float *>(h->xchg + xl.px);
    } else if ((rc = dalloc(h, &p.x, (size_t)p.cap * d.hidden * 4))) {
        return rc;
    }
    if ((rc = dalloc(h, &p.q, (size_t)p.cap * sl.q_heads * 128u * 4))) return rc;
    // all heads' positions (a rank writes its own heads; the others stay zero)
    if ((rc = dalloc(h, &p.att, (size_t)p.cap * d.q_dim * 4))) return rc;
    CU(h, cudaMemset(p.att, 0, (size_t)p.cap * d.q_dim * 4));
    if ((rc = dalloc(h, &p.ffn, (size_t)p.cap * sl.ffn_rows * 4))) return rc;
    if (d.has_qk_norm && (rc = dalloc(h, &p.kq, (size_t)p.cap * sl.kv_heads * 128u * 4))) return rc;
    if ((rc = dalloc(h, &p.xt, (size_t)tok_tiles * (max_cols / pf::kKBlock) * pf::kXTileBytes))) return rc;
    if ((rc = dalloc(h, &p.xscale, (size_t)p.tok_pad * 4))) return rc;
    // split-K partials: a split contraction runs at most one unit per CTA pair,
    // 2 x 128 x 256 floats each
    if ((rc = dalloc(h, &p.ws, (size_t)G * pf::kTokTile * pf::kRowTile * 4))) return rc;
    int pairs = 0;
    if (atlas_prefill_gemm_pairs(&pairs) != cudaSuccess || pairs < 1)
        return fail(h, ATLAS_ECUDA, "no CTA pair of the prefill contraction kernel fits this device");
    p.pairs = std::min((uint32_t)pairs, G / 2);
    p.max_units = prefill_max_units(h);
    if ((rc = dalloc(h, &p.apart, (size_t)p.max_units * 128 * 132 * 4))) return rc;
    const size_t actr = (size_t)((p.cap + 7) / 8) * d.kv_heads * 4;
    if ((rc = dalloc(h, &p.actr, actr))) return rc;
    CU(h, cudaMemset(p.actr, 0, actr));
    if ((rc = dalloc(h, &p.units, (size_t)p.max_units * 4))) return rc;
    if ((rc = dalloc(h, &p.ids, (size_t)p.cap * 4))) return rc;
    if ((rc = dalloc(h, &p.status, 256))) return rc;
    CU(h, cudaMemset(p.status, 0, 256));
    // tensor parallel: the last prompt token runs through the decode step
    if (h->tp > 1) return compute_weight_exponents(h);
    // tail program: rms_norm + head GEMV + argmax over x (the last token's row)
    std::vector<Phase> &P = p.tail.phases;
    Phase hd = gemv_phase(d.hidden, G, h->stage_bytes, false,
                          {seg_of(h->head, h->t_head, d.vocab, d.hidden, nullptr, h->logits)}, h->x, IN_RMSNORM,
                          h->out_norm, EPI_LOGITS);
    hd.partial_max = h->pmax;
    hd.partial_idx = h->pidx;
    P.push_back(hd);
    Phase am{};
    am.kind = PH_ARGMAX;
    am.layer = 0;
    am.argmax_items = std::min(hd.n_items, G);
    P.push_back(am);
    rc = finalize_program(h, p.tail, h);
    if (rc) return rc;
    p.tail.pg.advance = 0;
    return compute_weight_exponents(h);
}

pf::GemmSeg gseg(const uint8_t *w, uint32_t type, uint32_t rows, uint32_t cols, int wexp, const float *bias, float *out,
                 uint64_t head_stride, uint64_t tok_stride, uint32_t tok_off, bool rope)
{
    pf::GemmSeg s{};
    s.w = w;
    s.type = type;
    s.rows = rows;
    s.row_bytes = (uint64_t)(cols / 256) * block_bytes(type);
    s.wexp = wexp;
    s.rope = rope ? 1u : 0u;
    s.bias = bias;
    s.out = out;
    s.head_stride = head_stride;
    s.tok_stride = tok_stride;
    s.tok_off = tok_off;
    s.vec4 = (((uintptr_t)out & 15u) == 0 && head_stride % 4 == 0 && tok_stride % 4 == 0) ? 1u : 0u;
    return s;
}

// Split-K factor: enough K ranges to give every SM a unit when the tile count
// alone does not, keeping at least four 64-wide K blocks per range.
uint32_t plan_ksplit(uint32_t units, uint32_t kblocks, uint32_t grid)
{
    if (units >= grid) return 1;
    uint32_t s = std::min(grid / units, kblocks / 4);
    return s < 1 ? 1 : s;
}

// Fill the tiling fields of `a` and launch the contraction over the activation
// tiles already written for `tokens` tokens of `cols` inputs.
int launch_gemm(AtlasCuda *h, pf::GemmArgs &a, uint32_t cols, uint32_t tokens, uint32_t pos0)
{
    AtlasCuda::Prefill &p = h->pf;
    uint32_t tiles = 0;
    if (a.epi == pf::GEPI_SWIGLU) {
        tiles = (a.seg[0].rows + 127) / 128;
    } else {
        for (uint32_t s = 0; s < a.n_seg; ++s) {
            a.seg[s].tile0 = tiles;
            tiles += (a.seg[s].rows + pf::kRowTile - 1) / pf::kRowTile;
        }
    }
    a.n_tiles = tiles;
    a.tok_pairs = (tokens + pf::kPairTokens - 1) / pf::kPairTokens;
    a.kblocks = cols / pf::kKBlock;
    a.ksplit = plan_ksplit(a.n_tiles * a.tok_pairs, a.kblocks, p.pairs);
    a.tokens = tokens;
    a.pos0 = pos0;
    a.terms = p.terms;
    a.xt = p.xt;
    a.xscale = p.xscale;
    a.rope = reinterpret_cast<const float *>(h->rope);
    a.ws = p.ws;
    a.status = p.status;
    const uint32_t units = a.n_tiles * a.tok_pairs * a.ksplit;
    CU(h, atlas_launch_prefill_gemm(&a, 2 * (int)std::min(units, p.pairs), h->stream));
    h->launches += a.ksplit > 1 ? 2 : 1;   // contraction (+ split-K reduction)
    return ATLAS_OK;
}

int launch_split(AtlasCuda *h, const float *x, uint32_t cols, uint32_t tokens, const float *norm_w, uint32_t ldx = 0)
{
    const uint32_t tok_pad = (tokens + pf::kPairTokens - 1) / pf::kPairTokens * pf::kPairTokens;
    CU(h, atlas_launch_prefill_split(x, ldx ? ldx : cols, cols, tokens, tok_pad, norm_w, h->desc.rms_eps, h->pf.xt,
                                     h->pf.xscale, h->stream));
    ++h->launches;
    return ATLAS_OK;
}

// Attention units for `n` prompt tokens at positions pos0..pos0+n-1: per KV
// head and tile of 128 / group queries, the cached positions
// [0, pos0 + tile end) cut into spans of whole 64-key chunks. When one unit
// per tile fits in one wave over the SMs, the spans are the shortest that
// keep all units in one wave (every unit loads and splits its 128 query rows,
// so short spans pay that again and again: at 512 tokens of the 3B shape,
// 192-key spans take 1.72 ms for 4 layers where 64-key spans took 1.84);
// otherwise they are sized so that all units make about three waves.
int plan_attention(AtlasCuda *h, uint32_t n, uint32_t pos0, pf::AttnArgs &a)
{
    const AtlasModelDesc &d = h->desc;
    const AtlasTpSlice &sl = h->sl;
    // units of 128 query rows: qt tokens x group heads
    const uint32_t group = d.q_heads / d.kv_heads, qtok = std::max(1u, 128u / group);
    const uint32_t G = (uint32_t)h->sm_count, qt_n = (n + qtok - 1) / qtok;
    uint64_t chunks = 0;
    uint32_t max_chunks = 1;
    for (uint32_t qt = 0; qt < qt_n; ++qt) {
        const uint32_t c = (pos0 + std::min(qtok * qt + qtok, n) + 63) / 64;
        chunks += c;
        max_chunks = std::max(max_chunks, c);
    }
    chunks *= sl.kv_heads;
    uint32_t span_chunks = (uint32_t)std::max<uint64_t>(1, (chunks + 3 * G - 1) / (3 * G));
    if ((uint64_t)qt_n * sl.kv_heads <= G) {
        auto units = [&](uint32_t sc) {
            uint64_t u = 0;
            for (uint32_t qt = 0; qt < qt_n; ++qt)
                u += ((pos0 + std::min(qtok * qt + qtok, n) + 63) / 64 + sc - 1) / sc;
            return u * sl.kv_heads;
        };
        span_chunks = 1;
        while (span_chunks < max_chunks && units(span_chunks) > G) ++span_chunks;
    }
    std::vector<uint32_t> tab;
    for (;;) {
        tab.clear();
        const uint32_t span = 64 * span_chunks;
        for (uint32_t g = 0; g < sl.kv_heads; ++g)
            for (uint32_t qt = 0; qt < qt_n; ++qt) {
                const uint32_t kend = pos0 + std::min(qtok * qt + qtok, n), parts = (kend + span - 1) / span;
                for (uint32_t s = 0; s < parts; ++s) tab.push_back(g | (qt << 8) | (s << 20));
            }
        if (tab.size() <= h->pf.max_units && (d.max_context + span - 1) / span < 4096) break;
        ++span_chunks;
    }
    CU(h, cudaMemcpyAsync(h->pf.units, tab.data(), tab.size() * 4, cudaMemcpyHostToDevice, h->stream));
    // the table must stay valid until the copy ran: synchronize before it goes out of scope
    CU(h, cudaStreamSynchronize(h->stream));
    a = pf::AttnArgs{};
    a.q = h->pf.q;
    // the rank's heads at their places in the all-heads rows
    a.out = h->pf.att + (size_t)sl.q_head0 * 128u;
    a.out_stride = d.q_dim;
    a.kv_f16 = d.kv_fp16 ? 1u : 0u;
    a.q_tokens = qtok;
    a.part = h->pf.apart;
    a.ctr = h->pf.actr;
    a.status = h->pf.status;
    a.tokens = n;
    a.pos0 = pos0;
    a.q_heads = sl.q_heads;
    a.kv_heads = sl.kv_heads;
    a.max_context = d.max_context;
    a.q_tiles = qt_n;
    a.span = 64 * span_chunks;
    a.n_units = (uint32_t)tab.size();
    a.unit_tab = h->pf.units;
    return ATLAS_OK;
}

// One chunk of at most pf.cap prompt tokens through every layer
// (forward_prefill_batch, src/brain_runtime_batch.c:1644-1718); leaves the
// last token's final hidden state in x.
int prefill_chunk(AtlasCuda *h, const uint32_t *ids, uint32_t n, uint32_t pos0)
{
    const AtlasModelDesc &d = h->desc;
    const AtlasTpSlice &sl = h->sl;
    AtlasCuda::Prefill &p = h->pf;
    const bool tp = h->tp > 1;
    const uint32_t lq = sl.q_heads * 128u, lkv = sl.kv_heads * 128u, o_cols = sl.o_blocks * 256u;
    CU(h, cudaMemcpyAsync(p.ids, ids, (size_t)n * 4, cudaMemcpyHostToDevice, h->stream));
    CU(h, atlas_launch_prefill_embed(p.ids, n, h->embd, h->t_embd,
                                     (uint64_t)(d.hidden / block_elems(h->t_embd)) * block_bytes(h->t_embd), d.hidden,
                                     p.x, h->stream));
    ++h->launches;
    pf::AttnArgs at;
    int rc = plan_attention(h, n, pos0, at);
    if (rc) return rc;
    // tensor parallel: o and down leave partial rows in the exchange area, the
    // all-reduce adds every rank's to the residual
    d2::TpReduceArgs ar{};
    float *part = nullptr;
    if (tp) {
        const d2::TpLayout xl = d2::tp_layout((uint32_t)h->tp, d.hidden, d.max_prefill);
        for (int r = 0; r < h->tp; ++r) ar.peer[r] = h->peer[r];
        ar.tp = (uint32_t)h->tp;
        ar.rank = (uint32_t)h->rank;
        ar.part = xl.part;
        ar.px = xl.px;
        ar.n4 = n * d.hidden / 4u;
        ar.status = p.status;
        part = reinterpret_cast<float *>(h->xchg + xl.part);
    }
    auto allreduce = [&]() -> int {
        ar.seq = ++h->pf_seq;
        CU(h, atlas_tp_allreduce(&ar, (uint32_t)h->sm_count, h->stream));
        ++h->launches;
        return ATLAS_OK;
    };
    const uint64_t cache_head = (uint64_t)d.max_context * d.head_dim;
    for (uint32_t l = 0; l < d.layers; ++l) {
        const AtlasCuda::W &w = h->layers[l];
        // the sequence region the prompt belongs to (kv_off: 0 for sequence 0)
        float *kc = reinterpret_cast<float *>(static_cast<uint8_t *>(w.kc) + h->kv_off);
        float *vc = reinterpret_cast<float *>(static_cast<uint8_t *>(w.vc) + h->kv_off);
        // attention block: rms_norm -> Q, K, V (+bias, RoPE, KV-cache store) -> attention -> O (+residual)
        if ((rc = launch_split(h, p.x, d.hidden, n, w.attn_norm))) return rc;
        pf::GemmArgs g{};
        g.epi = pf::GEPI_STORE;
        g.n_seg = 3;
        const bool qkn = d.has_qk_norm != 0;
        g.seg[0] = gseg(w.q, w.tq, lq, d.hidden, w.eq, w.bq, p.q, 128, lq, 0, !qkn);
        g.seg[1] = qkn ? gseg(w.k, w.tk, lkv, d.hidden, w.ek, w.bk, p.kq, 128, lkv, 0, false)
                       : gseg(w.k, w.tk, lkv, d.hidden, w.ek, w.bk, kc, cache_head, d.head_dim, pos0, true);
        g.seg[2] = gseg(w.v, w.tv, lkv, d.hidden, w.ev, w.bv, vc, cache_head, d.head_dim, pos0, false);
        if (!qkn) g.seg[1].f16 = d.kv_fp16 ? 1u : 0u;   // element offsets either way
        g.seg[2].f16 = d.kv_fp16 ? 1u : 0u;
        if ((rc = launch_gemm(h, g, d.hidden, n, pos0))) return rc;
        if (qkn) {
            // qwen3: per-head RMSNorm, then RoPE; keys into the cache
            CU(h, atlas_launch_prefill_qknorm(p.q, sl.q_heads, p.kq, kc, sl.kv_heads, d.max_context, pos0, n, w.qn,
                                              w.kn, h->rope, d.rms_eps, d.kv_fp16 ? 1u : 0u, h->stream));
            ++h->launches;
        }
        at.k_cache = kc;
        at.v_cache = vc;
        CU(h, atlas_launch_prefill_attn_tc(&at, (int)std::min<uint32_t>(at.n_units, (uint32_t)h->sm_count),
                                           h->stream));
        ++h->launches;
        // the rank's attn_output blocks (other ranks' heads in them are zero)
        if ((rc = launch_split(h, p.att + (size_t)sl.o_block0 * 256u, o_cols, n, nullptr, d.q_dim))) return rc;
        g = pf::GemmArgs{};
        g.epi = tp ? pf::GEPI_STORE : pf::GEPI_RESID;
        g.n_seg = 1;
        g.seg[0] = gseg(w.o, w.to, d.hidden, o_cols, w.eo, nullptr, tp ? part : p.x, 128, d.hidden, 0, false);
        if ((rc = launch_gemm(h, g, o_cols, n, pos0))) return rc;
        if (tp && (rc = allreduce())) return rc;
        // feed-forward block: rms_norm -> gate, up -> SwiGLU -> down (+residual)
        if ((rc = launch_split(h, p.x, d.hidden, n, w.ffn_norm))) return rc;
        g = pf::GemmArgs{};
        g.epi = pf::GEPI_SWIGLU;
        g.n_seg = 2;
        g.seg[0] = gseg(w.gate, w.tg, sl.ffn_rows, d.hidden, w.eg, nullptr, p.ffn, 128, sl.ffn_rows, 0, false);
        g.seg[1] = gseg(w.up, w.tu, sl.ffn_rows, d.hidden, w.eu, nullptr, nullptr, 0, 0, 0, false);
        if ((rc = launch_gemm(h, g, d.hidden, n, pos0))) return rc;
        if ((rc = launch_split(h, p.ffn, sl.ffn_rows, n, nullptr))) return rc;
        g = pf::GemmArgs{};
        g.epi = tp ? pf::GEPI_STORE : pf::GEPI_RESID;
        g.n_seg = 1;
        g.seg[0] = gseg(w.down, w.td, d.hidden, sl.ffn_rows, w.ed, nullptr, tp ? part : p.x, 128, d.hidden, 0, false);
        if ((rc = launch_gemm(h, g, sl.ffn_rows, n, pos0))) return rc;
        if (tp && (rc = allreduce())) return rc;
    }
    if (!tp)
        CU(h, cudaMemcpyAsync(h->x, p.x + (size_t)(n - 1) * d.hidden, (size_t)d.hidden * 4, cudaMemcpyDeviceToDevice,
                              h->stream));
    return ATLAS_OK;
}

// ----------------------------------------------------- batched step (bt) --

struct BPlan {
    bt::BArgs a{};
    uint32_t grid = 0;
};

bt::BSeg bseg(const uint8_t *w, uint32_t type, uint32_t rows, uint32_t cols, uint32_t prow0)
{
    bt::BSeg s{};
    s.w = w;
    s.type = type;
    s.rows = rows;
    s.row_bytes = (uint64_t)(cols / 256u) * block_bytes(type);
    s.prow0 = prow0;
    return s;
}

// CTAs of one batched GEMV launch: K is cut into slices of at most
// kSplitMax blocks (the 8 inputs of a slice fit in shared memory); every
// (segment, slice) pair gets CTAs in proportion to its bytes, each a
// contiguous range of whole tiles; the ring is the deepest that fits.
int plan_mvb(AtlasCuda *h, BPlan &p, uint32_t cols, std::initializer_list<bt::BSeg> segs, uint32_t nseq)
{
    bt::BArgs &a = p.a;
    a = bt::BArgs{};
    a.cols = cols;
    a.nb = cols / 256u;
    a.nseq = nseq;
    if (!cols || cols % 256u || !nseq || nseq > bt::kMaxSeq) return fail(h, ATLAS_EINVAL, "mvb: bad shape");
    for (const bt::BSeg &sg : segs) {
        if (a.n_seg == 3) return fail(h, ATLAS_EINVAL, "mvb: too many segments");
        if ((sg.type != 12u && sg.type != 14u) || sg.rows % 16u || !sg.rows)
            return fail(h, ATLAS_EINVAL, "several sequences: matrices of type %u are not supported (Q4_K, Q6_K)",
                        sg.type);
        a.seg[a.n_seg++] = sg;
        a.prows = std::max(a.prows, sg.prow0 + sg.rows);
    }
    a.nsplit = (a.nb + bt::kSplitMax - 1u) / bt::kSplitMax;
    a.split_blocks = (a.nb + a.nsplit - 1u) / a.nsplit;
    a.nsplit = (a.nb + a.split_blocks - 1u) / a.split_blocks;
    const uint32_t G = (uint32_t)h->sm_count;
    struct Pair { uint32_t seg, split, tiles, n; double bytes; };
    std::vector<Pair> pr;
    double total = 0;
    for (uint32_t s = 0; s < a.n_seg; ++s)
        for (uint32_t k = 0; k < a.nsplit; ++k) {
            const uint32_t nbs = std::min(a.split_blocks, a.nb - k * a.split_blocks);
            const double by = (double)a.seg[s].rows * nbs * block_bytes(a.seg[s].type);
            pr.push_back(Pair{s, k, a.seg[s].rows / 16u, 1u, by});
            total += by;
        }
    uint32_t used = 0;
    for (Pair &q : pr) {
        q.n = std::min(q.tiles, (uint32_t)std::max(1.0, std::floor((double)G * q.bytes / total + 0.5)));
        used += q.n;
    }
    while (used > G) {
        size_t big = 0;
        for (size_t i = 1; i < pr.size(); ++i)
            if (pr[i].n > pr[big].n) big = i;
        if (pr[big].n <= 1) break;
        --pr[big].n;
        --used;
    }
    std::vector<bt::BCta> ctas;
    for (const Pair &q : pr)
        for (uint32_t c = 0; c < q.n; ++c)
            ctas.push_back(bt::BCta{q.seg, q.tiles * c / q.n, q.tiles * (c + 1) / q.n, q.split});
    p.grid = (uint32_t)ctas.size();
    uint32_t slot = 0;
    for (uint32_t s = 0; s < a.n_seg; ++s) slot = std::max(slot, a.seg[s].type == 12u ? 16u * 144u : 16u * 240u);
    a.nslot = 0;
    for (uint32_t ns = bt::kBMaxSlots; ns >= 2u && !a.nslot; --ns)
        if (bt::mvb_smem(a.split_blocks, ns, slot) <= 227u * 1024u) a.nslot = ns;
    if (!a.nslot) return fail(h, ATLAS_EINVAL, "mvb: no shared-memory plan");
    a.slot_bytes = slot;
    a.smem_bytes = (uint32_t)bt::mvb_smem(a.split_blocks, a.nslot, slot);
    bt::BCta *dc = nullptr;
    int rc = dalloc(h, &dc, ctas.size() * sizeof(bt::BCta));
    if (rc) return rc;
    CU(h, cudaMemcpy(dc, ctas.data(), ctas.size() * sizeof(bt::BCta), cudaMemcpyHostToDevice));
    a.cta = dc;
    a.pdl = 1u;
    return ATLAS_OK;
}

// A plan of a launch shape, made once per combination of block types
// (a Q4_K_M file's attn_v and ffn_down change type across layers).
int cached_mvb(AtlasCuda *h, std::vector<std::pair<std::vector<uint32_t>, BPlan>> &cache, BPlan &out, uint32_t cols,
               std::initializer_list<bt::BSeg> segs, uint32_t nseq)
{
    std::vector<uint32_t> key{cols, nseq};
    for (const bt::BSeg &sg : segs) {
        key.push_back(sg.type);
        key.push_back(sg.rows);
        key.push_back(sg.prow0);
    }
    const BPlan *f = nullptr;
    for (const auto &e : cache)
        if (e.first == key) f = &e.second;
    if (!f) {
        BPlan p;
        const int rc = plan_mvb(h, p, cols, segs, nseq);
        if (rc) return rc;
        cache.emplace_back(key, p);
        f = &cache.back().second;
    }
    out = *f;
    uint32_t i = 0;
    for (const bt::BSeg &sg : segs) out.a.seg[i++].w = sg.w;
    return ATLAS_OK;
}

// The batched step of nseq sequences as one CUDA graph (built on first use,
// rebuilt when nseq changes).
int build_graphb(AtlasCuda *h, uint32_t nseq)
{
    const AtlasModelDesc &d = h->desc;
    AtlasCuda::GraphB &b = h->gb;
    if (b.on && b.nseq == nseq) return ATLAS_OK;
    if (!h->g2.on) return fail(h, ATLAS_EINVAL, "several sequences: the decode step is not built");
    if (h->tp > 1 || h->other_types)
        return fail(h, ATLAS_EINVAL, "several sequences: one GPU and Q4_K / Q6_K matrices only");
    if (!nseq || nseq > h->max_batch)
        return fail(h, ATLAS_EINVAL, "%u sequences: the handle was created for at most %u (desc.max_batch)", nseq,
                    h->max_batch);
    if (b.exec) cudaGraphExecDestroy(b.exec);
    if (b.graph) cudaGraphDestroy(b.graph);
    b.exec = nullptr;
    b.graph = nullptr;
    b.on = false;
    const uint32_t B = h->max_batch, group = d.q_heads / d.kv_heads;
    const uint32_t qkvw = d.q_dim + 2u * d.kv_dim;
    const uint32_t C = d2::kAttnCluster;
    const uint32_t splits = std::max(C, (h->g2.splits / nseq) / C * C);
    int rc = ATLAS_OK;
    if (!b.st) {
        if ((rc = dalloc(h, &b.st, B * sizeof(d2::DecState))) || (rc = dalloc(h, &b.x, (size_t)B * d.hidden * 4)) ||
            (rc = dalloc(h, &b.qkv, (size_t)B * qkvw * 4)) || (rc = dalloc(h, &b.att, (size_t)B * d.q_dim * 4)) ||
            (rc = dalloc(h, &b.ffn, (size_t)B * d.ffn * 4)) || (rc = dalloc(h, &b.logits, (size_t)B * d.vocab * 4)) ||
            (rc = dalloc(h, &b.ssq, (size_t)B * ((d.hidden + bt::kRowChunk - 1u) / bt::kRowChunk) * 8)) ||
            (rc = dalloc(h, &b.apart, (size_t)B * d.kv_heads * (h->g2.splits / C) * group * d2::kRec * 4)) ||
            (rc = dalloc(h, &b.actr, (size_t)B * d.q_heads * 4)))
            return rc;
        CU(h, cudaMemset(b.st, 0, B * sizeof(d2::DecState)));
        CU(h, cudaMemset(b.actr, 0, (size_t)B * d.q_heads * 4));
        b.qkv_bias.assign(d.layers, nullptr);
        for (uint32_t l = 0; l < d.layers; ++l) {
            const AtlasCuda::W &w = h->layers[l];
            if (!w.bq && !w.bk && !w.bv) continue;
            float *bb = nullptr;
            if ((rc = dalloc(h, &bb, (size_t)qkvw * 4))) return rc;
            CU(h, cudaMemset(bb, 0, (size_t)qkvw * 4));
            if (w.bq) CU(h, cudaMemcpy(bb, w.bq, (size_t)d.q_dim * 4, cudaMemcpyDeviceToDevice));
            if (w.bk) CU(h, cudaMemcpy(bb + d.q_dim, w.bk, (size_t)d.kv_dim * 4, cudaMemcpyDeviceToDevice));
            if (w.bv) CU(h, cudaMemcpy(bb + d.q_dim + d.kv_dim, w.bv, (size_t)d.kv_dim * 4, cudaMemcpyDeviceToDevice));
            b.qkv_bias[l] = bb;
        }
        b.red_logits = (d.vocab + bt::kRowChunk - 1u) / bt::kRowChunk;
        if ((rc = dalloc(h, &b.pmax, (size_t)B * b.red_logits * 4)) || (rc = dalloc(h, &b.pidx, (size_t)B * b.red_logits * 4)))
            return rc;
    }
    // the launches' plans (per layer: q/k/v, o, gate/up, down; then the head)
    std::vector<std::pair<std::vector<uint32_t>, BPlan>> cache;
    std::vector<std::array<BPlan, 4>> lp(d.layers);
    BPlan hd;
    size_t part_floats = 0, smem = 0;
    for (uint32_t l = 0; l < d.layers; ++l) {
        const AtlasCuda::W &w = h->layers[l];
        if ((rc = cached_mvb(h, cache, lp[l][0], d.hidden,
                             {bseg(w.q, w.tq, d.q_dim, d.hidden, 0u), bseg(w.k, w.tk, d.kv_dim, d.hidden, d.q_dim),
                              bseg(w.v, w.tv, d.kv_dim, d.hidden, d.q_dim + d.kv_dim)},
                             nseq)) ||
            (rc = cached_mvb(h, cache, lp[l][1], d.q_dim, {bseg(w.o, w.to, d.hidden, d.q_dim, 0u)}, nseq)) ||
            (rc = cached_mvb(h, cache, lp[l][2], d.hidden,
                             {bseg(w.gate, w.tg, d.ffn, d.hidden, 0u), bseg(w.up, w.tu, d.ffn, d.hidden, d.ffn)}, nseq)) ||
            (rc = cached_mvb(h, cache, lp[l][3], d.ffn, {bseg(w.down, w.td, d.hidden, d.ffn, 0u)}, nseq)))
            return rc;
        for (const BPlan &p : lp[l]) {
            part_floats = std::max(part_floats, (size_t)p.a.nsplit * nseq * p.a.prows);
            smem = std::max<size_t>(smem, p.a.smem_bytes);
        }
    }
    if ((rc = cached_mvb(h, cache, hd, d.hidden, {bseg(h->head, h->t_head, d.vocab, d.hidden, 0u)}, nseq))) return rc;
    part_floats = std::max(part_floats, (size_t)hd.a.nsplit * nseq * hd.a.prows);
    smem = std::max<size_t>(smem, hd.a.smem_bytes);
    if (part_floats > b.part_cap) {
        if ((rc = dalloc(h, &b.part, part_floats * 4))) return rc;
        b.part_cap = part_floats;
    }
    CU(h, atlas_bt_setup(smem));

    d2::AttnArgs at{};
    at.q = b.qkv;
    at.k = b.qkv + d.q_dim;
    at.v = b.qkv + d.q_dim + d.kv_dim;
    at.att = b.att;
    at.part = b.apart;
    at.ctr = b.actr;
    at.rope = h->rope;
    at.st = b.st;
    at.q_heads = d.q_heads;
    at.kv_heads = d.kv_heads;
    at.max_context = d.max_context;
    at.splits = splits;
    at.kv_fp16 = d.kv_fp16 ? 1u : 0u;
    at.tc = h->g2.attn_tc ? 1u : 0u;
    at.eps = d.rms_eps;
    at.qkv_stride = qkvw;
    at.att_stride = d.q_dim;
    at.part_seq = d.kv_heads * (splits / C) * group * d2::kRec;
    at.ctr_seq = d.q_heads;
    at.cache_seq_bytes = h->kv_seq_bytes;
    const uint64_t embd_row = (uint64_t)(d.hidden / block_elems(h->t_embd)) * block_bytes(h->t_embd);
    const uint32_t nchunk = (d.hidden + bt::kRowChunk - 1u) / bt::kRowChunk;
    auto chunks = [](uint32_t rows) { return (rows + bt::kRowChunk - 1u) / bt::kRowChunk; };
    auto reduce = [&](const BPlan &p, uint32_t mode, uint32_t rows, const float *bias, float *out, uint32_t grid) {
        bt::BReduce r{};
        r.part = b.part;
        r.nsplit = p.a.nsplit;
        r.nseq = nseq;
        r.prows = p.a.prows;
        r.mode = mode;
        r.rows = rows;
        r.bias = bias;
        r.ssq = b.ssq;
        r.nssq = nchunk;
        r.hidden = d.hidden;
        r.eps = d.rms_eps;
        r.out = out;
        r.ostride = rows;
        r.pmax = b.pmax;
        r.pidx = b.pidx;
        r.pdl = 1u;
        return atlas_bt_launch_reduce(&r, grid, h->stream);
    };
    auto resid = [&](const BPlan &p) {
        bt::BResid r{};
        r.part = b.part;
        r.nsplit = p.a.nsplit;
        r.nseq = nseq;
        r.prows = p.a.prows;
        r.x = b.x;
        r.hidden = d.hidden;
        r.ssq = b.ssq;
        r.pdl = 1u;
        return atlas_bt_launch_resid(&r, h->stream);
    };
    auto mv = [&](BPlan p, const float *x, uint32_t xstride, const float *norm) {
        p.a.x = x;
        p.a.xstride = xstride;
        p.a.norm_w = norm;
        p.a.part = b.part;
        p.a.status = &b.st->status;
        return atlas_bt_launch_mv(&p.a, p.grid, h->stream);
    };
    CU(h, cudaStreamBeginCapture(h->stream, cudaStreamCaptureModeThreadLocal));
    uint32_t k = 0;
    cudaError_t e = atlas_bt_launch_embed(h->embd, embd_row, h->t_embd, d.hidden, d.vocab, b.x, b.ssq, b.st, nseq,
                                          h->stream);
    ++k;
    for (uint32_t l = 0; l < d.layers && e == cudaSuccess; ++l) {
        const AtlasCuda::W &w = h->layers[l];
        if ((e = mv(lp[l][0], b.x, d.hidden, w.attn_norm)) != cudaSuccess) break;
        if ((e = reduce(lp[l][0], bt::BRED_STORE, qkvw, b.qkv_bias[l], b.qkv, chunks(qkvw))) != cudaSuccess) break;
        at.k_cache = w.kc;
        at.v_cache = w.vc;
        at.q_norm = w.qn;
        at.k_norm = w.kn;
        if ((e = atlas_d2_launch_attn_b(&at, d.kv_heads * splits, nseq, h->stream)) != cudaSuccess) break;
        if ((e = mv(lp[l][1], b.att, d.q_dim, nullptr)) != cudaSuccess) break;
        if ((e = resid(lp[l][1])) != cudaSuccess) break;
        if ((e = mv(lp[l][2], b.x, d.hidden, w.ffn_norm)) != cudaSuccess) break;
        if ((e = reduce(lp[l][2], bt::BRED_SWIGLU, d.ffn, nullptr, b.ffn, chunks(d.ffn))) != cudaSuccess) break;
        if ((e = mv(lp[l][3], b.ffn, d.ffn, nullptr)) != cudaSuccess) break;
        if ((e = resid(lp[l][3])) != cudaSuccess) break;
        k += 9;
    }
    if (e == cudaSuccess && (e = mv(hd, b.x, d.hidden, h->out_norm)) == cudaSuccess &&
        (e = reduce(hd, bt::BRED_LOGITS, d.vocab, nullptr, b.logits, b.red_logits)) == cudaSuccess)
        e = atlas_bt_launch_argmax(b.pmax, b.pidx, b.red_logits, b.st, nseq, h->stream);
    k += 3;
    cudaGraph_t graph = nullptr;
    const cudaError_t e2 = cudaStreamEndCapture(h->stream, &graph);
    if (e != cudaSuccess || e2 != cudaSuccess) {
        if (graph) cudaGraphDestroy(graph);
        return fail(h, ATLAS_ECUDA, "batched graph capture failed: %s", cudaGetErrorString(e != cudaSuccess ? e : e2));
    }
    b.graph = graph;
    CU(h, cudaGraphInstantiate(&b.exec, graph, 0));
    b.kernels = k;
    b.nseq = nseq;
    b.on = true;
    return ATLAS_OK;
}

// `steps` replays of the batched step from each sequence's (token, position);
// out_dev[s * steps + i]: sequence s's pick after step i (advance mode).
int run_graphb(AtlasCuda *h, uint32_t nseq, const uint32_t *tok, const uint32_t *pos, uint32_t steps, bool advance)
{
    AtlasCuda::GraphB &b = h->gb;
    int rc = build_graphb(h, nseq);
    if (rc) return rc;
    const size_t need = (size_t)nseq * std::max(steps, 1u);
    if (need > b.out_cap) {
        uint32_t *p = nullptr;
        if ((rc = dalloc(h, &p, need * 4))) return rc;
        b.out_ids = p;
        b.out_cap = (uint32_t)need;
    }
    std::vector<d2::DecState> init(nseq);
    for (uint32_t s = 0; s < nseq; ++s) {
        init[s].pos = pos[s];
        init[s].token = tok[s];
        init[s].advance = advance ? 1u : 0u;
        init[s].max_steps = steps;
        init[s].out_ids = b.out_ids + (size_t)s * steps;
    }
    CU(h, cudaMemcpyAsync(b.st, init.data(), nseq * sizeof(d2::DecState), cudaMemcpyHostToDevice, h->stream));
    CU(h, cudaEventRecord(h->ev0, h->stream));
    for (uint32_t i = 0; i < std::max(steps, 1u); ++i) CU(h, cudaGraphLaunch(b.exec, h->stream));
    CU(h, cudaEventRecord(h->ev1, h->stream));
    h->launches += (uint64_t)std::max(steps, 1u) * b.kernels;
    std::vector<d2::DecState> out(nseq);
    CU(h, cudaMemcpyAsync(out.data(), b.st, nseq * sizeof(d2::DecState), cudaMemcpyDeviceToHost, h->stream));
    CU(h, cudaStreamSynchronize(h->stream));
    float ms = 0.f;
    cudaEventElapsedTime(&ms, h->ev0, h->ev1);
    h->last_ms = ms;
    h->total_ms += ms;
    for (uint32_t s = 0; s < nseq; ++s)
        if (out[s].status != kStatusOk) {
            const int code = status_to_code(h, out[s].status);
            cudaMemsetAsync(b.actr, 0, (size_t)h->max_batch * h->desc.q_heads * 4, h->stream);
            cudaMemsetAsync(b.st, 0, h->max_batch * sizeof(d2::DecState), h->stream);
            cudaStreamSynchronize(h->stream);
            return code;
        }
    return ATLAS_OK;
}

}  // namespace

extern "C" {

int atlas_cuda_device_info(int device, int *sm_count, int *cc_major, int *cc_minor)
{
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return ATLAS_ENODEV;
    cudaDeviceProp p{};
    if (cudaGetDeviceProperties(&p, device) != cudaSuccess) return ATLAS_ENODEV;
    if (sm_count) *sm_count = p.multiProcessorCount;
    if (cc_major) *cc_major = p.major;
    if (cc_minor) *cc_minor = p.minor;
    return ATLAS_OK;
}

const char *atlas_cuda_last_error(const AtlasCuda *h) { return h ? h->err.c_str() : g_tls_error; }

void atlas_cuda_destroy(AtlasCuda *h)
{
    if (!h) return;
    if (h->stream) cudaStreamSynchronize(h->stream);
    staging_close(h);
    if (h->g2.exec) cudaGraphExecDestroy(h->g2.exec);
    if (h->gb.exec) cudaGraphExecDestroy(h->gb.exec);
    if (h->gb.graph) cudaGraphDestroy(h->gb.graph);
    if (h->g2.graph) cudaGraphDestroy(h->g2.graph);
    for (int r = 0; r < (int)d2::kTpMax; ++r)
        if (h->peer_mapped[r]) cudaIpcCloseMemHandle(h->peer[r]);
    for (void *p : h->allocs) cudaFree(p);
    if (h->ev0) cudaEventDestroy(h->ev0);
    if (h->ev1) cudaEventDestroy(h->ev1);
    if (h->stream) cudaStreamDestroy(h->stream);
    delete h;
}

int atlas_cuda_create(const AtlasModelDesc *desc, const AtlasTensorDesc *tensors, uint32_t n_tensors, AtlasCuda **out)
{
    if (!desc || !tensors || !out) return fail(nullptr, ATLAS_EINVAL, "null argument");
    *out = nullptr;
    int sms = 0;
    if (device_ok(desc->device, &sms) != ATLAS_OK)
        return fail(nullptr, ATLAS_ENODEV, "device %d is not an sm_100 GPU (or no CUDA device)", desc->device);
    const AtlasModelDesc &d = *desc;
    if (d.head_dim != (uint32_t)kHeadDim || !d.q_heads || !d.kv_heads || d.q_heads % d.kv_heads ||
        d.q_heads / d.kv_heads > (uint32_t)kMaxGroup || d.q_dim != d.q_heads * d.head_dim ||
        d.kv_dim != d.kv_heads * d.head_dim || d.hidden % 256 || d.ffn % 256 || d.q_dim % 256 || !d.layers ||
        !d.vocab || d.max_context < 2)
        return fail(nullptr, ATLAS_EINVAL, "unsupported model shape (head_dim must be 128, dims multiples of 256)");
    const int tp = d.tp_size > 1 ? d.tp_size : 1;
    AtlasTpSlice sl{0u, d.q_heads, 0u, d.kv_heads, 0u, d.q_dim / 256u, 0u, d.q_dim, 0u, d.ffn, 0u, d.vocab};
    if (tp > 1) {
        if (const char *why = tp_slice_of(d, d.tp_rank, tp, sl))
            return fail(nullptr, ATLAS_EINVAL, "tensor parallel: %s", why);
    }
    AtlasCuda *h = new AtlasCuda();
    h->tp = tp;
    h->rank = tp > 1 ? d.tp_rank : 0;
    h->sl = sl;
    h->desc = d;
    if (h->desc.rms_eps <= 0.f) h->desc.rms_eps = 1e-6f;
    if (h->desc.rope_base <= 0.f) h->desc.rope_base = 1000000.0f;
    if (!h->desc.max_prefill) h->desc.max_prefill = 512;
    h->sm_count = sms;
    int rc = ATLAS_OK;
#define TRY(x) do { rc = (x); if (rc) { snprintf(g_tls_error, sizeof(g_tls_error), "%s", h->err.c_str()); atlas_cuda_destroy(h); return rc; } } while (0)
    if (cudaSetDevice(d.device) != cudaSuccess) TRY(fail(h, ATLAS_ECUDA, "cudaSetDevice failed"));
    if (cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking) != cudaSuccess)
        TRY(fail(h, ATLAS_ECUDA, "stream creation failed"));
    cudaEventCreate(&h->ev0);
    cudaEventCreate(&h->ev1);
    char name[96];
    staging_open(h);
    const AtlasTensorDesc *emb = find(tensors, n_tensors, "token_embd.weight");
    if (!emb) TRY(fail(h, ATLAS_EINVAL, "missing token_embd.weight"));
    TRY(upload_matrix(h, emb, d.hidden, d.vocab, &h->embd, &h->t_embd));
    const AtlasTensorDesc *outw = find(tensors, n_tensors, "output.weight");
    if (!outw || (outw->data == emb->data && outw->type == emb->type)) {
        // tied embeddings: one device copy (a rank's head rows are a row range of it)
        h->head = h->embd + (uint64_t)sl.vocab_row0 * (d.hidden / block_elems(h->t_embd)) * block_bytes(h->t_embd);
        h->t_head = h->t_embd;
    } else {
        TRY(upload_matrix_part(h, outw, d.hidden, d.vocab, sl.vocab_row0, sl.vocab_rows, 0, d.hidden / 256u,
                               &h->head, &h->t_head));
    }
    TRY(upload_vector(h, find(tensors, n_tensors, "output_norm.weight"), d.hidden, &h->out_norm));
    h->layers.resize(d.layers);
    const size_t esz = d.kv_fp16 ? 2 : 4;
    const size_t kv_layer = (size_t)sl.kv_heads * d.max_context * d.head_dim * esz;
    h->max_batch = std::max(1u, std::min(d.max_batch, bt::kMaxSeq));
    if (h->max_batch > 1 && tp > 1) TRY(fail(h, ATLAS_EINVAL, "several sequences: one GPU (tp_size 1) only"));
    h->kv_seq_bytes = kv_layer;
    const uint32_t hb = d.hidden / 256u, lq = sl.q_heads * 128u, lkv = sl.kv_heads * 128u;
    for (uint32_t l = 0; l < d.layers; ++l) {
        AtlasCuda::W &w = h->layers[l];
#define TN(suffix) (snprintf(name, sizeof(name), "blk.%u." suffix, l), find(tensors, n_tensors, name))
        // the rank's share (the whole tensor without tensor parallelism)
        TRY(upload_matrix_part(h, TN("attn_q.weight"), d.hidden, d.q_dim, sl.q_head0 * 128u, lq, 0, hb, &w.q, &w.tq));
        TRY(upload_matrix_part(h, TN("attn_k.weight"), d.hidden, d.kv_dim, sl.kv_head0 * 128u, lkv, 0, hb, &w.k, &w.tk));
        TRY(upload_matrix_part(h, TN("attn_v.weight"), d.hidden, d.kv_dim, sl.kv_head0 * 128u, lkv, 0, hb, &w.v, &w.tv));
        TRY(upload_matrix_part(h, TN("attn_output.weight"), d.q_dim, d.hidden, 0, d.hidden, sl.o_block0, sl.o_blocks,
                               &w.o, &w.to));
        TRY(upload_matrix_part(h, TN("ffn_gate.weight"), d.hidden, d.ffn, sl.ffn_row0, sl.ffn_rows, 0, hb, &w.gate,
                               &w.tg));
        TRY(upload_matrix_part(h, TN("ffn_up.weight"), d.hidden, d.ffn, sl.ffn_row0, sl.ffn_rows, 0, hb, &w.up, &w.tu));
        TRY(upload_matrix_part(h, TN("ffn_down.weight"), d.ffn, d.hidden, 0, d.hidden, sl.ffn_row0 / 256u,
                               sl.ffn_rows / 256u, &w.down, &w.td));
        TRY(upload_vector(h, TN("attn_norm.weight"), d.hidden, &w.attn_norm));
        TRY(upload_vector(h, TN("ffn_norm.weight"), d.hidden, &w.ffn_norm));
        // optional_bias: absent biases are skipped (src/brain_runtime.c:1540-1546)
        if (TN("attn_q.bias")) TRY(upload_vector(h, TN("attn_q.bias"), d.q_dim, &w.bq, sl.q_head0 * 128u, lq));
        if (TN("attn_k.bias")) TRY(upload_vector(h, TN("attn_k.bias"), d.kv_dim, &w.bk, sl.kv_head0 * 128u, lkv));
        if (TN("attn_v.bias")) TRY(upload_vector(h, TN("attn_v.bias"), d.kv_dim, &w.bv, sl.kv_head0 * 128u, lkv));
        if (d.has_qk_norm) {
            // qwen3 (src/brain_runtime.c:1727-1737): one weight vector per head dimension
            TRY(upload_vector(h, TN("attn_q_norm.weight"), d.head_dim, &w.qn));
            TRY(upload_vector(h, TN("attn_k_norm.weight"), d.head_dim, &w.kn));
        }
#undef TN
        TRY(dalloc(h, &w.kc, kv_layer * h->max_batch));
        TRY(dalloc(h, &w.vc, kv_layer * h->max_batch));
        for (uint32_t ty : {w.tq, w.tk, w.tv, w.to, w.tg, w.tu, w.td})
            if (d2::m4_other_type(ty)) h->other_types = true;
    }
    staging_close(h);   // every matrix is on the device (the stream is drained)
    if (d2::m4_other_type(h->t_head)) h->other_types = true;
    if (h->other_types && tp > 1)
        TRY(fail(h, ATLAS_EINVAL, "tensor parallel: Q4_K / Q6_K matrices only (the batched prefill is sliced)"));
    if (h->other_types) {
        TRY(dalloc(h, &h->d_in_ids, (size_t)d.max_context * 4));
        h->in_cap = d.max_context;
    }
    uint32_t big = d.ffn > d.q_dim ? d.ffn : d.q_dim;
    if (d.hidden > big) big = d.hidden;
    // the head's per-CTA (max, row) partials: one per SM, for every engine
    TRY(dalloc(h, &h->pmax, (size_t)sms * sizeof(float)));
    TRY(dalloc(h, &h->pidx, (size_t)sms * sizeof(uint32_t)));
    TRY(dalloc(h, &h->x, d.hidden * 4));
    TRY(dalloc(h, &h->q, lq * 4));
    TRY(dalloc(h, &h->k, lkv * 4));
    TRY(dalloc(h, &h->v, lkv * 4));
    TRY(dalloc(h, &h->att, d.q_dim * 4));   // all heads' positions; a rank writes its own heads only
    if (cudaMemset(h->att, 0, d.q_dim * 4) != cudaSuccess) TRY(fail(h, ATLAS_ECUDA, "memset failed"));
    TRY(dalloc(h, &h->ffn, (size_t)sl.ffn_rows * 4));
    TRY(dalloc(h, &h->logits, (size_t)sl.vocab_rows * 4));
    TRY(dalloc(h, &h->x2, d.hidden * 4));
    TRY(dalloc(h, &h->kpart, (size_t)d2::kMvMaxKParts * d.hidden * 4));
    if (tp > 1) {
        const d2::TpLayout xl = d2::tp_layout((uint32_t)tp, d.hidden, h->desc.max_prefill);
        TRY(dalloc(h, &h->xchg, xl.bytes));
        if (cudaMemset(h->xchg, 0, xl.bytes) != cudaSuccess) TRY(fail(h, ATLAS_ECUDA, "memset failed"));
        std::vector<uint8_t> init((size_t)(xl.part - xl.pmax), 0);
        for (uint32_t i = 0; i < (uint32_t)tp * d2::kTpPStride; ++i) {
            const float lo = -FLT_MAX;
            const uint32_t none = 0xffffffffu;
            memcpy(&init[4u * i], &lo, 4);
            memcpy(&init[xl.pidx - xl.pmax + 4u * i], &none, 4);
        }
        if (cudaMemcpy(h->xchg + xl.pmax, init.data(), init.size(), cudaMemcpyHostToDevice) != cudaSuccess)
            TRY(fail(h, ATLAS_ECUDA, "exchange area upload failed"));
        h->peer[h->rank] = h->xchg;
    }
    size_t nsplit_max = (d.max_context + kAttnChunk - 1) / kAttnChunk + 1;
    if (nsplit_max > (size_t)kMaxSplits) nsplit_max = kMaxSplits;
    TRY(dalloc(h, &h->part, (size_t)d.kv_heads * nsplit_max * (d.q_heads / d.kv_heads) * (d.head_dim + 4) * 4));
    TRY(dalloc(h, &h->split_ctr, 64 * sizeof(uint32_t) * (d.kv_heads + 1)));
    if (cudaMemset(h->split_ctr, 0, 64 * sizeof(uint32_t) * (d.kv_heads + 1)) != cudaSuccess)
        TRY(fail(h, ATLAS_ECUDA, "memset failed"));
    // RoPE table: the reference's angle formula, evaluated with the host libm.
    {
        const uint32_t half = d.head_dim / 2;
        std::vector<float2> tab((size_t)d.max_context * half);
        std::vector<float> freq(half);
        for (uint32_t p = 0; p < half; ++p)
            freq[p] = powf(h->desc.rope_base, -(2.0f * (float)p) / (float)d.head_dim);
        for (uint32_t pos = 0; pos < d.max_context; ++pos)
            for (uint32_t p = 0; p < half; ++p) {
                const float th = (float)pos * freq[p];
                tab[(size_t)pos * half + p] = make_float2(cosf(th), sinf(th));
            }
        TRY(dalloc(h, &h->rope, tab.size() * sizeof(float2)));
        if (cudaMemcpy(h->rope, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice) != cudaSuccess)
            TRY(fail(h, ATLAS_ECUDA, "rope upload failed"));
    }
    if (tp == 1 && h->other_types) {
        TRY(build_graph2(h));
    } else if (tp == 1) {
        TRY(build_decode_program(h));
        // graph decode step unless the persistent decode kernel is asked for
        // (qwen3's q/k norm exists in the graph step only)
        const char *eng = getenv("ATLAS_DECODE_ENGINE");
        if (!eng || strcmp(eng, "persistent") != 0 || d.has_qk_norm) TRY(build_graph2(h));
    }
    if (!h->other_types) TRY(alloc_prefill(h));
    // tensor parallel: the decode step is built by atlas_cuda_tp_connect
    if (cudaDeviceSynchronize() != cudaSuccess) TRY(fail(h, ATLAS_ECUDA, "device sync failed"));
#undef TRY
    *out = h;
    return ATLAS_OK;
}

int atlas_cuda_decode(AtlasCuda *h, uint32_t id, uint32_t pos, float *logits, uint32_t *argmax)
{
    if (!h) return fail(nullptr, ATLAS_EINVAL, "null handle");
    if (id >= h->desc.vocab) return fail(h, ATLAS_ERANGE, "token %u >= vocab %u", id, h->desc.vocab);
    if (pos >= h->desc.max_context) return fail(h, ATLAS_ERANGE, "position %u >= max_context %u", pos, h->desc.max_context);
    if (cudaSetDevice(h->desc.device) != cudaSuccess) return fail(h, ATLAS_ECUDA, "cudaSetDevice failed");
    uint32_t next = 0;
    int rc = run_decode(h, id, pos, 1, nullptr, &next, nullptr);
    if (rc) return rc;
    if (logits) {
        // the rank's vocab slice (all of it without tensor parallelism)
        CU(h, cudaMemcpyAsync(logits + h->sl.vocab_row0, h->logits, (size_t)h->sl.vocab_rows * 4,
                              cudaMemcpyDeviceToHost, h->stream));
        CU(h, cudaStreamSynchronize(h->stream));
    }
    if (argmax) *argmax = next;
    return ATLAS_OK;
}

int atlas_cuda_generate(AtlasCuda *h, uint32_t first, uint32_t pos0, uint32_t steps, uint32_t *out_ids)
{
    if (!h || !out_ids) return fail(h, ATLAS_EINVAL, "null argument");
    if (!steps) return ATLAS_OK;
    if (first >= h->desc.vocab) return fail(h, ATLAS_ERANGE, "token %u >= vocab", first);
    if ((uint64_t)pos0 + steps > h->desc.max_context) return fail(h, ATLAS_ERANGE, "positions exceed max_context");
    if (cudaSetDevice(h->desc.device) != cudaSuccess) return fail(h, ATLAS_ECUDA, "cudaSetDevice failed");
    if (steps > h->out_ids_cap) {
        uint32_t *p = nullptr;
        int rc = dalloc(h, &p, (size_t)steps * 4);
        if (rc) return rc;
        h->d_out_ids = p;
        h->out_ids_cap = steps;
    }
    int rc = run_decode(h, first, pos0, steps, h->d_out_ids, nullptr, nullptr);
    if (rc) return rc;
    CU(h, cudaMemcpyAsync(out_ids, h->d_out_ids, (size_t)steps * 4, cudaMemcpyDeviceToHost, h->stream));
    CU(h, cudaStreamSynchronize(h->stream));
    return ATLAS_OK;
}

int atlas_cuda_prefill_seq(AtlasCuda *h, uint32_t seq, const uint32_t *ids, uint32_t n, uint32_t pos0,
                           float *last_logits, uint32_t *argmax)
{
    if (!h) return fail(nullptr, ATLAS_EINVAL, "null handle");
    if (seq >= h->max_batch)
        return fail(h, ATLAS_ERANGE, "sequence %u >= desc.max_batch %u", seq, h->max_batch);
    if (seq && (h->tp > 1 || h->other_types))
        return fail(h, ATLAS_EINVAL, "several sequences: one GPU and Q4_K / Q6_K matrices only");
    h->kv_off = (uint64_t)seq * h->kv_seq_bytes;
    const int rc = atlas_cuda_prefill(h, ids, n, pos0, last_logits, argmax);
    h->kv_off = 0;
    return rc;
}

int atlas_cuda_generate_batch(AtlasCuda *h, uint32_t nseq, const uint32_t *first, const uint32_t *pos0,
                              uint32_t steps, uint32_t *out_ids)
{
    if (!h || !first || !pos0 || !out_ids) return fail(h, ATLAS_EINVAL, "null argument");
    if (!steps) return ATLAS_OK;
    if (!nseq || nseq > h->max_batch) return fail(h, ATLAS_ERANGE, "nseq %u: 1 .. %u", nseq, h->max_batch);
    for (uint32_t s = 0; s < nseq; ++s) {
        if (first[s] >= h->desc.vocab) return fail(h, ATLAS_ERANGE, "token %u >= vocab", first[s]);
        if ((uint64_t)pos0[s] + steps > h->desc.max_context)
            return fail(h, ATLAS_ERANGE, "sequence %u: positions exceed max_context", s);
    }
    if (cudaSetDevice(h->desc.device) != cudaSuccess) return fail(h, ATLAS_ECUDA, "cudaSetDevice failed");
    int rc = run_graphb(h, nseq, first, pos0, steps, true);
    if (rc) return rc;
    CU(h, cudaMemcpyAsync(out_ids, h->gb.out_ids, (size_t)nseq * steps * 4, cudaMemcpyDeviceToHost, h->stream));
    CU(h, cudaStreamSynchronize(h->stream));
    return ATLAS_OK;
}

int atlas_cuda_decode_batch(AtlasCuda *h, uint32_t nseq, const uint32_t *ids, const uint32_t *pos, float *logits,
                            uint32_t *argmax)
{
    if (!h || !ids || !pos) return fail(h, ATLAS_EINVAL, "null argument");
    if (!nseq || nseq > h->max_batch) return fail(h, ATLAS_ERANGE, "nseq %u: 1 .. %u", nseq, h->max_batch);
    for (uint32_t s = 0; s < nseq; ++s) {
        if (ids[s] >= h->desc.vocab) return fail(h, ATLAS_ERANGE, "token %u >= vocab", ids[s]);
        if (pos[s] >= h->desc.max_context) return fail(h, ATLAS_ERANGE, "position %u >= max_context", pos[s]);
    }
    if (cudaSetDevice(h->desc.device) != cudaSuccess) return fail(h, ATLAS_ECUDA, "cudaSetDevice failed");
    int rc = run_graphb(h, nseq, ids, pos, 1, true);
    if (rc) return rc;
    if (logits)
        CU(h, cudaMemcpyAsync(logits, h->gb.logits, (size_t)nseq * h->desc.vocab * 4, cudaMemcpyDeviceToHost,
                              h->stream));
    if (argmax) CU(h, cudaMemcpyAsync(argmax, h->gb.out_ids, (size_t)nseq * 4, cudaMemcpyDeviceToHost, h->stream));
    CU(h, cudaStreamSynchronize(h->stream));
    return ATLAS_OK;
}

// Batched prefill (forward_prefill_batch, src/brain_runtime_batch.c:1644):
// the prompt in chunks of up to max_prefill tokens through the tensor-core
// contractions, then rms_norm + head + argmax for the last token only (the
// reference's prompt loop asks for no logits before the last token,
// src/brain_runtime.c:2025-2028).
int atlas_cuda_prefill(AtlasCuda *h, const uint32_t *ids, uint32_t n, uint32_t pos0, float *last_logits,
                       uint32_t *argmax)
{
    if (!h || !ids || !n) return fail(h, ATLAS_EINVAL, "empty prefill");
    if ((uint64_t)pos0 + n > h->desc.max_context) return fail(h, ATLAS_ERANGE, "positions exceed max_context");
    for (uint32_t i = 0; i < n; ++i)
        if (ids[i] >= h->desc.vocab) return fail(h, ATLAS_ERANGE, "token %u >= vocab %u", ids[i], h->desc.vocab);
    if (cudaSetDevice(h->desc.device) != cudaSuccess) return fail(h, ATLAS_ECUDA, "cudaSetDevice failed");
    if (h->other_types) {
        // the decode step replayed over the prompt (prompt mode: each step's
        // token is the next prompt token), as the reference's prompt loop
        // runs forward_token per token (src/brain_runtime.c:2025-2028)
        CU(h, cudaMemcpyAsync(h->d_in_ids, ids, (size_t)n * 4, cudaMemcpyHostToDevice, h->stream));
        uint32_t next = 0;
        const int rc = run_graph2(h, ids[0], pos0, n, nullptr, &next, nullptr, h->d_in_ids, n);
        if (rc) return rc;
        if (last_logits) {
            CU(h, cudaMemcpyAsync(last_logits, h->logits, (size_t)h->desc.vocab * 4, cudaMemcpyDeviceToHost, h->stream));
            CU(h, cudaStreamSynchronize(h->stream));
        }
        if (argmax) *argmax = next;
        return ATLAS_OK;
    }
    if (h->tp > 1) {
        // tensor parallel: all but the last token through the batched
        // contractions (partial rows all-reduced over peer memory), then the
        // last one through the decode step (its layers, the split head and
        // the greedy pick across ranks)
        if (h->broken) return fail(h, ATLAS_ENCCL, "an earlier tensor-parallel step failed; recreate all ranks");
        if (!h->g2.on) return fail(h, ATLAS_EINVAL, "tensor parallel: call atlas_cuda_tp_connect first");
        AtlasCuda::Prefill &p = h->pf;
        CU(h, cudaEventRecord(h->ev0, h->stream));
        for (uint32_t off = 0; off + 1 < n; off += p.cap) {
            const int rc = prefill_chunk(h, ids + off, std::min(p.cap, n - 1 - off), pos0 + off);
            if (rc) return rc;
        }
        CU(h, cudaEventRecord(h->ev1, h->stream));
        uint32_t st = 0;
        CU(h, cudaMemcpyAsync(&st, p.status, 4, cudaMemcpyDeviceToHost, h->stream));
        CU(h, cudaStreamSynchronize(h->stream));
        float pms = 0.f;
        cudaEventElapsedTime(&pms, h->ev0, h->ev1);
        if (st != kStatusOk) {
            h->broken = true;
            return status_to_code(h, st);
        }
        uint32_t next = 0;
        int rc = run_graph2(h, ids[n - 1], pos0 + n - 1, 1, nullptr, &next, nullptr);
        if (rc) return rc;
        h->last_ms += pms;
        h->total_ms += pms;
        if (last_logits) {
            CU(h, cudaMemcpyAsync(last_logits + h->sl.vocab_row0, h->logits, (size_t)h->sl.vocab_rows * 4,
                                  cudaMemcpyDeviceToHost, h->stream));
            CU(h, cudaStreamSynchronize(h->stream));
        }
        if (argmax) *argmax = next;
        return ATLAS_OK;
    }
    AtlasCuda::Prefill &p = h->pf;
    CU(h, cudaEventRecord(h->ev0, h->stream));
    for (uint32_t off = 0; off < n; off += p.cap) {
        const int rc = prefill_chunk(h, ids + off, std::min(p.cap, n - off), pos0 + off);
        if (rc) return rc;
    }
    // tail program on x: rms_norm + head GEMV + greedy pick
    ProgramBuffers &pb = p.tail;
    StepState init{};
    init.max_steps = 1;
    const size_t soff = offsetof(StepState, pos);
    CU(h, cudaMemcpyAsync(reinterpret_cast<uint8_t *>(pb.d_state) + soff, reinterpret_cast<const uint8_t *>(&init) + soff,
                          sizeof(StepState) - soff, cudaMemcpyHostToDevice, h->stream));
    CU(h, atlas_launch_decode(&pb.pg, h->sm_count, h->stream));
    ++h->launches;
    CU(h, cudaEventRecord(h->ev1, h->stream));
    StepState out{};
    uint32_t st = 0;
    CU(h, cudaMemcpyAsync(&out, pb.d_state, sizeof(StepState), cudaMemcpyDeviceToHost, h->stream));
    CU(h, cudaMemcpyAsync(&st, p.status, 4, cudaMemcpyDeviceToHost, h->stream));
    CU(h, cudaStreamSynchronize(h->stream));
    float ms = 0.f;
    cudaEventElapsedTime(&ms, h->ev0, h->ev1);
    h->last_ms = ms;
    h->total_ms += ms;
    if (st != kStatusOk || out.status != kStatusOk) {
        const int rc = status_to_code(h, st != kStatusOk ? st : out.status);
        // clear what a failed launch may have left behind
        cudaMemsetAsync(p.status, 0, 4, h->stream);
        reset_program(h, pb);
        const AtlasModelDesc &d = h->desc;
        cudaMemsetAsync(p.actr, 0, (size_t)((p.cap + 7) / 8) * d.kv_heads * 4, h->stream);
        cudaStreamSynchronize(h->stream);
        return rc;
    }
    if (last_logits) {
        CU(h, cudaMemcpyAsync(last_logits, h->logits, (size_t)h->desc.vocab * 4, cudaMemcpyDeviceToHost, h->stream));
        CU(h, cudaStreamSynchronize(h->stream));
    }
    if (argmax) *argmax = out.next_token;
    return ATLAS_OK;
}

int atlas_cuda_tp_slice(const AtlasModelDesc *desc, int rank, int size, AtlasTpSlice *out)
{
    if (!desc || !out) return fail(nullptr, ATLAS_EINVAL, "null argument");
    if (const char *why = tp_slice_of(*desc, rank, size, *out)) return fail(nullptr, ATLAS_EINVAL, "tensor parallel: %s", why);
    return ATLAS_OK;
}

int atlas_cuda_tp_handle(AtlasCuda *h, void *out)
{
    if (!h || !out) return fail(h, ATLAS_EINVAL, "null argument");
    if (h->tp < 2 || !h->xchg) return fail(h, ATLAS_EINVAL, "not a tensor-parallel handle");
    static_assert(sizeof(cudaIpcMemHandle_t) == ATLAS_TP_HANDLE_BYTES, "IPC handle size");
    if (cudaSetDevice(h->desc.device) != cudaSuccess) return fail(h, ATLAS_ECUDA, "cudaSetDevice failed");
    cudaIpcMemHandle_t mh;
    CU(h, cudaIpcGetMemHandle(&mh, h->xchg));
    memcpy(out, &mh, sizeof(mh));
    return ATLAS_OK;
}

int atlas_cuda_tp_connect(AtlasCuda *h, const void *handles)
{
    if (!h || !handles) return fail(h, ATLAS_EINVAL, "null argument");
    if (h->tp < 2) return fail(h, ATLAS_EINVAL, "not a tensor-parallel handle");
    if (h->g2.on) return fail(h, ATLAS_EINVAL, "already connected");
    if (cudaSetDevice(h->desc.device) != cudaSuccess) return fail(h, ATLAS_ECUDA, "cudaSetDevice failed");
    const uint8_t *hb = static_cast<const uint8_t *>(handles);
    for (int r = 0; r < h->tp; ++r) {
        if (r == h->rank) continue;
        cudaIpcMemHandle_t mh;
        memcpy(&mh, hb + (size_t)r * ATLAS_TP_HANDLE_BYTES, sizeof(mh));
        void *p = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&p, mh, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess)
            return fail(h, ATLAS_ECUDA, "mapping rank %d's exchange area failed: %s", r, cudaGetErrorString(e));
        h->peer[r] = static_cast<uint8_t *>(p);
        h->peer_mapped[r] = true;
    }
    const int rc = build_graph2(h);
    if (rc) return rc;
    CU(h, cudaDeviceSynchronize());
    return ATLAS_OK;
}

int atlas_cuda_trace_step(AtlasCuda *h, uint32_t id, uint32_t pos, uint64_t *out_ns, size_t cap, uint32_t *n_ctas,
                          uint32_t *n_phases, uint32_t *phase_kinds)
{
    if (!h) return fail(h, ATLAS_EINVAL, "null handle");
    if (h->tp > 1 || h->desc.has_qk_norm || h->other_types)
        return fail(h, ATLAS_EINVAL, "tracing covers the single-GPU persistent engine (qwen2, Q4_K / Q6_K) only");
    const size_t np = h->decode.phases.size(), per = (size_t)h->sm_count * np, need = per * 12;
    if (n_ctas) *n_ctas = (uint32_t)h->sm_count;
    if (n_phases) *n_phases = (uint32_t)np;
    if (phase_kinds)
        for (size_t i = 0; i < np; ++i) phase_kinds[i] = h->decode.phases[i].kind * 16u + h->decode.phases[i].epilogue;
    if (!out_ns) return fail(h, ATLAS_EINVAL, "null trace buffer");
    if (cap < need) return fail(h, ATLAS_EINVAL, "trace buffer needs %zu slots", need);
    if (id >= h->desc.vocab || pos >= h->desc.max_context) return fail(h, ATLAS_ERANGE, "token or position out of range");
    if (cudaSetDevice(h->desc.device) != cudaSuccess) return fail(h, ATLAS_ECUDA, "cudaSetDevice failed");
    uint64_t *d = nullptr;
    CU(h, cudaMalloc(&d, need * sizeof(uint64_t)));
    CU(h, cudaMemset(d, 0, need * sizeof(uint64_t)));
    h->decode.pg.trace = d;
    h->decode.pg.trace_ext = d + per * 4;
    int rc = run_decode(h, id, pos, 1, nullptr, nullptr, nullptr);
    h->decode.pg.trace = nullptr;
    h->decode.pg.trace_ext = nullptr;
    if (rc == ATLAS_OK) {
        cudaError_t e = cudaMemcpy(out_ns, d, need * sizeof(uint64_t), cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) rc = fail(h, ATLAS_ECUDA, "trace readback: %s", cudaGetErrorString(e));
    }
    cudaFree(d);
    return rc;
}

int atlas_cuda_trace_graph(AtlasCuda *h, uint32_t id, uint32_t pos, uint64_t *out, size_t cap, uint32_t *n_launches,
                           uint32_t *n_ctas, uint32_t *n_words)
{
    if (!h) return fail(h, ATLAS_EINVAL, "null handle");
    AtlasCuda::Graph2 &g = h->g2;
    if (!g.on) return fail(h, ATLAS_EINVAL, "the decode step is not built (tensor parallel: call atlas_cuda_tp_connect)");
    const size_t need = (size_t)g.kernels * d2::kTraceCtas * d2::kTraceWords;
    if (n_launches) *n_launches = g.kernels;
    if (n_ctas) *n_ctas = d2::kTraceCtas;
    if (n_words) *n_words = d2::kTraceWords;
    if (!out) return ATLAS_OK;
    if (cap < need) return fail(h, ATLAS_EINVAL, "trace buffer needs %zu slots", need);
    if (id >= h->desc.vocab || pos >= h->desc.max_context) return fail(h, ATLAS_ERANGE, "token or position out of range");
    if (cudaSetDevice(h->desc.device) != cudaSuccess) return fail(h, ATLAS_ECUDA, "cudaSetDevice failed");
    if (!g.trace) {
        int rc = dalloc(h, &g.trace, need * sizeof(uint64_t));
        if (rc) return rc;
    }
    CU(h, cudaMemsetAsync(g.trace, 0, need * sizeof(uint64_t), h->stream));
    uint64_t *const on = g.trace, *const off = nullptr;
    CU(h, cudaMemcpyAsync(&g.st->trace, &on, sizeof(on), cudaMemcpyHostToDevice, h->stream));
    const int rc = run_graph2(h, id, pos, 1, nullptr, nullptr, nullptr);
    CU(h, cudaMemcpyAsync(&g.st->trace, &off, sizeof(off), cudaMemcpyHostToDevice, h->stream));
    CU(h, cudaStreamSynchronize(h->stream));
    if (rc) return rc;
    CU(h, cudaMemcpy(out, g.trace, need * sizeof(uint64_t), cudaMemcpyDeviceToHost));
    return ATLAS_OK;
}

int atlas_cuda_stats(const AtlasCuda *h, uint64_t *kernel_launches, double *last_ms)
{
    if (!h) return ATLAS_EINVAL;
    if (kernel_launches) *kernel_launches = h->launches;
    if (last_ms) *last_ms = h->last_ms;
    return ATLAS_OK;
}

int atlas_cuda_device_ms(const AtlasCuda *h, double *total_ms)
{
    if (!h || !total_ms) return ATLAS_EINVAL;
    *total_ms = h->total_ms;
    return ATLAS_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Stateless kernels for parity tests
// ---------------------------------------------------------------------------

namespace {

__global__ void dequant_kernel(uint32_t type, const uint8_t *blocks, uint64_t nblocks, float *out)
{
    const uint32_t be = block_elems(type), bb = block_bytes(type);
    const uint64_t total = nblocks * be;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x)
        out[i] = deq_elem(type, blocks + (i / be) * bb, (int)(i % be));
}

}  // namespace

extern "C" int atlas_cuda_dequant(uint32_t type, const void *d_blocks, uint64_t nblocks, float *d_out, void *stream)
{
    if (!block_bytes(type) || !d_blocks || !d_out) return fail(nullptr, ATLAS_EINVAL, "bad dequant arguments");
    int dev = 0;
    cudaGetDevice(&dev);
    if (device_ok(dev, nullptr) != ATLAS_OK) return fail(nullptr, ATLAS_ENODEV, "no sm_100 device");
    if (!nblocks) return ATLAS_OK;
    dequant_kernel<<<592, 256, 0, (cudaStream_t)stream>>>(type, (const uint8_t *)d_blocks, nblocks, d_out);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(nullptr, ATLAS_ECUDA, "dequant launch: %s", cudaGetErrorString(e));
    return ATLAS_OK;
}

extern "C" int atlas_cuda_gemv(uint32_t type, const void *d_weights, uint64_t rows, uint64_t cols, const float *d_x,
                               float *d_y, void *stream)
{
    if ((type != ATLAS_TYPE_Q4_K && type != ATLAS_TYPE_Q6_K) || !d_weights || !d_x || !d_y || !rows || !cols ||
        cols % 256 || rows > 0xffffffffu || cols > 49152)
        return fail(nullptr, ATLAS_EINVAL, "bad gemv arguments");
    if (type == ATLAS_TYPE_Q4_K && ((uintptr_t)d_weights & 15u))
        return fail(nullptr, ATLAS_EINVAL, "Q4_K weights must be 16-byte aligned");
    if ((uintptr_t)d_weights & 1u) return fail(nullptr, ATLAS_EINVAL, "weights must be 2-byte aligned");
    if (((uintptr_t)d_x & 15u) || ((uintptr_t)d_y & 3u))
        return fail(nullptr, ATLAS_EINVAL, "x must be 16-byte aligned and y 4-byte aligned");
    int dev = 0;
    cudaGetDevice(&dev);
    int sms = 0;
    if (dev < 0 || dev >= 16 || device_ok(dev, &sms) != ATLAS_OK) return fail(nullptr, ATLAS_ENODEV, "no sm_100 device");
    gv::GemvArgs a{};
    a.seg[0].w = (const uint8_t *)d_weights;
    a.seg[0].type = type;
    a.seg[0].rows = (uint32_t)rows;
    a.seg[0].row_bytes = (cols / 256) * block_bytes(type);
    a.seg[0].out = d_y;
    a.n_seg = 1;
    a.seg_start[0] = 0;
    a.seg_start[1] = (uint32_t)rows;
    a.cols = (uint32_t)cols;
    a.total_rows = (uint32_t)rows;
    a.rows_per_cta = gemv_rows_per_cta((uint32_t)rows, (uint32_t)sms);
    a.x = d_x;
    a.epi = gv::GV_STORE;
    const cudaError_t e = atlas_launch_gemv2(&a, (cudaStream_t)stream);
    if (e != cudaSuccess) return fail(nullptr, ATLAS_ECUDA, "gemv launch: %s", cudaGetErrorString(e));
    return ATLAS_OK;
}

// Y[tokens][rows] = X[tokens][cols] . W^T on the prefill contraction kernel.
// Scratch (activation tiles, split-K partials, counters) is allocated per call;
// the call synchronizes `stream` to read back the weight bound and the status.
extern "C" int atlas_cuda_gemm(uint32_t type, const void *d_weights, uint64_t rows, uint64_t cols, const float *d_x,
                               uint64_t tokens, float *d_y, void *stream)
{
    if ((type != ATLAS_TYPE_Q4_K && type != ATLAS_TYPE_Q6_K) || !d_weights || !d_x || !d_y || !rows || !cols ||
        !tokens || cols % 256 || rows > 0x7fffffffu || tokens > 0x7fffffffu || cols > pf::kSplitMaxCols)
        return fail(nullptr, ATLAS_EINVAL, "bad gemm arguments");
    if (type == ATLAS_TYPE_Q4_K && ((uintptr_t)d_weights & 15u))
        return fail(nullptr, ATLAS_EINVAL, "Q4_K weights must be 16-byte aligned");
    if ((uintptr_t)d_weights & 1u) return fail(nullptr, ATLAS_EINVAL, "weights must be 2-byte aligned");
    if (((uintptr_t)d_x & 3u) || ((uintptr_t)d_y & 3u)) return fail(nullptr, ATLAS_EINVAL, "x and y must be 4-byte aligned");
    int dev = 0;
    cudaGetDevice(&dev);
    int sms = 0;
    if (device_ok(dev, &sms) != ATLAS_OK) return fail(nullptr, ATLAS_ENODEV, "no sm_100 device");
    cudaStream_t s = (cudaStream_t)stream;
    const uint32_t tok_pairs = (uint32_t)((tokens + pf::kPairTokens - 1) / pf::kPairTokens);
    const uint32_t tiles = (uint32_t)((rows + pf::kRowTile - 1) / pf::kRowTile);
    uint32_t terms = 3;
    if (const char *t = getenv("ATLAS_PREFILL_TERMS")) {
        const int v = atoi(t);
        if (v >= 1 && v <= 3) terms = (uint32_t)v;
    }
    int pairs = 0;
    if (atlas_prefill_gemm_pairs(&pairs) != cudaSuccess || pairs < 1)
        return fail(nullptr, ATLAS_ECUDA, "no CTA pair of the contraction kernel fits this device");
    pairs = std::min(pairs, sms / 2);
    void *xt = nullptr, *xs = nullptr, *ws = nullptr, *st = nullptr;
    int rc = ATLAS_OK;
    cudaError_t e = cudaMalloc(&xt, (size_t)2 * tok_pairs * (cols / pf::kKBlock) * pf::kXTileBytes);
    if (e == cudaSuccess) e = cudaMalloc(&xs, (size_t)tok_pairs * pf::kPairTokens * 4);
    if (e == cudaSuccess) e = cudaMalloc(&ws, (size_t)sms * pf::kTokTile * pf::kRowTile * 4);
    if (e == cudaSuccess) e = cudaMalloc(&st, 256);
    if (e == cudaSuccess) e = cudaMemsetAsync(st, 0, 256, s);
    uint32_t bits = 0, status = 0;
    if (e == cudaSuccess)
        e = atlas_launch_wbound(type, (const uint8_t *)d_weights, rows * (cols / 256), (uint32_t *)st + 32, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(&bits, (uint32_t *)st + 32, 4, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e == cudaSuccess)
        e = atlas_launch_prefill_split(d_x, (uint32_t)cols, (uint32_t)cols, (uint32_t)tokens, tok_pairs * pf::kPairTokens,
                                       nullptr, 0.f, (uint8_t *)xt, (float *)xs, s);
    if (e == cudaSuccess) {
        float bound;
        memcpy(&bound, &bits, 4);
        pf::GemmArgs a{};
        a.epi = pf::GEPI_STORE;
        a.n_seg = 1;
        a.seg[0] = gseg((const uint8_t *)d_weights, type, (uint32_t)rows, (uint32_t)cols, weight_exponent(bound), nullptr,
                        d_y, 128, rows, 0, false);
        a.n_tiles = tiles;
        a.tok_pairs = tok_pairs;
        a.kblocks = (uint32_t)(cols / pf::kKBlock);
        a.ksplit = plan_ksplit(tiles * tok_pairs, a.kblocks, (uint32_t)pairs);
        a.tokens = (uint32_t)tokens;
        a.terms = terms;
        a.xt = (const uint8_t *)xt;
        a.xscale = (const float *)xs;
        a.ws = (float *)ws;
        a.status = (uint32_t *)st;
        const uint64_t units = (uint64_t)tiles * tok_pairs * a.ksplit;
        e = atlas_launch_prefill_gemm(&a, 2 * (int)std::min<uint64_t>(units, (uint64_t)pairs), s);
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(&status, st, 4, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) rc = fail(nullptr, ATLAS_ECUDA, "gemm: %s", cudaGetErrorString(e));
    else if (status != kStatusOk) rc = fail(nullptr, ATLAS_ETIMEOUT, "gemm: device status %u", status);
    cudaFree(xt);
    cudaFree(xs);
    cudaFree(ws);
    cudaFree(st);
    return rc;
}

// ---------------------------------------------------------------------------
// A GEMV entry point that allocates nothing
// ---------------------------------------------------------------------------
//
// For callers that cannot allocate device memory: a host that reserves all of
// HBM up front for weights and KV cache and hands plugins no allocator, or a
// path with a latency budget that cannot absorb cudaMalloc's implicit device
// synchronisation. atlas_cuda_gemv needs no scratch at all; this variant runs
// the persistent decode kernel (decode.cu) on one GEMV phase, and that kernel
// needs launch scratch - its phase descriptor, its phase counters and its step
// state. Here that scratch is a fixed 4 KB array of this module's static
// device memory, which every GPU that loads the library holds until the
// process exits.
#include <mutex>

namespace {

constexpr size_t kNoAllocScratchBytes = 4096;
__device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

constexpr size_t kNoAllocPhaseOff = 0;
constexpr size_t kNoAllocCtrOff = (sizeof(Phase) + 255) & ~size_t(255);
constexpr size_t kNoAllocStateOff = kNoAllocCtrOff + 256;
constexpr size_t kNoAllocNeeded = kNoAllocStateOff + sizeof(StepState);
static_assert(kNoAllocNeeded <= kNoAllocScratchBytes, "no-alloc scratch too small for the launch descriptor");
static_assert(sizeof(Phase) % 4 == 0 && kNoAllocNeeded % 4 == 0, "no-alloc scratch is written in words");

std::mutex g_noalloc_mu;
uint8_t *g_noalloc_ptr[64];  // device address of g_noalloc_scratch, per device

// Writes the phase descriptor (passed by value in the launch parameters, so
// no host memory is involved) into the scratch and zeroes the phase counters
// and the step state, which keep the previous call's values otherwise.
__global__ void noalloc_setup_kernel(const __grid_constant__ Phase ph, uint32_t *scratch)
{
    const uint32_t *src = reinterpret_cast<const uint32_t *>(&ph);
    for (uint32_t i = threadIdx.x; i < (uint32_t)(kNoAllocNeeded / 4); i += blockDim.x) {
        uint32_t v = 0u;
        if (i < (uint32_t)(sizeof(Phase) / 4)) v = src[i];
        else if (i < (uint32_t)(kNoAllocCtrOff / 4)) continue;
        scratch[i] = v;
    }
}

}  // namespace

extern "C" int atlas_cuda_gemv_noalloc(uint32_t type, const void *d_weights, uint64_t rows, uint64_t cols,
                                       const float *d_x, float *d_y, void *stream)
{
    if ((type != ATLAS_TYPE_Q4_K && type != ATLAS_TYPE_Q6_K) || !d_weights || !d_x || !d_y || !rows || !cols ||
        cols % 256 || rows > 0xffffffffu)
        return fail(nullptr, ATLAS_EINVAL, "bad gemv arguments");
    if (type == ATLAS_TYPE_Q4_K && ((uintptr_t)d_weights & 15u))
        return fail(nullptr, ATLAS_EINVAL, "Q4_K weights must be 16-byte aligned");
    if ((uintptr_t)d_weights & 1u) return fail(nullptr, ATLAS_EINVAL, "weights must be 2-byte aligned");
    if (((uintptr_t)d_x & 15u) || ((uintptr_t)d_y & 3u))
        return fail(nullptr, ATLAS_EINVAL, "x must be 16-byte aligned and y 4-byte aligned");
    int dev = 0;
    cudaGetDevice(&dev);
    int sms = 0;
    if (dev < 0 || dev >= 64 || device_ok(dev, &sms) != ATLAS_OK) return fail(nullptr, ATLAS_ENODEV, "no sm_100 device");
    uint32_t n_stages = 0, stage_bytes = 0;
    if (plan_smem(dev, (uint32_t)cols, n_stages, stage_bytes) != ATLAS_OK)
        return fail(nullptr, ATLAS_EINVAL,
                     "input length %llu exceeds the largest this kernel stages in shared memory",
                     (unsigned long long)cols);
    uint8_t *scratch = nullptr;
    {
        // Set-up, once per device, with that device current: the scratch's
        // device address (the symbol itself is only a host-side stand-in).
        std::lock_guard<std::mutex> lk(g_noalloc_mu);
        if (!g_noalloc_ptr[dev]) {
            void *p = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
            if (e != cudaSuccess || !p)
                return fail(nullptr, ATLAS_ECUDA, "cudaGetSymbolAddress(no-alloc scratch): %s", cudaGetErrorString(e));
            g_noalloc_ptr[dev] = static_cast<uint8_t *>(p);
        }
        scratch = g_noalloc_ptr[dev];
    }
    Phase ph = gemv_phase((uint32_t)cols, (uint32_t)sms, stage_bytes, false,
                          {seg_of((const uint8_t *)d_weights, type, (uint32_t)rows, (uint32_t)cols, nullptr, d_y)},
                          d_x, IN_RAW, nullptr, EPI_STORE);
    Program pg{};
    pg.phases = reinterpret_cast<const Phase *>(scratch + kNoAllocPhaseOff);
    pg.n_phases = 1;
    pg.phase_ctr = reinterpret_cast<uint32_t *>(scratch + kNoAllocCtrOff);
    pg.state = reinterpret_cast<StepState *>(scratch + kNoAllocStateOff);
    pg.n_stages = n_stages;
    pg.stage_bytes = stage_bytes;
    pg.max_cols = (uint32_t)cols;
    cudaStream_t s = (cudaStream_t)stream;
    noalloc_setup_kernel<<<1, 256, 0, s>>>(ph, reinterpret_cast<uint32_t *>(scratch));
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = atlas_launch_decode(&pg, sms, s);
    if (e != cudaSuccess) return fail(nullptr, ATLAS_ECUDA, "gemv (no-alloc) launch: %s", cudaGetErrorString(e));
    // The kernel's bounded waits record a status word in the scratch's step
    // state instead of hanging; read it back (into host stack memory, nothing
    // is allocated), so a timed-out wait is reported rather than a partial y.
    uint32_t st = 0;
    e = cudaMemcpyAsync(&st, scratch + kNoAllocStateOff + offsetof(StepState, status), sizeof(st),
                        cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return fail(nullptr, ATLAS_ECUDA, "gemv (no-alloc): %s", cudaGetErrorString(e));
    return status_to_code(nullptr, st);
}
