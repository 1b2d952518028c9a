// Streaming dequant-GEMV for the decode step (sm_100a), fp32 FMAs on CUDA
// cores: src/brain_runtime.c:1133-1185 (matvec_rows) with the block decoders
// of :960-1083 fused in.
//
// A CTA owns `rows_per_cta` consecutive output rows. It stages x (optionally
// rms_norm'ed exactly as the reference: double sum of squares, x * inv * w)
// in shared memory together with the sum of x over every 32-value group. Each
// warp takes one row at a time (for SwiGLU, the gate row then the up row of
// one output row); each lane takes the row's 64-value chunks ch = lane,
// lane + 32, ... (chunk kq of block ch / 4):
//   Q4_K: dot = (d*sc_2kq) sum q_lo*x - (dmin*m_2kq) sum x
//             + (d*sc_2kq+1) sum q_hi*x - (dmin*m_2kq+1) sum x
//   Q6_K: dot = sum over the four 16-value groups of (d*sc_g) sum (q-32)*x
// with the integer quants turned into floats exactly (byte -> 2^23 + q ->
// minus 2^23) and the products summed with packed fp32 FMAs (FFMA2), x read
// from shared memory as float4. The lane sums are reduced with shuffles.
//
// The raw bytes of a lane's next chunk are loaded before the current one is
// converted (two register buffers), and many small CTAs keep each SM's loads
// in flight. Launched with programmatic dependent launch, a kernel first pulls
// its weight rows towards L2 (they do not depend on the preceding kernel),
// then waits for the preceding kernel before reading x.
#include <cfloat>
#include <cmath>
#include <type_traits>
#include "common.cuh"
#include "quant.cuh"
#include "gemv.h"

namespace atlas {
namespace gv {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ void prefetch_l2(const void *p, uint32_t bytes)
{
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// floats of bytes k0, k0+1 of v (values < 256): 2^23 + q assembled bitwise,
// minus `bias` (2^23, or 2^23 + 32 for Q6_K's q - 32); exact.
__device__ __forceinline__ float2 bytes_f(uint32_t v, int k0, float bias)
{
    const float a = __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7440u | (uint32_t)k0));
    const float b = __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7440u | (uint32_t)(k0 + 1)));
    return __ffma2_rn(make_float2(a, b), make_float2(1.0f, 1.0f), make_float2(-bias, -bias));
}

// acc += q * x for the 4 bytes of w (4 quants) against x values xv.
__device__ __forceinline__ float2 dot4(uint32_t w, float4 xv, float bias, float2 acc)
{
    acc = __ffma2_rn(bytes_f(w, 0, bias), make_float2(xv.x, xv.y), acc);
    acc = __ffma2_rn(bytes_f(w, 2, bias), make_float2(xv.z, xv.w), acc);
    return acc;
}

// x is staged in shared memory with 4 floats of padding after every 64 (a
// lane reads its own 64-value chunk, so the lane stride becomes 272 bytes and
// a warp's float4 reads hit distinct banks).
__device__ __forceinline__ uint32_t xpad(uint32_t k) { return k + 4u * (k >> 6); }

// ---------------------------------------------------------------- Q4_K ----

struct RawQ4 {
    uint4 h, q0, q1;
};

__device__ __forceinline__ void load_q4(const uint8_t *row, uint32_t ch, RawQ4 &r)
{
    const uint8_t *blk = row + (size_t)(ch >> 2) * 144u;
    const uint32_t kq = ch & 3u;   // 64-value chunk: 32 quant bytes at 16 + 32kq
    r.h = __ldg(reinterpret_cast<const uint4 *>(blk));
    r.q0 = __ldg(reinterpret_cast<const uint4 *>(blk + 16 + 32 * kq));
    r.q1 = __ldg(reinterpret_cast<const uint4 *>(blk + 32 + 32 * kq));
}

// get_scale_min_k4 (src/brain_runtime.c:939-958) for sub-block j from the
// header words y (scale bytes 0-3), z (4-7), w (8-11).
__device__ __forceinline__ void k4_sm(uint32_t j, const uint4 &h, float d, float dmin, float &a, float &b)
{
    const uint32_t t = (j & 3u) * 8u;
    const uint32_t y = (h.y >> t) & 255u, z = (h.z >> t) & 255u, w = (h.w >> t) & 255u;
    const bool low = j < 4u;
    const uint32_t sc = low ? (y & 63u) : ((w & 15u) | ((y >> 6) << 4));
    const uint32_t mn = low ? (z & 63u) : ((w >> 4) | ((z >> 6) << 4));
    a = __fmul_rn(d, (float)sc);
    b = __fmul_rn(dmin, (float)mn);
}

__device__ __forceinline__ float dot_q4(const RawQ4 &r, uint32_t ch, const float *xs, const float *gs)
{
    const uint32_t kq = ch & 3u, base = (ch >> 2) * 256u + 64u * kq;
    const float4 *xl = reinterpret_cast<const float4 *>(xs + xpad(base));         // values 0..31: low nibbles
    const float4 *xh = reinterpret_cast<const float4 *>(xs + xpad(base) + 32u);   // values 32..63: high nibbles
    const uint32_t q[8] = {r.q0.x, r.q0.y, r.q0.z, r.q0.w, r.q1.x, r.q1.y, r.q1.z, r.q1.w};
    float2 al = make_float2(0.f, 0.f), ah = make_float2(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        al = dot4(q[i] & 0x0f0f0f0fu, xl[i], 8388608.0f, al);
        ah = dot4((q[i] >> 4) & 0x0f0f0f0fu, xh[i], 8388608.0f, ah);
    }
    const float d = h2f((uint16_t)(r.h.x & 0xffffu)), dmin = h2f((uint16_t)(r.h.x >> 16));
    float a0, b0, a1, b1;
    k4_sm(2u * kq, r.h, d, dmin, a0, b0);
    k4_sm(2u * kq + 1u, r.h, d, dmin, a1, b1);
    const float s0 = al.x + al.y, s1 = ah.x + ah.y;
    const float g0 = gs[base / 32u], g1 = gs[base / 32u + 1u];
    return fmaf(a0, s0, -b0 * g0) + fmaf(a1, s1, -b1 * g1);
}

// ---------------------------------------------------------------- Q6_K ----

struct RawQ6 {
    uint32_t ql[17], qh[9];
    uint32_t sc;   // the chunk's four int8 scales
    uint32_t dsh;  // d (low 16 bits), funnel shift of the words (bits 16..)
};

// chunk kq of block ch / 4 (values 64kq + 0..63) = runs j = 2(kq & 1) + hb of
// half n = kq / 2: ql[64n + 32hb + l] (nibble kq & 1), qh[32n + l] (bits 2j),
// scales [8n + 4(kq & 1) + 2hb + l / 16], d. Blocks are 2-byte aligned: the
// bytes are read as aligned words and realigned with funnel shifts.
__device__ __forceinline__ void load_q6(const uint8_t *row, uint32_t ch, RawQ6 &r)
{
    const uint8_t *blk = row + (size_t)(ch >> 2) * 210u;
    const uint32_t kq = ch & 3u, n = kq >> 1;
    const uintptr_t b = reinterpret_cast<uintptr_t>(blk);
    const uint32_t sh = (uint32_t)(b & 2u) * 8u;
    const uint32_t *ql = reinterpret_cast<const uint32_t *>((b + 64 * n) & ~(uintptr_t)3);
    const uint32_t *qh = reinterpret_cast<const uint32_t *>((b + 128 + 32 * n) & ~(uintptr_t)3);
#pragma unroll
    for (int i = 0; i < 16; ++i) r.ql[i] = __ldg(ql + i);
#pragma unroll
    for (int i = 0; i < 8; ++i) r.qh[i] = __ldg(qh + i);
    r.ql[16] = sh ? __ldg(ql + 16) : 0u;
    r.qh[8] = sh ? __ldg(qh + 8) : 0u;
    const unsigned short *sc = reinterpret_cast<const unsigned short *>(blk + 192 + 8 * n + 4 * (kq & 1u));
    r.sc = (uint32_t)__ldg(sc) | ((uint32_t)__ldg(sc + 1) << 16);
    r.dsh = (uint32_t)__ldg(reinterpret_cast<const unsigned short *>(blk + 208)) | (sh << 16);
}

__device__ __forceinline__ float dot_q6(const RawQ6 &r, uint32_t ch, const float *xs)
{
    const uint32_t kq = ch & 3u, sh = r.dsh >> 16, s4 = 4u * (kq & 1u);
    const float4 *xv = reinterpret_cast<const float4 *>(xs + xpad((ch >> 2) * 256u + 64u * kq));
    float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
    for (int hb = 0; hb < 2; ++hb) {
        const uint32_t s2 = s4 + 2u * (uint32_t)hb;
#pragma unroll
        for (int i = 0; i < 8; ++i) {   // values 32hb + 4i .. +3
            const int wl = 8 * hb + i;
            const uint32_t lw = __funnelshift_r(r.ql[wl], r.ql[wl + 1], sh);
            const uint32_t hw = __funnelshift_r(r.qh[i], r.qh[i + 1], sh);
            const uint32_t q = ((lw >> s4) & 0x0f0f0f0fu) | (((hw >> s2) & 0x03030303u) << 4);
            acc[2 * hb + (i >> 2)] = dot4(q, xv[8 * hb + i], 8388640.0f, acc[2 * hb + (i >> 2)]);   // q - 32
        }
    }
    const float d = h2f((uint16_t)(r.dsh & 0xffffu));
    float sum = 0.f;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
        const float a = __fmul_rn(d, (float)(int)(int8_t)(r.sc >> (8 * g)));
        sum = fmaf(a, acc[g].x + acc[g].y, sum);
    }
    return sum;
}

// ------------------------------------------------------------ row tasks ----

// Dot products of a warp's row tasks, lane by lane over 64-value chunks, the
// next chunk's bytes loaded while the current one converts. `row_of(k)`
// gives the k-th row task's row pointer (null: no such task); `done(k, v)`
// receives the warp-reduced dot of task k in every lane.
template <uint32_t TYPE, typename RowOf, typename Done>
__device__ __forceinline__ void run_tasks(uint32_t ntasks, uint32_t nch, uint32_t lane, const float *xs,
                                          const float *gs, RowOf row_of, Done done)
{
    using Raw = typename std::conditional<TYPE == 12u, RawQ4, RawQ6>::type;
    // every lane walks the same items (shuffles line up); chunks past the row end are skipped
    const uint32_t my = (nch + 31u) / 32u;   // chunk items per row
    const uint32_t total = ntasks * my;
    auto load = [&](uint32_t k, Raw &r) {
        const uint32_t ch = lane + 32u * (k % my);
        if (ch >= nch) return;
        const uint8_t *row = row_of(k / my);
        if constexpr (TYPE == 12u) load_q4(row, ch, r);
        else load_q6(row, ch, r);
    };
    auto dot = [&](uint32_t k, const Raw &r) -> float {
        const uint32_t ch = lane + 32u * (k % my);
        if (ch >= nch) return 0.f;
        if constexpr (TYPE == 12u) return dot_q4(r, ch, xs, gs);
        else return dot_q6(r, ch, xs);
    };
    Raw ra, rb;
    float acc = 0.f;
    uint32_t task = 0;
    auto finish_task = [&]() {
        float v = acc;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        done(task, v);
        acc = 0.f;
        ++task;
    };
    if (total) load(0, ra);
    for (uint32_t k = 0; k < total; k += 2) {
        if (k + 1 < total) load(k + 1, rb);
        acc += dot(k, ra);
        if ((k + 1) % my == 0) finish_task();
        if (k + 1 >= total) break;
        if (k + 2 < total) load(k + 2, ra);
        acc += dot(k + 1, rb);
        if ((k + 2) % my == 0) finish_task();
    }
}

__device__ __forceinline__ uint32_t seg_of_row(const GemvArgs &a, uint32_t r)
{
    uint32_t s = 0;
    while (s + 1 < a.n_seg && r >= a.seg_start[s + 1]) ++s;
    return s;
}

__global__ void __launch_bounds__(kThreads) gemv_kernel(const __grid_constant__ GemvArgs a)
{
    extern __shared__ float smem_f[];
    __shared__ double dred[kWarps];
    __shared__ float amax_s[kWarps];
    __shared__ uint32_t aidx_s[kWarps];
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const bool paired = a.epi == GV_SWIGLU;
    const uint32_t r0 = blockIdx.x * a.rows_per_cta;
    const uint32_t r1 = min(r0 + a.rows_per_cta, a.total_rows);
    const uint32_t nch = a.cols / 64u;

    // weights do not depend on the preceding kernel: while waiting for it,
    // pull the first two rows of every warp towards L2 (more would only queue
    // ahead of the demand loads)
    if (a.pdl && threadIdx.x < 2u * kWarps) {
        const uint32_t r = r0 + threadIdx.x;
        if (r < r1) {
            const uint32_t sgi = paired ? 0u : seg_of_row(a, r);
            const GemvSeg &sg = a.seg[sgi];
            const uint32_t lr = paired ? r : r - a.seg_start[sgi];
            for (uint32_t k = 0; k < (paired ? 2u : 1u); ++k) {
                const GemvSeg &s2 = a.seg[paired ? k : sgi];
                const uintptr_t b0 = reinterpret_cast<uintptr_t>(s2.w + (size_t)lr * s2.row_bytes);
                const uintptr_t s = b0 & ~(uintptr_t)15, e = (b0 + s2.row_bytes) & ~(uintptr_t)15;
                if (e > s) prefetch_l2(reinterpret_cast<const void *>(s), (uint32_t)(e - s));
            }
            (void)sg;
        }
    }
    if (a.pdl) pdl_wait();

    // stage x (rms_norm'ed when norm_w is set) and its 32-value group sums
    float *xs = smem_f, *gs = smem_f + a.cols + a.cols / 16u;
    float inv = 1.0f;
    if (a.norm_w) {
        double ss = 0.0;
        for (uint32_t i = threadIdx.x; i < a.cols / 4u; i += kThreads) {
            const float4 v = __ldcg(reinterpret_cast<const float4 *>(a.x) + i);
            ss += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) dred[warp] = ss;
        __syncthreads();
        double tot = 0.0;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) tot += dred[w];
        inv = 1.0f / sqrtf((float)(tot / (double)a.cols) + a.eps);   // src/brain_runtime.c:1355-1360
    }
    for (uint32_t g = threadIdx.x; g < a.cols / 32u; g += kThreads) {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float4 v = __ldcg(reinterpret_cast<const float4 *>(a.x + 32u * g) + i);
            if (a.norm_w) {
                const float4 wn = __ldg(reinterpret_cast<const float4 *>(a.norm_w + 32u * g) + i);
                v.x = __fmul_rn(__fmul_rn(v.x, inv), wn.x);
                v.y = __fmul_rn(__fmul_rn(v.y, inv), wn.y);
                v.z = __fmul_rn(__fmul_rn(v.z, inv), wn.z);
                v.w = __fmul_rn(__fmul_rn(v.w, inv), wn.w);
            }
            *reinterpret_cast<float4 *>(xs + xpad(32u * g + 4u * (uint32_t)i)) = v;
            s += (v.x + v.y) + (v.z + v.w);
        }
        gs[g] = s;
    }
    __syncthreads();

    // row tasks of this warp: rows r0 + warp, r0 + warp + 8, ... (SwiGLU: the
    // gate and the up row of each such output row, one after the other)
    const uint32_t nout = r1 > r0 + warp ? (r1 - r0 - warp + kWarps - 1u) / kWarps : 0u;
    float best = -FLT_MAX;
    uint32_t best_i = 0xffffffffu;
    if (paired) {
        float gate = 0.f;
        auto row_of = [&](uint32_t k) {
            const GemvSeg &sg = a.seg[k & 1u];
            return sg.w + (size_t)(r0 + warp + kWarps * (k >> 1)) * sg.row_bytes;
        };
        auto done = [&](uint32_t k, float v) {
            if (!(k & 1u)) { gate = v; return; }
            if (lane == 0)
                a.seg[0].out[r0 + warp + kWarps * (k >> 1)] = (gate / (1.0f + expf(-gate))) * v;   // src/brain_runtime.c:1755-1758
        };
        if (a.seg[0].type == 12u) run_tasks<12u>(2u * nout, nch, lane, xs, gs, row_of, done);
        else run_tasks<14u>(2u * nout, nch, lane, xs, gs, row_of, done);
    } else {
        // the rows of one warp may span segments of different types: one run per segment
        uint32_t k0 = 0;
        while (k0 < nout) {
            const uint32_t row0 = r0 + warp + kWarps * k0, sgi = seg_of_row(a, row0);
            const GemvSeg &sg = a.seg[sgi];
            const uint32_t end = a.seg_start[sgi + 1];
            uint32_t n = 0;
            while (k0 + n < nout && r0 + warp + kWarps * (k0 + n) < end) ++n;
            auto row_of = [&](uint32_t k) {
                return sg.w + (size_t)(row0 + kWarps * k - a.seg_start[sgi]) * sg.row_bytes;
            };
            auto done = [&](uint32_t k, float v) {
                if (lane != 0) return;
                const uint32_t lr = row0 + kWarps * k - a.seg_start[sgi];
                if (a.epi == GV_RESID) {
                    sg.out[lr] = __ldcg(sg.out + lr) + v;   // src/brain_runtime.c:1745, :1762
                } else {
                    sg.out[lr] = sg.bias ? v + __ldg(sg.bias + lr) : v;
                    if (a.epi == GV_LOGITS && (v > best || (v == best && lr < best_i))) { best = v; best_i = lr; }
                }
            };
            if (sg.type == 12u) run_tasks<12u>(n, nch, lane, xs, gs, row_of, done);
            else run_tasks<14u>(n, nch, lane, xs, gs, row_of, done);
            k0 += n;
        }
    }
    pdl_launch_dependents();
    if (a.epi == GV_LOGITS) {
        if (lane == 0) { amax_s[warp] = best; aidx_s[warp] = best_i; }
        __syncthreads();
        if (threadIdx.x == 0) {
            for (int w = 1; w < kWarps; ++w)
                if (amax_s[w] > best || (amax_s[w] == best && aidx_s[w] < best_i)) { best = amax_s[w]; best_i = aidx_s[w]; }
            a.pmax[blockIdx.x] = best;
            a.pidx[blockIdx.x] = best_i;
        }
    }
}

}  // namespace gv
}  // namespace atlas

using namespace atlas::gv;

extern "C" size_t atlas_gemv2_smem(uint32_t cols) { return ((size_t)cols + cols / 16u + cols / 32u) * 4u; }

extern "C" cudaError_t atlas_launch_gemv2(const GemvArgs *a, cudaStream_t stream)
{
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    const size_t smem = atlas_gemv2_smem(a->cols);
    if (smem > 200u * 1024u) return cudaErrorInvalidValue;
    const uint32_t grid = (a->total_rows + a->rows_per_cta - 1) / a->rows_per_cta;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = a->pdl ? 1 : 0;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gemv_kernel, *a);
}
