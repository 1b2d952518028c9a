// Batched prefill kernels (sm_100a): the dense contraction on tcgen05 tensor
// cores with Q4_K / Q6_K weights dequantized into shared memory, the
// activation split/tiling pass that feeds it, the embedding gather and the
// causal GQA attention over the KV cache.
//
// Contraction kernel, one CTA per SM, persistent over work units
// (row tile, token tile, K range):
//   warp 0      bulk-copies the pre-split activation tile of each 64-wide
//               K block (hi + lo binary16, already in the 128-byte swizzled
//               K-major layout) into the stage ring;
//   warps 6-13  dequantize the matching 256 weight rows x 64 K values
//               straight from the raw super-blocks in global memory
//               (bit-exact with src/brain_runtime.c:960-1083), scale them by
//               2^wexp, split them into binary16 hi/lo and store them
//               swizzled next to the activations;
//   warp 1      allocates 512 TMEM columns (two 128 x 256 fp32 accumulators)
//               and, from one thread, issues tcgen05.mma kind::f16
//               (M = 128 tokens, N = 256 rows, K = 16) for every product
//               term, committing each consumed stage back to the ring and the
//               finished accumulator to the epilogue;
//   warps 2-5   read the accumulator with tcgen05.ld (lane = token), undo
//               the power-of-two scales and apply the fused epilogue: bias,
//               RoPE and the KV-cache store for Q/K/V, residual add for
//               O / down, SwiGLU for gate+up. With split-K each unit stores
//               its partial tile and the last unit of a tile to arrive sums
//               the partials in K order and applies the epilogue.
// Every wait is bounded (2 s of globaltimer); on a timeout the CTA records a
// status, drains its outstanding copies and MMAs, frees its TMEM and exits.
#include <cfloat>
#include <cmath>
#include "common.cuh"
#include "quant.cuh"
#include "prefill.h"

namespace atlas {
namespace pf {

// ------------------------------------------------------- tcgen05 wrappers --

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t ncols)
{
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)), "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols)
{
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[tmem] (+)= A[smem] . B[smem]^T, both operands K-major binary16.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accum)
{
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
        ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum)
        : "memory");
}

// Arrive on `bar` once every tcgen05 operation this thread issued so far is done.
__device__ __forceinline__ void umma_commit(uint64_t *bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory operand descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (stride byte offset), leading byte offset 16 (unused by
// this layout), descriptor version 1, base offset 0 (1024-byte aligned tiles).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr)
{
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)(1024u >> 4) << 32) |
           ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}

// Instruction descriptor: fp32 accumulator, A = B = binary16, both K-major,
// N = 256, M = 128.
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(kRowTile >> 3) << 17) | ((uint32_t)(kTokTile >> 4) << 24);

// Byte offset of 16-byte chunk `chunk` (K elements 8*chunk..8*chunk+7) of
// operand row `row` in a 128-byte-swizzled K-major tile.
__host__ __device__ constexpr uint32_t sw128_off(uint32_t row, uint32_t chunk)
{
    return (row >> 3) * 1024u + (row & 7u) * 128u + ((chunk ^ (row & 7u)) << 4);
}

// --------------------------------------------------------- shared layout --

struct Bars {
    uint64_t xfull[kStages];   // activation copy landed (tx count)
    uint64_t wfull[kStages];   // 8 dequant warps stored their weight rows
    uint64_t empty[kStages];   // the MMAs reading the stage completed
    uint64_t acc_full[2];      // accumulator complete
    uint64_t acc_empty[2];     // epilogue done reading the accumulator
    uint64_t fin;              // teardown: all MMAs of this CTA completed
    uint32_t tmem;
    uint32_t status;
    uint32_t flag;
};

constexpr size_t kGemmSmem = (size_t)kStages * kStageBytes + 1024 + sizeof(Bars);

struct Unit {
    uint32_t tile, tt, ks, kb0, kb1;
};

__device__ __forceinline__ Unit unit_of(const GemmArgs &a, uint32_t u)
{
    Unit x;
    x.ks = u % a.ksplit;
    const uint32_t r = u / a.ksplit;
    x.tt = r % a.tok_tiles;
    x.tile = r / a.tok_tiles;
    x.kb0 = (uint32_t)((uint64_t)a.kblocks * x.ks / a.ksplit);
    x.kb1 = (uint32_t)((uint64_t)a.kblocks * (x.ks + 1) / a.ksplit);
    return x;
}

__device__ __forceinline__ uint32_t seg_of_tile(const GemmArgs &a, uint32_t tile)
{
    uint32_t s = 0;
    while (s + 1 < a.n_seg && tile >= a.seg[s + 1].tile0) ++s;
    return s;
}

// Teardown wait: bounded, ignores the error word (used to let in-flight copies
// and MMAs finish before the CTA frees its resources).
__device__ __forceinline__ bool mbar_drain(uint64_t *bar, uint32_t parity)
{
    const uint64_t t0 = global_ns();
    while (!mbar_try_wait(bar, parity))
        if (global_ns() - t0 > kWaitLimitNs) return false;
    return true;
}

// Warp-uniform bounded wait: every lane polls, the warp agrees on the outcome.
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity, volatile uint32_t *err)
{
    const bool ok = mbar_wait(bar, parity, err);
    return __all_sync(0xffffffffu, ok);
}

// -------------------------------------------------------------- dequant ----

// Float 2^23 + b for a byte b of v (k = byte index): exact small-integer
// conversion without I2F.
__device__ __forceinline__ float byte_f23(uint32_t v, int k)
{
    return __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7440u | (uint32_t)k));
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b)
{
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// Store 8 scaled weights as binary16 hi (and lo) at a swizzled chunk.
template <int TERMS>
__device__ __forceinline__ void store_chunk(uint8_t *bhi, uint32_t off, const float (&w)[8])
{
    uint4 hi;
    hi.x = pack_h2(w[0], w[1]);
    hi.y = pack_h2(w[2], w[3]);
    hi.z = pack_h2(w[4], w[5]);
    hi.w = pack_h2(w[6], w[7]);
    *reinterpret_cast<uint4 *>(bhi + off) = hi;
    if (TERMS >= 3) {
        const uint32_t h[4] = {hi.x, hi.y, hi.z, hi.w};
        uint32_t l[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&h[i]));
            l[i] = pack_h2(w[2 * i] - f.x, w[2 * i + 1] - f.y);
        }
        *reinterpret_cast<uint4 *>(bhi + kBTermBytes + off) = make_uint4(l[0], l[1], l[2], l[3]);
    }
}

// Raw bytes one dequant thread needs for one K block of one row.
struct Raw {
    uint32_t w[28];
    uint32_t sh;   // Q6_K: funnel shift (0 or 16) of the 4-byte aligned words
};

__device__ __forceinline__ void load_raw(uint32_t type, const uint8_t *blk, uint32_t kq, Raw &r)
{
    if (type == 12u) {
        // header (d, dmin, 12 scale bytes) + 32 quant bytes of chunk kq; 16-byte aligned
        const uint4 h = __ldg(reinterpret_cast<const uint4 *>(blk));
        const uint4 q0 = __ldg(reinterpret_cast<const uint4 *>(blk + 16 + 32 * kq));
        const uint4 q1 = __ldg(reinterpret_cast<const uint4 *>(blk + 32 + 32 * kq));
        r.w[0] = h.x; r.w[1] = h.y; r.w[2] = h.z; r.w[3] = h.w;
        r.w[4] = q0.x; r.w[5] = q0.y; r.w[6] = q0.z; r.w[7] = q0.w;
        r.w[8] = q1.x; r.w[9] = q1.y; r.w[10] = q1.z; r.w[11] = q1.w;
    } else {
        // Q6_K (2-byte aligned blocks): ql[64n .. 64n+63], qh[32n .. 32n+31],
        // scales[8n + 4(kq&1) .. +3], d, with n = kq / 2
        const uint32_t n = kq >> 1;
        const uintptr_t b = reinterpret_cast<uintptr_t>(blk);
        r.sh = (uint32_t)(b & 2u) * 8u;
        const uint32_t extra = r.sh ? 1u : 0u;
        const uint32_t *ql = reinterpret_cast<const uint32_t *>((b + 64 * n) & ~(uintptr_t)3);
        const uint32_t *qh = reinterpret_cast<const uint32_t *>((b + 128 + 32 * n) & ~(uintptr_t)3);
#pragma unroll
        for (int i = 0; i < 16; ++i) r.w[i] = __ldg(ql + i);
        r.w[16] = extra ? __ldg(ql + 16) : 0u;
#pragma unroll
        for (int i = 0; i < 8; ++i) r.w[17 + i] = __ldg(qh + i);
        r.w[25] = extra ? __ldg(qh + 8) : 0u;
        const unsigned short *sc = reinterpret_cast<const unsigned short *>(blk + 192 + 8 * n + 4 * (kq & 1));
        r.w[26] = (uint32_t)__ldg(sc) | ((uint32_t)__ldg(sc + 1) << 16);
        r.w[27] = (uint32_t)__ldg(reinterpret_cast<const unsigned short *>(blk + 208));
    }
}

// Dequantize the 64 values of one K block held in `r` (chunk kq of the
// super-block), scaled by p2 = 2^wexp, into swizzled row `row` of the tile.
template <int TERMS>
__device__ __forceinline__ void dequant_kblock(uint32_t type, const Raw &r, uint32_t kq, float p2, uint8_t *bhi,
                                               uint32_t row)
{
    if (type == 12u) {
        // src/brain_runtime.c:960-1015: y = (d*sc) * q - dmin*m per 32-value sub-block
        const float d = h2f((uint16_t)(r.w[0] & 0xffffu)), dmin = h2f((uint16_t)(r.w[0] >> 16));
        uint8_t scb[12];
#pragma unroll
        for (int i = 0; i < 12; ++i) scb[i] = (uint8_t)(r.w[1 + i / 4] >> (8 * (i % 4)));
        float a[2], bm[2];
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
            uint32_t sc, mn;
            k4_scale_min(2 * (int)kq + hf, scb, sc, mn);
            a[hf] = __fmul_rn(__fmul_rn(d, (float)sc), p2);      // exact: 2^wexp scaling
            bm[hf] = __fmul_rn(__fmul_rn(dmin, (float)mn), p2);
        }
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const int hf = c >> 2, wi = 4 + 2 * (c & 3);
            float w[8];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint32_t v = (r.w[wi + h] >> (4 * hf)) & 0x0f0f0f0fu;
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float q = byte_f23(v, k) - 8388608.0f;
                    w[4 * h + k] = fmaf(a[hf], q, -bm[hf]);   // == fl(fl(a*q) - b): a*q is exact
                }
            }
            store_chunk<TERMS>(bhi, sw128_off(row, (uint32_t)c), w);
        }
    } else {
        // src/brain_runtime.c:1049-1083: y = (d * sc) * (q - 32)
        const float d = h2f((uint16_t)r.w[27]);
        const uint32_t s4 = 4u * (kq & 1u);
        float ds[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
            ds[i] = __fmul_rn(__fmul_rn(d, (float)(int)(int8_t)(r.w[26] >> (8 * i))), p2);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const int hb = c >> 2, l8 = 2 * (c & 3);
            const uint32_t s2 = s4 + 2u * (uint32_t)hb;
            float w[8];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int qi = 8 * hb + l8 + h, hi = l8 + h;
                const uint32_t lw = __funnelshift_r(r.w[qi], r.w[qi + 1], r.sh);
                const uint32_t hw = __funnelshift_r(r.w[17 + hi], r.w[18 + hi], r.sh);
                const uint32_t q = ((lw >> s4) & 0x0f0f0f0fu) | (((hw >> s2) & 0x03030303u) << 4);
                const float sc = ds[2 * hb + ((c & 3) >> 1)];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float qf = byte_f23(q, k) - 8388640.0f;   // q - 32, exact
                    w[4 * h + k] = __fmul_rn(sc, qf);
                }
            }
            store_chunk<TERMS>(bhi, sw128_off(row, (uint32_t)c), w);
        }
    }
}

// ------------------------------------------------------------- epilogue ----

__device__ __forceinline__ float silu_mul(float z, float u)
{
    return (z / (1.0f + expf(-z))) * u;   // src/brain_runtime.c:1755-1758
}

// --------------------------------------------------------------- kernel ----

template <int TERMS>
__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ GemmArgs a)
{
    extern __shared__ uint8_t smem_raw[];
    const uint32_t base_addr = smem_addr(smem_raw);
    uint8_t *smem = smem_raw + (((base_addr + 1023u) & ~1023u) - base_addr);
    Bars *bars = reinterpret_cast<Bars *>(smem + (size_t)kStages * kStageBytes);
    volatile uint32_t *err = &bars->status;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t n_units = a.n_tiles * a.tok_tiles * a.ksplit;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&bars->xfull[s], 1);
            mbar_init(&bars->wfull[s], 8);
            mbar_init(&bars->empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bars->acc_full[b], 1);
            mbar_init(&bars->acc_empty[b], 4);
        }
        mbar_init(&bars->fin, 1);
        bars->status = kStatusOk;
        bars->flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(&bars->tmem, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem;

    if (warp == 0) {
        // ---------------------------------------------- activation copies --
        if (lane == 0) {
            const uint32_t xbytes = TERMS == 1 ? kATermBytes : 2 * kATermBytes;
            uint32_t it = 0;
            for (uint32_t u = blockIdx.x; u < n_units; u += gridDim.x) {
                const Unit un = unit_of(a, u);
                bool ok = true;
                for (uint32_t kb = un.kb0; kb < un.kb1; ++kb, ++it) {
                    const uint32_t s = it % kStages, ph = (it / kStages) & 1u;
                    if (!mbar_wait(&bars->empty[s], ph ^ 1u, err)) { ok = false; break; }
                    mbar_arrive_expect_tx(&bars->xfull[s], xbytes);
                    bulk_g2s(smem + (size_t)s * kStageBytes,
                             a.xt + ((size_t)un.tt * a.kblocks + kb) * kXTileBytes, xbytes, &bars->xfull[s]);
                }
                if (!ok) break;
            }
            // drain: every issued copy lands before the CTA may exit
            for (uint32_t i = 0; i < (uint32_t)kStages && i < it; ++i) {
                const uint32_t idx = it - 1 - i;
                mbar_drain(&bars->xfull[idx % kStages], (idx / kStages) & 1u);
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------- MMA issue --
        if (lane == 0) {
            uint32_t it = 0, lu = 0;
            for (uint32_t u = blockIdx.x; u < n_units; u += gridDim.x, ++lu) {
                const Unit un = unit_of(a, u);
                const uint32_t buf = lu & 1u, ap = (lu >> 1) & 1u;
                if (!mbar_wait(&bars->acc_empty[buf], ap ^ 1u, err)) break;
                tc_fence_after();
                const uint32_t d = tmem + buf * (uint32_t)kRowTile;
                bool ok = true;
                for (uint32_t kb = un.kb0; kb < un.kb1; ++kb, ++it) {
                    const uint32_t s = it % kStages, ph = (it / kStages) & 1u;
                    if (!mbar_wait(&bars->xfull[s], ph, err) || !mbar_wait(&bars->wfull[s], ph, err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t st = smem_addr(smem + (size_t)s * kStageBytes);
#pragma unroll
                    for (uint32_t k4 = 0; k4 < 4; ++k4) {
                        const uint64_t ah = sw128_desc(st + 32u * k4);
                        const uint64_t bh = sw128_desc(st + 2u * kATermBytes + 32u * k4);
                        umma_f16(d, ah, bh, kIdesc, (kb != un.kb0 || k4 != 0u) ? 1u : 0u);
                        if (TERMS >= 2) umma_f16(d, sw128_desc(st + kATermBytes + 32u * k4), bh, kIdesc, 1u);
                        if (TERMS >= 3)
                            umma_f16(d, ah, sw128_desc(st + 2u * kATermBytes + kBTermBytes + 32u * k4), kIdesc, 1u);
                    }
                    umma_commit(&bars->empty[s]);
                }
                if (!ok) break;
                umma_commit(&bars->acc_full[buf]);
            }
            // drain: all MMAs issued by this thread complete before TMEM is freed
            umma_commit(&bars->fin);
            mbar_drain(&bars->fin, 0);
        }
        __syncwarp();
    } else if (warp >= 6) {
        // ------------------------------------------------------ dequant --
        const uint32_t row = (warp - 6u) * 32u + lane;
        uint32_t it = 0;
        for (uint32_t u = blockIdx.x; u < n_units; u += gridDim.x) {
            const Unit un = unit_of(a, u);
            const GemmSeg *sg;
            uint32_t grow;
            if (a.epi == GEPI_SWIGLU) {
                sg = &a.seg[row >> 7];
                grow = un.tile * 128u + (row & 127u);
            } else {
                sg = &a.seg[seg_of_tile(a, un.tile)];
                grow = (un.tile - sg->tile0) * (uint32_t)kRowTile + row;
            }
            const bool valid = grow < sg->rows;
            const uint32_t type = sg->type;
            const float p2 = ldexpf(1.0f, sg->wexp);
            const uint8_t *wrow = sg->w + (size_t)(valid ? grow : 0u) * sg->row_bytes;
            const uint32_t bb = type == 12u ? 144u : 210u;
            bool ok = true;
            for (uint32_t kb = un.kb0; kb < un.kb1; ++kb, ++it) {
                const uint32_t s = it % kStages, ph = (it / kStages) & 1u;
                Raw r;
                if (valid) load_raw(type, wrow + (size_t)(kb >> 2) * bb, kb & 3u, r);
                if (!warp_wait(&bars->empty[s], ph ^ 1u, err)) { ok = false; break; }
                uint8_t *bhi = smem + (size_t)s * kStageBytes + 2u * kATermBytes;
                if (valid) {
                    dequant_kblock<TERMS>(type, r, kb & 3u, p2, bhi, row);
                } else {
#pragma unroll
                    for (uint32_t c = 0; c < 8; ++c) {
                        *reinterpret_cast<uint4 *>(bhi + sw128_off(row, c)) = make_uint4(0, 0, 0, 0);
                        if (TERMS >= 3)
                            *reinterpret_cast<uint4 *>(bhi + kBTermBytes + sw128_off(row, c)) = make_uint4(0, 0, 0, 0);
                    }
                }
                fence_proxy_async();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars->wfull[s]);
            }
            if (!ok) break;
        }
    } else {
        // ----------------------------------------------------- epilogue --
        // Each warp owns 32 token rows (its TMEM lane quarter) and handles them
        // independently, split-K arrivals included (one counter per quarter).
        const uint32_t quarter = warp & 3u, trow = quarter * 32u + lane;
        uint32_t lu = 0;
        for (uint32_t u = blockIdx.x; u < n_units; u += gridDim.x, ++lu) {
            const Unit un = unit_of(a, u);
            const uint32_t buf = lu & 1u, ap = (lu >> 1) & 1u;
            if (!warp_wait(&bars->acc_full[buf], ap, err)) break;
            tc_fence_after();
            const uint32_t tbase = tmem + ((quarter * 32u) << 16) + buf * (uint32_t)kRowTile;
            const uint32_t t = un.tt * (uint32_t)kTokTile + trow;
            const bool tvalid = t < a.tokens;
            const uint32_t tile_id = un.tile * a.tok_tiles + un.tt;
            bool reduce = false;
            if (a.ksplit > 1) {
                // store this K range's partial tile, then count arrivals
                float *dst = a.ws + ((size_t)(tile_id * a.ksplit + un.ks) * kTokTile + trow) * kRowTile;
                for (uint32_t c = 0; c < (uint32_t)kRowTile; c += 16) {
                    uint32_t r[16];
                    tmem_ld16(tbase + c, r);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; j += 4)
                        __stcg(reinterpret_cast<float4 *>(dst + c + j),
                               make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]), __uint_as_float(r[j + 2]),
                                           __uint_as_float(r[j + 3])));
                }
                tc_fence_before();
                __threadfence();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars->acc_empty[buf]);
                uint32_t last = 0;
                if (lane == 0) last = atom_acq_rel_add(a.ctr + tile_id * 4u + quarter, 1u) == a.ksplit - 1u ? 1u : 0u;
                last = __shfl_sync(0xffffffffu, last, 0);
                if (!last) continue;
                __threadfence();
                reduce = true;
            }
            // values of columns [c, c+16) of this thread's token row (accumulator scale)
            const float *wsrow = a.ws + ((size_t)tile_id * a.ksplit * kTokTile + trow) * kRowTile;
            auto fetch = [&](uint32_t c, float (&v)[16]) {
                if (!reduce) {
                    uint32_t r[16];
                    tmem_ld16(tbase + c, r);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = 0.f;
                    for (uint32_t k = 0; k < a.ksplit; ++k) {
                        const float4 *p = reinterpret_cast<const float4 *>(wsrow + (size_t)k * kTokTile * kRowTile + c);
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const float4 f = __ldcg(p + j);
                            v[4 * j] += f.x; v[4 * j + 1] += f.y; v[4 * j + 2] += f.z; v[4 * j + 3] += f.w;
                        }
                    }
                }
            };
            const float xs = tvalid ? __ldg(a.xscale + t) : 0.f;
            if (a.epi == GEPI_SWIGLU) {
                const GemmSeg &g = a.seg[0];
                const float sg = xs * ldexpf(1.0f, -g.wexp), su = xs * ldexpf(1.0f, -a.seg[1].wexp);
                for (uint32_t c = 0; c < 128u; c += 16) {
                    float vg[16], vu[16];
                    fetch(c, vg);
                    fetch(128u + c, vu);
                    const uint32_t r0 = un.tile * 128u + c;
                    if (tvalid) {
                        float *o = g.out + (size_t)(t + g.tok_off) * g.tok_stride;
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const uint32_t r = r0 + (uint32_t)j;
                            if (r < g.rows) o[(r >> 7) * g.head_stride + (r & 127u)] = silu_mul(vg[j] * sg, vu[j] * su);
                        }
                    }
                }
            } else {
                const GemmSeg &g = a.seg[seg_of_tile(a, un.tile)];
                const float s = xs * ldexpf(1.0f, -g.wexp);
                const uint32_t row0 = (un.tile - g.tile0) * (uint32_t)kRowTile;
                float *o = g.out + (size_t)(t + g.tok_off) * g.tok_stride;
                if (g.rope) {
                    const float2 *cs = reinterpret_cast<const float2 *>(a.rope) + (size_t)(a.pos0 + t) * 64u;
                    for (uint32_t hh = 0; hh < 2u; ++hh)
                        for (uint32_t c = 0; c < 64u; c += 16) {
                            float va[16], vb[16];
                            fetch(hh * 128u + c, va);
                            fetch(hh * 128u + 64u + c, vb);
                            if (tvalid) {
#pragma unroll
                                for (int j = 0; j < 16; ++j) {
                                    const uint32_t ra = row0 + hh * 128u + c + (uint32_t)j, rb = ra + 64u;
                                    if (rb >= g.rows) continue;
                                    float x0 = va[j] * s, x1 = vb[j] * s;
                                    if (g.bias) { x0 += __ldg(g.bias + ra); x1 += __ldg(g.bias + rb); }
                                    const float2 r = __ldg(cs + c + (uint32_t)j);   // src/brain_runtime.c:1391-1398
                                    const float y0 = __fsub_rn(__fmul_rn(x0, r.x), __fmul_rn(x1, r.y));
                                    const float y1 = __fadd_rn(__fmul_rn(x0, r.y), __fmul_rn(x1, r.x));
                                    o[(ra >> 7) * g.head_stride + (ra & 127u)] = y0;
                                    o[(rb >> 7) * g.head_stride + (rb & 127u)] = y1;
                                }
                            }
                        }
                } else {
                    for (uint32_t c = 0; c < (uint32_t)kRowTile; c += 16) {
                        float v[16];
                        fetch(c, v);
                        if (tvalid) {
#pragma unroll
                            for (int j = 0; j < 16; ++j) {
                                const uint32_t r = row0 + c + (uint32_t)j;
                                if (r >= g.rows) continue;
                                float *p = o + (r >> 7) * g.head_stride + (r & 127u);
                                float y = v[j] * s;
                                if (a.epi == GEPI_RESID) y = *p + y;   // src/brain_runtime.c:1745, :1762
                                else if (g.bias) y += __ldg(g.bias + r);
                                *p = y;
                            }
                        }
                    }
                }
            }
            if (!reduce) {
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars->acc_empty[buf]);
            } else if (lane == 0) {
                a.ctr[tile_id * 4u + quarter] = 0;   // ready for the next launch
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, 512);
    if (threadIdx.x == 0 && bars->status != kStatusOk) atomicCAS(a.status, kStatusOk, bars->status);
}

// ---------------------------------------------------- activation split ----

// One CTA per token row (padding rows of the last token tile included):
// optional rms_norm (src/brain_runtime.c:1338-1371: double sum of squares,
// out = x * inv * w), power-of-two scaling of the row into [2^14, 2^15),
// binary16 hi/lo split, stored as 128-byte-swizzled K-major tiles
// [token tile][K block][hi, lo][128 rows x 64].
__global__ void __launch_bounds__(256) split_kernel(const float *x, uint32_t ldx, uint32_t cols, uint32_t tokens,
                                                    const float *norm_w, float eps, uint8_t *xt, float *xscale)
{
    __shared__ double dred[8];
    __shared__ float fred[8];
    const uint32_t t = blockIdx.x, tl = t % kTokTile, tt = t / kTokTile, kbn = cols / kKBlock;
    const uint32_t nch = cols / 8;
    uint8_t *tile0 = xt + (size_t)tt * kbn * kXTileBytes;
    if (t >= tokens) {
        for (uint32_t ch = threadIdx.x; ch < nch; ch += blockDim.x) {
            uint8_t *p = tile0 + (size_t)(ch >> 3) * kXTileBytes + sw128_off(tl, ch & 7u);
            *reinterpret_cast<uint4 *>(p) = make_uint4(0, 0, 0, 0);
            *reinterpret_cast<uint4 *>(p + kATermBytes) = make_uint4(0, 0, 0, 0);
        }
        if (threadIdx.x == 0) xscale[t] = 0.f;
        return;
    }
    const float *xr = x + (size_t)t * ldx;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    float inv = 1.f;
    if (norm_w) {
        double ss = 0.0;
        for (uint32_t i = threadIdx.x; i < cols; i += blockDim.x) {
            const double v = xr[i];
            ss += v * v;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) dred[warp] = ss;
        __syncthreads();
        if (threadIdx.x == 0) {
            double tot = 0.0;
            for (int i = 0; i < 8; ++i) tot += dred[i];
            dred[0] = tot;
        }
        __syncthreads();
        inv = 1.0f / sqrtf((float)(dred[0] / (double)cols) + eps);
    }
    auto val = [&](uint32_t i) { return norm_w ? __fmul_rn(__fmul_rn(xr[i], inv), norm_w[i]) : xr[i]; };
    float amax = 0.f;
    for (uint32_t i = threadIdx.x; i < cols; i += blockDim.x) amax = fmaxf(amax, fabsf(val(i)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0) fred[warp] = amax;
    __syncthreads();
    amax = 0.f;
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fred[i]);
    int e = 0;
    if (amax > 0.f && amax <= FLT_MAX) frexpf(amax, &e);
    const int sx = amax > 0.f ? 15 - e : 0;
    const float p2 = ldexpf(1.0f, sx);
    for (uint32_t ch = threadIdx.x; ch < nch; ch += blockDim.x) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = val(ch * 8u + (uint32_t)j) * p2;
        uint32_t h[4], l[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            h[j] = pack_h2(v[2 * j], v[2 * j + 1]);
            const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&h[j]));
            l[j] = pack_h2(v[2 * j] - f.x, v[2 * j + 1] - f.y);
        }
        uint8_t *p = tile0 + (size_t)(ch >> 3) * kXTileBytes + sw128_off(tl, ch & 7u);
        *reinterpret_cast<uint4 *>(p) = make_uint4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<uint4 *>(p + kATermBytes) = make_uint4(l[0], l[1], l[2], l[3]);
    }
    if (threadIdx.x == 0) xscale[t] = ldexpf(1.0f, -sx);
}

// ------------------------------------------------------------ embedding ----

// x[t] = token_embd row ids[t] (load_embedding_row, src/brain_runtime.c:1311-1332).
__global__ void embed_kernel(const uint32_t *ids, uint32_t tokens, const uint8_t *embd, uint32_t type,
                             uint64_t row_bytes, uint32_t hidden, float *x)
{
    const uint32_t t = blockIdx.x;
    if (t >= tokens) return;
    const uint8_t *row = embd + (size_t)ids[t] * row_bytes;
    const uint32_t be = block_elems(type), bb = block_bytes(type);
    for (uint32_t i = threadIdx.x; i < hidden; i += blockDim.x)
        x[(size_t)t * hidden + i] = deq_elem(type, row + (size_t)(i / be) * bb, (int)(i % be));
}

// ------------------------------------------------------------ attention ----

// Causal GQA attention for prompt tokens (gqa_single_token per token,
// src/brain_runtime.c:1482-1528). A unit is (kv head g, tile of kQT query
// tokens, span of cached positions): the kQT x group query rows walk the
// span kKC keys at a time through shared memory (fp32 scores, online softmax,
// P.V); a (g, tile) whose keys fit one span writes its output directly,
// otherwise each span stores (acc, max, sum) and the last span to finish
// merges them.
constexpr uint32_t kQT = 8, kKC = 64, kRows = 64, kQPad = 132, kPPad = 68, kRec = 132;

struct AttnSmem {
    float q[kRows][kQPad];
    float k[kKC][kQPad];
    float v[kKC][128];
    float p[kRows][kPPad];
    uint32_t flag;
};

__global__ void __launch_bounds__(256, 1) attn_kernel(const __grid_constant__ AttnArgs a)
{
    extern __shared__ uint8_t smem_raw[];
    AttnSmem &sm = *reinterpret_cast<AttnSmem *>(smem_raw);
    const uint32_t tid = threadIdx.x, ty = tid >> 4, tx = tid & 15u;
    const uint32_t group = a.q_heads / a.kv_heads, qdim = a.q_heads * 128u;
    const float scale = 1.0f / sqrtf(128.0f);
    for (uint32_t u = blockIdx.x; u < a.n_units; u += gridDim.x) {
        const uint32_t code = a.unit_tab[u];
        const uint32_t g = code & 0xffu, qt = (code >> 8) & 0xfffu, part = code >> 20;
        const uint32_t t0 = qt * kQT, t1 = min(t0 + kQT, a.tokens);
        const uint32_t kend = a.pos0 + t1;                       // keys [0, kend) for this tile
        const uint32_t nparts = (kend + a.span - 1) / a.span;
        const uint32_t k0 = part * a.span, k1 = min(k0 + a.span, kend);
        __syncthreads();   // previous unit done with shared memory
        // queries (rows r = qi * group + h)
        for (uint32_t i = tid; i < kRows * 32u; i += 256u) {
            const uint32_t r = i >> 5, d4 = i & 31u, qi = r / group, h = r % group;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (r < kQT * group && t0 + qi < t1)
                v = __ldcg(reinterpret_cast<const float4 *>(a.q + (size_t)(t0 + qi) * qdim + (size_t)(g * group + h) * 128u) + d4);
            *reinterpret_cast<float4 *>(&sm.q[r][4 * d4]) = v;
        }
        float m[4], l[4], o[4][8];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            m[r] = -FLT_MAX;
            l[r] = 0.f;
#pragma unroll
            for (int j = 0; j < 8; ++j) o[r][j] = 0.f;
        }
        for (uint32_t p0 = k0; p0 < k1; p0 += kKC) {
        if (p0 != k0) __syncthreads();   // previous chunk's K / V / P consumed
        for (uint32_t i = tid; i < kKC * 32u; i += 256u) {
            const uint32_t j = i >> 5, d4 = i & 31u, pos = p0 + j;
            float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
            if (pos < k1) {
                const size_t off = ((size_t)g * a.max_context + pos) * 128u;
                kv = __ldcg(reinterpret_cast<const float4 *>(a.k_cache + off) + d4);
                vv = __ldcg(reinterpret_cast<const float4 *>(a.v_cache + off) + d4);
            }
            *reinterpret_cast<float4 *>(&sm.k[j][4 * d4]) = kv;
            *reinterpret_cast<float4 *>(&sm.v[j][4 * d4]) = vv;
        }
        __syncthreads();
        // scores: rows 4ty..4ty+3, keys tx + 16i
        float s[4][4];
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int i = 0; i < 4; ++i) s[r][i] = 0.f;
#pragma unroll 4
        for (uint32_t d = 0; d < 128u; d += 4) {
            float4 qv[4], kv[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) qv[r] = *reinterpret_cast<const float4 *>(&sm.q[4 * ty + r][d]);
#pragma unroll
            for (int i = 0; i < 4; ++i) kv[i] = *reinterpret_cast<const float4 *>(&sm.k[tx + 16 * i][d]);
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    s[r][i] = fmaf(qv[r].x, kv[i].x, s[r][i]);
                    s[r][i] = fmaf(qv[r].y, kv[i].y, s[r][i]);
                    s[r][i] = fmaf(qv[r].z, kv[i].z, s[r][i]);
                    s[r][i] = fmaf(qv[r].w, kv[i].w, s[r][i]);
                }
        }
        // online softmax (src/brain_runtime.c:1430-1476 computes the same
        // weights in one pass over all scores)
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const uint32_t row = 4 * ty + (uint32_t)r, qi = row / group;
            const uint32_t qpos = a.pos0 + t0 + qi;   // causal: keys <= qpos
            float mx = m[r];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t pos = p0 + tx + 16u * (uint32_t)i;
                const bool ok = row < kQT * group && t0 + qi < t1 && pos <= qpos && pos < k1;
                s[r][i] = ok ? s[r][i] * scale : -INFINITY;
                mx = fmaxf(mx, s[r][i]);
            }
#pragma unroll
            for (int sh = 8; sh > 0; sh >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, sh));
            const float corr = expf(m[r] - mx);
            float sum = 0.f;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float pv = s[r][i] == -INFINITY ? 0.f : expf(s[r][i] - mx);
                sm.p[4 * ty + r][tx + 16 * i] = pv;
                sum += pv;
            }
#pragma unroll
            for (int sh = 8; sh > 0; sh >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, sh);
            m[r] = mx;
            l[r] = fmaf(l[r], corr, sum);
#pragma unroll
            for (int j = 0; j < 8; ++j) o[r][j] *= corr;
        }
        __syncthreads();
        // P.V: rows 4ty..4ty+3, dims 8tx..8tx+7
        for (uint32_t j = 0; j < kKC; ++j) {
            const float4 v0 = *reinterpret_cast<const float4 *>(&sm.v[j][8 * tx]);
            const float4 v1 = *reinterpret_cast<const float4 *>(&sm.v[j][8 * tx + 4]);
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const float pv = sm.p[4 * ty + r][j];
                o[r][0] = fmaf(pv, v0.x, o[r][0]); o[r][1] = fmaf(pv, v0.y, o[r][1]);
                o[r][2] = fmaf(pv, v0.z, o[r][2]); o[r][3] = fmaf(pv, v0.w, o[r][3]);
                o[r][4] = fmaf(pv, v1.x, o[r][4]); o[r][5] = fmaf(pv, v1.y, o[r][5]);
                o[r][6] = fmaf(pv, v1.z, o[r][6]); o[r][7] = fmaf(pv, v1.w, o[r][7]);
            }
        }
        }   // key chunks of the span
        if (nparts == 1) {
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const uint32_t row = 4 * ty + (uint32_t)r, qi = row / group, h = row % group;
                if (row >= kQT * group || t0 + qi >= t1) continue;
                float *dst = a.out + (size_t)(t0 + qi) * qdim + (size_t)(g * group + h) * 128u + 8u * tx;
                const float inv = l[r] > 0.f ? 1.0f / l[r] : 0.f;
#pragma unroll
                for (int j = 0; j < 8; ++j) dst[j] = o[r][j] * inv;
            }
            continue;
        }
        // partial record of this span: acc[128], max, sum per row
        const uint32_t u0 = u - part;   // the tile's spans are consecutive units
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const uint32_t row = 4 * ty + (uint32_t)r;
            float *rec = a.part + ((size_t)u * kRows + row) * kRec;
#pragma unroll
            for (int j = 0; j < 8; j += 4)
                __stcg(reinterpret_cast<float4 *>(rec + 8 * tx + j), make_float4(o[r][j], o[r][j + 1], o[r][j + 2], o[r][j + 3]));
            if (tx == 0) { __stcg(rec + 128, m[r]); __stcg(rec + 129, l[r]); }
        }
        __threadfence();
        __syncthreads();
        if (tid == 0) {
            const uint32_t old = atom_acq_rel_add(a.ctr + g * a.q_tiles + qt, 1u);
            sm.flag = (old == nparts - 1u) ? 1u : 0u;
        }
        __syncthreads();
        if (!sm.flag) continue;
        __threadfence();
        // merge: rows 4ty..4ty+3, dims 8tx..8tx+7
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const uint32_t row = 4 * ty + (uint32_t)r, qi = row / group, h = row % group;
            if (row >= kQT * group || t0 + qi >= t1) continue;
            float M = -FLT_MAX;
            for (uint32_t c = 0; c < nparts; ++c) M = fmaxf(M, __ldcg(a.part + ((size_t)(u0 + c) * kRows + row) * kRec + 128));
            float L = 0.f, acc[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[j] = 0.f;
            for (uint32_t c = 0; c < nparts; ++c) {
                const float *rec = a.part + ((size_t)(u0 + c) * kRows + row) * kRec;
                const float mc = __ldcg(rec + 128);
                const float f = mc == -FLT_MAX ? 0.f : expf(mc - M);
                L = fmaf(f, __ldcg(rec + 129), L);
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[j] = fmaf(f, __ldcg(rec + 8 * tx + j), acc[j]);
            }
            const float inv = L > 0.f ? 1.0f / L : 0.f;
            float *dst = a.out + (size_t)(t0 + qi) * qdim + (size_t)(g * group + h) * 128u + 8u * tx;
#pragma unroll
            for (int j = 0; j < 8; ++j) dst[j] = acc[j] * inv;
        }
        if (tid == 0) a.ctr[g * a.q_tiles + qt] = 0;
    }
}

// ------------------------------------------------- weight scale bound ------

// Upper bound of |w| over a Q4_K / Q6_K tensor from its block headers, as
// float bits (non-negative floats order like unsigned integers).
__global__ void wbound_kernel(uint32_t type, const uint8_t *blocks, uint64_t nblocks, uint32_t *out_bits)
{
    float mx = 0.f;
    for (uint64_t b = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; b < nblocks; b += (uint64_t)gridDim.x * blockDim.x) {
        const uint8_t *p = blocks + b * (type == 12u ? 144u : 210u);
        float v;
        if (type == 12u) {
            const float d = fabsf(h2f_exact(ld_u16(p))), dm = fabsf(h2f_exact(ld_u16(p + 2)));
            v = d * 63.f * 15.f + dm * 63.f;
        } else {
            v = fabsf(h2f_exact(ld_u16(p + 208))) * 128.f * 32.f;
        }
        if (!(v <= FLT_MAX)) v = FLT_MAX;   // NaN / inf headers: clamp
        mx = fmaxf(mx, v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31u) == 0) atomicMax(out_bits, __float_as_uint(mx));
}

}  // namespace pf
}  // namespace atlas

using namespace atlas;
using namespace atlas::pf;

extern "C" size_t atlas_prefill_gemm_smem() { return kGemmSmem; }
extern "C" size_t atlas_prefill_attn_smem() { return sizeof(AttnSmem); }

extern "C" cudaError_t atlas_launch_prefill_gemm(const GemmArgs *a, int grid, cudaStream_t stream)
{
    static bool attr_set[3] = {false, false, false};
    const int ti = (int)a->terms - 1;
    if (ti < 0 || ti > 2) return cudaErrorInvalidValue;
    void (*fn)(GemmArgs) = ti == 0 ? gemm_kernel<1> : ti == 1 ? gemm_kernel<2> : gemm_kernel<3>;
    if (!attr_set[ti]) {
        cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemmSmem);
        if (e != cudaSuccess) return e;
        attr_set[ti] = true;
    }
    fn<<<grid, kThreads, kGemmSmem, stream>>>(*a);
    return cudaGetLastError();
}

extern "C" cudaError_t atlas_launch_prefill_split(const float *x, uint32_t ldx, uint32_t cols, uint32_t tokens,
                                                  uint32_t tok_pad, const float *norm_w, float eps, uint8_t *xt,
                                                  float *xscale, cudaStream_t stream)
{
    split_kernel<<<tok_pad, 256, 0, stream>>>(x, ldx, cols, tokens, norm_w, eps, xt, xscale);
    return cudaGetLastError();
}

extern "C" cudaError_t atlas_launch_prefill_embed(const uint32_t *ids, uint32_t tokens, const uint8_t *embd,
                                                  uint32_t type, uint64_t row_bytes, uint32_t hidden, float *x,
                                                  cudaStream_t stream)
{
    embed_kernel<<<tokens, 256, 0, stream>>>(ids, tokens, embd, type, row_bytes, hidden, x);
    return cudaGetLastError();
}

extern "C" cudaError_t atlas_launch_prefill_attn(const AttnArgs *a, int grid, cudaStream_t stream)
{
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(AttnSmem));
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    attn_kernel<<<grid, 256, sizeof(AttnSmem), stream>>>(*a);
    return cudaGetLastError();
}

extern "C" cudaError_t atlas_launch_wbound(uint32_t type, const uint8_t *blocks, uint64_t nblocks, uint32_t *out_bits,
                                           cudaStream_t stream)
{
    wbound_kernel<<<148, 256, 0, stream>>>(type, blocks, nblocks, out_bits);
    return cudaGetLastError();
}
