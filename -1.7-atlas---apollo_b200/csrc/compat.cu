// The reference's device-plugin ABI (include/gpu_matvec.h, replacing
// src/gpu_matvec.c's Direct3D 12 implementation) on B200.
//
// brain_gpu_init uploads the whole model file image once (as
// src/gpu_matvec.c:94-207 does); brain_gpu_matvec_batch runs up to three GEMVs
// whose weights are addressed by absolute file offset, with host input and
// output vectors, and blocks until the outputs are written
// (src/gpu_matvec.c:209-286). Q4_K / Q6_K rows go through the decode GEMV
// engine; the reference's other block types (Q5_0, Q5_1, Q8_0, Q5_K) through a
// one-warp-per-row kernel with the bit-exact element decoder. Errors return 0
// and are reported on stderr at most 4 times (src/gpu_matvec.c:211-218).
#include <cstdio>
#include <cstring>
#include <mutex>
#include "../../include/atlas_cuda.h"
#include "../../include/gpu_matvec.h"
#include "quant.cuh"

namespace {

struct CompatState {
    std::mutex mu;
    uint8_t *model = nullptr;
    size_t size = 0;
    float *in = nullptr, *out = nullptr;
    size_t in_cap = 0, out_cap = 0;
    cudaStream_t stream = nullptr;
    int device = -1;
    int reported = 0;
};

CompatState g_compat;

void report(const char *stage, const char *detail, size_t count)
{
    if (g_compat.reported < 4) {
        ++g_compat.reported;
        fprintf(stderr, "GPU matvec batch %s failed (%s), operations=%zu\n", stage, detail, count);
    }
}

// y[r] = sum_i deq(W[r, i]) x[i]: one warp per row, any block type of the reference.
__global__ void generic_gemv_kernel(uint32_t type, const uint8_t *w, uint64_t rows, uint64_t cols, const float *x,
                                    float *y)
{
    const uint32_t be = atlas::block_elems(type), bb = atlas::block_bytes(type);
    const uint64_t nb = cols / be;
    const uint64_t warp = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    for (uint64_t r = warp; r < rows; r += (gridDim.x * (uint64_t)blockDim.x) >> 5) {
        const uint8_t *row = w + r * nb * bb;
        float acc = 0.f;
        for (uint64_t i = lane; i < cols; i += 32) acc += atlas::deq_elem(type, row + (i / be) * bb, (int)(i % be)) * x[i];
        acc = atlas::warp_sum(acc);
        if (lane == 0) y[r] = acc;
    }
}

bool grow(float **p, size_t *cap, size_t n)
{
    if (n <= *cap) return true;
    if (*p) cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    if (cudaMalloc(p, n * sizeof(float)) != cudaSuccess) return false;
    *cap = n;
    return true;
}

}  // namespace

extern "C" {

void brain_gpu_shutdown(void)
{
    std::lock_guard<std::mutex> lk(g_compat.mu);
    if (g_compat.device >= 0) cudaSetDevice(g_compat.device);
    if (g_compat.stream) cudaStreamSynchronize(g_compat.stream);
    if (g_compat.model) cudaFree(g_compat.model);
    if (g_compat.in) cudaFree(g_compat.in);
    if (g_compat.out) cudaFree(g_compat.out);
    if (g_compat.stream) cudaStreamDestroy(g_compat.stream);
    g_compat.model = nullptr;
    g_compat.in = g_compat.out = nullptr;
    g_compat.in_cap = g_compat.out_cap = 0;
    g_compat.size = 0;
    g_compat.stream = nullptr;
    g_compat.device = -1;
}

int brain_gpu_init(const uint8_t *model, size_t model_size)
{
    brain_gpu_shutdown();
    if (!model || model_size < 4 || (model_size & 3u)) return 0;
    std::lock_guard<std::mutex> lk(g_compat.mu);
    int dev = 0, sms = 0, major = 0, minor = 0;
    cudaGetDevice(&dev);
    if (atlas_cuda_device_info(dev, &sms, &major, &minor) != ATLAS_OK || major != 10) {
        fprintf(stderr, "CUDA initialization failed: no sm_100 device.\n");
        return 0;
    }
    if (cudaMalloc(&g_compat.model, model_size) != cudaSuccess ||
        cudaMemcpy(g_compat.model, model, model_size, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaStreamCreateWithFlags(&g_compat.stream, cudaStreamNonBlocking) != cudaSuccess) {
        fprintf(stderr, "CUDA initialization failed during model upload.\n");
        if (g_compat.model) cudaFree(g_compat.model);
        g_compat.model = nullptr;
        return 0;
    }
    g_compat.size = model_size;
    g_compat.device = dev;
    return 1;
}

int brain_gpu_matvec_batch(const BrainGpuMatvec *ops, size_t count)
{
    std::lock_guard<std::mutex> lk(g_compat.mu);
    if (!g_compat.model || !ops || !count || count > 3) { report("arguments", "invalid", count); return 0; }
    cudaSetDevice(g_compat.device);
    size_t in_total = 0, out_total = 0;
    for (size_t i = 0; i < count; ++i) {
        const BrainGpuMatvec &op = ops[i];
        const uint32_t be = atlas::block_elems(op.type), bb = atlas::block_bytes(op.type);
        // rows, cols and offset above 2^32 are rejected first (as src/gpu_matvec.c:220-223
        // does); the tensor's extent is then checked by a division (rows x row bytes can
        // exceed 64 bits: 2^32 rows of 2^27 Q8_0 blocks of 34 bytes)
        if (!op.input || !op.output || !op.rows || !op.cols || !be || op.type == 1u || op.cols % be ||
            op.rows > 0xffffffffull || op.cols > 0xffffffffull || op.offset > 0xffffffffull ||
            op.offset > g_compat.size || op.rows > (g_compat.size - op.offset) / ((op.cols / be) * bb)) {
            report("arguments", "invalid operation", count);
            return 0;
        }
        in_total += op.cols;
        out_total += op.rows;
    }
    if (!grow(&g_compat.in, &g_compat.in_cap, in_total) || !grow(&g_compat.out, &g_compat.out_cap, out_total)) {
        report("allocation", "cudaMalloc", count);
        return 0;
    }
    cudaStream_t s = g_compat.stream;
    size_t io = 0, oo = 0;
    for (size_t i = 0; i < count; ++i) {
        const BrainGpuMatvec &op = ops[i];
        const uint8_t *w = g_compat.model + op.offset;
        if (cudaMemcpyAsync(g_compat.in + io, op.input, op.cols * sizeof(float), cudaMemcpyHostToDevice, s) !=
            cudaSuccess) { report("upload", "cudaMemcpyAsync", count); return 0; }
        const bool fast = (op.type == ATLAS_TYPE_Q4_K && !((uintptr_t)w & 15u)) ||
                          (op.type == ATLAS_TYPE_Q6_K && !((uintptr_t)w & 1u));
        int rc = ATLAS_OK;
        if (fast) {
            rc = atlas_cuda_gemv(op.type, w, op.rows, op.cols, g_compat.in + io, g_compat.out + oo, s);
        } else {
            generic_gemv_kernel<<<1184, 256, 0, s>>>(op.type, w, op.rows, op.cols, g_compat.in + io, g_compat.out + oo);
            if (cudaGetLastError() != cudaSuccess) rc = ATLAS_ECUDA;
        }
        if (rc != ATLAS_OK) { report("dispatch", atlas_cuda_last_error(nullptr), count); return 0; }
        if (cudaMemcpyAsync(op.output, g_compat.out + oo, op.rows * sizeof(float), cudaMemcpyDeviceToHost, s) !=
            cudaSuccess) { report("readback", "cudaMemcpyAsync", count); return 0; }
        io += op.cols;
        oo += op.rows;
    }
    const cudaError_t e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) { report("fence wait", cudaGetErrorString(e), count); return 0; }
    return 1;
}

int brain_gpu_matvec(uint64_t offset, uint32_t type, uint64_t rows, uint64_t cols, const float *input, float *output)
{
    BrainGpuMatvec op = {offset, rows, cols, type, input, output};
    return brain_gpu_matvec_batch(&op, 1);
}

}  // extern "C"
