/*
 * Device-plugin stub for the ORACLE build of the reference runtime.
 * The reference's Direct3D 12 plugin (src/gpu_matvec.c) cannot be built on
 * Linux; returning 0 from brain_gpu_init makes the runtime take its CPU path
 * ("CPU fallback", src/brain_runtime.c:1942-1947). Test infrastructure only.
 */
#include <stddef.h>
#include <stdint.h>
#include "gpu_matvec.h"

int brain_gpu_init(const uint8_t *model, size_t model_size)
{
    (void)model; (void)model_size;
    return 0;
}

int brain_gpu_matvec_batch(const BrainGpuMatvec *ops, size_t count)
{
    (void)ops; (void)count;
    return 0;
}

int brain_gpu_matvec(uint64_t offset, uint32_t type, uint64_t rows,
                     uint64_t cols, const float *input, float *output)
{
    (void)offset; (void)type; (void)rows; (void)cols; (void)input; (void)output;
    return 0;
}

void brain_gpu_shutdown(void) {}
