/*
 * The reference's device-plugin ABI (src/gpu_matvec.h:6-17), implemented by
 * libatlas_cuda on B200 so the reference runtime's hybrid path and its
 * `--gpu-check` self-test (src/brain_runtime.c:1958-1984) link against it
 * unchanged. Same names, field order and return convention: 1 = success,
 * 0 = failure (a message goes to stderr at most 4 times, as in
 * src/gpu_matvec.c:211-218).
 */
#ifndef BRAIN_GPU_MATVEC_H
#define BRAIN_GPU_MATVEC_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* One GEMV: `offset` is the absolute file offset of row 0's first block, `type`
   a ggml type id, `input` cols floats and `output` rows floats, both host memory.
   Replaces the struct of src/gpu_matvec.h:6-11. */
typedef struct {
    uint64_t offset, rows, cols;
    uint32_t type;
    const float *input;
    float *output;
} BrainGpuMatvec;

/* Copies the whole model file image to device memory; the caller keeps
   ownership of `model`. size must be a positive multiple of 4
   (src/gpu_matvec.c:98). Replaces src/gpu_matvec.h:13. */
int brain_gpu_init(const uint8_t *model, size_t model_size);

/* Runs 1..3 GEMVs and blocks until every output is written
   (src/gpu_matvec.c:209). Replaces src/gpu_matvec.h:14. */
int brain_gpu_matvec_batch(const BrainGpuMatvec *ops, size_t count);

/* Single-GEMV form (src/gpu_matvec.c:288). Replaces src/gpu_matvec.h:15-16. */
int brain_gpu_matvec(uint64_t offset, uint32_t type, uint64_t rows,
                     uint64_t cols, const float *input, float *output);

/* Frees the device copy; safe to call twice. Replaces src/gpu_matvec.h:17. */
void brain_gpu_shutdown(void);

#ifdef __cplusplus
}
#endif
#endif
