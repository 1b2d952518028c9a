/*
 * Host runtime: the reference's model/forward API (src/brain_runtime.c) on top
 * of libatlas_cuda. A caller that used the reference's gguf_open /
 * find_tensor / forward_token sequence uses the same steps here:
 *
 *   reference (src/brain_runtime.c)        this library
 *   ram_model_load + gguf_open :18, :401   atlas_rt_open   (mmap, no full-file copy)
 *   derive_model_shape :507                atlas_rt_shape  (tied output head and
 *                                                           context > 8192 accepted)
 *   find_tensor :920                       atlas_rt_find_tensor
 *   forward_token :1698                    atlas_rt_forward_token
 *   forward_prefill_batch (batch :1644)    atlas_rt_prefill
 *   decode loop :2036-2048 (greedy)        atlas_rt_generate
 *   gguf_close / ram_model_free            atlas_rt_close
 *
 * Return convention: ATLAS_OK (0) or a negative ATLAS_E* code (atlas_cuda.h);
 * atlas_rt_error() gives the message.
 */
#ifndef ATLAS_RUNTIME_H
#define ATLAS_RUNTIME_H
#include <stddef.h>
#include <stdint.h>
#include "atlas_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct AtlasRuntime AtlasRuntime;

/* ModelShape, src/brain_runtime.c:93-99 */
typedef struct {
    uint32_t hidden_size, q_dim, kv_dim, q_heads, kv_heads;
    uint32_t head_dim, ffn_size, layers, max_context, vocab_size;
    float rope_base;
    int32_t has_qk_norm;
    char architecture[64];
} AtlasShape;

/* TensorInfo, src/brain_runtime.c:138-144 (offset is relative to the data base). */
typedef struct {
    char name[256];
    uint32_t n_dims;
    uint64_t dims[4];
    uint32_t type;
    uint64_t offset;
} AtlasTensorInfo;

typedef struct {
    int32_t device;        /* CUDA device ordinal */
    uint32_t max_context;  /* KV positions to allocate; 0: the model's context (no 8192 cap) */
    uint32_t max_prefill;  /* 0: 512 */
    int32_t kv_fp16;       /* 1: fp16 KV cache instead of fp32 (atlas_cuda.h) */
    int32_t no_device;     /* 1: parse only (no GPU work) */
    int32_t tp_rank;       /* tensor parallel: this process's rank ... */
    int32_t tp_size;       /* ... of tp_size (0 or 1: one GPU); see atlas_cuda_tp_* */
    uint32_t max_batch;    /* sequences with a KV cache of their own (0 or 1: one); atlas_cuda_generate_batch */
} AtlasRtOptions;

int atlas_rt_open(const char *path, const AtlasRtOptions *opt, AtlasRuntime **out);
void atlas_rt_close(AtlasRuntime *rt);
const char *atlas_rt_error(const AtlasRuntime *rt);
int atlas_rt_shape(const AtlasRuntime *rt, AtlasShape *out);
uint64_t atlas_rt_data_base(const AtlasRuntime *rt);
/* 1 when the tensor exists (out filled), 0 otherwise - find_tensor's convention, not ATLAS_OK's. */
int atlas_rt_find_tensor(const AtlasRuntime *rt, const char *name, AtlasTensorInfo *out);
/* Raw bytes of the mapped file (for callers that address tensors by absolute offset). */
const uint8_t *atlas_rt_file_bytes(const AtlasRuntime *rt, uint64_t *size);
AtlasCuda *atlas_rt_device(AtlasRuntime *rt);

int atlas_rt_forward_token(AtlasRuntime *rt, uint32_t token, uint32_t pos, float *logits, uint32_t *argmax);
int atlas_rt_prefill(AtlasRuntime *rt, const uint32_t *ids, uint32_t n, uint32_t pos0, float *logits,
                     uint32_t *argmax);
int atlas_rt_generate(AtlasRuntime *rt, uint32_t first, uint32_t pos0, uint32_t steps, uint32_t *out_ids);

#ifdef __cplusplus
}
#endif
#endif
