/*
 * Seeded synthetic Qwen2-family GGUF writer.
 *
 * Produces the model files the parity tests and the benchmark run on: the
 * tensor set and names the reference runtime reads (src/brain_runtime.c:1698-1772,
 * derive_model_shape :507-583), GGUF v3 with 32-byte data alignment
 * (data base = align32(end of tensor directory), src/brain_runtime.c:433-434),
 * and a byte-level BPE vocabulary the reference tokenizer accepts
 * (load_tokenizer :748-790).
 *
 * Block contents follow the documented synthetic distributions:
 *   Q4_K: d, dmin = fp16(U[1e-4, 2e-3]); the 12 packed scale/min bytes and the
 *         128 nibble bytes uniform (every 6-bit scale/min and every nibble is
 *         then uniform);
 *   Q6_K: d = fp16(U[1e-4, 2e-3]); int8 scales U{-32..31}; ql/qh uniform
 *         (every 6-bit quant uniform in 0..63);
 *   norm weights 1 + N(0, 0.02) f32; biases N(0, 0.02) f32.
 * Tensor types: attn_q/k/output, ffn_gate/up Q4_K; attn_v, ffn_down,
 * token_embd, output Q6_K. Tied models emit an output.weight directory entry
 * whose offset aliases token_embd.weight (the reference requires the entry,
 * src/brain_runtime.c:529-531).
 *
 * Every block is a pure function of (seed, tensor index, block index), so the
 * bytes are identical on every machine and independent of thread count.
 */
#ifndef ATLAS_SYNTH_H
#define ATLAS_SYNTH_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    uint32_t hidden;          /* embedding length H */
    uint32_t layers;
    uint32_t q_heads;
    uint32_t kv_heads;
    uint32_t head_dim;        /* q_dim = q_heads * head_dim */
    uint32_t ffn;             /* feed-forward length F (multiple of 256) */
    uint32_t vocab;
    uint32_t context_length;  /* metadata qwen2.context_length */
    float rope_base;          /* metadata qwen2.rope.freq_base */
    int32_t tied;             /* 1: output.weight aliases token_embd.weight */
    int32_t qkv_bias;         /* 1: emit attn_q/k/v.bias */
    int32_t threads;          /* 0: all cores */
    uint64_t seed;
    int32_t qk_norm;          /* 1: a qwen3 file (architecture "qwen3", per-head
                                 blk.N.attn_q_norm / attn_k_norm.weight, head_dim floats) */
    int32_t alt_type;         /* 0, or another ggml block type the reference reads (1 F16,
                                 6 Q5_0, 7 Q5_1, 8 Q8_0, 13 Q5_K) for attn_q, ffn_gate,
                                 ffn_up, ffn_down and the head (token_embd.weight when
                                 tied, else output.weight): d (and dmin / m)
                                 fp16(U[1e-4, 2e-3]), every other byte uniform; F16
                                 elements fp16(U[-0.05, 0.05]) */
    int32_t layer_mix;        /* 1: odd layers' attn_v and ffn_down are Q4_K (types that
                                 change across layers, as in a Q4_K_M file) */
} AtlasSynthConfig;

/* Writes the model to `path`. Returns 0 on success, -1 on failure (errno-style
   message on stderr). */
int atlas_synth_write_gguf(const AtlasSynthConfig *cfg, const char *path);

/* Fills n Q4_K (144-byte) or Q6_K (210-byte) blocks for (seed, stream) with the
   distributions above; used by the kernel-level parity tests. */
void atlas_synth_q4k_blocks(uint64_t seed, uint64_t stream, uint8_t *dst, uint64_t n);
void atlas_synth_q6k_blocks(uint64_t seed, uint64_t stream, uint8_t *dst, uint64_t n);

/* Total file size the writer will produce for cfg (for callers sizing disks). */
uint64_t atlas_synth_file_size(const AtlasSynthConfig *cfg);

#ifdef __cplusplus
}
#endif
#endif
