/*
 * ORACLE: a CPU restatement of the reference's decode/prefill path.
 *
 * Test infrastructure only. tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg may load liboracle.so, and only as the checker; the product
 * library never links or calls it.
 *
 * Every function restates one reference function (cited in atlas_oracle.c) with
 * the same arithmetic order, so on the same inputs it reproduces the reference
 * bit for bit; the CPU test suite pins this against the reference compiled in
 * place (oracle/_ref) and against the committed golden fixtures.
 */
#ifndef ATLAS_ORACLE_H
#define ATLAS_ORACLE_H
#include <stddef.h>
#include <stdint.h>

typedef struct OracleModel OracleModel;

float oracle_half_to_float(uint16_t h);
size_t oracle_block_bytes(uint32_t type);
size_t oracle_block_elements(uint32_t type);
/* Dequantizes n consecutive blocks; returns 0 for an unsupported type. */
int oracle_dequant(uint32_t type, const uint8_t *src, float *dst, uint64_t nblocks);
/* y[r] = sum over the row's blocks and elements in order, one fp32 accumulator. */
int oracle_matvec_raw(uint32_t type, const uint8_t *data, uint64_t rows, uint64_t cols,
                      const float *x, float *y);

OracleModel *oracle_open(const char *path);
void oracle_close(OracleModel *m);
/* hidden, q_dim, kv_dim, q_heads, kv_heads, head_dim, ffn, layers, max_context, vocab, has_qk_norm */
int oracle_shape(const OracleModel *m, uint32_t *out11, float *rope_base);
int oracle_tensor(const OracleModel *m, const char *name, uint32_t *type, uint64_t *dims2,
                  const uint8_t **data);
int oracle_matvec(const OracleModel *m, const char *name, const float *x, float *y);
/* Allocates the KV cache for positions [0, max_positions). */
int oracle_session_begin(OracleModel *m, uint32_t max_positions);
int oracle_forward(OracleModel *m, uint32_t token, uint64_t pos, int want_logits, float *logits);
/* Greedy pick: first index of the maximum (exact ties never occur on this data). */
uint32_t oracle_argmax(const float *logits, uint64_t n);
/* Hidden state after output_norm of the last forward. */
int oracle_last_hidden(const OracleModel *m, float *out);
int oracle_kv_row(const OracleModel *m, uint32_t layer, uint64_t pos, float *k, float *v);

void oracle_rms_norm(const float *x, const float *w, float *out, size_t n, float eps);
void oracle_rope(float *q, float *k, int q_dim, int k_dim, int head_dim, float base, int pos);
void oracle_rope_table(int head_dim, float base, int pos, float *cos_out, float *sin_out);

#endif
