/*
 * ORACLE: CPU restatement of the reference decode path (test infrastructure
 * only; see atlas_oracle.h). Each function names the reference function it
 * restates; the arithmetic order, the precision of every accumulator and the
 * libm calls are the reference's, so results match it bit for bit.
 *
 * Rows of a GEMV are independent, so they are spread over OpenMP threads;
 * each row is still one sequential fp32 accumulation, as in the reference.
 */
#define _GNU_SOURCE
#include "atlas_oracle.h"

#include <fcntl.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

enum { TY_F32 = 0, TY_F16 = 1, TY_Q5_0 = 6, TY_Q5_1 = 7, TY_Q8_0 = 8,
       TY_Q4_K = 12, TY_Q5_K = 13, TY_Q6_K = 14 };

/* ---------------------------------------------------------------------------
 * Element formats
 * ------------------------------------------------------------------------- */

/* half_to_float, src/brain_runtime.c:203-247: exact binary16 -> binary32,
   subnormals renormalised, Inf/NaN keep the payload. */
float oracle_half_to_float(uint16_t h)
{
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t e = (h >> 10) & 31u, m = h & 1023u, bits;
    if (e == 31u) {
        bits = sign | 0x7f800000u | (m << 13);
    } else if (e != 0u) {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    } else if (m == 0u) {
        bits = sign;
    } else {
        int shift = 0;
        while (!(m & 0x400u)) { m <<= 1; ++shift; }
        bits = sign | ((uint32_t)(113 - shift) << 23) | ((m & 1023u) << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* quant_block_bytes / quant_block_elements, src/brain_runtime.c:117-136 */
size_t oracle_block_bytes(uint32_t type)
{
    switch (type) {
    case TY_F16: return 2;
    case TY_Q5_0: return 22;
    case TY_Q5_1: return 24;
    case TY_Q8_0: return 34;
    case TY_Q4_K: return 144;
    case TY_Q5_K: return 176;
    case TY_Q6_K: return 210;
    default: return 0;
    }
}

size_t oracle_block_elements(uint32_t type)
{
    if (type == TY_F16) return 1;
    if (type == TY_Q5_0 || type == TY_Q5_1 || type == TY_Q8_0) return 32;
    if (type == TY_Q4_K || type == TY_Q5_K || type == TY_Q6_K) return 256;
    return 0;
}

static inline uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* get_scale_min_k4, src/brain_runtime.c:939-958: the 12 packed bytes hold eight
   6-bit scales and eight 6-bit mins; entries 0-3 sit in the low 6 bits of bytes
   0-3 (scales) and 4-7 (mins); entries 4-7 combine a nibble of bytes 8-11 with
   the top two bits of bytes 0-7. */
static inline void k4_scale_min(int j, const uint8_t *p, unsigned *sc, unsigned *mn)
{
    if (j < 4) {
        *sc = p[j] & 63u;
        *mn = p[j + 4] & 63u;
    } else {
        *sc = (p[j + 4] & 15u) | ((unsigned)(p[j - 4] >> 6) << 4);
        *mn = (p[j + 4] >> 4) | ((unsigned)(p[j] >> 6) << 4);
    }
}

/* dequant_q4_k, src/brain_runtime.c:960-1015. Per 64-value chunk c: 32 bytes,
   low nibbles -> values 64c..64c+31 with (scale, min) pair 2c, high nibbles ->
   64c+32..64c+63 with pair 2c+1. value = fp32(d*sc) * q - fp32(dmin*m). */
static void deq_q4_k(const uint8_t *b, float *out)
{
    const float d = oracle_half_to_float(rd16(b));
    const float dmin = oracle_half_to_float(rd16(b + 2));
    const uint8_t *packed = b + 4, *qs = b + 16;
    for (int c = 0; c < 4; ++c) {
        unsigned s0, m0, s1, m1;
        k4_scale_min(2 * c, packed, &s0, &m0);
        k4_scale_min(2 * c + 1, packed, &s1, &m1);
        const float lo_scale = d * (float)s0, lo_min = dmin * (float)m0;
        const float hi_scale = d * (float)s1, hi_min = dmin * (float)m1;
        const uint8_t *q = qs + 32 * c;
        for (int l = 0; l < 32; ++l) out[64 * c + l] = lo_scale * (float)(q[l] & 15u) - lo_min;
        for (int l = 0; l < 32; ++l) out[64 * c + 32 + l] = hi_scale * (float)(q[l] >> 4) - hi_min;
    }
}

/* dequant_q5_k, src/brain_runtime.c:1017-1043: Q4_K plus a fifth bit per value
   from qh (bit 2c for the low half of chunk c, bit 2c+1 for the high half).
   The reference advances its qh pointer by 8 bytes per 64-value chunk
   (:1039), so chunk c reads qh[8c + i]; the D3D12 shader does the same
   (src/gpu_matvec.c:47, seg*8). Restated as is. */
static void deq_q5_k(const uint8_t *b, float *out)
{
    const float d = oracle_half_to_float(rd16(b));
    const float dmin = oracle_half_to_float(rd16(b + 2));
    const uint8_t *packed = b + 4, *qh = b + 16, *ql = b + 48;
    for (int c = 0; c < 4; ++c) {
        unsigned s0, m0, s1, m1;
        k4_scale_min(2 * c, packed, &s0, &m0);
        k4_scale_min(2 * c + 1, packed, &s1, &m1);
        const float a0 = d * (float)s0, b0 = dmin * (float)m0;
        const float a1 = d * (float)s1, b1 = dmin * (float)m1;
        const unsigned bit_lo = 1u << (2 * c), bit_hi = 1u << (2 * c + 1);
        for (int i = 0; i < 32; ++i) {
            const unsigned h = qh[8 * c + i];
            unsigned lo = (ql[32 * c + i] & 15u) + ((h & bit_lo) ? 16u : 0u);
            unsigned hi = (ql[32 * c + i] >> 4) + ((h & bit_hi) ? 16u : 0u);
            out[64 * c + i] = a0 * (float)lo - b0;
            out[64 * c + 32 + i] = a1 * (float)hi - b1;
        }
    }
}

/* dequant_q6_k, src/brain_runtime.c:1049-1083. Two 128-value halves h; lane l
   reads ql[64h+l], ql[64h+32+l], qh[32h+l] and yields four 6-bit values for
   positions 128h + 32k + l (k = 0..3); scale index 8h + l/16 + 2k.
   value = fp32(d * scale) * (q - 32). */
static void deq_q6_k(const uint8_t *b, float *out)
{
    const uint8_t *ql = b, *qh = b + 128;
    const int8_t *sc = (const int8_t *)(b + 192);
    const float d = oracle_half_to_float(rd16(b + 208));
    for (int h = 0; h < 2; ++h) {
        for (int l = 0; l < 32; ++l) {
            const unsigned a = ql[64 * h + l], c = ql[64 * h + 32 + l], hb = qh[32 * h + l];
            const int q[4] = {
                (int)((a & 15u) | ((hb & 3u) << 4)),
                (int)((c & 15u) | (((hb >> 2) & 3u) << 4)),
                (int)((a >> 4) | (((hb >> 4) & 3u) << 4)),
                (int)((c >> 4) | (((hb >> 6) & 3u) << 4)),
            };
            for (int k = 0; k < 4; ++k) {
                const float s = d * (float)sc[8 * h + l / 16 + 2 * k];
                out[128 * h + 32 * k + l] = s * (float)(q[k] - 32);
            }
        }
    }
}

/* dequant_block's small-block branches, src/brain_runtime.c:1085-1121 */
static void deq_small(uint32_t type, const uint8_t *b, float *out)
{
    const float d = oracle_half_to_float(rd16(b));
    if (type == TY_F16) { out[0] = d; return; }
    if (type == TY_Q8_0) {
        for (int i = 0; i < 32; ++i) out[i] = d * (float)(int8_t)b[2 + i];
        return;
    }
    uint32_t high;
    const uint8_t *nib;
    float m = 0.0f;
    if (type == TY_Q5_0) {
        memcpy(&high, b + 2, 4);
        nib = b + 6;
    } else {
        m = oracle_half_to_float(rd16(b + 2));
        memcpy(&high, b + 4, 4);
        nib = b + 8;
    }
    for (unsigned i = 0; i < 32; ++i) {
        unsigned q = i < 16 ? (nib[i & 15u] & 15u) : (nib[i & 15u] >> 4);
        q |= ((high >> i) & 1u) << 4;
        out[i] = type == TY_Q5_0 ? d * ((float)q - 16.0f) : d * (float)q + m;
    }
}

static int deq_one(uint32_t type, const uint8_t *b, float *out)
{
    switch (type) {
    case TY_Q4_K: deq_q4_k(b, out); return 1;
    case TY_Q5_K: deq_q5_k(b, out); return 1;
    case TY_Q6_K: deq_q6_k(b, out); return 1;
    case TY_F16: case TY_Q5_0: case TY_Q5_1: case TY_Q8_0: deq_small(type, b, out); return 1;
    default: return 0;
    }
}

int oracle_dequant(uint32_t type, const uint8_t *src, float *dst, uint64_t nblocks)
{
    const size_t bb = oracle_block_bytes(type), be = oracle_block_elements(type);
    if (!bb) return 0;
    int ok = 1;
#pragma omp parallel for schedule(static) if (nblocks > 4096)
    for (int64_t i = 0; i < (int64_t)nblocks; ++i)
        if (!deq_one(type, src + (uint64_t)i * bb, dst + (uint64_t)i * be)) ok = 0;
    return ok;
}

/* matvec_rows, src/brain_runtime.c:1133-1155: per row, blocks in order, each
   block dequantized then dotted element by element into ONE fp32 sum. */
int oracle_matvec_raw(uint32_t type, const uint8_t *data, uint64_t rows, uint64_t cols,
                      const float *x, float *y)
{
    const size_t bb = oracle_block_bytes(type), be = oracle_block_elements(type);
    if (!bb || !cols || cols % be) return 0;
    const uint64_t nb = cols / be;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < (int64_t)rows; ++r) {
        float w[256];
        float sum = 0.0f;
        for (uint64_t b = 0; b < nb; ++b) {
            deq_one(type, data + ((uint64_t)r * nb + b) * bb, w);
            const float *xb = x + b * be;
            for (size_t i = 0; i < be; ++i) sum += w[i] * xb[i];
        }
        y[r] = sum;
    }
    return 1;
}

/* ---------------------------------------------------------------------------
 * Vector ops
 * ------------------------------------------------------------------------- */

/* rms_norm, src/brain_runtime.c:1338-1371: sum of squares in double,
   inv = 1/sqrtf(float(mean) + eps), out = x * inv * w (left to right). */
void oracle_rms_norm(const float *x, const float *w, float *out, size_t n, float eps)
{
    double ss = 0.0;
    for (size_t i = 0; i < n; ++i) {
        const double v = x[i];
        ss += v * v;
    }
    const float inv = 1.0f / sqrtf((float)(ss / (double)n) + eps);
    for (size_t i = 0; i < n; ++i) out[i] = x[i] * inv * w[i];
}

/* rope's angle table, src/brain_runtime.c:1383-1387 */
void oracle_rope_table(int head_dim, float base, int pos, float *cos_out, float *sin_out)
{
    for (int p = 0; p < head_dim / 2; ++p) {
        const float freq = powf(base, -(2.0f * (float)p) / (float)head_dim);
        const float theta = (float)pos * freq;
        cos_out[p] = cosf(theta);
        sin_out[p] = sinf(theta);
    }
}

/* rope, src/brain_runtime.c:1377-1401: NEOX pairing (i, i + head_dim/2). */
void oracle_rope(float *q, float *k, int q_dim, int k_dim, int head_dim, float base, int pos)
{
    float c[256], s[256];
    const int half = head_dim / 2;
    oracle_rope_table(head_dim, base, pos, c, s);
    float *vecs[2] = {q, k};
    const int dims[2] = {q_dim, k_dim};
    for (int which = 0; which < 2; ++which) {
        float *v = vecs[which];
        for (int h0 = 0; h0 < dims[which]; h0 += head_dim)
            for (int p = 0; p < half; ++p) {
                const float a = v[h0 + p], b = v[h0 + p + half];
                v[h0 + p] = a * c[p] - b * s[p];
                v[h0 + p + half] = a * s[p] + b * c[p];
            }
    }
}

/* ---------------------------------------------------------------------------
 * GGUF reading (restates gguf_open / read_model_metadata / derive_model_shape,
 * src/brain_runtime.c:312-345, 401-445, 507-583) over an mmap of the file.
 * ------------------------------------------------------------------------- */

typedef struct {
    char name[256];
    uint32_t n_dims, type;
    uint64_t dims[4], offset;
} OTensor;

struct OracleModel {
    uint8_t *map;
    size_t size;
    uint64_t data_base;
    OTensor *t;
    uint64_t nt;
    char arch[64];
    uint32_t md_ctx, md_heads, md_kv_heads, md_layers;
    float md_rope;
    /* shape */
    uint32_t H, qd, kvd, nq, nkv, hd, F, L, max_ctx, V;
    int qk_norm;
    float rope_base;
    /* session */
    uint32_t cap;
    float *kc, *vc;
    float *x, *xn, *q, *k, *v, *att, *proj, *gate, *up, *ffn, *scores, *wts, *tmp;
};

typedef struct { const uint8_t *p, *end; int bad; } Cur;

static uint64_t cur_u(Cur *c, int n)
{
    if (c->bad || c->end - c->p < n) { c->bad = 1; return 0; }
    uint64_t v = 0;
    memcpy(&v, c->p, (size_t)n);
    c->p += n;
    return v;
}

static void cur_skip(Cur *c, uint64_t n)
{
    if (c->bad || (uint64_t)(c->end - c->p) < n) { c->bad = 1; return; }
    c->p += n;
}

static void skip_val(Cur *c, uint32_t type)
{
    static const int fixed[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
    if (type == 8) { cur_skip(c, cur_u(c, 8)); return; }
    if (type == 9) {
        uint32_t et = (uint32_t)cur_u(c, 4);
        uint64_t n = cur_u(c, 8);
        for (uint64_t i = 0; i < n && !c->bad; ++i) skip_val(c, et);
        return;
    }
    if (type > 12) { c->bad = 1; return; }
    cur_skip(c, (uint64_t)fixed[type]);
}

static int ends_with(const char *s, size_t n, const char *suffix)
{
    size_t k = strlen(suffix);
    return n >= k && memcmp(s + n - k, suffix, k) == 0;
}

static const OTensor *find_t(const OracleModel *m, const char *name)
{
    for (uint64_t i = 0; i < m->nt; ++i)
        if (!strcmp(m->t[i].name, name)) return &m->t[i];
    return NULL;
}

static int derive_shape(OracleModel *m)
{
    const OTensor *emb = find_t(m, "token_embd.weight"), *out = find_t(m, "output.weight");
    const OTensor *q = find_t(m, "blk.0.attn_q.weight"), *k = find_t(m, "blk.0.attn_k.weight");
    const OTensor *g = find_t(m, "blk.0.ffn_gate.weight");
    if (!emb || !out || !q || !k || !g) return 0;
    uint32_t max_layer = 0;
    int saw = 0;
    for (uint64_t i = 0; i < m->nt; ++i) {
        unsigned l;
        if (sscanf(m->t[i].name, "blk.%u.", &l) == 1) {
            if (!saw || l > max_layer) max_layer = l;
            saw = 1;
        }
    }
    m->H = (uint32_t)emb->dims[0];
    m->V = (uint32_t)out->dims[1];
    m->qd = (uint32_t)q->dims[1];
    m->kvd = (uint32_t)k->dims[1];
    m->F = (uint32_t)g->dims[1];
    m->nq = m->md_heads;
    if (!m->nq || m->qd % m->nq) return 0;
    m->hd = m->qd / m->nq;
    m->nkv = m->md_kv_heads ? m->md_kv_heads : m->kvd / m->hd;
    m->L = m->md_layers ? m->md_layers : (saw ? max_layer + 1 : 0);
    m->max_ctx = m->md_ctx ? m->md_ctx : 2048;
    if (m->max_ctx > 8192) m->max_ctx = 8192;
    m->rope_base = m->md_rope > 0.0f ? m->md_rope : 1000000.0f;
    m->qk_norm = !strcmp(m->arch, "qwen3");
    return (!strcmp(m->arch, "qwen2") || !strcmp(m->arch, "qwen3")) && m->H && m->L &&
           m->nkv && m->hd && m->nq % m->nkv == 0 && m->hd <= 512;
}

OracleModel *oracle_open(const char *path)
{
    int fd = open(path, O_RDONLY);
    if (fd < 0) return NULL;
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 24) { close(fd); return NULL; }
    void *map = mmap(NULL, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (map == MAP_FAILED) return NULL;
    OracleModel *m = (OracleModel *)calloc(1, sizeof(*m));
    if (!m) { munmap(map, (size_t)st.st_size); return NULL; }
    m->map = (uint8_t *)map;
    m->size = (size_t)st.st_size;
    Cur c = {m->map, m->map + m->size, 0};
    if ((uint32_t)cur_u(&c, 4) != 0x46554747u) goto fail;
    cur_u(&c, 4);
    m->nt = cur_u(&c, 8);
    uint64_t nkv = cur_u(&c, 8);
    for (uint64_t i = 0; i < nkv && !c.bad; ++i) {
        uint64_t kl = cur_u(&c, 8);
        if (kl >= 256 || (uint64_t)(c.end - c.p) < kl) { c.bad = 1; break; }
        const char *key = (const char *)c.p;
        c.p += kl;
        uint32_t ty = (uint32_t)cur_u(&c, 4);
        if (kl == 20 && !memcmp(key, "general.architecture", 20) && ty == 8) {
            uint64_t n = cur_u(&c, 8);
            size_t keep = n < sizeof(m->arch) - 1 ? (size_t)n : sizeof(m->arch) - 1;
            if ((uint64_t)(c.end - c.p) < n) { c.bad = 1; break; }
            memcpy(m->arch, c.p, keep);
            c.p += n;
            continue;
        }
        uint32_t *field = NULL;
        if (ends_with(key, kl, ".context_length")) field = &m->md_ctx;
        else if (ends_with(key, kl, ".attention.head_count_kv")) field = &m->md_kv_heads;
        else if (ends_with(key, kl, ".attention.head_count")) field = &m->md_heads;
        else if (ends_with(key, kl, ".block_count")) field = &m->md_layers;
        if (field && (ty == 4 || ty == 5)) { *field = (uint32_t)cur_u(&c, 4); continue; }
        if (ends_with(key, kl, ".rope.freq_base") && ty == 6) {
            uint32_t bits = (uint32_t)cur_u(&c, 4);
            memcpy(&m->md_rope, &bits, 4);
            continue;
        }
        skip_val(&c, ty);
    }
    if (c.bad || m->nt > 1000000) goto fail;
    m->t = (OTensor *)calloc((size_t)m->nt + 1, sizeof(OTensor));
    if (!m->t) goto fail;
    for (uint64_t i = 0; i < m->nt && !c.bad; ++i) {
        OTensor *t = &m->t[i];
        uint64_t nl = cur_u(&c, 8);
        if (nl >= sizeof(t->name) || (uint64_t)(c.end - c.p) < nl) { c.bad = 1; break; }
        memcpy(t->name, c.p, nl);
        c.p += nl;
        t->n_dims = (uint32_t)cur_u(&c, 4);
        if (t->n_dims > 4) { c.bad = 1; break; }
        for (uint32_t d = 0; d < t->n_dims; ++d) t->dims[d] = cur_u(&c, 8);
        t->type = (uint32_t)cur_u(&c, 4);
        t->offset = cur_u(&c, 8);
    }
    if (c.bad) goto fail;
    m->data_base = ((uint64_t)(c.p - m->map) + 31u) & ~(uint64_t)31u;
    if (!derive_shape(m)) goto fail;
    return m;
fail:
    oracle_close(m);
    return NULL;
}

static void session_free(OracleModel *m)
{
    float **bufs[] = {&m->kc, &m->vc, &m->x, &m->xn, &m->q, &m->k, &m->v, &m->att, &m->proj,
                      &m->gate, &m->up, &m->ffn, &m->scores, &m->wts, &m->tmp};
    for (size_t i = 0; i < sizeof(bufs) / sizeof(bufs[0]); ++i) { free(*bufs[i]); *bufs[i] = NULL; }
    m->cap = 0;
}

void oracle_close(OracleModel *m)
{
    if (!m) return;
    session_free(m);
    free(m->t);
    if (m->map) munmap(m->map, m->size);
    free(m);
}

int oracle_shape(const OracleModel *m, uint32_t *o, float *rope_base)
{
    o[0] = m->H; o[1] = m->qd; o[2] = m->kvd; o[3] = m->nq; o[4] = m->nkv; o[5] = m->hd;
    o[6] = m->F; o[7] = m->L; o[8] = m->max_ctx; o[9] = m->V; o[10] = (uint32_t)m->qk_norm;
    *rope_base = m->rope_base;
    return 1;
}

static const uint8_t *tensor_data(const OracleModel *m, const OTensor *t, uint64_t bytes)
{
    uint64_t at = m->data_base + t->offset;
    if (at > m->size || bytes > m->size - at) return NULL;
    return m->map + at;
}

static uint64_t tensor_nbytes(const OTensor *t)
{
    uint64_t el = 1;
    for (uint32_t d = 0; d < t->n_dims; ++d) el *= t->dims[d];
    if (t->type == TY_F32) return el * 4u;
    size_t be = oracle_block_elements(t->type);
    return be ? el / be * oracle_block_bytes(t->type) : 0;
}

int oracle_tensor(const OracleModel *m, const char *name, uint32_t *type, uint64_t *dims2,
                  const uint8_t **data)
{
    const OTensor *t = find_t(m, name);
    if (!t) return 0;
    *type = t->type;
    dims2[0] = t->dims[0];
    dims2[1] = t->n_dims > 1 ? t->dims[1] : 1;
    *data = tensor_data(m, t, tensor_nbytes(t));
    return *data != NULL;
}

int oracle_matvec(const OracleModel *m, const char *name, const float *x, float *y)
{
    const OTensor *t = find_t(m, name);
    if (!t || t->n_dims != 2) return 0;
    const uint8_t *d = tensor_data(m, t, tensor_nbytes(t));
    return d && oracle_matvec_raw(t->type, d, t->dims[1], t->dims[0], x, y);
}

/* load_f32_vector, src/brain_runtime.c:1280-1309 (F32 and F16 vectors) */
static int vec(const OracleModel *m, const char *name, float *out, size_t n)
{
    const OTensor *t = find_t(m, name);
    if (!t) return 0;
    uint64_t el = 1;
    for (uint32_t d = 0; d < t->n_dims; ++d) el *= t->dims[d];
    if (el != n) return 0;
    if (t->type == TY_F32) {
        const uint8_t *d = tensor_data(m, t, n * 4u);
        if (!d) return 0;
        memcpy(out, d, n * 4u);
        return 1;
    }
    if (t->type == TY_F16) {
        const uint8_t *d = tensor_data(m, t, n * 2u);
        if (!d) return 0;
        for (size_t i = 0; i < n; ++i) out[i] = oracle_half_to_float(rd16(d + 2 * i));
        return 1;
    }
    return 0;
}

static int mv(const OracleModel *m, int layer, const char *suffix, const float *x, float *y)
{
    char name[96];
    snprintf(name, sizeof(name), "blk.%d.%s", layer, suffix);
    return oracle_matvec(m, name, x, y);
}

/* optional_bias + add_bias, src/brain_runtime.c:1540-1561 */
static int bias(const OracleModel *m, int layer, const char *suffix, float *y, size_t n, float *tmp)
{
    char name[96];
    snprintf(name, sizeof(name), "blk.%d.%s", layer, suffix);
    if (!find_t(m, name)) return 1;
    if (!vec(m, name, tmp, n)) return 0;
    for (size_t i = 0; i < n; ++i) y[i] += tmp[i];
    return 1;
}

int oracle_session_begin(OracleModel *m, uint32_t max_positions)
{
    session_free(m);
    const size_t kv = (size_t)m->L * max_positions * m->kvd;
    size_t big = m->H > m->qd ? m->H : m->qd;
    if (m->F > big) big = m->F;
    m->kc = (float *)calloc(kv, 4); m->vc = (float *)calloc(kv, 4);
    m->x = (float *)calloc(m->H, 4); m->xn = (float *)calloc(m->H, 4);
    m->q = (float *)calloc(m->qd, 4); m->k = (float *)calloc(m->kvd, 4);
    m->v = (float *)calloc(m->kvd, 4); m->att = (float *)calloc(m->qd, 4);
    m->proj = (float *)calloc(m->H, 4); m->gate = (float *)calloc(m->F, 4);
    m->up = (float *)calloc(m->F, 4); m->ffn = (float *)calloc(m->F, 4);
    m->scores = (float *)calloc(max_positions, 4); m->wts = (float *)calloc(max_positions, 4);
    m->tmp = (float *)calloc(big, 4);
    m->cap = max_positions;
    return m->kc && m->vc && m->x && m->xn && m->q && m->k && m->v && m->att && m->proj &&
           m->gate && m->up && m->ffn && m->scores && m->wts && m->tmp;
}

/* gqa_single_token + head_dot + softmax, src/brain_runtime.c:1407-1528:
   append (k, v) at pos; per query head (kv head = head / (nq/nkv)):
   score_p = float(double dot) * (1/sqrtf(hd)); softmax with expf and a double
   sum divided back in float; out_i = float(sum_p double(w_p) * v_p,i). */
static void attend(OracleModel *m, int layer, uint64_t pos)
{
    const size_t stride = (size_t)m->cap * m->kvd;
    float *lk = m->kc + (size_t)layer * stride, *lv = m->vc + (size_t)layer * stride;
    memcpy(lk + pos * m->kvd, m->k, m->kvd * 4u);
    memcpy(lv + pos * m->kvd, m->v, m->kvd * 4u);
    const float scale = 1.0f / sqrtf((float)m->hd);
    const uint32_t group = m->nq / m->nkv;
    for (uint32_t h = 0; h < m->nq; ++h) {
        const uint32_t kvh = h / group;
        const float *qh = m->q + (size_t)h * m->hd;
        for (uint64_t p = 0; p <= pos; ++p) {
            const float *kp = lk + p * m->kvd + (size_t)kvh * m->hd;
            double dot = 0.0;
            for (uint32_t i = 0; i < m->hd; ++i) dot += (double)qh[i] * (double)kp[i];
            m->scores[p] = (float)dot * scale;
        }
        float mx = m->scores[0];
        for (uint64_t p = 1; p <= pos; ++p)
            if (m->scores[p] > mx) mx = m->scores[p];
        double total = 0.0;
        for (uint64_t p = 0; p <= pos; ++p) {
            m->wts[p] = expf(m->scores[p] - mx);
            total += m->wts[p];
        }
        if (total == 0.0) {
            for (uint64_t p = 0; p <= pos; ++p) m->wts[p] = 0.0f;
        } else {
            for (uint64_t p = 0; p <= pos; ++p) m->wts[p] /= (float)total;
        }
        for (uint32_t i = 0; i < m->hd; ++i) {
            double acc = 0.0;
            for (uint64_t p = 0; p <= pos; ++p)
                acc += (double)m->wts[p] * lv[p * m->kvd + (size_t)kvh * m->hd + i];
            m->att[(size_t)h * m->hd + i] = (float)acc;
        }
    }
}

/* forward_token, src/brain_runtime.c:1698-1772 */
int oracle_forward(OracleModel *m, uint32_t token, uint64_t pos, int want_logits, float *logits)
{
    if (!m->cap || pos >= m->cap || token >= m->V) return 0;
    const float eps = 1.0e-6f;
    /* load_embedding_row, src/brain_runtime.c:1311-1332 */
    {
        const OTensor *e = find_t(m, "token_embd.weight");
        const size_t bb = e ? oracle_block_bytes(e->type) : 0, be = e ? oracle_block_elements(e->type) : 0;
        if (!e || !bb || token >= e->dims[1]) return 0;
        const uint64_t nb = e->dims[0] / be;
        const uint8_t *row = tensor_data(m, e, (token + 1) * nb * bb);
        if (!row) return 0;
        row += (uint64_t)token * nb * bb;
        for (uint64_t b = 0; b < nb; ++b) deq_one(e->type, row + b * bb, m->x + b * be);
    }
    char name[96];
    for (int l = 0; l < (int)m->L; ++l) {
        snprintf(name, sizeof(name), "blk.%d.attn_norm.weight", l);
        if (!vec(m, name, m->tmp, m->H)) return 0;
        oracle_rms_norm(m->x, m->tmp, m->proj, m->H, eps);
        if (!mv(m, l, "attn_q.weight", m->proj, m->q) || !mv(m, l, "attn_k.weight", m->proj, m->k) ||
            !mv(m, l, "attn_v.weight", m->proj, m->v))
            return 0;
        if (!bias(m, l, "attn_q.bias", m->q, m->qd, m->tmp) ||
            !bias(m, l, "attn_k.bias", m->k, m->kvd, m->tmp) ||
            !bias(m, l, "attn_v.bias", m->v, m->kvd, m->tmp))
            return 0;
        if (m->qk_norm) {
            snprintf(name, sizeof(name), "blk.%d.attn_q_norm.weight", l);
            if (!vec(m, name, m->tmp, m->hd)) return 0;
            for (uint32_t b = 0; b < m->qd; b += m->hd) oracle_rms_norm(m->q + b, m->tmp, m->q + b, m->hd, eps);
            snprintf(name, sizeof(name), "blk.%d.attn_k_norm.weight", l);
            if (!vec(m, name, m->tmp, m->hd)) return 0;
            for (uint32_t b = 0; b < m->kvd; b += m->hd) oracle_rms_norm(m->k + b, m->tmp, m->k + b, m->hd, eps);
        }
        oracle_rope(m->q, m->k, (int)m->qd, (int)m->kvd, (int)m->hd, m->rope_base, (int)pos);
        attend(m, l, pos);
        if (!mv(m, l, "attn_output.weight", m->att, m->proj)) return 0;
        for (uint32_t i = 0; i < m->H; ++i) m->x[i] += m->proj[i];
        snprintf(name, sizeof(name), "blk.%d.ffn_norm.weight", l);
        if (!vec(m, name, m->tmp, m->H)) return 0;
        oracle_rms_norm(m->x, m->tmp, m->proj, m->H, eps);
        if (!mv(m, l, "ffn_gate.weight", m->proj, m->gate) || !mv(m, l, "ffn_up.weight", m->proj, m->up))
            return 0;
        for (uint32_t i = 0; i < m->F; ++i) {
            const float z = m->gate[i];
            m->ffn[i] = (z / (1.0f + expf(-z))) * m->up[i];
        }
        if (!mv(m, l, "ffn_down.weight", m->ffn, m->proj)) return 0;
        for (uint32_t i = 0; i < m->H; ++i) m->x[i] += m->proj[i];
    }
    if (!vec(m, "output_norm.weight", m->tmp, m->H)) return 0;
    oracle_rms_norm(m->x, m->tmp, m->xn, m->H, eps);
    if (want_logits && logits && !oracle_matvec(m, "output.weight", m->xn, logits)) return 0;
    return 1;
}

uint32_t oracle_argmax(const float *logits, uint64_t n)
{
    uint64_t best = 0;
    for (uint64_t i = 1; i < n; ++i)
        if (logits[i] > logits[best]) best = i;
    return (uint32_t)best;
}

int oracle_last_hidden(const OracleModel *m, float *out)
{
    if (!m->xn) return 0;
    memcpy(out, m->xn, m->H * 4u);
    return 1;
}

int oracle_kv_row(const OracleModel *m, uint32_t layer, uint64_t pos, float *k, float *v)
{
    if (!m->kc || layer >= m->L || pos >= m->cap) return 0;
    const size_t off = ((size_t)layer * m->cap + pos) * m->kvd;
    memcpy(k, m->kc + off, m->kvd * 4u);
    memcpy(v, m->vc + off, m->kvd * 4u);
    return 1;
}
