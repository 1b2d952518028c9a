/*
 * Seeded synthetic Qwen2-family GGUF writer (see include/atlas_synth.h).
 *
 * Layout written (GGUF v3, little endian):
 *   header, metadata (qwen2.* hyper-parameters + byte-level BPE tokenizer),
 *   tensor directory, zero padding to 32, tensor data (each tensor 32-aligned).
 * The reader side of this format is src/brain_runtime.c:401-445 (gguf_open),
 * :312-339 (metadata keys it consumes) and :748-790 (tokenizer arrays).
 */
#define _GNU_SOURCE
#include "atlas_synth.h"

#include <errno.h>
#include <math.h>
#include <omp.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

enum { T_F32 = 0, T_F16 = 1, T_Q5_0 = 6, T_Q5_1 = 7, T_Q8_0 = 8, T_Q4K = 12, T_Q5K = 13, T_Q6K = 14 };
enum { Q4K_BYTES = 144, Q6K_BYTES = 210, QK = 256, ALIGN = 32 };

/* ggml block geometry of the types the writer emits (src/brain_runtime.c:117-136) */
static uint32_t blk_elems(uint32_t t)
{
    return t == T_F16 ? 1u : (t == T_Q5_0 || t == T_Q5_1 || t == T_Q8_0) ? 32u : (t == T_F32 ? 1u : 256u);
}
static uint32_t blk_bytes(uint32_t t)
{
    switch (t) {
    case T_F16: return 2u;
    case T_Q5_0: return 22u;
    case T_Q5_1: return 24u;
    case T_Q8_0: return 34u;
    case T_Q4K: return Q4K_BYTES;
    case T_Q5K: return 176u;
    case T_Q6K: return Q6K_BYTES;
    default: return 0u;
    }
}

/* ---------------- counter-based random numbers ---------------- */

static inline uint64_t mix64(uint64_t z)
{
    z += 0x9e3779b97f4a7c15ULL;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
}

typedef struct { uint64_t s; } Rng;

static inline uint64_t rng_next(Rng *r)
{
    r->s += 0x9e3779b97f4a7c15ULL;
    uint64_t z = r->s;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
}

static inline Rng rng_for(uint64_t seed, uint64_t stream, uint64_t index)
{
    Rng r;
    r.s = mix64(seed ^ mix64(stream * 0x632be59bd9b4e019ULL + 1u) ^ mix64(index + 0x8cb92ba72f3d8dd7ULL));
    return r;
}

static inline double rng_uniform(Rng *r) { return (double)(rng_next(r) >> 11) * (1.0 / 9007199254740992.0); }

static double rng_normal(Rng *r)
{
    double u1 = rng_uniform(r), u2 = rng_uniform(r);
    if (u1 < 1e-300) u1 = 1e-300;
    return sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
}

static void fill_bytes(Rng *r, uint8_t *dst, size_t n)
{
    size_t i = 0;
    for (; i + 8 <= n; i += 8) {
        uint64_t v = rng_next(r);
        memcpy(dst + i, &v, 8);
    }
    if (i < n) {
        uint64_t v = rng_next(r);
        memcpy(dst + i, &v, n - i);
    }
}

/* IEEE binary32 -> binary16, round to nearest even (finite, normal-range input). */
static uint16_t f32_to_f16(float f)
{
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    int32_t e = (int32_t)((x >> 23) & 0xffu) - 127 + 15;
    uint32_t m = x & 0x7fffffu;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        /* subnormal half: shift the full significand */
        if (e < -10) return (uint16_t)sign;
        m |= 0x800000u;
        uint32_t shift = (uint32_t)(14 - e);
        uint32_t h = m >> shift, rem = m & ((1u << shift) - 1u), half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (h & 1u))) ++h;
        return (uint16_t)(sign | h);
    }
    uint32_t h = sign | ((uint32_t)e << 10) | (m >> 13);
    uint32_t rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
    return (uint16_t)h;
}

static inline uint16_t scale_f16(Rng *r) { return f32_to_f16((float)(1e-4 + 1.9e-3 * rng_uniform(r))); }

static void gen_q4k_block(Rng *r, uint8_t *b)
{
    uint16_t d = scale_f16(r), dmin = scale_f16(r);
    memcpy(b, &d, 2);
    memcpy(b + 2, &dmin, 2);
    fill_bytes(r, b + 4, Q4K_BYTES - 4); /* 12 scale/min bytes + 128 nibble bytes */
}

static void gen_q6k_block(Rng *r, uint8_t *b)
{
    fill_bytes(r, b, 192); /* ql[128], qh[64] */
    uint64_t v = rng_next(r), w = rng_next(r);
    for (int i = 0; i < 16; ++i) {
        uint64_t src = i < 8 ? v >> (8 * i) : w >> (8 * (i - 8));
        b[192 + i] = (uint8_t)(int8_t)((int)(src & 63u) - 32);
    }
    uint16_t d = scale_f16(r);
    memcpy(b + 208, &d, 2);
}

/* Blocks of the other types: scale fields as Q4_K's d, every other byte uniform. */
static void gen_other_block(Rng *r, uint32_t type, uint8_t *b)
{
    if (type == T_F16) {
        uint16_t h = f32_to_f16((float)(-0.05 + 0.1 * rng_uniform(r)));
        memcpy(b, &h, 2);
        return;
    }
    uint16_t d = scale_f16(r);
    memcpy(b, &d, 2);
    uint32_t head = 2;
    if (type == T_Q5_1 || type == T_Q5K) {   /* m / dmin */
        uint16_t m = scale_f16(r);
        memcpy(b + 2, &m, 2);
        head = 4;
    }
    fill_bytes(r, b + head, blk_bytes(type) - head);
}

void atlas_synth_q4k_blocks(uint64_t seed, uint64_t stream, uint8_t *dst, uint64_t n)
{
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i) {
        Rng r = rng_for(seed, stream, (uint64_t)i);
        gen_q4k_block(&r, dst + (uint64_t)i * Q4K_BYTES);
    }
}

void atlas_synth_q6k_blocks(uint64_t seed, uint64_t stream, uint8_t *dst, uint64_t n)
{
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i) {
        Rng r = rng_for(seed, stream, (uint64_t)i);
        gen_q6k_block(&r, dst + (uint64_t)i * Q6K_BYTES);
    }
}

/* ---------------- growable byte buffer ---------------- */

typedef struct { uint8_t *p; size_t n, cap; int oom; } Buf;

static void buf_put(Buf *b, const void *src, size_t n)
{
    if (b->oom) return;
    if (b->n + n > b->cap) {
        size_t cap = b->cap ? b->cap : 1u << 20;
        while (cap < b->n + n) cap *= 2;
        uint8_t *p = (uint8_t *)realloc(b->p, cap);
        if (!p) { b->oom = 1; return; }
        b->p = p;
        b->cap = cap;
    }
    memcpy(b->p + b->n, src, n);
    b->n += n;
}

static void put_u32(Buf *b, uint32_t v) { buf_put(b, &v, 4); }
static void put_u64(Buf *b, uint64_t v) { buf_put(b, &v, 8); }
static void put_str(Buf *b, const char *s) { put_u64(b, strlen(s)); buf_put(b, s, strlen(s)); }
static void kv_str(Buf *b, const char *k, const char *v) { put_str(b, k); put_u32(b, 8); put_str(b, v); }
static void kv_u32(Buf *b, const char *k, uint32_t v) { put_str(b, k); put_u32(b, 4); put_u32(b, v); }
static void kv_f32(Buf *b, const char *k, float v) { put_str(b, k); put_u32(b, 6); buf_put(b, &v, 4); }

/* ---------------- tokenizer vocabulary ---------------- */

/* GPT-2 byte -> code point map, as the reference's encode_chunk computes it
   (src/brain_runtime.c:717-724). */
static unsigned byte_code_point(unsigned b)
{
    int printable = (b >= 33 && b <= 126) || (b >= 161 && b <= 172) || (b >= 174 && b <= 255);
    if (printable) return b;
    unsigned offset = 0;
    for (unsigned x = 0; x < b; ++x) {
        int px = (x >= 33 && x <= 126) || (x >= 161 && x <= 172) || (x >= 174 && x <= 255);
        if (!px) ++offset;
    }
    return 256u + offset;
}

static size_t utf8_encode(unsigned cp, char *out)
{
    if (cp < 0x80u) { out[0] = (char)cp; out[1] = 0; return 1; }
    if (cp < 0x800u) {
        out[0] = (char)(0xc0u | (cp >> 6)); out[1] = (char)(0x80u | (cp & 63u)); out[2] = 0; return 2;
    }
    out[0] = (char)(0xe0u | (cp >> 12)); out[1] = (char)(0x80u | ((cp >> 6) & 63u));
    out[2] = (char)(0x80u | (cp & 63u)); out[3] = 0; return 3;
}

/* A few merges over byte symbols; "\xC4\xA0" is the symbol for a space byte. */
static const char *const k_merges[][2] = {
    {"t", "h"}, {"i", "n"}, {"e", "r"}, {"a", "n"}, {"o", "n"}, {"r", "e"},
    {"\xC4\xA0", "t"}, {"\xC4\xA0", "a"}, {"th", "e"}, {"\xC4\xA0t", "he"},
    {"e", "n"}, {"a", "t"}, {"o", "r"}, {"e", "s"}, {"i", "s"}, {"\xC4\xA0", "s"},
};
enum { N_MERGES = (int)(sizeof(k_merges) / sizeof(k_merges[0])) };

static void put_vocab(Buf *b, uint32_t vocab)
{
    put_str(b, "tokenizer.ggml.tokens");
    put_u32(b, 9);
    put_u32(b, 8);
    put_u64(b, vocab);
    char tmp[64];
    for (uint32_t i = 0; i < vocab; ++i) {
        if (i + 3 >= vocab) {
            const char *special[3] = {"<|endoftext|>", "<|im_start|>", "<|im_end|>"};
            put_str(b, special[i + 3 - vocab]);
        } else if (i < 256) {
            utf8_encode(byte_code_point(i), tmp);
            put_str(b, tmp);
        } else if (i < 256u + N_MERGES) {
            snprintf(tmp, sizeof(tmp), "%s%s", k_merges[i - 256][0], k_merges[i - 256][1]);
            put_str(b, tmp);
        } else {
            snprintf(tmp, sizeof(tmp), "w%u", i);
            put_str(b, tmp);
        }
    }
    put_str(b, "tokenizer.ggml.merges");
    put_u32(b, 9);
    put_u32(b, 8);
    put_u64(b, N_MERGES);
    for (int i = 0; i < N_MERGES; ++i) {
        snprintf(tmp, sizeof(tmp), "%s %s", k_merges[i][0], k_merges[i][1]);
        put_str(b, tmp);
    }
}

/* ---------------- tensor plan ---------------- */

typedef struct {
    char name[96];
    uint32_t type, n_dims;
    uint64_t dims[2];
    uint64_t offset, bytes;
    int alias_of;     /* -1, or the index whose data this entry reuses */
    int init;         /* 0 quant, 1 norm weight, 2 bias */
} Plan;

static uint64_t tensor_bytes(uint32_t type, uint64_t cols, uint64_t rows)
{
    if (type == T_F32) return cols * rows * 4u;
    return cols / blk_elems(type) * rows * blk_bytes(type);
}

static int build_plan(const AtlasSynthConfig *c, Plan **out, int *count)
{
    uint32_t H = c->hidden, qd = c->q_heads * c->head_dim, kvd = c->kv_heads * c->head_dim;
    int n = 3 + (int)c->layers * ((c->qkv_bias ? 12 : 9) + (c->qk_norm ? 2 : 0)) + 1;
    Plan *p = (Plan *)calloc((size_t)n, sizeof(Plan));
    if (!p) return -1;
    int k = 0;
#define ADD(NAME, TYPE, COLS, ROWS, INIT) do {                              \
        snprintf(p[k].name, sizeof(p[k].name), "%s", NAME);                 \
        p[k].type = TYPE; p[k].dims[0] = COLS; p[k].dims[1] = ROWS;         \
        p[k].n_dims = (ROWS) == 1 ? 1u : 2u; p[k].alias_of = -1;            \
        p[k].init = INIT; ++k;                                              \
    } while (0)
    const uint32_t alt = (uint32_t)c->alt_type;
    ADD("token_embd.weight", (alt && c->tied) ? alt : T_Q6K, H, c->vocab, 0);
    ADD("output_norm.weight", T_F32, H, 1, 1);
    ADD("output.weight", alt ? alt : T_Q6K, H, c->vocab, 0);   /* tied: an alias of token_embd, same type */
    if (c->tied) p[k - 1].alias_of = 0;
    char nm[96];
    for (uint32_t l = 0; l < c->layers; ++l) {
#define LADD(SUFFIX, TYPE, COLS, ROWS, INIT) do {                             \
        snprintf(nm, sizeof(nm), "blk.%u.%s", l, SUFFIX);                   \
        ADD(nm, TYPE, COLS, ROWS, INIT);                                    \
    } while (0)
        LADD("attn_norm.weight", T_F32, H, 1, 1);
        LADD("attn_q.weight", alt ? alt : T_Q4K, H, qd, 0);
        LADD("attn_k.weight", T_Q4K, H, kvd, 0);
        const int odd = c->layer_mix && (l & 1u);   /* types that change across layers */
        LADD("attn_v.weight", odd ? T_Q4K : T_Q6K, H, kvd, 0);
        if (c->qkv_bias) {
            LADD("attn_q.bias", T_F32, qd, 1, 2);
            LADD("attn_k.bias", T_F32, kvd, 1, 2);
            LADD("attn_v.bias", T_F32, kvd, 1, 2);
        }
        if (c->qk_norm) {
            LADD("attn_q_norm.weight", T_F32, c->head_dim, 1, 1);
            LADD("attn_k_norm.weight", T_F32, c->head_dim, 1, 1);
        }
        LADD("attn_output.weight", T_Q4K, qd, H, 0);
        LADD("ffn_norm.weight", T_F32, H, 1, 1);
        LADD("ffn_gate.weight", alt ? alt : T_Q4K, H, c->ffn, 0);
        LADD("ffn_up.weight", alt ? alt : T_Q4K, H, c->ffn, 0);
        LADD("ffn_down.weight", odd ? T_Q4K : alt ? alt : T_Q6K, c->ffn, H, 0);
#undef LADD
    }
#undef ADD
    uint64_t off = 0;
    for (int i = 0; i < k; ++i) {
        p[i].bytes = tensor_bytes(p[i].type, p[i].dims[0], p[i].dims[1]);
        if (p[i].alias_of >= 0) { p[i].offset = p[p[i].alias_of].offset; continue; }
        off = (off + ALIGN - 1) / ALIGN * ALIGN;
        p[i].offset = off;
        off += p[i].bytes;
    }
    *out = p;
    *count = k;
    return 0;
}

static int validate(const AtlasSynthConfig *c)
{
    if (!c->hidden || !c->layers || !c->q_heads || !c->kv_heads || !c->head_dim || !c->ffn ||
        !c->vocab || c->vocab < 256u + N_MERGES + 3u)
        return -1;
    uint32_t qd = c->q_heads * c->head_dim;
    if (c->hidden % QK || c->ffn % QK || qd % QK || c->q_heads % c->kv_heads) return -1;
    if (c->alt_type && (c->alt_type == T_Q4K || c->alt_type == T_Q6K || !blk_bytes((uint32_t)c->alt_type))) return -1;
    return 0;
}

static Buf build_header(const AtlasSynthConfig *c, const Plan *p, int n)
{
    Buf b = {0};
    put_u32(&b, 0x46554747u);
    put_u32(&b, 3);
    put_u64(&b, (uint64_t)n);
    put_u64(&b, 14);
    const char *arch = c->qk_norm ? "qwen3" : "qwen2";
    char key[96];
#define KEY(SUFFIX) (snprintf(key, sizeof(key), "%s.%s", arch, SUFFIX), key)
    kv_str(&b, "general.architecture", arch);
    kv_str(&b, "general.name", "atlas-synthetic");
    kv_u32(&b, "general.alignment", ALIGN);
    kv_u32(&b, KEY("block_count"), c->layers);
    kv_u32(&b, KEY("context_length"), c->context_length);
    kv_u32(&b, KEY("embedding_length"), c->hidden);
    kv_u32(&b, KEY("feed_forward_length"), c->ffn);
    kv_u32(&b, KEY("attention.head_count"), c->q_heads);
    kv_u32(&b, KEY("attention.head_count_kv"), c->kv_heads);
    kv_f32(&b, KEY("rope.freq_base"), c->rope_base);
    kv_f32(&b, KEY("attention.layer_norm_rms_epsilon"), 1e-6f);
#undef KEY
    kv_str(&b, "tokenizer.ggml.model", "gpt2");
    put_vocab(&b, c->vocab);
    for (int i = 0; i < n; ++i) {
        put_str(&b, p[i].name);
        put_u32(&b, p[i].n_dims);
        for (uint32_t d = 0; d < p[i].n_dims; ++d) put_u64(&b, p[i].dims[d]);
        put_u32(&b, p[i].type);
        put_u64(&b, p[i].offset);
    }
    static const uint8_t zeros[ALIGN] = {0};
    size_t pad = (ALIGN - b.n % ALIGN) % ALIGN;
    buf_put(&b, zeros, pad);
    return b;
}

uint64_t atlas_synth_file_size(const AtlasSynthConfig *c)
{
    Plan *p;
    int n;
    if (validate(c) || build_plan(c, &p, &n)) return 0;
    Buf h = build_header(c, p, n);
    uint64_t end = 0;
    for (int i = 0; i < n; ++i)
        if (p[i].offset + p[i].bytes > end) end = p[i].offset + p[i].bytes;
    uint64_t total = h.oom ? 0 : h.n + end;
    free(h.p);
    free(p);
    return total;
}

int atlas_synth_write_gguf(const AtlasSynthConfig *c, const char *path)
{
    if (validate(c)) { fprintf(stderr, "atlas_synth: invalid shape\n"); return -1; }
    Plan *p;
    int n;
    if (build_plan(c, &p, &n)) return -1;
    Buf h = build_header(c, p, n);
    if (h.oom) { free(h.p); free(p); return -1; }
    FILE *f = fopen(path, "wb");
    if (!f) { fprintf(stderr, "atlas_synth: %s: %s\n", path, strerror(errno)); free(h.p); free(p); return -1; }
    int rc = fwrite(h.p, 1, h.n, f) == h.n ? 0 : -1;
    free(h.p);
    if (c->threads > 0) omp_set_num_threads(c->threads);
    const size_t chunk = (size_t)64 << 20;
    uint8_t *buf = (uint8_t *)malloc(chunk);
    uint64_t written = 0;
    if (!buf) rc = -1;
    for (int t = 0; rc == 0 && t < n; ++t) {
        if (p[t].alias_of >= 0) continue;
        static const uint8_t zeros[ALIGN] = {0};
        if (p[t].offset > written) {
            if (fwrite(zeros, 1, (size_t)(p[t].offset - written), f) != p[t].offset - written) { rc = -1; break; }
            written = p[t].offset;
        }
        if (p[t].type == T_F32) {
            Rng r = rng_for(c->seed, (uint64_t)t, 0);
            uint64_t cnt = p[t].dims[0] * p[t].dims[1];
            float *v = (float *)buf;
            for (uint64_t i = 0; i < cnt; ++i) {
                double z = rng_normal(&r) * 0.02;
                v[i] = (float)(p[t].init == 1 ? 1.0 + z : z);
            }
            if (fwrite(buf, 4, cnt, f) != cnt) rc = -1;
            written += cnt * 4u;
            continue;
        }
        const uint32_t ty = p[t].type;
        size_t bb = blk_bytes(ty);
        uint64_t blocks = p[t].bytes / bb, per = chunk / bb;
        for (uint64_t b0 = 0; rc == 0 && b0 < blocks; b0 += per) {
            uint64_t m = blocks - b0 < per ? blocks - b0 : per;
#pragma omp parallel for schedule(static)
            for (int64_t i = 0; i < (int64_t)m; ++i) {
                Rng r = rng_for(c->seed, (uint64_t)t, b0 + (uint64_t)i);
                if (ty == T_Q4K) gen_q4k_block(&r, buf + (uint64_t)i * bb);
                else if (ty == T_Q6K) gen_q6k_block(&r, buf + (uint64_t)i * bb);
                else gen_other_block(&r, ty, buf + (uint64_t)i * bb);
            }
            if (fwrite(buf, 1, (size_t)(m * bb), f) != m * bb) rc = -1;
            written += m * bb;
        }
    }
    free(buf);
    free(p);
    if (fclose(f) != 0) rc = -1;
    if (rc) fprintf(stderr, "atlas_synth: write failed for %s\n", path);
    return rc;
}
