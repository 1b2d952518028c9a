/*
 * Host runtime (include/atlas_runtime.h): GGUF reader and the reference's
 * model/forward API over libatlas_cuda.
 *
 * The GGUF reader follows the reference's (src/brain_runtime.c:312-445,
 * 507-583): little-endian v2/v3 header, metadata keys matched by suffix
 * (.context_length, .attention.head_count[_kv], .block_count,
 * .rope.freq_base), general.architecture, tensor directory, data base aligned
 * up to 32 bytes. Differences, all documented in atlas_runtime.h: the file is
 * mmap'd instead of copied into RAM; a missing output.weight falls back to
 * token_embd.weight (tied head); the 8192-position cap is not applied.
 */
#define _GNU_SOURCE
#include "atlas_runtime.h"

#include <fcntl.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

struct AtlasRuntime {
    uint8_t *map;
    size_t size;
    uint64_t data_base;
    AtlasTensorInfo *t;
    uint64_t nt;
    size_t *slots;
    size_t cap;
    AtlasShape shape;
    uint32_t md_ctx, md_heads, md_kv_heads, md_layers;
    float md_rope;
    AtlasCuda *dev;
    char err[512];
};

static int rt_fail(AtlasRuntime *rt, int code, const char *fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    if (rt) vsnprintf(rt->err, sizeof(rt->err), fmt, ap);
    va_end(ap);
    return code;
}

typedef struct { const uint8_t *p, *end; int bad; } Cur;

static uint64_t rd(Cur *c, int n)
{
    if (c->bad || c->end - c->p < n) { c->bad = 1; return 0; }
    uint64_t v = 0;
    memcpy(&v, c->p, (size_t)n);
    c->p += n;
    return v;
}

static void skip(Cur *c, uint64_t n)
{
    if (c->bad || (uint64_t)(c->end - c->p) < n) { c->bad = 1; return; }
    c->p += n;
}

/* skip_value, src/brain_runtime.c:265-302 */
static void skip_value(Cur *c, uint32_t type, int depth)
{
    static const int fixed[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
    if (depth > 4) { c->bad = 1; return; }
    if (type == 8) { skip(c, rd(c, 8)); return; }
    if (type == 9) {
        const uint32_t et = (uint32_t)rd(c, 4);
        const uint64_t n = rd(c, 8);
        if (et != 8 && et != 9 && et <= 12) { skip(c, n * (uint64_t)fixed[et]); return; }
        for (uint64_t i = 0; i < n && !c->bad; ++i) skip_value(c, et, depth + 1);
        return;
    }
    if (type > 12) { c->bad = 1; return; }
    skip(c, (uint64_t)fixed[type]);
}

static int suffix(const char *k, size_t n, const char *s)
{
    const size_t m = strlen(s);
    return n >= m && !memcmp(k + n - m, s, m);
}

/* tensor_name_hash, src/brain_runtime.c:163-168: FNV-1a */
static size_t name_hash(const char *s)
{
    size_t h = (size_t)1469598103934665603ull;
    while (*s) { h ^= (unsigned char)*s++; h *= (size_t)1099511628211ull; }
    return h;
}

int atlas_rt_find_tensor(const AtlasRuntime *rt, const char *name, AtlasTensorInfo *out)
{
    if (!rt || !rt->slots) return 0;
    size_t s = name_hash(name) & (rt->cap - 1);
    while (rt->slots[s]) {
        const AtlasTensorInfo *t = &rt->t[rt->slots[s] - 1];
        if (!strcmp(t->name, name)) { if (out) *out = *t; return 1; }
        s = (s + 1) & (rt->cap - 1);
    }
    return 0;
}

static const AtlasTensorInfo *lookup(const AtlasRuntime *rt, const char *name)
{
    size_t s = name_hash(name) & (rt->cap - 1);
    while (rt->slots[s]) {
        const AtlasTensorInfo *t = &rt->t[rt->slots[s] - 1];
        if (!strcmp(t->name, name)) return t;
        s = (s + 1) & (rt->cap - 1);
    }
    return NULL;
}

/* derive_model_shape, src/brain_runtime.c:507-583 (tied-head fallback, no context cap) */
static int derive_shape(AtlasRuntime *rt, uint32_t max_context)
{
    AtlasShape *s = &rt->shape;
    const AtlasTensorInfo *emb = lookup(rt, "token_embd.weight"), *out = lookup(rt, "output.weight");
    const AtlasTensorInfo *q = lookup(rt, "blk.0.attn_q.weight"), *k = lookup(rt, "blk.0.attn_k.weight");
    const AtlasTensorInfo *g = lookup(rt, "blk.0.ffn_gate.weight");
    if (!out) out = emb;
    if (!emb || !q || !k || !g || emb->n_dims != 2 || out->n_dims != 2 || q->n_dims != 2 || k->n_dims != 2 ||
        g->n_dims != 2)
        return rt_fail(rt, ATLAS_EINVAL, "missing or malformed token_embd / attn_q / attn_k / ffn_gate");
    uint32_t max_layer = 0;
    int saw = 0;
    for (uint64_t i = 0; i < rt->nt; ++i) {
        unsigned l;
        if (sscanf(rt->t[i].name, "blk.%u.", &l) == 1) {
            if (!saw || l > max_layer) max_layer = l;
            saw = 1;
        }
    }
    s->hidden_size = (uint32_t)emb->dims[0];
    s->vocab_size = (uint32_t)out->dims[1];
    s->q_dim = (uint32_t)q->dims[1];
    s->kv_dim = (uint32_t)k->dims[1];
    s->ffn_size = (uint32_t)g->dims[1];
    s->q_heads = rt->md_heads;
    if (!s->q_heads || s->q_dim % s->q_heads) return rt_fail(rt, ATLAS_EINVAL, "bad head count");
    s->head_dim = s->q_dim / s->q_heads;
    s->kv_heads = rt->md_kv_heads ? rt->md_kv_heads : (s->head_dim ? s->kv_dim / s->head_dim : 0);
    s->layers = rt->md_layers ? rt->md_layers : (saw ? max_layer + 1 : 0);
    s->max_context = max_context ? max_context : (rt->md_ctx ? rt->md_ctx : 2048);
    s->rope_base = rt->md_rope > 0.0f ? rt->md_rope : 1000000.0f;
    s->has_qk_norm = !strcmp(s->architecture, "qwen3");
    if ((strcmp(s->architecture, "qwen2") && strcmp(s->architecture, "qwen3")) || !s->hidden_size || !s->layers ||
        !s->kv_heads || s->q_heads % s->kv_heads || s->kv_dim % s->head_dim || !s->vocab_size ||
        s->max_context < 2 || (s->head_dim & 1))
        return rt_fail(rt, ATLAS_EINVAL, "unsupported or incomplete architecture '%s'", s->architecture);
    return ATLAS_OK;
}

static int parse(AtlasRuntime *rt, uint32_t max_context)
{
    Cur c = {rt->map, rt->map + rt->size, 0};
    if ((uint32_t)rd(&c, 4) != 0x46554747u) return rt_fail(rt, ATLAS_EINVAL, "not a GGUF file (magic)");
    (void)rd(&c, 4);
    rt->nt = rd(&c, 8);
    const uint64_t nkv = rd(&c, 8);
    for (uint64_t i = 0; i < nkv && !c.bad; ++i) {
        const uint64_t kl = rd(&c, 8);
        if (kl >= 256 || (uint64_t)(c.end - c.p) < kl) { c.bad = 1; break; }
        const char *key = (const char *)c.p;
        c.p += kl;
        const uint32_t ty = (uint32_t)rd(&c, 4);
        if (kl == 20 && !memcmp(key, "general.architecture", 20) && ty == 8) {
            const uint64_t n = rd(&c, 8);
            if ((uint64_t)(c.end - c.p) < n) { c.bad = 1; break; }
            const size_t keep = n < sizeof(rt->shape.architecture) - 1 ? (size_t)n : sizeof(rt->shape.architecture) - 1;
            memcpy(rt->shape.architecture, c.p, keep);
            rt->shape.architecture[keep] = 0;
            c.p += n;
            continue;
        }
        uint32_t *field = NULL;
        if (suffix(key, kl, ".context_length")) field = &rt->md_ctx;
        else if (suffix(key, kl, ".attention.head_count_kv")) field = &rt->md_kv_heads;
        else if (suffix(key, kl, ".attention.head_count")) field = &rt->md_heads;
        else if (suffix(key, kl, ".block_count")) field = &rt->md_layers;
        if (field && (ty == 4 || ty == 5)) { *field = (uint32_t)rd(&c, 4); continue; }
        if (suffix(key, kl, ".rope.freq_base") && ty == 6) {
            const uint32_t bits = (uint32_t)rd(&c, 4);
            memcpy(&rt->md_rope, &bits, 4);
            continue;
        }
        skip_value(&c, ty, 0);
    }
    if (c.bad) return rt_fail(rt, ATLAS_EINVAL, "truncated or malformed GGUF metadata");
    if (rt->nt > 10000000u) return rt_fail(rt, ATLAS_EINVAL, "tensor count out of range");
    rt->cap = 8;
    while (rt->cap < rt->nt * 2) rt->cap *= 2;
    rt->t = (AtlasTensorInfo *)calloc(rt->nt ? rt->nt : 1, sizeof(AtlasTensorInfo));
    rt->slots = (size_t *)calloc(rt->cap, sizeof(size_t));
    if (!rt->t || !rt->slots) return rt_fail(rt, ATLAS_ENOMEM, "out of host memory");
    for (uint64_t i = 0; i < rt->nt && !c.bad; ++i) {
        AtlasTensorInfo *t = &rt->t[i];
        const uint64_t nl = rd(&c, 8);
        if (nl >= sizeof(t->name) || (uint64_t)(c.end - c.p) < nl) { c.bad = 1; break; }
        memcpy(t->name, c.p, nl);
        c.p += nl;
        t->n_dims = (uint32_t)rd(&c, 4);
        if (t->n_dims > 4) { c.bad = 1; break; }
        for (uint32_t d = 0; d < t->n_dims; ++d) t->dims[d] = rd(&c, 8);
        t->type = (uint32_t)rd(&c, 4);
        t->offset = rd(&c, 8);
        size_t s = name_hash(t->name) & (rt->cap - 1);
        while (rt->slots[s]) s = (s + 1) & (rt->cap - 1);
        rt->slots[s] = (size_t)i + 1;
    }
    if (c.bad) return rt_fail(rt, ATLAS_EINVAL, "truncated or malformed GGUF tensor directory");
    rt->data_base = ((uint64_t)(c.p - rt->map) + 31u) & ~(uint64_t)31u;
    return derive_shape(rt, max_context);
}

static uint64_t tensor_bytes(const AtlasTensorInfo *t)
{
    uint64_t e = 1;
    for (uint32_t d = 0; d < t->n_dims; ++d) e *= t->dims[d];
    switch (t->type) {
    case 0: return e * 4;
    case 1: return e * 2;
    case 6: return e / 32 * 22;
    case 7: return e / 32 * 24;
    case 8: return e / 32 * 34;
    case 12: return e / 256 * 144;
    case 13: return e / 256 * 176;
    case 14: return e / 256 * 210;
    default: return 0;
    }
}

int atlas_rt_open(const char *path, const AtlasRtOptions *opt, AtlasRuntime **out)
{
    if (!path || !out) return ATLAS_EINVAL;
    *out = NULL;
    AtlasRuntime *rt = (AtlasRuntime *)calloc(1, sizeof(*rt));
    if (!rt) return ATLAS_ENOMEM;
    AtlasRtOptions o;
    memset(&o, 0, sizeof(o));
    if (opt) o = *opt;
    int rc;
    const int fd = open(path, O_RDONLY);
    struct stat st;
    if (fd < 0 || fstat(fd, &st) != 0 || st.st_size < 24) {
        if (fd >= 0) close(fd);
        rc = rt_fail(rt, ATLAS_EINVAL, "cannot open %s", path);
        *out = rt;
        return rc;
    }
    void *m = mmap(NULL, (size_t)st.st_size, PROT_READ, MAP_SHARED, fd, 0);
    close(fd);
    if (m == MAP_FAILED) { *out = rt; return rt_fail(rt, ATLAS_ENOMEM, "mmap failed"); }
    rt->map = (uint8_t *)m;
    rt->size = (size_t)st.st_size;
    rc = parse(rt, o.max_context);
    if (rc || o.no_device) { *out = rt; return rc; }
    /* Tensor table for the device library: every tensor whose bytes lie inside the file. */
    AtlasTensorDesc *td = (AtlasTensorDesc *)calloc(rt->nt ? rt->nt : 1, sizeof(AtlasTensorDesc));
    if (!td) { *out = rt; return rt_fail(rt, ATLAS_ENOMEM, "out of host memory"); }
    uint32_t n = 0;
    for (uint64_t i = 0; i < rt->nt; ++i) {
        const AtlasTensorInfo *t = &rt->t[i];
        const uint64_t at = rt->data_base + t->offset, bytes = tensor_bytes(t);
        if (!bytes || at > rt->size || bytes > rt->size - at) continue;
        td[n].name = t->name;
        td[n].type = t->type;
        td[n].n_dims = t->n_dims;
        memcpy(td[n].dims, t->dims, sizeof(t->dims));
        td[n].data = rt->map + at;
        ++n;
    }
    madvise(rt->map, rt->size, MADV_SEQUENTIAL);
    const AtlasShape *s = &rt->shape;
    AtlasModelDesc d;
    memset(&d, 0, sizeof(d));
    d.hidden = s->hidden_size; d.q_dim = s->q_dim; d.kv_dim = s->kv_dim; d.q_heads = s->q_heads;
    d.kv_heads = s->kv_heads; d.head_dim = s->head_dim; d.ffn = s->ffn_size; d.layers = s->layers;
    d.vocab = s->vocab_size; d.max_context = s->max_context; d.max_prefill = o.max_prefill;
    d.rope_base = s->rope_base; d.rms_eps = 1.0e-6f; d.has_qk_norm = s->has_qk_norm;
    d.kv_fp16 = o.kv_fp16; d.device = o.device;
    d.tp_rank = o.tp_size > 1 ? o.tp_rank : 0; d.tp_size = o.tp_size > 1 ? o.tp_size : 1;
    d.max_batch = o.max_batch > 1 ? o.max_batch : 1;
    rc = atlas_cuda_create(&d, td, n, &rt->dev);
    free(td);
    if (rc) rt_fail(rt, rc, "%s", atlas_cuda_last_error(NULL));
    *out = rt;
    return rc;
}

void atlas_rt_close(AtlasRuntime *rt)
{
    if (!rt) return;
    if (rt->dev) atlas_cuda_destroy(rt->dev);
    if (rt->map) munmap(rt->map, rt->size);
    free(rt->t);
    free(rt->slots);
    free(rt);
}

const char *atlas_rt_error(const AtlasRuntime *rt) { return rt ? rt->err : "null runtime"; }

int atlas_rt_shape(const AtlasRuntime *rt, AtlasShape *out)
{
    if (!rt || !out) return ATLAS_EINVAL;
    *out = rt->shape;
    return ATLAS_OK;
}

uint64_t atlas_rt_data_base(const AtlasRuntime *rt) { return rt ? rt->data_base : 0; }

const uint8_t *atlas_rt_file_bytes(const AtlasRuntime *rt, uint64_t *size)
{
    if (!rt) return NULL;
    if (size) *size = rt->size;
    return rt->map;
}

AtlasCuda *atlas_rt_device(AtlasRuntime *rt) { return rt ? rt->dev : NULL; }

static int dev_rc(AtlasRuntime *rt, int rc)
{
    if (rc) rt_fail(rt, rc, "%s", atlas_cuda_last_error(rt->dev));
    return rc;
}

int atlas_rt_forward_token(AtlasRuntime *rt, uint32_t token, uint32_t pos, float *logits, uint32_t *argmax)
{
    if (!rt || !rt->dev) return ATLAS_EINVAL;
    return dev_rc(rt, atlas_cuda_decode(rt->dev, token, pos, logits, argmax));
}

int atlas_rt_prefill(AtlasRuntime *rt, const uint32_t *ids, uint32_t n, uint32_t pos0, float *logits, uint32_t *argmax)
{
    if (!rt || !rt->dev) return ATLAS_EINVAL;
    return dev_rc(rt, atlas_cuda_prefill(rt->dev, ids, n, pos0, logits, argmax));
}

int atlas_rt_generate(AtlasRuntime *rt, uint32_t first, uint32_t pos0, uint32_t steps, uint32_t *out_ids)
{
    if (!rt || !rt->dev) return ATLAS_EINVAL;
    return dev_rc(rt, atlas_cuda_generate(rt->dev, first, pos0, steps, out_ids));
}
