/*
 * atlas_dynamic_infer on libatlas_cuda: the reference CLI's contract
 * (run_main_utf8, src/brain_runtime.c:1921-2064) over the library's fast
 * path - batched prefill of the prompt, then the CUDA-graph decode step.
 *
 *   atlas_dynamic_infer model.gguf "prompt" [max_new 1..768] [min_new] [second_model.gguf] [--confidence]
 *   atlas_dynamic_infer model.gguf --gpu-check
 *
 * Kept from the reference: argv and its checks, exit codes (0 ok, 1 model /
 * inference failure, 2 usage), the chat template, the byte-level BPE
 * tokenizer and its pre-tokenization rules (:636-914), prompt truncation at
 * the reference's context (min(context_length, 8192), 2048 without one), the
 * sampler (atlas_sample_token :1783-1861: greedy when min_new is 0, else
 * top-40 at temperature 0.35 with a 1.12 repetition penalty over the last 32
 * generated tokens, xorshift64* seeded from the clock and the pid), the stop
 * tokens, the two-model routing and the confidence line (:1875-1913), stdout
 * text, the stderr device line. Greedy decoding without --confidence runs
 * whole chunks of steps on the GPU (picks made by the device); every other
 * mode reads each step's logits back for the host sampler.
 */
#include <ctype.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <unistd.h>

#include "atlas_runtime.h"
#include "gpu_matvec.h"

/* --------------------------------------------------- GGUF string arrays -- */

typedef struct {
    const uint8_t *p, *end;
} Rd;

static int rd_bytes(Rd *r, void *dst, size_t n)
{
    if ((size_t)(r->end - r->p) < n) return 0;
    memcpy(dst, r->p, n);
    r->p += n;
    return 1;
}
static int rd_u32(Rd *r, uint32_t *v) { return rd_bytes(r, v, 4); }
static int rd_u64(Rd *r, uint64_t *v) { return rd_bytes(r, v, 8); }

/* A GGUF string: u64 length + bytes (returned NUL-terminated, malloc'd). */
static char *rd_str(Rd *r)
{
    uint64_t n;
    if (!rd_u64(r, &n) || n > (uint64_t)(r->end - r->p) || n > (16u << 20)) return NULL;
    char *s = malloc((size_t)n + 1);
    if (!s) return NULL;
    memcpy(s, r->p, (size_t)n);
    s[n] = 0;
    r->p += n;
    return s;
}

static int skip_value(Rd *r, uint32_t type)
{
    static const uint8_t size[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
    if (type == 8) {   /* string */
        uint64_t n;
        if (!rd_u64(r, &n) || n > (uint64_t)(r->end - r->p)) return 0;
        r->p += n;
        return 1;
    }
    if (type == 9) {   /* array */
        uint32_t et;
        uint64_t n;
        if (!rd_u32(r, &et) || !rd_u64(r, &n)) return 0;
        for (uint64_t i = 0; i < n; ++i)
            if (!skip_value(r, et)) return 0;
        return 1;
    }
    if (type > 12) return 0;
    if ((size_t)(r->end - r->p) < size[type]) return 0;
    r->p += size[type];
    return 1;
}

typedef struct {
    char **s;
    uint32_t n;
} StrArr;

static void strarr_free(StrArr *a)
{
    for (uint32_t i = 0; i < a->n; ++i) free(a->s[i]);
    free(a->s);
    a->s = NULL;
    a->n = 0;
}

/* tokenizer.ggml.tokens and tokenizer.ggml.merges from the file's metadata
   (load_tokenizer, src/brain_runtime.c:880-914). */
static int read_tokenizer(const uint8_t *file, uint64_t size, StrArr *tok, StrArr *mrg)
{
    Rd r = {file, file + size};
    uint32_t magic, version;
    uint64_t nt, nkv;
    if (!rd_u32(&r, &magic) || !rd_u32(&r, &version) || !rd_u64(&r, &nt) || !rd_u64(&r, &nkv)) return 0;
    for (uint64_t i = 0; i < nkv; ++i) {
        char *key = rd_str(&r);
        uint32_t type;
        if (!key || !rd_u32(&r, &type)) { free(key); return 0; }
        StrArr *dst = NULL;
        if (type == 9) {
            if (!strcmp(key, "tokenizer.ggml.tokens")) dst = tok;
            else if (!strcmp(key, "tokenizer.ggml.merges")) dst = mrg;
        }
        if (dst) {
            uint32_t et;
            uint64_t n;
            if (!rd_u32(&r, &et) || !rd_u64(&r, &n) || et != 8 || n > 1000000 || dst->s) { free(key); return 0; }
            dst->s = calloc((size_t)n ? (size_t)n : 1, sizeof(char *));
            if (!dst->s) { free(key); return 0; }
            for (uint64_t j = 0; j < n; ++j) {
                dst->s[j] = rd_str(&r);
                if (!dst->s[j]) { dst->n = (uint32_t)j; free(key); return 0; }
            }
            dst->n = (uint32_t)n;
        } else if (!skip_value(&r, type)) {
            free(key);
            return 0;
        }
        free(key);
    }
    return tok->n && mrg->n;
}

/* ------------------------------------------------------- byte-level BPE -- */

/* Open-addressing tables: token string -> id, merge pair -> rank. */
typedef struct {
    StrArr tok, mrg;
    const char **left, **right;        /* merge i: left / right pieces (into mrg) */
    uint32_t *tslot, *mslot, tcap, mcap;
    uint32_t byte_cp[256];             /* byte -> code point of the byte-to-unicode map */
} Bpe;

static uint64_t fnv(const char *s, uint64_t h)
{
    for (; *s; ++s) { h ^= (unsigned char)*s; h *= 1099511628211ull; }
    return h;
}
static uint64_t hash_pair(const char *a, const char *b) { return fnv(b, fnv(a, 1469598103934665603ull) * 31u + 7u); }

/* printable bytes map to themselves, the others to 256, 257, ... in order (GPT-2's byte map) */
static int byte_printable(unsigned b) { return (b >= 33 && b <= 126) || (b >= 161 && b <= 172) || (b >= 174 && b <= 255); }

static int bpe_init(Bpe *t)
{
    unsigned extra = 0;
    for (unsigned b = 0; b < 256; ++b) t->byte_cp[b] = byte_printable(b) ? b : 256 + extra++;
    t->tcap = 1; while (t->tcap < 2 * t->tok.n) t->tcap <<= 1;
    t->mcap = 1; while (t->mcap < 2 * t->mrg.n) t->mcap <<= 1;
    t->tslot = calloc(t->tcap, 4);
    t->mslot = calloc(t->mcap, 4);
    t->left = calloc(t->mrg.n, sizeof(char *));
    t->right = calloc(t->mrg.n, sizeof(char *));
    if (!t->tslot || !t->mslot || !t->left || !t->right) return 0;
    for (uint32_t i = 0; i < t->tok.n; ++i) {
        uint32_t s = (uint32_t)fnv(t->tok.s[i], 1469598103934665603ull) & (t->tcap - 1);
        while (t->tslot[s]) s = (s + 1) & (t->tcap - 1);
        t->tslot[s] = i + 1;
    }
    for (uint32_t i = 0; i < t->mrg.n; ++i) {
        char *sp = strchr(t->mrg.s[i], ' ');
        if (!sp) return 0;
        *sp = 0;
        t->left[i] = t->mrg.s[i];
        t->right[i] = sp + 1;
        uint32_t s = (uint32_t)hash_pair(t->left[i], t->right[i]) & (t->mcap - 1);
        while (t->mslot[s]) s = (s + 1) & (t->mcap - 1);
        t->mslot[s] = i + 1;
    }
    return 1;
}

static int bpe_id(const Bpe *t, const char *s, uint32_t *id)
{
    uint32_t k = (uint32_t)fnv(s, 1469598103934665603ull) & (t->tcap - 1);
    for (; t->tslot[k]; k = (k + 1) & (t->tcap - 1))
        if (!strcmp(t->tok.s[t->tslot[k] - 1], s)) { *id = t->tslot[k] - 1; return 1; }
    return 0;
}

static uint32_t bpe_rank(const Bpe *t, const char *a, const char *b)
{
    uint32_t k = (uint32_t)hash_pair(a, b) & (t->mcap - 1);
    for (; t->mslot[k]; k = (k + 1) & (t->mcap - 1)) {
        const uint32_t i = t->mslot[k] - 1;
        if (!strcmp(t->left[i], a) && !strcmp(t->right[i], b)) return i;
    }
    return UINT32_MAX;
}

static size_t utf8_put(uint32_t cp, char *o)
{
    if (cp < 0x80) { o[0] = (char)cp; return 1; }
    if (cp < 0x800) { o[0] = (char)(0xc0 | (cp >> 6)); o[1] = (char)(0x80 | (cp & 63)); return 2; }
    if (cp < 0x10000) {
        o[0] = (char)(0xe0 | (cp >> 12)); o[1] = (char)(0x80 | ((cp >> 6) & 63)); o[2] = (char)(0x80 | (cp & 63));
        return 3;
    }
    o[0] = (char)(0xf0 | (cp >> 18)); o[1] = (char)(0x80 | ((cp >> 12) & 63));
    o[2] = (char)(0x80 | ((cp >> 6) & 63)); o[3] = (char)(0x80 | (cp & 63));
    return 4;
}

/* One pre-token: every byte as its mapped code point, then merges of the
   lowest-ranked adjacent pair (the leftmost on equal ranks) until none
   applies; the pieces' ids (encode_chunk, src/brain_runtime.c:696-737). */
static size_t encode_chunk(const Bpe *t, const char *bytes, size_t n, uint32_t *out, size_t cap)
{
    if (!n) return 0;
    char **parts = calloc(n, sizeof(char *));
    size_t count = 0, got = 0;
    if (!parts) return 0;
    for (size_t i = 0; i < n; ++i) {
        char tmp[5];
        const size_t len = utf8_put(t->byte_cp[(unsigned char)bytes[i]], tmp);
        tmp[len] = 0;
        if (!(parts[count] = strdup(tmp))) goto done;
        ++count;
    }
    while (count > 1) {
        uint32_t best = UINT32_MAX;
        size_t at = count;
        for (size_t i = 0; i + 1 < count; ++i) {
            const uint32_t r = bpe_rank(t, parts[i], parts[i + 1]);
            if (r < best) { best = r; at = i; }
        }
        if (at == count) break;
        const size_t la = strlen(parts[at]), lb = strlen(parts[at + 1]);
        char *j = malloc(la + lb + 1);
        if (!j) goto done;
        memcpy(j, parts[at], la);
        memcpy(j + la, parts[at + 1], lb + 1);
        free(parts[at]);
        free(parts[at + 1]);
        parts[at] = j;
        memmove(parts + at + 1, parts + at + 2, (count - at - 2) * sizeof(char *));
        --count;
    }
    if (count > cap) goto done;
    for (size_t i = 0; i < count; ++i)
        if (!bpe_id(t, parts[i], &out[i])) goto done;
    got = count;
done:
    for (size_t i = 0; i < count; ++i) free(parts[i]);
    free(parts);
    return got;
}

static int sp_byte(unsigned char c) { return c == ' ' || c == '\t' || c == '\n' || c == '\r'; }
static int word_byte(unsigned char c) { return (c >= 'a' && c <= 'z') || (c >= 'A' && c <= 'Z') || c >= 128; }

/* The reference's pre-tokenization (tokenize_text, src/brain_runtime.c:742-806):
   runs of newlines, of tabs, of spaces (one space stays with the next word),
   English contractions, then runs of letters, of up to 3 digits, or of other
   bytes (which take trailing newlines). */
static size_t tokenize_text(const Bpe *t, const char *text, uint32_t *out, size_t cap)
{
    const size_t n = strlen(text);
    size_t total = 0, pos = 0;
#define EMIT(from, len)                                                        \
    do {                                                                       \
        const size_t g_ = encode_chunk(t, text + (from), (len), out + total, cap - total); \
        if (!g_) return 0;                                                     \
        total += g_;                                                           \
    } while (0)
    while (pos < n) {
        size_t start = pos;
        if (sp_byte((unsigned char)text[pos])) {
            if (text[pos] == '\r' || text[pos] == '\n') {
                while (pos < n && (text[pos] == '\r' || text[pos] == '\n')) ++pos;
                EMIT(start, pos - start);
                continue;
            }
            if (text[pos] == '\t') {
                while (pos < n && text[pos] == '\t') ++pos;
                EMIT(start, pos - start);
                continue;
            }
            while (pos < n && text[pos] == ' ') ++pos;
            const size_t spaces = pos - start;
            if (pos == n) { EMIT(start, spaces); break; }
            if (spaces > 1) {
                EMIT(start, spaces - 1);
                start = pos - 1;
            } else if (!sp_byte((unsigned char)text[pos])) {
                start = pos - 1;
            }
        }
        const unsigned char c = (unsigned char)text[pos];
        if (c == '\'') {
            static const char *forms[] = {"'s", "'t", "'re", "'ve", "'m", "'ll", "'d"};
            size_t matched = 0;
            for (size_t f = 0; f < sizeof(forms) / sizeof(forms[0]) && !matched; ++f) {
                const size_t len = strlen(forms[f]);
                if (pos + len <= n && !strncasecmp(text + pos, forms[f], len)) matched = len;
            }
            if (matched) {
                EMIT(start, pos - start + matched);
                pos += matched;
                continue;
            }
        }
        const int kind = word_byte(c) ? 1 : ((c >= '0' && c <= '9') ? 2 : 3);
        size_t end = pos + 1;
        while (end < n) {
            const unsigned char d = (unsigned char)text[end];
            const int dk = word_byte(d) ? 1 : ((d >= '0' && d <= '9') ? 2 : (sp_byte(d) ? 0 : 3));
            if (dk != kind || dk == 0) break;
            if (kind == 2 && end - pos >= 3) break;
            ++end;
        }
        if (kind == 3)
            while (end < n && (text[end] == '\r' || text[end] == '\n')) ++end;
        EMIT(start, end - start);
        pos = end;
    }
#undef EMIT
    return total;
}

/* Special tokens written as <|name|> become their ids; the text between is
   tokenized (tokenize_prompt, src/brain_runtime.c:808-840). */
static size_t tokenize_prompt(const Bpe *t, const char *text, uint32_t *out, size_t cap)
{
    const size_t n = strlen(text);
    size_t total = 0, start = 0;
    for (size_t i = 0; i < n;) {
        if (i + 2 < n && text[i] == '<' && text[i + 1] == '|') {
            const char *e = strstr(text + i, "|>");
            if (e) {
                const size_t endpos = (size_t)(e - text) + 2;
                char *special = strndup(text + i, endpos - i);
                uint32_t id;
                if (!special) return 0;
                if (bpe_id(t, special, &id)) {
                    char *piece = strndup(text + start, i - start);
                    free(special);
                    if (!piece) return 0;
                    const size_t got = tokenize_text(t, piece, out + total, cap - total);
                    free(piece);
                    if ((i > start && !got) || total + got + 1 > cap) return 0;
                    total += got;
                    out[total++] = id;
                    i = endpos;
                    start = i;
                    continue;
                }
                free(special);
            }
        }
        ++i;
    }
    char *piece = strndup(text + start, n - start);
    if (!piece) return 0;
    const size_t got = tokenize_text(t, piece, out + total, cap - total);
    free(piece);
    if ((n > start && !got) || total + got > cap) return 0;
    return total + got;
}

/* Token text back to bytes: code points of the byte map -> their bytes;
   special tokens (<|...|>) print nothing (decode_token, :853-878). */
static void decode_token(const Bpe *t, uint32_t id, FILE *out)
{
    if (id >= t->tok.n) return;
    const unsigned char *s = (const unsigned char *)t->tok.s[id];
    if (s[0] == '<' && s[1] == '|') return;
    const size_t n = strlen((const char *)s);
    for (size_t i = 0; i < n;) {
        uint32_t cp = s[i];
        size_t used = 1;
        if ((s[i] & 0xe0) == 0xc0 && n - i >= 2) { cp = ((s[i] & 31u) << 6) | (s[i + 1] & 63u); used = 2; }
        else if ((s[i] & 0xf0) == 0xe0 && n - i >= 3) {
            cp = ((s[i] & 15u) << 12) | ((s[i + 1] & 63u) << 6) | (s[i + 2] & 63u);
            used = 3;
        } else if ((s[i] & 0xf8) == 0xf0 && n - i >= 4) {
            cp = ((s[i] & 7u) << 18) | ((s[i + 1] & 63u) << 12) | ((s[i + 2] & 63u) << 6) | (s[i + 3] & 63u);
            used = 4;
        }
        i += used;
        int found = 0;
        for (unsigned b = 0; b < 256 && !found; ++b)
            if (t->byte_cp[b] == cp) { fputc((int)b, out); found = 1; }
        if (!found && cp < 256) fputc((int)cp, out);
    }
}

/* ------------------------------------------------------------- sampler -- */

static uint64_t rng_next(uint64_t *s)   /* xorshift64*, as atlas_random_u64 (:1776-1781) */
{
    uint64_t x = *s;
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    *s = x;
    return x * 2685821657736338717ull;
}

static int is_stop(const char *tok) { return !strcmp(tok, "<|im_end|>") || !strcmp(tok, "<|endoftext|>"); }

/* atlas_sample_token (:1783-1861): the 40 largest (penalised) logits kept in
   a min-heap in vocabulary order, temperature 0.35, the 1.12 repetition
   penalty on the last 32 generated tokens (not when greedy), the pick's
   softmax probability as the step's confidence; greedy takes the heap's
   first largest entry. */
static uint32_t sample(const float *logits, const Bpe *t, uint32_t vocab, const uint32_t *hist, size_t nhist,
                       int allow_stop, int greedy, uint64_t *rng, float *confidence)
{
    enum { K = 40, RECENT = 32 };
    uint32_t ids[K] = {0};
    float vals[K];
    for (int k = 0; k < K; ++k) vals[k] = -INFINITY;
    float lmax = -INFINITY;
    double lsum = 0.0;
    const size_t first = nhist > RECENT ? nhist - RECENT : 0;
    unsigned cnt = 0;
    for (uint32_t i = 0; i < vocab; ++i) {
        if (!allow_stop && i < t->tok.n && is_stop(t->tok.s[i])) continue;
        float v = logits[i];
        for (size_t h = first; !greedy && h < nhist; ++h)
            if (hist[h] == i) { v = v < 0.0f ? v * 1.12f : v / 1.12f; break; }
        const float sc = v / 0.35f;
        if (sc > lmax) { lsum = lsum * exp((double)(lmax - sc)) + 1.0; lmax = sc; }
        else lsum += exp((double)(sc - lmax));
        if (cnt < K) {
            unsigned c = cnt++;
            vals[c] = v;
            ids[c] = i;
            while (c > 0) {
                const unsigned p = (c - 1) / 2;
                if (vals[p] <= vals[c]) break;
                float tv = vals[p]; vals[p] = vals[c]; vals[c] = tv;
                uint32_t ti = ids[p]; ids[p] = ids[c]; ids[c] = ti;
                c = p;
            }
        } else if (v > vals[0]) {
            unsigned p = 0;
            vals[0] = v;
            ids[0] = i;
            for (;;) {
                const unsigned l = 2 * p + 1;
                if (l >= K) break;
                const unsigned r = l + 1, c = (r < K && vals[r] < vals[l]) ? r : l;
                if (vals[p] <= vals[c]) break;
                float tv = vals[p]; vals[p] = vals[c]; vals[c] = tv;
                uint32_t ti = ids[p]; ids[p] = ids[c]; ids[c] = ti;
                p = c;
            }
        }
    }
    float mx = -INFINITY;
    for (unsigned k = 0; k < K; ++k) if (vals[k] > mx) mx = vals[k];
    if (!isfinite(mx)) return 0;
    float w[K], total = 0.0f;
    for (unsigned k = 0; k < K; ++k) {
        w[k] = isfinite(vals[k]) ? expf((vals[k] - mx) / 0.35f) : 0.0f;
        total += w[k];
    }
    unsigned best = 0;
    for (unsigned k = 1; k < K; ++k) if (vals[k] > vals[best]) best = k;
    if (confidence)
        *confidence = total > 0.0f && lsum > 0.0 ? (float)(exp((double)(vals[best] / 0.35f - lmax)) / lsum) : 0.0f;
    if (greedy) return ids[best];
    double pick = ((double)(rng_next(rng) >> 11) * (1.0 / 9007199254740992.0)) * total;
    for (unsigned k = 0; k < K; ++k)
        if ((pick -= w[k]) <= 0.0) return ids[k];
    return ids[best];
}

/* ------------------------------------------- request heuristics (text) -- */

static int has_term(const char *s, const char *e, const char *term)
{
    const size_t n = strlen(term);
    if (!n) return 0;
    for (const char *p = s; p + n <= e; ++p) {
        size_t i = 0;
        while (i < n && tolower((unsigned char)p[i]) == tolower((unsigned char)term[i])) ++i;
        if (i == n) return 1;
    }
    return 0;
}

/* The last user turn of a chat-formatted prompt (or the whole text). */
static void last_turn(const char *prompt, const char **s, const char **e)
{
    static const char tag[] = "<|im_start|>user\n";
    const char *last = prompt, *scan = prompt;
    while ((scan = strstr(scan, tag)) != NULL) { last = scan + sizeof(tag) - 1; scan = last; }
    const char *end = strstr(last, "<|im_end|>");
    *s = last;
    *e = end ? end : last + strlen(last);
}

/* request_coder_prior (:1875-1897): code-related terms of the last user turn
   (the first six weigh 2) route a two-model call to the first (coder) model. */
static float coder_prior(const char *prompt)
{
    static const char *terms[] = {"code", "program", "programming", "compiler", "compile", "debug", "implement",
                                  "source", "header", "pointer", "array", "syntax", "segfault", "algorithm",
                                  "makefile", "gcc", "api", "bug", "in c", "c code", "c program",
                                  "write a function", "implement a function", "c function", "function in c"};
    const char *s, *e;
    last_turn(prompt, &s, &e);
    float score = 0.0f;
    for (size_t i = 0; i < sizeof(terms) / sizeof(terms[0]); ++i)
        if (has_term(s, e, terms[i])) score += i < 6 ? 2.0f : 1.0f;
    if (score <= 0.0f) return 0.20f;
    const float p = 0.50f + 0.08f * score;
    return p > 0.85f ? 0.85f : p;
}

/* request_difficulty_factor (:1899-1913): reasoning or factual-question terms
   scale the confidence by 0.20. */
static float difficulty_factor(const char *prompt)
{
    static const char *terms[] = {"prove", "proof", "derive", "step by step", "reason through", "analyze",
                                  "analyse", "compare", "design", "debug", "optimize", "optimise", "edge case",
                                  "architecture", "trade-off", "tradeoff", "multiple constraints", "large problem",
                                  "complex problem", "break down", "multi-step", "multi step", "work through",
                                  "plan the steps", "why", "what is", "what are", "who is", "who was", "where is",
                                  "when did", "which one", "how does", "how do", "is it true", "explain",
                                  "definition", "historically", "cause of"};
    const char *s, *e;
    last_turn(prompt, &s, &e);
    for (size_t i = 0; i < sizeof(terms) / sizeof(terms[0]); ++i)
        if (has_term(s, e, terms[i])) return 0.20f;
    return 1.0f;
}

#ifdef ATLAS_CLI_LIBRARY
/* The tokenizer alone (tests compare it with the reference's): the ids of
   tokenize_prompt over the file's vocabulary, or -1. */
int cli_tokenize(const char *path, const char *text, uint32_t *out, uint64_t cap)
{
    FILE *f = fopen(path, "rb");
    if (!f) return -1;
    fseek(f, 0, SEEK_END);
    const long size = ftell(f);
    fseek(f, 0, SEEK_SET);
    uint8_t *buf = malloc((size_t)size);
    const int okr = buf && fread(buf, 1, (size_t)size, f) == (size_t)size;
    fclose(f);
    Bpe t;
    memset(&t, 0, sizeof(t));
    int n = -1;
    if (okr && read_tokenizer(buf, (uint64_t)size, &t.tok, &t.mrg) && bpe_init(&t))
        n = (int)tokenize_prompt(&t, text, out, (size_t)cap);
    strarr_free(&t.tok);
    strarr_free(&t.mrg);
    free(t.left); free(t.right); free(t.tslot); free(t.mslot);
    free(buf);
    return n;
}
#else

/* ------------------------------------------------------------ --gpu-check -- */

#include <cuda_runtime.h>

static uint32_t blk_elems(uint32_t t) { return t == 1 ? 1 : (t == 6 || t == 7 || t == 8) ? 32 : (t >= 12 && t <= 14) ? 256 : 0; }
static uint32_t blk_bytes(uint32_t t)
{
    switch (t) {
    case 1: return 2;
    case 6: return 22;
    case 7: return 24;
    case 8: return 34;
    case 12: return 144;
    case 13: return 176;
    case 14: return 210;
    default: return 0;
    }
}

/* The reference's self-test (:1958-1984): y = W x through the device plugin
   (brain_gpu_matvec, the reference's own entry point) against W dequantized
   bit-exactly on the GPU and multiplied in double on the host. */
static int gpu_check(AtlasRuntime *rt, const uint8_t *file, uint64_t size)
{
    const char *names[2] = {"blk.0.attn_q.weight", "blk.0.attn_v.weight"};
    const int init = brain_gpu_init(file, (size_t)size);
    int passed = 1;
    for (int which = 0; which < 2; ++which) {
        AtlasTensorInfo t;
        if (!atlas_rt_find_tensor(rt, names[which], &t) || t.n_dims != 2 || !blk_bytes(t.type)) { passed = 0; break; }
        const uint64_t cols = t.dims[0], rows = t.dims[1], n = rows * cols, nb = n / blk_elems(t.type);
        float *x = malloc(cols * 4), *gpu = malloc(rows * 4), *w = malloc(n * 4);
        void *d_blk = NULL, *d_w = NULL;
        int ok = x && gpu && w && init;
        if (ok) {
            for (uint64_t i = 0; i < cols; ++i) x[i] = sinf((float)i * 0.0137f) * 0.25f;
            ok = brain_gpu_matvec(atlas_rt_data_base(rt) + t.offset, t.type, rows, cols, x, gpu);
        }
        ok = ok && cudaMalloc(&d_blk, nb * blk_bytes(t.type)) == cudaSuccess && cudaMalloc(&d_w, n * 4) == cudaSuccess &&
             cudaMemcpy(d_blk, file + atlas_rt_data_base(rt) + t.offset, nb * blk_bytes(t.type),
                        cudaMemcpyHostToDevice) == cudaSuccess &&
             atlas_cuda_dequant(t.type, d_blk, nb, (float *)d_w, NULL) == ATLAS_OK &&
             cudaMemcpy(w, d_w, n * 4, cudaMemcpyDeviceToHost) == cudaSuccess;
        double max_error = 0.0, max_value = 0.0;
        for (uint64_t r = 0; ok && r < rows; ++r) {
            double ref = 0.0;
            for (uint64_t c = 0; c < cols; ++c) ref += (double)w[r * cols + c] * (double)x[c];
            const double e = fabs((double)gpu[r] - ref);
            if (e > max_error) max_error = e;
            if (fabs(ref) > max_value) max_value = fabs(ref);
        }
        ok = ok && max_error <= max_value * 0.005 + 0.002;   /* the reference's criterion */
        printf("%s GPU/CPU %s, max error %.6g\n", names[which], ok ? "PASS" : "FAIL", max_error);
        if (!ok) passed = 0;
        free(x); free(gpu); free(w);
        if (d_blk) cudaFree(d_blk);
        if (d_w) cudaFree(d_w);
    }
    brain_gpu_shutdown();
    return passed ? 0 : 1;
}

/* ------------------------------------------------------------------ main -- */

int main(int argc, char **argv)
{
    if (argc < 3 || argc > 7) {
        fprintf(stderr, "Usage: %s model.gguf \"prompt text\" [max_new_tokens] [min_new_tokens] [second_model.gguf]\n",
                argv[0]);
        return 2;
    }
    char *max_end = NULL, *min_end = NULL;
    const unsigned long gen_n = argc >= 4 ? strtoul(argv[3], &max_end, 10) : 32;
    const unsigned long min_n = argc >= 5 ? strtoul(argv[4], &min_end, 10) : 0;
    if (!gen_n || gen_n > 768 || (argc >= 4 && (!max_end || *max_end)) || min_n > gen_n ||
        (argc >= 5 && (!min_end || *min_end))) {
        fprintf(stderr, "max_new_tokens must be between 1 and 768\n");
        return 2;
    }
    const int emit_confidence = !strcmp(argv[argc - 1], "--confidence");
    const int paired = argc >= 6 && strcmp(argv[5], "--confidence") != 0;
    const float prior = paired ? coder_prior(argv[2]) : 1.0f;
    const int use_coder = paired && prior >= 0.50f, use_language = paired && !use_coder;
    const char *model = use_language ? argv[5] : argv[1];

    /* the reference's context: context_length (2048 without one), at most 8192 */
    AtlasRtOptions o;
    memset(&o, 0, sizeof(o));
    o.no_device = 1;
    AtlasRuntime *rt = NULL;
    if (atlas_rt_open(model, &o, &rt)) {
        fprintf(stderr, "%s\n", rt ? atlas_rt_error(rt) : "cannot open the model");
        atlas_rt_close(rt);
        return 1;
    }
    AtlasShape shape;
    atlas_rt_shape(rt, &shape);
    atlas_rt_close(rt);
    rt = NULL;
    const uint32_t ctx = shape.max_context > 8192u ? 8192u : shape.max_context;
    if (getenv("BRAIN_FORCE_CPU") || getenv("BRAIN_HYBRID"))
        fprintf(stderr, "BRAIN_FORCE_CPU / BRAIN_HYBRID ignored: every GEMV runs on the GPU\n");
    memset(&o, 0, sizeof(o));
    o.max_context = ctx;
    o.max_prefill = ctx < 512u ? ctx : 512u;
    if (atlas_rt_open(model, &o, &rt)) {
        fprintf(stderr, "%s\n", rt ? atlas_rt_error(rt) : "cannot open the model");
        atlas_rt_close(rt);
        return 1;
    }
    fprintf(stderr, "Inference device: NVIDIA B200 (libatlas_cuda)\n");
    uint64_t fsize = 0;
    const uint8_t *file = atlas_rt_file_bytes(rt, &fsize);
    Bpe tok;
    memset(&tok, 0, sizeof(tok));
    if (!file || !read_tokenizer(file, fsize, &tok.tok, &tok.mrg) || !bpe_init(&tok)) {
        fprintf(stderr, "Could not load tokenizer vocabulary and BPE merges from GGUF\n");
        atlas_rt_close(rt);
        return 1;
    }
    if (paired)
        fprintf(stderr, "Atlas assigned model weights: coder %.0f%%, language %.0f%%\n", use_coder ? 100.0f : 0.0f,
                use_language ? 100.0f : 0.0f);
    else
        fprintf(stderr, "Atlas using the single-model profile\n");
    int rc = 1;
    uint32_t *ids = NULL;
    float *logits = NULL;
    char *prompt = NULL;
    if (!strcmp(argv[2], "--gpu-check")) {
        rc = gpu_check(rt, file, fsize);
        goto out;
    }
    {
        const size_t max_ids = 8192;
        ids = malloc(max_ids * sizeof(uint32_t));
        prompt = malloc(strlen(argv[2]) + 128);
        if (!ids || !prompt) goto out;
        if (!strncmp(argv[2], "<|im_start|>", 12))
            snprintf(prompt, strlen(argv[2]) + 1, "%s", argv[2]);
        else
            snprintf(prompt, strlen(argv[2]) + 128, "<|im_start|>user\n%s<|im_end|>\n<|im_start|>assistant\n",
                     argv[2]);
        size_t pc = tokenize_prompt(&tok, prompt, ids, max_ids);
        if (!pc) {
            fprintf(stderr, "Prompt tokenization failed\n");
            goto out;
        }
        if (pc + gen_n >= ctx) {   /* keep the last tokens (the reference's truncation) */
            const size_t keep = ctx - gen_n - 1;
            memmove(ids, ids + pc - keep, keep * sizeof(uint32_t));
            pc = keep;
        }
        AtlasTensorInfo out_t;
        if (!atlas_rt_find_tensor(rt, "output.weight", &out_t)) {   /* 1: found */
            fprintf(stderr, "output.weight missing\n");
            goto out;
        }
        const uint32_t vocab = (uint32_t)out_t.dims[1];
        /* greedy without a confidence line: the picks are made on the device */
        const int device_picks = min_n == 0 && !emit_confidence;
        logits = device_picks ? NULL : malloc((size_t)vocab * sizeof(float));
        if (!device_picks && !logits) goto out;
        uint32_t next = 0;
        if (atlas_rt_prefill(rt, ids, (uint32_t)pc, 0, logits, &next)) {
            fprintf(stderr, "Inference failed: %s\n", atlas_rt_error(rt));
            goto out;
        }
        fprintf(stderr, "Prompt: %zu/%zu tokens\n", pc, pc);
        struct timespec ts, tr;
        clock_gettime(CLOCK_MONOTONIC, &ts);
        clock_gettime(CLOCK_REALTIME, &tr);
        uint64_t rng = ((uint64_t)ts.tv_sec * 1000000000ull + (uint64_t)ts.tv_nsec) ^ ((uint64_t)getpid() << 32) ^
                       ((uint64_t)tr.tv_sec * 1000ull + (uint64_t)tr.tv_nsec / 1000000ull);
        if (!rng) rng = 0x9e3779b97f4a7c15ull;
        double conf_sum = 0.0;
        unsigned conf_n = 0;
        int hit_limit = 1, ok = 1;
        uint32_t picks[64];
        size_t have = 0, used = 0;   /* device picks: picks[used..have) are the next steps' tokens */
        for (unsigned long step = 0; step < gen_n; ++step) {
            float c = 0.0f;
            if (device_picks) {
                if (step == 0) {
                    picks[0] = next;
                    have = 1;
                    used = 0;
                }
                if (used == have) {
                    /* more steps on the device: each pick fed back at the next position */
                    const size_t m = gen_n - step < 64 ? (size_t)(gen_n - step) : 64;
                    if (atlas_rt_generate(rt, picks[have - 1], (uint32_t)(pc + step - 1), (uint32_t)m, picks)) {
                        ok = 0;
                        break;
                    }
                    have = m;
                    used = 0;
                }
                next = picks[used++];
            } else {
                next = sample(logits, &tok, vocab, ids + pc, step, step >= min_n, min_n == 0, &rng, &c);
            }
            if (next < tok.tok.n && is_stop(tok.tok.s[next])) {
                hit_limit = 0;
                break;
            }
            conf_sum += c;
            ++conf_n;
            ids[pc + step] = next;
            decode_token(&tok, next, stdout);
            fflush(stdout);
            if (!device_picks && step + 1 < gen_n &&
                atlas_rt_forward_token(rt, next, (uint32_t)(pc + step), logits, NULL)) {
                ok = 0;
                break;
            }
        }
        fputc('\n', stdout);
        fflush(stdout);
        if (ok && emit_confidence) {
            float conf = conf_n ? (float)(conf_sum / conf_n) : 0.0f;
            conf *= difficulty_factor(argv[2]);
            if (hit_limit) conf *= 0.50f;
            fprintf(stdout, "\036ATLAS_CONFIDENCE=%.4f,TRUNCATED=%d\036\n", conf, hit_limit);
        }
        if (!ok) fprintf(stderr, "Inference failed: %s\n", atlas_rt_error(rt));
        rc = ok ? 0 : 1;
    }
out:
    free(ids);
    free(logits);
    free(prompt);
    strarr_free(&tok.tok);
    strarr_free(&tok.mrg);
    free(tok.left); free(tok.right); free(tok.tslot); free(tok.mslot);
    atlas_rt_close(rt);
    return rc;
}
#endif /* ATLAS_CLI_LIBRARY */
