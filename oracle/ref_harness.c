/*
 * ORACLE harness around the reference's own dynamic CPU runtime.
 *
 * Test infrastructure only (tests/, __graft_entry__.smoke and bench.py's CPU
 * baseline use it; the product never links it). It compiles
 * src/brain_runtime.c unchanged, in place, as part of this translation unit
 * (the reference's functions are file-static), and exports thin non-static
 * wrappers so tests can call the reference's own code paths:
 *   half_to_float            src/brain_runtime.c:203
 *   dequant_block (Q4_K/Q6_K/Q5_K/Q5_0/Q5_1/Q8_0/F16)  :1085
 *   tensor_matvec_cpu_range  :1162
 *   load_embedding_row       :1311
 *   rms_norm / rope          :1338 / :1377
 *   gqa_single_token         :1482
 *   forward_token            :1698
 *   atlas_sample_token       :1783 (greedy)
 *   run_main_utf8            :1921 (the CLI)
 */
#include "brain_runtime.c"

static GGUFFile g_ref_file;
static Work g_ref_work;
static float *g_ref_kc, *g_ref_vc, *g_ref_logits;
static uint64_t g_ref_vocab;

void ref_close(void);

int ref_open(const char *path)
{
    ref_close();
    if (!ram_model_load(path)) return 0;
    memset(&g_ref_file, 0, sizeof(g_ref_file));
    if (!gguf_open(path, &g_ref_file)) { ram_model_free(); return 0; }
    return 1;
}

static void ref_session_end_internal(void)
{
    free(g_ref_work.x); free(g_ref_work.norm); free(g_ref_work.q); free(g_ref_work.k);
    free(g_ref_work.v); free(g_ref_work.att); free(g_ref_work.proj); free(g_ref_work.gate);
    free(g_ref_work.up); free(g_ref_work.ffn); free(g_ref_work.bias);
    free(g_ref_work.scores); free(g_ref_work.weights);
    memset(&g_ref_work, 0, sizeof(g_ref_work));
    free(g_ref_kc); free(g_ref_vc); free(g_ref_logits);
    g_ref_kc = g_ref_vc = g_ref_logits = NULL;
    g_ref_vocab = 0;
}

void ref_close(void)
{
    ref_session_end_internal();
    if (g_ref_file.file || g_ref_file.tensor_index) gguf_close(&g_ref_file);
    if (g_ram_model.data) ram_model_free();
}

/* out: hidden, q_dim, kv_dim, q_heads, kv_heads, head_dim, ffn, layers, max_context, vocab, has_qk_norm */
int ref_shape(uint32_t *out, float *rope_base)
{
    out[0] = g_shape.hidden_size; out[1] = g_shape.q_dim; out[2] = g_shape.kv_dim;
    out[3] = g_shape.q_heads; out[4] = g_shape.kv_heads; out[5] = g_shape.head_dim;
    out[6] = g_shape.ffn_size; out[7] = g_shape.layers; out[8] = g_shape.max_context;
    out[9] = g_shape.vocab_size; out[10] = (uint32_t)g_shape.has_qk_norm;
    *rope_base = g_shape.rope_base;
    return 1;
}

uint64_t ref_data_base(void) { return g_ref_file.data_base; }

int ref_tensor(const char *name, uint32_t *type, uint32_t *n_dims, uint64_t *dims4, uint64_t *offset)
{
    TensorInfo t;
    if (!find_tensor(&g_ref_file, name, &t)) return 0;
    *type = t.type; *n_dims = t.n_dims;
    for (int i = 0; i < 4; ++i) dims4[i] = t.dims[i];
    *offset = t.offset;
    return 1;
}

float ref_half_to_float(uint16_t h) { return half_to_float(h); }

size_t ref_block_bytes(uint32_t type) { return quant_block_bytes(type); }
size_t ref_block_elements(uint32_t type) { return quant_block_elements(type); }

/* Dequantize n consecutive blocks of `type`. */
void ref_dequant_blocks(uint32_t type, const uint8_t *src, float *dst, size_t n)
{
    size_t bb = quant_block_bytes(type), be = quant_block_elements(type);
    for (size_t i = 0; i < n; ++i) dequant_block(type, src + i * bb, dst + i * be);
}

int ref_matvec_rows(const char *name, const float *x, float *y, uint64_t first, uint64_t last)
{
    TensorInfo t;
    if (!find_tensor(&g_ref_file, name, &t) || t.n_dims < 2) return 0;
    return tensor_matvec_cpu_range(&g_ref_file, &t, x, y, first, last);
}

int ref_matvec(const char *name, const float *x, float *y)
{
    TensorInfo t;
    if (!find_tensor(&g_ref_file, name, &t) || t.n_dims < 2) return 0;
    return tensor_matvec_cpu(&g_ref_file, &t, x, y);
}

int ref_embedding_row(uint32_t token, float *dst)
{
    TensorInfo t;
    if (!find_tensor(&g_ref_file, "token_embd.weight", &t)) return 0;
    return load_embedding_row(&g_ref_file, &t, token, dst);
}

int ref_vector(const char *name, float *dst, size_t n) { return vector_named(&g_ref_file, name, dst, n); }

void ref_rms_norm(const float *x, const float *w, float *out, size_t n) { rms_norm(x, w, out, n, RMS_EPS); }

void ref_rope(float *q, float *k, int q_dim, int k_dim, int pos) { rope(q, k, q_dim, k_dim, pos); }

int ref_session_begin(void)
{
    TensorInfo output;
    ref_session_end_internal();
    if (!find_tensor(&g_ref_file, "output.weight", &output)) return 0;
    g_ref_vocab = output.dims[1];
    Work *w = &g_ref_work;
    w->x = array_alloc(HIDDEN_SIZE, sizeof(float)); w->norm = array_alloc(HIDDEN_SIZE, sizeof(float));
    w->q = array_alloc(Q_DIM, sizeof(float)); w->k = array_alloc(KV_DIM, sizeof(float));
    w->v = array_alloc(KV_DIM, sizeof(float)); w->att = array_alloc(Q_DIM, sizeof(float));
    w->proj = array_alloc(HIDDEN_SIZE, sizeof(float)); w->gate = array_alloc(FFN_SIZE, sizeof(float));
    w->up = array_alloc(FFN_SIZE, sizeof(float)); w->ffn = array_alloc(FFN_SIZE, sizeof(float));
    w->bias = array_alloc(Q_DIM, sizeof(float));
    w->scores = array_alloc(MAX_CONTEXT, sizeof(float));
    w->weights = array_alloc(MAX_CONTEXT, sizeof(float));
    g_ref_kc = array_alloc((size_t)LAYERS * MAX_CONTEXT * KV_DIM, sizeof(float));
    g_ref_vc = array_alloc((size_t)LAYERS * MAX_CONTEXT * KV_DIM, sizeof(float));
    g_ref_logits = array_alloc((size_t)g_ref_vocab, sizeof(float));
    return w->x && w->norm && w->q && w->k && w->v && w->att && w->proj && w->gate &&
           w->up && w->ffn && w->bias && w->scores && w->weights && g_ref_kc && g_ref_vc &&
           g_ref_logits;
}

void ref_session_end(void) { ref_session_end_internal(); }

/* One decoder step; copies the logits out when want_logits (and logits != NULL). */
int ref_forward(uint32_t token, uint64_t pos, int want_logits, float *logits)
{
    if (!g_ref_logits) return 0;
    if (!forward_token(&g_ref_file, token, (size_t)pos, g_ref_kc, g_ref_vc, &g_ref_work,
                       g_ref_logits, g_ref_vocab, want_logits))
        return 0;
    if (want_logits && logits) memcpy(logits, g_ref_logits, (size_t)g_ref_vocab * sizeof(float));
    return 1;
}

/* Final hidden state after output_norm (w.proj) of the last forward. */
int ref_last_hidden(float *out)
{
    if (!g_ref_work.proj) return 0;
    memcpy(out, g_ref_work.proj, (size_t)HIDDEN_SIZE * sizeof(float));
    return 1;
}

/* Key/value cache rows written by the last forwards: layer, position -> kv_dim floats. */
int ref_kv_row(uint32_t layer, uint64_t pos, float *k_out, float *v_out)
{
    if (!g_ref_kc || layer >= (uint32_t)LAYERS || pos >= (uint64_t)MAX_CONTEXT) return 0;
    size_t off = ((size_t)layer * MAX_CONTEXT + (size_t)pos) * KV_DIM;
    memcpy(k_out, g_ref_kc + off, (size_t)KV_DIM * sizeof(float));
    memcpy(v_out, g_ref_vc + off, (size_t)KV_DIM * sizeof(float));
    return 1;
}

/* Benchmark helper: fills cache positions [filled, upto) of every layer by
   repeating rows [0, filled), so that forward_token can be timed at position
   `upto` without running upto prompt tokens first. The work of a decode step
   at a position does not depend on the cached values. */
int ref_fill_cache(uint64_t filled, uint64_t upto)
{
    if (!g_ref_kc || !filled || upto > (uint64_t)MAX_CONTEXT || filled > upto) return 0;
    for (size_t l = 0; l < (size_t)LAYERS; ++l)
        for (uint64_t p = filled; p < upto; ++p) {
            size_t dst = (l * MAX_CONTEXT + (size_t)p) * KV_DIM, src = (l * MAX_CONTEXT + (size_t)(p % filled)) * KV_DIM;
            memcpy(g_ref_kc + dst, g_ref_kc + src, (size_t)KV_DIM * sizeof(float));
            memcpy(g_ref_vc + dst, g_ref_vc + src, (size_t)KV_DIM * sizeof(float));
        }
    return 1;
}

/* Greedy pick exactly as atlas_sample_token(..., allow_stop=1, greedy=1). */
uint32_t ref_sample_greedy(const float *logits, uint64_t vocab)
{
    static char empty[1] = {0};
    Tokenizer tok;
    memset(&tok, 0, sizeof(tok));
    tok.tokens = (char **)malloc((size_t)vocab * sizeof(char *));
    if (!tok.tokens) return UINT32_MAX;
    for (uint64_t i = 0; i < vocab; ++i) tok.tokens[i] = empty;
    tok.token_count = (size_t)vocab;
    uint64_t rng = 1;
    float conf = 0.0f;
    uint32_t id = atlas_sample_token(logits, &tok, vocab, NULL, 0, 1, 1, &rng, &conf);
    free(tok.tokens);
    return id;
}

/* The reference's device plugin for forward_token's GEMVs, as run_main_utf8
   brings it up (src/brain_runtime.c:1941-1946): brain_gpu_init over the
   loaded file, hybrid row split when `hybrid`. Returns whether the plugin
   came up (the CPU build links a stub that never does). */
int ref_gpu_init(int hybrid)
{
    if (!g_ram_model.data) return 0;
    g_gpu_enabled = brain_gpu_init(g_ram_model.data, g_ram_model.size);
    g_hybrid_enabled = hybrid ? 1 : 0;
    return g_gpu_enabled;
}

void ref_gpu_shutdown(void)
{
    if (g_gpu_enabled) brain_gpu_shutdown();
    g_gpu_enabled = 0;
    g_hybrid_enabled = 0;
}

/* The reference CLI (argv contract of atlas_dynamic_infer). */
int ref_main(int argc, char **argv) { return run_main_utf8(argc, argv); }

/* tokenize_prompt (src/brain_runtime.c:808-840) with the opened file's
   tokenizer: the number of ids, or -1. */
int ref_tokenize(const char *text, uint32_t *out, uint64_t cap)
{
    Tokenizer tok;
    memset(&tok, 0, sizeof(tok));
    if (!load_tokenizer(&g_ref_file, &tok) || !tokenizer_index(&tok)) { tokenizer_free(&tok); return -1; }
    const size_t n = tokenize_prompt(&tok, text, out, (size_t)cap);
    tokenizer_free(&tok);
    return (int)n;
}
