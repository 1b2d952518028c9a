/*
 * ORACLE harness around the reference's batched-prefill CPU runtime
 * (src/brain_runtime_batch.c, fixed Qwen2-1.5B shape: hidden 1536, 28 layers,
 * 12/2 heads, FFN 8960, MAX_CONTEXT 2048, src/brain_runtime_batch.c:90-108,
 * :1505-1507). Test infrastructure only. Exports:
 *   forward_prefill_batch  src/brain_runtime_batch.c:1644 (chunks of <= 32)
 *   forward_token          src/brain_runtime_batch.c:1720
 */
#include "brain_runtime_batch.c"

static GGUFFile gb_file;
static Work gb_work;
static PrefillWork gb_prefill;
static float *gb_kc, *gb_vc, *gb_logits;
static uint64_t gb_vocab;

void refb_close(void)
{
    free(gb_work.x); free(gb_work.norm); free(gb_work.q); free(gb_work.k); free(gb_work.v);
    free(gb_work.att); free(gb_work.proj); free(gb_work.gate); free(gb_work.up);
    free(gb_work.ffn); free(gb_work.bias); free(gb_work.scores); free(gb_work.weights);
    memset(&gb_work, 0, sizeof(gb_work));
    prefill_work_free(&gb_prefill);
    free(gb_kc); free(gb_vc); free(gb_logits);
    gb_kc = gb_vc = gb_logits = NULL;
    if (gb_file.file || gb_file.tensor_index) gguf_close(&gb_file);
    if (g_ram_model.data) ram_model_free();
}

int refb_open(const char *path)
{
    refb_close();
    if (!ram_model_load(path)) return 0;
    memset(&gb_file, 0, sizeof(gb_file));
    if (!gguf_open(path, &gb_file)) { ram_model_free(); return 0; }
    TensorInfo output;
    if (!find_tensor(&gb_file, "output.weight", &output)) return 0;
    gb_vocab = output.dims[1];
    Work *w = &gb_work;
    w->x = array_alloc(HIDDEN_SIZE, sizeof(float)); w->norm = array_alloc(HIDDEN_SIZE, sizeof(float));
    w->q = array_alloc(Q_DIM, sizeof(float)); w->k = array_alloc(KV_DIM, sizeof(float));
    w->v = array_alloc(KV_DIM, sizeof(float)); w->att = array_alloc(Q_DIM, sizeof(float));
    w->proj = array_alloc(HIDDEN_SIZE, sizeof(float)); w->gate = array_alloc(FFN_SIZE, sizeof(float));
    w->up = array_alloc(FFN_SIZE, sizeof(float)); w->ffn = array_alloc(FFN_SIZE, sizeof(float));
    w->bias = array_alloc(Q_DIM, sizeof(float));
    w->scores = array_alloc(MAX_CONTEXT, sizeof(float));
    w->weights = array_alloc(MAX_CONTEXT, sizeof(float));
    gb_kc = array_alloc((size_t)LAYERS * MAX_CONTEXT * KV_DIM, sizeof(float));
    gb_vc = array_alloc((size_t)LAYERS * MAX_CONTEXT * KV_DIM, sizeof(float));
    gb_logits = array_alloc((size_t)gb_vocab, sizeof(float));
    return w->x && w->norm && w->q && w->k && w->v && w->att && w->proj && w->gate &&
           w->up && w->ffn && w->bias && w->scores && w->weights && gb_kc && gb_vc &&
           gb_logits && prefill_work_alloc(&gb_prefill);
}

/* Prefill tokens[0..n) at positions pos0.., in chunks of PREFILL_BATCH; logits of the last. */
int refb_prefill(const uint32_t *tokens, uint64_t n, uint64_t pos0, float *logits)
{
    uint64_t done = 0;
    while (done < n) {
        uint64_t m = n - done;
        if (m > PREFILL_BATCH) m = PREFILL_BATCH;
        if (!forward_prefill_batch(&gb_file, tokens + done, (size_t)m, (size_t)(pos0 + done),
                                   gb_kc, gb_vc, &gb_work, &gb_prefill, gb_logits, gb_vocab,
                                   done + m == n))
            return 0;
        done += m;
    }
    if (logits) memcpy(logits, gb_logits, (size_t)gb_vocab * sizeof(float));
    return 1;
}

int refb_forward(uint32_t token, uint64_t pos, int want_logits, float *logits)
{
    if (!forward_token(&gb_file, token, (size_t)pos, gb_kc, gb_vc, &gb_work, gb_logits,
                       gb_vocab, want_logits))
        return 0;
    if (want_logits && logits) memcpy(logits, gb_logits, (size_t)gb_vocab * sizeof(float));
    return 1;
}
