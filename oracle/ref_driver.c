/* ctypes-facing driver around the reference's own CPU forward.
 *
 * Test infrastructure only (the checker, never the product).  It is linked
 * against the UNMODIFIED reference sources under libffwd/ by oracle/Makefile
 * and calls the reference's lower-level CPU model API exactly as its backend
 * glue does (libffwd/backend_blas.c:35-83 loads with ffwd_model_load and
 * encodes with ffwd_model_encode_batch, libffwd/forward.c:628-652).
 */
#include "internal.h"
#include "threadpool.h"

#include <stdlib.h>

typedef struct {
    ffwd_model_t *model;
    ffwd_workspace_t *ws;
} ref_handle_t;

__attribute__((visibility("default"))) void ref_set_threads(int n) { tp_set_threads(n); }

__attribute__((visibility("default"))) void *ref_load(const char *dir) {
    ref_handle_t *h = calloc(1, sizeof(*h));
    if (!h)
        return NULL;
    h->model = ffwd_model_load(dir);
    if (!h->model) {
        free(h);
        return NULL;
    }
    h->ws = ffwd_workspace_new(h->model);
    if (!h->ws) {
        ffwd_model_free(h->model);
        free(h);
        return NULL;
    }
    return h;
}

__attribute__((visibility("default"))) void ref_free(void *p) {
    ref_handle_t *h = p;
    if (!h)
        return;
    ffwd_workspace_free(h->ws);
    ffwd_model_free(h->model);
    free(h);
}

/* Copies the parsed ffwd_config_t fields as ints/floats for the test harness. */
__attribute__((visibility("default"))) int ref_config(void *p, int *ints, float *floats) {
    ref_handle_t *h = p;
    const ffwd_config_t *c = ffwd_model_config(h->model);
    ints[0] = c->family;
    ints[1] = c->ffn_act;
    ints[2] = c->hidden_size;
    ints[3] = c->n_layers;
    ints[4] = c->n_heads;
    ints[5] = c->n_kv_heads;
    ints[6] = c->head_dim;
    ints[7] = c->intermediate_size;
    ints[8] = c->vocab_size;
    ints[9] = c->max_position_embeddings;
    ints[10] = c->position_id_offset;
    ints[11] = c->type_vocab_size;
    ints[12] = c->qk_norm;
    ints[13] = c->qkv_bias;
    ints[14] = c->attention_mode;
    ints[15] = c->pooling_mode;
    ints[16] = c->normalize_embeddings;
    ints[17] = c->append_terminal_token;
    floats[0] = c->rms_norm_eps;
    floats[1] = c->layer_norm_eps;
    floats[2] = c->rope_theta;
    return 0;
}

/* Packed batch: ids concatenated, lens[batch]. */
__attribute__((visibility("default"))) int
ref_encode(void *p, const int *ids, const int *lens, int batch, float *out) {
    ref_handle_t *h = p;
    ffwd_input_t *in = malloc((size_t)batch * sizeof(*in));
    if (!in)
        return -1;
    size_t off = 0;
    for (int b = 0; b < batch; b++) {
        in[b].ids = ids + off;
        in[b].n_tokens = lens[b];
        off += (size_t)(lens[b] > 0 ? lens[b] : 0);
    }
    int rc = ffwd_model_encode_batch(h->model, h->ws, in, batch, out);
    free(in);
    return rc;
}

/* Contextual spans (ffwd_model_encode_spans_batch, forward.c:528-589): ids
 * concatenated with lens[batch]; n_spans[batch] spans per document, their
 * (start, n_tokens) pairs concatenated in span_start / span_len. */
__attribute__((visibility("default"))) int
ref_encode_spans(void *p, const int *ids, const int *lens, int batch, const int *n_spans,
                 const int *span_start, const int *span_len, float *out) {
    ref_handle_t *h = p;
    int total = 0;
    for (int b = 0; b < batch; b++)
        total += n_spans[b];
    ffwd_context_input_t *in = malloc((size_t)batch * sizeof(*in));
    ffwd_span_t *sp = malloc((size_t)(total > 0 ? total : 1) * sizeof(*sp));
    if (!in || !sp) {
        free(in);
        free(sp);
        return -1;
    }
    size_t off = 0;
    int si = 0;
    for (int b = 0; b < batch; b++) {
        in[b].input.ids = ids + off;
        in[b].input.n_tokens = lens[b];
        in[b].spans = sp + si;
        in[b].n_spans = n_spans[b];
        for (int s = 0; s < n_spans[b]; s++, si++) {
            sp[si].start = span_start[si];
            sp[si].n_tokens = span_len[si];
        }
        off += (size_t)(lens[b] > 0 ? lens[b] : 0);
    }
    int rc = ffwd_model_encode_spans_batch(h->model, h->ws, in, batch, out);
    free(in);
    free(sp);
    return rc;
}

/* Final hidden states of one sequence (Qwen: after the final RMSNorm). */
__attribute__((visibility("default"))) int
ref_forward(void *p, const int *ids, int n, float *out_states) {
    ref_handle_t *h = p;
    return ffwd_model_forward_into(h->model, h->ws, ids, n, out_states);
}

/* ---- late interaction: the reference's CPU late model (libffwd/late.c,
 * late_blas.c), called as its MLX/BLAS backends do. */

typedef struct {
    ffwd_late_model_t *model;
    ffwd_late_workspace_t *ws;
} ref_late_t;

__attribute__((visibility("default"))) void *ref_late_load(const char *dir) {
    ref_late_t *h = calloc(1, sizeof(*h));
    if (!h)
        return NULL;
    h->model = ffwd_late_model_load(dir);
    if (!h->model || !(h->ws = ffwd_late_workspace_new(h->model))) {
        ffwd_late_model_free(h->model);
        free(h);
        return NULL;
    }
    return h;
}

__attribute__((visibility("default"))) void ref_late_free(void *p) {
    ref_late_t *h = p;
    if (!h)
        return;
    ffwd_late_workspace_free(h->ws);
    ffwd_late_model_free(h->model);
    free(h);
}

__attribute__((visibility("default"))) int ref_late_token_dim(void *p) {
    return ffwd_late_model_token_dim(((ref_late_t *)p)->model);
}

__attribute__((visibility("default"))) int
ref_late_encode_tokens(void *p, const int *ids, int n, int normalize, float *out) {
    ref_late_t *h = p;
    return ffwd_late_model_encode_tokens(h->model, h->ws, ids, n, normalize, out);
}

/* Documents concatenated: ids / lens[n_docs]; kept indices concatenated:
 * keep / n_keep[n_docs]. */
__attribute__((visibility("default"))) int
ref_late_encode_docs(void *p, const int *ids, const int *lens, const int *keep, const int *n_keep,
                     int n_docs, int normalize, float *out, int *out_offsets) {
    ref_late_t *h = p;
    const int **doc_ids = malloc((size_t)n_docs * sizeof(*doc_ids));
    const int **keeps = malloc((size_t)n_docs * sizeof(*keeps));
    if (!doc_ids || !keeps) {
        free(doc_ids);
        free(keeps);
        return -1;
    }
    size_t oi = 0, ok = 0;
    for (int d = 0; d < n_docs; d++) {
        doc_ids[d] = ids + oi;
        keeps[d] = keep + ok;
        oi += (size_t)lens[d];
        ok += (size_t)n_keep[d];
    }
    int rc = ffwd_late_model_encode_docs(h->model, h->ws, (const int *const *)doc_ids, lens,
                                         (const int *const *)keeps, n_keep, n_docs, normalize, out,
                                         out_offsets);
    free(doc_ids);
    free(keeps);
    return rc;
}

__attribute__((visibility("default"))) int
ref_late_maxsim_batch(const float *q, int nq, const float *docs, const int *offsets, int n_docs,
                      int dim, float *scores) {
    return ffwd_late_maxsim_batch(q, nq, docs, offsets, n_docs, dim, scores);
}
