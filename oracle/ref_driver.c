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

/* Final hidden states of one sequence (Qwen: after the final RMSNorm). */
__attribute__((visibility("default"))) int
ref_forward(void *p, const int *ids, int n, float *out_states) {
    ref_handle_t *h = p;
    return ffwd_model_forward_into(h->model, h->ws, ids, n, out_states);
}
