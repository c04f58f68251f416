/*
 * Reference-facing public API (libffwd/ffwd.h:137-215), implemented over the
 * B200 backend by ffwd_b200/backend/backend_b200.c and exported from
 * libffwd_b200_api.so.  The server and CLI of the reference call exactly these
 * functions, so linking this library in place of libffwd's CUDA backend keeps
 * them unchanged.  Types are layout-identical copies of libffwd/ffwd.h; when
 * the reference's ffwd.h is included first (in-tree build), its definitions
 * are used instead.
 */
#ifndef FFWD_B200_API_H
#define FFWD_B200_API_H

#include "ffwd_b200.h"

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#ifndef FFWD_H
typedef struct embed ffwd_t;

/* libffwd/ffwd.h:137-144 */
typedef struct {
    int n_threads;
    int gpu_quant_bits;
    int gpu_quant_group_size;
    const char *gpu_gemm_mode;
    const char *gpu_weight_dtype;
    double memory_utilization;
} ffwd_options_t;

/* ffwd_rerank_input_t (libffwd/ffwd.h:146-158) comes from ffwd_b200.h. */

FFWD_B200_API int ffwd_init(const ffwd_options_t *opts, char *err, size_t errlen);
FFWD_B200_API ffwd_t *ffwd_open(const char *model_dir, int is_late, const ffwd_options_t *opts,
                                char *err, size_t errlen);
FFWD_B200_API int ffwd_activate(ffwd_t *e, char *err, size_t errlen);
FFWD_B200_API void ffwd_worker_free(ffwd_t *e);
FFWD_B200_API void ffwd_free(ffwd_t *e);
FFWD_B200_API const ffwd_config_t *ffwd_config(const ffwd_t *e);
FFWD_B200_API int ffwd_token_dim(const ffwd_t *e);
FFWD_B200_API int ffwd_uses_dense_batches(const ffwd_t *e);
FFWD_B200_API int ffwd_encode_batch(ffwd_t *e, const ffwd_input_t *inputs, int batch, float *out);
FFWD_B200_API int ffwd_encode_spans_batch(ffwd_t *e, const ffwd_context_input_t *inputs, int batch,
                                          float *out);
FFWD_B200_API int ffwd_rerank(ffwd_t *e, const ffwd_rerank_input_t *in, float *scores);
FFWD_B200_API size_t ffwd_scratch_nbytes(const ffwd_t *e);
FFWD_B200_API const char *ffwd_capability(void);
FFWD_B200_API int ffwd_default_batch_wait_us(void);
FFWD_B200_API int ffwd_preflight(const char *const *paths, int n_paths, const ffwd_options_t *opts,
                                 char *err, size_t errlen);
FFWD_B200_API int ffwd_l2_normalize(float *vec, int dim);
FFWD_B200_API float ffwd_cosine_similarity(const float *a, const float *b, int dim);
FFWD_B200_API extern int ffwd_verbose;
#endif /* FFWD_H */

/* No counterpart in the reference: the backend context behind a pooled-model
 * handle (NULL before ffwd_activate or for a late-interaction model), so a
 * host can read ffwd_b200_shard_stats for its ffwd_encode_batch calls. */
FFWD_B200_API ffwd_b200_ctx_t *ffwd_b200_api_context(ffwd_t *e);

#ifdef __cplusplus
}
#endif

#endif /* FFWD_B200_API_H */
