/* B200 backend glue: implements the public API of libffwd/ffwd.h over the
 * ffwd_b200_* C ABI.  Drop-in replacement for libffwd/backend_cuda.c: same
 * two-phase load (open records the directory, activate loads on the
 * inference thread, backend_cuda.c:67-90), same option parsing and error
 * texts for --gpu-gemm-mode / --gpu-weight-dtype (backend_cuda.c:45-65), same
 * encode forwarding (backend_cuda.c:124-130) and constants
 * (ffwd_scratch_nbytes 0, ffwd_default_batch_wait_us 1000).
 *
 * Late-interaction models (is_late) load through ffwd_b200_late_load and serve
 * ffwd_token_dim / ffwd_rerank like backend_cuda.c:99-156, with MaxSim scored
 * on the device (ffwd_b200_late_rerank) instead of on the host. */
#include "ffwd_b200_api.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

struct embed {
    int is_late;
    char *dir;
    ffwd_b200_ctx_t *ctx;
    ffwd_b200_late_ctx_t *late_ctx;
};

FFWD_B200_API int ffwd_verbose = 0;

FFWD_B200_API const char *ffwd_capability(void) { return "NVIDIA CUDA (B200 sm_100a)"; }

FFWD_B200_API int ffwd_init(const ffwd_options_t *opts, char *err, size_t errlen) {
    if (!opts)
        return 0;
    if (opts->gpu_gemm_mode && ffwd_b200_set_fast_gemm(opts->gpu_gemm_mode) != 0) {
        snprintf(err, errlen, "--gpu-gemm-mode must be f32, tf32, bf16, or 16f");
        return -1;
    }
    if (opts->gpu_weight_dtype) {
        if (!strcmp(opts->gpu_weight_dtype, "bf16"))
            ffwd_b200_set_weights_bf16(1);
        else if (!strcmp(opts->gpu_weight_dtype, "f16") || !strcmp(opts->gpu_weight_dtype, "fp16"))
            ffwd_b200_set_weights_f16(1);
        else if (!strcmp(opts->gpu_weight_dtype, "f32"))
            ffwd_b200_set_weights_bf16(0);
        else {
            snprintf(err, errlen, "--gpu-weight-dtype must be f32, bf16, or f16");
            return -1;
        }
    }
    if (ffwd_verbose >= 1)
        fprintf(stderr, "Using %s\n", ffwd_capability());
    return 0;
}

FFWD_B200_API ffwd_b200_ctx_t *ffwd_b200_api_context(ffwd_t *b) { return b ? b->ctx : NULL; }

FFWD_B200_API ffwd_t *ffwd_open(const char *model_dir, int is_late, const ffwd_options_t *opts,
                                char *err, size_t errlen) {
    (void)opts;
    ffwd_t *b = (ffwd_t *)calloc(1, sizeof(*b));
    if (!b || !model_dir || !(b->dir = strdup(model_dir))) {
        snprintf(err, errlen, "out of memory");
        free(b);
        return NULL;
    }
    b->is_late = is_late;
    return b;
}

FFWD_B200_API int ffwd_activate(ffwd_t *b, char *err, size_t errlen) {
    if (b->is_late) {
        b->late_ctx = ffwd_b200_late_load(b->dir);
        if (!b->late_ctx) {
            snprintf(err, errlen, "failed to load late-interaction model");
            return -1;
        }
        return 0;
    }
    b->ctx = ffwd_b200_load(b->dir);
    if (!b->ctx) {
        snprintf(err, errlen, "failed to load model");
        return -1;
    }
    return 0;
}

FFWD_B200_API void ffwd_worker_free(ffwd_t *b) {
    if (!b)
        return;
    if (b->ctx) {
        ffwd_b200_free(b->ctx);
        b->ctx = NULL;
    }
    if (b->late_ctx) {
        ffwd_b200_late_free(b->late_ctx);
        b->late_ctx = NULL;
    }
}

FFWD_B200_API void ffwd_free(ffwd_t *b) {
    if (!b)
        return;
    ffwd_worker_free(b);
    free(b->dir);
    free(b);
}

FFWD_B200_API const ffwd_config_t *ffwd_config(const ffwd_t *b) {
    if (!b)
        return NULL;
    return b->is_late ? ffwd_b200_late_config(b->late_ctx) : ffwd_b200_config(b->ctx);
}

FFWD_B200_API int ffwd_token_dim(const ffwd_t *b) {
    return b && b->is_late ? ffwd_b200_late_token_dim(b->late_ctx) : 0;
}

FFWD_B200_API int ffwd_uses_dense_batches(const ffwd_t *b) {
    (void)b;
    return 0;
}

FFWD_B200_API int ffwd_encode_batch(ffwd_t *b, const ffwd_input_t *inputs, int batch, float *out) {
    return b ? ffwd_b200_encode_batch(b->ctx, inputs, batch, out) : -1;
}

FFWD_B200_API int ffwd_encode_spans_batch(ffwd_t *b, const ffwd_context_input_t *inputs, int batch,
                                          float *out) {
    return b ? ffwd_b200_encode_spans_batch(b->ctx, inputs, batch, out) : -1;
}

FFWD_B200_API int ffwd_rerank(ffwd_t *b, const ffwd_rerank_input_t *in, float *scores) {
    return b && b->late_ctx ? ffwd_b200_late_rerank(b->late_ctx, in, scores) : -1;
}

FFWD_B200_API size_t ffwd_scratch_nbytes(const ffwd_t *b) {
    (void)b;
    return 0;
}

FFWD_B200_API int ffwd_default_batch_wait_us(void) { return 1000; }

FFWD_B200_API int ffwd_preflight(const char *const *paths, int n_paths, const ffwd_options_t *opts,
                                 char *err, size_t errlen) {
    (void)paths;
    (void)n_paths;
    (void)opts;
    (void)err;
    (void)errlen;
    return 0;
}

/* Same contract as libffwd/vec.c:7-22. */
FFWD_B200_API int ffwd_l2_normalize(float *vec, int dim) {
    if (!vec || dim <= 0)
        return -1;
    float norm_sq = 0.0f;
    for (int i = 0; i < dim; i++)
        norm_sq += vec[i] * vec[i];
    if (!(norm_sq > 0.0f) || !isfinite(norm_sq))
        return -1;
    float inv = 1.0f / sqrtf(norm_sq);
    for (int i = 0; i < dim; i++)
        vec[i] *= inv;
    return 0;
}

/* Same contract as libffwd/vec.c:24-47. */
FFWD_B200_API float ffwd_cosine_similarity(const float *a, const float *b, int dim) {
    if (!a || !b || dim <= 0)
        return 0.0f;
    float dot = 0.0f, na = 0.0f, nb = 0.0f;
    for (int i = 0; i < dim; i++) {
        dot += a[i] * b[i];
        na += a[i] * a[i];
        nb += b[i] * b[i];
    }
    if (!(na > 0.0f) || !(nb > 0.0f) || !isfinite(na) || !isfinite(nb) || !isfinite(dot))
        return 0.0f;
    double denom = sqrt((double)na) * sqrt((double)nb);
    if (!(denom > 0.0) || !isfinite(denom))
        return 0.0f;
    return (float)((double)dot / denom);
}
