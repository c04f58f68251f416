/*
 * ffwd_b200 — B200 (sm_100a) backend for ffwd's packed, variable-length
 * embedding forward pass.
 *
 * C ABI.  The first group mirrors the reference backend interface in
 * libffwd/cuda.h one for one (ffwd_cuda_* -> ffwd_b200_*), so
 * libffwd/backend_cuda.c can call these instead; the shared types are
 * layout-identical copies of libffwd/ffwd.h so pointers pass straight through.
 * The second group has no counterpart in the reference (multi-GPU device set,
 * device-resident inputs, diagnostics).
 *
 * Conventions (as in the reference): 0 on success, -1 on failure, NULL on a
 * failed load; diagnostics go to stderr and to ffwd_b200_last_error().  A
 * context is used from one host thread at a time (the inference worker,
 * libffwd/ffwd.h:118-128).
 */
#ifndef FFWD_B200_H
#define FFWD_B200_H

#include <stddef.h>
#include <stdint.h>

#ifndef FFWD_B200_API
#    if defined(__GNUC__)
#        define FFWD_B200_API __attribute__((visibility("default")))
#    else
#        define FFWD_B200_API
#    endif
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- Shared types: identical layout to libffwd/ffwd.h:34-105 ------------- */
#ifndef FFWD_H
typedef enum {
    FFWD_ATTENTION_BIDIRECTIONAL = 0,
    FFWD_ATTENTION_CAUSAL = 1,
} ffwd_attention_mode_t;

typedef enum {
    FFWD_POOL_MEAN = 0,
    FFWD_POOL_LAST_TOKEN = 1,
    FFWD_POOL_CLS = 2,
} ffwd_pooling_mode_t;

typedef enum {
    FFWD_FAMILY_QWEN3 = 0,
    FFWD_FAMILY_BERT = 1,
} ffwd_family_t;

typedef enum {
    FFWD_ACT_GELU_ERF = 0,
    FFWD_ACT_GELU_TANH = 1,
} ffwd_act_t;

typedef struct {
    ffwd_family_t family;
    ffwd_act_t ffn_act;
    int hidden_size;
    int n_layers;
    int n_heads;
    int n_kv_heads;
    int head_dim;
    int q_dim;
    int kv_dim;
    int intermediate_size;
    int vocab_size;
    int max_position_embeddings;
    int position_id_offset;
    int type_vocab_size;
    float rms_norm_eps;
    float layer_norm_eps;
    float rope_theta;
    int qk_norm;
    int qkv_bias;
    ffwd_attention_mode_t attention_mode;
    ffwd_pooling_mode_t pooling_mode;
    int normalize_embeddings;
    int append_terminal_token;
} ffwd_config_t;

typedef struct {
    const int *ids;
    int n_tokens;
} ffwd_input_t;

typedef struct {
    int start;
    int n_tokens;
} ffwd_span_t;

typedef struct {
    ffwd_input_t input;
    const ffwd_span_t *spans;
    int n_spans;
} ffwd_context_input_t;

/* libffwd/ffwd.h:146-158 */
typedef struct {
    const int *query_ids;
    int query_n_tokens;
    int query_n_keep;
    const int *const *doc_ids;
    const int *doc_n_tokens;
    const int *const *doc_keep;
    const int *doc_n_keep;
    int n_docs;
} ffwd_rerank_input_t;
#endif /* FFWD_H */

typedef struct ffwd_b200_ctx ffwd_b200_ctx_t;

/* ---- Mirror of libffwd/cuda.h ---------------------------------------------- */

/* Process-wide GEMM mode, set before any load: "f32" | "tf32" | "bf16" | "16f".
 * Replaces ffwd_cuda_set_fast_gemm (cuda.h:22; parsing at cuda.cu:169-199).
 * With f32 weight storage, f32 runs split-bf16 3-pass GEMMs, tf32 kind::tf32
 * GEMMs (both with f32 attention); bf16 runs single-pass bf16 and 16f
 * single-pass f16 tensor-core GEMMs and attention.  16-bit weight storage: see
 * ffwd_b200_precision.
 * -1 on an unknown mode. */
FFWD_B200_API int ffwd_b200_set_fast_gemm(const char *mode);
/* Store weights as bf16 (on = 1) or as f32 (on = 0).
 * Replaces ffwd_cuda_set_weights_bf16 (cuda.h:23; cuda.cu:237-247). */
FFWD_B200_API int ffwd_b200_set_weights_bf16(int on);
/* Store weights as f16 (on = 1) or as f32 (on = 0).
 * Replaces ffwd_cuda_set_weights_f16 (cuda.h:24; cuda.cu:243-246). */
FFWD_B200_API int ffwd_b200_set_weights_f16(int on);
/* Back to the default storage: BF16 files as bf16, F32 and F16 files as f32
 * (cuda.cu:4225-4228).  No reference counterpart (its override lasts for the
 * process). */
FFWD_B200_API int ffwd_b200_set_weights_default(void);

/* Load config + safetensors from model_dir and upload to every device of the
 * current device set.  Replaces ffwd_cuda_load (cuda.h:26; cuda.cu:4306). */
FFWD_B200_API ffwd_b200_ctx_t *ffwd_b200_load(const char *model_dir);
/* Replaces ffwd_cuda_free (cuda.h:27). */
FFWD_B200_API void ffwd_b200_free(ffwd_b200_ctx_t *ctx);
/* Replaces ffwd_cuda_config (cuda.h:56). */
FFWD_B200_API const ffwd_config_t *ffwd_b200_config(const ffwd_b200_ctx_t *ctx);

/* One sequence -> out_embedding[hidden].  Replaces ffwd_cuda_encode_into
 * (cuda.h:58-59). */
FFWD_B200_API int ffwd_b200_encode_into(ffwd_b200_ctx_t *ctx, const int *token_ids, int n_tokens,
                                        float *out_embedding);
/* Malloc'd embedding or NULL.  Replaces ffwd_cuda_encode (cuda.h:60). */
FFWD_B200_API float *ffwd_b200_encode(ffwd_b200_ctx_t *ctx, const int *token_ids, int n_tokens);
/* Packed batch -> out_embeddings[batch * hidden] (host), input order.  Forward,
 * pooling and L2 normalisation run on the device(s); sequences are sharded
 * across the device set.  Replaces ffwd_cuda_encode_batch (cuda.h:61-64;
 * cuda.cu:5102-5140). */
FFWD_B200_API int ffwd_b200_encode_batch(ffwd_b200_ctx_t *ctx, const ffwd_input_t *inputs,
                                         int batch, float *out_embeddings);
/* Contextual spans: one forward per batch, each span mean-pooled over the
 * final hidden states, out[total_spans * hidden].  Replaces
 * ffwd_cuda_encode_spans_batch (cuda.h:65-68; cuda.cu:5142-5225). */
FFWD_B200_API int ffwd_b200_encode_spans_batch(ffwd_b200_ctx_t *ctx,
                                               const ffwd_context_input_t *inputs, int batch,
                                               float *out_embeddings);

/* ---- Late interaction: mirror of libffwd/cuda.h:30-60 ----------------------- */

typedef struct ffwd_b200_late_ctx ffwd_b200_late_ctx_t;

/* Load a late-interaction model: base model + 1_Dense/model.safetensors
 * `linear.weight` [token_dim, hidden] (token_dim <= 1024), on the first device
 * of the device set.  NULL without a 1_Dense head or with a bad projection.
 * Replaces ffwd_cuda_late_load (cuda.h:35; cuda.cu:5267-5296). */
FFWD_B200_API ffwd_b200_late_ctx_t *ffwd_b200_late_load(const char *model_dir);
/* Replaces ffwd_cuda_late_free (cuda.h:36). */
FFWD_B200_API void ffwd_b200_late_free(ffwd_b200_late_ctx_t *ctx);
/* Replaces ffwd_cuda_late_config (cuda.h:37). */
FFWD_B200_API const ffwd_config_t *ffwd_b200_late_config(const ffwd_b200_late_ctx_t *ctx);
/* Replaces ffwd_cuda_late_token_dim (cuda.h:38). */
FFWD_B200_API int ffwd_b200_late_token_dim(const ffwd_b200_late_ctx_t *ctx);
/* token_ids -> out_vectors[n_tokens * token_dim] (host), each vector the
 * projection of the final hidden state (decoders: after the final RMSNorm),
 * L2-normalised when `normalize`.  Replaces ffwd_cuda_late_encode_tokens
 * (cuda.h:41-42; cuda.cu:5364-5384). */
FFWD_B200_API int ffwd_b200_late_encode_tokens(ffwd_b200_late_ctx_t *ctx, const int *token_ids,
                                               int n_tokens, int normalize, float *out_vectors);
/* n_docs documents in one packed forward; document d's kept token vectors
 * (rows keep[d][0..n_keep[d])) back to back in out_vectors, out_offsets[n_docs
 * + 1] their prefix sum.  Replaces ffwd_cuda_late_encode_docs (cuda.h:50-58;
 * cuda.cu:5386-5452); the gather and normalisation run on the device. */
FFWD_B200_API int ffwd_b200_late_encode_docs(ffwd_b200_late_ctx_t *ctx, const int *const *doc_ids,
                                             const int *n_tokens, const int *const *keep,
                                             const int *n_keep, int n_docs, int normalize,
                                             float *out_vectors, int *out_offsets);
/* MaxSim scores of one query against n_docs candidates: query and candidates
 * in one packed forward, normalised vectors and scores computed on the device,
 * scores[n_docs] copied back.  Same result as the reference's ffwd_rerank
 * (backend_cuda.c:132-156: encode_tokens + encode_docs + host
 * ffwd_late_maxsim_batch, late.c:143-219). */
FFWD_B200_API int ffwd_b200_late_rerank(ffwd_b200_late_ctx_t *ctx, const ffwd_rerank_input_t *in,
                                        float *scores);

/* ---- No counterpart in the reference ------------------------------------ */

/* Output encodings of ffwd_b200_encode_batch_as. */
enum {
    FFWD_B200_OUT_F32 = 0,  /* float32 [batch * dims] */
    FFWD_B200_OUT_INT8 = 1, /* int8 round(tanh(x) * 127), clamped [batch * dims] */
    FFWD_B200_OUT_BINARY = 2 /* sign bits (x >= 0), 8 per byte, least significant bit first
                                [batch * dims / 8] */
};

/* ffwd_b200_encode_batch with the embedding's wire form produced on the device:
 * the first `dims` (1..hidden) values of each pooled embedding, L2-renormalised
 * when `renormalize` and dims < hidden (Matryoshka truncation), then encoded.
 * The reference's server applies the same steps to host floats
 * (tools/server/encode.c:20-61 quantize_int8_tanh / base64_binary, 107-122
 * truncate + renormalise); doing them on the device shrinks the copy back to
 * 1/4 (int8) or 1/32 (binary).  Binary needs dims % 8 == 0.  0 / -1. */
FFWD_B200_API int ffwd_b200_encode_batch_as(ffwd_b200_ctx_t *ctx, const ffwd_input_t *inputs,
                                            int batch, int dims, int renormalize, int encoding,
                                            void *out);

/* Device set used by the next ffwd_b200_load (replicated weights, sequences
 * sharded by LPT over estimated cost).  Default: $FFWD_B200_DEVICES
 * ("0,1,..."), else device 0. */
FFWD_B200_API int ffwd_b200_set_devices(const int *devices, int n_devices);

/* Largest packed token count one device forward holds; longer batches run as
 * several forwards of about equal size (sequences are never split).  Default
 * 262144 (about 6 GB of activations for a 1024-wide model). */
FFWD_B200_API int ffwd_b200_set_max_tokens(int max_tokens);

/* Device-resident entry (single device, index dev of the context's set): ids
 * and out already in that GPU's memory, host row offsets [batch + 1].  Work is
 * enqueued on the context's stream for that device; the call returns after
 * the stream completes when sync != 0.  The bench's kernel-only timing uses
 * this path. */
FFWD_B200_API int ffwd_b200_encode_device(ffwd_b200_ctx_t *ctx, int dev, const int *d_ids,
                                          const int *h_offsets, int batch, float *d_out, int sync);

/* No counterpart in the reference.  Same computation and arguments as
 * ffwd_b200_encode_device, for callers that cannot allocate device memory
 * while serving: hosts that hand all GPU memory to their own pool and forbid
 * other allocations, and latency-sensitive callers for whom cudaMalloc /
 * cudaFree (which can synchronise the device) are off limits on the request
 * path.  This entry allocates nothing: its working buffers live in a fixed
 * 32 MiB arena of device memory, reserved on a GPU when a model is loaded
 * there (ffwd_b200_load resolves the arena's address with that device
 * current) and held until the process exits.  Requests whose buffers do not
 * fit the arena (for example more than about 1300 tokens for a
 * Qwen3-0.6B-shaped model), more than 4096 sequences or 8192 attention work
 * items are rejected with -1 and a message; so are row offsets that do not
 * start at 0.  The attention work list is built in a static host array, so
 * the call needs only a small host stack.  All calls share the one arena and
 * it keeps the last call's contents, so calls whose GPU work overlaps (other
 * streams, other host threads) race.  The call synchronises the context's
 * stream and reads an error word back before it returns, so it must not be
 * called while any stream is being captured. */
FFWD_B200_API int ffwd_b200_encode_device_noalloc(ffwd_b200_ctx_t *ctx, int dev, const int *d_ids,
                                                  const int *h_offsets, int batch, float *d_out);

/* Re-issue `reps` launches of one op of layer `layer` on the buffers of the
 * last forward run on device index dev (enqueued, not synchronised), for
 * per-kernel timing: 0 QKV projection, 1 attention, 2 output projection,
 * 3 first norm, 4 FFN up / gate-up, 5 FFN down, 6 second norm; 7 the
 * embedding (+ first norm) and 8 the pooling (+ final norm, L2) of the whole
 * forward (layer ignored).  Ops that accumulate into the residual stream
 * change the buffers' values. */
FFWD_B200_API int ffwd_b200_run_op(ffwd_b200_ctx_t *ctx, int dev, int op, int layer, int reps);

/* Per device entry of the context, the last ffwd_b200_encode_batch /
 * _encode_batch_as call's shard: sequences, tokens and the host wall time in
 * ms of that entry's worker (packing through copied-out rows).  Writes up to
 * cap entries (any pointer may be NULL); returns the number of entries. */
FFWD_B200_API int ffwd_b200_shard_stats(const ffwd_b200_ctx_t *ctx, int *seqs, long long *tokens,
                                        double *ms, int cap);

/* Host-side fault injection for tests (no GPU fault is involved):
 * FFWD_B200_INJECT_SHARD, value = device entry: the next shard of an encode
 * call on that entry fails before anything is uploaded or launched;
 * FFWD_B200_INJECT_ALLOC, value = n: the next n workspace allocations return
 * cudaErrorMemoryAllocation; FFWD_B200_INJECT_NONE clears both.  Returns 0,
 * or -1 for an unknown kind. */
#define FFWD_B200_INJECT_NONE 0
#define FFWD_B200_INJECT_SHARD 1
#define FFWD_B200_INJECT_ALLOC 2
FFWD_B200_API int ffwd_b200_test_inject(int kind, int value);

/* Self-test of the kernels' bounded waits on GPU `device`: one thread waits
 * on an mbarrier that nothing arrives at, with a limit of limit_us
 * microseconds (1 .. 1000000).  The wait gives up, the kernel records its
 * error code and returns; the call then returns -1 with "device wait timed
 * out" and the context stays usable. */
FFWD_B200_API int ffwd_b200_selftest_wait(int device, int limit_us);

/* The CUDA stream (cudaStream_t) the context uses on device index dev. */
FFWD_B200_API void *ffwd_b200_stream(ffwd_b200_ctx_t *ctx, int dev);
/* Kernel launches issued by this process since load (all contexts). */
FFWD_B200_API long long ffwd_b200_launch_count(void);
/* Last error message of the calling thread ("" if none). */
FFWD_B200_API const char *ffwd_b200_last_error(void);
/* Precision plan chosen at load: 0 = single-pass bf16, 1 = single-pass f16,
 * 2 = split-bf16 2-pass, 3 = split-bf16 3-pass, 4 = tf32 (kind::tf32 GEMMs over
 * tf32-rounded f32 operands, split-bf16 attention). */
FFWD_B200_API int ffwd_b200_precision(const ffwd_b200_ctx_t *ctx);

/* Host-side LPT partition used by the sharder: assigns each of n items with
 * cost[i] to one of n_parts parts, minimising the largest part.  Writes
 * part[i].  Exposed for tests. */
FFWD_B200_API int ffwd_b200_lpt_partition(const double *cost, int n, int n_parts, int *part);

/* Attention work list of a packed batch (host; the list the forward builds),
 * exposed for tests: pairs of 128-row query blocks sharing a key/value head.
 * windows != 0: neighbouring sequences of at most 128 rows share items (the
 * list of the 16-bit plans).  offsets: [batch + 1] row offsets.  With items
 * NULL returns an upper bound of the count; else writes up to cap items as 7
 * ints each (seq, qt0, h0, qt1, h1, key tiles, window sequences: 0 for a
 * single-sequence item) and returns the count; -1 on bad arguments or when cap
 * is too small. */
FFWD_B200_API int ffwd_b200_attention_items(int causal, int windows, int n_heads, int n_kv_heads,
                                            const int *offsets, int batch, int *items, int cap);

/* Operator-level entry for tests: Y = X W^T with the tcgen05 GEMM on device
 * pointers (bf16 X [M, K], bf16 W [N, K], f32 Y [M, N]) on the stream of
 * device index 0 of no context (the current device, default stream).  bn is
 * 128 or 256.  x_lo / w_lo select the 2- / 3-pass split form when non-NULL. */
FFWD_B200_API int ffwd_b200_gemm_bf16(const void *x, const void *x_lo, const void *w,
                                      const void *w_lo, float *y, int M, int N, int K, int bn);
/* Y = X W^T in kind::tf32 (the tf32 plan's GEMM) on device pointers: f32 X [M, K],
 * f32 W [N, K] (read as tf32), f32 Y [M, N]; K a multiple of 64, N of bn. */
FFWD_B200_API int ffwd_b200_gemm_tf32(const float *x, const float *w, float *y, int M, int N, int K,
                                      int bn);

#ifdef __cplusplus
}
#endif

#endif /* FFWD_B200_H */
