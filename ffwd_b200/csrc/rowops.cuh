// Memory-bound row kernels of the forward: embedding gathers, RMSNorm,
// LayerNorm and pooling.  One warp per packed token row (128-bit loads,
// warp-shuffle reductions) except pooling (one CTA per sequence).
//
// Replace the reference's ffwd_lookup_kernel (libffwd/cuda.cu:409-429),
// bert_embed_layer_norm* (2195-2377), rms_norm_kernel (517-531),
// layer_norm_bias* (2382-2614), the pool kernels (2144-2190) and the host
// ffwd_l2_normalize (vec.c:7-22) after the D2H copy (cuda.cu:5133-5138).
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace fb {

// Encoding of the bf16 operand a row kernel writes for the next GEMM.
struct RowOut {
    __nv_bfloat16 *hi;  // bf16 value (RNE), or f16 when f16 is set
    __nv_bfloat16 *lo;  // remainder (x - hi) in bf16, or null (single-pass GEMMs)
    int f16;            // single-pass f16 operand (lo unused)
    float *tf32;        // when set: f32 rounded to tf32 instead (hi, lo unused)
};

// Qwen: x[t] = E[ids[t]] (f32 or bf16 table), xn = RMSNorm(x) * w (if w).
int embed_rms_launch(const int *ids, int T, const void *table, int table_bf16, int vocab, int H,
                     float *x, const float *w, float eps, RowOut xn, int *err, cudaStream_t s);

// BERT: x[t] = LN(E[ids[t]] + P[pos[t]] + type0) (f32) and its operand copy.
int embed_ln_launch(const int *ids, const int *pos, int T, const void *table, int table_bf16,
                    int vocab, const float *pos_table, const float *type0, const float *g,
                    const float *b, int H, float eps, float *x, RowOut xb, int *err,
                    cudaStream_t s);

// xn = RMSNorm(x) * w.
int rmsnorm_launch(const float *x, int T, int H, const float *w, float eps, RowOut xn,
                   cudaStream_t s);

// x = LN(x) * g + b in place, plus the operand copy.
int layernorm_launch(float *x, int T, int H, const float *g, const float *b, float eps,
                     RowOut xb, cudaStream_t s);

// Pooling of each sequence of the packed rows x [T, H]:
// mode 0 mean, 1 last token, 2 first token.  norm_w (Qwen final RMSNorm) is
// applied per pooled row when non-null; normalize applies L2.
int pool_launch(const float *x, const int *offsets, int batch, int H, int mode,
                const float *norm_w, float eps, int normalize, float *out, int *err,
                cudaStream_t s);

// Mean of each span of final hidden states (contextual spans): span i covers
// rows [starts[i], ends[i]); norm_w (Qwen final RMSNorm) applies per row.
int span_pool_launch(const float *x, const int *starts, const int *ends, int n_spans, int H,
                     const float *norm_w, float eps, float *out, cudaStream_t s);

// Output encodings of pooled embeddings emb [B, H] (server wire forms,
// tools/server/encode.c:20-61, 107-122): the first `dims` values, L2-renormalised
// when `renorm` (Matryoshka truncation), then enc 0: f32 [B, dims]; enc 1:
// int8 round(tanh(x) * 127) clamped to [-128, 127], [B, dims]; enc 2: one bit
// per value (x >= 0), 8 per byte least significant first, [B, dims / 8].
// A zero / non-finite truncated norm records kErrBadNorm.
int encode_rows_launch(const float *emb, int B, int H, int dims, int renorm, int enc, void *out,
                       int *err, cudaStream_t s);

}  // namespace fb
