// Packed variable-length attention over the fused QKV projection.
//
// Replaces the reference's attention dispatch (libffwd/cuda.cu
// cuda_attention_gemm 3369-3799): the mma.sync flash kernels
// (attn_stream_tc128_bf16_kv_ldm 1187-1478, attn_stream_bert_flash 1564-2142),
// the cuDNN ragged SDPA (cuda_sdpa.cu:252-341) and the materialised f32 path
// (3689-3797).  Semantics follow the CPU path (libffwd/attn.c:50-458):
// softmax(q k^T / sqrt(d)) v per sequence, key/value head = h / (nh / nkv),
// causal or bidirectional, sequences never attend across their boundary.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace fb {

// One work item of a CTA.  Tensor-core path: up to two query blocks
// (query tile, head) that share one key/value head, processed by the CTA's two
// softmax warpgroups over one stream of K/V tiles; qt1 = -1 when the second
// block is absent.  f32 path: (seq, qt0) with the head taken from blockIdx.y.
struct AttnItem {
    int seq;
    int qt0, h0;
    int qt1, h1;
    int cost;  // key tiles x blocks, for heaviest-first ordering
};

struct AttnParams {
    const int *offsets;     // [batch + 1] packed row offsets
    const AttnItem *items;  // [n_items]
    int n_items;
    int n_heads, n_kv_heads, head_dim;
    int q_col0, k_col0, v_col0;  // column of head 0 of Q / K / V inside a qkv row
    int causal;
    float scale;            // 1 / sqrt(head_dim)
    // bf16 tensor-core path: output bf16 [T, ldo]
    __nv_bfloat16 *out;
    int ldo;
    // f32 path
    const float *qkv_f32;   // [T, ldq]
    int ldq;
    __nv_bfloat16 *out_hi;  // split output (hi / lo) for the next 2- or 3-pass GEMM
    __nv_bfloat16 *out_lo;
    int *err;
};

// Build the work list of a packed batch (host).  tc selects the tensor-core
// pairing (128-row query tiles, two blocks per item) or the f32 path's items.
// Writes at most cap items to out, sorted heaviest first (ties in a fixed
// order); returns the count, or -1 if cap is too small.  Allocates nothing.
int attention_build_items(bool tc, int causal, int n_heads, int n_kv_heads, int head_dim,
                          const int *h_offsets, int batch, AttnItem *out, int cap);
// Number of items attention_build_items would write.
int attention_count_items(bool tc, int n_heads, int n_kv_heads, int head_dim, const int *h_offsets,
                          int batch);

// Tensor-core path.  `q_map` / `kv_map`: 2-D bf16 maps over the qkv matrix
// with boxes of 128 / 64 rows x min(head_dim, 64) columns (128-byte swizzle, or
// 64-byte for head_dim 32).
int attention_tc_launch(const CUtensorMap *q_map, const CUtensorMap *kv_map, const AttnParams &p,
                        cudaStream_t stream);

// f32 CUDA-core path for the exact (f32 / split-bf16) precision mode.  Items
// here use query tiles of attention_f32_qtile(head_dim) rows.
int attention_f32_qtile(int head_dim);
int attention_f32_launch(const AttnParams &p, cudaStream_t stream);

}  // namespace fb
