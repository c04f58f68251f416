// Packed variable-length attention over the fused QKV projection.
//
// Replaces the reference's attention dispatch (libffwd/cuda.cu
// cuda_attention_gemm 3369-3799): the mma.sync flash kernels
// (attn_stream_tc128_bf16_kv_ldm 1187-1478, attn_stream_bert_flash 1564-2142),
// the cuDNN ragged SDPA (cuda_sdpa.cu:252-341) and the materialised f32 path
// (3689-3797, replaced by the split-bf16 tensor-core kernel).  Semantics follow the CPU path (libffwd/attn.c:50-458):
// softmax(q k^T / sqrt(d)) v per sequence, key/value head = h / (nh / nkv),
// causal or bidirectional, sequences never attend across their boundary.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace fb {

// One work item: two query blocks of 128 rows that share their keys and
// values, block 0 = (query tile qt0, head h0), block 1 = (qt1, h1); qt1 = h1 =
// -1 when the item has block 0 only.  Tiles count from the first row of
// sequence `seq`.  nseq > 0 makes the item a window over the nseq consecutive
// short sequences seq .. seq + nseq - 1 (at most 128 rows when the two blocks
// are two heads, 256 when they are the window's two 128-row halves): its keys
// are the window's rows and each query row sees only its own sequence.
struct AttnItem {
    int seq;
    int qt0, h0;
    int qt1, h1;
    int cost;  // key tiles, for heaviest-first ordering
    int nseq;  // 0: one sequence; > 0: window of nseq short sequences
};

struct AttnParams {
    const int *offsets;     // [batch + 1] packed row offsets
    const AttnItem *items;  // [n_items]
    int n_items;
    int n_heads, n_kv_heads, head_dim;
    int q_col0, k_col0, v_col0;  // column of head 0 of Q / K / V inside a qkv row
    int causal;
    float scale;            // 1 / sqrt(head_dim)
    // 16-bit plans: qkv and output [T, ldo] in bf16, or f16 when f16 is set
    int f16;
    __nv_bfloat16 *out;
    int ldo;
    // exact plans (qkv as bf16 hi / lo matrices)
    __nv_bfloat16 *out_hi;  // split output (hi / lo) for the next 2- or 3-pass GEMM
    __nv_bfloat16 *out_lo;
    float *out_tf32;        // or, when set, f32 rounded to tf32 for a kind::tf32 GEMM
    int *err;
    int *sched;             // 16-bit plans: 2 ints (claim counter, exit count), zero
                            // before the first launch; the kernel rewinds them on exit
};

// Build the work list of a packed batch (host): pairs of 128-row query blocks
// sharing a key/value head (two query heads of a group, or two adjacent query
// tiles when every head has its own key/value head), ordered longest sequence
// first with the items of one key/value head together.  With `windows`,
// sequences of at most 128 rows that are neighbours in the packed layout share
// items (windows, see AttnItem), placed after the rest; only the 16-bit
// kernel reads windows.  Writes at most cap items to out; returns the count,
// or -1 if cap is too small.  Allocates nothing beyond a sequence order of
// `batch` ints.
int attention_build_items(int causal, int n_heads, int n_kv_heads, const int *h_offsets,
                          int batch, AttnItem *out, int cap, bool windows = false);
// Number of items attention_build_items would write without windows (an upper
// bound with them).
int attention_count_items(int n_heads, int n_kv_heads, const int *h_offsets, int batch);

// 16-bit plans.  `qkv_map`: 2-D 16-bit map over the qkv matrix with a box of
// 128 rows x min(head_dim, 64) columns (128-byte swizzle, or 64-byte for
// head_dim 32).
int attention_tc_launch(const CUtensorMap *qkv_map, const AttnParams &p, cudaStream_t stream);

// Tensor-core path of the exact plans: qkv as bf16 hi / lo matrices (two maps
// like `qkv_map` above); items are the tensor-core items (grid of 2 x n_items
// CTAs, one per query block); output split into out_hi / out_lo, or tf32-rounded
// f32 into out_tf32 when set.
int attention_split_launch(const CUtensorMap *qkv_hi_map, const CUtensorMap *qkv_lo_map,
                           const AttnParams &p, cudaStream_t stream);

}  // namespace fb
