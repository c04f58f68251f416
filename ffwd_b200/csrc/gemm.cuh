// Projection GEMM for the packed token matrix: Y[M, N] = X[M, K] * W[N, K]^T
// on the sm_100a tensor cores (tcgen05.mma, accumulators in TMEM, operands
// staged by TMA), with the layer's elementwise work fused into the epilogue.
//
// Replaces the reference's cuBLAS / cuBLASLt projections (libffwd/cuda.cu
// linear_ex 2905-2969, linear_lt 3058-3182, linear_accum 3030-3038) and the
// elementwise kernels that followed them (add_row_bias 402-407,
// rms_norm_rope_qk 538-606, silu_mul_packed 611-624, bias_gelu* 2616-2708).
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace fb {

// Epilogue kinds.
enum GemmEpi : int {
    kEpiStore = 0,   // out = acc (+ bias)
    kEpiGelu = 1,    // out = gelu(acc + bias)            (erf or tanh curve)
    kEpiResid = 2,   // resid[M, N] += acc (+ bias)       (f32, in place)
    kEpiSwiGLU = 3,  // tile = [gate | up] halves -> out = silu(gate) * up
    kEpiQKRope = 4,  // (+ bias) per-head RMSNorm (q/k heads) + NeoX RoPE
};

// Output encodings.
enum OutMode : int {
    kOutBF16 = 0,
    kOutF32 = 1,
    kOutSplit = 2,  // bf16 hi in `out`, bf16 lo (x - hi) in `out_lo`
    kOutF16 = 3,
    kOutTF32 = 4,   // f32 rounded to tf32 (operand of the next kind::tf32 GEMM)
};

struct GemmParams {
    int M, N, K;
    int epi;
    int out_mode;
    int op_f16;            // A and B are f16 (else bf16)
    void *out;
    void *out_lo;
    int ldo;               // output row stride (elements)
    float *resid;          // kEpiResid target [M, ldr]
    int ldr;
    const float *bias;     // [N] or null
    int gelu_tanh;         // kEpiGelu curve
    // kEpiQKRope
    const int *pos;        // [M] position of each packed row
    const float *rope_cos; // [n_pos, head_dim / 2]
    const float *rope_sin;
    const __half *rope_cos_h;  // the same tables in f16 (single-pass bf16 GEMM)
    const __half *rope_sin_h;
    const float *q_norm;   // [head_dim] or null (no QK-norm)
    const float *k_norm;
    int n_q_heads, n_kv_heads, head_dim;
    float eps;
    int *err;
};

// Host launcher.  Each tensor map is 2-D with a 128-byte box row and 128-byte
// swizzle: 16-bit (bf16, or f16 with op_f16) with 64-column boxes, or, for
// passes = 4, f32 with 32-column boxes.  A maps cover X (box rows 128), B maps
// cover W (box rows BN).  `passes` = 1: A*B; 2: (A + A_lo)*B;
// 3: A*B + A*B_lo + A_lo*B; 4: A*B in kind::tf32.
// Returns a cudaError_t value.
int gemm_launch(const CUtensorMap *a, const CUtensorMap *a_lo, const CUtensorMap *b,
                const CUtensorMap *b_lo, int bn, int passes, const GemmParams &p, int num_sms,
                cudaStream_t stream);

// Two-SM variant (cluster of two CTAs, tcgen05.mma.cta_group::2, M = 256 per
// pair) for single-pass bf16 with N a multiple of 256.  `b_half` maps W with a
// box of 128 rows x 64 columns (each CTA loads its half of a 256-row tile).
// `out` maps the epilogue's destination with a box of 128 rows x 32 columns:
// the output (bf16, 64-byte swizzle; or f32, 128-byte swizzle) or, for
// kEpiResid, the f32 residual (128-byte swizzle), which TMA adds into.
int gemm2_launch(const CUtensorMap *a, const CUtensorMap *b_half, const CUtensorMap *out,
                 const GemmParams &p, int num_sms, cudaStream_t stream);

}  // namespace fb
