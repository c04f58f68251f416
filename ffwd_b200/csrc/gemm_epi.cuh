// Fused GEMM epilogues shared by the 1-SM and 2-SM tcgen05 GEMM kernels:
// each epilogue thread owns one accumulator row (TMEM lane) of a 128-row tile
// and processes its columns 32 at a time; warpgroup g of kEpiGroups takes every
// kEpiGroups-th unit of the tile.
#pragma once

#include "gemm.cuh"
#include "ptx.cuh"

namespace fb {
namespace epi {

constexpr int kEpiGroups = 2;

__device__ __forceinline__ float gelu_erf(float x) {
    return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
}

__device__ __forceinline__ float gelu_tanh(float x) {
    float inner = 0.79788456080286536f * (x + 0.044715f * x * x * x);
    return 0.5f * x * (1.0f + tanhf(inner));
}

// GELU for 16-bit outputs (the single-pass two-SM GEMM), as x * sigmoid(u) =
// x / (1 + 2^-u'), two MUFU operations instead of erff / tanhf:
// - erf form: 0.5 (1 + erf(x / sqrt 2)) = sigmoid(q(x)) with q an odd quintic
//   fitted here (weighted least squares on |x| <= 8.5): erf matched to 3.7e-5,
//   GELU to 5.5e-5 absolute, far below the 16-bit output's rounding; |x| is
//   clamped to 8.5 inside q (beyond, GELU is x or 0 in f32);
// - tanh form: 0.5 (1 + tanh(v)) = sigmoid(2 v) exactly, v = sqrt(2 / pi) (x +
//   0.044715 x^3) as in the reference's gelu_new.
// The exact plans keep erff / tanhf (their outputs feed f32 comparisons).
__device__ __forceinline__ float gelu_erf_fast(float x) {
    const float c = fminf(fmaxf(x, -8.5f), 8.5f);
    const float c2 = c * c;
    // -2 log2(e) q(c): the exponent of 2 in the sigmoid's denominator.
    const float e = c * fmaf(fmaf(9.1122725e-4f, c2, -0.10617733f), c2, -2.3017271f);
    return __fdividef(x, 1.0f + ex2_approx(e));
}

__device__ __forceinline__ float gelu_tanh_fast(float x) {
    // -2 log2(e) sqrt(2 / pi) = -2.3022082; times 0.044715 = -0.1029432
    const float e = x * fmaf(-0.1029432f, x * x, -2.3022082f);
    return __fdividef(x, 1.0f + ex2_approx(e));
}

__device__ __forceinline__ void add_bias32(float (&v)[32], const float *bias, int col) {
    const float4 *b4 = reinterpret_cast<const float4 *>(bias + col);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        float4 b = __ldg(b4 + i);
        v[4 * i + 0] += b.x;
        v[4 * i + 1] += b.y;
        v[4 * i + 2] += b.z;
        v[4 * i + 3] += b.w;
    }
}

// SiLU(x) = x / (1 + e^-x) with the fast intrinsics: __expf (ex2.approx of
// x * log2 e) and __fdividef (reciprocal-multiply), a few instructions where
// expf and the IEEE division take tens; relative error about 1e-6 for |x| < 20,
// far below the bf16 rounding of the output and the 1e-4 gate of the exact
// plans.  For x below about -88, e^-x overflows and the result is -0, the limit.
__device__ __forceinline__ float silu_fast(float x) {
    return __fdividef(x, 1.0f + __expf(-x));
}

// Store 32 consecutive values of one row in the requested encoding.
__device__ __forceinline__ void store_row32(const GemmParams &p, int row, int col,
                                            const float (&v)[32]) {
    const size_t off = (size_t)row * p.ldo + col;
    if (p.out_mode == kOutF32) {
        float4 *o = reinterpret_cast<float4 *>(static_cast<float *>(p.out) + off);
#pragma unroll
        for (int i = 0; i < 8; ++i)
            o[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        return;
    }
    if (p.out_mode == kOutTF32) {
        float4 *o = reinterpret_cast<float4 *>(static_cast<float *>(p.out) + off);
#pragma unroll
        for (int i = 0; i < 8; ++i)
            o[i] = make_float4(round_tf32(v[4 * i]), round_tf32(v[4 * i + 1]),
                               round_tf32(v[4 * i + 2]), round_tf32(v[4 * i + 3]));
        return;
    }
    uint32_t hi[16];
    uint32_t lo[16];
    if (p.out_mode == kOutF16) {
#pragma unroll
        for (int i = 0; i < 16; ++i) hi[i] = pack_f16x2(v[2 * i], v[2 * i + 1]);
    } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            __nv_bfloat16 h0 = __float2bfloat16_rn(v[2 * i]);
            __nv_bfloat16 h1 = __float2bfloat16_rn(v[2 * i + 1]);
            __nv_bfloat162 hh(h0, h1);
            hi[i] = *reinterpret_cast<uint32_t *>(&hh);
            if (p.out_mode == kOutSplit)
                lo[i] = pack_bf16x2(v[2 * i] - __bfloat162float(h0),
                                    v[2 * i + 1] - __bfloat162float(h1));
        }
    }
    uint4 *o = reinterpret_cast<uint4 *>(static_cast<__nv_bfloat16 *>(p.out) + off);
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = make_uint4(hi[4 * i], hi[4 * i + 1], hi[4 * i + 2], hi[4 * i + 3]);
    if (p.out_mode == kOutSplit) {
        uint4 *ol = reinterpret_cast<uint4 *>(static_cast<__nv_bfloat16 *>(p.out_lo) + off);
#pragma unroll
        for (int i = 0; i < 4; ++i)
            ol[i] = make_uint4(lo[4 * i], lo[4 * i + 1], lo[4 * i + 2], lo[4 * i + 3]);
    }
}

// Writes each thread's row segments straight to global memory.
struct DirectSink {
    static constexpr bool kAllRows = false;  // rows past M skip their work
    static constexpr bool kFastGelu = false;  // erff / tanhf (also the exact plans)
    static constexpr bool kHalfRope = false;  // RoPE from the f32 tables
    const GemmParams &p;
    int grow;
    __device__ __forceinline__ void put(const float (&v)[32], int col) { store_row32(p, grow, col, v); }
    // Head-at-a-time output (the QK-norm / RoPE epilogue): stores go straight out.
    __device__ __forceinline__ void begin_head() {}
    __device__ __forceinline__ void stage32(const float (&v)[32], int col0, int local) {
        store_row32(p, grow, col0 + local, v);
    }
    __device__ __forceinline__ void commit_head(int) {}
    __device__ __forceinline__ void add(const float (&v)[32], int col) {
        float4 *r = reinterpret_cast<float4 *>(p.resid + (size_t)grow * p.ldr + col);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float4 x = r[i];
            x.x += v[4 * i];
            x.y += v[4 * i + 1];
            x.z += v[4 * i + 2];
            x.w += v[4 * i + 3];
            r[i] = x;
        }
    }
};

template <int BN, int EPI, typename Sink>
__device__ __forceinline__ void epilogue_tile(const GemmParams &p, uint32_t tbase, int grow,
                                              bool valid, int nb, int g, Sink &sink) {
    // Warpgroup g of kEpiGroups handles every kEpiGroups-th unit of the tile.
    const int n0 = nb * BN;
    if constexpr (EPI == kEpiStore || EPI == kEpiGelu) {
#pragma unroll 1
        for (int c = g; c < BN / 32; c += kEpiGroups) {
            float v[32];
            tmem_ld32(tbase + c * 32, v);
            tmem_wait_ld();
            if (!Sink::kAllRows && !valid) continue;
            const int col = n0 + c * 32;
            if (p.bias) add_bias32(v, p.bias, col);
            if constexpr (EPI == kEpiGelu && Sink::kFastGelu) {
                if (p.gelu_tanh) {
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = gelu_tanh_fast(v[i]);
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = gelu_erf_fast(v[i]);
                }
            } else if constexpr (EPI == kEpiGelu) {
                if (p.gelu_tanh) {
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = gelu_tanh(v[i]);
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = gelu_erf(v[i]);
                }
            }
            sink.put(v, col);
        }
    } else if constexpr (EPI == kEpiResid) {
#pragma unroll 1
        for (int c = g; c < BN / 32; c += kEpiGroups) {
            float v[32];
            tmem_ld32(tbase + c * 32, v);
            tmem_wait_ld();
            if (!Sink::kAllRows && !valid) continue;
            const int col = n0 + c * 32;
            if (p.bias) add_bias32(v, p.bias, col);
            sink.add(v, col);
        }
    } else if constexpr (EPI == kEpiSwiGLU) {
        const int o0 = nb * (BN / 2);
#pragma unroll 1
        for (int c = g; c < BN / 64; c += kEpiGroups) {
            float g[32], u[32];
            tmem_ld32(tbase + c * 32, g);
            tmem_ld32(tbase + BN / 2 + c * 32, u);
            tmem_wait_ld();
            if (!Sink::kAllRows && !valid) continue;
#pragma unroll
            for (int i = 0; i < 32; ++i) g[i] = silu_fast(g[i]) * u[i];
            sink.put(g, o0 + c * 32);
        }
    } else if constexpr (EPI == kEpiQKRope) {
        const int hd = p.head_dim;
        const int half = hd / 2;
        const int nq = p.n_q_heads, nkv = p.n_kv_heads;
        const int ps = valid ? __ldg(p.pos + grow) : 0;
#pragma unroll 1
        for (int h0 = g * hd; h0 < BN; h0 += kEpiGroups * hd) {
            const int col0 = n0 + h0;
            const int gh = col0 / hd;
            const bool is_q = gh < nq;
            const bool is_k = !is_q && gh < nq + nkv;
            sink.begin_head();
            if (!is_q && !is_k) {
#pragma unroll 1
                for (int c = 0; c < hd / 32; ++c) {
                    float v[32];
                    tmem_ld32(tbase + h0 + c * 32, v);
                    tmem_wait_ld();
                    if (!Sink::kAllRows && !valid) continue;
                    if (p.bias) add_bias32(v, p.bias, col0 + c * 32);
                    sink.stage32(v, col0, c * 32);
                }
                sink.commit_head(col0);
                continue;
            }
            const float *nw = is_q ? p.q_norm : p.k_norm;
            // f16 tables: the first chunk's cos / sin (64 halves) are loaded
            // before the sum-of-squares pass, later chunks' between the previous
            // chunk's two stores, so the L2 latency overlaps other work.
            const uint4 *c8 = reinterpret_cast<const uint4 *>(p.rope_cos_h + (size_t)ps * half);
            const uint4 *s8 = reinterpret_cast<const uint4 *>(p.rope_sin_h + (size_t)ps * half);
            uint4 cv[4], sv[4];
            if constexpr (Sink::kHalfRope) {
                if (half >= 32) {
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        cv[i] = __ldg(c8 + i);
                        sv[i] = __ldg(s8 + i);
                    }
                }
            }
            float inv = 1.0f;
            if (nw) {
                // Two 32-column TMEM loads per wait.
                float2 s2 = make_float2(0.0f, 0.0f);
#pragma unroll 1
                for (int c = 0; c < hd / 32; c += 2) {
                    float v[32], u[32];
                    tmem_ld32(tbase + h0 + c * 32, v);
                    tmem_ld32(tbase + h0 + c * 32 + 32, u);
                    tmem_wait_ld();
                    if (p.bias && valid) {
                        add_bias32(v, p.bias, col0 + c * 32);
                        add_bias32(u, p.bias, col0 + c * 32 + 32);
                    }
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const float2 x = make_float2(v[2 * i], v[2 * i + 1]);
                        s2 = fma_f32x2(x, x, s2);
                    }
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const float2 x = make_float2(u[2 * i], u[2 * i + 1]);
                        s2 = fma_f32x2(x, x, s2);
                    }
                }
                inv = 1.0f / sqrtf((s2.x + s2.y) / (float)hd + p.eps);
            }
            if constexpr (Sink::kHalfRope) {
#pragma unroll 1
                for (int c = 0; c < half / 32; ++c) {
                    float x1[32], x2[32];
                    tmem_ld32(tbase + h0 + c * 32, x1);
                    tmem_ld32(tbase + h0 + half + c * 32, x2);
                    tmem_wait_ld();
                    if (p.bias) {
                        add_bias32(x1, p.bias, col0 + c * 32);
                        add_bias32(x2, p.bias, col0 + half + c * 32);
                    }
                    // Packed pairs: x *= w (norm weight), then the rotation with
                    // the row's 1 / rms folded into cos and sin.
                    if (nw) {
                        const float4 *w1 = reinterpret_cast<const float4 *>(nw + c * 32);
                        const float4 *w2 = reinterpret_cast<const float4 *>(nw + half + c * 32);
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const float4 a = __ldg(w1 + i), b = __ldg(w2 + i);
                            const float2 p0 = mul_f32x2(make_float2(x1[4 * i], x1[4 * i + 1]), make_float2(a.x, a.y));
                            const float2 p1 = mul_f32x2(make_float2(x1[4 * i + 2], x1[4 * i + 3]), make_float2(a.z, a.w));
                            const float2 q0 = mul_f32x2(make_float2(x2[4 * i], x2[4 * i + 1]), make_float2(b.x, b.y));
                            const float2 q1 = mul_f32x2(make_float2(x2[4 * i + 2], x2[4 * i + 3]), make_float2(b.z, b.w));
                            x1[4 * i] = p0.x; x1[4 * i + 1] = p0.y; x1[4 * i + 2] = p1.x; x1[4 * i + 3] = p1.y;
                            x2[4 * i] = q0.x; x2[4 * i + 1] = q0.y; x2[4 * i + 2] = q1.x; x2[4 * i + 3] = q1.y;
                        }
                    }
                    const float2 inv2 = make_float2(inv, inv), ninv2 = make_float2(-inv, -inv);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const __half2 *ch = reinterpret_cast<const __half2 *>(&cv[i]);
                        const __half2 *sh = reinterpret_cast<const __half2 *>(&sv[i]);
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const float2 cf = __half22float2(ch[u]), sf = __half22float2(sh[u]);
                            const int e = 8 * i + 2 * u;
                            const float2 a = make_float2(x1[e], x1[e + 1]);
                            const float2 bb = make_float2(x2[e], x2[e + 1]);
                            const float2 ci = mul_f32x2(cf, inv2);
                            const float2 r1 = fma_f32x2(bb, mul_f32x2(sf, ninv2), mul_f32x2(a, ci));
                            const float2 r2 = fma_f32x2(a, mul_f32x2(sf, inv2), mul_f32x2(bb, ci));
                            x1[e] = r1.x; x1[e + 1] = r1.y;
                            x2[e] = r2.x; x2[e + 1] = r2.y;
                        }
                    }
                    sink.stage32(x1, col0, c * 32);
                    if (c + 1 < half / 32) {
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            cv[i] = __ldg(c8 + (c + 1) * 4 + i);
                            sv[i] = __ldg(s8 + (c + 1) * 4 + i);
                        }
                    }
                    sink.stage32(x2, col0, half + c * 32);
                }
                sink.commit_head(col0);
                continue;
            }
            const float *cs = p.rope_cos + (size_t)ps * half;
            const float *sn = p.rope_sin + (size_t)ps * half;
#pragma unroll 1
            for (int c = 0; c < half / 32; ++c) {
                float x1[32], x2[32];
                tmem_ld32(tbase + h0 + c * 32, x1);
                tmem_ld32(tbase + h0 + half + c * 32, x2);
                tmem_wait_ld();
                if (!Sink::kAllRows && !valid) continue;
                if (p.bias) {
                    add_bias32(x1, p.bias, col0 + c * 32);
                    add_bias32(x2, p.bias, col0 + half + c * 32);
                }
                if (nw) {
                    const float4 *w1 = reinterpret_cast<const float4 *>(nw + c * 32);
                    const float4 *w2 = reinterpret_cast<const float4 *>(nw + half + c * 32);
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const float4 a = __ldg(w1 + i), b = __ldg(w2 + i);
                        x1[4 * i] = x1[4 * i] * inv * a.x; x1[4 * i + 1] = x1[4 * i + 1] * inv * a.y;
                        x1[4 * i + 2] = x1[4 * i + 2] * inv * a.z; x1[4 * i + 3] = x1[4 * i + 3] * inv * a.w;
                        x2[4 * i] = x2[4 * i] * inv * b.x; x2[4 * i + 1] = x2[4 * i + 1] * inv * b.y;
                        x2[4 * i + 2] = x2[4 * i + 2] * inv * b.z; x2[4 * i + 3] = x2[4 * i + 3] * inv * b.w;
                    }
                }
                const float4 *c4 = reinterpret_cast<const float4 *>(cs + c * 32);
                const float4 *s4 = reinterpret_cast<const float4 *>(sn + c * 32);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float4 cv = __ldg(c4 + i), sv = __ldg(s4 + i);
                    const float cc[4] = {cv.x, cv.y, cv.z, cv.w};
                    const float ss[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const float a = x1[4 * i + u], b = x2[4 * i + u];
                        x1[4 * i + u] = a * cc[u] - b * ss[u];
                        x2[4 * i + u] = b * cc[u] + a * ss[u];
                    }
                }
                sink.stage32(x1, col0, c * 32);
                sink.stage32(x2, col0, half + c * 32);
            }
            sink.commit_head(col0);
        }
    }
}

}  // namespace epi
}  // namespace fb
