// tcgen05 projection GEMM with fused epilogues (see gemm.cuh).
//
// Kernel shape: persistent, one CTA per SM (the smem ring fills the SM), 192
// threads in three roles:
//   warp 0      TMA producer: streams 128x64 X tiles and BNx64 W tiles into a
//               STAGES-deep shared-memory ring (128-byte swizzle).
//   warp 1      allocates TMEM, then one lane issues tcgen05.mma (M=128, N=BN,
//               K=16 per instruction) into one of two TMEM accumulators and
//               frees ring slots / publishes accumulators with tcgen05.commit.
//   warps 2-5   epilogue: each thread owns one accumulator row (TMEM lane),
//               reads it with tcgen05.ld 32 columns at a time, applies the fused
//               elementwise work and writes the row segment to global memory.
// Two TMEM accumulators let the epilogue of tile i overlap the MMAs of tile i+1.
#include "gemm.cuh"
#include "ptx.cuh"

#include <cuda_runtime.h>

namespace fb {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = one 128-byte swizzle row
constexpr int kEpiGroups = 2;  // epilogue warpgroups (split each tile's columns)
constexpr int kThreads = 64 + 128 * kEpiGroups;

template <int BN, int PASSES>
struct GemmCfg {
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int N_A = PASSES >= 2 ? 2 : 1;
    static constexpr int N_B = PASSES == 3 ? 2 : 1;
    static constexpr int STAGE_BYTES = A_BYTES * N_A + B_BYTES * N_B;
    static constexpr int STAGES_RAW = (200 * 1024) / STAGE_BYTES;
    static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
    static constexpr int SMEM = STAGES * STAGE_BYTES + 1024;
    static constexpr int TMEM_COLS = 2 * BN;
};

__device__ __forceinline__ float gelu_erf(float x) {
    return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
}

__device__ __forceinline__ float gelu_tanh(float x) {
    float inner = 0.79788456080286536f * (x + 0.044715f * x * x * x);
    return 0.5f * x * (1.0f + tanhf(inner));
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
    uint32_t hi[16];
    uint32_t lo[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        __nv_bfloat16 h0 = __float2bfloat16_rn(v[2 * i]);
        __nv_bfloat16 h1 = __float2bfloat16_rn(v[2 * i + 1]);
        __nv_bfloat162 hh(h0, h1);
        hi[i] = *reinterpret_cast<uint32_t *>(&hh);
        if (p.out_mode == kOutSplit)
            lo[i] = pack_bf16x2(v[2 * i] - __bfloat162float(h0), v[2 * i + 1] - __bfloat162float(h1));
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

template <int BN, int EPI>
__device__ __forceinline__ void epilogue_tile(const GemmParams &p, uint32_t tbase, int grow,
                                              bool valid, int nb, int g) {
    // Warpgroup g of kEpiGroups handles every kEpiGroups-th unit of the tile.
    const int n0 = nb * BN;
    if constexpr (EPI == kEpiStore || EPI == kEpiGelu) {
#pragma unroll 1
        for (int c = g; c < BN / 32; c += kEpiGroups) {
            float v[32];
            tmem_ld32(tbase + c * 32, v);
            tmem_wait_ld();
            if (!valid) continue;
            const int col = n0 + c * 32;
            if (p.bias) add_bias32(v, p.bias, col);
            if constexpr (EPI == kEpiGelu) {
                if (p.gelu_tanh) {
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = gelu_tanh(v[i]);
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = gelu_erf(v[i]);
                }
            }
            store_row32(p, grow, col, v);
        }
    } else if constexpr (EPI == kEpiResid) {
#pragma unroll 1
        for (int c = g; c < BN / 32; c += kEpiGroups) {
            float v[32];
            tmem_ld32(tbase + c * 32, v);
            tmem_wait_ld();
            if (!valid) continue;
            const int col = n0 + c * 32;
            if (p.bias) add_bias32(v, p.bias, col);
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
    } else if constexpr (EPI == kEpiSwiGLU) {
        const int o0 = nb * (BN / 2);
#pragma unroll 1
        for (int c = g; c < BN / 64; c += kEpiGroups) {
            float g[32], u[32];
            tmem_ld32(tbase + c * 32, g);
            tmem_ld32(tbase + BN / 2 + c * 32, u);
            tmem_wait_ld();
            if (!valid) continue;
#pragma unroll
            for (int i = 0; i < 32; ++i) g[i] = (g[i] / (1.0f + expf(-g[i]))) * u[i];
            store_row32(p, grow, o0 + c * 32, g);
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
            if (!is_q && !is_k) {
#pragma unroll 1
                for (int c = 0; c < hd / 32; ++c) {
                    float v[32];
                    tmem_ld32(tbase + h0 + c * 32, v);
                    tmem_wait_ld();
                    if (!valid) continue;
                    if (p.bias) add_bias32(v, p.bias, col0 + c * 32);
                    store_row32(p, grow, col0 + c * 32, v);
                }
                continue;
            }
            const float *nw = is_q ? p.q_norm : p.k_norm;
            float inv = 1.0f;
            if (nw) {
                float ss = 0.0f;
#pragma unroll 1
                for (int c = 0; c < hd / 32; ++c) {
                    float v[32];
                    tmem_ld32(tbase + h0 + c * 32, v);
                    tmem_wait_ld();
                    if (p.bias && valid) add_bias32(v, p.bias, col0 + c * 32);
#pragma unroll
                    for (int i = 0; i < 32; ++i) ss += v[i] * v[i];
                }
                inv = 1.0f / sqrtf(ss / (float)hd + p.eps);
            }
            const float *cs = p.rope_cos + (size_t)ps * half;
            const float *sn = p.rope_sin + (size_t)ps * half;
#pragma unroll 1
            for (int c = 0; c < half / 32; ++c) {
                float x1[32], x2[32];
                tmem_ld32(tbase + h0 + c * 32, x1);
                tmem_ld32(tbase + h0 + half + c * 32, x2);
                tmem_wait_ld();
                if (!valid) continue;
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
                store_row32(p, grow, col0 + c * 32, x1);
                store_row32(p, grow, col0 + half + c * 32, x2);
            }
        }
    }
}

template <int BN, int PASSES, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmA2,
                const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmB2,
                const GemmParams p) {
    using C = GemmCfg<BN, PASSES>;
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t full_bar[C::STAGES];
    __shared__ __align__(8) uint64_t empty_bar[C::STAGES];
    __shared__ __align__(8) uint64_t tfull_bar[2];
    __shared__ __align__(8) uint64_t tempty_bar[2];
    __shared__ __align__(8) uint64_t drain_bar;
    __shared__ uint32_t tmem_base_sh;
    __shared__ int abort_sh;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));

    const int m_blocks = (p.M + BM - 1) / BM;
    const int n_blocks = p.N / BN;
    const int num_tiles = m_blocks * n_blocks;
    const int k_blocks = p.K / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull_bar[a], 1);
            mbar_init(&tempty_bar[a], 4 * kEpiGroups);
        }
        mbar_init(&drain_bar, 1);
        abort_sh = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        if (PASSES >= 2) tma_prefetch_desc(&tmA2);
        if (PASSES == 3) tma_prefetch_desc(&tmB2);
    }
    if (warp == 1) {
        tmem_alloc(&tmem_base_sh, C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = tmem_base_sh;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------------------------------------------------- producer
            const uint64_t pol_w = policy_evict_last();
            int it = 0;
            bool ok = true;
            for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
                const int mb = tile / n_blocks, nb = tile % n_blocks;
                for (int kb = 0; kb < k_blocks; ++kb) {
                    const int s = it % C::STAGES;
                    const uint32_t ph = (it / C::STAGES) & 1;
                    if (!mbar_wait(&empty_bar[s], ph ^ 1, p.err, &abort_sh)) {
                        ok = false;
                        break;
                    }
                    uint8_t *st = smem + s * C::STAGE_BYTES;
                    mbar_arrive_expect_tx(&full_bar[s], C::STAGE_BYTES);
                    tma_load_2d(st, &tmA, &full_bar[s], kb * BK, mb * BM);
                    if (PASSES >= 2) tma_load_2d(st + C::A_BYTES, &tmA2, &full_bar[s], kb * BK, mb * BM);
                    uint8_t *sb = st + C::A_BYTES * C::N_A;
                    tma_load_2d_hint(sb, &tmB, &full_bar[s], kb * BK, nb * BN, pol_w);
                    if (PASSES == 3)
                        tma_load_2d_hint(sb + C::B_BYTES, &tmB2, &full_bar[s], kb * BK, nb * BN, pol_w);
                    ++it;
                }
            }
            if (!ok) {
                // Drain: let every load already issued land before the CTA exits.
                for (int j = it - C::STAGES < 0 ? 0 : it - C::STAGES; j < it; ++j)
                    mbar_wait(&full_bar[j % C::STAGES], (j / C::STAGES) & 1, nullptr, nullptr);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------------------------------------------------- MMA issuer
            constexpr uint32_t IDESC = idesc_f16(BM, BN, 1, 1, 0, 0);
            int it = 0, lt = 0;
            bool ok = true;
            for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x, ++lt) {
                const int a = lt & 1;
                const uint32_t aph = (lt >> 1) & 1;
                if (!mbar_wait(&tempty_bar[a], aph ^ 1, p.err, &abort_sh)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + a * BN;
                for (int kb = 0; kb < k_blocks; ++kb) {
                    const int s = it % C::STAGES;
                    const uint32_t ph = (it / C::STAGES) & 1;
                    if (!mbar_wait(&full_bar[s], ph, p.err, &abort_sh)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(smem + s * C::STAGE_BYTES);
                    const uint32_t sa2 = sa + C::A_BYTES;
                    const uint32_t sb = sa + C::A_BYTES * C::N_A;
                    const uint32_t sb2 = sb + C::B_BYTES;
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
                        const uint64_t ad = smem_desc(sa + kk * 32, 16, 1024, kLayoutSW128);
                        const uint64_t bd = smem_desc(sb + kk * 32, 16, 1024, kLayoutSW128);
                        umma_f16(d, ad, bd, IDESC, (kb | kk) != 0);
                        if (PASSES >= 2) {
                            const uint64_t a2d = smem_desc(sa2 + kk * 32, 16, 1024, kLayoutSW128);
                            if (PASSES == 3) {
                                const uint64_t b2d = smem_desc(sb2 + kk * 32, 16, 1024, kLayoutSW128);
                                umma_f16(d, ad, b2d, IDESC, 1);
                            }
                            umma_f16(d, a2d, bd, IDESC, 1);
                        }
                    }
                    umma_commit(&empty_bar[s]);
                    ++it;
                }
                if (!ok) break;
                umma_commit(&tfull_bar[a]);
            }
            if (!ok) {
                // Drain: wait for every MMA already issued before TMEM is freed.
                umma_commit(&drain_bar);
                mbar_wait(&drain_bar, 0, nullptr, nullptr);
            }
        }
        __syncwarp();
    } else {
        // -------------------------------------------------------------- epilogue
        const int q = warp & 3;
        const int g = (warp - 2) >> 2;
        const int row = q * 32 + lane;
        int lt = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++lt) {
            const int a = lt & 1;
            const uint32_t aph = (lt >> 1) & 1;
            if (!mbar_wait(&tfull_bar[a], aph, p.err, &abort_sh)) break;
            tc_fence_after();
            const int mb = tile / n_blocks, nb = tile % n_blocks;
            const int grow = mb * BM + row;
            const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + a * BN;
            epilogue_tile<BN, EPI>(p, tbase, grow, grow < p.M, nb, g);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty_bar[a]);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::TMEM_COLS);
    }
}

template <int BN, int PASSES, int EPI>
int launch_t(const CUtensorMap *a, const CUtensorMap *a_lo, const CUtensorMap *b,
             const CUtensorMap *b_lo, const GemmParams &p, int num_sms, cudaStream_t stream) {
    using C = GemmCfg<BN, PASSES>;
    auto kern = gemm_kernel<BN, PASSES, EPI>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    const int tiles = ((p.M + BM - 1) / BM) * (p.N / BN);
    const int grid = tiles < num_sms ? tiles : num_sms;
    kern<<<grid, kThreads, C::SMEM, stream>>>(*a, a_lo ? *a_lo : *a, *b, b_lo ? *b_lo : *b, p);
    return cudaGetLastError();
}

template <int BN, int PASSES>
int launch_epi(const CUtensorMap *a, const CUtensorMap *a_lo, const CUtensorMap *b,
               const CUtensorMap *b_lo, const GemmParams &p, int num_sms, cudaStream_t s) {
    switch (p.epi) {
    case kEpiStore: return launch_t<BN, PASSES, kEpiStore>(a, a_lo, b, b_lo, p, num_sms, s);
    case kEpiGelu: return launch_t<BN, PASSES, kEpiGelu>(a, a_lo, b, b_lo, p, num_sms, s);
    case kEpiResid: return launch_t<BN, PASSES, kEpiResid>(a, a_lo, b, b_lo, p, num_sms, s);
    case kEpiSwiGLU: return launch_t<BN, PASSES, kEpiSwiGLU>(a, a_lo, b, b_lo, p, num_sms, s);
    case kEpiQKRope: return launch_t<BN, PASSES, kEpiQKRope>(a, a_lo, b, b_lo, p, num_sms, s);
    }
    return cudaErrorInvalidValue;
}

}  // namespace

int gemm_launch(const CUtensorMap *a, const CUtensorMap *a_lo, const CUtensorMap *b,
                const CUtensorMap *b_lo, int bn, int passes, const GemmParams &p, int num_sms,
                cudaStream_t stream) {
    if (p.M <= 0 || p.K % BK != 0 || p.N % bn != 0) return cudaErrorInvalidValue;
    if (passes >= 2 && !a_lo) return cudaErrorInvalidValue;
    if (passes == 3 && !b_lo) return cudaErrorInvalidValue;
    if (p.epi == kEpiQKRope && (p.head_dim % 64 != 0 || bn % p.head_dim != 0))
        return cudaErrorInvalidValue;
    if (bn == 256) {
        if (passes == 1) return launch_epi<256, 1>(a, a_lo, b, b_lo, p, num_sms, stream);
        if (passes == 2) return launch_epi<256, 2>(a, a_lo, b, b_lo, p, num_sms, stream);
        if (passes == 3) return launch_epi<256, 3>(a, a_lo, b, b_lo, p, num_sms, stream);
    } else if (bn == 128) {
        if (passes == 1) return launch_epi<128, 1>(a, a_lo, b, b_lo, p, num_sms, stream);
        if (passes == 2) return launch_epi<128, 2>(a, a_lo, b, b_lo, p, num_sms, stream);
        if (passes == 3) return launch_epi<128, 3>(a, a_lo, b, b_lo, p, num_sms, stream);
    }
    return cudaErrorInvalidValue;
}

}  // namespace fb
