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
#include "gemm_epi.cuh"
#include "launch_util.cuh"
#include "ptx.cuh"

#include <cuda_runtime.h>

namespace fb {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = one 128-byte swizzle row
using epi::kEpiGroups;
using epi::epilogue_tile;
constexpr int kThreads = 64 + 128 * kEpiGroups;

// PASSES 1-3: bf16 / f16 operands, 64 elements per 128-byte row; PASSES 4:
// tf32 (f32 operands), 32 elements per row.  Both take 4 MMAs of 32 bytes of K
// per stage.
template <int BN, int PASSES>
struct GemmCfg {
    static constexpr int KE = PASSES == 4 ? 32 : BK;  // K elements per stage
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int N_A = PASSES == 2 || PASSES == 3 ? 2 : 1;
    static constexpr int N_B = PASSES == 3 ? 2 : 1;
    static constexpr int STAGE_BYTES = A_BYTES * N_A + B_BYTES * N_B;
    static constexpr int STAGES_RAW = (200 * 1024) / STAGE_BYTES;
    static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
    static constexpr int SMEM = STAGES * STAGE_BYTES + 1024;
    static constexpr int TMEM_COLS = 2 * BN;
};

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
    const int k_blocks = p.K / C::KE;

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
        if (PASSES == 2 || PASSES == 3) tma_prefetch_desc(&tmA2);
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
    // Nothing above touches data of other kernels; wait for the stream's
    // previous kernel, then let the next one start launching.
    griddep_wait();
    griddep_launch();

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
                    tma_load_2d(st, &tmA, &full_bar[s], kb * C::KE, mb * BM);
                    if (C::N_A == 2)
                        tma_load_2d(st + C::A_BYTES, &tmA2, &full_bar[s], kb * C::KE, mb * BM);
                    uint8_t *sb = st + C::A_BYTES * C::N_A;
                    tma_load_2d_hint(sb, &tmB, &full_bar[s], kb * C::KE, nb * BN, pol_w);
                    if (PASSES == 3)
                        tma_load_2d_hint(sb + C::B_BYTES, &tmB2, &full_bar[s], kb * C::KE, nb * BN, pol_w);
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
            const int bf = p.op_f16 ? 0 : 1;
            const uint32_t IDESC = PASSES == 4 ? idesc_tf32(BM, BN) : idesc_f16(BM, BN, bf, bf, 0, 0);
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
                        if (PASSES == 4) {
                            umma_tf32(d, ad, bd, IDESC, (kb | kk) != 0);
                            continue;
                        }
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
            epi::DirectSink sink{p, grow};
            epilogue_tile<BN, EPI>(p, tbase, grow, grow < p.M, nb, g, sink);
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
    cudaError_t e = set_smem_once<gemm_kernel<BN, PASSES, EPI>>(C::SMEM);
    if (e != cudaSuccess) return e;
    const int tiles = ((p.M + BM - 1) / BM) * (p.N / BN);
    const int grid = tiles < num_sms ? tiles : num_sms;
    return launch_k(kern, dim3(grid), dim3(kThreads), C::SMEM, stream, *a, a_lo ? *a_lo : *a, *b,
                    b_lo ? *b_lo : *b, p);
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
    if ((passes == 2 || passes == 3) && !a_lo) return cudaErrorInvalidValue;
    if (passes == 3 && !b_lo) return cudaErrorInvalidValue;
    if (p.epi == kEpiQKRope && (p.head_dim % 64 != 0 || bn % p.head_dim != 0))
        return cudaErrorInvalidValue;
    if (bn == 256) {
        if (passes == 1) return launch_epi<256, 1>(a, a_lo, b, b_lo, p, num_sms, stream);
        if (passes == 2) return launch_epi<256, 2>(a, a_lo, b, b_lo, p, num_sms, stream);
        if (passes == 3) return launch_epi<256, 3>(a, a_lo, b, b_lo, p, num_sms, stream);
        if (passes == 4) return launch_epi<256, 4>(a, a_lo, b, b_lo, p, num_sms, stream);
    } else if (bn == 128) {
        if (passes == 1) return launch_epi<128, 1>(a, a_lo, b, b_lo, p, num_sms, stream);
        if (passes == 2) return launch_epi<128, 2>(a, a_lo, b, b_lo, p, num_sms, stream);
        if (passes == 3) return launch_epi<128, 3>(a, a_lo, b, b_lo, p, num_sms, stream);
        if (passes == 4) return launch_epi<128, 4>(a, a_lo, b, b_lo, p, num_sms, stream);
    }
    return cudaErrorInvalidValue;
}

}  // namespace fb
