// Two-SM tcgen05 projection GEMM (cta_group::2) with the fused epilogues of
// gemm_epi.cuh, for single-pass bf16 projections with N a multiple of 256.
//
// A cluster of two CTAs (two SMs) computes a 256 x 256 output tile: CTA r holds
// rows [128 r, 128 r + 128) of the X tile and rows [128 r, 128 r + 128) of the
// 256-row W tile in its own shared memory; the leader CTA (rank 0) issues
// tcgen05.mma.cta_group::2 with M = 256, which reads A from each CTA and the two
// W halves from both, and accumulates each CTA's 128 output rows in that CTA's
// TMEM.  Compared with the one-SM kernel every SM stages half as much W per
// FLOP.  Roles per CTA (320 threads):
//   warp 0      TMA producer for this CTA's halves; the transaction bytes of both
//               CTAs complete on the leader's stage barrier.
//   warp 1      TMEM allocation (both CTAs); on the leader, the MMA issuer.  Its
//               commits arrive on the barriers of both CTAs.
//   warps 2-9   epilogue of this CTA's 128 rows (two warpgroups split columns);
//               they release an accumulator on the leader's barrier.
// No TMA load here uses cluster multicast.
#include "gemm.cuh"
#include "gemm_epi.cuh"
#include "launch_util.cuh"
#include "ptx.cuh"

#include <cuda_runtime.h>

namespace fb {
namespace {

constexpr int BM = 128;  // rows per CTA
constexpr int BN = 256;  // output columns per tile
constexpr int BK = 64;
using epi::kEpiGroups;
using epi::epilogue_tile;
constexpr int kThreads = 64 + 128 * kEpiGroups;
constexpr int A_BYTES = BM * BK * 2;         // this CTA's X rows
constexpr int B_BYTES = (BN / 2) * BK * 2;   // this CTA's half of the W tile
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
// Shared memory per epilogue kind.  The QK-norm / RoPE epilogue writes a whole
// head (128 rows x 128 16-bit columns = two 64-column boxes, 32 KB) per
// warpgroup and stores it at once; it is epilogue-bound, so it keeps 4
// mainloop stages.  The others stage 64-byte row chunks (8 KB, two per
// warpgroup) and keep 6.
template <int EPI>
struct Cfg2 {
    static constexpr bool HEAD = EPI == kEpiQKRope;
    static constexpr int STAGES = HEAD ? 4 : 6;
    static constexpr int OFF_STAGING = STAGES * STAGE_BYTES;
    static constexpr int GROUP_STAGING = HEAD ? 32768 : 2 * 8192;
    static constexpr int SMEM = OFF_STAGING + kEpiGroups * GROUP_STAGING + 1024;
};
constexpr int STAGING_BYTES = 8192;  // one 128-row x 64-byte chunk
constexpr int TMEM_COLS = 2 * BN;
constexpr uint32_t kPeerMask = 0xFEFFFFFFu;  // clears the CTA-rank bit: leader's copy

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                     : "memory");
}

// Tile load into this CTA's shared memory, transaction bytes counted on the
// barrier at `bar_leader` (leader CTA).
__device__ __forceinline__ void tma_load_2d_pair(void *dst, const CUtensorMap *m, uint32_t bar_leader,
                                                 int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(bar_leader), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void umma_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accum) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accum)
        : "memory");
}

// Arrive on the barrier at this offset in both CTAs once the issued MMAs complete.
__device__ __forceinline__ void umma_commit_pair(uint64_t *bar) {
    const uint16_t mask = 0x3;
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
        " [%0], %1;" ::"r"(smem_u32(bar)),
        "h"(mask)
        : "memory");
}

// Arrive on the leader CTA's copy of `bar`.
__device__ __forceinline__ void arrive_leader(uint64_t *bar) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(remote) : "r"(smem_u32(bar)));
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote)
                 : "memory");
}

// Epilogue output through shared memory and TMA: each 64-byte row segment of
// the warpgroup's 128 rows (32 bf16 columns, or 16 f32 columns) is written to a
// staging chunk with the 64-byte swizzle and stored, or for the residual added
// (cp.reduce ... add), by one elected thread.  Two 8 KB chunks per warpgroup
// alternate (small chunks leave room for a sixth mainloop stage, which the
// K = 2048 / 3072 projections measured 2-5 % faster with); rows past M are
// clipped by the tensor map.
struct TmaSink {
    static constexpr bool kAllRows = true;  // every row takes part in the barriers
    static constexpr bool kFastGelu = true;  // 16-bit outputs: GELU through ex2
    static constexpr bool kHalfRope = true;  // single-pass bf16 only: RoPE from f16 tables
    const GemmParams &p;
    const CUtensorMap *map;
    uint8_t *stage;  // this warpgroup's two chunks
    int r, y0, g;
    bool elected;
    int k = 0;

    __device__ __forceinline__ uint8_t *acquire() {
        uint8_t *buf = stage + (k & 1) * STAGING_BYTES;
        if (elected) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
        named_bar(1 + g, 128);
        return buf;
    }
    __device__ __forceinline__ void publish(uint8_t *buf, int col, bool reduce) {
        fence_proxy_async_smem();
        named_bar(1 + g, 128);
        if (elected) {
            if (reduce)
                asm volatile(
                    "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group"
                    " [%0, {%2, %3}], [%1];" ::"l"(reinterpret_cast<uint64_t>(map)),
                    "r"(smem_u32(buf)), "r"(col), "r"(y0)
                    : "memory");
            else
                asm volatile(
                    "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group"
                    " [%0, {%2, %3}], [%1];" ::"l"(reinterpret_cast<uint64_t>(map)),
                    "r"(smem_u32(buf)), "r"(col), "r"(y0)
                    : "memory");
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
        ++k;
    }
    // 16 f32 values (64 bytes) of this row, 64-byte swizzle.
    __device__ __forceinline__ void put_f32(uint8_t *buf, const float (&v)[32], int h) {
#pragma unroll
        for (int c = 0; c < 4; ++c)
            *reinterpret_cast<float4 *>(buf + r * 64 + ((c ^ ((r >> 1) & 3)) * 16)) =
                make_float4(v[16 * h + 4 * c], v[16 * h + 4 * c + 1], v[16 * h + 4 * c + 2],
                            v[16 * h + 4 * c + 3]);
    }
    __device__ __forceinline__ void put(const float (&v)[32], int col) {
        if (p.out_mode == kOutF32) {
            for (int h = 0; h < 2; ++h) {
                uint8_t *buf = acquire();
                put_f32(buf, v, h);
                publish(buf, col + 16 * h, false);
            }
            return;
        }
        uint8_t *buf = acquire();
        {
            const bool f16 = p.out_mode == kOutF16;
#pragma unroll
            for (int c = 0; c < 4; ++c)
                *reinterpret_cast<uint4 *>(buf + r * 64 + ((c ^ ((r >> 1) & 3)) * 16)) =
                    make_uint4(pack16x2(v[8 * c], v[8 * c + 1], f16),
                               pack16x2(v[8 * c + 2], v[8 * c + 3], f16),
                               pack16x2(v[8 * c + 4], v[8 * c + 5], f16),
                               pack16x2(v[8 * c + 6], v[8 * c + 7], f16));
        }
        publish(buf, col, false);
    }
    __device__ __forceinline__ void add(const float (&v)[32], int col) {
        for (int h = 0; h < 2; ++h) {
            uint8_t *buf = acquire();
            put_f32(buf, v, h);
            publish(buf, col + 16 * h, true);
        }
    }
    __device__ __forceinline__ void finish() {
        if (elected) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    }
    // Head-at-a-time output (QK-norm / RoPE epilogue): the warpgroup's 128 rows
    // x 128 columns go to a 32 KB staging area as two 64-column boxes (128-byte
    // rows, 128-byte swizzle) and leave in two TMA stores, with one pair of
    // warpgroup barriers per head instead of one per 32 columns.
    __device__ __forceinline__ void begin_head() {
        if (elected) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
        named_bar(1 + g, 128);
    }
    __device__ __forceinline__ void stage32(const float (&v)[32], int, int local) {
        uint8_t *box = stage + (local >> 6) * 16384;
        const int j0 = (local & 63) >> 3;  // first 16-byte chunk of the 32 values
        const bool f16 = p.out_mode == kOutF16;
#pragma unroll
        for (int c = 0; c < 4; ++c)
            *reinterpret_cast<uint4 *>(box + r * 128 + (((j0 + c) ^ (r & 7)) * 16)) =
                make_uint4(pack16x2(v[8 * c], v[8 * c + 1], f16),
                           pack16x2(v[8 * c + 2], v[8 * c + 3], f16),
                           pack16x2(v[8 * c + 4], v[8 * c + 5], f16),
                           pack16x2(v[8 * c + 6], v[8 * c + 7], f16));
    }
    __device__ __forceinline__ void commit_head(int col0) {
        fence_proxy_async_smem();
        named_bar(1 + g, 128);
        if (elected) {
            for (int b = 0; b < p.head_dim / 64; ++b)
                asm volatile(
                    "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group"
                    " [%0, {%2, %3}], [%1];" ::"l"(reinterpret_cast<uint64_t>(map)),
                    "r"(smem_u32(stage + b * 16384)), "r"(col0 + 64 * b), "r"(y0)
                    : "memory");
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
    }
};

template <int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const __grid_constant__ CUtensorMap tmOut, const GemmParams p) {
    extern __shared__ uint8_t smem_raw[];
    using CF = Cfg2<EPI>;
    constexpr int STAGES = CF::STAGES;
    __shared__ __align__(8) uint64_t full_bar[STAGES];
    __shared__ __align__(8) uint64_t empty_bar[STAGES];
    __shared__ __align__(8) uint64_t tfull_bar[2];
    __shared__ __align__(8) uint64_t tempty_bar[2];
    __shared__ __align__(8) uint64_t drain_bar;
    __shared__ uint32_t tmem_base_sh;
    __shared__ int abort_sh;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));

    const int m_blocks = (p.M + 2 * BM - 1) / (2 * BM);
    const int n_blocks = p.N / BN;
    const int num_tiles = m_blocks * n_blocks;
    const int k_blocks = p.K / BK;
    const int pair = blockIdx.x >> 1;
    const int n_pairs = gridDim.x >> 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull_bar[a], 1);
            mbar_init(&tempty_bar[a], 2 * 4 * kEpiGroups);
        }
        mbar_init(&drain_bar, 1);
        abort_sh = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        tma_prefetch_desc(&tmOut);
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&tmem_base_sh)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // both CTAs' barriers initialised before any remote use
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
            (void)pol_w;
            int it = 0;
            bool ok = true;
            for (int tile = pair; ok && tile < num_tiles; tile += n_pairs) {
                const int mb = tile / n_blocks, nb = tile % n_blocks;
                for (int kb = 0; kb < k_blocks; ++kb) {
                    const int s = it % STAGES;
                    const uint32_t ph = (it / STAGES) & 1;
                    if (!mbar_wait(&empty_bar[s], ph ^ 1, p.err, &abort_sh)) {
                        ok = false;
                        break;
                    }
                    uint8_t *st = smem + s * STAGE_BYTES;
                    if (leader) mbar_arrive_expect_tx(&full_bar[s], 2 * STAGE_BYTES);
                    const uint32_t bar = smem_u32(&full_bar[s]) & kPeerMask;
                    tma_load_2d_pair(st, &tmA, bar, kb * BK, mb * 2 * BM + rank * BM);
                    tma_load_2d_pair(st + A_BYTES, &tmB, bar, kb * BK, nb * BN + rank * (BN / 2));
                    ++it;
                }
            }
            if (!ok && leader) {
                for (int j = it - STAGES < 0 ? 0 : it - STAGES; j < it; ++j)
                    mbar_wait(&full_bar[j % STAGES], (j / STAGES) & 1, nullptr, nullptr);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (leader && lane == 0) {
            // ---------------------------------------------------------- MMA issuer
            const int bf = p.op_f16 ? 0 : 1;
            const uint32_t IDESC = idesc_f16(2 * BM, BN, bf, bf, 0, 0);
            int it = 0, lt = 0;
            bool ok = true;
            for (int tile = pair; ok && tile < num_tiles; tile += n_pairs, ++lt) {
                const int a = lt & 1;
                const uint32_t aph = (lt >> 1) & 1;
                if (!mbar_wait(&tempty_bar[a], aph ^ 1, p.err, &abort_sh)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + a * BN;
                for (int kb = 0; kb < k_blocks; ++kb) {
                    const int s = it % STAGES;
                    const uint32_t ph = (it / STAGES) & 1;
                    if (!mbar_wait(&full_bar[s], ph, p.err, &abort_sh)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(smem + s * STAGE_BYTES);
                    const uint32_t sb = sa + A_BYTES;
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk)
                        umma_pair(d, smem_desc(sa + kk * 32, 16, 1024, kLayoutSW128),
                                  smem_desc(sb + kk * 32, 16, 1024, kLayoutSW128), IDESC,
                                  (kb | kk) != 0);
                    umma_commit_pair(&empty_bar[s]);
                    ++it;
                }
                if (!ok) break;
                umma_commit_pair(&tfull_bar[a]);
            }
            if (!ok) {
                asm volatile(
                    "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                        smem_u32(&drain_bar))
                    : "memory");
                mbar_wait(&drain_bar, 0, nullptr, nullptr);
            }
        }
        __syncwarp();
    } else {
        // -------------------------------------------------------------- epilogue
        const int q = warp & 3;
        const int g = (warp - 2) >> 2;
        const int row = q * 32 + lane;
        TmaSink sink{p, &tmOut, smem + CF::OFF_STAGING + g * CF::GROUP_STAGING, row, 0, g,
                     ((warp - 2) & 3) == 0 && lane == 0};
        int lt = 0;
        for (int tile = pair; tile < num_tiles; tile += n_pairs, ++lt) {
            const int a = lt & 1;
            const uint32_t aph = (lt >> 1) & 1;
            if (!mbar_wait(&tfull_bar[a], aph, p.err, &abort_sh)) break;
            tc_fence_after();
            const int mb = tile / n_blocks, nb = tile % n_blocks;
            const int grow = mb * 2 * BM + rank * BM + row;
            const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + a * BN;
            sink.y0 = mb * 2 * BM + rank * BM;
            epilogue_tile<BN, EPI>(p, tbase, grow, grow < p.M, nb, g, sink);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) arrive_leader(&tempty_bar[a]);
        }
        sink.finish();
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();  // no CTA leaves while its peer may still touch its barriers or smem
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                     "r"(TMEM_COLS)
                     : "memory");
    }
}

template <int EPI>
int launch2(const CUtensorMap *a, const CUtensorMap *b_half, const CUtensorMap *out,
            const GemmParams &p, int num_sms, cudaStream_t stream) {
    auto kern = gemm2_kernel<EPI>;
    cudaError_t e = set_smem_once<gemm2_kernel<EPI>>(Cfg2<EPI>::SMEM);
    if (e != cudaSuccess) return e;
    const int tiles = ((p.M + 2 * BM - 1) / (2 * BM)) * (p.N / BN);
    int grid = 2 * tiles;
    const int cap = num_sms & ~1;
    if (grid > cap) grid = cap;
    return launch_k(kern, dim3(grid), dim3(kThreads), Cfg2<EPI>::SMEM, stream, *a, *b_half, *out,
                    p);
}

}  // namespace

int gemm2_launch(const CUtensorMap *a, const CUtensorMap *b_half, const CUtensorMap *out,
                 const GemmParams &p, int num_sms, cudaStream_t stream) {
    if (p.out_mode == kOutSplit) return cudaErrorInvalidValue;
    if (p.M <= 0 || p.K % BK != 0 || p.N % BN != 0) return cudaErrorInvalidValue;
    if (p.epi == kEpiQKRope && (p.head_dim % 64 != 0 || BN % p.head_dim != 0))
        return cudaErrorInvalidValue;
    switch (p.epi) {
    case kEpiStore: return launch2<kEpiStore>(a, b_half, out, p, num_sms, stream);
    case kEpiGelu: return launch2<kEpiGelu>(a, b_half, out, p, num_sms, stream);
    case kEpiResid: return launch2<kEpiResid>(a, b_half, out, p, num_sms, stream);
    case kEpiSwiGLU: return launch2<kEpiSwiGLU>(a, b_half, out, p, num_sms, stream);
    case kEpiQKRope: return launch2<kEpiQKRope>(a, b_half, out, p, num_sms, stream);
    }
    return cudaErrorInvalidValue;
}

}  // namespace fb
