// Varlen attention kernels (see attention.cuh).
//
// Tensor-core kernel, one CTA per work item = up to two query blocks (128
// query rows of one head each) that share one key/value head; keys in tiles of
// 64.  384 threads:
//   warps 0-3   softmax of block 0, warps 4-7 softmax of block 1: one thread per
//               query row; reads its 64 scores of a key tile from TMEM, masks
//               (length, causal), writes P = exp2(s - m) as packed bf16 back into
//               the first 32 columns of its S buffer in TMEM and keeps the row
//               sum.  O accumulates in TMEM and is rescaled in place only when the
//               running row max grows by more than 2^8 (decided per warp:
//               tcgen05.ld/st are collective).
//   warp 8      TMA producer: both Q tiles once, then K_0 V_0 K_1 V_1 ... into a
//               six-slot ring of 64-key tiles.
//   warp 9      allocates TMEM (O0 | O1 | S0a S0b S1a S1b) and one lane issues
//               tcgen05.mma.  S is double-buffered per block: S_w(j+2) is computed
//               while the softmax works on S_w(j); O += P V takes P straight from
//               TMEM (tcgen05.mma with A in TMEM), so only K and V are read from
//               shared memory.  P_w(j) aliases S buffer j % 2: the MMA issuer
//               issues PV_w(j) before S_w(j + 2) (one thread's MMAs run in issue
//               order), and the softmax writes P only after S_w(j) was read.
// Masking follows the packed layout: key k of sequence b is visible to query q
// iff k < len(b) and (bidirectional or k <= q).
#include "attention.cuh"
#include "launch_util.cuh"
#include "ptx.cuh"

#include <algorithm>

namespace fb {
namespace {

constexpr int kTile = 128;  // query rows per block (and per AttnItem tile)
constexpr int kKT = 64;     // keys per key tile
constexpr int kAttnThreads = 384;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kRingSlots = 10;
constexpr float kRescaleLog2 = 8.0f;  // lazy O rescale threshold (factor 256)

template <int D>
struct AttnCfg {
    static constexpr int BOXC = D < 64 ? D : 64;                     // columns per TMA box
    static constexpr int NBOX = D / BOXC;                            // boxes per tile
    static constexpr int ROWB = BOXC * 2;                            // bytes per smem row
    static constexpr uint32_t LAYOUT = D == 32 ? kLayoutSW64 : kLayoutSW128;
    static constexpr int SBO = 8 * ROWB;                             // 8-row atom
    static constexpr int QBOX = kTile * ROWB;                        // Q box (128 rows)
    static constexpr int Q_BYTES = NBOX * QBOX;
    static constexpr int KVBOX = kKT * ROWB;                         // K/V box (64 rows)
    static constexpr int KV_BYTES = NBOX * KVBOX;
    static constexpr int OFF_Q = 0;                                  // Q0, Q1
    static constexpr int OFF_RING = 2 * Q_BYTES;
    static constexpr int SMEM = OFF_RING + kRingSlots * KV_BYTES + 1024;
    static constexpr int TMEM_COLS = 512;  // O0 [0,D) O1 [D,2D) S[w][b] at 256 + (2w + b) 64
};

// K-major operand (Q or K tile) descriptor of k-step 0; k-step kk adds koff(kk).
template <int D>
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base) {
    using C = AttnCfg<D>;
    return smem_desc(base, 16, C::SBO, C::LAYOUT);
}

template <int D>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmkv,
                   const AttnParams p) {
    using C = AttnCfg<D>;
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t q_full;
    __shared__ __align__(8) uint64_t ring_full[kRingSlots], ring_empty[kRingSlots];
    __shared__ __align__(8) uint64_t s_full[2][2], s_free[2][2], p_full[2][2], pv_done[2][2];
    __shared__ __align__(8) uint64_t drain;
    __shared__ uint32_t tmem_base_sh;
    __shared__ int abort_sh;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));

    const AttnItem item = p.items[blockIdx.x];
    const bool two = item.qt1 >= 0;
    const int kvh = item.h0 / (p.n_heads / p.n_kv_heads);
    const int seq0 = p.offsets[item.seq];
    const int L = p.offsets[item.seq + 1] - seq0;
    const int qt_max = two ? max(item.qt0, item.qt1) : item.qt0;
    const int kend = p.causal ? min(qt_max * kTile + kTile, L) : L;
    const int n_kt = (kend + kKT - 1) / kKT;

    if (threadIdx.x == 0) {
        mbar_init(&q_full, 1);
        for (int i = 0; i < kRingSlots; ++i) {
            mbar_init(&ring_full[i], 1);
            mbar_init(&ring_empty[i], 1);
        }
        for (int w = 0; w < 2; ++w)
            for (int b = 0; b < 2; ++b) {
                mbar_init(&s_full[w][b], 1);
                mbar_init(&s_free[w][b], 4);
                mbar_init(&p_full[w][b], 4);
                mbar_init(&pv_done[w][b], 1);
            }
        mbar_init(&drain, 1);
        abort_sh = 0;
        fence_barrier_init();
    }
    if (warp == kProducerWarp && lane == 0) {
        tma_prefetch_desc(&tmq);
        tma_prefetch_desc(&tmkv);
    }
    if (warp == kMmaWarp) {
        tmem_alloc(&tmem_base_sh, C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = tmem_base_sh;

    uint8_t *sQ = smem + C::OFF_Q;
    uint8_t *sRing = smem + C::OFF_RING;

    if (warp == kProducerWarp) {
        if (lane == 0) {
            // ------------------------------------------------------------ producer
            int issued = 0;
            bool ok = true;
            mbar_arrive_expect_tx(&q_full, (two ? 2 : 1) * C::Q_BYTES);
            for (int b = 0; b < C::NBOX; ++b)
                tma_load_2d(sQ + b * C::QBOX, &tmq, &q_full, p.q_col0 + item.h0 * D + b * C::BOXC,
                            seq0 + item.qt0 * kTile);
            if (two)
                for (int b = 0; b < C::NBOX; ++b)
                    tma_load_2d(sQ + C::Q_BYTES + b * C::QBOX, &tmq, &q_full,
                                p.q_col0 + item.h1 * D + b * C::BOXC, seq0 + item.qt1 * kTile);
            for (int i = 0; i < 2 * n_kt; ++i) {
                const int slot = i % kRingSlots;
                const uint32_t ph = (i / kRingSlots) & 1;
                if (!mbar_wait(&ring_empty[slot], ph ^ 1, p.err, &abort_sh)) {
                    ok = false;
                    break;
                }
                const int col = ((i & 1) ? p.v_col0 : p.k_col0) + kvh * D;
                const int row = seq0 + (i >> 1) * kKT;
                mbar_arrive_expect_tx(&ring_full[slot], C::KV_BYTES);
                for (int b = 0; b < C::NBOX; ++b)
                    tma_load_2d(sRing + slot * C::KV_BYTES + b * C::KVBOX, &tmkv, &ring_full[slot],
                                col + b * C::BOXC, row);
                ++issued;
            }
            if (!ok) {
                mbar_wait(&q_full, 0, nullptr, nullptr);
                for (int i = issued - kRingSlots < 0 ? 0 : issued - kRingSlots; i < issued; ++i)
                    mbar_wait(&ring_full[i % kRingSlots], (i / kRingSlots) & 1, nullptr, nullptr);
            }
        }
        __syncwarp();
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            // ------------------------------------------------------------ MMA issuer
            constexpr uint32_t IDESC_S = idesc_f16(128, kKT, 1, 1, 0, 0);
            constexpr uint32_t IDESC_O = idesc_f16(128, D, 1, 1, 0, 1);
            const int nw = two ? 2 : 1;
            // Descriptors are linear in the start address (16-byte units in the
            // low bits): each operand's descriptor is built once and offset.
            const uint64_t dQ = kmajor_desc<D>(smem_u32(sQ));
            const uint64_t dRingK = kmajor_desc<D>(smem_u32(sRing));
            const uint64_t dRingV = smem_desc(smem_u32(sRing), C::KVBOX, C::SBO, C::LAYOUT);
            auto kk_off = [](int kk) -> uint64_t {  // K-major k-step offset (16-byte units)
                const int e = kk * 16;
                return (uint64_t)(((e / C::BOXC) * C::QBOX + (e % C::BOXC) * 2) >> 4);
            };
            auto kk_offk = [](int kk) -> uint64_t {
                const int e = kk * 16;
                return (uint64_t)(((e / C::BOXC) * C::KVBOX + (e % C::BOXC) * 2) >> 4);
            };
            auto wait_slot = [&](int i) -> bool {
                return mbar_wait(&ring_full[i % kRingSlots], (i / kRingSlots) & 1, p.err, &abort_sh);
            };
            auto issue_s = [&](int w, int j) {
                const uint64_t dK = dRingK + (uint64_t)((((2 * j) % kRingSlots) * C::KV_BYTES) >> 4);
                const uint64_t dQw = dQ + (uint64_t)((w * C::Q_BYTES) >> 4);
                const uint32_t d = tmem_base + 256 + (2 * w + (j & 1)) * kKT;
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    umma_f16(d, dQw + kk_off(kk), dK + kk_offk(kk), IDESC_S, kk != 0);
            };
            auto issue_pv = [&](int w, int j) {
                const uint64_t dV =
                    dRingV + (uint64_t)((((2 * j + 1) % kRingSlots) * C::KV_BYTES) >> 4);
                const uint32_t tP = tmem_base + 256 + (2 * w + (j & 1)) * kKT;
                const uint32_t d = tmem_base + w * D;
#pragma unroll
                for (int kk = 0; kk < kKT / 16; ++kk)
                    umma_f16_ts(d, tP + kk * 8, dV + (uint64_t)((kk * 16 * C::ROWB) >> 4), IDESC_O,
                                (j | kk) != 0);
            };
            bool ok = mbar_wait(&q_full, 0, p.err, &abort_sh);
            // Prologue: S(0) and S(1) for both blocks.
            for (int j = 0; ok && j < 2 && j < n_kt; ++j) {
                if (!wait_slot(2 * j)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                for (int w = 0; w < nw; ++w) {
                    issue_s(w, j);
                    umma_commit(&s_full[w][j & 1]);
                }
                umma_commit(&ring_empty[(2 * j) % kRingSlots]);
            }
            for (int j = 0; ok && j < n_kt; ++j) {
                const int b = j & 1;
                const uint32_t ph = (j >> 1) & 1;
                const bool more = j + 2 < n_kt;
                if (!wait_slot(2 * j + 1)) {
                    ok = false;
                    break;
                }
                for (int w = 0; w < nw && ok; ++w) {
                    if (!mbar_wait(&p_full[w][b], ph, p.err, &abort_sh)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    issue_pv(w, j);
                    umma_commit(&pv_done[w][b]);
                    if (more) {
                        // S_w(j+2) reuses S buffer b once the softmax has read S_w(j).
                        if (!mbar_wait(&s_free[w][b], ph, p.err, &abort_sh) ||
                            (w == 0 && !wait_slot(2 * j + 4))) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        issue_s(w, j + 2);
                        umma_commit(&s_full[w][b]);
                    }
                }
                if (!ok) break;
                umma_commit(&ring_empty[(2 * j + 1) % kRingSlots]);
                if (more) umma_commit(&ring_empty[(2 * j + 4) % kRingSlots]);
            }
            if (!ok) {
                umma_commit(&drain);
                mbar_wait(&drain, 0, nullptr, nullptr);
            }
        }
        __syncwarp();
    } else if (warp < 8) {
        // ---------------------------------------------------------------- softmax
        const int w = warp >> 2;
        if (w == 0 || two) {
            const int quad = warp & 3;
            const int r = quad * 32 + lane;
            const int qt = w == 0 ? item.qt0 : item.qt1;
            const int h = w == 0 ? item.h0 : item.h1;
            const int q = qt * kTile + r;
            const float sl2 = p.scale * 1.4426950408889634f;
            const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
            const uint32_t tO = tmem_base + lane_off + w * D;
            float m_used = -INFINITY, l = 0.0f;
            bool ok = true;
            for (int j = 0; j < n_kt; ++j) {
                const int b = j & 1;
                const uint32_t ph = (j >> 1) & 1;
                if (!mbar_wait(&s_full[w][b], ph, p.err, &abort_sh)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t tS = tmem_base + lane_off + 256 + (2 * w + b) * kKT;
                float v0[32], v1[32];
                tmem_ld32(tS, v0);
                tmem_ld32(tS + 32, v1);
                tmem_wait_ld();
#define V(i) ((i) < 32 ? v0[(i)] : v1[(i) - 32])
                const int k0 = j * kKT;
                // Tiles wholly inside the sequence and below the diagonal need no mask.
                if (k0 + kKT > L || (p.causal && k0 + kKT - 1 > qt * kTile)) {
#pragma unroll
                    for (int i = 0; i < kKT; ++i) {
                        const int key = k0 + i;
                        if (!(key < L && (!p.causal || key <= q))) V(i) = -INFINITY;
                    }
                }
                float mxa[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) mxa[i] = V(i);
#pragma unroll
                for (int i = 8; i < kKT; ++i) mxa[i & 7] = fmaxf(mxa[i & 7], V(i));
                const float mx = fmaxf(fmaxf(fmaxf(mxa[0], mxa[1]), fmaxf(mxa[2], mxa[3])),
                                       fmaxf(fmaxf(mxa[4], mxa[5]), fmaxf(mxa[6], mxa[7])));
                const float m_new = fmaxf(m_used, mx * sl2);
                if (j == 0) {
                    m_used = m_new;
                } else if (__any_sync(0xffffffffu, m_new > m_used + kRescaleLog2)) {
                    // O_w may only change once PV_w(j-1) has completed; PV_w(j)
                    // waits for this block's P_w(j).
                    if (!mbar_wait(&pv_done[w][(j - 1) & 1], ((j - 1) >> 1) & 1, p.err, &abort_sh)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const float alpha = ex2_approx(m_used - m_new);
#pragma unroll 1
                    for (int c = 0; c < D / 32; ++c) {
                        float o[32];
                        tmem_ld32(tO + c * 32, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] *= alpha;
                        tmem_st32(tO + c * 32, o);
                    }
                    tmem_wait_st();
                    l *= alpha;
                    m_used = m_new;
                }
                // P_w(j) overwrites the S_w(j) columns just read (P_w(j-2) in the
                // other buffer may still be in use by PV_w(j-2)).
                uint32_t pk[32];
                float la[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const float p0 = ex2_approx(fmaf(V(2 * i), sl2, -m_used));
                    const float p1 = ex2_approx(fmaf(V(2 * i + 1), sl2, -m_used));
                    la[i & 3] += p0 + p1;
                    pk[i] = pack_bf16x2(p0, p1);
                }
#undef V
                tmem_st32u(tS, pk);
                tmem_wait_st();
                l += (la[0] + la[1]) + (la[2] + la[3]);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&s_free[w][b]);
                    mbar_arrive(&p_full[w][b]);
                }
            }
            const int jl = n_kt - 1;
            if (ok && mbar_wait(&pv_done[w][jl & 1], (jl >> 1) & 1, p.err, &abort_sh)) {
                tc_fence_after();
                const float inv = l > 0.0f ? 1.0f / l : 0.0f;
                __nv_bfloat16 *orow = p.out + (size_t)(seq0 + q) * p.ldo + h * D;
#pragma unroll 1
                for (int c = 0; c < D / 32; ++c) {
                    float o[32];
                    tmem_ld32(tO + c * 32, o);
                    tmem_wait_ld();
                    if (q < L) {
                        uint4 *op = reinterpret_cast<uint4 *>(orow + c * 32);
#pragma unroll
                        for (int u = 0; u < 4; ++u)
                            op[u] = make_uint4(pack_bf16x2(o[8 * u] * inv, o[8 * u + 1] * inv),
                                               pack_bf16x2(o[8 * u + 2] * inv, o[8 * u + 3] * inv),
                                               pack_bf16x2(o[8 * u + 4] * inv, o[8 * u + 5] * inv),
                                               pack_bf16x2(o[8 * u + 6] * inv, o[8 * u + 7] * inv));
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::TMEM_COLS);
    }
}

// ---------------------------------------------------------------- f32 path

constexpr int kF32Threads = 128;
constexpr int kF32Keys = 32;

// TPQ threads cooperate on one query (each owns D / TPQ dimensions).
template <int D, int TPQ>
__global__ void __launch_bounds__(kF32Threads)
    attn_f32_kernel(const AttnParams p) {
    constexpr int DS = D / TPQ;
    constexpr int QT = kF32Threads / TPQ;
    __shared__ float sk[kF32Keys][D];
    __shared__ float sv[kF32Keys][D];

    const AttnItem item = p.items[blockIdx.x];
    const int h = blockIdx.y;
    const int kvh = h / (p.n_heads / p.n_kv_heads);
    const int seq0 = p.offsets[item.seq];
    const int L = p.offsets[item.seq + 1] - seq0;
    const int qi = item.qt0 * QT + threadIdx.x / TPQ;
    const int part = threadIdx.x % TPQ;
    const bool qvalid = qi < L;
    const int kend = p.causal ? min(item.qt0 * QT + QT, L) : L;

    float qv[DS], acc[DS];
    {
        const float *qp = p.qkv_f32 + (size_t)(seq0 + (qvalid ? qi : 0)) * p.ldq + p.q_col0 + h * D +
                          part * DS;
#pragma unroll
        for (int i = 0; i < DS; ++i) {
            qv[i] = qp[i];
            acc[i] = 0.0f;
        }
    }
    float m = -INFINITY, l = 0.0f;
    for (int k0 = 0; k0 < kend; k0 += kF32Keys) {
        __syncthreads();
        for (int idx = threadIdx.x; idx < kF32Keys * D; idx += kF32Threads) {
            const int kr = idx / D, d = idx % D;
            const int key = k0 + kr;
            float kvv = 0.0f, vvv = 0.0f;
            if (key < L) {
                const float *row = p.qkv_f32 + (size_t)(seq0 + key) * p.ldq;
                kvv = row[p.k_col0 + kvh * D + d];
                vvv = row[p.v_col0 + kvh * D + d];
            }
            sk[kr][d] = kvv;
            sv[kr][d] = vvv;
        }
        __syncthreads();
        const int nk = min(kF32Keys, kend - k0);
        for (int kr = 0; kr < nk; ++kr) {
            const int key = k0 + kr;
            float dot = 0.0f;
#pragma unroll
            for (int i = 0; i < DS; ++i) dot += qv[i] * sk[kr][part * DS + i];
#pragma unroll
            for (int o = 1; o < TPQ; o <<= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
            if (p.causal && key > qi) continue;
            const float s = dot * p.scale;
            // Online update in the order of libffwd/attn.c:72-91.
            if (s > m) {
                const float corr = expf(m - s);
                l = l * corr + 1.0f;
#pragma unroll
                for (int i = 0; i < DS; ++i) acc[i] = acc[i] * corr + sv[kr][part * DS + i];
                m = s;
            } else {
                const float w = expf(s - m);
                l += w;
#pragma unroll
                for (int i = 0; i < DS; ++i) acc[i] += w * sv[kr][part * DS + i];
            }
        }
    }
    if (!qvalid) return;
    const float inv = l > 0.0f ? 1.0f / l : 0.0f;
    const size_t off = (size_t)(seq0 + qi) * p.ldo + h * D + part * DS;
#pragma unroll
    for (int i = 0; i < DS; ++i) {
        const float v = acc[i] * inv;
        __nv_bfloat16 hi = __float2bfloat16_rn(v);
        p.out_hi[off + i] = hi;
        p.out_lo[off + i] = __float2bfloat16_rn(v - __bfloat162float(hi));
    }
}

}  // namespace

int attention_tc_launch(const CUtensorMap *q_map, const CUtensorMap *kv_map, const AttnParams &p,
                        cudaStream_t stream) {
    if (p.n_items <= 0) return cudaSuccess;
    dim3 grid(p.n_items);
    cudaError_t e;
    switch (p.head_dim) {
    case 32:
        e = set_smem_once<attn_tc_kernel<32>>(AttnCfg<32>::SMEM);
        if (e != cudaSuccess) return e;
        attn_tc_kernel<32><<<grid, kAttnThreads, AttnCfg<32>::SMEM, stream>>>(*q_map, *kv_map, p);
        break;
    case 64:
        e = set_smem_once<attn_tc_kernel<64>>(AttnCfg<64>::SMEM);
        if (e != cudaSuccess) return e;
        attn_tc_kernel<64><<<grid, kAttnThreads, AttnCfg<64>::SMEM, stream>>>(*q_map, *kv_map, p);
        break;
    case 128:
        e = set_smem_once<attn_tc_kernel<128>>(AttnCfg<128>::SMEM);
        if (e != cudaSuccess) return e;
        attn_tc_kernel<128><<<grid, kAttnThreads, AttnCfg<128>::SMEM, stream>>>(*q_map, *kv_map, p);
        break;
    default:
        return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

int attention_f32_qtile(int head_dim) { return head_dim > 64 ? kF32Threads / 2 : kF32Threads; }

int attention_f32_launch(const AttnParams &p, cudaStream_t stream) {
    if (p.n_items <= 0) return cudaSuccess;
    dim3 grid(p.n_items, p.n_heads);
    switch (p.head_dim) {
    case 32: attn_f32_kernel<32, 1><<<grid, kF32Threads, 0, stream>>>(p); break;
    case 64: attn_f32_kernel<64, 1><<<grid, kF32Threads, 0, stream>>>(p); break;
    case 128: attn_f32_kernel<128, 2><<<grid, kF32Threads, 0, stream>>>(p); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

namespace {

int ceil_div(int a, int b) { return (a + b - 1) / b; }

}  // namespace

int attention_count_items(bool tc, int n_heads, int n_kv_heads, int head_dim, const int *h_offsets,
                          int batch) {
    const int rep = n_heads / n_kv_heads;
    long long n = 0;
    for (int b = 0; b < batch; ++b) {
        const int L = h_offsets[b + 1] - h_offsets[b];
        if (!tc) {
            n += ceil_div(L, attention_f32_qtile(head_dim));
        } else if (rep >= 2) {
            n += (long long)ceil_div(L, kTile) * n_kv_heads * ceil_div(rep, 2);
        } else {
            n += (long long)ceil_div(ceil_div(L, kTile), 2) * n_heads;
        }
    }
    return n > 0x7fffffff ? -1 : (int)n;
}

int attention_build_items(bool tc, int causal, int n_heads, int n_kv_heads, int head_dim,
                          const int *h_offsets, int batch, AttnItem *out, int cap) {
    const int rep = n_heads / n_kv_heads;
    int n = 0;
    auto push = [&](const AttnItem &it) -> bool {
        if (n >= cap) return false;
        out[n++] = it;
        return true;
    };
    for (int b = 0; b < batch; ++b) {
        const int L = h_offsets[b + 1] - h_offsets[b];
        if (!tc) {
            const int qt = attention_f32_qtile(head_dim);
            const int nq = ceil_div(L, qt);
            for (int t = 0; t < nq; ++t)
                if (!push(AttnItem{b, t, -1, -1, -1, causal ? t + 1 : nq})) return -1;
            continue;
        }
        const int nq = ceil_div(L, kTile);
        if (rep >= 2) {
            // Two q-heads of one kv head share every K/V tile.
            for (int t = 0; t < nq; ++t)
                for (int g = 0; g < n_kv_heads; ++g)
                    for (int pr = 0; pr < rep; pr += 2) {
                        const int h0 = g * rep + pr;
                        const bool has1 = pr + 1 < rep;
                        const int kt = causal ? t + 1 : nq;
                        if (!push(AttnItem{b, t, h0, has1 ? t : -1, has1 ? h0 + 1 : -1,
                                           kt * (has1 ? 2 : 1)}))
                            return -1;
                    }
        } else {
            // Full multi-head: two query tiles of one head share the K/V stream.
            for (int h = 0; h < n_heads; ++h)
                for (int t = 0; t < nq; t += 2) {
                    const bool has1 = t + 1 < nq;
                    const int kt = causal ? (has1 ? t + 2 : t + 1) : nq;
                    if (!push(AttnItem{b, t, h, has1 ? t + 1 : -1, has1 ? h : -1,
                                       kt * (has1 ? 2 : 1)}))
                        return -1;
                }
        }
    }
    std::sort(out, out + n, [](const AttnItem &x, const AttnItem &y) {
        if (x.cost != y.cost) return x.cost > y.cost;
        if (x.seq != y.seq) return x.seq < y.seq;
        if (x.qt0 != y.qt0) return x.qt0 < y.qt0;
        return x.h0 < y.h0;
    });
    return n;
}

}  // namespace fb
