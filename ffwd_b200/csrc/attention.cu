// Varlen attention kernels (see attention.cuh).
//
// Tensor-core kernel, one CTA per (query tile of 128 rows, head):
//   warp 0      TMA producer: Q tile once, then K_j / V_j key tiles (128 keys)
//               into a two-deep ring.
//   warp 1      allocates TMEM; one lane issues S_j = Q K_j^T (tcgen05.mma,
//               M=128 N=128, into one of two TMEM score buffers) one tile ahead
//               of the softmax, and O_j = P_j V_j (M=128, N=head_dim, V read as
//               an MN-major operand straight from its TMA tile).
//   warps 2-5   softmax, one thread per query row: reads its score row from
//               TMEM, applies the length / causal mask and the online-softmax
//               update, writes P_j as bf16 into a 128-byte-swizzled shared
//               tile for the next MMA, and folds O_j into f32 registers.
// Masking follows the packed layout: key k of sequence b is visible to query q
// iff k < len(b) and (bidirectional or k <= q).
#include "attention.cuh"
#include "ptx.cuh"

namespace fb {
namespace {

constexpr int kTile = 128;  // query rows and keys per tile
constexpr int kAttnThreads = 192;

template <int D>
struct AttnCfg {
    static constexpr int BOXC = D < 64 ? D : 64;                     // columns per TMA box
    static constexpr int NBOX = D / BOXC;                            // boxes per tile
    static constexpr int ROWB = BOXC * 2;                            // bytes per smem row
    static constexpr uint32_t LAYOUT = D == 32 ? kLayoutSW64 : kLayoutSW128;
    static constexpr int SBO = 8 * ROWB;                             // 8-row atom
    static constexpr int BOX_BYTES = kTile * ROWB;
    static constexpr int TILE_BYTES = NBOX * BOX_BYTES;              // Q, K or V tile
    static constexpr int P_BYTES = kTile * kTile * 2;                // 2 SW128 blocks
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_K = OFF_Q + TILE_BYTES;
    static constexpr int OFF_V = OFF_K + 2 * TILE_BYTES;
    static constexpr int OFF_P = OFF_V + 2 * TILE_BYTES;
    static constexpr int SMEM = OFF_P + P_BYTES + 1024;
    static constexpr int TMEM_COLS = 512;  // S0 [0,128) S1 [128,256) O [256, 256 + D)
};

// K-major operand (Q or K tile): k-step `kk` covers elements [16 kk, 16 kk + 16).
template <int D>
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int kk) {
    using C = AttnCfg<D>;
    const int e = kk * 16;
    const uint32_t addr = base + (e / C::BOXC) * C::BOX_BYTES + (e % C::BOXC) * 2;
    return smem_desc(addr, 16, C::SBO, C::LAYOUT);
}

template <int D>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tm, const AttnParams p) {
    using C = AttnCfg<D>;
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t q_full;
    __shared__ __align__(8) uint64_t k_full[2], k_empty[2], v_full[2], v_empty[2];
    __shared__ __align__(8) uint64_t s_full[2], s_free[2];
    __shared__ __align__(8) uint64_t p_full, o_full, o_free, drain;
    __shared__ uint32_t tmem_base_sh;
    __shared__ int abort_sh;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));

    const AttnItem item = p.items[blockIdx.x];
    const int h = blockIdx.y;
    const int kvh = h / (p.n_heads / p.n_kv_heads);
    const int seq0 = p.offsets[item.seq];
    const int L = p.offsets[item.seq + 1] - seq0;
    const int q0 = item.qtile * kTile;
    const int kend = p.causal ? min(q0 + kTile, L) : L;
    const int n_kt = (kend + kTile - 1) / kTile;

    if (threadIdx.x == 0) {
        mbar_init(&q_full, 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(&k_full[i], 1);
            mbar_init(&k_empty[i], 1);
            mbar_init(&v_full[i], 1);
            mbar_init(&v_empty[i], 1);
            mbar_init(&s_full[i], 1);
            mbar_init(&s_free[i], 4);
        }
        mbar_init(&p_full, 4);
        mbar_init(&o_full, 1);
        mbar_init(&o_free, 4);
        mbar_init(&drain, 1);
        abort_sh = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) tma_prefetch_desc(&tm);
    if (warp == 1) {
        tmem_alloc(&tmem_base_sh, C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = tmem_base_sh;

    uint8_t *sQ = smem + C::OFF_Q;
    uint8_t *sK = smem + C::OFF_K;
    uint8_t *sV = smem + C::OFF_V;
    uint8_t *sP = smem + C::OFF_P;

    if (warp == 0) {
        if (lane == 0) {
            int issued_k = 0, issued_v = 0;
            bool ok = true;
            mbar_arrive_expect_tx(&q_full, C::TILE_BYTES);
            for (int b = 0; b < C::NBOX; ++b)
                tma_load_2d(sQ + b * C::BOX_BYTES, &tm, &q_full, p.q_col0 + h * D + b * C::BOXC,
                            seq0 + q0);
            for (int j = 0; j < n_kt && ok; ++j) {
                const int s = j & 1;
                const uint32_t ph = (j >> 1) & 1;
                const int row = seq0 + j * kTile;
                if (!mbar_wait(&k_empty[s], ph ^ 1, p.err, &abort_sh)) { ok = false; break; }
                mbar_arrive_expect_tx(&k_full[s], C::TILE_BYTES);
                for (int b = 0; b < C::NBOX; ++b)
                    tma_load_2d(sK + s * C::TILE_BYTES + b * C::BOX_BYTES, &tm, &k_full[s],
                                p.k_col0 + kvh * D + b * C::BOXC, row);
                ++issued_k;
                if (!mbar_wait(&v_empty[s], ph ^ 1, p.err, &abort_sh)) { ok = false; break; }
                mbar_arrive_expect_tx(&v_full[s], C::TILE_BYTES);
                for (int b = 0; b < C::NBOX; ++b)
                    tma_load_2d(sV + s * C::TILE_BYTES + b * C::BOX_BYTES, &tm, &v_full[s],
                                p.v_col0 + kvh * D + b * C::BOXC, row);
                ++issued_v;
            }
            if (!ok) {
                mbar_wait(&q_full, 0, nullptr, nullptr);
                for (int j = issued_k - 2 < 0 ? 0 : issued_k - 2; j < issued_k; ++j)
                    mbar_wait(&k_full[j & 1], (j >> 1) & 1, nullptr, nullptr);
                for (int j = issued_v - 2 < 0 ? 0 : issued_v - 2; j < issued_v; ++j)
                    mbar_wait(&v_full[j & 1], (j >> 1) & 1, nullptr, nullptr);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t IDESC_S = idesc_f16(128, 128, 1, 1, 0, 0);
            constexpr uint32_t IDESC_O = idesc_f16(128, D, 1, 1, 0, 1);
            const uint32_t aQ = smem_u32(sQ);
            bool ok = mbar_wait(&q_full, 0, p.err, &abort_sh);
            auto issue_s = [&](int j) -> bool {
                const int s = j & 1;
                if (!mbar_wait(&k_full[s], (j >> 1) & 1, p.err, &abort_sh)) return false;
                if (!mbar_wait(&s_free[s], ((j >> 1) & 1) ^ 1, p.err, &abort_sh)) return false;
                tc_fence_after();
                const uint32_t aK = smem_u32(sK + s * C::TILE_BYTES);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    umma_f16(tmem_base + s * 128, kmajor_desc<D>(aQ, kk), kmajor_desc<D>(aK, kk),
                             IDESC_S, kk != 0);
                umma_commit(&s_full[s]);
                umma_commit(&k_empty[s]);
                return true;
            };
            if (ok && n_kt > 0) ok = issue_s(0);
            for (int j = 0; ok && j < n_kt; ++j) {
                if (j + 1 < n_kt && !issue_s(j + 1)) { ok = false; break; }
                const int s = j & 1;
                if (!mbar_wait(&p_full, j & 1, p.err, &abort_sh)) { ok = false; break; }
                if (!mbar_wait(&v_full[s], (j >> 1) & 1, p.err, &abort_sh)) { ok = false; break; }
                if (!mbar_wait(&o_free, (j & 1) ^ 1, p.err, &abort_sh)) { ok = false; break; }
                tc_fence_after();
                const uint32_t aP = smem_u32(sP);
                const uint32_t aV = smem_u32(sV + s * C::TILE_BYTES);
#pragma unroll
                for (int kk = 0; kk < kTile / 16; ++kk) {
                    // P: K-major over keys, two 64-key SW128 blocks.
                    const uint64_t pd = smem_desc(aP + (kk / 4) * (kTile * 128) + (kk % 4) * 32, 16,
                                                  1024, kLayoutSW128);
                    // V: MN-major (N = head_dim), 16 key rows per k-step.
                    const uint64_t vd = smem_desc(aV + kk * 16 * C::ROWB, C::BOX_BYTES, C::SBO,
                                                  C::LAYOUT);
                    umma_f16(tmem_base + 256, pd, vd, IDESC_O, kk != 0);
                }
                umma_commit(&o_full);
                umma_commit(&v_empty[s]);
            }
            if (!ok) {
                // Wait for the MMAs already issued before TMEM is released.
                umma_commit(&drain);
                mbar_wait(&drain, 0, nullptr, nullptr);
            }
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------ softmax
        const int quad = warp & 3;
        const int r = quad * 32 + lane;
        const int q = q0 + r;
        const float sl2 = p.scale * 1.4426950408889634f;
        const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
        float m = -1e30f, l = 0.0f, alpha_prev = 1.0f;
        float acc[D];
#pragma unroll
        for (int i = 0; i < D; ++i) acc[i] = 0.0f;
        bool ok = true;

        auto fold_o = [&](int j) -> bool {
            if (!mbar_wait(&o_full, j & 1, p.err, &abort_sh)) return false;
            tc_fence_after();
#pragma unroll
            for (int c = 0; c < D / 32; ++c) {
                float t[32];
                tmem_ld32(tmem_base + lane_off + 256 + c * 32, t);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i) acc[c * 32 + i] = acc[c * 32 + i] * alpha_prev + t[i];
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&o_free);
            return true;
        };

        for (int j = 0; j < n_kt; ++j) {
            const int s = j & 1;
            if (!mbar_wait(&s_full[s], (j >> 1) & 1, p.err, &abort_sh)) { ok = false; break; }
            tc_fence_after();
            const uint32_t sa = tmem_base + lane_off + s * 128;
            const int k0 = j * kTile;
            float mx = -INFINITY;
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
                float v[32];
                tmem_ld32(sa + c * 32, v);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const int key = k0 + c * 32 + i;
                    const bool vis = key < L && (!p.causal || key <= q);
                    mx = fmaxf(mx, vis ? v[i] * sl2 : -INFINITY);
                }
            }
            const float m_new = fmaxf(m, mx);
            const float alpha = exp2f(m - m_new);
            if (j > 0 && !fold_o(j - 1)) { ok = false; break; }
            float sum = 0.0f;
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
                float v[32];
                tmem_ld32(sa + c * 32, v);
                tmem_wait_ld();
                uint32_t pk[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int key = k0 + c * 32 + 2 * i;
                    const bool vis0 = key < L && (!p.causal || key <= q);
                    const bool vis1 = key + 1 < L && (!p.causal || key + 1 <= q);
                    const float p0 = vis0 ? exp2f(v[2 * i] * sl2 - m_new) : 0.0f;
                    const float p1 = vis1 ? exp2f(v[2 * i + 1] * sl2 - m_new) : 0.0f;
                    __nv_bfloat162 pb = __floats2bfloat162_rn(p0, p1);
                    // Row sum of the values the MMA will actually use.
                    const float2 pf = __bfloat1622float2(pb);
                    sum += pf.x + pf.y;
                    pk[i] = *reinterpret_cast<uint32_t *>(&pb);
                }
                // Keys [32c, 32c + 32) -> block c/2, 16-byte chunks 4(c%2) .. +3.
                uint8_t *rowp = sP + (c >> 1) * (kTile * 128) + r * 128;
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int chunk = (c & 1) * 4 + u;
                    *reinterpret_cast<uint4 *>(rowp + ((chunk ^ (r & 7)) * 16)) =
                        make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
                }
            }
            l = l * alpha + sum;
            tc_fence_before();
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&s_free[s]);
                mbar_arrive(&p_full);
            }
            alpha_prev = alpha;
            m = m_new;
        }
        if (ok && n_kt > 0) ok = fold_o(n_kt - 1);
        if (ok && q < L) {
            const float inv = l > 0.0f ? 1.0f / l : 0.0f;
            uint4 *o = reinterpret_cast<uint4 *>(p.out + (size_t)(seq0 + q) * p.ldo + h * D);
#pragma unroll
            for (int u = 0; u < D / 8; ++u)
                o[u] = make_uint4(pack_bf16x2(acc[8 * u] * inv, acc[8 * u + 1] * inv),
                                  pack_bf16x2(acc[8 * u + 2] * inv, acc[8 * u + 3] * inv),
                                  pack_bf16x2(acc[8 * u + 4] * inv, acc[8 * u + 5] * inv),
                                  pack_bf16x2(acc[8 * u + 6] * inv, acc[8 * u + 7] * inv));
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
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
    const int qi = item.qtile * QT + threadIdx.x / TPQ;
    const int part = threadIdx.x % TPQ;
    const bool qvalid = qi < L;
    const int kend = p.causal ? min(item.qtile * QT + QT, L) : L;

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

int attention_tc_launch(const CUtensorMap *qkv_map, const AttnParams &p, cudaStream_t stream) {
    if (p.n_items <= 0) return cudaSuccess;
    dim3 grid(p.n_items, p.n_heads);
    cudaError_t e;
    switch (p.head_dim) {
    case 32:
        e = cudaFuncSetAttribute(attn_tc_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 AttnCfg<32>::SMEM);
        if (e != cudaSuccess) return e;
        attn_tc_kernel<32><<<grid, kAttnThreads, AttnCfg<32>::SMEM, stream>>>(*qkv_map, p);
        break;
    case 64:
        e = cudaFuncSetAttribute(attn_tc_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 AttnCfg<64>::SMEM);
        if (e != cudaSuccess) return e;
        attn_tc_kernel<64><<<grid, kAttnThreads, AttnCfg<64>::SMEM, stream>>>(*qkv_map, p);
        break;
    case 128:
        e = cudaFuncSetAttribute(attn_tc_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 AttnCfg<128>::SMEM);
        if (e != cudaSuccess) return e;
        attn_tc_kernel<128><<<grid, kAttnThreads, AttnCfg<128>::SMEM, stream>>>(*qkv_map, p);
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

}  // namespace fb
