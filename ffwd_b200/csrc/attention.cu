// Varlen attention kernels (see attention.cuh).
//
// Tensor-core kernel: persistent, one CTA per SM.  A work item is a pair of
// query blocks (128 query rows each) that read the same keys and values: the
// two query heads of one key/value head (grouped-query models), or two
// adjacent query tiles of one head.  Each K/V tile is loaded once and used by
// both blocks, which halves the K/V traffic.  CTAs claim items in list order
// from a global counter; the list keeps the items of one (sequence, key/value
// head) together, so CTAs that run at the same time share K/V in L2.
// 320 threads:
//   warps 0-3   softmax of block 0, warps 4-7 block 1: one thread per query
//               row reads its 128 scores from TMEM, masks (length, causal),
//               writes P = exp2(s - m) as packed bf16 over the first half of
//               the same score columns and keeps the row sum.  O accumulates in
//               TMEM and is rescaled in place only when the running row max
//               grows by more than 2^8 (decided per warp: tcgen05.ld/st are
//               warp-collective).  At the end of an item it writes O / l.
//   warp 8      producer: claims items, publishes them to the other roles,
//               loads both Q tiles (double-buffered by item) and then
//               K_0 V_0 K_1 V_1 ... into a shared-memory ring.
//   warp 9      allocates TMEM (S0 | S1 | O0 | O1); one lane issues tcgen05.mma
//               in the order PV0(j) S0(j+1) PV1(j) S1(j+1): the tensor pipe works
//               on one block while the other block's softmax runs.  S_b(j+1)
//               overwrites the columns PV_b(j) reads P from; one thread's MMAs
//               execute in issue order, so that is safe.  After an item's last
//               tile the next item's first S follows directly.
// Masking follows the packed layout: key k of sequence b is visible to query q
// iff k < len(b) and (bidirectional or k <= q).
#include "attention.cuh"
#include "launch_util.cuh"
#include "ptx.cuh"

#include <algorithm>
#include <vector>

namespace fb {
namespace {

constexpr int kTile = 128;  // query rows per block and keys per key tile
constexpr int kAttnThreads = 320;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kItemSlots = 4;  // published-item ring
constexpr float kRescaleLog2 = 8.0f;  // lazy O rescale threshold (factor 256)
constexpr int kSmemCap = 232448 - 2048;  // dynamic shared memory budget (static part reserved)

template <int D>
struct AttnCfg {
    static constexpr int BOXC = D < 64 ? D : 64;                     // columns per TMA box
    static constexpr int NBOX = D / BOXC;                            // boxes per tile
    static constexpr int ROWB = BOXC * 2;                            // bytes per smem row
    static constexpr uint32_t LAYOUT = D == 32 ? kLayoutSW64 : kLayoutSW128;
    static constexpr int SBO = 8 * ROWB;                             // 8-row atom
    static constexpr int BOX_BYTES = kTile * ROWB;                   // 128-row box
    static constexpr int TILE_BYTES = NBOX * BOX_BYTES;              // Q, K or V tile
    static constexpr int OFF_Q = 0;  // Q[item parity][block]
    static constexpr int OFF_RING = 4 * TILE_BYTES;
    static constexpr int RING0 = (kSmemCap - 1024 - OFF_RING) / TILE_BYTES;
    static constexpr int RING = RING0 > 8 ? 8 : RING0;               // K/V ring slots
    static constexpr int SMEM = OFF_RING + RING * TILE_BYTES + 1024;
    static constexpr int TMEM_COLS = 512;  // S0 [0,128) S1 [128,256) O0 [256,384) O1 [384,512)
    static constexpr int CW = D < 32 ? D : 32;
    static_assert(RING >= 3, "K/V ring too small");
};

__device__ __forceinline__ float max3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

// Item geometry, recomputed by every role from the shared work list.  Rows
// and key tiles count from seq0; L rows (a window: all its sequences' rows).
struct ItemGeo {
    int seq0, L, kvh, n_kt;
    int qt0, h0, qt1, h1;
    int seq, nseq;  // first sequence; window size (0: not a window)
    bool store1;    // block 1 is a real block (else it repeats block 0, unstored)
};

__device__ __forceinline__ ItemGeo item_geo(const AttnParams &p, int idx) {
    const AttnItem it = p.items[idx];
    ItemGeo g;
    g.seq0 = p.offsets[it.seq];
    g.L = p.offsets[it.seq + (it.nseq > 0 ? it.nseq : 1)] - g.seq0;
    g.seq = it.seq;
    g.nseq = it.nseq;
    g.store1 = it.qt1 >= 0;
    g.qt0 = it.qt0;
    g.h0 = it.h0;
    g.qt1 = g.store1 ? it.qt1 : it.qt0;
    g.h1 = g.store1 ? it.h1 : it.h0;
    g.kvh = it.h0 / (p.n_heads / p.n_kv_heads);
    const int qmax = max(g.qt0, g.qt1);
    const int kend = p.causal ? min(qmax * kTile + kTile, g.L) : g.L;
    g.n_kt = (kend + kTile - 1) / kTile;
    return g;
}

template <int D, bool F16>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tm, const AttnParams p) {
    using C = AttnCfg<D>;
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t item_full[kItemSlots];
    __shared__ __align__(8) uint64_t q_full[2], q_empty[2];
    __shared__ __align__(8) uint64_t ring_full[C::RING], ring_empty[C::RING];
    __shared__ __align__(8) uint64_t s_full[2], s_free[2];
    __shared__ __align__(8) uint64_t o_full[2], o_free[2];
    __shared__ __align__(8) uint64_t drain;
    __shared__ int item_sh[kItemSlots];
    __shared__ ItemGeo geo_sh[kItemSlots];
    __shared__ uint32_t tmem_base_sh;
    __shared__ int abort_sh;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));

    if (threadIdx.x == 0) {
        for (int i = 0; i < kItemSlots; ++i) mbar_init(&item_full[i], 1);
        for (int b = 0; b < 2; ++b) {
            mbar_init(&q_full[b], 1);
            mbar_init(&q_empty[b], 1);
            mbar_init(&s_full[b], 1);
            mbar_init(&s_free[b], 4);
            mbar_init(&o_full[b], 1);
            mbar_init(&o_free[b], 4);
        }
        for (int i = 0; i < C::RING; ++i) {
            mbar_init(&ring_full[i], 1);
            mbar_init(&ring_empty[i], 1);
        }
        mbar_init(&drain, 1);
        abort_sh = 0;
        fence_barrier_init();
    }
    if (warp == kProducerWarp && lane == 0) tma_prefetch_desc(&tm);
    if (warp == kMmaWarp) {
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

    uint8_t *sQ = smem + C::OFF_Q;
    uint8_t *sRing = smem + C::OFF_RING;

    if (warp == kProducerWarp) {
        if (lane == 0) {
            // ------------------------------------------------------------ producer
            int e = 0;  // ring entry counter: K(g) is entry 2g, V(g) entry 2g + 1
            int k = 0;  // CTA-local item counter
            int q_issued = 0;
            bool ok = true;
            // Item k + 1 is claimed when item k starts and published (index and
            // geometry in shared memory) once item k's Q load is issued, so the
            // claim's atomic and the work-list reads stay off the path of the
            // roles that wait for the next item.
            auto claim = [&](int kk) -> int {
                const int idx = kk == 0 ? (int)blockIdx.x : (int)gridDim.x + atomicAdd(p.sched, 1);
                return idx < p.n_items ? idx : -1;
            };
            auto publish = [&](int kk, int idx) {
                item_sh[kk % kItemSlots] = idx;
                if (idx >= 0) geo_sh[kk % kItemSlots] = item_geo(p, idx);
                mbar_arrive(&item_full[kk % kItemSlots]);
            };
            int idx = claim(0);
            publish(0, idx);
            for (;; ++k) {
                if (idx < 0) break;
                const int idx_next = claim(k + 1);
                const ItemGeo g = geo_sh[k % kItemSlots];
                const int qb = k & 1;
                if (!mbar_wait(&q_empty[qb], ((k >> 1) & 1) ^ 1, p.err, &abort_sh)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&q_full[qb], 2 * C::TILE_BYTES);
                for (int blk = 0; blk < 2; ++blk)
                    for (int bx = 0; bx < C::NBOX; ++bx)
                        tma_load_2d(sQ + (qb * 2 + blk) * C::TILE_BYTES + bx * C::BOX_BYTES, &tm,
                                    &q_full[qb], p.q_col0 + (blk ? g.h1 : g.h0) * D + bx * C::BOXC,
                                    g.seq0 + (blk ? g.qt1 : g.qt0) * kTile);
                // Entry (k + 1) % 4 was last read for item k - 3.  The Q wait for
                // item k passed, so the MMA issuer has issued item k - 2's last S,
                // which needed the P of the tile before it: every role has
                // started item k - 3.
                publish(k + 1, idx_next);
                q_issued = k + 1;
                for (int t = 0; t < 2 * g.n_kt; ++t, ++e) {
                    const int slot = e % C::RING;
                    if (!mbar_wait(&ring_empty[slot], ((e / C::RING) & 1) ^ 1, p.err,
                                   &abort_sh)) {
                        ok = false;
                        break;
                    }
                    const int col = ((t & 1) ? p.v_col0 : p.k_col0) + g.kvh * D;
                    const int row = g.seq0 + (t >> 1) * kTile;
                    mbar_arrive_expect_tx(&ring_full[slot], C::TILE_BYTES);
                    for (int bx = 0; bx < C::NBOX; ++bx)
                        tma_load_2d(sRing + slot * C::TILE_BYTES + bx * C::BOX_BYTES, &tm,
                                    &ring_full[slot], col + bx * C::BOXC, row);
                }
                if (!ok) break;
                idx = idx_next;
            }
            if (!ok) {  // let loads in flight land before the CTA exits
                for (int j = e - C::RING < 0 ? 0 : e - C::RING; j < e; ++j)
                    mbar_wait(&ring_full[j % C::RING], (j / C::RING) & 1, nullptr, nullptr);
                for (int j = q_issued - 2 < 0 ? 0 : q_issued - 2; j < q_issued; ++j)
                    mbar_wait(&q_full[j & 1], (j >> 1) & 1, nullptr, nullptr);
            }
        }
        __syncwarp();
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            // ------------------------------------------------------------ MMA issuer
            // Issuing costs this thread about as long as the tensor pipe takes
            // to execute a 128 x 128 x 16 MMA, and a satisfied barrier wait
            // several times that, so the barrier of the next step is probed
            // (non-blocking) before the current MMAs are issued and only
            // waited on when the probe failed.
            constexpr int BF = F16 ? 0 : 1;
            constexpr uint32_t IDESC_S = idesc_f16(128, kTile, BF, BF, 0, 0);
            constexpr uint32_t IDESC_O = idesc_f16(128, D, BF, BF, 0, 1);
            const uint64_t dQ = smem_desc(smem_u32(sQ), 16, C::SBO, C::LAYOUT);
            const uint64_t dRingK = smem_desc(smem_u32(sRing), 16, C::SBO, C::LAYOUT);
            const uint64_t dRingV = smem_desc(smem_u32(sRing), C::BOX_BYTES, C::SBO, C::LAYOUT);
            auto kk_off = [](int kk) -> uint64_t {  // K-major k-step offset (16-byte units)
                const int e = kk * 16;
                return (uint64_t)(((e / C::BOXC) * C::BOX_BYTES + (e % C::BOXC) * 2) >> 4);
            };
            auto probe = [](uint64_t *bar, uint32_t parity) -> bool {
                return mbar_test_wait(smem_u32(bar), parity);
            };
            bool ok = true;
            auto need = [&](bool probed, uint64_t *bar, uint32_t parity) -> bool {
                if (probed) return true;
                if (!mbar_wait(bar, parity, p.err, &abort_sh)) ok = false;
                return ok;
            };
            auto ring_bar = [&](int e) { return &ring_full[e % C::RING]; };
            auto ring_par = [](int e) -> uint32_t { return (e / C::RING) & 1; };
            // Next item: its tile count, or 0 at the end of the list (or on failure).
            auto next_item = [&](int k) -> int {
                if (!mbar_wait(&item_full[k % kItemSlots], (k / kItemSlots) & 1, p.err, &abort_sh)) {
                    ok = false;
                    return 0;
                }
                return item_sh[k % kItemSlots] < 0 ? 0 : geo_sh[k % kItemSlots].n_kt;
            };
            // S_b(g) for block b of item k (Q buffer k & 1) against K(g).
            const uint32_t dhi = (uint32_t)(dQ >> 32);
            const uint32_t qlo = (uint32_t)dQ, klo = (uint32_t)dRingK, vlo = (uint32_t)dRingV;
            auto issue_s = [&](int b, int k, int g) {
                const uint32_t dK = klo + (uint32_t)((((2 * g) % C::RING) * C::TILE_BYTES) >> 4);
                const uint32_t dQb = qlo + (uint32_t)((((k & 1) * 2 + b) * C::TILE_BYTES) >> 4);
                const uint32_t d = tmem_base + b * kTile;
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    umma_f16_lo(d, dQb + (uint32_t)kk_off(kk), dK + (uint32_t)kk_off(kk), dhi,
                                IDESC_S, kk != 0);
                umma_commit(&s_full[b]);
            };
            // O_b (+)= P_b(g) V(g); P_b sits in the first half of S_b's columns.
            auto issue_pv = [&](int b, int g, bool first) {
                const uint32_t dV =
                    vlo + (uint32_t)((((2 * g + 1) % C::RING) * C::TILE_BYTES) >> 4);
                const uint32_t tP = tmem_base + b * kTile;
                const uint32_t dO = tmem_base + 256 + b * 128;
#pragma unroll
                for (int kk = 0; kk < kTile / 16; ++kk)
                    umma_f16_ts_lo(dO, tP + kk * 8, dV + (uint32_t)((kk * 16 * C::ROWB) >> 4), dhi,
                                   IDESC_O, !first || kk != 0);
            };
            int k = 0, g = 0;  // local item, global tile counter
            int n = next_item(0);
            // First item's S0(0), S1(0).
            if (n > 0) {
                if (!mbar_wait(&q_full[0], 0, p.err, &abort_sh) || !mbar_wait(ring_bar(0), 0, p.err, &abort_sh)) {
                    ok = false;
                    n = 0;
                } else {
                    tc_fence_after();
                    issue_s(0, 0, 0);
                    issue_s(1, 0, 0);
                    umma_commit(&ring_empty[0]);
                    if (n == 1) umma_commit(&q_empty[0]);
                }
            }
            bool pv_ok = false, s0_ok = false;  // probes: V(g) loaded, P_0(g) written
            while (ok && n > 0) {
                int n_next = 0;
                for (int j = 0; j < n; ++j, ++g) {
                    // ---- PV_0(g)
                    if (!need(pv_ok, ring_bar(2 * g + 1), ring_par(2 * g + 1)) ||
                        !need(s0_ok, &s_free[0], g & 1) ||
                        (j == 0 && !need(false, &o_free[0], (k & 1) ^ 1)))
                        break;
                    tc_fence_after();
                    const bool last = j + 1 == n;
                    bool k_ok = last ? false : probe(ring_bar(2 * g + 2), ring_par(2 * g + 2));
                    issue_pv(0, g, j == 0);
                    if (last) umma_commit(&o_full[0]);
                    // ---- S_0(g + 1): next tile of this item, or tile 0 of the next item
                    bool s1_ok;
                    if (!last) {
                        if (!need(k_ok, ring_bar(2 * g + 2), ring_par(2 * g + 2))) break;
                        tc_fence_after();
                        s1_ok = probe(&s_free[1], g & 1);
                        issue_s(0, k, g + 1);
                    } else {
                        n_next = next_item(k + 1);
                        if (!ok) break;
                        if (n_next > 0) {
                            if (!need(false, &q_full[(k + 1) & 1], ((k + 1) >> 1) & 1) ||
                                !need(false, ring_bar(2 * g + 2), ring_par(2 * g + 2)))
                                break;
                            tc_fence_after();
                        }
                        s1_ok = probe(&s_free[1], g & 1);
                        if (n_next > 0) issue_s(0, k + 1, g + 1);
                    }
                    // ---- PV_1(g)
                    if (!need(s1_ok, &s_free[1], g & 1) ||
                        (j == 0 && !need(false, &o_free[1], (k & 1) ^ 1)))
                        break;
                    tc_fence_after();
                    issue_pv(1, g, j == 0);
                    if (last) umma_commit(&o_full[1]);
                    umma_commit(&ring_empty[(2 * g + 1) % C::RING]);
                    // ---- S_1(g + 1)
                    const bool more = !last || n_next > 0;
                    if (more) {
                        pv_ok = probe(ring_bar(2 * g + 3), ring_par(2 * g + 3));
                        s0_ok = probe(&s_free[0], (g + 1) & 1);
                        issue_s(1, last ? k + 1 : k, g + 1);
                        umma_commit(&ring_empty[(2 * g + 2) % C::RING]);
                        const int n_cur = last ? n_next : n;
                        const int j_next = last ? 0 : j + 1;
                        if (j_next + 1 == n_cur) umma_commit(&q_empty[(last ? k + 1 : k) & 1]);
                    }
                }
                if (!ok) break;
                ++k;
                n = n_next;
            }
            if (!ok) {
                umma_commit(&drain);
                mbar_wait(&drain, 0, nullptr, nullptr);
            }
        }
        __syncwarp();
    } else if (warp < 8) {
        // ---------------------------------------------------------------- softmax
        const int b = warp >> 2;
        const int quad = warp & 3;
        const int r = quad * 32 + lane;
        const float sl2 = p.scale * 1.4426950408889634f;
        const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
        const uint32_t tS = tmem_base + lane_off + b * kTile;
        const uint32_t tO = tmem_base + lane_off + 256 + b * 128;
        // An item's O is written out after the next item's first P: the wait for
        // the item's last PV then overlaps that tile's softmax (PV_b of the
        // next item waits for both arrivals, so O_b still holds the item here).
        bool pend = false, p_store = false;
        __nv_bfloat16 *p_orow = nullptr;
        float p_l = 0.0f;
        int p_k = 0;
        auto flush = [&]() -> bool {
            pend = false;
            if (!mbar_wait(&o_full[b], p_k & 1, p.err, &abort_sh)) return false;
            tc_fence_after();
            const float inv = p_l > 0.0f ? 1.0f / p_l : 0.0f;
            // Read O_b into packed bf16 registers and release it at once (the
            // next item's first PV may start), then write the row with 32-byte
            // stores (one full sector each).  All of the row's columns are
            // loaded before one wait.
            uint32_t pk[D / 2];
            float o[D];
#pragma unroll
            for (int c = 0; c < D / C::CW; ++c) {
                if constexpr (C::CW == 32)
                    tmem_ld32(tO + c * 32, *reinterpret_cast<float(*)[32]>(&o[c * 32]));
                else
                    tmem_ld16(tO + c * 16, *reinterpret_cast<float(*)[16]>(&o[c * 16]));
            }
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < D / 2; ++i) pk[i] = pack16x2(o[2 * i] * inv, o[2 * i + 1] * inv, F16);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&o_free[b]);
            if (p_store) {
#pragma unroll
                for (int u = 0; u < D / 16; ++u)
                    asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(
                                     p_orow + u * 16),
                                 "r"(pk[8 * u]), "r"(pk[8 * u + 1]), "r"(pk[8 * u + 2]),
                                 "r"(pk[8 * u + 3]), "r"(pk[8 * u + 4]), "r"(pk[8 * u + 5]),
                                 "r"(pk[8 * u + 6]), "r"(pk[8 * u + 7])
                                 : "memory");
            }
            return true;
        };
        int g = 0;
        bool ok = true;
        for (int k = 0; ok; ++k) {
            if (!mbar_wait(&item_full[k % kItemSlots], (k / kItemSlots) & 1, p.err, &abort_sh))
                break;
            if (item_sh[k % kItemSlots] < 0) break;
            const ItemGeo it = geo_sh[k % kItemSlots];
            const int q = (b ? it.qt1 : it.qt0) * kTile + r;
            // Keys [lo, hi) (rows from seq0) are this row's sequence: the whole
            // item, or in a window the row's own sequence (none past the window).
            int lo = 0, hi = it.L;
            if (it.nseq > 0) {
                lo = hi = 0;
                if (q < it.L) {
                    int a = it.seq, z = it.seq + it.nseq - 1;
                    while (a < z) {
                        const int mid = (a + z + 1) >> 1;
                        if (p.offsets[mid] - it.seq0 <= q)
                            a = mid;
                        else
                            z = mid - 1;
                    }
                    lo = p.offsets[a] - it.seq0;
                    hi = p.offsets[a + 1] - it.seq0;
                }
            }
            if (p.causal) hi = min(hi, q + 1);
            float m_used = -INFINITY, l = 0.0f;
            for (int j = 0; j < it.n_kt; ++j, ++g) {
                if (!mbar_wait(&s_full[b], g & 1, p.err, &abort_sh)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                float s[kTile];
                tmem_ld32(tS, *reinterpret_cast<float(*)[32]>(&s[0]));
                tmem_ld32(tS + 32, *reinterpret_cast<float(*)[32]>(&s[32]));
                tmem_ld32(tS + 64, *reinterpret_cast<float(*)[32]>(&s[64]));
                tmem_ld32(tS + 96, *reinterpret_cast<float(*)[32]>(&s[96]));
                tmem_wait_ld();
                const int k0 = j * kTile;
                const int vlo = lo - k0, vhi = hi - k0;  // visible columns of this tile
                if (vlo > 0 || vhi < kTile) {
#pragma unroll
                    for (int i = 0; i < kTile; ++i) s[i] = i >= vlo && i < vhi ? s[i] : -INFINITY;
                }
                float mx[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) mx[u] = max3(s[u], s[4 + u], s[8 + u]);
#pragma unroll
                for (int i = 12; i + 8 <= kTile; i += 8)
#pragma unroll
                    for (int u = 0; u < 4; ++u) mx[u] = max3(mx[u], s[i + u], s[i + 4 + u]);
                mx[0] = max3(mx[0], mx[1], s[kTile - 4]);
                mx[2] = max3(mx[2], mx[3], s[kTile - 3]);
                const float rmax = max3(mx[0], mx[2], fmaxf(s[kTile - 2], s[kTile - 1]));
                const float m_new = fmaxf(m_used, rmax * sl2);
                const bool rescale = j > 0 && __any_sync(0xffffffffu, m_new > m_used + kRescaleLog2);
                const float m_old = m_used;
                if (j == 0 || rescale) m_used = m_new;
                // P over the first 64 columns of the score buffer: key 2c, 2c + 1 in
                // column c.  Key pairs are scaled with one packed f32x2 FMA.  (Moving
                // a share of the exponentials to an FMA-pipe polynomial was measured
                // slower, and with no exponentials at all the kernel is no faster:
                // the MMA-issuing thread, not the softmax, sets the pace.  A packed
                // add for the row sum was measured to cost registers: it spills.)
                float2 la[2] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f)};
                // (m_used is -inf only while the row has seen no visible key: then
                // every score is -inf and 0 keeps P at 0.)
                const float mu = m_used == -INFINITY ? 0.0f : m_used;
                const float2 scale2 = make_float2(sl2, sl2), neg_m2 = make_float2(-mu, -mu);
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    uint32_t pk[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const int e0 = h * 64 + 2 * i;
                        const float2 x = fma_f32x2(make_float2(s[e0], s[e0 + 1]), scale2, neg_m2);
                        const float2 pp = make_float2(ex2_approx(x.x), ex2_approx(x.y));
                        la[i & 1].x += pp.x; la[i & 1].y += pp.y;
                        pk[i] = pack16x2(pp.x, pp.y, F16);
                    }
                    tmem_st32u(tS + h * 32, pk);
                }
                tmem_wait_st();
                if (rescale) {
                    // PV_b(g - 1) has completed: S_b(g), whose completion this
                    // thread waited for, was issued after it.  PV_b(g) waits for
                    // the s_free arrival below.
                    // A row with no visible key before this tile (a window row
                    // whose sequence starts in a later key tile) holds O = 0, l = 0.
                    const float alpha = m_old == -INFINITY ? 0.0f : ex2_approx(m_old - m_used);
#pragma unroll 1
                    for (int c = 0; c < D / C::CW; ++c) {
                        float o[32];
                        tmem_ld32(tO + c * 32, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] *= alpha;
                        tmem_st32(tO + c * 32, o);
                    }
                    tmem_wait_st();
                    l *= alpha;
                }
                l += (la[0].x + la[1].x) + (la[0].y + la[1].y);
                if (j == 0 && pend && !flush()) {
                    ok = false;
                    break;
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&s_free[b]);
            }
            if (!ok) break;
            pend = true;
            p_store = q < it.L && (b == 0 || it.store1);
            p_orow = p.out + (size_t)(it.seq0 + q) * p.ldo + (b ? it.h1 : it.h0) * D;
            p_l = l;
            p_k = k;
        }
        if (ok && pend) flush();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::TMEM_COLS);
    }
    // The last CTA to finish rewinds the claim counter for the next launch.
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(p.sched + 1, 1) == (int)gridDim.x - 1) {
            atomicExch(p.sched, 0);
            atomicExch(p.sched + 1, 0);
        }
    }
}

// ---------------------------------------------------------------- split-bf16 path

// Tensor-core attention of the exact plans.  Q, K and V arrive as bf16 hi / lo
// pairs (x = hi + lo to about 2^-16 relative, written by the QKV projection's
// epilogue), and each product runs as three bf16 MMAs with f32 accumulation:
// S = Qh Kh^T + Qh Kl^T + Ql Kh^T and O += Ph Vh + Ph Vl + Pl Vh, the split-bf16
// scheme of the exact projections.  One CTA per 128-row query block (block b
// of work item blockIdx.x / 2), 192 threads:
//   warps 0-3   softmax: one thread per query row reads its 128 scores of tile
//               j from TMEM score buffer j % 2, masks them, and writes
//               P = exp2(s - m) split into bf16 hi (the buffer's columns 0-63,
//               keys 2c, 2c + 1 in column c) and lo (columns 64-127); O is
//               rescaled in place when the row max grows by more than 2^8 (after
//               waiting for PV(j - 1)); at the end it writes O / l.
//   warp 4      producer: Q hi and lo once, then K(0), K(1), V(0), K(2), V(1),
//               K(3), ... (each as hi and lo) into a ring of shared-memory
//               slots: the order the MMAs consume them.
//   warp 5      allocates TMEM (S0 [0, 128) | S1 [128, 256) | O [256, 256 + D));
//               one lane issues S(0), S(1), then per tile PV(j) (after the
//               softmax of tile j) and S(j + 2).  S(j + 2) goes to the buffer
//               P(j) sits in and follows PV(j) in issue order, so it overwrites
//               P(j) only after PV(j) has read it; meanwhile S(j + 1) is already
//               done, so the softmax of tile j + 1 overlaps PV(j) and S(j + 2).
constexpr int kSplitThreads = 192;
constexpr int kSplitProducerWarp = 4;
constexpr int kSplitMmaWarp = 5;

template <int D>
struct SplitCfg {
    using A = AttnCfg<D>;
    static constexpr int TILE_BYTES = A::TILE_BYTES;
    static constexpr int OFF_RING = 2 * TILE_BYTES;  // Q hi, Q lo
    static constexpr int RING0 = (kSmemCap - 1024 - OFF_RING) / TILE_BYTES;
    static constexpr int RING = RING0 > 8 ? 8 : RING0;
    static constexpr int SMEM = OFF_RING + RING * TILE_BYTES + 1024;
    static_assert(RING >= 5, "K/V ring too small");
};

template <int D>
__global__ void __launch_bounds__(kSplitThreads, 1)
    attn_split_kernel(const __grid_constant__ CUtensorMap tm_hi,
                      const __grid_constant__ CUtensorMap tm_lo, const AttnParams p) {
    using A = AttnCfg<D>;
    using C = SplitCfg<D>;
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t q_full;
    __shared__ __align__(8) uint64_t ring_full[C::RING], ring_empty[C::RING];
    __shared__ __align__(8) uint64_t s_full[2], p_ready[2], o_done, o_full, drain;
    __shared__ uint32_t tmem_base_sh;
    __shared__ int abort_sh;

    const AttnItem item = p.items[blockIdx.x >> 1];
    const int b = blockIdx.x & 1;
    if (b == 1 && item.qt1 < 0) return;  // the item has one block
    const int qt = b ? item.qt1 : item.qt0;
    const int h = b ? item.h1 : item.h0;
    const int kvh = h / (p.n_heads / p.n_kv_heads);
    const int seq0 = p.offsets[item.seq];
    const int L = p.offsets[item.seq + 1] - seq0;
    const int kend = p.causal ? min(qt * kTile + kTile, L) : L;
    const int n_kt = (kend + kTile - 1) / kTile;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t *sQ = smem;
    uint8_t *sRing = smem + C::OFF_RING;

    if (threadIdx.x == 0) {
        mbar_init(&q_full, 1);
        for (int i = 0; i < C::RING; ++i) {
            mbar_init(&ring_full[i], 1);
            mbar_init(&ring_empty[i], 1);
        }
        mbar_init(&s_full[0], 1);
        mbar_init(&s_full[1], 1);
        mbar_init(&p_ready[0], 4);  // per score buffer: a fast softmax warp may run a
        mbar_init(&p_ready[1], 4);  // tile ahead of the others, so one barrier would mix tiles
        mbar_init(&o_done, 1);
        mbar_init(&o_full, 1);
        mbar_init(&drain, 1);
        abort_sh = 0;
        fence_barrier_init();
    }
    if (warp == kSplitProducerWarp && lane == 0) {
        tma_prefetch_desc(&tm_hi);
        tma_prefetch_desc(&tm_lo);
    }
    if (warp == kSplitMmaWarp) {
        tmem_alloc(&tmem_base_sh, 512);
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

    if (warp == kSplitProducerWarp) {
        if (lane == 0) {
            // ------------------------------------------------------------ producer
            bool ok = true;
            int e = 0;
            mbar_arrive_expect_tx(&q_full, 2 * C::TILE_BYTES);
            for (int part = 0; part < 2; ++part)
                for (int bx = 0; bx < A::NBOX; ++bx)
                    tma_load_2d(sQ + part * C::TILE_BYTES + bx * A::BOX_BYTES, part ? &tm_lo : &tm_hi,
                                &q_full, p.q_col0 + h * D + bx * A::BOXC, seq0 + qt * kTile);
            // One part (hi and lo entries) of K or V of key tile `tile`.
            auto load_part = [&](bool is_v, int tile) {
                for (int part = 0; ok && part < 2; ++part, ++e) {
                    const int slot = e % C::RING;
                    if (!mbar_wait(&ring_empty[slot], ((e / C::RING) & 1) ^ 1, p.err, &abort_sh)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&ring_full[slot], C::TILE_BYTES);
                    const int col = (is_v ? p.v_col0 : p.k_col0) + kvh * D;
                    for (int bx = 0; bx < A::NBOX; ++bx)
                        tma_load_2d(sRing + slot * C::TILE_BYTES + bx * A::BOX_BYTES,
                                    part ? &tm_lo : &tm_hi, &ring_full[slot], col + bx * A::BOXC,
                                    seq0 + tile * kTile);
                }
            };
            // The order the MMA issuer consumes them.
            load_part(false, 0);
            if (n_kt > 1) load_part(false, 1);
            for (int j = 0; ok && j < n_kt; ++j) {
                load_part(true, j);
                if (j + 2 < n_kt) load_part(false, j + 2);
            }
            if (!ok) {  // let loads in flight land before the CTA exits
                for (int k = e - C::RING < 0 ? 0 : e - C::RING; k < e; ++k)
                    mbar_wait(&ring_full[k % C::RING], (k / C::RING) & 1, nullptr, nullptr);
                mbar_wait(&q_full, 0, nullptr, nullptr);
            }
        }
        __syncwarp();
    } else if (warp == kSplitMmaWarp) {
        if (lane == 0) {
            // ------------------------------------------------------------ MMA issuer
            constexpr uint32_t IDESC_S = idesc_f16(128, kTile, 1, 1, 0, 0);
            constexpr uint32_t IDESC_O = idesc_f16(128, D, 1, 1, 0, 1);
            const uint64_t dQh = smem_desc(smem_u32(sQ), 16, A::SBO, A::LAYOUT);
            const uint64_t dQl = dQh + (uint64_t)(C::TILE_BYTES >> 4);
            const uint64_t dRingK = smem_desc(smem_u32(sRing), 16, A::SBO, A::LAYOUT);
            const uint64_t dRingV = smem_desc(smem_u32(sRing), A::BOX_BYTES, A::SBO, A::LAYOUT);
            auto kk_off = [](int kk) -> uint64_t {  // K-major k-step offset (16-byte units)
                const int x = kk * 16;
                return (uint64_t)(((x / A::BOXC) * A::BOX_BYTES + (x % A::BOXC) * 2) >> 4);
            };
            auto slot_off = [](int e) -> uint64_t {
                return (uint64_t)(((e % C::RING) * C::TILE_BYTES) >> 4);
            };
            const uint32_t dO = tmem_base + 256;
            int e = 0;  // next ring entry
            bool ok = mbar_wait(&q_full, 0, p.err, &abort_sh);
            auto wait_part = [&]() -> bool {
                ok = ok && mbar_wait(&ring_full[e % C::RING], (e / C::RING) & 1, p.err, &abort_sh) &&
                     mbar_wait(&ring_full[(e + 1) % C::RING], ((e + 1) / C::RING) & 1, p.err,
                               &abort_sh);
                if (ok) tc_fence_after();
                return ok;
            };
            auto issue_s = [&](int j) {  // S(j) into buffer j % 2
                if (!wait_part()) return;
                const uint32_t dS = tmem_base + (j & 1) * kTile;
                const uint64_t dKh = dRingK + slot_off(e), dKl = dRingK + slot_off(e + 1);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    umma_f16(dS, dQh + kk_off(kk), dKh + kk_off(kk), IDESC_S, kk != 0);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    umma_f16(dS, dQh + kk_off(kk), dKl + kk_off(kk), IDESC_S, 1);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    umma_f16(dS, dQl + kk_off(kk), dKh + kk_off(kk), IDESC_S, 1);
                umma_commit(&s_full[j & 1]);
                umma_commit(&ring_empty[e % C::RING]);
                umma_commit(&ring_empty[(e + 1) % C::RING]);
                e += 2;
            };
            auto issue_pv = [&](int j) {  // O += P(j) V(j), P in buffer j % 2
                ok = ok && mbar_wait(&p_ready[j & 1], (j >> 1) & 1, p.err, &abort_sh);
                if (!wait_part()) return;
                const uint32_t tP = tmem_base + (j & 1) * kTile;
                const uint64_t dVh = dRingV + slot_off(e), dVl = dRingV + slot_off(e + 1);
#pragma unroll
                for (int kk = 0; kk < kTile / 16; ++kk) {
                    const uint64_t vo = (uint64_t)((kk * 16 * A::ROWB) >> 4);
                    umma_f16_ts(dO, tP + kk * 8, dVh + vo, IDESC_O, j != 0 || kk != 0);
                    umma_f16_ts(dO, tP + kk * 8, dVl + vo, IDESC_O, 1);
                    umma_f16_ts(dO, tP + 64 + kk * 8, dVh + vo, IDESC_O, 1);
                }
                umma_commit(&o_done);
                umma_commit(&ring_empty[e % C::RING]);
                umma_commit(&ring_empty[(e + 1) % C::RING]);
                e += 2;
            };
            issue_s(0);
            if (n_kt > 1) issue_s(1);
            for (int j = 0; ok && j < n_kt; ++j) {
                issue_pv(j);
                if (j + 2 < n_kt) issue_s(j + 2);
            }
            // o_full: every MMA of the block done (the softmax threads consume
            // o_done phases only when they rescale, so the last phases of o_done
            // cannot be told apart by parity).
            umma_commit(ok ? &o_full : &drain);
            if (!ok) mbar_wait(&drain, 0, nullptr, nullptr);
        }
        __syncwarp();
    } else {
        // ---------------------------------------------------------------- softmax
        const int r = warp * 32 + lane;
        const int q = qt * kTile + r;
        const float sl2 = p.scale * 1.4426950408889634f;
        const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
        const uint32_t tO = tmem_base + lane_off + 256;
        float m_used = -INFINITY, l = 0.0f;
        bool ok = true;
        for (int j = 0; j < n_kt; ++j) {
            const uint32_t tS = tmem_base + lane_off + (j & 1) * kTile;
            if (!mbar_wait(&s_full[j & 1], (j >> 1) & 1, p.err, &abort_sh)) {
                ok = false;
                break;
            }
            tc_fence_after();
            float s[kTile];
            tmem_ld32(tS, *reinterpret_cast<float(*)[32]>(&s[0]));
            tmem_ld32(tS + 32, *reinterpret_cast<float(*)[32]>(&s[32]));
            tmem_ld32(tS + 64, *reinterpret_cast<float(*)[32]>(&s[64]));
            tmem_ld32(tS + 96, *reinterpret_cast<float(*)[32]>(&s[96]));
            tmem_wait_ld();
            const int k0 = j * kTile;
            const int vis = p.causal ? min(L - k0, q - k0 + 1) : L - k0;
            float rmax = -INFINITY;
#pragma unroll
            for (int i = 0; i < kTile; ++i) {
                s[i] = i < vis ? s[i] * sl2 : -INFINITY;
                rmax = fmaxf(rmax, s[i]);
            }
            const float m_new = fmaxf(m_used, rmax);
            const bool rescale = j > 0 && __any_sync(0xffffffffu, m_new > m_used + kRescaleLog2);
            const float m_old = m_used;
            if (j == 0 || rescale) m_used = m_new;
            float la = 0.0f, lb = 0.0f;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                uint32_t ph[32], pl[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const int k = half * 64 + 2 * i;
                    const float p0 = ex2_approx(s[k] - m_used), p1 = ex2_approx(s[k + 1] - m_used);
                    la += p0;
                    lb += p1;
                    const __nv_bfloat16 h0 = __float2bfloat16_rn(p0), h1 = __float2bfloat16_rn(p1);
                    __nv_bfloat162 hh(h0, h1);
                    ph[i] = *reinterpret_cast<uint32_t *>(&hh);
                    pl[i] = pack_bf16x2(p0 - __bfloat162float(h0), p1 - __bfloat162float(h1));
                }
                tmem_st32u(tS + half * 32, ph);
                tmem_st32u(tS + 64 + half * 32, pl);
            }
            tmem_wait_st();
            if (rescale) {
                // O holds PV(0 .. j - 2) for sure (S(j) was issued after PV(j - 2)),
                // so o_done is in phase j - 1 or j: its parity names PV(j - 1)
                // unambiguously.  PV(j) waits for p_ready.
                if (!mbar_wait(&o_done, (j - 1) & 1, p.err, &abort_sh)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const float alpha = ex2_approx(m_old - m_used);
#pragma unroll 1
                for (int c = 0; c < D / A::CW; ++c) {
                    if constexpr (A::CW == 32) {
                        float o[32];
                        tmem_ld32(tO + c * 32, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] *= alpha;
                        tmem_st32(tO + c * 32, o);
                    } else {
                        float o[16];
                        tmem_ld16(tO + c * 16, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 16; ++i) o[i] *= alpha;
                        tmem_st16(tO + c * 16, o);
                    }
                }
                tmem_wait_st();
                l *= alpha;
            }
            l += la + lb;
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_ready[j & 1]);
        }
        if (ok && mbar_wait(&o_full, 0, p.err, &abort_sh)) {
            tc_fence_after();
            const float inv = l > 0.0f ? 1.0f / l : 0.0f;
            const size_t off = (size_t)(seq0 + q) * p.ldo + h * D;
#pragma unroll 1
            for (int c = 0; c < D / A::CW; ++c) {
                float o[32];
                if constexpr (A::CW == 32) {
                    tmem_ld32(tO + c * 32, o);
                } else {
                    tmem_ld16(tO + c * 16, *reinterpret_cast<float(*)[16]>(&o[0]));
                }
                tmem_wait_ld();
                if (q < L) {
#pragma unroll
                    for (int i = 0; i < A::CW; i += 4) {
                        float v[4];
#pragma unroll
                        for (int u = 0; u < 4; ++u) v[u] = o[i + u] * inv;
                        const size_t o4 = off + c * A::CW + i;
                        if (p.out_tf32) {
                            *reinterpret_cast<float4 *>(p.out_tf32 + o4) =
                                make_float4(round_tf32(v[0]), round_tf32(v[1]), round_tf32(v[2]),
                                            round_tf32(v[3]));
                        } else {
                            __nv_bfloat16 hi[4], lo[4];
#pragma unroll
                            for (int u = 0; u < 4; ++u) {
                                hi[u] = __float2bfloat16_rn(v[u]);
                                lo[u] = __float2bfloat16_rn(v[u] - __bfloat162float(hi[u]));
                            }
                            *reinterpret_cast<uint2 *>(p.out_hi + o4) = *reinterpret_cast<uint2 *>(hi);
                            *reinterpret_cast<uint2 *>(p.out_lo + o4) = *reinterpret_cast<uint2 *>(lo);
                        }
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kSplitMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem_base, 512);
    }
}

}  // namespace

int attention_tc_launch(const CUtensorMap *qkv_map, const AttnParams &p, cudaStream_t stream) {
    if (p.n_items <= 0) return cudaSuccess;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    dim3 grid(p.n_items < sms ? p.n_items : sms);  // persistent
    cudaError_t e;
#define ATTN_TC(DD, FF)                                                                      \
    do {                                                                                     \
        e = set_smem_once<attn_tc_kernel<DD, FF>>(AttnCfg<DD>::SMEM);                        \
        if (e != cudaSuccess) return e;                                                      \
        e = launch_k(attn_tc_kernel<DD, FF>, grid, dim3(kAttnThreads), AttnCfg<DD>::SMEM, stream, \
                     *qkv_map, p);                                                           \
        if (e != cudaSuccess) return e;                                                      \
    } while (0)
    const bool f16 = p.f16 != 0;
    switch (p.head_dim) {
    case 32:
        if (f16) ATTN_TC(32, true); else ATTN_TC(32, false);
        break;
    case 64:
        if (f16) ATTN_TC(64, true); else ATTN_TC(64, false);
        break;
    case 128:
        if (f16) ATTN_TC(128, true); else ATTN_TC(128, false);
        break;
    default:
        return cudaErrorInvalidValue;
    }
#undef ATTN_TC
    return cudaGetLastError();
}

int attention_split_launch(const CUtensorMap *qkv_hi_map, const CUtensorMap *qkv_lo_map,
                           const AttnParams &p, cudaStream_t stream) {
    if (p.n_items <= 0) return cudaSuccess;
    dim3 grid(2 * p.n_items);
    cudaError_t e;
#define ATTN_SPLIT(DD)                                                                     \
    do {                                                                                   \
        e = set_smem_once<attn_split_kernel<DD>>(SplitCfg<DD>::SMEM);                      \
        if (e != cudaSuccess) return e;                                                    \
        e = launch_k(attn_split_kernel<DD>, grid, dim3(kSplitThreads), SplitCfg<DD>::SMEM,  \
                     stream, *qkv_hi_map, *qkv_lo_map, p);                                 \
        if (e != cudaSuccess) return e;                                                    \
    } while (0)
    switch (p.head_dim) {
    case 32: ATTN_SPLIT(32); break;
    case 64: ATTN_SPLIT(64); break;
    case 128: ATTN_SPLIT(128); break;
    default: return cudaErrorInvalidValue;
    }
#undef ATTN_SPLIT
    return cudaGetLastError();
}

namespace {

int ceil_div(int a, int b) { return (a + b - 1) / b; }

}  // namespace

int attention_count_items(int n_heads, int n_kv_heads, const int *h_offsets, int batch) {
    const int rep = n_heads / n_kv_heads;
    long long n = 0;
    for (int b = 0; b < batch; ++b) {
        const int L = h_offsets[b + 1] - h_offsets[b];
        if (rep >= 2) {  // head pairs of each key/value head
            n += (long long)ceil_div(L, kTile) * n_kv_heads * ceil_div(rep, 2);
        } else {  // query-tile pairs of each head
            n += (long long)ceil_div(ceil_div(L, kTile), 2) * n_heads;
        }
    }
    return n > 0x7fffffff ? -1 : (int)n;
}

int attention_build_items(int causal, int n_heads, int n_kv_heads, const int *h_offsets,
                          int batch, AttnItem *out, int cap, bool windows) {
    const int rep = n_heads / n_kv_heads;
    int n = 0;
    auto push = [&](const AttnItem &it) -> bool {
        if (n >= cap) return false;
        out[n++] = it;
        return true;
    };
    auto len = [&](int b) { return h_offsets[b + 1] - h_offsets[b]; };
    // A sequence goes into a window when it fits one query tile.
    auto short_seq = [&](int b) { return windows && len(b) > 0 && len(b) <= kTile; };
    // Sequences longest first; within a sequence the items of one key/value head
    // (or head) stay together, heaviest query tile first, so the CTAs working at
    // the same time read the same keys and values.
    std::vector<int> order(batch);
    for (int b = 0; b < batch; ++b) order[b] = b;
    std::stable_sort(order.begin(), order.end(), [&](int x, int y) {
        return h_offsets[x + 1] - h_offsets[x] > h_offsets[y + 1] - h_offsets[y];
    });
    for (int b : order) {
        if (short_seq(b)) continue;
        const int L = len(b);
        const int nq = ceil_div(L, kTile);
        if (rep >= 2) {
            for (int kvh = 0; kvh < n_kv_heads; ++kvh)
                for (int t = nq - 1; t >= 0; --t)
                    for (int h = kvh * rep; h < (kvh + 1) * rep; h += 2) {
                        const bool pair = h + 1 < (kvh + 1) * rep;
                        if (!push(AttnItem{b, t, h, pair ? t : -1, pair ? h + 1 : -1,
                                           causal ? t + 1 : nq, 0}))
                            return -1;
                    }
        } else {
            for (int h = 0; h < n_heads; ++h)
                for (int t = nq - 1; t >= 0; t -= 2) {
                    const bool pair = t >= 1;
                    if (!push(AttnItem{b, pair ? t - 1 : t, h, pair ? t : -1, pair ? h : -1,
                                       causal ? t + 1 : nq, 0}))
                        return -1;
                }
        }
    }
    // Windows: runs of neighbouring short sequences, cut at 128 rows (two heads
    // per item) or 256 rows (the window's two halves per item).
    const int cap_rows = rep >= 2 ? kTile : 2 * kTile;
    for (int b = 0; b < batch;) {
        if (!short_seq(b)) {
            ++b;
            continue;
        }
        int e = b, rows = 0;
        while (e < batch && short_seq(e) && rows + len(e) <= cap_rows) rows += len(e++);
        const int nseq = e - b;
        const int nt = ceil_div(rows, kTile);
        if (rep >= 2) {
            for (int kvh = 0; kvh < n_kv_heads; ++kvh)
                for (int h = kvh * rep; h < (kvh + 1) * rep; h += 2) {
                    const bool pair = h + 1 < (kvh + 1) * rep;
                    if (!push(AttnItem{b, 0, h, pair ? 0 : -1, pair ? h + 1 : -1, 1, nseq}))
                        return -1;
                }
        } else {
            for (int h = 0; h < n_heads; ++h)
                if (!push(AttnItem{b, 0, h, nt > 1 ? 1 : -1, nt > 1 ? h : -1, nt, nseq}))
                    return -1;
        }
        b = e;
    }
    return n;
}

}  // namespace fb
