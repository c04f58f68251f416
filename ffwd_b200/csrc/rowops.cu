// Row kernels (see rowops.cuh).  Rows are processed in 8-element groups
// (one 16-byte bf16 load or two 16-byte f32 loads per lane); every pass of a
// kernel uses the same lane -> column mapping, so a thread only re-reads what
// it wrote itself.
#include "rowops.cuh"
#include "launch_util.cuh"
#include "ptx.cuh"

namespace fb {
namespace {

constexpr int kRowWarps = 8;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ void load8_f32(const float *p, float (&v)[8]) {
    const float4 a = reinterpret_cast<const float4 *>(p)[0];
    const float4 b = reinterpret_cast<const float4 *>(p)[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

__device__ __forceinline__ void store8_f32(float *p, const float (&v)[8]) {
    reinterpret_cast<float4 *>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4 *>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}

__device__ __forceinline__ void load8_bf16(const __nv_bfloat16 *p, float (&v)[8]) {
    const uint4 raw = __ldg(reinterpret_cast<const uint4 *>(p));
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        v[2 * i] = __uint_as_float(w[i] << 16);
        v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
}

__device__ __forceinline__ void load8_ro_f32(const float *p, float (&v)[8]) {
    const float4 a = __ldg(reinterpret_cast<const float4 *>(p));
    const float4 b = __ldg(reinterpret_cast<const float4 *>(p) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

__device__ __forceinline__ void store8_out(RowOut o, size_t off, const float (&v)[8]) {
    uint32_t hi[4], lo[4];
    if (o.tf32) {
        float4 *d = reinterpret_cast<float4 *>(o.tf32 + off);
        d[0] = make_float4(round_tf32(v[0]), round_tf32(v[1]), round_tf32(v[2]), round_tf32(v[3]));
        d[1] = make_float4(round_tf32(v[4]), round_tf32(v[5]), round_tf32(v[6]), round_tf32(v[7]));
        return;
    }
    if (o.f16) {
#pragma unroll
        for (int i = 0; i < 4; ++i) hi[i] = pack_f16x2(v[2 * i], v[2 * i + 1]);
        *reinterpret_cast<uint4 *>(o.hi + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        return;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __nv_bfloat16 h0 = __float2bfloat16_rn(v[2 * i]);
        const __nv_bfloat16 h1 = __float2bfloat16_rn(v[2 * i + 1]);
        __nv_bfloat162 hh(h0, h1);
        hi[i] = *reinterpret_cast<uint32_t *>(&hh);
        lo[i] = pack_bf16x2(v[2 * i] - __bfloat162float(h0), v[2 * i + 1] - __bfloat162float(h1));
    }
    *reinterpret_cast<uint4 *>(o.hi + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    if (o.lo) *reinterpret_cast<uint4 *>(o.lo + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
}

// Kernels below keep a whole row in registers when H <= NC * 256 (NC = 1..4:
// every hidden size of the BERT family and the 0.6B decoder): lane l holds the
// 8-element groups at columns l * 8 + k * 256, k < NC, so each row is read
// once and written once.  NC = 0 is the general path for wider rows, which
// re-reads the row (from L1 / L2) in each pass.  Per-lane partial sums run
// over k in increasing order in both forms, then a butterfly over the warp:
// both give the same bits.

template <int NC>
__device__ __forceinline__ bool col_ok(int c, int H) {
    return NC == 0 || c < H;
}

// ---------------------------------------------------------------- Qwen embed

template <bool BF16, int NC>
__global__ void __launch_bounds__(kRowWarps * 32)
    embed_rms_kernel(const int *ids, int T, const void *table, int vocab, int H, float *x,
                     const float *w, float eps, RowOut xn, int *err) {
    griddep_wait();  // inputs come from the stream's previous kernel
    griddep_launch();
    const int row = blockIdx.x * kRowWarps + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= T) return;
    int id = ids[row];
    const bool bad = id < 0 || id >= vocab;
    if (bad) {
        if (lane == 0) set_error(err, kErrBadTokenId);
        id = 0;
    }
    float *xr = x + (size_t)row * H;
    auto gather = [&](int c, float (&v)[8]) {
        if (BF16)
            load8_bf16(static_cast<const __nv_bfloat16 *>(table) + (size_t)id * H + c, v);
        else
            load8_ro_f32(static_cast<const float *>(table) + (size_t)id * H + c, v);
#pragma unroll
        for (int i = 0; i < 8; ++i)
            if (bad) v[i] = 0.0f;
    };
    float ss = 0.0f;
    if constexpr (NC > 0) {
        float v[NC][8];
#pragma unroll
        for (int k = 0; k < NC; ++k) {
            const int c = lane * 8 + k * 256;
            if (c < H) {
                gather(c, v[k]);
#pragma unroll
                for (int i = 0; i < 8; ++i) ss += v[k][i] * v[k][i];
                store8_f32(xr + c, v[k]);
            }
        }
        if (!w) return;
        ss = warp_sum(ss);
        const float inv = 1.0f / sqrtf(ss / (float)H + eps);
#pragma unroll
        for (int k = 0; k < NC; ++k) {
            const int c = lane * 8 + k * 256;
            if (c < H) {
                float g[8];
                load8_ro_f32(w + c, g);
#pragma unroll
                for (int i = 0; i < 8; ++i) v[k][i] = v[k][i] * inv * g[i];
                store8_out(xn, (size_t)row * H + c, v[k]);
            }
        }
    } else {
        for (int c = lane * 8; c < H; c += 256) {
            float v[8];
            gather(c, v);
#pragma unroll
            for (int i = 0; i < 8; ++i) ss += v[i] * v[i];
            store8_f32(xr + c, v);
        }
        if (!w) return;
        ss = warp_sum(ss);
        const float inv = 1.0f / sqrtf(ss / (float)H + eps);
        for (int c = lane * 8; c < H; c += 256) {
            float v[8], g[8];
            load8_f32(xr + c, v);
            load8_ro_f32(w + c, g);
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = v[i] * inv * g[i];
            store8_out(xn, (size_t)row * H + c, v);
        }
    }
}

// ---------------------------------------------------------------- RMSNorm

template <int NC>
__global__ void __launch_bounds__(kRowWarps * 32)
    rmsnorm_kernel(const float *x, int T, int H, const float *w, float eps, RowOut xn) {
    griddep_wait();  // x comes from the stream's previous kernel
    griddep_launch();
    // Last rows first: the residual GEMM before this kernel wrote them last
    // (they are likely still in L2), and the GEMM after it starts with the
    // first rows, which this kernel writes last.
    const int rf = blockIdx.x * kRowWarps + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (rf >= T) return;
    const int row = T - 1 - rf;
    const float *xr = x + (size_t)row * H;
    float ss = 0.0f;
    if constexpr (NC > 0) {
        float v[NC][8];
#pragma unroll
        for (int k = 0; k < NC; ++k) {
            const int c = lane * 8 + k * 256;
            if (c < H) {
                load8_f32(xr + c, v[k]);
#pragma unroll
                for (int i = 0; i < 8; ++i) ss += v[k][i] * v[k][i];
            }
        }
        ss = warp_sum(ss);
        const float inv = 1.0f / sqrtf(ss / (float)H + eps);
#pragma unroll
        for (int k = 0; k < NC; ++k) {
            const int c = lane * 8 + k * 256;
            if (c < H) {
                float g[8];
                load8_ro_f32(w + c, g);
#pragma unroll
                for (int i = 0; i < 8; ++i) v[k][i] = v[k][i] * inv * g[i];
                store8_out(xn, (size_t)row * H + c, v[k]);
            }
        }
    } else {
        for (int c = lane * 8; c < H; c += 256) {
            float v[8];
            load8_f32(xr + c, v);
#pragma unroll
            for (int i = 0; i < 8; ++i) ss += v[i] * v[i];
        }
        ss = warp_sum(ss);
        const float inv = 1.0f / sqrtf(ss / (float)H + eps);
        for (int c = lane * 8; c < H; c += 256) {
            float v[8], g[8];
            load8_f32(xr + c, v);
            load8_ro_f32(w + c, g);
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = v[i] * inv * g[i];
            store8_out(xn, (size_t)row * H + c, v);
        }
    }
}

// ---------------------------------------------------------------- LayerNorm

// Two-pass mean / variance as in libffwd/norm.c:107-138, over a row held in
// registers (v[k] = columns lane * 8 + k * 256); writes x and the operand copy.
template <int NC>
__device__ __forceinline__ void layernorm_regs(float (&v)[NC][8], float *xr, int H, int lane,
                                               const float *g, const float *b, float eps,
                                               RowOut xb, size_t off) {
    float sum = 0.0f;
#pragma unroll
    for (int k = 0; k < NC; ++k)
        if (lane * 8 + k * 256 < H) {
#pragma unroll
            for (int i = 0; i < 8; ++i) sum += v[k][i];
        }
    const float inv_h = 1.0f / (float)H;
    const float mean = warp_sum(sum) * inv_h;
    float var = 0.0f;
#pragma unroll
    for (int k = 0; k < NC; ++k)
        if (lane * 8 + k * 256 < H) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float d = v[k][i] - mean;
                var += d * d;
            }
        }
    var = warp_sum(var) * inv_h;
    const float inv_std = 1.0f / sqrtf(var + eps);
#pragma unroll
    for (int k = 0; k < NC; ++k) {
        const int c = lane * 8 + k * 256;
        if (c < H) {
            float gg[8], bb[8];
            load8_ro_f32(g + c, gg);
            load8_ro_f32(b + c, bb);
#pragma unroll
            for (int i = 0; i < 8; ++i) v[k][i] = gg[i] * (v[k][i] - mean) * inv_std + bb[i];
            store8_f32(xr + c, v[k]);
            store8_out(xb, off + c, v[k]);
        }
    }
}

// The same over a row in global memory (general widths).
__device__ __forceinline__ void layernorm_row(float *xr, int H, int lane, const float *g,
                                              const float *b, float eps, RowOut xb, size_t off) {
    float sum = 0.0f;
    for (int c = lane * 8; c < H; c += 256) {
        float v[8];
        load8_f32(xr + c, v);
#pragma unroll
        for (int i = 0; i < 8; ++i) sum += v[i];
    }
    const float inv_h = 1.0f / (float)H;
    const float mean = warp_sum(sum) * inv_h;
    float var = 0.0f;
    for (int c = lane * 8; c < H; c += 256) {
        float v[8];
        load8_f32(xr + c, v);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float d = v[i] - mean;
            var += d * d;
        }
    }
    var = warp_sum(var) * inv_h;
    const float inv_std = 1.0f / sqrtf(var + eps);
    for (int c = lane * 8; c < H; c += 256) {
        float v[8], gg[8], bb[8];
        load8_f32(xr + c, v);
        load8_ro_f32(g + c, gg);
        load8_ro_f32(b + c, bb);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = gg[i] * (v[i] - mean) * inv_std + bb[i];
        store8_f32(xr + c, v);
        store8_out(xb, off + c, v);
    }
}

template <int NC>
__global__ void __launch_bounds__(kRowWarps * 32)
    layernorm_kernel(float *x, int T, int H, const float *g, const float *b, float eps, RowOut xb) {
    griddep_wait();  // x comes from the stream's previous kernel
    griddep_launch();
    // Last rows first, as in rmsnorm_kernel (L2 reuse with the GEMMs around it).
    const int rf = blockIdx.x * kRowWarps + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (rf >= T) return;
    const int row = T - 1 - rf;
    float *xr = x + (size_t)row * H;
    if constexpr (NC > 0) {
        float v[NC][8];
#pragma unroll
        for (int k = 0; k < NC; ++k) {
            const int c = lane * 8 + k * 256;
            if (c < H) load8_f32(xr + c, v[k]);
        }
        layernorm_regs<NC>(v, xr, H, lane, g, b, eps, xb, (size_t)row * H);
    } else {
        layernorm_row(xr, H, lane, g, b, eps, xb, (size_t)row * H);
    }
}

template <bool BF16, int NC>
__global__ void __launch_bounds__(kRowWarps * 32)
    embed_ln_kernel(const int *ids, const int *pos, int T, const void *table, int vocab,
                    const float *pos_table, const float *type0, const float *g, const float *b,
                    int H, float eps, float *x, RowOut xb, int *err) {
    griddep_wait();  // inputs come from the stream's previous kernel
    griddep_launch();
    const int row = blockIdx.x * kRowWarps + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= T) return;
    int id = ids[row];
    const bool bad = id < 0 || id >= vocab;
    if (bad) {
        if (lane == 0) set_error(err, kErrBadTokenId);
        id = 0;
    }
    const int ps = pos[row];
    float *xr = x + (size_t)row * H;
    // Same association as libffwd/forward.c:362-365: (tok + pos) + type.
    auto gather = [&](int c, float (&v)[8]) {
        float pv[8], tv[8];
        if (BF16)
            load8_bf16(static_cast<const __nv_bfloat16 *>(table) + (size_t)id * H + c, v);
        else
            load8_ro_f32(static_cast<const float *>(table) + (size_t)id * H + c, v);
        load8_ro_f32(pos_table + (size_t)ps * H + c, pv);
        load8_ro_f32(type0 + c, tv);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = bad ? 0.0f : (v[i] + pv[i]) + tv[i];
    };
    if constexpr (NC > 0) {
        float v[NC][8];
#pragma unroll
        for (int k = 0; k < NC; ++k) {
            const int c = lane * 8 + k * 256;
            if (c < H) gather(c, v[k]);
        }
        layernorm_regs<NC>(v, xr, H, lane, g, b, eps, xb, (size_t)row * H);
    } else {
        for (int c = lane * 8; c < H; c += 256) {
            float v[8];
            gather(c, v);
            store8_f32(xr + c, v);
        }
        layernorm_row(xr, H, lane, g, b, eps, xb, (size_t)row * H);
    }
}

// ---------------------------------------------------------------- pooling

constexpr int kPoolThreads = 256;
constexpr int kPoolMaxCols = 16;  // H <= 4096

__device__ __forceinline__ float block_sum(float v, float *red) {
    v = warp_sum(v);
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    float t = 0.0f;
#pragma unroll
    for (int i = 0; i < kPoolThreads / 32; ++i) t += red[i];
    return t;
}

// mode 0: mean over [start, end); 1: row end-1; 2: row start.
__global__ void __launch_bounds__(kPoolThreads)
    pool_kernel(const float *x, const int *starts, const int *ends, int H, int mode,
                const float *norm_w, float eps, int normalize, float *out, int *err) {
    griddep_wait();  // inputs come from the stream's previous kernel
    griddep_launch();
    __shared__ float red[kPoolThreads / 32];
    const int b = blockIdx.x;
    const int s = starts[b], e = ends[b];
    float acc[kPoolMaxCols];
#pragma unroll
    for (int k = 0; k < kPoolMaxCols; ++k) acc[k] = 0.0f;

    auto add_row = [&](int r) {
        const float *xr = x + (size_t)r * H;
        float v[kPoolMaxCols];
        float ss = 0.0f;
#pragma unroll
        for (int k = 0; k < kPoolMaxCols; ++k) {
            const int d = threadIdx.x + k * kPoolThreads;
            v[k] = d < H ? xr[d] : 0.0f;
            ss += v[k] * v[k];
        }
        float inv = 1.0f;
        if (norm_w) inv = 1.0f / sqrtf(block_sum(ss, red) / (float)H + eps);
#pragma unroll
        for (int k = 0; k < kPoolMaxCols; ++k) {
            const int d = threadIdx.x + k * kPoolThreads;
            if (d < H) acc[k] += norm_w ? v[k] * inv * norm_w[d] : v[k];
        }
    };

    if (mode == 0) {
        for (int r = s; r < e; ++r) add_row(r);
        const float inv_len = 1.0f / (float)(e - s);
#pragma unroll
        for (int k = 0; k < kPoolMaxCols; ++k) acc[k] *= inv_len;
    } else {
        add_row(mode == 1 ? e - 1 : s);
    }
    if (normalize) {
        float ss = 0.0f;
#pragma unroll
        for (int k = 0; k < kPoolMaxCols; ++k) ss += acc[k] * acc[k];
        ss = block_sum(ss, red);
        if (!(ss > 0.0f) || !isfinite(ss)) {
            if (threadIdx.x == 0) set_error(err, kErrBadNorm);
            return;
        }
        const float inv = 1.0f / sqrtf(ss);
#pragma unroll
        for (int k = 0; k < kPoolMaxCols; ++k) acc[k] *= inv;
    }
#pragma unroll
    for (int k = 0; k < kPoolMaxCols; ++k) {
        const int d = threadIdx.x + k * kPoolThreads;
        if (d < H) out[(size_t)b * H + d] = acc[k];
    }
}

// Mean pooling without a per-row norm (the BERT family): a CTA per sequence
// whose threads are (row phase, 16-byte column) pairs, so a CTA keeps many
// row loads in flight; each thread sums the rows of its phase in order, four
// at a time, then the phases are added in order.  Deterministic: the same
// batch gives the same bits.
constexpr int kMeanThreads = 1024;

__global__ void __launch_bounds__(kMeanThreads)
    pool_mean_kernel(const float *x, const int *starts, const int *ends, int H, int normalize,
                     float *out, int *err) {
    griddep_wait();  // inputs come from the stream's previous kernel
    griddep_launch();
    __shared__ float4 part[kMeanThreads];
    __shared__ float red[kMeanThreads / 32];
    __shared__ float inv_sh;
    const int b = blockIdx.x;
    const int s = starts[b], e = ends[b];
    const int cols = H / 4;
    const int phases = kMeanThreads / cols;
    const int t = threadIdx.x;
    const int ph = t / cols, c4 = t - ph * cols;
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    auto add = [](float4 &a, const float4 v) {
        a.x += v.x;
        a.y += v.y;
        a.z += v.z;
        a.w += v.w;
    };
    if (ph < phases) {
        const float4 *xp = reinterpret_cast<const float4 *>(x) + c4;
        int r = s + ph;
        for (; r + 3 * phases < e; r += 4 * phases) {
            const float4 v0 = xp[(size_t)r * cols];
            const float4 v1 = xp[(size_t)(r + phases) * cols];
            const float4 v2 = xp[(size_t)(r + 2 * phases) * cols];
            const float4 v3 = xp[(size_t)(r + 3 * phases) * cols];
            add(acc, v0);
            add(acc, v1);
            add(acc, v2);
            add(acc, v3);
        }
        for (; r < e; r += phases) add(acc, xp[(size_t)r * cols]);
    }
    part[t] = acc;
    __syncthreads();
    float4 m = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    float ss = 0.0f;
    if (t < cols) {
        for (int q = 0; q < phases; ++q) add(m, part[q * cols + t]);
        const float inv_len = 1.0f / (float)(e - s);
        m.x *= inv_len;
        m.y *= inv_len;
        m.z *= inv_len;
        m.w *= inv_len;
        ss = m.x * m.x + m.y * m.y + m.z * m.z + m.w * m.w;
    }
    if (normalize) {
        ss = warp_sum(ss);
        if ((t & 31) == 0) red[t >> 5] = ss;
        __syncthreads();
        if (t == 0) {
            float tot = 0.0f;
            for (int w = 0; w < kMeanThreads / 32; ++w) tot += red[w];
            inv_sh = (tot > 0.0f && isfinite(tot)) ? 1.0f / sqrtf(tot) : 0.0f;
            if (inv_sh == 0.0f) set_error(err, kErrBadNorm);
        }
        __syncthreads();
        if (inv_sh == 0.0f) return;
        m.x *= inv_sh;
        m.y *= inv_sh;
        m.z *= inv_sh;
        m.w *= inv_sh;
    }
    if (t < cols) reinterpret_cast<float4 *>(out + (size_t)b * H)[t] = m;
}

constexpr int kEncThreads = 128;

// One CTA per pooled row.
__global__ void __launch_bounds__(kEncThreads)
    encode_rows_kernel(const float *emb, int H, int dims, int renorm, int enc, void *out,
                       int *err) {
    __shared__ float red[kEncThreads / 32];
    __shared__ float inv_sh;
    const int b = blockIdx.x;
    const float *e = emb + (size_t)b * H;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (renorm) {
        float ss = 0.0f;
        for (int i = threadIdx.x; i < dims; i += kEncThreads) ss += e[i] * e[i];
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        if (threadIdx.x == 0) {
            float t = 0.0f;
            for (int w = 0; w < kEncThreads / 32; ++w) t += red[w];
            if (!(t > 0.0f) || !isfinite(t)) {
                set_error(err, kErrBadNorm);
                t = 1.0f;
            }
            inv_sh = 1.0f / sqrtf(t);
        }
        __syncthreads();
    }
    const float inv = renorm ? inv_sh : 1.0f;
    if (enc == 0) {
        float *o = static_cast<float *>(out) + (size_t)b * dims;
        for (int i = threadIdx.x; i < dims; i += kEncThreads) o[i] = e[i] * inv;
    } else if (enc == 1) {
        int8_t *o = static_cast<int8_t *>(out) + (size_t)b * dims;
        for (int i = threadIdx.x; i < dims; i += kEncThreads) {
            int v = __float2int_rn(tanhf(e[i] * inv) * 127.0f);
            o[i] = (int8_t)(v > 127 ? 127 : (v < -128 ? -128 : v));
        }
    } else {
        // 32 values per warp step: bit i of the ballot is value base + i, so
        // its bytes are the wire bytes in order (dims is a multiple of 8).
        uint8_t *o = static_cast<uint8_t *>(out) + (size_t)b * (dims / 8);
        for (int base = warp * 32; base < dims; base += kEncThreads) {
            const int i = base + lane;
            const unsigned m = __ballot_sync(0xffffffffu, i < dims && e[i] * inv >= 0.0f);
            const int nbytes = min(4, (dims - base) / 8);
            if (lane < nbytes) o[base / 8 + lane] = (uint8_t)(m >> (8 * lane));
        }
    }
}

inline int row_blocks(int T) { return (T + kRowWarps - 1) / kRowWarps; }

}  // namespace

// Registers per row: NC 8-element groups per lane cover H <= NC * 256; 0 for
// wider rows (the re-reading path).
inline int row_groups(int H) { return H <= 256 ? 1 : H <= 512 ? 2 : H <= 768 ? 3 : H <= 1024 ? 4 : 0; }

#define FFWD_ROW_DISPATCH(H, KERNEL_NC)       \
    switch (row_groups(H)) {                  \
    case 1: KERNEL_NC(1); break;              \
    case 2: KERNEL_NC(2); break;              \
    case 3: KERNEL_NC(3); break;              \
    case 4: KERNEL_NC(4); break;              \
    default: KERNEL_NC(0); break;             \
    }

int embed_rms_launch(const int *ids, int T, const void *table, int table_bf16, int vocab, int H,
                     float *x, const float *w, float eps, RowOut xn, int *err, cudaStream_t s) {
    if (T <= 0) return cudaSuccess;
    cudaError_t e = cudaSuccess;
#define K(NC)                                                                                \
    e = table_bf16 ? launch_k(embed_rms_kernel<true, NC>, dim3(row_blocks(T)),               \
                              dim3(kRowWarps * 32), 0, s, ids, T, table, vocab, H, x, w, eps, \
                              xn, err)                                                       \
                   : launch_k(embed_rms_kernel<false, NC>, dim3(row_blocks(T)),              \
                              dim3(kRowWarps * 32), 0, s, ids, T, table, vocab, H, x, w, eps, \
                              xn, err)
    FFWD_ROW_DISPATCH(H, K)
#undef K
    return e;
}

int embed_ln_launch(const int *ids, const int *pos, int T, const void *table, int table_bf16,
                    int vocab, const float *pos_table, const float *type0, const float *g,
                    const float *b, int H, float eps, float *x, RowOut xb, int *err,
                    cudaStream_t s) {
    if (T <= 0) return cudaSuccess;
    cudaError_t e = cudaSuccess;
#define K(NC)                                                                                \
    e = table_bf16 ? launch_k(embed_ln_kernel<true, NC>, dim3(row_blocks(T)),                \
                              dim3(kRowWarps * 32), 0, s, ids, pos, T, table, vocab,         \
                              pos_table, type0, g, b, H, eps, x, xb, err)                    \
                   : launch_k(embed_ln_kernel<false, NC>, dim3(row_blocks(T)),               \
                              dim3(kRowWarps * 32), 0, s, ids, pos, T, table, vocab,         \
                              pos_table, type0, g, b, H, eps, x, xb, err)
    FFWD_ROW_DISPATCH(H, K)
#undef K
    return e;
}

int rmsnorm_launch(const float *x, int T, int H, const float *w, float eps, RowOut xn,
                   cudaStream_t s) {
    if (T <= 0) return cudaSuccess;
    cudaError_t e = cudaSuccess;
#define K(NC) \
    e = launch_k(rmsnorm_kernel<NC>, dim3(row_blocks(T)), dim3(kRowWarps * 32), 0, s, x, T, H, w, eps, xn)
    FFWD_ROW_DISPATCH(H, K)
#undef K
    return e;
}

int layernorm_launch(float *x, int T, int H, const float *g, const float *b, float eps,
                     RowOut xb, cudaStream_t s) {
    if (T <= 0) return cudaSuccess;
    cudaError_t e = cudaSuccess;
#define K(NC) \
    e = launch_k(layernorm_kernel<NC>, dim3(row_blocks(T)), dim3(kRowWarps * 32), 0, s, x, T, H, g, b, eps, xb)
    FFWD_ROW_DISPATCH(H, K)
#undef K
    return e;
}

int pool_launch(const float *x, const int *offsets, int batch, int H, int mode,
                const float *norm_w, float eps, int normalize, float *out, int *err,
                cudaStream_t s) {
    if (batch <= 0) return cudaSuccess;
    if (H > kPoolThreads * kPoolMaxCols) return cudaErrorInvalidValue;
    if (mode == 0 && !norm_w && H % 4 == 0)
        return launch_k(pool_mean_kernel, dim3(batch), dim3(kMeanThreads), 0, s, x, offsets,
                        offsets + 1, H, normalize, out, err);
    return launch_k(pool_kernel, dim3(batch), dim3(kPoolThreads), 0, s, x, offsets, offsets + 1, H,
                    mode, norm_w, eps, normalize, out, err);
}

int encode_rows_launch(const float *emb, int B, int H, int dims, int renorm, int enc, void *out,
                       int *err, cudaStream_t s) {
    if (B <= 0) return cudaSuccess;
    if (dims <= 0 || dims > H || enc < 0 || enc > 2 || (enc == 2 && dims % 8 != 0))
        return cudaErrorInvalidValue;
    encode_rows_kernel<<<B, kEncThreads, 0, s>>>(emb, H, dims, renorm, enc, out, err);
    return cudaGetLastError();
}

int span_pool_launch(const float *x, const int *starts, const int *ends, int n_spans, int H,
                     const float *norm_w, float eps, float *out, cudaStream_t s) {
    if (n_spans <= 0) return cudaSuccess;
    if (H > kPoolThreads * kPoolMaxCols) return cudaErrorInvalidValue;
    if (!norm_w && H % 4 == 0)
        pool_mean_kernel<<<n_spans, kMeanThreads, 0, s>>>(x, starts, ends, H, 0, out, nullptr);
    else
        pool_kernel<<<n_spans, kPoolThreads, 0, s>>>(x, starts, ends, H, 0, norm_w, eps, 0, out,
                                                      nullptr);
    return cudaGetLastError();
}

}  // namespace fb
