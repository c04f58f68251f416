// Late-interaction device kernels (see late.cuh).
#include "late.cuh"
#include "ptx.cuh"

#include <cfloat>

namespace fb {
namespace {

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

constexpr int kProjThreads = 128;
constexpr int kProjRows = 8;    // kept rows per CTA (W is read once per 8 rows)
constexpr int kProjChunk = 128; // hidden columns staged per step

// Thread t owns output columns t, t + 128, ... (NK of them); the CTA's 8 rows
// are staged 128 hidden columns at a time, each already scaled by the final
// RMSNorm (x * inv_rms * w, the pooling path's formula).
template <int NK>
__global__ void __launch_bounds__(kProjThreads)
    late_project_kernel(const float *x, int H, const int *rows, int n_rows, const float *final_norm,
                        float eps, const float *wt, int dim, int normalize, float *out, int *err) {
    __shared__ float xs[kProjRows][kProjChunk];
    __shared__ float scale[kProjRows];
    __shared__ float red[kProjRows][kProjThreads / 32];
    const int r0 = blockIdx.x * kProjRows;
    const int nr = min(kProjRows, n_rows - r0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // Final-norm scale of each row (two rows per warp).
    for (int r = warp; r < kProjRows; r += kProjThreads / 32) {
        float inv = 1.0f;
        if (final_norm && r < nr) {
            const float *xr = x + (size_t)rows[r0 + r] * H;
            float ss = 0.0f;
            for (int h = lane; h < H; h += 32) ss += xr[h] * xr[h];
            inv = 1.0f / sqrtf(warp_sum_f(ss) / (float)H + eps);
        }
        if (lane == 0) scale[r] = inv;
    }

    float acc[kProjRows][NK];
#pragma unroll
    for (int r = 0; r < kProjRows; ++r)
#pragma unroll
        for (int k = 0; k < NK; ++k) acc[r][k] = 0.0f;

    for (int h0 = 0; h0 < H; h0 += kProjChunk) {
        __syncthreads();  // scale written / previous chunk consumed
        for (int i = threadIdx.x; i < kProjRows * kProjChunk; i += kProjThreads) {
            const int r = i / kProjChunk, c = i % kProjChunk, h = h0 + c;
            float v = 0.0f;
            if (r < nr && h < H) {
                v = x[(size_t)rows[r0 + r] * H + h];
                if (final_norm) v = v * scale[r] * final_norm[h];
            }
            xs[r][c] = v;
        }
        __syncthreads();
        const int hn = min(kProjChunk, H - h0);
        for (int c = 0; c < hn; ++c) {
            const float *wrow = wt + (size_t)(h0 + c) * dim;
#pragma unroll
            for (int k = 0; k < NK; ++k) {
                const int o = threadIdx.x + k * kProjThreads;
                const float w = o < dim ? wrow[o] : 0.0f;
#pragma unroll
                for (int r = 0; r < kProjRows; ++r) acc[r][k] = fmaf(xs[r][c], w, acc[r][k]);
            }
        }
    }

    float inv[kProjRows];
#pragma unroll
    for (int r = 0; r < kProjRows; ++r) inv[r] = 1.0f;
    if (normalize) {
#pragma unroll
        for (int r = 0; r < kProjRows; ++r) {
            float ss = 0.0f;
#pragma unroll
            for (int k = 0; k < NK; ++k) ss += acc[r][k] * acc[r][k];
            ss = warp_sum_f(ss);
            if (lane == 0) red[r][warp] = ss;
        }
        __syncthreads();
#pragma unroll
        for (int r = 0; r < kProjRows; ++r) {
            float ss = 0.0f;
#pragma unroll
            for (int w = 0; w < kProjThreads / 32; ++w) ss += red[r][w];
            if (r < nr && (!(ss > 0.0f) || !isfinite(ss))) {
                if (threadIdx.x == 0) set_error(err, kErrBadNorm);
                ss = 1.0f;
            }
            inv[r] = 1.0f / sqrtf(ss);
        }
    }
#pragma unroll
    for (int r = 0; r < kProjRows; ++r) {
        if (r >= nr) break;
#pragma unroll
        for (int k = 0; k < NK; ++k) {
            const int o = threadIdx.x + k * kProjThreads;
            if (o < dim) out[(size_t)(r0 + r) * dim + o] = acc[r][k] * inv[r];
        }
    }
}

constexpr int kSimThreads = 128;
constexpr int kSimTile = 32;  // document vectors staged per step

// One CTA per document: the document's vectors pass through shared memory 32
// at a time; thread q keeps the best dot product of query vector q (read
// through L1) and the scores are summed in query order.
__global__ void __launch_bounds__(kSimThreads)
    late_maxsim_kernel(const float *qv, int nq, const float *dv, const int *doc_off, int dim,
                       float *scores) {
    extern __shared__ float sm[];
    float *best = sm;                     // [nq]
    float *tile = sm + ((nq + 3) & ~3);   // [kSimTile][dim]
    const int d = blockIdx.x;
    const int t0 = doc_off[d], t1 = doc_off[d + 1];
    for (int q = threadIdx.x; q < nq; q += kSimThreads) best[q] = -FLT_MAX;
    for (int tb = t0; tb < t1; tb += kSimTile) {
        const int nt = min(kSimTile, t1 - tb);
        __syncthreads();
        for (int i = threadIdx.x; i < nt * dim; i += kSimThreads)
            tile[i] = dv[(size_t)tb * dim + i];
        __syncthreads();
        for (int q = threadIdx.x; q < nq; q += kSimThreads) {
            const float *qr = qv + (size_t)q * dim;
            float b = best[q];
            for (int t = 0; t < nt; ++t) {
                const float *dr = tile + t * dim;
                float dot = 0.0f;
                for (int k = 0; k < dim; ++k) dot = fmaf(__ldg(qr + k), dr[k], dot);
                b = dot > b ? dot : b;
            }
            best[q] = b;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = 0.0f;
        for (int q = 0; q < nq; ++q) s += best[q];
        scores[d] = s;
    }
}

}  // namespace

int late_project_launch(const float *x, int H, const int *rows, int n_rows,
                        const float *final_norm, float eps, const float *wt, int dim,
                        int normalize, float *out, int *err, cudaStream_t s) {
    if (n_rows <= 0) return cudaSuccess;
    if (dim <= 0 || dim > kLateMaxDim) return cudaErrorInvalidValue;
    const dim3 grid((n_rows + kProjRows - 1) / kProjRows);
    const int nk = (dim + kProjThreads - 1) / kProjThreads;
#define LATE_PROJ(NK)                                                                           \
    late_project_kernel<NK><<<grid, kProjThreads, 0, s>>>(x, H, rows, n_rows, final_norm, eps, \
                                                           wt, dim, normalize, out, err)
    switch (nk) {
    case 1: LATE_PROJ(1); break;
    case 2: LATE_PROJ(2); break;
    case 3: LATE_PROJ(3); break;
    case 4: LATE_PROJ(4); break;
    case 5: LATE_PROJ(5); break;
    case 6: LATE_PROJ(6); break;
    case 7: LATE_PROJ(7); break;
    default: LATE_PROJ(8); break;
    }
#undef LATE_PROJ
    return cudaGetLastError();
}

int late_maxsim_launch(const float *q_vec, int nq, const float *doc_vec, const int *doc_off,
                       int n_docs, int dim, float *scores, cudaStream_t s) {
    if (n_docs <= 0) return cudaSuccess;
    if (nq <= 0 || dim <= 0 || dim > kLateMaxDim) return cudaErrorInvalidValue;
    const size_t smem = (size_t)(((nq + 3) & ~3) + kSimTile * dim) * sizeof(float);
    if (smem > 48 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(
            late_maxsim_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    late_maxsim_kernel<<<n_docs, kSimThreads, smem, s>>>(q_vec, nq, doc_vec, doc_off, dim, scores);
    return cudaGetLastError();
}

}  // namespace fb
