// Host runtime of the B200 backend: weight upload, per-device workspaces,
// the packed forward (BERT / XLM-R encoder and Qwen decoder families), the
// multi-GPU sharder and the C ABI of include/ffwd_b200.h.
//
// Reference counterparts (libffwd/cuda.cu): weight upload 249-400 and
// cuda_ctx_from_model 4212-4304; workspace growth ensure_buffers 3884-4125;
// input upload cuda_upload_packed_inputs 4433-4500; Qwen forward
// cuda_forward_batch 4975-5100; BERT forward cuda_forward_batch_bert
// 4634-4973; encode entry points 5102-5225.  The reference drives one GPU; the
// device set and the LPT sharder below have no counterpart there.
#include "ffwd_b200.h"
#include "attention.cuh"
#include "gemm.cuh"
#include "loader.h"
#include "ptx.cuh"
#include "late.cuh"
#include <sys/stat.h>
#include "rowops.cuh"

#include <algorithm>
#include <chrono>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <numeric>
#include <string>
#include <thread>
#include <vector>

namespace fb {
namespace {

// ------------------------------------------------------------------ globals

std::atomic<long long> g_launches{0};
int g_gemm_mode = 0;         // 0 f32, 1 tf32, 2 bf16, 3 16f (reference default: f32)
int g_weight_override = -1;  // -1 file dtype, 0 f32, 1 bf16, 2 f16
std::vector<int> g_devices;
bool g_devices_set = false;
int g_max_tokens = 262144;
thread_local std::string t_err;
// Host-side fault injection (ffwd_b200_test_inject): the device entry whose
// next shard fails before launch, and how many of the next workspace
// allocations fail.
std::atomic<int> g_inject_shard{-1};
std::atomic<int> g_inject_alloc{0};

void fail(const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    t_err = buf;
    fprintf(stderr, "ffwd_b200: %s\n", buf);
}

#define CK(expr)                                                                              \
    do {                                                                                      \
        cudaError_t _e = (cudaError_t)(expr);                                                 \
        if (_e != cudaSuccess) {                                                              \
            fail("%s failed: %s (%s:%d)", #expr, cudaGetErrorString(_e), __FILE__, __LINE__); \
            return -1;                                                                        \
        }                                                                                     \
    } while (0)

// Kernel launch wrappers return a cudaError_t value; count every launch.
#define LAUNCH(expr)             \
    do {                         \
        g_launches.fetch_add(1); \
        CK(expr);                \
    } while (0)

// ------------------------------------------------------------------ tensor maps

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// 2-D row-major matrix [rows, cols] of `esz`-byte elements; box = box_rows x box_cols.
int make_map_dt(CUtensorMap *m, const void *ptr, uint64_t rows, uint64_t cols, uint32_t box_rows,
                uint32_t box_cols, CUtensorMapSwizzle sw, CUtensorMapDataType dt, int esz) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) {
        fail("cuTensorMapEncodeTiled unavailable");
        return -1;
    }
    if (rows == 0) rows = 1;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * (uint64_t)esz};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, dt, 2, const_cast<void *>(ptr), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        fail("cuTensorMapEncodeTiled failed (%d) rows=%llu cols=%llu box=%ux%u", (int)r,
             (unsigned long long)rows, (unsigned long long)cols, box_rows, box_cols);
        return -1;
    }
    return 0;
}

// 2-D 16-bit row-major matrix [rows, cols]; box = box_rows x box_cols.  Also used
// for f16 operands: TMA loads copy the 2-byte elements without conversion.
int make_map(CUtensorMap *m, const void *ptr, uint64_t rows, uint64_t cols, uint32_t box_rows,
             uint32_t box_cols, CUtensorMapSwizzle sw) {
    return make_map_dt(m, ptr, rows, cols, box_rows, box_cols, sw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                       2);
}

// Destination map of the two-SM GEMM's TMA epilogue: 128 rows x 64 bytes (32
// 16-bit or 16 f32 columns), 64-byte swizzle.
int make_epi_map(CUtensorMap *m, const GemmParams &p) {
    if (p.epi == kEpiResid)
        return make_map_dt(m, p.resid, p.M, p.ldr, 128, 16, CU_TENSOR_MAP_SWIZZLE_64B,
                           CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4);
    if (p.out_mode == kOutF32)
        return make_map_dt(m, p.out, p.M, p.ldo, 128, 16, CU_TENSOR_MAP_SWIZZLE_64B,
                           CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4);
    if (p.epi == kEpiQKRope)  // whole heads: two 64-column boxes per store
        return make_map_dt(m, p.out, p.M, p.ldo, 128, 64, CU_TENSOR_MAP_SWIZZLE_128B,
                           p.out_mode == kOutF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                           2);
    return make_map_dt(m, p.out, p.M, p.ldo, 128, 32, CU_TENSOR_MAP_SWIZZLE_64B,
                       p.out_mode == kOutF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                             : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                       2);
}

// ------------------------------------------------------------------ model state

struct Mat {
    __nv_bfloat16 *hi = nullptr;
    __nv_bfloat16 *lo = nullptr;  // 3-pass mode only
    int rows = 0, cols = 0, bn = 128;
    CUtensorMap map_hi, map_lo;
    CUtensorMap map_half;  // 128-row box over hi, for the two-SM kernel (bn == 256)
};

struct LayerW {
    Mat qkv, o, up, down;  // up: fused interleaved [gate; up] (Qwen) or intermediate (BERT)
    float *b_qkv = nullptr, *b_o = nullptr, *b_up = nullptr, *b_down = nullptr;
    float *q_norm = nullptr, *k_norm = nullptr, *in_norm = nullptr, *post_norm = nullptr;
    float *ln1_g = nullptr, *ln1_b = nullptr, *ln2_g = nullptr, *ln2_b = nullptr;
    int swiglu_half = 128;
};

struct Workspace {
    int cap_t = 0, cap_b = 0, cap_items = 0, cap_spans = 0;
    int *ids = nullptr, *pos = nullptr, *offsets = nullptr, *err = nullptr;
    int *span_starts = nullptr, *span_ends = nullptr;
    AttnItem *items = nullptr;
    float *pooled = nullptr;
    float *x = nullptr;
    __nv_bfloat16 *xb = nullptr, *xb_lo = nullptr;
    void *qkv = nullptr;
    __nv_bfloat16 *att = nullptr, *att_lo = nullptr, *hmid = nullptr, *hmid_lo = nullptr;
    // pinned host staging
    int *h_ids = nullptr, *h_offsets = nullptr, *h_err = nullptr, *h_spans = nullptr;
    AttnItem *h_items = nullptr;
    float *h_out = nullptr;
};

// Per-forward state: shapes, activation tensor maps and the attention work
// list of the forward last prepared on a device (also lets single ops be
// re-issued for timing).
struct FwdState {
    int T = 0, B = 0, n_items = 0;
    CUtensorMap m_xb, m_xb_lo, m_att, m_att_lo, m_h, m_h_lo, m_qkv, m_qkv_lo;
    AttnParams ap{};
};

enum Op : int {
    kOpQKV = 0,
    kOpAttn = 1,
    kOpO = 2,
    kOpNorm1 = 3,
    kOpUp = 4,
    kOpDown = 5,
    kOpNorm2 = 6,
    kOpCount = 7,  // ops of one layer
    kOpEmbed = 7,  // positions + embedding (+ first norm), re-issued by ffwd_b200_run_op
    kOpPool = 8,   // pooling (+ final norm, L2) into ws.pooled, likewise
};

struct Device {
    int dev = 0;
    int num_sms = 148;
    cudaStream_t stream = nullptr;
    void *embed = nullptr;
    int embed_bf16 = 0;
    float *pos_table = nullptr, *type0 = nullptr, *emb_ln_g = nullptr, *emb_ln_b = nullptr;
    float *final_norm = nullptr;
    float *rope_cos = nullptr, *rope_sin = nullptr;
    __half *rope_cos_h = nullptr, *rope_sin_h = nullptr;  // f16 copies for the bf16 GEMM
    int rope_cap = 0;
    std::vector<LayerW> layers;
    Workspace ws;
    Workspace *active_ws = nullptr;  // when set, step() uses these buffers instead of ws
    FwdState fs;
    std::vector<void *> allocs;
    // Late interaction (first device of a late-interaction context).
    float *late_wt = nullptr;   // 1_Dense weight transposed: [hidden, token_dim] f32
    float *late_vec = nullptr;  // token vectors [late_cap_rows, token_dim]
    int *late_rows = nullptr, *late_doff = nullptr;
    float *late_scores = nullptr;
    int *h_late_rows = nullptr, *h_late_doff = nullptr;
    float *h_late_vec = nullptr, *h_late_scores = nullptr;
    size_t late_cap_rows = 0, late_cap_docs = 0;
    // Second set of pinned host staging buffers, so the host packs (and
    // launches) forward k + 1 of a long batch while the GPU runs forward k.
    struct Staging {
        int *ids = nullptr, *offsets = nullptr, *err = nullptr;
        AttnItem *items = nullptr;
        uint8_t *out = nullptr;
        size_t cap_ids = 0, cap_off = 0, cap_items = 0, cap_out = 0;
    } stg;
    cudaEvent_t fwd_done[2] = {nullptr, nullptr};
};

}  // namespace
}  // namespace fb

struct ffwd_b200_ctx {
    ffwd_config_t cfg;
    int prec = 0;      // 0 single pass, 2 / 3 split-bf16 passes, 4 kind::tf32
    bool f16 = false;  // single-pass operands in f16 (else bf16)
    std::vector<fb::Device> devs;
    float lin_flops_per_token = 0.0f;
    int token_dim = 0;  // late interaction: 1_Dense output width (0: pooled model)
    // Per device entry, the last encode_batch's share: sequences, tokens and
    // the host wall time of that shard's worker (packing to copied-out rows).
    struct Shard {
        int seqs = 0;
        long long tokens = 0;
        double ms = 0.0;
    };
    std::vector<Shard> last_shards;
};

// A late-interaction model: the base model context plus its 1_Dense head (on
// the base context's first device).
struct ffwd_b200_late_ctx {
    ffwd_b200_ctx *base = nullptr;
};

namespace fb {
namespace {

// ------------------------------------------------------------------ uploads

template <typename T>
int dev_alloc(Device &D, T **p, size_t count) {
    void *q = nullptr;
    CK(cudaMalloc(&q, std::max<size_t>(count, 1) * sizeof(T)));
    D.allocs.push_back(q);
    *p = static_cast<T *>(q);
    return 0;
}

template <typename T>
int upload(Device &D, T **p, const std::vector<T> &h) {
    if (dev_alloc(D, p, h.size())) return -1;
    CK(cudaMemcpy(*p, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice));
    return 0;
}

// Host copy of one (possibly fused) projection in its device encoding.
struct HostMat {
    std::vector<uint16_t> hi, lo;
    std::vector<float> f32;  // tf32 plan: f32 values rounded to tf32
    int rows = 0, cols = 0;
};

// f32 rounded to the nearest tf32 value, ties away from zero (the rounding of
// cvt.rna.tf32.f32); inf and NaN pass through.
float round_tf32_host(float v) {
    uint32_t u;
    memcpy(&u, &v, 4);
    if ((u & 0x7F800000u) != 0x7F800000u) u = (u + 0x1000u) & 0xFFFFE000u;
    memcpy(&v, &u, 4);
    return v;
}

// parts: row blocks concatenated in order (e.g. Wq, Wk, Wv).  interleave > 0
// reorders two equal parts [G; U] as G0 U0 G1 U1 ... in blocks of `interleave`
// rows, so one BN-wide GEMM tile holds matching gate and up columns.
// store: the device weight storage the values are first rounded to (0 f32,
// 1 bf16, 2 f16; libffwd/cuda.cu upload_weight 262-305).  The encoding is then
// f16 (out_f16, single-pass f16 GEMM), tf32-rounded f32 (out_tf32, kind::tf32
// GEMM), or bf16 hi (+ lo = bf16(v - hi) when split).
bool prep_mat(const std::vector<const TensorView *> &parts, const std::vector<std::string> &names,
              int cols, int store, bool split, bool out_f16, bool out_tf32, int interleave,
              HostMat &hm, std::string &err) {
    int rows = 0;
    for (size_t i = 0; i < parts.size(); ++i) {
        const TensorView *t = parts[i];
        if (!t || t->shape.size() != 2 || t->shape[1] != cols) {
            err = "missing or mis-shaped tensor " + names[i];
            return false;
        }
        rows += (int)t->shape[0];
    }
    hm.rows = rows;
    hm.cols = cols;
    if (out_tf32)
        hm.f32.resize((size_t)rows * cols);
    else
        hm.hi.resize((size_t)rows * cols);
    if (split) hm.lo.assign((size_t)rows * cols, 0);
    std::vector<int> src_part(rows), src_row(rows);
    {
        int r = 0;
        if (interleave > 0) {
            const int half = (int)parts[0]->shape[0];
            for (int blk = 0; blk < half / interleave; ++blk)
                for (int p = 0; p < 2; ++p)
                    for (int i = 0; i < interleave; ++i, ++r) {
                        src_part[r] = p;
                        src_row[r] = blk * interleave + i;
                    }
        } else {
            for (size_t p = 0; p < parts.size(); ++p)
                for (int i = 0; i < (int)parts[p]->shape[0]; ++i, ++r) {
                    src_part[r] = (int)p;
                    src_row[r] = i;
                }
        }
    }
    auto work = [&](int r0, int r1) {
        for (int r = r0; r < r1; ++r) {
            const TensorView *t = parts[src_part[r]];
            const size_t so = (size_t)src_row[r] * cols;
            uint16_t *dh = out_tf32 ? nullptr : hm.hi.data() + (size_t)r * cols;
            uint16_t *dl = split ? hm.lo.data() + (size_t)r * cols : nullptr;
            if (out_tf32) {
                for (int c = 0; c < cols; ++c) {
                    const uint16_t w = ((const uint16_t *)t->data)[so + c];
                    float v = t->dtype == DType::F32    ? ((const float *)t->data)[so + c]
                              : t->dtype == DType::BF16 ? bf16_to_f32(w)
                                                        : f16_to_f32(w);
                    if (store == 1) v = bf16_to_f32(f32_to_bf16_rne(v));
                    else if (store == 2) v = f16_to_f32(f32_to_f16_rne(v));
                    hm.f32[(size_t)r * cols + c] = round_tf32_host(v);
                }
            } else if (t->dtype == DType::BF16 && !out_f16 && store != 2) {
                memcpy(dh, (const uint16_t *)t->data + so, (size_t)cols * 2);
            } else if (t->dtype == DType::F16 && out_f16) {
                memcpy(dh, (const uint16_t *)t->data + so, (size_t)cols * 2);
            } else {
                for (int c = 0; c < cols; ++c) {
                    const uint16_t w = ((const uint16_t *)t->data)[so + c];
                    float v = t->dtype == DType::F32    ? ((const float *)t->data)[so + c]
                              : t->dtype == DType::BF16 ? bf16_to_f32(w)
                                                        : f16_to_f32(w);
                    if (store == 1) v = bf16_to_f32(f32_to_bf16_rne(v));
                    else if (store == 2) v = f16_to_f32(f32_to_f16_rne(v));
                    if (out_f16) {
                        dh[c] = f32_to_f16_rne(v);
                        continue;
                    }
                    const uint16_t h = f32_to_bf16_rne(v);
                    dh[c] = h;
                    if (dl) dl[c] = f32_to_bf16_rne(v - bf16_to_f32(h));
                }
            }
        }
    };
    const int nth = std::max(1, std::min(16, (int)std::thread::hardware_concurrency()));
    std::vector<std::thread> th;
    const int per = (rows + nth - 1) / nth;
    for (int i = 0; i < nth; ++i) {
        int a = i * per, b = std::min(rows, a + per);
        if (a < b) th.emplace_back(work, a, b);
    }
    for (auto &t : th) t.join();
    return true;
}

int upload_mat(Device &D, const HostMat &hm, int bn, Mat &m) {
    m.rows = hm.rows;
    m.cols = hm.cols;
    m.bn = bn;
    if (!hm.f32.empty()) {  // tf32 plan: f32 weights, 32-column (128-byte) boxes
        float *d = nullptr;
        if (dev_alloc(D, &d, hm.f32.size())) return -1;
        CK(cudaMemcpy(d, hm.f32.data(), hm.f32.size() * 4, cudaMemcpyHostToDevice));
        m.hi = reinterpret_cast<__nv_bfloat16 *>(d);
        return make_map_dt(&m.map_hi, d, m.rows, m.cols, bn, 32, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4);
    }
    if (dev_alloc(D, &m.hi, hm.hi.size())) return -1;
    CK(cudaMemcpy(m.hi, hm.hi.data(), hm.hi.size() * 2, cudaMemcpyHostToDevice));
    if (make_map(&m.map_hi, m.hi, m.rows, m.cols, bn, 64, CU_TENSOR_MAP_SWIZZLE_128B)) return -1;
    if (bn == 256 &&
        make_map(&m.map_half, m.hi, m.rows, m.cols, 128, 64, CU_TENSOR_MAP_SWIZZLE_128B))
        return -1;
    if (!hm.lo.empty()) {
        if (dev_alloc(D, &m.lo, hm.lo.size())) return -1;
        CK(cudaMemcpy(m.lo, hm.lo.data(), hm.lo.size() * 2, cudaMemcpyHostToDevice));
        if (make_map(&m.map_lo, m.lo, m.rows, m.cols, bn, 64, CU_TENSOR_MAP_SWIZZLE_128B)) return -1;
    }
    return 0;
}

int pick_bn(int n) { return n % 256 == 0 ? 256 : 128; }

// RoPE cos/sin cache exactly as libffwd/model_blas.c:85-123 computes it
// (f32 powf / cosf / sinf), keeping the first half (the halves are equal).
int ensure_rope(Device &D, const ffwd_config_t &c, int n_pos) {
    if (n_pos <= D.rope_cap) return 0;
    int cap = D.rope_cap > 0 ? D.rope_cap : 4096;
    while (cap < n_pos) cap *= 2;
    const int half = c.head_dim / 2;
    std::vector<float> hc((size_t)cap * half), hs((size_t)cap * half);
    for (int p = 0; p < cap; ++p) {
        const float fp = (float)p;
        for (int d = 0; d < half; ++d) {
            const float inv = 1.0f / powf(c.rope_theta, (float)(2 * d) / (float)c.head_dim);
            const float a = fp * inv;
            hc[(size_t)p * half + d] = cosf(a);
            hs[(size_t)p * half + d] = sinf(a);
        }
    }
    CK(cudaSetDevice(D.dev));
    CK(cudaStreamSynchronize(D.stream));
    std::vector<__half> hch(hc.size()), hsh(hs.size());
    for (size_t i = 0; i < hc.size(); ++i) {
        hch[i] = __float2half_rn(hc[i]);
        hsh[i] = __float2half_rn(hs[i]);
    }
    if (D.rope_cos) CK(cudaFree(D.rope_cos));
    if (D.rope_sin) CK(cudaFree(D.rope_sin));
    if (D.rope_cos_h) CK(cudaFree(D.rope_cos_h));
    if (D.rope_sin_h) CK(cudaFree(D.rope_sin_h));
    CK(cudaMalloc(&D.rope_cos, hc.size() * 4));
    CK(cudaMalloc(&D.rope_sin, hs.size() * 4));
    CK(cudaMalloc(&D.rope_cos_h, hch.size() * 2));
    CK(cudaMalloc(&D.rope_sin_h, hsh.size() * 2));
    CK(cudaMemcpy(D.rope_cos, hc.data(), hc.size() * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(D.rope_sin, hs.data(), hs.size() * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(D.rope_cos_h, hch.data(), hch.size() * 2, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(D.rope_sin_h, hsh.data(), hsh.size() * 2, cudaMemcpyHostToDevice));
    D.rope_cap = cap;
    return 0;
}

// ------------------------------------------------------------------ load

struct HostModel {
    ffwd_config_t cfg;
    int prec = 0;
    int store = 0;     // weight storage: 0 f32, 1 bf16, 2 f16
    bool f16 = false;  // single-pass operands are f16 (else bf16)
    std::string prefix;
    SafeTensors st;
};

int noalloc_scratch(int dev, uint8_t **out);

int load_device(HostModel &hm, Device &D, std::string &err) {
    const ffwd_config_t &c = hm.cfg;
    CK(cudaSetDevice(D.dev));
    CK(cudaStreamCreateWithFlags(&D.stream, cudaStreamNonBlocking));
    // Resolve the no-allocation arena now, so its module (and the arena) is
    // loaded when the model is, not on the first no-allocation request.
    uint8_t *arena = nullptr;
    if (noalloc_scratch(D.dev, &arena)) return -1;
    CK(cudaDeviceGetAttribute(&D.num_sms, cudaDevAttrMultiProcessorCount, D.dev));
    const bool split_w = hm.prec == 3;
    const int H = c.hidden_size, I = c.intermediate_size;
    const std::string &p = hm.prefix;
    auto T = [&](const std::string &n) { return hm.st.find(n); };
    auto vec = [&](const std::string &n, std::vector<int64_t> shape, float **dst) -> int {
        std::vector<float> h;
        if (!tensor_to_f32(T(n), shape, h, err, n)) return -1;
        return upload(D, dst, h);
    };
    auto mat = [&](std::vector<std::string> names, int cols, int interleave, int bn, Mat &m) -> int {
        std::vector<const TensorView *> parts;
        for (auto &n : names) parts.push_back(T(n));
        HostMat h;
        if (!prep_mat(parts, names, cols, hm.store, split_w, hm.f16, hm.prec == 4, interleave, h,
                      err))
            return -1;
        return upload_mat(D, h, bn, m);
    };

    // Embedding table: kept in the file dtype (it is only gathered).
    const std::string emb_name = c.family == FFWD_FAMILY_BERT ? p + "embeddings.word_embeddings.weight"
                                                              : p + "embed_tokens.weight";
    const TensorView *emb = T(emb_name);
    if (!emb || emb->shape != std::vector<int64_t>{c.vocab_size, H}) {
        err = "missing or mis-shaped " + emb_name;
        return -1;
    }
    if (emb->dtype == DType::BF16) {
        D.embed_bf16 = 1;
        void *q;
        CK(cudaMalloc(&q, emb->nbytes));
        D.allocs.push_back(q);
        CK(cudaMemcpy(q, emb->data, emb->nbytes, cudaMemcpyHostToDevice));
        D.embed = q;
    } else {
        std::vector<float> h;
        if (!tensor_to_f32(emb, {c.vocab_size, H}, h, err, emb_name)) return -1;
        float *q;
        if (upload(D, &q, h)) return -1;
        D.embed = q;
        D.embed_bf16 = 0;
    }

    D.layers.resize(c.n_layers);
    if (c.family == FFWD_FAMILY_BERT) {
        if (vec(p + "embeddings.position_embeddings.weight", {c.max_position_embeddings, H},
                &D.pos_table) ||
            vec(p + "embeddings.LayerNorm.weight", {H}, &D.emb_ln_g) ||
            vec(p + "embeddings.LayerNorm.bias", {H}, &D.emb_ln_b))
            return -1;
        {
            std::vector<float> h;
            const std::string n = p + "embeddings.token_type_embeddings.weight";
            if (!tensor_to_f32(T(n), {c.type_vocab_size, H}, h, err, n)) return -1;
            h.resize(H);  // token type 0
            if (upload(D, &D.type0, h)) return -1;
        }
        for (int i = 0; i < c.n_layers; ++i) {
            LayerW &l = D.layers[i];
            const std::string lp = p + "encoder.layer." + std::to_string(i) + ".";
            if (mat({lp + "attention.self.query.weight", lp + "attention.self.key.weight",
                     lp + "attention.self.value.weight"},
                    H, 0, pick_bn(3 * H), l.qkv) ||
                mat({lp + "attention.output.dense.weight"}, H, 0, pick_bn(H), l.o) ||
                mat({lp + "intermediate.dense.weight"}, H, 0, pick_bn(I), l.up) ||
                mat({lp + "output.dense.weight"}, I, 0, pick_bn(H), l.down))
                return -1;
            std::vector<float> bq, bk, bv;
            if (!tensor_to_f32(T(lp + "attention.self.query.bias"), {H}, bq, err, "query.bias") ||
                !tensor_to_f32(T(lp + "attention.self.key.bias"), {H}, bk, err, "key.bias") ||
                !tensor_to_f32(T(lp + "attention.self.value.bias"), {H}, bv, err, "value.bias"))
                return -1;
            bq.insert(bq.end(), bk.begin(), bk.end());
            bq.insert(bq.end(), bv.begin(), bv.end());
            if (upload(D, &l.b_qkv, bq)) return -1;
            if (vec(lp + "attention.output.dense.bias", {H}, &l.b_o) ||
                vec(lp + "attention.output.LayerNorm.weight", {H}, &l.ln1_g) ||
                vec(lp + "attention.output.LayerNorm.bias", {H}, &l.ln1_b) ||
                vec(lp + "intermediate.dense.bias", {I}, &l.b_up) ||
                vec(lp + "output.dense.bias", {H}, &l.b_down) ||
                vec(lp + "output.LayerNorm.weight", {H}, &l.ln2_g) ||
                vec(lp + "output.LayerNorm.bias", {H}, &l.ln2_b))
                return -1;
        }
    } else {
        const int qkv_out = c.q_dim + 2 * c.kv_dim;
        for (int i = 0; i < c.n_layers; ++i) {
            LayerW &l = D.layers[i];
            const std::string lp = p + "layers." + std::to_string(i) + ".";
            const int gu_bn = (I % 128 == 0) ? 256 : 128;
            l.swiglu_half = gu_bn / 2;
            if (mat({lp + "self_attn.q_proj.weight", lp + "self_attn.k_proj.weight",
                     lp + "self_attn.v_proj.weight"},
                    H, 0, qkv_out % 256 == 0 && 256 % c.head_dim == 0 ? 256 : 128, l.qkv) ||
                mat({lp + "self_attn.o_proj.weight"}, c.q_dim, 0, pick_bn(H), l.o) ||
                mat({lp + "mlp.gate_proj.weight", lp + "mlp.up_proj.weight"}, H, l.swiglu_half,
                    gu_bn, l.up) ||
                mat({lp + "mlp.down_proj.weight"}, I, 0, pick_bn(H), l.down))
                return -1;
            if (c.qkv_bias) {
                std::vector<float> bq, bk, bv;
                if (!tensor_to_f32(T(lp + "self_attn.q_proj.bias"), {c.q_dim}, bq, err, "q_proj.bias") ||
                    !tensor_to_f32(T(lp + "self_attn.k_proj.bias"), {c.kv_dim}, bk, err, "k_proj.bias") ||
                    !tensor_to_f32(T(lp + "self_attn.v_proj.bias"), {c.kv_dim}, bv, err, "v_proj.bias"))
                    return -1;
                bq.insert(bq.end(), bk.begin(), bk.end());
                bq.insert(bq.end(), bv.begin(), bv.end());
                if (upload(D, &l.b_qkv, bq)) return -1;
            }
            if (c.qk_norm && (vec(lp + "self_attn.q_norm.weight", {c.head_dim}, &l.q_norm) ||
                              vec(lp + "self_attn.k_norm.weight", {c.head_dim}, &l.k_norm)))
                return -1;
            if (vec(lp + "input_layernorm.weight", {H}, &l.in_norm) ||
                vec(lp + "post_attention_layernorm.weight", {H}, &l.post_norm))
                return -1;
        }
        if (vec(p + "norm.weight", {H}, &D.final_norm)) return -1;
        if (ensure_rope(D, c, 4096)) return -1;
    }
    return 0;
}

void free_device(Device &D) {
    cudaSetDevice(D.dev);
    if (D.stream) cudaStreamSynchronize(D.stream);
    for (void *q : D.allocs) cudaFree(q);
    D.allocs.clear();
    Workspace &w = D.ws;
    void *dptrs[] = {w.ids, w.pos, w.offsets, w.err, w.span_starts, w.span_ends, w.items, w.pooled,
                     w.x, w.xb, w.xb_lo, w.qkv, w.att, w.att_lo, w.hmid, w.hmid_lo, D.rope_cos,
                     D.rope_sin, D.rope_cos_h, D.rope_sin_h};
    for (void *q : dptrs)
        if (q) cudaFree(q);
    void *hptrs[] = {w.h_ids, w.h_offsets, w.h_err, w.h_items, w.h_out, w.h_spans};
    for (void *q : hptrs)
        if (q) cudaFreeHost(q);
    void *lptrs[] = {D.late_wt, D.late_vec, D.late_rows, D.late_doff, D.late_scores};
    for (void *q : lptrs)
        if (q) cudaFree(q);
    void *lhptrs[] = {D.h_late_rows, D.h_late_doff, D.h_late_vec, D.h_late_scores,
                      D.stg.ids, D.stg.offsets, D.stg.err, D.stg.items, D.stg.out};
    for (void *q : lhptrs)
        if (q) cudaFreeHost(q);
    for (cudaEvent_t e : D.fwd_done)
        if (e) cudaEventDestroy(e);
    if (D.stream) cudaStreamDestroy(D.stream);
    D = Device();
}

// ------------------------------------------------------------------ workspace

// Device and pinned allocations of the workspace.  ffwd_b200_test_inject can
// make the next ones fail, to exercise the out-of-memory paths.
cudaError_t ws_malloc(void **p, size_t bytes) {
    if (g_inject_alloc.load() > 0 && g_inject_alloc.fetch_sub(1) > 0) {
        *p = nullptr;
        return cudaErrorMemoryAllocation;
    }
    return cudaMalloc(p, bytes);
}

cudaError_t ws_malloc_host(void **p, size_t bytes) {
    if (g_inject_alloc.load() > 0 && g_inject_alloc.fetch_sub(1) > 0) {
        *p = nullptr;
        return cudaErrorMemoryAllocation;
    }
    return cudaMallocHost(p, bytes);
}

template <typename T>
int ws_free(T **p, bool host = false) {
    if (*p) {
        cudaError_t e = host ? cudaFreeHost(*p) : cudaFree(*p);
        *p = nullptr;
        CK(e);
    }
    return 0;
}

// Grow the workspace to T packed rows, B sequences, n_items attention items
// and n_spans spans.  A capacity is set only once all of its buffers exist,
// so a failed allocation leaves it at 0 and the next call allocates again.
int ensure_ws(ffwd_b200_ctx *ctx, Device &D, int T, int B, int n_items, int n_spans) {
    Workspace &w = D.ws;
    const ffwd_config_t &c = ctx->cfg;
    const bool exact = ctx->prec != 0;  // f32 qkv and attention
    const bool split = ctx->prec == 2 || ctx->prec == 3;
    const size_t ob = ctx->prec == 4 ? 4 : 2;  // bytes per GEMM operand element
    if (T > w.cap_t) {
        CK(cudaStreamSynchronize(D.stream));
        const int cap = std::max(T, std::min(g_max_tokens, std::max(T, 2 * w.cap_t)));
        w.cap_t = 0;
        void **bufs[] = {(void **)&w.ids, (void **)&w.pos, (void **)&w.x, (void **)&w.xb,
                         (void **)&w.xb_lo, &w.qkv, (void **)&w.att, (void **)&w.att_lo,
                         (void **)&w.hmid, (void **)&w.hmid_lo};
        for (void **b : bufs)
            if (ws_free(b)) return -1;
        if (ws_free(&w.h_ids, true)) return -1;
        const size_t t = (size_t)cap;
        const int H = c.hidden_size, qkv = c.q_dim + 2 * c.kv_dim;
        const int inter = c.intermediate_size;
        CK(ws_malloc((void **)&w.ids, t * 4));
        CK(ws_malloc((void **)&w.pos, t * 4));
        CK(ws_malloc((void **)&w.x, t * H * 4));
        CK(ws_malloc((void **)&w.xb, t * H * ob));
        CK(ws_malloc(&w.qkv, t * qkv * (exact ? 4 : 2)));
        CK(ws_malloc((void **)&w.att, t * c.q_dim * ob));
        CK(ws_malloc((void **)&w.hmid, t * inter * ob));
        if (split) {
            CK(ws_malloc((void **)&w.xb_lo, t * H * 2));
            CK(ws_malloc((void **)&w.att_lo, t * c.q_dim * 2));
            CK(ws_malloc((void **)&w.hmid_lo, t * inter * 2));
        }
        CK(ws_malloc_host((void **)&w.h_ids, t * 4));
        w.cap_t = cap;
    }
    // Pooled rows serve sequences and spans alike: size them for both.
    const int rows = std::max(B + 1, n_spans + 1);
    if (rows > w.cap_b) {
        CK(cudaStreamSynchronize(D.stream));
        const int cap = std::max(rows, 2 * w.cap_b);
        w.cap_b = 0;
        if (ws_free(&w.offsets) || ws_free(&w.pooled) || ws_free(&w.h_offsets, true) ||
            ws_free(&w.h_out, true))
            return -1;
        CK(ws_malloc((void **)&w.offsets, (size_t)cap * 4));
        CK(ws_malloc((void **)&w.pooled, (size_t)cap * c.hidden_size * 4));
        CK(ws_malloc_host((void **)&w.h_offsets, (size_t)cap * 4));
        CK(ws_malloc_host((void **)&w.h_out, (size_t)cap * c.hidden_size * 4));
        w.cap_b = cap;
    }
    if (n_items > w.cap_items) {
        CK(cudaStreamSynchronize(D.stream));
        const int cap = std::max(n_items, 2 * w.cap_items);
        w.cap_items = 0;
        if (ws_free(&w.items) || ws_free(&w.h_items, true)) return -1;
        CK(ws_malloc((void **)&w.items, (size_t)cap * sizeof(AttnItem)));
        CK(ws_malloc_host((void **)&w.h_items, (size_t)cap * sizeof(AttnItem)));
        w.cap_items = cap;
    }
    if (n_spans > w.cap_spans) {
        CK(cudaStreamSynchronize(D.stream));
        const int cap = std::max(n_spans, 2 * w.cap_spans);
        w.cap_spans = 0;
        if (ws_free(&w.span_starts) || ws_free(&w.span_ends) || ws_free(&w.h_spans, true))
            return -1;
        CK(ws_malloc((void **)&w.span_starts, (size_t)cap * 4));
        CK(ws_malloc((void **)&w.span_ends, (size_t)cap * 4));
        CK(ws_malloc_host((void **)&w.h_spans, (size_t)cap * 2 * 4));
        w.cap_spans = cap;
    }
    if (!w.err || !w.h_err) {
        // err[0]: device error word; err[2..3]: attention scheduler counters.
        if (ws_free(&w.err) || ws_free(&w.h_err, true)) return -1;
        CK(ws_malloc((void **)&w.err, 16));
        CK(cudaMemset(w.err, 0, 16));
        CK(ws_malloc_host((void **)&w.h_err, 4));
    }
    return 0;
}

// ------------------------------------------------------------------ forward

// Self-test of the bounded wait: one thread waits on an mbarrier that nothing
// ever arrives at, with a short limit; the wait records kErrWaitTimeout and
// the kernel returns.
__global__ void wait_selftest_kernel(int *err, uint64_t limit_ns) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
        abort_flag = 0;
    }
    __syncthreads();
    if (threadIdx.x == 0) mbar_wait(&bar, 0, err, &abort_flag, limit_ns);
}

__global__ void positions_kernel(const int *offsets, int pos_offset, int *pos) {
    const int b = blockIdx.x;
    const int s = offsets[b], e = offsets[b + 1];
    for (int t = s + threadIdx.x; t < e; t += blockDim.x) pos[t] = pos_offset + (t - s);
}

// Single-pass GEMMs with 256-wide tiles run on the two-SM kernel unless
// FFWD_B200_GEMM_2SM=0 (A/B comparisons).
bool use_gemm2() {
    static const bool on = [] {
        const char *e = getenv("FFWD_B200_GEMM_2SM");
        return !(e && e[0] == '0');
    }();
    return on;
}

// f16: single-pass operands (and 16-bit outputs) are f16 rather than bf16.
int gemm(Device &D, int prec, bool f16, const CUtensorMap *a, const CUtensorMap *a_lo, const Mat &w,
         GemmParams &p) {
    p.N = w.rows;
    p.K = w.cols;
    p.op_f16 = f16 && prec == 0;
    if (p.op_f16 && p.out_mode == kOutBF16) p.out_mode = kOutF16;
    const int passes = prec == 0 ? 1 : prec;  // 4: one kind::tf32 pass
    if (passes == 1 && w.bn == 256 && p.out_mode != kOutSplit && use_gemm2()) {
        CUtensorMap mo;
        if (make_epi_map(&mo, p)) return -1;
        LAUNCH(gemm2_launch(a, &w.map_half, &mo, p, D.num_sms, D.stream));
        return 0;
    }
    LAUNCH(gemm_launch(a, passes == 2 || passes == 3 ? a_lo : nullptr, &w.map_hi,
                       passes == 3 ? &w.map_lo : nullptr,
                       w.bn, passes, p, D.num_sms, D.stream));
    return 0;
}

// The exact plans (prec != 0) keep q, k and v as bf16 hi / lo matrices in the
// qkv buffer (4 bytes per element): hi first, then lo, each [T, qkv_dim].
__nv_bfloat16 *qkv_hi(const Workspace &w) { return static_cast<__nv_bfloat16 *>(w.qkv); }
__nv_bfloat16 *qkv_lo(const Workspace &w, int T, int qkv_dim) {
    return static_cast<__nv_bfloat16 *>(w.qkv) + (size_t)T * qkv_dim;
}

// Tensor maps over the GEMM operands of one forward and the qkv matrix (or its
// hi / lo pair) for the tensor-core attention: 16-bit with 64-column boxes,
// split-bf16 hi + lo, or tf32-rounded f32 with 32-column boxes.
int make_act_maps(const ffwd_b200_ctx *ctx, FwdState &fs, const Workspace &w, int T) {
    const ffwd_config_t &c = ctx->cfg;
    const int H = c.hidden_size, I = c.intermediate_size, qkv_dim = c.q_dim + 2 * c.kv_dim;
    const CUtensorMapSwizzle sw =
        c.head_dim == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
    const int hb = std::min(c.head_dim, 64);
    if (ctx->prec != 0 &&
        (make_map(&fs.m_qkv, qkv_hi(w), T, qkv_dim, 128, hb, sw) ||
         make_map(&fs.m_qkv_lo, qkv_lo(w, T, qkv_dim), T, qkv_dim, 128, hb, sw)))
        return -1;
    if (ctx->prec == 4) {
        auto m32 = [&](CUtensorMap *m, const void *ptr, int cols) {
            return make_map_dt(m, ptr, T, cols, 128, 32, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4);
        };
        return m32(&fs.m_xb, w.xb, H) || m32(&fs.m_att, w.att, c.q_dim) || m32(&fs.m_h, w.hmid, I)
                   ? -1
                   : 0;
    }
    if (make_map(&fs.m_xb, w.xb, T, H, 128, 64, CU_TENSOR_MAP_SWIZZLE_128B) ||
        make_map(&fs.m_att, w.att, T, c.q_dim, 128, 64, CU_TENSOR_MAP_SWIZZLE_128B) ||
        make_map(&fs.m_h, w.hmid, T, I, 128, 64, CU_TENSOR_MAP_SWIZZLE_128B))
        return -1;
    if (ctx->prec != 0)
        return make_map(&fs.m_xb_lo, w.xb_lo, T, H, 128, 64, CU_TENSOR_MAP_SWIZZLE_128B) ||
                       make_map(&fs.m_att_lo, w.att_lo, T, c.q_dim, 128, 64,
                                CU_TENSOR_MAP_SWIZZLE_128B) ||
                       make_map(&fs.m_h_lo, w.hmid_lo, T, I, 128, 64, CU_TENSOR_MAP_SWIZZLE_128B)
                   ? -1
                   : 0;
    return make_map(&fs.m_qkv, w.qkv, T, qkv_dim, 128, hb, sw) ? -1 : 0;
}

int embed_step(ffwd_b200_ctx *ctx, Device &D, const FwdState &fs, Workspace &w);

// Tensor maps, attention parameters, positions and the embedding (+ first
// norm) of one forward over the buffers of workspace w, whose ids, offsets and
// items (fs.n_items of them) already hold the packed batch (or are queued on
// D.stream before this).
int setup_forward(ffwd_b200_ctx *ctx, Device &D, FwdState &fs, Workspace &w, int T, int B) {
    const ffwd_config_t &c = ctx->cfg;
    fs.T = T;
    fs.B = B;
    if (make_act_maps(ctx, fs, w, T)) return -1;

    AttnParams &ap = fs.ap;
    ap = AttnParams{};
    ap.offsets = w.offsets;
    ap.items = w.items;
    ap.n_items = fs.n_items;
    ap.n_heads = c.n_heads;
    ap.n_kv_heads = c.n_kv_heads;
    ap.head_dim = c.head_dim;
    ap.q_col0 = 0;
    ap.k_col0 = c.q_dim;
    ap.v_col0 = c.q_dim + c.kv_dim;
    ap.causal = c.attention_mode == FFWD_ATTENTION_CAUSAL;
    ap.scale = 1.0f / sqrtf((float)c.head_dim);
    ap.out = w.att;
    ap.ldo = c.q_dim;
    ap.out_hi = w.att;
    ap.out_lo = w.att_lo;
    ap.err = w.err;
    ap.sched = w.err + 2;
    ap.f16 = ctx->f16 ? 1 : 0;
    ap.out_tf32 = ctx->prec == 4 ? reinterpret_cast<float *>(w.att) : nullptr;

    return embed_step(ctx, D, fs, w);
}

// Positions and the embedding (+ first norm) of the forward fs over w.
int embed_step(ffwd_b200_ctx *ctx, Device &D, const FwdState &fs, Workspace &w) {
    const ffwd_config_t &c = ctx->cfg;
    const bool split = ctx->prec == 2 || ctx->prec == 3;
    const int H = c.hidden_size, T = fs.T, B = fs.B;
    const bool bert = c.family == FFWD_FAMILY_BERT;
    const float eps = bert ? c.layer_norm_eps : c.rms_norm_eps;
    cudaStream_t s = D.stream;
    const RowOut xb_out{w.xb, split ? w.xb_lo : nullptr, ctx->f16 ? 1 : 0,
                        ctx->prec == 4 ? reinterpret_cast<float *>(w.xb) : nullptr};
    LAUNCH((positions_kernel<<<B, 256, 0, s>>>(w.offsets, bert ? c.position_id_offset : 0, w.pos),
            cudaGetLastError()));
    if (bert)
        LAUNCH(embed_ln_launch(w.ids, w.pos, T, D.embed, D.embed_bf16, c.vocab_size, D.pos_table,
                               D.type0, D.emb_ln_g, D.emb_ln_b, H, eps, w.x, xb_out, w.err, s));
    else
        LAUNCH(embed_rms_launch(w.ids, T, D.embed, D.embed_bf16, c.vocab_size, H, w.x,
                                D.layers[0].in_norm, eps, xb_out, w.err, s));
    return 0;
}

// Upload-independent preparation: RoPE cache, attention items, tensor maps,
// positions and the embedding (+ first norm).  ws.ids / ws.offsets must hold
// the packed batch; h_offsets is its host copy.
int prepare(ffwd_b200_ctx *ctx, Device &D, FwdState &fs, int T, int B, const int *h_offsets) {
    const ffwd_config_t &c = ctx->cfg;
    Workspace &w = D.ws;
    const bool bert = c.family == FFWD_FAMILY_BERT;
    cudaStream_t s = D.stream;

    int max_len = 0;
    for (int b = 0; b < B; ++b) max_len = std::max(max_len, h_offsets[b + 1] - h_offsets[b]);
    if (!bert && ensure_rope(D, c, max_len)) return -1;

    // Attention work list, heaviest first.
    {
        const int n = attention_count_items(c.n_heads, c.n_kv_heads, h_offsets, B);
        if (n < 0 || ensure_ws(ctx, D, T, B, n, 0)) return -1;
        fs.n_items = attention_build_items(c.attention_mode == FFWD_ATTENTION_CAUSAL, c.n_heads,
                                           c.n_kv_heads, h_offsets, B, w.h_items, w.cap_items,
                                           ctx->prec == 0);
        if (fs.n_items < 0) {
            fail("attention work list overflow");
            return -1;
        }
        CK(cudaMemcpyAsync(w.items, w.h_items, (size_t)fs.n_items * sizeof(AttnItem),
                           cudaMemcpyHostToDevice, s));
    }

    return setup_forward(ctx, D, fs, w, T, B);
}

// One op of layer li on the prepared forward.
int step(ffwd_b200_ctx *ctx, Device &D, FwdState &fs, int op, int li) {
    const ffwd_config_t &c = ctx->cfg;
    Workspace &w = D.active_ws ? *D.active_ws : D.ws;
    const int prec = ctx->prec;
    const bool exact = prec != 0;  // split-bf16 qkv and attention
    const bool split = prec == 2 || prec == 3;
    const int H = c.hidden_size, I = c.intermediate_size, T = fs.T;
    const int qkv_dim = c.q_dim + 2 * c.kv_dim;
    const bool bert = c.family == FFWD_FAMILY_BERT;
    const float eps = bert ? c.layer_norm_eps : c.rms_norm_eps;
    cudaStream_t s = D.stream;
    const LayerW &l = D.layers[li];
    const RowOut xb_out{w.xb, split ? w.xb_lo : nullptr, ctx->f16 ? 1 : 0,
                        ctx->prec == 4 ? reinterpret_cast<float *>(w.xb) : nullptr};
    switch (op) {
    case kOpQKV: {  // QKV projection (+ bias, + QK-norm and RoPE on the decoder)
        GemmParams p{};
        p.M = T;
        p.out = exact ? qkv_hi(w) : w.qkv;
        p.out_lo = exact ? qkv_lo(w, T, qkv_dim) : nullptr;
        p.ldo = qkv_dim;
        p.out_mode = exact ? kOutSplit : kOutBF16;
        p.bias = l.b_qkv;
        p.err = w.err;
        if (bert) {
            p.epi = kEpiStore;
        } else {
            p.epi = kEpiQKRope;
            p.pos = w.pos;
            p.rope_cos = D.rope_cos;
            p.rope_sin = D.rope_sin;
            p.rope_cos_h = D.rope_cos_h;
            p.rope_sin_h = D.rope_sin_h;
            p.q_norm = l.q_norm;
            p.k_norm = l.k_norm;
            p.n_q_heads = c.n_heads;
            p.n_kv_heads = c.n_kv_heads;
            p.head_dim = c.head_dim;
            p.eps = c.rms_norm_eps;
        }
        return gemm(D, prec, ctx->f16, &fs.m_xb, &fs.m_xb_lo, l.qkv, p);
    }
    case kOpAttn:
        if (exact)
            LAUNCH(attention_split_launch(&fs.m_qkv, &fs.m_qkv_lo, fs.ap, s));
        else
            LAUNCH(attention_tc_launch(&fs.m_qkv, fs.ap, s));
        return 0;
    case kOpO: {  // output projection + residual (+ bias)
        GemmParams p{};
        p.M = T;
        p.epi = kEpiResid;
        p.resid = w.x;
        p.ldr = H;
        p.bias = l.b_o;
        p.err = w.err;
        return gemm(D, prec, ctx->f16, &fs.m_att, &fs.m_att_lo, l.o, p);
    }
    case kOpNorm1:
        if (bert)
            LAUNCH(layernorm_launch(w.x, T, H, l.ln1_g, l.ln1_b, eps, xb_out, s));
        else
            LAUNCH(rmsnorm_launch(w.x, T, H, l.post_norm, eps, xb_out, s));
        return 0;
    case kOpUp: {  // FFN up (GELU) or gate/up (SwiGLU)
        GemmParams p{};
        p.M = T;
        p.out = w.hmid;
        p.out_lo = w.hmid_lo;
        p.ldo = I;
        p.out_mode = split ? kOutSplit : prec == 4 ? kOutTF32 : kOutBF16;
        p.err = w.err;
        if (bert) {
            p.epi = kEpiGelu;
            p.bias = l.b_up;
            p.gelu_tanh = c.ffn_act == FFWD_ACT_GELU_TANH;
        } else {
            p.epi = kEpiSwiGLU;
        }
        return gemm(D, prec, ctx->f16, &fs.m_xb, &fs.m_xb_lo, l.up, p);
    }
    case kOpDown: {  // FFN down + residual (+ bias)
        GemmParams p{};
        p.M = T;
        p.epi = kEpiResid;
        p.resid = w.x;
        p.ldr = H;
        p.bias = l.b_down;
        p.err = w.err;
        return gemm(D, prec, ctx->f16, &fs.m_h, &fs.m_h_lo, l.down, p);
    }
    case kOpNorm2:
        if (bert)
            LAUNCH(layernorm_launch(w.x, T, H, l.ln2_g, l.ln2_b, eps, xb_out, s));
        else if (li + 1 < c.n_layers)
            LAUNCH(rmsnorm_launch(w.x, T, H, D.layers[li + 1].in_norm, eps, xb_out, s));
        return 0;
    }
    fail("unknown op %d", op);
    return -1;
}

// The forward over the packed rows already uploaded to D.ws (ids, offsets on
// device; h_offsets on host).  Leaves final hidden states in ws.x.
int forward(ffwd_b200_ctx *ctx, Device &D, int T, int B, const int *h_offsets) {
    FwdState &fs = D.fs;
    if (prepare(ctx, D, fs, T, B, h_offsets)) return -1;
    for (int li = 0; li < ctx->cfg.n_layers; ++li)
        for (int op = 0; op < kOpCount; ++op)
            if (step(ctx, D, fs, op, li)) return -1;
    return 0;
}

int check_err(Device &D) {
    if (D.ws.h_err[0] != 0) {
        const int e = D.ws.h_err[0];
        fail("device error %d (%s)", e,
             e == kErrBadTokenId ? "invalid token id"
             : e == kErrBadNorm  ? "zero or non-finite embedding norm"
             : e == kErrWaitTimeout ? "device wait timed out"
                                    : "unknown");
        return -1;
    }
    return 0;
}

// Output form of pooled rows: the first `dims` values (L2-renormalised when
// `renorm`) as f32, tanh-int8 or sign bits (encode_rows_launch); row_bytes per
// output row.
struct OutSpec {
    int dims = 0, renorm = 0, enc = 0;
    size_t row_bytes = 0;
};

// Pinned staging of one forward: ids, row offsets, attention items, output
// rows and the error word.
struct HostSet {
    int *ids, *offsets, *err;
    AttnItem *items;
    uint8_t *out;
};

int grow_pinned(void **p, size_t *cap, size_t need) {
    if (need <= *cap) return 0;
    if (*p) CK(cudaFreeHost(*p));
    *p = nullptr;
    *cap = 0;
    CK(cudaMallocHost(p, need));
    *cap = need;
    return 0;
}

// Encode the sequences idx[] of inputs on device D (as one or more forwards of
// at most g_max_tokens packed rows), writing output rows to out + idx[i] *
// os.row_bytes.  With several forwards, two pinned staging sets alternate:
// forward k + 1 is packed and enqueued before the host waits for forward k,
// so the host's packing, work-list building and launches overlap the GPU.
int run_on_device(ffwd_b200_ctx *ctx, Device &D, const ffwd_input_t *inputs,
                  const std::vector<int> &idx, void *out, const OutSpec &os) {
    const ffwd_config_t &c = ctx->cfg;
    const int H = c.hidden_size;
    CK(cudaSetDevice(D.dev));
    {
        int entry = (int)(&D - ctx->devs.data());
        if (g_inject_shard.compare_exchange_strong(entry, -1)) {
            fail("injected failure of the shard on device entry %d", entry);
            return -1;
        }
    }
    // Forwards of at most g_max_tokens rows, sized evenly: with n forwards
    // needed, each aims at total / n tokens, so no small tail forward runs
    // the whole layer stack for a few sequences.
    long long total = 0;
    for (int i : idx) total += inputs[i].n_tokens;
    const long long n_fwd = (total + g_max_tokens - 1) / g_max_tokens;
    const long long aim = n_fwd > 1 ? (total + n_fwd - 1) / n_fwd : total;
    struct Chunk {
        size_t i0, i1;
        int T, B;
    };
    std::vector<Chunk> chunks;
    int maxT = 0, maxB = 0, maxItems = 0;
    std::vector<int> offs;
    for (size_t i0 = 0; i0 < idx.size();) {
        size_t i1 = i0;
        long long tok = 0;
        while (i1 < idx.size() &&
               (i1 == i0 || (tok + inputs[idx[i1]].n_tokens <= g_max_tokens && tok < aim))) {
            tok += inputs[idx[i1]].n_tokens;
            ++i1;
        }
        const int B = (int)(i1 - i0), T = (int)tok;
        offs.assign(1, 0);
        for (size_t i = i0; i < i1; ++i) offs.push_back(offs.back() + inputs[idx[i]].n_tokens);
        const int n_items = attention_count_items(c.n_heads, c.n_kv_heads, offs.data(), B);
        if (n_items < 0) {
            fail("attention work list too large");
            return -1;
        }
        chunks.push_back(Chunk{i0, i1, T, B});
        maxT = std::max(maxT, T);
        maxB = std::max(maxB, B);
        maxItems = std::max(maxItems, n_items);
        i0 = i1;
    }
    if (ensure_ws(ctx, D, maxT, maxB, maxItems, 0)) return -1;
    Workspace &w = D.ws;
    const HostSet set_a{w.h_ids, w.h_offsets, w.h_err, w.h_items, reinterpret_cast<uint8_t *>(w.h_out)};
    HostSet sets[2] = {set_a, set_a};
    if (chunks.size() > 1) {
        auto &g = D.stg;
        if (grow_pinned((void **)&g.ids, &g.cap_ids, (size_t)maxT * 4) ||
            grow_pinned((void **)&g.offsets, &g.cap_off, (size_t)(maxB + 1) * 4) ||
            grow_pinned((void **)&g.items, &g.cap_items, (size_t)maxItems * sizeof(AttnItem)) ||
            grow_pinned((void **)&g.out, &g.cap_out, (size_t)maxB * os.row_bytes))
            return -1;
        if (!g.err) CK(cudaMallocHost(&g.err, 16));
        for (auto &e : D.fwd_done)
            if (!e) CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        sets[1] = HostSet{g.ids, g.offsets, g.err, g.items, g.out};
    }
    auto use = [&](const HostSet &h) {
        w.h_ids = h.ids;
        w.h_offsets = h.offsets;
        w.h_err = h.err;
        w.h_items = h.items;
        w.h_out = reinterpret_cast<float *>(h.out);
    };
    // Copy forward k's rows out once its stream work is done.
    auto finish = [&](size_t k) -> int {
        const HostSet &h = sets[k & 1];
        if (chunks.size() > 1) CK(cudaEventSynchronize(D.fwd_done[k & 1]));
        else CK(cudaStreamSynchronize(D.stream));
        use(h);
        if (check_err(D)) return -1;
        for (size_t i = chunks[k].i0; i < chunks[k].i1; ++i)
            memcpy(static_cast<uint8_t *>(out) + (size_t)idx[i] * os.row_bytes,
                   h.out + (i - chunks[k].i0) * os.row_bytes, os.row_bytes);
        return 0;
    };
    auto enqueue = [&](size_t k) -> int {
        const Chunk &ch = chunks[k];
        use(sets[k & 1]);
        int off = 0;
        for (int b = 0; b < ch.B; ++b) {
            const ffwd_input_t &in = inputs[idx[ch.i0 + b]];
            w.h_offsets[b] = off;
            for (int t = 0; t < in.n_tokens; ++t) {
                const int id = in.ids[t];
                if (id < 0 || id >= c.vocab_size) {
                    fail("invalid token id %d at input %d position %d", id, idx[ch.i0 + b], t);
                    return -1;
                }
            }
            memcpy(w.h_ids + off, in.ids, (size_t)in.n_tokens * 4);
            off += in.n_tokens;
        }
        w.h_offsets[ch.B] = off;
        CK(cudaMemcpyAsync(w.ids, w.h_ids, (size_t)ch.T * 4, cudaMemcpyHostToDevice, D.stream));
        CK(cudaMemcpyAsync(w.offsets, w.h_offsets, (size_t)(ch.B + 1) * 4, cudaMemcpyHostToDevice,
                           D.stream));
        CK(cudaMemsetAsync(w.err, 0, 4, D.stream));
        if (forward(ctx, D, ch.T, ch.B, w.h_offsets)) return -1;
        LAUNCH(pool_launch(w.x, w.offsets, ch.B, H, c.pooling_mode,
                           c.family == FFWD_FAMILY_BERT ? nullptr : D.final_norm, c.rms_norm_eps,
                           c.normalize_embeddings, w.pooled, w.err, D.stream));
        const void *src = w.pooled;
        if (os.enc != 0 || os.dims != H || os.renorm) {
            // The FFN activation buffer is free after the forward: T >= B rows
            // of intermediate_size bf16 values, at least the 4 * H bytes of an
            // f32 row (intermediate_size >= 2 * hidden in every supported model).
            LAUNCH(encode_rows_launch(w.pooled, ch.B, H, os.dims, os.renorm, os.enc, w.hmid,
                                      w.err, D.stream));
            src = w.hmid;
        }
        CK(cudaMemcpyAsync(w.h_out, src, (size_t)ch.B * os.row_bytes, cudaMemcpyDeviceToHost,
                           D.stream));
        CK(cudaMemcpyAsync(w.h_err, w.err, 4, cudaMemcpyDeviceToHost, D.stream));
        if (chunks.size() > 1) CK(cudaEventRecord(D.fwd_done[k & 1], D.stream));
        return 0;
    };
    int rc = 0;
    for (size_t k = 0; rc == 0 && k < chunks.size(); ++k) {
        rc = enqueue(k);
        if (rc == 0 && k >= 1) rc = finish(k - 1);
    }
    if (rc == 0) rc = finish(chunks.size() - 1);
    if (rc != 0) cudaStreamSynchronize(D.stream);  // nothing in flight reads the staging
    use(set_a);
    return rc;
}

double seq_cost(const ffwd_b200_ctx *ctx, int L) {
    const ffwd_config_t &c = ctx->cfg;
    const double attn = c.attention_mode == FFWD_ATTENTION_CAUSAL ? 2.0 * c.q_dim * (L + 1.0)
                                                                  : 4.0 * c.q_dim * (double)L;
    return (double)L * ((double)ctx->lin_flops_per_token + attn * c.n_layers);
}

int validate_inputs(const ffwd_b200_ctx *ctx, const ffwd_input_t *inputs, int batch) {
    if (!ctx || !inputs || batch <= 0) {
        fail("invalid arguments");
        return -1;
    }
    long long total = 0;
    for (int b = 0; b < batch; ++b) {
        if (!inputs[b].ids || inputs[b].n_tokens <= 0) {
            fail("input %d is empty", b);
            return -1;
        }
        if (ctx->cfg.family == FFWD_FAMILY_BERT &&
            inputs[b].n_tokens > ctx->cfg.max_position_embeddings - ctx->cfg.position_id_offset) {
            fail("sequence length %d plus position offset %d exceeds max_position_embeddings %d",
                 inputs[b].n_tokens, ctx->cfg.position_id_offset,
                 ctx->cfg.max_position_embeddings);
            return -1;
        }
        total += inputs[b].n_tokens;
        if (total > INT32_MAX) {
            fail("batch too large");
            return -1;
        }
    }
    return 0;
}

// True if model_dir carries a 1_Dense projection head (a late-interaction
// model), libffwd/model.c:25-28.
bool has_late_projection(const std::string &dir) {
    struct stat st;
    return stat((dir + "/1_Dense/config.json").c_str(), &st) == 0 &&
           stat((dir + "/1_Dense/model.safetensors").c_str(), &st) == 0;
}

ffwd_b200_ctx *load_ctx(const char *model_dir);

}  // namespace
}  // namespace fb

using namespace fb;

// ====================================================================== C ABI

extern "C" {

FFWD_B200_API int ffwd_b200_set_fast_gemm(const char *mode) {
    if (!mode) return -1;
    if (!strcmp(mode, "f32")) g_gemm_mode = 0;
    else if (!strcmp(mode, "tf32")) g_gemm_mode = 1;
    else if (!strcmp(mode, "bf16")) g_gemm_mode = 2;
    else if (!strcmp(mode, "16f")) g_gemm_mode = 3;
    else return -1;
    return 0;
}

FFWD_B200_API int ffwd_b200_set_weights_bf16(int on) {
    g_weight_override = on ? 1 : 0;
    return 0;
}

FFWD_B200_API int ffwd_b200_set_weights_f16(int on) {
    g_weight_override = on ? 2 : 0;
    return 0;
}

FFWD_B200_API int ffwd_b200_set_weights_default(void) {
    g_weight_override = -1;
    return 0;
}

FFWD_B200_API int ffwd_b200_set_devices(const int *devices, int n) {
    if (n <= 0 || !devices) return -1;
    g_devices.assign(devices, devices + n);
    g_devices_set = true;
    return 0;
}

FFWD_B200_API int ffwd_b200_set_max_tokens(int max_tokens) {
    if (max_tokens < 1) return -1;
    g_max_tokens = max_tokens;
    return 0;
}

FFWD_B200_API const char *ffwd_b200_last_error(void) { return t_err.c_str(); }

FFWD_B200_API long long ffwd_b200_launch_count(void) { return g_launches.load(); }

FFWD_B200_API ffwd_b200_ctx_t *ffwd_b200_load(const char *model_dir) {
    t_err.clear();
    if (!model_dir) return nullptr;
    // A 1_Dense head makes the directory a late-interaction model, which is not
    // a pooled embedding model (libffwd/model.c:308-314).
    if (has_late_projection(model_dir)) {
        fail("load %s: late-interaction models require token-level MaxSim support and are not "
             "valid pooled embedding models (use ffwd_b200_late_load)",
             model_dir);
        return nullptr;
    }
    return load_ctx(model_dir);
}

}  // extern "C"

namespace fb {
namespace {

ffwd_b200_ctx *load_ctx(const char *model_dir) {
    auto hm = std::make_unique<HostModel>();
    std::string err;
    if (!parse_model_config(model_dir, hm->cfg, err) || !hm->st.open(model_dir, err)) {
        fail("load %s: %s", model_dir, err.c_str());
        return nullptr;
    }
    const ffwd_config_t &c = hm->cfg;
    if (c.family == FFWD_FAMILY_BERT) {
        if (hm->st.has("embeddings.word_embeddings.weight")) hm->prefix = "";
        else if (hm->st.has("bert.embeddings.word_embeddings.weight")) hm->prefix = "bert.";
        else if (hm->st.has("roberta.embeddings.word_embeddings.weight")) hm->prefix = "roberta.";
        else {
            fail("BERT-family word embeddings not found");
            return nullptr;
        }
    } else {
        if (hm->st.has("embed_tokens.weight")) hm->prefix = "";
        else if (hm->st.has("model.embed_tokens.weight")) hm->prefix = "model.";
        else {
            fail("neither embed_tokens.weight nor model.embed_tokens.weight was found");
            return nullptr;
        }
    }
    // Supported shapes of this backend.
    if (c.hidden_size % 128 != 0) {
        fail("hidden_size %d must be a multiple of 128", c.hidden_size);
        return nullptr;
    }
    if (c.head_dim != 32 && c.head_dim != 64 && c.head_dim != 128) {
        fail("head_dim %d unsupported (32, 64 or 128)", c.head_dim);
        return nullptr;
    }
    if (c.intermediate_size % 128 != 0 || c.hidden_size > 4096) {
        fail("intermediate_size must be a multiple of 128 and hidden_size <= 4096");
        return nullptr;
    }

    // Precision plan (mirrors libffwd/cuda.cu:189-247, 4225-4237, 5010-5019 and
    // linear_ex 2905-2964).  Weight storage follows the override, else the
    // file: BF16 files store bf16, F32 and F16 files f32 (the CPU model widens
    // F16 at load, model.c:158-172, so the embedding table reads as F32).
    //   decoder: bf16 storage -> bf16 operands; f16 storage -> activations cast
    //     to f16, f16 operands; f32 storage -> the GEMM mode (f32: split-bf16
    //     3-pass; tf32: one kind::tf32 pass; bf16 / 16f: single-pass bf16 / f16).
    //   BERT: f32 widens 16-bit storage back (bf16: 2-pass over exact bf16
    //     weights; f16 or f32: 3-pass, an f16 weight being exact as hi + lo);
    //     tf32 runs kind::tf32 over any storage (bf16 and f16 values are exact
    //     in tf32); bf16 / 16f run single-pass operands of the stored 16-bit
    //     type, or of the mode's type for f32 storage.
    const std::string probe = c.family == FFWD_FAMILY_BERT
                                  ? hm->prefix + "encoder.layer.0.attention.self.query.weight"
                                  : hm->prefix + "layers.0.self_attn.q_proj.weight";
    const TensorView *pt = hm->st.find(probe);
    if (!pt) {
        fail("tensor not found: %s", probe.c_str());
        return nullptr;
    }
    const int store = g_weight_override >= 0 ? g_weight_override : (pt->dtype == DType::BF16 ? 1 : 0);
    const bool exact = g_gemm_mode <= 1;
    int prec;
    bool f16 = false;
    const bool tf32 = g_gemm_mode == 1;
    if (c.family != FFWD_FAMILY_BERT) {
        if (store == 0 && exact) {
            prec = tf32 ? 4 : 3;
        } else {
            prec = 0;
            f16 = store == 2 || (store == 0 && g_gemm_mode == 3);
        }
    } else if (tf32) {
        prec = 4;
    } else if (exact) {
        prec = store == 1 ? 2 : 3;
    } else {
        prec = 0;
        f16 = store == 2 || (store == 0 && g_gemm_mode == 3);
    }
    hm->prec = prec;
    hm->store = store;
    hm->f16 = f16;

    auto *ctx = new ffwd_b200_ctx();
    ctx->cfg = c;
    ctx->prec = prec;
    ctx->f16 = f16;
    const int qkv_out = c.q_dim + 2 * c.kv_dim;
    ctx->lin_flops_per_token =
        2.0f * c.n_layers *
        ((float)c.hidden_size * qkv_out + (float)c.q_dim * c.hidden_size +
         (c.family == FFWD_FAMILY_BERT ? 2.0f : 3.0f) * c.hidden_size * c.intermediate_size);

    std::vector<int> devs = g_devices;
    if (!g_devices_set) {
        devs.clear();
        if (const char *e = getenv("FFWD_B200_DEVICES")) {
            std::string s(e);
            size_t pos = 0;
            while (pos < s.size()) {
                size_t q = s.find(',', pos);
                if (q == std::string::npos) q = s.size();
                if (q > pos) devs.push_back(atoi(s.substr(pos, q - pos).c_str()));
                pos = q + 1;
            }
        }
        if (devs.empty()) devs.push_back(0);
    }
    ctx->devs.resize(devs.size());
    for (size_t i = 0; i < devs.size(); ++i) {
        ctx->devs[i].dev = devs[i];
        if (load_device(*hm, ctx->devs[i], err)) {
            if (!err.empty()) fail("load %s on device %d: %s", model_dir, devs[i], err.c_str());
            ffwd_b200_free(ctx);
            return nullptr;
        }
    }
    return ctx;
}

}  // namespace
}  // namespace fb

extern "C" {

FFWD_B200_API void ffwd_b200_free(ffwd_b200_ctx_t *ctx) {
    if (!ctx) return;
    for (auto &D : ctx->devs) free_device(D);
    delete ctx;
}

FFWD_B200_API const ffwd_config_t *ffwd_b200_config(const ffwd_b200_ctx_t *ctx) {
    return ctx ? &ctx->cfg : nullptr;
}

FFWD_B200_API int ffwd_b200_precision(const ffwd_b200_ctx_t *ctx) {
    return ctx ? (ctx->prec == 0 && ctx->f16 ? 1 : ctx->prec) : -1;
}

FFWD_B200_API int ffwd_b200_lpt_partition(const double *cost, int n, int n_parts, int *part) {
    if (n < 0 || n_parts <= 0 || (n > 0 && (!cost || !part))) return -1;
    std::vector<int> order(n);
    std::iota(order.begin(), order.end(), 0);
    std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return cost[a] > cost[b]; });
    std::vector<double> load(n_parts, 0.0);
    for (int i : order) {
        int best = 0;
        for (int p = 1; p < n_parts; ++p)
            if (load[p] < load[best]) best = p;
        part[i] = best;
        load[best] += cost[i];
    }
    return 0;
}

FFWD_B200_API int ffwd_b200_attention_items(int causal, int windows, int n_heads, int n_kv_heads,
                                            const int *offsets, int batch, int *items, int cap) {
    if (batch < 0 || n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads || cap < 0 ||
        (batch > 0 && !offsets) || (cap > 0 && !items))
        return -1;
    const int n = attention_count_items(n_heads, n_kv_heads, offsets, batch);
    if (n < 0) return -1;
    if (!items) return n;
    std::vector<AttnItem> v(std::max(n, 1));
    const int got = attention_build_items(causal, n_heads, n_kv_heads, offsets, batch, v.data(), n,
                                          windows != 0);
    if (got < 0 || got > cap) return -1;
    for (int i = 0; i < got; ++i) {
        const AttnItem &it = v[i];
        int *o = items + 7 * i;
        o[0] = it.seq;
        o[1] = it.qt0;
        o[2] = it.h0;
        o[3] = it.qt1;
        o[4] = it.h1;
        o[5] = it.cost;
        o[6] = it.nseq;
    }
    return got;
}

}  // extern "C"

namespace fb {
namespace {

int encode_batch_impl(ffwd_b200_ctx_t *ctx, const ffwd_input_t *inputs, int batch, void *out,
                      const OutSpec &os) {
    const int nd = (int)ctx->devs.size();
    ctx->last_shards.assign(nd, ffwd_b200_ctx::Shard{});
    std::vector<std::vector<int>> idx(nd);
    if (nd == 1) {
        idx[0].resize(batch);
        std::iota(idx[0].begin(), idx[0].end(), 0);
    } else {
        std::vector<double> cost(batch);
        for (int b = 0; b < batch; ++b) cost[b] = seq_cost(ctx, inputs[b].n_tokens);
        std::vector<int> part(batch);
        ffwd_b200_lpt_partition(cost.data(), batch, nd, part.data());
        for (int b = 0; b < batch; ++b) idx[part[b]].push_back(b);
    }
    auto run = [&](int d) {
        auto &sh = ctx->last_shards[d];
        sh.seqs = (int)idx[d].size();
        for (int i : idx[d]) sh.tokens += inputs[i].n_tokens;
        const auto t0 = std::chrono::steady_clock::now();
        const int rc = run_on_device(ctx, ctx->devs[d], inputs, idx[d], out, os);
        sh.ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0)
                    .count();
        return rc;
    };
    if (nd == 1) return run(0);
    std::vector<int> rc(nd, 0);
    std::vector<std::string> errs(nd);
    std::vector<std::thread> th;
    for (int d = 0; d < nd; ++d) {
        if (idx[d].empty()) continue;
        th.emplace_back([&, d] {
            rc[d] = run(d);
            errs[d] = t_err;
        });
    }
    for (auto &t : th) t.join();
    for (int d = 0; d < nd; ++d)
        if (rc[d] != 0) {
            t_err = errs[d];
            return -1;
        }
    return 0;
}

}  // namespace
}  // namespace fb

extern "C" {

FFWD_B200_API int ffwd_b200_encode_batch(ffwd_b200_ctx_t *ctx, const ffwd_input_t *inputs,
                                         int batch, float *out) {
    t_err.clear();
    if (!out || validate_inputs(ctx, inputs, batch)) {
        if (!out) fail("null output");
        return -1;
    }
    const int H = ctx->cfg.hidden_size;
    return encode_batch_impl(ctx, inputs, batch, out, OutSpec{H, 0, 0, (size_t)H * 4});
}

FFWD_B200_API int ffwd_b200_encode_batch_as(ffwd_b200_ctx_t *ctx, const ffwd_input_t *inputs,
                                            int batch, int dims, int renormalize, int encoding,
                                            void *out) {
    t_err.clear();
    if (!out || validate_inputs(ctx, inputs, batch)) {
        if (!out) fail("null output");
        return -1;
    }
    const int H = ctx->cfg.hidden_size;
    if (dims <= 0 || dims > H || encoding < FFWD_B200_OUT_F32 || encoding > FFWD_B200_OUT_BINARY ||
        (encoding == FFWD_B200_OUT_BINARY && dims % 8 != 0)) {
        fail("invalid output form: dims %d (1..%d, a multiple of 8 for binary), encoding %d",
             dims, H, encoding);
        return -1;
    }
    const size_t row = encoding == FFWD_B200_OUT_F32    ? (size_t)dims * 4
                       : encoding == FFWD_B200_OUT_INT8 ? (size_t)dims
                                                        : (size_t)dims / 8;
    return encode_batch_impl(ctx, inputs, batch, out,
                             OutSpec{dims, renormalize && dims < H ? 1 : 0, encoding, row});
}

FFWD_B200_API int ffwd_b200_encode_into(ffwd_b200_ctx_t *ctx, const int *ids, int n, float *out) {
    ffwd_input_t in{ids, n};
    return ffwd_b200_encode_batch(ctx, &in, 1, out);
}

FFWD_B200_API float *ffwd_b200_encode(ffwd_b200_ctx_t *ctx, const int *ids, int n) {
    if (!ctx) return nullptr;
    float *out = (float *)malloc((size_t)ctx->cfg.hidden_size * sizeof(float));
    if (!out) return nullptr;
    if (ffwd_b200_encode_into(ctx, ids, n, out) != 0) {
        free(out);
        return nullptr;
    }
    return out;
}

FFWD_B200_API int ffwd_b200_encode_spans_batch(ffwd_b200_ctx_t *ctx,
                                               const ffwd_context_input_t *inputs, int batch,
                                               float *out) {
    t_err.clear();
    if (!ctx || !inputs || batch <= 0 || !out) {
        fail("invalid arguments");
        return -1;
    }
    std::vector<ffwd_input_t> packed(batch);
    int total_spans = 0;
    for (int b = 0; b < batch; ++b) {
        const ffwd_context_input_t &in = inputs[b];
        if (!in.input.ids || in.input.n_tokens <= 0 || !in.spans || in.n_spans <= 0) {
            fail("invalid span input %d", b);
            return -1;
        }
        for (int s = 0; s < in.n_spans; ++s) {
            const int st = in.spans[s].start, len = in.spans[s].n_tokens;
            if (st < 0 || len <= 0 || st > in.input.n_tokens || len > in.input.n_tokens - st) {
                fail("invalid span %d of input %d", s, b);
                return -1;
            }
        }
        packed[b] = in.input;
        total_spans += in.n_spans;
    }
    if (validate_inputs(ctx, packed.data(), batch)) return -1;
    const ffwd_config_t &c = ctx->cfg;
    Device &D = ctx->devs[0];
    CK(cudaSetDevice(D.dev));
    long long T64 = 0;
    for (auto &p : packed) T64 += p.n_tokens;
    const int T = (int)T64, H = c.hidden_size;
    if (ensure_ws(ctx, D, T, batch, 0, total_spans)) return -1;
    Workspace &w = D.ws;
    int off = 0, si = 0;
    for (int b = 0; b < batch; ++b) {
        const ffwd_input_t &in = packed[b];
        for (int t = 0; t < in.n_tokens; ++t)
            if (in.ids[t] < 0 || in.ids[t] >= c.vocab_size) {
                fail("invalid token id %d at input %d position %d", in.ids[t], b, t);
                return -1;
            }
        w.h_offsets[b] = off;
        memcpy(w.h_ids + off, in.ids, (size_t)in.n_tokens * 4);
        for (int s = 0; s < inputs[b].n_spans; ++s, ++si) {
            w.h_spans[si] = off + inputs[b].spans[s].start;
            w.h_spans[total_spans + si] = off + inputs[b].spans[s].start + inputs[b].spans[s].n_tokens;
        }
        off += in.n_tokens;
    }
    w.h_offsets[batch] = off;
    CK(cudaMemcpyAsync(w.ids, w.h_ids, (size_t)T * 4, cudaMemcpyHostToDevice, D.stream));
    CK(cudaMemcpyAsync(w.offsets, w.h_offsets, (size_t)(batch + 1) * 4, cudaMemcpyHostToDevice,
                       D.stream));
    CK(cudaMemcpyAsync(w.span_starts, w.h_spans, (size_t)total_spans * 4, cudaMemcpyHostToDevice,
                       D.stream));
    CK(cudaMemcpyAsync(w.span_ends, w.h_spans + total_spans, (size_t)total_spans * 4,
                       cudaMemcpyHostToDevice, D.stream));
    CK(cudaMemsetAsync(w.err, 0, 4, D.stream));
    if (forward(ctx, D, T, batch, w.h_offsets)) return -1;
    LAUNCH(span_pool_launch(w.x, w.span_starts, w.span_ends, total_spans, H,
                            c.family == FFWD_FAMILY_BERT ? nullptr : D.final_norm, c.rms_norm_eps,
                            w.pooled, D.stream));
    CK(cudaMemcpyAsync(w.h_out, w.pooled, (size_t)total_spans * H * 4, cudaMemcpyDeviceToHost,
                       D.stream));
    CK(cudaMemcpyAsync(w.h_err, w.err, 4, cudaMemcpyDeviceToHost, D.stream));
    CK(cudaStreamSynchronize(D.stream));
    if (check_err(D)) return -1;
    memcpy(out, w.h_out, (size_t)total_spans * H * 4);
    return 0;
}

FFWD_B200_API int ffwd_b200_encode_device(ffwd_b200_ctx_t *ctx, int dev, const int *d_ids,
                                          const int *h_offsets, int batch, float *d_out, int sync) {
    t_err.clear();
    if (h_offsets && batch > 0 && h_offsets[0] != 0) {
        fail("row offsets must start at 0 (got %d)", h_offsets[0]);
        return -1;
    }
    if (!ctx || dev < 0 || dev >= (int)ctx->devs.size() || !d_ids || !h_offsets || batch <= 0 ||
        !d_out) {
        fail("invalid arguments");
        return -1;
    }
    const ffwd_config_t &c = ctx->cfg;
    Device &D = ctx->devs[dev];
    CK(cudaSetDevice(D.dev));
    const int T = h_offsets[batch];
    for (int b = 0; b < batch; ++b) {
        const int L = h_offsets[b + 1] - h_offsets[b];
        if (L <= 0 || (c.family == FFWD_FAMILY_BERT &&
                       L > c.max_position_embeddings - c.position_id_offset)) {
            fail("invalid sequence length %d at %d", L, b);
            return -1;
        }
    }
    if (ensure_ws(ctx, D, T, batch, 0, 0)) return -1;
    Workspace &w = D.ws;
    memcpy(w.h_offsets, h_offsets, (size_t)(batch + 1) * 4);
    CK(cudaMemcpyAsync(w.ids, d_ids, (size_t)T * 4, cudaMemcpyDeviceToDevice, D.stream));
    CK(cudaMemcpyAsync(w.offsets, w.h_offsets, (size_t)(batch + 1) * 4, cudaMemcpyHostToDevice,
                       D.stream));
    CK(cudaMemsetAsync(w.err, 0, 4, D.stream));
    if (forward(ctx, D, T, batch, w.h_offsets)) return -1;
    LAUNCH(pool_launch(w.x, w.offsets, batch, c.hidden_size, c.pooling_mode,
                       c.family == FFWD_FAMILY_BERT ? nullptr : D.final_norm, c.rms_norm_eps,
                       c.normalize_embeddings, d_out, w.err, D.stream));
    if (sync) {
        CK(cudaMemcpyAsync(w.h_err, w.err, 4, cudaMemcpyDeviceToHost, D.stream));
        CK(cudaStreamSynchronize(D.stream));
        if (check_err(D)) return -1;
    }
    return 0;
}

FFWD_B200_API int ffwd_b200_run_op(ffwd_b200_ctx_t *ctx, int dev, int op, int layer, int reps) {
    t_err.clear();
    if (!ctx || dev < 0 || dev >= (int)ctx->devs.size() || op < 0 || op > kOpPool || layer < 0 ||
        layer >= ctx->cfg.n_layers || reps < 1) {
        fail("invalid arguments");
        return -1;
    }
    Device &D = ctx->devs[dev];
    if (D.fs.T <= 0) {
        fail("no prepared forward on device %d", dev);
        return -1;
    }
    CK(cudaSetDevice(D.dev));
    const ffwd_config_t &c = ctx->cfg;
    Workspace &w = D.ws;
    for (int r = 0; r < reps; ++r) {
        if (op == kOpEmbed) {
            if (embed_step(ctx, D, D.fs, w)) return -1;
        } else if (op == kOpPool) {
            LAUNCH(pool_launch(w.x, w.offsets, D.fs.B, c.hidden_size, c.pooling_mode,
                               c.family == FFWD_FAMILY_BERT ? nullptr : D.final_norm,
                               c.rms_norm_eps, c.normalize_embeddings, w.pooled, w.err, D.stream));
        } else if (step(ctx, D, D.fs, op, layer)) {
            return -1;
        }
    }
    return 0;
}

FFWD_B200_API int ffwd_b200_shard_stats(const ffwd_b200_ctx_t *ctx, int *seqs,
                                        long long *tokens, double *ms, int cap) {
    if (!ctx) return -1;
    const int n = (int)ctx->last_shards.size();
    for (int i = 0; i < n && i < cap; ++i) {
        if (seqs) seqs[i] = ctx->last_shards[i].seqs;
        if (tokens) tokens[i] = ctx->last_shards[i].tokens;
        if (ms) ms[i] = ctx->last_shards[i].ms;
    }
    return n;
}

FFWD_B200_API int ffwd_b200_test_inject(int kind, int value) {
    switch (kind) {
    case FFWD_B200_INJECT_NONE:
        g_inject_shard.store(-1);
        g_inject_alloc.store(0);
        return 0;
    case FFWD_B200_INJECT_SHARD:
        g_inject_shard.store(value);
        return 0;
    case FFWD_B200_INJECT_ALLOC:
        g_inject_alloc.store(value < 0 ? 0 : value);
        return 0;
    }
    return -1;
}

FFWD_B200_API int ffwd_b200_selftest_wait(int device, int limit_us) {
    t_err.clear();
    if (limit_us < 1 || limit_us > 1000000) {
        fail("limit_us must be in [1, 1000000]");
        return -1;
    }
    CK(cudaSetDevice(device));
    int *err = nullptr;
    CK(cudaMalloc(&err, 4));
    int h = 0;
    cudaError_t e = cudaMemset(err, 0, 4);
    if (e == cudaSuccess) {
        g_launches.fetch_add(1);
        wait_selftest_kernel<<<1, 32>>>(err, (uint64_t)limit_us * 1000ull);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpy(&h, err, 4, cudaMemcpyDeviceToHost);
    cudaFree(err);
    CK(e);
    if (h != 0) {
        fail("device error %d (%s)", h, h == kErrWaitTimeout ? "device wait timed out" : "unknown");
        return -1;
    }
    return 0;
}

FFWD_B200_API void *ffwd_b200_stream(ffwd_b200_ctx_t *ctx, int dev) {
    if (!ctx || dev < 0 || dev >= (int)ctx->devs.size()) return nullptr;
    return ctx->devs[dev].stream;
}

FFWD_B200_API int ffwd_b200_gemm_bf16(const void *x, const void *x_lo, const void *w,
                                      const void *w_lo, float *y, int M, int N, int K, int bn) {
    t_err.clear();
    if (!x || !w || !y || M <= 0 || N <= 0 || K <= 0 || (bn != 128 && bn != 256)) {
        fail("invalid arguments");
        return -1;
    }
    int dev = 0, sms = 148;
    CK(cudaGetDevice(&dev));
    CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    CUtensorMap ma, mal, mb, mbl;
    if (make_map(&ma, x, M, K, 128, 64, CU_TENSOR_MAP_SWIZZLE_128B) ||
        make_map(&mb, w, N, K, bn, 64, CU_TENSOR_MAP_SWIZZLE_128B))
        return -1;
    if (x_lo && make_map(&mal, x_lo, M, K, 128, 64, CU_TENSOR_MAP_SWIZZLE_128B)) return -1;
    if (w_lo && make_map(&mbl, w_lo, N, K, bn, 64, CU_TENSOR_MAP_SWIZZLE_128B)) return -1;
    const int passes = x_lo ? (w_lo ? 3 : 2) : 1;
    if (w_lo && !x_lo) {
        fail("w_lo requires x_lo");
        return -1;
    }
    GemmParams p{};
    p.M = M;
    p.N = N;
    p.K = K;
    p.epi = kEpiStore;
    p.out_mode = kOutF32;
    p.out = y;
    p.ldo = N;
    if (passes == 1 && bn == 256 && use_gemm2()) {
        CUtensorMap mh, mo;
        if (make_map(&mh, w, N, K, 128, 64, CU_TENSOR_MAP_SWIZZLE_128B) || make_epi_map(&mo, p))
            return -1;
        LAUNCH(gemm2_launch(&ma, &mh, &mo, p, sms, 0));
    } else {
        LAUNCH(gemm_launch(&ma, x_lo ? &mal : nullptr, &mb, w_lo ? &mbl : nullptr, bn, passes, p,
                           sms, 0));
    }
    CK(cudaDeviceSynchronize());
    return 0;
}

FFWD_B200_API int ffwd_b200_gemm_tf32(const float *x, const float *w, float *y, int M, int N, int K,
                                      int bn) {
    t_err.clear();
    if (!x || !w || !y || M <= 0 || N <= 0 || K <= 0 || K % 64 || (bn != 128 && bn != 256) ||
        N % bn) {
        fail("invalid arguments");
        return -1;
    }
    int dev = 0, sms = 148;
    CK(cudaGetDevice(&dev));
    CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    CUtensorMap ma, mb;
    if (make_map_dt(&ma, x, M, K, 128, 32, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4) ||
        make_map_dt(&mb, w, N, K, bn, 32, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4))
        return -1;
    GemmParams p{};
    p.M = M;
    p.N = N;
    p.K = K;
    p.epi = kEpiStore;
    p.out_mode = kOutF32;
    p.out = y;
    p.ldo = N;
    LAUNCH(gemm_launch(&ma, nullptr, &mb, nullptr, bn, 4, p, sms, 0));
    CK(cudaDeviceSynchronize());
    return 0;
}

}  // extern "C"

// ====================================================================== late interaction
//
// Mirrors libffwd/cuda.h:35-60 (ffwd_cuda_late_*) on top of the pooled
// engine: one packed forward, then the kept rows' token vectors (final norm,
// 1_Dense projection, L2) on the device.  ffwd_b200_late_rerank also scores
// MaxSim on the device; the reference scores on the host after copying every
// token vector back (backend_cuda.c:132-156).
namespace fb {
namespace {

int ensure_late(Device &D, size_t rows, size_t docs, int dim) {
    if (rows > D.late_cap_rows) {
        CK(cudaStreamSynchronize(D.stream));
        if (D.late_vec) CK(cudaFree(D.late_vec));
        if (D.late_rows) CK(cudaFree(D.late_rows));
        if (D.h_late_rows) CK(cudaFreeHost(D.h_late_rows));
        if (D.h_late_vec) CK(cudaFreeHost(D.h_late_vec));
        D.late_vec = nullptr;
        D.late_rows = D.h_late_rows = nullptr;
        D.h_late_vec = nullptr;
        const size_t cap = std::max(rows, 2 * D.late_cap_rows);
        D.late_cap_rows = 0;
        CK(cudaMalloc(&D.late_vec, cap * dim * sizeof(float)));
        CK(cudaMalloc(&D.late_rows, cap * sizeof(int)));
        CK(cudaMallocHost(&D.h_late_rows, cap * sizeof(int)));
        CK(cudaMallocHost(&D.h_late_vec, cap * dim * sizeof(float)));
        D.late_cap_rows = cap;
    }
    if (docs > D.late_cap_docs) {
        CK(cudaStreamSynchronize(D.stream));
        if (D.late_doff) CK(cudaFree(D.late_doff));
        if (D.late_scores) CK(cudaFree(D.late_scores));
        if (D.h_late_doff) CK(cudaFreeHost(D.h_late_doff));
        if (D.h_late_scores) CK(cudaFreeHost(D.h_late_scores));
        D.late_doff = D.h_late_doff = nullptr;
        D.late_scores = D.h_late_scores = nullptr;
        const size_t cap = std::max(docs, 2 * D.late_cap_docs);
        D.late_cap_docs = 0;
        CK(cudaMalloc(&D.late_doff, (cap + 1) * sizeof(int)));
        CK(cudaMalloc(&D.late_scores, cap * sizeof(float)));
        CK(cudaMallocHost(&D.h_late_doff, (cap + 1) * sizeof(int)));
        CK(cudaMallocHost(&D.h_late_scores, cap * sizeof(float)));
        D.late_cap_docs = cap;
    }
    return 0;
}

// One packed forward of inputs[0..n) on the context's first device, then the
// token vectors of the packed rows h_rows[0..n_rows) (filled by the caller
// into D.h_late_rows) into D.late_vec.  The stream is left running.
int late_forward(ffwd_b200_ctx *ctx, const ffwd_input_t *inputs, int n, int n_rows,
                 int normalize) {
    const ffwd_config_t &c = ctx->cfg;
    Device &D = ctx->devs[0];
    if (validate_inputs(ctx, inputs, n)) return -1;
    long long T = 0;
    for (int b = 0; b < n; ++b) T += inputs[b].n_tokens;
    if (T > g_max_tokens) {
        fail("late-interaction batch of %lld tokens exceeds the %d-token forward", T, g_max_tokens);
        return -1;
    }
    if (ensure_ws(ctx, D, (int)T, n, 0, 0)) return -1;
    Workspace &w = D.ws;
    int off = 0;
    for (int b = 0; b < n; ++b) {
        for (int t = 0; t < inputs[b].n_tokens; ++t) {
            const int id = inputs[b].ids[t];
            if (id < 0 || id >= c.vocab_size) {
                fail("invalid token id %d at input %d position %d", id, b, t);
                return -1;
            }
        }
        w.h_offsets[b] = off;
        memcpy(w.h_ids + off, inputs[b].ids, (size_t)inputs[b].n_tokens * 4);
        off += inputs[b].n_tokens;
    }
    w.h_offsets[n] = off;
    CK(cudaMemcpyAsync(w.ids, w.h_ids, (size_t)T * 4, cudaMemcpyHostToDevice, D.stream));
    CK(cudaMemcpyAsync(w.offsets, w.h_offsets, (size_t)(n + 1) * 4, cudaMemcpyHostToDevice,
                       D.stream));
    CK(cudaMemsetAsync(w.err, 0, 4, D.stream));
    if (forward(ctx, D, (int)T, n, w.h_offsets)) return -1;
    CK(cudaMemcpyAsync(D.late_rows, D.h_late_rows, (size_t)n_rows * 4, cudaMemcpyHostToDevice,
                       D.stream));
    LAUNCH(late_project_launch(w.x, c.hidden_size, D.late_rows, n_rows,
                               c.family == FFWD_FAMILY_BERT ? nullptr : D.final_norm,
                               c.rms_norm_eps, D.late_wt, ctx->token_dim, normalize, D.late_vec,
                               w.err, D.stream));
    return 0;
}

// Copy n_rows token vectors to out and check the device error word.
int late_fetch(ffwd_b200_ctx *ctx, int n_rows, float *out) {
    Device &D = ctx->devs[0];
    const size_t bytes = (size_t)n_rows * ctx->token_dim * sizeof(float);
    CK(cudaMemcpyAsync(D.h_late_vec, D.late_vec, bytes, cudaMemcpyDeviceToHost, D.stream));
    CK(cudaMemcpyAsync(D.ws.h_err, D.ws.err, 4, cudaMemcpyDeviceToHost, D.stream));
    CK(cudaStreamSynchronize(D.stream));
    if (check_err(D)) return -1;
    memcpy(out, D.h_late_vec, bytes);
    return 0;
}

// Reference input checks of ffwd_late_model_encode_docs (late_blas.c:117-134).
int late_check_docs(const int *const *doc_ids, const int *n_tokens, const int *const *keep,
                    const int *n_keep, int n_docs, long long *total_keep) {
    long long tk = 0;
    for (int d = 0; d < n_docs; ++d) {
        if (!doc_ids[d] || n_tokens[d] <= 0 || !keep[d] || n_keep[d] <= 0 ||
            n_keep[d] > n_tokens[d] || tk > INT32_MAX - n_keep[d]) {
            fail("document %d: empty, or kept count outside [1, n_tokens]", d);
            return -1;
        }
        for (int k = 0; k < n_keep[d]; ++k)
            if (keep[d][k] < 0 || keep[d][k] >= n_tokens[d]) {
                fail("document %d: kept index %d outside [0, %d)", d, keep[d][k], n_tokens[d]);
                return -1;
            }
        tk += n_keep[d];
    }
    *total_keep = tk;
    return 0;
}

}  // namespace
}  // namespace fb

extern "C" {

FFWD_B200_API ffwd_b200_late_ctx_t *ffwd_b200_late_load(const char *model_dir) {
    t_err.clear();
    if (!model_dir) return nullptr;
    if (!has_late_projection(model_dir)) {
        fail("late load %s: missing 1_Dense projection", model_dir);
        return nullptr;
    }
    SafeTensors st;
    std::string err;
    const std::string dense = std::string(model_dir) + "/1_Dense";
    if (!st.open(dense, err)) {
        fail("late load %s: cannot open %s/model.safetensors: %s", model_dir, dense.c_str(),
             err.c_str());
        return nullptr;
    }
    const TensorView *t = st.find("linear.weight");
    if (!t) {
        fail("late load %s: missing linear.weight", model_dir);
        return nullptr;
    }
    ffwd_b200_ctx *base = load_ctx(model_dir);
    if (!base) return nullptr;
    const int H = base->cfg.hidden_size;
    std::vector<float> w;
    if (t->shape.size() != 2 || t->shape[0] <= 0 || t->shape[0] > kLateMaxDim ||
        !tensor_to_f32(t, {t->shape[0], (int64_t)H}, w, err, "linear.weight")) {
        fail("late load %s: bad projection %s (token_dim must be in [1, %d], in = hidden %d)",
             model_dir, err.c_str(), kLateMaxDim, H);
        ffwd_b200_free(base);
        return nullptr;
    }
    const int dim = (int)t->shape[0];
    std::vector<float> wt((size_t)H * dim);
    for (int o = 0; o < dim; ++o)
        for (int h = 0; h < H; ++h) wt[(size_t)h * dim + o] = w[(size_t)o * H + h];
    Device &D = base->devs[0];
    if (cudaSetDevice(D.dev) != cudaSuccess || cudaMalloc(&D.late_wt, wt.size() * 4) != cudaSuccess ||
        cudaMemcpy(D.late_wt, wt.data(), wt.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
        fail("late load %s: projection upload failed", model_dir);
        ffwd_b200_free(base);
        return nullptr;
    }
    base->token_dim = dim;
    auto *ctx = new ffwd_b200_late_ctx();
    ctx->base = base;
    return ctx;
}

FFWD_B200_API void ffwd_b200_late_free(ffwd_b200_late_ctx_t *ctx) {
    if (!ctx) return;
    ffwd_b200_free(ctx->base);
    delete ctx;
}

FFWD_B200_API const ffwd_config_t *ffwd_b200_late_config(const ffwd_b200_late_ctx_t *ctx) {
    return ctx ? &ctx->base->cfg : nullptr;
}

FFWD_B200_API int ffwd_b200_late_token_dim(const ffwd_b200_late_ctx_t *ctx) {
    return ctx ? ctx->base->token_dim : 0;
}

FFWD_B200_API int ffwd_b200_late_encode_tokens(ffwd_b200_late_ctx_t *ctx, const int *token_ids,
                                               int n_tokens, int normalize, float *out_vectors) {
    t_err.clear();
    if (!ctx || !token_ids || n_tokens <= 0 || !out_vectors) {
        fail("invalid arguments");
        return -1;
    }
    ffwd_b200_ctx *b = ctx->base;
    Device &D = b->devs[0];
    CK(cudaSetDevice(D.dev));
    if (ensure_late(D, (size_t)n_tokens, 0, b->token_dim)) return -1;
    for (int i = 0; i < n_tokens; ++i) D.h_late_rows[i] = i;
    const ffwd_input_t in = {token_ids, n_tokens};
    if (late_forward(b, &in, 1, n_tokens, normalize)) return -1;
    return late_fetch(b, n_tokens, out_vectors);
}

FFWD_B200_API int ffwd_b200_late_encode_docs(ffwd_b200_late_ctx_t *ctx, const int *const *doc_ids,
                                             const int *n_tokens, const int *const *keep,
                                             const int *n_keep, int n_docs, int normalize,
                                             float *out_vectors, int *out_offsets) {
    t_err.clear();
    if (!ctx || !doc_ids || !n_tokens || !keep || !n_keep || n_docs <= 0 || !out_vectors ||
        !out_offsets) {
        fail("invalid arguments");
        return -1;
    }
    long long total_keep = 0;
    if (late_check_docs(doc_ids, n_tokens, keep, n_keep, n_docs, &total_keep)) return -1;
    ffwd_b200_ctx *b = ctx->base;
    Device &D = b->devs[0];
    CK(cudaSetDevice(D.dev));
    if (ensure_late(D, (size_t)total_keep, 0, b->token_dim)) return -1;
    std::vector<ffwd_input_t> inputs(n_docs);
    int pos = 0, start = 0;
    out_offsets[0] = 0;
    for (int d = 0; d < n_docs; ++d) {
        inputs[d] = ffwd_input_t{doc_ids[d], n_tokens[d]};
        for (int k = 0; k < n_keep[d]; ++k) D.h_late_rows[pos++] = start + keep[d][k];
        start += n_tokens[d];
        out_offsets[d + 1] = pos;
    }
    if (late_forward(b, inputs.data(), n_docs, (int)total_keep, normalize)) return -1;
    return late_fetch(b, (int)total_keep, out_vectors);
}

FFWD_B200_API int ffwd_b200_late_rerank(ffwd_b200_late_ctx_t *ctx, const ffwd_rerank_input_t *in,
                                        float *scores) {
    t_err.clear();
    if (!ctx || !in || !scores || !in->query_ids || in->query_n_tokens <= 0 ||
        in->query_n_keep <= 0 || in->query_n_keep > in->query_n_tokens || in->n_docs <= 0 ||
        !in->doc_ids || !in->doc_n_tokens || !in->doc_keep || !in->doc_n_keep) {
        fail("invalid arguments");
        return -1;
    }
    long long total_keep = 0;
    if (late_check_docs(in->doc_ids, in->doc_n_tokens, in->doc_keep, in->doc_n_keep, in->n_docs,
                        &total_keep))
        return -1;
    ffwd_b200_ctx *b = ctx->base;
    Device &D = b->devs[0];
    CK(cudaSetDevice(D.dev));
    const int qk = in->query_n_keep, dim = b->token_dim;
    if (ensure_late(D, (size_t)qk + total_keep, (size_t)in->n_docs, dim)) return -1;
    // Query and candidates in one packed forward; the query's first
    // query_n_keep vectors score against each candidate's kept vectors.
    std::vector<ffwd_input_t> inputs(in->n_docs + 1);
    inputs[0] = ffwd_input_t{in->query_ids, in->query_n_tokens};
    int pos = 0;
    for (int i = 0; i < qk; ++i) D.h_late_rows[pos++] = i;
    int start = in->query_n_tokens;
    D.h_late_doff[0] = 0;
    for (int d = 0; d < in->n_docs; ++d) {
        inputs[d + 1] = ffwd_input_t{in->doc_ids[d], in->doc_n_tokens[d]};
        for (int k = 0; k < in->doc_n_keep[d]; ++k) D.h_late_rows[pos++] = start + in->doc_keep[d][k];
        start += in->doc_n_tokens[d];
        D.h_late_doff[d + 1] = pos - qk;
    }
    if (late_forward(b, inputs.data(), in->n_docs + 1, pos, 1)) return -1;
    CK(cudaMemcpyAsync(D.late_doff, D.h_late_doff, (size_t)(in->n_docs + 1) * 4,
                       cudaMemcpyHostToDevice, D.stream));
    LAUNCH(late_maxsim_launch(D.late_vec, qk, D.late_vec + (size_t)qk * dim, D.late_doff,
                              in->n_docs, dim, D.late_scores, D.stream));
    CK(cudaMemcpyAsync(D.h_late_scores, D.late_scores, (size_t)in->n_docs * 4,
                       cudaMemcpyDeviceToHost, D.stream));
    CK(cudaMemcpyAsync(D.ws.h_err, D.ws.err, 4, cudaMemcpyDeviceToHost, D.stream));
    CK(cudaStreamSynchronize(D.stream));
    if (check_err(D)) return -1;
    memcpy(scores, D.h_late_scores, (size_t)in->n_docs * 4);
    return 0;
}

}  // extern "C"

// ====================================================================== no-allocation entry
//
// Scratch for ffwd_b200_encode_device_noalloc: a fixed arena in device global
// memory, reserved on every GPU that loads this library and held until the
// process exits.  It is shared by every call on a device and keeps the last
// call's contents.
namespace fb {
namespace {

constexpr size_t kNoAllocScratchBytes = 32u << 20;  // 32 MiB per device
constexpr int kNoAllocMaxItems = 8192;
constexpr int kNoAllocMaxBatch = 4096;
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch per device ordinal, resolved once per
// device (with that device current) when a model is loaded there.
uint8_t *g_noalloc_ptr[kNoAllocMaxDevices] = {};
std::mutex g_noalloc_mu;
// Host work list of the no-allocation entry, built under g_noalloc_mu (kept
// off the caller's stack: 8192 items are 192 KiB, more than many worker
// threads' stacks hold).
AttnItem g_noalloc_items[kNoAllocMaxItems];

int noalloc_scratch(int dev, uint8_t **out) {
    if (dev < 0 || dev >= kNoAllocMaxDevices) {
        fail("device ordinal %d out of range for the no-allocation scratch", dev);
        return -1;
    }
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            fail("cudaGetSymbolAddress(no-allocation scratch) failed on device %d: %s", dev,
                 cudaGetErrorString(e));
            return -1;
        }
        g_noalloc_ptr[dev] = static_cast<uint8_t *>(p);
    }
    *out = g_noalloc_ptr[dev];
    return 0;
}

// Bump carve of the arena (256-byte aligned pieces).  Returns false when the
// request does not fit.
struct Carver {
    uint8_t *base;
    size_t used = 0, cap;
    template <typename T>
    bool take(T **p, size_t count) {
        size_t off = (used + 255) & ~size_t(255);
        size_t bytes = count * sizeof(T);
        if (off + bytes > cap) return false;
        *p = reinterpret_cast<T *>(base + off);
        used = off + bytes;
        return true;
    }
};

}  // namespace
}  // namespace fb

extern "C" FFWD_B200_API int ffwd_b200_encode_device_noalloc(ffwd_b200_ctx_t *ctx, int dev,
                                                             const int *d_ids,
                                                             const int *h_offsets, int batch,
                                                             float *d_out) {
    t_err.clear();
    if (h_offsets && batch > 0 && h_offsets[0] != 0) {
        fail("row offsets must start at 0 (got %d)", h_offsets[0]);
        return -1;
    }
    if (!ctx || dev < 0 || dev >= (int)ctx->devs.size() || !d_ids || !h_offsets || batch <= 0 ||
        !d_out) {
        fail("invalid arguments");
        return -1;
    }
    const ffwd_config_t &c = ctx->cfg;
    Device &D = ctx->devs[dev];
    CK(cudaSetDevice(D.dev));
    const int T = h_offsets[batch];
    int max_len = 0;
    for (int b = 0; b < batch; ++b) {
        const int L = h_offsets[b + 1] - h_offsets[b];
        if (L <= 0 || (c.family == FFWD_FAMILY_BERT &&
                       L > c.max_position_embeddings - c.position_id_offset)) {
            fail("invalid sequence length %d at %d", L, b);
            return -1;
        }
        max_len = std::max(max_len, L);
    }
    if (batch > kNoAllocMaxBatch) {
        fail("no-allocation encode: batch %d exceeds the maximum %d", batch, kNoAllocMaxBatch);
        return -1;
    }
    if (c.family != FFWD_FAMILY_BERT && max_len > D.rope_cap) {
        fail("no-allocation encode: sequence length %d exceeds the loaded RoPE table (%d)", max_len,
             D.rope_cap);
        return -1;
    }

    // Carve the arena.
    uint8_t *base = nullptr;
    if (noalloc_scratch(D.dev, &base)) return -1;
    const bool exact = ctx->prec != 0;  // split-bf16 qkv and attention
    const bool split = ctx->prec == 2 || ctx->prec == 3;
    const int n_need = attention_count_items(c.n_heads, c.n_kv_heads, h_offsets, batch);
    if (n_need < 0 || n_need > kNoAllocMaxItems) {
        fail("no-allocation encode: more than %d attention work items", kNoAllocMaxItems);
        return -1;
    }
    const int H = c.hidden_size, I = c.intermediate_size, qkv_dim = c.q_dim + 2 * c.kv_dim;
    Workspace w{};
    Carver cv{base, 0, kNoAllocScratchBytes};
    const size_t ob16 = ctx->prec == 4 ? 2 : 1;  // 16-bit units per GEMM operand element
    bool ok = cv.take(&w.err, 4) && cv.take(&w.offsets, (size_t)batch + 1) &&
              cv.take(&w.items, (size_t)n_need) && cv.take(&w.ids, (size_t)T) &&
              cv.take(&w.pos, (size_t)T) && cv.take(&w.x, (size_t)T * H) &&
              cv.take(&w.xb, (size_t)T * H * ob16) && cv.take(&w.att, (size_t)T * c.q_dim * ob16) &&
              cv.take(&w.hmid, (size_t)T * I * ob16);
    if (ok) {
        uint8_t *q = nullptr;
        ok = cv.take(&q, (size_t)T * qkv_dim * (exact ? 4 : 2));
        w.qkv = q;
    }
    if (ok && split)
        ok = cv.take(&w.xb_lo, (size_t)T * H) && cv.take(&w.att_lo, (size_t)T * c.q_dim) &&
             cv.take(&w.hmid_lo, (size_t)T * I);
    if (!ok) {
        fail("no-allocation encode: %d tokens need more than the %zu-byte scratch maximum", T,
             kNoAllocScratchBytes);
        return -1;
    }
    w.cap_t = T;
    w.cap_b = batch + 1;
    w.cap_items = n_need;

    cudaStream_t s = D.stream;
    FwdState fs;
    CK(cudaMemsetAsync(w.err, 0, 16, s));  // error word and scheduler counters
    CK(cudaMemcpyAsync(w.ids, d_ids, (size_t)T * 4, cudaMemcpyDeviceToDevice, s));
    CK(cudaMemcpyAsync(w.offsets, h_offsets, (size_t)(batch + 1) * 4, cudaMemcpyHostToDevice, s));
    {
        // Attention work list, heaviest first (the builder prepare() uses).  The
        // copy from pageable memory has left the host array when it returns.
        std::lock_guard<std::mutex> lk(g_noalloc_mu);
        fs.n_items = attention_build_items(c.attention_mode == FFWD_ATTENTION_CAUSAL, c.n_heads,
                                           c.n_kv_heads, h_offsets, batch, g_noalloc_items,
                                           kNoAllocMaxItems, ctx->prec == 0);
        if (fs.n_items < 0 || fs.n_items > n_need) {
            fail("no-allocation encode: attention work list overflow");
            return -1;
        }
        CK(cudaMemcpyAsync(w.items, g_noalloc_items, (size_t)fs.n_items * sizeof(AttnItem),
                           cudaMemcpyHostToDevice, s));
    }

    // Forward on the arena buffers: same setup / step sequence as forward().
    if (setup_forward(ctx, D, fs, w, T, batch)) return -1;
    D.active_ws = &w;
    int rc = 0;
    for (int li = 0; li < c.n_layers && rc == 0; ++li)
        for (int op = 0; op < kOpCount && rc == 0; ++op) rc = step(ctx, D, fs, op, li);
    D.active_ws = nullptr;
    if (rc) return -1;
    LAUNCH(pool_launch(w.x, w.offsets, batch, H, c.pooling_mode,
                       c.family == FFWD_FAMILY_BERT ? nullptr : D.final_norm, c.rms_norm_eps,
                       c.normalize_embeddings, d_out, w.err, s));
    int h_err = 0;
    CK(cudaMemcpyAsync(&h_err, w.err, 4, cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    if (h_err) {
        fail("device error %d in no-allocation encode", h_err);
        return -1;
    }
    return 0;
}
