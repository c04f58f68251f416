// Model metadata + safetensors reader (see loader.h).
#include "loader.h"
#include "json.h"

#include <algorithm>
#include <cmath>
#include <climits>
#include <cstdio>
#include <cstring>
#include <dirent.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

namespace fb {

uint16_t f32_to_bf16_rne(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) return (uint16_t)((u >> 16) | 0x40);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

float bf16_to_f32(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

uint16_t f32_to_f16_rne(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    const uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    const uint32_t a = u & 0x7FFFFFFFu;
    if (a > 0x7F800000u) return sign | 0x7E00u;    // NaN
    if (a >= 0x477FF000u) return sign | 0x7C00u;   // |x| >= 65520 rounds to inf
    uint32_t r, rem, half;
    if (a < 0x38800000u) {                         // below 2^-14: subnormal result
        const uint32_t e = a >> 23;
        const uint32_t shift = 126 - e;            // value = m * 2^(e - 150); unit 2^-24
        if (shift > 24) return sign;
        const uint32_t m = (a & 0x7FFFFFu) | 0x800000u;
        r = m >> shift;
        rem = m & ((1u << shift) - 1);
        half = 1u << (shift - 1);
    } else {
        r = ((((a >> 23) - 112) << 10) | ((a & 0x7FFFFFu) >> 13));
        rem = a & 0x1FFFu;
        half = 0x1000u;
    }
    if (rem > half || (rem == half && (r & 1u))) ++r;  // a carry moves into the exponent
    return (uint16_t)(sign | r);
}

float f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1F;
    uint32_t mant = h & 0x3FF;
    uint32_t u;
    if (exp == 0) {
        if (mant == 0) {
            u = sign;
        } else {
            exp = 127 - 15 + 1;
            while (!(mant & 0x400)) {
                mant <<= 1;
                --exp;
            }
            mant &= 0x3FF;
            u = sign | (exp << 23) | (mant << 13);
        }
    } else if (exp == 31) {
        u = sign | 0x7F800000u | (mant << 13);
    } else {
        u = sign | ((exp + 127 - 15) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &u, 4);
    return f;
}

// ----------------------------------------------------------------- safetensors

SafeTensors::~SafeTensors() {
    for (auto &m : maps_)
        if (m.base) munmap(m.base, m.size);
}

bool SafeTensors::open_file(const std::string &path, std::string &err) {
    int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) {
        err = "cannot open " + path;
        return false;
    }
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 8) {
        ::close(fd);
        err = "bad safetensors file " + path;
        return false;
    }
    size_t size = (size_t)st.st_size;
    void *base = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (base == MAP_FAILED) {
        err = "mmap failed for " + path;
        return false;
    }
    maps_.push_back({base, size});
    uint64_t hlen;
    memcpy(&hlen, base, 8);
    if (hlen > size - 8) {
        err = "bad safetensors header size in " + path;
        return false;
    }
    json::Value root;
    if (!json::parse(std::string((const char *)base + 8, hlen), root) ||
        root.kind != json::Value::Object) {
        err = "bad safetensors header in " + path;
        return false;
    }
    const uint8_t *data0 = (const uint8_t *)base + 8 + hlen;
    const size_t data_size = size - 8 - hlen;
    for (const auto &kv : root.obj) {
        if (kv.first == "__metadata__") continue;
        const json::Value &v = kv.second;
        const json::Value *dt = v.get("dtype");
        const json::Value *sh = v.get("shape");
        const json::Value *off = v.get("data_offsets");
        if (!dt || !sh || !off || off->arr.size() != 2) {
            err = "bad tensor entry " + kv.first;
            return false;
        }
        TensorView t;
        t.dtype = dt->str == "F32" ? DType::F32 : dt->str == "BF16" ? DType::BF16
                                   : dt->str == "F16" ? DType::F16 : DType::Other;
        for (const auto &d : sh->arr) t.shape.push_back((int64_t)d.num);
        const size_t a = (size_t)off->arr[0].num, b = (size_t)off->arr[1].num;
        if (b < a || b > data_size) {
            err = "tensor data out of bounds for " + kv.first;
            return false;
        }
        t.data = data0 + a;
        t.nbytes = b - a;
        tensors_[kv.first] = t;
    }
    return true;
}

bool SafeTensors::open(const std::string &dir, std::string &err) {
    std::string single = dir + "/model.safetensors";
    struct stat st;
    if (stat(single.c_str(), &st) == 0) return open_file(single, err);
    DIR *d = opendir(dir.c_str());
    if (!d) {
        err = "cannot open model dir " + dir;
        return false;
    }
    std::vector<std::string> shards;
    int expected = 0;
    while (dirent *e = readdir(d)) {
        const char *n = e->d_name;
        if (strncmp(n, "model-", 6) != 0 || !strstr(n, ".safetensors")) continue;
        int idx = 0, tot = 0, used = 0;
        if (sscanf(n, "model-%d-of-%d.safetensors%n", &idx, &tot, &used) != 2 || n[used] != '\0' ||
            idx <= 0 || tot <= 0 || idx > tot) {
            closedir(d);
            err = std::string("bad shard name ") + n;
            return false;
        }
        if (expected && expected != tot) {
            closedir(d);
            err = "inconsistent shard totals";
            return false;
        }
        expected = tot;
        shards.push_back(n);
    }
    closedir(d);
    if (shards.empty() || (int)shards.size() != expected) {
        err = "no complete safetensors set in " + dir;
        return false;
    }
    std::sort(shards.begin(), shards.end());
    for (const auto &s : shards)
        if (!open_file(dir + "/" + s, err)) return false;
    return true;
}

const TensorView *SafeTensors::find(const std::string &name) const {
    auto it = tensors_.find(name);
    return it == tensors_.end() ? nullptr : &it->second;
}

bool tensor_to_f32(const TensorView *t, const std::vector<int64_t> &shape, std::vector<float> &out,
                   std::string &err, const std::string &name) {
    if (!t) {
        err = "tensor not found: " + name;
        return false;
    }
    if (t->shape != shape) {
        err = "bad shape for " + name;
        return false;
    }
    const int64_t n = t->numel();
    const size_t esz = t->dtype == DType::F32 ? 4 : 2;
    if (t->dtype == DType::Other || t->nbytes != (size_t)n * esz) {
        err = "unsupported dtype or size for " + name;
        return false;
    }
    out.resize((size_t)n);
    if (t->dtype == DType::F32) {
        memcpy(out.data(), t->data, (size_t)n * 4);
    } else {
        const uint16_t *s = (const uint16_t *)t->data;
        if (t->dtype == DType::BF16)
            for (int64_t i = 0; i < n; ++i) out[i] = bf16_to_f32(s[i]);
        else
            for (int64_t i = 0; i < n; ++i) out[i] = f16_to_f32(s[i]);
    }
    return true;
}

// ----------------------------------------------------------------- config

namespace {

bool read_file(const std::string &path, std::string &out) {
    FILE *f = fopen(path.c_str(), "rb");
    if (!f) return false;
    char buf[65536];
    size_t n;
    while ((n = fread(buf, 1, sizeof buf, f)) > 0) out.append(buf, n);
    fclose(f);
    return true;
}

int get_int(const json::Value &r, const char *k, int def) {
    const json::Value *v = r.get(k);
    return v && v->is_num() ? (int)v->num : def;
}

double get_double(const json::Value &r, const char *k, double def) {
    const json::Value *v = r.get(k);
    return v && v->is_num() ? v->num : def;
}

bool str_eq(const json::Value &r, const char *k, const char *s) {
    const json::Value *v = r.get(k);
    return v && v->kind == json::Value::String && v->str == s;
}

// -1 invalid type, 0 missing, 1 false, 2 true
int get_bool(const json::Value &r, const char *k) {
    const json::Value *v = r.get(k);
    if (!v) return 0;
    if (v->kind != json::Value::Bool) return v->kind == json::Value::Null ? 0 : -1;
    return v->b ? 2 : 1;
}

}  // namespace

bool parse_model_config(const std::string &dir, ffwd_config_t &cfg, std::string &err) {
    std::string text;
    if (!read_file(dir + "/config.json", text)) {
        err = "cannot open " + dir + "/config.json";
        return false;
    }
    json::Value root;
    if (!json::parse(text, root) || root.kind != json::Value::Object) {
        err = "invalid JSON in config.json";
        return false;
    }
    memset(&cfg, 0, sizeof cfg);
    cfg.hidden_size = get_int(root, "hidden_size", 0);
    cfg.n_layers = get_int(root, "num_hidden_layers", 0);
    cfg.n_heads = get_int(root, "num_attention_heads", 0);
    cfg.n_kv_heads = get_int(root, "num_key_value_heads", 0);
    cfg.head_dim = get_int(root, "head_dim", 128);
    cfg.intermediate_size = get_int(root, "intermediate_size", 0);
    cfg.vocab_size = get_int(root, "vocab_size", 151936);
    cfg.rms_norm_eps = (float)get_double(root, "rms_norm_eps", 1e-6);
    cfg.layer_norm_eps = (float)get_double(root, "layer_norm_eps", 1e-12);
    cfg.rope_theta = (float)get_double(root, "rope_theta", 1000000.0);
    cfg.max_position_embeddings = get_int(root, "max_position_embeddings", 0);
    cfg.position_id_offset = 0;
    cfg.type_vocab_size = get_int(root, "type_vocab_size", 2);
    cfg.family = FFWD_FAMILY_QWEN3;
    cfg.ffn_act = FFWD_ACT_GELU_ERF;
    cfg.qk_norm = 1;
    cfg.qkv_bias = 0;
    cfg.attention_mode = FFWD_ATTENTION_BIDIRECTIONAL;
    cfg.pooling_mode = FFWD_POOL_MEAN;
    cfg.normalize_embeddings = 0;
    cfg.append_terminal_token = 0;

    if (str_eq(root, "model_type", "qwen3")) {
        cfg.attention_mode = FFWD_ATTENTION_CAUSAL;
        cfg.pooling_mode = FFWD_POOL_LAST_TOKEN;
        cfg.normalize_embeddings = 1;
        cfg.append_terminal_token = 1;
    } else if (str_eq(root, "model_type", "qwen2")) {
        cfg.qk_norm = 0;
        cfg.qkv_bias = 1;
        cfg.attention_mode = FFWD_ATTENTION_CAUSAL;
    } else if (str_eq(root, "model_type", "bert") || str_eq(root, "model_type", "roberta") ||
               str_eq(root, "model_type", "xlm-roberta")) {
        cfg.family = FFWD_FAMILY_BERT;
        cfg.qk_norm = 0;
        cfg.qkv_bias = 1;
        cfg.attention_mode = FFWD_ATTENTION_BIDIRECTIONAL;
        cfg.n_kv_heads = cfg.n_heads;
        cfg.head_dim = cfg.n_heads > 0 ? cfg.hidden_size / cfg.n_heads : 0;
        if (str_eq(root, "model_type", "roberta") || str_eq(root, "model_type", "xlm-roberta")) {
            int pad = get_int(root, "pad_token_id", 1);
            if (pad < 0 || pad == INT_MAX) {
                err = "invalid RoBERTa pad_token_id";
                return false;
            }
            cfg.position_id_offset = pad + 1;
        }
        if (str_eq(root, "hidden_act", "gelu_new") || str_eq(root, "hidden_act", "gelu_pytorch_tanh"))
            cfg.ffn_act = FFWD_ACT_GELU_TANH;
        if (cfg.max_position_embeddings <= 0 ||
            cfg.position_id_offset >= cfg.max_position_embeddings || cfg.type_vocab_size <= 0 ||
            !std::isfinite(cfg.layer_norm_eps) || cfg.layer_norm_eps <= 0.0f) {
            err = "invalid BERT layer_norm_eps/max_position_embeddings";
            return false;
        }
    }
    int is_causal = get_bool(root, "is_causal");
    if (is_causal < 0) {
        err = "invalid is_causal";
        return false;
    }
    if (is_causal) cfg.attention_mode = is_causal == 2 ? FFWD_ATTENTION_CAUSAL : FFWD_ATTENTION_BIDIRECTIONAL;
    if (cfg.n_heads > 0 && cfg.head_dim > 0 && cfg.n_heads <= INT_MAX / cfg.head_dim)
        cfg.q_dim = cfg.n_heads * cfg.head_dim;
    if (cfg.n_kv_heads > 0 && cfg.head_dim > 0 && cfg.n_kv_heads <= INT_MAX / cfg.head_dim)
        cfg.kv_dim = cfg.n_kv_heads * cfg.head_dim;

    // sentence-transformers metadata (config.c:96-175)
    std::string meta;
    if (read_file(dir + "/1_Pooling/config.json", meta)) {
        json::Value pr;
        if (!json::parse(meta, pr)) {
            err = "invalid pooling metadata";
            return false;
        }
        int mean = get_bool(pr, "pooling_mode_mean_tokens");
        int last = get_bool(pr, "pooling_mode_lasttoken");
        int cls = get_bool(pr, "pooling_mode_cls_token");
        int mx = get_bool(pr, "pooling_mode_max_tokens");
        int sq = get_bool(pr, "pooling_mode_mean_sqrt_len_tokens");
        int wt = get_bool(pr, "pooling_mode_weightedmean_tokens");
        if (mean < 0 || last < 0 || cls < 0 || mx < 0 || sq < 0 || wt < 0) {
            err = "invalid pooling metadata";
            return false;
        }
        int supported = (mean == 2) + (last == 2) + (cls == 2);
        if (supported != 1 || mx == 2 || sq == 2 || wt == 2) {
            err = "unsupported Sentence Transformers pooling mode";
            return false;
        }
        cfg.pooling_mode = cls == 2 ? FFWD_POOL_CLS : last == 2 ? FFWD_POOL_LAST_TOKEN : FFWD_POOL_MEAN;
    }
    meta.clear();
    if (read_file(dir + "/modules.json", meta)) {
        json::Value mr;
        int normalize = 0;
        if (json::parse(meta, mr) && mr.kind == json::Value::Array)
            for (const auto &m : mr.arr)
                if (str_eq(m, "type", "sentence_transformers.models.Normalize")) normalize = 1;
        cfg.normalize_embeddings = normalize;
    }
    meta.clear();
    if (read_file(dir + "/tokenizer_config.json", meta)) {
        json::Value tr;
        if (json::parse(meta, tr)) {
            int add = get_bool(tr, "add_eos_token");
            if (add < 0) {
                err = "invalid add_eos_token metadata";
                return false;
            }
            if (add) cfg.append_terminal_token = add == 2;
        }
    }

    if (cfg.hidden_size <= 0 || cfg.n_layers <= 0 || cfg.n_heads <= 0 || cfg.n_kv_heads <= 0 ||
        cfg.head_dim <= 0 || cfg.intermediate_size <= 0 || cfg.vocab_size <= 0 || cfg.q_dim <= 0 ||
        cfg.kv_dim <= 0 || (cfg.head_dim & 1) || cfg.n_heads % cfg.n_kv_heads != 0 ||
        !std::isfinite(cfg.rms_norm_eps) || cfg.rms_norm_eps <= 0.0f ||
        !std::isfinite(cfg.rope_theta) || cfg.rope_theta <= 0.0f) {
        err = "invalid config";
        return false;
    }
    if (cfg.n_layers > 64) {
        err = "too many layers";
        return false;
    }
    return true;
}

}  // namespace fb
