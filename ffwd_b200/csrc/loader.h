// Host-side model metadata and weight access: config.json and
// sentence-transformers metadata parsing (same rules and defaults as
// libffwd/config.c:96-341) and an mmap'd safetensors reader (single
// model.safetensors or model-XXXXX-of-YYYYY shards, as
// libffwd/safetensors.c:351-467).
#pragma once

#include "ffwd_b200.h"

#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace fb {

enum class DType { F32, BF16, F16, Other };

struct TensorView {
    DType dtype = DType::Other;
    std::vector<int64_t> shape;
    const void *data = nullptr;
    size_t nbytes = 0;
    int64_t numel() const {
        int64_t n = 1;
        for (auto d : shape) n *= d;
        return n;
    }
};

class SafeTensors {
  public:
    ~SafeTensors();
    bool open(const std::string &dir, std::string &err);
    const TensorView *find(const std::string &name) const;
    bool has(const std::string &name) const { return find(name) != nullptr; }

  private:
    struct Map {
        void *base = nullptr;
        size_t size = 0;
    };
    bool open_file(const std::string &path, std::string &err);
    std::vector<Map> maps_;
    std::map<std::string, TensorView> tensors_;
};

// Parse config.json + metadata; returns false with a reason.
bool parse_model_config(const std::string &dir, ffwd_config_t &cfg, std::string &err);

// Tensor -> f32 (widening bf16 / f16 exactly); shape-checked.
bool tensor_to_f32(const TensorView *t, const std::vector<int64_t> &shape, std::vector<float> &out,
                   std::string &err, const std::string &name);

uint16_t f32_to_bf16_rne(float x);
float bf16_to_f32(uint16_t b);
float f16_to_f32(uint16_t h);
// IEEE binary16, round to nearest even (subnormals kept, overflow to inf).
uint16_t f32_to_f16_rne(float x);

}  // namespace fb
