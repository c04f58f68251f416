// Minimal JSON reader for model metadata (config.json, 1_Pooling/config.json,
// modules.json, tokenizer_config.json) and safetensors headers.  Supports the
// full JSON grammar except \u escapes beyond the BMP (kept as-is).
#pragma once

#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace fb {
namespace json {

struct Value {
    enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
    bool b = false;
    double num = 0.0;
    std::string str;
    std::vector<Value> arr;
    std::vector<std::pair<std::string, Value>> obj;

    const Value *get(const char *key) const {
        if (kind != Object) return nullptr;
        for (const auto &kv : obj)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
    bool is_num() const { return kind == Number; }
};

class Parser {
  public:
    Parser(const char *s, size_t n) : p_(s), end_(s + n) {}

    bool parse(Value &out) {
        ws();
        if (!value(out)) return false;
        ws();
        return true;
    }

  private:
    const char *p_;
    const char *end_;

    void ws() {
        while (p_ < end_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\r' || *p_ == '\t')) ++p_;
    }
    bool lit(const char *w) {
        size_t n = strlen(w);
        if ((size_t)(end_ - p_) < n || strncmp(p_, w, n) != 0) return false;
        p_ += n;
        return true;
    }
    bool string(std::string &s) {
        if (p_ >= end_ || *p_ != '"') return false;
        ++p_;
        while (p_ < end_ && *p_ != '"') {
            if (*p_ == '\\') {
                ++p_;
                if (p_ >= end_) return false;
                switch (*p_) {
                case 'n': s += '\n'; break;
                case 't': s += '\t'; break;
                case 'r': s += '\r'; break;
                case 'b': s += '\b'; break;
                case 'f': s += '\f'; break;
                case 'u': {
                    if (end_ - p_ < 5) return false;
                    unsigned cp = (unsigned)strtoul(std::string(p_ + 1, 4).c_str(), nullptr, 16);
                    if (cp < 0x80) {
                        s += (char)cp;
                    } else if (cp < 0x800) {
                        s += (char)(0xC0 | (cp >> 6));
                        s += (char)(0x80 | (cp & 0x3F));
                    } else {
                        s += (char)(0xE0 | (cp >> 12));
                        s += (char)(0x80 | ((cp >> 6) & 0x3F));
                        s += (char)(0x80 | (cp & 0x3F));
                    }
                    p_ += 4;
                    break;
                }
                default: s += *p_; break;
                }
                ++p_;
            } else {
                s += *p_++;
            }
        }
        if (p_ >= end_) return false;
        ++p_;
        return true;
    }
    bool value(Value &v) {
        ws();
        if (p_ >= end_) return false;
        char c = *p_;
        if (c == '{') {
            v.kind = Value::Object;
            ++p_;
            ws();
            if (p_ < end_ && *p_ == '}') {
                ++p_;
                return true;
            }
            while (true) {
                ws();
                std::string k;
                if (!string(k)) return false;
                ws();
                if (p_ >= end_ || *p_ != ':') return false;
                ++p_;
                Value child;
                if (!value(child)) return false;
                v.obj.emplace_back(std::move(k), std::move(child));
                ws();
                if (p_ < end_ && *p_ == ',') {
                    ++p_;
                    continue;
                }
                if (p_ < end_ && *p_ == '}') {
                    ++p_;
                    return true;
                }
                return false;
            }
        }
        if (c == '[') {
            v.kind = Value::Array;
            ++p_;
            ws();
            if (p_ < end_ && *p_ == ']') {
                ++p_;
                return true;
            }
            while (true) {
                Value child;
                if (!value(child)) return false;
                v.arr.push_back(std::move(child));
                ws();
                if (p_ < end_ && *p_ == ',') {
                    ++p_;
                    continue;
                }
                if (p_ < end_ && *p_ == ']') {
                    ++p_;
                    return true;
                }
                return false;
            }
        }
        if (c == '"') {
            v.kind = Value::String;
            return string(v.str);
        }
        if (lit("true")) {
            v.kind = Value::Bool;
            v.b = true;
            return true;
        }
        if (lit("false")) {
            v.kind = Value::Bool;
            v.b = false;
            return true;
        }
        if (lit("null")) {
            v.kind = Value::Null;
            return true;
        }
        char *e = nullptr;
        std::string tmp(p_, (size_t)(end_ - p_ < 64 ? end_ - p_ : 64));
        double d = strtod(tmp.c_str(), &e);
        if (e == tmp.c_str()) return false;
        v.kind = Value::Number;
        v.num = d;
        p_ += (e - tmp.c_str());
        return true;
    }
};

inline bool parse(const std::string &text, Value &out) {
    Parser ps(text.data(), text.size());
    return ps.parse(out);
}

}  // namespace json
}  // namespace fb
