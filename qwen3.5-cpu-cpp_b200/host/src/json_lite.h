// A small JSON reader (objects, arrays, strings, numbers, true/false/null) used for
// config.json and safetensors headers. Values keep document order.
#pragma once
#include <cstdint>
#include <memory>
#include <string>
#include <utility>
#include <vector>

namespace qwh {

struct JValue {
    enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
    bool b = false;
    double num = 0.0;
    std::string numtext;  // digits as written (exact int64 parsing)
    std::string str;
    std::vector<JValue> arr;
    std::vector<std::pair<std::string, JValue>> obj;

    const JValue* get(const std::string& key) const {
        if (kind != OBJ) return nullptr;
        for (const auto& kv : obj)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
    // First value named `key` in document order, searching nested objects depth-first.
    const JValue* find_deep(const std::string& key) const {
        if (kind == OBJ) {
            for (const auto& kv : obj) {
                if (kv.first == key) return &kv.second;
                if (const JValue* r = kv.second.find_deep(key)) return r;
            }
        } else if (kind == ARR) {
            for (const auto& v : arr)
                if (const JValue* r = v.find_deep(key)) return r;
        }
        return nullptr;
    }
    int64_t as_i64() const;
};

// Parses text[0, n). Returns false (and sets *err) on malformed input.
bool parse_json(const char* text, size_t n, JValue& out, std::string* err);

}  // namespace qwh
