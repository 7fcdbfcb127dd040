// SafeTensors: the Hugging Face .safetensors reader with the reference's interface
// (include/safetensors_loader.h:24-66). Files are memory-mapped rather than read into
// heap buffers; view() and get_row_f32() read the mapping in place, get_f32() converts
// once and caches, as in the reference.
#pragma once
#include <cstdint>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>
#include "weight_view.h"

class SafeTensors {
public:
    struct Entry {
        std::string dtype;  // "BF16" or "F32"
        std::vector<int64_t> shape;
        int shard = 0;
        size_t abs_offset = 0;
        size_t nbytes = 0;
        int64_t numel() const;
    };

    SafeTensors() = default;
    ~SafeTensors();
    SafeTensors(const SafeTensors&) = delete;
    SafeTensors& operator=(const SafeTensors&) = delete;

    // Every *.safetensors file of model_dir, in sorted name order.
    bool load_model(const std::string& model_dir);
    bool load(const std::string& path);

    const Entry* find(const std::string& name) const;
    bool has(const std::string& name) const { return find(name) != nullptr; }
    const float* get_f32(const std::string& name, int64_t* out_numel = nullptr);
    WeightView view(const std::string& name) const;
    bool get_row_f32(const std::string& name, int64_t row, float* dst) const;
    const std::unordered_map<std::string, Entry>& entries() const { return entries_; }

private:
    struct Shard {
        void* base = nullptr;
        size_t size = 0;
    };
    bool parse_shard(const std::string& path);
    void clear();
    const uint8_t* data_of(const Entry& e) const {
        return static_cast<const uint8_t*>(shards_[e.shard].base) + e.abs_offset;
    }
    std::vector<Shard> shards_;
    std::unordered_map<std::string, Entry> entries_;
    std::unordered_map<std::string, std::vector<float>> f32_cache_;
};

// Exact bf16 -> fp32 widening.
inline float bf16_to_f32(uint16_t h) {
    uint32_t bits = (uint32_t)h << 16;
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}
