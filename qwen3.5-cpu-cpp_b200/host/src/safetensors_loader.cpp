// SafeTensors over read-only memory maps. Same contract as the reference's
// src/safetensors_loader.cpp:125-298: all *.safetensors shards of a directory in sorted
// order, header = u64 length + JSON {name: {dtype, shape, data_offsets}}, every tensor
// bounds-checked against its file, BF16 widened exactly to fp32 on demand.
#include "safetensors_loader.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <filesystem>
#include <iostream>
#include <system_error>

#include "json_lite.h"

using qwh::JValue;

int64_t SafeTensors::Entry::numel() const {
    int64_t n = 1;
    for (int64_t d : shape) n *= d;
    return shape.empty() ? 0 : n;
}

SafeTensors::~SafeTensors() { clear(); }

void SafeTensors::clear() {
    for (auto& s : shards_)
        if (s.base && s.size) munmap(s.base, s.size);
    shards_.clear();
    entries_.clear();
    f32_cache_.clear();
}

bool SafeTensors::parse_shard(const std::string& path) {
    int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) {
        std::cerr << "[safetensors] cannot open '" << path << "'\n";
        return false;
    }
    struct stat stt;
    if (fstat(fd, &stt) != 0 || stt.st_size < 8) {
        ::close(fd);
        std::cerr << "[safetensors] file too small: '" << path << "'\n";
        return false;
    }
    const size_t size = (size_t)stt.st_size;
    void* base = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (base == MAP_FAILED) {
        std::cerr << "[safetensors] mmap failed: '" << path << "'\n";
        return false;
    }
    const int shard_idx = (int)shards_.size();
    shards_.push_back(Shard{base, size});
    const uint8_t* data = static_cast<const uint8_t*>(base);
    uint64_t header_len = 0;
    std::memcpy(&header_len, data, 8);
    if (header_len > size - 8) {
        std::cerr << "[safetensors] header length exceeds file: '" << path << "'\n";
        return false;
    }
    JValue hdr;
    std::string err;
    if (!qwh::parse_json(reinterpret_cast<const char*>(data) + 8, (size_t)header_len, hdr, &err) ||
        hdr.kind != JValue::OBJ) {
        std::cerr << "[safetensors] header parse error in '" << path << "': " << err << "\n";
        return false;
    }
    const size_t data_base = 8 + (size_t)header_len;
    for (const auto& kv : hdr.obj) {
        if (kv.first == "__metadata__") continue;
        const JValue& t = kv.second;
        const JValue* dt = t.get("dtype");
        const JValue* sh = t.get("shape");
        const JValue* off = t.get("data_offsets");
        if (!dt || dt->kind != JValue::STR || !sh || sh->kind != JValue::ARR || !off || off->kind != JValue::ARR ||
            off->arr.size() != 2) {
            std::cerr << "[safetensors] malformed entry '" << kv.first << "'\n";
            return false;
        }
        Entry e;
        e.dtype = dt->str;
        for (const auto& d : sh->arr) e.shape.push_back(d.as_i64());
        const int64_t a = off->arr[0].as_i64(), b = off->arr[1].as_i64();
        if (a < 0 || b < a) {
            std::cerr << "[safetensors] tensor '" << kv.first << "' has bad offsets\n";
            return false;
        }
        e.shard = shard_idx;
        e.abs_offset = data_base + (size_t)a;
        e.nbytes = (size_t)(b - a);
        if (e.abs_offset + e.nbytes > size) {
            std::cerr << "[safetensors] tensor '" << kv.first << "' out of range\n";
            return false;
        }
        const size_t esz = e.dtype == "F32" ? 4 : (e.dtype == "BF16" || e.dtype == "F16") ? 2 : 0;
        if (esz && (size_t)e.numel() * esz != e.nbytes) {
            std::cerr << "[safetensors] tensor '" << kv.first << "' size does not match its shape\n";
            return false;
        }
        entries_[kv.first] = std::move(e);
    }
    std::cout << "[safetensors] shard '" << path << "': " << (size / (1024 * 1024)) << " MB\n";
    return true;
}

bool SafeTensors::load(const std::string& path) {
    clear();
    return parse_shard(path);
}

bool SafeTensors::load_model(const std::string& model_dir) {
    clear();
    std::vector<std::string> files;
    std::error_code ec;
    for (const auto& de : std::filesystem::directory_iterator(model_dir, ec))
        if (de.path().extension() == ".safetensors") files.push_back(de.path().string());
    if (files.empty()) {
        std::cerr << "[safetensors] no .safetensors files in '" << model_dir << "'\n";
        return false;
    }
    std::sort(files.begin(), files.end());
    for (const auto& f : files)
        if (!parse_shard(f)) return false;
    std::cout << "[safetensors] " << files.size() << " shard(s), " << entries_.size() << " tensors\n";
    return true;
}

const SafeTensors::Entry* SafeTensors::find(const std::string& name) const {
    auto it = entries_.find(name);
    return it == entries_.end() ? nullptr : &it->second;
}

WeightView SafeTensors::view(const std::string& name) const {
    WeightView v;
    const Entry* e = find(name);
    if (!e) return v;
    v.numel = e->numel();
    if (e->dtype == "BF16") v.bf16 = reinterpret_cast<const uint16_t*>(data_of(*e));
    else if (e->dtype == "F32") v.f32 = reinterpret_cast<const float*>(data_of(*e));
    return v;
}

const float* SafeTensors::get_f32(const std::string& name, int64_t* out_numel) {
    auto cit = f32_cache_.find(name);
    if (cit != f32_cache_.end()) {
        if (out_numel) *out_numel = (int64_t)cit->second.size();
        return cit->second.data();
    }
    const Entry* e = find(name);
    if (!e) return nullptr;
    const int64_t n = e->numel();
    std::vector<float> buf((size_t)n);
    const uint8_t* src = data_of(*e);
    if (e->dtype == "F32") {
        std::memcpy(buf.data(), src, (size_t)n * 4);
    } else if (e->dtype == "BF16") {
        const uint16_t* s = reinterpret_cast<const uint16_t*>(src);
        for (int64_t i = 0; i < n; ++i) buf[(size_t)i] = bf16_to_f32(s[i]);
    } else {
        std::cerr << "[safetensors] unsupported dtype " << e->dtype << " for '" << name << "'\n";
        return nullptr;
    }
    auto res = f32_cache_.emplace(name, std::move(buf));
    if (out_numel) *out_numel = (int64_t)res.first->second.size();
    return res.first->second.data();
}

bool SafeTensors::get_row_f32(const std::string& name, int64_t row, float* dst) const {
    const Entry* e = find(name);
    if (!e || e->shape.size() != 2) return false;
    const int64_t rows = e->shape[0], cols = e->shape[1];
    if (row < 0 || row >= rows) return false;
    const uint8_t* base = data_of(*e);
    if (e->dtype == "F32") {
        std::memcpy(dst, reinterpret_cast<const float*>(base) + row * cols, (size_t)cols * 4);
    } else if (e->dtype == "BF16") {
        const uint16_t* s = reinterpret_cast<const uint16_t*>(base) + row * cols;
        for (int64_t i = 0; i < cols; ++i) dst[i] = bf16_to_f32(s[i]);
    } else {
        return false;
    }
    return true;
}
