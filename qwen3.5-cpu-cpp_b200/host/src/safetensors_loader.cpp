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

// ---------------------------------------------------------------- element access
// Tensor data stays in the file mapping. Every fp32 read goes through one routine that
// widens a run of elements (fp32 copied, bf16 exact), shared by the cached whole-tensor
// copy and the single-row read.
namespace {
enum class Elem { F32, BF16, Unsupported };

Elem elem_kind(const std::string& dtype) {
    if (dtype == "F32") return Elem::F32;
    if (dtype == "BF16") return Elem::BF16;
    return Elem::Unsupported;
}

// dst[0, count) <- elements [first, first + count) of the tensor whose data starts at base
bool widen_run(const uint8_t* base, Elem kind, int64_t first, int64_t count, float* dst) {
    if (kind == Elem::F32) {
        std::memcpy(dst, base + first * 4, (size_t)count * 4);
        return true;
    }
    if (kind == Elem::BF16) {
        const uint16_t* h = reinterpret_cast<const uint16_t*>(base) + first;
        std::transform(h, h + count, dst, bf16_to_f32);
        return true;
    }
    return false;
}
}  // namespace

WeightView SafeTensors::view(const std::string& name) const {
    WeightView out;
    const Entry* e = find(name);
    if (e == nullptr) return out;  // empty view: no such tensor
    out.numel = e->numel();
    const uint8_t* data = data_of(*e);
    switch (elem_kind(e->dtype)) {
        case Elem::BF16: out.bf16 = reinterpret_cast<const uint16_t*>(data); break;
        case Elem::F32: out.f32 = reinterpret_cast<const float*>(data); break;
        case Elem::Unsupported: break;  // element count only
    }
    return out;
}

const float* SafeTensors::get_f32(const std::string& name, int64_t* out_numel) {
    // One fp32 copy per tensor, made on the first request and kept for the object's lifetime.
    auto hit = f32_cache_.find(name);
    if (hit == f32_cache_.end()) {
        const Entry* e = find(name);
        if (e == nullptr) return nullptr;
        std::vector<float> widened((size_t)e->numel());
        if (!widen_run(data_of(*e), elem_kind(e->dtype), 0, e->numel(), widened.data())) {
            std::cerr << "[safetensors] '" << name << "': no fp32 reading of dtype " << e->dtype << "\n";
            return nullptr;
        }
        hit = f32_cache_.emplace(name, std::move(widened)).first;
    }
    if (out_numel) *out_numel = (int64_t)hit->second.size();
    return hit->second.data();
}

bool SafeTensors::get_row_f32(const std::string& name, int64_t row, float* dst) const {
    // Row `row` of a 2-D tensor, widened in place from the mapping (no cache).
    const Entry* e = find(name);
    if (e == nullptr || e->shape.size() != 2 || row < 0 || row >= e->shape[0]) return false;
    const int64_t width = e->shape[1];
    return widen_run(data_of(*e), elem_kind(e->dtype), row * width, width, dst);
}
