// Non-owning view of a checkpoint tensor in host memory, bf16 or fp32
// (include/weight_view.h:7-12 of the reference).
#pragma once
#include <cstdint>

struct WeightView {
    const uint16_t* bf16 = nullptr;
    const float* f32 = nullptr;
    int64_t numel = 0;
    bool ok() const { return bf16 != nullptr || f32 != nullptr; }
};
