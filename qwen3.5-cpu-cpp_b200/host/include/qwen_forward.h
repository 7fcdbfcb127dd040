// QwenForward: the whole-prompt forward pass with the reference's interface
// (include/qwen_forward.h:18-25): prefill(ids, logits) writes seq x vocab logits and
// leaves no decode state behind. Runs on a B200 through libqwen_cuda; the device copy
// of the weights is made on the first prefill() and reused afterwards.
#pragma once
#include <vector>
#include "model_config.h"
#include "safetensors_loader.h"

struct qwc_handle;

class QwenForward {
public:
    QwenForward(SafeTensors& weights, const ModelConfig& cfg) : w_(weights), cfg_(cfg) {}
    ~QwenForward();
    QwenForward(const QwenForward&) = delete;
    QwenForward& operator=(const QwenForward&) = delete;

    bool prefill(const std::vector<int>& ids, std::vector<float>& logits_out);

private:
    SafeTensors& w_;
    ModelConfig cfg_;
    qwc_handle* h_ = nullptr;
    int h_ctx_ = 0;
};
