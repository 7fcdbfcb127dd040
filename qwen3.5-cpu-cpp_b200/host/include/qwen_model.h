// QwenModel: stateful single-sequence incremental decoder with the reference's interface
// (include/qwen_model.h:21-32), executed on a B200 by libqwen_cuda. All device memory
// (weights, GDN recurrent + conv state, KV cache, scratch) is planned by the memory
// equation and allocated in the constructor; step() replays one captured CUDA graph and
// allocates nothing. The SafeTensors object must outlive the model only for the
// constructor (weights are copied to the device).
#pragma once
#include <string>
#include <vector>
#include "memory_budget.h"
#include "model_config.h"
#include "safetensors_loader.h"

struct qwc_handle;

class QwenModel {
public:
    QwenModel(SafeTensors& weights, const ModelConfig& cfg, int max_context);
    // Not in the reference: the GPU to run on and the KV cache type (QWC_DTYPE_F32, the
    // reference's fp32 cache and the default above, or QWC_DTYPE_BF16).
    QwenModel(SafeTensors& weights, const ModelConfig& cfg, int max_context, int device, int kv_dtype);
    ~QwenModel();
    QwenModel(const QwenModel&) = delete;
    QwenModel& operator=(const QwenModel&) = delete;

    void reset();
    const std::vector<float>& step(int token_id);  // logits [vocab], valid until the next call
    int position() const;
    std::vector<int> generate_greedy(const std::vector<int>& prompt, int n_new);
    const MemoryBudget& budget() const { return budget_; }
    bool ok() const { return ok_; }

    // Not in the reference: the greedy id of the last step() (computed on the device),
    // the C handle for callers that mix both interfaces, and the last error message.
    int last_argmax() const { return last_argmax_; }
    qwc_handle* handle() const { return h_; }
    const std::string& error() const { return err_; }

private:
    ModelConfig cfg_;
    int max_context_;
    bool ok_ = false;
    qwc_handle* h_ = nullptr;
    std::vector<float> logits_;
    MemoryBudget budget_;
    int last_argmax_ = -1;
    std::string err_;
};
