// QwenModel / QwenForward over libqwen_cuda, plus the host-side C entry points that
// need the C++ loaders (qwc_load_config, qwc_create_from_dir).
#include "qwen_model.h"

#include <iostream>

#include "capi_bridge.h"
#include "qwen_cuda.h"
#include "qwen_forward.h"

// ---------------------------------------------------------------- QwenModel
QwenModel::QwenModel(SafeTensors& weights, const ModelConfig& cfg, int max_context)
    : QwenModel(weights, cfg, max_context, 0, QWC_DTYPE_F32) {}

QwenModel::QwenModel(SafeTensors& weights, const ModelConfig& cfg, int max_context, int device, int kv_dtype)
    : cfg_(cfg), max_context_(max_context) {
    qwc_config c;
    qwh::to_c(cfg_, c);
    std::vector<std::string> names;
    std::vector<qwc_tensor> tensors;
    qwh::tensor_table(weights, names, tensors);
    int rc = qwc_create(&c, tensors.data(), (int)tensors.size(), max_context, kv_dtype, device, &h_);
    if (rc != QWC_OK) {
        err_ = qwc_last_error(nullptr);
        std::cerr << (rc == QWC_E_MISSING ? "" : "[qwen] ") << err_ << "\n";
        ok_ = false;
        h_ = nullptr;
        return;
    }
    ok_ = true;
    logits_.assign((size_t)cfg_.vocab_size, 0.0f);
    qwc_budget b{};
    qwc_get_budget(h_, &b);
    budget_ = qwh::from_c(b);
    std::cout << "[qwen] device arenas planned (max_context=" << max_context_ << "):\n"
              << "   weights (bf16):  " << budget_.weight_bytes / (1024 * 1024) << " MB\n"
              << "   gdn_state:       " << budget_.gdn_state_bytes / 1024 << " KB\n"
              << "   gdn_conv_state:  " << budget_.gdn_conv_bytes / 1024 << " KB\n"
              << "   kv_cache:        " << budget_.kv_cache_bytes / 1024 << " KB\n"
              << "   scratch+step:    " << budget_.activation_bytes / 1024 << " KB\n"
              << "   TOTAL (ex-file): " << budget_.total() / (1024 * 1024) << " MB\n";
}

QwenModel::~QwenModel() { qwc_destroy(h_); }

void QwenModel::reset() {
    if (h_ && qwc_reset(h_) != QWC_OK) err_ = qwc_last_error(h_);
}

int QwenModel::position() const { return h_ ? qwc_position(h_) : 0; }

const std::vector<float>& QwenModel::step(int token_id) {
    if (!h_) return logits_;
    if (qwc_step(h_, token_id, logits_.data(), &last_argmax_) != QWC_OK) {
        err_ = qwc_last_error(h_);
        std::cerr << "[qwen] step failed: " << err_ << "\n";
    }
    return logits_;
}

std::vector<int> QwenModel::generate_greedy(const std::vector<int>& prompt, int n_new) {
    std::vector<int> out;
    if (!h_ || prompt.empty() || n_new <= 0) {
        if (h_) reset();
        return out;
    }
    out.resize((size_t)n_new);
    if (qwc_generate_greedy(h_, prompt.data(), (int)prompt.size(), n_new, out.data()) != QWC_OK) {
        err_ = qwc_last_error(h_);
        std::cerr << "[qwen] generate_greedy failed: " << err_ << "\n";
        out.clear();
    }
    return out;
}

// ---------------------------------------------------------------- QwenForward
QwenForward::~QwenForward() { qwc_destroy(h_); }

bool QwenForward::prefill(const std::vector<int>& ids, std::vector<float>& logits_out) {
    const int T = (int)ids.size();
    if (T == 0) {
        logits_out.clear();
        return true;
    }
    if (!h_ || h_ctx_ < T) {
        qwc_destroy(h_);
        h_ = nullptr;
        qwc_config c;
        qwh::to_c(cfg_, c);
        std::vector<std::string> names;
        std::vector<qwc_tensor> tensors;
        qwh::tensor_table(w_, names, tensors);
        const int ctx = T < 4096 ? 4096 : T;
        if (qwc_create(&c, tensors.data(), (int)tensors.size(), ctx, QWC_DTYPE_F32, 0, &h_) != QWC_OK) {
            std::cerr << "[qwen] " << qwc_last_error(nullptr) << "\n";
            h_ = nullptr;
            return false;
        }
        h_ctx_ = ctx;
    }
    logits_out.assign((size_t)T * cfg_.vocab_size, 0.0f);
    if (qwc_forward_logits(h_, ids.data(), T, logits_out.data(), 0) != QWC_OK) {
        std::cerr << "[qwen] prefill failed: " << qwc_last_error(h_) << "\n";
        return false;
    }
    return true;
}

// ---------------------------------------------------------------- C entry points
namespace qwc {
void set_api_error(const char* msg);  // engine.cu: the message qwc_last_error(nullptr) returns
}

extern "C" int qwc_load_config(const char* path, qwc_config* out) {
    if (!path || !out) {
        qwc::set_api_error("qwc_load_config: null argument");
        return QWC_E_INVALID;
    }
    ModelConfig m;
    bool ok = load_model_config(path, m);
    qwh::to_c(m, *out);  // the defaults when the file cannot be read, as the reference does
    if (!ok) qwc::set_api_error((std::string("qwc_load_config: cannot read ") + path).c_str());
    return ok ? QWC_OK : QWC_E_IO;
}

static int create_from_dir(const char* model_dir, int max_context, int kv_dtype, int device, int rank, int world,
                           const void* unique_id, qwc_handle** out, const char* who) {
    if (!model_dir || !out) {
        qwc::set_api_error((std::string(who) + ": null argument").c_str());
        return QWC_E_INVALID;
    }
    *out = nullptr;
    const std::string dir(model_dir);
    ModelConfig m;
    if (!load_model_config(dir + "/config.json", m)) {
        qwc::set_api_error((std::string(who) + ": cannot read " + dir + "/config.json").c_str());
        return QWC_E_IO;
    }
    SafeTensors st;
    if (!st.load_model(dir)) {
        qwc::set_api_error((std::string(who) + ": cannot load the safetensors shards of " + dir).c_str());
        return QWC_E_IO;
    }
    qwc_config c;
    qwh::to_c(m, c);
    std::vector<std::string> names;
    std::vector<qwc_tensor> tensors;
    qwh::tensor_table(st, names, tensors);
    if (world == 1) return qwc_create(&c, tensors.data(), (int)tensors.size(), max_context, kv_dtype, device, out);
    return qwc_create_tp(&c, tensors.data(), (int)tensors.size(), max_context, kv_dtype, device, rank, world,
                         unique_id, out);
}

extern "C" int qwc_create_from_dir(const char* model_dir, int max_context, int kv_dtype, int device, qwc_handle** out) {
    return create_from_dir(model_dir, max_context, kv_dtype, device, 0, 1, nullptr, out, "qwc_create_from_dir");
}

extern "C" int qwc_create_from_dir_tp(const char* model_dir, int max_context, int kv_dtype, int device, int rank,
                                      int world, const void* unique_id, qwc_handle** out) {
    return create_from_dir(model_dir, max_context, kv_dtype, device, rank, world, unique_id, out,
                           "qwc_create_from_dir_tp");
}
