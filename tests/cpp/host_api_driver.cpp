// Test driver for the C++ drop-in API (host/include): a caller written the way the
// reference's main.cpp / server.cpp use QwenModel, QwenForward and SafeTensors, compiled
// against the headers and linked to libqwen_cuda.so. The Python tests run it and compare
// what it prints with the raw checkpoint bytes and with the C ABI.
//
//   host_api_driver st  <model_dir> <tensor> <row> <out.bin>
//       SafeTensors::view / get_f32 / get_row_f32 of one tensor, written to out.bin
//   host_api_driver gen <model_dir> <max_ctx> <n_new> <kv_dtype> <device> <ids...>
//       QwenModel: step() over the prompt, then generate_greedy(); prints one JSON line
//   host_api_driver fwd <model_dir> <out.bin> <ids...>
//       QwenForward::prefill: [T][vocab] logits written to out.bin
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <string>
#include <vector>

#include "model_config.h"
#include "qwen_cuda.h"
#include "qwen_forward.h"
#include "qwen_model.h"
#include "safetensors_loader.h"

namespace {

template <class T>
void put(std::ofstream& f, const T& v) { f.write(reinterpret_cast<const char*>(&v), sizeof(T)); }

int cmd_st(int argc, char** argv) {
    if (argc < 6) return 2;
    SafeTensors st;
    if (!st.load_model(argv[2])) return 3;
    const std::string name = argv[3];
    const long row = std::atol(argv[4]);
    std::ofstream f(argv[5], std::ios::binary);
    const WeightView v = st.view(name);
    put<int64_t>(f, v.numel);
    put<int32_t>(f, v.f32 ? 0 : (v.bf16 ? 1 : 2));
    int64_t n = -1;
    const float* a = st.get_f32(name, &n);
    const float* b = st.get_f32(name, nullptr);
    put<int64_t>(f, n);
    put<int32_t>(f, a != nullptr && a == b);  // the fp32 copy is made once and cached
    if (a) f.write(reinterpret_cast<const char*>(a), n * 4);
    const SafeTensors::Entry* e = st.find(name);
    const int64_t width = (e && e->shape.size() == 2) ? e->shape[1] : 0;
    std::vector<float> r((size_t)(width > 0 ? width : 1));
    const bool row_ok = st.get_row_f32(name, row, r.data());
    put<int32_t>(f, row_ok);
    put<int64_t>(f, width);
    if (row_ok) f.write(reinterpret_cast<const char*>(r.data()), width * 4);
    // a row past the end, a negative row and a missing tensor are refusals
    const bool oob = e && e->shape.size() == 2 && !st.get_row_f32(name, e->shape[0], r.data()) &&
                     !st.get_row_f32(name, -1, r.data());
    const bool missing = !st.view("no.such.tensor").ok() && st.get_f32("no.such.tensor") == nullptr &&
                         !st.get_row_f32("no.such.tensor", 0, r.data()) && !st.has("no.such.tensor");
    put<int32_t>(f, oob);
    put<int32_t>(f, missing);
    return f.good() ? 0 : 4;
}

int cmd_gen(int argc, char** argv) {
    if (argc < 8) return 2;
    const std::string dir = argv[2];
    const int max_ctx = std::atoi(argv[3]), n_new = std::atoi(argv[4]);
    const int kv = std::atoi(argv[5]), dev = std::atoi(argv[6]);
    std::vector<int> prompt;
    for (int i = 7; i < argc; ++i) prompt.push_back(std::atoi(argv[i]));
    ModelConfig cfg;
    if (!load_model_config(dir + "/config.json", cfg)) return 3;
    SafeTensors st;
    if (!st.load_model(dir)) return 3;
    QwenModel m(st, cfg, max_ctx, dev, kv);
    if (!m.ok()) {
        std::printf("{\"ok\": false}\n");
        return 5;
    }
    std::vector<int> step_argmax;
    double sum = 0.0, sq = 0.0;
    for (int t : prompt) {
        const std::vector<float>& lg = m.step(t);
        int best = 0;
        for (size_t i = 1; i < lg.size(); ++i)
            if (lg[i] > lg[best]) best = (int)i;  // strict '>': first index wins ties
        step_argmax.push_back(best);
        sum = 0.0;
        sq = 0.0;
        for (float x : lg) { sum += x; sq += (double)x * x; }
    }
    const int pos_after_prompt = m.position();
    const std::vector<int> gen = m.generate_greedy(prompt, n_new);
    std::printf("{\"ok\": true, \"position\": %d, \"last_sum\": %.9g, \"last_norm\": %.9g, \"step_argmax\": [",
                pos_after_prompt, sum, std::sqrt(sq));
    for (size_t i = 0; i < step_argmax.size(); ++i) std::printf("%s%d", i ? ", " : "", step_argmax[i]);
    std::printf("], \"greedy\": [");
    for (size_t i = 0; i < gen.size(); ++i) std::printf("%s%d", i ? ", " : "", gen[i]);
    std::printf("], \"final_position\": %d, \"weights_mb\": %llu}\n", m.position(),
                (unsigned long long)(m.budget().weight_bytes >> 20));
    return 0;
}

int cmd_fwd(int argc, char** argv) {
    if (argc < 5) return 2;
    const std::string dir = argv[2];
    std::vector<int> ids;
    for (int i = 4; i < argc; ++i) ids.push_back(std::atoi(argv[i]));
    ModelConfig cfg;
    if (!load_model_config(dir + "/config.json", cfg)) return 3;
    SafeTensors st;
    if (!st.load_model(dir)) return 3;
    QwenForward fw(st, cfg);
    std::vector<float> logits;
    if (!fw.prefill(ids, logits)) return 5;
    std::ofstream f(argv[3], std::ios::binary);
    f.write(reinterpret_cast<const char*>(logits.data()), (std::streamsize)(logits.size() * 4));
    return f.good() ? 0 : 4;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc < 2) return 2;
    const std::string c = argv[1];
    if (c == "st") return cmd_st(argc, argv);
    if (c == "gen") return cmd_gen(argc, argv);
    if (c == "fwd") return cmd_fwd(argc, argv);
    return 2;
}
