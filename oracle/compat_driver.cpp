// Compat check of the per-op Backend boundary -- TEST INFRASTRUCTURE ONLY.
//
// Linked by oracle/Makefile (target `compat`) from the UNMODIFIED reference
// sources (src/ minus main.cpp and runtime/generation_stats.cpp), with
// qwen2_model.cpp and llama_model.cpp compiled against the shim
// oracle/compat/smallm/backend/cpu_backend.h, so Qwen2Model / LlamaModel
// construct smallm::CUDABackend (include/smallm/backend/cuda_backend.h) and
// every Backend call of their forward pass (matmul_quantized, matmul,
// rmsnorm, rope, softmax, silu) runs on the GPU through the C ABI.
//
//   compat_driver <model.gguf> <n_new> "<prompt ids>" <logits.f32>
//       forward over the prompt, then n_new greedy steps (the first maximum,
//       greedy_sampler.cpp:8-14); prints "ids <generated ids...>" and writes
//       the last prompt token's logits to <logits.f32> (raw float32).
//
// Exit status 0 on success, 2 on a caught exception (message on stderr).
#include <cstdio>
#include <cstdlib>
#include <exception>
#include <memory>
#include <sstream>
#include <string>
#include <vector>

#include "smallm/config/common/config.h"
#include "smallm/core/gguf.h"
#include "smallm/model/llama_model.h"
#include "smallm/model/qwen2_model.h"

namespace {

uint32_t first_max(const std::vector<float>& v) {
    uint32_t best = 0;
    for (uint32_t i = 1; i < v.size(); ++i)
        if (v[i] > v[best]) best = i;
    return best;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc != 5) {
        std::fprintf(stderr, "usage: compat_driver <gguf> <n_new> <prompt ids> <logits.f32>\n");
        return 1;
    }
    try {
        smallm::GGUFModel g = smallm::load_gguf(argv[1]);
        const std::string arch = smallm::read_config(g)->architecture;
        std::unique_ptr<smallm::Model> model;
        if (arch == "qwen2") model = std::make_unique<smallm::Qwen2Model>(std::move(g));
        else model = std::make_unique<smallm::LlamaModel>(std::move(g));
        std::vector<uint32_t> prompt;
        {
            std::istringstream in(argv[3]);
            unsigned long v;
            while (in >> v) prompt.push_back(static_cast<uint32_t>(v));
        }
        std::vector<float> logits;
        uint32_t pos = 0;
        for (uint32_t t : prompt) logits = model->forward(t, pos++);
        if (std::FILE* f = std::fopen(argv[4], "wb")) {
            std::fwrite(logits.data(), sizeof(float), logits.size(), f);
            std::fclose(f);
        } else {
            throw std::runtime_error(std::string("cannot write ") + argv[4]);
        }
        const uint32_t n = (uint32_t)std::strtoul(argv[2], nullptr, 10);
        std::string out = "ids";
        for (uint32_t i = 0; i < n; ++i) {
            const uint32_t next = first_max(logits);
            out += " " + std::to_string(next);
            logits = model->forward(next, pos++);
        }
        std::printf("%s\n", out.c_str());
        return 0;
    } catch (const std::exception& e) {
        std::fprintf(stderr, "error: %s\n", e.what());
        return 2;
    }
}
