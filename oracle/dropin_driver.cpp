// Drop-in check of the C++ adapters -- TEST INFRASTRUCTURE ONLY.
//
// Built by oracle/Makefile (target `dropin`) from this file, the UNMODIFIED
// smallm-engine sources (the same set as libsmallm_ref.so: src/ minus
// main.cpp and runtime/generation_stats.cpp) and the adapter headers
// include/smallm/backend/cuda_backend.h and include/smallm/model/cuda_model.h,
// linked against libsmallm_cuda.so.  It shows the adapters compiling against
// the engine's own Backend/Model headers and the engine's own Generator,
// GreedySampler, GGUF loader and config reader driving the CUDA model:
//
//   dropin_driver generate <model.gguf> <n_new> "<ids of prompt 1>" "<ids of prompt 2>"
//       Generator::generate (src/runtime/generator.cpp:22-72) twice, the
//       second prompt sharing a prefix with the first (truncate_cache path);
//       prints one line per call: "ids <reused> <prefilled> <generated ids...>".
//   dropin_driver fastgen <model.gguf> <n_new> "<prompt ids>" <flags>
//       CudaModel::generate_greedy (one-pass prefill, device-chained greedy
//       steps); prints "fast <ids...>".
//   dropin_driver ops <seed>
//       CPUBackend vs CUDABackend on seeded inputs: rmsnorm, softmax, silu,
//       rope, F32 matmul; prints "op <name> <max |diff|> <max |ref|> <bits equal 0/1>".
//
// The prompt is a list of token ids (a whitespace-separated string); the
// tokenizer below maps ids to text and back, so the synthetic GGUF needs no
// vocabulary.  Exit status 0 on success, 2 on a caught exception (the
// message goes to stderr): without a GPU the CUDA classes throw, there is no
// CPU fallback.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <random>
#include <sstream>
#include <string>
#include <vector>

#include "smallm/backend/cpu_backend.h"
#include "smallm/backend/cuda_backend.h"
#include "smallm/model/cuda_model.h"
#include "smallm/runtime/generator.h"
#include "smallm/runtime/sampler/greedy_sampler.h"
#include "smallm/tokenizer/common/tokenizer.h"

namespace {

class IdTokenizer final : public smallm::Tokenizer {
public:
    explicit IdTokenizer(uint32_t vocab) : vocab_(vocab) {}
    std::vector<uint32_t> encode(const std::string& text) const override {
        std::istringstream in(text);
        std::vector<uint32_t> ids;
        unsigned long v;
        while (in >> v) ids.push_back(static_cast<uint32_t>(v));
        return ids;
    }
    std::string decode(const std::vector<uint32_t>& ids) const override {
        std::string s;
        for (uint32_t id : ids) s += " " + std::to_string(id);
        return s;
    }
    uint32_t vocab_size() const override { return vocab_; }
    int32_t bos_id() const override { return -1; }
    int32_t eos_id() const override { return -1; }

private:
    uint32_t vocab_;
};

int generate(const char* path, uint32_t n_new, const char* p1, const char* p2) {
    auto model = smallm::CudaModel::open(path);
    IdTokenizer tok(model->config().vocab_size);
    smallm::GreedySampler sampler;
    smallm::Generator gen(*model, tok, sampler);
    for (const char* p : {p1, p2}) {
        const std::string out = gen.generate(p, n_new);
        const auto& st = gen.last_stats();
        std::printf("ids %u %u%s\n", st.reused_tokens, st.prefill_tokens, out.c_str());
    }
    return 0;
}

int fastgen(const char* path, uint32_t n_new, const char* prompt, uint32_t flags) {
    auto model = smallm::CudaModel::open(path);
    IdTokenizer tok(model->config().vocab_size);
    const auto ids = model->generate_greedy(tok.encode(prompt), 0, n_new, flags);
    std::printf("fast%s\n", tok.decode(ids).c_str());
    return 0;
}

void report(const char* name, const std::vector<float>& ref, const std::vector<float>& got) {
    double diff = 0, mag = 0;
    for (size_t i = 0; i < ref.size(); ++i) {
        diff = std::fmax(diff, std::fabs((double)ref[i] - got[i]));
        mag = std::fmax(mag, std::fabs((double)ref[i]));
    }
    const int same = std::memcmp(ref.data(), got.data(), ref.size() * sizeof(float)) == 0;
    std::printf("op %s %.9g %.9g %d\n", name, diff, mag, same);
}

int ops(unsigned seed) {
    std::mt19937 rng(seed);
    std::normal_distribution<float> nd(0.f, 1.f);
    auto randv = [&](size_t n, float s) {
        std::vector<float> v(n);
        for (auto& x : v) x = nd(rng) * s;
        return v;
    };
    smallm::CPUBackend cpu;
    smallm::CUDABackend gpu;
    const uint32_t n = 4096, rows = 256, cols = 1000, heads = 8, hd = 128;
    {
        const auto x = randv(n, 1.f), w = randv(n, 1.f);
        std::vector<float> a(n), b(n);
        cpu.rmsnorm(x.data(), w.data(), n, 1e-5f, a.data());
        gpu.rmsnorm(x.data(), w.data(), n, 1e-5f, b.data());
        report("rmsnorm", a, b);
    }
    {
        auto a = randv(n, 3.f), b = a;
        cpu.softmax(a.data(), n);
        gpu.softmax(b.data(), n);
        report("softmax", a, b);
    }
    {
        auto a = randv(n, 3.f), b = a;
        cpu.silu(a.data(), n);
        gpu.silu(b.data(), n);
        report("silu", a, b);
    }
    {
        auto a = randv(heads * hd, 1.f), b = a;
        cpu.rope(a.data(), heads, hd, 77, 5e5f);
        gpu.rope(b.data(), heads, hd, 77, 5e5f);
        report("rope", a, b);
    }
    {
        const auto W = randv((size_t)rows * cols, 0.02f), x = randv(cols, 1.f);
        std::vector<float> a(rows), b(rows);
        cpu.matmul(W.data(), x.data(), rows, cols, a.data());
        gpu.matmul(W.data(), x.data(), rows, cols, b.data());
        report("matmul", a, b);
    }
    return 0;
}

}  // namespace

int main(int argc, char** argv) {
    try {
        if (argc == 6 && std::strcmp(argv[1], "generate") == 0)
            return generate(argv[2], (uint32_t)std::strtoul(argv[3], nullptr, 10), argv[4], argv[5]);
        if (argc == 6 && std::strcmp(argv[1], "fastgen") == 0)
            return fastgen(argv[2], (uint32_t)std::strtoul(argv[3], nullptr, 10), argv[4],
                           (uint32_t)std::strtoul(argv[5], nullptr, 10));
        if (argc == 3 && std::strcmp(argv[1], "ops") == 0)
            return ops((unsigned)std::strtoul(argv[2], nullptr, 10));
        std::fprintf(stderr, "usage: dropin_driver generate <gguf> <n_new> <prompt ids> <prompt ids>\n"
                             "       dropin_driver fastgen <gguf> <n_new> <prompt ids> <flags>\n"
                             "       dropin_driver ops <seed>\n");
        return 1;
    } catch (const std::exception& e) {
        std::fprintf(stderr, "error: %s\n", e.what());
        return 2;
    }
}
