// C-ABI harness over the UNMODIFIED smallm-engine sources -- TEST
// INFRASTRUCTURE ONLY.
//
// Compiled by oracle/Makefile together with the reference's own src/**/*.cpp
// (minus main.cpp and the stray runtime/generation_stats.cpp) into
// oracle/_ref/libsmallm_ref.so.  Tests use it to pin the C restatement
// (oracle/oracle.c) and to generate golden fixtures; the benchmark's
// reference arm times the reference's own decode loop through it.  The
// product never links it.
//
// Every entry point returns 0 on success and -1 on a caught C++ exception,
// whose message is kept for ref_last_error().
#include "smallm/backend/cpu_backend.h"
#include "smallm/config/common/config.h"
#include "smallm/core/common/quant_common.h"
#include "smallm/core/gguf.h"
#include "smallm/core/ops.h"
#include "smallm/core/tensor.h"
#include "smallm/model/llama_model.h"
#include "smallm/model/qwen2_model.h"
#include "smallm/runtime/generator.h"
#include "smallm/runtime/sampler/greedy_sampler.h"
#include "smallm/runtime/sampler/temperature_sampler.h"
#include "smallm/runtime/sampler/top_k_sampler.h"
#include "smallm/runtime/sampler/top_p_sampler.h"

#include <chrono>
#include <cstring>
#include <memory>
#include <sstream>
#include <string>
#include <vector>

namespace {

thread_local std::string g_err;

template <typename F>
int guarded(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

// A token-id "tokenizer" so the reference Generator can run unchanged:
// text is whitespace-separated decimal ids, decode prints ids the same way.
class IdTokenizer : public smallm::Tokenizer {
public:
    IdTokenizer(uint32_t v, int32_t eos) : v_(v), eos_(eos) {}
    std::vector<uint32_t> encode(const std::string& text) const override {
        std::vector<uint32_t> out;
        std::istringstream in(text);
        uint32_t id;
        while (in >> id) out.push_back(id);
        return out;
    }
    std::string decode(const std::vector<uint32_t>& ids) const override {
        std::string s;
        for (uint32_t id : ids) s += std::to_string(id) + " ";
        return s;
    }
    uint32_t vocab_size() const override { return v_; }
    int32_t bos_id() const override { return -1; }
    int32_t eos_id() const override { return eos_; }

private:
    uint32_t v_;
    int32_t eos_;
};

struct RefModel {
    std::unique_ptr<smallm::Model> model;
};

struct RefSampler {
    std::unique_ptr<smallm::Sampler> s;
};

// A GGUFModel that views a caller buffer; the mapping pointer is cleared
// before destruction so ~GGUFModel does not munmap memory it does not own.
struct BorrowedGGUF {
    smallm::GGUFModel m;
    ~BorrowedGGUF() { m.mapping = nullptr; }
};

}  // namespace

extern "C" {

const char* ref_last_error() { return g_err.c_str(); }

float ref_f16_to_f32(uint16_t h) { return smallm::f16_to_f32(h); }

// include/smallm/core/ops.h:18-19 -> src/core/ops.cpp:97-300
int ref_matmul_quantized(const uint8_t* W, uint32_t type, const float* x, uint32_t rows,
                         uint32_t cols, float* y) {
    return guarded([&] { smallm::ops::matmul_quantized(W, type, x, rows, cols, y); });
}

int ref_rmsnorm(const float* x, const float* w, uint32_t n, float eps, float* y) {
    return guarded([&] { smallm::ops::rmsnorm(x, w, n, eps, y); });
}
int ref_softmax(float* x, uint32_t n) { return guarded([&] { smallm::ops::softmax(x, n); }); }
int ref_silu(float* x, uint32_t n) { return guarded([&] { smallm::ops::silu(x, n); }); }
int ref_rope(float* x, uint32_t nh, uint32_t hd, uint32_t pos, float base) {
    return guarded([&] { smallm::ops::rope(x, nh, hd, pos, base); });
}
float ref_dot(const float* a, const float* b, uint32_t n) { return smallm::ops::dot(a, b, n); }
int ref_axpy(float* y, const float* v, float s, uint32_t n) {
    return guarded([&] { smallm::ops::axpy(y, v, s, n); });
}
int ref_mul(float* y, const float* v, uint32_t n) {
    return guarded([&] { smallm::ops::mul(y, v, n); });
}

// src/core/tensor.cpp:115-138 on raw block bytes: wraps them as a one-tensor
// GGUFModel (no file) and calls the reference dequantize_tensor.
int ref_dequantize(uint32_t type, const uint8_t* src, uint64_t count, float* out) {
    return guarded([&] {
        BorrowedGGUF g;
        g.m.mapping = src;
        g.m.tensor_data_offset = 0;
        smallm::GGUFTensorInfo t;
        t.name = "t";
        t.dims = {count};
        t.type = type;
        t.offset = 0;
        g.m.tensors.push_back(t);
        smallm::Tensor r = smallm::dequantize_tensor(g.m, "t");
        std::memcpy(out, r.data.data(), count * sizeof(float));
    });
}

// src/core/gguf.cpp:116-183 + src/config/common/config.cpp:14-21 dispatch.
void* ref_model_load(const char* path) {
    RefModel* rm = nullptr;
    int rc = guarded([&] {
        smallm::GGUFModel g = smallm::load_gguf(path);
        std::unique_ptr<smallm::ModelConfig> cfg = smallm::read_config(g);
        auto out = std::make_unique<RefModel>();
        if (cfg->architecture == "qwen2")
            out->model = std::make_unique<smallm::Qwen2Model>(std::move(g));
        else
            out->model = std::make_unique<smallm::LlamaModel>(std::move(g));
        rm = out.release();
    });
    return rc == 0 ? rm : nullptr;
}

void ref_model_free(void* h) { delete static_cast<RefModel*>(h); }

// fills cfg[0..9] = n_layers, embd, ffn, n_heads, n_kv_heads, vocab,
// context_length, head_dim, bits(rope_base), bits(rms_eps)
int ref_model_config(void* h, uint32_t* cfg) {
    return guarded([&] {
        const auto& c = static_cast<RefModel*>(h)->model->config();
        cfg[0] = c.n_layers; cfg[1] = c.embd_dim; cfg[2] = c.ffn_dim; cfg[3] = c.n_heads;
        cfg[4] = c.n_kv_heads; cfg[5] = c.vocab_size; cfg[6] = c.context_length;
        cfg[7] = c.head_dim();
        std::memcpy(&cfg[8], &c.rope_freq_base, 4);
        std::memcpy(&cfg[9], &c.rms_eps, 4);
    });
}

// include/smallm/model/common/model.h:22 Model::forward(token, pos) -> logits
int ref_model_forward(void* h, uint32_t token, uint32_t pos, float* logits) {
    return guarded([&] {
        std::vector<float> l = static_cast<RefModel*>(h)->model->forward(token, pos);
        std::memcpy(logits, l.data(), l.size() * sizeof(float));
    });
}

int ref_model_reset(void* h) { return guarded([&] { static_cast<RefModel*>(h)->model->reset_cache(); }); }
int ref_model_truncate(void* h, uint32_t n) {
    return guarded([&] { static_cast<RefModel*>(h)->model->truncate_cache(n); });
}
uint32_t ref_model_cached_length(void* h) { return static_cast<RefModel*>(h)->model->cached_length(); }

// kind: 0 greedy, 1 temperature(temp), 2 top-k(k, temp), 3 top-p(p, temp)
void* ref_sampler_new(int kind, uint32_t k, float p, float temp, uint64_t seed) {
    auto s = std::make_unique<RefSampler>();
    switch (kind) {
        case 0: s->s = std::make_unique<smallm::GreedySampler>(); break;
        case 1: s->s = std::make_unique<smallm::TemperatureSampler>(temp, seed); break;
        case 2: s->s = std::make_unique<smallm::TopKSampler>(k, temp, seed); break;
        case 3: s->s = std::make_unique<smallm::TopPSampler>(p, temp, seed); break;
        default: return nullptr;
    }
    return s.release();
}
void ref_sampler_free(void* s) { delete static_cast<RefSampler*>(s); }
int ref_sampler_sample(void* s, const float* logits, uint32_t n, uint32_t* out) {
    return guarded([&] {
        std::vector<float> l(logits, logits + n);
        *out = static_cast<RefSampler*>(s)->s->sample(l);
    });
}

// Runs the reference Generator (src/runtime/generator.cpp:22-72) unchanged:
// prompt ids -> up to max_new ids (EOS stop if eos >= 0).  stats[0..5] =
// prompt, reused, prefill, generated tokens, prefill_ms, decode_ms.
struct RefGen {
    IdTokenizer tok;
    std::unique_ptr<smallm::Generator> gen;
    RefGen(smallm::Model& m, smallm::Sampler& s, uint32_t v, int32_t eos) : tok(v, eos) {
        gen = std::make_unique<smallm::Generator>(m, tok, s);
    }
};
void* ref_generator_new(void* model, void* sampler, int32_t eos) {
    auto* m = static_cast<RefModel*>(model);
    return new RefGen(*m->model, *static_cast<RefSampler*>(sampler)->s,
                      m->model->config().vocab_size, eos);
}
void ref_generator_free(void* g) { delete static_cast<RefGen*>(g); }
int ref_generate(void* g, const uint32_t* prompt, uint32_t n, uint32_t max_new, uint32_t* out,
                 uint32_t* n_out, double* stats) {
    return guarded([&] {
        std::string text;
        for (uint32_t i = 0; i < n; ++i) text += std::to_string(prompt[i]) + " ";
        auto* rg = static_cast<RefGen*>(g);
        std::string res = rg->gen->generate(text, max_new);
        std::vector<uint32_t> ids = rg->tok.encode(res);
        for (size_t i = 0; i < ids.size(); ++i) out[i] = ids[i];
        *n_out = static_cast<uint32_t>(ids.size());
        const auto& s = rg->gen->last_stats();
        stats[0] = s.prompt_tokens; stats[1] = s.reused_tokens; stats[2] = s.prefill_tokens;
        stats[3] = s.generated_tokens; stats[4] = s.prefill_ms; stats[5] = s.decode_ms;
    });
}

// Greedy decode timed like generator.cpp:57-68 (steady_clock around the
// decode loop only): prompt prefill untimed, then `steps` forward+argmax
// steps.  ids[0..steps) receives the generated ids; *ms the decode time.
// The reference's decode loop (generator.cpp:47-67): the prompt through
// Model::forward token by token, then greedy steps (GreedySampler).  The
// first `warmup` greedy steps run untimed; the next `steps` are timed with
// steady_clock around the loop, as the reference's Generator times it.
// ids receives all warmup + steps greedy ids.
int ref_decode_timed(void* h, const uint32_t* prompt, uint32_t n, uint32_t warmup, uint32_t steps, uint32_t* ids,
                     double* ms) {
    return guarded([&] {
        auto& m = *static_cast<RefModel*>(h)->model;
        smallm::GreedySampler greedy;
        m.reset_cache();
        std::vector<float> logits;
        uint32_t pos = 0;
        for (uint32_t i = 0; i < n; ++i) logits = m.forward(prompt[i], pos++);
        for (uint32_t s = 0; s < warmup; ++s) {
            uint32_t next = greedy.sample(logits);
            ids[s] = next;
            logits = m.forward(next, pos++);
        }
        auto t0 = std::chrono::steady_clock::now();
        for (uint32_t s = 0; s < steps; ++s) {
            uint32_t next = greedy.sample(logits);
            ids[warmup + s] = next;
            logits = m.forward(next, pos++);
        }
        *ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    });
}

}  // extern "C"
