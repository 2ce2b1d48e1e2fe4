// smallm::CudaModel -- a device-resident Qwen2 / Llama decoder behind the
// engine's model interface, smallm::Model
// (include/smallm/model/common/model.h:16-43 of smallm-engine), so that the
// engine's Generator and samplers (src/runtime/) drive it unchanged.
// Header-only: it binds the C ABI of smallm_cuda.h (libsmallm_cuda.so) and
// is compiled inside the engine, next to qwen2_model.h, with the engine's
// include directory on the path.
//
// It replaces Qwen2Model(load_gguf(path)) / LlamaModel(...)
// (src/model/qwen2_model.cpp:28-65, llama_model.cpp:17-49): the weights are
// read from the same GGUF file once, kept in HBM, and every forward() is one
// CUDA-graph launch plus the copy of the logits back to the host.  Errors
// are std::runtime_error, as in the reference.
#pragma once

#include <cstdint>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "smallm/config/common/config.h"
#include "smallm/core/gguf.h"
#include "smallm/model/common/model.h"
#include "smallm_cuda.h"

namespace smallm {

class CudaModel final : public Model {
public:
    // cfg: the config the CPU model would get from read_config(load_gguf(path))
    // (src/config/common/config.cpp); max_ctx 0 = the GGUF context_length.
    CudaModel(const std::string& gguf_path, std::unique_ptr<ModelConfig> cfg, int device = 0,
              uint32_t max_ctx = 0)
        : Model(std::move(cfg)) {
        smallm_model_opts o{device, max_ctx, 0, 1, nullptr, 0};
        check(smallm_model_load(gguf_path.c_str(), &o, &m_));
        smallm_model_info info{};
        check(smallm_model_get_info(m_, &info));
        if (info.vocab != config().vocab_size || info.n_layers != config().n_layers ||
            info.embd != config().embd_dim) {
            smallm_model_free(m_);
            m_ = nullptr;
            throw std::runtime_error("CudaModel: the config does not describe " + gguf_path);
        }
    }

    // The config read the way the reference reads it, then the device model.
    static std::unique_ptr<CudaModel> open(const std::string& gguf_path, int device = 0, uint32_t max_ctx = 0) {
        std::unique_ptr<ModelConfig> cfg;
        {
            GGUFModel g = load_gguf(gguf_path);
            cfg = read_config(g);
        }
        return std::make_unique<CudaModel>(gguf_path, std::move(cfg), device, max_ctx);
    }

    ~CudaModel() override {
        if (m_) smallm_model_free(m_);
    }
    CudaModel(const CudaModel&) = delete;
    CudaModel& operator=(const CudaModel&) = delete;

    std::vector<float> forward(uint32_t token_id, uint32_t pos) override {
        std::vector<float> logits(config().vocab_size);
        check(smallm_model_forward(m_, token_id, pos, logits.data(), nullptr));
        cached_length_ = smallm_model_cached_length(m_);
        return logits;
    }
    void reset_cache() override {
        check(smallm_model_reset_cache(m_));
        cached_length_ = 0;
    }
    void truncate_cache(uint32_t n) override {
        check(smallm_model_truncate_cache(m_, n));
        cached_length_ = smallm_model_cached_length(m_);
    }

    // Beyond the reference's Model: the prompt in one pass per layer (the
    // same cache contents as tokens.size() forward calls) -> last logits.
    // The GEMMs run on the backend's tcgen05 tensor-core kernel; flags: 0.
    std::vector<float> prefill(const std::vector<uint32_t>& tokens, uint32_t start_pos, uint32_t flags = 0) {
        std::vector<float> logits(config().vocab_size);
        check(smallm_model_prefill(m_, tokens.data(), static_cast<uint32_t>(tokens.size()), start_pos,
                                   logits.data(), nullptr, flags));
        cached_length_ = smallm_model_cached_length(m_);
        return logits;
    }

    // Beyond the reference's Model: a greedy continuation without a host
    // round trip per token.  `prompt` is prefilled in one pass at positions
    // start_pos.. (flags as prefill()); its greedy id is the first of the n
    // returned ids, and the other n - 1 come from CUDA-graph steps chained on
    // the device, each feeding the previous step's argmax.  The cache then
    // holds start_pos + prompt.size() + n - 1 positions.
    std::vector<uint32_t> generate_greedy(const std::vector<uint32_t>& prompt, uint32_t start_pos, uint32_t n,
                                          uint32_t flags = 0) {
        std::vector<uint32_t> ids(n);
        if (n == 0) return ids;
        uint32_t first = 0;
        check(smallm_model_prefill(m_, prompt.data(), static_cast<uint32_t>(prompt.size()), start_pos, nullptr,
                                   &first, flags));
        ids[0] = first;
        if (n > 1) {
            const uint32_t pos = start_pos + static_cast<uint32_t>(prompt.size());
            check(smallm_model_decode_greedy_async(m_, first, pos, n - 1));
            check(smallm_model_decode_ids(m_, ids.data() + 1, n - 1));
        }
        cached_length_ = smallm_model_cached_length(m_);
        return ids;
    }

    smallm_model* handle() const { return m_; }

private:
    static void check(int rc) {
        if (rc != SMALLM_OK) throw std::runtime_error(std::string("CudaModel: ") + smallm_last_error());
    }
    smallm_model* m_ = nullptr;
};

}  // namespace smallm
