// smallm::CUDABackend -- the B200 backend behind the engine's own compute
// interface, smallm::Backend (include/smallm/backend/common/backend.h:12-38
// of smallm-engine).  Header-only: it binds the C ABI of smallm_cuda.h
// (libsmallm_cuda.so) and is compiled inside the engine, next to
// cpu_backend.h, with the engine's include directory on the path.
//
// Same contract as CPUBackend (src/backend/cpu_backend.cpp): the caller owns
// every buffer (host pointers), W stays valid for the model's lifetime (the
// GGUF mmap, src/core/tensor.cpp:148), errors are std::runtime_error.  The
// first call with a given W uploads and repacks it; later calls reuse the
// device copy.  Activations go host -> device -> host on every call, so this
// level is for parity and bisection; CudaModel (cuda_model.h) is the fast path.
#pragma once

#include <cstdint>
#include <stdexcept>
#include <string>

#include "smallm/backend/common/backend.h"
#include "smallm_cuda.h"

namespace smallm {

class CUDABackend final : public Backend {
public:
    explicit CUDABackend(int device = 0) { check(smallm_ctx_create(device, &ctx_)); }
    ~CUDABackend() override {
        if (ctx_) smallm_ctx_destroy(ctx_);
    }
    CUDABackend(const CUDABackend&) = delete;
    CUDABackend& operator=(const CUDABackend&) = delete;

    void matmul(const float* W, const float* x, uint32_t rows, uint32_t cols, float* y) override {
        check(smallm_backend_matmul(ctx_, W, x, rows, cols, y));
    }
    void matmul_quantized(const uint8_t* W, uint32_t type, const float* x, uint32_t rows, uint32_t cols,
                          float* y) override {
        check(smallm_backend_matmul_quantized(ctx_, W, type, x, rows, cols, y));
    }
    void rmsnorm(const float* x, const float* weight, uint32_t size, float eps, float* y) override {
        check(smallm_backend_rmsnorm(ctx_, x, weight, size, eps, y));
    }
    void softmax(float* x, uint32_t size) override { check(smallm_backend_softmax(ctx_, x, size)); }
    void silu(float* x, uint32_t size) override { check(smallm_backend_silu(ctx_, x, size)); }
    void rope(float* x, uint32_t n_heads, uint32_t head_dim, uint32_t pos, float freq_base) override {
        check(smallm_backend_rope(ctx_, x, n_heads, head_dim, pos, freq_base));
    }

    // Drop the device copies of every weight seen so far.
    void clear_weights() { check(smallm_ctx_clear_weights(ctx_)); }

private:
    static void check(int rc) {
        if (rc != SMALLM_OK) throw std::runtime_error(std::string("CUDABackend: ") + smallm_last_error());
    }
    smallm_ctx* ctx_ = nullptr;
};

}  // namespace smallm
