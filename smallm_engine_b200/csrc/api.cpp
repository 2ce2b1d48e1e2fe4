// extern "C" entry points of include/smallm_cuda.h.
#include <nccl.h>

#include <algorithm>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "engine.h"
#include "model.h"
#include "smallm_cuda.h"

using smallm::Error;

namespace {

thread_local std::string g_err;

template <typename F>
int guard(F&& f) {
    try {
        f();
        return SMALLM_OK;
    } catch (const Error& e) {
        g_err = e.what();
        return e.code;
    } catch (const std::bad_alloc&) {
        g_err = "out of host memory";
        return SMALLM_ERR_INVALID;
    } catch (const std::exception& e) {
        g_err = e.what();
        return SMALLM_ERR_INVALID;
    }
}

void need(bool ok, const char* msg) {
    if (!ok) throw Error(SMALLM_ERR_INVALID, msg);
}

// growable device buffer
struct DevBuf {
    void* p = nullptr;
    size_t n = 0;
    void* get(size_t bytes) {
        if (bytes > n) {
            if (p) cudaFree(p);
            p = nullptr;
            SM_CUDA(cudaMalloc(&p, bytes));
            n = bytes;
        }
        return p;
    }
    ~DevBuf() {
        if (p) cudaFree(p);
    }
};

}  // namespace

struct smallm_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    DevBuf a, b, c;
    // host weight pointer -> device copy (Backend::matmul_quantized compat)
    std::map<std::tuple<const void*, uint32_t, uint32_t, uint32_t>, smallm::QMat> cache;
    ~smallm_ctx() {
        for (auto& kv : cache) smallm::qmat_free(kv.second);
        if (stream) cudaStreamDestroy(stream);
    }
};

struct smallm_qmatrix {
    int device = 0;
    smallm::QMat m;
    ~smallm_qmatrix() { smallm::qmat_free(m); }
};

struct smallm_model {
    smallm::Model m;
};

static void set_dev(int d) { SM_CUDA(cudaSetDevice(d)); }

extern "C" {

const char* smallm_last_error(void) { return g_err.c_str(); }

int smallm_version(void) { return 100; }

int smallm_ctx_create(int device, smallm_ctx** out) {
    return guard([&] {
        need(out != nullptr, "out is NULL");
        *out = nullptr;
        int n = 0;
        SM_CUDA(cudaGetDeviceCount(&n));
        need(device >= 0 && device < n, "device ordinal out of range");
        set_dev(device);
        int major = 0;
        SM_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device));
        if (major < 10) throw Error(SMALLM_ERR_CUDA, "smallm: an sm_100 (Blackwell) device is required");
        auto c = std::make_unique<smallm_ctx>();
        c->device = device;
        SM_CUDA(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
        *out = c.release();
    });
}

int smallm_ctx_destroy(smallm_ctx* ctx) {
    return guard([&] {
        if (!ctx) return;
        set_dev(ctx->device);
        cudaStreamSynchronize(ctx->stream);
        delete ctx;
    });
}

void* smallm_ctx_stream(smallm_ctx* ctx) { return ctx ? (void*)ctx->stream : nullptr; }

int smallm_ctx_synchronize(smallm_ctx* ctx) {
    return guard([&] {
        need(ctx, "ctx is NULL");
        set_dev(ctx->device);
        SM_CUDA(cudaStreamSynchronize(ctx->stream));
    });
}

int smallm_ctx_clear_weights(smallm_ctx* ctx) {
    return guard([&] {
        need(ctx, "ctx is NULL");
        set_dev(ctx->device);
        SM_CUDA(cudaStreamSynchronize(ctx->stream));
        for (auto& kv : ctx->cache) smallm::qmat_free(kv.second);
        ctx->cache.clear();
    });
}

// Columns a Backend matmul row actually covers, as the reference computes it
// (src/core/ops.cpp:97-101, 184-187): quantized rows hold whole blocks only
// (cols / 32 blocks, cols / 256 super-blocks), so the tail of x is ignored;
// F32 rows (ops.cpp:15-26, 283-293) use every column.
static uint32_t matmul_cols(uint32_t type, uint32_t cols) {
    if (type == SMALLM_TYPE_F32) return cols;
    const uint32_t be = smallm::type_block_elems(type);
    return cols / be * be;
}

// Device copy of host matrix W (keyed by its address and shape).  F32 rows
// whose length is not a multiple of 32 are padded with zero columns to whole
// 32-element records; the padding multiplies zero-filled x entries.
static const smallm::QMat& cached_matrix(smallm_ctx* ctx, const uint8_t* W, uint32_t type, uint32_t rows,
                                         uint32_t cols) {
    auto key = std::make_tuple((const void*)W, type, rows, cols);
    auto it = ctx->cache.find(key);
    if (it != ctx->cache.end()) return it->second;
    smallm::QMat m;
    if (type == SMALLM_TYPE_F32 && cols % 32) {
        const uint32_t cp = (cols + 31) / 32 * 32;
        std::vector<float> pad((size_t)rows * cp, 0.f);
        for (uint32_t r = 0; r < rows; ++r)
            std::memcpy(pad.data() + (size_t)r * cp, W + (size_t)r * cols * 4, (size_t)cols * 4);
        smallm::qmat_upload(m, reinterpret_cast<const uint8_t*>(pad.data()), type, rows, cp, cp, 0, {},
                            ctx->stream);
    } else {
        smallm::qmat_upload(m, W, type, rows, cols, cols, 0, {}, ctx->stream);
    }
    return ctx->cache.emplace(key, m).first->second;
}

// y = m . x with host x (x_cols valid entries; the rest of m's columns read
// zeros) and host y.
static void gemv_host(smallm_ctx* ctx, const smallm::QMat& m, const float* x, uint32_t x_cols, float* y) {
    float* dx = static_cast<float*>(ctx->a.get(4ull * m.cols));
    float* dy = static_cast<float*>(ctx->b.get(4ull * m.rows));
    SM_CUDA(cudaMemcpyAsync(dx, x, 4ull * x_cols, cudaMemcpyHostToDevice, ctx->stream));
    if (x_cols < m.cols) SM_CUDA(cudaMemsetAsync(dx + x_cols, 0, 4ull * (m.cols - x_cols), ctx->stream));
    smallm::GemvArgs a;
    a.x = dx;
    a.y = dy;
    smallm::launch_gemv(m, smallm::GEMV_PRO_PLAIN, smallm::GEMV_EPI_STORE, a, ctx->stream);
    SM_CUDA(cudaMemcpyAsync(y, dy, 4ull * m.rows, cudaMemcpyDeviceToHost, ctx->stream));
    SM_CUDA(cudaStreamSynchronize(ctx->stream));
}

int smallm_backend_matmul(smallm_ctx* ctx, const float* W, const float* x, uint32_t rows, uint32_t cols,
                          float* y) {
    return smallm_backend_matmul_quantized(ctx, reinterpret_cast<const uint8_t*>(W), SMALLM_TYPE_F32, x, rows,
                                           cols, y);
}

int smallm_backend_matmul_quantized(smallm_ctx* ctx, const uint8_t* W, uint32_t type, const float* x,
                                    uint32_t rows, uint32_t cols, float* y) {
    return guard([&] {
        need(ctx != nullptr, "NULL argument");
        if (!smallm::type_supported(type))
            throw Error(SMALLM_ERR_UNSUPPORTED_TYPE, "unsupported tensor type: " + std::to_string(type));
        if (!rows) return;  // the reference's row loop runs zero times
        const uint32_t c = matmul_cols(type, cols);
        need(y && (c == 0 || (W && x)), "NULL argument");
        if (!c) {  // no whole block: every accumulator stays 0
            std::memset(y, 0, 4ull * rows);
            return;
        }
        set_dev(ctx->device);
        gemv_host(ctx, cached_matrix(ctx, W, type, rows, c), x, c, y);
    });
}

int smallm_backend_rmsnorm(smallm_ctx* ctx, const float* x, const float* weight, uint32_t size, float eps,
                           float* y) {
    return guard([&] {
        need(ctx && x && weight && y, "NULL argument");
        set_dev(ctx->device);
        if (!size) return;
        float* dx = static_cast<float*>(ctx->a.get(4ull * size));
        float* dw = static_cast<float*>(ctx->b.get(4ull * size));
        float* dy = static_cast<float*>(ctx->c.get(4ull * size));
        SM_CUDA(cudaMemcpyAsync(dx, x, 4ull * size, cudaMemcpyHostToDevice, ctx->stream));
        SM_CUDA(cudaMemcpyAsync(dw, weight, 4ull * size, cudaMemcpyHostToDevice, ctx->stream));
        smallm::launch_rmsnorm(dx, dw, size, eps, dy, ctx->stream);
        SM_CUDA(cudaMemcpyAsync(y, dy, 4ull * size, cudaMemcpyDeviceToHost, ctx->stream));
        SM_CUDA(cudaStreamSynchronize(ctx->stream));
    });
}

int smallm_backend_softmax(smallm_ctx* ctx, float* x, uint32_t size) {
    return guard([&] {
        need(ctx && (x || !size), "NULL argument");
        set_dev(ctx->device);
        if (!size) return;  // ops.cpp:44
        float* dx = static_cast<float*>(ctx->a.get(4ull * size));
        SM_CUDA(cudaMemcpyAsync(dx, x, 4ull * size, cudaMemcpyHostToDevice, ctx->stream));
        smallm::launch_softmax(dx, size, ctx->stream);
        SM_CUDA(cudaMemcpyAsync(x, dx, 4ull * size, cudaMemcpyDeviceToHost, ctx->stream));
        SM_CUDA(cudaStreamSynchronize(ctx->stream));
    });
}

int smallm_backend_silu(smallm_ctx* ctx, float* x, uint32_t size) {
    return guard([&] {
        need(ctx && (x || !size), "NULL argument");
        set_dev(ctx->device);
        if (!size) return;
        float* dx = static_cast<float*>(ctx->a.get(4ull * size));
        SM_CUDA(cudaMemcpyAsync(dx, x, 4ull * size, cudaMemcpyHostToDevice, ctx->stream));
        smallm::launch_silu(dx, size, ctx->stream);
        SM_CUDA(cudaMemcpyAsync(x, dx, 4ull * size, cudaMemcpyDeviceToHost, ctx->stream));
        SM_CUDA(cudaStreamSynchronize(ctx->stream));
    });
}

int smallm_backend_rope(smallm_ctx* ctx, float* x, uint32_t n_heads, uint32_t head_dim, uint32_t pos,
                        float freq_base) {
    return guard([&] {
        need(ctx && (x || !n_heads), "NULL argument");
        need(head_dim % 2 == 0, "head_dim must be even");
        set_dev(ctx->device);
        const size_t n = (size_t)n_heads * head_dim;
        if (!n) return;
        std::vector<float2> cs;
        smallm::rope_table(head_dim, 1, freq_base, cs, pos);
        float* dx = static_cast<float*>(ctx->a.get(4 * n));
        float2* dcs = static_cast<float2*>(ctx->b.get(cs.size() * sizeof(float2)));
        SM_CUDA(cudaMemcpyAsync(dx, x, 4 * n, cudaMemcpyHostToDevice, ctx->stream));
        SM_CUDA(cudaMemcpyAsync(dcs, cs.data(), cs.size() * sizeof(float2), cudaMemcpyHostToDevice, ctx->stream));
        smallm::launch_rope(dx, n_heads, head_dim, dcs, ctx->stream);
        SM_CUDA(cudaMemcpyAsync(x, dx, 4 * n, cudaMemcpyDeviceToHost, ctx->stream));
        SM_CUDA(cudaStreamSynchronize(ctx->stream));
    });
}

int smallm_qmatrix_upload(smallm_ctx* ctx, const uint8_t* W, uint32_t type, uint32_t rows, uint32_t cols,
                          smallm_qmatrix** out) {
    return guard([&] {
        need(ctx && W && out, "NULL argument");
        *out = nullptr;
        if (!smallm::type_supported(type))
            throw Error(SMALLM_ERR_UNSUPPORTED_TYPE, "unsupported tensor type: " + std::to_string(type));
        set_dev(ctx->device);
        auto q = std::make_unique<smallm_qmatrix>();
        q->device = ctx->device;
        smallm::qmat_upload(q->m, W, type, rows, cols, cols, 0, {}, ctx->stream);
        *out = q.release();
    });
}

int smallm_qmatrix_free(smallm_qmatrix* m) {
    return guard([&] {
        if (!m) return;
        set_dev(m->device);
        delete m;
    });
}

int smallm_qmatrix_bytes(const smallm_qmatrix* m, uint64_t* gguf_bytes, uint64_t* device_bytes) {
    return guard([&] {
        need(m, "NULL argument");
        if (gguf_bytes) *gguf_bytes = m->m.gguf_bytes;
        if (device_bytes) *device_bytes = m->m.dev_bytes;
    });
}

int smallm_gemv(smallm_ctx* ctx, const smallm_qmatrix* W, const float* x_dev, float* y_dev, void* stream) {
    return guard([&] {
        need(ctx && W && x_dev && y_dev, "NULL argument");
        set_dev(ctx->device);
        smallm::GemvArgs a;
        a.x = x_dev;
        a.y = y_dev;
        smallm::launch_gemv(W->m, smallm::GEMV_PRO_PLAIN, smallm::GEMV_EPI_STORE, a,
                            stream ? (cudaStream_t)stream : ctx->stream);
    });
}

int smallm_gemm_f16(smallm_ctx* ctx, const uint16_t* w_dev, const uint16_t* x_dev, uint32_t N, uint32_t K,
                    uint32_t T, float* y_dev, uint32_t ldy, void* stream) {
    return guard([&] {
        need(ctx && ((w_dev && x_dev && y_dev) || N == 0 || T == 0), "NULL argument");
        set_dev(ctx->device);
        smallm::launch_tc_gemm(reinterpret_cast<const __half*>(w_dev), N, K, reinterpret_cast<const __half*>(x_dev),
                               T, y_dev, ldy, stream ? (cudaStream_t)stream : ctx->stream);
    });
}

int smallm_gemv_residual_sum(smallm_ctx* ctx, const smallm_qmatrix* W, const float* x_res_dev,
                             const float* parts_dev, uint32_t n_parts, const uint32_t* flags_dev,
                             const uint32_t* epoch_dev, const float* norm_w_dev, float eps, float* x_out_dev,
                             float* y_dev, void* stream) {
    return guard([&] {
        need(ctx && W && x_res_dev && parts_dev && flags_dev && epoch_dev && norm_w_dev && x_out_dev && y_dev,
             "NULL argument");
        need(n_parts >= 1 && n_parts <= (uint32_t)smallm::kMaxTPRanks, "n_parts must be 1..8");
        set_dev(ctx->device);
        smallm::GemvArgs a;
        a.x = x_res_dev;
        a.x_res = x_res_dev;
        a.rx = parts_dev;
        a.rx_flag = flags_dev;
        a.epoch = epoch_dev;
        a.tp = n_parts;
        a.norm_w = norm_w_dev;
        a.eps = eps;
        a.x_out = x_out_dev;
        a.y = y_dev;
        smallm::launch_gemv(W->m, smallm::GEMV_PRO_RMS_SUM, smallm::GEMV_EPI_STORE, a,
                            stream ? (cudaStream_t)stream : ctx->stream);
    });
}

int smallm_ctx_device_errors(smallm_ctx* ctx, uint32_t* flags, int clear) {
    return guard([&] {
        need(ctx && flags, "NULL argument");
        set_dev(ctx->device);
        SM_CUDA(cudaDeviceSynchronize());
        *flags = smallm::gemv_error_flags(clear != 0);
    });
}

int smallm_attention_noalloc(smallm_ctx* ctx, const float* q_dev, const float* kcache_dev,
                             const float* vcache_dev, uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim,
                             uint32_t max_ctx, uint32_t pos, float* out_dev, void* stream) {
    return guard([&] {
        need(ctx && q_dev && kcache_dev && vcache_dev && out_dev, "NULL argument");
        set_dev(ctx->device);
        smallm::launch_attention_static(q_dev, kcache_dev, vcache_dev, n_heads, n_kv_heads, head_dim, max_ctx,
                                        pos, out_dev, stream ? (cudaStream_t)stream : ctx->stream);
    });
}

static void check_sampler(uint32_t kind, uint32_t k, float temperature) {
    need(kind <= SMALLM_SAMPLE_TOP_P, "unknown sampler kind");
    need(kind != SMALLM_SAMPLE_TOP_K || k >= 1, "top-k needs k >= 1");
    need(kind == SMALLM_SAMPLE_GREEDY || temperature > 0.f, "temperature must be positive");
}

int smallm_sample(smallm_ctx* ctx, const float* logits, uint32_t n, uint32_t kind, uint32_t k, float p,
                  float temperature, float u, uint32_t* token) {
    return guard([&] {
        need(ctx && logits && token && n > 0, "NULL argument or empty logits");
        check_sampler(kind, k, temperature);
        set_dev(ctx->device);
        float* dl = static_cast<float*>(ctx->a.get(4ull * n));
        uint32_t* scratch = static_cast<uint32_t*>(ctx->b.get(16ull * n + 16));
        SM_CUDA(cudaMemcpyAsync(dl, logits, 4ull * n, cudaMemcpyHostToDevice, ctx->stream));
        smallm::launch_sample(dl, n, kind, k, p, temperature, u, scratch, scratch + 4ull * n, ctx->stream);
        SM_CUDA(cudaMemcpyAsync(token, scratch + 4ull * n, 4, cudaMemcpyDeviceToHost, ctx->stream));
        SM_CUDA(cudaStreamSynchronize(ctx->stream));
    });
}

int smallm_model_prefill(smallm_model* m, const uint32_t* tokens, uint32_t n, uint32_t start_pos, float* logits,
                         uint32_t* argmax, uint32_t flags) {
    return guard([&] {
        need(m && (tokens || n == 0), "NULL argument");
        set_dev(m->m.device);
        m->m.prefill(tokens, n, start_pos, logits, argmax, flags);
    });
}

int smallm_model_sample(smallm_model* m, uint32_t kind, uint32_t k, float p, float temperature, float u,
                        uint32_t* token) {
    return guard([&] {
        need(m && token, "NULL argument");
        check_sampler(kind, k, temperature);
        set_dev(m->m.device);
        *token = m->m.sample(kind, k, p, temperature, u);
    });
}

int smallm_qmatrix_dequantize(smallm_ctx* ctx, const smallm_qmatrix* W, float* y_dev, void* stream) {
    return guard([&] {
        need(ctx && W && y_dev, "NULL argument");
        set_dev(ctx->device);
        smallm::launch_qmat_dequant(W->m, y_dev, stream ? (cudaStream_t)stream : ctx->stream);
    });
}

int smallm_dequantize(smallm_ctx* ctx, uint32_t type, const uint8_t* src, uint64_t count, float* out) {
    return guard([&] {
        need(ctx && (count == 0 || (src && out)), "NULL argument");
        if (!smallm::type_supported(type))
            throw Error(SMALLM_ERR_UNSUPPORTED_TYPE, "unsupported tensor type: " + std::to_string(type));
        const uint32_t be = smallm::type_block_elems(type);
        need(count % be == 0, "count is not a whole number of blocks");
        set_dev(ctx->device);
        if (!count) return;
        const uint64_t bytes = smallm::type_row_bytes(type, count);
        uint8_t* ds = static_cast<uint8_t*>(ctx->a.get(bytes));
        float* dy = static_cast<float*>(ctx->b.get(4 * count + 128));
        SM_CUDA(cudaMemcpyAsync(ds, src, bytes, cudaMemcpyHostToDevice, ctx->stream));
        smallm::launch_dequant_raw(type, ds, count, dy, ctx->stream);
        SM_CUDA(cudaMemcpyAsync(out, dy, 4 * count, cudaMemcpyDeviceToHost, ctx->stream));
        SM_CUDA(cudaStreamSynchronize(ctx->stream));
    });
}

int smallm_nccl_unique_id(void* out) {
    return guard([&] {
        need(out, "NULL argument");
        ncclUniqueId id;
        ncclResult_t r = ncclGetUniqueId(&id);
        if (r != ncclSuccess) throw Error(SMALLM_ERR_NCCL, std::string("ncclGetUniqueId: ") + ncclGetErrorString(r));
        std::memcpy(out, &id, sizeof(id));
    });
}

int smallm_host_alloc(size_t bytes, void** out) {
    return guard([&] {
        need(out, "NULL argument");
        *out = nullptr;
        SM_CUDA(cudaHostAlloc(out, bytes ? bytes : 16, cudaHostAllocPortable));
    });
}

int smallm_host_free(void* p) {
    return guard([&] {
        if (p) SM_CUDA(cudaFreeHost(p));
    });
}

int smallm_model_load(const char* gguf_path, const smallm_model_opts* opts, smallm_model** out) {
    return guard([&] {
        need(gguf_path && out, "NULL argument");
        *out = nullptr;
        smallm_model_opts o{};
        if (opts) o = *opts;
        int n = 0;
        SM_CUDA(cudaGetDeviceCount(&n));
        need(o.device >= 0 && o.device < n, "device ordinal out of range");
        auto m = std::make_unique<smallm_model>();
        m->m.load(gguf_path, o);
        *out = m.release();
    });
}

int smallm_model_free(smallm_model* m) {
    return guard([&] {
        if (!m) return;
        set_dev(m->m.device);
        cudaStreamSynchronize(m->m.stream);
        delete m;
    });
}

int smallm_model_get_info(const smallm_model* m, smallm_model_info* o) {
    return guard([&] {
        need(m && o, "NULL argument");
        const smallm::Model& M = m->m;
        std::memset(o, 0, sizeof(*o));
        std::strncpy(o->arch, M.arch.c_str(), sizeof(o->arch) - 1);
        o->n_layers = M.n_layers;
        o->embd = M.embd;
        o->ffn = M.ffn;
        o->n_heads = M.n_heads;
        o->n_kv_heads = M.n_kv;
        o->head_dim = M.hd;
        o->vocab = M.vocab;
        o->context_length = M.ctx;
        o->max_ctx = M.max_ctx;
        o->rope_freq_base = M.rope_base;
        o->rms_eps = M.eps;
        o->weight_bytes_per_token = M.weight_bytes;
        o->device_bytes = M.dev_bytes;
        o->step_launches = M.step_launch_count();
    });
}

void* smallm_model_stream(smallm_model* m) { return m ? (void*)m->m.stream : nullptr; }

int smallm_model_forward(smallm_model* m, uint32_t token, uint32_t pos, float* logits, uint32_t* argmax) {
    return guard([&] {
        need(m, "NULL argument");
        set_dev(m->m.device);
        m->m.forward(token, pos, logits, argmax);
    });
}

int smallm_model_reset_cache(smallm_model* m) {
    return guard([&] {
        need(m, "NULL argument");
        m->m.cached = 0;  // qwen2_model.cpp:69-71: only the bookkeeping is reset
    });
}

int smallm_model_truncate_cache(smallm_model* m, uint32_t n) {
    return guard([&] {
        need(m, "NULL argument");
        if (n < m->m.cached) m->m.cached = n;  // qwen2_model.cpp:73-75
    });
}

uint32_t smallm_model_cached_length(const smallm_model* m) { return m ? m->m.cached : 0; }

int smallm_model_decode_greedy_async(smallm_model* m, uint32_t token, uint32_t pos, uint32_t n_steps) {
    return guard([&] {
        need(m, "NULL argument");
        set_dev(m->m.device);
        m->m.decode_async(token, pos, n_steps);
    });
}

int smallm_model_decode_ids(smallm_model* m, uint32_t* ids, uint32_t n) {
    return guard([&] {
        need(m && (ids || !n), "NULL argument");
        set_dev(m->m.device);
        m->m.decode_ids(ids, n);
    });
}

const float* smallm_model_logits_device(smallm_model* m) { return m ? m->m.logits_local : nullptr; }

int smallm_model_trace_step(smallm_model* m, uint32_t token, uint32_t pos, uint64_t* out, uint32_t cap,
                            uint32_t* n) {
    return guard([&] {
        need(m && n && (out || !cap), "NULL argument");
        set_dev(m->m.device);
        std::vector<smallm::TraceSlot> t;
        m->m.trace_step(token, pos, t);
        *n = (uint32_t)t.size();
        uint64_t t0 = t.empty() ? 0 : t[0].t_start;
        for (const auto& r : t) t0 = std::min<uint64_t>(t0, r.t_start);
        for (uint32_t i = 0; i < t.size() && i < cap; ++i) {
            out[4 * i] = t[i].t_start - t0;
            out[4 * i + 1] = t[i].t_ready - t0;
            out[4 * i + 2] = t[i].t_end - t0;
            out[4 * i + 3] = t[i].kind;
        }
    });
}

}  // extern "C"
