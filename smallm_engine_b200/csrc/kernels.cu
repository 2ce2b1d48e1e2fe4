// Repack, dequantisation, embedding, attention, step bookkeeping and the
// op-level kernels, plus the GEMV launcher.
#include <cmath>
#include <cstring>
#include <mutex>
#include <set>
#include <tuple>
#include <unordered_map>

#include "engine.h"
#include "dequant.cuh"
#include "gemv.cuh"

namespace smallm {

void cuda_check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
        cudaGetLastError();
        throw Error(3, std::string(what) + ": " + cudaGetErrorString(e));
    }
}

uint32_t type_block_elems(uint32_t t) {
    switch (t) {
        case SM_T_F32: return 1;
        case SM_T_Q4_0: case SM_T_Q8_0: return 32;
        case SM_T_Q4_K: case SM_T_Q6_K: return 256;
        default: return 0;
    }
}
uint32_t type_block_bytes(uint32_t t) {
    switch (t) {
        case SM_T_F32: return 4;
        case SM_T_Q4_0: return 18;
        case SM_T_Q8_0: return 34;
        case SM_T_Q4_K: return 144;
        case SM_T_Q6_K: return 210;
        default: return 0;
    }
}
bool type_supported(uint32_t t) { return type_block_elems(t) != 0; }
uint64_t type_row_bytes(uint32_t t, uint64_t cols) {
    uint32_t be = type_block_elems(t);
    return be ? cols / be * type_block_bytes(t) : 0;
}

int device_sm_count() {
    int dev = 0, n = 0;
    SM_CUDA(cudaGetDevice(&dev));
    SM_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
    return n;
}

// ------------------------------------------------------------ layouts --

static uint32_t unit_elems(uint32_t t) {
    return (t == SM_T_Q4_K || t == SM_T_Q6_K) ? 64u : 32u;
}

static uint32_t align16(uint64_t v) { return (uint32_t)((v + 15) / 16 * 16); }

// Bytes of one storage row record (see QMat in engine.h).
static uint32_t record_stride(uint32_t t, uint32_t cols) {
    const uint32_t units = cols / unit_elems(t);
    switch (t) {
        case SM_T_F32: return cols * 4;
        case SM_T_Q4_0: return units * 16 + align16(units * 2);
        case SM_T_Q8_0: return units * 32 + align16(units * 2);
        case SM_T_Q4_K: return (cols / 256) * 144;
        case SM_T_Q6_K: return align16((uint64_t)units * 52 + (cols / 256) * 2);
        default: return 0;
    }
}

void qmat_alloc(QMat& m, uint32_t type, uint32_t rows, uint32_t cols) {
    if (!type_supported(type)) throw Error(2, "unsupported tensor type: " + std::to_string(type));
    const uint32_t be = type_block_elems(type);
    if (cols == 0 || rows == 0 || cols % (be < 32 ? 32 : be))
        throw Error(1, "matrix shape " + std::to_string(rows) + "x" + std::to_string(cols) +
                           " is not a whole number of blocks for type " + std::to_string(type));
    m.type = type;
    m.rows = rows;
    m.rows_pad = (rows + 31) / 32 * 32;
    m.cols = cols;
    m.units = cols / unit_elems(type);
    m.row_stride = record_stride(type, cols);
    m.gguf_bytes = (uint64_t)rows * type_row_bytes(type, cols);
    m.dev_bytes = (uint64_t)m.rows_pad * m.row_stride;
    SM_CUDA(cudaMalloc(&m.base, m.dev_bytes));
    SM_CUDA(cudaMemset(m.base, 0, m.dev_bytes));  // padding rows and record padding stay zero
}

void qmat_free(QMat& m) {
    if (m.base) cudaFree(m.base);
    m = QMat{};
}

// One thread per (storage row, 32-element unit) for Q4_0, Q8_0 and F32:
// quants to the front of the row record, f16 scales after them.  Source
// blocks are byte-addressed (18/34-byte GGUF blocks are not aligned).
__global__ void smallm_repack_blocks_kernel(const uint8_t* src, uint64_t src_row_bytes, uint64_t col_byte0,
                                     const uint32_t* row_map, uint32_t rows, uint32_t rows_pad,
                                     uint32_t nunits, uint32_t stride, uint32_t type, uint8_t* dst) {
    const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (uint64_t)rows_pad * nunits) return;
    const uint32_t p = (uint32_t)(idx / nunits), u = (uint32_t)(idx % nunits);
    const uint32_t srow = row_map ? row_map[p] : (p < rows ? p : 0xFFFFFFFFu);
    if (srow == 0xFFFFFFFFu) return;  // storage is zeroed
    const uint32_t bb = type == SM_T_Q4_0 ? 18 : (type == SM_T_Q8_0 ? 34 : 128);
    const uint32_t qb = type == SM_T_Q4_0 ? 16 : (type == SM_T_Q8_0 ? 32 : 128);
    const uint8_t* b = src + (uint64_t)srow * src_row_bytes + col_byte0 + (uint64_t)u * bb;
    uint8_t* row = dst + (uint64_t)p * stride;
    if (type == SM_T_F32) {
        for (uint32_t i = 0; i < 128; ++i) row[(size_t)u * 128 + i] = b[i];
    } else {
        for (uint32_t i = 0; i < qb; ++i) row[(size_t)u * qb + i] = b[2 + i];
        row[(size_t)nunits * qb + u * 2] = b[0];
        row[(size_t)nunits * qb + u * 2 + 1] = b[1];
    }
}

// Q4_K: super-blocks are copied whole (row permutation / column slice only).
__global__ void smallm_repack_q4k_kernel(const uint8_t* src, uint64_t src_row_bytes, uint64_t col_byte0,
                                  const uint32_t* row_map, uint32_t rows, uint32_t rows_pad, uint32_t nsb,
                                  uint32_t stride, uint8_t* dst) {
    const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (uint64_t)rows_pad * nsb) return;
    const uint32_t p = (uint32_t)(idx / nsb), k = (uint32_t)(idx % nsb);
    const uint32_t srow = row_map ? row_map[p] : (p < rows ? p : 0xFFFFFFFFu);
    if (srow == 0xFFFFFFFFu) return;
    const uint8_t* b = src + (uint64_t)srow * src_row_bytes + col_byte0 + (uint64_t)k * 144;
    uint8_t* o = dst + (uint64_t)p * stride + (uint64_t)k * 144;
    for (int i = 0; i < 144; ++i) o[i] = b[i];
}

// Q6_K: decode the 256 6-bit codes of a GGUF super-block (ql/qh layout of
// src/core/tensor.cpp:93-100) and re-encode them per 64-element unit: 32
// nibble bytes (byte k: element k low, element 32+k high) and 16 bytes of
// 2-bit high parts (byte k: elements k, 16+k, 32+k, 48+k).  The 16 int8
// scales keep their order (element e uses scale e/16) and d goes to the end
// of the record.  Lossless: every code and scale bit is preserved.
__global__ void smallm_repack_q6k_kernel(const uint8_t* src, uint64_t src_row_bytes, uint64_t col_byte0,
                                  const uint32_t* row_map, uint32_t rows, uint32_t rows_pad, uint32_t nsb,
                                  uint32_t stride, uint8_t* dst) {
    const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (uint64_t)rows_pad * nsb) return;
    const uint32_t p = (uint32_t)(idx / nsb), k = (uint32_t)(idx % nsb);
    const uint32_t srow = row_map ? row_map[p] : (p < rows ? p : 0xFFFFFFFFu);
    if (srow == 0xFFFFFFFFu) return;
    const uint8_t* b = src + (uint64_t)srow * src_row_bytes + col_byte0 + (uint64_t)k * 210;
    const uint32_t units = nsb * 4;
    uint8_t* row = dst + (uint64_t)p * stride;
    uint8_t* qo = row + (size_t)k * 4 * 48;
    uint8_t out[192];
    for (int i = 0; i < 192; ++i) out[i] = 0;
    for (int E = 0; E < 256; ++E) {
        const int h = E >> 7, w = E & 127, m = w >> 5, l = w & 31;
        const uint8_t qlb = b[h * 64 + l + ((m & 1) ? 32 : 0)];
        const uint8_t qhb = b[128 + h * 32 + l];
        const int lo4 = (m < 2) ? (qlb & 0xF) : (qlb >> 4);
        const int hi2 = (qhb >> (2 * m)) & 3;
        const int u = E >> 6, e = E & 63;
        uint8_t* ub = out + u * 48;
        if (e < 32) ub[e] |= (uint8_t)lo4;
        else ub[e - 32] |= (uint8_t)(lo4 << 4);
        ub[32 + (e & 15)] |= (uint8_t)(hi2 << (2 * (e >> 4)));
    }
    for (int i = 0; i < 192; ++i) qo[i] = out[i];
    uint8_t* so = row + (size_t)units * 48 + (size_t)k * 16;
    for (int i = 0; i < 16; ++i) so[i] = b[192 + i];
    uint8_t* dout = row + (size_t)units * 52 + (size_t)k * 2;
    dout[0] = b[208];
    dout[1] = b[209];
}

void qmat_repack(QMat& m, const RepackSource& s, cudaStream_t stream) {
    const uint64_t rb = type_row_bytes(m.type, s.src_cols);
    const uint64_t cb0 = type_row_bytes(m.type, s.col0);
    const int T = 256;
    if (m.type == SM_T_Q4_K || m.type == SM_T_Q6_K) {
        const uint32_t nsb = m.cols / 256;
        const uint64_t n = (uint64_t)m.rows_pad * nsb;
        if (m.type == SM_T_Q4_K)
            smallm_repack_q4k_kernel<<<(unsigned)((n + T - 1) / T), T, 0, stream>>>(s.src, rb, cb0, s.row_map, m.rows,
                                                                              m.rows_pad, nsb, m.row_stride, m.base);
        else
            smallm_repack_q6k_kernel<<<(unsigned)((n + T - 1) / T), T, 0, stream>>>(s.src, rb, cb0, s.row_map, m.rows,
                                                                              m.rows_pad, nsb, m.row_stride, m.base);
    } else {
        const uint64_t n = (uint64_t)m.rows_pad * m.units;
        smallm_repack_blocks_kernel<<<(unsigned)((n + T - 1) / T), T, 0, stream>>>(
            s.src, rb, cb0, s.row_map, m.rows, m.rows_pad, m.units, m.row_stride, m.type, m.base);
    }
    SM_CUDA(cudaGetLastError());
}

void qmat_upload(QMat& m, const uint8_t* host, uint32_t type, uint32_t rows, uint32_t cols,
                 uint64_t src_cols, uint64_t col0, const std::vector<uint32_t>& row_map,
                 cudaStream_t stream) {
    qmat_alloc(m, type, rows, cols);
    // stage only the source rows that are referenced
    uint32_t src_rows = rows;
    for (uint32_t r : row_map)
        if (r != 0xFFFFFFFFu && r + 1 > src_rows) src_rows = r + 1;
    const uint64_t bytes = (uint64_t)src_rows * type_row_bytes(type, src_cols);
    uint8_t* stage = nullptr;
    uint32_t* dmap = nullptr;
    try {
        SM_CUDA(cudaMalloc(&stage, bytes));
        SM_CUDA(cudaMemcpyAsync(stage, host, bytes, cudaMemcpyHostToDevice, stream));
        if (!row_map.empty()) {
            std::vector<uint32_t> full(row_map);
            full.resize(m.rows_pad, 0xFFFFFFFFu);
            SM_CUDA(cudaMalloc(&dmap, full.size() * 4));
            SM_CUDA(cudaMemcpyAsync(dmap, full.data(), full.size() * 4, cudaMemcpyHostToDevice, stream));
            RepackSource s{stage, src_cols, col0, dmap};
            qmat_repack(m, s, stream);
            SM_CUDA(cudaStreamSynchronize(stream));
        } else {
            RepackSource s{stage, src_cols, col0, nullptr};
            qmat_repack(m, s, stream);
            SM_CUDA(cudaStreamSynchronize(stream));
        }
    } catch (...) {
        if (stage) cudaFree(stage);
        if (dmap) cudaFree(dmap);
        qmat_free(m);
        throw;
    }
    cudaFree(stage);
    if (dmap) cudaFree(dmap);
}

// ------------------------------------------------------- dequantisation --


__global__ void smallm_qmat_dequant_kernel(const QMat m, float* y) {
    const uint32_t groups = m.cols / 32;
    const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (uint64_t)m.rows * groups) return;
    const uint32_t r = (uint32_t)(idx / groups), g = (uint32_t)(idx % groups);
    dequant_group(m, r, g, y + (size_t)r * m.cols + (size_t)g * 32);
}

void launch_qmat_dequant(const QMat& m, float* y, cudaStream_t stream) {
    const uint64_t n = (uint64_t)m.rows * (m.cols / 32);
    smallm_qmat_dequant_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(m, y);
    SM_CUDA(cudaGetLastError());
}


// Raw GGUF blocks (contiguous, byte-addressed) -> f32, one thread per 32
// elements, same arithmetic as dequant_group.
__global__ void smallm_dequant_raw_kernel(uint32_t type, const uint8_t* src, uint64_t count, float* out) {
    const uint64_t g = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (g * 32 >= count) return;
    float* o = out + g * 32;
    if (type == SM_T_F32) {
        const float* f = reinterpret_cast<const float*>(src) + g * 32;
        const uint64_t n = count - g * 32 < 32 ? count - g * 32 : 32;
        for (uint64_t i = 0; i < n; ++i) o[i] = f[i];
    } else if (type == SM_T_Q4_0) {
        const uint8_t* b = src + g * 18;
        const float d = f16_exact(b[0] | (b[1] << 8));
        for (int k = 0; k < 16; ++k) {
            o[k] = __fmul_rn(d, (float)((int)(b[2 + k] & 0xF) - 8));
            o[k + 16] = __fmul_rn(d, (float)((int)(b[2 + k] >> 4) - 8));
        }
    } else if (type == SM_T_Q8_0) {
        const uint8_t* b = src + g * 34;
        const float d = f16_exact(b[0] | (b[1] << 8));
        for (int k = 0; k < 32; ++k) o[k] = __fmul_rn(d, (float)(int8_t)b[2 + k]);
    } else if (type == SM_T_Q4_K) {
        const uint64_t sbi = g / 8;
        const uint32_t j = (uint32_t)(g % 8);
        const uint8_t* b = src + sbi * 144;
        const float d = f16_exact(b[0] | (b[1] << 8)), dmin = f16_exact(b[2] | (b[3] << 8));
        const uint8_t* sc = b + 4;
        int s, mm;
        if (j < 4) {
            s = sc[j] & 63;
            mm = sc[j + 4] & 63;
        } else {
            s = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
            mm = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
        }
        const float d1 = __fmul_rn(d, (float)s), m1 = __fmul_rn(dmin, (float)mm);
        const uint8_t* qs = b + 16 + (j / 2) * 32;
        for (int k = 0; k < 32; ++k) {
            const int v = (j & 1) ? (qs[k] >> 4) : (qs[k] & 0xF);
            o[k] = __fsub_rn(__fmul_rn(d1, (float)v), m1);
        }
    } else if (type == SM_T_Q6_K) {
        const uint64_t sbi = g / 8;
        const uint32_t gg = (uint32_t)(g % 8);
        const uint8_t* b = src + sbi * 210;
        const float d = f16_exact(b[208] | (b[209] << 8));
        const int8_t* sc = reinterpret_cast<const int8_t*>(b + 192);
        for (int k = 0; k < 32; ++k) {
            const int E = (int)gg * 32 + k;
            const int h = E >> 7, w = E & 127, m = w >> 5, l = w & 31;
            const uint8_t qlb = b[h * 64 + l + ((m & 1) ? 32 : 0)];
            const int lo4 = (m < 2) ? (qlb & 0xF) : (qlb >> 4);
            const int hi2 = (b[128 + h * 32 + l] >> (2 * m)) & 3;
            o[k] = __fmul_rn(__fmul_rn(d, (float)sc[E >> 4]), (float)((lo4 | (hi2 << 4)) - 32));
        }
    }
}

void launch_dequant_raw(uint32_t type, const uint8_t* src, uint64_t count, float* out, cudaStream_t stream) {
    const uint64_t groups = (count + 31) / 32;
    smallm_dequant_raw_kernel<<<(unsigned)((groups + 255) / 256), 256, 0, stream>>>(type, src, count, out);
    SM_CUDA(cudaGetLastError());
}

// --------------------------------------------------------------- launch --

void launch_kernel_ex(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl,
                      void** args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    if (pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    SM_CUDA(cudaLaunchKernelExC(&cfg, fn, args));
}

// ------------------------------------------------------------- embedding --

// One thread per 32-element group of the token's row.
__global__ void smallm_embed_kernel(const QMat m, DecodeState* st, float* x, TraceSlot* trace) {
    if (threadIdx.x == 0) trace_mark(trace, 0);
    pdl_launch_dependents();
    pdl_wait();
    if (threadIdx.x == 0) trace_mark(trace, 1);
    uint32_t tok = st->token;
    if (tok >= m.rows) tok = 0;  // the host validates ids; never read outside the table
    const uint32_t g = blockIdx.x * blockDim.x + threadIdx.x;
    if (g < m.cols / 32) dequant_group(m, tok, g, x + (size_t)g * 32);
    if (g == 0) st->argmax = 0ull;
    if (threadIdx.x == 0) trace_mark(trace, 2);
}

void launch_embed(const QMat& emb, DecodeState* st, float* x, cudaStream_t stream, bool pdl, TraceSlot* trace) {
    QMat m = emb;
    void* args[] = {&m, &st, &x, &trace};
    const uint32_t groups = m.cols / 32;
    launch_kernel_ex((const void*)smallm_embed_kernel, dim3((groups + 31) / 32), dim3(32), 0, stream, pdl, args);
}

// Prefill: X[t] = dequantized row tokens[t] for t < T (one thread per
// 32-element group).  Ids were validated on the host.
__global__ void smallm_embed_rows_kernel(const QMat m, const uint32_t* tokens, uint32_t T, float* X) {
    const uint32_t groups = m.cols / 32;
    const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (uint64_t)T * groups) return;
    const uint32_t t = (uint32_t)(idx / groups), g = (uint32_t)(idx % groups);
    dequant_group(m, tokens[t], g, X + (size_t)t * m.cols + (size_t)g * 32);
}

void launch_embed_rows(const QMat& emb, const uint32_t* tokens, uint32_t T, float* X, cudaStream_t stream) {
    const uint64_t n = (uint64_t)T * (emb.cols / 32);
    smallm_embed_rows_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(emb, tokens, T, X);
    SM_CUDA(cudaGetLastError());
}

__global__ void smallm_finalize_kernel(DecodeState* st, uint32_t* ids, uint32_t cap, TraceSlot* trace) {
    trace_mark(trace, 0);
    pdl_launch_dependents();
    pdl_wait();
    trace_mark(trace, 1);
    const uint32_t tok = argmax_key_index(st->argmax);
    st->token = tok;
    if (ids && st->step < cap) ids[st->step] = tok;
    st->step += 1;
    st->pos += 1;
    trace_mark(trace, 2);
}

void launch_finalize(DecodeState* st, uint32_t* ids, uint32_t cap, cudaStream_t stream, bool pdl, TraceSlot* trace) {
    void* args[] = {&st, &ids, &cap, &trace};
    launch_kernel_ex((const void*)smallm_finalize_kernel, dim3(1), dim3(1), 0, stream, pdl, args);
}

__global__ void smallm_finalize_tp_kernel(DecodeState* st, const unsigned long long* keys, int n, uint32_t* ids,
                                   uint32_t cap, unsigned int* epoch) {
    pdl_wait();
    if (epoch) *epoch += 1u;
    unsigned long long b = 0ull;
    for (int i = 0; i < n; ++i) b = keys[i] > b ? keys[i] : b;
    st->argmax = b;
    const uint32_t tok = argmax_key_index(b);
    st->token = tok;
    if (ids && st->step < cap) ids[st->step] = tok;
    st->step += 1;
    st->pos += 1;
    pdl_launch_dependents();
}

void launch_finalize_tp(DecodeState* st, const unsigned long long* keys, int n, uint32_t* ids, uint32_t cap,
                        unsigned int* epoch, cudaStream_t stream, bool pdl) {
    void* args[] = {&st, &keys, &n, &ids, &cap, &epoch};
    launch_kernel_ex((const void*)smallm_finalize_tp_kernel, dim3(1), dim3(1), 0, stream, pdl, args);
}

// ------------------------------------------------------------- op level --

// ops::rmsnorm (ops.cpp:29-40) on one CTA
__global__ void smallm_rmsnorm_kernel(const float* x, const float* w, uint32_t n, float eps, float* y) {
    __shared__ float red[32];
    float ss = 0.f;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) ss += x[i] * x[i];
    ss = block_sum(ss, red);
    const float inv = 1.0f / sqrtf(ss / (float)n + eps);
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) y[i] = (x[i] * inv) * w[i];
}

// ops::softmax (ops.cpp:43-57) in place on one CTA
__global__ void smallm_softmax_kernel(float* x, uint32_t n) {
    __shared__ float red[32];
    __shared__ float mx;
    float m = -INFINITY;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, x[i]);
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = red[0];
        for (int i = 1; i < (int)(blockDim.x >> 5); ++i) t = fmaxf(t, red[i]);
        mx = t;
    }
    __syncthreads();
    m = mx;
    float s = 0.f;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        const float e = expf(x[i] - m);
        x[i] = e;
        s += e;
    }
    s = block_sum(s, red);
    const float inv = 1.0f / s;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) x[i] *= inv;
}

// ops::silu (ops.cpp:60-65)
__global__ void smallm_silu_kernel(float* x, uint32_t n) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        const float v = x[i];
        x[i] = v / (1.0f + expf(-v));
    }
}

// ops::rope (ops.cpp:68-92) with the host table of (cos, sin)
__global__ void smallm_rope_kernel(float* x, uint32_t n_heads, uint32_t hd, const float2* cs) {
    const uint32_t half = hd / 2;
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_heads * half) return;
    const uint32_t h = i / half, k = i % half;
    float* v = x + (size_t)h * hd;
    const float x0 = v[k], x1 = v[k + half];
    const float2 c = cs[k];
    v[k] = fmaf(x0, c.x, -__fmul_rn(x1, c.y));
    v[k + half] = fmaf(x0, c.y, __fmul_rn(x1, c.x));
}

void launch_rmsnorm(const float* x, const float* w, uint32_t n, float eps, float* y, cudaStream_t s) {
    smallm_rmsnorm_kernel<<<1, 1024, 0, s>>>(x, w, n, eps, y);
    SM_CUDA(cudaGetLastError());
}
void launch_softmax(float* x, uint32_t n, cudaStream_t s) {
    smallm_softmax_kernel<<<1, 1024, 0, s>>>(x, n);
    SM_CUDA(cudaGetLastError());
}
void launch_silu(float* x, uint32_t n, cudaStream_t s) {
    if (!n) return;
    smallm_silu_kernel<<<(n + 255) / 256, 256, 0, s>>>(x, n);
    SM_CUDA(cudaGetLastError());
}
void launch_rope(float* x, uint32_t n_heads, uint32_t head_dim, const float2* cs, cudaStream_t s) {
    const uint32_t n = n_heads * (head_dim / 2);
    if (!n) return;
    smallm_rope_kernel<<<(n + 255) / 256, 256, 0, s>>>(x, n_heads, head_dim, cs);
    SM_CUDA(cudaGetLastError());
}

void rope_table(uint32_t hd, uint32_t positions, float base, std::vector<float2>& out, uint32_t first_pos) {
    const uint32_t half = hd / 2;
    out.resize((size_t)positions * half);
    std::vector<float> freq(half);
    for (uint32_t i = 0; i < half; ++i) {
        const float e = static_cast<float>(2 * i) / static_cast<float>(hd);
        freq[i] = 1.0f / std::pow(base, e);
    }
    for (uint32_t p = 0; p < positions; ++p)
        for (uint32_t i = 0; i < half; ++i) {
            const float th = static_cast<float>(p + first_pos) * freq[i];
            out[(size_t)p * half + i] = make_float2(std::cos(th), std::sin(th));
        }
}

// ----------------------------------------------------------------- GEMV --

__device__ unsigned int g_gemv_err;  // set by a bounded wait that gave up

template <class Fmt, int W>
static const void* pick(int pro, int epi) {
    if (pro == PRO_PLAIN && epi == EPI_STORE) return (const void*)smallm_qgemv_kernel<Fmt, PRO_PLAIN, EPI_STORE, W>;
    if (pro == PRO_PLAIN && epi == EPI_RESIDUAL) return (const void*)smallm_qgemv_kernel<Fmt, PRO_PLAIN, EPI_RESIDUAL, W>;
    if (pro == PRO_RMS && epi == EPI_STORE) return (const void*)smallm_qgemv_kernel<Fmt, PRO_RMS, EPI_STORE, W>;
    if (pro == PRO_RMS && epi == EPI_QKV) return (const void*)smallm_qgemv_kernel<Fmt, PRO_RMS, EPI_QKV, W>;
    if (pro == PRO_RMS && epi == EPI_SWIGLU) return (const void*)smallm_qgemv_kernel<Fmt, PRO_RMS, EPI_SWIGLU, W>;
    if (pro == PRO_RMS && epi == EPI_LOGITS) return (const void*)smallm_qgemv_kernel<Fmt, PRO_RMS, EPI_LOGITS, W>;
    // tensor parallel: row-parallel partials to peers, and the GEMVs that sum them
    if (pro == PRO_PLAIN && epi == EPI_PEER) return (const void*)smallm_qgemv_kernel<Fmt, PRO_PLAIN, EPI_PEER, W>;
    if (pro == PRO_RMS_SUM && epi == EPI_STORE) return (const void*)smallm_qgemv_kernel<Fmt, PRO_RMS_SUM, EPI_STORE, W>;
    if (pro == PRO_RMS_SUM && epi == EPI_QKV) return (const void*)smallm_qgemv_kernel<Fmt, PRO_RMS_SUM, EPI_QKV, W>;
    if (pro == PRO_RMS_SUM && epi == EPI_SWIGLU) return (const void*)smallm_qgemv_kernel<Fmt, PRO_RMS_SUM, EPI_SWIGLU, W>;
    if (pro == PRO_RMS_SUM && epi == EPI_LOGITS) return (const void*)smallm_qgemv_kernel<Fmt, PRO_RMS_SUM, EPI_LOGITS, W>;
    // the O projection after a multi-part attention: merge the parts as x is staged
    if (pro == PRO_MERGE && epi == EPI_RESIDUAL) return (const void*)smallm_qgemv_kernel<Fmt, PRO_MERGE, EPI_RESIDUAL, W>;
    if (pro == PRO_MERGE && epi == EPI_PEER) return (const void*)smallm_qgemv_kernel<Fmt, PRO_MERGE, EPI_PEER, W>;
    throw Error(1, "gemv: unsupported prologue/epilogue combination");
}

static const void* gemv_kernel_for(uint32_t type, int pro, int epi, uint32_t warps) {
    switch (type) {
        case SM_T_F32: return pick<FmtF32, 16>(pro, epi);
        case SM_T_Q4_0: return warps == 22 ? pick<FmtQ4_0, 22>(pro, epi) : pick<FmtQ4_0, 16>(pro, epi);
        case SM_T_Q8_0: return pick<FmtQ8_0, 16>(pro, epi);
        case SM_T_Q4_K: return pick<FmtQ4K, 16>(pro, epi);
        case SM_T_Q6_K: return pick<FmtQ6K, 16>(pro, epi);
        default: throw Error(2, "unsupported tensor type: " + std::to_string(type));
    }
}

constexpr size_t kSmemLimit = 227 * 1024;
constexpr uint32_t kMaxStages = 32;

// Consumer warps of the kernel for a matrix (gemv.cuh, kGemvMaxWarps).
static uint32_t gemv_warps(const QMat& m) {
    return m.type == SM_T_Q4_0 && m.units >= 256 ? 22u : 16u;
}

// Tiles of 4 rows; as many stages as shared memory (at most smem_cap bytes,
// 0 = the 227 KB limit) holds after the staged x.  The W consumer warps form
// NG <= 8 groups with private rings of >= 2 stages each, NG as large as the
// stages allow; a group has the fewest warps that still need the minimum
// number of 32-unit sweeps over K (measured: 448-unit rows run faster on 7-8
// warps with full sweeps than on 16 with 28 of 32 lanes busy).  Warps left
// over idle in the tile loop but share the x staging (measured on Q4_0
// 14336x4096: 11 groups of 2 warps, 9.51 us; 8 groups, 8.94 us).
constexpr uint32_t kGemvMaxGroups = 8;
GemvPlan gemv_plan(const QMat& m, size_t smem_cap) {
    GemvPlan pl;
    const size_t limit = smem_cap && smem_cap < kSmemLimit ? smem_cap : kSmemLimit;
    const uint32_t W = gemv_warps(m);
    pl.warps = W;
    // x records: three digits per 32-element block
    pl.xbytes = m.type == SM_T_F32 ? (size_t)m.cols * 4 : (size_t)(m.cols / 32) * kXrecBytes;
    // per stage: the tile, three mbarriers, the group's partial sums
    const size_t misc = kGemvMaxWarps * 4 + kGemvMaxWarps * 8 + 128;
    const uint32_t rt = 4;
    const size_t sb = (size_t)rt * m.row_stride;
    const size_t per_stage = sb + 24 + (size_t)W * 4 * 4;
    if (pl.xbytes + misc + 2 * per_stage > limit)
        throw Error(1, "gemv: rows of " + std::to_string(m.cols) + " columns do not fit the shared-memory pipeline");
    uint32_t smax = (uint32_t)((limit - pl.xbytes - misc) / per_stage);
    if (smax > kMaxStages) smax = kMaxStages;
    uint32_t ng = std::min(std::min(W / 2, kGemvMaxGroups), smax / 2);
    if (ng < 1) ng = 1;
    const uint32_t gmax = W / ng;
    const uint32_t sweeps = (m.units + 32 * gmax - 1) / (32 * gmax);
    uint32_t g = gmax;
    while (g > 1 && (m.units + 32 * (g - 1) - 1) / (32 * (g - 1)) <= sweeps) --g;
    pl.ngroups = ng;
    pl.gsize = g;
    pl.kring = smax / ng;
    pl.rt = rt;
    pl.stages = ng * pl.kring;
    pl.smem = pl.xbytes + (size_t)pl.stages * sb + 24 * (size_t)pl.stages + 8 + kGemvMaxWarps * 4 +
              kGemvMaxWarps * 8 + (size_t)pl.stages * g * 4 * 4;
    return pl;
}

unsigned int* device_error_flag() {
    static std::mutex mu;
    static std::unordered_map<int, unsigned int*> ptr;
    int dev = 0;
    SM_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> g(mu);
    auto it = ptr.find(dev);
    if (it == ptr.end()) {
        void* pe = nullptr;
        SM_CUDA(cudaGetSymbolAddress(&pe, g_gemv_err));
        it = ptr.emplace(dev, static_cast<unsigned int*>(pe)).first;
    }
    return it->second;
}

void set_smem_limit_once(const void* fn, int bytes) {
    static std::mutex mu;
    static std::set<std::tuple<int, const void*, int>> done;  // (device, kernel, bytes)
    int dev = 0;
    SM_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> g(mu);
    if (done.count({dev, fn, bytes})) return;
    SM_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    done.insert({dev, fn, bytes});
}

void launch_gemv(const QMat& m, int pro, int epi, const GemvArgs& a, cudaStream_t stream, bool pdl) {
    const GemvPlan pl = gemv_plan(m, a.smem_cap);
    const void* fn = gemv_kernel_for(m.type, pro, epi, pl.warps);
    unsigned int* err = device_error_flag();
    set_smem_limit_once(fn, (int)kSmemLimit);
    const uint32_t ntiles = m.rows_pad / pl.rt;
    uint32_t grid = (uint32_t)device_sm_count();
    if (grid > ntiles) grid = ntiles;

    GemvParams p{};
    p.w = m.base;
    p.row_stride = m.row_stride;
    p.rows = m.rows;
    p.rows_pad = m.rows_pad;
    p.cols = m.cols;
    p.units = m.units;
    p.rt = pl.rt;
    p.stages = pl.stages;
    p.ngroups = pl.ngroups;
    p.gsize = pl.gsize;
    p.kring = pl.kring;
    p.xbytes = (uint32_t)pl.xbytes;
    // hold back the ring fill behind x staging only when the rings cannot take
    // all of a CTA's tiles (measured: -0.9 us on 28672x4096 and 4096x14336 in
    // the decode step, +0.2 us on the 6144 / 4096-row matrices)
    p.hold = (ntiles + grid - 1) / grid > pl.stages ? 1u : ~0u;
    p.x = a.x;
    p.norm_w = a.norm_w;
    p.eps = a.eps;
    p.y = a.y;
    p.bias = a.bias;
    p.q_rows = a.q_rows;
    p.k_rows = a.k_rows;
    p.head_dim = a.head_dim;
    p.max_ctx = a.max_ctx;
    p.qout = a.qout;
    p.kcache = a.kcache;
    p.vcache = a.vcache;
    p.rope = a.rope;
    p.pos = a.pos;
    p.argmax = a.argmax;
    p.row_offset = a.row_offset;
    p.err = err;
    p.trace = a.trace;
    p.x_res = a.x_res;
    p.x_out = a.x_out;
    p.rx = a.rx;
    p.rx_flag = a.rx_flag;
    for (int r = 0; r < kMaxTPRanks; ++r) {
        p.peer_out[r] = a.peer_out[r];
        p.peer_flag[r] = a.peer_flag[r];
    }
    p.done_ctr = a.done_ctr;
    p.epoch = a.epoch;
    p.tp = a.tp;
    p.merge_parts = a.merge_parts < 1 ? 1 : a.merge_parts;
    p.merge_hd = a.merge_hd;
    p.merge_ml = a.merge_ml;
    if (pro == GEMV_PRO_MERGE && (p.merge_parts < 2 || !a.merge_ml || a.merge_hd == 0 || a.merge_hd % 4 ||
                                  m.cols % a.merge_hd))
        throw Error(1, "gemv: an attention-partial merge needs >= 2 parts, their (max, sum) and whole heads");
    if ((pro == GEMV_PRO_RMS_SUM || epi == GEMV_EPI_PEER) &&
        (a.tp < 1 || a.tp > (uint32_t)kMaxTPRanks || !a.epoch || (epi == GEMV_EPI_PEER && !a.done_ctr) ||
         (pro == GEMV_PRO_RMS_SUM && (!a.x_res || !a.x_out || !a.rx || !a.rx_flag))))
        throw Error(1, "gemv: incomplete tensor-parallel arguments");
    void* args[] = {&p};
    launch_kernel_ex(fn, dim3(grid), dim3((pl.warps + 1) * 32), pl.smem, stream, pdl, args);
}

unsigned int gemv_error_flags(bool clear) {
    unsigned int v = 0;
    SM_CUDA(cudaMemcpyFromSymbol(&v, g_gemv_err, sizeof(v)));
    if (clear && v) {
        unsigned int z = 0;
        SM_CUDA(cudaMemcpyToSymbol(g_gemv_err, &z, sizeof(z)));
    }
    return v;
}

}  // namespace smallm
