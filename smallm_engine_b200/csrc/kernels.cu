// Repack, dequantisation, embedding, attention, step bookkeeping and the
// op-level kernels, plus the GEMV launcher.
#include <cmath>
#include <cstring>
#include <mutex>
#include <unordered_map>

#include "engine.h"
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

void qmat_alloc(QMat& m, uint32_t type, uint32_t rows, uint32_t cols) {
    if (!type_supported(type)) throw Error(2, "unsupported tensor type: " + std::to_string(type));
    const uint32_t be = type_block_elems(type);
    if (cols == 0 || rows == 0 || cols % (be < 32 ? 32 : be))
        throw Error(1, "matrix shape " + std::to_string(rows) + "x" + std::to_string(cols) +
                           " is not a whole number of blocks for type " + std::to_string(type));
    m.type = type;
    m.rows = rows;
    m.rows_pad = (rows + 7) / 8 * 8;
    m.cols = cols;
    m.units = cols / unit_elems(type);
    m.gguf_bytes = (uint64_t)rows * type_row_bytes(type, cols);
    const uint64_t R = m.rows_pad;
    uint64_t qb = 0, sb = 0, db = 0;
    switch (type) {
        case SM_T_F32: qb = R * cols * 4; break;
        case SM_T_Q4_0: qb = R * m.units * 16; sb = R * m.units * 2; break;
        case SM_T_Q8_0: qb = R * m.units * 32; sb = R * m.units * 2; break;
        case SM_T_Q4_K: qb = R * (cols / 256) * 144; break;
        case SM_T_Q6_K: qb = R * m.units * 48; sb = R * m.units * 4; db = R * (cols / 256) * 2; break;
    }
    auto al = [](uint64_t v) { return (v + 255) / 256 * 256; };
    m.dev_bytes = al(qb) + al(sb) + al(db);
    SM_CUDA(cudaMalloc(&m.base, m.dev_bytes));
    m.q = m.base;
    m.s = sb ? m.base + al(qb) : nullptr;
    m.d = db ? m.base + al(qb) + al(sb) : nullptr;
}

void qmat_free(QMat& m) {
    if (m.base) cudaFree(m.base);
    m = QMat{};
}

// One thread per (storage row, GGUF block) for the 32-element block formats
// and F32 (32-element units), copying quants and scales into separate
// aligned streams.  Source blocks are byte-addressed (18/34-byte blocks are
// not aligned).
__global__ void repack_blocks_kernel(const uint8_t* src, uint64_t src_row_bytes, uint64_t col_byte0,
                                     const uint32_t* row_map, uint32_t rows, uint32_t rows_pad,
                                     uint32_t nunits, uint32_t type, uint8_t* q, uint8_t* s) {
    const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (uint64_t)rows_pad * nunits) return;
    const uint32_t p = (uint32_t)(idx / nunits), u = (uint32_t)(idx % nunits);
    const uint32_t srow = row_map ? row_map[p] : (p < rows ? p : 0xFFFFFFFFu);
    const uint32_t bb = type == SM_T_Q4_0 ? 18 : (type == SM_T_Q8_0 ? 34 : 128);
    const uint32_t qb = type == SM_T_Q4_0 ? 16 : (type == SM_T_Q8_0 ? 32 : 128);
    uint8_t* qo = q + idx * qb;
    if (srow == 0xFFFFFFFFu) {
        for (uint32_t i = 0; i < qb; ++i) qo[i] = 0;
        if (s) { s[idx * 2] = 0; s[idx * 2 + 1] = 0; }
        return;
    }
    const uint8_t* b = src + (uint64_t)srow * src_row_bytes + col_byte0 + (uint64_t)u * bb;
    if (type == SM_T_F32) {
        for (uint32_t i = 0; i < 128; ++i) qo[i] = b[i];
    } else {
        s[idx * 2] = b[0];
        s[idx * 2 + 1] = b[1];
        for (uint32_t i = 0; i < qb; ++i) qo[i] = b[2 + i];
    }
}

// Q4_K: super-blocks are copied whole (row permutation / column slice only).
__global__ void repack_q4k_kernel(const uint8_t* src, uint64_t src_row_bytes, uint64_t col_byte0,
                                  const uint32_t* row_map, uint32_t rows, uint32_t rows_pad, uint32_t nsb,
                                  uint8_t* q) {
    const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (uint64_t)rows_pad * nsb) return;
    const uint32_t p = (uint32_t)(idx / nsb), k = (uint32_t)(idx % nsb);
    const uint32_t srow = row_map ? row_map[p] : (p < rows ? p : 0xFFFFFFFFu);
    uint8_t* o = q + idx * 144;
    if (srow == 0xFFFFFFFFu) {
        for (int i = 0; i < 144; ++i) o[i] = 0;
        return;
    }
    const uint8_t* b = src + (uint64_t)srow * src_row_bytes + col_byte0 + (uint64_t)k * 144;
    for (int i = 0; i < 144; ++i) o[i] = b[i];
}

// Q6_K: decode the 256 6-bit codes of a GGUF super-block (ql/qh layout of
// src/core/tensor.cpp:93-100) and re-encode them per 64-element unit: 32
// nibble bytes (byte k: element k low, element 32+k high) and 16 bytes of
// 2-bit high parts (byte k: elements k, 16+k, 32+k, 48+k).  The 16 int8
// scales keep their order (element e uses scale e/16) and d goes to its own
// stream.  Lossless: every code and scale bit is preserved.
__global__ void repack_q6k_kernel(const uint8_t* src, uint64_t src_row_bytes, uint64_t col_byte0,
                                  const uint32_t* row_map, uint32_t rows, uint32_t rows_pad, uint32_t nsb,
                                  uint8_t* q, uint8_t* s, uint8_t* d) {
    const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (uint64_t)rows_pad * nsb) return;
    const uint32_t p = (uint32_t)(idx / nsb), k = (uint32_t)(idx % nsb);
    const uint32_t srow = row_map ? row_map[p] : (p < rows ? p : 0xFFFFFFFFu);
    uint8_t* qo = q + idx * 192;
    uint8_t* so = s + idx * 16;
    uint8_t* dout = d + idx * 2;
    if (srow == 0xFFFFFFFFu) {
        for (int i = 0; i < 192; ++i) qo[i] = 0;
        for (int i = 0; i < 16; ++i) so[i] = 0;
        dout[0] = dout[1] = 0;
        return;
    }
    const uint8_t* b = src + (uint64_t)srow * src_row_bytes + col_byte0 + (uint64_t)k * 210;
    for (int i = 0; i < 192; ++i) qo[i] = 0;
    for (int E = 0; E < 256; ++E) {
        const int h = E >> 7, w = E & 127, m = w >> 5, l = w & 31;
        const uint8_t qlb = b[h * 64 + l + ((m & 1) ? 32 : 0)];
        const uint8_t qhb = b[128 + h * 32 + l];
        const int lo4 = (m < 2) ? (qlb & 0xF) : (qlb >> 4);
        const int hi2 = (qhb >> (2 * m)) & 3;
        const int u = E >> 6, e = E & 63;
        uint8_t* ub = qo + u * 48;
        if (e < 32) ub[e] |= (uint8_t)lo4;
        else ub[e - 32] |= (uint8_t)(lo4 << 4);
        ub[32 + (e & 15)] |= (uint8_t)(hi2 << (2 * (e >> 4)));
    }
    for (int i = 0; i < 16; ++i) so[i] = b[192 + i];
    dout[0] = b[208];
    dout[1] = b[209];
}

void qmat_repack(QMat& m, const RepackSource& s, cudaStream_t stream) {
    const uint64_t rb = type_row_bytes(m.type, s.src_cols);
    const uint64_t cb0 = type_row_bytes(m.type, s.col0);
    const int T = 256;
    if (m.type == SM_T_Q4_K) {
        const uint32_t nsb = m.cols / 256;
        const uint64_t n = (uint64_t)m.rows_pad * nsb;
        repack_q4k_kernel<<<(unsigned)((n + T - 1) / T), T, 0, stream>>>(s.src, rb, cb0, s.row_map, m.rows,
                                                                          m.rows_pad, nsb, m.q);
    } else if (m.type == SM_T_Q6_K) {
        const uint32_t nsb = m.cols / 256;
        const uint64_t n = (uint64_t)m.rows_pad * nsb;
        repack_q6k_kernel<<<(unsigned)((n + T - 1) / T), T, 0, stream>>>(s.src, rb, cb0, s.row_map, m.rows,
                                                                          m.rows_pad, nsb, m.q, m.s, m.d);
    } else {
        const uint64_t n = (uint64_t)m.rows_pad * m.units;
        repack_blocks_kernel<<<(unsigned)((n + T - 1) / T), T, 0, stream>>>(
            s.src, rb, cb0, s.row_map, m.rows, m.rows_pad, m.units, m.type, m.q, m.s);
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
            SM_CUDA(cudaMalloc(&dmap, row_map.size() * 4));
            SM_CUDA(cudaMemcpyAsync(dmap, row_map.data(), row_map.size() * 4, cudaMemcpyHostToDevice, stream));
        }
        RepackSource s{stage, src_cols, col0, dmap};
        qmat_repack(m, s, stream);
        SM_CUDA(cudaStreamSynchronize(stream));
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

// 32 consecutive elements (group g of storage row r) of a repacked matrix,
// with the reference's exact arithmetic per type (src/core/tensor.cpp:20-111;
// Q4_K as gguf-py's Q4_K.dequantize_blocks).
__device__ void dequant_group(const QMat m, uint32_t r, uint32_t g, float* out) {
    switch (m.type) {
        case SM_T_F32: {
            const float* w = reinterpret_cast<const float*>(m.q) + (size_t)r * m.cols + (size_t)g * 32;
            for (int i = 0; i < 32; ++i) out[i] = w[i];
            break;
        }
        case SM_T_Q4_0: {
            const size_t i = (size_t)r * m.units + g;
            const uint8_t* q = m.q + i * 16;
            const float d = f16_exact(m.s[i * 2] | (m.s[i * 2 + 1] << 8));
            for (int k = 0; k < 16; ++k) {
                out[k] = __fmul_rn(d, (float)((int)(q[k] & 0xF) - 8));
                out[k + 16] = __fmul_rn(d, (float)((int)(q[k] >> 4) - 8));
            }
            break;
        }
        case SM_T_Q8_0: {
            const size_t i = (size_t)r * m.units + g;
            const int8_t* q = reinterpret_cast<const int8_t*>(m.q + i * 32);
            const float d = f16_exact(m.s[i * 2] | (m.s[i * 2 + 1] << 8));
            for (int k = 0; k < 32; ++k) out[k] = __fmul_rn(d, (float)q[k]);
            break;
        }
        case SM_T_Q4_K: {
            const uint32_t nsb = m.cols / 256, sbi = g / 8, j = g % 8;
            const uint8_t* b = m.q + ((size_t)r * nsb + sbi) * 144;
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
                out[k] = __fsub_rn(__fmul_rn(d1, (float)v), m1);
            }
            break;
        }
        case SM_T_Q6_K: {
            const uint32_t u = g / 2, sub = g % 2;
            const size_t i = (size_t)r * m.units + u;
            const uint8_t* ub = m.q + i * 48;
            const int8_t* sc = reinterpret_cast<const int8_t*>(m.s + i * 4);
            const size_t di = (size_t)r * (m.cols / 256) + u / 4;
            const float d = f16_exact(m.d[di * 2] | (m.d[di * 2 + 1] << 8));
            for (int k = 0; k < 32; ++k) {
                const int e = (int)sub * 32 + k;
                const int lo4 = e < 32 ? (ub[e] & 0xF) : (ub[e - 32] >> 4);
                const int hi2 = (ub[32 + (e & 15)] >> (2 * (e >> 4))) & 3;
                const int code = lo4 | (hi2 << 4);
                out[k] = __fmul_rn(__fmul_rn(d, (float)sc[e >> 4]), (float)(code - 32));
            }
            break;
        }
    }
}

__global__ void qmat_dequant_kernel(const QMat m, float* y) {
    const uint32_t groups = m.cols / 32;
    const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (uint64_t)m.rows * groups) return;
    const uint32_t r = (uint32_t)(idx / groups), g = (uint32_t)(idx % groups);
    dequant_group(m, r, g, y + (size_t)r * m.cols + (size_t)g * 32);
}

void launch_qmat_dequant(const QMat& m, float* y, cudaStream_t stream) {
    const uint64_t n = (uint64_t)m.rows * (m.cols / 32);
    qmat_dequant_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(m, y);
    SM_CUDA(cudaGetLastError());
}

// Raw GGUF blocks (contiguous, byte-addressed) -> f32, one thread per 32
// elements, same arithmetic as dequant_group.
__global__ void dequant_raw_kernel(uint32_t type, const uint8_t* src, uint64_t count, float* out) {
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
    dequant_raw_kernel<<<(unsigned)((groups + 255) / 256), 256, 0, stream>>>(type, src, count, out);
    SM_CUDA(cudaGetLastError());
}

// --------------------------------------------------------------- launch --

static void launch_ex(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl,
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

__global__ void embed_kernel(const QMat m, DecodeState* st, float* x) {
    pdl_wait();
    uint32_t tok = st->token;
    if (tok >= m.rows) tok = 0;  // the host validates ids; never read outside the table
    const uint32_t groups = m.cols / 32;
    for (uint32_t g = threadIdx.x; g < groups; g += blockDim.x) dequant_group(m, tok, g, x + (size_t)g * 32);
    if (threadIdx.x == 0) st->argmax = 0ull;
    pdl_launch_dependents();
}

void launch_embed(const QMat& emb, DecodeState* st, float* x, cudaStream_t stream, bool pdl) {
    QMat m = emb;
    void* args[] = {&m, &st, &x};
    launch_ex((const void*)embed_kernel, dim3(1), dim3(256), 0, stream, pdl, args);
}

__global__ void finalize_kernel(DecodeState* st, uint32_t* ids, uint32_t cap) {
    pdl_wait();
    const uint32_t tok = argmax_key_index(st->argmax);
    st->token = tok;
    if (ids && st->step < cap) ids[st->step] = tok;
    st->step += 1;
    st->pos += 1;
    pdl_launch_dependents();
}

void launch_finalize(DecodeState* st, uint32_t* ids, uint32_t cap, cudaStream_t stream, bool pdl) {
    void* args[] = {&st, &ids, &cap};
    launch_ex((const void*)finalize_kernel, dim3(1), dim3(1), 0, stream, pdl, args);
}

__global__ void finalize_tp_kernel(DecodeState* st, const unsigned long long* keys, int n, uint32_t* ids,
                                   uint32_t cap) {
    pdl_wait();
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
                        cudaStream_t stream, bool pdl) {
    void* args[] = {&st, &keys, &n, &ids, &cap};
    launch_ex((const void*)finalize_tp_kernel, dim3(1), dim3(1), 0, stream, pdl, args);
}

// ------------------------------------------------------------- attention --
//
// qwen2_model.cpp:111-133: for each query head h (kv head h / group):
// scores_t = dot(q_h, k_t) / sqrt(hd) for t <= pos, softmax, out_h = sum_t p_t v_t.
// Grid (n_kv, n_split): CTA (g, s) handles one chunk of positions for the
// `group` query heads sharing KV head g, so every K/V row is read once per
// step.  Partials (unnormalised out, running max, sum) go to scratch; the
// last CTA of each KV head (atomic ticket, no waiting) merges them.

constexpr int kAttnThreads = 128;
constexpr uint32_t kAttnMinChunk = 16;
constexpr int kAttnMaxGroup = 8;

uint32_t attention_splits(uint32_t n_kv, uint32_t max_ctx, int sm_count) {
    uint32_t s = (uint32_t)(2 * sm_count + n_kv - 1) / n_kv;
    const uint32_t cap = (max_ctx + kAttnMinChunk - 1) / kAttnMinChunk;
    if (s > cap) s = cap;
    return s < 1 ? 1 : s;
}

size_t attention_partial_floats(uint32_t n_heads, uint32_t hd, uint32_t n_split) {
    return (size_t)n_heads * n_split * (hd + 2);
}

__host__ __device__ static uint32_t attn_chunk_max(uint32_t max_ctx, uint32_t n_split) {
    uint32_t c = (max_ctx + n_split - 1) / n_split;
    return c < kAttnMinChunk ? kAttnMinChunk : c;
}

template <int HD>
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const AttnArgs a) {
    constexpr int EPL = HD / 32;  // elements per lane
    extern __shared__ float sm[];
    const uint32_t G = a.n_heads / a.n_kv;
    const uint32_t g = blockIdx.x, split = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nw = kAttnThreads / 32;
    const uint32_t chmax = attn_chunk_max(a.max_ctx, a.n_split);
    float* qs = sm;                    // [G][HD]
    float* sc = qs + G * HD;           // [G][chmax]
    float* ml = sc + G * chmax;        // [G][2] (max, sum)
    float* red = ml + 2 * kAttnMaxGroup;  // [PARTS-1][HD][kAttnMaxGroup] (slice-sum exchange)
    __shared__ unsigned int is_last;

    pdl_wait();
    const uint32_t n = *a.pos + 1;
    uint32_t chunk = (n + a.n_split - 1) / a.n_split;
    if (chunk < kAttnMinChunk) chunk = kAttnMinChunk;
    const uint32_t t0 = split * chunk;
    const uint32_t t1 = min(n, t0 + chunk);
    const uint32_t len = t0 < t1 ? t1 - t0 : 0;

    for (uint32_t i = tid; i < G * HD; i += kAttnThreads) qs[i] = a.q[(size_t)g * G * HD + i];
    __syncthreads();

    const float scale = 1.0f / sqrtf((float)HD);
    const float* kb = a.kcache + (size_t)g * a.max_ctx * HD;
    const float* vb = a.vcache + (size_t)g * a.max_ctx * HD;

    // phase A: scores, one warp per position, lanes split the head dim
    for (uint32_t t = t0 + warp; t < t1; t += nw) {
        const float* kr = kb + (size_t)t * HD;
        float kv[EPL];
#pragma unroll
        for (int e = 0; e < EPL; ++e) kv[e] = kr[lane + 32 * e];
#pragma unroll
        for (int h = 0; h < kAttnMaxGroup; ++h) {
            if (h < (int)G) {
                float p = 0.f;
#pragma unroll
                for (int e = 0; e < EPL; ++e) p = fmaf(qs[h * HD + lane + 32 * e], kv[e], p);
                p = warp_sum(p);
                if (lane == 0) sc[h * chmax + (t - t0)] = p * scale;
            }
        }
    }
    __syncthreads();

    // phase B: per-head max and exp (ops::softmax, ops.cpp:43-57, unnormalised)
    for (uint32_t h = warp; h < G; h += nw) {
        float m = -INFINITY;
        for (uint32_t i = lane; i < len; i += 32) m = fmaxf(m, sc[h * chmax + i]);
        m = warp_max(m);
        float l = 0.f;
        for (uint32_t i = lane; i < len; i += 32) {
            const float e = expf(sc[h * chmax + i] - m);
            sc[h * chmax + i] = e;
            l += e;
        }
        l = warp_sum(l);
        if (lane == 0) {
            ml[2 * h] = m;
            ml[2 * h + 1] = l;
        }
    }
    __syncthreads();

    // phase C: o[h][d] = sum_t p[h][t] * v[t][d]; thread -> (d, slice of the
    // positions); the PARTS slices are summed through shared memory
    constexpr int PARTS = kAttnThreads / HD;  // 4, 2, 1 for HD = 32, 64, 128
    const int d = tid % HD, part_i = tid / HD;
    float acc[kAttnMaxGroup];
#pragma unroll
    for (int h = 0; h < kAttnMaxGroup; ++h) acc[h] = 0.f;
    for (uint32_t i = part_i; i < len; i += PARTS) {
        const float v = vb[(size_t)(t0 + i) * HD + d];
#pragma unroll
        for (int h = 0; h < kAttnMaxGroup; ++h)
            if (h < (int)G) acc[h] = fmaf(sc[h * chmax + i], v, acc[h]);
    }
    if constexpr (PARTS > 1) {
        if (part_i > 0)
            for (int h = 0; h < kAttnMaxGroup; ++h) red[((part_i - 1) * HD + d) * kAttnMaxGroup + h] = acc[h];
        __syncthreads();
    }
    float* part = a.partial + ((size_t)g * a.n_split + split) * G * (HD + 2);
    if (part_i == 0) {
        for (uint32_t h = 0; h < G; ++h) {
            float o = acc[h];
#pragma unroll
            for (int k = 1; k < PARTS; ++k) o += red[((k - 1) * HD + d) * kAttnMaxGroup + h];
            part[h * (HD + 2) + d] = o;
            if (d == 0) {
                part[h * (HD + 2) + HD] = len ? ml[2 * h] : -INFINITY;
                part[h * (HD + 2) + HD + 1] = len ? ml[2 * h + 1] : 0.f;
            }
        }
    }

    // last CTA of this KV head merges the n_split partials
    __threadfence();
    __syncthreads();
    if (tid == 0) is_last = (atomicAdd(&a.counter[g], 1u) == a.n_split - 1) ? 1u : 0u;
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    const float* base = a.partial + (size_t)g * a.n_split * G * (HD + 2);
    const uint32_t nact = min(a.n_split, (n + chunk - 1) / chunk);
    for (uint32_t o = tid; o < G * HD; o += kAttnThreads) {
        const uint32_t h = o / HD, dd = o % HD;
        float M = -INFINITY;
        for (uint32_t s = 0; s < nact; ++s) M = fmaxf(M, base[(s * G + h) * (HD + 2) + HD]);
        float L = 0.f, O = 0.f;
        for (uint32_t s = 0; s < nact; ++s) {
            const float* r = base + (s * G + h) * (HD + 2);
            const float w = expf(r[HD] - M);
            L = fmaf(w, r[HD + 1], L);
            O = fmaf(w, r[dd], O);
        }
        a.out[((size_t)g * G + h) * HD + dd] = O / L;
    }
    if (tid == 0) a.counter[g] = 0u;
    pdl_launch_dependents();
}

void launch_attention(const AttnArgs& a, cudaStream_t stream, bool pdl) {
    const uint32_t G = a.n_heads / a.n_kv;
    if (G > (uint32_t)kAttnMaxGroup || a.n_heads % a.n_kv)
        throw Error(1, "attention: unsupported head grouping");
    const uint32_t chmax = attn_chunk_max(a.max_ctx, a.n_split);
    const size_t smem = sizeof(float) * ((size_t)G * a.hd + (size_t)G * chmax + 2 * kAttnMaxGroup +
                                         (size_t)(kAttnThreads - a.hd) * kAttnMaxGroup);
    AttnArgs aa = a;
    void* args[] = {&aa};
    const void* fn;
    if (a.hd == 32) fn = (const void*)attention_kernel<32>;
    else if (a.hd == 64) fn = (const void*)attention_kernel<64>;
    else if (a.hd == 128) fn = (const void*)attention_kernel<128>;
    else throw Error(1, "attention: head_dim must be 32, 64 or 128");
    if (smem > 200 * 1024) throw Error(1, "attention: context too long for one split");
    static bool attr_set = false;
    if (!attr_set) {
        SM_CUDA(cudaFuncSetAttribute(attention_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        SM_CUDA(cudaFuncSetAttribute(attention_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        SM_CUDA(cudaFuncSetAttribute(attention_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        attr_set = true;
    }
    launch_ex(fn, dim3(a.n_kv, a.n_split), dim3(kAttnThreads), smem, stream, pdl, args);
}

// ------------------------------------------------------------- op level --

// ops::rmsnorm (ops.cpp:29-40) on one CTA
__global__ void rmsnorm_kernel(const float* x, const float* w, uint32_t n, float eps, float* y) {
    __shared__ float red[32];
    float ss = 0.f;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) ss += x[i] * x[i];
    ss = block_sum(ss, red);
    const float inv = 1.0f / sqrtf(ss / (float)n + eps);
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) y[i] = (x[i] * inv) * w[i];
}

// ops::softmax (ops.cpp:43-57) in place on one CTA
__global__ void softmax_kernel(float* x, uint32_t n) {
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
__global__ void silu_kernel(float* x, uint32_t n) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        const float v = x[i];
        x[i] = v / (1.0f + expf(-v));
    }
}

// ops::rope (ops.cpp:68-92) with the host table of (cos, sin)
__global__ void rope_kernel(float* x, uint32_t n_heads, uint32_t hd, const float2* cs) {
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
    rmsnorm_kernel<<<1, 1024, 0, s>>>(x, w, n, eps, y);
    SM_CUDA(cudaGetLastError());
}
void launch_softmax(float* x, uint32_t n, cudaStream_t s) {
    softmax_kernel<<<1, 1024, 0, s>>>(x, n);
    SM_CUDA(cudaGetLastError());
}
void launch_silu(float* x, uint32_t n, cudaStream_t s) {
    if (!n) return;
    silu_kernel<<<(n + 255) / 256, 256, 0, s>>>(x, n);
    SM_CUDA(cudaGetLastError());
}
void launch_rope(float* x, uint32_t n_heads, uint32_t head_dim, const float2* cs, cudaStream_t s) {
    const uint32_t n = n_heads * (head_dim / 2);
    if (!n) return;
    rope_kernel<<<(n + 255) / 256, 256, 0, s>>>(x, n_heads, head_dim, cs);
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

template <class Fmt, int PRO, int EPI>
static const void* gemv_fn() {
    return (const void*)gemv_kernel<Fmt, PRO, EPI, 2>;
}

template <class Fmt>
static const void* pick(int pro, int epi) {
    if (pro == PRO_PLAIN && epi == EPI_STORE) return gemv_fn<Fmt, PRO_PLAIN, EPI_STORE>();
    if (pro == PRO_PLAIN && epi == EPI_RESIDUAL) return gemv_fn<Fmt, PRO_PLAIN, EPI_RESIDUAL>();
    if (pro == PRO_RMS && epi == EPI_STORE) return gemv_fn<Fmt, PRO_RMS, EPI_STORE>();
    if (pro == PRO_RMS && epi == EPI_QKV) return gemv_fn<Fmt, PRO_RMS, EPI_QKV>();
    if (pro == PRO_RMS && epi == EPI_SWIGLU) return gemv_fn<Fmt, PRO_RMS, EPI_SWIGLU>();
    if (pro == PRO_RMS && epi == EPI_LOGITS) return gemv_fn<Fmt, PRO_RMS, EPI_LOGITS>();
    throw Error(1, "gemv: unsupported prologue/epilogue combination");
}

static const void* gemv_kernel_for(uint32_t type, int pro, int epi) {
    switch (type) {
        case SM_T_F32: return pick<FmtF32>(pro, epi);
        case SM_T_Q4_0: return pick<FmtQ4_0>(pro, epi);
        case SM_T_Q8_0: return pick<FmtQ8_0>(pro, epi);
        case SM_T_Q4_K: return pick<FmtQ4K>(pro, epi);
        case SM_T_Q6_K: return pick<FmtQ6K>(pro, epi);
        default: throw Error(2, "unsupported tensor type: " + std::to_string(type));
    }
}

struct KernelInfo {
    int blocks_per_sm = 0;
    size_t smem = 0;
};

void launch_gemv(const QMat& m, int pro, int epi, const GemvArgs& a, cudaStream_t stream, bool pdl) {
    static std::mutex mu;
    static std::unordered_map<const void*, KernelInfo> info;
    const void* fn = gemv_kernel_for(m.type, pro, epi);
    const size_t smem = (size_t)m.cols * 4 + (size_t)(m.cols / 32) * 4;
    int bps;
    {
        std::lock_guard<std::mutex> g(mu);
        KernelInfo& ki = info[fn];
        if (ki.smem != smem) {
            SM_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024));
            SM_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&ki.blocks_per_sm, fn, kGemvThreads, smem));
            ki.smem = smem;
        }
        bps = ki.blocks_per_sm;
    }
    if (bps < 1) throw Error(1, "gemv: kernel does not fit on an SM (cols too large)");
    const uint32_t tiles = m.rows_pad / 2;
    const uint32_t warps = kGemvThreads / 32;
    uint32_t grid = (tiles + warps - 1) / warps;
    const uint32_t cap = (uint32_t)(bps * device_sm_count());
    if (grid > cap) grid = cap;

    GemvParams p{};
    p.q = m.q;
    p.s = m.s;
    p.d = m.d;
    p.rows = m.rows;
    p.rows_pad = m.rows_pad;
    p.cols = m.cols;
    p.units = m.units;
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
    void* args[] = {&p};
    launch_ex(fn, dim3(grid), dim3(kGemvThreads), smem, stream, pdl, args);
}

}  // namespace smallm
