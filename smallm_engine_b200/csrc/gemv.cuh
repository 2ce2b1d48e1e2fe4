// Batch-1 quantized GEMV for sm_100a: y = W . x with W in a repacked GGUF
// block layout streamed once from HBM.
//
// Design (bandwidth-bound, CUDA cores, no tensor cores):
//  * x (f32, K elements) is staged once per CTA in shared memory, optionally
//    RMS-normalised on the way in (fused ops::rmsnorm, src/core/ops.cpp:29-40).
//    The staging is XOR-swizzled per 16-byte granule so that the 32 lanes of
//    a warp, which read 32 different K-units at once, hit distinct banks.
//  * Persistent CTAs; each warp owns a tile of R consecutive (physical) rows
//    and its lanes stride the K dimension in "units" (one Q4_0/Q8_0 block of
//    32, or a quarter Q4_K/Q6_K super-block of 64 elements).  Every lane
//    issues 128-bit streaming loads, so a warp reads whole 512-byte segments.
//  * Dequantisation uses no int->float conversion instructions: a byte
//    permute builds 2^23 + q as an f32 bit pattern and one FADD removes the
//    offset exactly (byte_f in common.cuh).
//  * The R partial sums are combined with a reduce-scatter butterfly and
//    handed to a fused epilogue: plain store, residual add, Q/K/V bias + RoPE +
//    KV-cache append, SwiGLU, or logits + greedy argmax.
#pragma once

#include "common.cuh"

namespace smallm {

enum { PRO_PLAIN = 0, PRO_RMS = 1 };
enum { EPI_STORE = 0, EPI_RESIDUAL = 1, EPI_QKV = 2, EPI_SWIGLU = 3, EPI_LOGITS = 4 };

struct GemvParams {
    // repacked matrix (see repack kernels for the layouts)
    const uint8_t* q;
    const uint8_t* s;
    const uint8_t* d;
    uint32_t rows;      // logical rows; writes are masked to these
    uint32_t rows_pad;  // storage rows, a multiple of 8
    uint32_t cols;
    uint32_t units;     // cols / Fmt::UE
    // input vector and fused RMSNorm
    const float* x;
    const float* norm_w;
    float eps;
    // outputs
    float* y;           // STORE / RESIDUAL / SWIGLU / LOGITS destination
    const float* bias;  // optional per logical row bias (QKV)
    // QKV epilogue: physical rows [0, q_rows) are query pairs, [q_rows,
    // q_rows + k_rows) key pairs, the rest value rows (natural order).
    uint32_t q_rows, k_rows;
    uint32_t head_dim, max_ctx;
    float* qout;
    float* kcache;      // [n_kv][max_ctx][head_dim]
    float* vcache;
    const float2* rope; // [max_ctx][head_dim/2] (cos, sin)
    const uint32_t* pos;
    unsigned long long* argmax;
    uint32_t row_offset;  // LOGITS: global vocabulary index of storage row 0
};

// ---------------------------------------------------------------- formats --

// Q4_0: q stream [rows][units][16 B], s stream [rows][units] f16.
// Element i of a block is the low nibble of byte i, element i+16 the high
// nibble (src/core/tensor.cpp:57-63); value (q - 8) * d.
struct FmtQ4_0 {
    static constexpr int UE = 32, SUBS = 1, GS = 3;
    static constexpr bool XSUM = false;
    struct Raw { uint4 q; uint32_t s; };
    __device__ __forceinline__ static void load(const GemvParams& p, uint32_t row, uint32_t u, Raw& r) {
        size_t i = (size_t)row * p.units + u;
        r.q = ld_stream_u4(p.q + i * 16);
        r.s = ld_stream_u16(p.s + i * 2);
    }
    __device__ __forceinline__ static float dot(const Raw& r, int, const float (&x)[32], const float*, uint32_t) {
        const float M = 8388616.0f;  // 2^23 + 8
        const uint32_t w[4] = {r.q.x, r.q.y, r.q.z, r.q.w};
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            uint32_t lo = w[j] & 0x0F0F0F0Fu, hi = (w[j] >> 4) & 0x0F0F0F0Fu;
            a0 = fmaf(byte_f<0>(lo, M), x[4 * j + 0], a0);
            a1 = fmaf(byte_f<1>(lo, M), x[4 * j + 1], a1);
            a2 = fmaf(byte_f<2>(lo, M), x[4 * j + 2], a2);
            a3 = fmaf(byte_f<3>(lo, M), x[4 * j + 3], a3);
            a0 = fmaf(byte_f<0>(hi, M), x[16 + 4 * j + 0], a0);
            a1 = fmaf(byte_f<1>(hi, M), x[16 + 4 * j + 1], a1);
            a2 = fmaf(byte_f<2>(hi, M), x[16 + 4 * j + 2], a2);
            a3 = fmaf(byte_f<3>(hi, M), x[16 + 4 * j + 3], a3);
        }
        return ((a0 + a1) + (a2 + a3)) * h2f(r.s);
    }
};

// Q8_0: q stream [rows][units][32 B] (int8), s stream [rows][units] f16.
struct FmtQ8_0 {
    static constexpr int UE = 32, SUBS = 1, GS = 3;
    static constexpr bool XSUM = false;
    struct Raw { uint4 a, b; uint32_t s; };
    __device__ __forceinline__ static void load(const GemvParams& p, uint32_t row, uint32_t u, Raw& r) {
        size_t i = (size_t)row * p.units + u;
        r.a = ld_stream_u4(p.q + i * 32);
        r.b = ld_stream_u4(p.q + i * 32 + 16);
        r.s = ld_stream_u16(p.s + i * 2);
    }
    __device__ __forceinline__ static float dot(const Raw& r, int, const float (&x)[32], const float*, uint32_t) {
        const float M = 8388736.0f;  // 2^23 + 128 (bytes are biased by 128 first)
        const uint32_t w[8] = {r.a.x, r.a.y, r.a.z, r.a.w, r.b.x, r.b.y, r.b.z, r.b.w};
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            uint32_t u = w[j] ^ 0x80808080u;
            a0 = fmaf(byte_f<0>(u, M), x[4 * j + 0], a0);
            a1 = fmaf(byte_f<1>(u, M), x[4 * j + 1], a1);
            a2 = fmaf(byte_f<2>(u, M), x[4 * j + 2], a2);
            a3 = fmaf(byte_f<3>(u, M), x[4 * j + 3], a3);
        }
        return ((a0 + a1) + (a2 + a3)) * h2f(r.s);
    }
};

// Q4_K: GGUF super-blocks kept as they are, [rows][nsb][144 B] (144 = 9 x 16,
// so every super-block is 16-byte aligned): f16 d, f16 dmin, 12 bytes of
// 6-bit scales/mins, 128 bytes of nibbles.  A unit is a quarter super-block:
// sub-blocks 2k (low nibbles of qs[32k..32k+32)) and 2k+1 (high nibbles).
// Value of an element: (d*sc)*q - dmin*m (gguf-py Q4_K.dequantize_blocks).
struct FmtQ4K {
    static constexpr int UE = 64, SUBS = 2, GS = 4;
    static constexpr bool XSUM = true;
    struct Raw { uint4 h, a, b; };
    __device__ __forceinline__ static void load(const GemvParams& p, uint32_t row, uint32_t u, Raw& r) {
        const uint8_t* sb = p.q + ((size_t)row * (p.units >> 2) + (u >> 2)) * 144;
        r.h = ld_stream_u4(sb);
        r.a = ld_stream_u4(sb + 16 + (u & 3) * 32);
        r.b = ld_stream_u4(sb + 32 + (u & 3) * 32);
    }
    // 6-bit scale and min of sub-block j from the 12 packed bytes.
    __device__ __forceinline__ static void scale_min(const uint4& h, int j, int& sc, int& m) {
        const uint32_t s0 = h.y, s1 = h.z, s2 = h.w;  // scales bytes 0-3, 4-7, 8-11
        auto byte = [](uint32_t w, int k) { return (int)((w >> (8 * k)) & 0xFFu); };
        if (j < 4) {
            sc = byte(s0, j) & 63;
            m = byte(s1, j) & 63;
        } else {
            sc = (byte(s2, j - 4) & 0xF) | ((byte(s0, j - 4) >> 6) << 4);
            m = (byte(s2, j - 4) >> 4) | ((byte(s1, j - 4) >> 6) << 4);
        }
    }
    __device__ __forceinline__ static float dot(const Raw& r, int sub, const float (&x)[32], const float* xsum,
                                                uint32_t u) {
        const float M = 8388608.0f;  // 2^23
        const uint32_t w[8] = {r.a.x, r.a.y, r.a.z, r.a.w, r.b.x, r.b.y, r.b.z, r.b.w};
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            uint32_t n = sub ? ((w[j] >> 4) & 0x0F0F0F0Fu) : (w[j] & 0x0F0F0F0Fu);
            a0 = fmaf(byte_f<0>(n, M), x[4 * j + 0], a0);
            a1 = fmaf(byte_f<1>(n, M), x[4 * j + 1], a1);
            a2 = fmaf(byte_f<2>(n, M), x[4 * j + 2], a2);
            a3 = fmaf(byte_f<3>(n, M), x[4 * j + 3], a3);
        }
        int sc, m;
        scale_min(r.h, 2 * (u & 3) + sub, sc, m);
        const float d = h2f(r.h.x & 0xFFFFu), dmin = h2f(r.h.x >> 16);
        const float d1 = d * (float)sc, m1 = dmin * (float)m;
        return fmaf(d1, (a0 + a1) + (a2 + a3), -m1 * xsum[2 * u + sub]);
    }
};

// Q6_K re-encoded per 64-element unit (lossless re-arrangement of the 6-bit
// codes done by the repack kernel): q stream [rows][units][48 B] = 32 bytes
// of nibbles (byte k: element k low, element 32+k high) + 16 bytes of 2-bit
// high parts (byte k: elements k, 16+k, 32+k, 48+k in bits 0-1, 2-3, 4-5,
// 6-7); s stream [rows][units][4] int8 scales (one per 16 elements, element
// e of a super-block uses scale e/16); d stream [rows][nsb] f16.
// Value: (d*sc)*(q - 32) (src/core/tensor.cpp:97-106).
struct FmtQ6K {
    static constexpr int UE = 64, SUBS = 2, GS = 4;
    static constexpr bool XSUM = false;
    struct Raw { uint4 n0, n1, hb; uint32_t sc; uint32_t d; };
    __device__ __forceinline__ static void load(const GemvParams& p, uint32_t row, uint32_t u, Raw& r) {
        size_t i = (size_t)row * p.units + u;
        const uint8_t* qb = p.q + i * 48;
        r.n0 = ld_stream_u4(qb);
        r.n1 = ld_stream_u4(qb + 16);
        r.hb = ld_stream_u4(qb + 32);
        r.sc = ld_stream_u32(p.s + i * 4);
        r.d = ld_stream_u16(p.d + ((size_t)row * (p.units >> 2) + (u >> 2)) * 2);
    }
    __device__ __forceinline__ static float dot(const Raw& r, int sub, const float (&x)[32], const float*, uint32_t) {
        const float M = 8388640.0f;  // 2^23 + 32
        const uint32_t n[8] = {r.n0.x, r.n0.y, r.n0.z, r.n0.w, r.n1.x, r.n1.y, r.n1.z, r.n1.w};
        const uint32_t h[4] = {r.hb.x, r.hb.y, r.hb.z, r.hb.w};
        float g0 = 0.f, g1 = 0.f, g2 = 0.f, g3 = 0.f;  // g0,g1: first 16 elements; g2,g3: last 16
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            uint32_t q;
            if (sub == 0)
                q = (n[j] & 0x0F0F0F0Fu) | ((j < 4 ? (h[j] << 4) : (h[j - 4] << 2)) & 0x30303030u);
            else
                q = ((n[j] >> 4) & 0x0F0F0F0Fu) | ((j < 4 ? h[j] : (h[j - 4] >> 2)) & 0x30303030u);
            if (j < 4) {
                g0 = fmaf(byte_f<0>(q, M), x[4 * j + 0], g0);
                g1 = fmaf(byte_f<1>(q, M), x[4 * j + 1], g1);
                g0 = fmaf(byte_f<2>(q, M), x[4 * j + 2], g0);
                g1 = fmaf(byte_f<3>(q, M), x[4 * j + 3], g1);
            } else {
                g2 = fmaf(byte_f<0>(q, M), x[4 * j + 0], g2);
                g3 = fmaf(byte_f<1>(q, M), x[4 * j + 1], g3);
                g2 = fmaf(byte_f<2>(q, M), x[4 * j + 2], g2);
                g3 = fmaf(byte_f<3>(q, M), x[4 * j + 3], g3);
            }
        }
        const float d = h2f(r.d);
        const float sa = d * (float)(int8_t)((r.sc >> (16 * sub)) & 0xFFu);
        const float sb = d * (float)(int8_t)((r.sc >> (16 * sub + 8)) & 0xFFu);
        return fmaf(sb, g2 + g3, sa * (g0 + g1));
    }
};

// F32 (the reference's catch-all branch, ops.cpp:289-299): q stream
// [rows][cols] f32.
struct FmtF32 {
    static constexpr int UE = 32, SUBS = 1, GS = 3;
    static constexpr bool XSUM = false;
    struct Raw { uint4 v[8]; };
    __device__ __forceinline__ static void load(const GemvParams& p, uint32_t row, uint32_t u, Raw& r) {
        const uint8_t* b = p.q + ((size_t)row * p.cols + (size_t)u * 32) * 4;
#pragma unroll
        for (int i = 0; i < 8; ++i) r.v[i] = ld_stream_u4(b + 16 * i);
    }
    __device__ __forceinline__ static float dot(const Raw& r, int, const float (&x)[32], const float*, uint32_t) {
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            a0 = fmaf(__uint_as_float(r.v[i].x), x[4 * i + 0], a0);
            a1 = fmaf(__uint_as_float(r.v[i].y), x[4 * i + 1], a1);
            a2 = fmaf(__uint_as_float(r.v[i].z), x[4 * i + 2], a2);
            a3 = fmaf(__uint_as_float(r.v[i].w), x[4 * i + 3], a3);
        }
        return (a0 + a1) + (a2 + a3);
    }
};

// Swizzled granule index of float4 granule g of the staged x vector: the low
// 3 bits are XORed with the index of the K-unit the granule belongs to.
template <class Fmt>
__device__ __forceinline__ int xswz(int g) {
    return g ^ ((g >> Fmt::GS) & 7);
}

__device__ __forceinline__ float block_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < nw; ++i) t += red[i];
    return t;
}

constexpr int kGemvThreads = 512;

template <class Fmt, int PRO, int EPI, int R>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_kernel(const GemvParams p) {
    extern __shared__ float4 smem4[];
    float4* xs = smem4;
    float* xsum = reinterpret_cast<float*>(smem4 + p.cols / 4);
    __shared__ float red[32];
    __shared__ unsigned long long best_sh[32];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
    const int G = p.cols / 4;

    pdl_wait();

    // ---- stage x (fused RMSNorm: y = x * (1/sqrt(mean(x^2) + eps)) * w)
    const float4* x4 = reinterpret_cast<const float4*>(p.x);
    float ss = 0.f;
    for (int g = tid; g < G; g += blockDim.x) {
        float4 v = x4[g];
        if constexpr (PRO == PRO_RMS) ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        xs[xswz<Fmt>(g)] = v;
    }
    if constexpr (PRO == PRO_RMS) {
        ss = block_sum(ss, red);
        const float inv = 1.0f / sqrtf(ss / (float)p.cols + p.eps);
        const float4* w4 = reinterpret_cast<const float4*>(p.norm_w);
        for (int g = tid; g < G; g += blockDim.x) {
            float4 v = xs[xswz<Fmt>(g)];
            const float4 w = w4[g];
            v.x = (v.x * inv) * w.x;
            v.y = (v.y * inv) * w.y;
            v.z = (v.z * inv) * w.z;
            v.w = (v.w * inv) * w.w;
            xs[xswz<Fmt>(g)] = v;
        }
    }
    __syncthreads();
    if constexpr (Fmt::XSUM) {
        for (int b = tid; b < (int)(p.cols / 32); b += blockDim.x) {
            float t = 0.f;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                float4 v = xs[xswz<Fmt>(b * 8 + j)];
                t += (v.x + v.y) + (v.z + v.w);
            }
            xsum[b] = t;
        }
        __syncthreads();
    }

    unsigned long long best = 0ull;
    const uint32_t ntiles = p.rows_pad / R;
    for (uint32_t t = blockIdx.x * nwarps + warp; t < ntiles; t += gridDim.x * nwarps) {
        const uint32_t row0 = t * R;
        float acc[R];
#pragma unroll
        for (int r = 0; r < R; ++r) acc[r] = 0.f;

        // two K-units per lane per iteration: all their loads are issued
        // before any of them is consumed
        for (uint32_t u0 = lane; u0 < p.units; u0 += 64) {
            const bool two = u0 + 32 < p.units;
            typename Fmt::Raw raw[2][R];
#pragma unroll
            for (int r = 0; r < R; ++r) Fmt::load(p, row0 + r, u0, raw[0][r]);
            if (two) {
#pragma unroll
                for (int r = 0; r < R; ++r) Fmt::load(p, row0 + r, u0 + 32, raw[1][r]);
            }
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                if (k == 1 && !two) break;
                const uint32_t u = u0 + 32 * k;
#pragma unroll
                for (int sub = 0; sub < Fmt::SUBS; ++sub) {
                    float x[32];
                    const int g0 = (int)(u * Fmt::SUBS + sub) * 8;
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const float4 v = xs[xswz<Fmt>(g0 + j)];
                        x[4 * j + 0] = v.x;
                        x[4 * j + 1] = v.y;
                        x[4 * j + 2] = v.z;
                        x[4 * j + 3] = v.w;
                    }
#pragma unroll
                    for (int r = 0; r < R; ++r) acc[r] += Fmt::dot(raw[k][r], sub, x, xsum, u);
                }
            }
        }

        const float v = warp_reduce_rows<R>(acc, lane);
        constexpr int LPR = 32 / R;  // lanes holding each row's total
        const int rl = lane / LPR;   // row of this lane within the tile
        const uint32_t row = row0 + rl;
        const bool leader = (lane % LPR) == 0;

        if constexpr (EPI == EPI_STORE) {
            if (leader && row < p.rows) p.y[row] = v;
        } else if constexpr (EPI == EPI_RESIDUAL) {
            if (leader && row < p.rows) p.y[row] += v;  // x += W.h (ops::axpy, qwen2_model.cpp:178,184)
        } else if constexpr (EPI == EPI_LOGITS) {
            if (leader && row < p.rows) {
                p.y[row] = v;
                if (v == v) {  // a NaN never wins (greedy_sampler.cpp:11 compares with >)
                    const unsigned long long k = argmax_key(v, p.row_offset + row);
                    best = k > best ? k : best;
                }
            }
        } else if constexpr (EPI == EPI_SWIGLU) {
            // physical rows 2j / 2j+1 hold gate_j / up_j: h_j = silu(gate_j) * up_j
            // (ops::silu then ops::mul, qwen2_model.cpp:154-155)
            const float up = __shfl_down_sync(0xffffffffu, v, LPR);
            if (leader && (rl & 1) == 0 && row + 1 < p.rows) {
                const float g = v / (1.0f + expf(-v));
                p.y[row >> 1] = g * up;
            }
        } else if constexpr (EPI == EPI_QKV) {
            const float v1 = __shfl_down_sync(0xffffffffu, v, LPR);
            const uint32_t hd = p.head_dim, half = hd >> 1;
            const uint32_t pos = *p.pos;
            if (leader && row < p.rows) {
                if (row < p.q_rows + p.k_rows) {
                    if ((rl & 1) == 0) {
                        // a rotary pair (i, i + hd/2) of one head
                        const bool isq = row < p.q_rows;
                        const uint32_t pr = (isq ? row : row - p.q_rows) >> 1;  // pair index
                        const uint32_t head = pr / half, i = pr % half;
                        const uint32_t la = head * hd + i, lb = la + half;      // logical index in q or k
                        float x0 = v, x1 = v1;
                        if (p.bias) {
                            const uint32_t bo = isq ? 0u : p.q_rows;
                            x0 += p.bias[bo + la];
                            x1 += p.bias[bo + lb];
                        }
                        // ops::rope (ops.cpp:84-89) with the reference build's fused rounding
                        const float2 cs = p.rope[(size_t)pos * half + i];
                        const float o0 = fmaf(x0, cs.x, -__fmul_rn(x1, cs.y));
                        const float o1 = fmaf(x0, cs.y, __fmul_rn(x1, cs.x));
                        if (isq) {
                            p.qout[la] = o0;
                            p.qout[lb] = o1;
                        } else {
                            float* kr = p.kcache + ((size_t)head * p.max_ctx + pos) * hd;
                            kr[i] = o0;
                            kr[i + half] = o1;
                        }
                    }
                } else {
                    const uint32_t lv = row - p.q_rows - p.k_rows;
                    float val = v;
                    if (p.bias) val += p.bias[p.q_rows + p.k_rows + lv];
                    const uint32_t head = lv / hd, dd = lv % hd;
                    p.vcache[((size_t)head * p.max_ctx + pos) * hd + dd] = val;
                }
            }
        }
    }

    if constexpr (EPI == EPI_LOGITS) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
            best = other > best ? other : best;
        }
        if (lane == 0) best_sh[warp] = best;
        __syncthreads();
        if (tid == 0) {
            unsigned long long b = 0ull;
            for (int i = 0; i < nwarps; ++i) b = best_sh[i] > b ? best_sh[i] : b;
            if (b) atomicMax(p.argmax, b);
        }
    }
    pdl_launch_dependents();
}

}  // namespace smallm
