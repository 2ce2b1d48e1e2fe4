// Batched prefill: the kernels around the linear layers when T prompt tokens
// are processed at once (the reference feeds them one by one,
// src/runtime/generator.cpp:47-51).  The linear layers themselves are GEMMs
// over the T tokens (model.cu); these kernels restate, per token, the same
// arithmetic the decode step fuses into its GEMV prologues and epilogues:
// RMSNorm (ops.cpp:29-40), bias + RoPE + KV append (qwen2_model.cpp:97-110),
// causal GQA attention (qwen2_model.cpp:111-133), SiLU * up (ops.cpp:60-65,
// 325-330) and the residual adds.
#include "common.cuh"
#include "engine.h"

namespace smallm {

constexpr int kPreThreads = 256;

// Y[t] = X[t] * (1 / sqrt(mean(X[t]^2) + eps)) * w, one CTA per token.
__global__ void rmsnorm_rows_kernel(const float* X, const float* w, uint32_t n, float eps, float* Y) {
    __shared__ float red[32];
    const float* x = X + (size_t)blockIdx.x * n;
    float* y = Y + (size_t)blockIdx.x * n;
    float ss = 0.f;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) ss += x[i] * x[i];
    ss = block_sum(ss, red);
    const float inv = 1.0f / sqrtf(ss / (float)n + eps);
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) y[i] = (x[i] * inv) * w[i];
}

// The QKV GEMM's rows (storage order: query rotary pairs, key rotary pairs,
// value rows) of token t at position pos0 + t: bias, RoPE with the reference
// build's rounding, query into Q[t], key and value into the cache.  One
// thread per (token, even row of a pair or value row).
__global__ void qkv_post_kernel(const float* Y, uint32_t rows, uint32_t T, uint32_t q_rows, uint32_t k_rows,
                                uint32_t hd, const float* bias, const float2* rope, uint32_t pos0,
                                uint32_t max_ctx, float* Q, float* kc, float* vc) {
    const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (uint64_t)T * rows) return;
    const uint32_t t = (uint32_t)(idx / rows), row = (uint32_t)(idx % rows);
    const float* y = Y + (size_t)t * rows;
    const uint32_t pos = pos0 + t, half = hd >> 1;
    if (row < q_rows + k_rows) {
        if (row & 1) return;  // the even row of a pair does both
        const bool isq = row < q_rows;
        const uint32_t pr = (isq ? row : row - q_rows) >> 1;
        const uint32_t head = pr / half, ii = pr % half;
        const uint32_t la = head * hd + ii, lb = la + half;
        float x0 = y[row], x1 = y[row + 1];
        if (bias) {
            const uint32_t bo = isq ? 0u : q_rows;
            x0 += bias[bo + la];
            x1 += bias[bo + lb];
        }
        const float2 cs = rope[(size_t)pos * half + ii];
        const float o0 = fmaf(x0, cs.x, -__fmul_rn(x1, cs.y));
        const float o1 = fmaf(x0, cs.y, __fmul_rn(x1, cs.x));
        if (isq) {
            float* q = Q + (size_t)t * q_rows;
            q[la] = o0;
            q[lb] = o1;
        } else {
            float* kr = kc + ((size_t)head * max_ctx + pos) * hd;
            kr[ii] = o0;
            kr[ii + half] = o1;
        }
    } else {
        const uint32_t lv = row - q_rows - k_rows;
        float vv = y[row];
        if (bias) vv += bias[q_rows + k_rows + lv];
        const uint32_t head = lv / hd, dd = lv % hd;
        vc[((size_t)head * max_ctx + pos) * hd + dd] = vv;
    }
}

// Causal attention of token t (position pos0 + t) for the `group` query heads
// of KV head g: one CTA per (t, g), keys 0..pos0 + t in chunks of 32 staged in
// shared memory, online softmax across chunks (ops::softmax, ops.cpp:43-57).
constexpr uint32_t kPreChunk = 32;
constexpr int kPreMaxGroup = 8;

template <int HD>
__global__ void __launch_bounds__(128) attention_prefill_kernel(const float* Q, const float* kc, const float* vc,
                                                                uint32_t n_heads, uint32_t n_kv, uint32_t max_ctx,
                                                                uint32_t pos0, float* out) {
    constexpr int PARTS = 128 / HD;
    constexpr int DL = HD / 8, DV = DL / 4;
    __shared__ __align__(16) float ks[kPreChunk * HD];
    __shared__ __align__(16) float vs[kPreChunk * HD];
    __shared__ __align__(16) float qs[kPreMaxGroup * HD];
    __shared__ float sc[kPreMaxGroup * kPreChunk];
    __shared__ float corr[kPreMaxGroup], pm[kPreMaxGroup], pl[kPreMaxGroup];
    __shared__ float red[(128 - 32) * kPreMaxGroup + kPreMaxGroup];
    const uint32_t G = n_heads / n_kv;
    const uint32_t t = blockIdx.x, g = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t n = pos0 + t + 1;
    const float* q = Q + (size_t)t * n_heads * HD + (size_t)g * G * HD;
    for (uint32_t i = tid; i < G * HD; i += 128) qs[i] = q[i];
    if (tid < kPreMaxGroup) {
        pm[tid] = -INFINITY;
        pl[tid] = 0.f;
    }
    const float scale = 1.0f / sqrtf((float)HD);
    const int d = tid % HD, part = tid / HD;
    float acc[kPreMaxGroup];
#pragma unroll
    for (int h = 0; h < kPreMaxGroup; ++h) acc[h] = 0.f;
    const float* kb = kc + (size_t)g * max_ctx * HD;
    const float* vb = vc + (size_t)g * max_ctx * HD;
    for (uint32_t c0 = 0; c0 < n; c0 += kPreChunk) {
        const uint32_t len = min(kPreChunk, n - c0);
        __syncthreads();
        for (uint32_t i = tid; i < len * HD / 4; i += 128) {
            reinterpret_cast<float4*>(ks)[i] = reinterpret_cast<const float4*>(kb + (size_t)c0 * HD)[i];
            reinterpret_cast<float4*>(vs)[i] = reinterpret_cast<const float4*>(vb + (size_t)c0 * HD)[i];
        }
        __syncthreads();
        // scores: 8 lanes per key, uniform pass loop (all lanes reach the shuffles)
        const int l8 = tid & 7, grp = tid >> 3;
        for (uint32_t tb = 0; tb < len; tb += 16) {
            const uint32_t tt = tb + grp;
            const bool act = tt < len;
            float4 kv[DV];
#pragma unroll
            for (int j = 0; j < DV; ++j)
                kv[j] = act ? reinterpret_cast<const float4*>(ks + tt * HD)[l8 + 8 * j] : make_float4(0.f, 0.f, 0.f, 0.f);
            float s[kPreMaxGroup];
#pragma unroll
            for (int h = 0; h < kPreMaxGroup; ++h) {
                s[h] = 0.f;
                if (h < (int)G) {
#pragma unroll
                    for (int j = 0; j < DV; ++j) {
                        const float4 q4 = reinterpret_cast<const float4*>(qs + h * HD)[l8 + 8 * j];
                        s[h] = fmaf(q4.x, kv[j].x, s[h]);
                        s[h] = fmaf(q4.y, kv[j].y, s[h]);
                        s[h] = fmaf(q4.z, kv[j].z, s[h]);
                        s[h] = fmaf(q4.w, kv[j].w, s[h]);
                    }
                }
            }
#pragma unroll
            for (int o = 4; o >= 1; o >>= 1) {
#pragma unroll
                for (int h = 0; h < kPreMaxGroup; ++h)
                    if (h < (int)G) s[h] += __shfl_xor_sync(0xffffffffu, s[h], o);
            }
            if (l8 == 0 && act) {
#pragma unroll
                for (int h = 0; h < kPreMaxGroup; ++h)
                    if (h < (int)G) sc[h * kPreChunk + tt] = s[h] * scale;
            }
        }
        __syncthreads();
        for (uint32_t h = warp; h < G; h += 4) {
            const float sv = (uint32_t)lane < len ? sc[h * kPreChunk + lane] : -INFINITY;
            const float m_old = pm[h];
            const float m_new = fmaxf(m_old, warp_max(sv));
            const float e = (uint32_t)lane < len ? expf(sv - m_new) : 0.f;
            const float l = warp_sum(e);
            if ((uint32_t)lane < len) sc[h * kPreChunk + lane] = e;
            if (lane == 0) {
                const float cf = m_old == -INFINITY ? 0.f : expf(m_old - m_new);
                corr[h] = cf;
                pl[h] = fmaf(pl[h], cf, l);
                pm[h] = m_new;
            }
        }
        __syncthreads();
#pragma unroll
        for (int h = 0; h < kPreMaxGroup; ++h)
            if (h < (int)G) acc[h] *= corr[h];
        for (uint32_t tt = part; tt < len; tt += PARTS) {
            const float v = vs[tt * HD + d];
#pragma unroll
            for (int h = 0; h < kPreMaxGroup; ++h)
                if (h < (int)G) acc[h] = fmaf(sc[h * kPreChunk + tt], v, acc[h]);
        }
    }
    if constexpr (PARTS > 1) {
        __syncthreads();
        if (part > 0) {
#pragma unroll
            for (int h = 0; h < kPreMaxGroup; ++h) red[((part - 1) * HD + d) * kPreMaxGroup + h] = acc[h];
        }
        __syncthreads();
    }
    if (part == 0) {
        float* o = out + (size_t)t * n_heads * HD + (size_t)g * G * HD;
#pragma unroll
        for (int h = 0; h < kPreMaxGroup; ++h) {
            if (h < (int)G) {
                float v = acc[h];
#pragma unroll
                for (int k = 1; k < PARTS; ++k) v += red[((k - 1) * HD + d) * kPreMaxGroup + h];
                o[h * HD + d] = v / pl[h];
            }
        }
    }
}

// H[t][j] = silu(Y[t][2j]) * Y[t][2j+1] (gate / up rows interleaved).
__global__ void swiglu_rows_kernel(const float* Y, uint32_t ffn, uint32_t T, float* H) {
    const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (uint64_t)T * ffn) return;
    const uint32_t t = (uint32_t)(idx / ffn), j = (uint32_t)(idx % ffn);
    const float gv = Y[(size_t)t * 2 * ffn + 2 * j], uv = Y[(size_t)t * 2 * ffn + 2 * j + 1];
    H[idx] = (gv / (1.0f + expf(-gv))) * uv;
}

// X += Y (the residual, ops::axpy with a = 1).
__global__ void add_rows_kernel(float* X, const float* Y, uint64_t n) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) X[i] += Y[i];
}

static unsigned blocks_for(uint64_t n) { return (unsigned)((n + kPreThreads - 1) / kPreThreads); }

void launch_rmsnorm_rows(const float* X, const float* w, uint32_t n, uint32_t T, float eps, float* Y,
                         cudaStream_t s) {
    rmsnorm_rows_kernel<<<T, 1024, 0, s>>>(X, w, n, eps, Y);
    SM_CUDA(cudaGetLastError());
}

void launch_qkv_post(const float* Y, uint32_t rows, uint32_t T, uint32_t q_rows, uint32_t k_rows, uint32_t hd,
                     const float* bias, const float2* rope, uint32_t pos0, uint32_t max_ctx, float* Q, float* kc,
                     float* vc, cudaStream_t s) {
    qkv_post_kernel<<<blocks_for((uint64_t)T * rows), kPreThreads, 0, s>>>(Y, rows, T, q_rows, k_rows, hd, bias,
                                                                          rope, pos0, max_ctx, Q, kc, vc);
    SM_CUDA(cudaGetLastError());
}

void launch_attention_prefill(const float* Q, const float* kc, const float* vc, uint32_t n_heads, uint32_t n_kv,
                              uint32_t hd, uint32_t max_ctx, uint32_t pos0, uint32_t T, float* out,
                              cudaStream_t s) {
    if (n_heads % n_kv || n_heads / n_kv > (uint32_t)kPreMaxGroup)
        throw Error(1, "prefill attention: unsupported head grouping");
    const dim3 grid(T, n_kv);
    if (hd == 32) attention_prefill_kernel<32><<<grid, 128, 0, s>>>(Q, kc, vc, n_heads, n_kv, max_ctx, pos0, out);
    else if (hd == 64) attention_prefill_kernel<64><<<grid, 128, 0, s>>>(Q, kc, vc, n_heads, n_kv, max_ctx, pos0, out);
    else if (hd == 128) attention_prefill_kernel<128><<<grid, 128, 0, s>>>(Q, kc, vc, n_heads, n_kv, max_ctx, pos0, out);
    else throw Error(1, "prefill attention: head_dim must be 32, 64 or 128");
    SM_CUDA(cudaGetLastError());
}

void launch_swiglu_rows(const float* Y, uint32_t ffn, uint32_t T, float* H, cudaStream_t s) {
    swiglu_rows_kernel<<<blocks_for((uint64_t)T * ffn), kPreThreads, 0, s>>>(Y, ffn, T, H);
    SM_CUDA(cudaGetLastError());
}

void launch_add_rows(float* X, const float* Y, uint64_t n, cudaStream_t s) {
    add_rows_kernel<<<blocks_for(n), kPreThreads, 0, s>>>(X, Y, n);
    SM_CUDA(cudaGetLastError());
}

}  // namespace smallm
