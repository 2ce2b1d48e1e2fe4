// Batched prefill: the kernels around the linear layers when T prompt tokens
// are processed at once (the reference feeds them one by one,
// src/runtime/generator.cpp:47-51).  The linear layers themselves are GEMMs
// over the T tokens (model.cu); these kernels restate, per token, the same
// arithmetic the decode step fuses into its GEMV prologues and epilogues:
// RMSNorm (ops.cpp:29-40), bias + RoPE + KV append (qwen2_model.cpp:97-110),
// causal GQA attention (qwen2_model.cpp:111-133), SiLU * up (ops.cpp:60-65,
// 325-330) and the residual adds.
#include <algorithm>
#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "engine.h"

namespace smallm {

constexpr int kPreThreads = 256;

// Y[t] = X[t] * (1 / sqrt(mean(X[t]^2) + eps)) * w, one CTA per token.
// (Yh: the same values rounded to f16 instead, the tensor-core GEMM's input.)
__global__ void smallm_rmsnorm_rows_kernel(const float* X, const float* w, uint32_t n, float eps, float* Y, __half* Yh) {
    __shared__ float red[32];
    const float* x = X + (size_t)blockIdx.x * n;
    float ss = 0.f;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) ss += x[i] * x[i];
    ss = block_sum(ss, red);
    const float inv = 1.0f / sqrtf(ss / (float)n + eps);
    if (Yh) {
        __half* y = Yh + (size_t)blockIdx.x * n;
        for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) y[i] = __float2half_rn((x[i] * inv) * w[i]);
    } else {
        float* y = Y + (size_t)blockIdx.x * n;
        for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) y[i] = (x[i] * inv) * w[i];
    }
}

// The QKV GEMM's rows (storage order: query rotary pairs, key rotary pairs,
// value rows) of token t at position pos0 + t: bias, RoPE with the reference
// build's rounding, query into Q[t], key and value into the cache.  One
// thread per (token, even row of a pair or value row).
__global__ void smallm_qkv_post_kernel(const float* Y, uint32_t rows, uint32_t T, uint32_t q_rows, uint32_t k_rows,
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

// Causal attention over the prompt (the reference's per-token attention loop,
// src/model/qwen2_model.cpp:111-133, with ops::softmax, ops.cpp:43-57, for
// every prompt token at once).  One CTA of TOK warps (8, or 4 when 8-token
// blocks would leave fewer than two CTAs per SM) per (block of TOK query
// tokens, KV head g); warp w owns token t0 + w and its G query heads.
// Chunks of 32 keys (K rows padded to HD + 4 floats, so the lanes' float4
// reads of 32 different rows are conflict-free) are staged once in shared
// memory and used by all TOK tokens.  Scores: lane = key, so each row's online
// softmax (running max, sum, rescale) is a warp reduction; probabilities go
// through a warp-private shared-memory row to the PV product, where lane owns
// HD/32 output dimensions.  f32 throughout, expf as the reference.
constexpr uint32_t kPreChunk = 32;   // keys per chunk (= lanes)
constexpr int kPreMaxGroup = 8;      // query heads per KV head

template <int HD, int G, int TOK>
struct PreAttnSmem {
    static constexpr int KSTR = HD + 4;
    static constexpr size_t q = (size_t)TOK * G * HD;          // [token][head][HD]
    static constexpr size_t k = (size_t)kPreChunk * KSTR;      // [key][HD + 4]
    static constexpr size_t v = (size_t)kPreChunk * HD;        // [key][HD]
    static constexpr size_t p = (size_t)TOK * G * kPreChunk;
    static constexpr size_t bytes = 4 * (q + k + v + p);
};

// out (f32) or, when out_h is set, out_h (the same values rounded to f16,
// the tensor-core GEMM's input).
template <int HD, int G, int TOK>
__global__ void __launch_bounds__(32 * TOK) smallm_attention_prefill_kernel(const float* __restrict__ Q,
                                                                     const float* __restrict__ kc,
                                                                     const float* __restrict__ vc, uint32_t n_heads,
                                                                     uint32_t max_ctx, uint32_t pos0, uint32_t T,
                                                                     float* __restrict__ out, __half* out_h,
                                                                     uint32_t n_split, float* __restrict__ part) {
    using S = PreAttnSmem<HD, G, TOK>;
    constexpr uint32_t NT = 32 * TOK;  // threads
    constexpr int DPL = HD / 32;  // output dims per lane
    extern __shared__ __align__(16) float pre_smem[];
    float* qs = pre_smem;
    float* ks = qs + S::q;
    float* vs = ks + S::k;
    float* ps = vs + S::v;
    const uint32_t tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    // heaviest (last) token blocks first
    const uint32_t t0 = (gridDim.x - 1 - blockIdx.x) * TOK, g = blockIdx.y;
    const uint32_t t = t0 + w;
    const bool live = t < T;
    const uint32_t t_last = min(t0 + TOK, T) - 1;
    const uint32_t n_keys = pos0 + t_last + 1;  // keys the block's last token attends to
    const uint32_t my_keys = pos0 + t + 1;      // this warp's token (causal)

    // q tile: [token][head][HD]
    for (uint32_t i = tid; i < TOK * G * HD / 4; i += NT) {
        const uint32_t tok = i / (G * HD / 4), rem = i % (G * HD / 4);
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (t0 + tok < T)
            v = reinterpret_cast<const float4*>(Q + (size_t)(t0 + tok) * n_heads * HD + (size_t)g * G * HD)[rem];
        reinterpret_cast<float4*>(qs)[i] = v;
    }
    const float scale = 1.0f / sqrtf((float)HD);
    float m[G], l[G], acc[G][DPL];
#pragma unroll
    for (int i = 0; i < G; ++i) {
        m[i] = -INFINITY;
        l[i] = 0.f;
#pragma unroll
        for (int j = 0; j < DPL; ++j) acc[i][j] = 0.f;
    }
    const float* kb = kc + (size_t)g * max_ctx * HD;
    const float* vb = vc + (size_t)g * max_ctx * HD;
    const float* qw = qs + (size_t)w * G * HD;
    float* pw = ps + (size_t)w * G * kPreChunk;
    // this CTA's whole chunks of the block's keys (split blockIdx.z of n_split)
    const uint32_t per = ((n_keys + kPreChunk - 1) / kPreChunk + n_split - 1) / n_split * kPreChunk;
    const uint32_t k_begin = min(blockIdx.z * per, n_keys), k_end = min(k_begin + per, n_keys);
    for (uint32_t c0 = k_begin; c0 < k_end; c0 += kPreChunk) {
        const uint32_t len = min(kPreChunk, k_end - c0);
        __syncthreads();  // the previous chunk's K/V are no longer read
        for (uint32_t i = tid; i < len * HD / 4; i += NT) {
            const uint32_t key = i / (HD / 4), c4 = i % (HD / 4);
            reinterpret_cast<float4*>(ks + key * S::KSTR)[c4] =
                reinterpret_cast<const float4*>(kb + (size_t)(c0 + key) * HD)[c4];
            reinterpret_cast<float4*>(vs)[i] = reinterpret_cast<const float4*>(vb + (size_t)c0 * HD)[i];
        }
        __syncthreads();
        // scores of key c0 + lane for the G heads of this warp's token
        const bool valid = live && lane < len && c0 + lane < my_keys;
        float sc[G];
#pragma unroll
        for (int i = 0; i < G; ++i) sc[i] = 0.f;
        if (lane < len) {
            const float* kr = ks + lane * S::KSTR;
#pragma unroll 4
            for (int d = 0; d < HD; d += 4) {
                const float4 k4 = *reinterpret_cast<const float4*>(kr + d);
#pragma unroll
                for (int i = 0; i < G; ++i) {
                    const float4 q4 = *reinterpret_cast<const float4*>(qw + i * HD + d);
                    sc[i] = fmaf(q4.x, k4.x, sc[i]);
                    sc[i] = fmaf(q4.y, k4.y, sc[i]);
                    sc[i] = fmaf(q4.z, k4.z, sc[i]);
                    sc[i] = fmaf(q4.w, k4.w, sc[i]);
                }
            }
        }
        // online softmax per head (all lanes hold the row state)
        float corr[G];
#pragma unroll
        for (int i = 0; i < G; ++i) {
            const float sv = valid ? sc[i] * scale : -INFINITY;
            const float m_new = fmaxf(m[i], warp_max(sv));
            const float e = valid ? expf(sv - m_new) : 0.f;
            const float cf = m[i] == -INFINITY ? 0.f : expf(m[i] - m_new);
            l[i] = fmaf(l[i], cf, warp_sum(e));
            m[i] = m_new;
            corr[i] = cf;
            pw[i * kPreChunk + lane] = e;
        }
        __syncwarp();
#pragma unroll
        for (int i = 0; i < G; ++i)
#pragma unroll
            for (int j = 0; j < DPL; ++j) acc[i][j] *= corr[i];
        for (uint32_t key = 0; key < len; ++key) {
            float v[DPL];
            if constexpr (DPL == 4) {
                const float4 v4 = reinterpret_cast<const float4*>(vs + key * HD)[lane];
                v[0] = v4.x, v[1] = v4.y, v[2] = v4.z, v[3] = v4.w;
            } else if constexpr (DPL == 2) {
                const float2 v2 = reinterpret_cast<const float2*>(vs + key * HD)[lane];
                v[0] = v2.x, v[1] = v2.y;
            } else {
                v[0] = vs[key * HD + lane];
            }
#pragma unroll
            for (int i = 0; i < G; ++i) {
                const float p = pw[i * kPreChunk + key];
#pragma unroll
                for (int j = 0; j < DPL; ++j) acc[i][j] = fmaf(p, v[j], acc[i][j]);
            }
        }
        __syncwarp();  // pw is rewritten by the next chunk
    }
    if (live && n_split > 1) {
        // partial of this split: unnormalised output, running max and sum
        // ([token][head][split][HD + 2]); rows without a key here keep
        // m = -inf, l = 0 and weigh nothing in the merge
#pragma unroll
        for (int i = 0; i < G; ++i) {
            float* pr = part + (((size_t)t * n_heads + g * G + i) * n_split + blockIdx.z) * (HD + 2);
#pragma unroll
            for (int j = 0; j < DPL; ++j) pr[lane * DPL + j] = acc[i][j];
            if (lane == 0) {
                pr[HD] = m[i];
                pr[HD + 1] = l[i];
            }
        }
    } else if (live) {
        const size_t o = (size_t)t * n_heads * HD + (size_t)g * G * HD;
#pragma unroll
        for (int i = 0; i < G; ++i)
#pragma unroll
            for (int j = 0; j < DPL; ++j) {
                const float v = acc[i][j] / l[i];
                if (out_h) out_h[o + i * HD + lane * DPL + j] = __float2half_rn(v);
                else out[o + i * HD + lane * DPL + j] = v;
            }
    }
}

// Merge of the key splits of one (token, head): out = sum_s acc_s e^(m_s - M)
// / sum_s l_s e^(m_s - M), M = max_s m_s (split 0 holds key 0, so M is finite).
__global__ void smallm_attention_prefill_merge_kernel(const float* __restrict__ part, uint32_t n_split, uint32_t hd,
                                               float* __restrict__ out, __half* out_h) {
    const size_t row = blockIdx.x;  // token * n_heads + head
    const float* pr = part + row * n_split * (hd + 2);
    float M = -INFINITY;
    for (uint32_t s = 0; s < n_split; ++s) M = fmaxf(M, pr[s * (hd + 2) + hd]);
    for (uint32_t d = threadIdx.x; d < hd; d += blockDim.x) {
        float L = 0.f, O = 0.f;
        for (uint32_t s = 0; s < n_split; ++s) {
            const float* q = pr + s * (hd + 2);
            const float wgt = q[hd] == -INFINITY ? 0.f : expf(q[hd] - M);
            L = fmaf(q[hd + 1], wgt, L);
            O = fmaf(q[d], wgt, O);
        }
        const float v = O / L;
        if (out_h) out_h[row * hd + d] = __float2half_rn(v);
        else out[row * hd + d] = v;
    }
}

template <int HD, int G, int TOK>
static void launch_pre_attn_tok(const float* Q, const float* kc, const float* vc, uint32_t n_heads, uint32_t n_kv,
                                uint32_t max_ctx, uint32_t pos0, uint32_t T, float* out, __half* out_h,
                                float* part, cudaStream_t s) {
    using S = PreAttnSmem<HD, G, TOK>;
    static std::mutex mu;
    static std::unordered_map<int, bool> configured;
    int dev = 0;
    SM_CUDA(cudaGetDevice(&dev));
    {
        std::lock_guard<std::mutex> lk(mu);
        if (!configured.count(dev)) {
            SM_CUDA(cudaFuncSetAttribute(smallm_attention_prefill_kernel<HD, G, TOK>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S::bytes));
            configured[dev] = true;
        }
    }
    const uint32_t n_split = prefill_attention_splits(T, n_kv, pos0);
    const dim3 grid((T + TOK - 1) / TOK, n_kv, n_split);
    smallm_attention_prefill_kernel<HD, G, TOK><<<grid, 32 * TOK, S::bytes, s>>>(Q, kc, vc, n_heads, max_ctx, pos0, T, out,
                                                                          out_h, n_split, part);
    if (n_split > 1) {
        SM_CUDA(cudaGetLastError());
        smallm_attention_prefill_merge_kernel<<<T * n_heads, HD, 0, s>>>(part, n_split, HD, out, out_h);
    }
}

template <int HD, int G>
static void launch_pre_attn(const float* Q, const float* kc, const float* vc, uint32_t n_heads, uint32_t n_kv,
                            uint32_t max_ctx, uint32_t pos0, uint32_t T, float* out, __half* out_h, float* part,
                            cudaStream_t s) {
    // 8-token CTAs when they give at least two CTAs per SM, else 4-token ones
    // (more CTAs, so heavy and light causal blocks pack together)
    if (prefill_attention_tokens(T, n_kv) == 8)
        launch_pre_attn_tok<HD, G, 8>(Q, kc, vc, n_heads, n_kv, max_ctx, pos0, T, out, out_h, part, s);
    else
        launch_pre_attn_tok<HD, G, 4>(Q, kc, vc, n_heads, n_kv, max_ctx, pos0, T, out, out_h, part, s);
}

template <int HD>
static void launch_pre_attn_hd(uint32_t G, const float* Q, const float* kc, const float* vc, uint32_t n_heads,
                               uint32_t n_kv, uint32_t max_ctx, uint32_t pos0, uint32_t T, float* out,
                               __half* out_h, float* part, cudaStream_t s) {
    switch (G) {
        case 1: return launch_pre_attn<HD, 1>(Q, kc, vc, n_heads, n_kv, max_ctx, pos0, T, out, out_h, part, s);
        case 2: return launch_pre_attn<HD, 2>(Q, kc, vc, n_heads, n_kv, max_ctx, pos0, T, out, out_h, part, s);
        case 3: return launch_pre_attn<HD, 3>(Q, kc, vc, n_heads, n_kv, max_ctx, pos0, T, out, out_h, part, s);
        case 4: return launch_pre_attn<HD, 4>(Q, kc, vc, n_heads, n_kv, max_ctx, pos0, T, out, out_h, part, s);
        case 5: return launch_pre_attn<HD, 5>(Q, kc, vc, n_heads, n_kv, max_ctx, pos0, T, out, out_h, part, s);
        case 6: return launch_pre_attn<HD, 6>(Q, kc, vc, n_heads, n_kv, max_ctx, pos0, T, out, out_h, part, s);
        case 7: return launch_pre_attn<HD, 7>(Q, kc, vc, n_heads, n_kv, max_ctx, pos0, T, out, out_h, part, s);
        case 8: return launch_pre_attn<HD, 8>(Q, kc, vc, n_heads, n_kv, max_ctx, pos0, T, out, out_h, part, s);
        default: throw Error(1, "prefill attention: unsupported head grouping");
    }
}

// H[t][j] = silu(Y[t][2j]) * Y[t][2j+1] (gate / up rows interleaved).
// (Hh: the same values rounded to f16 instead, the tensor-core GEMM's input.)
__global__ void smallm_swiglu_rows_kernel(const float* Y, uint32_t ffn, uint32_t T, float* H, __half* Hh) {
    const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (uint64_t)T * ffn) return;
    const uint32_t t = (uint32_t)(idx / ffn), j = (uint32_t)(idx % ffn);
    const float gv = Y[(size_t)t * 2 * ffn + 2 * j], uv = Y[(size_t)t * 2 * ffn + 2 * j + 1];
    const float h = (gv / (1.0f + expf(-gv))) * uv;
    if (Hh) Hh[idx] = __float2half_rn(h);
    else H[idx] = h;
}

// X += Y (the residual, ops::axpy with a = 1).
__global__ void smallm_add_rows_kernel(float* X, const float* Y, uint64_t n) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) X[i] += Y[i];
}

static unsigned blocks_for(uint64_t n) { return (unsigned)((n + kPreThreads - 1) / kPreThreads); }

void launch_rmsnorm_rows(const float* X, const float* w, uint32_t n, uint32_t T, float eps, float* Y,
                         cudaStream_t s, __half* Yh) {
    smallm_rmsnorm_rows_kernel<<<T, 1024, 0, s>>>(X, w, n, eps, Y, Yh);
    SM_CUDA(cudaGetLastError());
}

void launch_qkv_post(const float* Y, uint32_t rows, uint32_t T, uint32_t q_rows, uint32_t k_rows, uint32_t hd,
                     const float* bias, const float2* rope, uint32_t pos0, uint32_t max_ctx, float* Q, float* kc,
                     float* vc, cudaStream_t s) {
    smallm_qkv_post_kernel<<<blocks_for((uint64_t)T * rows), kPreThreads, 0, s>>>(Y, rows, T, q_rows, k_rows, hd, bias,
                                                                          rope, pos0, max_ctx, Q, kc, vc);
    SM_CUDA(cudaGetLastError());
}

uint32_t prefill_attention_tokens(uint32_t T, uint32_t n_kv) {
    // 8-token CTAs when they give at least two CTAs per SM, else 4-token ones
    return (uint64_t)((T + 7) / 8) * n_kv >= 2ull * device_sm_count() ? 8u : 4u;
}

uint32_t prefill_attention_splits(uint32_t T, uint32_t n_kv, uint32_t pos0) {
    // split the keys of each token block until the grid has ~4 CTAs per SM,
    // keeping at least two 32-key chunks per split of the longest block
    const uint64_t ctas = (uint64_t)((T + prefill_attention_tokens(T, n_kv) - 1) / prefill_attention_tokens(T, n_kv)) *
                          n_kv;
    const uint64_t want = (4ull * device_sm_count() + ctas - 1) / ctas;
    const uint64_t chunks = ((uint64_t)pos0 + T + kPreChunk - 1) / kPreChunk;
    uint64_t n = std::min<uint64_t>(want, std::min<uint64_t>(8, chunks / 2));
    return n < 2 ? 1u : (uint32_t)n;
}

size_t prefill_attention_scratch_floats(uint32_t T, uint32_t n_heads, uint32_t n_kv, uint32_t hd, uint32_t pos0) {
    const uint32_t n = prefill_attention_splits(T, n_kv, pos0);
    return n > 1 ? (size_t)T * n_heads * n * (hd + 2) : 0;
}

void launch_attention_prefill(const float* Q, const float* kc, const float* vc, uint32_t n_heads, uint32_t n_kv,
                              uint32_t hd, uint32_t max_ctx, uint32_t pos0, uint32_t T, float* out,
                              cudaStream_t s, __half* out_h, float* part) {
    if (prefill_attention_splits(T, n_kv, pos0) > 1 && !part)
        throw Error(1, "prefill attention: key splits need scratch (prefill_attention_scratch_floats)");
    if (n_heads % n_kv || n_heads / n_kv > (uint32_t)kPreMaxGroup)
        throw Error(1, "prefill attention: unsupported head grouping");
    const uint32_t G = n_heads / n_kv;
    if (hd == 32) launch_pre_attn_hd<32>(G, Q, kc, vc, n_heads, n_kv, max_ctx, pos0, T, out, out_h, part, s);
    else if (hd == 64) launch_pre_attn_hd<64>(G, Q, kc, vc, n_heads, n_kv, max_ctx, pos0, T, out, out_h, part, s);
    else if (hd == 128) launch_pre_attn_hd<128>(G, Q, kc, vc, n_heads, n_kv, max_ctx, pos0, T, out, out_h, part, s);
    else throw Error(1, "prefill attention: head_dim must be 32, 64 or 128");
    SM_CUDA(cudaGetLastError());
}

void launch_swiglu_rows(const float* Y, uint32_t ffn, uint32_t T, float* H, cudaStream_t s, __half* Hh) {
    smallm_swiglu_rows_kernel<<<blocks_for((uint64_t)T * ffn), kPreThreads, 0, s>>>(Y, ffn, T, H, Hh);
    SM_CUDA(cudaGetLastError());
}

void launch_add_rows(float* X, const float* Y, uint64_t n, cudaStream_t s) {
    smallm_add_rows_kernel<<<blocks_for(n), kPreThreads, 0, s>>>(X, Y, n);
    SM_CUDA(cudaGetLastError());
}

}  // namespace smallm
