// Stochastic samplers on the device: temperature, top-k and top-p, the
// reference's TemperatureSampler / TopKSampler / TopPSampler
// (src/runtime/sampler/{temperature,top_k,top_p}_sampler.cpp).
//
// The uniform draw r comes from the host (std::mt19937 +
// uniform_real_distribution<float>, one draw per sample), so the random
// stream is the reference's.  One CTA of 1024 threads does the rest:
//   top-k / top-p: the candidates ordered by logit, largest first, ties by
//     index (a stable LSD radix sort of 32-bit keys, 4 passes of 8 bits, each
//     warp owning a contiguous chunk so the scatter stays stable);
//   e_i = exp((l_i - max) / T), sum, p_i = e_i / sum, cumulative sums (each
//     thread sums a contiguous chunk in order; a block scan joins the chunks);
//   top-p: the nucleus ends at the first cumulative >= p and r is scaled by
//     its mass (top_p_sampler.cpp:33-44);
//   the token is the first candidate with r <= cumulative, else the last.
// Differences from the reference come only from exp rounding and summation
// order (the chunked scan), i.e. only when r lies within ~1e-7 of a
// cumulative boundary.
#include "common.cuh"
#include "engine.h"
#include "smallm_cuda.h"

namespace smallm {

constexpr int kSampThreads = 1024;
constexpr int kSampWarps = kSampThreads / 32;

__device__ __forceinline__ uint32_t desc_key(float f) { return ~float_order_key(f); }

// Block-wide exclusive scan of one float per thread (in thread order); `tot`
// receives the total.
__device__ float block_exclusive_scan(float v, float* sh, float& tot) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) sh[warp] = x;
    __syncthreads();
    if (warp == 0) {
        float w = lane < kSampWarps ? sh[lane] : 0.f;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        sh[32 + lane] = w;  // inclusive over warps
    }
    __syncthreads();
    tot = sh[32 + kSampWarps - 1];
    const float before_warp = warp ? sh[32 + warp - 1] : 0.f;
    __syncthreads();
    return before_warp + x - v;
}

// One stable LSD pass: elements (key, idx) of `in` go to `out` ordered by
// digit (key >> shift) & 255; warp w owns a contiguous chunk of the input.
__device__ void radix_pass(const uint32_t* kin, const uint32_t* iin, uint32_t* kout, uint32_t* iout, uint32_t n,
                           int shift, uint32_t* hist /* [256][kSampWarps] */) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t chunk = (n + kSampWarps - 1) / kSampWarps;
    const uint32_t b = min(n, warp * chunk), e = min(n, b + chunk);
    for (uint32_t i = threadIdx.x; i < 256 * kSampWarps; i += kSampThreads) hist[i] = 0;
    __syncthreads();
    for (uint32_t i0 = b; i0 < e; i0 += 32) {
        const uint32_t i = i0 + lane;
        if (i < e) atomicAdd(&hist[((kin[i] >> shift) & 255) * kSampWarps + warp], 1u);
    }
    __syncthreads();
    // exclusive scan over (digit, warp) in that order: offsets of each
    // warp's run of each digit
    uint32_t sum = 0;
    if (threadIdx.x < 256) {
        const uint32_t d = threadIdx.x;
        for (int w = 0; w < kSampWarps; ++w) {
            const uint32_t c = hist[d * kSampWarps + w];
            hist[d * kSampWarps + w] = sum;
            sum += c;
        }
    }
    __shared__ uint32_t dtot[256];
    if (threadIdx.x < 256) dtot[threadIdx.x] = sum;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t run = 0;
        for (int d = 0; d < 256; ++d) {
            const uint32_t c = dtot[d];
            dtot[d] = run;
            run += c;
        }
    }
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < 256 * kSampWarps; i += kSampThreads) hist[i] += dtot[i / kSampWarps];
    __syncthreads();
    // stable scatter: within a step of 32, lanes with the same digit are
    // ranked by lane order; runs of a digit follow each other
    const uint32_t lt = (1u << lane) - 1u;
    for (uint32_t i0 = b; i0 < e; i0 += 32) {
        const uint32_t i = i0 + lane;
        const bool act = i < e;
        const uint32_t k = act ? kin[i] : 0u;
        const uint32_t d = act ? (k >> shift) & 255 : 256u + lane;  // inactive lanes never match
        const uint32_t peers = __match_any_sync(0xffffffffu, d);
        uint32_t pos = 0;
        if (act) pos = hist[d * kSampWarps + warp] + __popc(peers & lt);
        __syncwarp();
        if (act && (peers & lt) == 0) hist[d * kSampWarps + warp] += __popc(peers);
        __syncwarp();
        if (act) {
            kout[pos] = k;
            iout[pos] = iin[i];
        }
    }
    __syncthreads();
}

// kind 1 temperature, 2 top-k, 3 top-p.  scratch: 4 * n u32.
__global__ void __launch_bounds__(kSampThreads, 1)
    smallm_sample_kernel(const float* logits, uint32_t n, uint32_t kind, uint32_t k_arg, float p_arg, float temp, float r,
                  uint32_t* scratch, uint32_t* out) {
    __shared__ uint32_t hist[256 * kSampWarps];
    __shared__ float sh[64];
    __shared__ float smax[32];
    __shared__ uint32_t first_hit, cutoff_sh;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (kind == 0) {
        // greedy_sampler.cpp:8-14: the first maximum; NaN never wins
        __shared__ unsigned long long wbest[kSampWarps];
        unsigned long long b = 0ull;
        for (uint32_t i = tid; i < n; i += kSampThreads) {
            const float v = logits[i];
            if (v == v) {
                const unsigned long long key = argmax_key(v, i);
                b = key > b ? key : b;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long y = __shfl_xor_sync(0xffffffffu, b, o);
            b = y > b ? y : b;
        }
        if (lane == 0) wbest[warp] = b;
        __syncthreads();
        if (tid == 0) {
            for (int w = 0; w < kSampWarps; ++w) b = wbest[w] > b ? wbest[w] : b;
            *out = argmax_key_index(b);
        }
        return;
    }
    uint32_t* k0 = scratch;
    uint32_t* i0 = scratch + n;
    uint32_t* k1 = scratch + 2 * (size_t)n;
    uint32_t* i1 = scratch + 3 * (size_t)n;
    const bool sorted = kind != 1;
    uint32_t m = n;  // candidates
    if (sorted) {
        for (uint32_t i = tid; i < n; i += kSampThreads) {
            k0[i] = desc_key(logits[i]);
            i0[i] = i;
        }
        __syncthreads();
        radix_pass(k0, i0, k1, i1, n, 0, hist);
        radix_pass(k1, i1, k0, i0, n, 8, hist);
        radix_pass(k0, i0, k1, i1, n, 16, hist);
        radix_pass(k1, i1, k0, i0, n, 24, hist);  // sorted: k0 / i0
        if (kind == 2) m = min(k_arg, n);
    }
    // logit of candidate c
    auto cand = [&](uint32_t c) -> float { return sorted ? logits[i0[c]] : logits[c]; };
    // max (the first candidate when sorted; ops over the whole vector otherwise)
    float mx;
    if (sorted) {
        mx = cand(0);
    } else {
        float v = -INFINITY;
        for (uint32_t i = tid; i < n; i += kSampThreads) v = fmaxf(v, logits[i]);
        v = warp_max(v);
        if (lane == 0) smax[warp] = v;
        __syncthreads();
        if (warp == 0) {
            float w = lane < kSampWarps ? smax[lane] : -INFINITY;
            w = warp_max(w);
            if (lane == 0) smax[0] = w;
        }
        __syncthreads();
        mx = smax[0];
    }
    // contiguous chunk per thread
    const uint32_t chunk = (m + kSampThreads - 1) / kSampThreads;
    const uint32_t cb = min(m, tid * chunk), ce = min(m, cb + chunk);
    float esum = 0.f;
    for (uint32_t c = cb; c < ce; ++c) esum += expf((cand(c) - mx) / temp);
    float etot;
    block_exclusive_scan(esum, sh, etot);  // total of e_i
    // cumulative of p_i = e_i / sum
    float psum = 0.f;
    for (uint32_t c = cb; c < ce; ++c) psum += expf((cand(c) - mx) / temp) / etot;
    float ptot;
    const float pstart = block_exclusive_scan(psum, sh, ptot);
    uint32_t limit = m;
    float thresh = r;
    if (kind == 3) {
        // nucleus: first c with cumulative >= p; r is scaled by its mass
        if (tid == 0) cutoff_sh = m;
        __syncthreads();
        float cum = pstart;
        for (uint32_t c = cb; c < ce; ++c) {
            cum += expf((cand(c) - mx) / temp) / etot;
            if (cum >= p_arg) {
                atomicMin(&cutoff_sh, c + 1);
                break;
            }
        }
        __syncthreads();
        limit = cutoff_sh;
        // mass of the nucleus = cumulative at its last element
        __shared__ float nsum;
        if (limit >= cb + 1 && limit <= ce) {
            float cu = pstart;
            for (uint32_t c = cb; c < limit; ++c) cu += expf((cand(c) - mx) / temp) / etot;
            nsum = cu;
        }
        __syncthreads();
        thresh = r * nsum;
    }
    if (tid == 0) first_hit = limit;
    __syncthreads();
    float cum = pstart;
    for (uint32_t c = cb; c < ce && c < limit; ++c) {
        cum += expf((cand(c) - mx) / temp) / etot;
        if (thresh <= cum) {
            atomicMin(&first_hit, c);
            break;
        }
    }
    __syncthreads();
    if (tid == 0) {
        const uint32_t c = first_hit < limit ? first_hit : limit - 1;  // float-rounding fallback
        *out = sorted ? i0[c] : c;
    }
}

void launch_sample(const float* logits, uint32_t n, uint32_t kind, uint32_t k, float p, float temp, float r,
                   uint32_t* scratch, uint32_t* out, cudaStream_t stream) {
    smallm_sample_kernel<<<1, kSampThreads, 0, stream>>>(logits, n, kind, k, p, temp, r, scratch, out);
    SM_CUDA(cudaGetLastError());
}

}  // namespace smallm
