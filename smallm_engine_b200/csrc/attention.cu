// GQA decode attention over the device KV cache (split-K, flash-decoding).
//
// qwen2_model.cpp:111-133 (llama_model.cpp:297-317): for each query head h
// with KV head h / group, scores_t = dot(q_h, k_t) / sqrt(hd) over cached
// positions t <= pos, softmax, out_h = sum_t p_t v_t.
//
// Grid (n_kv, n_split).  CTA (g, s) owns one chunk of positions for the
// `group` query heads that share KV head g, so every K/V row is read from HBM
// once per step.  The chunk's K and V rows are contiguous in the head-major
// cache ([n_kv][max_ctx][hd]), so they arrive in shared memory through two
// TMA bulk copies completing on one mbarrier; scores, softmax and the V
// reduction then run from shared memory.  Each CTA writes an unnormalised
// partial (running max, sum, out); the last CTA of each KV head (atomic
// ticket, no waiting) merges the partials of the non-empty chunks.  This
// split-K kernel serves smallm_attention_noalloc; the decode step runs the
// cluster variant further down, which merges through distributed shared
// memory instead of global scratch.
#include <cooperative_groups.h>

#include <mutex>

#include "common.cuh"
#include "engine.h"
#include "smallm_cuda.h"

namespace smallm {

namespace cg = cooperative_groups;

constexpr int kAttnThreads = 128;
constexpr uint32_t kAttnMinChunk = 16;
constexpr uint32_t kAttnMaxChunk = 64;
constexpr int kAttnMaxGroup = 8;

uint32_t attention_splits(uint32_t n_kv, uint32_t max_ctx, int sm_count) {
    uint32_t s = (uint32_t)(2 * sm_count + n_kv - 1) / n_kv;
    const uint32_t lo = (max_ctx + kAttnMaxChunk - 1) / kAttnMaxChunk;   // chunks never exceed the maximum
    const uint32_t hi = (max_ctx + kAttnMinChunk - 1) / kAttnMinChunk;   // no split is always empty
    if (s > hi) s = hi;
    if (s < lo) s = lo;
    return s < 1 ? 1 : s;
}

size_t attention_partial_floats(uint32_t n_heads, uint32_t hd, uint32_t n_split) {
    return (size_t)n_heads * n_split * (hd + 2);
}

__host__ __device__ static uint32_t attn_chunk(uint32_t n, uint32_t n_split) {
    uint32_t c = (n + n_split - 1) / n_split;
    return c < kAttnMinChunk ? kAttnMinChunk : c;
}

__host__ __device__ static uint32_t attn_chunk_max(uint32_t max_ctx, uint32_t n_split) {
    return attn_chunk(max_ctx, n_split);
}

template <int HD>
__global__ void __launch_bounds__(kAttnThreads) smallm_attention_kernel(const AttnArgs a) {
    constexpr int EPL = HD / 32;               // head-dim elements per lane
    constexpr int PARTS = kAttnThreads / HD;   // position slices in the V pass
    extern __shared__ __align__(128) float sm[];
    const uint32_t G = a.n_heads / a.n_kv;
    const uint32_t g = blockIdx.x, split = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int nw = kAttnThreads / 32;
    const uint32_t chmax = attn_chunk_max(a.max_ctx, a.n_split);
    float* ks = sm;                            // [chmax][HD]
    float* vs = ks + (size_t)chmax * HD;       // [chmax][HD]
    float* qs = vs + (size_t)chmax * HD;       // [G][HD]
    float* sc = qs + G * HD;                   // [G][chmax]
    float* ml = sc + G * chmax;                // [G][2]
    float* red = ml + 2 * kAttnMaxGroup;       // [PARTS-1][HD][kAttnMaxGroup]
    __shared__ __align__(8) uint64_t bar;
    __shared__ unsigned int is_last;

    if (tid == 0) trace_mark(a.trace, 0);
    pdl_launch_dependents();
    pdl_wait();
    if (tid == 0) trace_mark(a.trace, 1);
    const uint32_t n = (a.pos ? *a.pos : a.pos_value) + 1;
    const uint32_t chunk = attn_chunk(n, a.n_split);
    const uint32_t t0 = split * chunk;
    const uint32_t t1 = min(n, t0 + chunk);
    const uint32_t len = t0 < t1 ? t1 - t0 : 0;
    float* part = a.partial + ((size_t)g * a.n_split + split) * G * (HD + 2);

    if (len > 0) {
        if (tid == 0) {
            mbar_init(&bar, 1);
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        }
        __syncthreads();
        if (tid == 0) {
            const uint32_t bytes = len * HD * 4;
            mbar_arrive_expect_tx(&bar, 2 * bytes);
            bulk_g2s(ks, a.kcache + ((size_t)g * a.max_ctx + t0) * HD, bytes, &bar);
            bulk_g2s(vs, a.vcache + ((size_t)g * a.max_ctx + t0) * HD, bytes, &bar);
        }
        for (uint32_t i = tid; i < G * HD; i += kAttnThreads) qs[i] = a.q[(size_t)g * G * HD + i];
        __syncthreads();
        const bool ok = mbar_wait(&bar, 0);
        if (!ok) {
            if (tid == 0 && a.err) atomicOr(a.err, 4u);
            // the two copies may still be landing in ks / vs: wait once more
            // (bounded) before the CTA reuses that memory or exits; the error
            // bit stays raised and the math below skips the staged rows
            mbar_wait(&bar, 0);
        }
        const float scale = 1.0f / sqrtf((float)HD);

        // scores: one warp per position, lanes split the head dimension
        for (uint32_t t = warp; t < len; t += nw) {
            float kv[EPL];
#pragma unroll
            for (int e = 0; e < EPL; ++e) kv[e] = ok ? ks[t * HD + lane + 32 * e] : 0.f;
#pragma unroll
            for (int h = 0; h < kAttnMaxGroup; ++h) {
                if (h < (int)G) {
                    float p = 0.f;
#pragma unroll
                    for (int e = 0; e < EPL; ++e) p = fmaf(qs[h * HD + lane + 32 * e], kv[e], p);
                    p = warp_sum(p);
                    if (lane == 0) sc[h * chmax + t] = p * scale;
                }
            }
        }
        __syncthreads();

        // softmax numerators and sums per head (ops::softmax, ops.cpp:43-57)
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

        // o[h][d] = sum_t p[h][t] v[t][d]: thread -> (d, slice of positions)
        const int d = tid % HD, pi = tid / HD;
        float acc[kAttnMaxGroup];
#pragma unroll
        for (int h = 0; h < kAttnMaxGroup; ++h) acc[h] = 0.f;
        for (uint32_t i = pi; i < len; i += PARTS) {
            const float v = ok ? vs[i * HD + d] : 0.f;
#pragma unroll
            for (int h = 0; h < kAttnMaxGroup; ++h)
                if (h < (int)G) acc[h] = fmaf(sc[h * chmax + i], v, acc[h]);
        }
        if constexpr (PARTS > 1) {
            if (pi > 0)
                for (int h = 0; h < kAttnMaxGroup; ++h) red[((pi - 1) * HD + d) * kAttnMaxGroup + h] = acc[h];
            __syncthreads();
        }
        if (pi == 0) {
            for (uint32_t h = 0; h < G; ++h) {
                float o = acc[h];
#pragma unroll
                for (int k = 1; k < PARTS; ++k) o += red[((k - 1) * HD + d) * kAttnMaxGroup + h];
                part[h * (HD + 2) + d] = o;
                if (d == 0) {
                    part[h * (HD + 2) + HD] = ml[2 * h];
                    part[h * (HD + 2) + HD + 1] = ml[2 * h + 1];
                }
            }
        }
    }

    // last CTA of this KV head merges the partials of the non-empty chunks
    __threadfence();
    __syncthreads();
    if (tid == 0) is_last = (atomicAdd(&a.counter[g], 1u) == a.n_split - 1) ? 1u : 0u;
    __syncthreads();
    if (!is_last) {
        if (tid == 0) trace_mark(a.trace, 2);
        return;
    }
    __threadfence();
    const float* base = a.partial + (size_t)g * a.n_split * G * (HD + 2);
    const uint32_t nact = min(a.n_split, (n + chunk - 1) / chunk);
    // (max, sum) of every active chunk and head in one parallel load; the
    // per-chunk weights exp(m_s - M) / L then come from shared memory, and
    // the partial outputs are summed with loads independent of the sum.
    float* wts = sm;  // [nact][G] weights (the K/V staging is no longer needed)
    for (uint32_t i = tid; i < nact * G; i += kAttnThreads) {
        const float* r = base + (size_t)i * (HD + 2);
        wts[i] = __ldcg(r + HD);
        wts[nact * G + i] = __ldcg(r + HD + 1);
    }
    __syncthreads();
    if (tid < (int)G) {
        float M = -INFINITY;
        for (uint32_t s = 0; s < nact; ++s) M = fmaxf(M, wts[s * G + tid]);
        float L = 0.f;
        for (uint32_t s = 0; s < nact; ++s) {
            const float w = expf(wts[s * G + tid] - M);
            wts[s * G + tid] = w;
            L = fmaf(w, wts[nact * G + s * G + tid], L);
        }
        for (uint32_t s = 0; s < nact; ++s) wts[s * G + tid] /= L;
    }
    __syncthreads();
    for (uint32_t o = tid; o < G * HD; o += kAttnThreads) {
        const uint32_t h = o / HD, dd = o % HD;
        float O = 0.f;
#pragma unroll 8
        for (uint32_t s = 0; s < nact; ++s) O = fmaf(wts[s * G + h], __ldcg(base + (s * G + h) * (HD + 2) + dd), O);
        a.out[((size_t)g * G + h) * HD + dd] = O;
    }
    if (tid == 0) a.counter[g] = 0u;
    __syncthreads();
    if (tid == 0) trace_mark(a.trace, 2);
}

size_t attention_smem(uint32_t n_heads, uint32_t n_kv, uint32_t hd, uint32_t max_ctx, uint32_t n_split) {
    const uint32_t G = n_heads / n_kv;
    const uint32_t chmax = attn_chunk_max(max_ctx, n_split);
    const size_t main = 2 * (size_t)chmax * hd + (size_t)G * hd + (size_t)G * chmax + 2 * kAttnMaxGroup +
                        (size_t)(kAttnThreads - hd) * kAttnMaxGroup;
    const size_t combine = 2 * (size_t)n_split * G;  // the merging CTA's (max, sum) staging
    return sizeof(float) * (main > combine ? main : combine);
}

void launch_attention(const AttnArgs& a, cudaStream_t stream, bool pdl) {
    const uint32_t G = a.n_heads / a.n_kv;
    if (G > (uint32_t)kAttnMaxGroup || a.n_heads % a.n_kv)
        throw Error(1, "attention: unsupported head grouping");
    const size_t smem = attention_smem(a.n_heads, a.n_kv, a.hd, a.max_ctx, a.n_split);
    if (smem > 200 * 1024) throw Error(1, "attention: chunk does not fit in shared memory");
    AttnArgs aa = a;
    void* args[] = {&aa};
    const void* fn;
    if (a.hd == 32) fn = (const void*)smallm_attention_kernel<32>;
    else if (a.hd == 64) fn = (const void*)smallm_attention_kernel<64>;
    else if (a.hd == 128) fn = (const void*)smallm_attention_kernel<128>;
    else throw Error(1, "attention: head_dim must be 32, 64 or 128");
    // the shared-memory limit is a per-device attribute of each function: set
    // it once per (device, kernel)
    set_smem_limit_once(fn, 200 * 1024);
    launch_kernel_ex(fn, dim3(a.n_kv, a.n_split), dim3(kAttnThreads), smem, stream, pdl, args);
}

// ---------------------------------------------------------------------------
// Cluster attention: the decode step's attention.
//
// One thread-block cluster of C CTAs per KV head; CTA c of the cluster owns
// the c-th of C equal contiguous ranges of positions 0..pos.  It stages its
// range in chunks sized for the model's context (32-256 positions, usually
// the whole range in one; K and V rows: two bulk copies on one mbarrier),
// scores the `group` query heads of the KV head against them, and keeps a
// running (max, sum, unnormalised output) per head across its chunks (online
// softmax).
//
// Before the dependency wait.  The position is fixed for the whole step (only
// the step's last kernel advances it) and rows below it were written by
// earlier steps, so the first chunk's rows other than the new one are copied
// into shared memory while the QKV kernel still runs; the QKV kernel leaves
// room on each SM for this kernel's CTAs.  After the wait only q and the new
// row are read (the position is re-read, and a mismatch reloads the chunk).
//
// Merge.  Each CTA pushes its partial into its peers' shared memory: the
// (max, sum) of every head to every CTA, and each output element to the CTA
// that merges it (CTA j merges a 1/C slice), then arrives on each peer's
// merge mbarrier.  A CTA waits only for its own C arrivals, merges its slice
// and writes it.  A split cluster barrier publishes the mbarrier
// initialisation (arrive at the start, wait before the first push) and keeps
// every CTA alive until all of its peers' pushes are done (arrive after the
// pushes, wait at the end).  No global scratch, no atomics, one launch.
// 4 warps per CTA, or 8 when a CTA's chunk holds 64 positions or more (long
// contexts: half the score and V passes; measured on the TinyLlama shape)
__host__ __device__ constexpr int cattn_threads(uint32_t chunk) { return chunk >= 64 ? 256 : 128; }
constexpr uint32_t kCAttnChunkUnit = 32;  // chunks are 1..kCAttnMaxUnits units of positions
constexpr uint32_t kCAttnMaxUnits = 8;
constexpr uint32_t kCAttnMaxCluster = 16;
constexpr uint32_t kCAttnMaxParts = 4;  // clusters per KV head

// Clusters per KV head for contexts up to max_ctx: with few KV heads one
// cluster of C CTAs per head leaves most SMs idle, so long contexts
// (>= 1024 positions) split each head's positions over up to 4 clusters
// while n_kv * parts * C stays within the SMs.
uint32_t attention_cluster_parts(uint32_t n_kv, uint32_t C, uint32_t max_ctx, int sm_count) {
    if (max_ctx < 1024) return 1;
    uint32_t parts = 1;
    while (parts < kCAttnMaxParts && n_kv * (parts * 2) * C <= (uint32_t)sm_count) parts *= 2;
    return parts;
}

__host__ __device__ constexpr size_t cattn_smem_floats(uint32_t G, uint32_t hd, uint32_t chunk) {
    // (the V-pass slice partials below are sized for the chunk's thread count)
    return 2 * (size_t)chunk * hd                          // ks, vs
           + (size_t)G * hd                                // qs
           + (size_t)G * chunk                             // sc
           + 3 * kAttnMaxGroup                             // corr, pm, pl
           + (size_t)(cattn_threads(chunk) - hd) * kAttnMaxGroup  // V-pass slice partials
           + (size_t)G * hd + kCAttnMaxCluster             // received output slices: C x ceil(G hd / C)
           + 2 * (size_t)kCAttnMaxCluster * kAttnMaxGroup  // received (max, sum) per CTA and head
           + (size_t)kAttnMaxGroup * kCAttnMaxCluster;     // merge weights
}

// Positions [b, e) of CTA `rank` of the cluster for part kp of a KV head's
// positions 0..n-1 split into `parts` equal ranges, each over C CTAs.
__device__ __forceinline__ void cattn_range(uint32_t n, uint32_t parts, uint32_t kp, uint32_t C, uint32_t rank,
                                            uint32_t& b, uint32_t& e) {
    const uint32_t pp = (n + parts - 1) / parts;
    const uint32_t pb = min(n, kp * pp), pe = min(n, pb + pp);
    const uint32_t per = (pe - pb + C - 1) / C;
    b = min(pe, pb + rank * per);
    e = min(pe, b + per);
}

template <int HD, int T>
__global__ void __launch_bounds__(T) smallm_attention_cluster_kernel(const AttnArgs a) {
    constexpr int kCAttnThreads = T;           // 128 or 256 (cattn_threads of the chunk)
    constexpr int PARTS = kCAttnThreads / HD;  // position slices in the V pass
    constexpr int DL = HD / 8;                 // head-dim elements per lane in the score pass
    constexpr int DV = DL / 4;                 // ... as float4
    extern __shared__ __align__(128) float sm[];
    __shared__ __align__(8) uint64_t bar, bar_pre, mrg;
    __shared__ uint32_t pre_n, pre_rows, early;
    cg::cluster_group cluster = cg::this_cluster();
    const uint32_t C = cluster.num_blocks();
    const uint32_t rank = cluster.block_rank();
    const uint32_t G = a.n_heads / a.n_kv;
    const uint32_t NP = a.parts;               // clusters per KV head
    const uint32_t g = blockIdx.x / C / NP;    // KV head of this cluster
    const uint32_t kp = blockIdx.x / C % NP;   // its part of the head's positions
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int nw = kCAttnThreads / 32;
    const uint32_t S = (G * HD + C - 1) / C;  // outputs merged per CTA
    const uint32_t CH = a.chunk;  // positions per chunk (a multiple of kCAttnChunkUnit)
    float* ks = sm;
    float* vs = ks + (size_t)CH * HD;
    float* qs = vs + (size_t)CH * HD;
    float* sc = qs + G * HD;
    float* corr = sc + G * CH;
    float* pm = corr + kAttnMaxGroup;
    float* pl = pm + kAttnMaxGroup;
    float* red = pl + kAttnMaxGroup;
    float* rpo = red + (kCAttnThreads - HD) * kAttnMaxGroup;  // [C][S]
    float* rm = rpo + G * HD + kCAttnMaxCluster;               // [C][G]
    float* rl = rm + kCAttnMaxCluster * kAttnMaxGroup;         // [C][G]
    float* wts = rl + kCAttnMaxCluster * kAttnMaxGroup;        // [G][kCAttnMaxCluster]

    if (tid == 0) {
        trace_mark(a.trace, 0);
        mbar_init(&bar, 1);
        mbar_init(&bar_pre, 1);
        mbar_init(&mrg, 1);
        // the merge barrier completes when every peer's pushed bytes are in:
        // (its slice of outputs + its (max, sum) per head) from each of the C CTAs
        const uint32_t lo = min(G * HD, rank * S), slice = min(S, G * HD - lo);
        mbar_arrive_expect_tx(&mrg, C * (slice + 2 * G) * 4);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    cluster_arrive_relaxed();  // matched by the cluster_wait before the first push
    pdl_launch_dependents();
    if (tid == 0) {
        const uint32_t n0 = min(*(volatile const uint32_t*)a.pos + 1, a.max_ctx);
        uint32_t b0, e0;
        cattn_range(n0, NP, kp, C, rank, b0, e0);
        // rows below the position are final; the new row comes after the wait
        const uint32_t fin = min(min(e0, b0 + CH), n0 - 1);
        const uint32_t rows = fin > b0 ? fin - b0 : 0u;
        if (rows) {
            const uint32_t bytes = rows * HD * 4;
            const size_t off = ((size_t)g * a.max_ctx + b0) * HD;
            mbar_arrive_expect_tx(&bar_pre, 2 * bytes);
            bulk_g2s(ks, a.kcache + off, bytes, &bar_pre);
            bulk_g2s(vs, a.vcache + off, bytes, &bar_pre);
        }
        // warm L2 with the rest of the range (longer contexts)
        if (e0 > b0 + CH) {
            const uint32_t bytes = (e0 - b0 - CH) * HD * 4;
            const size_t off = ((size_t)g * a.max_ctx + b0 + CH) * HD;
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a.kcache + off), "r"(bytes) : "memory");
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a.vcache + off), "r"(bytes) : "memory");
        }
        pre_n = n0;
        pre_rows = rows;
    }
    pdl_wait();
    if (tid == 0) {
        trace_mark(a.trace, 1);
        // the rest of the first chunk (from the row the QKV kernel has just
        // written) is copied right away, overlapping the q load
        const uint32_t n1 = pre_n;
        uint32_t b1, e1;
        cattn_range(n1, NP, kp, C, rank, b1, e1);
        const uint32_t len1 = min(CH, e1 - b1);
        uint32_t e = 0;
        if (pre_rows < len1) {
            const uint32_t bytes = (len1 - pre_rows) * HD * 4;
            const size_t off = ((size_t)g * a.max_ctx + b1 + pre_rows) * HD;
            mbar_arrive_expect_tx(&bar, 2 * bytes);
            bulk_g2s(ks + pre_rows * HD, a.kcache + off, bytes, &bar);
            bulk_g2s(vs + pre_rows * HD, a.vcache + off, bytes, &bar);
            e = 1;
        }
        early = e;
    }
    {
        const float4* q4 = reinterpret_cast<const float4*>(a.q + (size_t)g * G * HD);
        for (uint32_t i = tid; i < G * HD / 4; i += kCAttnThreads) reinterpret_cast<float4*>(qs)[i] = q4[i];
    }
    if (tid < kAttnMaxGroup) {
        pm[tid] = -INFINITY;
        pl[tid] = 0.f;
    }
    bool ok = true;
    __syncthreads();  // pre_n / pre_rows / early
    // The position read before the wait is the step's: only the step's last
    // kernel advances it (checked once more at the end).
    const uint32_t n = pre_n;
    uint32_t t_begin, t_end;
    cattn_range(n, NP, kp, C, rank, t_begin, t_end);
    if (pre_rows) {  // the first chunk's rows copied before the dependency wait
        if (!mbar_wait(&bar_pre, 0)) {
            ok = false;
            if (tid == 0 && a.err) atomicOr(a.err, 4u);
        }
    }
    const float scale = 1.0f / sqrtf((float)HD);
    const int d = tid % HD, part = tid / HD;
    float acc[kAttnMaxGroup];
#pragma unroll
    for (int h = 0; h < kAttnMaxGroup; ++h) acc[h] = 0.f;
    // The chunk is sized for the step's longest range (attention_cluster_chunk),
    // so at most one chunk after the first remains; the first arrived whole
    // before the wait but for the new row.
    uint32_t phase = 0;
    for (uint32_t c0 = t_begin; c0 < t_end; c0 += CH) {
        const uint32_t len = min(CH, t_end - c0);
        const bool first = c0 == t_begin;
        __syncthreads();  // the previous chunk's K/V/scores are no longer read (and q is staged)
        if (!first && tid == 0) {
            const uint32_t bytes = len * HD * 4;
            const size_t off = ((size_t)g * a.max_ctx + c0) * HD;
            mbar_arrive_expect_tx(&bar, 2 * bytes);
            bulk_g2s(ks, a.kcache + off, bytes, &bar);
            bulk_g2s(vs, a.vcache + off, bytes, &bar);
        }
        if (!first || early) {
            if (!mbar_wait(&bar, phase)) {
                ok = false;
                if (tid == 0 && a.err) atomicOr(a.err, 4u);
            }
            phase ^= 1u;
        }
        // scores: 8 lanes per position, lane k of the 8 holds elements
        // 4k + 32j .. +3 (conflict-free float4 rows), 16 positions per pass.
        // The pass loop is uniform across the CTA (all lanes reach the
        // shuffles); groups past the chunk's end compute on zeros.
        const int l8 = tid & 7, grp = tid >> 3;
        for (uint32_t tb = 0; tb < len; tb += kCAttnThreads / 8) {
            const uint32_t t = tb + grp;
            const bool act = ok && t < len;
            float4 kv[DV];
#pragma unroll
            for (int j = 0; j < DV; ++j)
                kv[j] = act ? reinterpret_cast<const float4*>(ks + t * HD)[l8 + 8 * j] : make_float4(0.f, 0.f, 0.f, 0.f);
            // heads unrolled so their dot products and shuffles interleave
            float s[kAttnMaxGroup];
#pragma unroll
            for (int h = 0; h < kAttnMaxGroup; ++h) {
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
                for (int h = 0; h < kAttnMaxGroup; ++h)
                    if (h < (int)G) s[h] += __shfl_xor_sync(0xffffffffu, s[h], o);
            }
            if (l8 == 0 && t < len) {
#pragma unroll
                for (int h = 0; h < kAttnMaxGroup; ++h)
                    if (h < (int)G) sc[h * CH + t] = s[h] * scale;
            }
        }
        __syncthreads();
        // online softmax (ops::softmax, ops.cpp:43-57, across chunks)
        for (uint32_t h = warp; h < G; h += nw) {
            float mx = -INFINITY;
            for (uint32_t t = lane; t < len; t += 32) mx = fmaxf(mx, sc[h * CH + t]);
            const float m_old = pm[h];
            const float m_new = fmaxf(m_old, warp_max(mx));
            float l = 0.f;
            for (uint32_t t = lane; t < len; t += 32) {
                const float e = expf(sc[h * CH + t] - m_new);
                sc[h * CH + t] = e;
                l += e;
            }
            l = warp_sum(l);
            if (lane == 0) {
                const float cf = m_old == -INFINITY ? 0.f : expf(m_old - m_new);
                corr[h] = cf;
                pl[h] = fmaf(pl[h], cf, l);
                pm[h] = m_new;
            }
        }
        __syncthreads();
        // o[h][d] = o[h][d] * corr[h] + sum_t p[h][t] v[t][d]
#pragma unroll
        for (int h = 0; h < kAttnMaxGroup; ++h)
            if (h < (int)G) acc[h] *= corr[h];
        for (uint32_t t = part; t < len; t += PARTS) {
            const float v = ok ? vs[t * HD + d] : 0.f;
#pragma unroll
            for (int h = 0; h < kAttnMaxGroup; ++h)
                if (h < (int)G) acc[h] = fmaf(sc[h * CH + t], v, acc[h]);
        }
    }
    if constexpr (PARTS > 1) {
        __syncthreads();
        if (part > 0) {
#pragma unroll
            for (int h = 0; h < kAttnMaxGroup; ++h) red[((part - 1) * HD + d) * kAttnMaxGroup + h] = acc[h];
        }
        __syncthreads();
        if (part == 0) {
#pragma unroll
            for (int h = 0; h < kAttnMaxGroup; ++h)
#pragma unroll
                for (int k = 1; k < PARTS; ++k) acc[h] += red[((k - 1) * HD + d) * kAttnMaxGroup + h];
        }
    }
    __syncthreads();  // pm / pl final
    cluster_wait();   // every peer's merge barrier is initialised
    // push this CTA's partial with asynchronous remote stores that count
    // their bytes on the receiver's merge barrier: output h*HD + d to the CTA
    // merging it (row `rank` of its slice table), (max, sum) to every CTA
    if (part == 0) {
#pragma unroll
        for (int h = 0; h < kAttnMaxGroup; ++h) {
            if (h < (int)G) {
                const uint32_t o = (uint32_t)h * HD + d, j = o / S;
                st_async_remote(rpo + rank * S + (o - j * S), j, acc[h], &mrg);
            }
        }
    }
    for (uint32_t i = tid; i < C * G; i += kCAttnThreads) {
        const uint32_t j = i / G, h = i % G;
        st_async_remote(rm + rank * G + h, j, pm[h], &mrg);
        st_async_remote(rl + rank * G + h, j, pl[h], &mrg);
    }
    cluster_arrive_release();  // matched at the end: peers stay alive until every push has landed
    // merge this CTA's slice once all C partials are here
    if (!mbar_wait(&mrg, 0)) {
        ok = false;
        if (tid == 0 && a.err) atomicOr(a.err, 4u);
    }
    // weights of the C partials per head: warp h, lane c
    for (uint32_t h = warp; h < G; h += nw) {
        const float mc = (uint32_t)lane < C ? rm[lane * G + h] : -INFINITY;
        const float lc = (uint32_t)lane < C ? rl[lane * G + h] : 0.f;
        const float M = warp_max(mc);
        const float e = mc == -INFINITY ? 0.f : expf(mc - M);
        const float L = warp_sum(e * lc);
        // a part of a KV head with no positions yet (parts > 1, short
        // context) has L = 0: its output is zero and its weight below is zero
        if ((uint32_t)lane < C) wts[h * kCAttnMaxCluster + lane] = L > 0.f ? e / L : 0.f;
        if (NP > 1 && rank == 0 && lane == 0) {
            float* ml = a.part_ml + ((size_t)kp * a.n_heads + (size_t)g * G + h) * 2;
            ml[0] = M;
            ml[1] = L;
        }
    }
    __syncthreads();
    for (uint32_t ol = tid; ol < S; ol += kCAttnThreads) {
        const uint32_t o = rank * S + ol;
        if (o >= G * HD) break;
        const float* w = wts + (o / HD) * kCAttnMaxCluster;
        float O = 0.f;
        for (uint32_t c = 0; c < C; ++c) O = fmaf(w[c], rpo[c * S + ol], O);
        // one part: the head's output; several: this part's normalised
        // output, weighted by (M, L) when the next kernel stages it
        float* dst = NP > 1 ? a.part_out + (size_t)kp * a.n_heads * HD : a.out;
        dst[(size_t)g * G * HD + o] = O;
    }
    cluster_wait();
    if (tid == 0 && a.err && min(*(volatile const uint32_t*)a.pos + 1, a.max_ctx) != pre_n)
        atomicOr(a.err, 32u);  // the position moved during the step: results invalid
    if (tid == 0) trace_mark(a.trace, 2);
}

size_t attention_cluster_smem(uint32_t n_heads, uint32_t n_kv, uint32_t hd, uint32_t chunk) {
    return 4 * cattn_smem_floats(n_heads / n_kv, hd, chunk);
}

// Positions per chunk of the cluster attention for contexts up to max_ctx
// over clusters of C: a CTA's longest range rounded up to 32, at most 256
// positions and 96 KB of K/V rows.  With the whole range in one chunk a CTA
// copies all its rows but the step's new one before the dependency wait
// (while the QKV kernel runs) and scores them in one pass (measured on the
// TinyLlama shape at ~2050 positions: 32-position chunks, one at a time,
// took ~20 us per layer).
uint32_t attention_cluster_chunk(uint32_t max_ctx, uint32_t C, uint32_t hd, uint32_t parts) {
    const uint32_t per = ((max_ctx + parts - 1) / parts + C - 1) / C;
    uint32_t u = (per + kCAttnChunkUnit - 1) / kCAttnChunkUnit;
    u = u < 1 ? 1 : (u > kCAttnMaxUnits ? kCAttnMaxUnits : u);
    while (u > 1 && 2ull * u * kCAttnChunkUnit * hd * 4 > 96 * 1024) --u;
    return u * kCAttnChunkUnit;
}

static const void* cattn_fn(uint32_t hd, uint32_t chunk) {
    const bool wide = cattn_threads(chunk) == 256;
    if (hd == 32) return wide ? (const void*)smallm_attention_cluster_kernel<32, 256>
                              : (const void*)smallm_attention_cluster_kernel<32, 128>;
    if (hd == 64) return wide ? (const void*)smallm_attention_cluster_kernel<64, 256>
                              : (const void*)smallm_attention_cluster_kernel<64, 128>;
    if (hd == 128) return wide ? (const void*)smallm_attention_cluster_kernel<128, 256>
                               : (const void*)smallm_attention_cluster_kernel<128, 128>;
    throw Error(SMALLM_ERR_INVALID, "attention: head_dim must be 32, 64 or 128");
}

uint32_t attention_cluster_size(uint32_t n_heads, uint32_t n_kv, uint32_t hd, uint32_t chunk) {
    const void* fn = cattn_fn(hd, chunk);
    const size_t smem = 4 * cattn_smem_floats(n_heads / n_kv, hd, chunk);
    SM_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    SM_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
#ifndef SMALLM_ATTN_CLUSTER
#define SMALLM_ATTN_CLUSTER 16u  // largest cluster tried (a power of two <= kCAttnMaxCluster)
#endif
    for (uint32_t C = SMALLM_ATTN_CLUSTER; C > 1; C /= 2) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(n_kv * C);
        cfg.blockDim = dim3(cattn_threads(chunk));
        cfg.dynamicSmemBytes = smem;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = C;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int nclusters = 0;
        if (cudaOccupancyMaxActiveClusters(&nclusters, fn, &cfg) == cudaSuccess && nclusters > 0) return C;
        (void)cudaGetLastError();
    }
    return 1;
}

void launch_attention_cluster(const AttnArgs& a, uint32_t C, cudaStream_t stream, bool pdl) {
    const uint32_t G = a.n_heads / a.n_kv;
    if (G > (uint32_t)kAttnMaxGroup || a.n_heads % a.n_kv)
        throw Error(SMALLM_ERR_INVALID, "attention: unsupported head grouping");
    if (C < 1 || C > kCAttnMaxCluster) throw Error(SMALLM_ERR_INVALID, "attention: bad cluster size");
    const void* fn = cattn_fn(a.hd, a.chunk);
    cudaLaunchConfig_t cfg = {};
    if (a.parts < 1 || a.parts > kCAttnMaxParts || (a.parts > 1 && (!a.part_out || !a.part_ml)))
        throw Error(SMALLM_ERR_INVALID, "attention: bad part count or missing part buffers");
    cfg.gridDim = dim3(a.n_kv * a.parts * C);
    cfg.blockDim = dim3(cattn_threads(a.chunk));
    if (a.chunk < kCAttnChunkUnit || a.chunk > kCAttnChunkUnit * kCAttnMaxUnits || a.chunk % kCAttnChunkUnit)
        throw Error(SMALLM_ERR_INVALID, "attention: bad chunk size");
    cfg.dynamicSmemBytes = 4 * cattn_smem_floats(G, a.hd, a.chunk);
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = C;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.numAttrs = 1;
    if (pdl) {
        attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[1].val.programmaticStreamSerializationAllowed = 1;
        cfg.numAttrs = 2;
    }
    cfg.attrs = attr;
    AttnArgs aa = a;
    void* args[] = {&aa};
    SM_CUDA(cudaLaunchKernelExC(&cfg, fn, args));
}

// ---------------------------------------------------------------------------
// The same attention kernel with library-owned static scratch.
//
// A loaded model allocates its attention scratch once, at load.  A caller that
// keeps its own q / K / V on the device and wants only this kernel may be
// unable to let the library allocate at all: a serving engine that has handed
// the GPU's memory to its own KV-block pool has none left for cudaMalloc to
// find, and cudaMalloc / cudaFree can synchronise the device, which a
// latency-bound decode loop cannot absorb.  For those callers the split-K
// partials and the per-KV-head tickets live in this one
// fixed array of the module, so a call allocates nothing.
//
// Layout: [0, kAttnStaticPartialBytes) partials, then kAttnStaticMaxKv
// tickets (u32, must be zero before a launch; the merging CTA of each KV head
// puts its ticket back to zero).  The position goes to the kernel as a
// parameter.  Tickets start at zero because the first call on a device clears
// them on its stream before its launch.  Every call on a device shares this
// array, so calls whose kernels overlap in time (other streams, other threads)
// race on it; callers must order them.
constexpr size_t kAttnStaticPartialBytes = 4u << 20;  // 4 MiB
constexpr uint32_t kAttnStaticMaxKv = 256;
constexpr size_t kAttnStaticTicketOff = kAttnStaticPartialBytes;
constexpr size_t kAttnStaticBytes = kAttnStaticTicketOff + 4 * kAttnStaticMaxKv;
static __device__ __align__(256) unsigned char g_attn_scratch[kAttnStaticBytes];

constexpr int kAttnStaticMaxDevices = 64;
static std::mutex g_attn_static_mu;
static unsigned char* g_attn_static_base[kAttnStaticMaxDevices];

// Device address of g_attn_scratch on the current device; the first call for a
// device looks it up (once, with that device current) and zeroes the tickets on
// `stream`, ahead of that call's launch.
static unsigned char* attention_static_scratch(cudaStream_t stream) {
    int dev = 0;
    SM_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kAttnStaticMaxDevices) throw Error(SMALLM_ERR_RANGE, "attention (static scratch): device ordinal too large");
    std::lock_guard<std::mutex> lock(g_attn_static_mu);
    if (!g_attn_static_base[dev]) {
        void* p = nullptr;
        const cudaError_t rc = cudaGetSymbolAddress(&p, g_attn_scratch);
        if (rc != cudaSuccess || !p)
            throw Error(SMALLM_ERR_CUDA, std::string("attention (static scratch): cudaGetSymbolAddress failed: ") +
                                             cudaGetErrorString(rc));
        unsigned char* base = static_cast<unsigned char*>(p);
        SM_CUDA(cudaMemsetAsync(base + kAttnStaticTicketOff, 0, 4 * kAttnStaticMaxKv, stream));
        g_attn_static_base[dev] = base;
    }
    return g_attn_static_base[dev];
}

void launch_attention_static(const float* q, const float* kcache, const float* vcache, uint32_t n_heads,
                             uint32_t n_kv, uint32_t hd, uint32_t max_ctx, uint32_t pos, float* out,
                             cudaStream_t stream) {
    if (!n_heads || !n_kv || n_heads % n_kv || n_heads / n_kv > (uint32_t)kAttnMaxGroup)
        throw Error(SMALLM_ERR_INVALID, "attention: n_heads must be a multiple of n_kv_heads, at most 8 per KV head");
    if (hd != 32 && hd != 64 && hd != 128) throw Error(SMALLM_ERR_INVALID, "attention: head_dim must be 32, 64 or 128");
    if (pos >= max_ctx) throw Error(SMALLM_ERR_RANGE, "attention: pos must be below max_ctx");
    if (n_kv > kAttnStaticMaxKv)
        throw Error(SMALLM_ERR_RANGE, "attention (static scratch): more than 256 KV heads");
    const uint32_t n_split = attention_splits(n_kv, max_ctx, device_sm_count());
    const size_t need = 4 * attention_partial_floats(n_heads, hd, n_split);
    if (need > kAttnStaticPartialBytes)
        throw Error(SMALLM_ERR_RANGE, "attention (static scratch): this shape needs " + std::to_string(need) +
                                          " bytes of partials for max_ctx " + std::to_string(max_ctx) +
                                          "; the static scratch holds 4194304 (lower max_ctx or n_heads)");
    if (attention_smem(n_heads, n_kv, hd, max_ctx, n_split) > 200 * 1024)
        throw Error(SMALLM_ERR_INVALID, "attention: chunk does not fit in shared memory");
    // K and V rows reach shared memory through bulk copies, whose global
    // source must be 16-byte aligned (row offsets are whole rows of head_dim
    // floats, so the base pointers decide)
    if ((reinterpret_cast<uintptr_t>(kcache) | reinterpret_cast<uintptr_t>(vcache)) & 15u)
        throw Error(SMALLM_ERR_INVALID, "attention: kcache_dev and vcache_dev must be 16-byte aligned");
    unsigned char* base = attention_static_scratch(stream);
    AttnArgs a;
    a.q = q;
    a.kcache = kcache;
    a.vcache = vcache;
    a.out = out;
    a.partial = reinterpret_cast<float*>(base);
    a.counter = reinterpret_cast<unsigned int*>(base + kAttnStaticTicketOff);
    a.pos = nullptr;
    a.pos_value = pos;
    a.n_heads = n_heads;
    a.n_kv = n_kv;
    a.hd = hd;
    a.max_ctx = max_ctx;
    a.n_split = n_split;
    a.err = device_error_flag();
    launch_attention(a, stream, false);
}

}  // namespace smallm
