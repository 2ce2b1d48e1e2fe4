// Shared device helpers for the sm_100a kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "trace.h"

#define SM_T_F32 0u
#define SM_T_Q4_0 2u
#define SM_T_Q8_0 8u
#define SM_T_Q4_K 12u
#define SM_T_Q6_K 14u

namespace smallm {

constexpr int kWarp = 32;

// IEEE half -> float by integer ops, bit-identical to the reference's
// f16_to_f32 (include/smallm/core/common/quant_common.h:15-40) including
// NaN payloads; used wherever dequantized values must match exactly.
__device__ __forceinline__ float f16_exact(uint32_t h) {
    uint32_t sign = (h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t mant = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0) {
        if (mant == 0) {
            bits = sign;
        } else {
            // normalise: shift the leading 1 of the 10-bit mantissa to bit 10
            int lz = __clz(mant) - 21;  // leading zeros within the 11-bit field
            mant = (mant << lz) & 0x3FFu;
            bits = sign | ((uint32_t)(113 - lz) << 23) | (mant << 13);
        }
    } else if (exp == 0x1F) {
        bits = sign | 0x7F800000u | (mant << 13);
    } else {
        bits = sign | ((exp + 112u) << 23) | (mant << 13);
    }
    return __uint_as_float(bits);
}

// Hardware half -> float; exact for every finite half (the GEMV hot loops
// use this for block scales).
__device__ __forceinline__ float h2f(uint32_t h) {
    return __half2float(__ushort_as_half((unsigned short)h));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Sum over the whole CTA (all threads must call it); `red` holds >= 32 floats.
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

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Reduce R per-lane partial sums across the warp so that every lane of the
// group of 32/R lanes starting at r*(32/R) ends with the full sum of row r.
// log2(R) reduce-scatter halvings, then plain butterflies.
template <int R>
__device__ __forceinline__ float warp_reduce_rows(float (&acc)[R], int lane) {
    static_assert(R == 1 || R == 2 || R == 4 || R == 8, "R must be 1, 2, 4 or 8");
    if constexpr (R == 1) {
        return warp_sum(acc[0]);
    } else {
        float v[R];
#pragma unroll
        for (int i = 0; i < R; ++i) v[i] = acc[i];
        int cnt = R;
        int off = 16;
#pragma unroll
        for (int step = 0; step < 3; ++step) {
            if (cnt == 1) break;
            const bool upper = (lane & off) != 0;
            const int h = cnt / 2;
#pragma unroll
            for (int i = 0; i < R / 2; ++i) {
                if (i < h) {
                    float keep = upper ? v[i + h] : v[i];
                    float send = upper ? v[i] : v[i + h];
                    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
                }
            }
            cnt = h;
            off >>= 1;
        }
        float s = v[0];
        for (; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
        return s;
    }
}

// Order-preserving map of a float to uint32 (larger float -> larger key).
__device__ __forceinline__ uint32_t float_order_key(float f) {
    uint32_t b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Pack (value, index) so that the maximum of the packed keys is the maximum
// value with the lowest index on ties: the reference's greedy sampler keeps
// the first strict maximum (src/runtime/sampler/greedy_sampler.cpp:8-14).
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
    return ((unsigned long long)float_order_key(v) << 32) | (0xFFFFFFFFu - idx);
}
// Index of a packed key; an empty key (no non-NaN candidate) maps to 0, the
// reference's answer when nothing beats logits[0].
__host__ __device__ __forceinline__ uint32_t argmax_key_index(unsigned long long k) {
    return k ? 0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull) : 0u;
}

// Programmatic dependent launch controls (no-ops when the kernel was not
// launched with the attribute).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------------------- kernel tracing --
// Kernels of the production graph get a null slot and skip all of it.
__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void trace_mark(TraceSlot* s, int which) {
    if (!s) return;
    const unsigned long long t = global_ns();
    if (which == 0) atomicMin(&s->t_start, t);
    else if (which == 1) atomicMin(&s->t_ready, t);
    else atomicMax(&s->t_end, t);
}

// ------------------------------------------- mbarriers and bulk copies --

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
// System-scope acquire load / release store of a flag another GPU writes or
// reads (peer memory over NVLink).
__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(unsigned int* p, unsigned int v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Wait for phase `parity` of the barrier to complete; gives up after about
// 2^31 SM cycles (~1 s) and returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    const uint32_t a = smem_u32(bar);
    const long long t0 = clock64();
    for (;;) {
        uint32_t ok;
        // the suspend-time hint (ns) lets the hardware park the thread until
        // the phase completes instead of returning early into a spin loop
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}"
            : "=r"(ok)
            : "r"(a), "r"(parity), "r"(1000000u)
            : "memory");
        if (ok) return true;
        if (clock64() - t0 > (1ll << 31)) return false;
    }
}
// Asynchronous store of one float into CTA `rank`'s shared memory at the
// offset of `p` in this CTA, completing 4 bytes on that CTA's barrier at the
// offset of `bar` (the receiver expects the bytes with mbar_arrive_expect_tx
// and sees the data once the phase completes).
__device__ __forceinline__ void st_async_remote(float* p, uint32_t rank, float v, uint64_t* bar) {
    uint32_t ra, rb;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(smem_u32(p)), "r"(rank));
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rb) : "r"(smem_u32(bar)), "r"(rank));
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(ra),
                 "r"(__float_as_uint(v)), "r"(rb)
                 : "memory");
}
// Split cluster barrier (every thread of every CTA of the cluster executes
// both, arrive first).
__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive_release() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// 1-D bulk copy global -> shared completing on `bar` (both addresses and the
// size are multiples of 16 bytes).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
}  // namespace smallm
