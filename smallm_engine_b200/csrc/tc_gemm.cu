// Tensor-core GEMM of the batched prefill (sm_100a, tcgen05 + TMA):
//
//   Y[T][ldy] (f32, columns 0..N) = X[T][K] . W[N][K]^T      X, W: f16, row-major
//
// The prefill's linear layers are the one dense contraction of the engine
// (the reference runs them as one matmul_quantized per token,
// src/core/ops.cpp:103-184, called from Model::forward once per prompt token,
// src/runtime/generator.cpp:47-51).  A persistent grid (one CTA per SM)
// walks 128 x BN output tiles of W-rows x tokens (BN = 64, 128 or 256):
//   - warp 0, one lane: TMA producer.  2-D tiled bulk tensor copies of a
//     128 x 64 W tile and a BN x 64 X tile per stage (64 f16 = one 128-byte
//     row, 128-byte swizzle) into a ring of stages, completing on the stage's
//     mbarrier;
//   - warp 1, one lane: MMA issuer.  Four tcgen05.mma kind::f16 (K = 16 each)
//     per stage into an f32 accumulator in tensor memory; tcgen05.commit
//     frees the stage when its MMAs have read it.  Tiles alternate between two
//     accumulators (2 x BN TMEM columns), so one tile's epilogue overlaps the
//     next tile's MMAs;
//   - warps 2..5: epilogue.  Each reads its 32 accumulator lanes (tcgen05.ld
//     32x32b) and stores them: lane = W row, so a warp's stores of one
//     token's 32 outputs are one 128-byte line.
// Every mbarrier wait is bounded (mbar_wait: ~2^31 cycles); a wait that gives
// up raises bit 6 of the device error word and the CTA finishes without
// further MMAs, so the host sees an error instead of a hang.  On every exit
// path the producer first waits (bounded) for the last copy it issued into
// each stage and the MMA thread for all of its MMAs, so nothing lands in
// shared or tensor memory after the CTA has released them.
//
// Operands are f16 (11-bit significands, like TF32's): products are exact in
// the f32 accumulator.  No cluster launch: every CTA loads its own tiles.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "engine.h"
#include "smallm_cuda.h"

namespace smallm {
namespace {

constexpr uint32_t kBM = 128;  // W rows per tile: the MMA's M (one row per TMEM lane)
constexpr uint32_t kBK = 64;   // K per stage: 64 f16 = one 128-byte swizzle row
constexpr uint32_t kUK = 16;   // K of one tcgen05.mma kind::f16
constexpr unsigned kErrTcGemm = 64u;

template <uint32_t BN>
struct TcCfg {
    static_assert(BN == 64 || BN == 128 || BN == 256, "token tile");
    static constexpr uint32_t a_bytes = kBM * kBK * 2;  // 16 KB
    static constexpr uint32_t b_bytes = BN * kBK * 2;   // 8 / 16 / 32 KB
    static constexpr uint32_t stage_bytes = a_bytes + b_bytes;
    static constexpr uint32_t stages = 192u * 1024u / stage_bytes;  // 8 / 6 / 4
    static constexpr uint32_t tmem_cols = 2 * BN;                   // two f32 accumulators
    static constexpr size_t smem = 1024 + (size_t)stages * stage_bytes + 512;
};
constexpr uint32_t kThreads = 192;  // warp 0 TMA, warp 1 MMA, warps 2..5 epilogue

// ---- PTX wrappers ----------------------------------------------------------

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int32_t x, int32_t y,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// Shared-memory matrix descriptor of a K-major tile written by TMA with the
// 128-byte swizzle: rows of 128 bytes, 8-row groups 1024 bytes apart (stride
// byte offset), descriptor version 1, layout type 2 (SWIZZLE_128B).  The tile
// base is 1024-byte aligned, so the base-offset field stays 0 and stepping K
// by 16 elements adds 32 bytes to the start address.
__device__ __forceinline__ uint64_t smem_desc_sw128(const void* p) {
    const uint64_t addr = (smem_u32(p) >> 4) & 0x3FFFu;
    return addr | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor: f16 A and B (format 0), f32 D (format 1), both
// K-major, N = BN (bits 17..22 hold N/8), M = 128 (bits 24..28 hold M/16).
template <uint32_t BN>
__host__ __device__ constexpr uint32_t idesc_f16_f32() {
    return (1u << 4) | ((BN >> 3) << 17) | ((kBM >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive f32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
        "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---- the kernel --------------------------------------------------------------

template <uint32_t BN>
__global__ void __launch_bounds__(kThreads, 1)
    smallm_tc_gemm_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tx,
                   float* __restrict__ y, uint32_t N, uint32_t T, uint32_t K, uint32_t ldy, unsigned int* err) {
    using C = TcCfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte aligned base (the swizzle pattern is a function of the address)
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* sa = smem;
    uint8_t* sb = smem + C::stages * C::a_bytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(sb + C::stages * C::b_bytes);
    uint64_t* empty = full + C::stages;
    uint64_t* acc_full = empty + C::stages;  // [2] MMA -> epilogue: accumulator b complete
    uint64_t* acc_empty = acc_full + 2;      // [2] epilogue -> MMA: accumulator b drained
    uint64_t* mma_done = acc_empty + 2;      // every MMA this CTA issued has completed
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t nk = (K + kBK - 1) / kBK;
    const uint32_t n_t = (T + BN - 1) / BN;                 // token tiles (fastest: CTAs running
    const uint32_t tiles = n_t * ((N + kBM - 1) / kBM);     // together share W rows in L2)

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < C::stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (uint32_t b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 128);
        }
        mbar_init(mma_done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tw)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tx)) : "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(C::tmem_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // producer: a stage is refilled once the MMAs of its previous use completed
            uint32_t it = 0;
            uint32_t last[C::stages];  // last use issued into each stage
#pragma unroll
            for (uint32_t st = 0; st < C::stages; ++st) last[st] = ~0u;
            for (uint32_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
                const int32_t t0 = (int32_t)((tile % n_t) * BN), m0 = (int32_t)((tile / n_t) * kBM);
                bool ok = true;
                for (uint32_t kb = 0; kb < nk; ++kb, ++it) {
                    const uint32_t s = it % C::stages, use = it / C::stages;
                    if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[s], C::stage_bytes);
                    tma_load_2d(sa + s * C::a_bytes, &tw, (int32_t)(kb * kBK), m0, &full[s]);
                    tma_load_2d(sb + s * C::b_bytes, &tx, (int32_t)(kb * kBK), t0, &full[s]);
                    last[s] = use;
                }
                if (!ok) {
                    atomicOr(err, kErrTcGemm);
                    break;
                }
            }
            // no copy may still be landing in shared memory when the CTA exits
            // (immediate when the MMA warp has consumed them all)
#pragma unroll
            for (uint32_t st = 0; st < C::stages; ++st)
                if (last[st] != ~0u && !mbar_wait(&full[st], last[st] & 1)) atomicOr(err, kErrTcGemm);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // MMA issuer: tile j accumulates into TMEM columns (j & 1) * BN
            constexpr uint32_t idesc = idesc_f16_f32<BN>();
            uint32_t it = 0, j = 0;
            for (uint32_t tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++j) {
                const uint32_t b = j & 1, buse = j >> 1;
                if (buse > 0 && !mbar_wait(&acc_empty[b], (buse - 1) & 1)) {
                    atomicOr(err, kErrTcGemm);
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + b * BN;
                bool ok = true;
                for (uint32_t kb = 0; kb < nk; ++kb, ++it) {
                    const uint32_t s = it % C::stages, use = it / C::stages;
                    if (!mbar_wait(&full[s], use & 1)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t da = smem_desc_sw128(sa + s * C::a_bytes);
                    const uint64_t db = smem_desc_sw128(sb + s * C::b_bytes);
#pragma unroll
                    for (uint32_t k = 0; k < kBK / kUK; ++k)  // +32 bytes = +2 in the 16-byte address field
                        mma_f16(d, da + 2 * k, db + 2 * k, idesc, (kb | k) != 0);
                    mma_commit(&empty[s]);
                }
                mma_commit(&acc_full[b]);  // arrives when every MMA issued so far has completed
                if (!ok) {
                    atomicOr(err, kErrTcGemm);
                    break;
                }
            }
            // the tensor memory is freed below only after every MMA completed
            mma_commit(mma_done);
            if (!mbar_wait(mma_done, 0)) atomicOr(err, kErrTcGemm);
        }
    } else {
        // epilogue warps 2..5: warp w reads TMEM lanes (W rows) 32 (w % 4) .. + 31
        const uint32_t q = warp & 3;
        const uint32_t lane_base = tmem + ((q * 32u) << 16);
        uint32_t j = 0;
        for (uint32_t tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++j) {
            const uint32_t b = j & 1, buse = j >> 1;
            const uint32_t t0 = (tile % n_t) * BN, m = (tile / n_t) * kBM + q * 32 + lane;
            const bool ok = mbar_wait(&acc_full[b], buse & 1);
            __syncwarp();
            tc_fence_after();
#pragma unroll 1
            for (uint32_t c = 0; c < BN; c += 32) {
                uint32_t r[32];
                tmem_ld32(lane_base + b * BN + c, r);
                if (ok && m < N) {
#pragma unroll
                    for (uint32_t i = 0; i < 32; ++i) {
                        const uint32_t t = t0 + c + i;
                        if (t < T) y[(size_t)t * ldy + m] = __uint_as_float(r[i]);
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&acc_empty[b]);
            if (!ok) {
                if (lane == 0) atomicOr(err, kErrTcGemm);
                break;
            }
        }
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::tmem_cols)
                     : "memory");
    }
}

__global__ void smallm_f32_to_f16_kernel(const float* __restrict__ src, __half* __restrict__ dst, uint64_t n) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t n4 = n / 4;
    const float4* s4 = reinterpret_cast<const float4*>(src);
    __half2* d2 = reinterpret_cast<__half2*>(dst);
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
        const float4 v = s4[i];
        d2[2 * i] = __floats2half2_rn(v.x, v.y);
        d2[2 * i + 1] = __floats2half2_rn(v.z, v.w);
    }
    for (uint64_t i = 4 * n4 + (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        dst[i] = __float2half_rn(src[i]);
}

// ---- host side ---------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static std::mutex mu;
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    std::lock_guard<std::mutex> g(mu);
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        SM_CUDA(cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q));
        if (q != cudaDriverEntryPointSuccess || !p)
            throw Error(SMALLM_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
        fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// 2-D f16 map over a row-major [outer][inner] matrix, box = box_outer rows of
// 64 elements, 128-byte swizzle, zero fill outside the matrix.
CUtensorMap f16_map(const void* base, uint64_t inner, uint64_t outer, uint32_t box_outer) {
    CUtensorMap m;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {inner * 2};
    const cuuint32_t box[2] = {kBK, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = tensor_map_encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims,
                                            strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw Error(SMALLM_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
    return m;
}

template <uint32_t BN>
void launch_tc(const CUtensorMap& tw, const CUtensorMap& tx, float* Y, uint32_t N, uint32_t T, uint32_t K,
               uint32_t ldy, cudaStream_t s) {
    using C = TcCfg<BN>;
    static std::mutex mu;
    static std::unordered_map<int, bool> configured;
    int dev = 0;
    SM_CUDA(cudaGetDevice(&dev));
    {
        std::lock_guard<std::mutex> g(mu);
        if (!configured.count(dev)) {
            SM_CUDA(cudaFuncSetAttribute(smallm_tc_gemm_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)C::smem));
            configured[dev] = true;
        }
    }
    const uint64_t tiles = (uint64_t)((T + BN - 1) / BN) * ((N + kBM - 1) / kBM);
    const uint32_t grid = (uint32_t)std::min<uint64_t>(tiles, (uint64_t)device_sm_count());
    smallm_tc_gemm_kernel<BN><<<grid, kThreads, C::smem, s>>>(tw, tx, Y, N, T, K, ldy, device_error_flag());
    SM_CUDA(cudaGetLastError());
}

}  // namespace

// Token-tile width from a wave model of the persistent grid: per 64-wide K
// stage a 128 x BN tile costs max(MMA, shared-memory operand reads) =
// max(2 BN, 128 + BN) SM cycles (M=128, N=BN, K=16 MMAs at ~8 K flop/cycle;
// 16 KB of W plus BN x 128 bytes of X read at 128 bytes/cycle), and the
// grid runs ceil(tiles / SMs) rounds of tiles.  Ties go to the wider tile
// (fewer re-reads of W).
uint32_t tc_gemm_token_tile(uint32_t N, uint32_t T) {
    const uint64_t sms = (uint64_t)device_sm_count(), n_m = (N + kBM - 1) / kBM;
    uint32_t best = 64;
    uint64_t best_cost = ~0ull;
    for (uint32_t bn : {256u, 128u, 64u}) {
        const uint64_t tiles = (uint64_t)((T + bn - 1) / bn) * n_m;
        const uint64_t cost = (tiles + sms - 1) / sms * std::max<uint64_t>(2 * bn, 128 + bn);
        if (cost < best_cost) {
            best_cost = cost;
            best = bn;
        }
    }
    return best;
}

void launch_tc_gemm(const __half* W, uint32_t N, uint32_t K, const __half* X, uint32_t T, float* Y, uint32_t ldy,
                    cudaStream_t s) {
    if (N == 0 || T == 0) return;
    if (K == 0 || K % 8 != 0) throw Error(SMALLM_ERR_INVALID, "tc_gemm: K must be a positive multiple of 8");
    if (ldy < N) throw Error(SMALLM_ERR_INVALID, "tc_gemm: ldy < N");
    if ((reinterpret_cast<uintptr_t>(W) | reinterpret_cast<uintptr_t>(X)) & 15)
        throw Error(SMALLM_ERR_INVALID, "tc_gemm: W and X must be 16-byte aligned");
    const uint32_t bn = tc_gemm_token_tile(N, T);
    const CUtensorMap tw = f16_map(W, K, N, kBM);
    const CUtensorMap tx = f16_map(X, K, T, bn);
    if (bn == 256) launch_tc<256>(tw, tx, Y, N, T, K, ldy, s);
    else if (bn == 128) launch_tc<128>(tw, tx, Y, N, T, K, ldy, s);
    else launch_tc<64>(tw, tx, Y, N, T, K, ldy, s);
}

void launch_f32_to_f16(const float* src, __half* dst, uint64_t n, cudaStream_t s) {
    if (!n) return;
    if ((reinterpret_cast<uintptr_t>(src) & 15) || (reinterpret_cast<uintptr_t>(dst) & 7))
        throw Error(SMALLM_ERR_INVALID, "f32_to_f16: src must be 16-byte and dst 8-byte aligned");
    const uint64_t want = (n / 4 + 255) / 256;
    const uint32_t grid = (uint32_t)std::min<uint64_t>(std::max<uint64_t>(want, 1), 8ull * device_sm_count());
    smallm_f32_to_f16_kernel<<<grid, 256, 0, s>>>(src, dst, n);
    SM_CUDA(cudaGetLastError());
}

}  // namespace smallm
