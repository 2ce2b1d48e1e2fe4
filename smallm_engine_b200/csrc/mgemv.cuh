// Batch-1 GEMV on the integer tensor cores for the 32-element block formats
// Q4_0 and Q8_0: y = W . x, x in three-digit block fixed point (gemv.cuh).
//
// Why mma.sync.m16n8k32 and not tcgen05: every 32-element block carries its
// own weight scale, so each block's integer dot must be scaled before it
// joins the row sum.  A tcgen05 MMA accumulates over K in tensor memory; a
// per-block result would need one tcgen05.ld per block and tile.  The
// register-fed m16n8k32 MMA hands a 16-row x 32-element product straight back
// to the threads that scale it.  The MMA replaces 24 IDP4A per block and row
// (three digits x eight 4-element words) by 1/16 of an instruction.
//
// Device layout (qmat_alloc / qmat_repack): storage rows in tiles of 16; a
// tile holds its block pairs (blocks 2p, 2p+1) in order, pair_bytes each, so
// a tile (or a run of its pairs) is one contiguous range for a bulk copy.
// Lane L = 4g + t (g < 8, t < 4) of a warp owns, per pair:
//   Q4_0 (576 B): 16 B at 16 L = word t (nibble bytes 4t..4t+3) of
//     (row g, block 2p), (row g+8, 2p), (row g, 2p+1), (row g+8, 2p+1);
//     a word's low nibbles are elements 4t..4t+3 and its high nibbles
//     elements 16+4t..16+4t+3 (src/core/tensor.cpp:57-63), which are exactly
//     the k-slots of the MMA's A fragment registers (rows g and g+8,
//     k = 4t..4t+3 and 16+4t..16+4t+3): two masks and a shift per word.
//   Q8_0 (1088 B): 16 B at 16 L for block 2p (codes 4t..4t+3 of row g, of
//     row g+8, codes 16+4t..16+4t+3 of row g, of row g+8), the same for
//     block 2p+1 at 512 + 16 L: the A fragments as stored.
//   then 64 B of f16 scales: lane L's at 2 L, for row g + 8 (t & 1) and
//     block 2p + (t >> 1) -- the (row, block) that lane finishes.
//
// x, staged per CTA in shared memory: per pair 32 lanes x 8 B, lane (g, t)'s
// B fragment (column g): digit g of block 2p (g < 3) or digit g - 4 of block
// 2p+1 (4 <= g < 7), elements 4t..4t+3 and 16+4t..16+4t+3, zero for g = 3, 7;
// then per block {int offset, float scale}.
//
// A pair is two MMAs into one accumulator: block 2p's three digit sums land
// in columns 0-2, block 2p+1's in columns 4-6 (each MMA's B operand is zero in
// the other half).  Lane (g, t) then holds sums for rows g and g+8 of block
// 2p + (t >> 1); two shuffles between lanes t and t^1 give each lane the
// three sums S0, S1, S2 of ONE (row, block): row g + 8 (t & 1).  Its exact
// integer dot is S0 + 2^8 S1 + 2^16 S2 (Q4_0: plus the block's offset
// -8 sum X for the codes' -8), converted once and multiplied by weight scale
// times x scale.  Per pair and lane: one 16-byte weight load, one scale, one
// 8-byte x load and one constant load, 2 MMAs, 2 shuffles and about 20
// integer/float instructions -- against ~90 for the IDP4A path.
#pragma once

#include "gemv.cuh"

namespace smallm {

constexpr int kMgemvWarps = 16;               // consumer warps (one producer warp more)
constexpr uint32_t kXfragPairBytes = 256;     // x fragments of one block pair
constexpr uint32_t kXconstBytes = 8;          // {offset, scale} of one block
constexpr uint32_t kMgemvPartFloats = kMgemvWarps * 16;  // per stage: every warp's 16 row partials

__device__ __forceinline__ void mma_u8s8(int (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_s8s8(int (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Q4_0: codes 0..15 as unsigned bytes; the -8 rides on x as the block offset.
// sum_i q_i X_i < 15 * 32 * 2^21 and |8 sum X| <= 2^29: the join is exact in int32.
struct MmaQ4_0 {
    static constexpr uint32_t kPairBytes = 576, kScaleOff = 512;
    static constexpr bool kOffset = true;
    __device__ __forceinline__ static void frags(const uint8_t* pw, int lane, uint32_t (&ab)[4], uint32_t (&an)[4]) {
        const uint4 w = *reinterpret_cast<const uint4*>(pw + lane * 16);
        constexpr uint32_t m = 0x0F0F0F0Fu;
        ab[0] = w.x & m;
        ab[1] = w.y & m;
        ab[2] = (w.x >> 4) & m;
        ab[3] = (w.y >> 4) & m;
        an[0] = w.z & m;
        an[1] = w.w & m;
        an[2] = (w.z >> 4) & m;
        an[3] = (w.w >> 4) & m;
    }
    __device__ __forceinline__ static void mma(int (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
        mma_u8s8(c, a, b0, b1);
    }
    __device__ __forceinline__ static float join(int s0, int s1, int s2, int off) {
        return __int2float_rn(s0 + 256 * s1 + 65536 * s2 + off);
    }
};

// Q8_0: signed codes; sum_i q_i X_i reaches 2^33, so the top digit joins in float.
struct MmaQ8_0 {
    static constexpr uint32_t kPairBytes = 1088, kScaleOff = 1024;
    static constexpr bool kOffset = false;
    __device__ __forceinline__ static void frags(const uint8_t* pw, int lane, uint32_t (&ab)[4], uint32_t (&an)[4]) {
        const uint4 a = *reinterpret_cast<const uint4*>(pw + lane * 16);
        const uint4 b = *reinterpret_cast<const uint4*>(pw + 512 + lane * 16);
        ab[0] = a.x;
        ab[1] = a.y;
        ab[2] = a.z;
        ab[3] = a.w;
        an[0] = b.x;
        an[1] = b.y;
        an[2] = b.z;
        an[3] = b.w;
    }
    __device__ __forceinline__ static void mma(int (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
        mma_s8s8(c, a, b0, b1);
    }
    __device__ __forceinline__ static float join(int s0, int s1, int s2, int) {
        return fmaf(__int2float_rn(s2), 65536.0f, __int2float_rn(s0 + 256 * s1));
    }
};

// The x fragments and constants of one 32-element block, built by the 8
// aligned lanes of a group (lane & 7 = j holds elements 4j..4j+3).  All 32
// lanes call it (shuffles); lanes with act == false write nothing.  Same
// fixed point as build_xrec_lane: X_i = rint(x_i 2^(21-e)), 2^e > max|x_i|,
// as balanced signed-byte digits X = D2 2^16 + D1 2^8 + D0.
template <bool kOffset>
__device__ __forceinline__ void build_xfrag_lane(float4 q, int lane, bool act, uint32_t blk, uint8_t* xfrag,
                                                 uint8_t* xconst) {
    constexpr int B = kXrecBits;
    const int j = lane & 7;
    float m = fmaxf(fmaxf(fabsf(q.x), fabsf(q.y)), fmaxf(fabsf(q.z), fabsf(q.w)));
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const bool finite = m <= 3.4028235e38f;  // false for inf and NaN
    if (!finite || m < 1e-30f) m = 0.f;      // tiny blocks contribute below f32 resolution
    const int e = (int)((__float_as_uint(m) >> 23) & 0xFFu) - 126;  // 2^e > m (m is 0 or normal)
    const float up = m > 0.f ? __uint_as_float((uint32_t)(B - e + 127) << 23) : 0.f;
    constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23: one FMA rounds x * 2^(B-e) to an integer
    constexpr uint32_t kMagicBits = 0x4B400000u;
    // X = rint(x * 2^(B-e)) (|X| <= 2^21) from the low mantissa bits; its
    // balanced signed-byte digits are the bytes of (X + 0x808080) ^ 0x808080
    // (adding 128 per byte makes every byte's carry explicit; the XOR maps
    // byte b to the int8 pattern of b - 128).  Four elements' digit words are
    // then gathered per digit with byte permutes.
    const uint32_t b0 = __float_as_uint(fmaf(q.x, up, kMagic)), b1 = __float_as_uint(fmaf(q.y, up, kMagic));
    const uint32_t b2 = __float_as_uint(fmaf(q.z, up, kMagic)), b3 = __float_as_uint(fmaf(q.w, up, kMagic));
    constexpr uint32_t kBias = 0x808080u;
    const uint32_t e0 = (b0 - kMagicBits + kBias) ^ kBias, e1 = (b1 - kMagicBits + kBias) ^ kBias;
    const uint32_t e2 = (b2 - kMagicBits + kBias) ^ kBias, e3 = (b3 - kMagicBits + kBias) ^ kBias;
    const uint32_t w01 = __byte_perm(e0, e1, 0x5140), w23 = __byte_perm(e2, e3, 0x5140);
    const uint32_t v01 = __byte_perm(e0, e1, 0x0062), v23 = __byte_perm(e2, e3, 0x0062);
    const uint32_t p[3] = {__byte_perm(w01, w23, 0x5410), __byte_perm(w01, w23, 0x7632),
                           __byte_perm(v01, v23, 0x5410)};
    int sx = (int)((b0 + b1) + (b2 + b3) - 4u * kMagicBits);
    if constexpr (kOffset) {
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) sx += __shfl_xor_sync(0xffffffffu, sx, o);
    }
    if (act) {
        // word j of each digit -> lane (digit + 4h) * 4 + (j & 3), register j >> 2
        const uint32_t h = blk & 1u, tl = (uint32_t)j & 3u, sl = (uint32_t)j >> 2;
        uint32_t* fr = reinterpret_cast<uint32_t*>(xfrag + (size_t)(blk >> 1) * kXfragPairBytes);
#pragma unroll
        for (int d = 0; d < 3; ++d) fr[(((uint32_t)d + 4u * h) * 4u + tl) * 2u + sl] = p[d];
        fr[((3u + 4u * h) * 4u + tl) * 2u + sl] = 0u;
        if (j == 0) {
            const float nan = __int_as_float(0x7FC00000);  // propagate like the reference's f32 math
            const float scale = __uint_as_float((uint32_t)(e - B + 127) << 23);
            int2 c;
            c.x = kOffset ? -8 * sx : 0;
            c.y = __float_as_int(!finite ? nan : (m > 0.f ? scale : 0.f));
            *reinterpret_cast<int2*>(xconst + (size_t)blk * kXconstBytes) = c;
        }
    }
}

// acc += this lane's (row, block) products over pairs [pa, pb) of a run of
// pairs at `pairs` whose first pair is global pair p0 (x is indexed
// globally).  Lane (g, t) accumulates row g + 8 (t & 1) of the 16-row tile.
template <class M>
__device__ __forceinline__ float mma_pairs(const uint8_t* pairs, uint32_t pa, uint32_t pb, uint32_t p0,
                                           const uint8_t* xfrag, const uint8_t* xconst, int lane, float acc) {
    const uint32_t t = (uint32_t)lane & 3u, g = (uint32_t)lane >> 2;
    const bool odd = (t & 1u) != 0u;
    const uint32_t mlo = g < 4 ? 0xFFFFFFFFu : 0u;
    const uint8_t* xf_lane = xfrag + (size_t)lane * 8;
    const uint8_t* xc_lane = xconst + (size_t)(t >> 1) * kXconstBytes;
#pragma unroll 2
    for (uint32_t i = pa; i < pb; ++i) {
        const uint8_t* pw = pairs + (size_t)i * M::kPairBytes;
        uint32_t ab[4], an[4];
        M::frags(pw, lane, ab, an);
        const uint32_t sc = *reinterpret_cast<const uint16_t*>(pw + M::kScaleOff + lane * 2);
        const uint2 xf = *reinterpret_cast<const uint2*>(xf_lane + (size_t)(p0 + i) * kXfragPairBytes);
        const int2 xc = *reinterpret_cast<const int2*>(xc_lane + (size_t)(p0 + i) * 2 * kXconstBytes);
        int c[4] = {0, 0, 0, 0};
        M::mma(c, ab, xf.x & mlo, xf.y & mlo);
        M::mma(c, an, xf.x & ~mlo, xf.y & ~mlo);
        // even t: S0, S1 of row g are c0, c1, S2 is the partner's c0;
        // odd t: S0, S1 of row g+8 are the partner's c2, c3, S2 is its own c2
        const int r1 = __shfl_xor_sync(0xffffffffu, odd ? c[0] : c[2], 1);
        const int r2 = __shfl_xor_sync(0xffffffffu, c[3], 1);
        const int s0 = odd ? r1 : c[0], s1 = odd ? r2 : c[1], s2 = odd ? c[2] : r1;
        acc = fmaf(M::join(s0, s1, s2, xc.x), h2f(sc) * __int_as_float(xc.y), acc);
    }
    return acc;
}

// ------------------------------------------------------------------ kernel --

// Tiles of rt = 16 nr rows (nr = 2 when a 16-row tile is small), each
// streamed as nchunk pieces of at most cpairs pairs (nchunk > 1 only with
// nr = 1) through an S-stage ring by one producer lane (bulk copies,
// mbarrier transaction counts).  Warp w takes row group w / (16 / nr) and a
// 1/(16 / nr) share of each piece's pairs; a lane keeps one row partial
// across the chunks of a tile.  Every warp counts itself done with a piece;
// the LAST one (no warp waits for another) sums the warps' row partials of a
// tile's last piece, releases the stage to the producer and runs the fused
// epilogue (gemv_epilogue_row).  (A fixed warp that waited for the others
// and then ran the epilogue fell one epilogue further behind per piece and
// held the stages: two copies in flight instead of four.)  Every wait is
// bounded: on timeout the kernel raises an error bit and skips the math.
template <class M, int PRO, int EPI>
__global__ void __launch_bounds__((kMgemvWarps + 1) * 32, 1) smallm_mgemv_kernel(const GemvParams p) {
    constexpr int W = kMgemvWarps;
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* xfrag = smem;
    uint8_t* xconst = smem + (size_t)p.upairs * kXfragPairBytes;
    uint8_t* stage0 = smem + p.xbytes;
    const uint32_t S = p.stages;
    uint64_t* full = reinterpret_cast<uint64_t*>(stage0 + (size_t)S * p.piece_bytes);
    uint64_t* empty = full + S;
    uint32_t* cnt = reinterpret_cast<uint32_t*>(empty + S);                         // [S] warps done
    uint64_t* xready = reinterpret_cast<uint64_t*>(cnt + 2 * ((S + 1) / 2));
    float* red = reinterpret_cast<float*>(xready + 1);                              // [W]
    unsigned long long* best_sh = reinterpret_cast<unsigned long long*>(red + W);  // [W]
    float* part = reinterpret_cast<float*>(best_sh + W);                            // [S][W][16]

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t ntiles = p.rows_pad / p.rt;
    const uint32_t NC = p.nchunk;
    const uint32_t my_tiles = blockIdx.x < ntiles ? (ntiles - blockIdx.x + gridDim.x - 1) / gridDim.x : 0u;
    const uint32_t npieces = my_tiles * NC;

    if (tid == 0) trace_mark(p.trace, 0);
    if (tid == 0) {
        for (uint32_t s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
            cnt[s] = 0u;
        }
        mbar_init(xready, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    // the next kernel of the step may launch now: it reads what this one
    // writes only after its own griddepcontrol.wait
    pdl_launch_dependents();

    if (warp == W) {
        // producer: weights do not depend on the previous kernel.  Pieces
        // from p.hold on wait until x is staged (a full ring's burst would
        // queue the x loads behind it).
        if (lane == 0) {
            const size_t tile_bytes = (size_t)p.rt * p.row_stride;
            const uint32_t nr = p.rt / 16;
            for (uint32_t j = 0; j < npieces; ++j) {
                const uint32_t s = j % S;
                if (j == p.hold && !mbar_wait(xready, 0)) {
                    atomicOr(p.err, 1u);
                    break;
                }
                if (j >= S && !mbar_wait(&empty[s], ((j / S) - 1) & 1)) {
                    atomicOr(p.err, 1u);  // consumers then time out once and skip their work
                    break;
                }
                const uint32_t t = blockIdx.x + (j / NC) * gridDim.x, c = j % NC;
                const uint32_t pc = min(p.cpairs, p.upairs - c * p.cpairs);
                const uint32_t bytes = nr * pc * p.pair_bytes;
                mbar_arrive_expect_tx(&full[s], bytes);
                bulk_g2s(stage0 + (size_t)s * p.piece_bytes, p.w + t * tile_bytes + (size_t)c * p.cpairs * p.pair_bytes,
                         bytes, &full[s]);
            }
        }
        return;
    }

    const float inv = gemv_stage_x<W, PRO>(p, warp, lane, p.upairs * 16u, red,
                                           [&](float4 q, int ln, bool act, uint32_t g) {
                                               build_xfrag_lane<M::kOffset>(q, ln, act, g >> 3, xfrag, xconst);
                                           });
    if (tid == 0) mbar_arrive(xready);  // the producer may fill the rest of the ring

    unsigned long long best = 0ull;
    bool dead = false;  // a bounded wait gave up: skip the math, keep the counting protocol
    const uint32_t WK = (uint32_t)W / (p.rt / 16);
    const uint32_t rg = (uint32_t)warp / WK, kp = (uint32_t)warp % WK;
    float acc = 0.f;
    for (uint32_t j = 0; j < npieces; ++j) {
        const uint32_t s = j % S, c = j % NC;
        if (!dead && !mbar_wait(&full[s], (j / S) & 1u)) {
            dead = true;
            if (lane == 0) atomicOr(p.err, 2u);
        }
        const uint32_t pc = min(p.cpairs, p.upairs - c * p.cpairs);
        const uint8_t* run = stage0 + (size_t)s * p.piece_bytes + (size_t)rg * pc * p.pair_bytes;
        if (!dead) acc = mma_pairs<M>(run, kp * pc / WK, (kp + 1) * pc / WK, c * p.cpairs, xfrag, xconst, lane, acc);
        const bool lastc = c == NC - 1;
        float* ps = part + (size_t)s * kMgemvPartFloats;
        if (lastc) {
            // lanes t and t^2 hold the two blocks of each pair of the same row
            const float v = acc + __shfl_xor_sync(0xffffffffu, acc, 2);
            acc = 0.f;
            if ((lane & 3) < 2) ps[warp * 16 + (lane >> 2) + 8 * (lane & 1)] = v;
        }
        __syncwarp();
        uint32_t last = 0u;
        if (lane == 0) {
            __threadfence_block();
            last = atomicAdd(&cnt[s], 1u) == (uint32_t)W - 1u ? 1u : 0u;
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (!last) continue;
        __threadfence_block();
        // the last warp: lane L sums row L of the tile (nr = 2: lanes 16-31 the second row group)
        const uint32_t rgl = (uint32_t)lane / 16, rl = (uint32_t)lane % 16;
        float r = 0.f;
        if (lastc && rgl < p.rt / 16)
            for (uint32_t k = 0; k < WK; ++k) r += ps[(rgl * WK + k) * 16 + rl];
        __syncwarp();
        if (lane == 0) {
            cnt[s] = 0u;
            mbar_arrive(&empty[s]);  // every reader of the stage and its partials is done
        }
        if (!lastc) continue;
        r *= inv;  // 1/rms of the fused RMSNorm (1 if plain)
        const float r_next = __shfl_down_sync(0xffffffffu, r, 1);  // partner row of a pair
        const uint32_t row = (blockIdx.x + (j / NC) * gridDim.x) * p.rt + (uint32_t)lane;
        if (rgl < p.rt / 16 && !dead) gemv_epilogue_row<EPI>(p, row, r, r_next, best);
    }

    if constexpr (EPI == EPI_LOGITS) {
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
            best = other > best ? other : best;
        }
        if (lane == 0) best_sh[warp] = best;
        consumers_sync<W>();
        if (tid == 0) {
            unsigned long long b = 0ull;
            for (int k = 0; k < W; ++k) b = best_sh[k] > b ? best_sh[k] : b;
            if (b) atomicMax(p.argmax, b);
        }
    }
    if constexpr (EPI == EPI_PEER) {
        // every row partial of this CTA is stored (at the peers too); the last
        // CTA to finish raises this rank's flag at every rank
        __threadfence_system();
        consumers_sync<W>();
        if (tid == 0 && atomicAdd(p.done_ctr, 1u) == gridDim.x - 1) {
            *p.done_ctr = 0u;
            __threadfence_system();
            const unsigned int e = __ldcg(p.epoch) + 1u;
            for (uint32_t r = 0; r < p.tp; ++r) st_release_sys(p.peer_flag[r], e);
        }
    }
    if (p.trace) {
        consumers_sync<W>();
        if (tid == 0) trace_mark(p.trace, 2);
    }
}

}  // namespace smallm
