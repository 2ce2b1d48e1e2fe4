// Batch-1 quantized GEMV for sm_100a: y = W . x, W in a repacked GGUF block
// layout streamed once from HBM, CUDA cores only.
//
// Memory side -- a TMA bulk-copy pipeline.  The device layout stores every
// row as one contiguous, 16-byte padded record (quants, then scales), so a
// tile of RT consecutive rows is ONE contiguous range.  One elected lane of a
// producer warp streams tiles into an S-stage shared-memory ring with
// cp.async.bulk (completion through mbarrier transaction counts).
//
// Compute side -- warp groups with private rings.  A tile is 4 rows.  The W
// consumer warps form NG groups of G warps; group g owns a ring of k stages
// and takes tiles g, g+NG, g+2NG, ..., its j-th tile landing in stage
// g*k + j%k, so every mbarrier wait is on the next phase of a stage only
// that group uses (parity waits are only unambiguous that way).  Producer
// lane g serves ring g, so a slow group never stalls another's loads.  The G
// warps of a group split the tile's K-units; each reduces its 4 partial row
// sums with one butterfly, and with G > 1 the partials meet in shared memory
// behind a per-stage "done" mbarrier, after which the group leader runs the
// epilogue and releases the stage.  No CTA-wide barrier sits inside the tile
// loop.  Every wait is bounded: on timeout the kernel raises an error flag
// and skips the remaining math.
//
// Math side -- integer dot products.  In the prologue each CTA turns x (f32;
// times the RMSNorm weight when the norm is fused, ops::rmsnorm,
// src/core/ops.cpp:29-40) into block fixed point: per 32-element block,
// X_i = rint(x_i * 2^(21-e)) with 2^e > max|x_i|, split into three balanced
// signed bytes ("digits"), so x is held to 2^-21 of the block maximum, the
// order of the f32 rounding of the reference's FMA chain.  A block's integer
// weight codes q meet x through IDP4A, one exact sum S_d = sum_i q_i D_d,i per
// digit; the digits are joined in float and the block needs one float scale
// (weight scale * 2^(e-21)).  4-bit codes are masked in place (the high
// nibble as 16 q, no shift), so a 32-weight block costs 8 masks and 24 IDP4A.
// The norm's 1/rms is a scalar and is applied to the row results in the
// epilogue.
//
// Epilogues (fused): plain store, residual add, Q/K/V bias + RoPE + KV-cache
// append, SwiGLU, logits + greedy argmax.
#pragma once

#include "common.cuh"

namespace smallm {

enum { PRO_PLAIN = 0, PRO_RMS = 1, PRO_RMS_SUM = 2, PRO_MERGE = 3 };
enum { EPI_STORE = 0, EPI_RESIDUAL = 1, EPI_QKV = 2, EPI_SWIGLU = 3, EPI_LOGITS = 4, EPI_PEER = 5 };
constexpr int kMaxTP = 8;

// Consumer warps per CTA (one producer warp more; a kernel template
// parameter): 16, or 22 for Q4_0 rows of >= 256 units (8192 columns), where
// the extra warps share the x staging of the long row (measured on the
// 4096x14336 down projection: 11.86 -> 10.86 us; on 4096-column rows they
// cost 0.26 us).  22 warps fit 72 registers per thread with room left on the
// SM for the decode attention's CTAs; the other formats' dots need more
// registers than 22 warps allow (Fmt::WIDE).
constexpr int kGemvMaxWarps = 22;
constexpr int kMaxRT = 32;                                   // storage rows pad to this

struct GemvParams {
    // repacked matrix: rows_pad records of row_stride bytes
    const uint8_t* w;
    uint32_t row_stride;
    uint32_t rows;      // logical rows; writes are masked to these
    uint32_t rows_pad;  // storage rows (multiple of kMaxRT)
    uint32_t cols;
    uint32_t units;     // cols / Fmt::UE
    uint32_t rt;        // rows per tile (4)
    uint32_t stages;    // pipeline depth = ngroups * kring
    uint32_t ngroups;   // warp groups; each owns a private ring of kring stages
    uint32_t gsize;     // warps per group; they split each tile's K-units
    uint32_t kring;     // stages per ring
    uint32_t xbytes;    // bytes of the staged x region
    uint32_t hold;      // the producer's j-th tile per ring waits for x to be staged (~0u: never)
    // input vector and fused RMSNorm
    const float* x;
    const float* norm_w;
    float eps;
    // outputs
    float* y;
    const float* bias;
    // QKV epilogue: storage rows [0, q_rows) are query rotary pairs, [q_rows,
    // q_rows + k_rows) key pairs, the rest value rows in natural order.
    uint32_t q_rows, k_rows;
    uint32_t head_dim, max_ctx;
    float* qout;
    float* kcache;      // [n_kv][max_ctx][head_dim]
    float* vcache;
    const float2* rope; // [max_ctx][head_dim/2] (cos, sin)
    const uint32_t* pos;
    unsigned long long* argmax;
    uint32_t row_offset;  // LOGITS: global vocabulary index of storage row 0
    unsigned int* err;    // set non-zero when a bounded wait gives up
    TraceSlot* trace;     // null outside traced steps
    // Tensor-parallel residual, all-reduced through peer memory instead of a
    // separate collective.  EPI_PEER (row-parallel O / down): each finished
    // row's partial goes straight into every rank's receive buffer, and the
    // kernel's last CTA raises this rank's arrival flag at every rank.
    // PRO_RMS_SUM (the next GEMV): waits for all ranks' flags, takes
    // x = x_res + sum over ranks of the partials (rank order: identical bits on
    // every rank), CTA 0 stores it to x_out, then the RMSNorm prologue runs.
    const float* x_res;             // PRO_RMS_SUM: residual before the add
    float* x_out;                   // PRO_RMS_SUM: residual after the add
    const float* rx;                // PRO_RMS_SUM: [tp][cols] received partials
    const unsigned int* rx_flag;    // PRO_RMS_SUM: [tp] arrival flags (epoch + 1 when ready)
    float* peer_out[kMaxTP];        // EPI_PEER: rank q's receive slot for this rank's partial
    unsigned int* peer_flag[kMaxTP];// EPI_PEER: this rank's arrival flag at rank q
    unsigned int* done_ctr;         // EPI_PEER: finished CTAs, zero between launches
    const unsigned int* epoch;      // steps completed so far (same on every rank)
    uint32_t tp;
    // PRO_MERGE: x is the merge of merge_parts attention partials
    // ([parts][cols], normalised per part) with per-head (max, sum) weights
    // merge_ml [parts][cols / merge_hd][2]
    uint32_t merge_parts, merge_hd;
    const float* merge_ml;
};

// Granule g (elements 4g..4g+3) of x merged from attention partials: part k
// of head h weighs exp(M_k - M) L_k over the head's parts (a part with no
// positions has L_k = 0), the same sum on every CTA.
__device__ __forceinline__ float4 merge_granule(const GemvParams& p, uint32_t g) {
    const uint32_t cols = p.cols, h = 4 * g / p.merge_hd, nh = cols / p.merge_hd;
    float M = -INFINITY;
    for (uint32_t k = 0; k < p.merge_parts; ++k)
        if (p.merge_ml[((size_t)k * nh + h) * 2 + 1] > 0.f) M = fmaxf(M, p.merge_ml[((size_t)k * nh + h) * 2]);
    float wsum = 0.f;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    for (uint32_t k = 0; k < p.merge_parts; ++k) {
        const float L = p.merge_ml[((size_t)k * nh + h) * 2 + 1];
        const float w = L > 0.f ? expf(p.merge_ml[((size_t)k * nh + h) * 2] - M) * L : 0.f;
        const float4 v = reinterpret_cast<const float4*>(p.x + (size_t)k * cols)[g];
        wsum += w;
        o.x = fmaf(w, v.x, o.x);
        o.y = fmaf(w, v.y, o.y);
        o.z = fmaf(w, v.z, o.z);
        o.w = fmaf(w, v.w, o.w);
    }
    const float r = 1.0f / wsum;
    return make_float4(o.x * r, o.y * r, o.z * r, o.w * r);
}

// ------------------------------------------------------- x in fixed point --

// Shared-memory record of one 32-element block of x: X_i = rint(x_i 2^(21-e))
// (2^e > the block's max |x|) as three balanced signed-byte digits,
// X = D2 2^16 + D1 2^8 + D0, plus four format-specific words (XK below).
struct XRec {
    uint32_t d[3][8];   // digits, 4 elements per word (d[0] least significant)
    int32_t s0, s1;     // XK_PLAIN / XK_NIB: sum of X over elements 0-15 / 16-31;
    uint32_t s2;        //   s2 = bits of the f32 sum of x.  XK_NIB_SD: s0, s1, s2 =
                        //   sum over the block of D0, D1, D2
    float xs;           // x_i ~= X_i xs; XK_NIB / XK_NIB_SD fold in 1/16 (see the dots)
};
constexpr int kXrecBytes = 112;
constexpr int kXrecBits = 21;
static_assert(sizeof(XRec) == kXrecBytes, "XRec layout");
enum { XK_PLAIN = 0, XK_NIB = 1, XK_NIB_SD = 2 };

// Exact int -> float for |v| < 2^22 (IADD + FADD, no conversion unit).
__device__ __forceinline__ float i2f_small(int v) {
    return __int_as_float(0x4B400000 + v) - 12582912.0f;
}

// Build the record of one 32-element block cooperatively: the 8 aligned lanes
// of a group each hold one float4 (elements 4j..4j+3, j = lane & 7).  All 32
// lanes must call it (shuffles); lanes with act == false hold zeros and write
// nothing.  x is held to 2^-21 of the block maximum, the order of the f32
// rounding of the reference's FMA chain.
template <int XK>
__device__ __forceinline__ void build_xrec_lane(float4 q, int lane, bool act, uint8_t* rec) {
    constexpr int B = kXrecBits;
    const int j = lane & 7;
    float m = fmaxf(fmaxf(fabsf(q.x), fabsf(q.y)), fmaxf(fabsf(q.z), fabsf(q.w)));
    float s = (q.x + q.y) + (q.z + q.w);
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        s += __shfl_xor_sync(0xffffffffu, s, o);
    }
    const bool finite = m <= 3.4028235e38f;  // false for inf and NaN
    if (!finite || m < 1e-30f) m = 0.f;      // tiny blocks contribute below f32 resolution
    // m = f * 2^e with f in [0.5, 1) (m is 0 or normal): e = biased exponent - 126,
    // so 2^e > m; 2^(B-e) and the record's scale are built from their exponent
    // bits (both stay in the normal range for 1e-30 <= m <= FLT_MAX)
    const int e = (int)((__float_as_uint(m) >> 23) & 0xFFu) - 126;
    const float up = m > 0.f ? __uint_as_float((uint32_t)(B - e + 127) << 23) : 0.f;
    // X = rint(x * 2^(B-e)): x * 2^(B-e) is exact and |X| <= 2^B < 2^22, so
    // one FMA with 1.5 * 2^23 rounds it (ties to even) into the low mantissa
    // bits: bits = 0x4B400000 + X
    constexpr float kMagic = 12582912.0f;
    constexpr uint32_t kMagicBits = 0x4B400000u;
    const float v[4] = {q.x, q.y, q.z, q.w};
    uint32_t bits[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) bits[k] = __float_as_uint(fmaf(v[k], up, kMagic));
    // Balanced digits X = D2 2^16 + D1 2^8 + D0 (|X| <= 2^21): they are the
    // bytes of (X + 0x808080) ^ 0x808080 -- adding 128 per byte makes every
    // byte's carry explicit and the XOR maps byte b to the int8 pattern of
    // b - 128 -- gathered per digit across the 4 elements with byte permutes.
    constexpr uint32_t kBias = 0x808080u;
    uint32_t el[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) el[k] = (bits[k] - kMagicBits + kBias) ^ kBias;
    const uint32_t w01 = __byte_perm(el[0], el[1], 0x5140), w23 = __byte_perm(el[2], el[3], 0x5140);
    const uint32_t v01 = __byte_perm(el[0], el[1], 0x0062), v23 = __byte_perm(el[2], el[3], 0x0062);
    const uint32_t p[3] = {__byte_perm(w01, w23, 0x5410), __byte_perm(w01, w23, 0x7632),
                           __byte_perm(v01, v23, 0x5410)};
    int ds[3] = {0, 0, 0};  // this lane's digit sums (XK_NIB_SD)
    if constexpr (XK == XK_NIB_SD) {
#pragma unroll
        for (int d = 0; d < 3; ++d) ds[d] = __dp4a((int)p[d], 0x01010101, 0);
    }
    int t0, t1;
    uint32_t t2;
    if constexpr (XK == XK_NIB_SD) {
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
            ds[0] += __shfl_xor_sync(0xffffffffu, ds[0], o);
            ds[1] += __shfl_xor_sync(0xffffffffu, ds[1], o);
            ds[2] += __shfl_xor_sync(0xffffffffu, ds[2], o);
        }
        t0 = ds[0];
        t1 = ds[1];
        t2 = (uint32_t)ds[2];
    } else {
        int sx = (int)((bits[0] + bits[1]) + (bits[2] + bits[3]) - 4u * kMagicBits);
        sx += __shfl_xor_sync(0xffffffffu, sx, 1);
        sx += __shfl_xor_sync(0xffffffffu, sx, 2);  // lanes 0-3: elements 0-15, lanes 4-7: 16-31
        const int sx_other = __shfl_xor_sync(0xffffffffu, sx, 4);
        t0 = sx;
        t1 = sx_other;
        t2 = __float_as_uint(s);
    }
    if (act) {
        uint32_t* w = reinterpret_cast<uint32_t*>(rec);
#pragma unroll
        for (int d = 0; d < 3; ++d) w[8 * d + j] = p[d];
        if (j == 0) {
            const float nan = __int_as_float(0x7FC00000);  // propagate like the reference's f32 math
            // 4-bit codes produce 16 sum q X (high nibbles stay in place)
            const int scale_e = e - B - (XK == XK_PLAIN ? 0 : 4);
            const float scale = __uint_as_float((uint32_t)(scale_e + 127) << 23);
            w[24] = (uint32_t)t0;
            w[25] = (uint32_t)t1;
            w[26] = !finite && XK != XK_NIB_SD ? __float_as_uint(nan) : t2;
            reinterpret_cast<float*>(w)[27] = !finite ? nan : (m > 0.f ? scale : 0.f);
        }
    }
}

__device__ __forceinline__ void load_xrec(const uint8_t* base, uint32_t blk, XRec& r) {
    const uint4* p = reinterpret_cast<const uint4*>(base + (size_t)blk * kXrecBytes);
#pragma unroll
    for (int i = 0; i < kXrecBytes / 16; ++i) reinterpret_cast<uint4*>(&r)[i] = p[i];
}

// IDP4A with an unsigned first operand: unsigned x unsigned / unsigned x signed bytes.
__device__ __forceinline__ int dp4a_uu(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Three-digit records: sum_i q_i x_i of one block = xs * (2^16 S2 + 2^8 S1 +
// S0), joined in float by combine() (each S exact and below 2^22).
__device__ __forceinline__ float combine(int s0, int s1, int s2) {
    return fmaf(i2f_small(s2), 65536.0f, fmaf(i2f_small(s1), 256.0f, i2f_small(s0)));
}

// ---------------------------------------------------------------- formats --
// Device row records (kernels.cu: qmat_alloc / repack):
//  Q4_0  [units][16 B nibbles] [units][f16 d]          unit = one 32-block
//  Q8_0  [units][32 B int8]    [units][f16 d]          unit = one 32-block
//  Q4_K  [nsb][144 B GGUF super-block]                 unit = quarter super-block (64)
//  Q6_K  [units][48 B codes]   [units][4 x i8 scale] [nsb][f16 d]   unit = 64
//  F32   [cols][f32]                                   unit = 32 values

// Q4_0: element i of a block is the low nibble of byte i, element i+16 the
// high nibble (src/core/tensor.cpp:57-63); value (q - 8) * d.  Low nibbles
// are masked to q, high nibbles masked in place to 16 q (no shift); per digit
// 16 sum (q - 8) D = 16 L + H - 128 sum D is exact in int32 and below 2^21,
// and the three digits are joined in float (the record's scale carries 1/16).
struct FmtQ4_0 {
    static constexpr int UE = 32, SUBS = 1, WIDE = 22, XK = XK_NIB_SD;
    static constexpr int STEP_RPT = 4;  // rows per thread and piece in the persistent step
    static constexpr bool F32X = false;
    struct Raw { uint4 q; uint32_t s; };
    __device__ __forceinline__ static void load(const uint8_t* row, uint32_t u, uint32_t units, Raw& r) {
        r.q = *reinterpret_cast<const uint4*>(row + (size_t)u * 16);
        r.s = *reinterpret_cast<const uint16_t*>(row + (size_t)units * 16 + (size_t)u * 2);
    }
    __device__ __forceinline__ static float dot(const Raw& r, int, const XRec& x, uint32_t) {
        const uint32_t w[4] = {r.q.x, r.q.y, r.q.z, r.q.w};
        int l0 = 0, l1 = 0, l2 = 0, h0 = 0, h1 = 0, h2 = 0;  // low nibbles (q) / high nibbles in place (16 q)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t lo = w[j] & 0x0F0F0F0Fu, hi = w[j] & 0xF0F0F0F0u;
            l0 = dp4a_us(lo, x.d[0][j], l0);
            l1 = dp4a_us(lo, x.d[1][j], l1);
            l2 = dp4a_us(lo, x.d[2][j], l2);
            h0 = dp4a_us(hi, x.d[0][4 + j], h0);
            h1 = dp4a_us(hi, x.d[1][4 + j], h1);
            h2 = dp4a_us(hi, x.d[2][4 + j], h2);
        }
        const int v0 = 16 * l0 + h0 - 128 * x.s0;
        const int v1 = 16 * l1 + h1 - 128 * x.s1;
        const int v2 = 16 * l2 + h2 - 128 * (int)x.s2;
        return combine(v0, v1, v2) * (h2f(r.s) * x.xs);
    }
};

// Q8_0: int8 codes; value q * d.
struct FmtQ8_0 {
    static constexpr int UE = 32, SUBS = 1, WIDE = 16, XK = XK_PLAIN;
    static constexpr int STEP_RPT = 2;  // rows per thread and piece in the persistent step (registers)
    static constexpr bool F32X = false;
    struct Raw { uint4 a, b; uint32_t s; };
    __device__ __forceinline__ static void load(const uint8_t* row, uint32_t u, uint32_t units, Raw& r) {
        const uint4* q = reinterpret_cast<const uint4*>(row + (size_t)u * 32);
        // lanes with bit 2 of u set read the upper half first, so the 8 lanes
        // of each quarter-warp touch distinct banks in both loads
        const uint32_t f = (u >> 2) & 1u;
        const uint4 first = q[f], second = q[f ^ 1u];
        r.a = f ? second : first;
        r.b = f ? first : second;
        r.s = *reinterpret_cast<const uint16_t*>(row + (size_t)units * 32 + (size_t)u * 2);
    }
    __device__ __forceinline__ static float dot(const Raw& r, int, const XRec& x, uint32_t) {
        const uint32_t w[8] = {r.a.x, r.a.y, r.a.z, r.a.w, r.b.x, r.b.y, r.b.z, r.b.w};
        int s0 = 0, s1 = 0, s2 = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            s0 = __dp4a((int)w[j], (int)x.d[0][j], s0);
            s1 = __dp4a((int)w[j], (int)x.d[1][j], s1);
            s2 = __dp4a((int)w[j], (int)x.d[2][j], s2);
        }
        return combine(s0, s1, s2) * (h2f(r.s) * x.xs);
    }
};

// Q4_K: GGUF super-blocks {f16 d, f16 dmin, 12 B packed 6-bit scales/mins,
// 128 B nibbles}; a unit is a quarter super-block: sub-block 2k = low
// nibbles of qs[32k..32k+32), sub-block 2k+1 = high nibbles.
// Value: (d*sc)*q - dmin*m (gguf-py Q4_K.dequantize_blocks).
struct FmtQ4K {
    static constexpr int UE = 64, SUBS = 2, WIDE = 16, XK = XK_NIB;
    static constexpr bool F32X = false;
    struct Raw { uint4 h, a, b; };
    __device__ __forceinline__ static void load(const uint8_t* row, uint32_t u, uint32_t, Raw& r) {
        const uint8_t* sb = row + (size_t)(u >> 2) * 144;
        r.h = *reinterpret_cast<const uint4*>(sb);
        r.a = *reinterpret_cast<const uint4*>(sb + 16 + (u & 3) * 32);
        r.b = *reinterpret_cast<const uint4*>(sb + 32 + (u & 3) * 32);
    }
    __device__ __forceinline__ static void scale_min(const uint4& h, int j, int& sc, int& m) {
        const uint32_t s0 = h.y, s1 = h.z, s2 = h.w;  // scale bytes 0-3, 4-7, 8-11
        auto byte = [](uint32_t w, int k) { return (int)((w >> (8 * k)) & 0xFFu); };
        if (j < 4) {
            sc = byte(s0, j) & 63;
            m = byte(s1, j) & 63;
        } else {
            sc = (byte(s2, j - 4) & 0xF) | ((byte(s0, j - 4) >> 6) << 4);
            m = (byte(s2, j - 4) >> 4) | ((byte(s1, j - 4) >> 6) << 4);
        }
    }
    __device__ __forceinline__ static float dot(const Raw& r, int sub, const XRec& x, uint32_t u) {
        const uint32_t w[8] = {r.a.x, r.a.y, r.a.z, r.a.w, r.b.x, r.b.y, r.b.z, r.b.w};
        // sub-block 1's high nibbles stay in place: its sums are 16 sum q X
        const uint32_t mask = sub ? 0xF0F0F0F0u : 0x0F0F0F0Fu;
        int s0 = 0, s1 = 0, s2 = 0;  // each below 32 * 240 * 128 < 2^22
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t n = w[j] & mask;
            s0 = dp4a_us(n, x.d[0][j], s0);
            s1 = dp4a_us(n, x.d[1][j], s1);
            s2 = dp4a_us(n, x.d[2][j], s2);
        }
        int sc, m;
        scale_min(r.h, 2 * (int)(u & 3) + sub, sc, m);
        const float d = h2f(r.h.x & 0xFFFFu), dmin = h2f(r.h.x >> 16);
        const float d1 = d * (float)sc, m1 = dmin * (float)m;
        const float xs = sub ? x.xs : x.xs * 16.0f;  // x.xs carries 1/16 for in-place high nibbles
        return fmaf(d1 * xs, combine(s0, s1, s2), -m1 * __uint_as_float(x.s2));
    }
};

// Q6_K re-encoded per 64-element unit by the repack kernel: 32 bytes of
// nibbles (byte k: element k low, element 32+k high) and 16 bytes of 2-bit
// high parts (byte k: elements k, 16+k, 32+k, 48+k in bits 0-1, 2-3, 4-5,
// 6-7); 4 int8 scales per unit (element e of a super-block uses scale e/16);
// f16 d per super-block.  Value: (d*sc)*(q - 32) (src/core/tensor.cpp:97-106).
struct FmtQ6K {
    static constexpr int UE = 64, SUBS = 2, WIDE = 16, XK = XK_PLAIN;
    static constexpr bool F32X = false;
    struct Raw { uint4 n0, n1, hb; uint32_t sc; uint32_t d; };
    __device__ __forceinline__ static void load(const uint8_t* row, uint32_t u, uint32_t units, Raw& r) {
        const uint8_t* qb = row + (size_t)u * 48;
        r.n0 = *reinterpret_cast<const uint4*>(qb);
        r.n1 = *reinterpret_cast<const uint4*>(qb + 16);
        r.hb = *reinterpret_cast<const uint4*>(qb + 32);
        r.sc = *reinterpret_cast<const uint32_t*>(row + (size_t)units * 48 + (size_t)u * 4);
        r.d = *reinterpret_cast<const uint16_t*>(row + (size_t)units * 52 + (size_t)(u >> 2) * 2);
    }
    __device__ __forceinline__ static float dot(const Raw& r, int sub, const XRec& x, uint32_t) {
        const uint32_t n[8] = {r.n0.x, r.n0.y, r.n0.z, r.n0.w, r.n1.x, r.n1.y, r.n1.z, r.n1.w};
        const uint32_t h[4] = {r.hb.x, r.hb.y, r.hb.z, r.hb.w};
        int a0 = 0, a1 = 0, a2 = 0, b0 = 0, b1 = 0, b2 = 0;  // first / second 16 elements
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            uint32_t q;
            if (sub == 0)
                q = (n[j] & 0x0F0F0F0Fu) | ((j < 4 ? (h[j] << 4) : (h[j - 4] << 2)) & 0x30303030u);
            else
                q = ((n[j] >> 4) & 0x0F0F0F0Fu) | ((j < 4 ? h[j] : (h[j - 4] >> 2)) & 0x30303030u);
            if (j < 4) {
                a0 = __dp4a((int)q, (int)x.d[0][j], a0);
                a1 = __dp4a((int)q, (int)x.d[1][j], a1);
                a2 = __dp4a((int)q, (int)x.d[2][j], a2);
            } else {
                b0 = __dp4a((int)q, (int)x.d[0][j], b0);
                b1 = __dp4a((int)q, (int)x.d[1][j], b1);
                b2 = __dp4a((int)q, (int)x.d[2][j], b2);
            }
        }
        // codes are q + 32: subtract 32 * sum X per 16-element group
        const float va = fmaf(-32.0f, (float)x.s0, combine(a0, a1, a2));
        const float vb = fmaf(-32.0f, (float)x.s1, combine(b0, b1, b2));
        const float sa = (float)(int8_t)((r.sc >> (16 * sub)) & 0xFFu);
        const float sbv = (float)(int8_t)((r.sc >> (16 * sub + 8)) & 0xFFu);
        return (h2f(r.d) * x.xs) * fmaf(sbv, vb, sa * va);
    }
};

// F32 (the reference's catch-all branch, ops.cpp:289-299): plain f32 FMAs
// against an f32 copy of x.
struct FmtF32 {
    static constexpr int UE = 32, SUBS = 1, WIDE = 16, XK = XK_PLAIN;
    static constexpr bool F32X = true;
};

// Named barrier over the consumer warps only (the producer never joins).
template <int W>
__device__ __forceinline__ void consumers_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(W * 32) : "memory");
}

// Fused epilogue of one finished row (v = the row's W.x after 1/rms).  The
// pair epilogues (RoPE, SwiGLU) run on the even row of a pair and read the
// odd row's value from v_next; `best` collects the LOGITS argmax key.
template <int EPI, class P>  // P: GemvParams, or any struct with the same output fields
__device__ __forceinline__ void gemv_epilogue_row(const P& p, uint32_t row, float v, float v_next,
                                                  unsigned long long& best) {
    if constexpr (EPI == EPI_STORE) {
        if (row < p.rows) p.y[row] = v;
    } else if constexpr (EPI == EPI_PEER) {
        if (row < p.rows)
            for (uint32_t r = 0; r < p.tp; ++r) p.peer_out[r][row] = v;  // NVLink stores to peers
    } else if constexpr (EPI == EPI_RESIDUAL) {
        // x += W.h (ops::axpy, qwen2_model.cpp:178,184); the residual is read
        // from L2, where other CTAs of a persistent step may have updated it
        if (row < p.rows) p.y[row] = __ldcg(p.y + row) + v;
    } else if constexpr (EPI == EPI_LOGITS) {
        if (row < p.rows) {
            p.y[row] = v;
            if (v == v) {  // a NaN never wins (greedy_sampler.cpp:11 compares with >)
                const unsigned long long k = argmax_key(v, p.row_offset + row);
                best = k > best ? k : best;
            }
        }
    } else if constexpr (EPI == EPI_SWIGLU) {
        // storage rows 2j / 2j+1 hold gate_j / up_j (ops::silu then ops::mul,
        // qwen2_model.cpp:154-155)
        if ((row & 1) == 0 && row + 1 < p.rows) {
            const float g = v / (1.0f + expf(-v));
            p.y[row >> 1] = g * v_next;
        }
    } else if constexpr (EPI == EPI_QKV) {
        const uint32_t hd = p.head_dim, half = hd >> 1;
        const uint32_t pos = *p.pos;
        if (row < p.q_rows + p.k_rows) {
            if ((row & 1) == 0 && row + 1 < p.rows) {
                const bool isq = row < p.q_rows;
                const uint32_t pr = (isq ? row : row - p.q_rows) >> 1;  // rotary pair index
                const uint32_t head = pr / half, ii = pr % half;
                const uint32_t la = head * hd + ii, lb = la + half;
                float x0 = v, x1 = v_next;
                if (p.bias) {
                    const uint32_t bo = isq ? 0u : p.q_rows;
                    x0 += p.bias[bo + la];
                    x1 += p.bias[bo + lb];
                }
                // ops::rope (ops.cpp:84-89) with the reference build's fused rounding
                const float2 cs = p.rope[(size_t)pos * half + ii];
                const float o0 = fmaf(x0, cs.x, -__fmul_rn(x1, cs.y));
                const float o1 = fmaf(x0, cs.y, __fmul_rn(x1, cs.x));
                if (isq) {
                    p.qout[la] = o0;
                    p.qout[lb] = o1;
                } else {
                    float* kr = p.kcache + ((size_t)head * p.max_ctx + pos) * hd;
                    kr[ii] = o0;
                    kr[ii + half] = o1;
                }
            }
        } else if (row < p.rows) {
            const uint32_t lv = row - p.q_rows - p.k_rows;
            float vv = v;
            if (p.bias) vv += p.bias[p.q_rows + p.k_rows + lv];
            const uint32_t head = lv / hd, dd = lv % hd;
            p.vcache[((size_t)head * p.max_ctx + pos) * hd + dd] = vv;
        }
    }
}

// ------------------------------------------------------------------ kernel --

template <class Fmt, int PRO, int EPI, int W>  // W consumer warps; warp W is the producer
__global__ void __launch_bounds__((W + 1) * 32, 1) smallm_qgemv_kernel(const GemvParams p) {
    static_assert(W <= kGemvMaxWarps && W <= Fmt::WIDE, "consumer warps");
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* xreg = smem;                                   // x records (or f32 x)
    uint8_t* stage0 = smem + p.xbytes;                      // S stages
    const uint32_t sbytes = p.rt * p.row_stride;            // bytes per stage
    uint64_t* full = reinterpret_cast<uint64_t*>(stage0 + (size_t)p.stages * sbytes);
    uint64_t* empty = full + p.stages;
    uint64_t* done = empty + p.stages;
    uint64_t* xready = done + p.stages;                                 // x records staged
    float* red = reinterpret_cast<float*>(xready + 1);                  // [kGemvMaxWarps]
    unsigned long long* best_sh = reinterpret_cast<unsigned long long*>(red + kGemvMaxWarps);
    float* part = reinterpret_cast<float*>(best_sh + kGemvMaxWarps);   // [stages][gsize][4]

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t ntiles = p.rows_pad / p.rt;
    const uint32_t NG = p.ngroups, G = p.gsize, K = p.kring;

    if (tid == 0) trace_mark(p.trace, 0);
    if (tid == 0) {
        for (uint32_t s = 0; s < p.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
            mbar_init(&done[s], G);
        }
        mbar_init(xready, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    // let the next kernel of the step launch now: it only reads what this one
    // writes after its own griddepcontrol.wait, and its producer warp can
    // start streaming weights while this kernel drains
    pdl_launch_dependents();

    if (warp == W) {
        // ---------------- producer: weights do not depend on the previous kernel
        // lane g feeds ring g: the group's j-th tile (CTA tile g + j*NG) goes
        // to stage g*K + j%K once the group has released that stage.  When
        // the ring cannot hold all of the CTA's tiles anyway, only the first
        // tile per ring is fetched before the consumers have staged x (tile
        // p.hold onwards waits): a full ring's burst would queue the x loads
        // behind it.
        if ((uint32_t)lane < NG) {
            const uint32_t g = lane;
            uint32_t j = 0;
            for (uint32_t t = blockIdx.x + g * gridDim.x; t < ntiles; t += NG * gridDim.x, ++j) {
                const uint32_t s = g * K + j % K;
                if (j == p.hold && !mbar_wait(xready, 0)) {
                    atomicOr(p.err, 1u);
                    break;
                }
                if (j >= K && !mbar_wait(&empty[s], ((j / K) - 1) & 1)) {
                    atomicOr(p.err, 1u);  // consumers then time out once and skip their work
                    break;
                }
                mbar_arrive_expect_tx(&full[s], sbytes);
                bulk_g2s(stage0 + (size_t)s * sbytes, p.w + (size_t)t * sbytes, sbytes, &full[s]);
            }
        }
        return;
    }

    // ---------------- consumers: stage x (after the producer of x finished)
    const int ctid = tid;  // 0 .. 32 * W - 1
    // RMSNorm is linear in x given its scalar: the records hold x * w and the
    // epilogue multiplies each row result by 1/rms, so x is read only once.
    // 8 consecutive lanes own the 8 float4 granules of one 32-element block;
    // loads are issued in batches of kB granules per thread before any of them
    // is used (one batch covers 8192 columns with the norm, 16384 without),
    // and the norm weights (constant) are fetched before the wait.
    constexpr int kB = PRO == PRO_PLAIN ? 8 : 4;
    constexpr uint32_t kStride = W * 32;
    const float4* x4 = reinterpret_cast<const float4*>(p.x);
    const float4* w4 = reinterpret_cast<const float4*>(p.norm_w);
    const uint32_t ngr = p.cols / 4;  // a multiple of 8: whole blocks are in or out
    constexpr bool kRms = PRO == PRO_RMS || PRO == PRO_RMS_SUM;
    float4 wpre[kB];
    if constexpr (kRms) {
#pragma unroll
        for (int k = 0; k < kB; ++k) {
            const uint32_t g = ctid + k * kStride;
            wpre[k] = g < ngr ? w4[g] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    pdl_wait();
    if (ctid == 0) trace_mark(p.trace, 1);
    if constexpr (PRO == PRO_RMS_SUM) {
        // every rank's partial of the previous row-parallel GEMV must have
        // arrived (bounded wait; on timeout the error flag is raised and the
        // step's result is not valid)
        if (ctid == 0) {
            const unsigned int want = __ldcg(p.epoch) + 1u;
            const long long t0 = clock64();
            for (uint32_t r = 0; r < p.tp; ++r) {
                while (ld_acquire_sys(p.rx_flag + r) != want) {
                    if (clock64() - t0 > (1ll << 31)) {
                        atomicOr(p.err, 8u);
                        break;
                    }
                    __nanosleep(32);
                }
            }
        }
        consumers_sync<W>();
    }
    const float4* xr4 = reinterpret_cast<const float4*>(p.rx);
    float ss = 0.f;
    for (uint32_t g0 = 0; g0 < ngr; g0 += kB * kStride) {
        float4 xq[kB];
#pragma unroll
        for (int k = 0; k < kB; ++k) {
            const uint32_t g = g0 + ctid + k * kStride;
            if constexpr (PRO == PRO_RMS_SUM) {
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (g < ngr) {
                    v = reinterpret_cast<const float4*>(p.x_res)[g];
                    for (uint32_t r = 0; r < p.tp; ++r) {  // rank order: the same sum on every rank
                        const float4 d = __ldcg(xr4 + (size_t)r * ngr + g);
                        v.x += d.x;
                        v.y += d.y;
                        v.z += d.z;
                        v.w += d.w;
                    }
                    if (blockIdx.x == 0) reinterpret_cast<float4*>(p.x_out)[g] = v;
                }
                xq[k] = v;
            } else if constexpr (PRO == PRO_MERGE) {
                xq[k] = g < ngr ? merge_granule(p, g) : make_float4(0.f, 0.f, 0.f, 0.f);
            } else {
                xq[k] = g < ngr ? x4[g] : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
#pragma unroll
        for (int k = 0; k < kB; ++k) {
            const uint32_t g = g0 + ctid + k * kStride;
            // a warp whose first granule lies past the end has no block here
            // (warp-uniform, so the shuffles inside stay whole-warp)
            if (g0 + (uint32_t)warp * 32 + k * kStride >= ngr) continue;
            const bool act = g < ngr;
            float4 q = xq[k];
            if constexpr (kRms) {
                ss += q.x * q.x + q.y * q.y + q.z * q.z + q.w * q.w;
                const float4 w = g0 == 0 ? wpre[k] : (act ? w4[g] : make_float4(0.f, 0.f, 0.f, 0.f));
                q.x *= w.x;
                q.y *= w.y;
                q.z *= w.z;
                q.w *= w.w;
            }
            if constexpr (Fmt::F32X) {
                if (act) reinterpret_cast<float4*>(xreg)[g] = q;
            } else {
                // uniform across the warp: all lanes reach the shuffles inside
                build_xrec_lane<Fmt::XK>(q, lane, act, xreg + (size_t)(g >> 3) * kXrecBytes);
            }
        }
    }
    float inv = 1.0f;
    if constexpr (kRms) {
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
    }
    consumers_sync<W>();
    if (ctid == 0) mbar_arrive(xready);  // the producer may fill the rest of the rings
    if constexpr (kRms) {
        float t = 0.f;
#pragma unroll
        for (int k = 0; k < W; ++k) t += red[k];
        inv = 1.0f / sqrtf(t / (float)p.cols + p.eps);
    }

    unsigned long long best = 0ull;
    // A warp whose bounded wait gave up marks itself dead: it skips the math
    // but still releases its stages.
    bool dead = false;
    const uint32_t grp = (uint32_t)warp / G, gpart = (uint32_t)warp % G;
    const bool working = grp < NG;  // warps beyond NG * G idle
    const uint32_t ua = (uint32_t)(((uint64_t)p.units * gpart) / G);       // this warp's K-units
    const uint32_t ub = (uint32_t)(((uint64_t)p.units * (gpart + 1)) / G);
    const uint32_t first = working ? blockIdx.x + grp * gridDim.x : ntiles;
    uint32_t j = 0;
    for (uint32_t t = first; t < ntiles; t += NG * gridDim.x, ++j) {
        const uint32_t s = grp * K + j % K;
        const uint32_t ph = (j / K) & 1;
        if (!dead && !mbar_wait(&full[s], ph)) {
            dead = true;
            if (lane == 0) atomicOr(p.err, 2u);
        }
        const uint8_t* rows4 = stage0 + (size_t)s * sbytes;
        constexpr uint32_t sub4 = 0;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        if (!dead) {
            if constexpr (Fmt::F32X) {
                for (uint32_t u = ua + lane; u < ub; u += 32) {
                    float xv[32];
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const float4 q = reinterpret_cast<const float4*>(xreg)[u * 8 + j];
                        xv[4 * j] = q.x;
                        xv[4 * j + 1] = q.y;
                        xv[4 * j + 2] = q.z;
                        xv[4 * j + 3] = q.w;
                    }
#pragma unroll
                    for (int r = 0; r < 4; ++r) {
                        const float4* wr = reinterpret_cast<const float4*>(rows4 + (size_t)r * p.row_stride) + u * 8;
                        float a = 0.f;
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            const float4 q = wr[j];
                            a = fmaf(q.x, xv[4 * j], a);
                            a = fmaf(q.y, xv[4 * j + 1], a);
                            a = fmaf(q.z, xv[4 * j + 2], a);
                            a = fmaf(q.w, xv[4 * j + 3], a);
                        }
                        acc[r] += a;
                    }
                }
            } else {
                for (uint32_t u = ua + lane; u < ub; u += 32) {
                    typename Fmt::Raw raw[4];
#pragma unroll
                    for (int r = 0; r < 4; ++r) Fmt::load(rows4 + (size_t)r * p.row_stride, u, p.units, raw[r]);
#pragma unroll
                    for (int sb = 0; sb < Fmt::SUBS; ++sb) {
                        XRec xr;
                        load_xrec(xreg, u * Fmt::SUBS + sb, xr);
#pragma unroll
                        for (int r = 0; r < 4; ++r) acc[r] += Fmt::dot(raw[r], sb, xr, u);
                    }
                }
            }
        }
        // lanes 8r..8r+7 hold this warp's partial of row r (of the tile's 4)
        float v = warp_reduce_rows<4>(acc, lane);
        if (G > 1) {
            // partials of the group's warps meet in shared memory; the leader
            // (gpart 0) waits for all of them, sums and runs the epilogue
            float* ps = part + (size_t)s * G * 4;
            if ((lane & 7) == 0) ps[gpart * 4 + (lane >> 3)] = v;
            __syncwarp();
            if (lane == 0) mbar_arrive(&done[s]);  // also: this warp no longer reads the stage
            if (gpart != 0) continue;
            if (!dead && !mbar_wait(&done[s], ph)) {
                dead = true;
                if (lane == 0) atomicOr(p.err, 4u);
            }
            v = 0.f;
            for (uint32_t k = 0; k < G; ++k) v += ps[k * 4 + (lane >> 3)];
        }
        // every reader of the stage is done: release it to the producer
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        v *= inv;  // 1/rms of the fused RMSNorm (1 if plain)
        const float v_next = __shfl_down_sync(0xffffffffu, v, 8);  // partner row of a pair
        const uint32_t rl = (uint32_t)lane >> 3;
        const uint32_t row = t * p.rt + sub4 + rl;
        if ((lane & 7) != 0 || dead) continue;

        gemv_epilogue_row<EPI>(p, row, v, v_next, best);
    }

    if constexpr (EPI == EPI_LOGITS) {
#pragma unroll
        for (int o = 8; o < 32; o <<= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
            best = other > best ? other : best;
        }
        if (lane == 0) best_sh[warp] = best;
        consumers_sync<W>();
        if (ctid == 0) {
            unsigned long long b = 0ull;
            for (int k = 0; k < W; ++k) b = best_sh[k] > b ? best_sh[k] : b;
            if (b) atomicMax(p.argmax, b);
        }
    }
    if constexpr (EPI == EPI_PEER) {
        // every row partial of this CTA is stored (at the peers too); the last
        // CTA to finish raises this rank's flag at every rank.  One thread
        // fences after the CTA barrier: the barrier orders the other threads'
        // peer stores before its system-scope fence, which is cumulative (a
        // fence in every thread cost each CTA an NVLink round trip per thread)
        consumers_sync<W>();
        if (ctid == 0) __threadfence_system();
        if (ctid == 0 && atomicAdd(p.done_ctr, 1u) == gridDim.x - 1) {
            *p.done_ctr = 0u;
            __threadfence_system();
            const unsigned int e = __ldcg(p.epoch) + 1u;
            for (uint32_t r = 0; r < p.tp; ++r) st_release_sys(p.peer_flag[r], e);
        }
    }
    if (p.trace) {
        consumers_sync<W>();
        if (ctid == 0) trace_mark(p.trace, 2);
    }
}

}  // namespace smallm
