// Exact dequantisation of one 32-element group of a repacked matrix (shared by
// the embedding, the dequant kernels and the persistent decode step).
#pragma once

#include "common.cuh"
#include "engine.h"

namespace smallm {

// Tiled Q4_0 / Q8_0 storage (mgemv.cuh): rows in tiles of 16, a tile = its
// block pairs (blocks 2p, 2p+1) of pair_bytes; units pad to even.
// Byte offsets of storage row r, block u within the matrix:
__device__ __forceinline__ size_t tiled_pair_base(uint32_t row_stride, uint32_t pair_bytes, uint32_t r, uint32_t u) {
    return (size_t)(r / 16) * 16 * row_stride + (size_t)(u >> 1) * pair_bytes;
}
// Q4_0 nibble byte i (0..15: element i in the low nibble, i + 16 in the high)
__device__ __forceinline__ size_t tiled_q4_0_byte(uint32_t row_stride, uint32_t r, uint32_t u, uint32_t i) {
    const uint32_t rr = r % 16, g = rr % 8, hi = rr / 8, h = u & 1u;
    return tiled_pair_base(row_stride, 576, r, u) + (g * 4 + i / 4) * 16 + (2 * h + hi) * 4 + i % 4;
}
// Q8_0 code k (0..31)
__device__ __forceinline__ size_t tiled_q8_0_byte(uint32_t row_stride, uint32_t r, uint32_t u, uint32_t k) {
    const uint32_t rr = r % 16, g = rr % 8, hi = rr / 8, h = u & 1u;
    return tiled_pair_base(row_stride, 1088, r, u) + h * 512 + (g * 4 + (k % 16) / 4) * 16 + (2 * (k / 16) + hi) * 4 +
           k % 4;
}
// f16 scale of (r, u); scale_off 512 (Q4_0) or 1024 (Q8_0)
__device__ __forceinline__ size_t tiled_scale_byte(uint32_t row_stride, uint32_t pair_bytes, uint32_t scale_off,
                                                   uint32_t r, uint32_t u) {
    const uint32_t rr = r % 16, g = rr % 8, hi = rr / 8, h = u & 1u;
    return tiled_pair_base(row_stride, pair_bytes, r, u) + scale_off + (4 * g + 2 * h + hi) * 2;
}

// 32 consecutive elements (group g of storage row r) of a repacked matrix,
// with the reference's exact arithmetic per type (src/core/tensor.cpp:20-111;
// Q4_K as gguf-py's Q4_K.dequantize_blocks).
static __device__ __forceinline__ void dequant_group(const QMat m, uint32_t r, uint32_t g, float* out) {
    const uint8_t* row = m.base + (size_t)r * m.row_stride;
    switch (m.type) {
        case SM_T_F32: {
            const float* w = reinterpret_cast<const float*>(row) + (size_t)g * 32;
            for (int i = 0; i < 32; ++i) out[i] = w[i];
            break;
        }
        case SM_T_Q4_0: {
            const uint8_t* s = m.base + tiled_scale_byte(m.row_stride, 576, 512, r, g);
            const float d = f16_exact(s[0] | (s[1] << 8));
            for (uint32_t k = 0; k < 16; ++k) {
                const uint8_t q = m.base[tiled_q4_0_byte(m.row_stride, r, g, k)];
                out[k] = __fmul_rn(d, (float)((int)(q & 0xF) - 8));
                out[k + 16] = __fmul_rn(d, (float)((int)(q >> 4) - 8));
            }
            break;
        }
        case SM_T_Q8_0: {
            const uint8_t* s = m.base + tiled_scale_byte(m.row_stride, 1088, 1024, r, g);
            const float d = f16_exact(s[0] | (s[1] << 8));
            for (uint32_t k = 0; k < 32; ++k)
                out[k] = __fmul_rn(d, (float)(int8_t)m.base[tiled_q8_0_byte(m.row_stride, r, g, k)]);
            break;
        }
        case SM_T_Q4_K: {
            const uint32_t sbi = g / 8, j = g % 8;
            const uint8_t* b = row + (size_t)sbi * 144;
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
            const uint8_t* ub = row + (size_t)u * 48;
            const int8_t* sc = reinterpret_cast<const int8_t*>(row + (size_t)m.units * 48 + (size_t)u * 4);
            const uint8_t* dp = row + (size_t)m.units * 52 + (size_t)(u / 4) * 2;
            const float d = f16_exact(dp[0] | (dp[1] << 8));
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

}  // namespace smallm
