// Exact dequantisation of one 32-element group of a repacked matrix (shared by
// the embedding, the dequant kernels and the persistent decode step).
#pragma once

#include "common.cuh"
#include "engine.h"

namespace smallm {

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
            const uint8_t* q = row + (size_t)g * 16;
            const uint8_t* s = row + (size_t)m.units * 16 + (size_t)g * 2;
            const float d = f16_exact(s[0] | (s[1] << 8));
            for (int k = 0; k < 16; ++k) {
                out[k] = __fmul_rn(d, (float)((int)(q[k] & 0xF) - 8));
                out[k + 16] = __fmul_rn(d, (float)((int)(q[k] >> 4) - 8));
            }
            break;
        }
        case SM_T_Q8_0: {
            const int8_t* q = reinterpret_cast<const int8_t*>(row + (size_t)g * 32);
            const uint8_t* s = row + (size_t)m.units * 32 + (size_t)g * 2;
            const float d = f16_exact(s[0] | (s[1] << 8));
            for (int k = 0; k < 32; ++k) out[k] = __fmul_rn(d, (float)q[k]);
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
