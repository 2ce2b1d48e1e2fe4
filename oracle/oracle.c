/*
 * CPU oracle for the smallm-engine decode path -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's arithmetic for the batch-1
 * decode path.  It exists so that tests, the smoke check and the CPU
 * baseline leg of the benchmark can check the CUDA backend against the
 * reference semantics.  Nothing in the product links or calls it.
 *
 * Every function cites the reference file:line it restates (paths are
 * relative to the smallm-engine source tree).  The accumulation order of
 * matmul_quantized copies the reference's 8-lane AVX2 order (lane-wise FMA,
 * then the lo128+hi128 / hadd / hadd horizontal sum) so that this restatement
 * agrees with the reference bit for bit; tests pin that against the reference
 * compiled from its own sources.
 *
 * Q4_K has no reference implementation (the reference's GEMV silently reads
 * it as F32 and its dequantizer throws).  Its block format and dequant follow
 * the published GGUF Q4_K layout as implemented by gguf-py 0.19.0
 * (gguf/quants.py, class Q4_K): d, dmin (f16), 12 bytes of packed 6-bit
 * scales/mins, 128 bytes of nibbles; value = (d*sc)*q - (dmin*m).
 *
 * Build: see oracle/Makefile (gcc -O2 -mfma -fopenmp -ffp-contract=off).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define T_F32 0u
#define T_F16 1u
#define T_Q4_0 2u
#define T_Q8_0 8u
#define T_Q4_K 12u
#define T_Q6_K 14u

/* include/smallm/core/common/quant_common.h:15-40 (IEEE half -> float, exact) */
float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t mant = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0) {
        if (mant == 0) {
            bits = sign;
        } else {
            int e = -1;
            do { mant <<= 1; ++e; } while ((mant & 0x400u) == 0);
            mant &= 0x3FFu;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (mant << 13);
        }
    } else if (exp == 0x1F) {
        bits = sign | 0x7F800000u | (mant << 13);
    } else {
        bits = sign | ((exp - 15u + 127u) << 23) | (mant << 13);
    }
    float out;
    memcpy(&out, &bits, 4);
    return out;
}

static inline uint16_t rd16(const uint8_t* p) { uint16_t v; memcpy(&v, p, 2); return v; }

/* ---- block dequantizers: src/core/tensor.cpp:20-111 ---- */

/* tensor.cpp:26-43: out[i] = scale * q[i] */
static void dq_q8_0(const uint8_t* src, uint64_t count, float* out) {
    for (uint64_t b = 0; b < count / 32; ++b, src += 34) {
        float s = orc_f16_to_f32(rd16(src));
        const int8_t* q = (const int8_t*)(src + 2);
        for (int i = 0; i < 32; ++i) out[b * 32 + i] = s * (float)q[i];
    }
}

/* tensor.cpp:45-67: low nibble -> element i, high nibble -> element i+16, offset 8 */
static void dq_q4_0(const uint8_t* src, uint64_t count, float* out) {
    for (uint64_t b = 0; b < count / 32; ++b, src += 18) {
        float s = orc_f16_to_f32(rd16(src));
        const uint8_t* q = src + 2;
        for (int i = 0; i < 16; ++i) {
            out[b * 32 + i] = s * (float)((int)(q[i] & 0x0F) - 8);
            out[b * 32 + i + 16] = s * (float)((int)(q[i] >> 4) - 8);
        }
    }
}

/* tensor.cpp:68-111: 210-byte super-block ql[128] qh[64] i8 scales[16] f16 d;
 * value = (d * sc) * q, left to right as the reference evaluates it. */
static void dq_q6_k(const uint8_t* src, uint64_t count, float* out) {
    for (uint64_t b = 0; b < count / 256; ++b, src += 210) {
        const uint8_t* ql = src;
        const uint8_t* qh = src + 128;
        const int8_t* sc = (const int8_t*)(src + 192);
        float d = orc_f16_to_f32(rd16(src + 208));
        float* dst = out + b * 256;
        for (int half = 0; half < 2; ++half) {
            const uint8_t* qlh = ql + half * 64;
            const uint8_t* qhh = qh + half * 32;
            const int8_t* sch = sc + half * 8;
            float* dh = dst + half * 128;
            for (int l = 0; l < 32; ++l) {
                uint8_t h = qhh[l];
                int q0 = (int)((qlh[l] & 0x0F) | (((h >> 0) & 3) << 4)) - 32;
                int q1 = (int)((qlh[l + 32] & 0x0F) | (((h >> 2) & 3) << 4)) - 32;
                int q2 = (int)((qlh[l] >> 4) | (((h >> 4) & 3) << 4)) - 32;
                int q3 = (int)((qlh[l + 32] >> 4) | (((h >> 6) & 3) << 4)) - 32;
                dh[l] = d * (float)sch[l / 16] * (float)q0;
                dh[l + 32] = d * (float)sch[2 + l / 16] * (float)q1;
                dh[l + 64] = d * (float)sch[4 + l / 16] * (float)q2;
                dh[l + 96] = d * (float)sch[6 + l / 16] * (float)q3;
            }
        }
    }
}

/* Q4_K scale/min unpack for sub-block j (gguf-py quants.py Q4_K.get_scale_min). */
static void q4k_scale_min(const uint8_t* s, int j, int* sc, int* m) {
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
        *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

/* Q4_K (gguf-py quants.py Q4_K.dequantize_blocks): 144-byte super-block
 * {f16 d, f16 dmin, u8 scales[12], u8 qs[128]}; sub-block j (32 values) reads
 * qs[(j/2)*32 + l], low nibble for even j, high nibble for odd j;
 * value = (d*sc_j)*q - (dmin*m_j). */
static void dq_q4_k(const uint8_t* src, uint64_t count, float* out) {
    for (uint64_t b = 0; b < count / 256; ++b, src += 144) {
        float d = orc_f16_to_f32(rd16(src));
        float dmin = orc_f16_to_f32(rd16(src + 2));
        const uint8_t* s = src + 4;
        const uint8_t* qs = src + 16;
        for (int j = 0; j < 8; ++j) {
            int sc, m;
            q4k_scale_min(s, j, &sc, &m);
            float d1 = d * (float)sc;
            float m1 = dmin * (float)m;
            const uint8_t* q = qs + (j / 2) * 32;
            for (int l = 0; l < 32; ++l) {
                int v = (j & 1) ? (q[l] >> 4) : (q[l] & 0x0F);
                float p = d1 * (float)v;
                out[b * 256 + j * 32 + l] = p - m1;
            }
        }
    }
}

/* tensor.cpp:115-138 dequantize_tensor dispatch (+ Q4_K, see header).
 * Returns 0 on success, -1 for an unsupported type (the reference throws). */
int orc_dequantize(uint32_t type, const uint8_t* src, uint64_t count, float* out) {
    switch (type) {
        case T_F32: memcpy(out, src, count * 4); return 0;
        case T_Q8_0: dq_q8_0(src, count, out); return 0;
        case T_Q4_0: dq_q4_0(src, count, out); return 0;
        case T_Q6_K: dq_q6_k(src, count, out); return 0;
        case T_Q4_K: dq_q4_k(src, count, out); return 0;
        default: return -1;
    }
}

/* bytes of one row of `cols` elements in the given type (0 if unsupported) */
uint64_t orc_row_bytes(uint32_t type, uint64_t cols) {
    switch (type) {
        case T_F32: return cols * 4;
        case T_F16: return cols * 2;
        case T_Q4_0: return cols / 32 * 18;
        case T_Q8_0: return cols / 32 * 34;
        case T_Q4_K: return cols / 256 * 144;
        case T_Q6_K: return cols / 256 * 210;
        default: return 0;
    }
}

/* the reference's 8-lane horizontal sum (ops.cpp:130-136): lo128+hi128, hadd, hadd */
static inline float hsum8(const float a[8]) {
    float t0 = a[0] + a[4], t1 = a[1] + a[5], t2 = a[2] + a[6], t3 = a[3] + a[7];
    float u0 = t0 + t1, u1 = t2 + t3;
    return u0 + u1;
}

/* ---- ops::matmul_quantized, src/core/ops.cpp:97-300 ---- */

static float row_q8_0(const uint8_t* row, const float* x, uint32_t nb) {   /* ops.cpp:103-137 */
    float acc[8] = {0};
    for (uint32_t b = 0; b < nb; ++b, row += 34) {
        float s = orc_f16_to_f32(rd16(row));
        const int8_t* q = (const int8_t*)(row + 2);
        const float* xb = x + b * 32;
        for (int i = 0; i < 32; i += 8)
            for (int l = 0; l < 8; ++l) acc[l] = fmaf((float)q[i + l] * s, xb[i + l], acc[l]);
    }
    return hsum8(acc);
}

static float row_q4_0(const uint8_t* row, const float* x, uint32_t nb) {   /* ops.cpp:139-184 */
    float acc[8] = {0};
    for (uint32_t b = 0; b < nb; ++b, row += 18) {
        float s = orc_f16_to_f32(rd16(row));
        const uint8_t* q = row + 2;
        const float* xb = x + b * 32;
        for (int i = 0; i < 16; i += 8) {
            for (int l = 0; l < 8; ++l)
                acc[l] = fmaf((float)((int)(q[i + l] & 0x0F) - 8) * s, xb[i + l], acc[l]);
            for (int l = 0; l < 8; ++l)
                acc[l] = fmaf((float)((int)(q[i + l] >> 4) - 8) * s, xb[16 + i + l], acc[l]);
        }
    }
    return hsum8(acc);
}

static float row_q6_k(const uint8_t* row, const float* x, uint32_t nsb) {  /* ops.cpp:185-288 */
    float acc[8] = {0};
    for (uint32_t sb = 0; sb < nsb; ++sb, row += 210) {
        const uint8_t* ql = row;
        const uint8_t* qh = row + 128;
        const int8_t* sc = (const int8_t*)(row + 192);
        float d = orc_f16_to_f32(rd16(row + 208));
        const float* xb = x + sb * 256;
        for (int half = 0; half < 2; ++half) {
            const uint8_t* qlh = ql + half * 64;
            const uint8_t* qhh = qh + half * 32;
            const int8_t* sch = sc + half * 8;
            const float* xh = xb + half * 128;
            for (int l = 0; l < 32; l += 8) {
                int si = l / 16;
                float s0 = d * (float)sch[si], s1 = d * (float)sch[2 + si];
                float s2 = d * (float)sch[4 + si], s3 = d * (float)sch[6 + si];
                float f0[8], f1[8], f2[8], f3[8];
                for (int k = 0; k < 8; ++k) {
                    int lo = qlh[l + k], hi = qlh[l + k + 32], h = qhh[l + k];
                    f0[k] = (float)(((lo & 0x0F) | ((h & 3) << 4)) - 32) * s0;
                    f1[k] = (float)(((hi & 0x0F) | (((h >> 2) & 3) << 4)) - 32) * s1;
                    f2[k] = (float)(((lo >> 4) | (((h >> 4) & 3) << 4)) - 32) * s2;
                    f3[k] = (float)(((hi >> 4) | (((h >> 6) & 3) << 4)) - 32) * s3;
                }
                for (int k = 0; k < 8; ++k) acc[k] = fmaf(f0[k], xh[l + k], acc[k]);
                for (int k = 0; k < 8; ++k) acc[k] = fmaf(f1[k], xh[l + k + 32], acc[k]);
                for (int k = 0; k < 8; ++k) acc[k] = fmaf(f2[k], xh[l + k + 64], acc[k]);
                for (int k = 0; k < 8; ++k) acc[k] = fmaf(f3[k], xh[l + k + 96], acc[k]);
            }
        }
    }
    return hsum8(acc);
}

/* Q4_K: no reference GEMV.  Dequantize one super-block (as dq_q4_k) and
 * accumulate in the same 8-lane FMA pattern in element order. */
static float row_q4_k(const uint8_t* row, const float* x, uint32_t nsb) {
    float acc[8] = {0};
    float w[256];
    for (uint32_t sb = 0; sb < nsb; ++sb, row += 144) {
        dq_q4_k(row, 256, w);
        const float* xb = x + sb * 256;
        for (int i = 0; i < 256; i += 8)
            for (int l = 0; l < 8; ++l) acc[l] = fmaf(w[i + l], xb[i + l], acc[l]);
    }
    return hsum8(acc);
}

/* ops.cpp:289-299: the reference's catch-all branch reads W as f32
 * (separate multiply and add: GCC does not contract this loop). */
static float row_f32(const float* wr, const float* x, uint32_t cols) {
    float acc = 0.0f;
    for (uint32_t c = 0; c < cols; ++c) acc += wr[c] * x[c];
    return acc;
}

/* y[rows] = W[rows, cols] . x[cols]; returns -1 for types other than
 * F32/Q4_0/Q8_0/Q4_K/Q6_K (the reference would silently read them as F32).
 * Quantized rows hold cols / 32 (cols / 256) whole blocks (ops.cpp:101,186),
 * so trailing columns are ignored and a row without a whole block gives 0. */
int orc_matmul_quantized(const uint8_t* W, uint32_t type, const float* x,
                         uint32_t rows, uint32_t cols, float* y) {
    if (type != T_F32 && type != T_Q4_0 && type != T_Q8_0 && type != T_Q4_K && type != T_Q6_K) return -1;
    uint64_t rb = orc_row_bytes(type, cols);
    long r;
#pragma omp parallel for schedule(static)
    for (r = 0; r < (long)rows; ++r) {
        const uint8_t* row = W + (uint64_t)r * rb;
        float v;
        switch (type) {
            case T_Q8_0: v = row_q8_0(row, x, cols / 32); break;
            case T_Q4_0: v = row_q4_0(row, x, cols / 32); break;
            case T_Q6_K: v = row_q6_k(row, x, cols / 256); break;
            case T_Q4_K: v = row_q4_k(row, x, cols / 256); break;
            default: v = row_f32((const float*)row, x, cols); break;
        }
        y[r] = v;
    }
    return 0;
}

/* ---- elementwise ops, src/core/ops.cpp ---- */

/* ops.cpp:29-40 (the sum of squares is a separate multiply and add, as the
 * reference build compiles it) */
void orc_rmsnorm(const float* x, const float* w, uint32_t n, float eps, float* y) {
    float ss = 0.0f;
    for (uint32_t i = 0; i < n; ++i) ss += x[i] * x[i];
    float inv = 1.0f / sqrtf(ss / (float)n + eps);
    for (uint32_t i = 0; i < n; ++i) y[i] = x[i] * inv * w[i];
}

/* ops.cpp:43-57 */
void orc_softmax(float* x, uint32_t n) {
    if (n == 0) return;
    float m = x[0];
    for (uint32_t i = 1; i < n; ++i) m = x[i] > m ? x[i] : m;
    float s = 0.0f;
    for (uint32_t i = 0; i < n; ++i) { x[i] = expf(x[i] - m); s += x[i]; }
    float inv = 1.0f / s;
    for (uint32_t i = 0; i < n; ++i) x[i] *= inv;
}

/* ops.cpp:60-65 */
void orc_silu(float* x, uint32_t n) {
    for (uint32_t i = 0; i < n; ++i) { float v = x[i]; x[i] = v / (1.0f + expf(-v)); }
}

/* ops.cpp:68-92: NeoX rotation of pairs (i, i + hd/2).  The reference is
 * built with GCC's default FP contraction, which fuses the rotation as
 * fma(x0, c, -(x1*s)) and fma(x0, s, x1*c); written out explicitly here. */
void orc_rope(float* x, uint32_t n_heads, uint32_t hd, uint32_t pos, float base) {
    for (uint32_t h = 0; h < n_heads; ++h) {
        float* v = x + (uint64_t)h * hd;
        for (uint32_t i = 0; i < hd / 2; ++i) {
            float e = (float)(2 * i) / (float)hd;
            float f = 1.0f / powf(base, e);
            float th = (float)pos * f;
            float c = cosf(th), s = sinf(th);
            float x0 = v[i], x1 = v[i + hd / 2];
            v[i] = fmaf(x0, c, -(x1 * s));
            v[i + hd / 2] = fmaf(x0, s, x1 * c);
        }
    }
}

/* ops.cpp:304-324: 8-lane FMA, horizontal sum, scalar tail (multiply then
 * add, unfused in the reference build) */
float orc_dot(const float* a, const float* b, uint32_t n) {
    float acc[8] = {0};
    uint32_t i = 0;
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; ++l) acc[l] = fmaf(a[i + l], b[i + l], acc[l]);
    float s = hsum8(acc);
    for (; i < n; ++i) s += a[i] * b[i];
    return s;
}

/* ops.cpp:327-337: y += scale * v (the scalar tail is fused in the
 * reference build) */
void orc_axpy(float* y, const float* v, float scale, uint32_t n) {
    uint32_t i = 0;
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; ++l) y[i + l] = fmaf(v[i + l], scale, y[i + l]);
    for (; i < n; ++i) y[i] = fmaf(scale, v[i], y[i]);
}

/* ops.cpp:339-347: y *= v */
void orc_mul(float* y, const float* v, uint32_t n) {
    for (uint32_t i = 0; i < n; ++i) y[i] *= v[i];
}

/* src/model/qwen2_model.cpp:111-133 (llama_model.cpp:297-317 is the same):
 * per query head h, scores over cached positions 0..pos with kv head h/group,
 * softmax, weighted sum of V.  k/v caches are position-major
 * [ctx][n_kv*hd] as in include/smallm/model/common/kv_cache.h:15-27. */
void orc_attention(const float* q, const float* kc, const float* vc, uint32_t n_head,
                   uint32_t n_kv, uint32_t hd, uint32_t pos, float* out, float* scratch) {
    uint32_t kv_dim = n_kv * hd, group = n_head / n_kv;
    float scale = 1.0f / sqrtf((float)hd);
    memset(out, 0, sizeof(float) * n_head * hd);
    for (uint32_t h = 0; h < n_head; ++h) {
        const float* qh = q + h * hd;
        uint32_t kvh = h / group;
        for (uint32_t t = 0; t <= pos; ++t)
            scratch[t] = orc_dot(qh, kc + (uint64_t)t * kv_dim + kvh * hd, hd) * scale;
        orc_softmax(scratch, pos + 1);
        for (uint32_t t = 0; t <= pos; ++t)
            orc_axpy(out + h * hd, vc + (uint64_t)t * kv_dim + kvh * hd, scratch[t], hd);
    }
}

/* src/runtime/sampler/greedy_sampler.cpp:8-14: first index of the strict max */
uint32_t orc_argmax(const float* logits, uint32_t n) {
    uint32_t best = 0;
    for (uint32_t i = 1; i < n; ++i) if (logits[i] > logits[best]) best = i;
    return best;
}
