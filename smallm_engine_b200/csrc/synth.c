/*
 * Seeded synthetic weight generation for GGUF files (host only).
 *
 * Values are i.i.d. normal from a counter-based generator: element pair p of
 * a tensor keyed by `key` draws two 64-bit words mix(key, 2p), mix(key, 2p+1)
 * (splitmix64 finaliser) and maps them through Box-Muller in double
 * precision, so any element range can be produced in parallel and the bytes
 * do not depend on the thread count.
 *
 * Quantizers:
 *   Q8_0, Q4_0  the ggml reference quantizers as gguf-py 0.19.0 restates them
 *               (gguf/quants.py Q8_0.quantize_blocks, Q4_0.quantize_blocks),
 *               evaluated in f32 in the same order, fp16 scales rounded to
 *               nearest even -- byte-identical to gguf-py.
 *   Q6_K, Q4_K  a plain absmax / min-max quantizer of this project's own into
 *               the GGUF block layouts (gguf-py has no K-quant quantizer).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define T_F32 0u
#define T_Q4_0 2u
#define T_Q8_0 8u
#define T_Q4_K 12u
#define T_Q6_K 14u

static inline uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* normal sample for element i of stream `key` */
static inline double normal_at(uint64_t key, uint64_t i) {
    uint64_t p = i >> 1;
    uint64_t a = mix64(key ^ mix64(2 * p));
    uint64_t b = mix64(key ^ mix64(2 * p + 1));
    double u1 = ((double)(a >> 11) + 1.0) * (1.0 / 9007199254740992.0);
    double u2 = (double)(b >> 11) * (1.0 / 9007199254740992.0);
    double r = sqrt(-2.0 * log(u1));
    double t = 6.283185307179586 * u2;
    return (i & 1) ? r * sin(t) : r * cos(t);
}

/* float -> IEEE half, round to nearest even (NaN kept quiet, overflow -> inf) */
uint16_t synth_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0));
    if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* rounds to >= 65520 */
    if (ax < 0x38800000u) {                                   /* result subnormal or zero */
        if (ax < 0x33000000u) return (uint16_t)sign;          /* < 2^-25: rounds to 0 */
        uint32_t e = ax >> 23;
        uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
        uint32_t shift = 126 - e; /* 14 + (112 - e) */
        uint32_t q = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t e = (ax >> 23) - 112;
    uint32_t m = ax & 0x7FFFFFu;
    uint32_t q = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1))) q++;
    return (uint16_t)(sign | q);
}

static float f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16, exp = (h >> 10) & 0x1Fu, mant = h & 0x3FFu, bits;
    if (exp == 0) {
        if (mant == 0) bits = sign;
        else {
            exp = 113;
            while ((mant & 0x400u) == 0) { mant <<= 1; --exp; }
            bits = sign | (exp << 23) | ((mant & 0x3FFu) << 13);
        }
    } else if (exp == 0x1F) bits = sign | 0x7F800000u | (mant << 13);
    else bits = sign | ((exp + 112u) << 23) | (mant << 13);
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static void put16(uint8_t* p, uint16_t v) { memcpy(p, &v, 2); }

/* gguf-py Q8_0.quantize_blocks: d = amax/127, q = roundf(x * (1/d)) */
static void q8_0_block(const float* x, uint8_t* out) {
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) { float a = fabsf(x[i]); if (a > amax) amax = a; }
    float d = amax / 127.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    put16(out, synth_f32_to_f16(d));
    for (int i = 0; i < 32; ++i) {
        float v = x[i] * id;
        out[2 + i] = (uint8_t)(int8_t)roundf(v);
    }
}

/* gguf-py Q4_0.quantize_blocks: max = element of largest |x| (first one),
 * d = max / -8, q = min(15, trunc(x * (1/d) + 8.5)) */
static void q4_0_block(const float* x, uint8_t* out) {
    int im = 0;
    float amax = fabsf(x[0]);
    for (int i = 1; i < 32; ++i) { float a = fabsf(x[i]); if (a > amax) { amax = a; im = i; } }
    float d = x[im] / -8.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    put16(out, synth_f32_to_f16(d));
    uint8_t q[32];
    for (int i = 0; i < 32; ++i) {
        float v = truncf(x[i] * id + 8.5f);
        int qi = (int)v;
        q[i] = (uint8_t)(qi > 15 ? 15 : qi);
    }
    for (int i = 0; i < 16; ++i) out[2 + i] = (uint8_t)(q[i] | (q[i + 16] << 4));
}

static inline int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* Q6_K: 16 sub-blocks of 16 with int8 scales under an f16 super scale d. */
static void q6_k_block(const float* x, uint8_t* out) {
    float sub[16], smax = 0.0f;
    for (int s = 0; s < 16; ++s) {
        float a = 0.0f;
        for (int i = 0; i < 16; ++i) { float v = fabsf(x[s * 16 + i]); if (v > a) a = v; }
        sub[s] = a / 31.0f;
        if (sub[s] > smax) smax = sub[s];
    }
    uint16_t dh = synth_f32_to_f16(smax / 127.0f);
    float d = f16_to_f32(dh);
    int8_t sc[16];
    for (int s = 0; s < 16; ++s) sc[s] = (int8_t)(d > 0.0f ? clampi((int)lrintf(sub[s] / d), 0, 127) : 0);
    uint8_t q[256];
    for (int e = 0; e < 256; ++e) {
        float eff = d * (float)sc[e / 16];
        int v = eff > 0.0f ? clampi((int)lrintf(x[e] / eff), -32, 31) : 0;
        q[e] = (uint8_t)(v + 32);
    }
    uint8_t* ql = out;
    uint8_t* qh = out + 128;
    memset(out, 0, 210);
    for (int h = 0; h < 2; ++h)
        for (int l = 0; l < 32; ++l) {
            int b = h * 128;
            uint8_t q0 = q[b + l], q1 = q[b + 32 + l], q2 = q[b + 64 + l], q3 = q[b + 96 + l];
            ql[h * 64 + l] = (uint8_t)((q0 & 0xF) | ((q2 & 0xF) << 4));
            ql[h * 64 + 32 + l] = (uint8_t)((q1 & 0xF) | ((q3 & 0xF) << 4));
            qh[h * 32 + l] = (uint8_t)((q0 >> 4) | ((q1 >> 4) << 2) | ((q2 >> 4) << 4) | ((q3 >> 4) << 6));
        }
    memcpy(out + 192, sc, 16);
    put16(out + 208, dh);
}

/* Q4_K: 8 sub-blocks of 32 with 6-bit scale and min under f16 d and dmin. */
static void q4_k_block(const float* x, uint8_t* out) {
    float scl[8], mins[8], smax = 0.0f, mmax = 0.0f;
    for (int j = 0; j < 8; ++j) {
        float lo = 0.0f, hi = x[j * 32];
        for (int i = 0; i < 32; ++i) {
            float v = x[j * 32 + i];
            if (v < lo) lo = v;
            if (v > hi) hi = v;
        }
        if (hi < 0.0f) hi = 0.0f;
        scl[j] = (hi - lo) / 15.0f;
        mins[j] = -lo;
        if (scl[j] > smax) smax = scl[j];
        if (mins[j] > mmax) mmax = mins[j];
    }
    uint16_t dh = synth_f32_to_f16(smax / 63.0f), mh = synth_f32_to_f16(mmax / 63.0f);
    float d = f16_to_f32(dh), dmin = f16_to_f32(mh);
    int sc[8], m[8];
    for (int j = 0; j < 8; ++j) {
        sc[j] = d > 0.0f ? clampi((int)lrintf(scl[j] / d), 0, 63) : 0;
        m[j] = dmin > 0.0f ? clampi((int)lrintf(mins[j] / dmin), 0, 63) : 0;
    }
    memset(out, 0, 144);
    put16(out, dh);
    put16(out + 2, mh);
    uint8_t* s = out + 4;
    for (int j = 0; j < 4; ++j) {
        s[j] = (uint8_t)(sc[j] | ((sc[j + 4] >> 4) << 6));
        s[j + 4] = (uint8_t)(m[j] | ((m[j + 4] >> 4) << 6));
        s[j + 8] = (uint8_t)((sc[j + 4] & 0xF) | ((m[j + 4] & 0xF) << 4));
    }
    uint8_t* qs = out + 16;
    for (int j = 0; j < 8; ++j) {
        float ed = d * (float)sc[j], em = dmin * (float)m[j];
        for (int l = 0; l < 32; ++l) {
            int v = ed > 0.0f ? clampi((int)lrintf((x[j * 32 + l] + em) / ed), 0, 15) : 0;
            if (j & 1) qs[(j / 2) * 32 + l] |= (uint8_t)(v << 4);
            else qs[(j / 2) * 32 + l] |= (uint8_t)v;
        }
    }
}

static int block_elems(uint32_t type) {
    switch (type) {
        case T_F32: return 1;
        case T_Q4_0: case T_Q8_0: return 32;
        case T_Q4_K: case T_Q6_K: return 256;
        default: return 0;
    }
}
static int block_bytes(uint32_t type) {
    switch (type) {
        case T_F32: return 4;
        case T_Q4_0: return 18;
        case T_Q8_0: return 34;
        case T_Q4_K: return 144;
        case T_Q6_K: return 210;
        default: return 0;
    }
}

/* quantize `count` floats (a multiple of the block size) into `out` */
int synth_quantize(uint32_t type, const float* x, uint64_t count, uint8_t* out) {
    int be = block_elems(type), bb = block_bytes(type);
    if (be == 0 || count % (uint64_t)be) return -1;
    long nb = (long)(count / (uint64_t)be), b;
#pragma omp parallel for schedule(static)
    for (b = 0; b < nb; ++b) {
        const float* xb = x + (uint64_t)b * be;
        uint8_t* ob = out + (uint64_t)b * bb;
        switch (type) {
            case T_F32: memcpy(ob, xb, 4); break;
            case T_Q8_0: q8_0_block(xb, ob); break;
            case T_Q4_0: q4_0_block(xb, ob); break;
            case T_Q6_K: q6_k_block(xb, ob); break;
            default: q4_k_block(xb, ob); break;
        }
    }
    return 0;
}

/* mean + std * N(0,1) for elements [0, count) of stream `key` */
void synth_normals(uint64_t key, uint64_t count, float mean, float std, float* out) {
    long i;
#pragma omp parallel for schedule(static)
    for (i = 0; i < (long)count; ++i) out[i] = (float)((double)mean + (double)std * normal_at(key, (uint64_t)i));
}

/* Generate and quantize a whole tensor in one parallel pass:
 * element values mean + std * N(0,1) from stream `key`. */
int synth_fill(uint32_t type, uint64_t key, uint64_t count, float mean, float std, uint8_t* out) {
    int be = block_elems(type), bb = block_bytes(type);
    if (be == 0 || count % (uint64_t)be) return -1;
    long nb = (long)(count / (uint64_t)be), b;
#pragma omp parallel for schedule(static)
    for (b = 0; b < nb; ++b) {
        float xb[256];
        for (int i = 0; i < be; ++i)
            xb[i] = (float)((double)mean + (double)std * normal_at(key, (uint64_t)b * be + i));
        uint8_t* ob = out + (uint64_t)b * bb;
        switch (type) {
            case T_F32: memcpy(ob, xb, 4); break;
            case T_Q8_0: q8_0_block(xb, ob); break;
            case T_Q4_0: q4_0_block(xb, ob); break;
            case T_Q6_K: q6_k_block(xb, ob); break;
            default: q4_k_block(xb, ob); break;
        }
    }
    return 0;
}
