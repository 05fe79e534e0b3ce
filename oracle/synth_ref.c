/*
 * TEST INFRASTRUCTURE ONLY -- the CPU side of the synthetic BASELINE family
 * for the oracle and the timed CPU reference arm.  Nothing in the product
 * links this file.
 *
 * The reference itself loads its experts from a GGUF checkpoint
 * (reference/weights.py:118-179); this build stands in seeded synthetic
 * weights.  So that the CPU reference arm reads exactly the bytes the GPU
 * bench reads, without loading the product library, this file restates the
 * product's published generator from its specification:
 *   - Philox4x32-10 (Salmon et al., SC 2011), counter = (group lo, group hi,
 *     stream lo, stream hi), key = seed; four 24-bit uniforms per block;
 *   - Box-Muller with this project's polynomial ln and sin/cos (atanh series
 *     to s^9 around m in [sqrt(1/2), sqrt(2)); Taylor to a^9 / a^10 on a
 *     quarter turn folded to [0, pi/4]), every step one correctly rounded
 *     binary32 operation (compiled with -ffp-contract=off, fmaf explicit);
 *   - the project's IQ4_XS quantiser (the reference and gguf 0.19 have none):
 *     per 32-value sub-block the largest-magnitude element maps to the
 *     codebook's extreme entry, d = s_max / -32 stored as fp16, 6-bit
 *     sub-block steps rint(s / d) clamped to [-32, 31], codes by the midpoint
 *     rule with the lower entry on a tie, entry 8 for a zero step.
 * tests/test_oracle.py pins the bytes against the product's host generator,
 * tests/test_gpu_parity.py against the device one.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

typedef struct {
    uint32_t v[4];
} ctr4;

static ctr4 philox10(ctr4 c, uint32_t k0, uint32_t k1) {
    for (int round = 0; round < 10; ++round) {
        const uint64_t p0 = (uint64_t)0xD2511F53u * c.v[0];
        const uint64_t p1 = (uint64_t)0xCD9E8D57u * c.v[2];
        ctr4 n;
        n.v[0] = (uint32_t)(p1 >> 32) ^ c.v[1] ^ k0;
        n.v[1] = (uint32_t)p1;
        n.v[2] = (uint32_t)(p0 >> 32) ^ c.v[3] ^ k1;
        n.v[3] = (uint32_t)p0;
        c = n;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    return c;
}

static uint32_t fbits(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}
static float bitsf(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* ln u for u in [2^-24, 1]. */
static float synth_ln(float u) {
    const uint32_t b = fbits(u);
    int e = (int)(b >> 23) - 127;
    float m = bitsf((b & 0x7FFFFFu) | 0x3F800000u);
    if (m > 1.41421353816986083984375f) {
        m = m * 0.5f;
        e += 1;
    }
    const float s = (m - 1.0f) / (m + 1.0f);
    const float z = s * s;
    float p = fmaf(z, 0.111111111f, 0.142857143f);
    p = fmaf(z, p, 0.2f);
    p = fmaf(z, p, 0.333333343f);
    p = fmaf(z, p, 1.0f);
    const float lnm = (s * p) * 2.0f;
    const float fe = (float)e;
    return fmaf(fe, 0.693115234375f, fmaf(fe, 3.19461832987e-05f, lnm));
}

static void quarter_sincos(float g, float* s, float* c) {
    const float a = g * 1.57079637050628662109375f;
    const float z = a * a;
    float ps = fmaf(z, 2.75573192e-06f, -1.98412698e-04f);
    ps = fmaf(z, ps, 8.33333377e-03f);
    ps = fmaf(z, ps, -1.66666672e-01f);
    ps = z * ps;
    *s = fmaf(a, ps, a);
    float pc = fmaf(z, -2.75573192e-07f, 2.48015876e-05f);
    pc = fmaf(z, pc, -1.38888892e-03f);
    pc = fmaf(z, pc, 4.16666679e-02f);
    pc = fmaf(z, pc, -0.5f);
    *c = fmaf(z, pc, 1.0f);
}

static void turn_sincos(float u, float* sn, float* cs) {
    const float t = u * 4.0f;
    const int q = (int)t;
    const float f = t + -(float)q;
    float s, c;
    if (f <= 0.5f) quarter_sincos(f, &s, &c);
    else quarter_sincos(1.0f + -f, &c, &s);
    if (q == 0) { *sn = s; *cs = c; }
    else if (q == 1) { *sn = c; *cs = -s; }
    else if (q == 2) { *sn = -s; *cs = -c; }
    else { *sn = -c; *cs = s; }
}

static void group4(uint64_t seed, uint64_t sid, uint64_t g, float std_dev, float out[4]) {
    ctr4 c = {{(uint32_t)g, (uint32_t)(g >> 32), (uint32_t)sid, (uint32_t)(sid >> 32)}};
    const ctr4 r = philox10(c, (uint32_t)seed, (uint32_t)(seed >> 32));
    const float step = 5.9604644775390625e-8f; /* 2^-24 */
    const float u0 = fmaf((float)(r.v[0] >> 8), step, step);
    const float u1 = (float)(r.v[1] >> 8) * step;
    const float u2 = fmaf((float)(r.v[2] >> 8), step, step);
    const float u3 = (float)(r.v[3] >> 8) * step;
    const float a = sqrtf(synth_ln(u0) * -2.0f);
    const float b = sqrtf(synth_ln(u2) * -2.0f);
    float s0, c0, s1, c1;
    turn_sincos(u1, &s0, &c0);
    turn_sincos(u3, &s1, &c1);
    out[0] = (a * c0) * std_dev;
    out[1] = (a * s0) * std_dev;
    out[2] = (b * c1) * std_dev;
    out[3] = (b * s1) * std_dev;
}

/* ---- fp16 conversion and the quantiser ------------------------------------ */

static uint16_t to_half(float f) {
    const uint32_t u = fbits(f);
    const uint32_t sign = (u >> 16) & 0x8000u;
    const uint32_t ex = (u >> 23) & 0xFFu;
    uint32_t mant = u & 0x7FFFFFu;
    if (ex == 255) return (uint16_t)(sign | 0x7C00u | (mant ? 0x200u : 0u));
    const int e = (int)ex - 112;
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    if (e <= 0) { /* subnormal or zero half */
        if (e < -10) return (uint16_t)sign;
        mant |= 0x800000u;
        const int sh = 14 - e;
        uint32_t m = mant >> sh;
        const uint32_t rem = mant & ((1u << sh) - 1u), half = 1u << (sh - 1);
        if (rem > half || (rem == half && (m & 1u))) ++m;
        return (uint16_t)(sign | m);
    }
    uint32_t h = sign | ((uint32_t)e << 10) | (mant >> 13);
    const uint32_t rem = mant & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
    return (uint16_t)h;
}

static float from_half(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16, ex = (h >> 10) & 0x1Fu, mant = h & 0x3FFu;
    if (ex == 0) {
        const float v = (float)mant * 5.9604644775390625e-8f;
        return sign ? -v : v;
    }
    if (ex == 31) return bitsf(sign | 0x7F800000u | (mant << 13));
    return bitsf(sign | ((ex + 112u) << 23) | (mant << 13));
}

static void quantize256(const float* x, uint8_t* out) {
    static const float mids[15] = {-115.5f, -93.5f, -74.0f, -57.0f, -42.0f, -28.5f, -16.0f, -4.5f,
                                   7.0f,    19.0f,  31.5f,  45.5f,  61.0f,  79.0f,  101.0f};
    float sub[8];
    int top = 0;
    float top_abs = -1.0f;
    for (int ib = 0; ib < 8; ++ib) {
        float best = -1.0f, val = 0.0f;
        for (int j = 0; j < 32; ++j) {
            const float v = x[32 * ib + j], a = fabsf(v);
            if (a > best) { best = a; val = v; }
        }
        sub[ib] = val / -127.0f;
        if (fabsf(sub[ib]) > top_abs) { top_abs = fabsf(sub[ib]); top = ib; }
    }
    const uint16_t d16 = to_half(sub[top] / -32.0f);
    const float d = from_half(d16);
    uint8_t scl[4] = {0, 0, 0, 0};
    uint16_t sch = 0;
    memset(out + 8, 0, 128);
    for (int ib = 0; ib < 8; ++ib) {
        int l = 0;
        if (d != 0.0f) {
            float r = rintf(sub[ib] / d);
            r = r < -32.0f ? -32.0f : (r > 31.0f ? 31.0f : r);
            l = (int)r;
        }
        const int ls = l + 32;
        scl[ib >> 1] |= (uint8_t)((ls & 15) << (4 * (ib & 1)));
        sch |= (uint16_t)(((ls >> 4) & 3) << (2 * ib));
        const float dl = d * (float)l;
        for (int j = 0; j < 32; ++j) {
            int code = 8;
            if (dl != 0.0f) {
                const float t = x[32 * ib + j] / dl;
                code = 0;
                while (code < 15 && t > mids[code]) ++code;
            }
            /* value j of the sub-block: low nibble of byte j (j < 16), high nibble of byte j - 16 */
            out[8 + 16 * ib + (j & 15)] |= (uint8_t)(code << (j < 16 ? 0 : 4));
        }
    }
    out[0] = (uint8_t)d16;
    out[1] = (uint8_t)(d16 >> 8);
    out[2] = (uint8_t)sch;
    out[3] = (uint8_t)(sch >> 8);
    memcpy(out + 4, scl, 4);
}

/* ---- exported -------------------------------------------------------------- */

void oracle_synth_f32(uint64_t seed, uint64_t sid, int64_t n, float std_dev, float* out) {
    const int64_t groups = (n + 3) / 4;
#pragma omp parallel for schedule(static)
    for (int64_t g = 0; g < groups; ++g) {
        float v[4];
        group4(seed, sid, (uint64_t)g, std_dev, v);
        for (int i = 0; i < 4 && 4 * g + i < n; ++i) out[4 * g + i] = v[i];
    }
}

void oracle_synth_iq4xs(uint64_t seed, uint64_t sid, int64_t n_values, float std_dev, uint8_t* out) {
    const int64_t blocks = n_values / 256;
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < blocks; ++b) {
        float v[256];
        for (int i = 0; i < 64; ++i) group4(seed, sid, (uint64_t)(b * 64 + i), std_dev, v + 4 * i);
        quantize256(v, out + 136 * b);
    }
}

void oracle_quantize_iq4xs(const float* values, int64_t n_values, uint8_t* out) {
    const int64_t blocks = n_values / 256;
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < blocks; ++b) quantize256(values + 256 * b, out + 136 * b);
}
