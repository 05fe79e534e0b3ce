// The seeded weight generator of the synthetic BASELINE family, shared by the
// device kernels and the host entry points.
//
// A value stream is keyed by (seed, stream id); value n of the stream is
// normal(group n / 4)[n % 4] * std, where a group's four N(0, 1) values come
// from one Philox4x32-10 block (Salmon, Moraes, Dror, Shaw, "Parallel random
// numbers: as easy as 1, 2, 3", SC 2011; counter = (group lo, group hi,
// stream lo, stream hi), key = seed) through the Box-Muller transform.
//
// Every floating-point step is one IEEE-754 binary32 operation with
// round-to-nearest (add, multiply, fused multiply-add, divide, square root),
// spelled out so that no compiler contracts or reorders it, and the two
// transcendental functions Box-Muller needs are this file's own polynomials:
//   ln u   = e ln 2 + 2 atanh(s), s = (m - 1) / (m + 1), u = m 2^e with
//            m in [sqrt(1/2), sqrt(2)): the odd series of atanh to s^9
//            (|s| <= 0.1716, truncation below 3e-9 relative);
//   sin, cos of (pi / 2) g for g in [0, 1/2]: their Taylor series to a^9
//            and a^10 (a <= pi / 4, truncation below 1e-8);
// the quadrant of 2 pi u1 taken from the exact product 4 u1.  The host and
// the device therefore produce the same bits for every value, and the test
// oracle's C restatement of this generator reproduces them too.
#pragma once

#include <stdint.h>

#include "iq4xs.cuh"

#if !defined(__CUDACC__)
#include <math.h>
#endif

#if defined(__CUDA_ARCH__)
#define QMOE_FADD(a, b) __fadd_rn((a), (b))
#define QMOE_FMUL(a, b) __fmul_rn((a), (b))
#define QMOE_FFMA(a, b, c) __fmaf_rn((a), (b), (c))
#define QMOE_FSQRT(a) __fsqrt_rn(a)
#define QMOE_UMULHI(a, b) __umulhi((a), (b))
#else
#define QMOE_FADD(a, b) ((a) + (b))
#define QMOE_FMUL(a, b) ((a) * (b))
#define QMOE_FFMA(a, b, c) fmaf((a), (b), (c))
#define QMOE_FSQRT(a) sqrtf(a)
#define QMOE_UMULHI(a, b) ((uint32_t)(((uint64_t)(a) * (uint64_t)(b)) >> 32))
#endif

struct qmoe_u4 {
    uint32_t x, y, z, w;
};

// Philox4x32-10: ten rounds of the published round function and key schedule.
QMOE_HD qmoe_u4 qmoe_philox4x32_10(qmoe_u4 c, uint32_t k0, uint32_t k1) {
    for (int r = 0; r < 10; ++r) {
        const uint32_t hi0 = QMOE_UMULHI(0xD2511F53u, c.x), lo0 = 0xD2511F53u * c.x;
        const uint32_t hi1 = QMOE_UMULHI(0xCD9E8D57u, c.z), lo1 = 0xCD9E8D57u * c.z;
        const qmoe_u4 n = {hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0};
        c = n;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    return c;
}

// Natural logarithm of u in [2^-25, 1] (normal binary32).
QMOE_HD float qmoe_synth_ln(float u) {
    const uint32_t b = qmoe_f32_bits(u);
    int e = (int)(b >> 23) - 127;
    float m = qmoe_bits_f32((b & 0x7FFFFFu) | 0x3F800000u);  // [1, 2)
    if (m > 1.41421353816986083984375f) {                     // above sqrt(2): halve (exact)
        m = QMOE_FMUL(m, 0.5f);
        e += 1;
    }
    const float s = qmoe_div(QMOE_FADD(m, -1.0f), QMOE_FADD(m, 1.0f));
    const float z = QMOE_FMUL(s, s);
    float p = QMOE_FFMA(z, 0.111111111f, 0.142857143f);  // 1/9, 1/7
    p = QMOE_FFMA(z, p, 0.2f);                            // 1/5
    p = QMOE_FFMA(z, p, 0.333333343f);                    // 1/3
    p = QMOE_FFMA(z, p, 1.0f);
    const float at2 = QMOE_FMUL(QMOE_FMUL(s, p), 2.0f);  // 2 atanh(s) = ln m
    const float fe = (float)e;                            // exact (|e| <= 25)
    // ln 2 split so that e * hi is exact: hi has 12 significant bits.
    return QMOE_FFMA(fe, 0.693115234375f, QMOE_FFMA(fe, 3.19461832987e-05f, at2));
}

// sin and cos of a = (pi / 2) g, g in [0, 1/2].
QMOE_HD void qmoe_synth_sincos_quarter(float g, float* s, float* c) {
    const float a = QMOE_FMUL(g, 1.57079637050628662109375f);
    const float z = QMOE_FMUL(a, a);
    float ps = QMOE_FFMA(z, 2.75573192e-06f, -1.98412698e-04f);  // 1/9!, -1/7!
    ps = QMOE_FFMA(z, ps, 8.33333377e-03f);                       // 1/5!
    ps = QMOE_FFMA(z, ps, -1.66666672e-01f);                      // -1/3!
    ps = QMOE_FMUL(z, ps);
    *s = QMOE_FFMA(a, ps, a);
    float pc = QMOE_FFMA(z, -2.75573192e-07f, 2.48015876e-05f);  // -1/10!, 1/8!
    pc = QMOE_FFMA(z, pc, -1.38888892e-03f);                      // -1/6!
    pc = QMOE_FFMA(z, pc, 4.16666679e-02f);                       // 1/4!
    pc = QMOE_FFMA(z, pc, -0.5f);                                 // -1/2!
    *c = QMOE_FFMA(z, pc, 1.0f);
}

// sin and cos of 2 pi u for u = j 2^-24, j an integer in [0, 2^24).
QMOE_HD void qmoe_synth_sincos2pi(float u, float* sn, float* cs) {
    const float t = QMOE_FMUL(u, 4.0f);  // exact
    const int q = (int)t;                 // quadrant 0..3
    const float f = QMOE_FADD(t, -(float)q);  // exact, [0, 1)
    float s, c;
    if (f <= 0.5f) {
        qmoe_synth_sincos_quarter(f, &s, &c);
    } else {  // sin((pi/2) f) = cos((pi/2)(1 - f)) and the converse
        qmoe_synth_sincos_quarter(QMOE_FADD(1.0f, -f), &c, &s);
    }
    switch (q) {
        case 0: *sn = s; *cs = c; break;
        case 1: *sn = c; *cs = -s; break;
        case 2: *sn = -s; *cs = -c; break;
        default: *sn = -c; *cs = s; break;
    }
}

// Four N(0, 1) values of counter group g of stream (seed, sid).
QMOE_HD void qmoe_synth_normal4(uint64_t seed, uint64_t sid, uint64_t g, float out[4]) {
    const qmoe_u4 ctr = {(uint32_t)g, (uint32_t)(g >> 32), (uint32_t)sid, (uint32_t)(sid >> 32)};
    const qmoe_u4 r = qmoe_philox4x32_10(ctr, (uint32_t)seed, (uint32_t)(seed >> 32));
    // 24-bit uniforms: u0, u2 in (0, 1] (never 0, for the logarithm), u1, u3 in [0, 1).
    const float u0 = QMOE_FFMA((float)(r.x >> 8), 5.9604644775390625e-8f, 5.9604644775390625e-8f);
    const float u1 = QMOE_FMUL((float)(r.y >> 8), 5.9604644775390625e-8f);
    const float u2 = QMOE_FFMA((float)(r.z >> 8), 5.9604644775390625e-8f, 5.9604644775390625e-8f);
    const float u3 = QMOE_FMUL((float)(r.w >> 8), 5.9604644775390625e-8f);
    const float a = QMOE_FSQRT(QMOE_FMUL(qmoe_synth_ln(u0), -2.0f));
    const float b = QMOE_FSQRT(QMOE_FMUL(qmoe_synth_ln(u2), -2.0f));
    float s0, c0, s1, c1;
    qmoe_synth_sincos2pi(u1, &s0, &c0);
    qmoe_synth_sincos2pi(u3, &s1, &c1);
    out[0] = QMOE_FMUL(a, c0);
    out[1] = QMOE_FMUL(a, s0);
    out[2] = QMOE_FMUL(b, c1);
    out[3] = QMOE_FMUL(b, s1);
}

// Values [4g, 4g + 4) of the stream scaled by std_dev.
QMOE_HD void qmoe_synth_values4(uint64_t seed, uint64_t sid, uint64_t g, float std_dev, float out[4]) {
    float z[4];
    qmoe_synth_normal4(seed, sid, g, z);
    for (int i = 0; i < 4; ++i) out[i] = QMOE_FMUL(z[i], std_dev);
}

// Super-block b of the stream's IQ4_XS form: values [256 b, 256 b + 256)
// quantised by qmoe_quantize_superblock.
QMOE_HD void qmoe_synth_superblock(uint64_t seed, uint64_t sid, uint64_t b, float std_dev, uint8_t* out) {
    float v[256];
    for (int i = 0; i < 64; ++i) qmoe_synth_values4(seed, sid, b * 64 + (uint64_t)i, std_dev, v + 4 * i);
    qmoe_quantize_superblock(v, out);
}
