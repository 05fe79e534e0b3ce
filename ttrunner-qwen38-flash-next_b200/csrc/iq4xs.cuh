// IQ4_XS format helpers shared by every kernel and by the host quantiser.
//
// Super-block layout (256 values, 136 bytes; gguf/reader.py:107 TYPE_TRAITS):
//   bytes 0..1   d        fp16 super-block scale
//   bytes 2..3   scales_h u16, 2 high bits of each sub-block scale
//   bytes 4..7   scales_l 4 bytes, low nibble pairs of the sub-block scales
//   bytes 8..135 qs       128 bytes, 16 per 32-value sub-block
// Sub-block ib (0..7): ls = ((scales_l >> 4*ib) & 15) | (((scales_h >> 2*ib) & 3) << 4),
// dl = d * (ls - 32); value ib*32 + j = kv[qs[16*ib + j] & 15] * dl and value
// ib*32 + 16 + j = kv[qs[16*ib + j] >> 4] * dl for j < 16
// (gguf/quants.py:112-129).  d*(ls-32) is exact in fp32 (11 x 6 bits) and so is
// its product with a codebook entry (<= 7 bits), so any evaluation order of
// the decode gives the reference's bits.
#pragma once

#include <stdint.h>

#if defined(__CUDACC__)
#include <cuda_fp16.h>
#define QMOE_HD __host__ __device__ __forceinline__
#else
#define QMOE_HD static inline
#endif

#define QMOE_SB_VALUES 256
#define QMOE_SB_BYTES 136

// The iq4nl codebook (gguf/_codebooks.py:9), a format constant.
#define QMOE_KV0 (-127)
#define QMOE_KV_TABLE {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113}

// The same table packed four int8 entries per word, little-endian, for byte
// permutes: entries 0..3, 4..7, 8..11, 12..15.
#define QMOE_KV_W0 0xBFAD9881u
#define QMOE_KV_W1 0xF6EADDCFu
#define QMOE_KV_W2 0x26190D01u
#define QMOE_KV_W3 0x71594535u

// ---------------------------------------------------------------------------
// IEEE binary16 conversions written out with integer operations, so the
// host quantiser and the device quantiser share one definition bit for bit.
QMOE_HD uint32_t qmoe_f32_bits(float f) {
    uint32_t u;
    __builtin_memcpy(&u, &f, 4);
    return u;
}
QMOE_HD float qmoe_bits_f32(uint32_t u) {
    float f;
    __builtin_memcpy(&f, &u, 4);
    return f;
}

// binary16 -> binary32 (exact).
QMOE_HD float qmoe_half_bits_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t exp = (h >> 10) & 0x1Fu;
    const uint32_t mant = h & 0x3FFu;
    if (exp == 0) {
        // zero or subnormal: mant * 2^-24, exact in binary32
        const float v = (float)mant * 5.9604644775390625e-8f;
        return sign ? -v : v;
    }
    if (exp == 31) return qmoe_bits_f32(sign | 0x7F800000u | (mant << 13));
    return qmoe_bits_f32(sign | ((exp + 112u) << 23) | (mant << 13));
}

// binary32 -> binary16, round to nearest, ties to even; overflow -> inf.
QMOE_HD uint16_t qmoe_float_to_half_bits(float f) {
    const uint32_t u = qmoe_f32_bits(f);
    const uint32_t sign = (u >> 16) & 0x8000u;
    const uint32_t exp = (u >> 23) & 0xFFu;
    uint32_t mant = u & 0x7FFFFFu;
    if (exp == 255) return (uint16_t)(sign | 0x7C00u | (mant ? 0x200u : 0u));
    const int e = (int)exp - 112;  // biased binary16 exponent
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        mant |= 0x800000u;
        const int shift = 14 - e;
        uint32_t m = mant >> shift;
        const uint32_t rem = mant & ((1u << shift) - 1u);
        const uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (m & 1u))) ++m;
        return (uint16_t)(sign | m);
    }
    uint32_t h = sign | ((uint32_t)e << 10) | (mant >> 13);
    const uint32_t rem = mant & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;  // a carry may roll into inf
    return (uint16_t)h;
}

// IEEE single-precision operations that the compiler may not contract into
// an FMA, so host and device produce the same bits.
QMOE_HD float qmoe_div(float a, float b) {
#if defined(__CUDA_ARCH__)
    return __fdiv_rn(a, b);
#else
    return a / b;
#endif
}
QMOE_HD float qmoe_mul(float a, float b) {
#if defined(__CUDA_ARCH__)
    return __fmul_rn(a, b);
#else
    return a * b;
#endif
}
QMOE_HD float qmoe_rint(float a) {
#if defined(__CUDA_ARCH__)
    return rintf(a);
#else
    return __builtin_rintf(a);
#endif
}

// Sub-block scale index (6 bits) of sub-block ib from the 8-byte header
// words: h0 = bytes 0..3 (d | scales_h << 16), h1 = bytes 4..7 (scales_l).
QMOE_HD int qmoe_iq4xs_ls(uint32_t h0, uint32_t h1, int ib) {
    const uint32_t lo = (h1 >> (4 * ib)) & 0xFu;
    const uint32_t hi = ((h0 >> 16) >> (2 * ib)) & 0x3u;
    return (int)(lo | (hi << 4));
}

// ---------------------------------------------------------------------------
// Quantiser: 256 fp32 values -> one 136-byte IQ4_XS super-block.
//
// The reference has no IQ4_XS quantiser (gguf 0.19's quantize() raises for
// it), so this is this project's own, kept simple and deterministic:
//  1. per 32-value sub-block, the element of largest magnitude (first on
//     ties) maps to the codebook's extreme entry: s_ib = xmax / -127;
//  2. the super-block scale makes the largest |s_ib| the extreme 6-bit
//     step: d = s_max / -32, stored as fp16;
//  3. l_ib = clamp(rint(s_ib / d16), -32, 31), ls = l_ib + 32;
//  4. each value takes the codebook entry nearest to x / (d16 * l_ib), the
//     lower entry on an exact midpoint; a zero step codes every value as
//     entry 8 (+1, the entry nearest zero).
// Only IEEE-rounded operations are used, so host and device agree bitwise.
QMOE_HD void qmoe_quantize_superblock(const float* x, uint8_t* out) {
    const float kv_mid[15] = {-115.5f, -93.5f, -74.0f, -57.0f, -42.0f, -28.5f, -16.0f, -4.5f,
                              7.0f,    19.0f,  31.5f,  45.5f,  61.0f,  79.0f,  101.0f};
    float s[8];
    int best_ib = 0;
    float best_abs = -1.0f;
    for (int ib = 0; ib < 8; ++ib) {
        float amax = -1.0f, xmax = 0.0f;
        for (int j = 0; j < 32; ++j) {
            const float v = x[ib * 32 + j];
            const float a = v < 0.0f ? -v : v;
            if (a > amax) {
                amax = a;
                xmax = v;
            }
        }
        s[ib] = qmoe_div(xmax, (float)QMOE_KV0);
        const float as = s[ib] < 0.0f ? -s[ib] : s[ib];
        if (as > best_abs) {
            best_abs = as;
            best_ib = ib;
        }
    }
    const float d = qmoe_div(s[best_ib], -32.0f);
    const uint16_t d16 = qmoe_float_to_half_bits(d);
    const float df = qmoe_half_bits_to_float(d16);

    uint16_t scales_h = 0;
    uint8_t scales_l[4] = {0, 0, 0, 0};
    for (int ib = 0; ib < 8; ++ib) {
        int l = 0;
        if (df != 0.0f) {
            float r = qmoe_rint(qmoe_div(s[ib], df));
            if (r < -32.0f) r = -32.0f;
            if (r > 31.0f) r = 31.0f;
            l = (int)r;
        }
        const int ls = l + 32;
        scales_l[ib / 2] |= (uint8_t)((ls & 0xF) << (4 * (ib % 2)));
        scales_h |= (uint16_t)(((ls >> 4) & 3) << (2 * ib));
        const float dl = qmoe_mul(df, (float)l);
        uint8_t* qs = out + 8 + 16 * ib;
        for (int j = 0; j < 16; ++j) {
            int q[2];
            for (int half = 0; half < 2; ++half) {
                const float v = x[ib * 32 + 16 * half + j];
                int code = 8;
                if (dl != 0.0f) {
                    const float t = qmoe_div(v, dl);
                    code = 0;
                    for (int m = 0; m < 15; ++m) code += (t > kv_mid[m]) ? 1 : 0;
                }
                q[half] = code;
            }
            qs[j] = (uint8_t)(q[0] | (q[1] << 4));
        }
    }
    out[0] = (uint8_t)(d16 & 0xFF);
    out[1] = (uint8_t)(d16 >> 8);
    out[2] = (uint8_t)(scales_h & 0xFF);
    out[3] = (uint8_t)(scales_h >> 8);
    out[4] = scales_l[0];
    out[5] = scales_l[1];
    out[6] = scales_l[2];
    out[7] = scales_l[3];
}

#if defined(__CUDACC__)
// ---------------------------------------------------------------------------
// Device decode primitives.

// Generic byte permute (PTX prmt default mode): selector nibble bit 3 set
// replicates the selected byte's sign bit into the whole byte.
__device__ __forceinline__ uint32_t qmoe_prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// Eight 4-bit codes in one word -> their int8 codebook values.  Nibbles 0..3
// land in bytes 0..3 of `lo`, nibbles 4..7 in bytes 0..3 of `hi`.  Two table
// permutes per four codes (entries 0..7 and 8..15), a sign-replicating permute
// that turns each code's bit 3 into a byte mask, and one 3-input logic op.
__device__ __forceinline__ void qmoe_lut8(uint32_t w, uint32_t& lo, uint32_t& hi) {
    const uint32_t a = w << 4;
    const uint32_t wm = w & 0x77777777u;
    uint32_t r0 = qmoe_prmt(QMOE_KV_W0, QMOE_KV_W1, w);
    uint32_t r1 = qmoe_prmt(QMOE_KV_W2, QMOE_KV_W3, wm);
    uint32_t m = qmoe_prmt(a, w, 0xD9C8u);
    lo = (r0 & ~m) | (r1 & m);
    r0 = qmoe_prmt(QMOE_KV_W0, QMOE_KV_W1, w >> 16);
    r1 = qmoe_prmt(QMOE_KV_W2, QMOE_KV_W3, wm >> 16);
    m = qmoe_prmt(a, w, 0xFBEAu);
    hi = (r0 & ~m) | (r1 & m);
}

// The codebook shifted by +128 (entries 1..241, all unsigned bytes), packed
// the same way: the prefill dequant places these bytes under an fp32
// exponent to turn them into floats.
#define QMOE_KVB_W0 0x3F2D1801u
#define QMOE_KVB_W1 0x766A5D4Fu
#define QMOE_KVB_W2 0xA6998D81u
#define QMOE_KVB_W3 0xF1D9C5B5u

// qmoe_lut8 with the +128-shifted codebook.
__device__ __forceinline__ void qmoe_lut8_biased(uint32_t w, uint32_t& lo, uint32_t& hi) {
    const uint32_t a = w << 4;
    const uint32_t wm = w & 0x77777777u;
    uint32_t r0 = qmoe_prmt(QMOE_KVB_W0, QMOE_KVB_W1, w);
    uint32_t r1 = qmoe_prmt(QMOE_KVB_W2, QMOE_KVB_W3, wm);
    uint32_t m = qmoe_prmt(a, w, 0xD9C8u);
    lo = (r0 & ~m) | (r1 & m);
    r0 = qmoe_prmt(QMOE_KVB_W0, QMOE_KVB_W1, w >> 16);
    r1 = qmoe_prmt(QMOE_KVB_W2, QMOE_KVB_W3, wm >> 16);
    m = qmoe_prmt(a, w, 0xFBEAu);
    hi = (r0 & ~m) | (r1 & m);
}

// Integer dot product of one 32-value sub-block with an activation block in
// int16 pair form: xp[p] = x[p] | x[16+p] << 16 for p < 16 (the order in
// which a qs byte holds its two codes).  q0..q3 are the sub-block's 16 qs
// bytes as words.  Exact in int32.
__device__ __forceinline__ int qmoe_subblock_dot(uint32_t q0, uint32_t q1, uint32_t q2, uint32_t q3,
                                                 const int* xp, int acc) {
    // Four independent dp2a chains (one per qs word), summed at the end:
    // integer addition is exact, so the order does not change the result,
    // and the chains overlap instead of queueing on one accumulator.
    uint32_t lo0, hi0, lo1, hi1, lo2, hi2, lo3, hi3;
    qmoe_lut8(q0, lo0, hi0);
    qmoe_lut8(q1, lo1, hi1);
    qmoe_lut8(q2, lo2, hi2);
    qmoe_lut8(q3, lo3, hi3);
    int a0 = __dp2a_lo(xp[0], (int)lo0, 0);
    int a1 = __dp2a_lo(xp[4], (int)lo1, 0);
    int a2 = __dp2a_lo(xp[8], (int)lo2, 0);
    int a3 = __dp2a_lo(xp[12], (int)lo3, 0);
    a0 = __dp2a_hi(xp[1], (int)lo0, a0);
    a1 = __dp2a_hi(xp[5], (int)lo1, a1);
    a2 = __dp2a_hi(xp[9], (int)lo2, a2);
    a3 = __dp2a_hi(xp[13], (int)lo3, a3);
    a0 = __dp2a_lo(xp[2], (int)hi0, a0);
    a1 = __dp2a_lo(xp[6], (int)hi1, a1);
    a2 = __dp2a_lo(xp[10], (int)hi2, a2);
    a3 = __dp2a_lo(xp[14], (int)hi3, a3);
    a0 = __dp2a_hi(xp[3], (int)hi0, a0);
    a1 = __dp2a_hi(xp[7], (int)hi1, a1);
    a2 = __dp2a_hi(xp[11], (int)hi2, a2);
    a3 = __dp2a_hi(xp[15], (int)hi3, a3);
    return acc + ((a0 + a1) + (a2 + a3));
}

// The codebook split for a select-free look-up: T1 = entries 0..7 (all
// negative), T2 = entries 8..15 plus one (all positive), four bytes a word.
// For a code c with bit 3 set, a byte permute of T1 with selector c yields
// the sign of T1[c & 7], i.e. -1, and one of T2 with selector c ^ 8 yields
// T2[c & 7] = kv[c] + 1; with bit 3 clear the first yields kv[c] and the
// second the sign of a positive byte, 0.  The two bytes always sum to kv[c].
#define QMOE_KV_T2_W0 0x271A0E02u
#define QMOE_KV_T2_W1 0x725A4636u

// qmoe_subblock_dot without the mask select: each word's eight codes as two
// byte-permute pairs (T1 with the codes, T2 with bit 3 flipped) whose byte
// sums are the codebook values, dotted separately (the sum is the same exact
// int32).  Seven ALU instructions per eight codes instead of twelve, at the
// price of twice the dp2a.
__device__ __forceinline__ int qmoe_subblock_dot_t2(uint32_t q0, uint32_t q1, uint32_t q2, uint32_t q3,
                                                    const int* xp, int acc) {
    const uint32_t qw[4] = {q0, q1, q2, q3};
    int a[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        const uint32_t q = qw[w], f = q ^ 0x88888888u;
        const uint32_t qh = q >> 16, fh = f >> 16;
        const uint32_t p1l = qmoe_prmt(QMOE_KV_W0, QMOE_KV_W1, q), p2l = qmoe_prmt(QMOE_KV_T2_W0, QMOE_KV_T2_W1, f);
        const uint32_t p1h = qmoe_prmt(QMOE_KV_W0, QMOE_KV_W1, qh), p2h = qmoe_prmt(QMOE_KV_T2_W0, QMOE_KV_T2_W1, fh);
        int v = __dp2a_lo(xp[4 * w], (int)p1l, 0);
        v = __dp2a_lo(xp[4 * w], (int)p2l, v);
        v = __dp2a_hi(xp[4 * w + 1], (int)p1l, v);
        v = __dp2a_hi(xp[4 * w + 1], (int)p2l, v);
        v = __dp2a_lo(xp[4 * w + 2], (int)p1h, v);
        v = __dp2a_lo(xp[4 * w + 2], (int)p2h, v);
        v = __dp2a_hi(xp[4 * w + 3], (int)p1h, v);
        a[w] = __dp2a_hi(xp[4 * w + 3], (int)p2h, v);
    }
    return acc + ((a[0] + a[1]) + (a[2] + a[3]));
}

// qmoe_subblock_dot in two halves, for one sub-block dotted with several
// activation blocks: the codes' codebook bytes once (w[0..7]: lo, hi of each
// qs word), then a dp2a pass per activation block.  Same exact int32 sum.
__device__ __forceinline__ void qmoe_subblock_decode(uint32_t q0, uint32_t q1, uint32_t q2, uint32_t q3,
                                                     uint32_t (&w)[8]) {
    qmoe_lut8(q0, w[0], w[1]);
    qmoe_lut8(q1, w[2], w[3]);
    qmoe_lut8(q2, w[4], w[5]);
    qmoe_lut8(q3, w[6], w[7]);
}
__device__ __forceinline__ int qmoe_subblock_dot_decoded(const uint32_t (&w)[8], const int* xp) {
    int a0 = __dp2a_lo(xp[0], (int)w[0], 0);
    int a1 = __dp2a_lo(xp[4], (int)w[2], 0);
    int a2 = __dp2a_lo(xp[8], (int)w[4], 0);
    int a3 = __dp2a_lo(xp[12], (int)w[6], 0);
    a0 = __dp2a_hi(xp[1], (int)w[0], a0);
    a1 = __dp2a_hi(xp[5], (int)w[2], a1);
    a2 = __dp2a_hi(xp[9], (int)w[4], a2);
    a3 = __dp2a_hi(xp[13], (int)w[6], a3);
    a0 = __dp2a_lo(xp[2], (int)w[1], a0);
    a1 = __dp2a_lo(xp[6], (int)w[3], a1);
    a2 = __dp2a_lo(xp[10], (int)w[5], a2);
    a3 = __dp2a_lo(xp[14], (int)w[7], a3);
    a0 = __dp2a_hi(xp[3], (int)w[1], a0);
    a1 = __dp2a_hi(xp[7], (int)w[3], a1);
    a2 = __dp2a_hi(xp[11], (int)w[5], a2);
    a3 = __dp2a_hi(xp[15], (int)w[7], a3);
    return (a0 + a1) + (a2 + a3);
}

// Block floating point for an activation sub-block: the power-of-two step
// 2^(e-14), e the binary exponent of the block's largest magnitude
// (|x| < 2^e), so every |x / step| < 2^14 fits int16 with a bit to spare.
// bf16 inputs within 2^-6 of the block maximum convert exactly.
__device__ __forceinline__ int qmoe_block_exponent(float amax) {
    int e;
    frexpf(amax, &e);  // amax = f * 2^e, f in [0.5, 1)
    return e;
}
#endif  // __CUDACC__
