/*
 * TEST INFRASTRUCTURE ONLY -- the CPU oracle for parity checks.  Nothing in
 * the product links this file; tests/ load it as a checker.
 *
 * Plain-C restatements of the reference's decode of the real checkpoint's
 * other expert formats, ttrunner_qwen38_flash_next/gguf/quants.py:
 *   Q8_0   :33-37  (32 values, 34 bytes: fp16 d, 32 int8)
 *   IQ4_NL :100-108 (32 values, 18 bytes: fp16 d, 16 bytes of 4-bit codes)
 *   IQ3_S  :132-165 (256 values, 110 bytes: fp16 d, qs[64], qh[8], signs[32],
 *                    scales[4]; grid gguf/_codebooks.py:12-80)
 * with the block traits of gguf/reader.py:85-108.  Pinned against the
 * reference's own outputs (tests/golden/formats_dequant.npz).
 */
#include <stdint.h>
#include <string.h>

#include "iq3s_grid.inc"

static const int8_t kKv[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};

static float f16(const uint8_t* p) {
    const uint16_t h = (uint16_t)(p[0] | (p[1] << 8));
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t exp = (h >> 10) & 0x1Fu;
    const uint32_t mant = h & 0x3FFu;
    uint32_t bits;
    float f;
    if (exp == 0) {
        f = (float)mant * 5.9604644775390625e-8f;
        return sign ? -f : f;
    }
    if (exp == 31) bits = sign | 0x7F800000u | (mant << 13);
    else bits = sign | ((exp + 112u) << 23) | (mant << 13);
    memcpy(&f, &bits, 4);
    return f;
}

/* quants.py:33-37 */
static void q8_0(const uint8_t* raw, int64_t nb, float* out) {
    for (int64_t b = 0; b < nb; ++b) {
        const uint8_t* blk = raw + b * 34;
        const float d = f16(blk);
        for (int j = 0; j < 32; ++j) out[b * 32 + j] = d * (float)(int8_t)blk[2 + j];
    }
}

/* quants.py:100-108 */
static void iq4_nl(const uint8_t* raw, int64_t nb, float* out) {
    for (int64_t b = 0; b < nb; ++b) {
        const uint8_t* blk = raw + b * 18;
        const float d = f16(blk);
        for (int j = 0; j < 16; ++j) {
            out[b * 32 + j] = (float)kKv[blk[2 + j] & 0xF] * d;
            out[b * 32 + 16 + j] = (float)kKv[blk[2 + j] >> 4] * d;
        }
    }
}

/* quants.py:132-165 */
static void iq3_s(const uint8_t* raw, int64_t nb, float* out) {
    for (int64_t b = 0; b < nb; ++b) {
        const uint8_t* blk = raw + b * 110;
        const float d = f16(blk);
        const uint8_t* qs = blk + 2;
        const uint8_t* qh = blk + 66;
        const uint8_t* signs = blk + 74;
        const uint8_t* scales = blk + 106;
        for (int ib32 = 0; ib32 < 8; ++ib32) {
            const int sc = (scales[ib32 / 2] >> (4 * (ib32 % 2))) & 0xF;           /* :144 */
            const float db = d * (1.0f + 2.0f * (float)sc);                          /* :145 */
            const int h = qh[ib32];
            for (int l = 0; l < 4; ++l) {
                const int idx1 = qs[ib32 * 8 + 2 * l] | ((h << (8 - 2 * l)) & 256);  /* :153 */
                const int idx2 = qs[ib32 * 8 + 2 * l + 1] | ((h << (7 - 2 * l)) & 256);
                const uint32_t g1 = oracle_iq3s_grid[idx1], g2 = oracle_iq3s_grid[idx2];
                const uint8_t sg = signs[ib32 * 4 + l];
                for (int k = 0; k < 4; ++k) {
                    const float v1 = (float)((g1 >> (8 * k)) & 0xFF) * ((sg >> k) & 1 ? -1.0f : 1.0f);
                    const float v2 = (float)((g2 >> (8 * k)) & 0xFF) * ((sg >> (4 + k)) & 1 ? -1.0f : 1.0f);
                    out[b * 256 + ib32 * 32 + l * 8 + k] = v1 * db;                   /* :162-164 */
                    out[b * 256 + ib32 * 32 + l * 8 + 4 + k] = v2 * db;
                }
            }
        }
    }
}

void oracle_dequant_iq4xs(const uint8_t* raw, int64_t n_blocks, float* out);

/* GGML type ids (gguf/reader.py:53-74): 8 Q8_0, 20 IQ4_NL, 21 IQ3_S, 23 IQ4_XS.
 * Returns 0, or -1 for another type. */
int oracle_dequant(int type, const uint8_t* raw, int64_t n_values, float* out) {
    switch (type) {
        case 8: q8_0(raw, n_values / 32, out); return 0;
        case 20: iq4_nl(raw, n_values / 32, out); return 0;
        case 21: iq3_s(raw, n_values / 256, out); return 0;
        case 23: oracle_dequant_iq4xs(raw, n_values / 256, out); return 0;
        default: return -1;
    }
}
