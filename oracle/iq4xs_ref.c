/*
 * TEST INFRASTRUCTURE ONLY -- the CPU oracle for parity checks.  Nothing in
 * the product links this file; tests/, __graft_entry__.smoke() and bench.py's
 * CPU-baseline leg load it as a checker.
 *
 * Plain-C restatement of the reference's IQ4_XS decode,
 * ttrunner_qwen38_flash_next/gguf/quants.py:112-129 (_dequant_iq4_xs), with
 * the codebook of gguf/_codebooks.py:9 (KVALUES_IQ4NL) and the block traits
 * of gguf/reader.py:107 (256 values, 136 bytes).  Pinned against the
 * reference's own outputs (tests/golden/iq4xs_dequant.npz).
 */
#include <stdint.h>
#include <string.h>

static const int8_t kKvalues[16] = {-127, -104, -83, -65, -49, -35, -22, -10,
                                    1,    13,   25,  38,  53,  69,  89,  113};

/* IEEE binary16 -> binary32, exact (quants.py:28 `_f16`: view as float16, astype float32). */
static float half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t exp = (h >> 10) & 0x1Fu;
    const uint32_t mant = h & 0x3FFu;
    uint32_t bits;
    float f;
    if (exp == 0) {
        f = (float)mant * 5.9604644775390625e-8f; /* mant * 2^-24 */
        return sign ? -f : f;
    }
    if (exp == 31) bits = sign | 0x7F800000u | (mant << 13);
    else bits = sign | ((exp + 112u) << 23) | (mant << 13);
    memcpy(&f, &bits, 4);
    return f;
}

/* quants.py:112-129, one super-block at a time. */
void oracle_dequant_iq4xs(const uint8_t* raw, int64_t n_blocks, float* out) {
#pragma omp parallel for schedule(static) if (n_blocks >= 4096)
    for (int64_t b = 0; b < n_blocks; ++b) {
        const uint8_t* blk = raw + b * 136;
        const float d = half_to_float((uint16_t)(blk[0] | (blk[1] << 8)));      /* :115 */
        const uint32_t scales_h = (uint32_t)blk[2] | ((uint32_t)blk[3] << 8);   /* :116 */
        const uint8_t* scales_l = blk + 4;                                       /* :117 */
        const uint8_t* qs = blk + 8;                                             /* :118 */
        float* o = out + b * 256;
        for (int ib = 0; ib < 8; ++ib) {                                         /* :121 */
            const uint32_t ls = (((uint32_t)scales_l[ib / 2] >> (4 * (ib % 2))) & 0xF) |
                                (((scales_h >> (2 * ib)) & 3) << 4);              /* :122-124 */
            const float dl = d * ((float)ls - 32.0f);                            /* :125 */
            const uint8_t* q = qs + ib * 16;                                     /* :126 */
            for (int j = 0; j < 16; ++j) {
                o[ib * 32 + j] = (float)kKvalues[q[j] & 0xF] * dl;               /* :127 */
                o[ib * 32 + 16 + j] = (float)kKvalues[q[j] >> 4] * dl;           /* :128 */
            }
        }
    }
}
