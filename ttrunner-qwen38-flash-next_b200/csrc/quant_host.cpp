// Host IQ4_XS quantiser: the loader-side half of the synthetic weight
// builder.  Shares qmoe_quantize_superblock with the device quantiser; this
// file is compiled with -ffp-contract=off so both produce identical bytes.
#include <stdint.h>

#include "../../include/qmoe_b200.h"
#include "iq4xs.cuh"

extern "C" int qmoe_quantize_iq4xs_host(const float* values, int64_t n_values, void* out_blocks,
                                        int n_threads) {
    if (n_values < 0 || n_values % QMOE_SB_VALUES) return QMOE_ERR_INVALID_ARG;
    if (n_values == 0) return QMOE_OK;
    if (!values || !out_blocks) return QMOE_ERR_INVALID_ARG;
    const int64_t n_blocks = n_values / QMOE_SB_VALUES;
    uint8_t* out = static_cast<uint8_t*>(out_blocks);
    if (n_threads < 1) n_threads = 1;
#pragma omp parallel for num_threads(n_threads) schedule(static)
    for (int64_t b = 0; b < n_blocks; ++b) {
        qmoe_quantize_superblock(values + b * QMOE_SB_VALUES, out + b * QMOE_SB_BYTES);
    }
    return QMOE_OK;
}

// The seeded generator on the host: the same bits as qmoe_synth_iq4xs /
// qmoe_synth_f32 on the device (synth.cuh uses only correctly rounded
// binary32 operations).
#include "synth.cuh"

extern "C" int qmoe_synth_iq4xs_host(uint64_t seed, uint64_t stream_id, int64_t n_values, float std_dev,
                                     void* out_blocks, int n_threads) {
    if (n_values < 0 || n_values % QMOE_SB_VALUES) return QMOE_ERR_INVALID_ARG;
    if (n_values == 0) return QMOE_OK;
    if (!out_blocks) return QMOE_ERR_INVALID_ARG;
    const int64_t n_blocks = n_values / QMOE_SB_VALUES;
    uint8_t* out = static_cast<uint8_t*>(out_blocks);
    if (n_threads < 1) n_threads = 1;
#pragma omp parallel for num_threads(n_threads) schedule(static)
    for (int64_t b = 0; b < n_blocks; ++b) qmoe_synth_superblock(seed, stream_id, (uint64_t)b, std_dev, out + b * QMOE_SB_BYTES);
    return QMOE_OK;
}

extern "C" int qmoe_synth_f32_host(uint64_t seed, uint64_t stream_id, int64_t n_values, float std_dev, float* out,
                                   int n_threads) {
    if (n_values < 0) return QMOE_ERR_INVALID_ARG;
    if (n_values == 0) return QMOE_OK;
    if (!out) return QMOE_ERR_INVALID_ARG;
    const int64_t n_groups = (n_values + 3) / 4;
    if (n_threads < 1) n_threads = 1;
#pragma omp parallel for num_threads(n_threads) schedule(static)
    for (int64_t g = 0; g < n_groups; ++g) {
        float v[4];
        qmoe_synth_values4(seed, stream_id, (uint64_t)g, std_dev, v);
        for (int i = 0; i < 4 && 4 * g + i < n_values; ++i) out[4 * g + i] = v[i];
    }
    return QMOE_OK;
}
