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
