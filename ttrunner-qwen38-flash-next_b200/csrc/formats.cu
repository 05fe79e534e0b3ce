// The real checkpoint's other expert formats (the reference's gguf/quants.py;
// tt/plan.py:90-103 puts IQ3_S on gate|up and IQ4_NL, or Q8_0 for the first
// layers, on down): a bit-exact decode to fp32 and the MoE block's expert
// stages on weights of any of them.
//
//   Q8_0    32 values in 34 bytes: fp16 d, 32 int8            (quants.py:33-37)
//   IQ4_NL  32 values in 18 bytes: fp16 d, 16 bytes of codes  (quants.py:100-108)
//   IQ3_S   256 values in 110 bytes: fp16 d, qs[64], qh[8], signs[32],
//           scales[4]; 9-bit grid indices, one sign bit per value,
//           d * (1 + 2 sc) per 32 values                       (quants.py:132-165)
//   IQ4_XS  the format of the rest of this library            (quants.py:112-129)
//
// Every weight is decoded with the reference's own arithmetic (one fp32
// multiply by the block scale), so this decode is bitwise the reference's.
// The MoE block's expert stages on these formats run on the integer core of
// the rest of the library (experts.cu: fmt_gateup_kernel, fmt_down_kernel).
#include "common.cuh"

namespace qmoe {
namespace {

#define QMOE_IQ3S_GRID_DEF __device__ uint32_t g_iq3s_grid[512]
#include "iq3s_grid.inc"
#undef QMOE_IQ3S_GRID_DEF

__device__ float g_kvf[16] = {-127.f, -104.f, -83.f, -65.f, -49.f, -35.f, -22.f, -10.f,
                              1.f, 13.f, 25.f, 38.f, 53.f, 69.f, 89.f, 113.f};

// The two code tables in shared memory, where lanes with different codes read
// them in one pass (a constant-bank read serialises on distinct addresses).
struct FmtTables {
    uint32_t grid[512];
    float kv[16];
};

__device__ __forceinline__ void load_tables(FmtTables& t) {
    for (int i = threadIdx.x; i < 512; i += blockDim.x) t.grid[i] = g_iq3s_grid[i];
    if (threadIdx.x < 16) t.kv[threadIdx.x] = g_kvf[threadIdx.x];
    __syncthreads();
}


__device__ __forceinline__ float f16_at(const uint8_t* p) {
    return __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
}

// Values 0..31 of 32-value sub-block sb of a row in format fmt.
__device__ __forceinline__ void decode32(int fmt, const uint8_t* row, int64_t sb, float (&v)[32],
                                         const FmtTables& tb) {
    if (fmt == QMOE_FMT_Q8_0) {
        const uint8_t* blk = row + (size_t)sb * 34;
        const float d = f16_at(blk);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = d * (float)(int8_t)blk[2 + j];
    } else if (fmt == QMOE_FMT_IQ4_NL) {
        const uint8_t* blk = row + (size_t)sb * 18;
        const float d = f16_at(blk);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const uint8_t q = blk[2 + j];
            v[j] = tb.kv[q & 0xF] * d;
            v[16 + j] = tb.kv[q >> 4] * d;
        }
    } else if (fmt == QMOE_FMT_IQ4_XS) {
        const uint8_t* blk = row + (size_t)(sb >> 3) * 136;
        const int ib = sb & 7;
        const float d = f16_at(blk);
        const uint32_t sh = (uint32_t)blk[2] | ((uint32_t)blk[3] << 8);
        const uint32_t ls = (((uint32_t)blk[4 + ib / 2] >> (4 * (ib % 2))) & 0xF) | (((sh >> (2 * ib)) & 3) << 4);
        const float dl = d * ((float)ls - 32.0f);
        const uint8_t* q = blk + 8 + ib * 16;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            v[j] = tb.kv[q[j] & 0xF] * dl;
            v[16 + j] = tb.kv[q[j] >> 4] * dl;
        }
    } else {  // QMOE_FMT_IQ3_S
        const uint8_t* blk = row + (size_t)(sb >> 3) * 110;
        const int ib32 = sb & 7;
        const float d = f16_at(blk);
        const int sc = (blk[106 + ib32 / 2] >> (4 * (ib32 % 2))) & 0xF;
        const float db = d * (1.0f + 2.0f * (float)sc);
        const uint8_t* qs = blk + 2 + ib32 * 8;
        const int h = blk[66 + ib32];
        const uint8_t* sg = blk + 74 + ib32 * 4;
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const uint32_t g1 = tb.grid[qs[2 * l] | ((h << (8 - 2 * l)) & 256)];
            const uint32_t g2 = tb.grid[qs[2 * l + 1] | ((h << (7 - 2 * l)) & 256)];
            const int s = sg[l];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float a = (float)((g1 >> (8 * k)) & 0xFF) * (((s >> k) & 1) ? -1.0f : 1.0f);
                const float b = (float)((g2 >> (8 * k)) & 0xFF) * (((s >> (4 + k)) & 1) ? -1.0f : 1.0f);
                v[l * 8 + k] = a * db;
                v[l * 8 + 4 + k] = b * db;
            }
        }
    }
}

__global__ void fmt_dequant_kernel(int fmt, const uint8_t* __restrict__ raw, int64_t n_sub, float* __restrict__ out) {
    __shared__ FmtTables tb;
    load_tables(tb);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_sub; i += (int64_t)gridDim.x * blockDim.x) {
        float v[32];
        decode32(fmt, raw, i, v, tb);
        float4* o = reinterpret_cast<float4*>(out + i * 32);
#pragma unroll
        for (int q = 0; q < 8; ++q) o[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    }
}

}  // namespace

// Bytes of a row of n values in format fmt (0: not a whole number of blocks or unknown format).
size_t fmt_row_bytes(int fmt, int64_t n) {
    switch (fmt) {
        case QMOE_FMT_Q8_0: return n % 32 ? 0 : (size_t)(n / 32) * 34;
        case QMOE_FMT_IQ4_NL: return n % 32 ? 0 : (size_t)(n / 32) * 18;
        case QMOE_FMT_IQ3_S: return n % 256 ? 0 : (size_t)(n / 256) * 110;
        case QMOE_FMT_IQ4_XS: return n % 256 ? 0 : (size_t)(n / 256) * 136;
        default: return 0;
    }
}

cudaError_t launch_fmt_dequant(int fmt, const uint8_t* raw, int64_t n_values, float* out, cudaStream_t s) {
    const int64_t n_sub = n_values / 32;
    int64_t g = (n_sub + 255) / 256;
    const int64_t cap = (int64_t)device_sm_count() * 16;
    if (g > cap) g = cap;
    if (g < 1) g = 1;
    const unsigned grid = (unsigned)g;
    fmt_dequant_kernel<<<grid, 256, 0, s>>>(fmt, raw, n_sub, out);
    return cudaGetLastError();
}

}  // namespace qmoe
