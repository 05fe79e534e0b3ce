// IQ4_XS decode, the device quantiser and the seeded weight generator.
#include "common.cuh"
#include "synth.cuh"

namespace qmoe {
namespace {

// One thread per 32-value sub-block.  Values are written exactly as the
// reference computes them: kv[q] * (d * (ls - 32)) in fp32
// (gguf/quants.py:112-129).
__global__ void dequant_kernel(const uint8_t* __restrict__ blocks, int64_t n_sub,
                               float* __restrict__ out) {
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= n_sub) return;
    const int64_t sb = t >> 3;
    const int ib = (int)(t & 7);
    const uint8_t* blk = blocks + sb * QMOE_SB_BYTES;
    const uint2 hdr = *reinterpret_cast<const uint2*>(blk);
    const uint2 qa = *reinterpret_cast<const uint2*>(blk + 8 + 16 * ib);
    const uint2 qb = *reinterpret_cast<const uint2*>(blk + 16 + 16 * ib);
    const float d = __half2float(__ushort_as_half((unsigned short)(hdr.x & 0xFFFFu)));
    const int ls = qmoe_iq4xs_ls(hdr.x, hdr.y, ib);
    const float dl = d * (float)(ls - 32);
    const uint32_t q[4] = {qa.x, qa.y, qb.x, qb.y};
    const int kv[16] = QMOE_KV_TABLE;
    float v[32];
#pragma unroll
    for (int w = 0; w < 4; ++w) {
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const uint32_t byte = (q[w] >> (8 * b)) & 0xFFu;
            v[4 * w + b] = (float)kv[byte & 0xF] * dl;
            v[16 + 4 * w + b] = (float)kv[byte >> 4] * dl;
        }
    }
    float4* o = reinterpret_cast<float4*>(out + t * 32);
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
}

__global__ void quantize_kernel(const float* __restrict__ x, int64_t n_blocks,
                                uint8_t* __restrict__ out) {
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= n_blocks) return;
    float v[256];
    const float4* src = reinterpret_cast<const float4*>(x + b * 256);
#pragma unroll 8
    for (int i = 0; i < 64; ++i) {
        const float4 f = src[i];
        v[4 * i] = f.x;
        v[4 * i + 1] = f.y;
        v[4 * i + 2] = f.z;
        v[4 * i + 3] = f.w;
    }
    uint8_t blk[QMOE_SB_BYTES];
    qmoe_quantize_superblock(v, blk);
    uint8_t* dst = out + b * QMOE_SB_BYTES;
#pragma unroll
    for (int i = 0; i < QMOE_SB_BYTES / 8; ++i) {
        uint2 w;
        memcpy(&w, blk + 8 * i, 8);
        *reinterpret_cast<uint2*>(dst + 8 * i) = w;
    }
}

// One counter group (four values) per thread; the arithmetic is the shared
// exact generator of synth.cuh, so the host entry points give the same bits.
__global__ void synth_f32_kernel(uint64_t seed, uint64_t sid, int64_t n, float std_dev,
                                 float* __restrict__ out) {
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (4 * g >= n) return;
    float v[4];
    qmoe_synth_values4(seed, sid, (uint64_t)g, std_dev, v);
    for (int i = 0; i < 4 && 4 * g + i < n; ++i) out[4 * g + i] = v[i];
}

// One super-block (64 counter groups, then the quantiser) per thread.
__global__ void synth_iq4xs_kernel(uint64_t seed, uint64_t sid, int64_t n_blocks, float std_dev,
                                   uint8_t* __restrict__ out) {
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= n_blocks) return;
    uint8_t blk[QMOE_SB_BYTES];
    qmoe_synth_superblock(seed, sid, (uint64_t)b, std_dev, blk);
    uint8_t* dst = out + b * QMOE_SB_BYTES;
#pragma unroll
    for (int i = 0; i < QMOE_SB_BYTES / 8; ++i) {
        uint2 w;
        memcpy(&w, blk + 8 * i, 8);
        *reinterpret_cast<uint2*>(dst + 8 * i) = w;
    }
}

inline unsigned grid_for(int64_t n, int block) { return (unsigned)((n + block - 1) / block); }

}  // namespace

cudaError_t launch_dequant(const uint8_t* blocks, int64_t n_blocks, float* out, cudaStream_t s) {
    if (n_blocks == 0) return cudaSuccess;
    const int64_t n_sub = n_blocks * 8;
    dequant_kernel<<<grid_for(n_sub, 256), 256, 0, s>>>(blocks, n_sub, out);
    return cudaGetLastError();
}

cudaError_t launch_quantize(const float* x, int64_t n_blocks, uint8_t* out, cudaStream_t s) {
    if (n_blocks == 0) return cudaSuccess;
    quantize_kernel<<<grid_for(n_blocks, 128), 128, 0, s>>>(x, n_blocks, out);
    return cudaGetLastError();
}

cudaError_t launch_synth_iq4xs(uint64_t seed, uint64_t sid, int64_t n_blocks, float std_dev,
                               uint8_t* out, cudaStream_t s) {
    if (n_blocks == 0) return cudaSuccess;
    synth_iq4xs_kernel<<<grid_for(n_blocks, 128), 128, 0, s>>>(seed, sid, n_blocks, std_dev, out);
    return cudaGetLastError();
}

cudaError_t launch_synth_f32(uint64_t seed, uint64_t sid, int64_t n, float std_dev, float* out,
                             cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    synth_f32_kernel<<<grid_for((n + 3) / 4, 256), 256, 0, s>>>(seed, sid, n, std_dev, out);
    return cudaGetLastError();
}

}  // namespace qmoe
