// IQ4_XS decode, the device quantiser and the seeded weight generator.
#include "common.cuh"

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

// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as
// easy as 1, 2, 3", SC 2011): counter = (group lo, group hi, stream lo,
// stream hi), key = seed.
__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint2 k) {
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        const uint32_t hi0 = __umulhi(0xD2511F53u, c.x), lo0 = 0xD2511F53u * c.x;
        const uint32_t hi1 = __umulhi(0xCD9E8D57u, c.z), lo1 = 0xCD9E8D57u * c.z;
        c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
        k.x += 0x9E3779B9u;
        k.y += 0xBB67AE85u;
    }
    return c;
}

// Four N(0,1) values for counter group g (Box-Muller on two uniform pairs).
__device__ __forceinline__ float4 normal4(uint64_t seed, uint64_t sid, uint64_t g) {
    const uint4 r = philox4x32_10(make_uint4((uint32_t)g, (uint32_t)(g >> 32), (uint32_t)sid,
                                             (uint32_t)(sid >> 32)),
                                  make_uint2((uint32_t)seed, (uint32_t)(seed >> 32)));
    const float u0 = (float)(r.x >> 8) * 5.9604644775390625e-8f + 2.98023223876953125e-8f;
    const float u1 = (float)(r.y >> 8) * 5.9604644775390625e-8f;
    const float u2 = (float)(r.z >> 8) * 5.9604644775390625e-8f + 2.98023223876953125e-8f;
    const float u3 = (float)(r.w >> 8) * 5.9604644775390625e-8f;
    const float a = sqrtf(-2.0f * logf(u0));
    const float b = sqrtf(-2.0f * logf(u2));
    float s0, c0, s1, c1;
    sincospif(2.0f * u1, &s0, &c0);
    sincospif(2.0f * u3, &s1, &c1);
    return make_float4(a * c0, a * s0, b * c1, b * s1);
}

__global__ void synth_f32_kernel(uint64_t seed, uint64_t sid, int64_t n, float std_dev,
                                 float* __restrict__ out) {
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (4 * g >= n) return;
    const float4 z = normal4(seed, sid, (uint64_t)g);
    const float v[4] = {z.x * std_dev, z.y * std_dev, z.z * std_dev, z.w * std_dev};
    for (int i = 0; i < 4 && 4 * g + i < n; ++i) out[4 * g + i] = v[i];
}

__global__ void synth_iq4xs_kernel(uint64_t seed, uint64_t sid, int64_t n_blocks, float std_dev,
                                   uint8_t* __restrict__ out) {
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= n_blocks) return;
    float v[256];
#pragma unroll 4
    for (int i = 0; i < 64; ++i) {
        const float4 z = normal4(seed, sid, (uint64_t)(b * 64 + i));
        v[4 * i] = z.x * std_dev;
        v[4 * i + 1] = z.y * std_dev;
        v[4 * i + 2] = z.z * std_dev;
        v[4 * i + 3] = z.w * std_dev;
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
