// The hyper-connection mixer around the MoE block: the reference's gated
// residual (reference/model.py:53-81; device ops tt/ops.py:2627
// gated_residual_mix and :2825 reinject).
//
//   normed  = rms_norm(hyper, norm_w, eps, group = hidden)     hyper [M, hc * D]
//   t       = normed . [down_w; inject_w]^T                    [M, rank + hc]
//   mixed   = mean_s sigmoid(up_w[s D + d] . silu(t[:rank] / hc)) * normed[s D + d]
//   inject  = 2 sigmoid(t[rank + s] / hc)
//   reinject: out = hyper + branch (outer) inject
//
// Three launches: the streams' inverse RMS; the down and inject rows (a warp
// per row, the tokens' normalised streams staged in shared memory a group of
// tokens at a time, every row read once per group); the up rows, the gate and
// the mean over the streams (a warp per output column).  fp32 throughout; the
// MoE block reads `mixed` as its input and its output is the `branch` that
// the reinjection adds back into every stream.
#include "common.cuh"

namespace qmoe {
namespace {

constexpr int kHcWarps = 8;
constexpr int kHcGroup = 4;               // tokens staged per pass of the down rows
constexpr size_t kHcSmem = 200 * 1024;    // dynamic shared memory ceiling per CTA

__device__ __forceinline__ float load_val(const void* p, int f32, size_t i) {
    return f32 ? reinterpret_cast<const float*>(p)[i] : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}

// inv[m * hc + s] = 1 / sqrt(mean(x^2) + eps) over stream s of token m.
__global__ void __launch_bounds__(256) hc_rms_kernel(const void* hyper, int f32, int D, int hc, float eps,
                                                     float* inv) {
    __shared__ float part[8];
    const int ms = blockIdx.x, m = ms / hc, s = ms % hc;
    const size_t base = ((size_t)m * hc + s) * D;
    float acc = 0.0f;
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
        const float v = load_val(hyper, f32, base + i);
        acc = fmaf(v, v, acc);
    }
    acc = warp_sum(acc);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.0f;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += part[w];
        inv[ms] = 1.0f / sqrtf(t / (float)D + eps);
    }
}

// t[m * R1 + j] = normed_m . row_j for rows j < rank (down_w) and rank..rank+hc (inject_w).
__global__ void __launch_bounds__(kHcWarps * 32) hc_down_kernel(const void* hyper, int f32, int M, int D, int hc,
                                                                int rank, int group, const float* __restrict__ norm_w,
                                                                const float* __restrict__ down_w,
                                                                const float* __restrict__ inject_w,
                                                                const float* __restrict__ inv, float* t) {
    extern __shared__ __align__(16) float xn[];  // [group][hc * D]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int N = hc * D, R1 = rank + hc;
    const int row = blockIdx.x * kHcWarps + warp;
    const float* w = row >= R1 ? nullptr : row < rank ? down_w + (size_t)row * N : inject_w + (size_t)(row - rank) * N;
    for (int m0 = 0; m0 < M; m0 += group) {
        const int G = min(group, M - m0);
        __syncthreads();
        for (int i = threadIdx.x; i < G * N; i += blockDim.x) {
            const int g = i / N, c = i - g * N;
            const float v = load_val(hyper, f32, (size_t)(m0 + g) * N + c);
            xn[i] = (v * inv[(m0 + g) * hc + c / D]) * norm_w[c];
        }
        __syncthreads();
        if (row >= R1) continue;
        float acc[kHcGroup];
#pragma unroll
        for (int g = 0; g < kHcGroup; ++g) acc[g] = 0.0f;
        for (int c = lane * 4; c < N; c += 128) {
            const float4 wv = __ldg(reinterpret_cast<const float4*>(w + c));
#pragma unroll
            for (int g = 0; g < kHcGroup; ++g) {
                if (g < G) {
                    const float4 x = *reinterpret_cast<const float4*>(xn + (size_t)g * N + c);
                    acc[g] = fmaf(wv.x, x.x, acc[g]);
                    acc[g] = fmaf(wv.y, x.y, acc[g]);
                    acc[g] = fmaf(wv.z, x.z, acc[g]);
                    acc[g] = fmaf(wv.w, x.w, acc[g]);
                }
            }
        }
#pragma unroll
        for (int g = 0; g < kHcGroup; ++g) {
            if (g < G) {
                const float v = warp_sum(acc[g]);
                if (lane == 0) t[(size_t)(m0 + g) * R1 + row] = v;
            }
        }
    }
}

// mixed[m][d] = (1 / hc) sum_s sigmoid(up_w[s D + d] . silu(t[m][:rank] / hc)) * normed[m][s D + d];
// block 0 also writes inject[m][s] = 2 sigmoid(t[m][rank + s] / hc).
__global__ void __launch_bounds__(kHcWarps * 32) hc_up_kernel(const void* hyper, int f32, int M, int D, int hc,
                                                              int rank, const float* __restrict__ norm_w,
                                                              const float* __restrict__ up_w,
                                                              const float* __restrict__ inv, const float* t,
                                                              float* mixed, float* inject) {
    extern __shared__ __align__(16) float mix1[];  // [M][rank]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int N = hc * D, R1 = rank + hc;
    const float rhc = 1.0f / (float)hc;
    for (int i = threadIdx.x; i < M * rank; i += blockDim.x) {
        const int m = i / rank, r = i - m * rank;
        const float z = __ldcg(t + (size_t)m * R1 + r) / (float)hc;
        mix1[i] = silu(z);
    }
    if (blockIdx.x == 0) {
        for (int i = threadIdx.x; i < M * hc; i += blockDim.x) {
            const int m = i / hc, s = i - m * hc;
            inject[i] = 2.0f * sigmoid(__ldcg(t + (size_t)m * R1 + rank + s) / (float)hc);
        }
    }
    __syncthreads();
    const int d = blockIdx.x * kHcWarps + warp;
    if (d >= D) return;
    for (int m = 0; m < M; ++m) {
        float acc = 0.0f;
        for (int s = 0; s < hc; ++s) {
            const float* row = up_w + ((size_t)s * D + d) * rank;
            float u = 0.0f;
            for (int r = lane; r < rank; r += 32) u = fmaf(__ldg(row + r), mix1[m * rank + r], u);
            u = warp_sum(u);
            const size_t c = (size_t)s * D + d;
            const float xn = (load_val(hyper, f32, (size_t)m * N + c) * inv[m * hc + s]) * norm_w[c];
            acc += sigmoid(u) * xn;
        }
        if (lane == 0) mixed[(size_t)m * D + d] = acc * rhc;
    }
}

// out[m][s D + d] = hyper[m][s D + d] + branch[m][d] * inject[m][s]
__global__ void hc_reinject_kernel(const void* hyper, int h_f32, const void* branch, int b_f32,
                                   const float* __restrict__ inject, int M, int D, int hc, float* out) {
    const size_t n = (size_t)M * hc * D;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const size_t m = i / ((size_t)hc * D), c = i - m * hc * D;
        const int s = (int)(c / D), d = (int)(c - (size_t)s * D);
        out[i] = load_val(hyper, h_f32, i) + load_val(branch, b_f32, m * D + d) * inject[m * hc + s];
    }
}

}  // namespace

size_t hc_workspace_bytes(int M, int hc, int rank) {
    return (((size_t)M * hc * 4 + 255) & ~(size_t)255) + (size_t)M * (rank + hc) * 4;
}

// Tokens staged per pass of the down rows: up to kHcGroup, as shared memory allows.
int hc_group(int M, int hc, int D) {
    const int fit = (int)(kHcSmem / ((size_t)hc * D * 4));
    return max(1, min(min(M, kHcGroup), fit));
}
size_t hc_down_smem(int M, int hc, int D) { return (size_t)hc_group(M, hc, D) * hc * D * 4; }
size_t hc_up_smem(int M, int rank) { return (size_t)M * rank * 4; }

cudaError_t launch_hc_mix(const void* hyper, int f32, int M, int D, int hc, int rank, float eps,
                          const float* norm_w, const float* down_w, const float* up_w, const float* inject_w,
                          float* mixed, float* inject, unsigned char* ws, cudaStream_t s) {
    float* inv = reinterpret_cast<float*>(ws);
    float* t = reinterpret_cast<float*>(ws + (((size_t)M * hc * 4 + 255) & ~(size_t)255));
    hc_rms_kernel<<<(unsigned)(M * hc), 256, 0, s>>>(hyper, f32, D, hc, eps, inv);
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return err;
    const size_t dsm = hc_down_smem(M, hc, D);
    err = smem_opt_in(reinterpret_cast<const void*>(hc_down_kernel), (int)dsm);
    if (err != cudaSuccess) return err;
    hc_down_kernel<<<(unsigned)((rank + hc + kHcWarps - 1) / kHcWarps), kHcWarps * 32, dsm, s>>>(
        hyper, f32, M, D, hc, rank, hc_group(M, hc, D), norm_w, down_w, inject_w, inv, t);
    err = cudaGetLastError();
    if (err != cudaSuccess) return err;
    const size_t usm = hc_up_smem(M, rank);
    err = smem_opt_in(reinterpret_cast<const void*>(hc_up_kernel), (int)usm);
    if (err != cudaSuccess) return err;
    hc_up_kernel<<<(unsigned)((D + kHcWarps - 1) / kHcWarps), kHcWarps * 32, usm, s>>>(
        hyper, f32, M, D, hc, rank, norm_w, up_w, inv, t, mixed, inject);
    return cudaGetLastError();
}

cudaError_t launch_hc_reinject(const void* hyper, int h_f32, const void* branch, int b_f32, const float* inject,
                               int M, int D, int hc, float* out, cudaStream_t s) {
    const size_t n = (size_t)M * hc * D;
    const unsigned grid = (unsigned)min((n + 255) / 256, (size_t)device_sm_count() * 8);
    hc_reinject_kernel<<<grid, 256, 0, s>>>(hyper, h_f32, branch, b_f32, inject, M, D, hc, out);
    return cudaGetLastError();
}

}  // namespace qmoe
