// Router GEMV, top-k selection and renormalisation in one launch.
//
// Behaviour follows reference/model.py:399-403: logits = x . W_r^T in fp32,
// softmax, top-k, weights divided by their sum.  The global softmax
// denominator is common to every expert, so ranking and renormalising use the
// numerators exp(l_i - l_max) alone: w_i = p_i / sum_topk p_j.  Ties go to the lower expert id, the
// rule of scripts/kernels/router_select.cpp:163-164 (EXACT_TOPK mode).
//
// Layout: every warp owns one router row (512 rows + the shared-expert gate
// vector as row E), reads it once with 128-bit loads and dots it with all M
// tokens held in shared memory.  The last CTA to finish (arrival counter)
// runs the selection, so no second launch and no host round trip.
#include <math.h>

#include "common.cuh"

namespace qmoe {
namespace {

constexpr int kRouteWarps = 4;
constexpr int kCandCap = 192;  // candidate slots per warp before the tie fallback

__device__ __forceinline__ bool better(float a, int ia, float b, int ib) {
    return a > b || (a == b && ia < ib);
}

// Top-k of E logits (E % 32 == 0, E <= 1024, k <= 16) for one token, by one
// warp.  Selection is on p_i = exp(l_i - l_max), the softmax numerators: the
// reference ranks fp32 softmax probabilities (reference/model.py:400-401),
// so logits closer together than fp32 resolves after exp must tie there too
// (they do when activations are tiny), and ties go to the lower id.  Writes
// the k (p, id) pairs in descending order to sv/si; returns l_max.
//
// Every element of the top k is at least as good as T0, the k-th best of the
// 32 per-lane maxima (those k maxima are k distinct elements not worse than
// T0), so only elements not worse than T0 are ranked.  With distinct values
// that is typically k to 2k candidates; a run of ties larger than the
// candidate buffer falls back to k rounds of warp arg-max.
__device__ float warp_topk(const float* __restrict__ logits, int E, int k, float* cv, int* ci,
                           float* sv, int* si) {
    const int lane = threadIdx.x & 31;
    const int npl = E >> 5;
    float v[32];
    float lmax = -INFINITY;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        if (j < npl) {
            float t = __ldcg(logits + lane + 32 * j);
            if (t != t) t = -INFINITY;  // NaN ranks last
            v[j] = t;
            lmax = fmaxf(lmax, t);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, o));
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        if (j < npl) {
            v[j] = expf(v[j] - lmax);
            if (better(v[j], lane + 32 * j, bv, bi)) {
                bv = v[j];
                bi = lane + 32 * j;
            }
        }
    }
    int rank = 0;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        const float ov = __shfl_sync(0xffffffffu, bv, j);
        const int oi = __shfl_sync(0xffffffffu, bi, j);
        rank += better(ov, oi, bv, bi) ? 1 : 0;
    }
    const unsigned sel = __ballot_sync(0xffffffffu, rank == k - 1);
    const int src = __ffs(sel) - 1;
    const float tv = __shfl_sync(0xffffffffu, bv, src);
    const int ti = __shfl_sync(0xffffffffu, bi, src);

    int c = 0;
#pragma unroll
    for (int j = 0; j < 32; ++j)
        if (j < npl && !better(tv, ti, v[j], lane + 32 * j)) ++c;
    int incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    const int total = __shfl_sync(0xffffffffu, incl, 31);

    if (total <= kCandCap) {
        int pos = incl - c;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            if (j < npl && !better(tv, ti, v[j], lane + 32 * j)) {
                cv[pos] = v[j];
                ci[pos] = lane + 32 * j;
                ++pos;
            }
        }
        __syncwarp();
        for (int cc = lane; cc < total; cc += 32) {
            const float mv = cv[cc];
            const int mi = ci[cc];
            int r = 0;
            for (int j = 0; j < total; ++j) r += better(cv[j], ci[j], mv, mi) ? 1 : 0;
            if (r < k) {
                sv[r] = mv;
                si[r] = mi;
            }
        }
        __syncwarp();
        return lmax;
    }

    // Fallback for long runs of equal values: k rounds of warp arg-max.
    uint32_t taken = 0;
    for (int r = 0; r < k; ++r) {
        float lv = -INFINITY;
        int li = 0x7fffffff;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            if (j < npl && !((taken >> j) & 1u) && better(v[j], lane + 32 * j, lv, li)) {
                lv = v[j];
                li = lane + 32 * j;
            }
        }
        float wv = lv;
        int wi = li;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, wv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, wi, o);
            if (better(ov, oi, wv, wi)) {
                wv = ov;
                wi = oi;
            }
        }
        if (lane == 0) {
            sv[r] = wv;
            si[r] = wi;
        }
        if (li == wi && li != 0x7fffffff) taken |= 1u << ((wi - lane) >> 5);
    }
    __syncwarp();
    return lmax;
}

template <int MAXM>
__global__ void __launch_bounds__(kRouteWarps * 32) route_kernel(RouteArgs a) {
    extern __shared__ __align__(16) float xs[];  // [M][D]
    __shared__ float s_cv[kRouteWarps][kCandCap];
    __shared__ int s_ci[kRouteWarps][kCandCap];
    __shared__ float s_sv[kRouteWarps][kMaxTopK];
    __shared__ int s_si[kRouteWarps][kMaxTopK];
    __shared__ unsigned int s_last;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int M = a.M, D = a.D, E = a.E;
    for (int i = tid; i < M * D; i += blockDim.x) xs[i] = load_act(a.x, a.x_f32, (size_t)i);
    __syncthreads();

    const int rows = E + (a.gate_vec ? 1 : 0);
    const int row = blockIdx.x * kRouteWarps + warp;
    if (row < rows) {
        const float* w = row < E ? a.router + (size_t)row * D : a.gate_vec;
        float acc[MAXM];
#pragma unroll
        for (int m = 0; m < MAXM; ++m) acc[m] = 0.0f;
        // 16 independent 128-bit loads in flight per lane before any use.
        for (int c0 = 0; c0 < D; c0 += 16 * 128) {
            float4 wv[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int c = c0 + i * 128 + lane * 4;
                wv[i] = c < D ? __ldg(reinterpret_cast<const float4*>(w + c)) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int c = c0 + i * 128 + lane * 4;
                if (c >= D) break;
#pragma unroll
                for (int m = 0; m < MAXM; ++m) {
                    if (m < M) {
                        const float4 xv = *reinterpret_cast<const float4*>(xs + m * D + c);
                        acc[m] = fmaf(wv[i].x, xv.x, acc[m]);
                        acc[m] = fmaf(wv[i].y, xv.y, acc[m]);
                        acc[m] = fmaf(wv[i].z, xv.z, acc[m]);
                        acc[m] = fmaf(wv[i].w, xv.w, acc[m]);
                    }
                }
            }
        }
#pragma unroll
        for (int m = 0; m < MAXM; ++m) {
            if (m < M) {
                const float s = warp_sum(acc[m]);
                if (lane == 0) a.logits[(size_t)m * (E + 1) + row] = s;
            }
        }
    }

    // Last CTA to arrive selects.
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const unsigned prev = atomicAdd(a.counter, 1u);
        s_last = (prev == gridDim.x - 1) ? 1u : 0u;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();

    for (int m = warp; m < M; m += kRouteWarps) {
        const float* lg = a.logits + (size_t)m * (E + 1);
        if (E == 0) {  // gate-vector row only (standalone shared expert)
            if (lane == 0 && a.shared_logit) a.shared_logit[m] = __ldcg(lg);
            continue;
        }
        const float lmax = warp_topk(lg, E, a.k, s_cv[warp], s_ci[warp], s_sv[warp], s_si[warp]);
        const float e = lane < a.k ? s_sv[warp][lane] : 0.0f;
        const float sum = warp_sum(e);
        if (lane < a.k) {
            if (!(fabsf(lmax) <= 3.0e38f)) record_status(a.status, QMOE_ERR_NOT_FINITE);
            a.ids[m * a.k + lane] = s_si[warp][lane];
            a.weights[m * a.k + lane] = e / sum;
        }
        if (lane == 0 && a.shared_logit) {
            a.shared_logit[m] = a.gate_vec ? __ldcg(lg + E) : 0.0f;
        }
        __syncwarp();
    }
    __syncthreads();
    if (tid == 0) *a.counter = 0u;  // ready for the next launch / graph replay
}

template <int MAXM>
cudaError_t launch_route_t(const RouteArgs& a, cudaStream_t s) {
    const int rows = a.E + (a.gate_vec ? 1 : 0);
    const unsigned grid = (unsigned)((rows + kRouteWarps - 1) / kRouteWarps);
    const size_t smem = (size_t)a.M * a.D * sizeof(float);
    cudaError_t err = cudaFuncSetAttribute(route_kernel<MAXM>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess) return err;
    route_kernel<MAXM><<<grid, kRouteWarps * 32, smem, s>>>(a);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_route(const RouteArgs& a, cudaStream_t s) {
    if (a.M <= 1) return launch_route_t<1>(a, s);
    if (a.M <= 4) return launch_route_t<4>(a, s);
    if (a.M <= 8) return launch_route_t<8>(a, s);
    return launch_route_t<16>(a, s);
}

}  // namespace qmoe
