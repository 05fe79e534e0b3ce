// Router GEMV, top-k selection and renormalisation in one launch.
//
// Behaviour follows reference/model.py:399-403: logits = x . W_r^T in fp32,
// softmax, top-k, weights divided by their sum.  The global softmax
// denominator is common to every expert, so ranking and renormalising use the
// numerators exp(l_i - l_max) alone: w_i = p_i / sum_topk p_j.  Ties go to the lower expert id, the
// rule of scripts/kernels/router_select.cpp:163-164 (EXACT_TOPK mode).  The
// same launch also runs that select's tie-admitting threshold mode
// (router_select.cpp:223-255; warp_select_threshold in topk.cuh).
//
// Layout: every warp owns one router row (512 rows + the shared-expert gate
// vector as row E), reads it once with 128-bit loads and dots it with all M
// tokens held in shared memory.  The last CTA to finish (arrival counter)
// runs the selection, so no second launch and no host round trip.
#include <math.h>

#include "common.cuh"
#include "topk.cuh"

namespace qmoe {
namespace {

// kRouteWarps warps per CTA: one router row each, then one token each in the
// selecting CTA (4 for up to 4 tokens, else one per token).
template <int MAXM, int kRouteWarps>
__global__ void __launch_bounds__(kRouteWarps * 32) route_kernel(RouteArgs a) {
    extern __shared__ __align__(16) float xs[];  // [M][D]
    __shared__ __align__(16) float s_cv[kRouteWarps][kCandCap];
    __shared__ int s_ci[kRouteWarps][kCandCap];
    __shared__ float s_sv[kRouteWarps][kMaxTopK];
    __shared__ int s_si[kRouteWarps][kMaxTopK];
    __shared__ unsigned int s_last;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int M = a.M, D = a.D, E = a.E;
    stage_act(xs, a.x, a.x_f32, M * D);
    __syncthreads();
    if (a.xconv) {
        // x in block floating point for the gate|up kernel, a warp per
        // 32-value block over the grid (block b = token b / (D/32)).
        const int nb = M * (D >> 5);
        float* xsf = reinterpret_cast<float*>(a.xconv + (size_t)nb * 16);
        for (int b = blockIdx.x * kRouteWarps + warp; b < nb; b += gridDim.x * kRouteWarps) {
            float st;
            const int pw = warp_block_fp(xs[b * 32 + lane], &st);
            if (lane < 16) a.xconv[b * 16 + lane] = pw;
            if (lane == 0) xsf[b] = st;
        }
    }

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

    if (MAXM == 1 && M == 1 && !a.thr_mode && E > 0 && E % (32 * kRouteWarps) == 0 &&
        E / (32 * kRouteWarps) <= 8) {
        // One token: the CTA's warps share it.  Warp w ranks ids w*E/W ..,
        // keys (p bits << 32 | ~id) with p = exp(l - l_max); each warp's k-th
        // best lane maximum is a lower bound of the top k (k distinct keys
        // reach it), so the largest of those bounds, T0, is one too, and only
        // keys >= T0 (about k to 2k) are ranked: ties go to the lower id as
        // in warp_topk.
        __shared__ float s_mx[kRouteWarps];
        __shared__ unsigned long long s_t[kRouteWarps];
        __shared__ int s_n;
        const int npl = E / (32 * kRouteWarps);
        const int id0 = warp * 32 * npl + lane;
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = __ldcg(a.logits + id0 + 32 * (j < npl ? j : npl - 1));
        float mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if (j < npl) {
                if (v[j] != v[j]) v[j] = -INFINITY;  // NaN ranks last
                mx = fmaxf(mx, v[j]);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) s_mx[warp] = mx;
        if (tid == 0) s_n = 0;
        __syncthreads();
        float lmax = s_mx[0];
#pragma unroll
        for (int w = 1; w < kRouteWarps; ++w) lmax = fmaxf(lmax, s_mx[w]);
        unsigned long long key[8], best = 0ull;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            key[j] = 0ull;
            if (j < npl) {
                const unsigned id = (unsigned)(id0 + 32 * j);
                key[j] = ((unsigned long long)__float_as_uint(expf(v[j] - lmax)) << 32) | (0xFFFFFFFFu - id);
                best = key[j] > best ? key[j] : best;
            }
        }
        int gt = 0;
#pragma unroll
        for (int i = 0; i < 32; ++i) gt += __shfl_sync(0xffffffffu, best, i) > best ? 1 : 0;
        const unsigned selb = __ballot_sync(0xffffffffu, gt == a.k - 1);
        const unsigned long long tw = __shfl_sync(0xffffffffu, best, __ffs(selb) - 1);
        if (lane == 0) s_t[warp] = tw;
        __syncthreads();
        unsigned long long t0 = s_t[0];
#pragma unroll
        for (int w = 1; w < kRouteWarps; ++w) t0 = s_t[w] > t0 ? s_t[w] : t0;
        unsigned long long* cand = reinterpret_cast<unsigned long long*>(&s_cv[0][0]);
        constexpr int kCap = kRouteWarps * kCandCap / 2;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if (j < npl && key[j] >= t0) {
                const int pos = atomicAdd(&s_n, 1);
                if (pos < kCap) cand[pos] = key[j];
            }
        }
        __syncthreads();
        const int n = s_n;
        if (warp == 0) {
            float lm = lmax;
            if (n <= kCap) {
                for (int c = lane; c < n; c += 32) {
                    const unsigned long long ck = cand[c];
                    int r = 0;
                    for (int j = 0; j < n; ++j) r += cand[j] > ck ? 1 : 0;
                    if (r < a.k) {
                        s_sv[0][r] = __uint_as_float((unsigned)(ck >> 32));
                        s_si[0][r] = (int)(0xFFFFFFFFu - (unsigned)ck);
                    }
                }
                __syncwarp();
            } else {  // long runs of ties: the one-warp selection
                lm = warp_topk(a.logits, E, a.k, s_cv[0], s_ci[0], s_sv[0], s_si[0]);
            }
            const float e = lane < a.k ? s_sv[0][lane] : 0.0f;
            const float sum = warp_sum(e);
            if (lane < a.k) {
                if (!(fabsf(lm) <= 3.0e38f)) record_status(a.status, QMOE_ERR_NOT_FINITE);
                a.ids[lane] = s_si[0][lane];
                a.weights[lane] = e / sum;
            }
            if (lane == 0 && a.shared_logit) a.shared_logit[0] = a.gate_vec ? __ldcg(a.logits + E) : 0.0f;
        }
        __syncthreads();
        if (tid == 0) *a.counter = 0u;
        return;
    }

    for (int m = warp; m < M; m += kRouteWarps) {
        const float* lg = a.logits + (size_t)m * (E + 1);
        if (E == 0) {  // gate-vector row only (standalone shared expert)
            if (lane == 0 && a.shared_logit) a.shared_logit[m] = __ldcg(lg);
            continue;
        }
        if (a.thr_mode) {
            const float lmax = warp_select_threshold(lg, E, a.thr_k, a.k, a.e_lo, a.e_hi, a.thr_mode == 2,
                                                     a.ids + m * a.k, a.weights + m * a.k);
            if (lane == 0) {
                if (!(fabsf(lmax) <= 3.0e38f)) record_status(a.status, QMOE_ERR_NOT_FINITE);
                if (a.shared_logit) a.shared_logit[m] = a.gate_vec ? __ldcg(lg + E) : 0.0f;
            }
            __syncwarp();
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
    constexpr int kRouteWarps = MAXM < 4 ? 4 : MAXM;
    const int rows = a.E + (a.gate_vec ? 1 : 0);
    const unsigned grid = (unsigned)((rows + kRouteWarps - 1) / kRouteWarps);
    const size_t smem = (size_t)a.M * a.D * sizeof(float);
    cudaError_t err = smem_opt_in(reinterpret_cast<const void*>(route_kernel<MAXM, kRouteWarps>), (int)smem);
    if (err != cudaSuccess) return err;
    route_kernel<MAXM, kRouteWarps><<<grid, kRouteWarps * 32, smem, s>>>(a);
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
