// Warp-level top-k selection shared by the router kernel and the stack kernel.
#pragma once

#include "common.cuh"

namespace qmoe {

constexpr int kCandCap = 192;  // candidate slots per warp before the tie fallback

__device__ __forceinline__ bool topk_better(float a, int ia, float b, int ib) {
    return a > b || (a == b && ia < ib);
}

// Order-preserving map of a float to an unsigned integer (for redux.sync max).
__device__ __forceinline__ unsigned topk_ord(float f) {
    const unsigned b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
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
// `load(j)` gives this lane's logit lane + 32 j (j < E / 32 <= NPL); the
// per-lane values stay in registers.
template <int NPL, class Load>
__device__ __forceinline__ float warp_topk_fn(Load load, int E, int k, float* cv, int* ci, float* sv, int* si) {
    const int lane = threadIdx.x & 31;
    const int npl = E >> 5;
    float v[NPL];
    float lmax = -INFINITY;
    // Every load issued before any use (a load past npl re-reads the last
    // valid one and is never used).
#pragma unroll
    for (int j = 0; j < NPL; ++j) v[j] = load(j < npl ? j : npl - 1);
#pragma unroll
    for (int j = 0; j < NPL; ++j) {
        if (j < npl) {
            float t = v[j];
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
    for (int j = 0; j < NPL; ++j) {
        if (j < npl) {
            v[j] = expf(v[j] - lmax);
            if (topk_better(v[j], lane + 32 * j, bv, bi)) {
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
        rank += topk_better(ov, oi, bv, bi) ? 1 : 0;
    }
    const unsigned sel = __ballot_sync(0xffffffffu, rank == k - 1);
    const int src = __ffs(sel) - 1;
    const float tv = __shfl_sync(0xffffffffu, bv, src);
    const int ti = __shfl_sync(0xffffffffu, bi, src);

    int c = 0;
#pragma unroll
    for (int j = 0; j < NPL; ++j)
        if (j < npl && !topk_better(tv, ti, v[j], lane + 32 * j)) ++c;
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
        for (int j = 0; j < NPL; ++j) {
            if (j < npl && !topk_better(tv, ti, v[j], lane + 32 * j)) {
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
            for (int j = 0; j < total; ++j) r += topk_better(cv[j], ci[j], mv, mi) ? 1 : 0;
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
        for (int j = 0; j < NPL; ++j) {
            if (j < npl && !((taken >> j) & 1u) && topk_better(v[j], lane + 32 * j, lv, li)) {
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
            if (topk_better(ov, oi, wv, wi)) {
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

// The warp top-k of E fp32 logits in global memory (read through L2).
// (E <= 512: 16 per lane, the register arrays sized to fit.)
static __device__ __noinline__ float warp_topk(const float* __restrict__ logits, int E, int k, float* cv, int* ci,
                                               float* sv, int* si) {
    auto load = [&](int j) { return __ldcg(logits + (threadIdx.x & 31) + 32 * j); };
    if (E <= 512) return warp_topk_fn<16>(load, E, k, cv, ci, sv, si);
    return warp_topk_fn<32>(load, E, k, cv, ci, sv, si);
}


// Tie-admitting threshold routing for one token by one warp: the reference's
// device select in its non-exact mode (scripts/kernels/router_select.cpp:
// 223-255, the ttnn chain of tt/moe.py:308-327).  The softmax probabilities
// p_e (numerators exp(l_e - l_max) over their sum; each lane sums its ids in
// order, then a butterfly over the lanes), rounded to bf16 when probs_bf16;
// the threshold t is the k-th largest p counting equal values separately;
// total = the sum of every p_e >= t; then the k_sel largest positive p_e >= t
// with ids in [e_lo, e_hi), ties to the lower id, written as (id, p_e / total
// via the reciprocal) to ids/weights, the remaining slots as (e_lo, 0).
// E % 32 == 0, E <= 1024, k <= 16, k_sel <= 16.  Returns l_max.
static __device__ __noinline__ float warp_select_threshold(const float* __restrict__ lg, int E, int k, int k_sel,
                                                           int e_lo, int e_hi, int probs_bf16, int32_t* ids,
                                                           float* weights) {
    const int lane = threadIdx.x & 31;
    const int npl = E >> 5;
    float v[32];
    float lmax = -INFINITY;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        if (j < npl) {
            float t = __ldcg(lg + lane + 32 * j);
            if (t != t) t = -INFINITY;  // NaN ranks last
            v[j] = t;
            lmax = fmaxf(lmax, t);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, o));
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        if (j < npl) {
            v[j] = expf(v[j] - lmax);
            s += v[j];
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        if (j < npl) {
            float pj = v[j] / s;
            if (probs_bf16) pj = __bfloat162float(__float2bfloat16_rn(pj));
            v[j] = pj;
        }
    }
    // One round of warp arg-max (value, lowest id) over this lane's values
    // that `ok` admits and `taken` has not marked; marks the winner.
    auto argmax = [&](uint32_t& taken, auto ok, float& wv, int& wi) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            if (j < npl && !((taken >> j) & 1u) && ok(j) && topk_better(v[j], lane + 32 * j, bv, bi)) {
                bv = v[j];
                bi = lane + 32 * j;
            }
        }
        wv = bv;
        wi = bi;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, wv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, wi, o);
            if (topk_better(ov, oi, wv, wi)) {
                wv = ov;
                wi = oi;
            }
        }
        if (bi == wi && bi != 0x7fffffff) taken |= 1u << ((wi - lane) >> 5);
    };
    uint32_t taken = 0;
    float thr = 0.0f;
    for (int r = 0; r < k; ++r) {
        float wv;
        int wi;
        argmax(taken, [&](int) { return true; }, wv, wi);
        thr = wi != 0x7fffffff ? wv : 0.0f;
    }
    float tot = 0.0f;
#pragma unroll
    for (int j = 0; j < 32; ++j)
        if (j < npl && v[j] >= thr) tot += v[j];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
    const float inv = tot > 0.0f ? 1.0f / tot : 0.0f;
    taken = 0;
    for (int r = 0; r < k_sel; ++r) {
        float wv;
        int wi;
        argmax(
            taken,
            [&](int j) {
                const int id = lane + 32 * j;
                return id >= e_lo && id < e_hi && v[j] > 0.0f && v[j] >= thr;
            },
            wv, wi);
        if (lane == 0) {
            const bool got = wi != 0x7fffffff;
            ids[r] = got ? wi : e_lo;
            weights[r] = got ? wv * inv : 0.0f;
        }
    }
    __syncwarp();
    return lmax;
}

}  // namespace qmoe
