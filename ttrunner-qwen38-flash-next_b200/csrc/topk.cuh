// Warp-level top-k selection shared by the router kernel and the stack kernel.
#pragma once

#include "common.cuh"

namespace qmoe {

constexpr int kCandCap = 192;  // candidate slots per warp before the tie fallback

__device__ __forceinline__ bool topk_better(float a, int ia, float b, int ib) {
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
static __device__ __noinline__ float warp_topk(const float* __restrict__ logits, int E, int k, float* cv, int* ci,
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
    for (int j = 0; j < 32; ++j)
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
        for (int j = 0; j < 32; ++j) {
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
        for (int j = 0; j < 32; ++j) {
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

}  // namespace qmoe

namespace qmoe {

// Top-k of E <= 2 * blockDim.x logits by the whole CTA (k <= blockDim.x / 32),
// same selection rule as warp_topk: rank p_i = exp(l_i - l_max) descending,
// lower id on ties, via unique 64-bit keys (p bits << 32 | ~id).
//   1. block max of the logits (order-preserving integer keys, redux.sync);
//   2. each warp's largest key; T0 = the k-th largest warp maximum, which is
//      not above the k-th largest key overall (k distinct keys reach it);
//   3. keys >= T0 are the candidates (k..~2k for distinct logits, up to all
//      of them for a long run of ties), each ranked against all candidates.
// Results in tkv (p values) and tki (ids), descending.  Returns l_max.
// Scratch (shared): cand[max(E, nwarps * k)] u64, wmax[nwarps + 1] u64, red[nwarps] u32, cnt.
__device__ __forceinline__ unsigned topk_ord(float f) {
    const unsigned b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Top-k of E <= blockDim.x logits (E % 32 == 0, k <= 16) by the whole CTA in a
// fixed number of steps, whatever the ties: one logit per thread; the block
// maximum; unique keys (p bits << 32 | ~id) on p = exp(l - l_max); every warp
// ranks its 32 keys (shuffles) and keeps its k best in rank order; then each of
// the E/32 * k survivors counts the survivors of the other warps above it
// (broadcast reads) -- its global rank.  `logit(i)` gives logit i's address.
// Results: tkv (p values) and tki (ids), descending.  Returns l_max.
// Scratch (shared): cand[E/32 * k] u64, red[nwarps] u32.
template <class LogitAt>
__device__ __forceinline__ float block_topk_ranked(LogitAt logit, int E, int k, unsigned long long* cand,
                                                   unsigned* red, float* tkv, int* tki) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    float l = -INFINITY;
    if (tid < E) {
        l = __ldcg(logit(tid));
        if (l != l) l = -INFINITY;  // NaN ranks last
    }
    const unsigned m = __reduce_max_sync(0xffffffffu, topk_ord(l));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    unsigned mm = 0;
    for (int w = 0; w < nw; ++w) mm = max(mm, red[w]);
    const float lmax = __uint_as_float((mm & 0x80000000u) ? (mm & 0x7FFFFFFFu) : ~mm);
    const unsigned long long key =
        tid < E ? ((unsigned long long)__float_as_uint(expf(l - lmax)) << 32) | (0xFFFFFFFFu - (unsigned)tid) : 0ull;
    const unsigned kh = (unsigned)(key >> 32), kl = (unsigned)key;
    int rank = 0;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        const unsigned oh = __shfl_sync(0xffffffffu, kh, j), ol = __shfl_sync(0xffffffffu, kl, j);
        rank += (oh > kh || (oh == kh && ol > kl)) ? 1 : 0;
    }
    const int nl = E >> 5;  // lists: one per warp holding logits
    if (warp < nl && rank < k) cand[warp * k + rank] = key;
    __syncthreads();
    const int nc = nl * k;
    for (int i = tid; i < nc; i += blockDim.x) {
        const unsigned long long c = cand[i];
        const int w = i / k;
        int r = i - w * k;
        for (int w2 = 0; w2 < nl; ++w2) {
            if (w2 == w) continue;
            const unsigned long long* L = cand + w2 * k;
            for (int j = 0; j < k; ++j) r += L[j] > c ? 1 : 0;
        }
        if (r < k) {
            tkv[r] = __uint_as_float((unsigned)(c >> 32));
            tki[r] = (int)(0xFFFFFFFFu - (unsigned)c);
        }
    }
    __syncthreads();
    return lmax;
}

static __device__ __noinline__ float block_topk(const float* __restrict__ logits, int E, int k,
                                                unsigned long long* cand, unsigned long long* wmax,
                                                unsigned* red, int* cnt, float* tkv, int* tki) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nt = blockDim.x, nw = nt >> 5;
    float l0 = -INFINITY, l1 = -INFINITY;
    if (tid < E) {
        l0 = __ldcg(logits + tid);
        if (l0 != l0) l0 = -INFINITY;
    }
    if (tid + nt < E) {
        l1 = __ldcg(logits + tid + nt);
        if (l1 != l1) l1 = -INFINITY;
    }
    unsigned m = __reduce_max_sync(0xffffffffu, max(topk_ord(l0), topk_ord(l1)));
    if (lane == 0) red[warp] = m;
    if (tid == 0) *cnt = 0;
    __syncthreads();
    unsigned mm = 0;
    for (int w = 0; w < nw; ++w) mm = max(mm, red[w]);
    const float lmax = __uint_as_float((mm & 0x80000000u) ? (mm & 0x7FFFFFFFu) : ~mm);
    const int i0 = tid, i1 = tid + nt;
    const unsigned long long k0 =
        i0 < E ? ((unsigned long long)__float_as_uint(expf(l0 - lmax)) << 32) | (0xFFFFFFFFu - (unsigned)i0) : 0ull;
    const unsigned long long k1 =
        i1 < E ? ((unsigned long long)__float_as_uint(expf(l1 - lmax)) << 32) | (0xFFFFFFFFu - (unsigned)i1) : 0ull;
    const unsigned long long best = k0 > k1 ? k0 : k1;
    const unsigned hi = (unsigned)(best >> 32), lo = (unsigned)best;
    const unsigned mh = __reduce_max_sync(0xffffffffu, hi);
    const unsigned ml = __reduce_max_sync(0xffffffffu, hi == mh ? lo : 0u);
    if (lane == 0) wmax[warp] = ((unsigned long long)mh << 32) | ml;
    __syncthreads();
    if (tid < nw) {
        const unsigned long long v = wmax[tid];
        int r = 0;
        for (int w = 0; w < nw; ++w) r += wmax[w] > v ? 1 : 0;
        if (r == k - 1) wmax[nw] = v;
    }
    __syncthreads();
    const unsigned long long T0 = wmax[nw];
    if (i0 < E && k0 >= T0) cand[atomicAdd(cnt, 1)] = k0;
    if (i1 < E && k1 >= T0) cand[atomicAdd(cnt, 1)] = k1;
    __syncthreads();
    const int C = *cnt;
    if (C <= 64) {
        for (int c = tid; c < C; c += nt) {
            const unsigned long long v = cand[c];
            int r = 0;
            for (int j = 0; j < C; ++j) r += cand[j] > v ? 1 : 0;
            if (r < k) {
                tkv[r] = __uint_as_float((unsigned)(v >> 32));
                tki[r] = (int)(0xFFFFFFFFu - (unsigned)v);
            }
        }
        __syncthreads();
        return lmax;
    }
    // Many candidates: a long run of equal probabilities (activations small
    // enough that exp rounds them together).  Each warp extracts its own top
    // k by k rounds of warp arg-max (no block barrier), then warp 0 merges the
    // nw * k survivors the same way -- cost independent of the ties.
    unsigned long long a0 = i0 < E ? k0 : 0ull, a1 = i1 < E ? k1 : 0ull;
    for (int r = 0; r < k; ++r) {
        const unsigned long long b = a0 > a1 ? a0 : a1;
        const unsigned bh = (unsigned)(b >> 32), bl = (unsigned)b;
        const unsigned wh = __reduce_max_sync(0xffffffffu, bh);
        const unsigned wl = __reduce_max_sync(0xffffffffu, bh == wh ? bl : 0u);
        const unsigned long long m = ((unsigned long long)wh << 32) | wl;
        if (lane == 0) cand[warp * k + r] = m;
        if (a0 == m) a0 = 0ull;
        if (a1 == m) a1 = 0ull;
    }
    __syncthreads();
    if (warp == 0) {
        const int n = nw * k;  // <= 16 * 16 = 256: up to 8 per lane
        unsigned long long c[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) c[j] = (lane + 32 * j) < n ? cand[lane + 32 * j] : 0ull;
        for (int r = 0; r < k; ++r) {
            unsigned long long b = 0ull;
#pragma unroll
            for (int j = 0; j < 8; ++j) b = c[j] > b ? c[j] : b;
            const unsigned bh = (unsigned)(b >> 32), bl = (unsigned)b;
            const unsigned wh = __reduce_max_sync(0xffffffffu, bh);
            const unsigned wl = __reduce_max_sync(0xffffffffu, bh == wh ? bl : 0u);
            const unsigned long long m = ((unsigned long long)wh << 32) | wl;
            if (lane == 0) {
                tkv[r] = __uint_as_float(wh);
                tki[r] = (int)(0xFFFFFFFFu - wl);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (c[j] == m) c[j] = 0ull;
        }
    }
    __syncthreads();
    return lmax;
}

}  // namespace qmoe
