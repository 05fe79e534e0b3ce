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

struct NoStamp {
    __device__ void operator()(int, unsigned long long = 0) const {}
};

// Order-preserving map of a float to an unsigned integer (for redux.sync max).
__device__ __forceinline__ unsigned topk_ord(float f) {
    const unsigned b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Top-k of E logits (E <= blockDim.x, E a multiple of the warp count, k <= 16)
// by the whole CTA in a fixed number of steps.  Same selection rule as
// warp_topk: unique keys (p bits << 32 | ~id) on p = exp(l - l_max).  Thread
// (warp w, lane l) holds expert l * nw + w, so every warp sees experts spread
// over the whole id range:
//   1. the block maximum of the logits;
//   2. each warp's largest key; T0 = the k-th largest of the nw warp maxima.
//      Every member of the top k is >= T0 (k distinct keys reach it);
//   3. keys >= T0 are the candidates: about k for distinct probabilities, and
//      still about k when many tie (each warp's maximum is then its lowest
//      tied id, so T0 is the k-th lowest tied id); each candidate is ranked
//      against all, up to 256 of them; beyond that (adversarial ties), k
//      rounds of block arg-max.
// `logit(i)` loads logit i (from L2: it is read once); `between()` runs while
// the loads are in flight.  Shared scratch: cand[256] u64, wmax[nw + 1] u64,
// red[nw] u32, cnt (int).  Writes tkv (p values, not normalised) and tki
// (ids), descending; returns l_max.  Every thread of the CTA must call it.
template <class LogitAt, class Between, class Stamp = NoStamp>
__device__ __forceinline__ float block_topk_threshold(LogitAt logit, int E, int k, unsigned long long* cand,
                                                      unsigned long long* wmax, unsigned* red, int* cnt, float* tkv,
                                                      int* tki, Between between, Stamp stamp = Stamp()) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    const int e = lane * nw + warp;
    float l = -INFINITY;
    if (e < E) l = logit(e);
    stamp(0, (unsigned long long)__float_as_uint(l));
    between();  // caller's work that overlaps the logit loads
    stamp(1, 0ull);
    if (l != l) l = -INFINITY;  // NaN ranks last
    const unsigned m = __reduce_max_sync(0xffffffffu, topk_ord(l));
    if (lane == 0) red[warp] = m;
    if (tid == 0) *cnt = 0;
    __syncthreads();
    unsigned mm = 0;
    for (int w = 0; w < nw; ++w) mm = max(mm, red[w]);
    const float lmax = __uint_as_float((mm & 0x80000000u) ? (mm & 0x7FFFFFFFu) : ~mm);
    const unsigned long long key =
        e < E ? ((unsigned long long)__float_as_uint(expf(l - lmax)) << 32) | (0xFFFFFFFFu - (unsigned)e) : 0ull;
    const unsigned kh = (unsigned)(key >> 32), kl = (unsigned)key;
    const unsigned mh = __reduce_max_sync(0xffffffffu, kh);
    const unsigned ml = __reduce_max_sync(0xffffffffu, kh == mh ? kl : 0u);
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
    stamp(2, T0);
    const bool is_c = e < E && key >= T0;
    const unsigned bal = __ballot_sync(0xffffffffu, is_c);
    int base = 0;
    if (lane == 0 && bal) base = atomicAdd(cnt, __popc(bal));
    base = __shfl_sync(0xffffffffu, base, 0);
    const int pos = base + __popc(bal & ((1u << lane) - 1u));
    if (is_c && pos < 256) cand[pos] = key;
    __syncthreads();
    const int C = *cnt;
    if (C <= 256) {
        for (int i = tid; i < C; i += blockDim.x) {
            const unsigned long long ci = cand[i];
            int r = 0;
            for (int j = 0; j < C; ++j) r += cand[j] > ci ? 1 : 0;
            if (r < k) {
                tkv[r] = __uint_as_float((unsigned)(ci >> 32));
                tki[r] = (int)(0xFFFFFFFFu - (unsigned)ci);
            }
        }
        __syncthreads();
        stamp(3, 0ull);
        return lmax;
    }
    // Adversarial ties: k rounds of block arg-max over the keys.
    unsigned long long mine = key;
    for (int r = 0; r < k; ++r) {
        const unsigned h = (unsigned)(mine >> 32), lo = (unsigned)mine;
        const unsigned wh = __reduce_max_sync(0xffffffffu, h);
        const unsigned wl = __reduce_max_sync(0xffffffffu, h == wh ? lo : 0u);
        if (lane == 0) cand[warp] = ((unsigned long long)wh << 32) | wl;
        __syncthreads();
        unsigned long long best = 0ull;
        for (int w = 0; w < nw; ++w) best = cand[w] > best ? cand[w] : best;
        if (tid == 0) {
            tkv[r] = __uint_as_float((unsigned)(best >> 32));
            tki[r] = (int)(0xFFFFFFFFu - (unsigned)best);
        }
        if (mine == best) mine = 0ull;
        __syncthreads();
    }
    return lmax;
}

}  // namespace qmoe
