// The whole batch-1 MoE decode stack in one persistent launch.
//
// One CTA per SM (cooperative launch, so all CTAs are co-resident), looping
// over the layers.  Every layer is the reference's `_moe` (reference/model.py
// :387-417) in two phases separated by grid barriers:
//
//   B  every CTA ranks the E router logits (block top-k, lower id on ties);
//      warps 0 and 1 start bulk copies (cp.async.bulk, mbarrier completion)
//      of only this CTA's slice of the selected experts' gate|up rows and
//      down rows while x converts to block floating point; all warps decode
//      the shared expert's rows of the slice (prefetched), then the routed
//      gate|up rows as their chunks land -> h slice.
//   C  while the next layer's shared rows and router columns stream in (HBM
//      is otherwise idle here): the full h (k + 1 slots) -> block floating
//      point; this CTA's output rows of every selected expert's down (resident
//      since phase B) and of the shared expert, a warp per row ->
//      out[j] = sum_s w_s D_s[j].h_s + sigmoid(g.x) D_sh[j].h_sh; then the NEXT
//      layer's router logits restricted to these rows, sum_j R[e][j] x[j] over
//      this CTA's j, added into a logit accumulator with atomics.
//
// The barrier after C therefore publishes both the next layer's input and
// its complete router logits: two grid barriers per layer.  A prologue
// computes layer 0's logits the same way.
//
// Sharded over R ranks (one process and one GPU each; the reference's
// split of every expert's intermediate rows, tt/plan.py:70-103), each rank
// runs this kernel on its slice of every expert (I / R gate|up row pairs and
// the matching down columns) and its phase-C rows are partial sums.  The
// reduction over ranks happens inside the kernel: CTA c sends its partial
// rows to CTA c of every peer as 8-byte words (value bits, flag) stored
// straight into the peer's memory over NVLink, each word its own completion
// signal, and sums the R partials of its rows in rank order once the peers'
// words are in.  Every rank then holds bitwise the same next-layer input, and
// computes the router partials from it as on one GPU; on R > 1 ranks the
// logits accumulate in fp64, where a sum of fp32 partials is exact unless
// their magnitudes span more than 2^21, so every rank ranks the same logits
// and selects the same experts.  On one rank the accumulation is fp32 and
// its last bits depend on arrival order (selection reads it only after the
// barrier).
//
// Activations between layers are fp32 rounded to bf16 where they are read
// (bf16 activations, fp32 accumulation).  All waits are bounded in time
// (%globaltimer): a grid barrier, copy or exchange that does not complete
// sets QMOE_ERR_TIMEOUT and an abort word; every CTA waits (bounded) for its
// own copies in flight and returns.  No trap, no unbounded spin.
#include <cuda.h>  // CUtensorMap

#include "common.cuh"
#include "ptx.cuh"
#include "tma_host.cuh"
#include "topk.cuh"

namespace qmoe {
namespace {

constexpr int kSKWarps = 16;
constexpr int kSKThreads = kSKWarps * 32;
constexpr unsigned long long kTimeoutNs = 200ull * 1000 * 1000;
// A peer rank's rows may arrive late by as much as the ranks' launch skew.
constexpr unsigned long long kXchgTimeoutNs = 4000ull * 1000 * 1000;
constexpr int kSKChunk = 8;      // routed row pairs per gate|up bulk-copy chunk
constexpr int kSKMaxChunks = 6;  // chunks of a CTA's pairs (<= 40 pairs per CTA)
constexpr int kRColW = 20;      // router columns per tensor-copy box (80 B): covers 16 from a 16-byte-aligned start
constexpr int kRBoxRows = 256;  // router rows per tensor-copy box

struct SKLayer {
    const float* router;
    const float* gate_vec;
    const uint8_t* gate_up;
    const uint8_t* down;
    const uint8_t* sh_gate_up;
    const uint8_t* sh_down;
};

}  // namespace

constexpr int kSKMaxLayers = 64;

struct SKArgs {
    // In-kernel exchange over R ranks (R == 1: none).  xr[q]: rank q's receive
    // words [2 parities][R][D] as mapped in this process (xr[rank] local);
    // epoch: this rank's count of completed launches, which makes every
    // exchange's flag value new.
    int R, rank;
    int ib0;                              // first sub-block of a down row's slice inside its super-block
    unsigned long long* xr[kMaxXchgRanks];
    unsigned* epoch;
    const __nv_bfloat16* x;  // [D] layer-0 input
    float* out;              // [D] last layer's output
    __nv_bfloat16* act;      // [D] layer activation, bf16 (workspace)
    unsigned* hmax;          // two buffers of per-block max |h| bits (workspace)
    float* logits;           // two accumulators of G lines x 32 floats (logits 4g..4g+3 at a line's front)
    float* h;                // [(K + 1) * I] (workspace)
    unsigned* sync;          // 8 counters, 128 B apart, then the abort word
    unsigned long long* trace;  // [2][64][kTraceSlots] phase stamps of CTA 0 and the last CTA, or null
    __nv_bfloat16* act_trace;      // [n_layers][D]: every layer's output rounded to bf16, or null
    int* ids_trace;                // [n_layers][K]: the selected ids in rank order, or null
    float* w_trace;                // [n_layers][K]: their renormalised weights, or null
    const __nv_bfloat16* teacher;  // [n_layers][D]: layer L's input in place of layer L-1's output, or null
    int* status;
    int n_layers, D, I, E, K;
    SKLayer L[kSKMaxLayers];
    // Per layer: the router [E][D] and the gate vector [1][D] as 2-D tensors
    // for TMA copies of this CTA's column slice (boxes of kRColW columns).
    CUtensorMap rmap[kSKMaxLayers];
    CUtensorMap gmap[kSKMaxLayers];
};

// Shared-memory carve-up (byte offsets), a function of the shape and grid.
struct SKLayout {
    int NSQ, NP, NJ, NJR, RJ;
    unsigned xq, xs, rcol, xo, sgu, sdn, gbuf, ubuf, dbuf, hq, hs, gv, uv, sgv, suv, cand, wmax, red, tkv, tki, misc, bars,
        total;
};

__host__ __device__ constexpr unsigned sk_take(unsigned& o, unsigned bytes) {
    const unsigned r = o;
    o = (o + bytes + 127u) & ~127u;
    return r;
}

// Bytes of a down row of I values: whole super-blocks, or (a rank's slice of
// fewer than 256 columns) the super-block's 8-byte header then the slice's
// I / 32 16-byte code groups.
__host__ __device__ constexpr int sk_down_row_bytes(int I) { return I >= 256 ? (I / 256) * 136 : 8 + 16 * (I / 32); }

__host__ __device__ constexpr SKLayout sk_layout(int D, int I, int E, int K, int n) {
    SKLayout s{};
    const unsigned RB = (unsigned)(D / 256) * 136, DRB = (unsigned)sk_down_row_bytes(I);
    const unsigned NSB = D / 32, NSBH = I / 32;
    s.NSQ = (I + n - 1) / n;
    s.NP = (K * I + n - 1) / n;
    s.NJ = (D + n - 1) / n;
    // Down rows whose size is not a multiple of 16 bytes are copied in pairs
    // from an even row, so that every bulk copy starts 16-byte aligned: up
    // to two extra rows per slot, and an even row count keeps slots aligned.
    s.NJR = DRB % 16 ? (s.NJ + 3) & ~1 : s.NJ;
    s.RJ = kRColW;  // the tensor-copy box's row pitch
    unsigned o = 0;
    s.xq = sk_take(o, NSB * 64);
    s.xs = sk_take(o, NSB * 4);
    s.rcol = sk_take(o, (unsigned)(((E + kRBoxRows - 1) / kRBoxRows) * kRBoxRows + 1) * kRColW * 4);
    s.xo = sk_take(o, (unsigned)(s.NJ > kRColW ? s.NJ : kRColW) * 4);  // the router-column window's x
    s.sgu = sk_take(o, 2u * s.NSQ * RB);
    s.sdn = sk_take(o, (unsigned)s.NJR * DRB);
    s.gbuf = sk_take(o, (unsigned)s.NP * RB);
    s.ubuf = sk_take(o, (unsigned)s.NP * RB);
    s.dbuf = sk_take(o, (unsigned)K * s.NJR * DRB);
    s.hq = sk_take(o, (unsigned)(K + 1) * NSBH * 64);
    s.hs = sk_take(o, (unsigned)(K + 1) * NSBH * 4);
    s.gv = sk_take(o, s.NP * 4);
    s.uv = sk_take(o, s.NP * 4);
    s.sgv = sk_take(o, s.NSQ * 4);
    s.suv = sk_take(o, s.NSQ * 4);
    s.cand = sk_take(o, 256 * 8);
    s.wmax = sk_take(o, (kSKWarps + 1) * 8);
    s.red = sk_take(o, kSKWarps * 4);
    s.tkv = sk_take(o, kMaxTopK * 4);
    s.tki = sk_take(o, kMaxTopK * 4);
    s.misc = sk_take(o, 64);
    s.bars = sk_take(o, (4 + kSKMaxChunks) * 8);
    s.total = o;
    return s;
}

// The shapes the single launch is built for: everything that sizes or
// places data is a compile-time constant, so the layer loop keeps only its
// data in registers.  I is the intermediate width this rank holds: 512 (the
// BASELINE family) unsharded, 512 / R on each of R ranks.
template <int D_, int E_, int K_, int NSM_, int I_ = 512>
struct SKShape {
    static constexpr int D = D_, E = E_, K = K_, NSM = NSM_, I = I_;
    static constexpr int DRB = sk_down_row_bytes(I_);
    static constexpr bool kPairRows = DRB % 16 != 0;
    static constexpr SKLayout S = sk_layout(D_, I_, E_, K_, NSM_);
    static_assert(E_ <= kSKThreads && E_ % 32 == 0, "one router row per thread");
    static_assert(I_ % 32 == 0 && I_ <= 512 && (I_ >= 256 ? I_ % 256 == 0 : 256 % I_ == 0), "intermediate slice");
    static_assert((K_ + 1) * (I_ / 32) <= kStackHmaxBlocks, "block maxima of h");
    static_assert(K_ * I_ / NSM_ + 1 <= I_, "a CTA's routed rows span at most two experts");
    static_assert((K_ * I_ + NSM_ - 1) / NSM_ <= kSKChunk * (kSKMaxChunks - 1), "chunks of a CTA's pairs");
    static_assert((D_ + NSM_ - 1) / NSM_ + 3 <= kRColW, "router column slice: one box per CTA");
    static_assert(D_ % 2 == 0, "down rows copied in pairs");
};

namespace {

using ptx::mbar_expect_tx;
using ptx::mbar_init;
using ptx::mbar_test;
using ptx::now_ns;

// Bounded wait for the phase of `bar` with parity `par`; false on timeout.
__device__ bool mbar_wait(uint64_t* bar, uint32_t par) {
    if (mbar_test(bar, par)) return true;
    const unsigned long long t0 = now_ns();
    while (!ptx::mbar_test_sleep(bar, par, 20000u)) {
        if (now_ns() - t0 > kTimeoutNs) return false;
    }
    return true;
}

__device__ __forceinline__ unsigned* abort_word(unsigned* sync) { return sync + 8 * 32; }

// Phase trace: thread `rec` (0 unless stated) of CTA 0 and of the last CTA
// stamp their SM's cycle counter (clock64) at each phase boundary.
__device__ __forceinline__ void trace_mark(const SKArgs& a, int L, int k, int rec = 0) {
    if (a.trace && (int)threadIdx.x == rec) {
        if (blockIdx.x == 0) a.trace[L * kTraceSlots + k] = (unsigned long long)clock64();
        else if (blockIdx.x == gridDim.x - 1) a.trace[(64 + L) * kTraceSlots + k] = (unsigned long long)clock64();
    }
}

// trace_mark taken only once `dep` has been computed (the clock read consumes it).
__device__ __forceinline__ void trace_mark_after(const SKArgs& a, int L, int k, unsigned long long dep) {
    if (a.trace && threadIdx.x == 0 && (blockIdx.x == 0 || blockIdx.x == gridDim.x - 1)) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%clock64;" : "=l"(t) : "l"(dep));
        a.trace[(blockIdx.x == 0 ? L : 64 + L) * kTraceSlots + k] = t;
    }
}

// Grid barrier over all CTAs: arrival on one of 8 counters (128 B apart, so
// arrivals spread over 8 lines instead of queueing on one), then warp 0
// polls all 8 with acquire loads until each reached gen x (its CTA count).
// Counters only grow within a launch; the host zeroes them before it.
__device__ bool grid_sync(unsigned* sync, unsigned gen, int* status, int* s_ok) {
    __syncthreads();
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        if (lane == 0)  // release: orders this CTA's writes and atomics (after bar.sync) before the arrival
            asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(sync + 32 * (blockIdx.x & 7)) : "memory");
        const int i = lane & 7;
        const unsigned n = gridDim.x;
        const unsigned cnt = n > (unsigned)i ? (n - (unsigned)i + 7u) / 8u : 0u;
        const unsigned target = gen * cnt;
        const unsigned long long t0 = now_ns();
        bool ok = true;
        for (unsigned it = 0;; ++it) {
            unsigned v = target, ab = 0;
            if (lane < 8)
                asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(sync + 32 * i) : "memory");
            if (__all_sync(0xffffffffu, (int)(v - target) >= 0)) break;
            if ((it & 31u) == 31u) {
                if (lane == 0)
                    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(ab) : "l"(abort_word(sync)) : "memory");
                if (__any_sync(0xffffffffu, ab != 0u)) {
                    ok = false;
                    break;
                }
            }
            if (now_ns() - t0 > kTimeoutNs) {
                ok = false;
                if (lane == 0) {
                    record_status(status, QMOE_ERR_TIMEOUT);
                    atomicExch(abort_word(sync), 1u);
                }
                break;
            }
        }
        if (lane == 0) *s_ok = ok ? 1 : 0;
    }
    __syncthreads();
    return *s_ok != 0;
}

// Two IQ4_XS rows of D = 1024 * SBL2 values (a pair's gate and up rows)
// dotted with the activation in block floating point held in registers,
// decoded side by side so that their loads, decodes and reductions overlap;
// lane l owns sub-blocks l*SBL2 .. l*SBL2+SBL2-1, all in one super-block, so
// one header load per row.
template <int SBL2>
__device__ __forceinline__ void row_dot2(const uint8_t* row_a, const uint8_t* row_b, const int (&xr)[SBL2][16],
                                         const float (&xs)[SBL2], int lane, float& out_a, float& out_b) {
    const int b0 = lane * SBL2;
    const uint8_t* blk_a = row_a + (b0 >> 3) * QMOE_SB_BYTES;
    const uint8_t* blk_b = row_b + (b0 >> 3) * QMOE_SB_BYTES;
    const uint2 ha = *reinterpret_cast<const uint2*>(blk_a);
    const uint2 hb = *reinterpret_cast<const uint2*>(blk_b);
    const float da = __half2float(__ushort_as_half((unsigned short)(ha.x & 0xFFFFu)));
    const float db = __half2float(__ushort_as_half((unsigned short)(hb.x & 0xFFFFu)));
    float acc_a = 0.0f, acc_b = 0.0f;
#pragma unroll
    for (int i = 0; i < SBL2; ++i) {
        const int ib = (b0 + i) & 7;
        const uint2 a0 = *reinterpret_cast<const uint2*>(blk_a + 8 + 16 * ib);
        const uint2 a1 = *reinterpret_cast<const uint2*>(blk_a + 16 + 16 * ib);
        const uint2 c0 = *reinterpret_cast<const uint2*>(blk_b + 8 + 16 * ib);
        const uint2 c1 = *reinterpret_cast<const uint2*>(blk_b + 16 + 16 * ib);
        const int Sa = qmoe_subblock_dot(a0.x, a0.y, a1.x, a1.y, xr[i], 0);
        const int Sb = qmoe_subblock_dot(c0.x, c0.y, c1.x, c1.y, xr[i], 0);
        const float dla = da * (float)(qmoe_iq4xs_ls(ha.x, ha.y, ib) - 32);
        const float dlb = db * (float)(qmoe_iq4xs_ls(hb.x, hb.y, ib) - 32);
        acc_a = fmaf(dla * xs[i], (float)Sa, acc_a);
        acc_b = fmaf(dlb * xs[i], (float)Sb, acc_b);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        acc_a += __shfl_xor_sync(0xffffffffu, acc_a, o);
        acc_b += __shfl_xor_sync(0xffffffffu, acc_b, o);
    }
    out_a = acc_a;
    out_b = acc_b;
}

// Block floating point of a 32-value block given its largest |v| as float
// bits (the same step and rounding as warp_block_fp): the pair word of
// values j and j + 16 (v0, v1) and, in *step, the block's step.
__device__ __forceinline__ int block_fp_pair(float v0, float v1, unsigned mb, float* step) {
    const int E = (int)(mb >> 23);
    int q0 = 0, q1 = 0;
    float st = 0.0f;
    if (E >= 255) {
        st = __uint_as_float(0x7fc00000u);
    } else if (E >= 1) {
        const int k = 140 - E, k1 = k >> 1, k2 = k - k1;
        const float s1 = __uint_as_float((unsigned)(127 + k1) << 23);
        const float s2 = __uint_as_float((unsigned)(127 + k2) << 23);
        q0 = __float2int_rn((v0 * s1) * s2);
        q1 = __float2int_rn((v1 * s1) * s2);
        st = E >= 14 ? __uint_as_float((unsigned)(E - 13) << 23) : __uint_as_float(1u << (E + 9));
    }
    *step = st;
    return (q0 & 0xFFFF) | (q1 << 16);
}

// One 32-value block to block floating point, lane j holding value j.
__device__ __forceinline__ void convert_block(float v, int* q16, float* step, int lane) {
    float st;
    const int pw = warp_block_fp(v, &st);
    if (lane < 16) q16[lane] = pw;
    if (lane == 0) *step = st;
}

// The activation's block-floating-point words and steps for row_dot2: lane l
// takes sub-blocks l*SBL2 .. l*SBL2+SBL2-1.
template <int SBL2>
__device__ __forceinline__ void load_xr(const int* xq, const float* xs, int lane, int (&xr)[SBL2][16],
                                        float (&xsr)[SBL2]) {
#pragma unroll
    for (int i = 0; i < SBL2; ++i) {
        const int b = lane * SBL2 + i;
        const int4* src = reinterpret_cast<const int4*>(xq + b * 16);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int4 w4 = src[q];
            xr[i][4 * q] = w4.x;
            xr[i][4 * q + 1] = w4.y;
            xr[i][4 * q + 2] = w4.z;
            xr[i][4 * q + 3] = w4.w;
        }
        xsr[i] = xs[b];
    }
}

// Sub-block t of one down row dotted with its slot's activation block (hq in
// the [quad][sub-block][4 words] layout), scaled: d*(ls-32) * step * S.  A
// row of whole super-blocks has ib0 = 0; a rank's slice of fewer than 8
// sub-blocks stores them after the super-block's header and takes its scales
// from sub-block ib0 on.
__device__ __forceinline__ float down_unit_one(const uint8_t* row, const int* hq, const float* hs, int nsbh, int t,
                                               int ib0) {
    const uint8_t* blk = row + (t >> 3) * QMOE_SB_BYTES;
    const int ib = t & 7;
    const uint2 hdr = *reinterpret_cast<const uint2*>(blk);
    const uint2 q0 = *reinterpret_cast<const uint2*>(blk + 8 + 16 * ib);
    const uint2 q1 = *reinterpret_cast<const uint2*>(blk + 16 + 16 * ib);
    int xp[16];
#pragma unroll
    for (int v = 0; v < 4; ++v) {
        const int4 w4 = *reinterpret_cast<const int4*>(hq + (v * nsbh + t) * 4);
        xp[4 * v] = w4.x;
        xp[4 * v + 1] = w4.y;
        xp[4 * v + 2] = w4.z;
        xp[4 * v + 3] = w4.w;
    }
    const int Sd = qmoe_subblock_dot(q0.x, q0.y, q1.x, q1.y, xp, 0);
    const float dl = __half2float(__ushort_as_half((unsigned short)(hdr.x & 0xFFFFu))) *
                     (float)(qmoe_iq4xs_ls(hdr.x, hdr.y, ib0 + ib) - 32);
    return dl * hs[t] * (float)Sd;
}

// Shape-derived constants and this CTA's static slices.
struct SKPart {
    int D, I, E, K, RB, DRB, NSBH;
    size_t GUE, DNE;
    int sq_lo, sq_hi, p_lo, p_hi, j_lo, j_hi;
    int jc_lo, jc_hi;  // down rows copied: [j_lo, j_hi), widened to even bounds for rows of 8 mod 16 bytes
};

template <class SH>
__device__ __forceinline__ SKPart sk_part() {
    SKPart p;
    constexpr int n = SH::NSM;
    const int c = blockIdx.x;
    p.D = SH::D;
    p.I = SH::I;
    p.E = SH::E;
    p.K = SH::K;
    p.RB = (SH::D >> 8) * QMOE_SB_BYTES;
    p.DRB = SH::DRB;
    p.NSBH = SH::I >> 5;
    p.GUE = (size_t)2 * SH::I * p.RB;
    p.DNE = (size_t)SH::D * p.DRB;
    constexpr int P = SH::K * SH::I;
    p.sq_lo = c * SH::I / n;
    p.sq_hi = (c + 1) * SH::I / n;
    p.p_lo = c * P / n;
    p.p_hi = (c + 1) * P / n;
    p.j_lo = c * SH::D / n;
    p.j_hi = (c + 1) * SH::D / n;
    p.jc_lo = SH::kPairRows ? p.j_lo & ~1 : p.j_lo;
    p.jc_hi = SH::kPairRows ? (p.j_hi + 1) & ~1 : p.j_hi;
    return p;
}

// Shared-expert gate|up rows of this CTA's slice (thread 0 only).
__device__ __forceinline__ void issue_sgu(const SKLayer& W, const SKPart& p, const SKLayout& S, unsigned char* sm,
                                          uint64_t* bar) {
    const int nsq = p.sq_hi - p.sq_lo;
    uint8_t* sgu = sm + S.sgu;
    mbar_expect_tx(bar, (uint32_t)(2 * nsq * p.RB));
    if (nsq > 0) {
        ptx::bulk_g2s(sgu, W.sh_gate_up + (size_t)p.sq_lo * p.RB, (uint32_t)(nsq * p.RB), bar);
        ptx::bulk_g2s(sgu + (size_t)S.NSQ * p.RB, W.sh_gate_up + (size_t)(p.I + p.sq_lo) * p.RB,
                      (uint32_t)(nsq * p.RB), bar);
    }
}

// Shared-expert down rows of this CTA's output slice (thread 0 only).
__device__ __forceinline__ void issue_sdn(const SKLayer& W, const SKPart& p, const SKLayout& S, unsigned char* sm,
                                          uint64_t* bar) {
    const int nc = p.jc_hi - p.jc_lo;
    mbar_expect_tx(bar, (uint32_t)(nc * p.DRB));
    if (nc > 0) ptx::bulk_g2s(sm + S.sdn, W.sh_down + (size_t)p.jc_lo * p.DRB, (uint32_t)(nc * p.DRB), bar);
}

// Router columns of this CTA's output rows, for every router row and the gate
// vector (row E), as 2-D tensor copies (thread 0 only): boxes of kRColW
// columns from j_lo rounded down to a 16-byte boundary, kRBoxRows rows each;
// rcol row e at e * kRColW floats, the gate vector after the last box.
__device__ __forceinline__ void issue_rcol(const CUtensorMap* rmap, const CUtensorMap* gmap, const SKPart& p,
                                           const SKLayout& S, unsigned char* sm, uint64_t* bar) {
    float* rcol = reinterpret_cast<float*>(sm + S.rcol);
    const int nbox = (p.E + kRBoxRows - 1) / kRBoxRows, rows = p.E < kRBoxRows ? p.E : kRBoxRows;
    const int x = p.j_lo & ~3;
    mbar_expect_tx(bar, (uint32_t)((nbox * rows + 1) * kRColW * 4));
    for (int b = 0; b < nbox; ++b) ptx::tma_load_2d(rcol + b * rows * kRColW, rmap, x, b * rows, bar);
    ptx::tma_load_2d(rcol + nbox * kRBoxRows * kRColW, gmap, x, 0, bar);
}

// Row r of the router-column window (kRColW floats from column j_lo & ~3)
// dotted with x over the same window: 16-byte loads (the 8 rows a quarter
// warp reads, 80 bytes apart, fall in 8 distinct bank groups).  The window's
// columns outside this CTA's rows hold x = 0 and add exact zeros, so the sum
// runs over the CTA's columns in order, as a plain loop over them would
// (router weights are finite).
__device__ __forceinline__ float rcol_dot(const float* row, const float4* x4) {
    const float4* r4 = reinterpret_cast<const float4*>(row);
    float v = 0.0f;
#pragma unroll
    for (int q = 0; q < kRColW / 4; ++q) {
        const float4 r = r4[q], x = x4[q];
        v = fmaf(r.x, x.x, v);
        v = fmaf(r.y, x.y, v);
        v = fmaf(r.z, x.z, v);
        v = fmaf(r.w, x.w, v);
    }
    return v;
}

// This CTA's share of the router logits: thread e (and thread 0 for the gate
// row E) sums rcol[e][j] * x[j] over its columns j.  fp32 accumulators: four
// consecutive experts combine into one vector atomic add on their line; fp64
// (f64): one atomic add per logit, four per line.
__device__ __forceinline__ void router_partial(const SKPart& p, const SKLayout& S, const unsigned char* sm,
                                               float* acc_buf, bool f64) {
    const float4* x4 = reinterpret_cast<const float4*>(sm + S.xo);
    const float* rcol = reinterpret_cast<const float*>(sm + S.rcol);
    const int e = threadIdx.x, lane = threadIdx.x & 31;
    const int gate_row = ((p.E + kRBoxRows - 1) / kRBoxRows) * kRBoxRows;
    float v = 0.0f;
    if (e < p.E) v = rcol_dot(rcol + e * kRColW, x4);
    if (f64) {
        double* acc64 = reinterpret_cast<double*>(acc_buf);
        if (e < p.E)
            asm volatile("red.global.add.f64 [%0], %1;" ::"l"(acc64 + (e >> 2) * 16 + (e & 3)), "d"((double)v)
                         : "memory");
        if (e == 0) {
            const float g = rcol_dot(rcol + gate_row * kRColW, x4);
            asm volatile("red.global.add.f64 [%0], %1;" ::"l"(acc64 + (p.E >> 2) * 16 + (p.E & 3)), "d"((double)g)
                         : "memory");
        }
        return;
    }
    const float v1 = __shfl_down_sync(0xffffffffu, v, 1), v2 = __shfl_down_sync(0xffffffffu, v, 2),
                v3 = __shfl_down_sync(0xffffffffu, v, 3);
    if (e < p.E && (lane & 3) == 0)
        asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(acc_buf + (e >> 2) * 32), "f"(v), "f"(v1),
                     "f"(v2), "f"(v3)
                     : "memory");
    if (e == 0) atomicAdd(acc_buf + (p.E >> 2) * 32 + (p.E & 3), rcol_dot(rcol + gate_row * kRColW, x4));
}

// This CTA's routed pairs [p_lo, p_hi) fall in at most two expert slots: the
// first len0 pairs in the first.
__device__ __forceinline__ int seg0_len(const SKPart& p) {
    const int np = p.p_hi - p.p_lo, r0 = p.p_lo % p.I;
    return np < p.I - r0 ? np : p.I - r0;
}

// The selected experts' gate|up rows, issued by warp 0 in chunks of kSKChunk
// pairs, each chunk with its own mbarrier so decoding starts as the first
// chunk lands; a chunk that crosses the expert boundary is two pieces.  Lane c
// posts chunk c's expected bytes; then lane 2q / 2q + 1 copies piece q's gate /
// up rows (contiguous in the expert).
__device__ __forceinline__ void issue_gate_up(const SKLayer& W, const SKPart& p, const SKLayout& S, unsigned char* sm,
                                              const int* ids, uint64_t* bar_ch, int lane) {
    const int np = p.p_hi - p.p_lo, len0 = seg0_len(p);
    const int nch = (np + kSKChunk - 1) / kSKChunk;
    if (lane < kSKMaxChunks) {
        const int u0 = lane * kSKChunk, u1 = min(u0 + kSKChunk, np);
        mbar_expect_tx(bar_ch + lane, u1 > u0 ? (uint32_t)(2 * (u1 - u0) * p.RB) : 0u);
    }
    __syncwarp();
    // piece q: chunk c = the q-th chunk, except that the chunk holding the
    // boundary contributes two pieces
    const int cb = len0 < np ? len0 / kSKChunk : nch;  // chunk that contains pair len0 (if len0 is interior)
    const bool split = len0 < np && len0 % kSKChunk != 0;
    const int npieces = nch + (split ? 1 : 0);
    const int q = lane >> 1, up = lane & 1;
    if (q < npieces) {
        int c, u0, u1;
        if (!split || q <= cb) {
            c = q;
            u0 = c * kSKChunk;
            u1 = min(u0 + kSKChunk, np);
            if (split && q == cb) u1 = len0;  // first piece of the boundary chunk
        } else {
            c = q - 1;
            u0 = c == cb ? len0 : c * kSKChunk;
            u1 = min(c * kSKChunk + kSKChunk, np);
        }
        if (u1 > u0) {
            const int pp = p.p_lo + u0, s = pp / p.I, r = pp - s * p.I;
            const uint8_t* src = W.gate_up + (size_t)ids[s] * p.GUE + (size_t)(up ? p.I + r : r) * p.RB;
            ptx::bulk_g2s(sm + (up ? S.ubuf : S.gbuf) + (size_t)u0 * p.RB, src, (uint32_t)((u1 - u0) * p.RB),
                          bar_ch + c);
        }
    }
}

// The selected experts' rows of this CTA's output slice of their down, one
// copy per slot (issued by warp 1 beside warp 0's gate|up copies; needed only
// in phase C).
__device__ __forceinline__ void issue_down(const SKLayer& W, const SKPart& p, const SKLayout& S, unsigned char* sm,
                                           const int* ids, uint64_t* bar_dn, int lane) {
    const int nc = p.jc_hi - p.jc_lo;
    if (lane == 0) mbar_expect_tx(bar_dn, (uint32_t)(p.K * nc * p.DRB));
    __syncwarp();
    if (lane < p.K && nc > 0)
        ptx::bulk_g2s(sm + S.dbuf + (size_t)lane * S.NJR * p.DRB,
                      W.down + (size_t)ids[lane] * p.DNE + (size_t)p.jc_lo * p.DRB, (uint32_t)(nc * p.DRB), bar_dn);
}

// XC: this launch exchanges partial rows with peer ranks (a.R > 1); one rank
// compiles without any of it.
template <class SH, bool XC>
__global__ void __launch_bounds__(kSKThreads, 1) stack_kernel(const __grid_constant__ SKArgs a) {
    extern __shared__ __align__(128) unsigned char sm[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const SKPart p = sk_part<SH>();
    constexpr SKLayout S = SH::S;
    constexpr int SBL2 = SH::D / 1024;
    constexpr int D = SH::D, I = SH::I, E = SH::E, K = SH::K;
    const int nsq = p.sq_hi - p.sq_lo, np = p.p_hi - p.p_lo, nj = p.j_hi - p.j_lo;
    constexpr int G = (E + 1 + 3) / 4;  // accumulator lines per logit buffer

    int* xq = reinterpret_cast<int*>(sm + S.xq);
    float* xs = reinterpret_cast<float*>(sm + S.xs);
    // xo: x over the router-column window [j_lo & ~3, +kRColW); row j of this
    // CTA's slice at xo[xw + j], the rest zero
    float* xo = reinterpret_cast<float*>(sm + S.xo);
    const int xw = p.j_lo & 3;
    const uint8_t* sgu = sm + S.sgu;
    const uint8_t* sdn = sm + S.sdn;
    const uint8_t* gbuf = sm + S.gbuf;
    const uint8_t* ubuf = sm + S.ubuf;
    const uint8_t* dbuf = sm + S.dbuf;
    int* hq = reinterpret_cast<int*>(sm + S.hq);
    float* hs = reinterpret_cast<float*>(sm + S.hs);
    float* gv = reinterpret_cast<float*>(sm + S.gv);
    float* uv = reinterpret_cast<float*>(sm + S.uv);
    float* sgv = reinterpret_cast<float*>(sm + S.sgv);
    float* suv = reinterpret_cast<float*>(sm + S.suv);
    unsigned long long* cand = reinterpret_cast<unsigned long long*>(sm + S.cand);
    unsigned long long* wmax = reinterpret_cast<unsigned long long*>(sm + S.wmax);
    unsigned* red = reinterpret_cast<unsigned*>(sm + S.red);
    float* tkv = reinterpret_cast<float*>(sm + S.tkv);
    int* tki = reinterpret_cast<int*>(sm + S.tki);
    int* s_ok = reinterpret_cast<int*>(sm + S.misc);
    int* s_cnt = reinterpret_cast<int*>(sm + S.misc) + 8;
    float* s_glogit = reinterpret_cast<float*>(sm + S.misc) + 12;
    unsigned* s_epoch = reinterpret_cast<unsigned*>(sm + S.misc) + 2;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S.bars);
    uint64_t* bar_sgu = bars;
    uint64_t* bar_sdn = bars + 1;
    uint64_t* bar_rc = bars + 2;
    uint64_t* bar_dn = bars + 3;
    uint64_t* bar_ch = bars + 4;
    constexpr int nbars = 4 + kSKMaxChunks;

    if (tid == 0) {
        for (int i = 0; i < nbars; ++i) mbar_init(bars + i, 1);
        ptx::fence_mbar_init();
        *s_epoch = XC ? __ldcg(a.epoch) : 0u;
    }
    __syncthreads();
    constexpr bool xchg = XC;
    const int ib0 = SH::I >= 256 ? 0 : a.ib0;  // whole super-blocks start at sub-block 0
    const unsigned epoch = *s_epoch;
    // Phases issued (kept by thread 0 in registers), for the bounded drain:
    // the prefetch barriers (shared rows, shared down rows, router columns) and
    // the per-layer routed copies (chunks and down rows, issued together).
    int iss_pre = 0, iss_sdn = 0, iss_routed = 0;
    if (tid == 0) {
        issue_sgu(a.L[0], p, S, sm, bar_sgu);
        issue_sdn(a.L[0], p, S, sm, bar_sdn);
        issue_rcol(&a.rmap[0], &a.gmap[0], p, S, sm, bar_rc);
        iss_pre = iss_sdn = 1;
    }

    // ---------------- prologue: layer 0's router logits --------------------
    if (tid < kRColW) {
        const int j = tid - xw;
        const __nv_bfloat16* x0 = a.teacher ? a.teacher : a.x;
        xo[tid] = j >= 0 && j < nj ? __bfloat162float(x0[p.j_lo + j]) : 0.0f;
    }
    bool ok = !__syncthreads_or(!mbar_wait(bar_rc, 0));
    if (ok) router_partial(p, S, sm, a.logits + (size_t)(blockIdx.x % kStackLogitReplicas) * G * 32, xchg);
    else if (tid == 0) {
        record_status(a.status, QMOE_ERR_TIMEOUT);
        atomicExch(abort_word(a.sync), 1u);
    }
    unsigned gen = 0;
    ok = grid_sync(a.sync, ++gen, a.status, s_ok) && ok;

    for (int L = 0; L < a.n_layers && ok; ++L) {
        const SKLayer& W = a.L[L];
        const uint32_t par = (uint32_t)(L & 1);
        const bool last = L + 1 == a.n_layers;
        const float* lg = a.logits + (size_t)(L & 1) * kStackLogitReplicas * G * 32;
        float* lg_next = a.logits + (size_t)((L + 1) & 1) * kStackLogitReplicas * G * 32;

        // ---------------- phase B: top-k, gate|up ----------------------------
        trace_mark(a, L, 0);
        // x loads, then the selection's logit loads; x converts to block
        // floating point while the logits are in flight (each warp 4 blocks).
        constexpr int NXB = D / 32, XPW = (NXB + kSKWarps - 1) / kSKWarps;
        float xv[XPW];
#pragma unroll
        for (int i = 0; i < XPW; ++i) {
            const int b = warp + i * kSKWarps;
            xv[i] = 0.0f;
            if (b < NXB)
                xv[i] = a.teacher ? __bfloat162float(a.teacher[(size_t)L * D + b * 32 + lane])
                        : L == 0  ? __bfloat162float(a.x[b * 32 + lane])
                                  : __bfloat162float(__ushort_as_bfloat16(
                                       __ldcg(reinterpret_cast<const unsigned short*>(a.act) + b * 32 + lane)));
        }
        // logit i: fp32 at float (i / 4) * 32 + i % 4, or fp64 at double (i / 4) * 16 + i % 4
        const double* lg64 = reinterpret_cast<const double*>(lg);
        auto logit_at = [&](int i) {
            return xchg ? (float)__ldcg(lg64 + (i >> 2) * 16 + (i & 3)) : __ldcg(lg + (i >> 2) * 32 + (i & 3));
        };
        if (tid == 0) *s_glogit = logit_at(E);
        const float lmax = block_topk_threshold(
            logit_at, E, K, cand, wmax, red, s_cnt, tkv, tki,
            [&]() {
#pragma unroll
                for (int i = 0; i < XPW; ++i) {
                    const int b = warp + i * kSKWarps;
                    if (b < NXB) convert_block(xv[i], xq + b * 16, xs + b, lane);
                }
            },
            [&](int pt, unsigned long long d) { trace_mark_after(a, L, 12 + pt, d); });
        trace_mark(a, L, 1);
        if (a.ids_trace && blockIdx.x == 0 && tid < K) {
            float ps = 0.0f;
            for (int s2 = 0; s2 < K; ++s2) ps += tkv[s2];
            a.ids_trace[L * K + tid] = tki[tid];
            a.w_trace[L * K + tid] = tkv[tid] * (1.0f / ps);
        }
        // Warps 0 and 1 issue the routed copies; the others stay off the
        // shared-memory pipe meanwhile (traffic there slows the issue).
        if (warp == 0) {
            if (lane == 0) {
                ptx::fence_proxy_async();
                if (!(fabsf(lmax) <= 3.0e38f)) record_status(a.status, QMOE_ERR_NOT_FINITE);
            }
            issue_gate_up(W, p, S, sm, tki, bar_ch, lane);
            if (tid == 0) ++iss_routed;
            trace_mark(a, L, 2);
        } else if (warp == 1) {
            if (lane == 0) ptx::fence_proxy_async();
            issue_down(W, p, S, sm, tki, bar_dn, lane);
            trace_mark(a, L, 3, 32);
        } else if (blockIdx.x == 0 && !last) {
            // CTA 0 clears the other logit accumulator for the next layer's sums
            // (read last in the previous layer's phase B; first added to after
            // this layer's second barrier).
            for (int g = tid - 64; g < kStackLogitReplicas * G; g += kSKThreads - 64) {
                *reinterpret_cast<float4*>(lg_next + g * 32) = make_float4(0.f, 0.f, 0.f, 0.f);
                if constexpr (XC)  // four fp64 logits per line
                    *reinterpret_cast<float4*>(lg_next + g * 32 + 4) = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
        __syncthreads();
        trace_mark(a, L, 4);
        {
            int xr[SBL2][16];
            float xsr[SBL2];
            load_xr<SBL2>(xq, xs, lane, xr, xsr);
            // Row tasks: the shared expert's 2 * nsq rows (prefetched), then the
            // routed pairs' gate and up rows as their chunks land.
            const bool w_ok = mbar_wait(bar_sgu, par);
            // Pair tasks: the shared expert's nsq pairs (prefetched), then the
            // routed pairs as their chunks land; a warp decodes a pair's gate
            // and up rows side by side.
            for (int t = warp; t < nsq + np && ok && w_ok; t += kSKWarps) {
                const uint8_t *rg, *ru;
                float *dg, *du;
                if (t < nsq) {
                    rg = sgu + (size_t)t * p.RB;
                    ru = sgu + (size_t)(S.NSQ + t) * p.RB;
                    dg = sgv + t;
                    du = suv + t;
                } else {
                    const int u = t - nsq;
                    if (!mbar_wait(bar_ch + u / kSKChunk, par)) {
                        ok = false;
                        break;
                    }
                    if (u % kSKChunk == 0) trace_mark(a, L, 18 + u / kSKChunk, 32 * warp);  // chunk landed
                    rg = gbuf + (size_t)u * p.RB;
                    ru = ubuf + (size_t)u * p.RB;
                    dg = gv + u;
                    du = uv + u;
                }
                float g, up;
                row_dot2<SBL2>(rg, ru, xr, xsr, lane, g, up);
                if (lane == 0) {
                    *dg = g;
                    *du = up;
                }
            }
            if (!w_ok) ok = false;
        }
        if (__syncthreads_or(!ok)) {
            if (tid == 0) {
                record_status(a.status, QMOE_ERR_TIMEOUT);
                atomicExch(abort_word(a.sync), 1u);
            }
            ok = false;
            break;
        }
        trace_mark(a, L, 5);
        {
            // h slice and its blocks' running max |h| (bits of non-negative
            // floats order like unsigned integers; NaN above infinity)
            // Each warp reduces first: one atomic per block a warp's 32 h
            // values touch (at most three).
            unsigned* hm = a.hmax + (L & 1) * kStackHmaxWords;
            const int n_h = np + nsq;  // routed slice, then the shared slice
            for (int i0 = warp * 32; i0 < n_h; i0 += kSKThreads) {
                const int i = i0 + lane;
                int hidx = -1;
                float v = 0.0f;
                if (i < np) {
                    v = silu(gv[i]) * uv[i];
                    hidx = p.p_lo + i;
                } else if (i < n_h) {
                    v = silu(sgv[i - np]) * suv[i - np];
                    hidx = K * I + p.sq_lo + (i - np);
                }
                if (hidx >= 0) a.h[hidx] = v;
                const unsigned bits = hidx >= 0 ? __float_as_uint(fabsf(v)) : 0u;
                const int b = hidx >= 0 ? hidx >> 5 : -1;
                // lanes grouped by block (up to three groups where the routed
                // slice meets the shared one); one atomic per group
                const unsigned grp = __match_any_sync(0xffffffffu, b);
                const unsigned m = __reduce_max_sync(grp, bits);
                if (b >= 0 && lane == __ffs(grp) - 1)  // no return value: nothing waits for the L2 round trip
                    asm volatile("red.global.max.u32 [%0], %1;" ::"l"(hm + b * 32), "r"(m) : "memory");
            }
        }
        trace_mark(a, L, 6);
        if (!grid_sync(a.sync, ++gen, a.status, s_ok)) {
            ok = false;
            break;
        }
        trace_mark(a, L, 7);

        // ---------------- phase C: down + combine, next layer's logits -------
        // The next layer's shared rows and router columns stream in now, while
        // HBM is otherwise idle (their buffers were last read before the barrier).
        if (!last && tid == 0) {
            ptx::fence_proxy_async();
            issue_sgu(a.L[L + 1], p, S, sm, bar_sgu);
            issue_rcol(&a.rmap[L + 1], &a.gmap[L + 1], p, S, sm, bar_rc);
            ++iss_pre;
        }
        {
            // h -> block floating point with the producers' block maxima: lanes
            // 0-15 / 16-31 take one block each, element l and l + 16 per lane.
            const unsigned* hm = a.hmax + (L & 1) * kStackHmaxWords;
            constexpr int NBH = (K + 1) * (I / 32), NIT = (NBH + 2 * kSKWarps - 1) / (2 * kSKWarps);
            const int half = lane >> 4, hl = lane & 15;
            float v0[NIT], v1[NIT];
            unsigned mb[NIT];
#pragma unroll
            for (int i = 0; i < NIT; ++i) {
                const int b = warp + kSKWarps * (2 * i + half);
                v0[i] = v1[i] = 0.0f;
                mb[i] = 0u;
                if (b < NBH) {
                    v0[i] = __ldcg(a.h + (size_t)b * 32 + hl);
                    v1[i] = __ldcg(a.h + (size_t)b * 32 + 16 + hl);
                    mb[i] = __ldcg(hm + b * 32);
                }
            }
#pragma unroll
            for (int i = 0; i < NIT; ++i) {
                const int b = warp + kSKWarps * (2 * i + half);
                if (b < NBH) {
                    float st;
                    const int pw = block_fp_pair(v0[i], v1[i], mb[i], &st);
                    const int slot = b / (I / 32), t = b - slot * (I / 32);
                    // word w = 4*quad + (w & 3) of block t of the slot
                    hq[slot * p.NSBH * 16 + ((hl >> 2) * p.NSBH + t) * 4 + (hl & 3)] = pw;
                    if (hl == 0) hs[b] = st;
                }
            }
            // CTA 0 clears the other block-maximum buffer for the next layer
            // (read last in the previous layer's phase C).
            if (blockIdx.x == 0 && !last)
                for (int i = tid; i < kStackHmaxBlocks; i += kSKThreads)
                    a.hmax[((L + 1) & 1) * kStackHmaxWords + i * 32] = 0u;
        }
        __syncthreads();
        trace_mark(a, L, 8);
        {
            const bool d_ok = mbar_wait(bar_dn, par) && mbar_wait(bar_sdn, par);
            if (__syncthreads_or(!d_ok)) {
                if (tid == 0) {
                    record_status(a.status, QMOE_ERR_TIMEOUT);
                    atomicExch(abort_word(a.sync), 1u);
                }
                ok = false;
                break;
            }
        }
        trace_mark(a, L, 9);
        // Down + combine: a warp per output row j; its lanes walk the row's
        // (slot, sub-block) pairs of all k + 1 slots with the slot weight folded
        // in, so one reduction per row.  Slot K is the shared expert.
        float psum = 0.0f;
        for (int s2 = 0; s2 < K; ++s2) psum += tkv[s2];
        const float inv_psum = 1.0f / psum, gate = sigmoid(*s_glogit);
        const int jo = p.j_lo - p.jc_lo;  // row j_lo's place in the copied rows
        // exchange: this layer's flag value and receive parity (both change
        // with every exchange, across launches too)
        const unsigned fval = epoch * 64u + (unsigned)L + 1u;
        const int xpar = (int)((epoch * (unsigned)a.n_layers + (unsigned)L) & 1u);
        for (int j = warp; j < nj; j += kSKWarps) {
            float acc = 0.0f;
            constexpr int NT = (K + 1) * (I / 32);
            for (int t = lane; t < NT; t += 32) {
                const int s = t / (I / 32), b = t - s * (I / 32);
                const uint8_t* row = s < K ? dbuf + ((size_t)s * S.NJR + jo + j) * p.DRB : sdn + (size_t)(jo + j) * p.DRB;
                const float wgt = s < K ? tkv[s] * inv_psum : gate;
                acc += wgt * down_unit_one(row, hq + s * p.NSBH * 16, hs + s * p.NSBH, p.NSBH, b, ib0);
            }
            acc = warp_sum(acc);
            if constexpr (!xchg) {
                if (lane == 0) {
                    const __nv_bfloat16 xb = __float2bfloat16_rn(acc);
                    if (last) a.out[p.j_lo + j] = acc;
                    else a.act[p.j_lo + j] = xb;
                    if (a.act_trace) a.act_trace[(size_t)L * D + p.j_lo + j] = xb;
                    xo[xw + j] = __bfloat162float(a.teacher && !last ? a.teacher[(size_t)(L + 1) * D + p.j_lo + j] : xb);
                }
            } else {
                // this rank's partial of row j: kept, and stored into every
                // peer as one word (value bits, flag)
                if (lane == 0) xo[xw + j] = acc;
                if (lane < a.R && lane != a.rank)
                    ptx::st_relaxed_sys_u64(
                        a.xr[lane] + ((size_t)(xpar * a.R + a.rank) * D + p.j_lo + j),
                        ((unsigned long long)fval << 32) | __float_as_uint(acc));
            }
        }
        if constexpr (xchg) {
            trace_mark(a, L, 16);
            __syncthreads();
            // Row j_lo + tid: the R partials summed in rank order (the same
            // order, so the same bits, on every rank) once the peers' words
            // carry this exchange's flag.
            bool x_ok = true;
            if (tid < nj) {
                const unsigned long long* rx = a.xr[a.rank] + (size_t)xpar * a.R * D + p.j_lo + tid;
                float v = 0.0f;
                for (int q = 0; q < a.R && x_ok; ++q) {
                    float pv;
                    if (q == a.rank) {
                        pv = xo[xw + tid];
                    } else {
                        unsigned long long w = ptx::ld_relaxed_sys_u64(rx + (size_t)q * D);
                        if ((unsigned)(w >> 32) != fval) {
                            const unsigned long long t0 = now_ns();
                            do {
                                if (now_ns() - t0 > kXchgTimeoutNs) {
                                    x_ok = false;
                                    break;
                                }
                                w = ptx::ld_relaxed_sys_u64(rx + (size_t)q * D);
                            } while ((unsigned)(w >> 32) != fval);
                        }
                        pv = __uint_as_float((unsigned)w);
                    }
                    v = q == 0 ? pv : v + pv;
                }
                const __nv_bfloat16 xb = __float2bfloat16_rn(v);
                if (last) a.out[p.j_lo + tid] = v;
                else a.act[p.j_lo + tid] = xb;
                if (a.act_trace) a.act_trace[(size_t)L * D + p.j_lo + tid] = xb;
                xo[xw + tid] =
                    __bfloat162float(a.teacher && !last ? a.teacher[(size_t)(L + 1) * D + p.j_lo + tid] : xb);
            }
            if (__syncthreads_or(!x_ok)) {
                if (tid == 0) {
                    record_status(a.status, QMOE_ERR_TIMEOUT);
                    atomicExch(abort_word(a.sync), 1u);
                }
                ok = false;
                break;
            }
            trace_mark(a, L, 17);
        }
        // the next layer's router columns
        if (__syncthreads_or(!last && !mbar_wait(bar_rc, (uint32_t)((L + 1) & 1)))) {
            if (tid == 0) {
                record_status(a.status, QMOE_ERR_TIMEOUT);
                atomicExch(abort_word(a.sync), 1u);
            }
            ok = false;
            break;
        }
        trace_mark(a, L, 10);
        // warp 1 issues the next layer's shared down rows (thread 0 also adds the gate row below)
        if (tid == 32 && !last) {
            ptx::fence_proxy_async();
            issue_sdn(a.L[L + 1], p, S, sm, bar_sdn);
        }
        if (tid == 0 && !last) ++iss_sdn;
        if (!last) {
            router_partial(p, S, sm, lg_next + (size_t)(blockIdx.x % kStackLogitReplicas) * G * 32, xchg);
            trace_mark(a, L, 11);
            if (!grid_sync(a.sync, ++gen, a.status, s_ok)) {
                ok = false;
                break;
            }
        }
    }

    // This rank's launch count, read by every CTA at its start (all read it
    // before the prologue's barrier, which CTA 0 has passed).
    if (xchg && blockIdx.x == 0 && tid == 0) *a.epoch = epoch + 1u;

    // Stopped early: let this CTA's copies in flight land (bounded) before exit.
    if (!ok && tid == 0) {
        if (iss_pre > 0) {
            (void)mbar_wait(bar_sgu, (uint32_t)((iss_pre - 1) & 1));
            (void)mbar_wait(bar_rc, (uint32_t)((iss_pre - 1) & 1));
        }
        if (iss_sdn > 0) (void)mbar_wait(bar_sdn, (uint32_t)((iss_sdn - 1) & 1));
        if (iss_routed > 0) {
            const uint32_t q = (uint32_t)((iss_routed - 1) & 1);
            (void)mbar_wait(bar_dn, q);
            for (int c = 0; c < kSKMaxChunks; ++c) (void)mbar_wait(bar_ch + c, q);
        }
    }
}

}  // namespace

namespace {

// BASELINE configs 1-2 on a 148-SM B200: the whole layer (I = 512), or one
// rank's slice of every expert's intermediate rows on 2, 4 or 8 ranks.
using SKShapeC2 = SKShape<2048, 512, 10, 148>;
using SKShapeC2R2 = SKShape<2048, 512, 10, 148, 256>;
using SKShapeC2R4 = SKShape<2048, 512, 10, 148, 128>;
using SKShapeC2R8 = SKShape<2048, 512, 10, 148, 64>;
using SKShapeTest = SKShape<1024, 64, 10, 148>;  // a small member of the family (tests)

template <class SH>
void (*entry(unsigned* smem, bool xc))(SKArgs) {
    *smem = SH::S.total;
    if constexpr (SH::I < 512) {
        if (xc) return stack_kernel<SH, true>;
    }
    return xc ? nullptr : stack_kernel<SH, false>;
}

// The compiled instantiation for these shapes on this device (xc: with the
// exchange between ranks), or null.
void (*pick_kernel(const qmoe_dims& d, int n_sm, unsigned* smem, bool xc))(SKArgs) {
    if (n_sm != 148 || d.top_k != 10 || d.inter != 512) return nullptr;
    if (d.hidden == 2048 && d.n_experts == 512) {
        switch (d.inter_local) {
            case 512: return entry<SKShapeC2>(smem, xc);
            case 256: return entry<SKShapeC2R2>(smem, xc);
            case 128: return entry<SKShapeC2R4>(smem, xc);
            case 64: return entry<SKShapeC2R8>(smem, xc);
            default: return nullptr;
        }
    }
    if (d.hidden == 1024 && d.n_experts == 64 && d.inter_local == 512) return entry<SKShapeTest>(smem, xc);
    return nullptr;
}

// The down rows in the format the kernel reads for I local columns: whole
// super-blocks, or one segment (header + I / 32 code groups) of one.
bool down_format_ok(int I, int nseg, int nsub) {
    return I >= 256 ? (nseg == I / 256 && nsub == 8) : (nseg == 1 && nsub == I / 32);
}

}  // namespace

// fp32 [rows][cols] row-major (cols * 4 bytes a multiple of 16, base 16-byte
// aligned) as a 2-D tensor with boxes of kRColW columns x min(rows, kRBoxRows)
// rows; reads past the last column return zeros.
static cudaError_t encode_rows_map(CUtensorMap* m, const float* base, int cols, int rows) {
    return encode_2d(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, base, (unsigned long long)cols, (unsigned long long)rows,
                     (unsigned long long)cols * 4, kRColW, (unsigned)(rows < kRBoxRows ? rows : kRBoxRows));
}

bool stack_kernel_supported(const qmoe_dims& d, int M, int n_layers, int R) {
    if (M != 1 || n_layers < 1 || n_layers > kSKMaxLayers || R < 1 || R > kMaxXchgRanks) return false;
    if (d.expert_lo != 0 || d.expert_hi != d.n_experts) return false;
    const int I = d.inter_local;
    if (!down_format_ok(I, d.down_nseg, d.down_nsub) || (I >= 256 && d.down_ib0 != 0)) return false;
    // the shared expert sliced like the routed ones (variant B of the family: equal widths)
    if (d.sh_inter_local != I || d.sh_down_nseg != d.down_nseg || d.sh_down_nsub != d.down_nsub ||
        d.sh_down_ib0 != d.down_ib0)
        return false;
    if (R > 1 && I * R != d.inter) return false;
    unsigned smem = 0;
    return pick_kernel(d, device_sm_count(), &smem, R > 1) != nullptr && smem <= 227u * 1024u;
}

cudaError_t launch_stack_kernel(const void* x, float* out, float* act, float* h, unsigned* sync,
                                unsigned long long* trace, int* status, const qmoe_layer_weights* layers, int n_layers,
                                const qmoe_dims& d, const XchgDesc* xc, const StackTraceBufs& tb, cudaStream_t stream) {
    SKArgs a{};
    a.act_trace = tb.act;
    a.ids_trace = tb.ids;
    a.w_trace = tb.weights;
    a.teacher = tb.teacher;
    a.R = xc ? xc->R : 1;
    a.rank = xc ? xc->rank : 0;
    a.ib0 = d.down_ib0;
    if (xc) {
        for (int q = 0; q < xc->R; ++q)
            a.xr[q] = reinterpret_cast<unsigned long long*>(xc->buf[q] + kXchgHeader);
        a.epoch = reinterpret_cast<unsigned*>(xc->buf[xc->rank]);
    }
    a.trace = trace;
    a.x = reinterpret_cast<const __nv_bfloat16*>(x);
    a.out = out;
    a.act = reinterpret_cast<__nv_bfloat16*>(act);
    // the single launch keeps its logits in the accumulators behind the barrier words
    a.logits = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(sync) + 1152);
    a.hmax = reinterpret_cast<unsigned*>(reinterpret_cast<unsigned char*>(sync) + 1152 + stack_logit_bytes(d.n_experts));
    a.h = h;
    a.sync = sync;
    a.status = status;
    a.n_layers = n_layers;
    a.D = d.hidden;
    a.I = d.inter;
    a.E = d.n_experts;
    a.K = d.top_k;
    for (int l = 0; l < n_layers; ++l) {
        a.L[l].router = layers[l].router;
        a.L[l].gate_vec = layers[l].gate_vec;
        a.L[l].gate_up = reinterpret_cast<const uint8_t*>(layers[l].gate_up);
        a.L[l].down = reinterpret_cast<const uint8_t*>(layers[l].down);
        a.L[l].sh_gate_up = reinterpret_cast<const uint8_t*>(layers[l].sh_gate_up);
        a.L[l].sh_down = reinterpret_cast<const uint8_t*>(layers[l].sh_down);
    }
    const int n = device_sm_count();
    unsigned smem = 0;
    void (*kern)(SKArgs) = pick_kernel(d, n, &smem, xc != nullptr);
    if (!kern) return cudaErrorInvalidValue;
    for (int l = 0; l < n_layers; ++l) {
        cudaError_t e = encode_rows_map(&a.rmap[l], layers[l].router, d.hidden, d.n_experts);
        if (e == cudaSuccess) e = encode_rows_map(&a.gmap[l], layers[l].gate_vec, d.hidden, 1);
        if (e != cudaSuccess) return e;
    }
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess) return err;
    // Barrier counters, the abort word, both logit accumulators and both
    // block-maximum buffers start at zero for every launch.
    err = cudaMemsetAsync(sync, 0, stack_sync_bytes(d.n_experts), stream);
    if (err != cudaSuccess) return err;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)n);
    cfg.blockDim = dim3(kSKThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, a);
}

}  // namespace qmoe
