// The whole batch-1 MoE decode stack in one persistent launch.
//
// One 512-thread CTA per SM (a cooperative launch, so all are co-resident and
// may wait on one another), every CTA doing the same work on its own slices.
// Every layer is the reference's `_moe` (reference/model.py:387-417):
//
//   routing  once every CTA has added its share of the layer's router
//            logits (below) and arrived on the logit counters, every CTA
//            reads the E + 1 exact sums and ranks them itself (block top-k on
//            the softmax numerators, ties to the lower id): the same logits
//            give every CTA the same experts.
//   B        a CTA then starts all its copies at once: its fixed slice of the
//            k * I routed (gate row, up row) pairs of the selected experts,
//            then its rows of their down projections (cp.async.bulk into
//            shared memory, an mbarrier per chunk, several lanes issuing).
//            While they stream in it reads the layer input x, converts it to
//            block floating point and decodes its slice of the shared
//            expert's pairs (rows prefetched); then the routed pairs as their
//            chunks land, each pair split over D / 1024 warps (one 32-value
//            sub-block of each row per lane), two pairs at a time per warp,
//            decoded from IQ4_XS in registers; SwiGLU; its h values go out as
//            words and it arrives on the h counters.
//   C        once the h round is complete, every CTA copies all (k + 1) * I h
//            words into shared memory with one bulk copy, converts them to
//            block floating point, starts the next layer's prefetches,
//            computes its D / 148 output rows of the routed experts'
//            weighted down projections plus the gated shared expert,
//            publishes them as the next layer's activation words, adds its
//            share of the next layer's logits, sum_{j in its rows} R[e][j]
//            x[j] for every expert e (and the gate vector, row E), into the
//            fp64 accumulators, and arrives on the logit counters.
//
// A round's counters are 8 words on separate lines: a CTA arrives on word
// c % 8 with release semantics; a waiter's 8 lanes poll the 8 words, then
// acquire.  fp32 partials whose magnitudes span less than 2^21 sum exactly in
// fp64, in any order: the logits do not depend on arrival order, so reruns
// give the same bits and every rank of a sharded stack selects the same
// experts.  The accumulators rotate over three buffers (layer % 3): a CTA
// clears its lines of the buffer two layers on after the h round, when every
// CTA has read it, and its arrival on the logit counters orders the clearing
// before anyone adds into it again.  The activation and h words carry tags
// derived from the layer's stamp, launch_counter * 64 + layer + 1 (the
// counter lives in the workspace and advances every launch), checked when
// they are read: activation words are bf16 with a 16-bit tag, h words fp32
// with their low 8 mantissa bits replaced by an 8-bit tag (the block floating
// point they feed keeps 14 bits of the block maximum).
//
// Sharded over R ranks (one process and one GPU each; the reference's split
// of every expert's intermediate rows, tt/plan.py:70-103), each rank runs
// this kernel on its slice of every expert and its phase-C rows are partial
// sums.  CTA c stores its partial rows into CTA c's receive slots on every
// peer as 8-byte words (value bits, flag) over NVLink and sums the R partials
// of its rows in rank order once the peers' words are in: every rank ends the
// layer with bitwise the same activation.
//
// All waits are bounded in time (%globaltimer): a wait that runs out sets
// QMOE_ERR_TIMEOUT and an abort word that every other wait checks; each CTA
// then waits (bounded) for its own copies in flight and returns.  No trap,
// no unbounded spin.
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
constexpr int kSKChunk = 8;      // routed row pairs per gate|up copy chunk
constexpr int kSKMaxChunks = 6;  // chunks of a worker's pairs (<= 48 pairs)
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
    // xepoch: this rank's count of completed exchange launches.
    int R, rank;
    int ib0;  // first sub-block of a down row's slice inside its super-block
    unsigned long long* xr[kMaxXchgRanks];
    unsigned* xepoch;
    const __nv_bfloat16* x;  // [D] layer-0 input
    float* out;              // [D] last layer's output
    unsigned char* sync;     // the synchronisation area (common.cuh)
    unsigned long long* trace;     // phase stamps of worker 0 and the routing CTA, or null
    __nv_bfloat16* act_trace;      // [n_layers][D]: every layer's output rounded to bf16, or null
    int* ids_trace;                // [n_layers][K]: the selected ids in rank order, or null
    float* w_trace;                // [n_layers][K]: their renormalised weights, or null
    const __nv_bfloat16* teacher;  // [n_layers][D]: layer L's input in place of layer L-1's output, or null
    int* status;
    int n_layers;
    SKLayer L[kSKMaxLayers];
    // Per layer: the router [E][D] and the gate vector [1][D] as 2-D tensors
    // for TMA copies of a worker's column slice (boxes of kRColW columns).
    CUtensorMap rmap[kSKMaxLayers];
    CUtensorMap gmap[kSKMaxLayers];
};

// Shared-memory carve-up (byte offsets), a function of the shape.
struct SKLayout {
    int NSQ, NP, NJ, NJR;
    unsigned xq, xs, rcol, xo, sgu, sdn, gbuf, ubuf, dbuf, hq, hs, gp, up, sgp, sup, dpart, cand, wmax, red, tkv,
        tki, misc, bars, total;
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

// Column splits of a gate|up row pair over warps: one 32-value sub-block of
// each row per lane.
__host__ __device__ constexpr int sk_splits(int D) { return D / 1024; }

__host__ __device__ constexpr SKLayout sk_layout(int D, int I, int E, int K, int n) {
    SKLayout s{};
    const unsigned RB = (unsigned)(D / 256) * 136, DRB = (unsigned)sk_down_row_bytes(I);
    const unsigned NSB = D / 32, NSBH = I / 32, SPL = (unsigned)sk_splits(D);
    s.NSQ = (I + n - 1) / n;
    s.NP = (K * I + n - 1) / n;
    s.NJ = (D + n - 1) / n;
    // Down rows whose size is not a multiple of 16 bytes are copied in pairs
    // from an even row, so that every bulk copy starts 16-byte aligned: up
    // to two extra rows per slot, and an even row count keeps slots aligned.
    s.NJR = DRB % 16 ? (s.NJ + 3) & ~1 : s.NJ;
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
    s.gp = sk_take(o, s.NP * SPL * 4);
    s.up = sk_take(o, s.NP * SPL * 4);
    s.sgp = sk_take(o, s.NSQ * SPL * 4);
    s.sup = sk_take(o, s.NSQ * SPL * 4);
    s.dpart = sk_take(o, kSKWarps * 16 * 4);
    s.cand = sk_take(o, 256 * 8);
    s.wmax = sk_take(o, (kSKWarps + 1) * 8);
    s.red = sk_take(o, kSKWarps * 4);
    s.tkv = sk_take(o, kMaxTopK * 4);
    s.tki = sk_take(o, kMaxTopK * 4);
    s.misc = sk_take(o, 64);
    s.bars = sk_take(o, (5 + kSKMaxChunks) * 8);
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
    static constexpr int NW = NSM_;  // every CTA works
    static constexpr int DRB = sk_down_row_bytes(I_);
    static constexpr bool kPairRows = DRB % 16 != 0;
    static constexpr SKLayout S = sk_layout(D_, I_, E_, K_, NW);
    static_assert(E_ <= kSKThreads && E_ % 32 == 0, "one logit per thread");
    static_assert(I_ % 32 == 0 && I_ <= 512 && (I_ >= 256 ? I_ % 256 == 0 : 256 % I_ == 0), "intermediate slice");
    static_assert(K_ <= kMaxTopK && 2 * K_ < 32, "routing record: one word per lane");
    static_assert(K_ * I_ / NW + 1 <= I_, "a worker's routed rows span at most two experts");
    static_assert((K_ * I_ + NW - 1) / NW <= kSKChunk * kSKMaxChunks, "chunks of a worker's pairs");
    static_assert((D_ + NW - 1) / NW <= 16, "a lane per output row in the down phase");
    static_assert((D_ + NW - 1) / NW + 3 <= kRColW, "router column slice: one box per worker");
    static_assert(D_ % 1024 == 0 && kSKWarps % (D_ / 1024) == 0, "gate|up column splits");
    static_assert((K_ * I_ + NW - 1) / NW <= kSKThreads, "h writers");
    static_assert(D_ % 2 == 0, "down rows copied in pairs");
    static_assert(S.total <= 227u * 1024u, "shared memory of one CTA");
};

namespace {

using ptx::mbar_expect_tx;
using ptx::mbar_init;
using ptx::mbar_test;
using ptx::now_ns;

// ---- memory-model helpers ------------------------------------------------
__device__ __forceinline__ unsigned ld_relaxed_u32(const unsigned* p) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ double ld_relaxed_f64(const double* p) {
    double v;
    asm volatile("ld.relaxed.gpu.global.f64 %0, [%1];" : "=d"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_u32(unsigned* p, unsigned v) {
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

// Bounded wait for the phase of `bar` with parity `par`; false on timeout.
__device__ bool mbar_wait(uint64_t* bar, uint32_t par) {
    if (mbar_test(bar, par)) return true;
    const unsigned long long t0 = now_ns();
    while (!ptx::mbar_test_sleep(bar, par, 20000u)) {
        if (now_ns() - t0 > kTimeoutNs) return false;
    }
    return true;
}

// Phase trace: thread `rec` (0 unless stated) of worker 0 and of the routing
// CTA stamp their SM's cycle counter (clock64) at each phase boundary.
__device__ __forceinline__ void trace_mark(const SKArgs& a, int L, int k, int rec = 0) {
#if defined(QMOE_SK_FULLTRACE)
    // development builds: every CTA, on the GPU-wide clock (ns)
    if (a.trace && (int)threadIdx.x == rec)
        a.trace[((size_t)L * kFullTraceCtas + blockIdx.x) * kTraceSlots + k] = now_ns();
#else
    if (a.trace && (int)threadIdx.x == rec) {
        if (blockIdx.x == 0) a.trace[L * kTraceSlots + k] = (unsigned long long)clock64();
        else if (blockIdx.x == gridDim.x - 1) a.trace[(64 + L) * kTraceSlots + k] = (unsigned long long)clock64();
    }
#endif
}

// The sync area as the kernel sees it.
struct SKSync {
    unsigned* abortw;
    unsigned* xcnt;              // logit-round counters: 8 words, 32 apart
    unsigned* hcnt;              // h-round counters
    double* logits;              // [3 buffers][E + 1 lines][16 doubles]: logit i at the start of line i
    unsigned* xw;                // the activation words [D]
    unsigned* hw;                // the h words [(K + 1) I]
};

__device__ __forceinline__ void sk_fail(const SKSync& s, int* status) {
    record_status(status, QMOE_ERR_TIMEOUT);
    atomicExch(s.abortw, 1u);
}

// A warp's wait loop: `more()` re-polls and returns true while something this
// lane needs is still missing.  Checks the abort word every 32 rounds and
// gives up after kTimeoutNs (recording the timeout).
template <class More>
__device__ __forceinline__ bool poll_warp(More more, const SKSync& s, int* status) {
    unsigned long long t0 = 0;
    for (unsigned it = 0;; ++it) {
        if (!__any_sync(0xffffffffu, more())) return true;
        if (it == 0) t0 = now_ns();
        __nanosleep(32);
        if ((it & 31u) == 31u) {
            unsigned ab = 0;
            if ((threadIdx.x & 31) == 0) ab = ld_relaxed_u32(s.abortw);
            if (__any_sync(0xffffffffu, ab != 0u)) return false;
            if (now_ns() - t0 > kTimeoutNs) {
                if ((threadIdx.x & 31) == 0) sk_fail(s, status);
                return false;
            }
        }
    }
}

// Arrival of worker c on a round's counters (one thread; every earlier write
// of the CTA ordered before it by the caller's barrier and the release).
__device__ __forceinline__ void arrive(unsigned* cnt, int c) {
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(cnt + 32 * (c & 7)) : "memory");
}

// One warp waits until round r (1-based) of nw workers is complete on the 8
// counters (lane i < 8 polls word i, whose workers number (nw - i + 7) / 8),
// then acquires.  Bounded; false on a timeout or an abort.
__device__ bool wait_round(const unsigned* cnt, unsigned r, int nw, const SKSync& s, int* status) {
    const int lane = threadIdx.x & 31;
    const unsigned target = lane < 8 && lane < nw ? r * (unsigned)((nw - lane + 7) / 8) : 0u;
    const unsigned* w = cnt + 32 * (lane & 7);
    const bool got = poll_warp(
        [&]() { return lane < 8 && (int)(ld_relaxed_u32(w) - target) < 0; }, s, status);
    fence_acq_rel_gpu();
    __syncwarp();
    return got;
}

// ---- the decode core --------------------------------------------------------
__device__ __forceinline__ int sk_dot(uint32_t q0, uint32_t q1, uint32_t q2, uint32_t q3, const int* xp) {
#if defined(QMOE_SK_CORE_MASK)
    return qmoe_subblock_dot(q0, q1, q2, q3, xp, 0);
#else
    return qmoe_subblock_dot_t2(q0, q1, q2, q3, xp, 0);
#endif
}

// Sub-block sb of a gate row and of an up row dotted with the activation's
// block sb (16 pair words + step in registers), scaled: the lane's shares of
// the two row sums.
__device__ __forceinline__ void pair_dot(const uint8_t* rg, const uint8_t* ru, int sb, const int (&xr)[16], float xst,
                                         float& g, float& u) {
    const uint8_t* bg = rg + (sb >> 3) * QMOE_SB_BYTES;
    const uint8_t* bu = ru + (sb >> 3) * QMOE_SB_BYTES;
    const int ib = sb & 7;
    const uint2 hg = *reinterpret_cast<const uint2*>(bg);
    const uint2 hu = *reinterpret_cast<const uint2*>(bu);
    const uint2 g0 = *reinterpret_cast<const uint2*>(bg + 8 + 16 * ib);
    const uint2 g1 = *reinterpret_cast<const uint2*>(bg + 16 + 16 * ib);
    const uint2 u0 = *reinterpret_cast<const uint2*>(bu + 8 + 16 * ib);
    const uint2 u1 = *reinterpret_cast<const uint2*>(bu + 16 + 16 * ib);
    const int Sg = sk_dot(g0.x, g0.y, g1.x, g1.y, xr);
    const int Su = sk_dot(u0.x, u0.y, u1.x, u1.y, xr);
    const float dg = __half2float(__ushort_as_half((unsigned short)(hg.x & 0xFFFFu))) *
                     (float)(qmoe_iq4xs_ls(hg.x, hg.y, ib) - 32);
    const float du = __half2float(__ushort_as_half((unsigned short)(hu.x & 0xFFFFu))) *
                     (float)(qmoe_iq4xs_ls(hu.x, hu.y, ib) - 32);
    g = (dg * xst) * (float)Sg;
    u = (du * xst) * (float)Su;
}

// The two row sums of a warp (lane values g, u): lanes 0..15 end with the
// sum of g, lanes 16..31 with the sum of u (six shuffles).
__device__ __forceinline__ float pair_reduce(float g, float u, int lane) {
    const float og = __shfl_xor_sync(0xffffffffu, g, 16);
    const float ou = __shfl_xor_sync(0xffffffffu, u, 16);
    float v = lane < 16 ? g + og : u + ou;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Sub-block t of one down row dotted with its slot's activation block (hq in
// the [quad][sub-block][4 words] layout), scaled: d*(ls-32) * step * S.  A
// row of whole super-blocks has ib0 = 0; a rank's slice of fewer than 8
// sub-blocks stores them after the super-block's header and takes its scales
// from sub-block ib0 on.
__device__ __forceinline__ float down_unit(const uint8_t* row, const int* hq, float hstep, int nsbh, int t, int ib0) {
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
    const int Sd = sk_dot(q0.x, q0.y, q1.x, q1.y, xp);
    const float dl = __half2float(__ushort_as_half((unsigned short)(hdr.x & 0xFFFFu))) *
                     (float)(qmoe_iq4xs_ls(hdr.x, hdr.y, ib0 + ib) - 32);
    return (dl * hstep) * (float)Sd;
}

// Shape-derived constants and a worker's static slices.
struct SKPart {
    int D, I, E, K, RB, DRB, NSBH;
    size_t GUE, DNE;
    int sq_lo, sq_hi, p_lo, p_hi, j_lo, j_hi;
    int jc_lo, jc_hi;  // down rows copied: [j_lo, j_hi), widened to even bounds for rows of 8 mod 16 bytes
};

template <class SH>
__device__ __forceinline__ SKPart sk_part() {
    SKPart p;
    constexpr int n = SH::NW;
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

// Shared-expert gate|up rows of this worker's slice (one thread).
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

// Shared-expert down rows of this worker's output slice (one thread).
__device__ __forceinline__ void issue_sdn(const SKLayer& W, const SKPart& p, const SKLayout& S, unsigned char* sm,
                                          uint64_t* bar) {
    const int nc = p.jc_hi - p.jc_lo;
    mbar_expect_tx(bar, (uint32_t)(nc * p.DRB));
    if (nc > 0) ptx::bulk_g2s(sm + S.sdn, W.sh_down + (size_t)p.jc_lo * p.DRB, (uint32_t)(nc * p.DRB), bar);
}

// Router columns of this worker's output rows, for every router row and the
// gate vector (row E), as 2-D tensor copies (one thread): boxes of kRColW
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
// columns outside this worker's rows hold x = 0 and add exact zeros, so the
// sum runs over its columns in order, as a plain loop over them would
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

// This worker's share of the router logits: thread e (and thread 0 for the
// gate row E) sums rcol[e][j] * x[j] over its columns j in fp32 and adds it to
// logit e's fp64 accumulator, one per 128-byte line.
__device__ __forceinline__ void router_partial(const SKPart& p, const SKLayout& S, const unsigned char* sm,
                                               double* acc) {
    const float4* x4 = reinterpret_cast<const float4*>(sm + S.xo);
    const float* rcol = reinterpret_cast<const float*>(sm + S.rcol);
    const int e = threadIdx.x;
    const int gate_row = ((p.E + kRBoxRows - 1) / kRBoxRows) * kRBoxRows;
    if (e < p.E) {
        const float v = rcol_dot(rcol + e * kRColW, x4);
        asm volatile("red.global.add.f64 [%0], %1;" ::"l"(acc + (size_t)e * 16), "d"((double)v) : "memory");
    }
    if (e == 0) {
        const float g = rcol_dot(rcol + gate_row * kRColW, x4);
        asm volatile("red.global.add.f64 [%0], %1;" ::"l"(acc + (size_t)p.E * 16), "d"((double)g) : "memory");
    }
}

// This worker's routed pairs [p_lo, p_hi) fall in at most two expert slots: the
// first len0 pairs in the first.
__device__ __forceinline__ int seg0_len(const SKPart& p) {
    const int np = p.p_hi - p.p_lo, r0 = p.p_lo % p.I;
    return np < p.I - r0 ? np : p.I - r0;
}

// Chunk c of this worker's routed pairs (kSKChunk pairs; gate rows into gbuf,
// up rows into ubuf, both in pair order), completing on bar (one thread).
// A chunk that crosses the expert boundary is two pieces per half.
__device__ __forceinline__ void issue_chunk(const SKLayer& W, const SKPart& p, const SKLayout& S, unsigned char* sm,
                                            const int* ids, int c, uint64_t* bar) {
    const int np = p.p_hi - p.p_lo, len0 = seg0_len(p);
    const int u0 = c * kSKChunk, u1 = min(u0 + kSKChunk, np);
    mbar_expect_tx(bar, (uint32_t)(2 * (u1 - u0) * p.RB));
    int a = u0;
    while (a < u1) {
        const int b = a < len0 ? min(u1, len0) : u1;  // one piece inside one expert
        const int pp = p.p_lo + a, s = pp / p.I, r = pp - s * p.I;
        const uint8_t* base = W.gate_up + (size_t)ids[s] * p.GUE;
        const uint32_t bytes = (uint32_t)((b - a) * p.RB);
        ptx::bulk_g2s(sm + S.gbuf + (size_t)a * p.RB, base + (size_t)r * p.RB, bytes, bar);
        ptx::bulk_g2s(sm + S.ubuf + (size_t)a * p.RB, base + (size_t)(p.I + r) * p.RB, bytes, bar);
        a = b;
    }
}

// The selected experts' rows of this worker's output slice of their down, one
// copy per slot, issued by lanes 0..K-1 of one warp (lane 0 posts the bytes).
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
    constexpr SKLayout S = SH::S;
    constexpr int D = SH::D, I = SH::I, E = SH::E, K = SH::K, NW = SH::NW;
    constexpr int NSB = D / 32, NSBH = I / 32, NH = (K + 1) * I, NHB = NH / 32;
    constexpr int SPL = sk_splits(D), NSTREAM = kSKWarps / SPL;
    constexpr size_t G = (size_t)(E + 1) * 16;  // doubles per logit buffer
    static_assert(NH * 4 <= (int)(S.ubuf - S.gbuf) + S.NP * (D / 256) * 136, "h words staged in the gate|up buffers");
    static_assert(D * 4 <= (((E + kRBoxRows - 1) / kRBoxRows) * kRBoxRows + 1) * kRColW * 4,
                  "activation words staged in the router-column buffer");

    const SKPart p = sk_part<SH>();
    const int nsq = p.sq_hi - p.sq_lo, np = p.p_hi - p.p_lo, nj = p.j_hi - p.j_lo;
    const int nch = (np + kSKChunk - 1) / kSKChunk;
    const int c = blockIdx.x;
    int* xq = reinterpret_cast<int*>(sm + S.xq);
    float* xs = reinterpret_cast<float*>(sm + S.xs);
    // xo: x over the router-column window [j_lo & ~3, +kRColW); row j of this
    // CTA's slice at xo[xwin + j], the rest zero
    float* xo = reinterpret_cast<float*>(sm + S.xo);
    const int xwin = p.j_lo & 3;
    unsigned* xstage = reinterpret_cast<unsigned*>(sm + S.rcol);  // the activation words, between uses of rcol
    unsigned* hstage = reinterpret_cast<unsigned*>(sm + S.gbuf);  // the h words, once the gate|up rows are used
    const uint8_t* sgu = sm + S.sgu;
    const uint8_t* sdn = sm + S.sdn;
    const uint8_t* gbuf = sm + S.gbuf;
    const uint8_t* ubuf = sm + S.ubuf;
    const uint8_t* dbuf = sm + S.dbuf;
    int* hq = reinterpret_cast<int*>(sm + S.hq);
    float* hs = reinterpret_cast<float*>(sm + S.hs);
    float* gp = reinterpret_cast<float*>(sm + S.gp);
    float* up = reinterpret_cast<float*>(sm + S.up);
    float* sgp = reinterpret_cast<float*>(sm + S.sgp);
    float* sup = reinterpret_cast<float*>(sm + S.sup);
    float* dpart = reinterpret_cast<float*>(sm + S.dpart);
    unsigned long long* cand = reinterpret_cast<unsigned long long*>(sm + S.cand);
    unsigned long long* wmax = reinterpret_cast<unsigned long long*>(sm + S.wmax);
    unsigned* red = reinterpret_cast<unsigned*>(sm + S.red);
    float* tkv = reinterpret_cast<float*>(sm + S.tkv);
    int* tki = reinterpret_cast<int*>(sm + S.tki);
    // s_misc: [0] ok flag, [1] launch counter, [2] exchange counter, [8] top-k count; float [12] the gate
    unsigned* s_misc = reinterpret_cast<unsigned*>(sm + S.misc);
    int* s_cnt = reinterpret_cast<int*>(sm + S.misc) + 8;
    float* s_gate = reinterpret_cast<float*>(sm + S.misc) + 12;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S.bars);
    uint64_t* bar_sgu = bars;
    uint64_t* bar_sdn = bars + 1;
    uint64_t* bar_rc = bars + 2;
    uint64_t* bar_dn = bars + 3;
    uint64_t* bar_h = bars + 4;
    uint64_t* bar_ch = bars + 5;
    constexpr int nbars = 5 + kSKMaxChunks;
    const int ib0 = SH::I >= 256 ? 0 : a.ib0;

    SKSync sy;
    sy.abortw = reinterpret_cast<unsigned*>(a.sync + kStackAbortOff);
    sy.xcnt = reinterpret_cast<unsigned*>(a.sync + kStackXCountOff);
    sy.hcnt = reinterpret_cast<unsigned*>(a.sync + kStackHCountOff);
    sy.logits = reinterpret_cast<double*>(a.sync + kStackLogitOff);
    sy.xw = reinterpret_cast<unsigned*>(a.sync + stack_xw_off(E));
    sy.hw = reinterpret_cast<unsigned*>(a.sync + stack_hw_off(E, D));

    if (tid == 0) {
        for (int i = 0; i < nbars; ++i) mbar_init(bars + i, 1);
        ptx::fence_mbar_init();
        s_misc[1] = ld_relaxed_u32(reinterpret_cast<const unsigned*>(a.sync));
        s_misc[2] = XC ? __ldcg(a.xepoch) : 0u;
    }
    __syncthreads();
    const unsigned lc = s_misc[1];      // this launch's counter (tags)
    const unsigned xepoch = s_misc[2];  // exchange launch counter (peer flags)
    auto stamp_of = [&](int L) { return lc * 64u + (unsigned)L + 1u; };
    // Phases issued (kept by thread 0 in registers), for the bounded drain.
    int iss_sgu = 0, iss_rc = 0, iss_sdn = 0, iss_routed = 0, iss_h = 0;
    bool ok = true;
    if (tid == 0) {
        issue_rcol(&a.rmap[0], &a.gmap[0], p, S, sm, bar_rc);
        issue_sgu(a.L[0], p, S, sm, bar_sgu);
        issue_sdn(a.L[0], p, S, sm, bar_sdn);
        iss_sgu = iss_rc = iss_sdn = 1;
    }

    // ---------------- prologue: layer 0's router logits --------------------
    if (tid < kRColW) {
        const int j = tid - xwin;
        const __nv_bfloat16* x0 = a.teacher ? a.teacher : a.x;
        xo[tid] = j >= 0 && j < nj ? __bfloat162float(x0[p.j_lo + j]) : 0.0f;
    }
    ok = !__syncthreads_or(!mbar_wait(bar_rc, 0));
    if (!ok && tid == 0) sk_fail(sy, a.status);
    if (ok) {
        router_partial(p, S, sm, sy.logits);
        __syncthreads();
        if (tid == 0) arrive(sy.xcnt, c);
    }

    for (int L = 0; L < a.n_layers && ok; ++L) {
        const SKLayer& W = a.L[L];
        const uint32_t par = (uint32_t)(L & 1);
        const bool last = L + 1 == a.n_layers;
        const unsigned stamp = stamp_of(L);
        double* lg = sy.logits + (size_t)(L % 3) * G;
        trace_mark(a, L, 0);

        // ---- routing: every CTA's logit partials of the layer are in ---------
        if (warp == 0) {
            const bool got = wait_round(sy.xcnt, (unsigned)(L + 1), NW, sy, a.status);
            if (lane == 0) s_misc[0] = got ? 1u : 0u;
        }
        __syncthreads();
        if (!s_misc[0]) {
            ok = false;
            break;
        }
        trace_mark(a, L, 1);
        {
            // logit i: the fp64 word at the start of line i
            auto logit_at = [&](int i) { return (float)ld_relaxed_f64(lg + (size_t)i * 16); };
            if (tid == 0) *s_gate = logit_at(E);
            const float lmax = block_topk_threshold(logit_at, E, K, cand, wmax, red, s_cnt, tkv, tki, []() {});
            if (warp == 0) {
                float ps = 0.0f;
                for (int i = 0; i < K; ++i) ps += tkv[i];
                const float inv = 1.0f / ps;
                __syncwarp();
                if (lane < K) tkv[lane] = tkv[lane] * inv;
                if (lane == 0) {
                    *s_gate = sigmoid(*s_gate);
                    if (!(fabsf(lmax) <= 3.0e38f)) record_status(a.status, QMOE_ERR_NOT_FINITE);
                }
                __syncwarp();
                if (a.ids_trace && c == 0 && lane < K) {
                    a.ids_trace[L * K + lane] = tki[lane];
                    a.w_trace[L * K + lane] = tkv[lane];
                }
                // all of this CTA's copies at once: the gate|up chunks (lane
                // c: chunk c), then the down rows (lanes 0..k-1)
                ptx::fence_proxy_async();  // every issuing lane
                if (lane < nch) issue_chunk(W, p, S, sm, tki, lane, bar_ch + lane);
                issue_down(W, p, S, sm, tki, bar_dn, lane);
                if (lane == 0) ++iss_routed;
            }
        }
        __syncthreads();
        trace_mark(a, L, 2);

        // ---- x_L: block floating point (xq, xs) ------------------------------
        // (complete: every CTA wrote its rows before arriving on the logit
        // counters this CTA acquired)
        {
            const unsigned t16 = stamp & 0xFFFFu;
            if (L > 0 && !a.teacher) {
                for (int i = tid * 4; i < D; i += kSKThreads * 4) {
                    uint4 v;
                    asm volatile("ld.relaxed.gpu.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                                 : "l"(sy.xw + i)
                                 : "memory");
                    *reinterpret_cast<uint4*>(xstage + i) = v;
                }
            } else {
                const __nv_bfloat16* src = a.teacher ? a.teacher + (size_t)L * D : a.x;
                for (int i = tid; i < D; i += kSKThreads) xstage[i] = (t16 << 16) | __bfloat16_as_ushort(src[i]);
            }
            __syncthreads();
            constexpr int XPW = (NSB + kSKWarps - 1) / kSKWarps;
            unsigned xv[XPW];
#pragma unroll
            for (int i = 0; i < XPW; ++i) {
                const int b = warp + i * kSKWarps;
                xv[i] = b < NSB ? xstage[b * 32 + lane] : (t16 << 16);
            }
            // the tags check what the counters guarantee (bounded, normally no round)
            const bool got = poll_warp(
                [&]() {
                    bool miss = false;
#pragma unroll
                    for (int i = 0; i < XPW; ++i) {
                        const int b = warp + i * kSKWarps;
                        if (b < NSB && (xv[i] >> 16) != t16) {
                            xv[i] = ld_relaxed_u32(sy.xw + b * 32 + lane);
                            miss = true;
                        }
                    }
                    return miss;
                },
                sy, a.status);
            if (got) {
#pragma unroll
                for (int i = 0; i < XPW; ++i) {
                    const int b = warp + i * kSKWarps;
                    if (b < NSB) {
                        float st;
                        const int pw =
                            warp_block_fp(__bfloat162float(__ushort_as_bfloat16((unsigned short)xv[i])), &st);
                        if (lane < 16) xq[b * 16 + lane] = pw;
                        if (lane == 0) xs[b] = st;
                    }
                }
            }
            if (__syncthreads_or(!got)) {
                ok = false;
                break;
            }
        }
        trace_mark(a, L, 3);
        // This warp's column split of every row pair: lane l owns sub-block
        // hf * 32 + l; the activation block in registers.
        const int hf = warp % SPL, stream = warp / SPL, sb = hf * 32 + lane;
        int xr[16];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int4 w4 = reinterpret_cast<const int4*>(xq + sb * 16)[q];
            xr[4 * q] = w4.x;
            xr[4 * q + 1] = w4.y;
            xr[4 * q + 2] = w4.z;
            xr[4 * q + 3] = w4.w;
        }
        const float xst = xs[sb];
        // ---- the shared expert's pairs (rows prefetched) --------------------
        if (__syncthreads_or(!mbar_wait(bar_sgu, par))) {
            if (tid == 0) sk_fail(sy, a.status);
            ok = false;
            break;
        }
        for (int t = stream; t < nsq; t += NSTREAM) {
            float g, u;
            pair_dot(sgu + (size_t)t * p.RB, sgu + (size_t)(S.NSQ + t) * p.RB, sb, xr, xst, g, u);
            const float v = pair_reduce(g, u, lane);
            if (lane == 0) sgp[t * SPL + hf] = v;
            if (lane == 16) sup[t * SPL + hf] = v;
        }
        trace_mark(a, L, 4);

        // ---- routed pairs as their chunks land, two per warp at a time ------
        for (int u = stream; u < np && ok; u += 2 * NSTREAM) {
            const int u2 = u + NSTREAM;
            const bool two = u2 < np;
            if (!mbar_wait(bar_ch + u / kSKChunk, par) || (two && !mbar_wait(bar_ch + u2 / kSKChunk, par))) {
                ok = false;
                break;
            }
            if (hf == 0 && u % kSKChunk == 0) trace_mark(a, L, 16 + min(u / kSKChunk, 5), 32 * warp);
            float g, v, g2 = 0.0f, v2 = 0.0f;
            pair_dot(gbuf + (size_t)u * p.RB, ubuf + (size_t)u * p.RB, sb, xr, xst, g, v);
            if (two) pair_dot(gbuf + (size_t)u2 * p.RB, ubuf + (size_t)u2 * p.RB, sb, xr, xst, g2, v2);
            const float r = pair_reduce(g, v, lane);
            const float r2 = pair_reduce(g2, v2, lane);
            if (lane == 0) gp[u * SPL + hf] = r;
            if (lane == 16) up[u * SPL + hf] = r;
            if (two && lane == 0) gp[u2 * SPL + hf] = r2;
            if (two && lane == 16) up[u2 * SPL + hf] = r2;
        }
        if (__syncthreads_or(!ok)) {
            if (tid == 0) sk_fail(sy, a.status);
            ok = false;
            break;
        }
        trace_mark(a, L, 5);
        // h words: the routed pairs, then the shared ones (slot K)
        if (tid < np + nsq) {
            const bool routed = tid < np;
            const int i = routed ? tid : tid - np;
            const float* gq = routed ? gp : sgp;
            const float* uq = routed ? up : sup;
            float gs = 0.0f, us = 0.0f;
            for (int q = 0; q < SPL; ++q) {
                gs += gq[i * SPL + q];
                us += uq[i * SPL + q];
            }
            const float h = silu(gs) * us;
            st_relaxed_u32(sy.hw + (routed ? p.p_lo + i : K * I + p.sq_lo + i),
                           (__float_as_uint(h) & 0xFFFFFF00u) | (stamp & 0xFFu));
        }
        __syncthreads();
        if (tid == 0) arrive(sy.hcnt, c);
        trace_mark(a, L, 6);

        // ---------------- phase C --------------------------------------------
        // Every CTA's h is in once the h round is complete: one bulk copy of
        // all of it into the (consumed) gate|up buffers, then the next layer's
        // prefetches behind it.
        if (warp == 0) {
            const bool got = wait_round(sy.hcnt, (unsigned)(L + 1), NW, sy, a.status);
            if (lane == 0) {
                s_misc[0] = got ? 1u : 0u;
                if (got) {
                    ptx::fence_proxy_async_global();  // the acquired h words, then the async-proxy read
                    ptx::fence_proxy_async();
                    mbar_expect_tx(bar_h, (uint32_t)(NH * 4));
                    ptx::bulk_g2s(hstage, sy.hw, (uint32_t)(NH * 4), bar_h);
                    ++iss_h;
                    if (!last) {
                        issue_sgu(a.L[L + 1], p, S, sm, bar_sgu);
                        issue_rcol(&a.rmap[L + 1], &a.gmap[L + 1], p, S, sm, bar_rc);
                        ++iss_sgu;
                        ++iss_rc;
                    }
                }
            }
        }
        __syncthreads();
        if (!s_misc[0]) {
            ok = false;
            break;
        }
        trace_mark(a, L, 7);
        // this CTA's lines of the accumulator two layers on: every CTA has read
        // it (layer L - 1's logits) before arriving on this h round
        for (int i = c + tid * NW; i <= E; i += kSKThreads * NW)
            sy.logits[(size_t)((L + 2) % 3) * G + (size_t)i * 16] = 0.0;
        {
            // the h words -> block floating point (hq, hs)
            if (__syncthreads_or(!mbar_wait(bar_h, par))) {
                if (tid == 0) sk_fail(sy, a.status);
                ok = false;
                break;
            }
            constexpr int HPW = (NHB + kSKWarps - 1) / kSKWarps;
            const unsigned t8 = stamp & 0xFFu;
            unsigned hv[HPW];
#pragma unroll
            for (int i = 0; i < HPW; ++i) {
                const int b = warp + i * kSKWarps;
                hv[i] = b < NHB ? hstage[b * 32 + lane] : t8;
            }
            const bool got = poll_warp(
                [&]() {
                    bool miss = false;
#pragma unroll
                    for (int i = 0; i < HPW; ++i) {
                        const int b = warp + i * kSKWarps;
                        if (b < NHB && (hv[i] & 0xFFu) != t8) {
                            hv[i] = ld_relaxed_u32(sy.hw + b * 32 + lane);
                            miss = true;
                        }
                    }
                    return miss;
                },
                sy, a.status);
            if (got) {
#pragma unroll
                for (int i = 0; i < HPW; ++i) {
                    const int b = warp + i * kSKWarps;
                    if (b < NHB) {
                        float st;
                        const int pw = warp_block_fp(__uint_as_float(hv[i] & 0xFFFFFF00u), &st);
                        const int slot = b / NSBH, t = b - slot * NSBH;
                        // word w = 4*quad + (w & 3) of block t of the slot
                        if (lane < 16) hq[slot * NSBH * 16 + ((lane >> 2) * NSBH + t) * 4 + (lane & 3)] = pw;
                        if (lane == 0) hs[b] = st;
                    }
                }
            }
            if (__syncthreads_or(!got)) {
                ok = false;
                break;
            }
        }
        trace_mark(a, L, 8);
        {
            const bool d_ok = mbar_wait(bar_dn, par) && mbar_wait(bar_sdn, par);
            if (__syncthreads_or(!d_ok)) {
                if (tid == 0) sk_fail(sy, a.status);
                ok = false;
                break;
            }
        }
        trace_mark(a, L, 9);
        // Down + combine: lane j (of 16) of a half-warp owns output row j; the
        // 32 half-warps split the (k + 1) * I / 32 (slot, sub-block) columns,
        // so a half-warp reads each column's activation words once (a
        // broadcast); per-row partials summed over the warps in warp order.
        {
            constexpr int NT = (K + 1) * NSBH;
            const int jr = lane & 15, grp = warp * 2 + (lane >> 4);
            const int t0 = grp * NT / (2 * kSKWarps), t1 = (grp + 1) * NT / (2 * kSKWarps);
            const int jo = p.j_lo - p.jc_lo;  // row j_lo's place in the copied rows
            float acc0 = 0.0f, acc1 = 0.0f, acc2 = 0.0f, acc3 = 0.0f;
            if (jr < nj) {
                auto unit = [&](int t) {
                    const int s = t / NSBH, b = t - s * NSBH;
                    const uint8_t* row =
                        s < K ? dbuf + ((size_t)s * S.NJR + jo + jr) * p.DRB : sdn + (size_t)(jo + jr) * p.DRB;
                    const float wgt = s < K ? tkv[s] : *s_gate;
                    return wgt * down_unit(row, hq + s * NSBH * 16, hs[t], NSBH, b, ib0);
                };
                int t = t0;
                for (; t + 3 < t1; t += 4) {  // four independent chains
                    acc0 += unit(t);
                    acc1 += unit(t + 1);
                    acc2 += unit(t + 2);
                    acc3 += unit(t + 3);
                }
                for (; t < t1; ++t) acc0 += unit(t);
            }
            float acc = (acc0 + acc1) + (acc2 + acc3);
            acc += __shfl_xor_sync(0xffffffffu, acc, 16);
            if (lane < 16) dpart[warp * 16 + lane] = acc;
        }
        __syncthreads();
        trace_mark(a, L, 10);
        // this CTA's rows of the layer output (partial sums when sharded)
        float v = 0.0f;
        if (tid < nj) {
            for (int w = 0; w < kSKWarps; ++w) v += dpart[w * 16 + tid];
        }
        // the shared down rows have been read: the next layer's stream in
        if (tid == 0 && !last) {
            ptx::fence_proxy_async();
            issue_sdn(a.L[L + 1], p, S, sm, bar_sdn);
            ++iss_sdn;
        }
        if constexpr (XC) {
            // this rank's partial of row j_lo + tid, stored into every peer as
            // one word (value bits, flag); then the R partials in rank order
            const unsigned fval = xepoch * 64u + (unsigned)L + 1u;
            const int xpar = (int)((xepoch * (unsigned)a.n_layers + (unsigned)L) & 1u);
            if (tid < nj) {
                for (int q = 0; q < a.R; ++q)
                    if (q != a.rank)
                        ptx::st_relaxed_sys_u64(a.xr[q] + ((size_t)(xpar * a.R + a.rank) * D + p.j_lo + tid),
                                                ((unsigned long long)fval << 32) | __float_as_uint(v));
            }
            trace_mark(a, L, 22);
            bool x_ok = true;
            if (tid < nj) {
                const unsigned long long* rx = a.xr[a.rank] + (size_t)xpar * a.R * D + p.j_lo + tid;
                float sum = 0.0f;
                for (int q = 0; q < a.R && x_ok; ++q) {
                    float pv;
                    if (q == a.rank) {
                        pv = v;
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
                    sum = q == 0 ? pv : sum + pv;
                }
                v = sum;
            }
            if (__syncthreads_or(!x_ok)) {
                if (tid == 0) sk_fail(sy, a.status);
                ok = false;
                break;
            }
            trace_mark(a, L, 23);
        }
        if (tid < nj) {
            const __nv_bfloat16 xb = __float2bfloat16_rn(v);
            if (last) a.out[p.j_lo + tid] = v;
            else st_relaxed_u32(sy.xw + p.j_lo + tid, ((stamp_of(L + 1) & 0xFFFFu) << 16) | __bfloat16_as_ushort(xb));
            if (a.act_trace) a.act_trace[(size_t)L * D + p.j_lo + tid] = xb;
            xo[xwin + tid] =
                __bfloat162float(a.teacher && !last ? a.teacher[(size_t)(L + 1) * D + p.j_lo + tid] : xb);
        }
        trace_mark(a, L, 11);
        if (last) break;
        // the next layer's router partial, then the arrival on the logit counters
        if (__syncthreads_or(!mbar_wait(bar_rc, (uint32_t)((L + 1) & 1)))) {
            if (tid == 0) sk_fail(sy, a.status);
            ok = false;
            break;
        }
        router_partial(p, S, sm, sy.logits + (size_t)((L + 1) % 3) * G);
        __syncthreads();
        if (tid == 0) arrive(sy.xcnt, c);
        trace_mark(a, L, 12);
    }

    // The launch counters, read by every CTA at its start (before its first
    // arrival, which every CTA waits for before its first layer).
    if (c == 0 && tid == 0) {
        st_relaxed_u32(reinterpret_cast<unsigned*>(a.sync), lc + 1u);
        if (XC) *a.xepoch = xepoch + 1u;
    }

    // Stopped early: let this CTA's copies in flight land (bounded) before exit.
    if (!ok && tid == 0) {
        if (iss_sgu > 0) (void)mbar_wait(bar_sgu, (uint32_t)((iss_sgu - 1) & 1));
        if (iss_rc > 0) (void)mbar_wait(bar_rc, (uint32_t)((iss_rc - 1) & 1));
        if (iss_sdn > 0) (void)mbar_wait(bar_sdn, (uint32_t)((iss_sdn - 1) & 1));
        if (iss_h > 0) (void)mbar_wait(bar_h, (uint32_t)((iss_h - 1) & 1));
        if (iss_routed > 0) {
            const uint32_t q = (uint32_t)((iss_routed - 1) & 1);
            (void)mbar_wait(bar_dn, q);
            for (int ch = 0; ch < nch; ++ch) (void)mbar_wait(bar_ch + ch, q);
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

cudaError_t launch_stack_kernel(const void* x, float* out, unsigned char* sync, unsigned long long* trace,
                                int* status, const qmoe_layer_weights* layers, int n_layers, const qmoe_dims& d,
                                const XchgDesc* xc, const StackTraceBufs& tb, cudaStream_t stream) {
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
        a.xepoch = reinterpret_cast<unsigned*>(xc->buf[xc->rank]);
    }
    a.trace = trace;
    a.x = reinterpret_cast<const __nv_bfloat16*>(x);
    a.out = out;
    a.sync = sync;
    a.status = status;
    a.n_layers = n_layers;
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
    cudaError_t err = smem_opt_in(reinterpret_cast<const void*>(kern), (int)smem);
    if (err != cudaSuccess) return err;
    // The abort word, the round counters and the three logit accumulators
    // start at zero for every launch; the launch counter (offset 0) and the
    // tagged words are kept.
    err = cudaMemsetAsync(sync + kStackAbortOff, 0, kStackLogitOff + stack_logit_bytes(d.n_experts) - kStackAbortOff,
                          stream);
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
