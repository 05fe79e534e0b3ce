// The whole batch-1 MoE decode stack in one persistent launch.
//
// One 512-thread CTA per SM (a cooperative launch, so all are co-resident and
// may wait on one another), every CTA doing the same work on its own slices.
// Every layer is the reference's `_moe` (reference/model.py:387-417):
//
//   A        every CTA gathers the layer input x (the D activation words
//            that all CTAs published at the end of the last layer),
//            converts it to block floating point, computes its own few of
//            the E + 1 router logits (the expert rows and the gate vector
//            are split over the CTAs, each row a fixed-order fp32 dot
//            product with x) and publishes them as words; then it gathers
//            all E + 1 and ranks them itself (block top-k on the softmax
//            numerators, ties to the lower id): the same logits give every
//            CTA the same experts.
//   B        a CTA starts the copies of its fixed slice of the k * I routed
//            (gate row, up row) pairs of the selected experts (cp.async.bulk
//            into shared memory, an mbarrier per chunk, several lanes
//            issuing), decodes its slice of the shared expert's pairs (rows
//            prefetched), then the routed pairs as their chunks land, each
//            pair split over D / 1024 warps (one 32-value sub-block of each
//            row per lane), two pairs at a time per warp, decoded from IQ4_XS
//            in registers; SwiGLU; its h values go out as words, and it
//            starts the copies of its rows of the selected experts' down
//            projections.
//   C        once every CTA's h is in, a CTA copies all (k + 1) * I h words
//            into shared memory with one bulk copy, converts them to block
//            floating point, starts the next layer's prefetches (shared
//            gate|up rows, its router rows), computes its D / 148 output rows
//            of the routed experts' weighted down projections plus the gated
//            shared expert, and publishes them as the next layer's
//            activation words.
//
// Every word one CTA publishes for others carries a tag derived from the
// layer's stamp, launch_counter * 64 + layer + 1 (the counter lives in the
// workspace and advances every launch): activation words are bf16 with a
// 16-bit tag, logit words fp32 with the whole stamp beside it, h words fp32
// with their low 8 mantissa bits replaced by an 8-bit tag (the block floating
// point they feed keeps 14 bits of the block maximum).  A reader checks the
// tags and re-reads what is not yet there, so no fence orders the data: each
// round (activation, logits, h) also has arrival counters (8 words on
// separate lines; a CTA adds 1 to word c % 8 after its words, relaxed; a
// waiter's 8 lanes poll them) that only say when to start reading, so that
// the CTAs do not poll the data itself.  Each logit is one
// CTA's fixed-order sum, so reruns give the same bits and every rank of a
// sharded stack selects the same experts.
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
#include "common.cuh"
#include "ptx.cuh"
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
constexpr int kSKMaxRRows = 4;   // router rows (logits) per CTA

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
    unsigned long long* trace;     // phase stamps of CTA 0 and the last CTA, or null
    __nv_bfloat16* act_trace;      // [n_layers][D]: every layer's output rounded to bf16, or null
    int* ids_trace;                // [n_layers][K]: the selected ids in rank order, or null
    float* w_trace;                // [n_layers][K]: their renormalised weights, or null
    const __nv_bfloat16* teacher;  // [n_layers][D]: layer L's input in place of layer L-1's output, or null
    int* status;
    int n_layers;
    SKLayer L[kSKMaxLayers];
};

// Shared-memory carve-up (byte offsets), a function of the shape.
struct SKLayout {
    int NSQ, NP, NJ, NJR;
    unsigned xq, xs, xstage, rrow, rpart, sgu, sdn, gbuf, ubuf, dbuf, hq, hs, gp, up, sgp, sup, dpart, cand,
        wmax, red, lf, tkv, tki, misc, bars, total;
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
    s.xstage = sk_take(o, (unsigned)D * 4);                   // the activation words
    s.rrow = sk_take(o, (unsigned)kSKMaxRRows * D * 4);       // this CTA's router rows
    s.rpart = sk_take(o, (unsigned)kSKWarps * kSKMaxRRows * 4);
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
    s.cand = sk_take(o, kCandCap * 8);  // the top-k's candidates
    s.wmax = sk_take(o, kSKWarps * 8);
    s.red = sk_take(o, kSKWarps * 4);
    s.lf = sk_take(o, (unsigned)E * 4);  // the logits
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
    static_assert(E_ <= kSKThreads && E_ % 32 == 0 && E_ >= kSKWarps, "one logit per thread");
    static_assert(I_ % 32 == 0 && I_ <= 512 && (I_ >= 256 ? I_ % 256 == 0 : 256 % I_ == 0), "intermediate slice");
    static_assert(K_ <= kMaxTopK && K_ <= kSKWarps && 2 * K_ < 32, "top-k");
    static_assert(K_ * I_ / NW + 1 <= I_, "a worker's routed rows span at most two experts");
    static_assert((K_ * I_ + NW - 1) / NW <= kSKChunk * kSKMaxChunks, "chunks of a worker's pairs");
    static_assert((D_ + NW - 1) / NW <= 16, "a lane per output row in the down phase");
    static_assert((E_ + 1 + NW - 1) / NW <= kSKMaxRRows, "router rows per CTA");
    static_assert(D_ % kSKThreads == 0 && D_ / kSKThreads <= 4, "router dot: columns per thread");
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
__device__ __forceinline__ uint4 ld_relaxed_v4(const unsigned* p) {
    uint4 v;
    asm volatile("ld.relaxed.gpu.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_u32(unsigned* p, unsigned v) {
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Bounded wait for the phase of `bar` with parity `par`; false on timeout.
__device__ bool mbar_wait(uint64_t* bar, uint32_t par) {
    if (mbar_test(bar, par)) return true;
    const unsigned long long t0 = now_ns();
    while (!ptx::mbar_test_sleep(bar, par, 20000u)) {
        if (now_ns() - t0 > kTimeoutNs) return false;
    }
    return true;
}

// Phase trace: thread `rec` (0 unless stated) of CTA 0 and of the last CTA
// stamp their SM's cycle counter (clock64) at each phase boundary.
__device__ __forceinline__ void trace_mark(const SKArgs& a, int L, int k, int rec = 0) {
#if defined(QMOE_SK_FULLTRACE)
    // development builds: every CTA; slot 13 holds the GPU-wide clock (ns)
    // taken with slot 0, to place the CTAs' cycle counts on one time line
    if (a.trace && (int)threadIdx.x == rec)
        a.trace[((size_t)L * kFullTraceCtas + blockIdx.x) * kTraceSlots + k] =
            k == 13 ? now_ns() : (unsigned long long)clock64();
#else
    if (a.trace && (int)threadIdx.x == rec) {
        if (blockIdx.x == 0) a.trace[L * kTraceSlots + k] = (unsigned long long)clock64();
        else if (blockIdx.x == gridDim.x - 1) a.trace[(64 + L) * kTraceSlots + k] = (unsigned long long)clock64();
    }
#endif
}

// Development-build stamps (slots the product build leaves to the exchange
// or unused).
__device__ __forceinline__ void dev_mark(const SKArgs& a, int L, int k, int rec = 0) {
#if defined(QMOE_SK_FULLTRACE)
    trace_mark(a, L, k, rec);
#endif
}

// The sync area as the kernel sees it.
struct SKSync {
    unsigned* abortw;
    unsigned* xcnt;           // activation-round counters: 8 words, 32 apart
    unsigned* hcnt;           // h-round counters
    unsigned* lcnt;           // logit-round counters
    unsigned long long* lw;   // the logit words [E + 1]: fp32 bits | stamp << 32
    unsigned* xw;             // the activation words [D]
    unsigned* hw;             // the h words [(K + 1) I]
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

// Arrival of worker c on a round's counters (one thread, after the CTA's
// words of the round: a hint for when to read them, the tags decide).
__device__ __forceinline__ void arrive(unsigned* cnt, int c) {
    asm volatile("red.relaxed.gpu.global.add.u32 [%0], 1;" ::"l"(cnt + 32 * (c & 7)) : "memory");
}

// One warp waits until round r (1-based) of nw workers is complete on the 8
// counters (lane i < 8 polls word i, whose workers number (nw - i + 7) / 8).
// Bounded; false on a timeout or an abort.
__device__ bool wait_round(const unsigned* cnt, unsigned r, int nw, const SKSync& s, int* status) {
    const int lane = threadIdx.x & 31;
    const unsigned target = lane < 8 && lane < nw ? r * (unsigned)((nw - lane + 7) / 8) : 0u;
    const unsigned* w = cnt + 32 * (lane & 7);
    return poll_warp([&]() { return lane < 8 && (int)(ld_relaxed_u32(w) - target) < 0; }, s, status);
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
    int e_lo, e_hi;    // router logits [e_lo, e_hi) of the E + 1 (row E: the gate vector)
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
    p.e_lo = c * (SH::E + 1) / n;
    p.e_hi = (c + 1) * (SH::E + 1) / n;
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

// This CTA's router rows of a layer (one thread): rows [e_lo, e_hi) of the
// router, the gate vector in place of row E.
__device__ __forceinline__ void issue_rrow(const SKLayer& W, const SKPart& p, const SKLayout& S, unsigned char* sm,
                                           uint64_t* bar) {
    const int ne = p.e_hi - p.e_lo, nr = min(p.e_hi, p.E) - p.e_lo;
    float* rrow = reinterpret_cast<float*>(sm + S.rrow);
    mbar_expect_tx(bar, (uint32_t)(ne * p.D * 4));
    if (nr > 0) ptx::bulk_g2s(rrow, W.router + (size_t)p.e_lo * p.D, (uint32_t)(nr * p.D * 4), bar);
    if (p.e_hi > p.E) ptx::bulk_g2s(rrow + (size_t)(p.E - p.e_lo) * p.D, W.gate_vec, (uint32_t)(p.D * 4), bar);
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
    static_assert(NH * 4 <= (int)(S.ubuf - S.gbuf) + S.NP * (D / 256) * 136, "h words staged in the gate|up buffers");

    const SKPart p = sk_part<SH>();
    const int nsq = p.sq_hi - p.sq_lo, np = p.p_hi - p.p_lo, nj = p.j_hi - p.j_lo, ne = p.e_hi - p.e_lo;
    const int nch = (np + kSKChunk - 1) / kSKChunk;
    const int c = blockIdx.x;
    int* xq = reinterpret_cast<int*>(sm + S.xq);
    float* xs = reinterpret_cast<float*>(sm + S.xs);
    unsigned* xstage = reinterpret_cast<unsigned*>(sm + S.xstage);
    const float* rrow = reinterpret_cast<const float*>(sm + S.rrow);
    float* rpart = reinterpret_cast<float*>(sm + S.rpart);
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
    float* lf = reinterpret_cast<float*>(sm + S.lf);
    int* s_cnt = reinterpret_cast<int*>(sm + S.misc) + 8;
    float* tkv = reinterpret_cast<float*>(sm + S.tkv);
    int* tki = reinterpret_cast<int*>(sm + S.tki);
    // s_misc: [0] ok flag, [1] launch counter, [2] exchange counter, [3] down
    // copies issued (by the last warp), [8] top-k candidates; float [12] the gate
    unsigned* s_misc = reinterpret_cast<unsigned*>(sm + S.misc);
    float* s_gate = reinterpret_cast<float*>(sm + S.misc) + 12;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S.bars);
    uint64_t* bar_sgu = bars;
    uint64_t* bar_sdn = bars + 1;
    uint64_t* bar_rr = bars + 2;
    uint64_t* bar_dn = bars + 3;
    uint64_t* bar_h = bars + 4;
    uint64_t* bar_ch = bars + 5;
    constexpr int nbars = 5 + kSKMaxChunks;
    const int ib0 = SH::I >= 256 ? 0 : a.ib0;

    SKSync sy;
    sy.abortw = reinterpret_cast<unsigned*>(a.sync + kStackAbortOff);
    sy.xcnt = reinterpret_cast<unsigned*>(a.sync + kStackXCountOff);
    sy.hcnt = reinterpret_cast<unsigned*>(a.sync + kStackHCountOff);
    sy.lcnt = reinterpret_cast<unsigned*>(a.sync + kStackLCountOff);
    sy.lw = reinterpret_cast<unsigned long long*>(a.sync + kStackLogitOff);
    sy.xw = reinterpret_cast<unsigned*>(a.sync + stack_xw_off(E));
    sy.hw = reinterpret_cast<unsigned*>(a.sync + stack_hw_off(E, D));

    if (tid == 0) {
        for (int i = 0; i < nbars; ++i) mbar_init(bars + i, 1);
        ptx::fence_mbar_init();
        s_misc[1] = ld_relaxed_u32(reinterpret_cast<const unsigned*>(a.sync));
        s_misc[2] = XC ? __ldcg(a.xepoch) : 0u;
        s_misc[3] = 0u;
    }
    __syncthreads();
    const unsigned lc = s_misc[1];      // this launch's counter (tags)
    const unsigned xepoch = s_misc[2];  // exchange launch counter (peer flags)
    auto stamp_of = [&](int L) { return lc * 64u + (unsigned)L + 1u; };
    // Phases issued (kept by thread 0 in registers), for the bounded drain.
    int iss_sgu = 0, iss_rr = 0, iss_sdn = 0, iss_gu = 0, iss_h = 0;
    bool ok = true;
    if (tid == 0) {
        issue_rrow(a.L[0], p, S, sm, bar_rr);
        issue_sgu(a.L[0], p, S, sm, bar_sgu);
        issue_sdn(a.L[0], p, S, sm, bar_sdn);
        iss_sgu = iss_rr = iss_sdn = 1;
    }

    for (int L = 0; L < a.n_layers && ok; ++L) {
        const SKLayer& W = a.L[L];
        const uint32_t par = (uint32_t)(L & 1);
        const bool last = L + 1 == a.n_layers;
        const unsigned stamp = stamp_of(L);
        const unsigned t16 = stamp & 0xFFFFu;
        trace_mark(a, L, 0);
        dev_mark(a, L, 13);

        // ---- A: x_L, this CTA's logits, all logits, the experts -------------
        if (L > 0 && !a.teacher) {
            // every CTA's output rows of the last layer: the counters say when
            // to read, the tags check what was read
            if (warp == 0) {
                const bool got = wait_round(sy.xcnt, (unsigned)L, NW, sy, a.status);
                if (lane == 0) s_misc[0] = got ? 1u : 0u;
            }
            __syncthreads();
            if (!s_misc[0]) {
                ok = false;
                break;
            }
            for (int i = tid * 4; i < D; i += kSKThreads * 4)
                *reinterpret_cast<uint4*>(xstage + i) = ld_relaxed_v4(sy.xw + i);
        } else {
            const __nv_bfloat16* src = a.teacher ? a.teacher + (size_t)L * D : a.x;
            for (int i = tid; i < D; i += kSKThreads) xstage[i] = (t16 << 16) | __bfloat16_as_ushort(src[i]);
        }
        __syncthreads();
        trace_mark(a, L, 1);
        {
            // the tags: bounded re-reads of what is missing, written back
            constexpr int XPW = (NSB + kSKWarps - 1) / kSKWarps;
            unsigned xv[XPW];
#pragma unroll
            for (int i = 0; i < XPW; ++i) {
                const int b = warp + i * kSKWarps;
                xv[i] = b < NSB ? xstage[b * 32 + lane] : (t16 << 16);
            }
            bool miss_any = false;
            bool got = poll_warp(
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
                    miss_any = miss_any || miss;
                    return miss;
                },
                sy, a.status);
            if (__any_sync(0xffffffffu, miss_any)) {
#pragma unroll
                for (int i = 0; i < XPW; ++i) {
                    const int b = warp + i * kSKWarps;
                    if (b < NSB) xstage[b * 32 + lane] = xv[i];
                }
            }
            const bool rr_ok = mbar_wait(bar_rr, par);
            if (!rr_ok && tid == 0) sk_fail(sy, a.status);
            if (__syncthreads_or(!got || !rr_ok)) {
                ok = false;
                break;
            }
        }
        trace_mark(a, L, 2);
        {
            // this CTA's logits: each a fixed-order fp32 dot product (a
            // thread's CPT columns in order, the warp's lanes by a butterfly,
            // the warps in order), published as words
            constexpr int CPT = D / kSKThreads;
            float xf[CPT];
#pragma unroll
            for (int j = 0; j < CPT; ++j)
                xf[j] = __bfloat162float(__ushort_as_bfloat16((unsigned short)xstage[tid * CPT + j]));
            float acc[kSKMaxRRows];
#pragma unroll
            for (int r = 0; r < kSKMaxRRows; ++r) {
                acc[r] = 0.0f;
                if (r < ne) {
#pragma unroll
                    for (int j = 0; j < CPT; ++j) acc[r] = fmaf(rrow[(size_t)r * D + tid * CPT + j], xf[j], acc[r]);
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
                for (int r = 0; r < kSKMaxRRows; ++r) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
            }
            if (lane < kSKMaxRRows) {
                float mine = acc[0];
#pragma unroll
                for (int r = 1; r < kSKMaxRRows; ++r) mine = lane == r ? acc[r] : mine;
                rpart[warp * kSKMaxRRows + lane] = mine;
            }
            __syncthreads();
            if (warp == 0) {
                if (lane < ne) {
                    float v = 0.0f;
                    for (int w = 0; w < kSKWarps; ++w) v += rpart[w * kSKMaxRRows + lane];
                    st_relaxed_u64(sy.lw + p.e_lo + lane, ((unsigned long long)stamp << 32) | __float_as_uint(v));
                }
                __syncwarp();
                if (lane == 0) arrive(sy.lcnt, c);
            }
        }
        dev_mark(a, L, 22);
        // Every logit once the round is counted in (thread t: logit t, thread
        // 0 also the gate's; tags checked), into lf[] with each warp's
        // largest in red[].
        if (warp == 0) {
            const bool got = wait_round(sy.lcnt, (unsigned)(L + 1), NW, sy, a.status);
            if (lane == 0) s_misc[0] = got ? 1u : 0u;
        }
        __syncthreads();
        if (!s_misc[0]) {
            ok = false;
            break;
        }
        {
            unsigned long long w = 0ull, wg = 0ull;
            bool have = tid >= E, hg = tid != 0;
            const bool got = poll_warp(
                [&]() {
                    if (!have) w = ld_relaxed_u64(sy.lw + tid);
                    if (!hg) wg = ld_relaxed_u64(sy.lw + E);
                    have = have || (unsigned)(w >> 32) == stamp;
                    hg = hg || (unsigned)(wg >> 32) == stamp;
                    return !have || !hg;
                },
                sy, a.status);
            float l = -INFINITY;
            if (tid < E) {
                l = __uint_as_float((unsigned)w);
                if (l != l) l = -INFINITY;  // NaN ranks last
                lf[tid] = l;
            }
            if (tid == 0) {
                *s_gate = __uint_as_float((unsigned)wg);
                *s_cnt = 0;
            }
            const unsigned m = __reduce_max_sync(0xffffffffu, topk_ord(l));
            if (lane == 0) red[warp] = m;
            if (__syncthreads_or(!got)) {
                ok = false;
                break;
            }
        }
        dev_mark(a, L, 23);
        // Top-k on keys (p bits << 32 | ~id), p = exp(l - l_max): thread
        // (warp w, lane l) takes id l * 16 + w, so every warp sees ids spread
        // over the whole range; t0 = the k-th largest of the 16 warp maxima
        // (k distinct keys reach it, so every member of the top k does); the
        // keys >= t0 are the candidates, about k even when all tie.
        float lmax;
        int n_cand;
        unsigned long long key;
        {
            const unsigned mm = __reduce_max_sync(0xffffffffu, lane < kSKWarps ? red[lane] : 0u);
            lmax = __uint_as_float((mm & 0x80000000u) ? (mm & 0x7FFFFFFFu) : ~mm);
            const int e = lane * kSKWarps + warp;
            key = e < E ? ((unsigned long long)__float_as_uint(expf(lf[e] - lmax)) << 32) | (0xFFFFFFFFu - (unsigned)e)
                        : 0ull;
            const unsigned kh = (unsigned)(key >> 32), kl = (unsigned)key;
            const unsigned mh = __reduce_max_sync(0xffffffffu, kh);
            const unsigned ml = __reduce_max_sync(0xffffffffu, kh == mh ? kl : 0u);
            if (lane == 0) wmax[warp] = ((unsigned long long)mh << 32) | ml;
            __syncthreads();
            const unsigned long long wv = lane < kSKWarps ? wmax[lane] : 0ull;
            int gt = 0;
#pragma unroll
            for (int j = 0; j < kSKWarps; ++j) gt += __shfl_sync(0xffffffffu, wv, j) > wv ? 1 : 0;
            const unsigned sel = __ballot_sync(0xffffffffu, lane < kSKWarps && gt == K - 1);
            const unsigned long long t0 = __shfl_sync(0xffffffffu, wv, __ffs(sel) - 1);
            const bool is_c = e < E && key >= t0;
            const unsigned bal = __ballot_sync(0xffffffffu, is_c);
            int base = 0;
            if (lane == 0 && bal) base = atomicAdd(s_cnt, __popc(bal));
            base = __shfl_sync(0xffffffffu, base, 0);
            const int pos = base + __popc(bal & ((1u << lane) - 1u));
            if (is_c && pos < kCandCap) cand[pos] = key;
            __syncthreads();
            n_cand = *s_cnt;
            if (n_cand > 32) {
                // adversarial ties: the whole CTA ranks (up to kCandCap
                // candidates), or k rounds of block arg-max
                if (n_cand <= kCandCap) {
                    for (int i = tid; i < n_cand; i += kSKThreads) {
                        const unsigned long long ci = cand[i];
                        int rr = 0;
                        for (int j = 0; j < n_cand; ++j) rr += cand[j] > ci ? 1 : 0;
                        if (rr < K) {
                            tkv[rr] = __uint_as_float((unsigned)(ci >> 32));
                            tki[rr] = (int)(0xFFFFFFFFu - (unsigned)ci);
                        }
                    }
                    __syncthreads();
                } else {
                    unsigned long long mine = key;
                    for (int rd = 0; rd < K; ++rd) {
                        const unsigned h = (unsigned)(mine >> 32), lo = (unsigned)mine;
                        const unsigned wh = __reduce_max_sync(0xffffffffu, h);
                        const unsigned wl = __reduce_max_sync(0xffffffffu, h == wh ? lo : 0u);
                        if (lane == 0) cand[warp] = ((unsigned long long)wh << 32) | wl;
                        __syncthreads();
                        unsigned long long best = 0ull;
                        for (int w2 = 0; w2 < kSKWarps; ++w2) best = cand[w2] > best ? cand[w2] : best;
                        if (tid == 0) {
                            tkv[rd] = __uint_as_float((unsigned)(best >> 32));
                            tki[rd] = (int)(0xFFFFFFFFu - (unsigned)best);
                        }
                        if (mine == best) mine = 0ull;
                        __syncthreads();
                    }
                }
            }
        }
        if (tid == 0 && !(fabsf(lmax) <= 3.0e38f)) record_status(a.status, QMOE_ERR_NOT_FINITE);
        // Warp 0: the ranking of up to 32 candidates, this CTA's gate|up
        // copies, the weights.  Warps 1..: x to block floating point, then the
        // shared expert's pairs.
        bool a_ok = true;
        if (warp == 0) {
            if (n_cand <= 32) {
                const unsigned long long ci = lane < n_cand ? cand[lane] : 0ull;
                int rr = 0;
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const unsigned long long o = __shfl_sync(0xffffffffu, ci, j);
                    rr += (j < n_cand && o > ci) ? 1 : 0;
                }
                if (lane < n_cand && rr < K) {
                    tkv[rr] = __uint_as_float((unsigned)(ci >> 32));
                    tki[rr] = (int)(0xFFFFFFFFu - (unsigned)ci);
                }
                __syncwarp();
            }
            dev_mark(a, L, 15);
            ptx::fence_proxy_async();  // every issuing lane
            if (lane < nch) issue_chunk(W, p, S, sm, tki, lane, bar_ch + lane);
            if (lane == 0) ++iss_gu;
            trace_mark(a, L, 3);
            float ps = 0.0f;
            for (int i = 0; i < K; ++i) ps += tkv[i];
            const float inv = 1.0f / ps;
            __syncwarp();
            if (lane < K) tkv[lane] = tkv[lane] * inv;
            if (lane == 0) *s_gate = sigmoid(*s_gate);
            __syncwarp();
            if (a.ids_trace && c == 0 && lane < K) {
                a.ids_trace[L * K + lane] = tki[lane];
                a.w_trace[L * K + lane] = tkv[lane];
            }
            dev_mark(a, L, 24);
        } else {
            constexpr int XW = kSKWarps - 1, XPW = (NSB + XW - 1) / XW;
#pragma unroll
            for (int i = 0; i < XPW; ++i) {
                const int b = warp - 1 + i * XW;
                if (b < NSB) {
                    float st;
                    const int pw =
                        warp_block_fp(__bfloat162float(__ushort_as_bfloat16((unsigned short)xstage[b * 32 + lane])), &st);
                    if (lane < 16) xq[b * 16 + lane] = pw;
                    if (lane == 0) xs[b] = st;
                }
            }
            asm volatile("bar.sync 1, %0;" ::"r"(XW * 32) : "memory");
            dev_mark(a, L, 14, 32);
            // the shared expert's pairs (rows prefetched), on the streams
            // without warp 0
            const int hf = warp % SPL, stream = warp / SPL, sb = hf * 32 + lane;
            if (stream > 0) {
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
                if (!mbar_wait(bar_sgu, par)) {
                    a_ok = false;
                } else {
                    for (int t = stream - 1; t < nsq; t += NSTREAM - 1) {
                        float g, u;
                        pair_dot(sgu + (size_t)t * p.RB, sgu + (size_t)(S.NSQ + t) * p.RB, sb, xr, xst, g, u);
                        const float v = pair_reduce(g, u, lane);
                        if (lane == 0) sgp[t * SPL + hf] = v;
                        if (lane == 16) sup[t * SPL + hf] = v;
                    }
                }
            }
        }
        if (__syncthreads_or(!a_ok)) {
            if (tid == 0) sk_fail(sy, a.status);
            ok = false;
            break;
        }
        trace_mark(a, L, 4);

        // ---- B: gate|up pairs ------------------------------------------------
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
        // the routed pairs as their chunks land, two per warp at a time
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
        dev_mark(a, L, 25);
        __syncthreads();
        if (tid == 0) arrive(sy.hcnt, c);
        trace_mark(a, L, 6);
        // the down rows of the selected experts, needed once every h is in:
        // issued now, behind the gate|up rows
        if (warp == kSKWarps - 1) {
            ptx::fence_proxy_async();  // every issuing lane (dbuf was read in the last layer's phase C)
            issue_down(W, p, S, sm, tki, bar_dn, lane);
            if (lane == 0) s_misc[3] += 1u;
            dev_mark(a, L, 26, 32 * (kSKWarps - 1));
        }

        // ---- C: down, the next layer's input ---------------------------------
        // Once every CTA's h is counted in: one bulk copy of all of it into
        // the (consumed) gate|up buffers, then the next layer's prefetches
        // behind it.
        if (warp == 0) {
            const bool got = wait_round(sy.hcnt, (unsigned)(L + 1), NW, sy, a.status);
            if (lane == 0) {
                s_misc[0] = got ? 1u : 0u;
                if (got) {
                    ptx::fence_proxy_async();  // gbuf was read by the generic proxy
                    mbar_expect_tx(bar_h, (uint32_t)(NH * 4));
                    ptx::bulk_g2s(hstage, sy.hw, (uint32_t)(NH * 4), bar_h);
                    ++iss_h;
                    if (!last) {
                        issue_sgu(a.L[L + 1], p, S, sm, bar_sgu);
                        issue_rrow(a.L[L + 1], p, S, sm, bar_rr);
                        ++iss_sgu;
                        ++iss_rr;
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
        {
            // the h words -> block floating point (hq, hs)
            if (__syncthreads_or(!mbar_wait(bar_h, par))) {
                if (tid == 0) sk_fail(sy, a.status);
                ok = false;
                break;
            }
            dev_mark(a, L, 27);
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
        }
        trace_mark(a, L, 11);
        if (last) break;
        __syncthreads();
        if (tid == 0) arrive(sy.xcnt, c);
        trace_mark(a, L, 12);
    }

    // The launch counter, read by every CTA at its start (before its first
    // arrival on the h counters, which every CTA waits for in every layer).
    if (c == 0 && tid == 0) {
        st_relaxed_u32(reinterpret_cast<unsigned*>(a.sync), lc + 1u);
        if (XC) *a.xepoch = xepoch + 1u;
    }

    // Stopped early: let this CTA's copies in flight land (bounded) before exit.
    __syncthreads();
    if (!ok && tid == 0) {
        if (iss_sgu > 0) (void)mbar_wait(bar_sgu, (uint32_t)((iss_sgu - 1) & 1));
        if (iss_rr > 0) (void)mbar_wait(bar_rr, (uint32_t)((iss_rr - 1) & 1));
        if (iss_sdn > 0) (void)mbar_wait(bar_sdn, (uint32_t)((iss_sdn - 1) & 1));
        if (iss_h > 0) (void)mbar_wait(bar_h, (uint32_t)((iss_h - 1) & 1));
        if (s_misc[3] > 0u) (void)mbar_wait(bar_dn, (s_misc[3] - 1u) & 1u);
        if (iss_gu > 0) {
            const uint32_t q = (uint32_t)((iss_gu - 1) & 1);
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
    cudaError_t err = smem_opt_in(reinterpret_cast<const void*>(kern), (int)smem);
    if (err != cudaSuccess) return err;
    // The abort word and the round counters start at zero for every launch;
    // the launch counter (offset 0) and the tagged words are kept.
    err = cudaMemsetAsync(sync + kStackAbortOff, 0, kStackLogitOff - kStackAbortOff, stream);
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
