// The whole batch-1 MoE decode stack in one persistent launch.
//
// One CTA per SM (cooperative launch, so all CTAs are co-resident), looping
// over the layers.  Every layer is the reference's `_moe` (reference/model.py
// :387-417) in three phases separated by grid barriers:
//
//   A  x (bf16) -> block floating point in shared memory; this CTA's router
//      rows (fp32, already in shared memory) -> logits; this CTA's shared-
//      expert gate|up rows (already in shared memory) -> shared h.
//   B  every CTA ranks the 512 logits itself (warp top-k, lower id on ties),
//      then TMA bulk copies (cp.async.bulk, one thread issuing, mbarrier
//      completion) bring only its slice of the selected experts' gate|up rows
//      and down rows into shared memory; gate|up rows are decoded as their
//      4-pair chunks land -> routed h.
//   C  the full h (11 x 512) -> block floating point; this CTA's output rows
//      of every selected expert's down (already in shared memory) and of the
//      shared expert -> out[j] = sum_s w_s D_s[j].h_s + sigmoid(g.x) D_sh[j].h_sh.
//      Meanwhile the next layer's router rows and shared-expert rows stream
//      in, so phase A of the next layer starts on resident data.
//
// The layer output is written in fp32 and rounded to bf16 when the next layer
// loads it (bf16 activations, fp32 accumulation).  All waits are bounded in
// time (%globaltimer): a grid barrier or copy that does not complete sets
// QMOE_ERR_TIMEOUT and an abort word, every CTA waits (bounded) for its own
// copies in flight and returns.  No trap, no unbounded spin.
#include "common.cuh"
#include "topk.cuh"

namespace qmoe {
namespace {

constexpr int kSKWarps = 16;
constexpr int kSKThreads = kSKWarps * 32;
constexpr int kSKChunk = 4;        // routed row pairs per bulk-copy chunk
constexpr int kSKMaxChunks = 32;
constexpr unsigned long long kTimeoutNs = 200ull * 1000 * 1000;

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
    const __nv_bfloat16* x;  // [D] layer-0 input
    float* out;              // [D] last layer's output
    float* act;              // [D] layer activation (workspace)
    float* logits;           // [E + 1] (workspace); row E is the shared-expert gate
    float* h;                // [(K + 1) * I] (workspace)
    unsigned* sync;          // 8 counters, 128 B apart, then the abort word
    unsigned long long* trace;  // [2][64][16] phase stamps of CTA 0 and the last CTA, or null
    int* status;
    int n_layers, D, I, E, K;
    SKLayer L[kSKMaxLayers];
};

// Shared-memory carve-up (byte offsets), a function of the shape and grid.
struct SKLayout {
    int NR, NSQ, NP, NJ, NCH;
    unsigned xf, xq, xs, rbuf, sgu, sdn, gbuf, ubuf, dbuf, hq, hs, gv, uv, sgv, suv, rpart, dpart,
        cand, wmax, red, tkv, tki, misc, issued, bars, total;
};

__host__ __device__ constexpr unsigned sk_take(unsigned& o, unsigned bytes) {
    const unsigned r = o;
    o = (o + bytes + 127u) & ~127u;
    return r;
}

__host__ __device__ constexpr SKLayout sk_layout(int D, int I, int E, int K, int n) {
    SKLayout s{};
    const unsigned RB = (unsigned)(D / 256) * 136, DRB = (unsigned)(I / 256) * 136;
    const unsigned NSB = D / 32, NSBH = I / 32;
    s.NR = (E + 1 + n - 1) / n;
    s.NSQ = (I + n - 1) / n;
    s.NP = (K * I + n - 1) / n;
    s.NJ = (D + n - 1) / n;
    s.NCH = (s.NP + kSKChunk - 1) / kSKChunk;
    unsigned o = 0;
    s.xf = sk_take(o, D * 4);
    s.xq = sk_take(o, NSB * 64);
    s.xs = sk_take(o, NSB * 4);
    s.rbuf = sk_take(o, (unsigned)s.NR * D * 4);
    s.sgu = sk_take(o, 2u * s.NSQ * RB);
    s.sdn = sk_take(o, (unsigned)s.NJ * DRB);
    s.gbuf = sk_take(o, (unsigned)s.NP * RB);
    s.ubuf = sk_take(o, (unsigned)s.NP * RB);
    s.dbuf = sk_take(o, (unsigned)K * s.NJ * DRB);
    s.hq = sk_take(o, (unsigned)(K + 1) * NSBH * 64);
    s.hs = sk_take(o, (unsigned)(K + 1) * NSBH * 4);
    s.gv = sk_take(o, s.NP * 4);
    s.uv = sk_take(o, s.NP * 4);
    s.sgv = sk_take(o, s.NSQ * 4);
    s.suv = sk_take(o, s.NSQ * 4);
    s.rpart = sk_take(o, s.NR * 4 * 4);
    s.dpart = sk_take(o, (unsigned)s.NJ * (K + 1) * 4);
    s.cand = sk_take(o, (unsigned)(E > 256 ? E : 256) * 8);  // the tie fallback keeps 16 x k
    s.wmax = sk_take(o, (kSKWarps + 1) * 8);
    s.red = sk_take(o, kSKWarps * 4);
    s.tkv = sk_take(o, kMaxTopK * 4);
    s.tki = sk_take(o, kMaxTopK * 4);
    s.misc = sk_take(o, 64);
    s.issued = sk_take(o, (4 + kSKMaxChunks) * 4);
    s.bars = sk_take(o, (4 + kSKMaxChunks) * 8);
    s.total = o;
    return s;
}

// The shapes the single launch is built for: everything that sizes or
// places data is a compile-time constant, so the layer loop keeps only its
// data in registers.  Inter is 512 (the BASELINE family).
template <int D_, int E_, int K_, int NSM_>
struct SKShape {
    static constexpr int D = D_, E = E_, K = K_, NSM = NSM_, I = 512;
    static constexpr SKLayout S = sk_layout(D_, 512, E_, K_, NSM_);
};

namespace {

// ---- PTX wrappers: mbarrier, bulk copy, proxy fence, timer ---------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Global -> shared bulk copy into this CTA's own shared memory; dst, src 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_addr(dst)),
                 "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ unsigned long long now_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait for the phase of `bar` with parity `par`; false on timeout.
__device__ bool mbar_wait(uint64_t* bar, uint32_t par) {
    if (mbar_test(bar, par)) return true;
    const unsigned long long t0 = now_ns();
    while (!mbar_test(bar, par)) {
        if (now_ns() - t0 > kTimeoutNs) return false;
    }
    return true;
}

__device__ __forceinline__ unsigned* abort_word(unsigned* sync) { return sync + 8 * 32; }

// Phase trace: thread 0 of CTA 0 and of the last CTA stamp their SM's cycle
// counter (clock64) at each phase boundary.
__device__ __forceinline__ void trace_mark(const SKArgs& a, int L, int k) {
    if (a.trace && threadIdx.x == 0) {
        if (blockIdx.x == 0) a.trace[L * 16 + k] = (unsigned long long)clock64();
        else if (blockIdx.x == gridDim.x - 1) a.trace[(64 + L) * 16 + k] = (unsigned long long)clock64();
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
        if (lane == 0)  // release: orders this CTA's writes (after bar.sync) before the arrival
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

// One IQ4_XS row of D = 1024 * SBL2 values dotted with the activation in
// block floating point held in registers; lane l owns sub-blocks
// l*SBL2 .. l*SBL2+SBL2-1, all in one super-block, so one header load.
template <int SBL2>
__device__ __forceinline__ float row_dot(const uint8_t* row, const int (&xr)[SBL2][16], const float (&xs)[SBL2],
                                      int lane) {
    const int b0 = lane * SBL2;
    const uint8_t* blk = row + (b0 >> 3) * QMOE_SB_BYTES;
    const uint2 hdr = *reinterpret_cast<const uint2*>(blk);
    const float d = __half2float(__ushort_as_half((unsigned short)(hdr.x & 0xFFFFu)));
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < SBL2; ++i) {
        const int ib = (b0 + i) & 7;
        const uint2 q0 = *reinterpret_cast<const uint2*>(blk + 8 + 16 * ib);
        const uint2 q1 = *reinterpret_cast<const uint2*>(blk + 16 + 16 * ib);
        const int S = qmoe_subblock_dot(q0.x, q0.y, q1.x, q1.y, xr[i], 0);
        const float dl = d * (float)(qmoe_iq4xs_ls(hdr.x, hdr.y, ib) - 32);
        acc = fmaf(dl * xs[i], (float)S, acc);
    }
    return warp_sum(acc);
}

// One 32-value block to block floating point (out of line: one copy of the
// code serves the x and the h conversions).
__device__ __forceinline__ void convert_block(float v, int* q16, float* step, int lane) {
    float st;
    const int pw = warp_block_fp(v, &st);
    if (lane < 16) q16[lane] = pw;
    if (lane == 0) *step = st;
}

// One (output row, expert slot) down unit, lanes 0-15 or 16-31 of a warp
// each taking sub-blocks hl, hl+16, ...; returns the lane's share.  hq holds
// the slot's activation blocks as [word quad v][sub-block t][4 words], so the
// 16 lanes of a unit read 16 consecutive 16-byte chunks per quad.
__device__ __forceinline__ float down_unit(const uint8_t* row, const int* hq, const float* hs, int nsbh, int hl) {
    float acc = 0.0f;
    for (int t = hl; t < nsbh; t += 16) {
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
                         (float)(qmoe_iq4xs_ls(hdr.x, hdr.y, ib) - 32);
        acc = fmaf(dl * hs[t], (float)Sd, acc);
    }
    return acc;
}

// Shape-derived constants and this CTA's static slices.
struct SKPart {
    int D, I, E, K, RB, DRB, NSBH;
    size_t GUE, DNE;
    int rr_lo, rr_hi, sq_lo, sq_hi, p_lo, p_hi, j_lo, j_hi;
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
    p.DRB = (SH::I >> 8) * QMOE_SB_BYTES;
    p.NSBH = SH::I >> 5;
    p.GUE = (size_t)2 * SH::I * p.RB;
    p.DNE = (size_t)SH::D * p.DRB;
    constexpr int R = SH::E + 1, P = SH::K * SH::I;
    p.rr_lo = c * R / n;
    p.rr_hi = (c + 1) * R / n;
    p.sq_lo = c * SH::I / n;
    p.sq_hi = (c + 1) * SH::I / n;
    p.p_lo = c * P / n;
    p.p_hi = (c + 1) * P / n;
    p.j_lo = c * SH::D / n;
    p.j_hi = (c + 1) * SH::D / n;
    return p;
}

// Router rows + shared-expert gate|up rows of one layer (thread 0 only).
__device__ __forceinline__ void issue_phase_a(const SKLayer& W, const SKPart& p, const SKLayout& S, unsigned char* sm,
                              uint64_t* bar_r, uint64_t* bar_sgu) {
    const int nr = p.rr_hi - p.rr_lo, nsq = p.sq_hi - p.sq_lo;
    float* rbuf = reinterpret_cast<float*>(sm + S.rbuf);
    mbar_expect_tx(bar_r, (uint32_t)(nr * p.D * 4));
    const int r_end = p.rr_hi < p.E ? p.rr_hi : p.E;
    if (r_end > p.rr_lo)
        bulk_g2s(rbuf, W.router + (size_t)p.rr_lo * p.D, (uint32_t)((r_end - p.rr_lo) * p.D * 4), bar_r);
    if (p.rr_hi > p.E) bulk_g2s(rbuf + (size_t)(p.E - p.rr_lo) * p.D, W.gate_vec, (uint32_t)(p.D * 4), bar_r);
    uint8_t* sgu = sm + S.sgu;
    mbar_expect_tx(bar_sgu, (uint32_t)(2 * nsq * p.RB));
    if (nsq > 0) {
        bulk_g2s(sgu, W.sh_gate_up + (size_t)p.sq_lo * p.RB, (uint32_t)(nsq * p.RB), bar_sgu);
        bulk_g2s(sgu + (size_t)S.NSQ * p.RB, W.sh_gate_up + (size_t)(p.I + p.sq_lo) * p.RB,
                 (uint32_t)(nsq * p.RB), bar_sgu);
    }
}

// Shared-expert down rows of this CTA's output slice (thread 0 only).
__device__ __forceinline__ void issue_sdn(const SKLayer& W, const SKPart& p, const SKLayout& S, unsigned char* sm, uint64_t* bar) {
    const int nj = p.j_hi - p.j_lo;
    mbar_expect_tx(bar, (uint32_t)(nj * p.DRB));
    if (nj > 0) bulk_g2s(sm + S.sdn, W.sh_down + (size_t)p.j_lo * p.DRB, (uint32_t)(nj * p.DRB), bar);
}

// The selected experts' slices, issued by warp 0: lane 0 first posts every
// barrier's expected bytes, then lane i issues chunk i's gate|up row copies
// and, for i < K, expert slot i's down rows.  Chunks are kSKChunk row pairs
// with their own mbarrier so decoding starts on the first chunk to land.
__device__ __forceinline__ void issue_routed(const SKLayer& W, const SKPart& p, const SKLayout& S, unsigned char* sm,
                             const int* ids, uint64_t* bar_ch, uint64_t* bar_dn, int lane) {
    const int np = p.p_hi - p.p_lo, nj = p.j_hi - p.j_lo;
    if (lane == 0) {
        fence_proxy_async();
        for (int ch = 0; ch < S.NCH; ++ch) {
            const int u0 = ch * kSKChunk;
            const int u1 = (u0 + kSKChunk < np) ? u0 + kSKChunk : np;
            mbar_expect_tx(bar_ch + ch, u1 > u0 ? (uint32_t)(2 * (u1 - u0) * p.RB) : 0u);
        }
        mbar_expect_tx(bar_dn, (uint32_t)(p.K * nj * p.DRB));
    }
    __syncwarp();
    uint8_t* gbuf = sm + S.gbuf;
    uint8_t* ubuf = sm + S.ubuf;
    for (int ch = lane; ch < S.NCH; ch += 32) {
        const int u0 = ch * kSKChunk;
        const int u1 = (u0 + kSKChunk < np) ? u0 + kSKChunk : np;
        int u = u0;
        while (u < u1) {
            const int pp = p.p_lo + u;
            const int s = pp / p.I, r = pp - s * p.I;
            const int seg = (u1 - u) < (p.I - r) ? (u1 - u) : (p.I - r);
            const uint8_t* eb = W.gate_up + (size_t)ids[s] * p.GUE;
            bulk_g2s(gbuf + (size_t)u * p.RB, eb + (size_t)r * p.RB, (uint32_t)(seg * p.RB), bar_ch + ch);
            bulk_g2s(ubuf + (size_t)u * p.RB, eb + (size_t)(p.I + r) * p.RB, (uint32_t)(seg * p.RB), bar_ch + ch);
            u += seg;
        }
    }
    if (nj > 0) {
        uint8_t* dbuf = sm + S.dbuf;
        for (int s = lane; s < p.K; s += 32)
            bulk_g2s(dbuf + (size_t)s * S.NJ * p.DRB, W.down + (size_t)ids[s] * p.DNE + (size_t)p.j_lo * p.DRB,
                     (uint32_t)(nj * p.DRB), bar_dn);
    }
}

template <class SH>
__global__ void __launch_bounds__(kSKThreads, 1) stack_kernel(const __grid_constant__ SKArgs a) {
    extern __shared__ __align__(128) unsigned char sm[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const SKPart p = sk_part<SH>();
    constexpr SKLayout S = SH::S;
    constexpr int SBL2 = SH::D / 1024;
    constexpr int NSB = 32 * SBL2;
    constexpr int D = SH::D, I = SH::I, E = SH::E, K = SH::K;
    const int nr = p.rr_hi - p.rr_lo, nsq = p.sq_hi - p.sq_lo, np = p.p_hi - p.p_lo, nj = p.j_hi - p.j_lo;

    float* xf = reinterpret_cast<float*>(sm + S.xf);
    int* xq = reinterpret_cast<int*>(sm + S.xq);
    float* xs = reinterpret_cast<float*>(sm + S.xs);
    const float* rbuf = reinterpret_cast<const float*>(sm + S.rbuf);
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
    float* rpart = reinterpret_cast<float*>(sm + S.rpart);
    float* dpart = reinterpret_cast<float*>(sm + S.dpart);
    unsigned long long* cand = reinterpret_cast<unsigned long long*>(sm + S.cand);
    unsigned long long* wmax = reinterpret_cast<unsigned long long*>(sm + S.wmax);
    unsigned* red = reinterpret_cast<unsigned*>(sm + S.red);
    float* tkv = reinterpret_cast<float*>(sm + S.tkv);
    int* tki = reinterpret_cast<int*>(sm + S.tki);
    int* s_ok = reinterpret_cast<int*>(sm + S.misc);
    float* s_gate = reinterpret_cast<float*>(sm + S.misc) + 4;
    int* s_cnt = reinterpret_cast<int*>(sm + S.misc) + 8;
    float* s_glogit = reinterpret_cast<float*>(sm + S.misc) + 12;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S.bars);
    uint64_t* bar_r = bars;
    uint64_t* bar_sgu = bars + 1;
    uint64_t* bar_sdn = bars + 2;
    uint64_t* bar_dn = bars + 3;
    uint64_t* bar_ch = bars + 4;
    const int nbars = 4 + S.NCH;

    if (tid == 0) {
        for (int i = 0; i < nbars; ++i) mbar_init(bars + i, 1);
        fence_mbar_init();
    }
    __syncthreads();
    // Phases issued per barrier (kept by thread 0), for the bounded drain.
    int* issued = reinterpret_cast<int*>(sm + S.issued);
    if (tid == 0) {
        for (int i = 0; i < nbars; ++i) issued[i] = 0;
        issue_phase_a(a.L[0], p, S, sm, bar_r, bar_sgu);
        issue_sdn(a.L[0], p, S, sm, bar_sdn);
        issued[0] = issued[1] = issued[2] = 1;
    }

    unsigned gen = 0;
    bool ok = true;
    for (int L = 0; L < a.n_layers && ok; ++L) {
        const SKLayer& W = a.L[L];
        const uint32_t par = (uint32_t)(L & 1);
        const bool last = L + 1 == a.n_layers;

        // ---------------- phase A: x, router rows, shared gate|up --------
        trace_mark(a, L, 0);
        {
            // every load of x issued before any store (D <= 4 * kSKThreads)
            float v[4];
#pragma unroll
            for (int k4 = 0; k4 < 4; ++k4) {
                const int i = tid + k4 * kSKThreads;
                v[k4] = 0.0f;
                if (i < D) v[k4] = L == 0 ? __bfloat162float(a.x[i]) : __ldcg(a.act + i);
            }
#pragma unroll
            for (int k4 = 0; k4 < 4; ++k4) {
                const int i = tid + k4 * kSKThreads;
                if (i < D) xf[i] = L == 0 ? v[k4] : __bfloat162float(__float2bfloat16_rn(v[k4]));
            }
        }
        __syncthreads();
        trace_mark(a, L, 1);
#pragma unroll 1
        for (int b = warp; b < NSB; b += kSKWarps) convert_block(xf[b * 32 + lane], xq + b * 16, xs + b, lane);
        __syncthreads();
        int xr[SBL2][16];
        float xsr[SBL2];
#pragma unroll
        for (int i = 0; i < SBL2; ++i) {
            const int b = lane * SBL2 + i;
            const int4* src = reinterpret_cast<const int4*>(xq + b * 16);
#pragma unroll
            for (int v = 0; v < 4; ++v) {
                const int4 w4 = src[v];
                xr[i][4 * v] = w4.x;
                xr[i][4 * v + 1] = w4.y;
                xr[i][4 * v + 2] = w4.z;
                xr[i][4 * v + 3] = w4.w;
            }
            xsr[i] = xs[b];
        }
        trace_mark(a, L, 2);
        {
            const bool w_ok = mbar_wait(bar_r, par) && mbar_wait(bar_sgu, par);
            if (__syncthreads_or(!w_ok)) {  // block-uniform decision
                if (tid == 0) {
                    record_status(a.status, QMOE_ERR_TIMEOUT);
                    atomicExch(abort_word(a.sync), 1u);
                }
                ok = false;
                break;
            }
        }
        trace_mark(a, L, 3);
        // router: work item = (row, quarter of the columns)
        for (int it = warp; it < nr * 4; it += kSKWarps) {
            const int r = it >> 2, q = it & 3;
            const float* wr = rbuf + (size_t)r * D;
            const int cols = D >> 2;
            float acc = 0.0f;
            for (int c4 = q * cols + lane * 4; c4 < (q + 1) * cols; c4 += 128) {
                const float4 w4 = *reinterpret_cast<const float4*>(wr + c4);
                const float4 x4 = *reinterpret_cast<const float4*>(xf + c4);
                acc = fmaf(w4.x, x4.x, acc);
                acc = fmaf(w4.y, x4.y, acc);
                acc = fmaf(w4.z, x4.z, acc);
                acc = fmaf(w4.w, x4.w, acc);
            }
            acc = warp_sum(acc);
            if (lane == 0) rpart[it] = acc;
        }
        // shared expert gate|up rows
        for (int t = warp; t < 2 * nsq; t += kSKWarps) {
            const uint8_t* row = sgu + (size_t)((t & 1) ? (S.NSQ + (t >> 1)) : (t >> 1)) * p.RB;
            const float v = row_dot<SBL2>(row, xr, xsr, lane);
            if (lane == 0) ((t & 1) ? suv : sgv)[t >> 1] = v;
        }
        __syncthreads();
        trace_mark(a, L, 4);
        if (tid < nr) a.logits[p.rr_lo + tid] = (rpart[4 * tid] + rpart[4 * tid + 1]) + (rpart[4 * tid + 2] + rpart[4 * tid + 3]);
        if (tid >= 64 && tid - 64 < nsq) {
            const int q = tid - 64;
            a.h[(size_t)K * I + p.sq_lo + q] = silu(sgv[q]) * suv[q];
        }
        trace_mark(a, L, 5);
        if (!grid_sync(a.sync, ++gen, a.status, s_ok)) {
            ok = false;
            break;
        }
        trace_mark(a, L, 6);

        // ---------------- phase B: top-k, routed gate|up ------------------
        if (tid == kSKThreads - 1) *s_glogit = __ldcg(a.logits + E);  // overlaps the top-k's loads
        const float lmax = block_topk(a.logits, E, K, cand, wmax, red, s_cnt, tkv, tki);
        if (warp == 0) {
            const float e = lane < K ? tkv[lane] : 0.0f;
            const float sum = warp_sum(e);
            if (lane < K) tkv[lane] = e / sum;
            if (lane == 0) {
                *s_gate = sigmoid(*s_glogit);
                if (!(fabsf(lmax) <= 3.0e38f)) record_status(a.status, QMOE_ERR_NOT_FINITE);
            }
            trace_mark(a, L, 7);
        }
        __syncthreads();

        if (warp == 0) {
            issue_routed(W, p, S, sm, tki, bar_ch, bar_dn, lane);
            if (tid == 0)
                for (int i = 3; i < nbars; ++i) ++issued[i];
        }
        trace_mark(a, L, 8);
        for (int t = warp; t < 2 * np; t += kSKWarps) {
            const int u = t >> 1;
            if (!mbar_wait(bar_ch + u / kSKChunk, par)) {
                ok = false;
                break;
            }
            const uint8_t* row = ((t & 1) ? ubuf : gbuf) + (size_t)u * p.RB;
            const float v = row_dot<SBL2>(row, xr, xsr, lane);
            if (lane == 0) ((t & 1) ? uv : gv)[u] = v;
        }
        if (__syncthreads_or(!ok)) {
            if (tid == 0) {
                record_status(a.status, QMOE_ERR_TIMEOUT);
                atomicExch(abort_word(a.sync), 1u);
            }
            ok = false;
            break;
        }
        trace_mark(a, L, 9);
        for (int u = tid; u < np; u += kSKThreads) a.h[p.p_lo + u] = silu(gv[u]) * uv[u];
        trace_mark(a, L, 10);
        if (!grid_sync(a.sync, ++gen, a.status, s_ok)) {
            ok = false;
            break;
        }
        trace_mark(a, L, 11);

        // ---------------- phase C: down + combine --------------------------
        if (tid == 0 && !last) {
            fence_proxy_async();
            issue_phase_a(a.L[L + 1], p, S, sm, bar_r, bar_sgu);
            ++issued[0];
            ++issued[1];
        }
        {
            const int nbh = (K + 1) * p.NSBH;
            constexpr int NB = 12;
            for (int b0 = warp; b0 < nbh; b0 += NB * kSKWarps) {
                float v[NB];
#pragma unroll
                for (int i = 0; i < NB; ++i) {
                    const int b = b0 + i * kSKWarps;
                    v[i] = b < nbh ? __ldcg(a.h + (size_t)b * 32 + lane) : 0.0f;
                }
#pragma unroll
                for (int i = 0; i < NB; ++i) {
                    const int b = b0 + i * kSKWarps;
                    if (b < nbh) {
                        float st;
                        const int pw = warp_block_fp(v[i], &st);
                        const int slot = b / p.NSBH, t = b - slot * p.NSBH;
                        // word w = 4*quad + (w & 3) of block t of the slot
                        if (lane < 16) hq[slot * p.NSBH * 16 + ((lane >> 2) * p.NSBH + t) * 4 + (lane & 3)] = pw;
                        if (lane == 0) hs[b] = st;
                    }
                }
            }
        }
        __syncthreads();
        trace_mark(a, L, 12);
        {
            const bool w_ok = mbar_wait(bar_dn, par) && mbar_wait(bar_sdn, par);
            if (__syncthreads_or(!w_ok)) {
                if (tid == 0) {
                    record_status(a.status, QMOE_ERR_TIMEOUT);
                    atomicExch(abort_word(a.sync), 1u);
                }
                ok = false;
                break;
            }
        }
        trace_mark(a, L, 13);
        {
            // (output row j, expert slot s) per half-warp; slot K is the shared expert
            const int K1 = K + 1, nu = nj * K1, half = lane >> 4, hl = lane & 15;
            for (int u0 = 2 * warp; u0 < nu; u0 += 2 * kSKWarps) {
                const int u = u0 + half;
                float acc = 0.0f;
                if (u < nu) {
                    const int j = u / K1, s = u - j * K1;
                    const uint8_t* row = s < K ? dbuf + ((size_t)s * S.NJ + j) * p.DRB : sdn + (size_t)j * p.DRB;
                    acc = down_unit(row, hq + s * p.NSBH * 16, hs + s * p.NSBH, p.NSBH, hl);
                }
#pragma unroll
                for (int o = 8; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
                if (u < nu && hl == 0) dpart[u] = acc;
            }
        }
        __syncthreads();
        trace_mark(a, L, 14);
        for (int j = tid; j < nj; j += kSKThreads) {
            const float* dp = dpart + j * (K + 1);
            float o = 0.0f;
            for (int s = 0; s < K; ++s) o = fmaf(tkv[s], dp[s], o);
            o = fmaf(*s_gate, dp[K], o);
            (last ? a.out : a.act)[p.j_lo + j] = o;
        }
        __syncthreads();
        if (tid == 0 && !last) {
            fence_proxy_async();
            issue_sdn(a.L[L + 1], p, S, sm, bar_sdn);
            ++issued[2];
        }
        trace_mark(a, L, 15);
        if (!last && !grid_sync(a.sync, ++gen, a.status, s_ok)) {
            ok = false;
            break;
        }

    }

    // Stopped early: let this CTA's copies in flight land (bounded) before exit.
    if (!ok && tid == 0) {
        for (int i = 0; i < nbars; ++i)
            if (issued[i] > 0) (void)mbar_wait(bars + i, (uint32_t)((issued[i] - 1) & 1));
    }
}

}  // namespace

namespace {

using SKShapeC2 = SKShape<2048, 512, 10, 148>;    // BASELINE configs 1-2 on a 148-SM B200
using SKShapeTest = SKShape<1024, 64, 10, 148>;   // a small member of the family (tests)

// The compiled instantiation for these shapes on this device, or null.
void (*pick_kernel(const qmoe_dims& d, int n_sm, unsigned* smem))(SKArgs) {
    if (n_sm == 148 && d.hidden == 2048 && d.n_experts == 512 && d.top_k == 10) {
        *smem = SKShapeC2::S.total;
        return stack_kernel<SKShapeC2>;
    }
    if (n_sm == 148 && d.hidden == 1024 && d.n_experts == 64 && d.top_k == 10) {
        *smem = SKShapeTest::S.total;
        return stack_kernel<SKShapeTest>;
    }
    return nullptr;
}

}  // namespace

bool stack_kernel_supported(const qmoe_dims& d, int M, int n_layers) {
    if (M != 1 || n_layers < 1 || n_layers > kSKMaxLayers) return false;
    if (d.inter != 512 || d.inter_local != 512 || d.down_nseg != 2 || d.down_nsub != 8 || d.down_ib0 != 0)
        return false;
    if (d.sh_inter_local != 512 || d.sh_down_nseg != 2 || d.sh_down_nsub != 8 || d.sh_down_ib0 != 0) return false;
    if (d.expert_lo != 0 || d.expert_hi != d.n_experts) return false;
    unsigned smem = 0;
    return pick_kernel(d, device_sm_count(), &smem) != nullptr && smem <= 227u * 1024u;
}

cudaError_t launch_stack_kernel(const void* x, float* out, float* act, float* logits, float* h, unsigned* sync,
                                unsigned long long* trace, int* status, const qmoe_layer_weights* layers, int n_layers,
                                const qmoe_dims& d, cudaStream_t stream) {
    SKArgs a{};
    a.trace = trace;
    a.x = reinterpret_cast<const __nv_bfloat16*>(x);
    a.out = out;
    a.act = act;
    a.logits = logits;
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
    void (*kern)(SKArgs) = pick_kernel(d, n, &smem);
    if (!kern) return cudaErrorInvalidValue;
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess) return err;
    // Barrier counters and the abort word start at zero for every launch.
    err = cudaMemsetAsync(sync, 0, 1152, stream);
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
