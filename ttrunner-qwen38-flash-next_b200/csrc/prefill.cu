// Chunked prefill / large verify chunks: T tokens through one MoE layer.
//
// Reference: TTModel._prefill_ffn_half (tt/model.py:2812-2907), which calls
// moe.route (tt/moe.py:308-327) and apply_experts / expert_ffn (tt/moe.py:
// 330-368, 1057-1152); per token the arithmetic is reference/model.py:387-417
// (router softmax top-k renormalised, SwiGLU experts, sigmoid-gated shared
// expert).  Only here is the expert work a dense contraction: every selected
// expert sees a group of tokens, so its IQ4_XS rows are expanded to bf16 once
// per group in shared memory and fed to the 5th-generation tensor cores
// (tcgen05.mma, accumulators in tensor memory).
//
// One stream, no host round trip:
//   1. x -> bf16 copy, when x is fp32 or not 16-byte aligned;
//   2. router logits [T][E + 1] in fp32 (row E: the shared-expert gate vector);
//   3. top-k per token (warp per token, the decode path's selection rule);
//   4. grouping: per-expert counts, offsets, n-tiles of <= 64 tokens, and slot
//      rows ordered by token (deterministic); groups of at most 8 tokens are
//      listed apart for the grouped GEMV (no bf16 expansion);
//   5. gate|up grouped GEMM + SwiGLU epilogue -> h [rows][I] bf16, and the
//      small groups' gate|up GEMV -> h;
//   6. out = 0, then the down grouped GEMM and the small groups' down GEMV,
//      both with a gate-weighted scatter-add.
// The shared expert is group E: every token, weight sigmoid(x . gate_vec).
#include <atomic>

#include <math.h>

#include "common.cuh"
#include "ptx.cuh"
#include "tma_host.cuh"
#include "topk.cuh"

namespace qmoe {
namespace {

constexpr int kPfMaxTokens = 8192;
constexpr int kPfTraceSlots = 64;
constexpr size_t kPfTraceBytes = kPfTraceSlots * 8 * 8;
constexpr unsigned long long kPfTimeoutNs = 1000ull * 1000 * 1000;

// ---- grouped GEMM geometry --------------------------------------------------
constexpr int kGM = 128;            // MMA M: weight rows per tile
constexpr int kGNMax = 64;          // tokens per n-tile (MMA N, padded to 16)
constexpr int kGAtomK = 64;         // K of one 128-byte swizzle atom row of bf16
constexpr int kGSlotK = 128;        // K per operand slot: two atoms, one handshake
constexpr int kGSlots = 3;          // slot ring depth (A expanded weights and B token rows together)
constexpr int kGStageK = 512;       // K per IQ4_XS stage: two super-blocks of every row
constexpr int kGStageRowB = 2 * QMOE_SB_BYTES;  // 272 bytes of one row per stage
constexpr int kGStages = 2;
constexpr int kGAtomBytes = kGM * kGAtomK * 2;      // 16 KB: 128 rows x 64 K of A
constexpr int kGSlotBytes = 2 * kGAtomBytes;        // 32 KB A slot
constexpr int kGBAtomBytes = kGNMax * kGAtomK * 2;  // 8 KB: 64 token rows x 64 K of B
constexpr int kGBSlotBytes = 2 * kGBAtomBytes;      // 16 KB B slot
constexpr int kGSlotsPerStage = kGStageK / kGSlotK; // 4
constexpr int kGStageBytes = kGM * kGStageRowB;  // 34,816
constexpr int kGTmemCols = 2 * kGNMax;  // two accumulator buffers
// warp roles
// Dequant: two groups of kNDqG warps; group g expands the slots whose running
// index is g mod 2, so two slots are expanded at once.
// A warp issues on scheduler (warp mod 4).  The single MMA-issuing thread
// shares its scheduler only with the light roles (stage loads, B copies, one
// epilogue warp), so the expansion warps do not take its issue slots: with
// four expansion warps beside it, each step of its per-slot loop waited
// several hundred cycles.  Warps 20-23 are the epilogue (TMEM lane quarter =
// warp mod 4), warp 18 has no role, the other 16 expand.
constexpr int kNDqG = 8, kNDqGroups = 2;
constexpr int kWLoad = 6, kWGather = 10, kWMma = 2, kWIdle = 18, kNDq = kNDqG * kNDqGroups, kWEp0 = 20, kNEp = 4;
constexpr int kGWarps = 24;
constexpr int kGThreads = kGWarps * 32;
// Expansion index 0..15 of a warp that is none of the above.
__host__ __device__ constexpr int dq_index(int w) { return w - (w > 2) - (w > 6) - (w > 10) - (w > 18); }
static_assert(dq_index(19) == kNDq - 1 && dq_index(0) == 0, "16 expansion warps");

// shared-memory carve-up from a 1024-aligned base
constexpr int kOffA = 0;
constexpr int kOffB = kOffA + kGSlots * kGSlotBytes;
constexpr int kOffStage = kOffB + kGSlots * kGBSlotBytes;
constexpr int kOffBars = kOffStage + kGStages * kGStageBytes;
constexpr int kNBars = 2 * kGStages + 2 * kGSlots + 2 * 2 + 1;
constexpr int kOffMisc = kOffBars + kNBars * 8;
constexpr int kGSmemBytes = kOffMisc + 64 + 1024;  // + slack to align the base
static_assert(kOffStage % 1024 == 0 && kOffB % 1024 == 0, "operand tiles must be 1024-aligned");
static_assert(kGSmemBytes <= 232448, "dynamic shared memory above the 227 KB opt-in limit");

struct GemmArgs {
    int mode;  // 0: gate|up + SwiGLU -> h; 1: down + weighted scatter-add -> out
    int D, I, E, T;
    const uint8_t* gate_up;
    const uint8_t* down;
    const uint8_t* sh_gate_up;
    const uint8_t* sh_down;
    size_t gu_expert_bytes, dn_expert_bytes;
    const __nv_bfloat16* x;  // [T][D], 16-byte aligned
    __nv_bfloat16* h;        // [rows][I]
    const int* slot_tok;     // [rows]
    const float* slot_w;     // [rows]
    const int4* ntiles;      // {group, first token of the tile in the group, count, slot row}
    const int* meta;         // meta[0]: number of n-tiles
    float* out;              // [T][D]
    int* status;
    unsigned long long* trace;  // CTA 0's per-slot clock stamps [64 slots][8] (workspace)
    // This mode's weights as 2-D uint16 tensors [rows][row bytes / 2]: the
    // routed experts' (rows of all experts stacked) and the shared expert's.
    // A stage is boxes of 136 elements (272 bytes: two super-blocks) x 64
    // rows (gate|up: a gate box and an up box) or x 128 rows (down).
    CUtensorMap wmap;
    CUtensorMap shmap;
    // B operand rows as a bf16 tensor [slot rows][K] (the expert-sorted copy of x
    // for gate|up, h for down), boxes of 64 columns x 128 rows in the 128-byte
    // swizzle layout the MMA descriptors read.
    CUtensorMap bmap;
};

struct PfSmem {
    unsigned char* base;
    uint64_t* bars;
    __device__ uint8_t* a_slot(int s) const { return base + kOffA + s * kGSlotBytes; }
    __device__ uint8_t* b_slot(int s) const { return base + kOffB + s * kGBSlotBytes; }
    __device__ uint8_t* stage(int s) const { return base + kOffStage + s * kGStageBytes; }
    __device__ uint64_t* iq_full(int s) const { return bars + s; }
    __device__ uint64_t* iq_empty(int s) const { return bars + kGStages + s; }
    __device__ uint64_t* s_full(int s) const { return bars + 2 * kGStages + s; }
    __device__ uint64_t* s_empty(int s) const { return bars + 2 * kGStages + kGSlots + s; }
    __device__ uint64_t* acc_full(int b) const { return bars + 2 * kGStages + 2 * kGSlots + b; }
    __device__ uint64_t* acc_empty(int b) const { return bars + 2 * kGStages + 2 * kGSlots + 2 + b; }
    __device__ uint64_t* fin() const { return bars + 2 * kGStages + 2 * kGSlots + 4; }
    __device__ uint32_t* tmem_holder() const { return reinterpret_cast<uint32_t*>(base + kOffMisc); }
    __device__ volatile int* abort_flag() const { return reinterpret_cast<volatile int*>(base + kOffMisc + 16); }
};

// Bounded wait on an mbarrier phase; false (and the CTA's abort flag set) on
// timeout, or when another role already gave up (unless `honour_abort` is
// false: the drains before exit wait for in-flight work regardless).
__device__ bool pf_wait(uint64_t* bar, uint32_t par, volatile int* abort_flag, int* status,
                        bool honour_abort = true) {
    if (ptx::mbar_probe(bar, par)) return true;
    const unsigned long long t0 = ptx::now_ns();
    for (unsigned it = 0;; ++it) {
        if (ptx::mbar_test_sleep(bar, par, 20000u)) return true;
        if ((it & 3u) == 3u) {
            if (honour_abort && *abort_flag) return false;
            if (ptx::now_ns() - t0 > kPfTimeoutNs) {
                *abort_flag = 1;
                record_status(status, QMOE_ERR_TIMEOUT);
                return false;
            }
        }
    }
}
// The same, by every lane of a warp, agreeing on the outcome.
__device__ __forceinline__ bool pf_wait_warp(uint64_t* bar, uint32_t par, volatile int* abort_flag, int* status) {
    const bool ok = pf_wait(bar, par, abort_flag, status);
    return __all_sync(0xffffffffu, ok);
}

// CTA 0 stamps its SM clock for slot `it` (< kPfTraceSlots), event k.
__device__ __forceinline__ void pf_stamp(const GemmArgs& a, int it, int k) {
    if (a.trace && blockIdx.x == 0 && it < kPfTraceSlots)
        a.trace[it * 8 + k] = (unsigned long long)clock64();
}

struct TileInfo {
    int g, cnt, row0, mt, N;
    const uint8_t* w;  // this group's weight tensor for the mode
};

__device__ __forceinline__ TileInfo tile_info(const GemmArgs& a, int t, int MT) {
    TileInfo ti;
    const int4 nd = __ldg(a.ntiles + t / MT);
    ti.g = nd.x;
    ti.cnt = nd.z;
    ti.row0 = nd.w;
    ti.mt = t % MT;
    ti.N = (ti.cnt + 15) & ~15;
    if (a.mode == 0)
        ti.w = ti.g < a.E ? a.gate_up + (size_t)ti.g * a.gu_expert_bytes : a.sh_gate_up;
    else
        ti.w = ti.g < a.E ? a.down + (size_t)ti.g * a.dn_expert_bytes : a.sh_down;
    return ti;
}

// (x0 - bias) * scale and (x1 - bias) * scale with sm_100's packed fp32
// instructions: an exact subtraction of the 2^23 bias, then one rounding.
__device__ __forceinline__ void sub_mul_f32x2(float& x0, float& x1, float bias, float scale) {
    asm("{\n .reg .b64 v, b, s;\n mov.b64 v, {%0, %1};\n mov.b64 b, {%2, %2};\n mov.b64 s, {%3, %3};\n"
        " add.rn.f32x2 v, v, b;\n mul.rn.f32x2 v, v, s;\n mov.b64 {%0, %1}, v;\n}"
        : "+f"(x0), "+f"(x1)
        : "f"(-bias), "f"(scale));
}

// One 32-value sub-block of IQ4_XS (header words h0/h1, qs words q0..q3) to
// 32 bf16 in natural order, as four 16-byte chunks.  Each code's codebook
// entry + 128 is placed under the exponent of 2^23 (an exact float 2^23 + b),
// the bias removed exactly, the result scaled by d*(ls-32) and rounded to bf16.
__device__ __forceinline__ void dequant_subblock_bf16(uint32_t h0, uint32_t h1, int ib, uint32_t q0, uint32_t q1,
                                                      uint32_t q2, uint32_t q3, uint4 (&c)[4]) {
    const float d = __half2float(__ushort_as_half((unsigned short)(h0 & 0xFFFFu)));
    const float dl = d * (float)(qmoe_iq4xs_ls(h0, h1, ib) - 32);
    const uint32_t q[4] = {q0, q1, q2, q3};
    uint32_t pk[4][4];  // [word][lo-pair, hi-pair, lo-pair(high nibbles), hi-pair(high nibbles)]
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        uint32_t lo, hi;
        qmoe_lut8_biased(q[w], lo, hi);
        // lo bytes: values 4w, 16+4w, 4w+1, 16+4w+1; hi: 4w+2, 18+4w, 4w+3, 19+4w
        float v[8];
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            v[b] = __uint_as_float(qmoe_prmt(lo, 0x4B000000u, 0x7540u + (uint32_t)b));
            v[4 + b] = __uint_as_float(qmoe_prmt(hi, 0x4B000000u, 0x7540u + (uint32_t)b));
        }
        // (v - (2^23 + 128)) * dl, two values per packed instruction (the
        // same two roundings as the scalar form)
        sub_mul_f32x2(v[0], v[2], 8388736.0f, dl);
        sub_mul_f32x2(v[4], v[6], 8388736.0f, dl);
        sub_mul_f32x2(v[1], v[3], 8388736.0f, dl);
        sub_mul_f32x2(v[5], v[7], 8388736.0f, dl);
        const __nv_bfloat162 p0 = __floats2bfloat162_rn(v[0], v[2]);  // values 4w, 4w+1
        const __nv_bfloat162 p1 = __floats2bfloat162_rn(v[4], v[6]);  // 4w+2, 4w+3
        const __nv_bfloat162 p2 = __floats2bfloat162_rn(v[1], v[3]);  // 16+4w, 16+4w+1
        const __nv_bfloat162 p3 = __floats2bfloat162_rn(v[5], v[7]);  // 16+4w+2, 16+4w+3
        pk[w][0] = *reinterpret_cast<const uint32_t*>(&p0);
        pk[w][1] = *reinterpret_cast<const uint32_t*>(&p1);
        pk[w][2] = *reinterpret_cast<const uint32_t*>(&p2);
        pk[w][3] = *reinterpret_cast<const uint32_t*>(&p3);
    }
    c[0] = make_uint4(pk[0][0], pk[0][1], pk[1][0], pk[1][1]);  // values 0..7
    c[1] = make_uint4(pk[2][0], pk[2][1], pk[3][0], pk[3][1]);  // 8..15
    c[2] = make_uint4(pk[0][2], pk[0][3], pk[1][2], pk[1][3]);  // 16..23
    c[3] = make_uint4(pk[2][2], pk[2][3], pk[3][2], pk[3][3]);  // 24..31
}

// Byte offset of 16-byte chunk `c` (0..7) of row `r` in a 128-byte-swizzled
// K-major tile.
__device__ __forceinline__ uint32_t sw128_off(int r, int c) {
    return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

// Grouped GEMM, persistent: one CTA per SM walks tiles t = blockIdx.x,
// + gridDim.x, ...; tile t = (n-tile t / MT, m-tile t % MT).  mode 0: M rows
// interleave the gate and up rows of 64 intermediate rows (even = gate,
// odd = up), K = D; mode 1: 128 down rows, K = I.
__global__ void __launch_bounds__(kGThreads, 1) grouped_gemm_kernel(const __grid_constant__ GemmArgs a) {
    extern __shared__ unsigned char smem_raw[];
    PfSmem S;
    S.base = reinterpret_cast<unsigned char*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    S.bars = reinterpret_cast<uint64_t*>(S.base + kOffBars);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    volatile int* abort_flag = S.abort_flag();

    if (tid == 0) {
        for (int s = 0; s < kGStages; ++s) {
            ptx::mbar_init(S.iq_full(s), 1);
            ptx::mbar_init(S.iq_empty(s), kNDq);
        }
        // A slot full: the 8 expansion warps of its group and the B copy (one
        // arrival with the copy's bytes); empty: the MMAs that read it.
        for (int s = 0; s < kGSlots; ++s) {
            ptx::mbar_init(S.s_full(s), kNDqG + 1);
            ptx::mbar_init(S.s_empty(s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            ptx::mbar_init(S.acc_full(b), 1);
            ptx::mbar_init(S.acc_empty(b), kNEp);
        }
        ptx::mbar_init(S.fin(), 1);
        *abort_flag = 0;
        ptx::fence_mbar_init();
    }
    if (warp == kWMma) {
        ptx::tmem_alloc(S.tmem_holder(), kGTmemCols);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem_base = *S.tmem_holder();

    const int MT = a.mode == 0 ? a.I / 64 : a.D / kGM;
    const int K = a.mode == 0 ? a.D : a.I;
    const int nslots = K / kGSlotK;
    const int n_tiles = __ldg(a.meta) * MT;

    if (warp == kWLoad) {
        // ---- IQ4_XS stage producer: 128 rows x 272 bytes per stage --------
        int st_it = 0;
        int last_issue[kGStages] = {-1, -1};
        bool ok = true;
        for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
            const TileInfo ti = tile_info(a, t, MT);
            for (int kst = 0; kst < K / kGStageK; ++kst) {
                const int st = st_it % kGStages;
                if (!pf_wait_warp(S.iq_empty(st), ((st_it / kGStages) & 1) ^ 1, abort_flag, a.status)) {
                    ok = false;
                    break;
                }
                if (lane == 0) {
                    // gate|up: gate rows mt*64.. -> stage rows 0-63, up rows -> 64-127;
                    // down: rows mt*128.. -> stage rows 0-127
                    const CUtensorMap* map = ti.g < a.E ? &a.wmap : &a.shmap;
                    const int rows_per_e = a.mode == 0 ? 2 * a.I : a.D;
                    const int y0 = (ti.g < a.E ? ti.g * rows_per_e : 0) + ti.mt * (a.mode == 0 ? 64 : kGM);
                    const int x = kst * (kGStageRowB / 2);
                    ptx::mbar_expect_tx(S.iq_full(st), kGStageBytes);
                    uint8_t* dst = S.stage(st);
                    if (a.mode == 0) {
                        ptx::tma_load_2d(dst, map, x, y0, S.iq_full(st));
                        ptx::tma_load_2d(dst + 64 * kGStageRowB, map, x, y0 + a.I, S.iq_full(st));
                    } else {
                        ptx::tma_load_2d(dst, map, x, y0, S.iq_full(st));
                    }
                }
                __syncwarp();
                if (lane == 0) pf_stamp(a, st_it * (kGStageK / kGSlotK), 6);
                last_issue[st] = st_it;
                ++st_it;
            }
        }
        // Copies still in flight land before the CTA leaves (bounded).
        if (!ok && lane == 0) {
            for (int s = 0; s < kGStages; ++s)
                if (last_issue[s] >= 0)
                    (void)pf_wait(S.iq_full(s), (last_issue[s] / kGStages) & 1, abort_flag, a.status, false);
        }
    } else if (warp == kWGather) {
        // ---- B operand: two 2-D tensor copies per slot (2 x 64 K x 64 rows)
        // into the slot's B half, counted on the slot's full barrier --------
        if (lane == 0) {
            int it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
                const TileInfo ti = tile_info(a, t, MT);
                for (int ks = 0; ks < nslots; ++ks) {
                    const int slot = it % kGSlots;
                    if (!pf_wait(S.s_empty(slot), ((it / kGSlots) & 1) ^ 1, abort_flag, a.status)) {
                        ok = false;
                        break;
                    }
                    ptx::mbar_expect_tx(S.s_full(slot), kGBSlotBytes);
                    ptx::tma_load_2d(S.b_slot(slot), &a.bmap, ks * kGSlotK, ti.row0, S.s_full(slot));
                    ptx::tma_load_2d(S.b_slot(slot) + kGBAtomBytes, &a.bmap, ks * kGSlotK + kGAtomK, ti.row0,
                                     S.s_full(slot));
                    pf_stamp(a, it, 0);
                    ++it;
                }
            }
            // The last copies land before the CTA leaves (bounded: after an
            // abort the expansion arrivals on those slots may never come, and
            // each wait then ends at the time limit).
            if (!ok)
                for (int j = 1; j <= kGSlots && it - j >= 0; ++j)
                    (void)pf_wait(S.s_full((it - j) % kGSlots), ((it - j) / kGSlots) & 1, abort_flag, a.status,
                                  false);
        }
        __syncwarp();
    } else if (warp == kWMma) {
        // ---- MMA issue: one thread --------------------------------------
        if (lane == 0) {
            int it = 0, tc = 0;
            bool ok = true, issued = false;
            // Slot s's descriptor is slot 0's plus s * slot bytes / 16 in the
            // start-address field (the rings lie below 256 KB of shared
            // memory, so the 14-bit field does not overflow).
            const uint64_t desc_a0 = ptx::desc_sw128(ptx::smem_addr(S.a_slot(0)));
            const uint64_t desc_b0 = ptx::desc_sw128(ptx::smem_addr(S.b_slot(0)));
            for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
                const TileInfo ti = tile_info(a, t, MT);
                const uint32_t idesc = ptx::idesc_bf16(kGM, ti.N);
                const int ab = tc & 1;
                if (!pf_wait(S.acc_empty(ab), ((tc >> 1) & 1) ^ 1, abort_flag, a.status)) {
                    ok = false;
                    break;
                }
                ptx::tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(ab * kGNMax);
                const uint32_t idesc_t = idesc;
                for (int ks = 0; ks < nslots; ++ks) {
                    const int slot = it % kGSlots;
                    if (!pf_wait(S.s_full(slot), (it / kGSlots) & 1, abort_flag, a.status)) {
                        ok = false;
                        break;
                    }
                    pf_stamp(a, it, 1);
                    pf_stamp(a, it, 2);
                    ptx::tc_fence_after();
                    // descriptors of the slot's atoms, advanced 32 bytes (2 in
                    // the start-address field) per K = 16 step
                    const uint64_t da = desc_a0 + (uint64_t)(slot * (kGSlotBytes >> 4));
                    const uint64_t db = desc_b0 + (uint64_t)(slot * (kGBSlotBytes >> 4));
#pragma unroll
                    for (int k = 0; k < kGSlotK / 16; ++k) {
                        const int atom = k >> 2, kk = k & 3;
                        ptx::mma_bf16(d_tmem, da + (uint64_t)(atom * (kGAtomBytes >> 4) + 2 * kk),
                                      db + (uint64_t)(atom * (kGBAtomBytes >> 4) + 2 * kk), idesc_t,
                                      (ks | k) != 0 ? 1u : 0u);
                    }
                    ptx::mma_commit(S.s_empty(slot));
                    pf_stamp(a, it, 3);
                    issued = true;
                    ++it;
                }
                if (!ok) break;
                ptx::mma_commit(S.acc_full(ab));
                ++tc;
            }
            // Every MMA issued completes before the tensor memory is released.
            if (issued) {
                ptx::mma_commit(S.fin());
                (void)pf_wait(S.fin(), 0, abort_flag, a.status, false);
            }
        }
        __syncwarp();
    } else if (warp == kWIdle) {
    } else if (warp < kWEp0) {
        // ---- dequant: IQ4_XS stage -> bf16 A slot -----------------------
        const int dq = dq_index(warp), grp = dq / kNDqG;
        const int d = (dq % kNDqG) * 32 + lane;  // 0..255 within the group
        const int m = d & (kGM - 1), sub = d >> 7;
        int it = 0, st_it = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
            for (int ks = 0; ks < nslots; ++ks) {
                const int st = st_it % kGStages;
                if ((ks % kGSlotsPerStage) == 0) {
                    if (!pf_wait_warp(S.iq_full(st), (st_it / kGStages) & 1, abort_flag, a.status)) {
                        ok = false;
                        break;
                    }
                    if (dq == 0 && lane == 0) pf_stamp(a, it, 7);
                }
                const int slot = it % kGSlots;
                if ((it & 1) == grp) {
                    if (!pf_wait_warp(S.s_empty(slot), ((it / kGSlots) & 1) ^ 1, abort_flag, a.status)) {
                        ok = false;
                        break;
                    }
                    if (dq % kNDqG == 0 && lane == 0) pf_stamp(a, it, 4);
                    // stage row of M row m: gate|up stages hold the gate box then the up box
                    const int srow = a.mode == 0 ? ((m & 1) ? 64 + (m >> 1) : (m >> 1)) : m;
                    uint8_t* dst = S.a_slot(slot);
                    // this thread's two of the slot's four sub-blocks: sub and
                    // sub + 2, i.e. half `sub` of each atom's 64 K
#pragma unroll
                    for (int h2 = 0; h2 < 2; ++h2) {
                        const int sbq = sub + 2 * h2;
                        const int sbk = (ks % kGSlotsPerStage) * 4 + sbq;  // sub-block within the stage row (0..15)
                        const uint8_t* blk = S.stage(st) + srow * kGStageRowB + (sbk >> 3) * QMOE_SB_BYTES;
                        const int ib = sbk & 7;
                        const uint2 hd = *reinterpret_cast<const uint2*>(blk);
                        const uint2 qa = *reinterpret_cast<const uint2*>(blk + 8 + 16 * ib);
                        const uint2 qb = *reinterpret_cast<const uint2*>(blk + 16 + 16 * ib);
                        uint4 cv[4];
                        dequant_subblock_bf16(hd.x, hd.y, ib, qa.x, qa.y, qb.x, qb.y, cv);
                        uint8_t* at = dst + h2 * kGAtomBytes;
#pragma unroll
                        for (int j = 0; j < 4; ++j) *reinterpret_cast<uint4*>(at + sw128_off(m, sub * 4 + j)) = cv[j];
                    }
                    ptx::fence_proxy_async();
                    __syncwarp();
                    if (lane == 0) ptx::mbar_arrive(S.s_full(slot));
                    if (dq % kNDqG == 0 && lane == 0) pf_stamp(a, it, 5);
                }
                ++it;
                if ((ks % kGSlotsPerStage) == kGSlotsPerStage - 1 || ks == nslots - 1) {
                    __syncwarp();
                    if (lane == 0) ptx::mbar_arrive(S.iq_empty(st));
                    ++st_it;
                }
            }
        }
    } else {
        // ---- epilogue: TMEM -> registers -> h (mode 0) or out (mode 1) ---
        const int q = warp & 3;          // TMEM lane quarter this warp may read
        const int m = q * 32 + lane;     // M row of this thread
        int tc = 0;
        for (int t = blockIdx.x; t < n_tiles; t += gridDim.x) {
            const TileInfo ti = tile_info(a, t, MT);
            const int ab = tc & 1;
            // this tile's token ids and weights (down), one per lane and column
            // half, loaded before the accumulator wait and broadcast per column
            int tok_r[2] = {0, 0};
            float w_r[2] = {0.0f, 0.0f};
            if (a.mode == 1) {
#pragma unroll
                for (int hlf = 0; hlf < 2; ++hlf) {
                    const int n = hlf * 32 + lane;
                    if (n < ti.cnt) {
                        tok_r[hlf] = __ldg(a.slot_tok + ti.row0 + n);
                        w_r[hlf] = __ldg(a.slot_w + ti.row0 + n);
                    }
                }
            }
            if (!pf_wait_warp(S.acc_full(ab), (tc >> 1) & 1, abort_flag, a.status)) break;
            ptx::tc_fence_after();
            const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * kGNMax);
            for (int c0 = 0; c0 < ti.N; c0 += 16) {
                float v[16];
                ptx::tmem_ld16(tbase + (uint32_t)c0, v);
                if (a.mode == 0) {
                    const int r = ti.mt * 64 + (m >> 1);
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const float other = __shfl_xor_sync(0xffffffffu, v[j], 1);
                        const int n = c0 + j;
                        if (!(m & 1) && n < ti.cnt)
                            a.h[(size_t)(ti.row0 + n) * a.I + r] = __float2bfloat16_rn(silu(v[j]) * other);
                    }
                } else {
                    const int row = ti.mt * kGM + m;
                    const int hlf = c0 >> 5;  // c0 + j < 64 stays in one half: c0 is a multiple of 16
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int n = c0 + j;
                        const int tok = __shfl_sync(0xffffffffu, tok_r[hlf], n & 31);
                        const float w = __shfl_sync(0xffffffffu, w_r[hlf], n & 31);
                        if (n < ti.cnt && (unsigned)tok < (unsigned)a.T)
                            atomicAdd(a.out + (size_t)tok * a.D + row, w * v[j]);
                    }
                }
            }
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(S.acc_empty(ab));
            ++tc;
        }
    }

    ptx::tc_fence_before();
    __syncthreads();
    if (warp == kWMma) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem_base, kGTmemCols);
    }
}

// ---- router, top-k, grouping -------------------------------------------------

// xg[r] = x[slot_tok[r]] for every slot row r < meta[1] (bf16 rows of D): the
// gate|up B operand in expert-sorted order, so each tile's token rows are one
// contiguous box.
__global__ void __launch_bounds__(256) pf_gather_kernel(const __nv_bfloat16* __restrict__ x, int D,
                                                        const int* __restrict__ slot_tok, const int* __restrict__ meta,
                                                        int T, __nv_bfloat16* __restrict__ xg) {
    const int r = blockIdx.x;
    if (r >= __ldg(meta + 1)) return;
    const int tok = __ldg(slot_tok + r);
    if ((unsigned)tok >= (unsigned)T) return;
    const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)tok * D);
    uint4* dst = reinterpret_cast<uint4*>(xg + (size_t)r * D);
    for (int i = threadIdx.x; i < D / 8; i += blockDim.x) dst[i] = __ldg(src + i);
}

// bf16 copy of the activations (fp32 input is rounded to bf16, the activation
// dtype between layers).
__global__ void pf_convert_kernel(const void* x, int x_f32, size_t n, __nv_bfloat16* xb) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        xb[i] = __float2bfloat16_rn(load_act(x, x_f32, i));
}

// logits[t][e] = x_t . R_e in fp32 for e < E and the gate vector at e = E.
// Tile: 64 tokens x 64 router rows, K step 32, 4 x 4 outputs per thread.
// Router logits of a chunk, fp32: logits[t][e] = x_t . R_e, row E the gate
// vector (zero without one).  64 x 64 tiles of (tokens, router rows), 256
// threads each holding a 4 x 4 block; K in steps of 32, each step's operands
// loaded with 16-byte loads one step ahead of the arithmetic.  When the tiles
// alone would leave SMs idle (small chunks), grid.z splits K into equal
// chunks whose partials go to part[z] and are summed in chunk order by
// pf_logit_reduce_kernel: the same bits on every run.
constexpr int kRtK = 32;   // K per step
constexpr int kRtM = 128;  // tokens per tile (8 per thread)
constexpr int kRtN = 64;   // router rows per tile (4 per thread)

// out[t][e] = x[t] . W[e] over this CTA's K chunk, fp32 (x from its bf16 copy), each thread
// accumulating its 8 x 4 outputs over k in ascending order.
__global__ void __launch_bounds__(256) pf_router_kernel(const __nv_bfloat16* __restrict__ xb, int T, int D,
                                                        const float* __restrict__ router,
                                                        const float* __restrict__ gate_vec, int E, int k_chunk,
                                                        float* __restrict__ out) {
    __shared__ __align__(16) float xs[kRtK][kRtM + 4];
    __shared__ __align__(16) float rs[kRtK][kRtN + 4];
    const int t0 = blockIdx.x * kRtM, e0 = blockIdx.y * kRtN, tid = threadIdx.x;
    const int kb = blockIdx.z * k_chunk, nsteps = k_chunk / kRtK;
    const int tr = tid >> 4, tcol = tid & 15;
    // loader: rows lr and lr + 64 of the x tile and row lr of the router tile, 8 consecutive k at lk
    const int lr = tid >> 2, lk = (tid & 3) * 8;
    const __nv_bfloat16* xrow0 = t0 + lr < T ? xb + (size_t)(t0 + lr) * D + kb + lk : nullptr;
    const __nv_bfloat16* xrow1 = t0 + lr + 64 < T ? xb + (size_t)(t0 + lr + 64) * D + kb + lk : nullptr;
    const int e = e0 + lr;
    const float* rrow = e < E ? router + (size_t)e * D + kb + lk : (e == E && gate_vec ? gate_vec + kb + lk : nullptr);
    uint4 xa = make_uint4(0u, 0u, 0u, 0u), xc = xa;
    float4 r0 = make_float4(0.f, 0.f, 0.f, 0.f), r1 = r0;
    if (xrow0) xa = __ldg(reinterpret_cast<const uint4*>(xrow0));
    if (xrow1) xc = __ldg(reinterpret_cast<const uint4*>(xrow1));
    if (rrow) {
        r0 = __ldg(reinterpret_cast<const float4*>(rrow));
        r1 = __ldg(reinterpret_cast<const float4*>(rrow) + 1);
    }
    float acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
    for (int st = 0; st < nsteps; ++st) {
        {
            const __nv_bfloat162* xp = reinterpret_cast<const __nv_bfloat162*>(&xa);
            const __nv_bfloat162* xq = reinterpret_cast<const __nv_bfloat162*>(&xc);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float2 f = __bfloat1622float2(xp[q]);
                const float2 g = __bfloat1622float2(xq[q]);
                xs[lk + 2 * q][lr] = f.x;
                xs[lk + 2 * q + 1][lr] = f.y;
                xs[lk + 2 * q][lr + 64] = g.x;
                xs[lk + 2 * q + 1][lr + 64] = g.y;
            }
            rs[lk + 0][lr] = r0.x;
            rs[lk + 1][lr] = r0.y;
            rs[lk + 2][lr] = r0.z;
            rs[lk + 3][lr] = r0.w;
            rs[lk + 4][lr] = r1.x;
            rs[lk + 5][lr] = r1.y;
            rs[lk + 6][lr] = r1.z;
            rs[lk + 7][lr] = r1.w;
        }
        __syncthreads();
        if (st + 1 < nsteps) {  // the next step's operands, in flight during this step's arithmetic
            const int off = (st + 1) * kRtK;
            if (xrow0) xa = __ldg(reinterpret_cast<const uint4*>(xrow0 + off));
            if (xrow1) xc = __ldg(reinterpret_cast<const uint4*>(xrow1 + off));
            if (rrow) {
                r0 = __ldg(reinterpret_cast<const float4*>(rrow + off));
                r1 = __ldg(reinterpret_cast<const float4*>(rrow + off) + 1);
            }
        }
#pragma unroll 8
        for (int kk = 0; kk < kRtK; ++kk) {
            const float4 x0 = *reinterpret_cast<const float4*>(&xs[kk][tr * 8]);
            const float4 x1 = *reinterpret_cast<const float4*>(&xs[kk][tr * 8 + 4]);
            const float4 rq = *reinterpret_cast<const float4*>(&rs[kk][tcol * 4]);
            const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w}, rv[4] = {rq.x, rq.y, rq.z, rq.w};
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(xv[i], rv[j], acc[i][j]);
        }
        __syncthreads();
    }
    float* o = out + (size_t)blockIdx.z * T * (E + 1);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int tt = t0 + tr * 8 + i;
        if (tt >= T) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int ee = e0 + tcol * 4 + j;
            if (ee <= E) o[(size_t)tt * (E + 1) + ee] = acc[i][j];
        }
    }
}

// logits[i] = part[0][i] + part[1][i] + ... in chunk order.
__global__ void __launch_bounds__(256) pf_logit_reduce_kernel(const float* __restrict__ part, int S, size_t n,
                                                              float* __restrict__ logits) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        float v = part[i];
        for (int s = 1; s < S; ++s) v += part[(size_t)s * n + i];
        logits[i] = v;
    }
}

// K chunks of the router GEMM for a chunk of T tokens: enough CTAs to cover
// the SMs, each chunk a multiple of 128 columns.
int router_splits(int T, int E, int D) {
    const int tiles = ((T + kRtM - 1) / kRtM) * ((E + 1 + kRtN - 1) / kRtN);
    int S = 1;
    while (S * 2 * tiles <= 2 * 148 && D % (S * 2 * 128) == 0) S *= 2;
    return S;
}

constexpr int kTopkWarps = 8;

// Top-k per token, warp per token; weights renormalised over the k; the
// shared-expert logit is the gate-vector row (0 without a gate vector).
// thr_mode != 0: the tie-admitting threshold select at the thr_k-th
// probability instead (warp_select_threshold), k slots.
__global__ void __launch_bounds__(kTopkWarps * 32) pf_topk_kernel(const float* __restrict__ logits, int T, int E,
                                                                  int k, int has_gate, int32_t* ids, float* weights,
                                                                  float* shared_logit, int* status, int thr_mode,
                                                                  int thr_k) {
    __shared__ float cv[kTopkWarps][kCandCap];
    __shared__ int ci[kTopkWarps][kCandCap];
    __shared__ float sv[kTopkWarps][kMaxTopK];
    __shared__ int si[kTopkWarps][kMaxTopK];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int t = blockIdx.x * kTopkWarps + warp;
    if (t >= T) return;
    const float* lg = logits + (size_t)t * (E + 1);
    if (thr_mode) {
        const float lmax = warp_select_threshold(lg, E, thr_k, k, 0, E, thr_mode == 2, ids + (size_t)t * k,
                                                 weights + (size_t)t * k);
        if (lane == 0) {
            if (!(fabsf(lmax) <= 3.0e38f)) record_status(status, QMOE_ERR_NOT_FINITE);
            if (shared_logit) shared_logit[t] = has_gate ? __ldcg(lg + E) : 0.0f;
        }
        return;
    }
    const float lmax = warp_topk(lg, E, k, cv[warp], ci[warp], sv[warp], si[warp]);
    const float e = lane < k ? sv[warp][lane] : 0.0f;
    const float sum = warp_sum(e);
    if (lane < k) {
        if (!(fabsf(lmax) <= 3.0e38f)) record_status(status, QMOE_ERR_NOT_FINITE);
        ids[(size_t)t * k + lane] = si[warp][lane];
        weights[(size_t)t * k + lane] = e / sum;
    }
    if (lane == 0 && shared_logit) shared_logit[t] = has_gate ? __ldcg(lg + E) : 0.0f;
}

// counts[g] += 1 for every in-range routed id; out-of-range ids are skipped
// and reported.
__global__ void pf_count_kernel(const int32_t* __restrict__ ids, int n, int E, int* counts, int* status) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int g = ids[i];
    if (g >= 0 && g < E) atomicAdd(counts + g, 1);
    else record_status(status, QMOE_ERR_DEVICE_RANGE);
}

// One CTA: counts[E] = shared-group size, exclusive scans of counts (slot rows)
// and of the n-tile counts, and the n-tile table.
constexpr int kScanThreads = 1024;
// Groups of at most gv_max tokens are listed in gv instead (the grouped GEMV
// path); the others are cut into n-tiles of <= kGNMax tokens for the
// tensor-core path.  meta: [0] n-tiles, [1] slot rows, [2] small groups.
__global__ void __launch_bounds__(kScanThreads) pf_scan_kernel(int* counts, int G, int shared_count, int gv_max,
                                                               int* offsets, int4* ntiles, int4* gv, int* meta) {
    __shared__ int s_rows[kScanThreads / 32], s_nt[kScanThreads / 32], s_ns[kScanThreads / 32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // G <= 1025 groups: thread tid owns groups 2*tid and 2*tid + 1.
    int c[2], nt[2], sg[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const int g = 2 * tid + j;
        c[j] = 0;
        if (g < G) c[j] = g == G - 1 ? shared_count : counts[g];
        sg[j] = c[j] > 0 && c[j] <= gv_max ? 1 : 0;
        nt[j] = sg[j] ? 0 : (c[j] + kGNMax - 1) / kGNMax;
    }
    if (2 * tid + 1 == G - 1 || 2 * tid == G - 1) counts[G - 1] = shared_count;
    int r = c[0] + c[1], n = nt[0] + nt[1], ns = sg[0] + sg[1];
    int ri = r, ni = n, nsi = ns;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int yr = __shfl_up_sync(0xffffffffu, ri, o), yn = __shfl_up_sync(0xffffffffu, ni, o),
                  ys = __shfl_up_sync(0xffffffffu, nsi, o);
        if (lane >= o) {
            ri += yr;
            ni += yn;
            nsi += ys;
        }
    }
    if (lane == 31) {
        s_rows[warp] = ri;
        s_nt[warp] = ni;
        s_ns[warp] = nsi;
    }
    __syncthreads();
    if (warp == 0) {
        int vr = s_rows[lane], vn = s_nt[lane], vs = s_ns[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int yr = __shfl_up_sync(0xffffffffu, vr, o), yn = __shfl_up_sync(0xffffffffu, vn, o),
                      ys = __shfl_up_sync(0xffffffffu, vs, o);
            if (lane >= o) {
                vr += yr;
                vn += yn;
                vs += ys;
            }
        }
        s_rows[lane] = vr;
        s_nt[lane] = vn;
        s_ns[lane] = vs;
    }
    __syncthreads();
    const int wr = warp > 0 ? s_rows[warp - 1] : 0, wn = warp > 0 ? s_nt[warp - 1] : 0,
              ws = warp > 0 ? s_ns[warp - 1] : 0;
    // exclusive prefixes of this thread's first group
    int row = wr + ri - r, nti = wn + ni - n, nsg = ws + nsi - ns;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const int g = 2 * tid + j;
        if (g < G) {
            offsets[g] = row;
            if (sg[j]) gv[nsg] = make_int4(g, row, c[j], 0);
            for (int q = 0; q < nt[j]; ++q) {
                const int n0 = q * kGNMax;
                ntiles[nti + q] = make_int4(g, n0, min(kGNMax, c[j] - n0), row + n0);
            }
        }
        row += c[j];
        nti += nt[j];
        nsg += sg[j];
    }
    if (tid == kScanThreads - 1) {
        meta[0] = nti;  // tensor-core n-tiles
        meta[1] = row;  // total slot rows
        meta[2] = nsg;  // small groups
        offsets[G] = row;
    }
}

// ---- small groups: grouped GEMV ---------------------------------------------
// A group of at most kGvMax tokens (most experts of a short chunk: ~2.7
// tokens each at T = 128) is not worth expanding to bf16 for the tensor
// cores: a warp decodes each weight row once with the decode path's integer
// core (4-bit codes through the codebook, dp2a against the activations in
// block floating point) and dots it with every token of the group.  Items are
// (group, block of rows); the CTAs walk them persistently.
constexpr int kGvMax = 8;     // largest group the GEMV path takes (the default threshold)
constexpr int kGvWarps = 8;
constexpr int kGvPairs = 64;  // gate|up row pairs per item
constexpr int kGvRows = 256;  // down rows per item

struct GvArgs {
    int D, I, E;
    const uint8_t* gate_up;
    const uint8_t* down;
    const uint8_t* sh_gate_up;
    const uint8_t* sh_down;
    size_t gu_expert_bytes, dn_expert_bytes;
    const int4* gv;     // small groups {group, first slot row, tokens, 0}
    const int* meta;    // meta[2]: number of small groups
    const int* slot_tok;
    const float* slot_w;
    const int* xq;      // [T][4 quads][D/32 blocks][4 words]: x in block floating point
    const float* xs;    // [T][D/32] steps
    __nv_bfloat16* h;   // [rows][I]
    float* out;         // [T][D]
};

// x -> block floating point in the [quad][block][4 words] order: lanes on
// consecutive blocks read consecutive 16-byte chunks of shared memory.
__global__ void __launch_bounds__(256) pf_xq_kernel(const __nv_bfloat16* __restrict__ xb, int T, int D,
                                                    const int* __restrict__ meta, int* __restrict__ xq,
                                                    float* __restrict__ xs) {
    if (__ldg(meta + 2) == 0) return;  // no small groups in this chunk
    const int lane = threadIdx.x & 31, nb = D >> 5;
    const size_t n = (size_t)T * nb;
    for (size_t w = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; w < n;
         w += ((size_t)gridDim.x * blockDim.x) >> 5) {
        const int t = (int)(w / nb), b = (int)(w % nb);
        const float v = __bfloat162float(xb[(size_t)t * D + b * 32 + lane]);
        float st;
        const int pw = warp_block_fp(v, &st);
        if (lane < 16) xq[(((size_t)t * 4 + (lane >> 2)) * nb + b) * 4 + (lane & 3)] = pw;
        if (lane == 0) xs[(size_t)t * nb + b] = st;
    }
}

// gate|up + SwiGLU of the small groups -> h (bf16, the tensor-core path's rows).
// SBL: 32-value blocks of a row per lane (blocks lane, lane + 32, ...).
template <int SBL>
__global__ void __launch_bounds__(kGvWarps * 32) pf_gv_gateup_kernel(const __grid_constant__ GvArgs a) {
    extern __shared__ __align__(16) unsigned char gsm[];
    __shared__ int s_tok[kGvMax];
    const int D = a.D, nb = D >> 5, words = nb * 16;
    int* sxq = reinterpret_cast<int*>(gsm);                         // [kGvMax][4][nb][4]
    float* sxs = reinterpret_cast<float*>(sxq + (size_t)kGvMax * words);  // [kGvMax][nb]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ipg = a.I / kGvPairs;
    const int n_items = __ldg(a.meta + 2) * ipg;
    const int row_bytes = (D >> 8) * QMOE_SB_BYTES;
    for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
        const int4 grp = __ldg(a.gv + it / ipg);
        const int g = grp.x, row0 = grp.y, cnt = min(grp.z, kGvMax), r0 = (it % ipg) * kGvPairs;
        __syncthreads();  // the previous item's activations are no longer read
        if (tid < cnt) s_tok[tid] = __ldg(a.slot_tok + row0 + tid);
        __syncthreads();
        for (int m = 0; m < cnt; ++m) {
            const int4* src = reinterpret_cast<const int4*>(a.xq + (size_t)s_tok[m] * words);
            int4* dst = reinterpret_cast<int4*>(sxq + (size_t)m * words);
            for (int i = tid; i < words / 4; i += blockDim.x) dst[i] = __ldg(src + i);
            for (int i = tid; i < nb; i += blockDim.x) sxs[m * nb + i] = __ldg(a.xs + (size_t)s_tok[m] * nb + i);
        }
        __syncthreads();
        const uint8_t* base = g < a.E ? a.gate_up + (size_t)g * a.gu_expert_bytes : a.sh_gate_up;
        for (int pi = warp; pi < kGvPairs; pi += kGvWarps) {
            const int r = r0 + pi;
            const uint8_t* grow = base + (size_t)r * row_bytes;
            const uint8_t* urow = base + (size_t)(a.I + r) * row_bytes;
            uint2 hg[SBL], hu[SBL], qg[SBL][2], qu[SBL][2];
#pragma unroll
            for (int i = 0; i < SBL; ++i) {
                const int b = lane + 32 * i;
                if (b < nb) {
                    const int off = (b >> 3) * QMOE_SB_BYTES, q = off + 8 + 16 * (b & 7);
                    hg[i] = __ldg(reinterpret_cast<const uint2*>(grow + off));
                    hu[i] = __ldg(reinterpret_cast<const uint2*>(urow + off));
                    qg[i][0] = __ldg(reinterpret_cast<const uint2*>(grow + q));
                    qg[i][1] = __ldg(reinterpret_cast<const uint2*>(grow + q + 8));
                    qu[i][0] = __ldg(reinterpret_cast<const uint2*>(urow + q));
                    qu[i][1] = __ldg(reinterpret_cast<const uint2*>(urow + q + 8));
                }
            }
            float accg[kGvMax], accu[kGvMax];
#pragma unroll
            for (int m = 0; m < kGvMax; ++m) accg[m] = accu[m] = 0.0f;
#pragma unroll
            for (int i = 0; i < SBL; ++i) {
                const int b = lane + 32 * i;
                if (b >= nb) continue;
                const int ib = b & 7;
                const float dg = __half2float(__ushort_as_half((unsigned short)(hg[i].x & 0xFFFFu))) *
                                 (float)(qmoe_iq4xs_ls(hg[i].x, hg[i].y, ib) - 32);
                const float du = __half2float(__ushort_as_half((unsigned short)(hu[i].x & 0xFFFFu))) *
                                 (float)(qmoe_iq4xs_ls(hu[i].x, hu[i].y, ib) - 32);
                uint32_t wg[8], wu[8];  // the codes' codebook bytes, decoded once for every token
                qmoe_subblock_decode(qg[i][0].x, qg[i][0].y, qg[i][1].x, qg[i][1].y, wg);
                qmoe_subblock_decode(qu[i][0].x, qu[i][0].y, qu[i][1].x, qu[i][1].y, wu);
#pragma unroll
                for (int m = 0; m < kGvMax; ++m) {
                    if (m < cnt) {
                        int xp[16];
#pragma unroll
                        for (int v = 0; v < 4; ++v) {
                            const int4 w4 = *reinterpret_cast<const int4*>(sxq + (((size_t)m * 4 + v) * nb + b) * 4);
                            xp[4 * v] = w4.x;
                            xp[4 * v + 1] = w4.y;
                            xp[4 * v + 2] = w4.z;
                            xp[4 * v + 3] = w4.w;
                        }
                        const float st = sxs[m * nb + b];
                        const int sgv = qmoe_subblock_dot_decoded(wg, xp);
                        const int suv = qmoe_subblock_dot_decoded(wu, xp);
                        accg[m] = fmaf(dg * st, (float)sgv, accg[m]);
                        accu[m] = fmaf(du * st, (float)suv, accu[m]);
                    }
                }
            }
#pragma unroll
            for (int m = 0; m < kGvMax; ++m) {
                if (m < cnt) {
                    const float gs = warp_sum(accg[m]), us = warp_sum(accu[m]);
                    if (lane == 0) a.h[(size_t)(row0 + m) * a.I + r] = __float2bfloat16_rn(silu(gs) * us);
                }
            }
        }
    }
}

// down of the small groups, weighted and scatter-added into out: a half
// warp per output row (two rows at a time), its lanes on the row's blocks.
__global__ void __launch_bounds__(kGvWarps * 32) pf_gv_down_kernel(const __grid_constant__ GvArgs a) {
    extern __shared__ __align__(16) unsigned char dsm[];
    __shared__ int s_tok[kGvMax];
    __shared__ float s_w[kGvMax];
    const int D = a.D, I = a.I, nbh = I >> 5;
    int* shq = reinterpret_cast<int*>(dsm);                               // [kGvMax][4][nbh][4]
    float* shs = reinterpret_cast<float*>(shq + (size_t)kGvMax * nbh * 16);  // [kGvMax][nbh]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, half = lane >> 4, hl = lane & 15;
    const int ipg = D / kGvRows;
    const int n_items = __ldg(a.meta + 2) * ipg;
    const int drb = (I >> 8) * QMOE_SB_BYTES;
    for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
        const int4 grp = __ldg(a.gv + it / ipg);
        const int g = grp.x, row0 = grp.y, cnt = min(grp.z, kGvMax), j0 = (it % ipg) * kGvRows;
        __syncthreads();
        if (tid < cnt) {
            s_tok[tid] = __ldg(a.slot_tok + row0 + tid);
            s_w[tid] = __ldg(a.slot_w + row0 + tid);
        }
        // the group's h rows -> block floating point, a warp per 32-value block
        for (int blk = warp; blk < cnt * nbh; blk += kGvWarps) {
            const int m = blk / nbh, b = blk - m * nbh;
            const float v = __bfloat162float(a.h[(size_t)(row0 + m) * I + b * 32 + lane]);
            float st;
            const int pw = warp_block_fp(v, &st);
            if (lane < 16) shq[(((size_t)m * 4 + (lane >> 2)) * nbh + b) * 4 + (lane & 3)] = pw;
            if (lane == 0) shs[m * nbh + b] = st;
        }
        __syncthreads();
        const uint8_t* base = g < a.E ? a.down + (size_t)g * a.dn_expert_bytes : a.sh_down;
        for (int jj = 2 * warp + half; jj < kGvRows; jj += 2 * kGvWarps) {
            const int j = j0 + jj;
            const uint8_t* row = base + (size_t)j * drb;
            float acc[kGvMax];
#pragma unroll
            for (int m = 0; m < kGvMax; ++m) acc[m] = 0.0f;
            for (int t = hl; t < nbh; t += 16) {
                const uint8_t* blk = row + (t >> 3) * QMOE_SB_BYTES;
                const int ib = t & 7;
                const uint2 hd = __ldg(reinterpret_cast<const uint2*>(blk));
                const uint2 q0 = __ldg(reinterpret_cast<const uint2*>(blk + 8 + 16 * ib));
                const uint2 q1 = __ldg(reinterpret_cast<const uint2*>(blk + 16 + 16 * ib));
                const float dl = __half2float(__ushort_as_half((unsigned short)(hd.x & 0xFFFFu))) *
                                 (float)(qmoe_iq4xs_ls(hd.x, hd.y, ib) - 32);
                uint32_t wd[8];
                qmoe_subblock_decode(q0.x, q0.y, q1.x, q1.y, wd);
#pragma unroll
                for (int m = 0; m < kGvMax; ++m) {
                    if (m < cnt) {
                        int xp[16];
#pragma unroll
                        for (int v = 0; v < 4; ++v) {
                            const int4 w4 = *reinterpret_cast<const int4*>(shq + (((size_t)m * 4 + v) * nbh + t) * 4);
                            xp[4 * v] = w4.x;
                            xp[4 * v + 1] = w4.y;
                            xp[4 * v + 2] = w4.z;
                            xp[4 * v + 3] = w4.w;
                        }
                        const int S = qmoe_subblock_dot_decoded(wd, xp);
                        acc[m] = fmaf(dl * shs[m * nbh + t], (float)S, acc[m]);
                    }
                }
            }
#pragma unroll
            for (int m = 0; m < kGvMax; ++m) {
                if (m < cnt) {
                    float v = acc[m];
#pragma unroll
                    for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                    if (hl == 0) atomicAdd(a.out + (size_t)s_tok[m] * D + j, s_w[m] * v);
                }
            }
        }
    }
}

// Slot rows in token order: warp per routed group scans every token's ids
// (held in shared memory) and ranks its hits with a ballot; the shared group
// lists every token.
// Slot rows: a thread per (token, slot) entry takes the next free row of its
// group, counting the group's size (left by the count and scan kernels)
// down with an atomic, then a thread per token fills the shared group's rows
// in token order.  The order within a routed group is the arrival order: a
// token's results do not depend on its column in a tile (each accumulator
// column sums over K in the same order), so only the rows' bookkeeping sees
// it.
__global__ void __launch_bounds__(256) pf_place_kernel(const int32_t* __restrict__ ids,
                                                       const float* __restrict__ weights,
                                                       const float* __restrict__ shared_logit, int T, int k, int E,
                                                       int has_shared, const int* __restrict__ offsets, int* counts,
                                                       int* slot_tok, float* slot_w) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const int n = T * k;
    if (i < n) {
        // Every (token, slot) naming g is placed, so the rows match the counts even when a
        // caller's routing repeats an expert within a token.
        const int g = ids[i];
        if (g >= 0 && g < E) {
            const int r = offsets[g] + atomicSub(counts + g, 1) - 1;
            slot_tok[r] = i / k;
            slot_w[r] = weights[i];
        }
    } else if (has_shared && i < n + T) {
        const int t = i - n, base = offsets[E];
        slot_tok[base + t] = t;
        slot_w[base + t] = sigmoid(shared_logit[t]);
    }
}

}  // namespace

// ---- workspace and launches ---------------------------------------------------

struct PfLayout {
    size_t status, meta, trace, xb, logits, part, ids, weights, slog, counts, offsets, ntiles, gv, slot_tok, slot_w, h,
        xg, xq, xs, total;
    int max_ntiles, rows;
};

static size_t pf_align(size_t v) { return (v + 255) / 256 * 256; }

PfLayout pf_layout(const qmoe_dims& d, int T) {
    PfLayout L{};
    const int E = d.n_experts, k = d.top_k, G = E + 1;
    L.rows = T * (k + 1);
    L.max_ntiles = G + L.rows / kGNMax + 1;
    size_t o = 0;
    L.status = 0;
    L.meta = 64;
    L.trace = 256;  // [64 slots][8] u64 clock stamps of CTA 0's pipeline (per launch)
    o = 256 + kPfTraceBytes;
    L.xb = o;
    o = pf_align(o + (size_t)T * d.hidden * 2);
    L.logits = o;
    o = pf_align(o + (size_t)T * G * 4);
    L.part = o;  // the router's K-chunk partials when it splits K
    {
        const int S = router_splits(T, E, d.hidden);
        o = pf_align(o + (S > 1 ? (size_t)S * T * G * 4 : 0));
    }
    L.ids = o;
    o = pf_align(o + (size_t)T * k * 4);
    L.weights = o;
    o = pf_align(o + (size_t)T * k * 4);
    L.slog = o;
    o = pf_align(o + (size_t)T * 4);
    L.counts = o;
    o = pf_align(o + (size_t)G * 4);
    L.offsets = o;
    o = pf_align(o + (size_t)(G + 1) * 4);
    L.ntiles = o;
    o = pf_align(o + (size_t)L.max_ntiles * 16);
    L.gv = o;  // small groups
    o = pf_align(o + (size_t)G * 16);
    L.slot_tok = o;
    o = pf_align(o + (size_t)L.rows * 4);
    L.slot_w = o;
    o = pf_align(o + (size_t)L.rows * 4);
    L.h = o;
    o = pf_align(o + (size_t)L.rows * d.inter * 2);
    L.xg = o;
    o = pf_align(o + (size_t)L.rows * d.hidden * 2);
    L.xq = o;  // x in block floating point, for the small groups
    o = pf_align(o + (size_t)T * (d.hidden / 32) * 64);
    L.xs = o;
    o = pf_align(o + (size_t)T * (d.hidden / 32) * 4);
    L.total = o;
    return L;
}

int prefill_max_tokens() { return kPfMaxTokens; }

// Largest expert group the grouped GEMV takes (0: every group goes to the
// tensor-core path).  One process-wide setting for every device and thread,
// read once per call when the call is issued; atomic, so a setter on one
// thread and a prefill issued on another do not race.
static std::atomic<int> g_small_group_max{kGvMax};
int prefill_small_group_max(int n) {
    if (n < 0) return g_small_group_max.load();
    return g_small_group_max.exchange(n < kGvMax ? n : kGvMax);
}

// Whether the grouped GEMM's CTA 0 stamps its pipeline clocks into the
// workspace (off by default: the stamps cost CTA 0, and with it the launch,
// tens of cycles per slot).  Process-wide, atomic like the setting above.
static std::atomic<int> g_pf_trace{0};
int prefill_trace(int enable) {
    if (enable < 0) return g_pf_trace.load();
    return g_pf_trace.exchange(enable ? 1 : 0);
}

size_t prefill_workspace_bytes(const qmoe_dims& d, int T) { return pf_layout(d, T).total; }

void prefill_route_buffers(const qmoe_dims& d, int T, unsigned char* ws, int32_t** ids, float** weights,
                           float** shared_logit) {
    const PfLayout L = pf_layout(d, T);
    *ids = reinterpret_cast<int32_t*>(ws + L.ids);
    *weights = reinterpret_cast<float*>(ws + L.weights);
    *shared_logit = reinterpret_cast<float*>(ws + L.slog);
}

bool prefill_supported(const qmoe_dims& d) {
    if (d.expert_lo != 0 || d.expert_hi != d.n_experts) return false;  // unsharded only
    if (d.inter_local != d.inter || d.down_ib0 != 0 || d.down_nsub != 8 || d.down_nseg * 256 != d.inter)
        return false;
    if (d.hidden % kGStageK || d.inter % kGStageK) return false;
    if (d.n_experts + 1 > 2 * kScanThreads) return false;
    if (d.n_experts > 32767) return false;  // ids held as int16 while grouping
    if (d.sh_inter_local != 0 &&
        (d.sh_inter_local != d.inter || d.sh_down_ib0 != 0 || d.sh_down_nsub != 8 || d.sh_down_nseg * 256 != d.inter))
        return false;
    return true;
}

const __nv_bfloat16* prefill_act_bf16(const void* x, int x_f32, bool x_ok, int T, const qmoe_dims& d,
                                      unsigned char* ws, cudaStream_t s) {
    if (x_ok) return reinterpret_cast<const __nv_bfloat16*>(x);
    const PfLayout L = pf_layout(d, T);
    __nv_bfloat16* xc = reinterpret_cast<__nv_bfloat16*>(ws + L.xb);
    const size_t n = (size_t)T * d.hidden;
    const size_t blocks = (n + 255) / 256;
    pf_convert_kernel<<<(unsigned)(blocks < 4096 ? blocks : 4096), 256, 0, s>>>(x, x_f32, n, xc);
    return xc;
}

cudaError_t launch_prefill_route(const __nv_bfloat16* xb, int T, const qmoe_layer_weights& w, const qmoe_dims& d,
                                 unsigned char* ws, int32_t* ids, float* weights, float* shared_logit,
                                 cudaStream_t s, int thr_mode, int thr_k) {
    const PfLayout L = pf_layout(d, T);
    int* status = reinterpret_cast<int*>(ws + L.status);
    const int E = d.n_experts;
    const int S = router_splits(T, E, d.hidden);
    float* logits = reinterpret_cast<float*>(ws + L.logits);
    dim3 grid((unsigned)((T + kRtM - 1) / kRtM), (unsigned)((E + 1 + kRtN - 1) / kRtN), (unsigned)S);
    pf_router_kernel<<<grid, 256, 0, s>>>(xb, T, d.hidden, w.router, w.gate_vec, E, d.hidden / S,
                                          S > 1 ? reinterpret_cast<float*>(ws + L.part) : logits);
    if (S > 1) {
        const size_t n = (size_t)T * (E + 1);
        const size_t blocks = (n + 255) / 256;
        pf_logit_reduce_kernel<<<(unsigned)(blocks < 1184 ? blocks : 1184), 256, 0, s>>>(
            reinterpret_cast<const float*>(ws + L.part), S, n, logits);
    }
    pf_topk_kernel<<<(unsigned)((T + kTopkWarps - 1) / kTopkWarps), kTopkWarps * 32, 0, s>>>(
        reinterpret_cast<const float*>(ws + L.logits), T, E, d.top_k, w.gate_vec ? 1 : 0, ids, weights,
        shared_logit, status, thr_mode, thr_k);
    return cudaGetLastError();
}

cudaError_t launch_prefill_experts(const __nv_bfloat16* xb, int T, const int32_t* ids, const float* weights,
                                   const float* shared_logit, const qmoe_layer_weights& w, const qmoe_dims& d,
                                   float* out, unsigned char* ws, cudaStream_t s) {
    const PfLayout L = pf_layout(d, T);
    const int E = d.n_experts, k = d.top_k, G = E + 1;
    const bool has_shared = d.sh_inter_local > 0;
    int* status = reinterpret_cast<int*>(ws + L.status);
    int* meta = reinterpret_cast<int*>(ws + L.meta);
    int* counts = reinterpret_cast<int*>(ws + L.counts);
    int* offsets = reinterpret_cast<int*>(ws + L.offsets);
    int4* ntiles = reinterpret_cast<int4*>(ws + L.ntiles);
    int* slot_tok = reinterpret_cast<int*>(ws + L.slot_tok);
    float* slot_w = reinterpret_cast<float*>(ws + L.slot_w);
    __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(ws + L.h);

    cudaError_t err = cudaMemsetAsync(counts, 0, (size_t)G * 4, s);
    if (err != cudaSuccess) return err;
    const int n = T * k;
    pf_count_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(ids, n, E, counts, status);
    int4* gv = reinterpret_cast<int4*>(ws + L.gv);
    pf_scan_kernel<<<1, kScanThreads, 0, s>>>(counts, G, has_shared ? T : 0, g_small_group_max.load(), offsets, ntiles, gv,
                                              meta);
    pf_place_kernel<<<(unsigned)((n + T + 255) / 256), 256, 0, s>>>(ids, weights, shared_logit, T, k, E,
                                                                 has_shared ? 1 : 0, offsets, counts, slot_tok,
                                                                 slot_w);

    GemmArgs a{};
    a.D = d.hidden;
    a.I = d.inter;
    a.E = E;
    a.T = T;
    a.gate_up = reinterpret_cast<const uint8_t*>(w.gate_up);
    a.down = reinterpret_cast<const uint8_t*>(w.down);
    a.sh_gate_up = reinterpret_cast<const uint8_t*>(w.sh_gate_up);
    a.sh_down = reinterpret_cast<const uint8_t*>(w.sh_down);
    a.gu_expert_bytes = (size_t)2 * d.inter * (d.hidden / 256) * QMOE_SB_BYTES;
    a.dn_expert_bytes = (size_t)d.hidden * (d.inter / 256) * QMOE_SB_BYTES;
    a.x = xb;
    a.h = h;
    a.slot_tok = slot_tok;
    a.slot_w = slot_w;
    a.ntiles = ntiles;
    a.meta = meta;
    a.out = out;
    a.status = status;
    a.trace = g_pf_trace.load() ? reinterpret_cast<unsigned long long*>(ws + L.trace) : nullptr;
    err = smem_opt_in(reinterpret_cast<const void*>(grouped_gemm_kernel), kGSmemBytes);
    if (err != cudaSuccess) return err;
    const int n_sm = device_sm_count();
    const unsigned long long rb = (unsigned long long)(d.hidden / 256) * QMOE_SB_BYTES;
    const unsigned long long drb = (unsigned long long)(d.inter / 256) * QMOE_SB_BYTES;
    __nv_bfloat16* xg = reinterpret_cast<__nv_bfloat16*>(ws + L.xg);
    pf_gather_kernel<<<(unsigned)L.rows, 256, 0, s>>>(xb, d.hidden, slot_tok, meta, T, xg);
    a.mode = 0;
    err = encode_2d(&a.bmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, xg, (unsigned long long)d.hidden,
                    (unsigned long long)L.rows, (unsigned long long)d.hidden * 2, kGAtomK, kGNMax,
                    CU_TENSOR_MAP_SWIZZLE_128B);
    if (err != cudaSuccess) return err;
    err = encode_2d(&a.wmap, CU_TENSOR_MAP_DATA_TYPE_UINT16, w.gate_up, rb / 2, (unsigned long long)E * 2 * d.inter, rb,
                    kGStageRowB / 2, 64);
    if (err == cudaSuccess && has_shared)
        err = encode_2d(&a.shmap, CU_TENSOR_MAP_DATA_TYPE_UINT16, w.sh_gate_up, rb / 2, 2ull * d.inter, rb,
                        kGStageRowB / 2, 64);
    if (err != cudaSuccess) return err;
    grouped_gemm_kernel<<<(unsigned)n_sm, kGThreads, kGSmemBytes, s>>>(a);

    // the small groups (grouped GEMV), gate|up
    GvArgs v{};
    v.D = d.hidden;
    v.I = d.inter;
    v.E = E;
    v.gate_up = a.gate_up;
    v.down = a.down;
    v.sh_gate_up = a.sh_gate_up;
    v.sh_down = a.sh_down;
    v.gu_expert_bytes = a.gu_expert_bytes;
    v.dn_expert_bytes = a.dn_expert_bytes;
    v.gv = gv;
    v.meta = meta;
    v.slot_tok = slot_tok;
    v.slot_w = slot_w;
    v.xq = reinterpret_cast<int*>(ws + L.xq);
    v.xs = reinterpret_cast<float*>(ws + L.xs);
    v.h = h;
    v.out = out;
    const int nb = d.hidden / 32;
    {
        const size_t n = (size_t)T * nb;
        const size_t blocks = (n + 7) / 8;
        pf_xq_kernel<<<(unsigned)(blocks < 4096 ? blocks : 4096), 256, 0, s>>>(xb, T, d.hidden, meta,
                                                                              reinterpret_cast<int*>(ws + L.xq),
                                                                              reinterpret_cast<float*>(ws + L.xs));
        const size_t gsm = (size_t)kGvMax * nb * 16 * 4 + (size_t)kGvMax * nb * 4;
        void (*gk)(GvArgs) = nb <= 32 ? pf_gv_gateup_kernel<1> : nb <= 64 ? pf_gv_gateup_kernel<2>
                                                                           : pf_gv_gateup_kernel<4>;
        err = smem_opt_in(reinterpret_cast<const void*>(gk), (int)gsm);
        if (err != cudaSuccess) return err;
        int per_sm = 1;  // persistent: as many CTAs as stay resident
        err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gk, kGvWarps * 32, gsm);
        if (err != cudaSuccess) return err;
        gk<<<(unsigned)(n_sm * (per_sm > 0 ? per_sm : 1)), kGvWarps * 32, gsm, s>>>(v);
    }

    err = cudaMemsetAsync(out, 0, (size_t)T * d.hidden * 4, s);
    if (err != cudaSuccess) return err;
    {
        const int nbh = d.inter / 32;
        const size_t dsm = (size_t)kGvMax * nbh * 16 * 4 + (size_t)kGvMax * nbh * 4;
        err = smem_opt_in(reinterpret_cast<const void*>(pf_gv_down_kernel), (int)dsm);
        if (err != cudaSuccess) return err;
        int per_sm = 1;
        err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, pf_gv_down_kernel, kGvWarps * 32, dsm);
        if (err != cudaSuccess) return err;
        pf_gv_down_kernel<<<(unsigned)(n_sm * (per_sm > 0 ? per_sm : 1)), kGvWarps * 32, dsm, s>>>(v);
    }
    a.mode = 1;
    err = encode_2d(&a.bmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, h, (unsigned long long)d.inter, (unsigned long long)L.rows,
                    (unsigned long long)d.inter * 2, kGAtomK, kGNMax, CU_TENSOR_MAP_SWIZZLE_128B);
    if (err != cudaSuccess) return err;
    err = encode_2d(&a.wmap, CU_TENSOR_MAP_DATA_TYPE_UINT16, w.down, drb / 2, (unsigned long long)E * d.hidden, drb,
                    kGStageRowB / 2, kGM);
    if (err == cudaSuccess && has_shared)
        err = encode_2d(&a.shmap, CU_TENSOR_MAP_DATA_TYPE_UINT16, w.sh_down, drb / 2, (unsigned long long)d.hidden,
                        drb, kGStageRowB / 2, kGM);
    if (err != cudaSuccess) return err;
    grouped_gemm_kernel<<<(unsigned)n_sm, kGThreads, kGSmemBytes, s>>>(a);
    return cudaGetLastError();
}

}  // namespace qmoe
