// Gathered expert GEMVs on IQ4_XS weights.
//
//  gate|up:  h[m][slot][r] = silu(G_e[r] . x_m) * (U_e[r] . x_m) for every
//            selected expert e of token m (reference/model.py:411-414; the
//            device pair gather_gemv MODE 2 + fused_swiglu, tt/moe.py:946-953)
//            and the shared expert in slot k (reference/model.py:392-394).
//  down:     out[m][j] = sum_s w[m][s] * D_e[j] . h[m][s]
//                        + sigmoid(x_m . g) * D_sh[j] . h[m][k]
//            (reference/model.py:395-397, 413-417; gather_gemv MODE 0,
//            tt/moe.py:958-975, which stacks experts on K to do the combine).
//
// Only the selected experts' super-blocks are read; nothing is copied or
// dequantised to memory.  Each warp owns one weight row (gate|up: a row pair
// r, I+r; down: an output row j across every selected expert), lanes split
// the row's 32-value sub-blocks (the k-split), and a shuffle reduction folds
// the lanes.  Sub-block sums are exact int32 dot products of the 4-bit codes'
// int8 codebook values with the activation in block floating point (int16
// mantissas, one power-of-two step per 32 values); the fp32 accumulation
// then applies d * (ls - 32) and the activation step.
//
// Tokens that share an expert share its weight reads: the kernels first
// build, per CTA, the list of distinct local experts and which tokens (and
// in which top-k slot) use each one.
#include "common.cuh"

namespace qmoe {
namespace {

constexpr int kWarps = 8;

struct Plan {
    int n;                                   // distinct routed local experts
    int expert[kMaxUnique];                  // local expert index
    uint32_t mask[kMaxUnique];               // tokens using it
    int8_t slot[kMaxUnique][kMaxTokens];     // top-k slot per token
};

__device__ __forceinline__ uint2 ldg2(const uint8_t* p) {
    return __ldg(reinterpret_cast<const uint2*>(p));
}

// Distinct local experts over the M x k routing table, in first-use order.
__device__ void build_plan(const ExpertArgs& a, Plan& p, int* owner /* smem [E] */) {
    const int tid = threadIdx.x;
    const int Mk = a.M * a.k;
    if (a.M == 1) {
        if (tid < 32) {
            const int lane = tid;
            int id = lane < a.k ? a.ids[lane] : -1;
            if (lane < a.k && (id < 0 || id >= a.E)) {
                record_status(a.status, QMOE_ERR_DEVICE_RANGE);
                id = -1;
            }
            const bool local = id >= a.e_lo && id < a.e_hi;
            const unsigned b = __ballot_sync(0xffffffffu, local);
            if (local) {
                const int pos = __popc(b & ((1u << lane) - 1u));
                p.expert[pos] = id - a.e_lo;
                p.mask[pos] = 1u;
                p.slot[pos][0] = (int8_t)lane;
            }
            if (lane == 0) p.n = __popc(b);
        }
        __syncthreads();
        return;
    }
    const int n_loc = a.e_hi - a.e_lo;
    for (int i = tid; i < n_loc; i += blockDim.x) owner[i] = 0x7fffffff;
    __syncthreads();
    for (int t = tid; t < Mk; t += blockDim.x) {
        const int id = a.ids[t];
        if (id < 0 || id >= a.E) {
            record_status(a.status, QMOE_ERR_DEVICE_RANGE);
            continue;
        }
        if (id >= a.e_lo && id < a.e_hi) atomicMin(&owner[id - a.e_lo], t);
    }
    __syncthreads();
    // Serial compaction in t order by one warp: Mk <= 256.
    if (tid < 32) {
        int base = 0;
        for (int t0 = 0; t0 < Mk; t0 += 32) {
            const int t = t0 + tid;
            bool first = false;
            int id = -1;
            if (t < Mk) {
                id = a.ids[t];
                first = id >= a.e_lo && id < a.e_hi && owner[id - a.e_lo] == t;
            }
            const unsigned b = __ballot_sync(0xffffffffu, first);
            if (first) {
                const int pos = base + __popc(b & ((1u << tid) - 1u));
                p.expert[pos] = id - a.e_lo;
                p.mask[pos] = 0u;
                owner[id - a.e_lo] = -1 - pos;  // owner now holds -(pos + 1)
            }
            base += __popc(b);
        }
        if (tid == 0) p.n = base;
    }
    __syncthreads();
    for (int t = tid; t < Mk; t += blockDim.x) {
        const int id = a.ids[t];
        if (id >= a.e_lo && id < a.e_hi) {
            const int pos = -1 - owner[id - a.e_lo];
            const int m = t / a.k, s = t % a.k;
            atomicOr(&p.mask[pos], 1u << m);
            p.slot[pos][m] = (int8_t)s;
        }
    }
    __syncthreads();
}

// Convert n 32-value blocks to block floating point, one warp per block, with
// NB blocks' loads issued per warp before any conversion (one memory round
// trip per NB * kWarps blocks instead of one per block) and the NB blocks'
// reductions and shuffles issued together.
// load(b, lane) -> float: value `lane` of block b; store(b, lane, pair, step).
template <int NB, typename LoadF, typename StoreF>
__device__ __forceinline__ void convert_blocks(int n, LoadF load, StoreF store) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int b0 = warp; b0 < n; b0 += NB * kWarps) {
        float v[NB];
#pragma unroll
        for (int i = 0; i < NB; ++i) {
            const int b = b0 + i * kWarps;
            v[i] = b < n ? load(b, lane) : 0.0f;
        }
        int pw[NB];
        float st[NB];
        warp_block_fp_n<NB>(v, pw, st);
#pragma unroll
        for (int i = 0; i < NB; ++i) {
            const int b = b0 + i * kWarps;
            if (b < n) store(b, lane, pw[i], st[i]);
        }
    }
}

// qmoe_subblock_dot on codes already through the codebook look-up (lo/hi
// of the four qs words), for a sub-block dotted with several tokens.
__device__ __forceinline__ int subblock_dot_lut(const uint32_t (&lo)[4], const uint32_t (&hi)[4], const int* xp) {
    int a0 = __dp2a_lo(xp[0], (int)lo[0], 0);
    int a1 = __dp2a_lo(xp[4], (int)lo[1], 0);
    int a2 = __dp2a_lo(xp[8], (int)lo[2], 0);
    int a3 = __dp2a_lo(xp[12], (int)lo[3], 0);
    a0 = __dp2a_hi(xp[1], (int)lo[0], a0);
    a1 = __dp2a_hi(xp[5], (int)lo[1], a1);
    a2 = __dp2a_hi(xp[9], (int)lo[2], a2);
    a3 = __dp2a_hi(xp[13], (int)lo[3], a3);
    a0 = __dp2a_lo(xp[2], (int)hi[0], a0);
    a1 = __dp2a_lo(xp[6], (int)hi[1], a1);
    a2 = __dp2a_lo(xp[10], (int)hi[2], a2);
    a3 = __dp2a_lo(xp[14], (int)hi[3], a3);
    a0 = __dp2a_hi(xp[3], (int)hi[0], a0);
    a1 = __dp2a_hi(xp[7], (int)hi[1], a1);
    a2 = __dp2a_hi(xp[11], (int)hi[2], a2);
    a3 = __dp2a_hi(xp[15], (int)hi[3], a3);
    return (a0 + a1) + (a2 + a3);
}

// ---------------------------------------------------------------------------
// gate|up + SwiGLU.  SBL = 32-value sub-blocks per lane along D (D / 1024).
template <int MAXM, int SBL>
__global__ void __launch_bounds__(kWarps * 32, (MAXM == 1 || SBL > 2) ? 1 : 3) gateup_kernel(ExpertArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ Plan plan;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int D = a.D, M = a.M;
    const int nsb = D >> 5;
    int* xq = reinterpret_cast<int*>(smem);                        // [M][nsb][16]
    float* xs = reinterpret_cast<float*>(xq + (size_t)M * nsb * 16);  // [M][nsb]
    int* owner = reinterpret_cast<int*>(xs + (size_t)M * nsb);     // [E_loc]

    build_plan(a, plan, owner);
    if (a.xconv) {
        // converted once by the route launch; the same layout as xq then xs,
        // copied with 16-byte loads, eight in flight per thread
        const int n16 = M * nsb * 68 / 16;
        const uint4* src = reinterpret_cast<const uint4*>(a.xconv);
        uint4* dst = reinterpret_cast<uint4*>(smem);
        constexpr int U = 8;
        for (int i0 = tid; i0 < n16; i0 += blockDim.x * U) {
            uint4 v[U];
#pragma unroll
            for (int u = 0; u < U; ++u)
                if (i0 + u * (int)blockDim.x < n16) v[u] = __ldcg(src + i0 + u * blockDim.x);
#pragma unroll
            for (int u = 0; u < U; ++u)
                if (i0 + u * (int)blockDim.x < n16) dst[i0 + u * blockDim.x] = v[u];
        }
    } else {
        convert_blocks<16>(
            M * nsb, [&](int b, int ln) { return load_act(a.x, a.x_f32, (size_t)b * 32 + ln); },
            [&](int b, int ln, int pw, float st) {
                if (ln < 16) xq[(size_t)b * 16 + ln] = pw;
                if (ln == 0) xs[b] = st;
            });
    }
    __syncthreads();

    // M == 1: the lane's activation blocks stay in registers for every row.
    int xr[SBL][16];
    float xsr[SBL];
    if (MAXM == 1) {
#pragma unroll
        for (int i = 0; i < SBL; ++i) {
            const int b = lane + 32 * i;
#pragma unroll
            for (int v = 0; v < 4; ++v) {
                const int4 w4 = b < nsb ? reinterpret_cast<const int4*>(xq + b * 16)[v] : make_int4(0, 0, 0, 0);
                xr[i][4 * v] = w4.x;
                xr[i][4 * v + 1] = w4.y;
                xr[i][4 * v + 2] = w4.z;
                xr[i][4 * v + 3] = w4.w;
            }
            xsr[i] = b < nsb ? xs[b] : 0.0f;
        }
    }

    const int row_bytes = (D >> 8) * QMOE_SB_BYTES;
    const int n_routed = plan.n;
    const int has_sh = (a.sh_gate_up != nullptr && a.sh_I_loc > 0) ? 1 : 0;
    const int T = n_routed * a.I_loc + has_sh * a.sh_I_loc;
    const int gw = blockIdx.x * kWarps + warp, nw = gridDim.x * kWarps;

    for (int t = gw; t < T; t += nw) {
        const uint8_t* base;
        int r, u, rows;
        if (t < n_routed * a.I_loc) {
            u = t / a.I_loc;
            r = t - u * a.I_loc;
            base = a.gate_up + (size_t)plan.expert[u] * a.gu_expert_bytes;
            rows = a.I_loc;
        } else {
            u = n_routed;
            r = t - n_routed * a.I_loc;
            base = a.sh_gate_up;
            rows = a.sh_I_loc;
        }
        const uint8_t* grow = base + (size_t)r * row_bytes;
        const uint8_t* urow = base + (size_t)(rows + r) * row_bytes;

        // Issue every load of this row pair before any decode.
        uint2 hg[SBL], hu[SBL], qg[SBL][2], qu[SBL][2];
#pragma unroll
        for (int i = 0; i < SBL; ++i) {
            const int b = lane + 32 * i;
            if (b < nsb) {
                const int off = (b >> 3) * QMOE_SB_BYTES, q = off + 8 + 16 * (b & 7);
                hg[i] = ldg2(grow + off);
                hu[i] = ldg2(urow + off);
                qg[i][0] = ldg2(grow + q);
                qg[i][1] = ldg2(grow + q + 8);
                qu[i][0] = ldg2(urow + q);
                qu[i][1] = ldg2(urow + q + 8);
            }
        }

        const uint32_t tmask = (u < n_routed) ? plan.mask[u] : ((M >= 32) ? 0xffffffffu : ((1u << M) - 1u));
        const int slot_sh = a.k;
        float dg[SBL], du[SBL];
#pragma unroll
        for (int i = 0; i < SBL; ++i) {
            const int ib = (lane + 32 * i) & 7;
            if (lane + 32 * i >= nsb) {
                dg[i] = du[i] = 0.0f;
                continue;
            }
            dg[i] = qmoe_half_bits_to_float((uint16_t)(hg[i].x & 0xFFFFu)) *
                    (float)(qmoe_iq4xs_ls(hg[i].x, hg[i].y, ib) - 32);
            du[i] = qmoe_half_bits_to_float((uint16_t)(hu[i].x & 0xFFFFu)) *
                    (float)(qmoe_iq4xs_ls(hu[i].x, hu[i].y, ib) - 32);
        }
        if (MAXM == 1) {
            float accg = 0.0f, accu = 0.0f;
#pragma unroll
            for (int i = 0; i < SBL; ++i) {
                if (lane + 32 * i >= nsb) continue;
                const int sg = qmoe_subblock_dot(qg[i][0].x, qg[i][0].y, qg[i][1].x, qg[i][1].y, xr[i], 0);
                const int su = qmoe_subblock_dot(qu[i][0].x, qu[i][0].y, qu[i][1].x, qu[i][1].y, xr[i], 0);
                accg = fmaf(dg[i] * xsr[i], (float)sg, accg);
                accu = fmaf(du[i] * xsr[i], (float)su, accu);
            }
            const float g = warp_sum(accg);
            const float uu = warp_sum(accu);
            if (lane == 0 && (tmask & 1u)) {
                const int slot = (u < n_routed) ? plan.slot[u][0] : slot_sh;
                a.h[(size_t)slot * a.h_stride + r] = silu(g) * uu;
            }
            continue;
        }
        // Several tokens: the codes go through the codebook once, then each
        // token that uses the unit (warp-uniform, usually one) takes one pass.
        uint32_t glo[SBL][4], ghi[SBL][4], ulo[SBL][4], uhi[SBL][4];
#pragma unroll
        for (int i = 0; i < SBL; ++i) {
            qmoe_lut8(qg[i][0].x, glo[i][0], ghi[i][0]);
            qmoe_lut8(qg[i][0].y, glo[i][1], ghi[i][1]);
            qmoe_lut8(qg[i][1].x, glo[i][2], ghi[i][2]);
            qmoe_lut8(qg[i][1].y, glo[i][3], ghi[i][3]);
            qmoe_lut8(qu[i][0].x, ulo[i][0], uhi[i][0]);
            qmoe_lut8(qu[i][0].y, ulo[i][1], uhi[i][1]);
            qmoe_lut8(qu[i][1].x, ulo[i][2], uhi[i][2]);
            qmoe_lut8(qu[i][1].y, ulo[i][3], uhi[i][3]);
        }
        for (uint32_t mm = tmask; mm; mm &= mm - 1u) {
            const int m = __ffs(mm) - 1;
            float accg = 0.0f, accu = 0.0f;
#pragma unroll
            for (int i = 0; i < SBL; ++i) {
                const int b = lane + 32 * i;
                if (b >= nsb) continue;
                int xp[16];
                const int4* src = reinterpret_cast<const int4*>(xq + ((size_t)m * nsb + b) * 16);
#pragma unroll
                for (int v = 0; v < 4; ++v) {
                    const int4 w4 = src[v];
                    xp[4 * v] = w4.x;
                    xp[4 * v + 1] = w4.y;
                    xp[4 * v + 2] = w4.z;
                    xp[4 * v + 3] = w4.w;
                }
                const float st = xs[m * nsb + b];
                const int sg = subblock_dot_lut(glo[i], ghi[i], xp);
                const int su = subblock_dot_lut(ulo[i], uhi[i], xp);
                accg = fmaf(dg[i] * st, (float)sg, accg);
                accu = fmaf(du[i] * st, (float)su, accu);
            }
            const float g = warp_sum(accg);
            const float uu = warp_sum(accu);
            if (lane == 0) {
                const int slot = (u < n_routed) ? plan.slot[u][m] : slot_sh;
                a.h[((size_t)m * (a.k + 1) + slot) * a.h_stride + r] = silu(g) * uu;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// The h rows of every (token, slot) to block floating point once, for the
// down kernel's CTAs to copy (M > 1; with M = 1 each CTA converts its own).
// A warp per 32-value block reads all of it before writing, so hconv may be
// h itself.
__global__ void __launch_bounds__(kWarps * 32) convert_h_kernel(ExpertArgs a) {
    const int lane = threadIdx.x & 31;
    const int K1 = a.k + 1;
    const int I_max = a.I_loc > a.sh_I_loc ? a.I_loc : a.sh_I_loc;
    const int nsbh = I_max >> 5;
    const int i = blockIdx.x * kWarps + (threadIdx.x >> 5);
    if (i >= a.M * K1 * nsbh) return;
    const int b = i % nsbh, ms = i / nsbh, m = ms / K1, s = ms % K1;
    int nv;
    if (s < a.k) {
        const int id = a.ids[m * a.k + s];
        nv = (id >= a.e_lo && id < a.e_hi) ? (a.I_loc >> 5) : 0;
    } else {
        nv = (a.sh_down != nullptr && a.sh_I_loc > 0) ? (a.sh_I_loc >> 5) : 0;
    }
    const float v = b < nv ? a.h[(size_t)ms * a.h_stride + b * 32 + lane] : 0.0f;
    float st;
    const int pw = warp_block_fp(v, &st);
    __syncwarp();
    float* dst = a.hconv + (size_t)ms * a.hconv_stride + b * 32;
    if (lane < 16) dst[lane] = __int_as_float(pw);
    if (lane == 16) dst[16] = st;
}

// ---------------------------------------------------------------------------
// down + weighted combine + gated shared expert.
// The down kernels' common start: the expert plan, the per-(token, slot)
// combine weights and valid h block counts, and every h block in block
// floating point in shared memory (hq pair words, hs steps).
struct DownShared {
    Plan plan;
    float w[kMaxTokens][kMaxTopK + 1];
    int nvalid[kMaxTokens][kMaxTopK + 1];
};

__device__ __forceinline__ void down_prologue(const ExpertArgs& a, DownShared& sh, int* hq, float* hs, int* owner,
                                              bool stage_h = true) {
    const int tid = threadIdx.x;
    const int M = a.M, K1 = a.k + 1;
    const int I_max = a.I_loc > a.sh_I_loc ? a.I_loc : a.sh_I_loc;
    const int nsbh = I_max >> 5;
    build_plan(a, sh.plan, owner);
    const int has_sh = (a.sh_down != nullptr && a.sh_I_loc > 0) ? 1 : 0;
    for (int i = tid; i < M * K1; i += blockDim.x) {
        const int m = i / K1, s = i % K1;
        float w;
        if (s < a.k) w = a.weights[m * a.k + s];
        else w = (has_sh && a.shared_logit) ? sigmoid(a.shared_logit[m]) : (has_sh ? 1.0f : 0.0f);
        sh.w[m][s] = w;
    }
    // Which (token, slot) h rows are in use, then convert them to block
    // floating point.
    for (int i = tid; i < M * K1; i += blockDim.x) {
        const int m = i / K1, s = i % K1;
        int nv = 0;
        if (s < a.k) {
            const int id = a.ids[m * a.k + s];
            nv = (id >= a.e_lo && id < a.e_hi) ? (a.I_loc >> 5) : 0;
        } else {
            nv = has_sh ? (a.sh_I_loc >> 5) : 0;
        }
        sh.nvalid[m][s] = nv;
    }
    __syncthreads();
    if (!stage_h) return;
    if (a.hconv) {
        // converted once by convert_h_kernel: 16 pair words and the step per
        // block; blocks past a slot's valid count were written as zeros.  A
        // thread per block, four blocks' loads in flight before any store.
        constexpr int U = 4;
        const int nblk = M * K1 * nsbh;
        for (int i0 = tid; i0 < nblk; i0 += blockDim.x * U) {
            float4 q[U][4];
            float st[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int i = i0 + u * blockDim.x;
                if (i < nblk) {
                    const int b = i % nsbh, ms = i / nsbh;
                    const float* src = a.hconv + (size_t)ms * a.hconv_stride + b * 32;
#pragma unroll
                    for (int v = 0; v < 4; ++v) q[u][v] = __ldcg(reinterpret_cast<const float4*>(src) + v);
                    st[u] = __ldcg(src + 16);
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int i = i0 + u * blockDim.x;
                if (i < nblk) {
                    float4* d = reinterpret_cast<float4*>(hq + (size_t)i * 16);
#pragma unroll
                    for (int v = 0; v < 4; ++v) d[v] = q[u][v];
                    hs[i] = st[u];
                }
            }
        }
    } else {
        convert_blocks<8>(
            M * K1 * nsbh,
            [&](int i, int ln) {
                const int b = i % nsbh, ms = i / nsbh;
                return b < sh.nvalid[ms / K1][ms % K1] ? a.h[(size_t)ms * a.h_stride + b * 32 + ln] : 0.0f;
            },
            [&](int i, int ln, int pw, float st) {
                if (ln < 16) hq[(size_t)i * 16 + ln] = pw;
                if (ln == 0) hs[i] = st;
            });
    }
    __syncthreads();
}

template <int MAXM>
__global__ void __launch_bounds__(kWarps * 32) down_kernel(ExpertArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ DownShared sh;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int M = a.M, K1 = a.k + 1;
    const int I_max = a.I_loc > a.sh_I_loc ? a.I_loc : a.sh_I_loc;
    const int nsbh = I_max >> 5;                                     // h blocks per slot
    int* hq = reinterpret_cast<int*>(smem);                          // [M][k+1][nsbh][16]
    float* hs = reinterpret_cast<float*>(hq + (size_t)M * K1 * nsbh * 16);  // [M][k+1][nsbh]
    int* owner = reinterpret_cast<int*>(hs + (size_t)M * K1 * nsbh);
    down_prologue(a, sh, hq, hs, owner);
    const Plan& plan = sh.plan;
    const int has_sh = (a.sh_down != nullptr && a.sh_I_loc > 0) ? 1 : 0;

    const int nsb_r = a.dn_nseg * a.dn_nsub;
    const int nsb_s = a.sh_nseg * a.sh_nsub;
    const int rb_r = a.dn_nseg * (8 + 16 * a.dn_nsub);
    const int rb_s = a.sh_nseg * (8 + 16 * a.sh_nsub);
    const int n_routed = plan.n;
    const int P = n_routed * nsb_r + has_sh * nsb_s;
    const uint32_t all = (M >= 32) ? 0xffffffffu : ((1u << M) - 1u);
    const int gw = blockIdx.x * kWarps + warp, nw = gridDim.x * kWarps;

    for (int j = gw; j < a.D; j += nw) {
        float acc[MAXM];
#pragma unroll
        for (int m = 0; m < MAXM; ++m) acc[m] = 0.0f;
        // Batches of kPB (expert, sub-block) pairs per lane: every load of a
        // batch is issued before any decode.
        constexpr int kPB = 6;
        for (int p0 = lane; p0 < P; p0 += 32 * kPB) {
            uint2 hdr[kPB], q0[kPB], q1[kPB];
            int ib[kPB];
#pragma unroll
            for (int i = 0; i < kPB; ++i) {
                const int p = p0 + 32 * i;
                if (p < P) {
                    int u, t, nsub, ib0;
                    const uint8_t* row;
                    if (p < n_routed * nsb_r) {
                        u = p / nsb_r;
                        t = p - u * nsb_r;
                        row = a.down + (size_t)plan.expert[u] * a.dn_expert_bytes + (size_t)j * rb_r;
                        nsub = a.dn_nsub;
                        ib0 = a.dn_ib0;
                    } else {
                        t = p - n_routed * nsb_r;
                        row = a.sh_down + (size_t)j * rb_s;
                        nsub = a.sh_nsub;
                        ib0 = a.sh_ib0;
                    }
                    const int seg = t / nsub, ibl = t - seg * nsub;
                    const uint8_t* sp = row + seg * (8 + 16 * nsub);
                    hdr[i] = ldg2(sp);
                    q0[i] = ldg2(sp + 8 + 16 * ibl);
                    q1[i] = ldg2(sp + 16 + 16 * ibl);
                    ib[i] = ib0 + ibl;
                }
            }
#pragma unroll
            for (int i = 0; i < kPB; ++i) {
                const int p = p0 + 32 * i;
                if (p >= P) break;
                int u, t;
                if (p < n_routed * nsb_r) {
                    u = p / nsb_r;
                    t = p - u * nsb_r;
                } else {
                    u = n_routed;
                    t = p - n_routed * nsb_r;
                }
                const float dl = qmoe_half_bits_to_float((uint16_t)(hdr[i].x & 0xFFFFu)) *
                                 (float)(qmoe_iq4xs_ls(hdr[i].x, hdr[i].y, ib[i]) - 32);
                const uint32_t tmask = (u < n_routed) ? plan.mask[u] : all;
#pragma unroll
                for (int m = 0; m < MAXM; ++m) {
                    if (m < M && ((tmask >> m) & 1u)) {
                        const int s = (u < n_routed) ? plan.slot[u][m] : a.k;
                        const size_t hb = ((size_t)m * K1 + s) * nsbh + t;
                        int xp[16];
                        const int4* src = reinterpret_cast<const int4*>(hq + hb * 16);
#pragma unroll
                        for (int v = 0; v < 4; ++v) {
                            const int4 w4 = src[v];
                            xp[4 * v] = w4.x;
                            xp[4 * v + 1] = w4.y;
                            xp[4 * v + 2] = w4.z;
                            xp[4 * v + 3] = w4.w;
                        }
                        const int S = qmoe_subblock_dot(q0[i].x, q0[i].y, q1[i].x, q1[i].y, xp, 0);
                        acc[m] = fmaf(sh.w[m][s] * dl * hs[hb], (float)S, acc[m]);
                    }
                }
            }
        }
#pragma unroll
        for (int m = 0; m < MAXM; ++m) {
            if (m < M) {
                const float v = warp_sum(acc[m]);
                if (lane == 0) a.out[(size_t)m * a.D + j] = v;
            }
        }
    }
}

// down + combine for several tokens with R = 32 / NSB output rows per warp
// (NSB = the sub-blocks of a down row, routed and shared alike): lane
// (rr, t) takes sub-block t of row j0 + rr of every unit (a routed expert or
// the shared one), so the tokens that use a unit are the same for the whole
// warp and the token loop does not diverge; each sub-block is looked up in
// the codebook once for all its tokens.  US warps split a row group's units
// and add their sums in a fixed order.  Grid: exactly D / (R * kWarps / US)
// CTAs.
template <int MAXM, int NSB, int US>
__global__ void __launch_bounds__(kWarps * 32, 3) down_rows_kernel(ExpertArgs a) {
    constexpr int R = 32 / NSB, G = kWarps / US;
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ DownShared sh;
    __shared__ float part[kWarps][R][MAXM];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int M = a.M, K1 = a.k + 1;
    const int I_max = a.I_loc > a.sh_I_loc ? a.I_loc : a.sh_I_loc;
    const int nsbh = I_max >> 5;
    int* hq = reinterpret_cast<int*>(smem);                          // [M][k+1][nsbh][16]
    float* hs = reinterpret_cast<float*>(hq + (size_t)M * K1 * nsbh * 16);  // [M][k+1][nsbh]
    int* owner = reinterpret_cast<int*>(hs + (size_t)M * K1 * nsbh);
    down_prologue(a, sh, hq, hs, owner);
    const Plan& plan = sh.plan;
    const int has_sh = (a.sh_down != nullptr && a.sh_I_loc > 0) ? 1 : 0;

    const int rr = lane / NSB, t = lane % NSB;
    const int g = warp % G, sp = warp / G;
    const int n_units = plan.n + has_sh;
    const int u_lo = sp * n_units / US, u_hi = (sp + 1) * n_units / US;
    const int rb_r = a.dn_nseg * (8 + 16 * a.dn_nsub);
    const int rb_s = a.sh_nseg * (8 + 16 * a.sh_nsub);
    const int seg_r = t / a.dn_nsub, ibl_r = t - seg_r * a.dn_nsub;
    const int seg_s = t / a.sh_nsub, ibl_s = t - seg_s * a.sh_nsub;
    const int off_r = seg_r * (8 + 16 * a.dn_nsub), off_s = seg_s * (8 + 16 * a.sh_nsub);
    const uint32_t all = (M >= 32) ? 0xffffffffu : ((1u << M) - 1u);
    const int j = (blockIdx.x * G + g) * R + rr;

    float acc[MAXM];
#pragma unroll
    for (int m = 0; m < MAXM; ++m) acc[m] = 0.0f;
    constexpr int kUB = 6;
    for (int u0 = u_lo; u0 < u_hi; u0 += kUB) {
        uint2 hdr[kUB], q0[kUB], q1[kUB];
#pragma unroll
        for (int i = 0; i < kUB; ++i) {
            const int u = u0 + i;
            if (u < u_hi) {
                const uint8_t* sp_;
                int ibl;
                if (u < plan.n) {
                    sp_ = a.down + (size_t)plan.expert[u] * a.dn_expert_bytes + (size_t)j * rb_r + off_r;
                    ibl = ibl_r;
                } else {
                    sp_ = a.sh_down + (size_t)j * rb_s + off_s;
                    ibl = ibl_s;
                }
                hdr[i] = ldg2(sp_);
                q0[i] = ldg2(sp_ + 8 + 16 * ibl);
                q1[i] = ldg2(sp_ + 16 + 16 * ibl);
            }
        }
#pragma unroll
        for (int i = 0; i < kUB; ++i) {
            const int u = u0 + i;
            if (u >= u_hi) break;
            const bool routed = u < plan.n;
            const int ib = routed ? a.dn_ib0 + ibl_r : a.sh_ib0 + ibl_s;
            const float dl = qmoe_half_bits_to_float((uint16_t)(hdr[i].x & 0xFFFFu)) *
                             (float)(qmoe_iq4xs_ls(hdr[i].x, hdr[i].y, ib) - 32);
            uint32_t lo[4], hi[4];
            qmoe_lut8(q0[i].x, lo[0], hi[0]);
            qmoe_lut8(q0[i].y, lo[1], hi[1]);
            qmoe_lut8(q1[i].x, lo[2], hi[2]);
            qmoe_lut8(q1[i].y, lo[3], hi[3]);
            // the unit's tokens (warp-uniform), one pass each; the sum goes to
            // its accumulator by a predicated select, so acc stays in registers
            for (uint32_t mm = routed ? plan.mask[u] : all; mm; mm &= mm - 1u) {
                const int m = __ffs(mm) - 1;
                const int s = routed ? plan.slot[u][m] : a.k;
                const size_t hb = ((size_t)m * K1 + s) * nsbh + t;
                int xp[16];
                const int4* src = reinterpret_cast<const int4*>(hq + hb * 16);
#pragma unroll
                for (int v = 0; v < 4; ++v) {
                    const int4 w4 = src[v];
                    xp[4 * v] = w4.x;
                    xp[4 * v + 1] = w4.y;
                    xp[4 * v + 2] = w4.z;
                    xp[4 * v + 3] = w4.w;
                }
                const float f = sh.w[m][s] * dl * hs[hb];
                const float S = (float)subblock_dot_lut(lo, hi, xp);
#pragma unroll
                for (int q = 0; q < MAXM; ++q)
                    if (q == m) acc[q] = fmaf(f, S, acc[q]);
            }
        }
    }
#pragma unroll
    for (int m = 0; m < MAXM; ++m) {
#pragma unroll
        for (int o = NSB / 2; o > 0; o >>= 1) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], o);
    }
    if (US == 1) {
        if (t == 0) {
#pragma unroll
            for (int m = 0; m < MAXM; ++m)
                if (m < M) a.out[(size_t)m * a.D + j] = acc[m];
        }
        return;
    }
    if (t == 0) {
#pragma unroll
        for (int m = 0; m < MAXM; ++m) part[warp][rr][m] = acc[m];
    }
    __syncthreads();
    if (sp == 0 && t == 0) {
#pragma unroll
        for (int m = 0; m < MAXM; ++m) {
            if (m < M) {
                float v = part[g][rr][m];
#pragma unroll
                for (int q = 1; q < US; ++q) v += part[q * G + g][rr][m];
                a.out[(size_t)m * a.D + j] = v;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// The checkpoint's other expert formats (IQ3_S, IQ4_NL, Q8_0; IQ4_XS too) on
// the same integer core: each 32-value sub-block becomes eight int8x4 words
// in the core's pair order (values j and j + 16 side by side, as the block
// floating-point activation pairs them) and one fp32 scale, then dp2a against
// the activation.  IQ4_NL codes are laid out as one IQ4_XS sub-block (the
// same codebook); Q8_0 bytes are the values; IQ3_S grid bytes (odd, 1..15)
// take their signs as (g ^ m) + (m & 1) per byte, never carrying.

#define QMOE_IQ3S_GRID_DEF __device__ uint32_t g_iq3s_grid_core[512]
#include "iq3s_grid.inc"
#undef QMOE_IQ3S_GRID_DEF

struct FmtSel {
    int gu, dn, sgu, sdn;          // GGML types
    int gu_rb, dn_rb, sgu_rb, sdn_rb;  // bytes per row
};

__device__ __forceinline__ uint32_t ld_u16(const uint8_t* p) { return *reinterpret_cast<const unsigned short*>(p); }
// four bytes at a 2-byte aligned address
__device__ __forceinline__ uint32_t ld_w16(const uint8_t* p) { return ld_u16(p) | (ld_u16(p + 2) << 16); }

// Natural-order words N[n] (values 4n .. 4n+3) -> the core's (lo, hi) words.
__device__ __forceinline__ void pair_order(const uint32_t (&N)[8], uint32_t (&lo)[4], uint32_t (&hi)[4]) {
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        lo[w] = qmoe_prmt(N[w], N[w + 4], 0x5140u);  // values 4w, 4w+16, 4w+1, 4w+17
        hi[w] = qmoe_prmt(N[w], N[w + 4], 0x7362u);  // 4w+2, 4w+18, 4w+3, 4w+19
    }
}

// Four unsigned grid bytes with sign bits s4 (bit k: byte k negative).
__device__ __forceinline__ uint32_t signed_bytes(uint32_t g, uint32_t s4) {
    const uint32_t m01 = (s4 * 0x00204081u) & 0x01010101u;
    return (g ^ (m01 * 0xFFu)) + m01;
}

// Sub-block sb of a row in `fmt` as core words and its scale (gguf/quants.py
// IQ4_XS 112-129, IQ4_NL 101-109, Q8_0 33-37, IQ3_S 132-165).
__device__ __forceinline__ float fmt_words(int fmt, const uint8_t* row, int sb, const uint32_t* grid,
                                           uint32_t (&lo)[4], uint32_t (&hi)[4]) {
    if (fmt == QMOE_FMT_IQ4_XS) {
        const uint8_t* blk = row + (sb >> 3) * QMOE_SB_BYTES;
        const int ib = sb & 7;
        const uint2 h = ldg2(blk), q0 = ldg2(blk + 8 + 16 * ib), q1 = ldg2(blk + 16 + 16 * ib);
        qmoe_lut8(q0.x, lo[0], hi[0]);
        qmoe_lut8(q0.y, lo[1], hi[1]);
        qmoe_lut8(q1.x, lo[2], hi[2]);
        qmoe_lut8(q1.y, lo[3], hi[3]);
        return qmoe_half_bits_to_float((uint16_t)(h.x & 0xFFFFu)) * (float)(qmoe_iq4xs_ls(h.x, h.y, ib) - 32);
    }
    if (fmt == QMOE_FMT_IQ4_NL) {
        const uint8_t* blk = row + sb * 18;
#pragma unroll
        for (int w = 0; w < 4; ++w) qmoe_lut8(ld_w16(blk + 2 + 4 * w), lo[w], hi[w]);
        return qmoe_half_bits_to_float((uint16_t)ld_u16(blk));
    }
    uint32_t N[8];
    if (fmt == QMOE_FMT_Q8_0) {
        const uint8_t* blk = row + sb * 34;
#pragma unroll
        for (int n = 0; n < 8; ++n) N[n] = ld_w16(blk + 2 + 4 * n);
        pair_order(N, lo, hi);
        return qmoe_half_bits_to_float((uint16_t)ld_u16(blk));
    }
    // IQ3_S
    const uint8_t* blk = row + (sb >> 3) * 110;
    const int ib32 = sb & 7;
    const uint32_t qs01 = ld_w16(blk + 2 + 8 * ib32), qs23 = ld_w16(blk + 6 + 8 * ib32);
    const uint32_t h = blk[66 + ib32];
    const uint32_t sg = ld_w16(blk + 74 + 4 * ib32);
    const int sc = (blk[106 + ib32 / 2] >> (4 * (ib32 % 2))) & 0xF;
#pragma unroll
    for (int l = 0; l < 4; ++l) {
        const uint32_t qw = l < 2 ? qs01 : qs23;
        const int sh = (l & 1) * 16;
        const uint32_t i1 = ((qw >> sh) & 0xFFu) | ((h << (8 - 2 * l)) & 256u);
        const uint32_t i2 = ((qw >> (sh + 8)) & 0xFFu) | ((h << (7 - 2 * l)) & 256u);
        const uint32_t s8 = (sg >> (8 * l)) & 0xFFu;
        N[2 * l] = signed_bytes(grid[i1], s8 & 0xFu);
        N[2 * l + 1] = signed_bytes(grid[i2], s8 >> 4);
    }
    pair_order(N, lo, hi);
    return qmoe_half_bits_to_float((uint16_t)ld_u16(blk)) * (1.0f + 2.0f * (float)sc);
}

// gate|up + SwiGLU on formatted weights: gateup_kernel's plan and task
// layout (warp per row pair of a distinct expert; x converted by the route
// launch), each row pair's sub-blocks decoded once for all its tokens.
template <int MAXM, int SBL>
__global__ void __launch_bounds__(kWarps * 32) fmt_gateup_kernel(ExpertArgs a, FmtSel f) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ Plan plan;
    __shared__ uint32_t s_grid[512];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int D = a.D, M = a.M;
    const int nsb = D >> 5;
    int* xq = reinterpret_cast<int*>(smem);
    float* xs = reinterpret_cast<float*>(xq + (size_t)M * nsb * 16);
    int* owner = reinterpret_cast<int*>(xs + (size_t)M * nsb);
    for (int i = tid; i < 512; i += blockDim.x) s_grid[i] = g_iq3s_grid_core[i];
    build_plan(a, plan, owner);
    {
        const int n16 = M * nsb * 68 / 16;
        const uint4* src = reinterpret_cast<const uint4*>(a.xconv);
        uint4* dst = reinterpret_cast<uint4*>(smem);
        constexpr int U = 8;
        for (int i0 = tid; i0 < n16; i0 += blockDim.x * U) {
            uint4 v[U];
#pragma unroll
            for (int u = 0; u < U; ++u)
                if (i0 + u * (int)blockDim.x < n16) v[u] = __ldcg(src + i0 + u * blockDim.x);
#pragma unroll
            for (int u = 0; u < U; ++u)
                if (i0 + u * (int)blockDim.x < n16) dst[i0 + u * blockDim.x] = v[u];
        }
    }
    __syncthreads();

    const int n_routed = plan.n;
    const int has_sh = (a.sh_gate_up != nullptr && a.sh_I_loc > 0) ? 1 : 0;
    const int T = n_routed * a.I_loc + has_sh * a.sh_I_loc;
    const int gw = blockIdx.x * kWarps + warp, nw = gridDim.x * kWarps;
    for (int t = gw; t < T; t += nw) {
        const uint8_t *grow, *urow;
        int u, r, fmt;
        if (t < n_routed * a.I_loc) {
            u = t / a.I_loc;
            r = t - u * a.I_loc;
            grow = a.gate_up + (size_t)plan.expert[u] * a.gu_expert_bytes + (size_t)r * f.gu_rb;
            urow = grow + (size_t)a.I_loc * f.gu_rb;
            fmt = f.gu;
        } else {
            u = n_routed;
            r = t - n_routed * a.I_loc;
            grow = a.sh_gate_up + (size_t)r * f.sgu_rb;
            urow = grow + (size_t)a.sh_I_loc * f.sgu_rb;
            fmt = f.sgu;
        }
        uint32_t glo[SBL][4], ghi[SBL][4], ulo[SBL][4], uhi[SBL][4];
        float dg[SBL], du[SBL];
#pragma unroll
        for (int i = 0; i < SBL; ++i) {
            const int b = lane + 32 * i;
            if (b < nsb) {
                dg[i] = fmt_words(fmt, grow, b, s_grid, glo[i], ghi[i]);
                du[i] = fmt_words(fmt, urow, b, s_grid, ulo[i], uhi[i]);
            } else {
                dg[i] = du[i] = 0.0f;
            }
        }
        const uint32_t tmask = (u < n_routed) ? plan.mask[u] : ((M >= 32) ? 0xffffffffu : ((1u << M) - 1u));
        for (uint32_t mm = tmask; mm; mm &= mm - 1u) {
            const int m = __ffs(mm) - 1;
            float accg = 0.0f, accu = 0.0f;
#pragma unroll
            for (int i = 0; i < SBL; ++i) {
                const int b = lane + 32 * i;
                if (b >= nsb) continue;
                int xp[16];
                const int4* src = reinterpret_cast<const int4*>(xq + ((size_t)m * nsb + b) * 16);
#pragma unroll
                for (int v = 0; v < 4; ++v) {
                    const int4 w4 = src[v];
                    xp[4 * v] = w4.x;
                    xp[4 * v + 1] = w4.y;
                    xp[4 * v + 2] = w4.z;
                    xp[4 * v + 3] = w4.w;
                }
                const float st = xs[m * nsb + b];
                accg = fmaf(dg[i] * st, (float)subblock_dot_lut(glo[i], ghi[i], xp), accg);
                accu = fmaf(du[i] * st, (float)subblock_dot_lut(ulo[i], uhi[i], xp), accu);
            }
            const float g = warp_sum(accg);
            const float uu = warp_sum(accu);
            if (lane == 0) {
                const int slot = (u < n_routed) ? plan.slot[u][m] : a.k;
                a.h[((size_t)m * (a.k + 1) + slot) * a.h_stride + r] = silu(g) * uu;
            }
        }
    }
}

// down + combine on formatted weights: down_kernel's layout (warp per output
// row, lanes over (unit, sub-block) pairs, h in block floating point), each
// pair decoded once for all the unit's tokens.
template <int MAXM>
__global__ void __launch_bounds__(kWarps * 32) fmt_down_kernel(ExpertArgs a, FmtSel f) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ DownShared sh;
    __shared__ uint32_t s_grid[512];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int M = a.M, K1 = a.k + 1;
    const int I_max = a.I_loc > a.sh_I_loc ? a.I_loc : a.sh_I_loc;
    const int nsbh = I_max >> 5;
    int* hq = reinterpret_cast<int*>(smem);
    float* hs = reinterpret_cast<float*>(hq + (size_t)M * K1 * nsbh * 16);
    int* owner = reinterpret_cast<int*>(hs + (size_t)M * K1 * nsbh);
    for (int i = tid; i < 512; i += blockDim.x) s_grid[i] = g_iq3s_grid_core[i];
    down_prologue(a, sh, hq, hs, owner);
    const Plan& plan = sh.plan;
    const int has_sh = (a.sh_down != nullptr && a.sh_I_loc > 0) ? 1 : 0;
    const int nsb_r = a.I_loc >> 5, nsb_s = a.sh_I_loc >> 5;
    const int n_routed = plan.n;
    const int P = n_routed * nsb_r + has_sh * nsb_s;
    const uint32_t all = (M >= 32) ? 0xffffffffu : ((1u << M) - 1u);
    const int gw = blockIdx.x * kWarps + warp, nw = gridDim.x * kWarps;
    for (int j = gw; j < a.D; j += nw) {
        float acc[MAXM];
#pragma unroll
        for (int m = 0; m < MAXM; ++m) acc[m] = 0.0f;
        for (int p = lane; p < P; p += 32) {
            int u, t, fmt;
            const uint8_t* row;
            if (p < n_routed * nsb_r) {
                u = p / nsb_r;
                t = p - u * nsb_r;
                row = a.down + (size_t)plan.expert[u] * a.dn_expert_bytes + (size_t)j * f.dn_rb;
                fmt = f.dn;
            } else {
                u = n_routed;
                t = p - n_routed * nsb_r;
                row = a.sh_down + (size_t)j * f.sdn_rb;
                fmt = f.sdn;
            }
            uint32_t lo[4], hi[4];
            const float dl = fmt_words(fmt, row, t, s_grid, lo, hi);
            for (uint32_t mm = u < n_routed ? plan.mask[u] : all; mm; mm &= mm - 1u) {
                const int m = __ffs(mm) - 1;
                const int s = (u < n_routed) ? plan.slot[u][m] : a.k;
                const size_t hb = ((size_t)m * K1 + s) * nsbh + t;
                int xp[16];
                const int4* src = reinterpret_cast<const int4*>(hq + hb * 16);
#pragma unroll
                for (int v = 0; v < 4; ++v) {
                    const int4 w4 = src[v];
                    xp[4 * v] = w4.x;
                    xp[4 * v + 1] = w4.y;
                    xp[4 * v + 2] = w4.z;
                    xp[4 * v + 3] = w4.w;
                }
                const float fs = sh.w[m][s] * dl * hs[hb];
                const float S = (float)subblock_dot_lut(lo, hi, xp);
#pragma unroll
                for (int q = 0; q < MAXM; ++q)
                    if (q == m) acc[q] = fmaf(fs, S, acc[q]);
            }
        }
#pragma unroll
        for (int m = 0; m < MAXM; ++m) {
            if (m < M) {
                const float v = warp_sum(acc[m]);
                if (lane == 0) a.out[(size_t)m * a.D + j] = v;
            }
        }
    }
}

template <typename K>
cudaError_t launch_with_smem(K kernel, unsigned grid, size_t smem, const ExpertArgs& a,
                             cudaStream_t s) {
    cudaError_t err = smem_opt_in(reinterpret_cast<const void*>(kernel), (int)smem);
    if (err != cudaSuccess) return err;
    kernel<<<grid, kWarps * 32, smem, s>>>(a);
    return cudaGetLastError();
}

template <int MAXM>
int gateup_resident(int sbl, size_t smem) {
    int n = 0;
    const void* k = sbl == 1   ? reinterpret_cast<const void*>(gateup_kernel<MAXM, 1>)
                    : sbl == 2 ? reinterpret_cast<const void*>(gateup_kernel<MAXM, 2>)
                    : sbl == 3 ? reinterpret_cast<const void*>(gateup_kernel<MAXM, 3>)
                               : reinterpret_cast<const void*>(gateup_kernel<MAXM, 4>);
    if (smem_opt_in(k, (int)smem) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, kWarps * 32, smem) != cudaSuccess || n < 1)
        n = 1;
    return n;
}

template <int MAXM>
cudaError_t launch_gateup_m(const ExpertArgs& a, cudaStream_t s) {
    const int nsb = a.D >> 5;
    const size_t smem = (size_t)a.M * nsb * (16 * 4 + 4) + (size_t)(a.e_hi - a.e_lo) * 4;
    const int n_units = a.M * a.k + 1;
    const long tasks = (long)n_units * (a.I_loc > a.sh_I_loc ? a.I_loc : a.sh_I_loc);
    unsigned grid = (unsigned)((tasks + kWarps - 1) / kWarps);
    const int sbl = (nsb + 31) / 32;
    // Every CTA copies the converted x and plans the experts first, so one
    // wave of resident CTAs takes the row pairs in strides (a second, partial
    // wave would repeat that work for a few row pairs).
    grid = min(grid, (unsigned)(device_sm_count() * gateup_resident<MAXM>(sbl, smem)));
    switch (sbl) {
        case 1: return launch_with_smem(gateup_kernel<MAXM, 1>, grid, smem, a, s);
        case 2: return launch_with_smem(gateup_kernel<MAXM, 2>, grid, smem, a, s);
        case 3: return launch_with_smem(gateup_kernel<MAXM, 3>, grid, smem, a, s);
        default: return launch_with_smem(gateup_kernel<MAXM, 4>, grid, smem, a, s);
    }
}

template <int MAXM>
cudaError_t launch_down_m(const ExpertArgs& a, cudaStream_t s) {
    const int I_max = a.I_loc > a.sh_I_loc ? a.I_loc : a.sh_I_loc;
    const size_t smem = (size_t)a.M * (a.k + 1) * (I_max >> 5) * (16 * 4 + 4) +
                        (size_t)(a.e_hi - a.e_lo) * 4;
    const unsigned grid = (unsigned)((a.D + kWarps - 1) / kWarps);
    if (a.hconv) {
        // h to block floating point once (not once per CTA), then the CTAs copy it
        const int nb = a.M * (a.k + 1) * (I_max >> 5);
        convert_h_kernel<<<(unsigned)((nb + kWarps - 1) / kWarps), kWarps * 32, 0, s>>>(a);
        cudaError_t err = cudaGetLastError();
        if (err != cudaSuccess) return err;
        // Rows-per-warp layout when the routed and shared down rows have 8 or
        // 16 sub-blocks (and D fills the exact grid); else a row per warp.
        const int nsb_r = a.dn_nseg * a.dn_nsub;
        const bool sh_ok = a.sh_down == nullptr || a.sh_I_loc == 0 || a.sh_nseg * a.sh_nsub == nsb_r;
        if (sh_ok && (nsb_r == 16 || nsb_r == 8)) {
            const int R = 32 / nsb_r;
            if (a.D % (R * kWarps / 2) == 0) {
                const unsigned g2 = (unsigned)(a.D / (R * kWarps / 2));
                return nsb_r == 16 ? launch_with_smem(down_rows_kernel<MAXM, 16, 2>, g2, smem, a, s)
                                   : launch_with_smem(down_rows_kernel<MAXM, 8, 2>, g2, smem, a, s);
            }
        }
        return launch_with_smem(down_kernel<MAXM>, grid, smem, a, s);
    }
    ExpertArgs b = a;
    b.hconv = nullptr;
    return launch_with_smem(down_kernel<MAXM>, grid, smem, b, s);
}

}  // namespace

size_t gateup_smem_bytes(const ExpertArgs& a) {
    return (size_t)a.M * (a.D >> 5) * (16 * 4 + 4) + (size_t)(a.e_hi - a.e_lo) * 4;
}
size_t down_smem_bytes(const ExpertArgs& a) {
    const int I_max = a.I_loc > a.sh_I_loc ? a.I_loc : a.sh_I_loc;
    return (size_t)a.M * (a.k + 1) * (I_max >> 5) * (16 * 4 + 4) + (size_t)(a.e_hi - a.e_lo) * 4;
}

cudaError_t launch_gateup(const ExpertArgs& a, cudaStream_t s) {
    if (a.M <= 1) return launch_gateup_m<1>(a, s);
    if (a.M <= 4) return launch_gateup_m<4>(a, s);
    if (a.M <= 8) return launch_gateup_m<8>(a, s);
    return launch_gateup_m<16>(a, s);
}

cudaError_t launch_down(const ExpertArgs& a, cudaStream_t s) {
    if (a.M <= 1) return launch_down_m<1>(a, s);
    if (a.M <= 4) return launch_down_m<4>(a, s);
    if (a.M <= 8) return launch_down_m<8>(a, s);
    return launch_down_m<16>(a, s);
}

// The block's expert stages on formatted weights (x already converted by the
// route launch into `xconv`).
cudaError_t launch_fmt_experts(const void* x, int x_f32, int M, const qmoe_dims& d, const qmoe_formats& fm,
                               const qmoe_layer_weights& w, const int32_t* ids, const float* weights,
                               const float* shared_logit, float* h, int h_stride, const int* xconv, float* out,
                               int* status, cudaStream_t s) {
    ExpertArgs a{};
    a.x = x;
    a.x_f32 = x_f32;
    a.M = M;
    a.D = d.hidden;
    a.k = d.top_k;
    a.e_lo = 0;
    a.e_hi = d.n_experts;
    a.E = d.n_experts;
    a.ids = ids;
    a.weights = weights;
    a.shared_logit = d.sh_inter_local > 0 ? shared_logit : nullptr;
    a.gate_up = (const uint8_t*)w.gate_up;
    a.I_loc = d.inter;
    a.sh_gate_up = d.sh_inter_local > 0 ? (const uint8_t*)w.sh_gate_up : nullptr;
    a.sh_I_loc = d.sh_inter_local;
    a.h = h;
    a.h_stride = h_stride;
    a.xconv = xconv;
    a.down = (const uint8_t*)w.down;
    a.sh_down = d.sh_inter_local > 0 ? (const uint8_t*)w.sh_down : nullptr;
    a.out = out;
    a.status = status;
    FmtSel f{};
    f.gu = fm.gate_up;
    f.dn = fm.down;
    f.sgu = fm.sh_gate_up;
    f.sdn = fm.sh_down;
    f.gu_rb = (int)fmt_row_bytes(fm.gate_up, d.hidden);
    f.dn_rb = (int)fmt_row_bytes(fm.down, d.inter);
    f.sgu_rb = d.sh_inter_local > 0 ? (int)fmt_row_bytes(fm.sh_gate_up, d.hidden) : 0;
    f.sdn_rb = d.sh_inter_local > 0 ? (int)fmt_row_bytes(fm.sh_down, d.sh_inter_local) : 0;
    a.gu_expert_bytes = (size_t)2 * d.inter * f.gu_rb;
    a.dn_expert_bytes = (size_t)d.hidden * f.dn_rb;

    const int nsb = d.hidden >> 5;
    const size_t smem_g = (size_t)M * nsb * 68 + (size_t)d.n_experts * 4;
    const long tasks = (long)(M * d.top_k + 1) * (d.inter > d.sh_inter_local ? d.inter : d.sh_inter_local);
    unsigned grid = (unsigned)((tasks + kWarps - 1) / kWarps);
    if (M > 1) grid = min(grid, (unsigned)device_sm_count() * 3u);
    const int sbl = (nsb + 31) / 32;
    cudaError_t err;
    auto gu = [&](auto kern) {
        cudaError_t e = smem_opt_in(reinterpret_cast<const void*>(kern), (int)smem_g);
        if (e != cudaSuccess) return e;
        kern<<<grid, kWarps * 32, smem_g, s>>>(a, f);
        return cudaGetLastError();
    };
#define QMOE_FMT_GU(MM)                                               \
    switch (sbl) {                                                     \
        case 1: err = gu(fmt_gateup_kernel<MM, 1>); break;             \
        case 2: err = gu(fmt_gateup_kernel<MM, 2>); break;             \
        case 3: err = gu(fmt_gateup_kernel<MM, 3>); break;             \
        default: err = gu(fmt_gateup_kernel<MM, 4>); break;            \
    }
    if (M <= 1) { QMOE_FMT_GU(1) } else if (M <= 4) { QMOE_FMT_GU(4) } else if (M <= 8) { QMOE_FMT_GU(8) } else { QMOE_FMT_GU(16) }
#undef QMOE_FMT_GU
    if (err != cudaSuccess) return err;

    const int I_max = d.inter > d.sh_inter_local ? d.inter : d.sh_inter_local;
    const size_t smem_d = (size_t)M * (d.top_k + 1) * (I_max >> 5) * 68 + (size_t)d.n_experts * 4;
    if (M > 1) {
        a.hconv = h;
        a.hconv_stride = h_stride;
        const int nb = M * (d.top_k + 1) * (I_max >> 5);
        convert_h_kernel<<<(unsigned)((nb + kWarps - 1) / kWarps), kWarps * 32, 0, s>>>(a);
        err = cudaGetLastError();
        if (err != cudaSuccess) return err;
    }
    const unsigned grid_d = (unsigned)((d.hidden + kWarps - 1) / kWarps);
    auto dn = [&](auto kern) {
        cudaError_t e = smem_opt_in(reinterpret_cast<const void*>(kern), (int)smem_d);
        if (e != cudaSuccess) return e;
        kern<<<grid_d, kWarps * 32, smem_d, s>>>(a, f);
        return cudaGetLastError();
    };
    if (M <= 1) return dn(fmt_down_kernel<1>);
    if (M <= 4) return dn(fmt_down_kernel<4>);
    if (M <= 8) return dn(fmt_down_kernel<8>);
    return dn(fmt_down_kernel<16>);
}

}  // namespace qmoe
