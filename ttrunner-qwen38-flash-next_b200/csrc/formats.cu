// The real checkpoint's other expert formats (the reference's gguf/quants.py;
// tt/plan.py:90-103 puts IQ3_S on gate|up and IQ4_NL, or Q8_0 for the first
// layers, on down): a bit-exact decode to fp32 and the MoE block's expert
// stages on weights of any of them.
//
//   Q8_0    32 values in 34 bytes: fp16 d, 32 int8            (quants.py:33-37)
//   IQ4_NL  32 values in 18 bytes: fp16 d, 16 bytes of codes  (quants.py:100-108)
//   IQ3_S   256 values in 110 bytes: fp16 d, qs[64], qh[8], signs[32],
//           scales[4]; 9-bit grid indices, one sign bit per value,
//           d * (1 + 2 sc) per 32 values                       (quants.py:132-165)
//   IQ4_XS  the format of the rest of this library            (quants.py:112-129)
//
// Every weight is decoded with the reference's own arithmetic (one fp32
// multiply by the block scale), so the decode is bitwise the reference's.  The
// expert stages decode a 32-value sub-block per lane into fp32 and accumulate
// its dot product with the fp32 activation: a warp per (token, slot, row pair)
// for gate|up + SwiGLU, a warp per (token, output row) for the down and the
// weighted combine with the gated shared expert.  These formats take this
// general path; the IQ4_XS path keeps its integer decode core.
#include "common.cuh"

namespace qmoe {
namespace {

#define QMOE_IQ3S_GRID_DEF __device__ uint32_t g_iq3s_grid[512]
#include "iq3s_grid.inc"
#undef QMOE_IQ3S_GRID_DEF

__device__ float g_kvf[16] = {-127.f, -104.f, -83.f, -65.f, -49.f, -35.f, -22.f, -10.f,
                              1.f, 13.f, 25.f, 38.f, 53.f, 69.f, 89.f, 113.f};

// The two code tables in shared memory, where lanes with different codes read
// them in one pass (a constant-bank read serialises on distinct addresses).
struct FmtTables {
    uint32_t grid[512];
    float kv[16];
};

__device__ __forceinline__ void load_tables(FmtTables& t) {
    for (int i = threadIdx.x; i < 512; i += blockDim.x) t.grid[i] = g_iq3s_grid[i];
    if (threadIdx.x < 16) t.kv[threadIdx.x] = g_kvf[threadIdx.x];
    __syncthreads();
}

constexpr int kFmtWarps = 8;

__device__ __forceinline__ float f16_at(const uint8_t* p) {
    return __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
}

// Activation values off .. off + 31 as load_act returns them; 16-byte loads
// when x is 16-byte aligned (off is a multiple of 32).
__device__ __forceinline__ void load_act32(const void* x, int x_f32, bool vec, size_t off, float (&xv)[32]) {
    if (!vec) {
#pragma unroll
        for (int j = 0; j < 32; ++j) xv[j] = load_act(x, x_f32, off + j);
        return;
    }
    if (x_f32) {
        const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(x) + off);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 v = __ldg(p + i);
            xv[4 * i] = __bfloat162float(__float2bfloat16_rn(v.x));
            xv[4 * i + 1] = __bfloat162float(__float2bfloat16_rn(v.y));
            xv[4 * i + 2] = __bfloat162float(__float2bfloat16_rn(v.z));
            xv[4 * i + 3] = __bfloat162float(__float2bfloat16_rn(v.w));
        }
        return;
    }
    const uint4* p = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(x) + off);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint4 v = __ldg(p + i);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            xv[8 * i + 2 * q] = __uint_as_float(w[q] << 16);
            xv[8 * i + 2 * q + 1] = __uint_as_float(w[q] & 0xFFFF0000u);
        }
    }
}

// Values 0..31 of 32-value sub-block sb of a row in format fmt.
__device__ __forceinline__ void decode32(int fmt, const uint8_t* row, int64_t sb, float (&v)[32],
                                         const FmtTables& tb) {
    if (fmt == QMOE_FMT_Q8_0) {
        const uint8_t* blk = row + (size_t)sb * 34;
        const float d = f16_at(blk);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = d * (float)(int8_t)blk[2 + j];
    } else if (fmt == QMOE_FMT_IQ4_NL) {
        const uint8_t* blk = row + (size_t)sb * 18;
        const float d = f16_at(blk);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const uint8_t q = blk[2 + j];
            v[j] = tb.kv[q & 0xF] * d;
            v[16 + j] = tb.kv[q >> 4] * d;
        }
    } else if (fmt == QMOE_FMT_IQ4_XS) {
        const uint8_t* blk = row + (size_t)(sb >> 3) * 136;
        const int ib = sb & 7;
        const float d = f16_at(blk);
        const uint32_t sh = (uint32_t)blk[2] | ((uint32_t)blk[3] << 8);
        const uint32_t ls = (((uint32_t)blk[4 + ib / 2] >> (4 * (ib % 2))) & 0xF) | (((sh >> (2 * ib)) & 3) << 4);
        const float dl = d * ((float)ls - 32.0f);
        const uint8_t* q = blk + 8 + ib * 16;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            v[j] = tb.kv[q[j] & 0xF] * dl;
            v[16 + j] = tb.kv[q[j] >> 4] * dl;
        }
    } else {  // QMOE_FMT_IQ3_S
        const uint8_t* blk = row + (size_t)(sb >> 3) * 110;
        const int ib32 = sb & 7;
        const float d = f16_at(blk);
        const int sc = (blk[106 + ib32 / 2] >> (4 * (ib32 % 2))) & 0xF;
        const float db = d * (1.0f + 2.0f * (float)sc);
        const uint8_t* qs = blk + 2 + ib32 * 8;
        const int h = blk[66 + ib32];
        const uint8_t* sg = blk + 74 + ib32 * 4;
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const uint32_t g1 = tb.grid[qs[2 * l] | ((h << (8 - 2 * l)) & 256)];
            const uint32_t g2 = tb.grid[qs[2 * l + 1] | ((h << (7 - 2 * l)) & 256)];
            const int s = sg[l];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float a = (float)((g1 >> (8 * k)) & 0xFF) * (((s >> k) & 1) ? -1.0f : 1.0f);
                const float b = (float)((g2 >> (8 * k)) & 0xFF) * (((s >> (4 + k)) & 1) ? -1.0f : 1.0f);
                v[l * 8 + k] = a * db;
                v[l * 8 + 4 + k] = b * db;
            }
        }
    }
}

__global__ void fmt_dequant_kernel(int fmt, const uint8_t* __restrict__ raw, int64_t n_sub, float* __restrict__ out) {
    __shared__ FmtTables tb;
    load_tables(tb);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_sub; i += (int64_t)gridDim.x * blockDim.x) {
        float v[32];
        decode32(fmt, raw, i, v, tb);
        float4* o = reinterpret_cast<float4*>(out + i * 32);
#pragma unroll
        for (int q = 0; q < 8; ++q) o[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    }
}

// Arguments of the two expert stages on formatted weights.
struct FmtArgs {
    const void* x;
    int x_f32;
    int M, D, I, Ish, E, k;
    int f_gu, f_dn, f_sgu, f_sdn;
    size_t gu_row, dn_row, sgu_row, sdn_row;  // bytes per row
    const uint8_t* gate_up;                   // [E][2I rows]
    const uint8_t* down;                      // [E][D rows]
    const uint8_t* sh_gate_up;                // [2 Ish rows] or null
    const uint8_t* sh_down;                   // [D rows]
    const int32_t* ids;                       // [M][k]
    const float* weights;                     // [M][k]
    const float* shared_logit;                // [M] or null
    float* h;                                 // [M][k + 1][h_stride]
    int h_stride;
    float* out;                               // [M][D]
    int* status;
};

// h[m][s][r] = silu(G_e[r] . x_m) * (U_e[r] . x_m); slot k: the shared expert.
__global__ void __launch_bounds__(kFmtWarps * 32) fmt_gateup_kernel(FmtArgs a) {
    __shared__ FmtTables tb;
    load_tables(tb);
    const int lane = threadIdx.x & 31;
    const bool xvec = (reinterpret_cast<uintptr_t>(a.x) & 15) == 0;
    const int K1 = a.k + 1, Imax = max(a.I, a.Ish);
    const long tasks = (long)a.M * K1 * Imax;
    const int nsb = a.D >> 5;
    for (long t = (long)blockIdx.x * kFmtWarps + (threadIdx.x >> 5); t < tasks; t += (long)gridDim.x * kFmtWarps) {
        const int r = (int)(t % Imax);
        const int ms = (int)(t / Imax), m = ms / K1, s = ms % K1;
        const uint8_t *grow, *urow;
        int fmt;
        if (s < a.k) {
            if (r >= a.I) continue;
            const int e = a.ids[m * a.k + s];
            if (e < 0 || e >= a.E) {
                if (lane == 0 && r == 0) record_status(a.status, QMOE_ERR_DEVICE_RANGE);
                continue;
            }
            grow = a.gate_up + ((size_t)e * 2 * a.I + r) * a.gu_row;
            urow = grow + (size_t)a.I * a.gu_row;
            fmt = a.f_gu;
        } else {
            if (!a.sh_gate_up || r >= a.Ish) continue;
            grow = a.sh_gate_up + (size_t)r * a.sgu_row;
            urow = grow + (size_t)a.Ish * a.sgu_row;
            fmt = a.f_sgu;
        }
        float g = 0.0f, u = 0.0f;
        for (int sb = lane; sb < nsb; sb += 32) {
            float xv[32];
            load_act32(a.x, a.x_f32, xvec, (size_t)m * a.D + sb * 32, xv);
            float w[32];
            decode32(fmt, grow, sb, w, tb);
#pragma unroll
            for (int j = 0; j < 32; ++j) g = fmaf(w[j], xv[j], g);
            decode32(fmt, urow, sb, w, tb);
#pragma unroll
            for (int j = 0; j < 32; ++j) u = fmaf(w[j], xv[j], u);
        }
        g = warp_sum(g);
        u = warp_sum(u);
        if (lane == 0) a.h[((size_t)m * K1 + s) * a.h_stride + r] = silu(g) * u;
    }
}

// out[m][j] = sum_s w[m][s] D_e[j] . h[m][s] + sigmoid(shared logit) Dsh[j] . h[m][k]
__global__ void __launch_bounds__(kFmtWarps * 32) fmt_down_kernel(FmtArgs a) {
    __shared__ FmtTables tb;
    load_tables(tb);
    const int lane = threadIdx.x & 31;
    const int K1 = a.k + 1;
    const int nr = a.I >> 5, ns = a.Ish >> 5;
    const int units = a.k * nr + (a.sh_down ? ns : 0);
    const long tasks = (long)a.M * a.D;
    for (long t = (long)blockIdx.x * kFmtWarps + (threadIdx.x >> 5); t < tasks; t += (long)gridDim.x * kFmtWarps) {
        const int m = (int)(t / a.D), j = (int)(t % a.D);
        float acc = 0.0f;
        for (int q = lane; q < units; q += 32) {
            const uint8_t* row;
            int fmt, sb, s;
            float w;
            if (q < a.k * nr) {
                s = q / nr;
                sb = q - s * nr;
                const int e = a.ids[m * a.k + s];
                if (e < 0 || e >= a.E) continue;
                row = a.down + ((size_t)e * a.D + j) * a.dn_row;
                fmt = a.f_dn;
                w = a.weights[m * a.k + s];
            } else {
                s = a.k;
                sb = q - a.k * nr;
                row = a.sh_down + (size_t)j * a.sdn_row;
                fmt = a.f_sdn;
                w = a.shared_logit ? sigmoid(a.shared_logit[m]) : 1.0f;
            }
            float v[32];
            decode32(fmt, row, sb, v, tb);
            const float4* hh = reinterpret_cast<const float4*>(a.h + ((size_t)m * K1 + s) * a.h_stride + sb * 32);
            float d = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float4 h4 = hh[i];
                d = fmaf(v[4 * i], h4.x, d);
                d = fmaf(v[4 * i + 1], h4.y, d);
                d = fmaf(v[4 * i + 2], h4.z, d);
                d = fmaf(v[4 * i + 3], h4.w, d);
            }
            acc = fmaf(w, d, acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) a.out[(size_t)m * a.D + j] = acc;
    }
}

}  // namespace

// Bytes of a row of n values in format fmt (0: not a whole number of blocks or unknown format).
size_t fmt_row_bytes(int fmt, int64_t n) {
    switch (fmt) {
        case QMOE_FMT_Q8_0: return n % 32 ? 0 : (size_t)(n / 32) * 34;
        case QMOE_FMT_IQ4_NL: return n % 32 ? 0 : (size_t)(n / 32) * 18;
        case QMOE_FMT_IQ3_S: return n % 256 ? 0 : (size_t)(n / 256) * 110;
        case QMOE_FMT_IQ4_XS: return n % 256 ? 0 : (size_t)(n / 256) * 136;
        default: return 0;
    }
}

cudaError_t launch_fmt_dequant(int fmt, const uint8_t* raw, int64_t n_values, float* out, cudaStream_t s) {
    const int64_t n_sub = n_values / 32;
    int64_t g = (n_sub + 255) / 256;
    const int64_t cap = (int64_t)device_sm_count() * 16;
    if (g > cap) g = cap;
    if (g < 1) g = 1;
    const unsigned grid = (unsigned)g;
    fmt_dequant_kernel<<<grid, 256, 0, s>>>(fmt, raw, n_sub, out);
    return cudaGetLastError();
}

cudaError_t launch_fmt_experts(const void* x, int x_f32, int M, const qmoe_dims& d, const qmoe_formats& f,
                               const qmoe_layer_weights& w, const int32_t* ids, const float* weights,
                               const float* shared_logit, float* h, int h_stride, float* out, int* status,
                               cudaStream_t s) {
    FmtArgs a{};
    a.x = x;
    a.x_f32 = x_f32;
    a.M = M;
    a.D = d.hidden;
    a.I = d.inter;
    a.Ish = d.sh_inter_local;
    a.E = d.n_experts;
    a.k = d.top_k;
    a.f_gu = f.gate_up;
    a.f_dn = f.down;
    a.f_sgu = f.sh_gate_up;
    a.f_sdn = f.sh_down;
    a.gu_row = fmt_row_bytes(f.gate_up, d.hidden);
    a.dn_row = fmt_row_bytes(f.down, d.inter);
    a.sgu_row = fmt_row_bytes(f.sh_gate_up, d.hidden);
    a.sdn_row = fmt_row_bytes(f.sh_down, d.sh_inter_local > 0 ? d.sh_inter_local : 32);
    a.gate_up = (const uint8_t*)w.gate_up;
    a.down = (const uint8_t*)w.down;
    a.sh_gate_up = d.sh_inter_local > 0 ? (const uint8_t*)w.sh_gate_up : nullptr;
    a.sh_down = d.sh_inter_local > 0 ? (const uint8_t*)w.sh_down : nullptr;
    a.ids = ids;
    a.weights = weights;
    a.shared_logit = d.sh_inter_local > 0 ? shared_logit : nullptr;
    a.h = h;
    a.h_stride = h_stride;
    a.out = out;
    a.status = status;
    const long cap = (long)device_sm_count() * 8;
    const long gt = (long)M * (d.top_k + 1) * (d.inter > d.sh_inter_local ? d.inter : d.sh_inter_local);
    long g1 = (gt + kFmtWarps - 1) / kFmtWarps;
    if (g1 > cap) g1 = cap;
    fmt_gateup_kernel<<<(unsigned)g1, kFmtWarps * 32, 0, s>>>(a);
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return err;
    long g2 = ((long)M * d.hidden + kFmtWarps - 1) / kFmtWarps;
    if (g2 > cap) g2 = cap;
    fmt_down_kernel<<<(unsigned)g2, kFmtWarps * 32, 0, s>>>(a);
    return cudaGetLastError();
}

}  // namespace qmoe
