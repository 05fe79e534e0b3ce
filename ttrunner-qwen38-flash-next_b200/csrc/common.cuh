// Internal declarations shared by the kernel translation units.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <map>
#include <mutex>

#include "../../include/qmoe_b200.h"
#include "iq4xs.cuh"

namespace qmoe {

constexpr int kMaxTokens = 16;     // decode / verify GEMV path
constexpr int kMaxTopK = 16;
constexpr int kMaxExperts = 1024;
constexpr int kMaxHidden = 4096;
constexpr int kMaxUnique = kMaxTokens * kMaxTopK + 1;

// Workspace layout (bytes from the workspace base), sized for max_tokens.
struct WsLayout {
    size_t status;      // int32 status word + padding
    size_t counter;     // uint32 arrival counter of the router's last-CTA select
    size_t logits;      // fp32 [max_tokens][n_experts + 1]
    size_t ids;         // int32 [max_tokens][top_k]
    size_t weights;     // fp32 [max_tokens][top_k]
    size_t shared;      // fp32 [max_tokens]
    size_t h;           // fp32 [max_tokens][top_k + 1][h_stride]
    size_t act;         // fp32 [max_tokens][hidden]: the stack kernel's layer activation
    size_t sync;        // the stack kernel's synchronisation area (stack_sync_bytes)
    size_t trace;       // u64: the stack kernel's phase timestamps (kTraceBytes)
    size_t act_trace;   // bf16 [64 layers][hidden]: the single launch's per-layer outputs
    size_t route_trace; // int32 [64][16] ids, then fp32 [64][16] weights, per layer
    size_t total;
    int h_stride;
};

WsLayout ws_layout(const qmoe_dims& d, int max_tokens);

// A kernel's opt-in to at least `bytes` of dynamic shared memory, made only
// when it raises what this process already set for (kernel, device), instead
// of before every launch.
inline cudaError_t smem_opt_in(const void* fn, int bytes) {
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, int> set_to;
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    std::lock_guard<std::mutex> g(mu);
    int& cur = set_to[std::make_pair(fn, dev)];
    if (bytes <= cur) return cudaSuccess;
    err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (err == cudaSuccess) cur = bytes;
    return err;
}

// The stack kernel's synchronisation area (the workspace's `sync` region),
// byte offsets from its base, every item on its own 128-byte lines:
//   0      launch counter (u32; kept across launches: the tags below use it)
//   128    abort word (u32)
//   256    arrival counters of the activation rounds: 8 lines (u32 at each start)
//   1280   arrival counters of the h rounds: 8 lines
//   2304   arrival counters of the logit rounds: 8 lines
//   3328   the router logits as tagged words: E + 1 u64
//   then   the layer activation as tagged words: D u32
//   then   SwiGLU activations h as tagged words: (k + 1) x I u32
// [128, 3328) is zeroed before every launch; the tagged words carry the
// launch counter in their tags instead.
constexpr size_t kStackAbortOff = 128;
constexpr size_t kStackXCountOff = 256;
constexpr size_t kStackHCountOff = 1280;
constexpr size_t kStackLCountOff = 2304;
constexpr size_t kStackLogitOff = 3328;
__host__ __device__ constexpr size_t stack_logit_bytes(int E) { return ((size_t)(E + 2) * 8 + 127) & ~(size_t)127; }
__host__ __device__ constexpr size_t stack_xw_off(int E) { return kStackLogitOff + stack_logit_bytes(E); }
__host__ __device__ constexpr size_t stack_hw_off(int E, int D) { return stack_xw_off(E) + (((size_t)D * 4 + 127) & ~(size_t)127); }
__host__ __device__ constexpr size_t stack_sync_bytes(int E, int D, int K, int I) {
    return stack_hw_off(E, D) + (size_t)(K + 1) * I * 4;
}

// Phase stamps per layer in the stack kernel's trace ([2][64 layers][slots]).
#if defined(QMOE_SK_FULLTRACE)
constexpr int kTraceSlots = 32;      // development builds: more points,
constexpr int kFullTraceCtas = 160;  // every CTA's stamps
constexpr size_t kTraceBytes = (size_t)64 * kFullTraceCtas * kTraceSlots * 8;
#else
constexpr int kTraceSlots = 24;
constexpr size_t kTraceBytes = (size_t)2 * 64 * kTraceSlots * 8;
#endif

// In-kernel exchange between ranks: a rank's exchange buffer holds its
// launch counter (first 128 bytes), then the receive words
// u64 [2 parities][R][hidden] that the peers store into.
constexpr int kMaxXchgRanks = 8;
constexpr size_t kXchgHeader = 128;
inline size_t xchg_bytes(int R, int hidden) { return kXchgHeader + (size_t)2 * R * hidden * 8; }

// Where the stack kernel exchanges partial rows with its peers.
struct XchgDesc {
    int R, rank;
    unsigned char* buf[kMaxXchgRanks];  // every rank's exchange buffer as mapped here
};

// Launch arguments of the routing kernel.
struct RouteArgs {
    const void* x;
    int x_f32;
    int M, D, E, k;
    const float* router;
    const float* gate_vec;  // may be null
    float* logits;          // [M][E + 1] workspace
    unsigned int* counter;
    int32_t* ids;           // [M][k]
    float* weights;         // [M][k]
    float* shared_logit;    // [M] or null
    int* status;
    // Selection: 0 exact top-k (k slots); 1, 2 tie-admitting threshold at the
    // thr_k-th probability (fp32, bf16 probabilities), the k slots filled from
    // experts [e_lo, e_hi).
    int thr_mode, thr_k, e_lo, e_hi;
    // Non-null: the launch also writes x in block floating point for the
    // gate|up kernel, [M][D/32][16] pair words then [M][D/32] steps.
    int* xconv;
};

// Arguments shared by the two expert kernels.
struct ExpertArgs {
    const void* x;          // gate|up input
    int x_f32;
    int M, D, k;
    int e_lo, e_hi, E;
    const int32_t* ids;     // [M][k]
    const float* weights;   // [M][k]
    const float* shared_logit;  // [M] or null
    // gate|up
    const uint8_t* gate_up;
    size_t gu_expert_bytes;
    int I_loc;              // gate rows (= up rows) per routed expert
    const uint8_t* sh_gate_up;
    int sh_I_loc;           // 0: no shared expert
    float* h;               // [M][k+1][h_stride]
    int h_stride;
    // the h blocks in block floating point for M > 1: block b of (token m,
    // slot s) at float (m * (k+1) + s) * h_stride + 32 b, 16 pair words then
    // the step (the workspace's h region; may be h itself)
    float* hconv;           // null: the down kernel converts h itself
    int hconv_stride;
    // x in block floating point as the route launch wrote it (RouteArgs::xconv);
    // null: the gate|up kernel converts x itself
    const int* xconv;
    // down
    const uint8_t* down;
    size_t dn_expert_bytes;
    int dn_nseg, dn_nsub, dn_ib0;
    const uint8_t* sh_down;
    int sh_nseg, sh_nsub, sh_ib0;
    float* out;             // [M][D]
    int* status;
};

cudaError_t launch_route(const RouteArgs& a, cudaStream_t s);
cudaError_t launch_gateup(const ExpertArgs& a, cudaStream_t s);
cudaError_t launch_down(const ExpertArgs& a, cudaStream_t s);
cudaError_t launch_dequant(const uint8_t* blocks, int64_t n_blocks, float* out, cudaStream_t s);
cudaError_t launch_quantize(const float* x, int64_t n_blocks, uint8_t* out, cudaStream_t s);
cudaError_t launch_synth_iq4xs(uint64_t seed, uint64_t sid, int64_t n_blocks, float std_dev,
                               uint8_t* out, cudaStream_t s);
cudaError_t launch_synth_f32(uint64_t seed, uint64_t sid, int64_t n, float std_dev, float* out,
                             cudaStream_t s);

int device_sm_count();

// Per-layer records of the single-launch stack and its teacher input (all may be null).
struct StackTraceBufs {
    __nv_bfloat16* act;              // [n_layers][hidden] each layer's output, bf16
    int* ids;                        // [n_layers][top_k]
    float* weights;                  // [n_layers][top_k]
    const __nv_bfloat16* teacher;    // [n_layers][hidden] each layer's input, or null (the chain)
};

// The single-launch decode stack kernel (stack_kernel.cu).  R ranks exchange
// their partial rows inside the kernel when R > 1.
// xc: null for one rank.
bool stack_kernel_supported(const qmoe_dims& d, int M, int n_layers, int R);
cudaError_t launch_stack_kernel(const void* x, float* out, unsigned char* sync, unsigned long long* trace,
                                int* status, const qmoe_layer_weights* layers, int n_layers, const qmoe_dims& d,
                                const XchgDesc* xc, const StackTraceBufs& tb, cudaStream_t stream);

// The other expert formats (formats.cu).
size_t fmt_row_bytes(int fmt, int64_t n);
cudaError_t launch_fmt_dequant(int fmt, const uint8_t* raw, int64_t n_values, float* out, cudaStream_t s);
cudaError_t launch_fmt_experts(const void* x, int x_f32, int M, const qmoe_dims& d, const qmoe_formats& f,
                               const qmoe_layer_weights& w, const int32_t* ids, const float* weights,
                               const float* shared_logit, float* h, int h_stride, const int* xconv, float* out,
                               int* status, cudaStream_t s);

// The hyper-connection mixer (hc.cu).
size_t hc_workspace_bytes(int M, int hc, int rank);
size_t hc_down_smem(int M, int hc, int D);
size_t hc_up_smem(int M, int rank);
cudaError_t launch_hc_mix(const void* hyper, int f32, int M, int D, int hc, int rank, float eps,
                          const float* norm_w, const float* down_w, const float* up_w, const float* inject_w,
                          float* mixed, float* inject, unsigned char* ws, cudaStream_t s);
cudaError_t launch_hc_reinject(const void* hyper, int h_f32, const void* branch, int b_f32, const float* inject,
                               int M, int D, int hc, float* out, cudaStream_t s);

// Prefill / large verify chunks (prefill.cu).
int prefill_max_tokens();
int prefill_small_group_max(int n);
int prefill_trace(int enable);
bool prefill_supported(const qmoe_dims& d);
struct PfLayout;
size_t prefill_workspace_bytes(const qmoe_dims& d, int T);
// The activations as bf16 [T][hidden], 16-byte aligned: x itself when it already is, else a copy
// in the workspace.
const __nv_bfloat16* prefill_act_bf16(const void* x, int x_f32, bool x_ok, int T, const qmoe_dims& d,
                                      unsigned char* ws, cudaStream_t s);
// thr_mode, thr_k: as RouteArgs (0: exact top-k).
cudaError_t launch_prefill_route(const __nv_bfloat16* xb, int T, const qmoe_layer_weights& w, const qmoe_dims& d,
                                 unsigned char* ws, int32_t* ids, float* weights, float* shared_logit,
                                 cudaStream_t s, int thr_mode = 0, int thr_k = 0);
cudaError_t launch_prefill_experts(const __nv_bfloat16* xb, int T, const int32_t* ids, const float* weights,
                                   const float* shared_logit, const qmoe_layer_weights& w, const qmoe_dims& d,
                                   float* out, unsigned char* ws, cudaStream_t s);
// Device pointers to the prefill workspace's routing table (ids, weights, shared logit).
void prefill_route_buffers(const qmoe_dims& d, int T, unsigned char* ws, int32_t** ids, float** weights,
                           float** shared_logit);

}  // namespace qmoe

#if defined(__CUDACC__)
namespace qmoe {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Activation element i of row m as float: bf16 as stored, or fp32 rounded to
// bf16 (the activation dtype between layers).
__device__ __forceinline__ float load_act(const void* x, int x_f32, size_t i) {
    if (x_f32) {
        const float v = reinterpret_cast<const float*>(x)[i];
        return __bfloat162float(__float2bfloat16_rn(v));
    }
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[i]);
}

// x[0, n) as load_act returns it, into shared memory (16-byte aligned): every
// load of a thread's batch is issued before any store, 16-byte loads when x is
// 16-byte aligned and n a multiple of 8.
__device__ __forceinline__ void stage_act(float* dst, const void* x, int x_f32, int n) {
    constexpr int U = 8;
    const int nt = blockDim.x;
    if ((reinterpret_cast<uintptr_t>(x) & 15) == 0 && (n & 7) == 0) {
        const int n8 = n >> 3;
        const uint4* src = reinterpret_cast<const uint4*>(x);
        for (int g0 = threadIdx.x; g0 < n8; g0 += nt * U) {
            uint4 lo[U], hi[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int g = g0 + u * nt;
                if (g < n8) {
                    if (x_f32) {
                        lo[u] = __ldcg(src + 2 * g);
                        hi[u] = __ldcg(src + 2 * g + 1);
                    } else {
                        lo[u] = __ldcg(src + g);
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int g = g0 + u * nt;
                if (g >= n8) break;
                float4 a, b;
                if (x_f32) {
                    auto r = [](uint32_t w) { return __bfloat162float(__float2bfloat16_rn(__uint_as_float(w))); };
                    a = make_float4(r(lo[u].x), r(lo[u].y), r(lo[u].z), r(lo[u].w));
                    b = make_float4(r(hi[u].x), r(hi[u].y), r(hi[u].z), r(hi[u].w));
                } else {
                    auto l = [](uint32_t w) { return __uint_as_float(w << 16); };
                    auto h = [](uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); };
                    a = make_float4(l(lo[u].x), h(lo[u].x), l(lo[u].y), h(lo[u].y));
                    b = make_float4(l(lo[u].z), h(lo[u].z), l(lo[u].w), h(lo[u].w));
                }
                reinterpret_cast<float4*>(dst)[2 * g] = a;
                reinterpret_cast<float4*>(dst)[2 * g + 1] = b;
            }
        }
        return;
    }
    for (int i0 = threadIdx.x; i0 < n; i0 += nt * U) {
        float v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) v[u] = i0 + u * nt < n ? load_act(x, x_f32, (size_t)(i0 + u * nt)) : 0.0f;
#pragma unroll
        for (int u = 0; u < U; ++u)
            if (i0 + u * nt < n) dst[i0 + u * nt] = v[u];
    }
}

__device__ __forceinline__ void record_status(int* status, int code) {
    if (status) atomicCAS(status, 0, code);
}

// Block floating point of one 32-value activation block, one value per lane
// (lane j holds value j).  The step is 2^(e-14) with |x| < 2^e for the
// block's largest |x|, so every mantissa fits int16 with a bit to spare;
// values within 2^-6 of the block maximum convert exactly from bf16.
// Returns, in lanes 0..15, the pair word q_j | q_(16+j) << 16 -- the order in
// which an IQ4_XS qs byte holds its two codes; *step gets the step in every
// lane.  Zero or subnormal blocks give zeros; a non-finite value gives a NaN
// step so the result is NaN, as in fp32 arithmetic.
__device__ __forceinline__ int warp_block_fp(float v, float* step) {
    const unsigned mb = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(v)));
    const int E = (int)(mb >> 23);  // biased exponent of the block maximum
    int q = 0;
    float st = 0.0f;
    if (E >= 255) {
        st = __uint_as_float(0x7fc00000u);
    } else if (E >= 1) {
        const int k = 140 - E;  // q = rint(v * 2^k), k in [-114, 139]
        const int k1 = k >> 1, k2 = k - k1;
        const float s1 = __uint_as_float((unsigned)(127 + k1) << 23);
        const float s2 = __uint_as_float((unsigned)(127 + k2) << 23);
        // rint((v * s1) * s2) on the FMA pipe: the product is exact (powers of
        // two) and below 2^15 in magnitude, so adding 1.5 * 2^23 rounds it to
        // an integer in the low mantissa bits (round to nearest even).
        q = __float_as_int(fmaf(v * s1, s2, 12582912.0f)) - 0x4B400000;
        st = E >= 14 ? __uint_as_float((unsigned)(E - 13) << 23) : __uint_as_float(1u << (E + 9));
    }
    const int hi = __shfl_down_sync(0xffffffffu, q, 16);
    *step = st;
    return (q & 0xFFFF) | (hi << 16);
}

// warp_block_fp for N blocks at once (v[i]: this lane's value of block i),
// the same arithmetic step by step for every block before the next step, so
// the blocks' warp reductions and shuffles are in flight together instead of
// one block's chain after another's.
template <int N>
__device__ __forceinline__ void warp_block_fp_n(const float (&v)[N], int (&pw)[N], float (&step)[N]) {
    unsigned mb[N];
#pragma unroll
    for (int i = 0; i < N; ++i) mb[i] = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(v[i])));
    int q[N];
#pragma unroll
    for (int i = 0; i < N; ++i) {
        const int E = (int)(mb[i] >> 23);
        q[i] = 0;
        step[i] = 0.0f;
        if (E >= 255) {
            step[i] = __uint_as_float(0x7fc00000u);
        } else if (E >= 1) {
            const int k = 140 - E;
            const int k1 = k >> 1, k2 = k - k1;
            const float s1 = __uint_as_float((unsigned)(127 + k1) << 23);
            const float s2 = __uint_as_float((unsigned)(127 + k2) << 23);
            q[i] = __float_as_int(fmaf(v[i] * s1, s2, 12582912.0f)) - 0x4B400000;
            step[i] = E >= 14 ? __uint_as_float((unsigned)(E - 13) << 23) : __uint_as_float(1u << (E + 9));
        }
    }
#pragma unroll
    for (int i = 0; i < N; ++i) {
        const int hi = __shfl_down_sync(0xffffffffu, q[i], 16);
        pw[i] = (q[i] & 0xFFFF) | (hi << 16);
    }
}

__device__ __forceinline__ float silu(float g) { return g / (1.0f + expf(-g)); }
__device__ __forceinline__ float sigmoid(float z) { return 1.0f / (1.0f + expf(-z)); }

}  // namespace qmoe
#endif
