/*
 * qmoe_b200.h -- C ABI of the B200 (sm_100a) qwen4exp MoE block.
 *
 * Plain pointers and sizes only.  Every pointer named "device" must point to
 * CUDA device memory of the current device; `stream` is a cudaStream_t passed
 * as void* (NULL = legacy default stream).  Every function returns an int
 * status (QMOE_OK = 0); qmoe_status_string() names it.  Kernels never trap:
 * device-side range violations (an expert id outside [0, n_experts)) are
 * recorded in the workspace status word and read back by qmoe_read_status().
 *
 * Weight formats (all little-endian, GGUF byte order):
 *   - router:   fp32 [n_experts, hidden] row-major       (blk.L.ffn_gate_inp.weight)
 *   - gate_vec: fp32 [hidden]                             (blk.L.ffn_gate_inp_shexp.weight)
 *   - gate_up:  IQ4_XS, per local expert 2*inter_local rows of `hidden`
 *               values: gate rows [0, inter_local) then up rows
 *               [inter_local, 2*inter_local).  Row = hidden/256 super-blocks of
 *               136 bytes (blk.L.ffn_gate_exps / ffn_up_exps, rows concatenated).
 *   - down:     IQ4_XS row slices, per local expert `hidden` rows; a row holds
 *               `down_nseg` segments of (8-byte super-block header + down_nsub
 *               sub-blocks of 16 bytes of qs).  Unsliced rows (n_seg = inter/256,
 *               n_sub = 8) are exactly the GGUF bytes of blk.L.ffn_down_exps.
 * The shared expert uses the same formats with one expert.
 */
#ifndef QMOE_B200_H
#define QMOE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum qmoe_status_code {
    QMOE_OK = 0,
    QMOE_ERR_INVALID_ARG = 1,      /* null pointer, negative size, bad enum        */
    QMOE_ERR_UNSUPPORTED = 2,      /* shape outside what the kernels are built for */
    QMOE_ERR_ALIGNMENT = 3,        /* a pointer breaks the 16-byte alignment rule  */
    QMOE_ERR_WORKSPACE = 4,        /* workspace missing or too small               */
    QMOE_ERR_CUDA = 5,             /* a CUDA runtime call failed                   */
    QMOE_ERR_DEVICE_RANGE = 6,     /* a kernel saw an expert id out of range       */
    QMOE_ERR_NOT_FINITE = 7,       /* a kernel saw a non-finite router logit       */
    QMOE_ERR_TIMEOUT = 8           /* a bounded device wait (grid barrier or bulk
                                      copy) ran out: the kernel stopped early     */
};

/* Activation element types accepted by the entry points. */
enum qmoe_act_dtype {
    QMOE_ACT_BF16 = 0,   /* bf16 activations (the reference's device dtype)        */
    QMOE_ACT_F32 = 1     /* fp32, rounded to bf16 on load (layer chaining)         */
};

/* One layer's weights.  sh_* may be NULL: no shared expert on this rank. */
typedef struct qmoe_layer_weights {
    const float* router;        /* [n_experts, hidden] fp32                        */
    const float* gate_vec;      /* [hidden] fp32 or NULL (no shared expert)        */
    const void* gate_up;        /* local routed experts, IQ4_XS                    */
    const void* down;           /* local routed experts, IQ4_XS row slices         */
    const void* sh_gate_up;     /* shared expert gate|up or NULL                   */
    const void* sh_down;        /* shared expert down or NULL                      */
} qmoe_layer_weights;

/* Shapes and the shard this rank holds.
 *   variant A (expert axis):        expert_lo/expert_hi = this rank's window.
 *   variant B (intermediate axis):  inter_local = inter/n, down_ib0/down_nsub
 *                                   describe the column slice of each down row. */
typedef struct qmoe_dims {
    int hidden;          /* D: multiple of 256, <= 4096                          */
    int inter;           /* I: full expert intermediate (multiple of 256)        */
    int n_experts;       /* E: multiple of 32, <= 1024                           */
    int top_k;           /* k: 1..16                                             */
    int expert_lo;       /* first local expert id                                */
    int expert_hi;       /* one past the last local expert id (== lo: none)      */
    int inter_local;     /* rows of gate (and of up) held per routed expert     */
    int down_nseg;       /* segments per routed down row                         */
    int down_nsub;       /* 32-value sub-blocks per segment (1..8)               */
    int down_ib0;        /* first sub-block index inside the super-block          */
    int sh_inter_local;  /* shared expert rows of gate per rank (0 = none)       */
    int sh_down_nseg;
    int sh_down_nsub;
    int sh_down_ib0;
} qmoe_dims;

/* ---- library ------------------------------------------------------------ */
const char* qmoe_status_string(int status);
int qmoe_version(void);
/* Largest token count the decode/verify (GEMV) kernels accept. */
int qmoe_max_tokens(void);

/* Workspace bytes for calls with up to `max_tokens` rows.  The workspace must
 * be zero-filled once before first use (qmoe_workspace_init). */
size_t qmoe_workspace_bytes(const qmoe_dims* dims, int max_tokens);
int qmoe_workspace_init(void* workspace, size_t bytes, void* stream);
/* Copies the device status word to *status_out (synchronising `stream`) and
 * clears it.  *status_out is QMOE_OK or a QMOE_ERR_* code. */
int qmoe_read_status(void* workspace, int* status_out, void* stream);

/* ---- IQ4_XS ------------------------------------------------------------- */
/* Replaces gguf/quants.py:112-129 (_dequant_iq4_xs) through dequantize()
 * (gguf/quants.py:214).  blocks: device, n_blocks*136 bytes; out: device
 * fp32, n_blocks*256 values.  Bit-exact with the reference. */
int qmoe_dequant_iq4xs_f32(const void* blocks, int64_t n_blocks, float* out, void* stream);

/* Synthetic-weight builder (the reference converts a real checkpoint with
 * tt/convert.py:151; this project generates seeded weights instead).
 * Host quantiser: fp32 -> IQ4_XS, n_values a multiple of 256. */
int qmoe_quantize_iq4xs_host(const float* values, int64_t n_values, void* out_blocks, int n_threads);
/* Same quantiser on the device (bit-identical to the host one). */
int qmoe_quantize_iq4xs(const float* values, int64_t n_values, void* out_blocks, void* stream);
/* Device generator: N(0, std^2) values from a counter-based RNG keyed by
 * (seed, stream_id), quantised to IQ4_XS (synth_iq4xs) or kept fp32. */
int qmoe_synth_iq4xs(uint64_t seed, uint64_t stream_id, int64_t n_values, float std_dev,
                     void* out_blocks, void* stream);
int qmoe_synth_f32(uint64_t seed, uint64_t stream_id, int64_t n_values, float std_dev,
                   float* out, void* stream);
/* The same two generators on the host (OpenMP, n_threads >= 1), bit-identical
 * to the device ones: every arithmetic step is a correctly rounded binary32
 * operation.  out: host memory. */
int qmoe_synth_iq4xs_host(uint64_t seed, uint64_t stream_id, int64_t n_values, float std_dev,
                          void* out_blocks, int n_threads);
int qmoe_synth_f32_host(uint64_t seed, uint64_t stream_id, int64_t n_values, float std_dev,
                        float* out, int n_threads);

/* ---- the MoE block, by stage --------------------------------------------- */
/* Router + top-k + renormalise.  Replaces reference/model.py:399-403 and the
 * device pair tt/moe.py:199-237 (ksgemv router, softmax, fused_router_select /
 * scripts/kernels/router_select.cpp:159-273 with EXACT_TOPK).  Selection is on
 * fp32 logits, ties to the lower expert id; weights are the softmax over the
 * k selected, in descending order.  ids/weights: device [M, k];
 * shared_logit: device [M] (x . gate_vec, before the sigmoid) or NULL. */
int qmoe_route(const void* x, int x_dtype, int n_tokens, const qmoe_layer_weights* w,
               const qmoe_dims* dims, int32_t* ids, float* weights, float* shared_logit,
               void* workspace, size_t workspace_bytes, void* stream);

/* Gathered gate|up GEMV + SwiGLU over the selected experts and the shared one.
 * Replaces tt/moe.py:946-953 (gather_gemv MODE 2 + fused_swiglu) and the
 * shared half of tt/moe.py:999-1028.  h: device fp32 [M, k+1, h_stride]; slot
 * k holds the shared expert. */
/* Router with the tie-admitting threshold select: the reference device
 * select's other mode (scripts/kernels/router_select.cpp:223-255,
 * TT_ROUTER_EXACT_TOPK=0; the ttnn chain tt/moe.py:308-327).  Softmax
 * probabilities p_e over all E experts (rounded to bf16 when probs_bf16 = 1,
 * as the ttnn chain compares them); t = the top_k-th largest p counting
 * equal values separately; total = the sum of every p_e >= t.  The
 * dims->top_k slots (K_SEL, >= top_k) take the largest positive p_e >= t
 * among experts [expert_lo, expert_hi), descending, ties to the lower id, as
 * (id, p_e * (1 / total)); slots left over hold (expert_lo, 0), which the
 * expert stages compute with weight 0.  The probability sums run over each
 * lane's ids in order and then a butterfly over 32 lanes (the oracle's
 * route_threshold restates that order).  ids/weights: device [M, dims->top_k]. */
int qmoe_route_threshold(const void* x, int x_dtype, int n_tokens, const qmoe_layer_weights* w,
                         const qmoe_dims* dims, int top_k, int probs_bf16, int32_t* ids, float* weights,
                         float* shared_logit, void* workspace, size_t workspace_bytes, void* stream);
int qmoe_gateup_swiglu(const void* x, int x_dtype, int n_tokens, const int32_t* ids,
                       const qmoe_layer_weights* w, const qmoe_dims* dims, float* h,
                       int h_stride, void* workspace, size_t workspace_bytes, void* stream);

/* Gathered down GEMV fused with the routing-weighted sum and the
 * sigmoid-gated shared expert.  Replaces tt/moe.py:958-975 (gather_gemv
 * MODE 0, the combine) and tt/moe.py:1029-1044.  out: device fp32 [M, hidden]
 * (this rank's partial sum when sharded). */
int qmoe_down_combine(const float* h, int h_stride, int n_tokens, const int32_t* ids,
                      const float* weights, const float* shared_logit,
                      const qmoe_layer_weights* w, const qmoe_dims* dims, float* out,
                      void* workspace, size_t workspace_bytes, void* stream);

/* The whole block: routed experts + shared expert, x [M, hidden] -> out fp32
 * [M, hidden].  Replaces TTModel._moe_block (tt/model.py:2010-2052: moe_block
 * tt/moe.py:159 + shared_expert tt/moe.py:983) before its all-reduce, and the
 * oracle Qwen4ExpModel._moe (reference/model.py:387-417). */
int qmoe_moe_block(const void* x, int x_dtype, int n_tokens, const qmoe_layer_weights* w,
                   const qmoe_dims* dims, float* out, void* workspace, size_t workspace_bytes,
                   void* stream);

/* 1 when qmoe_stack_decode runs these shapes as one persistent launch (one
 * token, hidden 1024 or 2048, inter 512 with a 512-row shared expert, the
 * whole expert range and the shared expert sliced like the routed ones,
 * <= 64 layers, operands 16-byte aligned), else 0 (three launches per
 * layer).  The whole-stack analogue of the traced step (tt/traced.py:261-277),
 * which replays all 48 layers' MoE ops at once. */
int qmoe_stack_single_launch(const qmoe_dims* dims, int n_tokens, int n_layers);

/* Tracing: the single-launch stack kernel stamps its SM's cycle counter at 24
 * points of every layer into the workspace (unused points stay 0): CTA 0
 * and the last CTA each at layer start, x gathered, x checked, ranked and
 * gate|up copies issued, shared pairs done, gate|up pairs done, h words
 * written, h round complete, h converted, down rows landed, down done,
 * output rows written, arrived (0-12), gate|up chunks 0-5
 * landed (16-21), and with an exchange between ranks partial rows sent,
 * peers' rows summed (22-23).  Copies the n_layers x 24 stamps of CTA 0 and
 * then those of the last CTA (2 x n_layers x 24 values; the two are
 * different SMs' clocks) of the last launch made with this workspace and
 * n_tokens to host_out (synchronises `stream`).  The reference's analogue is
 * its section profiler (tt/bench.py:33-78). */
int qmoe_read_stack_trace(void* workspace, const qmoe_dims* dims, int n_tokens, int n_layers,
                          uint64_t* host_out, void* stream);

/* The single launch's per-layer record of its last call with this workspace
 * (n_tokens = 1): act_out [n_layers, hidden] bf16 bits, each layer's output
 * rounded to bf16 (the next layer's input); ids_out [n_layers, top_k] the
 * selected experts in rank order; weights_out [n_layers, top_k] their
 * renormalised routing weights.  Any of the three may be NULL.  Host buffers;
 * synchronises `stream`.  The analogue of the reference's per-layer probe
 * (reference/model.py:37-40, `probe(layer, hidden)`). */
int qmoe_read_stack_route_trace(void* workspace, const qmoe_dims* dims, int n_tokens, int n_layers,
                                uint16_t* act_out, int32_t* ids_out, float* weights_out, void* stream);

/* The single-launch stack with every layer's input supplied: layer L reads
 * x_layers[L] (device bf16 [n_layers, hidden]) instead of layer L-1's output,
 * everything else exactly as qmoe_stack_decode with one token (the same
 * kernel, the same phases and inter-layer handoff of the router logits).
 * Layer-by-layer checks of the whole launch use it with a well-conditioned
 * input per layer (the reference's decode_vs_reference harness feeds each
 * layer the reference's own hidden state, scripts/dev/decode_vs_reference.py).
 * out: the last layer's fp32 output; the per-layer outputs are in the route
 * trace.  QMOE_ERR_UNSUPPORTED where the single launch does not apply. */
int qmoe_stack_decode_teacher(const void* x_layers, const qmoe_layer_weights* layers, int n_layers,
                              const qmoe_dims* dims, float* out, void* workspace, size_t workspace_bytes,
                              void* stream);

/* The shared expert alone: sigmoid(x . gate_vec) * down(silu(gate x) * up x).
 * Replaces tt/moe.py:983-1044 (shared_expert) and reference/model.py:392-397.
 * Uses gate_vec, sh_gate_up and sh_down of `w`; routed fields are ignored. */
int qmoe_shared_expert(const void* x, int x_dtype, int n_tokens, const qmoe_layer_weights* w,
                       const qmoe_dims* dims, float* out, void* workspace, size_t workspace_bytes,
                       void* stream);

/* A stack of n_layers blocks, the output of layer L (rounded to bf16) feeding
 * layer L+1; the per-layer MoE calls of TTModel.step (tt/model.py:2056,
 * 48 x _moe_block) with nothing between them.  layers: host array of
 * n_layers weight sets; x: device bf16 [M, hidden]; out: device fp32
 * [M, hidden] (the last layer's output); act: device fp32 scratch
 * [M, hidden] or NULL (then `out` is used).  Stream-ordered, no host sync,
 * no allocation: capturable into a CUDA graph. */
int qmoe_stack_decode(const void* x, int n_tokens, const qmoe_layer_weights* layers,
                      int n_layers, const qmoe_dims* dims, float* out, void* workspace,
                      size_t workspace_bytes, void* stream);

/* ---- the stack sharded over the GPUs of one node ---------------------------
 * One process per GPU, rank r of n_ranks (2, 4 or 8) holding the slice
 * [r * inter / n, (r + 1) * inter / n) of every expert's intermediate rows
 * (gate/up rows and the matching down columns; the shared expert sliced the
 * same way): the reference's shipped shard plan (tt/plan.py:70-103).  Where
 * the reference all-reduces each layer's partial output over its fabric
 * (TTModel._moe_block, tt/model.py:2041-2052; tt/ops.py:97-111), here the
 * single-launch stack kernel of every rank stores its partial rows straight
 * into the peers' exchange buffers over NVLink and sums the n partials of
 * its rows in rank order, so every rank ends each layer with bitwise the same
 * activation and routes identically.
 *
 * Each rank allocates its exchange buffer with qmoe_xchg_alloc (zeroed; the
 * 64-byte CUDA IPC handle goes to the peers through the caller's own
 * channel, e.g. an all-gather), maps every peer's with qmoe_xchg_open, and
 * passes all of them in a qmoe_xchg.  The buffers carry a launch counter:
 * every rank must make the same sequence of qmoe_stack_decode_xchg calls with
 * the same n_layers, and after a call that reports an error (a peer that
 * never arrived: QMOE_ERR_TIMEOUT after a bounded wait) every rank resets
 * its buffer with qmoe_xchg_reset (or frees and allocates them anew).  Unmap peers (qmoe_xchg_close) and
 * free (qmoe_xchg_free) only when no rank has a launch in flight. */
typedef struct qmoe_xchg {
    int rank;
    int n_ranks;
    void* buf[8]; /* every rank's exchange buffer as mapped in this process; buf[rank] is this rank's own */
} qmoe_xchg;

#define QMOE_XCHG_HANDLE_BYTES 64

size_t qmoe_xchg_bytes(int n_ranks, int hidden);
/* cudaMalloc + zero (synchronous) on the current device; ipc_handle receives
 * QMOE_XCHG_HANDLE_BYTES bytes for the peers. */
int qmoe_xchg_alloc(int n_ranks, int hidden, void** buf, void* ipc_handle);
/* Maps a peer's exchange buffer into this process (peer access enabled). */
int qmoe_xchg_open(const void* ipc_handle, void** peer_buf);
int qmoe_xchg_close(void* peer_buf);
int qmoe_xchg_free(void* buf);
/* Zeroes this rank's own exchange buffer (launch counter and receive words),
 * stream-ordered.  After a call that failed on any rank (a host-side launch
 * error, or QMOE_ERR_TIMEOUT from a peer that never arrived), the ranks'
 * launch counters disagree; every rank then calls this on its own buffer,
 * with no launch in flight anywhere and a barrier across the ranks before
 * and after, and the exchange starts again from launch 0. */
int qmoe_xchg_reset(void* buf, int n_ranks, int hidden, void* stream);
/* 1 when qmoe_stack_decode_xchg runs these dims (this rank's slice) on
 * n_ranks ranks: the shapes of qmoe_stack_single_launch with
 * inter_local * n_ranks == inter. */
int qmoe_stack_xchg_supported(const qmoe_dims* dims, int n_ranks, int n_tokens, int n_layers);
/* qmoe_stack_decode on this rank's slice with the per-layer sum over ranks
 * inside the launch: out [1, hidden] fp32 is the full (summed) last layer's
 * output, the same bits on every rank.  Stream-ordered, capturable into a
 * CUDA graph (one launch per call). */
int qmoe_stack_decode_xchg(const void* x, int n_tokens, const qmoe_layer_weights* layers, int n_layers,
                           const qmoe_dims* dims, const qmoe_xchg* xc, float* out, void* workspace,
                           size_t workspace_bytes, void* stream);

/* The MoE block for callers that cannot allocate device memory: the same
 * computation as qmoe_moe_block, with no workspace argument.  No counterpart
 * in the reference: it exists for hosts bound through a plain C ABI (cgo,
 * JNI, N-API) without a device allocator, plug-ins whose process's device
 * memory belongs to another framework's allocator, and serving loops that
 * forbid allocation after start-up.  It calls no cudaMalloc, cudaFree or
 * allocating library routine; its scratch is a file-scope device array of
 * QMOE_NOALLOC_SCRATCH_BYTES that every GPU loading the library holds until
 * the process exits.  Calls needing more scratch than that (see
 * qmoe_workspace_bytes) return QMOE_ERR_WORKSPACE.  All calls on a device
 * share the array: calls that overlap on the GPU race, so order them.  The
 * first call on a device looks up the array's address and must come before
 * any stream capture. */
#define QMOE_NOALLOC_SCRATCH_BYTES (1u << 20)
int qmoe_moe_block_noalloc(const void* x, int x_dtype, int n_tokens, const qmoe_layer_weights* w,
                           const qmoe_dims* dims, float* out, void* stream);
/* The device-side status of the no-allocation calls on the current device:
 * the first error any of them recorded since the last read (QMOE_OK if none;
 * QMOE_ERR_NOT_FINITE for a non-finite router logit), copied to *status_out,
 * then cleared.  Synchronises `stream`; order it after the calls it reports
 * on.  No counterpart in the reference (its fused kernels have no status
 * word); it allocates nothing. */
int qmoe_noalloc_read_status(int* status_out, void* stream);

/* ---- Chunked prefill and large verify chunks: T tokens through one layer ----
 * Replaces TTModel._prefill_ffn_half (tt/model.py:2812-2907): moe.route
 * (tt/moe.py:308-327), apply_experts / expert_ffn (tt/moe.py:330-368,
 * 1057-1152) and shared_expert (tt/moe.py:983) over a chunk.  Tokens are
 * grouped per expert on the device; each group runs as an IQ4_XS -> bf16
 * expansion in shared memory feeding tcgen05 tensor-core tiles (fp32
 * accumulation), SwiGLU, then the down projection scatter-added into out
 * with the routing weights.  Unsharded dims only (expert window = all
 * experts, whole intermediate rows); hidden and inter multiples of 512;
 * 1 <= n_tokens <= qmoe_prefill_max_tokens() and n_tokens * top_k <= 102400.
 * Weight tensors 16-byte aligned.  Stream-ordered, no host sync.  Routed
 * outputs are summed with fp32 atomics, so the low bits of `out` may differ
 * between runs. */
int qmoe_prefill_max_tokens(void);
/* Experts that see at most this many tokens of a chunk (default 8, at most
 * 8) skip the bf16 expansion and run as a grouped GEMV: each IQ4_XS row is
 * decoded once with the decode path's integer core and dotted with every
 * token of the group; larger groups take the tcgen05 grouped GEMM.  n >= 0
 * sets it (0: every group on the tensor cores), n < 0 only queries; returns
 * the previous value.  One process-wide setting for every device and thread
 * (an atomic: setting it while another thread issues a prefill is safe), read
 * once when a call is issued.  The
 * reference has no counterpart (its prefill runs every group through the
 * same matmul, tt/moe.py:330-368). */
int qmoe_prefill_small_group_max(int n);
/* Diagnostics: enable != 0 makes the grouped GEMM's CTA 0 stamp its pipeline
 * clock (%clock64) per A slot into the prefill workspace (bytes 256 .. 4351:
 * [64 slots][8 events] u64: B copy issued, MMA thread past the A and B waits,
 * MMAs issued, expansion past its slot wait and done, stage issued, expansion
 * past the stage wait); 0 turns it off (the default: the stamps slow CTA 0);
 * < 0 only queries.  Returns the previous value.  Process-wide, like
 * qmoe_prefill_small_group_max.  The reference's counterpart is its section
 * profiler (tt/bench.py:33-78). */
int qmoe_prefill_trace(int enable);
size_t qmoe_prefill_workspace_bytes(const qmoe_dims* dims, int n_tokens);
/* ids [T, top_k] int32 and weights [T, top_k] fp32 (renormalised, descending,
 * ties to the lower id); shared_logit [T] (x . gate_vec) or NULL. */
int qmoe_prefill_route(const void* x, int x_dtype, int n_tokens, const qmoe_layer_weights* w,
                       const qmoe_dims* dims, int32_t* ids, float* weights, float* shared_logit,
                       void* workspace, size_t workspace_bytes, void* stream);
/* The same with the tie-admitting threshold select (as qmoe_route_threshold;
 * the whole expert range only); ids/weights [T, dims->top_k]. */
int qmoe_prefill_route_threshold(const void* x, int x_dtype, int n_tokens, const qmoe_layer_weights* w,
                                 const qmoe_dims* dims, int top_k, int probs_bf16, int32_t* ids, float* weights,
                                 float* shared_logit, void* workspace, size_t workspace_bytes, void* stream);
/* out [T, hidden] fp32 = sum_s weights[t,s] * expert_{ids[t,s]}(x_t)
 *                      + sigmoid(shared_logit[t]) * shared(x_t) (when the dims
 * carry a shared expert; shared_logit is then required).  Out-of-range ids
 * are skipped and set QMOE_ERR_DEVICE_RANGE in the workspace status word. */
int qmoe_prefill_experts(const void* x, int x_dtype, int n_tokens, const int32_t* ids,
                         const float* weights, const float* shared_logit,
                         const qmoe_layer_weights* w, const qmoe_dims* dims, float* out,
                         void* workspace, size_t workspace_bytes, void* stream);
/* qmoe_prefill_route followed by qmoe_prefill_experts. */
int qmoe_prefill(const void* x, int x_dtype, int n_tokens, const qmoe_layer_weights* w,
                 const qmoe_dims* dims, float* out, void* workspace, size_t workspace_bytes,
                 void* stream);

/* ---- the real checkpoint's other expert formats ---------------------------- */
/* GGML block formats by their GGML type ids (the reference's gguf/reader.py:53-74):
 * Q8_0 (32 values, 34 bytes), IQ4_NL (32, 18), IQ3_S (256, 110), IQ4_XS (256, 136).
 * The reference's checkpoint stores gate|up as IQ3_S and down as IQ4_NL, or
 * Q8_0 in its first layers (tt/plan.py:90-103). */
enum qmoe_format {
    QMOE_FMT_Q8_0 = 8,
    QMOE_FMT_IQ4_NL = 20,
    QMOE_FMT_IQ3_S = 21,
    QMOE_FMT_IQ4_XS = 23
};

/* The format of each expert tensor of a layer. */
typedef struct qmoe_formats {
    int gate_up;     /* routed experts' fused gate|up rows  */
    int down;        /* routed experts' down rows           */
    int sh_gate_up;  /* shared expert's gate|up rows        */
    int sh_down;     /* shared expert's down rows           */
} qmoe_formats;

/* Bytes of a row of n_values values in `format`; 0 when n_values is not a
 * whole number of its blocks or the format is unknown. */
size_t qmoe_format_row_bytes(int format, int64_t n_values);
/* Decode n_values values of `format` to fp32, bitwise the reference's
 * gguf.quants.dequantize (quants.py:33-37 Q8_0, :100-108 IQ4_NL, :112-129
 * IQ4_XS, :132-165 IQ3_S).  blocks 16-byte aligned; out fp32 16-byte aligned. */
int qmoe_dequant_f32(int format, const void* blocks, int64_t n_values, float* out, void* stream);
/* The MoE block (as qmoe_moe_block: routed experts + gated shared expert,
 * reference/model.py:387-417) on expert tensors of the given formats, laid
 * out as the IQ4_XS ones are (gate_up [E][2I rows], down [E][D rows], rows of
 * qmoe_format_row_bytes bytes).  Unsharded dims only (the whole expert range
 * and intermediate width); shared expert optional (sh_inter_local = 0).
 * Routing is the exact top-k; each 32-value sub-block becomes int8 words and
 * a scale (the codebook or grid values, signs applied) dotted with x and h in
 * block floating point, as the IQ4_XS path does.  Every weight tensor 16-byte
 * aligned (QMOE_ERR_ALIGNMENT otherwise).  out [M, hidden] fp32. */
int qmoe_moe_block_formats(const void* x, int x_dtype, int n_tokens, const qmoe_layer_weights* w,
                           const qmoe_dims* dims, const qmoe_formats* formats, float* out,
                           void* workspace, size_t workspace_bytes, void* stream);

/* ---- the hyper-connection mixer around the block ------------------------ */
/* The reference's gated residual (reference/model.py:53-81; device ops
 * tt/ops.py:2627 gated_residual_mix and :2825 reinject): the MoE block reads
 * `mixed` and its output (the branch) goes back into every residual stream
 * weighted by `inject`.  hyper [M, hc * hidden] holds hc residual streams. */
typedef struct qmoe_hc_weights {
    const float* norm_w;    /* [hc * hidden] RMS-norm weights, stream-major          */
    const float* down_w;    /* [rank, hc * hidden]                                    */
    const float* up_w;      /* [hc * hidden, rank]                                    */
    const float* inject_w;  /* [hc, hc * hidden]                                      */
} qmoe_hc_weights;

typedef struct qmoe_hc_dims {
    int hidden;  /* per-stream width: multiple of 32                                  */
    int hc;      /* streams: 1..16                                                   */
    int rank;    /* width of the low-rank gate: 1..4096                              */
    float eps;   /* RMS-norm epsilon (the config's rms_norm_eps)                      */
} qmoe_hc_dims;

/* Workspace bytes of qmoe_hc_mix for n_tokens tokens (256-byte aligned base). */
size_t qmoe_hc_workspace_bytes(const qmoe_hc_dims* dims, int n_tokens);
/* normed = rms_norm(hyper, norm_w, eps) per stream of `hidden` values
 * (reference/layers.py:31-43); mixed [M, hidden] fp32 = mean over the streams
 * of sigmoid(up_w . silu(down_w . normed / hc)) * normed; inject [M, hc] fp32
 * = 2 sigmoid(inject_w . normed / hc) (model.py:62-77).  hyper: device, bf16 or
 * fp32 (hyper_dtype); weights fp32; all 16-byte aligned.  fp32 arithmetic. */
int qmoe_hc_mix(const void* hyper, int hyper_dtype, int n_tokens, const qmoe_hc_weights* w,
                const qmoe_hc_dims* dims, float* mixed, float* inject, void* workspace,
                size_t workspace_bytes, void* stream);
/* out [M, hc * hidden] fp32 = hyper + branch (outer) inject, stream s of token m
 * adding branch[m] * inject[m][s] (model.py:80-81).  branch [M, hidden] bf16 or
 * fp32 (branch_dtype); out may be hyper itself when that is fp32. */
int qmoe_hc_reinject(const void* hyper, int hyper_dtype, const void* branch, int branch_dtype,
                     const float* inject, int n_tokens, const qmoe_hc_dims* dims, float* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* QMOE_B200_H */
