// extern "C" entry points: argument checks, workspace layout, launches.
#include <stdio.h>
#include <string.h>

#include "common.cuh"

namespace qmoe {

size_t gateup_smem_bytes(const ExpertArgs& a);
size_t down_smem_bytes(const ExpertArgs& a);

namespace {

constexpr size_t kSmemLimit = 200 * 1024;  // dynamic shared memory ceiling per CTA

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
bool aligned(const void* p, size_t a) { return ((uintptr_t)p % a) == 0; }

int check_dims(const qmoe_dims* d) {
    if (!d) return QMOE_ERR_INVALID_ARG;
    if (d->hidden < 256 || d->hidden > kMaxHidden || d->hidden % 256) return QMOE_ERR_UNSUPPORTED;
    if (d->inter < 32 || d->inter % 32) return QMOE_ERR_UNSUPPORTED;
    if (d->n_experts < 32 || d->n_experts > kMaxExperts || d->n_experts % 32) return QMOE_ERR_UNSUPPORTED;
    if (d->top_k < 1 || d->top_k > kMaxTopK || d->top_k > d->n_experts) return QMOE_ERR_UNSUPPORTED;
    if (d->expert_lo < 0 || d->expert_hi > d->n_experts || d->expert_lo > d->expert_hi)
        return QMOE_ERR_INVALID_ARG;
    if (d->inter_local < 32 || d->inter_local % 32 || d->inter_local > d->inter) return QMOE_ERR_UNSUPPORTED;
    if (d->down_nseg < 1 || d->down_nsub < 1 || d->down_nsub > 8 || d->down_ib0 < 0 ||
        d->down_ib0 + d->down_nsub > 8 || d->down_nseg * d->down_nsub * 32 != d->inter_local)
        return QMOE_ERR_UNSUPPORTED;
    if (d->sh_inter_local < 0 || d->sh_inter_local % 32 || d->sh_inter_local > 8192) return QMOE_ERR_UNSUPPORTED;
    if (d->sh_inter_local > 0 &&
        (d->sh_down_nseg < 1 || d->sh_down_nsub < 1 || d->sh_down_nsub > 8 || d->sh_down_ib0 < 0 ||
         d->sh_down_ib0 + d->sh_down_nsub > 8 ||
         d->sh_down_nseg * d->sh_down_nsub * 32 != d->sh_inter_local))
        return QMOE_ERR_UNSUPPORTED;
    return QMOE_OK;
}

int check_tokens(int M) { return (M >= 1 && M <= kMaxTokens) ? QMOE_OK : QMOE_ERR_UNSUPPORTED; }

int check_act(const void* x, int x_dtype) {
    if (!x) return QMOE_ERR_INVALID_ARG;
    if (x_dtype != QMOE_ACT_BF16 && x_dtype != QMOE_ACT_F32) return QMOE_ERR_INVALID_ARG;
    if (!aligned(x, x_dtype == QMOE_ACT_F32 ? 4 : 2)) return QMOE_ERR_ALIGNMENT;
    return QMOE_OK;
}

int check_weights_route(const qmoe_layer_weights* w) {
    if (!w || !w->router) return QMOE_ERR_INVALID_ARG;
    if (!aligned(w->router, 16)) return QMOE_ERR_ALIGNMENT;
    if (w->gate_vec && !aligned(w->gate_vec, 16)) return QMOE_ERR_ALIGNMENT;
    return QMOE_OK;
}

int check_weights_experts(const qmoe_layer_weights* w, const qmoe_dims* d) {
    if (!w) return QMOE_ERR_INVALID_ARG;
    if (d->expert_hi > d->expert_lo) {  // an empty window holds no routed experts
        if (!w->gate_up || !w->down) return QMOE_ERR_INVALID_ARG;
        if (!aligned(w->gate_up, 8) || !aligned(w->down, 8)) return QMOE_ERR_ALIGNMENT;
    }
    if (d->sh_inter_local > 0) {
        if (!w->sh_gate_up || !w->sh_down) return QMOE_ERR_INVALID_ARG;
        if (!aligned(w->sh_gate_up, 8) || !aligned(w->sh_down, 8)) return QMOE_ERR_ALIGNMENT;
    }
    return QMOE_OK;
}

int cuda_status(cudaError_t e) {
    if (e == cudaSuccess) return QMOE_OK;
    fprintf(stderr, "qmoe: CUDA error %s\n", cudaGetErrorString(e));
    return QMOE_ERR_CUDA;
}

ExpertArgs expert_args(const void* x, int x_dtype, int M, const int32_t* ids, const float* weights,
                       const float* shared_logit, const qmoe_layer_weights* w, const qmoe_dims* d,
                       float* h, int h_stride, float* out, int* status) {
    ExpertArgs a{};
    a.x = x;
    a.x_f32 = x_dtype == QMOE_ACT_F32;
    a.M = M;
    a.D = d->hidden;
    a.k = d->top_k;
    a.e_lo = d->expert_lo;
    a.e_hi = d->expert_hi;
    a.E = d->n_experts;
    a.ids = ids;
    a.weights = weights;
    a.shared_logit = shared_logit;
    a.gate_up = (const uint8_t*)w->gate_up;
    a.I_loc = d->inter_local;
    a.gu_expert_bytes = (size_t)2 * d->inter_local * (d->hidden / 256) * QMOE_SB_BYTES;
    a.sh_gate_up = d->sh_inter_local > 0 ? (const uint8_t*)w->sh_gate_up : nullptr;
    a.sh_I_loc = d->sh_inter_local;
    a.h = h;
    a.h_stride = h_stride;
    a.down = (const uint8_t*)w->down;
    a.dn_nseg = d->down_nseg;
    a.dn_nsub = d->down_nsub;
    a.dn_ib0 = d->down_ib0;
    a.dn_expert_bytes = (size_t)d->hidden * d->down_nseg * (8 + 16 * d->down_nsub);
    a.sh_down = d->sh_inter_local > 0 ? (const uint8_t*)w->sh_down : nullptr;
    a.sh_nseg = d->sh_inter_local > 0 ? d->sh_down_nseg : 1;
    a.sh_nsub = d->sh_inter_local > 0 ? d->sh_down_nsub : 1;
    a.sh_ib0 = d->sh_inter_local > 0 ? d->sh_down_ib0 : 0;
    a.out = out;
    a.status = status;
    return a;
}

int check_smem(const ExpertArgs& a) {
    if (gateup_smem_bytes(a) > kSmemLimit || down_smem_bytes(a) > kSmemLimit) return QMOE_ERR_UNSUPPORTED;
    return QMOE_OK;
}

int route_smem_ok(int M, int D) {
    return (size_t)M * D * sizeof(float) <= kSmemLimit - 16 * 1024 ? QMOE_OK : QMOE_ERR_UNSUPPORTED;
}

struct Ws {
    WsLayout L;
    unsigned char* base;
    int* status() const { return (int*)(base + L.status); }
    unsigned int* counter() const { return (unsigned int*)(base + L.counter); }
    float* logits() const { return (float*)(base + L.logits); }
    int32_t* ids() const { return (int32_t*)(base + L.ids); }
    float* weights() const { return (float*)(base + L.weights); }
    float* shared() const { return (float*)(base + L.shared); }
    float* h() const { return (float*)(base + L.h); }
    float* act() const { return (float*)(base + L.act); }
    unsigned* sync() const { return (unsigned*)(base + L.sync); }
    unsigned long long* trace() const { return (unsigned long long*)(base + L.trace); }
    StackTraceBufs trace_bufs(int top_k, const void* teacher = nullptr) const {
        StackTraceBufs t{};
        t.act = (__nv_bfloat16*)(base + L.act_trace);
        t.ids = (int*)(base + L.route_trace);
        t.weights = (float*)(base + L.route_trace) + 64 * kMaxTopK;
        t.teacher = (const __nv_bfloat16*)teacher;
        (void)top_k;
        return t;
    }
};

int get_ws(void* workspace, size_t bytes, const qmoe_dims* d, int M, Ws* ws) {
    if (!workspace) return QMOE_ERR_WORKSPACE;
    if (!aligned(workspace, 256)) return QMOE_ERR_ALIGNMENT;
    ws->L = ws_layout(*d, M);
    if (bytes < ws->L.total) return QMOE_ERR_WORKSPACE;
    ws->base = (unsigned char*)workspace;
    return QMOE_OK;
}

#define QMOE_TRY(expr)                 \
    do {                               \
        const int _rc = (expr);        \
        if (_rc != QMOE_OK) return _rc; \
    } while (0)

int run_route(const void* x, int x_dtype, int M, const qmoe_layer_weights* w, const qmoe_dims* d,
              int32_t* ids, float* weights, float* shared_logit, const Ws& ws, cudaStream_t s, int thr_mode = 0,
              int thr_k = 0, int* xconv = nullptr) {
    RouteArgs r{};
    r.x = x;
    r.x_f32 = x_dtype == QMOE_ACT_F32;
    r.M = M;
    r.D = d->hidden;
    r.E = d->n_experts;
    r.k = d->top_k;
    r.router = w->router;
    r.gate_vec = w->gate_vec;
    r.logits = ws.logits();
    r.counter = ws.counter();
    r.ids = ids;
    r.weights = weights;
    r.shared_logit = shared_logit;
    r.status = ws.status();
    r.thr_mode = thr_mode;
    r.thr_k = thr_k;
    r.e_lo = d->expert_lo;
    r.e_hi = d->expert_hi;
    r.xconv = xconv;
    return cuda_status(launch_route(r, s));
}

int run_block(const void* x, int x_dtype, int M, const qmoe_layer_weights* w, const qmoe_dims* d,
              float* out, const Ws& ws, cudaStream_t s) {
    // The route launch also leaves x in block floating point (the workspace's
    // act region) for every gate|up CTA to copy.
    int* xconv = (int*)ws.act();
    QMOE_TRY(run_route(x, x_dtype, M, w, d, ws.ids(), ws.weights(), ws.shared(), ws, s, 0, 0, xconv));
    ExpertArgs a = expert_args(x, x_dtype, M, ws.ids(), ws.weights(), ws.shared(), w, d, ws.h(),
                               ws.L.h_stride, out, ws.status());
    a.xconv = xconv;
    a.hconv = ws.h();
    a.hconv_stride = ws.L.h_stride;
    QMOE_TRY(cuda_status(launch_gateup(a, s)));
    return cuda_status(launch_down(a, s));
}

}  // namespace

WsLayout ws_layout(const qmoe_dims& d, int max_tokens) {
    WsLayout L{};
    const int M = max_tokens;
    const int hmax = d.inter_local > d.sh_inter_local ? d.inter_local : d.sh_inter_local;
    L.h_stride = (int)align_up((size_t)hmax, 32);
    size_t off = 0;
    L.status = off;
    L.counter = off + 64;
    off = 256;
    L.logits = off;
    off = align_up(off + (size_t)M * (d.n_experts + 1) * 4, 256);
    L.ids = off;
    off = align_up(off + (size_t)M * d.top_k * 4, 256);
    L.weights = off;
    off = align_up(off + (size_t)M * d.top_k * 4, 256);
    L.shared = off;
    off = align_up(off + (size_t)M * 4, 256);
    L.h = off;
    off = align_up(off + (size_t)M * (d.top_k + 1) * L.h_stride * 4, 256);
    L.act = off;
    off = align_up(off + (size_t)M * d.hidden * 4, 256);
    L.sync = off;
    off = align_up(off + stack_sync_bytes(d.n_experts, d.hidden, d.top_k, d.inter_local), 256);
    L.trace = off;
    off = align_up(off + kTraceBytes, 256);
    L.act_trace = off;
    off = align_up(off + (size_t)64 * d.hidden * 2, 256);
    L.route_trace = off;
    off = align_up(off + (size_t)64 * kMaxTopK * 8, 256);
    L.total = off;
    return L;
}

int device_sm_count() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
    return n;
}

}  // namespace qmoe

using namespace qmoe;

extern "C" {

const char* qmoe_status_string(int status) {
    switch (status) {
        case QMOE_OK: return "ok";
        case QMOE_ERR_INVALID_ARG: return "invalid argument";
        case QMOE_ERR_UNSUPPORTED: return "unsupported shape";
        case QMOE_ERR_ALIGNMENT: return "misaligned pointer";
        case QMOE_ERR_WORKSPACE: return "workspace missing or too small";
        case QMOE_ERR_CUDA: return "CUDA runtime error";
        case QMOE_ERR_DEVICE_RANGE: return "expert id out of range";
        case QMOE_ERR_NOT_FINITE: return "non-finite router logit";
        case QMOE_ERR_TIMEOUT: return "a bounded device wait timed out";
        default: return "unknown status";
    }
}

int qmoe_version(void) { return 1; }
int qmoe_max_tokens(void) { return kMaxTokens; }

size_t qmoe_workspace_bytes(const qmoe_dims* dims, int max_tokens) {
    if (check_dims(dims) != QMOE_OK || check_tokens(max_tokens) != QMOE_OK) return 0;
    return ws_layout(*dims, max_tokens).total;
}

int qmoe_workspace_init(void* workspace, size_t bytes, void* stream) {
    if (!workspace) return QMOE_ERR_WORKSPACE;
    return cuda_status(cudaMemsetAsync(workspace, 0, bytes, (cudaStream_t)stream));
}

int qmoe_read_status(void* workspace, int* status_out, void* stream) {
    if (!workspace || !status_out) return QMOE_ERR_INVALID_ARG;
    int v = 0;
    cudaStream_t s = (cudaStream_t)stream;
    QMOE_TRY(cuda_status(cudaMemcpyAsync(&v, workspace, sizeof(int), cudaMemcpyDeviceToHost, s)));
    QMOE_TRY(cuda_status(cudaStreamSynchronize(s)));
    QMOE_TRY(cuda_status(cudaMemsetAsync(workspace, 0, sizeof(int), s)));
    *status_out = v;
    return QMOE_OK;
}

int qmoe_dequant_iq4xs_f32(const void* blocks, int64_t n_blocks, float* out, void* stream) {
    if (n_blocks < 0) return QMOE_ERR_INVALID_ARG;
    if (n_blocks == 0) return QMOE_OK;
    if (!blocks || !out) return QMOE_ERR_INVALID_ARG;
    if (!aligned(blocks, 8) || !aligned(out, 16)) return QMOE_ERR_ALIGNMENT;
    return cuda_status(launch_dequant((const uint8_t*)blocks, n_blocks, out, (cudaStream_t)stream));
}

int qmoe_quantize_iq4xs(const float* values, int64_t n_values, void* out_blocks, void* stream) {
    if (n_values < 0 || n_values % 256) return QMOE_ERR_INVALID_ARG;
    if (n_values == 0) return QMOE_OK;
    if (!values || !out_blocks) return QMOE_ERR_INVALID_ARG;
    if (!aligned(values, 16) || !aligned(out_blocks, 8)) return QMOE_ERR_ALIGNMENT;
    return cuda_status(launch_quantize(values, n_values / 256, (uint8_t*)out_blocks, (cudaStream_t)stream));
}

int qmoe_synth_iq4xs(uint64_t seed, uint64_t stream_id, int64_t n_values, float std_dev,
                     void* out_blocks, void* stream) {
    if (n_values < 0 || n_values % 256) return QMOE_ERR_INVALID_ARG;
    if (n_values == 0) return QMOE_OK;
    if (!out_blocks) return QMOE_ERR_INVALID_ARG;
    if (!aligned(out_blocks, 8)) return QMOE_ERR_ALIGNMENT;
    return cuda_status(launch_synth_iq4xs(seed, stream_id, n_values / 256, std_dev,
                                          (uint8_t*)out_blocks, (cudaStream_t)stream));
}

int qmoe_synth_f32(uint64_t seed, uint64_t stream_id, int64_t n_values, float std_dev, float* out,
                   void* stream) {
    if (n_values < 0) return QMOE_ERR_INVALID_ARG;
    if (n_values == 0) return QMOE_OK;
    if (!out) return QMOE_ERR_INVALID_ARG;
    return cuda_status(launch_synth_f32(seed, stream_id, n_values, std_dev, out, (cudaStream_t)stream));
}

int qmoe_route(const void* x, int x_dtype, int n_tokens, const qmoe_layer_weights* w,
               const qmoe_dims* dims, int32_t* ids, float* weights, float* shared_logit,
               void* workspace, size_t workspace_bytes, void* stream) {
    QMOE_TRY(check_dims(dims));
    QMOE_TRY(check_tokens(n_tokens));
    QMOE_TRY(check_act(x, x_dtype));
    QMOE_TRY(check_weights_route(w));
    QMOE_TRY(route_smem_ok(n_tokens, dims->hidden));
    if (!ids || !weights) return QMOE_ERR_INVALID_ARG;
    Ws ws;
    QMOE_TRY(get_ws(workspace, workspace_bytes, dims, n_tokens, &ws));
    return run_route(x, x_dtype, n_tokens, w, dims, ids, weights, shared_logit, ws, (cudaStream_t)stream);
}

int qmoe_route_threshold(const void* x, int x_dtype, int n_tokens, const qmoe_layer_weights* w,
                         const qmoe_dims* dims, int top_k, int probs_bf16, int32_t* ids, float* weights,
                         float* shared_logit, void* workspace, size_t workspace_bytes, void* stream) {
    QMOE_TRY(check_dims(dims));
    QMOE_TRY(check_tokens(n_tokens));
    QMOE_TRY(check_act(x, x_dtype));
    QMOE_TRY(check_weights_route(w));
    QMOE_TRY(route_smem_ok(n_tokens, dims->hidden));
    if (!ids || !weights) return QMOE_ERR_INVALID_ARG;
    if (top_k < 1 || top_k > kMaxTopK || (probs_bf16 != 0 && probs_bf16 != 1)) return QMOE_ERR_INVALID_ARG;
    Ws ws;
    QMOE_TRY(get_ws(workspace, workspace_bytes, dims, n_tokens, &ws));
    return run_route(x, x_dtype, n_tokens, w, dims, ids, weights, shared_logit, ws, (cudaStream_t)stream,
                     probs_bf16 ? 2 : 1, top_k);
}

int qmoe_gateup_swiglu(const void* x, int x_dtype, int n_tokens, const int32_t* ids,
                       const qmoe_layer_weights* w, const qmoe_dims* dims, float* h, int h_stride,
                       void* workspace, size_t workspace_bytes, void* stream) {
    QMOE_TRY(check_dims(dims));
    QMOE_TRY(check_tokens(n_tokens));
    QMOE_TRY(check_act(x, x_dtype));
    QMOE_TRY(check_weights_experts(w, dims));
    if (!ids || !h) return QMOE_ERR_INVALID_ARG;
    if (h_stride < dims->inter_local || h_stride < dims->sh_inter_local) return QMOE_ERR_INVALID_ARG;
    Ws ws;
    QMOE_TRY(get_ws(workspace, workspace_bytes, dims, n_tokens, &ws));
    ExpertArgs a = expert_args(x, x_dtype, n_tokens, ids, nullptr, nullptr, w, dims, h, h_stride,
                               nullptr, ws.status());
    QMOE_TRY(check_smem(a));
    return cuda_status(launch_gateup(a, (cudaStream_t)stream));
}

int qmoe_down_combine(const float* h, int h_stride, int n_tokens, const int32_t* ids,
                      const float* weights, const float* shared_logit, const qmoe_layer_weights* w,
                      const qmoe_dims* dims, float* out, void* workspace, size_t workspace_bytes,
                      void* stream) {
    QMOE_TRY(check_dims(dims));
    QMOE_TRY(check_tokens(n_tokens));
    QMOE_TRY(check_weights_experts(w, dims));
    if (!h || !ids || !weights || !out) return QMOE_ERR_INVALID_ARG;
    if (h_stride < dims->inter_local || h_stride < dims->sh_inter_local) return QMOE_ERR_INVALID_ARG;
    if (!aligned(h, 16) || h_stride % 4) return QMOE_ERR_ALIGNMENT;
    Ws ws;
    QMOE_TRY(get_ws(workspace, workspace_bytes, dims, n_tokens, &ws));
    ExpertArgs a = expert_args(nullptr, QMOE_ACT_F32, n_tokens, ids, weights, shared_logit, w, dims,
                               (float*)h, h_stride, out, ws.status());
    a.hconv = ws.h();  // the caller's h stays as given
    a.hconv_stride = ws.L.h_stride;
    QMOE_TRY(check_smem(a));
    return cuda_status(launch_down(a, (cudaStream_t)stream));
}

int qmoe_moe_block(const void* x, int x_dtype, int n_tokens, const qmoe_layer_weights* w,
                   const qmoe_dims* dims, float* out, void* workspace, size_t workspace_bytes,
                   void* stream) {
    QMOE_TRY(check_dims(dims));
    QMOE_TRY(check_tokens(n_tokens));
    QMOE_TRY(check_act(x, x_dtype));
    QMOE_TRY(check_weights_route(w));
    QMOE_TRY(check_weights_experts(w, dims));
    QMOE_TRY(route_smem_ok(n_tokens, dims->hidden));
    if (!out) return QMOE_ERR_INVALID_ARG;
    // out may alias an fp32 x: the router and gate|up launches finish reading
    // x before the down launch writes out (stream order).
    Ws ws;
    QMOE_TRY(get_ws(workspace, workspace_bytes, dims, n_tokens, &ws));
    ExpertArgs probe = expert_args(x, x_dtype, n_tokens, nullptr, nullptr, nullptr, w, dims, ws.h(),
                                   ws.L.h_stride, out, nullptr);
    QMOE_TRY(check_smem(probe));
    return run_block(x, x_dtype, n_tokens, w, dims, out, ws, (cudaStream_t)stream);
}

int qmoe_shared_expert(const void* x, int x_dtype, int n_tokens, const qmoe_layer_weights* w,
                       const qmoe_dims* dims, float* out, void* workspace, size_t workspace_bytes,
                       void* stream) {
    QMOE_TRY(check_dims(dims));
    QMOE_TRY(check_tokens(n_tokens));
    QMOE_TRY(check_act(x, x_dtype));
    if (!w || !w->gate_vec || !w->sh_gate_up || !w->sh_down || !out) return QMOE_ERR_INVALID_ARG;
    if (dims->sh_inter_local <= 0) return QMOE_ERR_INVALID_ARG;
    if (!aligned(w->gate_vec, 16) || !aligned(w->sh_gate_up, 8) || !aligned(w->sh_down, 8))
        return QMOE_ERR_ALIGNMENT;
    QMOE_TRY(route_smem_ok(n_tokens, dims->hidden));
    Ws ws;
    QMOE_TRY(get_ws(workspace, workspace_bytes, dims, n_tokens, &ws));
    qmoe_dims d = *dims;  // no routed experts: an empty window
    d.expert_lo = d.expert_hi = 0;
    qmoe_layer_weights sw = *w;
    sw.gate_up = sw.down = nullptr;
    cudaStream_t s = (cudaStream_t)stream;
    RouteArgs r{};
    r.x = x;
    r.x_f32 = x_dtype == QMOE_ACT_F32;
    r.M = n_tokens;
    r.D = d.hidden;
    r.E = 0;  // the gate-vector row alone
    r.k = d.top_k;
    r.gate_vec = w->gate_vec;
    r.logits = ws.logits();
    r.counter = ws.counter();
    r.shared_logit = ws.shared();
    r.status = ws.status();
    QMOE_TRY(cuda_status(launch_route(r, s)));
    // Any in-range ids will do: none falls in the empty window.
    QMOE_TRY(cuda_status(cudaMemsetAsync(ws.ids(), 0, (size_t)n_tokens * d.top_k * 4, s)));
    ExpertArgs a = expert_args(x, x_dtype, n_tokens, ws.ids(), ws.weights(), ws.shared(), &sw, &d,
                               ws.h(), ws.L.h_stride, out, ws.status());
    QMOE_TRY(check_smem(a));
    QMOE_TRY(cuda_status(launch_gateup(a, s)));
    return cuda_status(launch_down(a, s));
}

int qmoe_read_stack_trace(void* workspace, const qmoe_dims* dims, int n_tokens, int n_layers,
                          uint64_t* host_out, void* stream) {
    QMOE_TRY(check_dims(dims));
    if (!workspace || !host_out || n_layers < 1 || n_layers > 64) return QMOE_ERR_INVALID_ARG;
    const WsLayout L = ws_layout(*dims, n_tokens);
    cudaStream_t s = (cudaStream_t)stream;
#if defined(QMOE_SK_FULLTRACE)
    QMOE_TRY(cuda_status(cudaMemcpyAsync(host_out, (unsigned char*)workspace + L.trace,
                                         (size_t)n_layers * kFullTraceCtas * kTraceSlots * 8, cudaMemcpyDeviceToHost,
                                         s)));
    return cuda_status(cudaStreamSynchronize(s));
#endif
    const size_t rows = (size_t)n_layers * kTraceSlots * sizeof(uint64_t);
    QMOE_TRY(cuda_status(cudaMemcpyAsync(host_out, (unsigned char*)workspace + L.trace, rows,
                                         cudaMemcpyDeviceToHost, s)));
    QMOE_TRY(cuda_status(cudaMemcpyAsync(host_out + (size_t)n_layers * kTraceSlots,
                                         (unsigned char*)workspace + L.trace + 64 * kTraceSlots * sizeof(uint64_t),
                                         rows, cudaMemcpyDeviceToHost, s)));
    return cuda_status(cudaStreamSynchronize(s));
}

int qmoe_stack_single_launch(const qmoe_dims* dims, int n_tokens, int n_layers) {
    if (check_dims(dims) != QMOE_OK) return 0;
    return stack_kernel_supported(*dims, n_tokens, n_layers, 1) ? 1 : 0;
}

int qmoe_stack_decode(const void* x, int n_tokens, const qmoe_layer_weights* layers, int n_layers,
                      const qmoe_dims* dims, float* out, void* workspace, size_t workspace_bytes,
                      void* stream) {
    QMOE_TRY(check_dims(dims));
    QMOE_TRY(check_tokens(n_tokens));
    QMOE_TRY(check_act(x, QMOE_ACT_BF16));
    if (!layers || n_layers < 1 || !out) return QMOE_ERR_INVALID_ARG;
    QMOE_TRY(route_smem_ok(n_tokens, dims->hidden));
    for (int l = 0; l < n_layers; ++l) {
        QMOE_TRY(check_weights_route(&layers[l]));
        QMOE_TRY(check_weights_experts(&layers[l], dims));
    }
    Ws ws;
    QMOE_TRY(get_ws(workspace, workspace_bytes, dims, n_tokens, &ws));
    ExpertArgs probe = expert_args(x, QMOE_ACT_BF16, n_tokens, nullptr, nullptr, nullptr, &layers[0],
                                   dims, ws.h(), ws.L.h_stride, out, nullptr);
    QMOE_TRY(check_smem(probe));
    cudaStream_t s = (cudaStream_t)stream;
    // One token, BASELINE-family shapes, unsharded, every operand 16-byte
    // aligned: the whole stack is one persistent launch.
    bool aligned16 = aligned(x, 16) && aligned(out, 16);
    for (int l = 0; l < n_layers && aligned16; ++l) {
        const qmoe_layer_weights& w = layers[l];
        aligned16 = w.gate_vec && w.sh_gate_up && w.sh_down && aligned(w.router, 16) && aligned(w.gate_vec, 16) &&
                    aligned(w.gate_up, 16) && aligned(w.down, 16) && aligned(w.sh_gate_up, 16) &&
                    aligned(w.sh_down, 16);
    }
    if (aligned16 && stack_kernel_supported(*dims, n_tokens, n_layers, 1))
        return cuda_status(launch_stack_kernel(x, out, (unsigned char*)ws.sync(), ws.trace(), ws.status(), layers,
                                               n_layers, *dims, nullptr, ws.trace_bufs(dims->top_k), s));
    // Otherwise three launches per layer. Layer L+1 reads `out` (layer L's result) in its router and gate|up
    // launches; its down launch overwrites `out` only after both, in stream
    // order, so one buffer carries the activation through the stack.
    for (int l = 0; l < n_layers; ++l) {
        const void* in = l == 0 ? x : (const void*)out;
        const int dt = l == 0 ? QMOE_ACT_BF16 : QMOE_ACT_F32;
        QMOE_TRY(run_block(in, dt, n_tokens, &layers[l], dims, out, ws, s));
    }
    return QMOE_OK;
}

int qmoe_stack_decode_teacher(const void* x_layers, const qmoe_layer_weights* layers, int n_layers,
                              const qmoe_dims* dims, float* out, void* workspace, size_t workspace_bytes,
                              void* stream) {
    QMOE_TRY(check_dims(dims));
    QMOE_TRY(check_act(x_layers, QMOE_ACT_BF16));
    if (!layers || n_layers < 1 || !out) return QMOE_ERR_INVALID_ARG;
    if (!aligned(x_layers, 16) || !aligned(out, 16)) return QMOE_ERR_ALIGNMENT;
    for (int l = 0; l < n_layers; ++l) {
        const qmoe_layer_weights& w = layers[l];
        QMOE_TRY(check_weights_route(&w));
        QMOE_TRY(check_weights_experts(&w, dims));
        if (!w.gate_vec || !w.sh_gate_up || !w.sh_down) return QMOE_ERR_UNSUPPORTED;
        if (!aligned(w.gate_up, 16) || !aligned(w.down, 16) || !aligned(w.sh_gate_up, 16) || !aligned(w.sh_down, 16))
            return QMOE_ERR_ALIGNMENT;
    }
    if (!stack_kernel_supported(*dims, 1, n_layers, 1)) return QMOE_ERR_UNSUPPORTED;
    Ws ws;
    QMOE_TRY(get_ws(workspace, workspace_bytes, dims, 1, &ws));
    return cuda_status(launch_stack_kernel(x_layers, out, (unsigned char*)ws.sync(), ws.trace(), ws.status(),
                                           layers, n_layers, *dims, nullptr, ws.trace_bufs(dims->top_k, x_layers),
                                           (cudaStream_t)stream));
}

int qmoe_read_stack_route_trace(void* workspace, const qmoe_dims* dims, int n_tokens, int n_layers,
                                uint16_t* act_out, int32_t* ids_out, float* weights_out, void* stream) {
    QMOE_TRY(check_dims(dims));
    if (!workspace || n_layers < 1 || n_layers > 64) return QMOE_ERR_INVALID_ARG;
    QMOE_TRY(check_tokens(n_tokens));
    Ws ws;
    ws.L = ws_layout(*dims, n_tokens);
    ws.base = (unsigned char*)workspace;
    const StackTraceBufs t = ws.trace_bufs(dims->top_k);
    cudaStream_t s = (cudaStream_t)stream;
    if (act_out)
        QMOE_TRY(cuda_status(cudaMemcpyAsync(act_out, t.act, (size_t)n_layers * dims->hidden * 2,
                                             cudaMemcpyDeviceToHost, s)));
    if (ids_out)
        QMOE_TRY(cuda_status(cudaMemcpyAsync(ids_out, t.ids, (size_t)n_layers * dims->top_k * 4,
                                             cudaMemcpyDeviceToHost, s)));
    if (weights_out)
        QMOE_TRY(cuda_status(cudaMemcpyAsync(weights_out, t.weights, (size_t)n_layers * dims->top_k * 4,
                                             cudaMemcpyDeviceToHost, s)));
    return cuda_status(cudaStreamSynchronize(s));
}

// ---- the stack sharded over ranks, exchange inside the kernel ----------------

static int check_stack_operands(const void* x, int n_tokens, const qmoe_layer_weights* layers, int n_layers,
                                const qmoe_dims* dims, const float* out) {
    QMOE_TRY(check_dims(dims));
    QMOE_TRY(check_tokens(n_tokens));
    QMOE_TRY(check_act(x, QMOE_ACT_BF16));
    if (!layers || n_layers < 1 || !out) return QMOE_ERR_INVALID_ARG;
    for (int l = 0; l < n_layers; ++l) {
        QMOE_TRY(check_weights_route(&layers[l]));
        QMOE_TRY(check_weights_experts(&layers[l], dims));
    }
    return QMOE_OK;
}

size_t qmoe_xchg_bytes(int n_ranks, int hidden) {
    if (n_ranks < 1 || n_ranks > kMaxXchgRanks || hidden < 1 || hidden > kMaxHidden) return 0;
    return xchg_bytes(n_ranks, hidden);
}

int qmoe_xchg_alloc(int n_ranks, int hidden, void** buf, void* ipc_handle) {
    if (!buf || !ipc_handle) return QMOE_ERR_INVALID_ARG;
    const size_t bytes = qmoe_xchg_bytes(n_ranks, hidden);
    if (!bytes) return QMOE_ERR_UNSUPPORTED;
    void* p = nullptr;
    QMOE_TRY(cuda_status(cudaMalloc(&p, bytes)));
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaMemset(p, 0, bytes);
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        return cuda_status(e);
    }
    static_assert(sizeof(h) == QMOE_XCHG_HANDLE_BYTES, "CUDA IPC handle size");
    memcpy(ipc_handle, &h, sizeof(h));
    *buf = p;
    return QMOE_OK;
}

int qmoe_xchg_open(const void* ipc_handle, void** peer_buf) {
    if (!ipc_handle || !peer_buf) return QMOE_ERR_INVALID_ARG;
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof(h));
    return cuda_status(cudaIpcOpenMemHandle(peer_buf, h, cudaIpcMemLazyEnablePeerAccess));
}

int qmoe_xchg_close(void* peer_buf) {
    if (!peer_buf) return QMOE_ERR_INVALID_ARG;
    return cuda_status(cudaIpcCloseMemHandle(peer_buf));
}

int qmoe_xchg_free(void* buf) {
    if (!buf) return QMOE_ERR_INVALID_ARG;
    return cuda_status(cudaFree(buf));
}

int qmoe_xchg_reset(void* buf, int n_ranks, int hidden, void* stream) {
    if (!buf) return QMOE_ERR_INVALID_ARG;
    const size_t bytes = qmoe_xchg_bytes(n_ranks, hidden);
    if (!bytes) return QMOE_ERR_UNSUPPORTED;
    return cuda_status(cudaMemsetAsync(buf, 0, bytes, (cudaStream_t)stream));
}

int qmoe_stack_xchg_supported(const qmoe_dims* dims, int n_ranks, int n_tokens, int n_layers) {
    if (check_dims(dims) != QMOE_OK || n_ranks < 2 || n_ranks > kMaxXchgRanks) return 0;
    return stack_kernel_supported(*dims, n_tokens, n_layers, n_ranks) ? 1 : 0;
}

int qmoe_stack_decode_xchg(const void* x, int n_tokens, const qmoe_layer_weights* layers, int n_layers,
                           const qmoe_dims* dims, const qmoe_xchg* xc, float* out, void* workspace,
                           size_t workspace_bytes, void* stream) {
    QMOE_TRY(check_stack_operands(x, n_tokens, layers, n_layers, dims, out));
    if (!xc || xc->n_ranks < 2 || xc->n_ranks > kMaxXchgRanks || xc->rank < 0 || xc->rank >= xc->n_ranks)
        return QMOE_ERR_INVALID_ARG;
    XchgDesc desc{};
    desc.R = xc->n_ranks;
    desc.rank = xc->rank;
    for (int q = 0; q < xc->n_ranks; ++q) {
        if (!xc->buf[q]) return QMOE_ERR_INVALID_ARG;
        if (!aligned(xc->buf[q], 256)) return QMOE_ERR_ALIGNMENT;
        desc.buf[q] = (unsigned char*)xc->buf[q];
    }
    if (!aligned(x, 16) || !aligned(out, 16)) return QMOE_ERR_ALIGNMENT;
    for (int l = 0; l < n_layers; ++l) {
        const qmoe_layer_weights& w = layers[l];
        if (!w.gate_vec || !w.sh_gate_up || !w.sh_down) return QMOE_ERR_INVALID_ARG;
        if (!aligned(w.router, 16) || !aligned(w.gate_vec, 16) || !aligned(w.gate_up, 16) || !aligned(w.down, 16) ||
            !aligned(w.sh_gate_up, 16) || !aligned(w.sh_down, 16))
            return QMOE_ERR_ALIGNMENT;
    }
    if (!stack_kernel_supported(*dims, n_tokens, n_layers, xc->n_ranks)) return QMOE_ERR_UNSUPPORTED;
    Ws ws;
    QMOE_TRY(get_ws(workspace, workspace_bytes, dims, n_tokens, &ws));
    return cuda_status(launch_stack_kernel(x, out, (unsigned char*)ws.sync(), ws.trace(), ws.status(), layers,
                                           n_layers, *dims, &desc, ws.trace_bufs(dims->top_k), (cudaStream_t)stream));
}

// ---- prefill / large verify chunks ------------------------------------------

static int check_prefill(const qmoe_dims* dims, int n_tokens) {
    QMOE_TRY(check_dims(dims));
    if (!prefill_supported(*dims)) return QMOE_ERR_UNSUPPORTED;
    if (n_tokens < 1 || n_tokens > prefill_max_tokens()) return QMOE_ERR_UNSUPPORTED;
    // the grouping pass holds every routed id of the chunk in shared memory as int16
    if ((size_t)n_tokens * dims->top_k * 2 > 200 * 1024) return QMOE_ERR_UNSUPPORTED;
    return QMOE_OK;
}

static int check_prefill_experts_weights(const qmoe_layer_weights* w, const qmoe_dims* d) {
    if (!w || !w->gate_up || !w->down) return QMOE_ERR_INVALID_ARG;
    if (!aligned(w->gate_up, 16) || !aligned(w->down, 16)) return QMOE_ERR_ALIGNMENT;
    if (d->sh_inter_local > 0) {
        if (!w->sh_gate_up || !w->sh_down) return QMOE_ERR_INVALID_ARG;
        if (!aligned(w->sh_gate_up, 16) || !aligned(w->sh_down, 16)) return QMOE_ERR_ALIGNMENT;
    }
    return QMOE_OK;
}

static int get_prefill_ws(void* workspace, size_t bytes, const qmoe_dims* d, int T) {
    if (!workspace) return QMOE_ERR_WORKSPACE;
    if (!aligned(workspace, 256)) return QMOE_ERR_ALIGNMENT;
    if (bytes < prefill_workspace_bytes(*d, T)) return QMOE_ERR_WORKSPACE;
    return QMOE_OK;
}

namespace {
int check_hc(const qmoe_hc_dims* d, int M) {
    if (!d) return QMOE_ERR_INVALID_ARG;
    if (d->hidden < 32 || d->hidden % 32 || d->hc < 1 || d->hc > 16 || d->rank < 1 || d->rank > 4096 ||
        !(d->eps >= 0.0f))
        return QMOE_ERR_INVALID_ARG;
    if (M < 1 || M > 1024) return QMOE_ERR_INVALID_ARG;
    if (hc_down_smem(1, d->hc, d->hidden) > kSmemLimit || hc_up_smem(M, d->rank) > kSmemLimit)
        return QMOE_ERR_UNSUPPORTED;
    return QMOE_OK;
}
}  // namespace

size_t qmoe_hc_workspace_bytes(const qmoe_hc_dims* dims, int n_tokens) {
    if (check_hc(dims, n_tokens) != QMOE_OK) return 0;
    return hc_workspace_bytes(n_tokens, dims->hc, dims->rank);
}

int qmoe_hc_mix(const void* hyper, int hyper_dtype, int n_tokens, const qmoe_hc_weights* w,
                const qmoe_hc_dims* dims, float* mixed, float* inject, void* workspace,
                size_t workspace_bytes, void* stream) {
    QMOE_TRY(check_hc(dims, n_tokens));
    QMOE_TRY(check_act(hyper, hyper_dtype));
    if (!w || !w->norm_w || !w->down_w || !w->up_w || !w->inject_w || !mixed || !inject)
        return QMOE_ERR_INVALID_ARG;
    if (!aligned(w->norm_w, 16) || !aligned(w->down_w, 16) || !aligned(w->up_w, 16) ||
        !aligned(w->inject_w, 16))
        return QMOE_ERR_ALIGNMENT;
    if (!workspace) return QMOE_ERR_WORKSPACE;
    if (!aligned(workspace, 256)) return QMOE_ERR_ALIGNMENT;
    if (workspace_bytes < hc_workspace_bytes(n_tokens, dims->hc, dims->rank)) return QMOE_ERR_WORKSPACE;
    return cuda_status(launch_hc_mix(hyper, hyper_dtype == QMOE_ACT_F32, n_tokens, dims->hidden, dims->hc,
                                     dims->rank, dims->eps, w->norm_w, w->down_w, w->up_w, w->inject_w, mixed,
                                     inject, (unsigned char*)workspace, (cudaStream_t)stream));
}

int qmoe_hc_reinject(const void* hyper, int hyper_dtype, const void* branch, int branch_dtype,
                     const float* inject, int n_tokens, const qmoe_hc_dims* dims, float* out, void* stream) {
    QMOE_TRY(check_hc(dims, n_tokens));
    QMOE_TRY(check_act(hyper, hyper_dtype));
    QMOE_TRY(check_act(branch, branch_dtype));
    if (!inject || !out) return QMOE_ERR_INVALID_ARG;
    if (out == hyper && hyper_dtype != QMOE_ACT_F32) return QMOE_ERR_INVALID_ARG;
    return cuda_status(launch_hc_reinject(hyper, hyper_dtype == QMOE_ACT_F32, branch, branch_dtype == QMOE_ACT_F32,
                                          inject, n_tokens, dims->hidden, dims->hc, out, (cudaStream_t)stream));
}

size_t qmoe_format_row_bytes(int format, int64_t n_values) {
    return n_values > 0 ? fmt_row_bytes(format, n_values) : 0;
}

int qmoe_dequant_f32(int format, const void* blocks, int64_t n_values, float* out, void* stream) {
    if (!blocks || !out || n_values < 0 || (n_values > 0 && fmt_row_bytes(format, n_values) == 0))
        return QMOE_ERR_INVALID_ARG;
    if (!aligned(blocks, 16) || !aligned(out, 16)) return QMOE_ERR_ALIGNMENT;
    if (n_values == 0) return QMOE_OK;
    return cuda_status(launch_fmt_dequant(format, (const uint8_t*)blocks, n_values, out, (cudaStream_t)stream));
}

int qmoe_moe_block_formats(const void* x, int x_dtype, int n_tokens, const qmoe_layer_weights* w,
                           const qmoe_dims* dims, const qmoe_formats* f, float* out, void* workspace,
                           size_t workspace_bytes, void* stream) {
    QMOE_TRY(check_dims(dims));
    QMOE_TRY(check_tokens(n_tokens));
    QMOE_TRY(check_act(x, x_dtype));
    QMOE_TRY(check_weights_route(w));
    QMOE_TRY(route_smem_ok(n_tokens, dims->hidden));
    if (!f || !out || !w->gate_up || !w->down) return QMOE_ERR_INVALID_ARG;
    if (dims->expert_lo != 0 || dims->expert_hi != dims->n_experts || dims->inter_local != dims->inter)
        return QMOE_ERR_UNSUPPORTED;
    const bool sh = dims->sh_inter_local > 0;
    if (fmt_row_bytes(f->gate_up, dims->hidden) == 0 || fmt_row_bytes(f->down, dims->inter) == 0 ||
        (sh && (fmt_row_bytes(f->sh_gate_up, dims->hidden) == 0 ||
                fmt_row_bytes(f->sh_down, dims->sh_inter_local) == 0 || !w->sh_gate_up || !w->sh_down)))
        return QMOE_ERR_INVALID_ARG;
    if (dims->inter % 32 || (sh && dims->sh_inter_local % 32)) return QMOE_ERR_UNSUPPORTED;
    if (!aligned(w->gate_up, 16) || !aligned(w->down, 16) || (sh && (!aligned(w->sh_gate_up, 16) ||
                                                                     !aligned(w->sh_down, 16))))
        return QMOE_ERR_ALIGNMENT;
    Ws ws;
    QMOE_TRY(get_ws(workspace, workspace_bytes, dims, n_tokens, &ws));
    cudaStream_t s = (cudaStream_t)stream;
    int* xconv = (int*)ws.act();
    QMOE_TRY(run_route(x, x_dtype, n_tokens, w, dims, ws.ids(), ws.weights(), ws.shared(), ws, s, 0, 0, xconv));
    return cuda_status(launch_fmt_experts(x, x_dtype == QMOE_ACT_F32, n_tokens, *dims, *f, *w, ws.ids(),
                                          ws.weights(), ws.shared(), ws.h(), ws.L.h_stride, xconv, out,
                                          ws.status(), s));
}

int qmoe_prefill_max_tokens(void) { return prefill_max_tokens(); }
int qmoe_prefill_small_group_max(int n) { return prefill_small_group_max(n); }
int qmoe_prefill_trace(int enable) { return prefill_trace(enable); }

size_t qmoe_prefill_workspace_bytes(const qmoe_dims* dims, int n_tokens) {
    if (check_dims(dims) != QMOE_OK || n_tokens < 1 || n_tokens > prefill_max_tokens()) return 0;
    return prefill_workspace_bytes(*dims, n_tokens);
}

namespace {
int prefill_route_impl(const void* x, int x_dtype, int n_tokens, const qmoe_layer_weights* w,
                       const qmoe_dims* dims, int32_t* ids, float* weights, float* shared_logit,
                       void* workspace, size_t workspace_bytes, void* stream, int thr_mode, int thr_k) {
    // Routing alone needs only valid dims and a chunk size the workspace covers.
    QMOE_TRY(check_dims(dims));
    if (n_tokens < 1 || n_tokens > prefill_max_tokens()) return QMOE_ERR_UNSUPPORTED;
    QMOE_TRY(check_act(x, x_dtype));
    QMOE_TRY(check_weights_route(w));
    if (!ids || !weights) return QMOE_ERR_INVALID_ARG;
    QMOE_TRY(get_prefill_ws(workspace, workspace_bytes, dims, n_tokens));
    cudaStream_t s = (cudaStream_t)stream;
    unsigned char* ws = (unsigned char*)workspace;
    const bool x_ok = x_dtype == QMOE_ACT_BF16 && aligned(x, 16);
    const __nv_bfloat16* xb = prefill_act_bf16(x, x_dtype == QMOE_ACT_F32, x_ok, n_tokens, *dims, ws, s);
    return cuda_status(
        launch_prefill_route(xb, n_tokens, *w, *dims, ws, ids, weights, shared_logit, s, thr_mode, thr_k));
}
}  // namespace

int qmoe_prefill_route(const void* x, int x_dtype, int n_tokens, const qmoe_layer_weights* w,
                       const qmoe_dims* dims, int32_t* ids, float* weights, float* shared_logit,
                       void* workspace, size_t workspace_bytes, void* stream) {
    return prefill_route_impl(x, x_dtype, n_tokens, w, dims, ids, weights, shared_logit, workspace,
                              workspace_bytes, stream, 0, 0);
}

int qmoe_prefill_route_threshold(const void* x, int x_dtype, int n_tokens, const qmoe_layer_weights* w,
                                 const qmoe_dims* dims, int top_k, int probs_bf16, int32_t* ids, float* weights,
                                 float* shared_logit, void* workspace, size_t workspace_bytes, void* stream) {
    if (top_k < 1 || top_k > kMaxTopK || (probs_bf16 != 0 && probs_bf16 != 1)) return QMOE_ERR_INVALID_ARG;
    if (dims && (dims->expert_lo != 0 || dims->expert_hi != dims->n_experts)) return QMOE_ERR_UNSUPPORTED;
    return prefill_route_impl(x, x_dtype, n_tokens, w, dims, ids, weights, shared_logit, workspace,
                              workspace_bytes, stream, probs_bf16 ? 2 : 1, top_k);
}

int qmoe_prefill_experts(const void* x, int x_dtype, int n_tokens, const int32_t* ids, const float* weights,
                         const float* shared_logit, const qmoe_layer_weights* w, const qmoe_dims* dims, float* out,
                         void* workspace, size_t workspace_bytes, void* stream) {
    QMOE_TRY(check_prefill(dims, n_tokens));
    QMOE_TRY(check_act(x, x_dtype));
    QMOE_TRY(check_prefill_experts_weights(w, dims));
    if (!ids || !weights || !out) return QMOE_ERR_INVALID_ARG;
    if (dims->sh_inter_local > 0 && !shared_logit) return QMOE_ERR_INVALID_ARG;
    QMOE_TRY(get_prefill_ws(workspace, workspace_bytes, dims, n_tokens));
    cudaStream_t s = (cudaStream_t)stream;
    unsigned char* ws = (unsigned char*)workspace;
    const bool x_ok = x_dtype == QMOE_ACT_BF16 && aligned(x, 16);
    // out may alias an fp32 x: x is read (converted to bf16) before out is cleared.
    const __nv_bfloat16* xb = prefill_act_bf16(x, x_dtype == QMOE_ACT_F32, x_ok, n_tokens, *dims, ws, s);
    return cuda_status(launch_prefill_experts(xb, n_tokens, ids, weights, shared_logit, *w, *dims, out, ws, s));
}

int qmoe_prefill(const void* x, int x_dtype, int n_tokens, const qmoe_layer_weights* w, const qmoe_dims* dims,
                 float* out, void* workspace, size_t workspace_bytes, void* stream) {
    QMOE_TRY(check_prefill(dims, n_tokens));
    QMOE_TRY(check_act(x, x_dtype));
    QMOE_TRY(check_weights_route(w));
    QMOE_TRY(check_prefill_experts_weights(w, dims));
    if (!out) return QMOE_ERR_INVALID_ARG;
    QMOE_TRY(get_prefill_ws(workspace, workspace_bytes, dims, n_tokens));
    cudaStream_t s = (cudaStream_t)stream;
    unsigned char* ws = (unsigned char*)workspace;
    const bool x_ok = x_dtype == QMOE_ACT_BF16 && aligned(x, 16);
    const __nv_bfloat16* xb = prefill_act_bf16(x, x_dtype == QMOE_ACT_F32, x_ok, n_tokens, *dims, ws, s);
    int32_t* ids;
    float* wts;
    float* slog;
    prefill_route_buffers(*dims, n_tokens, ws, &ids, &wts, &slog);
    QMOE_TRY(cuda_status(launch_prefill_route(xb, n_tokens, *w, *dims, ws, ids, wts, slog, s)));
    // An fp32 x that aliases out is safe: fp32 input is always read through its bf16 copy, made
    // before out is cleared.
    return cuda_status(launch_prefill_experts(xb, n_tokens, ids, wts, slog, *w, *dims, out, ws, s));
}

}  // extern "C"
