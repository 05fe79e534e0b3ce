// qmoe_moe_block_noalloc: the MoE block with no workspace argument and no
// allocation of any kind.
//
// Who needs it: callers that cannot hand the library device memory.  Examples
// are a host engine bound through cgo / JNI / N-API that has no device
// allocator of its own, a plug-in loaded into a process whose device memory
// belongs to another framework's caching allocator, or a real-time serving
// loop whose rules forbid allocation after start-up.  Such callers pass only
// their inputs and outputs; the block's scratch (router logits, the routing
// table, the SwiGLU activations, the status and arrival words) lives in the
// file-scope array below, which the loader places in device memory when the
// library's module loads on a device.
//
// Limits and sharing:
//   * The array holds QMOE_NOALLOC_SCRATCH_BYTES (1 MiB, include/qmoe_b200.h)
//     on every GPU that loads the library, for the life of the process.  A
//     call whose scratch (qmoe_workspace_bytes(dims, n_tokens)) would exceed it
//     is rejected with QMOE_ERR_WORKSPACE before anything is launched.
//   * Every call on a device shares the one array and it keeps the last
//     call's contents, so two calls that overlap on the GPU (different
//     streams, or different host threads) race and corrupt each other;
//     callers must order them.  The router's arrival counter, which must
//     start at zero, is cleared (stream-ordered) at the start of every call.
//   * The first call on a device (of either entry point below) looks up the
//     array's device address (cudaGetSymbolAddress with that device current),
//     caches it and zeroes the status word once; make that first call before
//     any stream capture.
//   * Device-side status: the kernels record the first error they meet (a
//     non-finite router logit, QMOE_ERR_NOT_FINITE; a bounded wait that ran
//     out) in the array's status word, which keeps it across calls until
//     qmoe_noalloc_read_status copies it out and clears it.
#include <mutex>

#include "common.cuh"

static __device__ __align__(256) unsigned char g_qmoe_noalloc_scratch[QMOE_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_by_device[kMaxDevices] = {};

// The device address of g_qmoe_noalloc_scratch on the current device.  In
// host code the array's name is only a host-side stand-in, never a device
// pointer, so the address is looked up once per device and cached.
int scratch_on_current_device(void** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return QMOE_ERR_CUDA;
    if (dev < 0 || dev >= kMaxDevices) return QMOE_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_by_device[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_qmoe_noalloc_scratch) != cudaSuccess || !p) return QMOE_ERR_CUDA;
        // The status word (and the rest of the first 256 bytes) starts at zero.
        if (cudaMemset(p, 0, 256) != cudaSuccess) return QMOE_ERR_CUDA;
        g_scratch_by_device[dev] = p;
    }
    *out = g_scratch_by_device[dev];
    return QMOE_OK;
}

}  // namespace

extern "C" int qmoe_moe_block_noalloc(const void* x, int x_dtype, int n_tokens,
                                      const qmoe_layer_weights* w, const qmoe_dims* dims, float* out,
                                      void* stream) {
    const size_t need = qmoe_workspace_bytes(dims, n_tokens);
    if (need == 0) return dims ? QMOE_ERR_UNSUPPORTED : QMOE_ERR_INVALID_ARG;
    if (need > QMOE_NOALLOC_SCRATCH_BYTES) return QMOE_ERR_WORKSPACE;
    void* scratch = nullptr;
    const int rc = scratch_on_current_device(&scratch);
    if (rc != QMOE_OK) return rc;
    // The router's arrival counter (at byte 64, after the status word) starts
    // at zero for every call; the status word keeps errors until read.
    if (cudaMemsetAsync(static_cast<unsigned char*>(scratch) + 64, 0, 192, (cudaStream_t)stream) != cudaSuccess)
        return QMOE_ERR_CUDA;
    return qmoe_moe_block(x, x_dtype, n_tokens, w, dims, out, scratch, QMOE_NOALLOC_SCRATCH_BYTES, stream);
}

extern "C" int qmoe_noalloc_read_status(int* status_out, void* stream) {
    if (!status_out) return QMOE_ERR_INVALID_ARG;
    void* scratch = nullptr;
    const int rc = scratch_on_current_device(&scratch);
    if (rc != QMOE_OK) return rc;
    return qmoe_read_status(scratch, status_out, stream);
}
