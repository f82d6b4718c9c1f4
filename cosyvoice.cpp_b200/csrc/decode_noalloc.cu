// decode_noalloc.cu -- cvattn_decode for callers that cannot allocate device memory.
//
// Some callers of the decode path may not call cudaMalloc at all.  Examples:
// a ggml custom-op callback that runs inside ggml_backend_sched_graph_compute
// and is handed only its input and output tensors (ggml plans every buffer
// before the graph runs), and a real-time streaming worker that must not take
// the driver's allocation lock or risk the implicit device synchronization an
// allocation can cause.  cvattn_decode needs a workspace for its split-KV
// partials and per-sequence ticket counters; this entry point supplies that
// workspace from a fixed array in device memory instead.
//
// The scratch is a file-scope __device__ array of CVATTN_DECODE_NOALLOC_SCRATCH_BYTES
// (8 MiB).  Every GPU that loads the library holds its own copy until the
// process exits.  Requests whose workspace would exceed it are rejected with
// CVATTN_ERR_LENGTH before anything is launched.  All calls on a device share
// the one array, so calls whose kernels overlap on that GPU (several streams,
// several host threads) race on it; serialize them.  The array keeps the last
// call's partials; the ticket counters, which must start at zero, are cleared
// on the caller's stream at the start of every call.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/cvattn.h"
#include "internal.h"

namespace {

constexpr size_t kScratchBytes = CVATTN_DECODE_NOALLOC_SCRATCH_BYTES;

// Device-side scratch.  In host code this name is only a stand-in for the
// symbol: its device address comes from cudaGetSymbolAddress, per device.
static __device__ __align__(256) unsigned char g_decode_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_addr[kMaxDevices] = {};
std::mutex g_setup_mutex;

// Device address of the scratch on `dev`, looked up once per device with that
// device current (the caller's device is restored afterwards).
cudaError_t scratch_address(int dev, void** out) {
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch_addr[dev]) {
        int prev = -1;
        cudaError_t e = cudaGetDevice(&prev);
        if (e != cudaSuccess) return e;
        if (prev != dev && (e = cudaSetDevice(dev)) != cudaSuccess) return e;
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_decode_scratch);
        if (prev != dev) cudaSetDevice(prev);
        if (e != cudaSuccess) return e;
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return cudaSuccess;
}

}  // namespace

// The device of a context (capi.cpp).
int cvattn_context_device(const cvattn_context* ctx);

extern "C" cvattn_status cvattn_decode_noalloc(cvattn_context* ctx, void* stream, const cvattn_decode_params* p) {
    // the same argument checks as cvattn_decode, before the workspace size is asked,
    // so both entry points give the same status for the same bad parameters
    if (!ctx || !p || !p->q || !p->out || !p->kv_len) return CVATTN_ERR_INVALID_ARGUMENT;
    if (p->n_seq < 0 || p->max_kv_len < 0 || p->n_q_heads <= 0) return CVATTN_ERR_INVALID_ARGUMENT;
    if (p->n_seq == 0) return CVATTN_OK;
    const size_t need = cvattn_decode_workspace_size(p->k.type, p->v.type, p->n_seq, p->max_kv_len, p->n_q_heads,
                                                     p->k.n_heads, p->k.head_dim);
    if (need == 0) return CVATTN_ERR_UNSUPPORTED;
    if (need > kScratchBytes) return CVATTN_ERR_LENGTH;  // beyond the static scratch: nothing launched
    const int dev = cvattn_context_device(ctx);
    void* scratch = nullptr;
    cudaError_t e = scratch_address(dev, &scratch);
    if (e != cudaSuccess) return CVATTN_ERR_CUDA;
    // the per-sequence ticket counters lead the workspace (256-byte aligned block);
    // cleared with the context's device current
    int prev = -1;
    if (cudaGetDevice(&prev) != cudaSuccess) return CVATTN_ERR_CUDA;
    if (prev != dev && cudaSetDevice(dev) != cudaSuccess) return CVATTN_ERR_CUDA;
    const size_t counter_bytes = cvattn::decode_ticket_bytes(p->n_seq, p->k.n_heads);
    e = cudaMemsetAsync(scratch, 0, counter_bytes, reinterpret_cast<cudaStream_t>(stream));
    if (prev != dev) cudaSetDevice(prev);
    if (e != cudaSuccess) return CVATTN_ERR_CUDA;
    cvattn_decode_params q = *p;
    q.workspace = scratch;
    q.workspace_size = kScratchBytes;
    return cvattn_decode(ctx, stream, &q);
}
