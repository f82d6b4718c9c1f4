// capi.cpp -- the extern "C" boundary of libcvattn.so (declared in include/cvattn.h).
//
// Argument validation, the per-worker context (device status word), type
// negotiation, host<->device KV copies, the cvattn_kv_cache host object and
// the DiT step planner.  Kernels live in kv_append.cu, decode*.cu and
// flash_tc.cu; nothing here computes attention on the CPU.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <vector>

#include "../../include/cvattn.h"
#include "internal.h"

using namespace cvattn;

namespace {

// ggml_row_size for the KV types (host side).
int64_t type_row_bytes(int t, int64_t n) {
    switch (t) {
    case CVATTN_TYPE_F32: return n * 4;
    case CVATTN_TYPE_F16: return n * 2;
    case CVATTN_TYPE_Q4_0: return n / 32 * 18;
    case CVATTN_TYPE_Q4_1: return n / 32 * 20;
    case CVATTN_TYPE_Q5_0: return n / 32 * 22;
    case CVATTN_TYPE_Q5_1: return n / 32 * 24;
    case CVATTN_TYPE_Q8_0: return n / 32 * 34;
    default: return 0;
    }
}

bool known_type(int t) {
    return t == CVATTN_TYPE_F32 || t == CVATTN_TYPE_F16 || t == CVATTN_TYPE_Q4_0 || t == CVATTN_TYPE_Q4_1 ||
           t == CVATTN_TYPE_Q5_0 || t == CVATTN_TYPE_Q5_1 || t == CVATTN_TYPE_Q8_0;
}

int block_elems(int t) { return (t == CVATTN_TYPE_F32 || t == CVATTN_TYPE_F16) ? 1 : 32; }

cvattn_status from_cuda(cudaError_t e) {
    if (e == cudaSuccess) return CVATTN_OK;
    if (e == cudaErrorMemoryAllocation) return CVATTN_ERR_ALLOC;
    if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) return CVATTN_ERR_NO_DEVICE;
    return CVATTN_ERR_CUDA;
}

cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// A tensor description is usable when its type is known, its rows hold whole
// blocks, strides cover a row and the data pointer is set.
bool tensor_ok(const cvattn_tensor* t) {
    if (!t || !t->data || !known_type(t->type)) return false;
    if (t->n_heads <= 0 || t->head_dim <= 0 || t->ne1 <= 0 || t->ne2 <= 0) return false;
    const int64_t row_elems = (int64_t)t->n_heads * t->head_dim;
    if (row_elems % 32) return false;
    const int64_t rb = type_row_bytes(t->type, row_elems);
    if (t->nb1 < rb || (t->ne2 > 1 && t->nb2 < t->nb1 * t->ne1)) return false;
    if ((t->nb1 & 1) || (t->nb2 & 1) || (reinterpret_cast<uintptr_t>(t->data) & 1)) return false;
    return true;
}

// Makes `device` current for the lifetime of the guard and restores the
// caller's device afterwards, so a call made while another GPU is current
// still runs on the context's device.
class DeviceGuard {
public:
    explicit DeviceGuard(int device) {
        if (cudaGetDevice(&prev_) != cudaSuccess) {
            err_ = cudaErrorNoDevice;
            return;
        }
        if (prev_ != device) err_ = cudaSetDevice(device);
    }
    ~DeviceGuard() {
        int cur = -1;
        if (cudaGetDevice(&cur) == cudaSuccess && cur != prev_ && prev_ >= 0) cudaSetDevice(prev_);
    }
    cudaError_t error() const { return err_; }
    DeviceGuard(const DeviceGuard&) = delete;
    DeviceGuard& operator=(const DeviceGuard&) = delete;

private:
    int prev_ = -1;
    cudaError_t err_ = cudaSuccess;
};

}  // namespace

// ------------------------------------------------------------------ context

struct cvattn_context {
    int device;
    int* status;  // device word; 0 = clean
};

// The device of a context, for the entry points defined in other files.
int cvattn_context_device(const cvattn_context* ctx) { return ctx ? ctx->device : -1; }

extern "C" {

const char* cvattn_status_string(cvattn_status s) {
    switch (s) {
    case CVATTN_OK: return "ok";
    case CVATTN_ERR_INVALID_ARGUMENT: return "invalid argument";
    case CVATTN_ERR_UNSUPPORTED: return "unsupported type pair or head shape";
    case CVATTN_ERR_LENGTH: return "sequence longer than the KV cache";
    case CVATTN_ERR_ALLOC: return "device allocation failed";
    case CVATTN_ERR_CUDA: return "CUDA runtime error";
    case CVATTN_ERR_DEVICE: return "a kernel skipped a bad device-resident index";
    case CVATTN_ERR_NO_DEVICE: return "no CUDA device";
    case CVATTN_ERR_TIMEOUT: return "bounded in-kernel wait expired";
    }
    return "unknown status";
}

int32_t cvattn_status_to_ggml(cvattn_status s) {
    if (s == CVATTN_OK) return 0;          // GGML_STATUS_SUCCESS
    if (s == CVATTN_ERR_ALLOC) return -2;  // GGML_STATUS_ALLOC_FAILED
    return -1;                             // GGML_STATUS_FAILED
}

int32_t cvattn_abi_version(void) { return CVATTN_ABI_VERSION; }

size_t cvattn_abi_sizeof(int32_t which) {
    switch (which) {
    case 0: return sizeof(cvattn_tensor);
    case 1: return sizeof(cvattn_decode_params);
    case 2: return sizeof(cvattn_flash_params);
    case 3: return sizeof(cvattn_kv_cache_params);
    case 4: return sizeof(cvattn_dit_step);
    case 5: return sizeof(cvattn_rope_params);
    default: return 0;
    }
}

size_t cvattn_row_size(int32_t type, int64_t n) {
    if (!known_type(type) || n < 0 || n % block_elems(type)) return 0;
    return (size_t)type_row_bytes(type, n);
}

// ------------------------------------------------------- types / capability

// The flash kernel serves every query count; the decode kernel is a faster
// path for one query row that cvattn_kv_cache_attention picks when it applies.
int32_t cvattn_supports(int32_t k_type, int32_t v_type, int32_t head_dim, int32_t n_q_heads, int32_t n_kv_heads) {
    return flash_supported(k_type, v_type, head_dim, n_q_heads, n_kv_heads) ? 1 : 0;
}

// src/cosyvoice-loader.cpp:498-510
int32_t cvattn_kv_fallback_type(int32_t t) {
    switch (t) {
    case CVATTN_TYPE_Q4_0: return CVATTN_TYPE_Q4_1;
    case CVATTN_TYPE_Q4_1: return CVATTN_TYPE_Q5_0;
    case CVATTN_TYPE_Q5_0: return CVATTN_TYPE_Q5_1;
    case CVATTN_TYPE_Q5_1: return CVATTN_TYPE_Q8_0;
    case CVATTN_TYPE_Q8_0: return CVATTN_TYPE_F16;
    case CVATTN_TYPE_F16: return CVATTN_TYPE_F32;
    default: return -1;
    }
}

// include/cosyvoice.h:32-42 enum order: F32, F16, Q8_0, Q5_1, Q5_0, Q4_1, Q4_0.
int32_t cvattn_kv_cache_type_to_ggml(int32_t t) {
    static const int32_t map[7] = {CVATTN_TYPE_F32, CVATTN_TYPE_F16, CVATTN_TYPE_Q8_0, CVATTN_TYPE_Q5_1,
                                   CVATTN_TYPE_Q5_0, CVATTN_TYPE_Q4_1, CVATTN_TYPE_Q4_0};
    return (t >= 0 && t < 7) ? map[t] : -1;
}

int32_t cvattn_ggml_to_kv_cache_type(int32_t g) {
    for (int32_t i = 0; i < 7; ++i)
        if (cvattn_kv_cache_type_to_ggml(i) == g) return i;
    return -1;
}

static uint32_t make_separate(uint32_t k, uint32_t v, uint32_t fb) {
    return k | (v << 5) | (fb << 10) | (1u << 31);
}

// Flash-attention branch of cosyvoice_check_kv_cache_types
// (src/cosyvoice-loader.cpp:568-632), probing with cvattn_supports.
cvattn_status cvattn_negotiate_kv_types(uint32_t u, int32_t kv_fallback, int32_t head_dim, int32_t n_q_heads,
                                        int32_t n_kv_heads, int32_t* k_type, int32_t* v_type,
                                        uint32_t* resolved_union, int32_t* fattn) {
    if (!k_type || !v_type || !resolved_union || !fattn) return CVATTN_ERR_INVALID_ARGUMENT;
    auto check = [&](int32_t k, int32_t v) {
        return k >= 0 && v >= 0 && cvattn_supports(k, v, head_dim, n_q_heads, n_kv_heads) != 0;
    };
    const bool separate = (u >> 31) & 1u;
    const int32_t uk = (int32_t)(u & 0x1f), uv = (int32_t)((u >> 5) & 0x1f), ufb = (int32_t)((u >> 10) & 0x1f);
    int32_t kt = -1, vt = -1;
    *fattn = check(CVATTN_TYPE_F32, CVATTN_TYPE_F32) ? 1 : 0;
    if (!*fattn) return CVATTN_ERR_UNSUPPORTED;  // the engine implements the flash path only
    if (kv_fallback) {
        bool done = false;
        int32_t cur;
        if (separate) {
            kt = cvattn_kv_cache_type_to_ggml(uk);
            vt = cvattn_kv_cache_type_to_ggml(uv);
            if (check(kt, vt)) {
                u = make_separate((uint32_t)uk, (uint32_t)uv, (uint32_t)uv);
                done = true;
            }
            cur = cvattn_kv_cache_type_to_ggml(ufb);
        } else {
            cur = cvattn_kv_cache_type_to_ggml((int32_t)u);
        }
        if (!done) {
            if (cur < 0) return CVATTN_ERR_INVALID_ARGUMENT;
            do {
                if (check(cur, cur)) {
                    kt = vt = cur;
                    u = (uint32_t)cvattn_ggml_to_kv_cache_type(cur);
                    break;
                }
                cur = cvattn_kv_fallback_type(cur);
            } while (cur != CVATTN_TYPE_F32 && cur >= 0);
            if (kt < 0) {  // fell through to f32 without a check, as the reference loop does
                kt = vt = CVATTN_TYPE_F32;
            }
            if (separate)
                u = make_separate((uint32_t)cvattn_ggml_to_kv_cache_type(kt), (uint32_t)cvattn_ggml_to_kv_cache_type(vt),
                                  (uint32_t)cvattn_ggml_to_kv_cache_type(vt));
        }
    } else if (separate) {
        kt = cvattn_kv_cache_type_to_ggml(uk);
        vt = cvattn_kv_cache_type_to_ggml(uv);
        *fattn = check(kt, vt) ? 1 : 0;
        if (*fattn) u = make_separate((uint32_t)uk, (uint32_t)uv, (uint32_t)uv);
    } else {
        kt = vt = cvattn_kv_cache_type_to_ggml((int32_t)u);
        *fattn = check(kt, vt) ? 1 : 0;
    }
    if (kt < 0 || vt < 0) return CVATTN_ERR_INVALID_ARGUMENT;
    *k_type = kt;
    *v_type = vt;
    *resolved_union = u;
    return *fattn ? CVATTN_OK : CVATTN_ERR_UNSUPPORTED;
}

// ------------------------------------------------------------------ context

cvattn_status cvattn_context_create(int32_t device, cvattn_context** out) {
    if (!out) return CVATTN_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) return CVATTN_ERR_NO_DEVICE;
    if (device < 0 || device >= n) return CVATTN_ERR_INVALID_ARGUMENT;
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return from_cuda(e);
    int* st = nullptr;
    e = cudaMalloc(&st, sizeof(int));
    if (e != cudaSuccess) return from_cuda(e);
    e = cudaMemset(st, 0, sizeof(int));
    if (e != cudaSuccess) {
        cudaFree(st);
        return from_cuda(e);
    }
    cvattn_context* c = new (std::nothrow) cvattn_context{device, st};
    if (!c) {
        cudaFree(st);
        return CVATTN_ERR_ALLOC;
    }
    *out = c;
    return CVATTN_OK;
}

void cvattn_context_destroy(cvattn_context* ctx) {
    if (!ctx) return;
    DeviceGuard dg(ctx->device);
    cudaFree(ctx->status);
    delete ctx;
}

cvattn_status cvattn_context_sync_status(cvattn_context* ctx, void* stream, int32_t* detail) {
    if (!ctx) return CVATTN_ERR_INVALID_ARGUMENT;
    DeviceGuard dg(ctx->device);
    if (dg.error() != cudaSuccess) return from_cuda(dg.error());
    int v = 0;
    cudaError_t e = cudaMemcpyAsync(&v, ctx->status, sizeof(int), cudaMemcpyDeviceToHost, as_stream(stream));
    if (e == cudaSuccess) e = cudaStreamSynchronize(as_stream(stream));
    if (e == cudaSuccess && v != 0) e = cudaMemsetAsync(ctx->status, 0, sizeof(int), as_stream(stream));
    if (e == cudaSuccess) e = cudaStreamSynchronize(as_stream(stream));
    if (e != cudaSuccess) return from_cuda(e);
    if (detail) *detail = v;
    if ((v & 0xff) == 3) return CVATTN_ERR_TIMEOUT;
    return v ? CVATTN_ERR_DEVICE : CVATTN_OK;
}

// ---------------------------------------------------------------- append

cvattn_status cvattn_kv_append(cvattn_context* ctx, void* stream, const cvattn_tensor* cache, const float* src,
                               int64_t src_nb1, int64_t src_nb2, const int32_t* pos, int64_t pos_nb1, int32_t n_new,
                               int32_t batch) {
    if (!ctx || !tensor_ok(cache) || n_new < 0 || batch < 0 || batch > cache->ne2) return CVATTN_ERR_INVALID_ARGUMENT;
    if (n_new == 0 || batch == 0) return CVATTN_OK;
    if (!src || !pos || (src_nb1 & 3) || (src_nb2 & 3) || (pos_nb1 & 3) || pos_nb1 < 0)
        return CVATTN_ERR_INVALID_ARGUMENT;
    if (reinterpret_cast<uintptr_t>(src) & 3) return CVATTN_ERR_INVALID_ARGUMENT;
    DeviceGuard dg(ctx->device);
    if (dg.error() != cudaSuccess) return from_cuda(dg.error());
    return from_cuda(launch_kv_append(as_stream(stream), *cache, src, src_nb1, src_nb2, pos, pos_nb1 / 4, n_new, batch,
                                      ctx->status));
}

// ------------------------------------------------------------------ RoPE

// Validates a RoPE description and forms its device form (theta_scale with the
// C library's powf, as ggml's CPU backend does).
static bool rope_dev(const cvattn_rope_params* r, RopeDev& d) {
    if (!r || (r->mode != CVATTN_ROPE_NORMAL && r->mode != CVATTN_ROPE_NEOX)) return false;
    if (r->unit_len <= 0 || r->n_dims < 2 || (r->n_dims & 1) || r->n_dims > r->unit_len) return false;
    if (!(r->freq_base > 0.0f) || !std::isfinite(r->freq_scale) || !std::isfinite(r->attn_factor)) return false;
    d.mode = r->mode;
    d.n_dims = r->n_dims;
    d.unit_len = r->unit_len;
    d.theta_scale = powf(r->freq_base, -2.0f / (float)r->n_dims);
    d.freq_scale = r->freq_scale;
    d.attn_factor = r->attn_factor;
    return true;
}

cvattn_status cvattn_rope(void* stream, const cvattn_rope_params* rope, const float* x, int64_t x_nb1, float* out,
                          int64_t out_nb1, const int32_t* pos, int32_t n_rows, int32_t row_len) {
    RopeDev d;
    if (!rope_dev(rope, d) || n_rows < 0 || row_len <= 0 || row_len % rope->unit_len) return CVATTN_ERR_INVALID_ARGUMENT;
    if (n_rows == 0) return CVATTN_OK;
    if (!x || !out || !pos || (x_nb1 & 3) || (out_nb1 & 3) || x_nb1 < 4 * (int64_t)row_len ||
        out_nb1 < 4 * (int64_t)row_len || (reinterpret_cast<uintptr_t>(x) & 3) || (reinterpret_cast<uintptr_t>(out) & 3))
        return CVATTN_ERR_INVALID_ARGUMENT;
    if (x == out) {
        if (x_nb1 != out_nb1) return CVATTN_ERR_INVALID_ARGUMENT;  // in place: same rows
    } else {
        // distinct buffers must not overlap
        const auto* xb = reinterpret_cast<const uint8_t*>(x);
        const auto* ob = reinterpret_cast<const uint8_t*>(out);
        if (ob < xb + (int64_t)n_rows * x_nb1 && xb < ob + (int64_t)n_rows * out_nb1) return CVATTN_ERR_INVALID_ARGUMENT;
    }
    return from_cuda(launch_rope(as_stream(stream), d, x, x_nb1 / 4, out, out_nb1 / 4, pos, n_rows, row_len));
}

cvattn_status cvattn_kv_append_rope(cvattn_context* ctx, void* stream, const cvattn_tensor* cache, const float* src,
                                    int64_t src_nb1, int64_t src_nb2, const int32_t* pos, int64_t pos_nb1,
                                    int32_t n_new, int32_t batch, const cvattn_rope_params* rope) {
    RopeDev d;
    if (!rope_dev(rope, d) || !tensor_ok(cache) || (cache->n_heads * cache->head_dim) % rope->unit_len)
        return CVATTN_ERR_INVALID_ARGUMENT;
    if (!ctx || n_new < 0 || batch < 0 || batch > cache->ne2) return CVATTN_ERR_INVALID_ARGUMENT;
    if (n_new == 0 || batch == 0) return CVATTN_OK;
    if (!src || !pos || (src_nb1 & 3) || (src_nb2 & 3) || (pos_nb1 & 3) || pos_nb1 < 0)
        return CVATTN_ERR_INVALID_ARGUMENT;
    if (reinterpret_cast<uintptr_t>(src) & 3) return CVATTN_ERR_INVALID_ARGUMENT;
    DeviceGuard dg(ctx->device);
    if (dg.error() != cudaSuccess) return from_cuda(dg.error());
    return from_cuda(launch_kv_append(as_stream(stream), *cache, src, src_nb1, src_nb2, pos, pos_nb1 / 4, n_new, batch,
                                      ctx->status, &d));
}

cvattn_status cvattn_kv_dequantize(cvattn_context* ctx, void* stream, const cvattn_tensor* cache, int32_t n_rows,
                                   float* dst) {
    if (!ctx || !tensor_ok(cache) || n_rows < 0 || n_rows > cache->ne1 || (n_rows && !dst))
        return CVATTN_ERR_INVALID_ARGUMENT;
    DeviceGuard dg(ctx->device);
    if (dg.error() != cudaSuccess) return from_cuda(dg.error());
    return from_cuda(launch_kv_dequant(as_stream(stream), *cache, n_rows, dst));
}

// ---------------------------------------------------------------- decode

size_t cvattn_decode_workspace_size(int32_t k_type, int32_t v_type, int32_t n_seq, int32_t max_kv_len,
                                    int32_t n_q_heads, int32_t n_kv_heads, int32_t head_dim) {
    if (!decode_supported(k_type, v_type, head_dim, n_q_heads, n_kv_heads)) return 0;
    return decode_workspace_bytes(k_type, v_type, n_seq, max_kv_len, n_q_heads, n_kv_heads, head_dim);
}

cvattn_status cvattn_workspace_init(void* stream, void* workspace, size_t bytes) {
    if (!workspace && bytes) return CVATTN_ERR_INVALID_ARGUMENT;
    if (!bytes) return CVATTN_OK;
    return from_cuda(cudaMemsetAsync(workspace, 0, bytes, as_stream(stream)));
}

static cvattn_status decode_impl(cvattn_context* ctx, void* stream, const cvattn_decode_params* p,
                                 const cvattn_rope_params* rope) {
    if (!ctx || !p || !p->q || !p->out || !p->kv_len) return CVATTN_ERR_INVALID_ARGUMENT;
    if (p->n_seq < 0 || p->max_kv_len < 0 || p->n_q_heads <= 0) return CVATTN_ERR_INVALID_ARGUMENT;
    if (p->n_seq == 0) return CVATTN_OK;
    const cvattn_tensor& k = p->k;
    const cvattn_tensor& v = p->v;
    if (!p->k_seq_ptrs && !tensor_ok(&k)) return CVATTN_ERR_INVALID_ARGUMENT;
    if (!p->v_seq_ptrs && !tensor_ok(&v)) return CVATTN_ERR_INVALID_ARGUMENT;
    if (!known_type(k.type) || !known_type(v.type) || k.n_heads != v.n_heads || k.head_dim != v.head_dim)
        return CVATTN_ERR_INVALID_ARGUMENT;
    if (!decode_supported(k.type, v.type, k.head_dim, p->n_q_heads, k.n_heads)) return CVATTN_ERR_UNSUPPORTED;
    // rows must be packed (one ggml row per position) for the chunk stream
    if (k.nb1 != type_row_bytes(k.type, (int64_t)k.n_heads * k.head_dim) ||
        v.nb1 != type_row_bytes(v.type, (int64_t)v.n_heads * v.head_dim))
        return CVATTN_ERR_UNSUPPORTED;
    if (!p->k_seq_ptrs && k.ne2 < p->n_seq) return CVATTN_ERR_INVALID_ARGUMENT;
    if (!p->v_seq_ptrs && v.ne2 < p->n_seq) return CVATTN_ERR_INVALID_ARGUMENT;
    if (p->max_kv_len > k.ne1 || p->max_kv_len > v.ne1) return CVATTN_ERR_LENGTH;
    if ((p->k_new == nullptr) != (p->v_new == nullptr)) return CVATTN_ERR_INVALID_ARGUMENT;
    if ((p->flags & CVATTN_DECODE_EMIT_PARTIAL) && !p->partial_ml) return CVATTN_ERR_INVALID_ARGUMENT;
    if (p->q_seq_stride < (int64_t)p->n_q_heads * k.head_dim || p->out_seq_stride < (int64_t)p->n_q_heads * k.head_dim)
        return CVATTN_ERR_INVALID_ARGUMENT;
    // q and out rows are accessed as 16-byte vectors
    if ((reinterpret_cast<uintptr_t>(p->q) & 15) || (reinterpret_cast<uintptr_t>(p->out) & 15) || (p->q_seq_stride & 3) ||
        (p->out_seq_stride & 3))
        return CVATTN_ERR_INVALID_ARGUMENT;
    const size_t need = decode_workspace_bytes(k.type, v.type, p->n_seq, p->max_kv_len, p->n_q_heads, k.n_heads,
                                               k.head_dim);
    if (!p->workspace || p->workspace_size < need) return CVATTN_ERR_INVALID_ARGUMENT;
    RopeDev rd;
    if (rope) {
        if (!rope_dev(rope, rd)) return CVATTN_ERR_INVALID_ARGUMENT;
        if (rope->unit_len != k.head_dim || rope->n_dims != k.head_dim || !decode_rope_supported(*p))
            return CVATTN_ERR_UNSUPPORTED;
    }
    DeviceGuard dg(ctx->device);
    if (dg.error() != cudaSuccess) return from_cuda(dg.error());
    if (p->max_kv_len == 0) {
        // nothing visible anywhere: ggml's S == 0 convention gives zeros
        for (int32_t s = 0; s < p->n_seq; ++s) {
            cudaError_t e = cudaMemsetAsync(p->out + (int64_t)s * p->out_seq_stride, 0,
                                            sizeof(float) * p->n_q_heads * k.head_dim, as_stream(stream));
            if (e != cudaSuccess) return from_cuda(e);
        }
        return CVATTN_OK;
    }
    return from_cuda(launch_decode(as_stream(stream), *p, ctx->status, rope ? &rd : nullptr));
}

cvattn_status cvattn_decode(cvattn_context* ctx, void* stream, const cvattn_decode_params* p) {
    return decode_impl(ctx, stream, p, nullptr);
}

cvattn_status cvattn_decode_rope(cvattn_context* ctx, void* stream, const cvattn_decode_params* p,
                                 const cvattn_rope_params* rope) {
    if (!rope) return CVATTN_ERR_INVALID_ARGUMENT;
    return decode_impl(ctx, stream, p, rope);
}

cvattn_status cvattn_combine(void* stream, const float* partial_o, const float* partial_ml, int32_t n_parts,
                             int32_t n_rows, int32_t head_dim, float* out) {
    if (n_parts <= 0 || n_rows < 0 || head_dim <= 0 || (n_rows && (!partial_o || !partial_ml || !out)))
        return CVATTN_ERR_INVALID_ARGUMENT;
    return from_cuda(launch_combine(as_stream(stream), partial_o, partial_ml, n_parts, n_rows, head_dim, out));
}

// ------------------------------------------------------------------ flash

cvattn_status cvattn_flash(cvattn_context* ctx, void* stream, const cvattn_flash_params* p) {
    if (!ctx || !p || !p->q || !p->out) return CVATTN_ERR_INVALID_ARGUMENT;
    if (p->n_q < 0 || p->n_kv < 0 || p->batch < 0 || p->n_q_heads <= 0) return CVATTN_ERR_INVALID_ARGUMENT;
    if (p->n_q == 0 || p->batch == 0) return CVATTN_OK;
    if (!tensor_ok(&p->k) || !tensor_ok(&p->v)) return CVATTN_ERR_INVALID_ARGUMENT;
    if (p->k.n_heads != p->v.n_heads || p->k.head_dim != p->v.head_dim) return CVATTN_ERR_INVALID_ARGUMENT;
    if (!flash_supported(p->k.type, p->v.type, p->k.head_dim, p->n_q_heads, p->k.n_heads)) return CVATTN_ERR_UNSUPPORTED;
    if (p->n_kv > p->k.ne1 || p->n_kv > p->v.ne1) return CVATTN_ERR_LENGTH;
    if (p->batch > p->k.ne2 || p->batch > p->v.ne2) return CVATTN_ERR_INVALID_ARGUMENT;
    if (p->mask_mode < CVATTN_MASK_NONE || p->mask_mode > CVATTN_MASK_CHUNK) return CVATTN_ERR_INVALID_ARGUMENT;
    if (p->mask_mode == CVATTN_MASK_EXPLICIT && (!p->mask || p->mask_nb1 < p->n_kv)) return CVATTN_ERR_INVALID_ARGUMENT;
    if (p->mask_mode == CVATTN_MASK_CHUNK) {
        if (p->n_chunk_bounds < 0 || p->n_chunk_bounds > CVATTN_MAX_CHUNK_BOUNDS) return CVATTN_ERR_INVALID_ARGUMENT;
        for (int32_t i = 1; i < p->n_chunk_bounds; ++i)
            if (p->chunk_bounds[i] < p->chunk_bounds[i - 1]) return CVATTN_ERR_INVALID_ARGUMENT;
    }
    DeviceGuard dg(ctx->device);
    if (dg.error() != cudaSuccess) return from_cuda(dg.error());
    return from_cuda(launch_flash(as_stream(stream), *p, ctx->status));
}

// ------------------------------------------------------------ copies

static cvattn_status copy_rows(void* stream, const cvattn_tensor* t, int32_t n_tokens, void* host, bool to_host) {
    if (!tensor_ok(t) || n_tokens < 0 || n_tokens > t->ne1 || (n_tokens && !host)) return CVATTN_ERR_INVALID_ARGUMENT;
    const size_t bytes = (size_t)t->nb1 * (size_t)n_tokens;
    if (!bytes) return CVATTN_OK;
    for (int64_t b = 0; b < t->ne2; ++b) {
        char* dev = static_cast<char*>(t->data) + b * t->nb2;
        char* h = static_cast<char*>(host) + (size_t)b * bytes;
        cudaError_t e = to_host ? cudaMemcpyAsync(h, dev, bytes, cudaMemcpyDeviceToHost, as_stream(stream))
                                : cudaMemcpyAsync(dev, h, bytes, cudaMemcpyHostToDevice, as_stream(stream));
        if (e != cudaSuccess) return from_cuda(e);
    }
    return CVATTN_OK;
}

cvattn_status cvattn_kv_copy_to_host(void* stream, const cvattn_tensor* t, int32_t n_tokens, void* host) {
    return copy_rows(stream, t, n_tokens, host, true);
}

cvattn_status cvattn_kv_copy_from_host(void* stream, const cvattn_tensor* t, int32_t n_tokens, const void* host) {
    return copy_rows(stream, t, n_tokens, const_cast<void*>(host), false);
}

}  // extern "C"

// ------------------------------------------------------ KV cache object

struct cvattn_kv_cache {
    cvattn_context* ctx = nullptr;
    cvattn_kv_cache_params p{};
    char* base = nullptr;           // one device allocation
    size_t bytes = 0;
    std::vector<size_t> k_off, v_off;  // per (slot * layers + layer)
    int64_t k_nb1 = 0, v_nb1 = 0;
    uint32_t cur_len = 0;
    uint32_t view_len = 0;          // cur_len + rows appended by the last update
    int cur_slot = 0;
    // offloaded host slots (src/cosyvoice-kv-cache.cpp:19-32), in pinned memory so
    // the copies run asynchronously; `done` marks the end of the last copy that
    // touched the slot (later copies on another stream wait for it, and the host
    // waits for it before it reads, resizes or frees the buffer)
    struct host_slot {
        uint32_t len = 0;
        char* buffer = nullptr;
        size_t bytes = 0;           // bytes holding len positions of every layer
        size_t capacity = 0;
        cudaEvent_t done = nullptr;
        bool pending = false;       // `done` was recorded and may not have completed
    };
    std::vector<host_slot> offloaded;
    // decode workspace, sized at creation for the largest supported query-head
    // count (8 per KV head) and max_seq positions: the attention call never allocates
    void* ws = nullptr;
    size_t ws_bytes = 0;
    int32_t* d_len = nullptr;       // device kv lengths [batch]
};

static size_t al256(size_t x) { return (x + 255) & ~size_t(255); }

static cvattn_tensor cache_tensor(const cvattn_kv_cache* c, int layer, int slot, int which) {
    cvattn_tensor t{};
    const int idx = slot * c->p.layers + layer;
    t.data = c->base + (which ? c->v_off[idx] : c->k_off[idx]);
    t.type = which ? c->p.v_type : c->p.k_type;
    t.n_heads = c->p.n_kv_heads;
    t.head_dim = which ? c->p.v_head_dim : c->p.k_head_dim;
    t.ne1 = c->p.max_seq;
    t.ne2 = c->p.batch;
    t.nb1 = which ? c->v_nb1 : c->k_nb1;
    t.nb2 = t.nb1 * (int64_t)c->p.max_seq;
    return t;
}

// Waits for the copies that last touched a host slot (host side).
static cudaError_t host_slot_wait(cvattn_kv_cache::host_slot& hs) {
    if (!hs.pending) return cudaSuccess;
    cudaError_t e = cudaEventSynchronize(hs.done);
    if (e == cudaSuccess) hs.pending = false;
    return e;
}

static void host_slot_free(cvattn_kv_cache::host_slot& hs) {
    host_slot_wait(hs);
    if (hs.buffer) cudaFreeHost(hs.buffer);
    hs.buffer = nullptr;
    hs.capacity = hs.bytes = 0;
    hs.len = 0;
}

// Host bytes of one offloaded slot holding n positions: per layer K for every
// batch entry, then V (src/cosyvoice-kv-cache.cpp:153-172).
static size_t host_slot_bytes(const cvattn_kv_cache* c, uint32_t n) {
    return ((size_t)c->k_nb1 + (size_t)c->v_nb1) * n * (size_t)c->p.batch * (size_t)c->p.layers;
}

// Copies positions [0, n) of every batch entry of t to or from host, where the
// host rows of batch entry b start at host + b * n * t.nb1: one strided copy
// covers the whole batch.
static cudaError_t copy_rows_2d(cudaStream_t s, const cvattn_tensor& t, uint32_t n, char* host, bool to_host) {
    const size_t w = (size_t)t.nb1 * n;
    if (!w) return cudaSuccess;
    if (to_host)
        return cudaMemcpy2DAsync(host, w, t.data, (size_t)t.nb2, w, (size_t)t.ne2, cudaMemcpyDeviceToHost, s);
    return cudaMemcpy2DAsync(t.data, (size_t)t.nb2, host, w, w, (size_t)t.ne2, cudaMemcpyHostToDevice, s);
}

extern "C" {

void cvattn_kv_cache_destroy(cvattn_kv_cache* c) {
    if (!c) return;
    DeviceGuard dg(c->ctx->device);
    for (auto& hs : c->offloaded) {
        host_slot_free(hs);
        if (hs.done) cudaEventDestroy(hs.done);
    }
    cudaFree(c->base);
    cudaFree(c->d_len);
    if (c->ws) cudaFree(c->ws);
    delete c;
}

cvattn_status cvattn_kv_cache_create(cvattn_context* ctx, const cvattn_kv_cache_params* p, cvattn_kv_cache** out) {
    if (!ctx || !p || !out) return CVATTN_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    if (p->layers <= 0 || p->n_kv_heads <= 0 || p->k_head_dim <= 0 || p->v_head_dim <= 0 || p->max_seq == 0 ||
        p->max_seq > 0x7fffffffu || p->batch <= 0 || p->n_slots <= 0 || p->n_offloaded_slots < 0 ||
        !known_type(p->k_type) || !known_type(p->v_type))
        return CVATTN_ERR_INVALID_ARGUMENT;
    const int64_t ke = (int64_t)p->k_head_dim * p->n_kv_heads, ve = (int64_t)p->v_head_dim * p->n_kv_heads;
    if (ke % 32 || ve % 32) return CVATTN_ERR_INVALID_ARGUMENT;
    DeviceGuard dg(ctx->device);
    if (dg.error() != cudaSuccess) return from_cuda(dg.error());
    cvattn_kv_cache* c = new (std::nothrow) cvattn_kv_cache();
    if (!c) return CVATTN_ERR_ALLOC;
    c->ctx = ctx;
    c->p = *p;
    c->k_nb1 = type_row_bytes(p->k_type, ke);
    c->v_nb1 = type_row_bytes(p->v_type, ve);
    const size_t kb = al256((size_t)c->k_nb1 * p->max_seq * p->batch);
    const size_t vb = al256((size_t)c->v_nb1 * p->max_seq * p->batch);
    size_t off = 0;
    const int n = p->layers * p->n_slots;
    c->k_off.resize(n);
    c->v_off.resize(n);
    for (int i = 0; i < n; ++i) {  // K then V per (slot, layer): reset_buffer order, kv-cache.cpp:134-145
        c->k_off[i] = off;
        off += kb;
        c->v_off[i] = off;
        off += vb;
    }
    c->bytes = off;
    c->offloaded.resize(p->n_offloaded_slots);
    cudaError_t e = cudaMalloc(&c->base, off);
    if (e == cudaSuccess) e = cudaMalloc(&c->d_len, sizeof(int32_t) * p->batch);
    // the decode workspace for the largest query-head count the engine supports
    if (e == cudaSuccess && p->k_head_dim == p->v_head_dim &&
        decode_supported(p->k_type, p->v_type, p->k_head_dim, 8 * p->n_kv_heads, p->n_kv_heads)) {
        const size_t need = decode_workspace_bytes(p->k_type, p->v_type, p->batch, (int)p->max_seq,
                                                   8 * p->n_kv_heads, p->n_kv_heads, p->k_head_dim);
        e = cudaMalloc(&c->ws, need);
        if (e == cudaSuccess) {
            c->ws_bytes = need;
            e = cudaMemset(c->ws, 0, need);
        }
    }
    for (auto& hs : c->offloaded)
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&hs.done, cudaEventDisableTiming);
    if (e != cudaSuccess) {
        cvattn_kv_cache_destroy(c);
        return from_cuda(e);
    }
    *out = c;
    return CVATTN_OK;
}

cvattn_status cvattn_kv_cache_tensor(cvattn_kv_cache* c, int32_t layer, int32_t slot, int32_t which,
                                     cvattn_tensor* out) {
    if (!c || !out || layer < 0 || layer >= c->p.layers || slot < 0 || slot >= c->p.n_slots || (which != 0 && which != 1))
        return CVATTN_ERR_INVALID_ARGUMENT;
    *out = cache_tensor(c, layer, slot, which);
    return CVATTN_OK;
}

size_t cvattn_kv_cache_device_bytes(const cvattn_kv_cache* c) { return c ? c->bytes : 0; }

uint32_t cvattn_kv_cache_get_len(const cvattn_kv_cache* c) { return c ? c->cur_len : 0; }

void cvattn_kv_cache_set_len(cvattn_kv_cache* c, uint32_t len) {
    if (!c) return;
    c->cur_len = len;
    c->view_len = len;
}

cvattn_status cvattn_kv_cache_update(cvattn_kv_cache* c, void* stream, int32_t layer, const float* k, const float* v,
                                     const int32_t* pos, int64_t pos_nb1, int32_t n_new) {
    if (!c || layer < 0 || layer >= c->p.layers || n_new < 0) return CVATTN_ERR_INVALID_ARGUMENT;
    if ((uint64_t)c->cur_len + (uint64_t)n_new > c->p.max_seq) return CVATTN_ERR_LENGTH;
    const cvattn_tensor kt = cache_tensor(c, layer, c->cur_slot, 0);
    const cvattn_tensor vt = cache_tensor(c, layer, c->cur_slot, 1);
    const int64_t kr = (int64_t)kt.n_heads * kt.head_dim * 4, vr = (int64_t)vt.n_heads * vt.head_dim * 4;
    cvattn_status s = cvattn_kv_append(c->ctx, stream, &kt, k, kr, kr * n_new, pos, pos_nb1, n_new, c->p.batch);
    if (s == CVATTN_OK) s = cvattn_kv_append(c->ctx, stream, &vt, v, vr, vr * n_new, pos, pos_nb1, n_new, c->p.batch);
    if (s == CVATTN_OK) c->view_len = c->cur_len + (uint32_t)n_new;
    return s;
}

cvattn_status cvattn_kv_cache_attention(cvattn_kv_cache* c, void* stream, int32_t layer, const float* q, int32_t n_q,
                                        int32_t n_q_heads, int32_t mask_mode, const uint16_t* mask, int64_t mask_nb1,
                                        float* out) {
    if (!c || layer < 0 || layer >= c->p.layers || !q || !out || n_q <= 0 || n_q_heads <= 0)
        return CVATTN_ERR_INVALID_ARGUMENT;
    const cvattn_tensor kt = cache_tensor(c, layer, c->cur_slot, 0);
    const cvattn_tensor vt = cache_tensor(c, layer, c->cur_slot, 1);
    const int32_t n_kv = (int32_t)c->view_len;
    const int64_t D = kt.head_dim;
    if (n_q == 1 && mask_mode == CVATTN_MASK_NONE && n_kv > 0 && c->ws &&
        decode_supported(kt.type, vt.type, kt.head_dim, n_q_heads, kt.n_heads)) {
        cvattn_decode_params dp{};
        dp.q = q;
        dp.q_seq_stride = n_q_heads * D;
        dp.out = out;
        dp.out_seq_stride = n_q_heads * D;
        dp.k = kt;
        dp.v = vt;
        dp.n_seq = c->p.batch;
        dp.n_q_heads = n_q_heads;
        dp.max_kv_len = n_kv;
        dp.scale = 1.0f / std::sqrt((float)D);
        dp.workspace = c->ws;
        dp.workspace_size = c->ws_bytes;
        dp.kv_len = c->d_len;
        // the view length goes to the device with a tiny kernel (no host buffer, no
        // synchronization, capturable); the same launch clears the ticket counters,
        // so a decode that gave up on an earlier call cannot leave them stale
        {
            DeviceGuard dg(c->ctx->device);
            if (dg.error() != cudaSuccess) return from_cuda(dg.error());
            cudaError_t e = launch_fill_lengths(as_stream(stream), c->d_len, c->p.batch, n_kv,
                                                static_cast<uint32_t*>(c->ws),
                                                (int)(decode_ticket_bytes(c->p.batch, c->p.n_kv_heads) / 4));
            if (e != cudaSuccess) return from_cuda(e);
        }
        return cvattn_decode(c->ctx, stream, &dp);
    }
    cvattn_flash_params fp{};
    fp.q = q;
    fp.q_nb_tok = n_q_heads * D;
    fp.q_nb_head = D;
    fp.q_nb_batch = (int64_t)n_q * n_q_heads * D;
    fp.out = out;
    fp.k = kt;
    fp.v = vt;
    fp.n_q = n_q;
    fp.n_kv = n_kv;
    fp.n_q_heads = n_q_heads;
    fp.batch = c->p.batch;
    fp.scale = 1.0f / std::sqrt((float)D);
    fp.mask_mode = mask_mode;
    fp.mask = mask;
    fp.mask_nb1 = mask_nb1;
    fp.causal_offset = n_kv - n_q;
    return cvattn_flash(c->ctx, stream, &fp);
}

void cvattn_kv_cache_shift(cvattn_kv_cache* c, uint32_t n) {
    if (!c) return;
    c->cur_len += n;
    c->view_len = c->cur_len;
}

int32_t cvattn_kv_cache_bind_slot(cvattn_kv_cache* c, int32_t slot) {
    if (!c || slot < 0 || slot >= c->p.n_slots) return 0;
    c->cur_slot = slot;
    return 1;
}

cvattn_status cvattn_kv_cache_slide_slot(cvattn_kv_cache* c) {
    if (!c || c->cur_slot + 1 >= c->p.n_slots) return CVATTN_ERR_INVALID_ARGUMENT;
    c->cur_slot++;
    return CVATTN_OK;
}

int32_t cvattn_kv_cache_current_slot(const cvattn_kv_cache* c) { return c ? c->cur_slot : -1; }

cvattn_status cvattn_kv_cache_offload_slot(cvattn_kv_cache* c, void* stream, int32_t slot_idx, uint32_t n_tokens) {
    if (!c || slot_idx < 0 || slot_idx >= (int32_t)c->offloaded.size() || n_tokens > c->p.max_seq)
        return CVATTN_ERR_INVALID_ARGUMENT;
    DeviceGuard dg(c->ctx->device);
    if (dg.error() != cudaSuccess) return from_cuda(dg.error());
    auto& hs = c->offloaded[slot_idx];
    const cudaStream_t s = as_stream(stream);
    const size_t need = host_slot_bytes(c, n_tokens);
    cudaError_t e = cudaSuccess;
    if (need > hs.capacity) {  // grow: the old buffer may still be read by an earlier load
        host_slot_free(hs);
        e = cudaHostAlloc(reinterpret_cast<void**>(&hs.buffer), need, cudaHostAllocDefault);
        if (e != cudaSuccess) {
            hs.buffer = nullptr;
            return from_cuda(e);
        }
        hs.capacity = need;
    } else if (hs.pending) {  // an earlier load from this buffer must finish before it is overwritten
        e = cudaStreamWaitEvent(s, hs.done, 0);
        if (e != cudaSuccess) return from_cuda(e);
    }
    hs.len = n_tokens;
    hs.bytes = need;
    const size_t kn = (size_t)c->k_nb1 * n_tokens, vn = (size_t)c->v_nb1 * n_tokens;
    const size_t per_layer = (kn + vn) * c->p.batch;
    // offload_cache reads kv_cache_layers[i], the layers of device slot 0, which every
    // offloadable step shares (src/cosyvoice-kv-cache.cpp:163-172; token2wav binds slot
    // 0 for offload steps, src/cosyvoice-token2wav.cpp:390)
    for (int l = 0; l < c->p.layers && e == cudaSuccess; ++l) {
        char* kdst = hs.buffer + (size_t)l * per_layer;
        char* vdst = kdst + kn * c->p.batch;
        e = copy_rows_2d(s, cache_tensor(c, l, 0, 0), n_tokens, kdst, true);
        if (e == cudaSuccess) e = copy_rows_2d(s, cache_tensor(c, l, 0, 1), n_tokens, vdst, true);
    }
    if (e == cudaSuccess) e = cudaEventRecord(hs.done, s);
    if (e == cudaSuccess) hs.pending = true;
    return from_cuda(e);
}

cvattn_status cvattn_kv_cache_load_slot(cvattn_kv_cache* c, void* stream, int32_t slot_idx) {
    if (!c || slot_idx < 0 || slot_idx >= (int32_t)c->offloaded.size()) return CVATTN_ERR_INVALID_ARGUMENT;
    DeviceGuard dg(c->ctx->device);
    if (dg.error() != cudaSuccess) return from_cuda(dg.error());
    auto& hs = c->offloaded[slot_idx];
    c->cur_len = hs.len;
    c->view_len = hs.len;
    if (hs.len == 0) return CVATTN_OK;
    const cudaStream_t s = as_stream(stream);
    cudaError_t e = cudaSuccess;
    if (hs.pending) e = cudaStreamWaitEvent(s, hs.done, 0);  // the offload may run on another stream
    const size_t kn = (size_t)c->k_nb1 * hs.len, vn = (size_t)c->v_nb1 * hs.len;
    const size_t per_layer = (kn + vn) * c->p.batch;
    // load_cache writes kv_cache_layers[i + cur_slot_idx * layers] (src/cosyvoice-kv-cache.cpp:233-243)
    for (int l = 0; l < c->p.layers && e == cudaSuccess; ++l) {
        char* ksrc = hs.buffer + (size_t)l * per_layer;
        char* vsrc = ksrc + kn * c->p.batch;
        e = copy_rows_2d(s, cache_tensor(c, l, c->cur_slot, 0), hs.len, ksrc, false);
        if (e == cudaSuccess) e = copy_rows_2d(s, cache_tensor(c, l, c->cur_slot, 1), hs.len, vsrc, false);
    }
    if (e == cudaSuccess) e = cudaEventRecord(hs.done, s);
    if (e == cudaSuccess) hs.pending = true;
    return from_cuda(e);
}

cvattn_status cvattn_kv_cache_offloaded_slot(cvattn_kv_cache* c, int32_t slot_idx, const void** data, size_t* bytes,
                                             uint32_t* n_tokens) {
    if (!c || slot_idx < 0 || slot_idx >= (int32_t)c->offloaded.size() || !data || !bytes)
        return CVATTN_ERR_INVALID_ARGUMENT;
    auto& hs = c->offloaded[slot_idx];
    DeviceGuard dg(c->ctx->device);
    if (dg.error() != cudaSuccess) return from_cuda(dg.error());
    cudaError_t e = host_slot_wait(hs);
    if (e != cudaSuccess) return from_cuda(e);
    *data = hs.buffer;
    *bytes = hs.bytes;
    if (n_tokens) *n_tokens = hs.len;
    return CVATTN_OK;
}

size_t cvattn_kv_cache_offloaded_size(const cvattn_kv_cache* c) {
    if (!c) return 0;
    size_t n = 0;
    for (const auto& s : c->offloaded) n += s.capacity;
    return n;
}

void cvattn_kv_cache_clear_offloaded(cvattn_kv_cache* c) {
    if (!c) return;
    DeviceGuard dg(c->ctx->device);
    for (auto& s : c->offloaded) host_slot_free(s);
}

// ------------------------------------------------------------- DiT plan

// dit_sched_config (src/cosyvoice-token2wav.cpp:100-167).
cvattn_status cvattn_dit_sched_plan(int32_t n, int32_t n_offloadable, int32_t n_fixed, int64_t cut_len, uint32_t offset,
                                    int32_t streaming, int32_t kv_slidable, cvattn_dit_step* out) {
    if (!out || n < 2 || n_offloadable < 0 || n_fixed < 0 || n_offloadable + n_fixed > n) return CVATTN_ERR_INVALID_ARGUMENT;
    for (int i = 0; i < n; ++i) out[i] = cvattn_dit_step{};
    if (!streaming) {
        out[0].rebuild = 1;
        out[1].rebuild = 1;
        out[n - 1].rebuild = 1;
        out[n - 1].cut_len = cut_len;
        return CVATTN_OK;
    }
    if (offset != 0) cut_len = 0;
    const int n_no_cache = n - n_offloadable - n_fixed;
    for (int i = 0; i < n; ++i) {
        cvattn_dit_step& s = out[i];
        s.rebuild = (i <= 1 || (offset != 0 && i == n_no_cache - 1) || i == n_no_cache || (i == n - 1 && cut_len != 0) ||
                     (!kv_slidable && i >= n_no_cache))
                        ? 1
                        : 0;
        s.cache_kv = i >= n_no_cache;
        s.offload = i >= n_no_cache && i < n_no_cache + n_offloadable;
        s.load = s.offload && offset != 0;
        s.mask = i < n_no_cache && offset != 0;
        s.cut_len = (i == n - 1 && offset == 0) ? cut_len : 0;
        if (i == n_no_cache - 1 && offset != 0) s.cut_len = offset;
        s.slice = offset != 0 && i == n_no_cache;
        s.slide = (kv_slidable && s.cache_kv && (!s.offload || i == n_no_cache + n_offloadable - 1) && i != n - 1) ? 1 : 0;
    }
    return CVATTN_OK;
}

}  // extern "C"
