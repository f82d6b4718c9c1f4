// kv_append.cu -- fused quantize-on-write of new K/V rows into a ggml-layout
// cache tensor: the ggml_set_rows of cosyvoice_kv_cache::update_cache
// (src/cosyvoice-kv-cache.cpp:315-316,321-322), plus the inverse
// (dequantize rows to f32) used for slot export and tests.
//
// Large launches of 4- and 5-bit rows without a RoPE: one thread per 32-element block
// (quantize_block_thread, a sequential scan); q8_0, f16 / f32, RoPE'd rows and small
// launches: one warp per row, one lane per element (quantize_block_warp in common.cuh).
// Both are bit-identical to ggml's reference quantizers.
// HBM-bound: reads 128 B of f32 per group, writes 18-128 B.
//
// With a RoPE the K rows are rotated on the way in, as ggml_rope_ext does
// before update_cache (src/cosyvoice-llm.cpp:57,180; src/cosyvoice-graph.cpp:355);
// the standalone rope kernel covers Q and other callers.
#include <atomic>

#include "common.cuh"
#include "internal.h"
#include "rope.cuh"

namespace cvattn {

// One warp per source row (t, b): the row's position is looked up once, then
// the warp walks the row's 32-element groups (coalesced 128-byte loads, the
// iterations independent of each other).
template <int T>
__global__ void __launch_bounds__(256) kv_append_kernel(
    uint8_t* __restrict__ cache, int64_t nb1, int64_t nb2, int64_t capacity, int groups_per_row,
    const float* __restrict__ src, int64_t src_nb1, int64_t src_nb2,
    const int32_t* __restrict__ pos, int64_t pos_stride, int n_new, int batch, int* status, RopeDev rope) {
    const int lane = threadIdx.x & 31;
    const unsigned rw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);  // row (t, b), t fastest
    if (rw >= (unsigned)n_new * (unsigned)batch) return;
    const int b = (int)(rw / (unsigned)n_new);
    const int t = (int)(rw - (unsigned)b * (unsigned)n_new);
    const int p = pos[t + (int64_t)b * pos_stride];
    if (p < 0 || p >= capacity) {
        if (lane == 0) record_status(status, kStatusBadPosition);
        return;
    }
    const float* row = reinterpret_cast<const float*>(reinterpret_cast<const uint8_t*>(src) + t * src_nb1 + b * src_nb2);
    uint8_t* dst_row = cache + b * nb2 + (int64_t)p * nb1;
    // eight groups' loads in flight before any of them is quantized
    constexpr int kBatch = 8;
    for (int g0 = 0; g0 < groups_per_row; g0 += kBatch) {
        float x[kBatch];
#pragma unroll
        for (int i = 0; i < kBatch; ++i) x[i] = g0 + i < groups_per_row ? row[(g0 + i) * 32 + lane] : 0.0f;
        if (rope.n_dims > 0) {
#pragma unroll
            for (int i = 0; i < kBatch; ++i) {
                const int e = (g0 + i) * 32 + lane;
                int k;
                bool first;
                const int pe = rope_pair(rope, e, k, first);
                if (g0 + i < groups_per_row && pe >= 0)
                    x[i] = rope_rotate(x[i], row[pe], rope_cs(rope, rope_theta(rope, p, k)), first);
            }
        }
#pragma unroll
        for (int i = 0; i < kBatch; ++i)
            if (g0 + i < groups_per_row)  // uniform per warp
                quantize_block_warp<T>(x[i], dst_row + (int64_t)(g0 + i) * group_bytes(T), lane);
    }
}

// Quantize the 32 values of one 4- or 5-bit block into dst (2-byte aligned) with one thread:
// the sequential first-occurrence scans of ggml's reference quantizers (gguf-py quants.py
// Q4_0 :220-252, Q4_1 :254-289, Q5_0 :291-331, Q5_1 :333-376) and the same IEEE fp32
// operations as quantize_block_warp, so the bytes are the same.
template <int T>
__device__ __forceinline__ void quantize_block_thread(const float (&x)[32], uint8_t* dst) {
    using B = BlockTraits<T>;
    static_assert(T != kQ8_0, "q8_0 appends keep the warp form");
    constexpr bool kMin = B::HAS_MIN, k5 = B::OFF_QH >= 0;
    constexpr int kMax = k5 ? 31 : 15;
    float d, lo = 0.0f;
    if constexpr (kMin) {  // min and max, first occurrence (strict comparisons)
        float mn = x[0], mx = x[0];
#pragma unroll
        for (int j = 1; j < 32; ++j) {
            if (x[j] < mn) mn = x[j];
            if (x[j] > mx) mx = x[j];
        }
        d = __fdiv_rn(__fsub_rn(mx, mn), k5 ? 31.0f : 15.0f);
        lo = mn;
    } else {  // the value of largest magnitude, first occurrence
        float amax = 0.0f, mx = 0.0f;
#pragma unroll
        for (int j = 0; j < 32; ++j)
            if (amax < fabsf(x[j])) {
                amax = fabsf(x[j]);
                mx = x[j];
            }
        d = __fdiv_rn(mx, k5 ? -16.0f : -8.0f);
    }
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    int q[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        const int v = kMin ? (int)truncf(__fadd_rn(__fmul_rn(__fsub_rn(x[j], lo), id), 0.5f))
                           : (int)truncf(__fadd_rn(__fmul_rn(x[j], id), k5 ? 16.5f : 8.5f));
        q[j] = min(kMax, max(0, v));
    }
    store_u16(dst, f2h(d));
    if constexpr (kMin) store_u16(dst + 2, f2h(lo));
    if constexpr (k5) {  // bit e of qh: the fifth bit of element e
        uint32_t qh = 0;
#pragma unroll
        for (int j = 0; j < 32; ++j) qh |= (uint32_t)((q[j] >> 4) & 1) << j;
        store_u16(dst + B::OFF_QH, (uint16_t)qh);
        store_u16(dst + B::OFF_QH + 2, (uint16_t)(qh >> 16));
    }
#pragma unroll
    for (int j = 0; j < 16; j += 2)  // byte j: element j (low nibble) and element j + 16 (high)
        store_u16(dst + B::OFF_QS + j, (uint16_t)(((q[j] & 15) | ((q[j + 16] & 15) << 4)) |
                                                  (((q[j + 1] & 15) | ((q[j + 17] & 15) << 4)) << 8)));
}

// Block-quantized append without a RoPE: one thread per 32-element block (row (t, b), block
// g fastest), its 128 bytes of f32 read as eight 16-byte loads, the block quantized by a
// sequential scan (no warp reductions): ~5x fewer instructions per block than the warp form.
constexpr int kAppendBlockThreadsPerSm = 512;  // smallest launch (blocks per SM) that takes this form

template <int T>
__global__ void __launch_bounds__(256) kv_append_block_kernel(
    uint8_t* __restrict__ cache, int64_t nb1, int64_t nb2, int64_t capacity, int groups_per_row,
    const float* __restrict__ src, int64_t src_nb1, int64_t src_nb2,
    const int32_t* __restrict__ pos, int64_t pos_stride, int n_new, int batch, int* status) {
    const int64_t gi = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gi >= (int64_t)n_new * batch * groups_per_row) return;
    const int g = (int)(gi % groups_per_row);
    const int64_t rw = gi / groups_per_row;  // row (t, b), t fastest
    const int b = (int)(rw / n_new);
    const int t = (int)(rw - (int64_t)b * n_new);
    const int p = pos[t + (int64_t)b * pos_stride];
    if (p < 0 || p >= capacity) {
        if (g == 0) record_status(status, kStatusBadPosition);
        return;
    }
    const float4* s4 =
        reinterpret_cast<const float4*>(reinterpret_cast<const uint8_t*>(src) + t * src_nb1 + b * src_nb2) + 8 * g;
    float x[32];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 v = __ldcs(s4 + i);  // read once
        x[4 * i] = v.x; x[4 * i + 1] = v.y; x[4 * i + 2] = v.z; x[4 * i + 3] = v.w;
    }
    quantize_block_thread<T>(x, cache + b * nb2 + (int64_t)p * nb1 + (int64_t)g * group_bytes(T));
}

// Standalone RoPE: rows of row_len floats (row r at x + r * x_nb1f, out + r * out_nb1f;
// x may equal out).  One thread per pair (or per unrotated element), so a pair
// is read before either of its elements is written.
__global__ void __launch_bounds__(256) rope_kernel(const float* x, int64_t x_nb1f, float* out, int64_t out_nb1f,
                                                   const int32_t* __restrict__ pos, int n_rows, int row_len,
                                                   RopeDev rope) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)n_rows * row_len) return;
    const int r = (int)(idx / row_len), e = (int)(idx % row_len);
    const float* xr = x + r * x_nb1f;
    float* orow = out + r * out_nb1f;
    int k;
    bool first;
    const int pe = rope_pair(rope, e, k, first);
    if (pe < 0) {
        orow[e] = xr[e];
        return;
    }
    if (!first) return;  // the pair's first element writes both
    const float a = xr[e], bb = xr[pe];
    const float2 cs = rope_cs(rope, rope_theta(rope, pos[r], k));
    orow[e] = rope_rotate(a, bb, cs, true);
    orow[pe] = rope_rotate(bb, a, cs, false);
}

template <int T>
__global__ void __launch_bounds__(256) kv_dequant_kernel(
    const uint8_t* __restrict__ cache, int64_t nb1, int64_t nb2, int groups_per_row, int n_rows, int batch,
    float* __restrict__ dst) {
    const int lane = threadIdx.x & 31;
    const int64_t w = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int64_t total = (int64_t)n_rows * batch * groups_per_row;
    if (w >= total) return;
    const int g = (int)(w % groups_per_row);
    const int64_t r = w / groups_per_row;
    const int t = (int)(r % n_rows);
    const int b = (int)(r / n_rows);
    const uint8_t* grp = cache + b * nb2 + (int64_t)t * nb1 + (int64_t)g * group_bytes(T);
    dst[(((int64_t)b * n_rows + t) * groups_per_row + g) * 32 + lane] = dequant_elem<T>(grp, lane);
}

cudaError_t launch_kv_append(cudaStream_t stream, const cvattn_tensor& c, const float* src, int64_t src_nb1,
                             int64_t src_nb2, const int32_t* pos, int64_t pos_stride, int n_new, int batch,
                             int* status, const RopeDev* rope) {
    const RopeDev rp = rope ? *rope : RopeDev{0, 0, 1, 1.0f, 1.0f, 1.0f};
    const int row_elems = c.n_heads * c.head_dim;
    const int groups = row_elems / 32;
    const int64_t rows = (int64_t)n_new * batch;  // one warp per row
    if (rows == 0) return cudaSuccess;
    if (rows > 0x7fffffffLL) return cudaErrorInvalidValue;
    const unsigned grid = (unsigned)((rows + 7) / 8);
    uint8_t* base = static_cast<uint8_t*>(c.data);
    // 4- and 5-bit caches without a RoPE, f32 rows 16-byte aligned, and enough blocks for at
    // least 512 threads per SM: a thread per block.  Smaller launches (the LLM's 256-token
    // prefill calls hold 8,192 blocks) keep a warp per block, which has 32x the threads in flight.
    // q8_0 keeps the warp form too: a thread's 17 two-byte stores, 34 bytes apart across the warp,
    // spread each store instruction over ~34 sectors, and that costs more than the warp form's
    // reductions (DiT step, 1.2 M blocks: 143 us as a thread per block, 94 us as a warp per block).
    const bool block_type = c.type == kQ4_0 || c.type == kQ4_1 || c.type == kQ5_0 || c.type == kQ5_1;
    const int64_t blocks = rows * groups;
    if (block_type && rp.n_dims == 0 && blocks >= (int64_t)current_sm_count() * kAppendBlockThreadsPerSm &&
        ((reinterpret_cast<uintptr_t>(src) | (uintptr_t)src_nb1 | (uintptr_t)src_nb2) & 15) == 0) {
        const unsigned gridb = (unsigned)((blocks + 255) / 256);
        if ((blocks + 255) / 256 > 0x7fffffffLL) return cudaErrorInvalidValue;
#define CVATTN_APPEND_BLOCK_CASE(T)                                                                          \
    case T:                                                                                                  \
        kv_append_block_kernel<T><<<gridb, 256, 0, stream>>>(base, c.nb1, c.nb2, c.ne1, groups, src, src_nb1, \
                                                             src_nb2, pos, pos_stride, n_new, batch, status);  \
        return cudaGetLastError();
        switch (c.type) {
            CVATTN_APPEND_BLOCK_CASE(kQ4_0)
            CVATTN_APPEND_BLOCK_CASE(kQ4_1)
            CVATTN_APPEND_BLOCK_CASE(kQ5_0)
            CVATTN_APPEND_BLOCK_CASE(kQ5_1)
        default: break;
        }
#undef CVATTN_APPEND_BLOCK_CASE
    }
#define CVATTN_APPEND_CASE(T)                                                                              \
    case T:                                                                                                \
        kv_append_kernel<T><<<grid, 256, 0, stream>>>(base, c.nb1, c.nb2, c.ne1, groups, src, src_nb1,     \
                                                      src_nb2, pos, pos_stride, n_new, batch, status, rp); \
        break;
    switch (c.type) {
        CVATTN_APPEND_CASE(kF32)
        CVATTN_APPEND_CASE(kF16)
        CVATTN_APPEND_CASE(kQ4_0)
        CVATTN_APPEND_CASE(kQ4_1)
        CVATTN_APPEND_CASE(kQ5_0)
        CVATTN_APPEND_CASE(kQ5_1)
        CVATTN_APPEND_CASE(kQ8_0)
    default: return cudaErrorInvalidValue;
    }
#undef CVATTN_APPEND_CASE
    return cudaGetLastError();
}

cudaError_t launch_rope(cudaStream_t stream, const RopeDev& rope, const float* x, int64_t x_nb1f, float* out,
                        int64_t out_nb1f, const int32_t* pos, int n_rows, int row_len) {
    const int64_t n = (int64_t)n_rows * row_len;
    if (n == 0) return cudaSuccess;
    rope_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(x, x_nb1f, out, out_nb1f, pos, n_rows, row_len, rope);
    return cudaGetLastError();
}

cudaError_t launch_kv_dequant(cudaStream_t stream, const cvattn_tensor& c, int n_rows, float* dst) {
    const int row_elems = c.n_heads * c.head_dim;
    const int groups = row_elems / 32;
    const int64_t warps = (int64_t)n_rows * c.ne2 * groups;
    if (warps == 0) return cudaSuccess;
    const unsigned grid = (unsigned)((warps + 7) / 8);
    const uint8_t* base = static_cast<const uint8_t*>(c.data);
#define CVATTN_DEQ_CASE(T)                                                                                  \
    case T:                                                                                                 \
        kv_dequant_kernel<T><<<grid, 256, 0, stream>>>(base, c.nb1, c.nb2, groups, n_rows, (int)c.ne2, dst); \
        break;
    switch (c.type) {
        CVATTN_DEQ_CASE(kF32)
        CVATTN_DEQ_CASE(kF16)
        CVATTN_DEQ_CASE(kQ4_0)
        CVATTN_DEQ_CASE(kQ4_1)
        CVATTN_DEQ_CASE(kQ5_0)
        CVATTN_DEQ_CASE(kQ5_1)
        CVATTN_DEQ_CASE(kQ8_0)
    default: return cudaErrorInvalidValue;
    }
#undef CVATTN_DEQ_CASE
    return cudaGetLastError();
}

// ------------------------------------------------------- per-device state

namespace {
constexpr int kMaxDevices = 64;
std::atomic<int> g_sm_count[kMaxDevices];  // 0 = not looked up yet
}  // namespace

int device_sm_count(int device) {
    if (device < 0 || device >= kMaxDevices) return 0;
    int n = g_sm_count[device].load(std::memory_order_relaxed);
    if (n == 0) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
        g_sm_count[device].store(n, std::memory_order_relaxed);
    }
    return n;
}

int current_sm_count() {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    return device_sm_count(dev);
}

// ------------------------------------------------- lengths and tickets

__global__ void fill_lengths_kernel(int32_t* __restrict__ lens, int n, int32_t value, uint32_t* __restrict__ tickets,
                                    int n_tickets) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) lens[i] = value;
    if (i < n_tickets) tickets[i] = 0u;
}

cudaError_t launch_fill_lengths(cudaStream_t stream, int32_t* lens, int n, int32_t value, uint32_t* tickets,
                                int n_tickets) {
    const int m = n > n_tickets ? n : n_tickets;
    if (m <= 0) return cudaSuccess;
    fill_lengths_kernel<<<(m + 255) / 256, 256, 0, stream>>>(lens, n, value, tickets, n_tickets);
    return cudaGetLastError();
}

}  // namespace cvattn
