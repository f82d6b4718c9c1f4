// common.cuh -- shared device helpers for the cvattn kernels (sm_100a only).
//
// Contents: ggml KV block type traits, the bit-exact block quantizers used by
// the append kernels, raw-block readers used by the attention kernels, and thin
// inline-PTX wrappers (mbarrier, bulk async copies, packed f32x2 FMA, tcgen05).
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/cvattn.h"

namespace cvattn {

// ------------------------------------------------------------------ types --

enum : int { kF32 = 0, kF16 = 1, kQ4_0 = 2, kQ4_1 = 3, kQ5_0 = 6, kQ5_1 = 7, kQ8_0 = 8 };

// Block layout of each ggml type (ggml-common.h block_q*; restated from gguf-py
// quants.py:220-401): elements per block, bytes per block, byte offsets of the
// f16 scale d, the f16 min m (the _1 types), the 32-bit high-bit plane qh (q5
// types) and the quants.
template <int T> struct BlockTraits;
template <> struct BlockTraits<kF32>  { static constexpr int QK = 1,  BYTES = 4,  OFF_M = -1, OFF_QH = -1, OFF_QS = 0; static constexpr bool HAS_MIN = false; };
template <> struct BlockTraits<kF16>  { static constexpr int QK = 1,  BYTES = 2,  OFF_M = -1, OFF_QH = -1, OFF_QS = 0; static constexpr bool HAS_MIN = false; };
template <> struct BlockTraits<kQ4_0> { static constexpr int QK = 32, BYTES = 18, OFF_M = -1, OFF_QH = -1, OFF_QS = 2; static constexpr bool HAS_MIN = false; };
template <> struct BlockTraits<kQ4_1> { static constexpr int QK = 32, BYTES = 20, OFF_M = 2,  OFF_QH = -1, OFF_QS = 4; static constexpr bool HAS_MIN = true; };
template <> struct BlockTraits<kQ5_0> { static constexpr int QK = 32, BYTES = 22, OFF_M = -1, OFF_QH = 2,  OFF_QS = 6; static constexpr bool HAS_MIN = false; };
template <> struct BlockTraits<kQ5_1> { static constexpr int QK = 32, BYTES = 24, OFF_M = 2,  OFF_QH = 4,  OFF_QS = 8; static constexpr bool HAS_MIN = true; };
template <> struct BlockTraits<kQ8_0> { static constexpr int QK = 32, BYTES = 34, OFF_M = -1, OFF_QH = -1, OFF_QS = 2; static constexpr bool HAS_MIN = false; };

// Bytes of one head (head_dim elements) and of n elements.
template <int T> __host__ __device__ constexpr int head_bytes(int head_dim) {
    return head_dim / BlockTraits<T>::QK * BlockTraits<T>::BYTES;
}

__host__ __device__ constexpr int64_t type_row_bytes(int t, int64_t n) {
    switch (t) {
    case kF32: return n * 4;
    case kF16: return n * 2;
    case kQ4_0: return n / 32 * 18;
    case kQ4_1: return n / 32 * 20;
    case kQ5_0: return n / 32 * 22;
    case kQ5_1: return n / 32 * 24;
    case kQ8_0: return n / 32 * 34;
    default: return 0;
    }
}

__host__ __device__ constexpr bool type_known(int t) {
    return t == kF32 || t == kF16 || t == kQ4_0 || t == kQ4_1 || t == kQ5_0 || t == kQ5_1 || t == kQ8_0;
}

// Device status word codes (cvattn_context_sync_status detail).
enum : int {
    kStatusBadPosition = 1,   // append position outside [0, capacity)
    kStatusBadLength = 2,     // kv_len outside [0, capacity] or above max_kv_len
    kStatusTimeout = 3,       // bounded mbarrier wait gave up
};

__device__ __forceinline__ void record_status(int* status, int code) {
    if (status) atomicCAS(status, 0, code);
}

// --------------------------------------------------------------- f16 bits --

__device__ __forceinline__ float h2f(uint16_t b) { return __half2float(__ushort_as_half(b)); }
__device__ __forceinline__ uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }

// ------------------------------------------------- warp-level quantizers --
//
// One warp quantizes one 32-element block; lane j holds element j.  The
// arithmetic follows ggml's reference quantizers as restated by gguf-py
// quants.py (Q4_0 :220-252, Q4_1 :254-289, Q5_0 :291-331, Q5_1 :333-376,
// Q8_0 :378-401): every product / sum / quotient is a single IEEE fp32
// operation (explicit _rn intrinsics, no FMA contraction), d = max/-8 etc. is
// divided exactly, and the reciprocal id = 1/d is an IEEE division.
// Reductions reproduce ggml's sequential "first element wins" scans: the
// (value, lane) pair with the smaller lane wins a tie, so -0.0 vs +0.0 ties
// resolve as ggml's loops do.

__device__ __forceinline__ float warp_max_abs(float a) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    return a;
}

// Signed value of largest magnitude, first occurrence: the largest magnitude by
// a max reduction, then the lowest lane holding it (a ballot) gives the value.
__device__ __forceinline__ float warp_signed_absmax(float x, int lane) {
    (void)lane;
    const float a = warp_max_abs(fabsf(x));
    // ggml keeps max = 0.0f until some |v| > 0: an all-zero block gives +0.0
    if (a == 0.0f) return 0.0f;
    const uint32_t hit = __ballot_sync(0xffffffffu, fabsf(x) == a);
    return __shfl_sync(0xffffffffu, x, __ffs(hit) - 1);
}

// Minimum / maximum, first occurrence (values that compare equal, -0.0 and +0.0,
// resolve to the lower lane, as ggml's sequential scans do).
__device__ __forceinline__ void warp_min_max(float x, int lane, float& mn, float& mx) {
    (void)lane;
    float vmin = x, vmax = x;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        vmin = fminf(vmin, __shfl_xor_sync(0xffffffffu, vmin, o));
        vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, o));
    }
    const uint32_t hmin = __ballot_sync(0xffffffffu, x == vmin);
    const uint32_t hmax = __ballot_sync(0xffffffffu, x == vmax);
    mn = __shfl_sync(0xffffffffu, x, __ffs(hmin) - 1);
    mx = __shfl_sync(0xffffffffu, x, __ffs(hmax) - 1);
}

__device__ __forceinline__ void store_u16(uint8_t* p, uint16_t v) {
    // block starts are 2-byte aligned for every ggml block type
    *reinterpret_cast<uint16_t*>(p) = v;
}

// Quantize element x (lane j of a warp) of one block into dst[0, BYTES) and, when
// dst2 is not null, the same bytes into dst2 (one computation, two stores).
// Every lane must call it (warp-collective); dst2 is the same on every lane.
template <int T>
__device__ __forceinline__ void quantize_block_warp(float x, uint8_t* dst, int lane, uint8_t* dst2 = nullptr) {
    if constexpr (T == kQ8_0) {
        float amax = warp_max_abs(fabsf(x));
        float d = __fdiv_rn(amax, 127.0f);
        float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        int q = (int)roundf(__fmul_rn(x, id));          // ties away from zero (np_roundf)
        const uint16_t dh = f2h(d);
        if (lane == 0) store_u16(dst, dh);
        dst[2 + lane] = (uint8_t)(int8_t)q;
        if (dst2) {
            if (lane == 0) store_u16(dst2, dh);
            dst2[2 + lane] = (uint8_t)(int8_t)q;
        }
    } else if constexpr (T == kQ4_0 || T == kQ5_0) {
        constexpr float kDiv = T == kQ4_0 ? -8.0f : -16.0f;
        constexpr float kOff = T == kQ4_0 ? 8.5f : 16.5f;
        constexpr int kMax = T == kQ4_0 ? 15 : 31;
        float mx = warp_signed_absmax(x, lane);
        float d = __fdiv_rn(mx, kDiv);
        float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        int q = (int)truncf(__fadd_rn(__fmul_rn(x, id), kOff));
        q = min(kMax, max(0, q));
        int hi = __shfl_down_sync(0xffffffffu, q, 16);
        uint32_t qh = 0;
        if constexpr (T == kQ5_0) qh = __ballot_sync(0xffffffffu, (q >> 4) & 1);
        const uint16_t dh = f2h(d);
        const uint8_t qs = (uint8_t)((q & 15) | ((hi & 15) << 4));
        for (int k = 0; k < 2; ++k) {
            uint8_t* o = k ? dst2 : dst;
            if (!o) break;
            if (lane == 0) store_u16(o, dh);
            if constexpr (T == kQ5_0)
                if (lane == 0) { store_u16(o + 2, (uint16_t)qh); store_u16(o + 4, (uint16_t)(qh >> 16)); }
            if (lane < 16) o[BlockTraits<T>::OFF_QS + lane] = qs;
        }
    } else if constexpr (T == kQ4_1 || T == kQ5_1) {
        constexpr float kDiv = T == kQ4_1 ? 15.0f : 31.0f;
        constexpr int kMax = T == kQ4_1 ? 15 : 31;
        float mn, mx;
        warp_min_max(x, lane, mn, mx);
        float d = __fdiv_rn(__fsub_rn(mx, mn), kDiv);
        float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        int q = (int)truncf(__fadd_rn(__fmul_rn(__fsub_rn(x, mn), id), 0.5f));
        q = min(kMax, max(0, q));
        int hi = __shfl_down_sync(0xffffffffu, q, 16);
        uint32_t qh = 0;
        if constexpr (T == kQ5_1) qh = __ballot_sync(0xffffffffu, (q >> 4) & 1);
        const uint16_t dh = f2h(d), mh = f2h(mn);
        const uint8_t qs = (uint8_t)((q & 15) | ((hi & 15) << 4));
        for (int k = 0; k < 2; ++k) {
            uint8_t* o = k ? dst2 : dst;
            if (!o) break;
            if (lane == 0) { store_u16(o, dh); store_u16(o + 2, mh); }
            if constexpr (T == kQ5_1)
                if (lane == 0) { store_u16(o + 4, (uint16_t)qh); store_u16(o + 6, (uint16_t)(qh >> 16)); }
            if (lane < 16) o[BlockTraits<T>::OFF_QS + lane] = qs;
        }
    } else if constexpr (T == kF16) {
        const uint16_t h = f2h(x);
        store_u16(dst + 2 * lane, h);
        if (dst2) store_u16(dst2 + 2 * lane, h);
    } else {  // kF32
        reinterpret_cast<float*>(dst)[lane] = x;
        if (dst2) reinterpret_cast<float*>(dst2)[lane] = x;
    }
}

// Quantize one 32-element group (a block for the quantized types, 32
// consecutive elements for F16/F32) to dst_a and, if non-null, also dst_b.
template <int T>
__device__ __forceinline__ void quantize_group_warp2(float x, uint8_t* dst_a, uint8_t* dst_b, int lane) {
    quantize_block_warp<T>(x, dst_a, lane, dst_b);
}

// Runtime-type dispatch of the warp quantizer (group = 32 elements).
__device__ __forceinline__ void quantize_group_rt(int t, float x, uint8_t* dst, int lane) {
    switch (t) {
    case kQ8_0: quantize_block_warp<kQ8_0>(x, dst, lane); break;
    case kQ4_0: quantize_block_warp<kQ4_0>(x, dst, lane); break;
    case kQ4_1: quantize_block_warp<kQ4_1>(x, dst, lane); break;
    case kQ5_0: quantize_block_warp<kQ5_0>(x, dst, lane); break;
    case kQ5_1: quantize_block_warp<kQ5_1>(x, dst, lane); break;
    case kF16:  quantize_block_warp<kF16>(x, dst, lane); break;
    default:    quantize_block_warp<kF32>(x, dst, lane); break;
    }
}

// Bytes a 32-element group occupies in a row of type t.
__host__ __device__ constexpr int group_bytes(int t) {
    switch (t) {
    case kF32: return 128;
    case kF16: return 64;
    case kQ4_0: return 18;
    case kQ4_1: return 20;
    case kQ5_0: return 22;
    case kQ5_1: return 24;
    case kQ8_0: return 34;
    default: return 0;
    }
}

// ----------------------------------------------------------- dequantizers --
//
// Element i (0..31) of a 32-element group as gguf-py's dequantize_blocks
// computes it: d*q for the symmetric types, d*q + m for the _1 types (d*q is
// exact in fp32 so an FMA gives the same value).

template <int T>
__device__ __forceinline__ float dequant_elem(const uint8_t* g, int i) {
    if constexpr (T == kF32) {
        return reinterpret_cast<const float*>(g)[i];
    } else if constexpr (T == kF16) {
        return h2f(reinterpret_cast<const uint16_t*>(g)[i]);
    } else {
        using B = BlockTraits<T>;
        float d = h2f(*reinterpret_cast<const uint16_t*>(g));
        if constexpr (T == kQ8_0) {
            return d * (float)(int8_t)g[B::OFF_QS + i];
        } else {
            int nib = (g[B::OFF_QS + (i & 15)] >> ((i >> 4) * 4)) & 15;
            int q = nib;
            if constexpr (B::OFF_QH >= 0) {
                uint32_t qh = (uint32_t)*reinterpret_cast<const uint16_t*>(g + B::OFF_QH) |
                              ((uint32_t)*reinterpret_cast<const uint16_t*>(g + B::OFF_QH + 2) << 16);
                q |= ((qh >> i) & 1) << 4;
            }
            if constexpr (B::HAS_MIN) {
                float m = h2f(*reinterpret_cast<const uint16_t*>(g + B::OFF_M));
                return d * (float)q + m;
            } else {
                constexpr int off = B::OFF_QH >= 0 ? 16 : 8;
                return d * (float)(q - off);
            }
        }
    }
}

__device__ __forceinline__ float dequant_elem_rt(int t, const uint8_t* g, int i) {
    switch (t) {
    case kQ8_0: return dequant_elem<kQ8_0>(g, i);
    case kQ4_0: return dequant_elem<kQ4_0>(g, i);
    case kQ4_1: return dequant_elem<kQ4_1>(g, i);
    case kQ5_0: return dequant_elem<kQ5_0>(g, i);
    case kQ5_1: return dequant_elem<kQ5_1>(g, i);
    case kF16:  return dequant_elem<kF16>(g, i);
    default:    return dequant_elem<kF32>(g, i);
    }
}

// ----------------------------------------------------------------- f32x2 --

// Packed fp32 FMA (sm_100+): two independent IEEE fp32 FMAs per instruction.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    unsigned long long ra = *reinterpret_cast<unsigned long long*>(&a);
    unsigned long long rb = *reinterpret_cast<unsigned long long*>(&b);
    unsigned long long rc = *reinterpret_cast<unsigned long long*>(&c);
    unsigned long long rd;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(rd) : "l"(ra), "l"(rb), "l"(rc));
    return *reinterpret_cast<float2*>(&rd);
}

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// -------------------------------------------------------------- mbarrier --

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(smem_addr(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(smem_addr(bar)), "r"(parity) : "memory");
    return ok != 0;
}

// Programmatic dependent launch.  launch_dependents lets the next kernel in the
// stream (launched with programmatic stream serialization) start its own
// prologue on SMs this grid frees; wait blocks until every prerequisite grid
// has completed and its memory is visible (immediately after a kernel that
// never triggers).  Everything that reads inputs or writes outputs sits behind
// the wait.
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Non-blocking probe of a phase (for issuers that poll several barriers).
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(smem_addr(bar)), "r"(parity) : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// try_wait with an explicit suspend-time hint (ns) so one poll never sleeps long.
__device__ __forceinline__ bool mbar_try_wait_hint(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns) : "memory");
    return ok != 0;
}

// Wall-clock budget of one bounded wait.  A wait that runs out records
// kStatusTimeout plus its call-site code (status word = 0x100 * site + 3) and
// returns false; callers then stop issuing work and fall through to teardown.
constexpr uint64_t kWaitBudgetNs = 2000000000ull;

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status, int site = 0) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (;;) {
        if (mbar_try_wait_hint(bar, parity, 1000u)) return true;
        if (global_timer_ns() - t0 > kWaitBudgetNs) {
            record_status(status, kStatusTimeout | (site << 8));
            return false;
        }
    }
}

// ------------------------------------------------------ bulk async copies --

// Global -> shared bulk copy (TMA engine, non-tensor form).  Both addresses
// 16-byte aligned, bytes a multiple of 16.  Completion is signalled on bar as
// transaction bytes.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        :: "r"(smem_addr(smem_dst)), "l"(gmem_src), "r"(bytes), "r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

}  // namespace cvattn
