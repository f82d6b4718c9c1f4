// flash_tc.cuh -- tcgen05/TMEM flash attention for the multi-query paths:
// Qwen2 causal prefill (src/cosyvoice-llm.cpp:62 with the mask of :20-29 /
// :101-108) and DiT attention, cached (src/cosyvoice-graph.cpp:363-366) or
// uncached (:373-377), with the streaming chunk mask of
// src/cosyvoice-token2wav.cpp:285-298 and an arbitrary explicit f16 mask.
//
// Semantics: ggml_flash_attn_ext with scale = 1/sqrt(D), max_bias = 0,
// softcap = 0; query head h reads KV head h / (Hq / Hkv); output f32 in
// ggml's result order [batch][n_q][Hq][D].  Operands are converted to f16 for
// the tensor cores (ggml's CUDA backend does the same); accumulation, softmax
// statistics and the output are f32.
//
// CTA = one tile of 128 query rows x one query head x one batch entry.
//   warps 0-3  softmax + epilogue: thread t owns query row t (TMEM lane t)
//   warps 4-7  producer: K/V tile (128 keys x 64 dims) of any ggml KV type
//              -> f16 in 128B-swizzled shared memory, double-buffered; for an
//              f16 cache one thread issues TMA tensor loads instead
//   warp 8     MMA issuer (one thread): S = Q K^T (M=128, N=128, K=64) into
//              TMEM columns [0,128); O += P V (M=128, N=64, K=128) into TMEM
//              columns [128,192); P comes from shared memory.
// Softmax keeps a reference max per row and only rescales O (in TMEM) when a
// tile raises the row max by more than 2^8, so P <= 256 stays exact in f16
// and most tiles need no correction pass.  Fully masked key tiles (causal /
// chunk) are never loaded.
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "tc.cuh"

namespace cvattn {
namespace fa {

constexpr int BM = 128;
constexpr int BN = 128;
constexpr int D = 64;
constexpr int kThreads = 288;
constexpr int kSoftmax = 128;
constexpr int kProducer = 128;
constexpr int kMmaWarp = 8;
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kSCol = 0;
constexpr uint32_t kOCol = 128;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

// shared memory carve-up (offsets from a 1024-aligned base)
constexpr int kQOff = 0;                 // 16 KB  Q tile, f16, SW128
constexpr int kKOff = 16 * 1024;         // 2 x 16 KB
constexpr int kVOff = 48 * 1024;         // 2 x 16 KB
constexpr int kPOff = 80 * 1024;         // 32 KB: keys 0-63 | keys 64-127
constexpr int kBarOff = 112 * 1024;      // mbarriers, TMEM address, error flag
constexpr int kSmemBytes = kBarOff + 128;  // two CTAs fit one SM (TMEM: 2 x 256 columns)

struct Params {
    const float* q;
    int64_t q_nb_tok, q_nb_head, q_nb_batch;
    float* out;
    const uint8_t* k;
    const uint8_t* v;
    int64_t k_nb1, k_nb2, v_nb1, v_nb2;
    int k_head_bytes, v_head_bytes;
    int n_q, n_kv, Hq, G, batch;
    float scale_log2;
    int mask_mode;
    const uint16_t* mask;
    int64_t mask_nb1, mask_nb2;
    int causal_offset;
    int n_bounds;
    int bounds[CVATTN_MAX_CHUNK_BOUNDS];
    int key_offset, row_offset;
    int use_tma;
    int staged;  // block-quantized K and V: the staged producer's copy form (flash_pipe), 0 = none
    int raw_bytes, raw_k_bytes;  // its chunk form: raw buffer bytes and the K part (whole rows of 64 keys)
    int halves;  // persistent kernel: softmax warpgroups per query tile (1 or 2)
    int* status;
};

struct Bars {
    uint64_t kv_full[2];
    uint64_t kv_empty[2];
    uint64_t q_full;
    uint64_t s_full;
    uint64_t p_ready;
    uint64_t pv_done;
    uint32_t tmem_base;
    int err;
};

__device__ __forceinline__ int block_end(const Params& p, int r) {
    for (int i = 0; i < p.n_bounds; ++i)
        if (p.bounds[i] > r) return p.bounds[i];
    return 0x7fffffff;  // no boundary above r: every column of the chunk region
}

// Number of key tiles a query tile needs (keys beyond it are masked for every row).
__device__ __forceinline__ int key_limit(const Params& p, int i0) {
    const int last = min(i0 + BM, p.n_q) - 1;
    int kmax = p.n_kv;
    if (p.mask_mode == CVATTN_MASK_CAUSAL) {
        kmax = min(kmax, p.causal_offset + last + 1);
    } else if (p.mask_mode == CVATTN_MASK_CHUNK) {
        const int be = block_end(p, last + p.row_offset);
        if (be != 0x7fffffff) kmax = min(kmax, p.key_offset + be);
    }
    return max(kmax, 0);
}

// Convert one head row (64 elements) of a ggml KV type to 64 f16 and store it
// as row r of a 128B-swizzled tile.  Rows past n_kv are zero.
template <int T>
__device__ __forceinline__ void store_row_f16(const uint8_t* src, bool valid, uint8_t* tile, int r) {
    uint32_t w[32];
    if (valid) {
        if constexpr (T == kF16) {
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const uint4 v = *reinterpret_cast<const uint4*>(src + 16 * c);
                w[4 * c] = v.x; w[4 * c + 1] = v.y; w[4 * c + 2] = v.z; w[4 * c + 3] = v.w;
            }
        } else if constexpr (T == kF32) {
#pragma unroll
            for (int c = 0; c < 16; ++c) {
                const float4 v = *reinterpret_cast<const float4*>(src + 16 * c);
                w[2 * c] = tc::pack_f16x2(v.x, v.y);
                w[2 * c + 1] = tc::pack_f16x2(v.z, v.w);
            }
        } else {
            constexpr int GB = group_bytes(T);
#pragma unroll
            for (int blk = 0; blk < 2; ++blk) {
                const uint8_t* g = src + blk * GB;
#pragma unroll
                for (int i = 0; i < 32; i += 2)
                    w[blk * 16 + i / 2] = tc::pack_f16x2(dequant_elem<T>(g, i), dequant_elem<T>(g, i + 1));
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) w[i] = 0u;
    }
#pragma unroll
    for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4*>(tile + tc::sw128_offset(r, c)) = make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
}

// Bounded wait shared by the warp roles: gives up after kWaitBudgetNs or as
// soon as another role has flagged an error, so every thread reaches teardown.
__device__ __forceinline__ bool wait_or_flag(uint64_t* bar, uint32_t parity, Bars* B, int* status, int site) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (;;) {
        if (mbar_try_wait_hint(bar, parity, 1000u)) return true;
        if (*reinterpret_cast<volatile int*>(&B->err)) return false;
        if (global_timer_ns() - t0 > kWaitBudgetNs) {
            record_status(status, kStatusTimeout | (site << 8));
            *reinterpret_cast<volatile int*>(&B->err) = 1;
            return false;
        }
    }
}

template <int KT, int VT>
__global__ void __launch_bounds__(kThreads, 2)
    flash_kernel(const __grid_constant__ Params p, const __grid_constant__ CUtensorMap kmap,
                 const __grid_constant__ CUtensorMap vmap) {
    // 128B-swizzled operand tiles need 1024-byte alignment; the kernel uses no
    // static shared memory, so the dynamic window starts at offset 0.
    extern __shared__ __align__(1024) uint8_t smem[];
    Bars* B = reinterpret_cast<Bars*>(smem + kBarOff);
    if (smem_addr(smem) & 1023u) {
        if (threadIdx.x == 0) record_status(p.status, kStatusTimeout);
        return;
    }
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int i0 = qt * BM;
    const int g = h / p.G;
    const int kmax = key_limit(p, i0);
    const int n_tiles = (kmax + BN - 1) / BN;

    if (tid == 0) {
        mbar_init(&B->kv_full[0], p.use_tma ? 1 : kProducer);
        mbar_init(&B->kv_full[1], p.use_tma ? 1 : kProducer);
        mbar_init(&B->kv_empty[0], 1);
        mbar_init(&B->kv_empty[1], 1);
        mbar_init(&B->q_full, kSoftmax);
        mbar_init(&B->s_full, 1);
        mbar_init(&B->p_ready, kSoftmax);
        mbar_init(&B->pv_done, 1);
        B->err = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        tc::tmem_alloc(&B->tmem_base, kTmemCols);
        tc::tmem_relinquish();
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tmem = B->tmem_base;

    if (warp < 4) {
        // ============================ softmax / epilogue: row r = tid
        const int r = tid;
        const int i = i0 + r;
        const bool row_ok = i < p.n_q;
        {   // Q row -> f16 swizzled
            const float* qrow = p.q + (int64_t)b * p.q_nb_batch + (int64_t)i * p.q_nb_tok + (int64_t)h * p.q_nb_head;
            uint32_t w[32];
#pragma unroll
            for (int c = 0; c < 16; ++c) {
                float4 v = row_ok ? *reinterpret_cast<const float4*>(qrow + 4 * c) : make_float4(0.f, 0.f, 0.f, 0.f);
                const float sc = p.scale_log2;  // scores leave the MMA already in log2 units
                w[2 * c] = tc::pack_f16x2(v.x * sc, v.y * sc);
                w[2 * c + 1] = tc::pack_f16x2(v.z * sc, v.w * sc);
            }
#pragma unroll
            for (int c = 0; c < 8; ++c)
                *reinterpret_cast<uint4*>(smem + kQOff + tc::sw128_offset(r, c)) =
                    make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
            fence_proxy_async_smem();
            mbar_arrive(&B->q_full);
        }
        const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
        const int be = (p.mask_mode == CVATTN_MASK_CHUNK) ? block_end(p, i + p.row_offset) : 0;
        const uint16_t* mrow = (p.mask_mode == CVATTN_MASK_EXPLICIT && row_ok)
                                   ? p.mask + (int64_t)b * p.mask_nb2 + (int64_t)i * p.mask_nb1
                                   : nullptr;
        float m_ref = -INFINITY, l = 0.0f;
        // visible score in log2 units, or -inf
        auto score = [&](uint32_t bits, int j) -> float {
            float s = __uint_as_float(bits);
            bool vis = j < p.n_kv && row_ok;
            if (p.mask_mode == CVATTN_MASK_CAUSAL) vis = vis && (j <= p.causal_offset + i);
            else if (p.mask_mode == CVATTN_MASK_CHUNK) vis = vis && (j < p.key_offset || j - p.key_offset < be);
            else if (p.mask_mode == CVATTN_MASK_EXPLICIT && vis) s += h2f(mrow[j]) * 1.4426950408889634f;
            return vis ? s : -INFINITY;
        };
        // first key index at which some row of this query tile may be masked
        int full_below = p.n_kv;
        if (p.mask_mode == CVATTN_MASK_CAUSAL) full_below = min(full_below, p.causal_offset + i0 + 1);
        else if (p.mask_mode == CVATTN_MASK_CHUNK) {
            const int be0 = block_end(p, i0 + p.row_offset);
            full_below = min(full_below, be0 == 0x7fffffff ? p.n_kv : p.key_offset + be0);
        } else if (p.mask_mode == CVATTN_MASK_EXPLICIT) full_below = 0;
        for (int jt = 0; jt < n_tiles; ++jt) {
            // waits are made warp-uniform: the tcgen05.ld/st below are warp-collective
            if (!__all_sync(0xffffffffu, wait_or_flag(&B->s_full, jt & 1, B, p.status, 1))) break;
            tc::fence_after();
            const bool full = (jt + 1) * BN <= full_below;
            // pass 1: tile max
            float mt = -INFINITY;
            for (int c = 0; c < 4; ++c) {
                uint32_t sv[32];
                tc::tmem_ld32(tmem + lane_base + kSCol + 32 * c, sv);
                tc::tmem_ld_wait();
                if (full) {
#pragma unroll
                    for (int e = 0; e < 32; ++e) mt = fmaxf(mt, __uint_as_float(sv[e]));
                } else {
#pragma unroll
                    for (int e = 0; e < 32; ++e) mt = fmaxf(mt, score(sv[e], jt * BN + 32 * c + e));
                }
            }
            float alpha = 1.0f;
            if (mt > m_ref + kRescaleThreshold) {
                alpha = (m_ref == -INFINITY) ? 0.0f : fast_exp2(m_ref - mt);
                m_ref = mt;
                l *= alpha;
            }
            if (jt > 0) {
                if (!__all_sync(0xffffffffu, wait_or_flag(&B->pv_done, (jt - 1) & 1, B, p.status, 2))) break;
                tc::fence_after();
                // correction O *= alpha in TMEM; tcgen05.ld/st are warp-collective,
                // so the whole warp takes the branch if any of its rows needs it
                if (__any_sync(0xffffffffu, alpha != 1.0f)) {
                    for (int c = 0; c < 2; ++c) {
                        uint32_t ov[32];
                        tc::tmem_ld32(tmem + lane_base + kOCol + 32 * c, ov);
                        tc::tmem_ld_wait();
#pragma unroll
                        for (int e = 0; e < 32; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
                        tc::tmem_st32(tmem + lane_base + kOCol + 32 * c, ov);
                    }
                    tc::tmem_st_wait();
                }
            }
            // pass 2: P = 2^(s - m_ref) -> f16 into the swizzled P tile
            const float mu = (m_ref == -INFINITY) ? 0.0f : m_ref;
            for (int c = 0; c < 4; ++c) {
                uint32_t sv[32];
                tc::tmem_ld32(tmem + lane_base + kSCol + 32 * c, sv);
                tc::tmem_ld_wait();
                uint32_t pw[16];
                if (full) {
                    const float2 neg_mu = make_float2(-mu, -mu), one = make_float2(1.0f, 1.0f);
                    float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
                    for (int e = 0; e < 32; e += 2) {
                        const float2 x = ffma2(make_float2(__uint_as_float(sv[e]), __uint_as_float(sv[e + 1])), one, neg_mu);
                        const float2 pp = make_float2(fast_exp2(x.x), fast_exp2(x.y));
                        acc = ffma2(pp, one, acc);
                        pw[e / 2] = tc::pack_f16x2(pp.x, pp.y);
                    }
                    l += acc.x + acc.y;
                } else {
#pragma unroll
                    for (int e = 0; e < 32; e += 2) {
                        const float s0 = score(sv[e], jt * BN + 32 * c + e);
                        const float s1 = score(sv[e + 1], jt * BN + 32 * c + e + 1);
                        const float p0 = fast_exp2(s0 - mu), p1 = fast_exp2(s1 - mu);
                        l += p0 + p1;
                        pw[e / 2] = tc::pack_f16x2(p0, p1);
                    }
                }
                uint8_t* half = smem + kPOff + (c >> 1) * 16384;
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4)
                    *reinterpret_cast<uint4*>(half + tc::sw128_offset(r, (c & 1) * 4 + q4)) =
                        make_uint4(pw[4 * q4], pw[4 * q4 + 1], pw[4 * q4 + 2], pw[4 * q4 + 3]);
            }
            fence_proxy_async_smem();
            tc::fence_before();
            mbar_arrive(&B->p_ready);
        }
        // epilogue
        float o[64];
        bool have = __all_sync(0xffffffffu, n_tiles > 0 && !*reinterpret_cast<volatile int*>(&B->err));
        if (have && __all_sync(0xffffffffu, wait_or_flag(&B->pv_done, (n_tiles - 1) & 1, B, p.status, 3))) {
            tc::fence_after();
            for (int c = 0; c < 2; ++c) {
                uint32_t ov[32];
                tc::tmem_ld32(tmem + lane_base + kOCol + 32 * c, ov);
                tc::tmem_ld_wait();
#pragma unroll
                for (int e = 0; e < 32; ++e) o[32 * c + e] = __uint_as_float(ov[e]);
            }
        } else {
            have = false;
        }
        if (row_ok) {
            const float inv = (have && l > 0.0f) ? 1.0f / l : 0.0f;
            float* orow = p.out + (((int64_t)b * p.n_q + i) * p.Hq + h) * D;
#pragma unroll
            for (int c = 0; c < 16; ++c)
                *reinterpret_cast<float4*>(orow + 4 * c) =
                    have ? make_float4(o[4 * c] * inv, o[4 * c + 1] * inv, o[4 * c + 2] * inv, o[4 * c + 3] * inv)
                         : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    } else if (warp < 8) {
        // ============================ producer
        const int r = tid - kSoftmax;
        if (p.use_tma) {
            if (r == 0) {
                tc::prefetch_tmap(&kmap);
                tc::prefetch_tmap(&vmap);
                for (int jt = 0; jt < n_tiles; ++jt) {
                    const int s = jt & 1;
                    if (jt >= 2 && !wait_or_flag(&B->kv_empty[s], ((jt >> 1) - 1) & 1, B, p.status, 4)) break;
                    mbar_arrive_expect_tx(&B->kv_full[s], 2 * BN * D * 2);
                    tc::tma_load_3d(smem + kKOff + s * 16384, &kmap, g * D, jt * BN, b, &B->kv_full[s]);
                    tc::tma_load_3d(smem + kVOff + s * 16384, &vmap, g * D, jt * BN, b, &B->kv_full[s]);
                }
            }
        } else {
            const uint8_t* kbase = p.k + (int64_t)b * p.k_nb2 + (int64_t)g * p.k_head_bytes;
            const uint8_t* vbase = p.v + (int64_t)b * p.v_nb2 + (int64_t)g * p.v_head_bytes;
            for (int jt = 0; jt < n_tiles; ++jt) {
                const int s = jt & 1;
                if (jt >= 2 && !wait_or_flag(&B->kv_empty[s], ((jt >> 1) - 1) & 1, B, p.status, 5)) break;
                const int key = jt * BN + r;
                const bool valid = key < p.n_kv;
                store_row_f16<KT>(kbase + (int64_t)key * p.k_nb1, valid, smem + kKOff + s * 16384, r);
                store_row_f16<VT>(vbase + (int64_t)key * p.v_nb1, valid, smem + kVOff + s * 16384, r);
                fence_proxy_async_smem();
                mbar_arrive(&B->kv_full[s]);
            }
        }
    } else if (warp == kMmaWarp && lane == 0) {
        // ============================ MMA issuer
        const uint32_t idesc_s = tc::idesc_f16_f32(128, 128, false);
        const uint32_t idesc_o = tc::idesc_f16_f32(128, 64, true);
        const uint32_t sq = smem_addr(smem + kQOff), sp = smem_addr(smem + kPOff);
        bool ok = n_tiles == 0 || wait_or_flag(&B->q_full, 0, B, p.status, 6);
        for (int jt = 0; ok && jt <= n_tiles; ++jt) {
            if (jt > 0) {
                // P(jt-1) ready and S(jt-1) consumed
                if (!wait_or_flag(&B->p_ready, (jt - 1) & 1, B, p.status, 7)) break;
                tc::fence_after();
                const int sv = (jt - 1) & 1;
                const uint32_t vaddr = smem_addr(smem + kVOff + sv * 16384);
#pragma unroll
                for (int kk = 0; kk < BN / 16; ++kk) {
                    const uint64_t a = tc::sdesc_sw128(sp + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
                    const uint64_t bb = tc::sdesc_sw128(vaddr + kk * 2048, 16, 1024);
                    tc::mma_ss(tmem + kOCol, a, bb, idesc_o, (jt > 1 || kk > 0) ? 1u : 0u);
                }
                tc::mma_commit(&B->pv_done);
                tc::mma_commit(&B->kv_empty[sv]);
            }
            if (jt < n_tiles) {
                const int s = jt & 1;
                if (!wait_or_flag(&B->kv_full[s], (jt >> 1) & 1, B, p.status, 8)) break;
                tc::fence_after();
                const uint32_t kaddr = smem_addr(smem + kKOff + s * 16384);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint64_t a = tc::sdesc_sw128(sq + kk * 32, 16, 1024);
                    const uint64_t bb = tc::sdesc_sw128(kaddr + kk * 32, 16, 1024);
                    tc::mma_ss(tmem + kSCol, a, bb, idesc_s, kk > 0 ? 1u : 0u);
                }
                tc::mma_commit(&B->s_full);
            }
        }
    }

    tc::fence_before();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after();
        tc::tmem_dealloc(tmem, kTmemCols);
    }
}

template <int KT>
cudaError_t launch_for_k(cudaStream_t s, int v_type, const Params& p, const CUtensorMap& km, const CUtensorMap& vm,
                         dim3 grid);
template <> cudaError_t launch_for_k<kF32>(cudaStream_t, int, const Params&, const CUtensorMap&, const CUtensorMap&, dim3);
template <> cudaError_t launch_for_k<kF16>(cudaStream_t, int, const Params&, const CUtensorMap&, const CUtensorMap&, dim3);
template <> cudaError_t launch_for_k<kQ4_0>(cudaStream_t, int, const Params&, const CUtensorMap&, const CUtensorMap&, dim3);
template <> cudaError_t launch_for_k<kQ4_1>(cudaStream_t, int, const Params&, const CUtensorMap&, const CUtensorMap&, dim3);
template <> cudaError_t launch_for_k<kQ5_0>(cudaStream_t, int, const Params&, const CUtensorMap&, const CUtensorMap&, dim3);
template <> cudaError_t launch_for_k<kQ5_1>(cudaStream_t, int, const Params&, const CUtensorMap&, const CUtensorMap&, dim3);
template <> cudaError_t launch_for_k<kQ8_0>(cudaStream_t, int, const Params&, const CUtensorMap&, const CUtensorMap&, dim3);

}  // namespace fa
}  // namespace cvattn
