// decode_tc.cuh -- tensor-core (tcgen05 / TMEM) split-KV decode for the
// Qwen2 shape (2 KV heads x head_dim 64, up to 8 query heads per KV head).
//
// Same semantics, arguments, workspace and combine as decode.cuh (one query
// row per sequence, ggml_flash_attn_ext with f32 precision,
// src/cosyvoice-kv-cache.cpp:379-386, fused update_cache append :316,322),
// but both contractions run on the 5th-generation tensor cores while keeping
// fp32-level accuracy:
//   - every ggml block stores integer quants q and an f16 scale d (and min m);
//     q is exact in f16, so K and V tiles hold q itself (the f16 value for an
//     f16 cache) and the scales stay aside in fp32;
//   - Q is split per head into f16 hi + lo parts after an exact power-of-two
//     scaling, so Q.q = (Q_hi + Q_lo).q with products exact in the fp32
//     accumulator; S = d0*(Sblk0) + d1*(Sblk1) (+ m * sum Q) per key.
//   - P' = p * d_V (scaled by an exact power of two per group column) is
//     split into hi + lo f16 the same way for O = sum_k P'(k) q_V(k).
// CTA = one sequence x one chunk of 128 positions (both KV heads):
//   1. one thread streams the chunk's raw K/V rows HBM->SMEM (cp.async.bulk);
//   2. all warps convert the raw blocks to 128B-swizzled f16 tiles + scales;
//   3. tcgen05.mma S^T[key][h|hi,lo] = K_g . Q_g^T (M=128 keys, N=16, K=16 x 4)
//      into TMEM, one accumulator per (kv head, 32-element group);
//   4. thread = key: scores from TMEM, chunk max / sum by warp shuffles,
//      P' row (64 f16: kv head x group x hi/lo x 8 heads) into SMEM;
//   5. tcgen05.mma O^T[(g,dim)][n] = V^T . P' (M=128 (kv head, dim) rows,
//      N=64, K=128 keys; both operands MN-major) into TMEM;
//   6. thread = (kv head, dim) row reads its group's 16 columns; partials and
//      the last-CTA log-sum-exp combine are as in decode.cuh.
#pragma once

#include "decode.cuh"
#include "tc.cuh"

namespace cvattn {
namespace dtc {

using dec::Args;

constexpr int kD = 64;
constexpr int kC = 128;          // positions per CTA (the MMA M dimension)
constexpr int kThreads = 256;
constexpr int kHP = 8;           // query heads per KV head, padded
constexpr uint32_t kTmemCols = 128;
constexpr uint32_t kSCol = 0;    // 4 accumulators x 16 columns
constexpr uint32_t kOCol = 64;   // 64 columns

__host__ __device__ constexpr int round_up(int x, int a) { return (x + a - 1) / a * a; }

struct Smem {
    int raw, ktile, vtile, qtile, dk, mk, dv, mv, qsum, esc, vsc, red, ml, pm, bars, total;
    __host__ __device__ Smem(int rowK, int rowV, bool k_min, bool v_min) {
        int o = 0;
        raw = o;   o += round_up(kC * (rowK + rowV), 1024);  // raw chunk, later the P' tile (16 KB)
        ktile = o; o += 2 * 16384;                           // [g][128 keys x 64 dims] f16, SW128 K-major
        vtile = o; o += 2 * 16384;                           // [g][128 keys x 64 dims] f16, MN-major atoms
        qtile = o; o += 2 * 2048;                            // [g][16 rows x 64 dims] f16, SW128 K-major
        dk = o;    o += 2 * 2 * kC * 4;
        mk = o;    o += k_min ? 2 * 2 * kC * 4 : 0;
        dv = o;    o += 2 * 2 * kC * 4;
        mv = o;    o += v_min ? 2 * 2 * kC * 4 : 0;
        qsum = o;  o += 2 * 2 * kHP * 4;
        esc = o;   o += 2 * kHP * 4;
        vsc = o;   o += 16;
        red = o;   o += 8 * 32 * 4;
        ml = o;    o += 2 * kHP * 2 * 4;
        pm = o;    o += 2 * 2 * kHP * 4;
        bars = o;  o += 64;
        total = round_up(o, 128);
    }
};

// ------------------------------------------------- raw group -> f16 exact --

__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
    __half2 r = __hsub2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
}

constexpr uint32_t kF16x2_1024 = 0x64006400u;  // (1024, 1024)
constexpr uint32_t kF16x2_1032 = 0x64086408u;  // (1032, 1032)
constexpr uint32_t kF16x2_1040 = 0x64106410u;  // (1040, 1040)
constexpr uint32_t kF16x2_1152 = 0x64806480u;  // (1152, 1152)

// 32 elements of one group as exact f16 raw values (w[i] = elements 2i, 2i+1)
// plus the group's scale and min: element = d * raw + m.  The raw values are
// centred (q - 8 for 4-bit, q - 16 for 5-bit quants; q8_0 is signed already)
// and the min absorbs the offset (m = min + 8 d or min + 16 d), so sums of
// d * raw over many positions do not cancel against the min term.
template <int T>
__device__ __forceinline__ void convert_group(const uint8_t* g, uint32_t (&w)[16], float& d, float& m) {
    if constexpr (T == kF16) {
#pragma unroll
        for (int i = 0; i < 16; ++i) w[i] = reinterpret_cast<const uint32_t*>(g)[i];
        d = 1.0f;
        m = 0.0f;
    } else if constexpr (T == kQ8_0) {
        d = h2f(*reinterpret_cast<const uint16_t*>(g));
        m = 0.0f;
        // 32-bit loads of the (2-byte aligned) quants; byte pairs never straddle
        // a word, so one PRMT per pair builds (1024 + b0 ^ 0x80, 1024 + b1 ^ 0x80).
        const uint8_t* qs = g + 2;
        const uint32_t* wp = reinterpret_cast<const uint32_t*>(reinterpret_cast<uintptr_t>(qs) & ~uintptr_t(3));
        if (reinterpret_cast<uintptr_t>(qs) & 2) {  // pair i: high half of word (i+1)/2 when i is even
            uint32_t x[9];
#pragma unroll
            for (int j = 0; j < 9; ++j) x[j] = wp[j] ^ 0x80808080u;
#pragma unroll
            for (int i = 0; i < 16; ++i)
                w[i] = hsub2_u32(__byte_perm(x[(i + 1) >> 1], 0x6464u, (i & 1) ? 0x5140u : 0x5342u), kF16x2_1152);
        } else {
            uint32_t x[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) x[j] = wp[j] ^ 0x80808080u;
#pragma unroll
            for (int i = 0; i < 16; ++i)
                w[i] = hsub2_u32(__byte_perm(x[i >> 1], 0x6464u, (i & 1) ? 0x5342u : 0x5140u), kF16x2_1152);
        }
    } else {
        using B = BlockTraits<T>;
        d = h2f(*reinterpret_cast<const uint16_t*>(g));
        constexpr float kCentre = B::OFF_QH >= 0 ? 16.0f : 8.0f;
        m = B::HAS_MIN ? fmaf(kCentre, d, h2f(*reinterpret_cast<const uint16_t*>(g + 2))) : 0.0f;
        uint32_t qh = 0;
        if constexpr (B::OFF_QH >= 0)
            qh = (uint32_t)*reinterpret_cast<const uint16_t*>(g + B::OFF_QH) |
                 ((uint32_t)*reinterpret_cast<const uint16_t*>(g + B::OFF_QH + 2) << 16);
        constexpr uint32_t bias = B::OFF_QH >= 0 ? kF16x2_1040 : kF16x2_1032;
        // Quant byte pair p (bytes 2p, 2p+1) spread to [b0, 0, b1, 0]: its low nibbles
        // are elements 2p, 2p+1, its high nibbles elements 16 + 2p, 17 + 2p.  The
        // quants start 2-byte aligned, so a pair never straddles a 32-bit word.
        const uint8_t* qs = g + B::OFF_QS;
        const uint32_t* wp = reinterpret_cast<const uint32_t*>(reinterpret_cast<uintptr_t>(qs) & ~uintptr_t(3));
        uint32_t r[8];
        if (reinterpret_cast<uintptr_t>(qs) & 2) {  // pair p: high half of word (p+1)/2 when p is even
            uint32_t x[5];
#pragma unroll
            for (int j = 0; j < 5; ++j) x[j] = wp[j];
#pragma unroll
            for (int p = 0; p < 8; ++p) r[p] = __byte_perm(x[(p + 1) >> 1], 0u, (p & 1) ? 0x4140u : 0x4342u);
        } else {
            uint32_t x[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) x[j] = wp[j];
#pragma unroll
            for (int p = 0; p < 8; ++p) r[p] = __byte_perm(x[p >> 1], 0u, (p & 1) ? 0x4342u : 0x4140u);
        }
#pragma unroll
        for (int p = 0; p < 8; ++p) {
            uint32_t lo = (r[p] & 0x000F000Fu) | 0x64006400u;         // (1024 + nibble, 1024 + nibble)
            uint32_t hi = ((r[p] >> 4) & 0x000F000Fu) | 0x64006400u;
            if constexpr (B::OFF_QH >= 0) {  // 5th bits: element e takes bit e of qh, at bit 4 / 20 of its pair
                lo |= (((qh >> (2 * p)) & 3u) * 0x80010u) & 0x00100010u;
                hi |= (((qh >> (16 + 2 * p)) & 3u) * 0x80010u) & 0x00100010u;
            }
            w[p] = hsub2_u32(lo, bias);
            w[8 + p] = hsub2_u32(hi, bias);
        }
    }
}

__device__ __forceinline__ float pow2f(int e) {  // exact 2^e, e in [-126, 127]
    return __int_as_float((127 + e) << 23);
}

// Power-of-two factor bringing a positive magnitude into [128, 256).
__device__ __forceinline__ int norm_exp(float amax) {
    if (!(amax > 0.0f)) return 0;
    const int ex = ((__float_as_int(amax) >> 23) & 0xff) - 127;
    int e = 7 - ex;
    return e > 100 ? 100 : (e < -100 ? -100 : e);
}

template <int KT, int VT>
__global__ void __launch_bounds__(kThreads, 2) decode_tc_kernel(const Args a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int seq = blockIdx.y, chunk = blockIdx.x;
    const int G = a.G, Hq = a.Hq;
    constexpr int GBK = group_bytes(KT), GBV = group_bytes(VT);
    constexpr int headK = 2 * GBK, headV = 2 * GBV, rowK = 2 * headK, rowV = 2 * headV;
    constexpr bool K_MIN = BlockTraits<KT>::HAS_MIN, V_MIN = BlockTraits<VT>::HAS_MIN;
    const Smem L(rowK, rowV, K_MIN, V_MIN);
    const bool emit_partial = (a.flags & CVATTN_DECODE_EMIT_PARTIAL) != 0;

    const int len = a.kv_len[seq];
    float* out = a.out + (int64_t)seq * a.out_seq_stride;
    if (len <= 0 || len > a.capacity || len > a.max_kv_len) {
        if (chunk == 0) {
            for (int i = tid; i < Hq * kD; i += kThreads) out[i] = 0.0f;
            if (emit_partial)
                for (int i = tid; i < Hq; i += kThreads) {
                    a.partial_ml[((int64_t)seq * Hq + i) * 2] = -INFINITY;
                    a.partial_ml[((int64_t)seq * Hq + i) * 2 + 1] = 0.0f;
                }
            if (len != 0 && tid == 0) record_status(a.status, kStatusBadLength);
        }
        return;
    }
    const int p0 = chunk * kC;
    if (p0 >= len) return;
    if (smem_addr(smem) & 1023u) {  // swizzled tiles need 1024-byte alignment
        if (tid == 0) record_status(a.status, kStatusTimeout | (9 << 8));
        return;
    }
    const int n = min(kC, len - p0);
    const int nchunks = (len + kC - 1) / kC;

    uint8_t* Kraw = smem + L.raw;
    uint8_t* Vraw = Kraw + kC * rowK;
    uint8_t* ktile = smem + L.ktile;
    uint8_t* vtile = smem + L.vtile;
    uint8_t* qtile = smem + L.qtile;
    uint8_t* ptile = smem + L.raw;  // aliases the raw chunk after conversion
    float* dk = reinterpret_cast<float*>(smem + L.dk);
    float* mk = reinterpret_cast<float*>(smem + L.mk);
    float* dv = reinterpret_cast<float*>(smem + L.dv);
    float* mv = reinterpret_cast<float*>(smem + L.mv);
    float* qsum = reinterpret_cast<float*>(smem + L.qsum);
    float* esc = reinterpret_cast<float*>(smem + L.esc);
    uint32_t* vsc = reinterpret_cast<uint32_t*>(smem + L.vsc);
    float* red = reinterpret_cast<float*>(smem + L.red);
    float* ML = reinterpret_cast<float*>(smem + L.ml);
    float* PM = reinterpret_cast<float*>(smem + L.pm);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);  // 0 bulk, 1 S done, 2 O done
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.bars + 32);

    const uint8_t* kb = a.k_seq_ptrs ? reinterpret_cast<const uint8_t*>(a.k_seq_ptrs[seq]) : a.k_base + seq * a.k_nb2;
    const uint8_t* vb = a.v_seq_ptrs ? reinterpret_cast<const uint8_t*>(a.v_seq_ptrs[seq]) : a.v_base + seq * a.v_nb2;

    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        mbar_init(&bars[2], 1);
        fence_mbar_init();
    }
    if (tid < 4) vsc[tid] = 0u;
    if (warp == 0) {
        tc::tmem_alloc(tmem_slot, kTmemCols);
        tc::tmem_relinquish();
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tmem = *tmem_slot;

    // ---- 1. raw chunk -> SMEM
    const uint32_t kbytes = (uint32_t)(n * rowK), vbytes = (uint32_t)(n * rowV);
    const uint8_t* ksrc = kb + (int64_t)p0 * rowK;
    const uint8_t* vsrc = vb + (int64_t)p0 * rowV;
    const uint32_t kbulk = ((reinterpret_cast<uintptr_t>(ksrc) & 15) == 0) ? (kbytes & ~15u) : 0u;
    const uint32_t vbulk = ((reinterpret_cast<uintptr_t>(vsrc) & 15) == 0) ? (vbytes & ~15u) : 0u;
    if (tid == 0) {
        mbar_arrive_expect_tx(&bars[0], kbulk + vbulk);
        if (kbulk) bulk_g2s(Kraw, ksrc, kbulk, &bars[0]);
        if (vbulk) bulk_g2s(Vraw, vsrc, vbulk, &bars[0]);
    }
    for (uint32_t i = kbulk / 2 + tid; i < kbytes / 2; i += kThreads)
        reinterpret_cast<uint16_t*>(Kraw)[i] = reinterpret_cast<const uint16_t*>(ksrc)[i];
    for (uint32_t i = vbulk / 2 + tid; i < vbytes / 2; i += kThreads)
        reinterpret_cast<uint16_t*>(Vraw)[i] = reinterpret_cast<const uint16_t*>(vsrc)[i];

    // ---- 2. Q hi/lo tiles: thread = (kv head g, tile row, 8-dim chunk)
    {
        const int g = tid >> 7, row = (tid >> 3) & 15, c = tid & 7;
        const int h = row & 7;
        const bool lo_row = row >= 8;
        float x[8];
        if (h < G) {
            const float* qr = a.q + (int64_t)seq * a.q_seq_stride + (g * G + h) * kD + 8 * c;
            const float4 u = *reinterpret_cast<const float4*>(qr);
            const float4 v = *reinterpret_cast<const float4*>(qr + 4);
            x[0] = u.x; x[1] = u.y; x[2] = u.z; x[3] = u.w; x[4] = v.x; x[5] = v.y; x[6] = v.z; x[7] = v.w;
        } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) x[e] = 0.0f;
        }
        float am = 0.0f, part = 0.0f;
#pragma unroll
        for (int e = 0; e < 8; ++e) { am = fmaxf(am, fabsf(x[e])); part += x[e]; }
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
        const int ex = norm_exp(am);
        const float sc = pow2f(ex);
        uint32_t wv[4];
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
            const float y0 = x[e] * sc, y1 = x[e + 1] * sc;
            const __half h0 = __float2half_rn(y0), h1 = __float2half_rn(y1);
            if (!lo_row) {
                wv[e / 2] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
            } else {
                wv[e / 2] = tc::pack_f16x2(y0 - __half2float(h0), y1 - __half2float(h1));
            }
        }
        *reinterpret_cast<uint4*>(qtile + g * 2048 + tc::sw128_offset(row, c)) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
        if (!lo_row && c == 0) esc[g * kHP + h] = pow2f(-ex);
        if constexpr (K_MIN) {
            part += __shfl_xor_sync(0xffffffffu, part, 1);
            part += __shfl_xor_sync(0xffffffffu, part, 2);
            if (!lo_row && (c & 3) == 0) qsum[(g * 2 + (c >> 2)) * kHP + h] = part;
        }
    }

    const bool bulk_ok = mbar_wait(&bars[0], 0, a.status, 1);
    if (!__syncthreads_and(bulk_ok)) goto teardown;

    // ---- fused append of this step's row (position len-1)
    if (a.k_new && chunk == nchunks - 1) {
        const int r = len - 1 - p0;
        for (int gi = warp; gi < 8; gi += kThreads / 32) {
            const bool isv = gi >= 4;
            const int g2 = gi & 3;
            const float xv = (isv ? a.v_new : a.k_new)[(int64_t)seq * 2 * kD + g2 * 32 + lane];
            if (!isv) {
                quantize_block_warp<KT>(xv, Kraw + r * rowK + g2 * GBK, lane);
                quantize_block_warp<KT>(xv, const_cast<uint8_t*>(kb) + (int64_t)(len - 1) * rowK + g2 * GBK, lane);
            } else {
                quantize_block_warp<VT>(xv, Vraw + r * rowV + g2 * GBV, lane);
                quantize_block_warp<VT>(xv, const_cast<uint8_t*>(vb) + (int64_t)(len - 1) * rowV + g2 * GBV, lane);
            }
        }
        __syncthreads();
    }

    // ---- 3. raw groups -> f16 exact tiles + scales; items (K|V, g, blk, key)
#pragma unroll
    for (int it = 0; it < 4; ++it) {
        const int item = tid + it * kThreads;
        const int key = item & (kC - 1);
        const int rest = item >> 7;
        const int g = (rest >> 1) & 1, blk = rest & 1;
        uint32_t w[16];
        float d = 0.0f, m = 0.0f;
        if (it < 2) {
            if (key < n) convert_group<KT>(Kraw + key * rowK + g * headK + blk * GBK, w, d, m);
            else {
#pragma unroll
                for (int i = 0; i < 16; ++i) w[i] = 0u;
            }
            uint8_t* tile = ktile + g * 16384;
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4)
                *reinterpret_cast<uint4*>(tile + tc::sw128_offset(key, blk * 4 + c4)) =
                    make_uint4(w[4 * c4], w[4 * c4 + 1], w[4 * c4 + 2], w[4 * c4 + 3]);
            dk[(g * 2 + blk) * kC + key] = d;
            if constexpr (K_MIN) mk[(g * 2 + blk) * kC + key] = m;
        } else {
            if (key < n) convert_group<VT>(Vraw + key * rowV + g * headV + blk * GBV, w, d, m);
            else {
#pragma unroll
                for (int i = 0; i < 16; ++i) w[i] = 0u;
            }
            uint8_t* tile = vtile + g * 16384;
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4)
                *reinterpret_cast<uint4*>(tile + tc::sw128_offset(key, blk * 4 + c4)) =
                    make_uint4(w[4 * c4], w[4 * c4 + 1], w[4 * c4 + 2], w[4 * c4 + 3]);
            dv[(g * 2 + blk) * kC + key] = d;
            if constexpr (V_MIN) mv[(g * 2 + blk) * kC + key] = m;
            // a warp covers 32 keys of one (g, blk): reduce, then one atomic per warp
            const float dmax = dec::warp_max(fabsf(d));
            if (lane == 0) atomicMax(&vsc[g * 2 + blk], __float_as_uint(dmax));
        }
    }
    fence_proxy_async_smem();
    tc::fence_before();
    __syncthreads();

    // ---- 4. S^T = K_g . Q_g^T, one accumulator of 16 columns per (g, blk)
    if (tid == 0) {
        tc::fence_after();
        const uint32_t idesc = tc::idesc_f16_f32(128, 16, false);
#pragma unroll
        for (int g = 0; g < 2; ++g)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const uint64_t ad = tc::sdesc_sw128(smem_addr(ktile + g * 16384) + kk * 32, 16, 1024);
                const uint64_t bd = tc::sdesc_sw128(smem_addr(qtile + g * 2048) + kk * 32, 16, 1024);
                tc::mma_ss(tmem + kSCol + (g * 2 + (kk >> 1)) * 16, ad, bd, idesc, (kk & 1) ? 1u : 0u);
            }
        tc::mma_commit(&bars[1]);
    }
    {
        const bool s_ok = mbar_wait(&bars[1], 0, a.status, 2);
        if (!__syncthreads_and(s_ok)) goto teardown;
    }
    tc::fence_after();

    // ---- 5. softmax over the chunk: thread = (kv head g, key)
    {
        const int g = warp >> 2, key = tid & (kC - 1);
        const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
        uint32_t sv[32];
        tc::tmem_ld32(tmem + lane_base + kSCol + g * 32, sv);
        tc::tmem_ld_wait();
        const float d0 = dk[(g * 2) * kC + key], d1 = dk[(g * 2 + 1) * kC + key];
        float s[kHP];
#pragma unroll
        for (int h = 0; h < kHP; ++h) {
            float t = d0 * (__uint_as_float(sv[h]) + __uint_as_float(sv[8 + h])) +
                      d1 * (__uint_as_float(sv[16 + h]) + __uint_as_float(sv[24 + h]));
            t *= esc[g * kHP + h];
            if constexpr (K_MIN)
                t += mk[(g * 2) * kC + key] * qsum[(g * 2) * kHP + h] + mk[(g * 2 + 1) * kC + key] * qsum[(g * 2 + 1) * kHP + h];
            s[h] = (key < n && h < G) ? t * a.scale_log2 : -INFINITY;
        }
#pragma unroll
        for (int h = 0; h < kHP; ++h) {
            const float v = dec::warp_max(s[h]);
            if (lane == 0) red[warp * 32 + h] = v;
        }
        __syncthreads();
        float p[kHP];
#pragma unroll
        for (int h = 0; h < kHP; ++h) {
            float mm = red[(g * 4) * 32 + h];
#pragma unroll
            for (int w2 = 1; w2 < 4; ++w2) mm = fmaxf(mm, red[(g * 4 + w2) * 32 + h]);
            p[h] = (s[h] == -INFINITY) ? 0.0f : fast_exp2(s[h] - mm);
            if (warp == g * 4 && lane == h) ML[(g * kHP + h) * 2] = mm;
        }
#pragma unroll
        for (int h = 0; h < kHP; ++h) {
            const float v = dec::warp_sum(p[h]);
            if (lane == 0) red[warp * 32 + 8 + h] = v;
        }
        if constexpr (V_MIN) {
#pragma unroll
            for (int b2 = 0; b2 < 2; ++b2) {
                const float mvk = mv[(g * 2 + b2) * kC + key];
#pragma unroll
                for (int h = 0; h < kHP; ++h) {
                    const float v = dec::warp_sum(p[h] * mvk);
                    if (lane == 0) red[warp * 32 + 16 + b2 * 8 + h] = v;
                }
            }
        }
        // P' row of this key: columns g*32 + blk*16 + {hi: h, lo: 8 + h}
#pragma unroll
        for (int b2 = 0; b2 < 2; ++b2) {
            const int vex = norm_exp(__uint_as_float(vsc[g * 2 + b2]));
            const float dvk = dv[(g * 2 + b2) * kC + key] * pow2f(vex);
            uint32_t hi[4], lo[4];
#pragma unroll
            for (int h = 0; h < kHP; h += 2) {
                const float x0 = p[h] * dvk, x1 = p[h + 1] * dvk;
                const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
                hi[h / 2] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
                lo[h / 2] = tc::pack_f16x2(x0 - __half2float(h0), x1 - __half2float(h1));
            }
            *reinterpret_cast<uint4*>(ptile + tc::sw128_offset(key, g * 4 + b2 * 2)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
            *reinterpret_cast<uint4*>(ptile + tc::sw128_offset(key, g * 4 + b2 * 2 + 1)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        }
    }
    fence_proxy_async_smem();
    tc::fence_before();
    __syncthreads();
    if (tid < 16) {  // per (g, h): chunk sum and the min-term sums
        const int g = tid >> 3, h = tid & 7;
        float l = 0.0f;
#pragma unroll
        for (int w2 = 0; w2 < 4; ++w2) l += red[(g * 4 + w2) * 32 + 8 + h];
        ML[(g * kHP + h) * 2 + 1] = l;
        if constexpr (V_MIN) {
#pragma unroll
            for (int b2 = 0; b2 < 2; ++b2) {
                float s2 = 0.0f;
#pragma unroll
                for (int w2 = 0; w2 < 4; ++w2) s2 += red[(g * 4 + w2) * 32 + 16 + b2 * 8 + h];
                PM[(g * 2 + b2) * kHP + h] = s2;
            }
        }
    }

    // ---- 6. O^T = V^T . P' (M = 128 (g, dim) rows, N = 64, K = 128 keys)
    if (tid == 0) {
        tc::fence_after();
        const uint32_t idesc = tc::idesc_f16_f32(128, 64, true, true);
#pragma unroll
        for (int kk = 0; kk < kC / 16; ++kk) {
            const uint64_t ad = tc::sdesc_sw128(smem_addr(vtile) + kk * 2048, 16384, 1024);
            const uint64_t bd = tc::sdesc_sw128(smem_addr(ptile) + kk * 2048, 16, 1024);
            tc::mma_ss(tmem + kOCol, ad, bd, idesc, kk > 0 ? 1u : 0u);
        }
        tc::mma_commit(&bars[2]);
    }
    {
        const bool o_ok = mbar_wait(&bars[2], 0, a.status, 3);
        if (!__syncthreads_and(o_ok)) goto teardown;
    }
    tc::fence_after();

    // ---- 7. chunk result: thread = (g, dim) row of O^T
    {
        const bool single = nchunks == 1;
        float* wso = a.ws_o + (((int64_t)seq * a.ws_chunks + chunk) * Hq) * kD;
        float* wsml = a.ws_ml + (((int64_t)seq * a.ws_chunks + chunk) * Hq) * 2;
        if (warp < 4) {
            const int g = tid >> 6, dim = tid & 63, blk = dim >> 5;
            const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
            uint32_t ov[16];
            tc::tmem_ld16(tmem + lane_base + kOCol + g * 32 + blk * 16, ov);
            tc::tmem_ld_wait();
            const float inv_vs = pow2f(-norm_exp(__uint_as_float(vsc[g * 2 + blk])));
#pragma unroll
            for (int h = 0; h < kHP; ++h) {
                if (h >= G) break;
                float o = (__uint_as_float(ov[h]) + __uint_as_float(ov[8 + h])) * inv_vs;
                if constexpr (V_MIN) o += PM[(g * 2 + blk) * kHP + h];
                const int qh = g * G + h;
                const float m = ML[(g * kHP + h) * 2], l = ML[(g * kHP + h) * 2 + 1];
                if (single) {
                    out[qh * kD + dim] = emit_partial ? o : o / l;
                    if (emit_partial && dim == 0) {
                        a.partial_ml[((int64_t)seq * Hq + qh) * 2] = m;
                        a.partial_ml[((int64_t)seq * Hq + qh) * 2 + 1] = l;
                    }
                } else {
                    wso[qh * kD + dim] = o;
                    if (dim == 0) {
                        wsml[qh * 2] = m;
                        wsml[qh * 2 + 1] = l;
                    }
                }
            }
        }
        if (!single) {
            // last CTA of the sequence merges the chunk partials
            __threadfence();
            __syncthreads();
            int* flag = reinterpret_cast<int*>(smem + L.bars + 48);
            if (tid == 0) {
                const uint32_t prev = atomicAdd(&a.ws_cnt[seq], 1u);
                *flag = (prev == (uint32_t)(nchunks - 1)) ? 1 : 0;
            }
            __syncthreads();
            if (*flag) {
                __threadfence();
                combine_chunks(a, seq, nchunks, out, reinterpret_cast<float*>(ktile));  // K tiles are free now
            }
        }
    }

teardown:
    tc::fence_before();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after();
        tc::tmem_dealloc(tmem, kTmemCols);
    }
}

template <int KT>
cudaError_t launch_for_k(cudaStream_t s, const Args& a, int v_type, dim3 grid);
template <> cudaError_t launch_for_k<kF16>(cudaStream_t, const Args&, int, dim3);
template <> cudaError_t launch_for_k<kQ4_0>(cudaStream_t, const Args&, int, dim3);
template <> cudaError_t launch_for_k<kQ4_1>(cudaStream_t, const Args&, int, dim3);
template <> cudaError_t launch_for_k<kQ5_0>(cudaStream_t, const Args&, int, dim3);
template <> cudaError_t launch_for_k<kQ5_1>(cudaStream_t, const Args&, int, dim3);
template <> cudaError_t launch_for_k<kQ8_0>(cudaStream_t, const Args&, int, dim3);

inline bool supported_type(int t) { return t == kF16 || t == kQ4_0 || t == kQ4_1 || t == kQ5_0 || t == kQ5_1 || t == kQ8_0; }

inline int smem_bytes(int k_type, int v_type) {
    const int rowK = (int)type_row_bytes(k_type, 2 * kD), rowV = (int)type_row_bytes(v_type, 2 * kD);
    return Smem(rowK, rowV, k_type == kQ4_1 || k_type == kQ5_1, v_type == kQ4_1 || v_type == kQ5_1).total;
}

}  // namespace dtc
}  // namespace cvattn
