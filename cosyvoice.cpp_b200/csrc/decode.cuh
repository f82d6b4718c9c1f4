// decode.cuh -- GQA split-KV decode attention over ggml-layout KV rows.
//
// Reference semantics: ggml_flash_attn_ext with one query row per sequence,
// no mask, scale 1/sqrt(D), f32 precision requested
// (src/cosyvoice-kv-cache.cpp:379-386, called from src/cosyvoice-llm.cpp:62
// for every layer of llm_decode, src/cosyvoice-llm.cpp:204-318), optionally
// fused with that token's update_cache append (src/cosyvoice-kv-cache.cpp:316,322).
//
// Design (one CTA = one sequence x one chunk of C consecutive positions, all
// KV heads):
//   1. the chunk's K and V rows are contiguous bytes in a ggml cache tensor;
//      one thread streams them into shared memory with cp.async.bulk (TMA
//      engine) -- HBM -> SMEM with no register staging.
//   2. QK: one thread per (kv head, 32-element group, key) computes the raw
//      dot product of the group's integer quants with the G query heads of
//      that KV head using packed fp32 FMAs (fma.rn.f32x2), then applies the
//      group scale (and min).  All arithmetic is fp32 on exactly dequantized
//      values.
//   3. softmax per (kv head, q head) row inside the chunk: warp-shuffle max
//      and sum, exp2 in log2 units.
//   4. PV: one thread per (kv head, dim pair, key split); p * d_group is
//      folded before the packed FMA with the raw V quants.
//   5. chunk partials (unnormalized O, max, sum) go to the workspace; the last
//      CTA of a sequence to finish (atomic ticket, no spinning) merges them
//      with a log-sum-exp combine and writes the output.
#pragma once

#include "common.cuh"

namespace cvattn {
namespace dec {

constexpr int kD = 64;          // head_dim
constexpr int kNB = kD / 32;    // 32-element groups per head
constexpr int kThreads = 256;
constexpr int kHP = 8;          // query heads per KV head, padded
constexpr int kKQ = 4;          // key splits in the PV phase

struct Args {
    const float* q;
    int64_t q_seq_stride;
    float* out;
    int64_t out_seq_stride;
    const uint8_t* k_base;
    const uint8_t* v_base;
    int64_t k_nb2, v_nb2;
    int64_t capacity;
    const uint64_t* k_seq_ptrs;
    const uint64_t* v_seq_ptrs;
    const int32_t* kv_len;
    const float* k_new;
    const float* v_new;
    float* partial_ml;
    int n_seq, Hq, Hkv, G, C, flags;
    int max_kv_len;  // host bound the grid and workspace were sized for
    float scale_log2;
    float* ws_o;
    float* ws_ml;
    uint32_t* ws_cnt;
    int ws_chunks;  // chunk stride of the workspace arrays
    int* status;
    // RoPE of Q and the appended K row at position kv_len - 1 (streaming kernel;
    // rope_n_dims = 0: none)
    int rope_mode, rope_n_dims;
    float rope_theta_scale, rope_freq_scale, rope_attn_factor;
};

// Shared-memory carve-up, identical on host and device.
struct Smem {
    int k, v, q2, qsum, s, pd, pm, ml, bar, flag, total;
    __host__ __device__ static int al(int x) { return (x + 127) & ~127; }
    __host__ __device__ Smem(int C, int Hkv, int rowK, int rowV, bool v_min) {
        int o = 0;
        k = o; o += al(C * rowK);
        v = o; o += al(C * rowV);
        q2 = o; o += al(Hkv * 32 * kHP * 8);
        qsum = o; o += al(Hkv * kNB * kHP * 4);
        s = o;
        {
            int s_bytes = kNB * Hkv * kHP * C * 4;
            int ored = kKQ * Hkv * kHP * 32 * 8 + kKQ * Hkv * kNB * kHP * 4;
            o += al(s_bytes > ored ? s_bytes : ored);
        }
        pd = o; o += al(Hkv * C * kNB * kHP * 8);
        pm = o; o += v_min ? al(Hkv * C * kNB * kHP * 4) : 0;
        ml = o; o += al(Hkv * kHP * 2 * 4);
        bar = o; o += 16;
        flag = o; o += 16;
        total = al(o);
    }
};

// Raw values of one 32-element group.  pair(i) returns elements (i, i+1),
// i even: q - offset for the symmetric block types, q for the _1 types, the
// value itself for F16/F32.  d / m are the group's scale and min (1 / 0 for
// the float types), so element = d * raw + m exactly as gguf-py dequantizes.
template <int T> struct Group;

template <> struct Group<kF32> {
    const uint8_t* p;
    __device__ explicit Group(const uint8_t* g) : p(g) {}
    __device__ float d() const { return 1.0f; }
    __device__ float m() const { return 0.0f; }
    __device__ float2 pair(int i) const { return *reinterpret_cast<const float2*>(p + 4 * i); }
};

template <> struct Group<kF16> {
    const uint8_t* p;
    __device__ explicit Group(const uint8_t* g) : p(g) {}
    __device__ float d() const { return 1.0f; }
    __device__ float m() const { return 0.0f; }
    __device__ float2 pair(int i) const { return __half22float2(*reinterpret_cast<const __half2*>(p + 2 * i)); }
};

template <> struct Group<kQ8_0> {
    const uint8_t* p;
    __device__ explicit Group(const uint8_t* g) : p(g) {}
    __device__ float d() const { return h2f(*reinterpret_cast<const uint16_t*>(p)); }
    __device__ float m() const { return 0.0f; }
    __device__ float2 pair(int i) const {
        uint32_t w = *reinterpret_cast<const uint16_t*>(p + 2 + i);
        return make_float2((float)(int8_t)(w & 0xffu), (float)(int8_t)(w >> 8));
    }
};

template <int T, int OFF_QS, int BIAS, bool MIN>
struct Group4 {
    const uint8_t* p;
    __device__ explicit Group4(const uint8_t* g) : p(g) {}
    __device__ float d() const { return h2f(*reinterpret_cast<const uint16_t*>(p)); }
    __device__ float m() const { return MIN ? h2f(*reinterpret_cast<const uint16_t*>(p + 2)) : 0.0f; }
    __device__ float2 pair(int i) const {
        uint32_t w = *reinterpret_cast<const uint16_t*>(p + OFF_QS + (i & 15));
        int sh = (i >> 4) << 2;
        return make_float2((float)((int)((w >> sh) & 15u) - BIAS), (float)((int)((w >> (8 + sh)) & 15u) - BIAS));
    }
};
template <> struct Group<kQ4_0> : Group4<kQ4_0, 2, 8, false> { using Group4::Group4; };
template <> struct Group<kQ4_1> : Group4<kQ4_1, 4, 0, true> { using Group4::Group4; };

template <int T, int OFF_QH, int OFF_QS, int BIAS, bool MIN>
struct Group5 {
    const uint8_t* p;
    uint32_t qh;
    __device__ explicit Group5(const uint8_t* g)
        : p(g),
          qh((uint32_t)*reinterpret_cast<const uint16_t*>(g + OFF_QH) |
             ((uint32_t)*reinterpret_cast<const uint16_t*>(g + OFF_QH + 2) << 16)) {}
    __device__ float d() const { return h2f(*reinterpret_cast<const uint16_t*>(p)); }
    __device__ float m() const { return MIN ? h2f(*reinterpret_cast<const uint16_t*>(p + 2)) : 0.0f; }
    __device__ float2 pair(int i) const {
        uint32_t w = *reinterpret_cast<const uint16_t*>(p + OFF_QS + (i & 15));
        int sh = (i >> 4) << 2;
        int a = (int)((w >> sh) & 15u) | (int)(((qh >> i) & 1u) << 4);
        int b = (int)((w >> (8 + sh)) & 15u) | (int)(((qh >> (i + 1)) & 1u) << 4);
        return make_float2((float)(a - BIAS), (float)(b - BIAS));
    }
};
template <> struct Group<kQ5_0> : Group5<kQ5_0, 2, 6, 16, false> { using Group5::Group5; };
template <> struct Group<kQ5_1> : Group5<kQ5_1, 4, 8, 0, true> { using Group5::Group5; };

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Log-sum-exp merge of one sequence's chunk partials by the CTA that finished
// last.  All (head, chunk) statistics are fetched in one parallel pass into
// shared memory (independent L2 loads), then every output element sums its
// chunks with independent loads.  scratch: >= Hq * (nchunks + 2) floats.
__device__ __forceinline__ void combine_chunks(const Args& a, int seq, int nchunks, float* out, float* scratch) {
    const int Hq = a.Hq, tid = threadIdx.x, nt = blockDim.x;
    const bool emit_partial = (a.flags & CVATTN_DECODE_EMIT_PARTIAL) != 0;
    float* W = scratch;                      // [Hq][nchunks]: m_c, then weights
    float* Lc = scratch + Hq * nchunks;      // [Hq][nchunks]: l_c
    float* MLc = Lc + Hq * nchunks;          // [Hq][2]: M, L
    const float* seq_ml = a.ws_ml + ((int64_t)seq * a.ws_chunks) * Hq * 2;
    const float* seq_o = a.ws_o + ((int64_t)seq * a.ws_chunks) * Hq * kD;
    for (int i = tid; i < Hq * nchunks; i += nt) {
        const int h = i / nchunks, c = i % nchunks;
        const float2 ml = __ldcg(reinterpret_cast<const float2*>(seq_ml + ((int64_t)c * Hq + h) * 2));
        W[i] = ml.x;
        Lc[i] = ml.y;
    }
    __syncthreads();
    for (int h = tid; h < Hq; h += nt) {
        float M = -INFINITY;
        for (int c = 0; c < nchunks; ++c) M = fmaxf(M, W[h * nchunks + c]);
        float Ls = 0.0f;
        for (int c = 0; c < nchunks; ++c) {
            const float w = fast_exp2(W[h * nchunks + c] - M);
            W[h * nchunks + c] = w;
            Ls += w * Lc[h * nchunks + c];
        }
        MLc[h * 2] = M;
        MLc[h * 2 + 1] = Ls;
    }
    __syncthreads();
    for (int it = tid; it < Hq * kD / 4; it += nt) {
        const int h = (it * 4) / kD, dd = (it * 4) % kD;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
        for (int c = 0; c < nchunks; ++c) {
            const float w = W[h * nchunks + c];
            const float4 v = __ldcg(reinterpret_cast<const float4*>(seq_o + ((int64_t)c * Hq + h) * kD + dd));
            acc.x = fmaf(w, v.x, acc.x); acc.y = fmaf(w, v.y, acc.y);
            acc.z = fmaf(w, v.z, acc.z); acc.w = fmaf(w, v.w, acc.w);
        }
        const float inv = emit_partial ? 1.0f : 1.0f / MLc[h * 2 + 1];
        *reinterpret_cast<float4*>(out + h * kD + dd) = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
    }
    if (emit_partial)
        for (int h = tid; h < Hq; h += nt) {
            a.partial_ml[((int64_t)seq * Hq + h) * 2] = MLc[h * 2];
            a.partial_ml[((int64_t)seq * Hq + h) * 2 + 1] = MLc[h * 2 + 1];
        }
    if (tid == 0) a.ws_cnt[seq] = 0u;  // leave the ticket zeroed for the next call
}

// GT: unroll bound for the query heads of one KV head (the actual count a.G <= GT).
template <int KT, int VT, int GT>
__global__ void __launch_bounds__(kThreads) decode_kernel(const Args a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int seq = blockIdx.y, chunk = blockIdx.x;
    const int C = a.C, Hkv = a.Hkv, G = a.G, Hq = a.Hq;
    constexpr int GBK = group_bytes(KT), GBV = group_bytes(VT);
    constexpr int headK = GBK * kNB, headV = GBV * kNB;
    constexpr bool K_MIN = BlockTraits<KT>::HAS_MIN, V_MIN = BlockTraits<VT>::HAS_MIN;
    const int rowK = Hkv * headK, rowV = Hkv * headV;
    const Smem L(C, Hkv, rowK, rowV, V_MIN);
    const bool emit_partial = (a.flags & CVATTN_DECODE_EMIT_PARTIAL) != 0;

    const int len = a.kv_len[seq];
    float* out = a.out + (int64_t)seq * a.out_seq_stride;
    if (len <= 0 || len > a.capacity || len > a.max_kv_len) {
        // empty or invalid sequence: zero output, flag invalid lengths
        if (chunk == 0) {
            for (int i = tid; i < Hq * kD; i += kThreads) out[(i / kD) * kD + (i % kD)] = 0.0f;
            if (emit_partial)
                for (int i = tid; i < Hq; i += kThreads) {
                    a.partial_ml[((int64_t)seq * Hq + i) * 2] = -INFINITY;
                    a.partial_ml[((int64_t)seq * Hq + i) * 2 + 1] = 0.0f;
                }
            if (len != 0 && tid == 0) record_status(a.status, kStatusBadLength);
        }
        return;
    }
    const int p0 = chunk * C;
    if (p0 >= len) return;
    const int n = min(C, len - p0);
    const int nchunks = (len + C - 1) / C;

    const uint8_t* kb = a.k_seq_ptrs ? reinterpret_cast<const uint8_t*>(a.k_seq_ptrs[seq]) : a.k_base + seq * a.k_nb2;
    const uint8_t* vb = a.v_seq_ptrs ? reinterpret_cast<const uint8_t*>(a.v_seq_ptrs[seq]) : a.v_base + seq * a.v_nb2;
    uint8_t* Ks = smem + L.k;
    uint8_t* Vs = smem + L.v;
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L.bar);

    // ---- 1. stream the chunk into shared memory
    const uint32_t kbytes = (uint32_t)(n * rowK), vbytes = (uint32_t)(n * rowV);
    const uint8_t* ksrc = kb + (int64_t)p0 * rowK;
    const uint8_t* vsrc = vb + (int64_t)p0 * rowV;
    const uint32_t kbulk = ((reinterpret_cast<uintptr_t>(ksrc) & 15) == 0) ? (kbytes & ~15u) : 0u;
    const uint32_t vbulk = ((reinterpret_cast<uintptr_t>(vsrc) & 15) == 0) ? (vbytes & ~15u) : 0u;
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) {
        mbar_arrive_expect_tx(bar, kbulk + vbulk);
        if (kbulk) bulk_g2s(Ks, ksrc, kbulk, bar);
        if (vbulk) bulk_g2s(Vs, vsrc, vbulk, bar);
    }
    for (uint32_t i = kbulk / 2 + tid; i < kbytes / 2; i += kThreads)
        reinterpret_cast<uint16_t*>(Ks)[i] = reinterpret_cast<const uint16_t*>(ksrc)[i];
    for (uint32_t i = vbulk / 2 + tid; i < vbytes / 2; i += kThreads)
        reinterpret_cast<uint16_t*>(Vs)[i] = reinterpret_cast<const uint16_t*>(vsrc)[i];

    // ---- 2. query heads into shared memory as (d, d+1) pairs, heads padded to kHP
    float2* Q2 = reinterpret_cast<float2*>(smem + L.q2);  // [Hkv][32][kHP]
    const float* qs = a.q + (int64_t)seq * a.q_seq_stride;
    for (int i = tid; i < Hkv * 32 * kHP; i += kThreads) {
        const int hh = i % kHP, ip = (i / kHP) % 32, g = i / (kHP * 32);
        float2 v = make_float2(0.0f, 0.0f);
        if (hh < G) v = *reinterpret_cast<const float2*>(qs + (g * G + hh) * kD + 2 * ip);
        Q2[i] = v;
    }
    float* Qsum = reinterpret_cast<float*>(smem + L.qsum);  // [Hkv][kNB][kHP]
    if constexpr (K_MIN) {
        for (int i = tid; i < Hkv * kNB * kHP; i += kThreads) {
            const int hh = i % kHP, blk = (i / kHP) % kNB, g = i / (kHP * kNB);
            float s = 0.0f;
            if (hh < G)
                for (int e = 0; e < 32; ++e) s += qs[(g * G + hh) * kD + blk * 32 + e];
            Qsum[i] = s;
        }
    }

    if (!mbar_wait(bar, 0, a.status, 1)) return;
    __syncthreads();

    // ---- fused append of this step's row (position len-1) into cache and chunk copy
    if (a.k_new && chunk == nchunks - 1) {
        const int r = len - 1 - p0;
        const int groups = Hkv * kNB;
        for (int gi = warp; gi < 2 * groups; gi += kThreads / 32) {
            const bool isv = gi >= groups;
            const int g2 = isv ? gi - groups : gi;
            const float x = (isv ? a.v_new : a.k_new)[(int64_t)seq * Hkv * kD + g2 * 32 + lane];
            if (!isv) {
                quantize_block_warp<KT>(x, Ks + r * rowK + g2 * GBK, lane);
                quantize_block_warp<KT>(x, const_cast<uint8_t*>(kb) + (int64_t)(len - 1) * rowK + g2 * GBK, lane);
            } else {
                quantize_block_warp<VT>(x, Vs + r * rowV + g2 * GBV, lane);
                quantize_block_warp<VT>(x, const_cast<uint8_t*>(vb) + (int64_t)(len - 1) * rowV + g2 * GBV, lane);
            }
        }
        __syncthreads();
    }

    // ---- 3. scores: one item per (kv head, group, key)
    float* S = reinterpret_cast<float*>(smem + L.s);  // [kNB][Hkv][kHP][C]
    for (int it = tid; it < Hkv * kNB * C; it += kThreads) {
        const int key = it % C, gb = it / C, blk = gb % kNB, g = gb / kNB;
        if (key >= n) continue;
        const Group<KT> grp(Ks + key * rowK + g * headK + blk * GBK);
        float2 acc[GT];
#pragma unroll
        for (int h = 0; h < GT; ++h) acc[h] = make_float2(0.0f, 0.0f);
        const float4* qrow = reinterpret_cast<const float4*>(Q2 + (g * 32 + blk * 16) * kHP);
#pragma unroll 4
        for (int ip = 0; ip < 16; ++ip) {
            const float2 kv = grp.pair(2 * ip);
#pragma unroll
            for (int h2 = 0; h2 < (GT + 1) / 2; ++h2) {
                const float4 qq = qrow[ip * (kHP / 2) + h2];
                acc[2 * h2] = ffma2(make_float2(qq.x, qq.y), kv, acc[2 * h2]);
                if (2 * h2 + 1 < GT) acc[2 * h2 + 1] = ffma2(make_float2(qq.z, qq.w), kv, acc[2 * h2 + 1]);
            }
        }
        const float d = grp.d();
#pragma unroll
        for (int h = 0; h < GT; ++h) {
            float s = d * (acc[h].x + acc[h].y);
            if constexpr (K_MIN) s = fmaf(grp.m(), Qsum[(g * kNB + blk) * kHP + h], s);
            S[((blk * Hkv + g) * kHP + h) * C + key] = s * a.scale_log2;
        }
    }
    __syncthreads();

    // ---- 4. softmax inside the chunk, one warp per (kv head, q head) row
    float* ML = reinterpret_cast<float*>(smem + L.ml);  // [Hkv*kHP][2]
    for (int r = warp; r < Hkv * G; r += kThreads / 32) {
        const int g = r / G, h = r % G;
        float sv[4];
        float m = -INFINITY;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int key = lane + 32 * j;
            float s = -INFINITY;
            if (key < n) {
                s = 0.0f;
#pragma unroll
                for (int blk = 0; blk < kNB; ++blk) s += S[((blk * Hkv + g) * kHP + h) * C + key];
            }
            sv[j] = s;
            m = fmaxf(m, s);
        }
        m = warp_max(m);
        float l = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int key = lane + 32 * j;
            if (key < n) {
                const float p = fast_exp2(sv[j] - m);
                l += p;
                S[(g * kHP + h) * C + key] = p;  // blk-0 slot now holds p
            }
        }
        l = warp_sum(l);
        if (lane == 0) {
            ML[(g * kHP + h) * 2] = m;
            ML[(g * kHP + h) * 2 + 1] = l;
        }
    }
    __syncthreads();

    // ---- p * d_group (and p * m_group) per (kv head, key, group)
    float2* Pd = reinterpret_cast<float2*>(smem + L.pd);  // [Hkv][C][kNB][kHP]
    float* Pm = reinterpret_cast<float*>(smem + L.pm);    // [Hkv][C][kNB][kHP]
    for (int it = tid; it < Hkv * C * kNB; it += kThreads) {
        const int blk = it % kNB, key = (it / kNB) % C, g = it / (kNB * C);
        if (key >= n) continue;
        const Group<VT> grp(Vs + key * rowV + g * headV + blk * GBV);
        const float dv = grp.d();
        float mv = 0.0f;
        if constexpr (V_MIN) mv = grp.m();
#pragma unroll
        for (int h = 0; h < GT; ++h) {
            const float p = h < G ? S[(g * kHP + h) * C + key] : 0.0f;
            Pd[it * kHP + h] = make_float2(p * dv, p * dv);
            if constexpr (V_MIN) Pm[it * kHP + h] = p * mv;
        }
    }
    __syncthreads();

    // ---- 5. PV: one item per (kv head, key split, dim pair)
    float2* Ored = reinterpret_cast<float2*>(smem + L.s);  // [kKQ][Hkv][kHP][32]
    float* PMred = reinterpret_cast<float*>(smem + L.s + kKQ * Hkv * kHP * 32 * 8);  // [kKQ][Hkv][kNB][kHP]
    for (int it = tid; it < Hkv * kKQ * 32; it += kThreads) {
        const int ip32 = it % 32, kq = (it / 32) % kKQ, g = it / (32 * kKQ);
        const int blk = ip32 / 16, i = 2 * (ip32 % 16);
        float2 acc[GT];
        float pm[GT];
#pragma unroll
        for (int h = 0; h < GT; ++h) { acc[h] = make_float2(0.0f, 0.0f); pm[h] = 0.0f; }
        for (int key = kq; key < n; key += kKQ) {
            const Group<VT> grp(Vs + key * rowV + g * headV + blk * GBV);
            const float2 vv = grp.pair(i);
            const float4* pd = reinterpret_cast<const float4*>(Pd + ((g * C + key) * kNB + blk) * kHP);
#pragma unroll
            for (int h2 = 0; h2 < (GT + 1) / 2; ++h2) {
                const float4 pp = pd[h2];
                acc[2 * h2] = ffma2(make_float2(pp.x, pp.y), vv, acc[2 * h2]);
                if (2 * h2 + 1 < GT) acc[2 * h2 + 1] = ffma2(make_float2(pp.z, pp.w), vv, acc[2 * h2 + 1]);
            }
            if constexpr (V_MIN) {
                const float* pmr = Pm + ((g * C + key) * kNB + blk) * kHP;
#pragma unroll
                for (int h = 0; h < GT; ++h) pm[h] += pmr[h];
            }
        }
#pragma unroll
        for (int h = 0; h < GT; ++h) Ored[((kq * Hkv + g) * kHP + h) * 32 + ip32] = acc[h];
        if constexpr (V_MIN) {
            if ((ip32 & 15) == 0)
#pragma unroll
                for (int h = 0; h < GT; ++h) PMred[((kq * Hkv + g) * kNB + blk) * kHP + h] = pm[h];
        }
    }
    __syncthreads();

    // ---- 6. chunk result: unnormalized O, running max and sum
    float* wso = a.ws_o + (((int64_t)seq * a.ws_chunks + chunk) * Hq) * kD;
    float* wsml = a.ws_ml + (((int64_t)seq * a.ws_chunks + chunk) * Hq) * 2;
    const bool single = nchunks == 1;
    for (int it = tid; it < Hq * 32; it += kThreads) {
        const int ip32 = it % 32, h = it / 32, g = h / G, hh = h % G;
        float2 o = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int kq = 0; kq < kKQ; ++kq) {
            const float2 v = Ored[((kq * Hkv + g) * kHP + hh) * 32 + ip32];
            o.x += v.x;
            o.y += v.y;
        }
        if constexpr (V_MIN) {
            const int blk = ip32 / 16;
            float s = 0.0f;
#pragma unroll
            for (int kq = 0; kq < kKQ; ++kq) s += PMred[((kq * Hkv + g) * kNB + blk) * kHP + hh];
            o.x += s;
            o.y += s;
        }
        const float m = ML[(g * kHP + hh) * 2], l = ML[(g * kHP + hh) * 2 + 1];
        if (single) {
            if (emit_partial) {
                *reinterpret_cast<float2*>(out + h * kD + 2 * ip32) = o;
                if (ip32 == 0) {
                    a.partial_ml[((int64_t)seq * Hq + h) * 2] = m;
                    a.partial_ml[((int64_t)seq * Hq + h) * 2 + 1] = l;
                }
            } else {
                const float inv = 1.0f / l;
                *reinterpret_cast<float2*>(out + h * kD + 2 * ip32) = make_float2(o.x * inv, o.y * inv);
            }
        } else {
            *reinterpret_cast<float2*>(wso + h * kD + 2 * ip32) = o;
            if (ip32 == 0) {
                wsml[h * 2] = m;
                wsml[h * 2 + 1] = l;
            }
        }
    }
    if (single) return;

    // ---- 7. last CTA of the sequence merges the chunk partials
    __threadfence();
    __syncthreads();
    int* flag = reinterpret_cast<int*>(smem + L.flag);
    if (tid == 0) {
        const uint32_t prev = atomicAdd(&a.ws_cnt[seq], 1u);
        *flag = (prev == (uint32_t)(nchunks - 1)) ? 1 : 0;
    }
    __syncthreads();
    if (!*flag) return;
    __threadfence();
    combine_chunks(a, seq, nchunks, out, reinterpret_cast<float*>(smem + L.pd));
}

}  // namespace dec
}  // namespace cvattn

namespace cvattn {
namespace dec {
// Per-K-type launcher (one translation unit per K type, see decode_inst.cu).
template <int KT>
cudaError_t launch_for_k(cudaStream_t s, const Args& a, int v_type, dim3 grid, int smem);
template <> cudaError_t launch_for_k<kF32>(cudaStream_t, const Args&, int, dim3, int);
template <> cudaError_t launch_for_k<kF16>(cudaStream_t, const Args&, int, dim3, int);
template <> cudaError_t launch_for_k<kQ4_0>(cudaStream_t, const Args&, int, dim3, int);
template <> cudaError_t launch_for_k<kQ4_1>(cudaStream_t, const Args&, int, dim3, int);
template <> cudaError_t launch_for_k<kQ5_0>(cudaStream_t, const Args&, int, dim3, int);
template <> cudaError_t launch_for_k<kQ5_1>(cudaStream_t, const Args&, int, dim3, int);
template <> cudaError_t launch_for_k<kQ8_0>(cudaStream_t, const Args&, int, dim3, int);
}  // namespace dec
}  // namespace cvattn
