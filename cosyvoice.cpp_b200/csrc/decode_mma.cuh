// decode_mma.cuh -- register-resident split-KV decode on warp-level tensor-core
// MMAs (mma.sync m16n8k16, f16 operands, f32 accumulators).
//
// Same contract as the other decode kernels (one query row per sequence,
// ggml_flash_attn_ext with f32 precision, src/cosyvoice-kv-cache.cpp:379-386;
// optional fused update_cache append :316,322; split partials merged by the
// last writer), and the same exact-integer arithmetic:
//   * K and V quants are integers, exact in f16: a block's quants (centred for
//     the 4/5-bit types) go straight from the raw ggml bytes into MMA operand
//     registers; its f16 scale (and min) stays aside in f32;
//   * Q is scaled per head by an exact power of two and split into f16
//     hi + lo, so the QK products are exact in the f32 accumulator;
//   * P' = p * d_V * 2^ev is split into f16 hi + lo the same way for P.V.
//
// Work split: an item is (sequence, 64-position chunk) for both KV heads.  A
// warp pair walks one contiguous range of items; warp 2i + g handles KV head g.
// The pair's first lane streams the raw K/V rows of each item into a 2-slot
// ring with cp.async.bulk (TMA engine); everything else stays in registers:
//   S^T-free layout: S[head][pos] = A(Q) . B(K^T) with A rows 0-7 = Q_hi of the
//   8 (padded) query heads of the group and rows 8-15 = Q_lo, so the f32
//   accumulator row h holds the hi part and row h + 8 the lo part of head h;
//   the C fragment of two 8-position tiles is, element for element, the A
//   fragment of P' for the P.V MMA (A rows = P'_hi / P'_lo of each head, k =
//   the 16 positions), and B = V[16 positions][8 dims].
// The dot products run over the K-dimension in any order, so each thread takes
// the quants of a block that are cheapest to reach for its type (8 contiguous
// bytes for q8_0, the nibbles of 4 contiguous bytes for the 4/5-bit types) and
// Q is loaded in the same order; the output dims of P.V follow the V type's
// own order the same way.
//
// Online softmax per head row with a lazy reference max (raised only when a
// score exceeds it by more than 2^8, then O is rescaled in registers), a
// power-of-two factor per V block that moves only when an item's V scales
// leave [2^-3, 2^7) of it, and runs that end at a sequence boundary: a run
// that covers a whole sequence writes the output, otherwise its partial goes to
// the workspace slot of its first chunk and an acq_rel ticket per (sequence,
// KV head) elects the last writer, which merges the runs listed from the cut.
#pragma once

#include <type_traits>

#include "decode_stream.cuh"

namespace cvattn {
namespace dmma {

using dec::Args;

constexpr int kD = 64;
constexpr int kC = 64;          // positions per item
constexpr int kHP = 8;          // query heads per KV head, padded (the 8 A rows)
constexpr int kStages = 2;      // raw-row ring per warp pair
constexpr int kMaxPairs = 6;
constexpr int kMaxThreads = 64 * kMaxPairs;
constexpr int kMaxSeq = 512;    // prefix table in shared memory
constexpr float kLazyLog2 = 8.0f;
constexpr int kEvMin = -3, kEvMax = 6;
constexpr int kSmemLimit = 227 * 1024;  // dynamic shared memory of one CTA
constexpr int kMaxTasks = 4 * kMaxPairs;  // merges a CTA can be elected for: two per warp
constexpr int kMaxMergeRuns = 64;         // runs a CTA-wide merge takes (more: the warp merges alone)
constexpr int kMergeBatch = 10;
constexpr long kLatencyItemsPerSm = 16;   // launches with at most this many items per SM ...
constexpr int kLatencyPairs = 4;          // ... run this many warp pairs per CTA           // runs whose (max, sum) and outputs a merging thread loads at once

// A merge the CTA was elected for: the runs of (sequence seq, KV head g), whose
// nruns workspace slots are listed at int offset `slots` of the scale tables.
struct MergeTask {
    int seq, g, nruns, slots;
};

__host__ __device__ constexpr int rup(int x, int a) { return (x + a - 1) / a * a; }

// Shared memory: prefix table, lengths, barriers (full / empty per pair and
// slot), error flag, the per-warp scale tables of the current item, then the raw
// rings of the pairs.  A warp's scale table holds, per position pair q (positions
// 2q, 2q + 1 of the item), float4s {x[2q][blk 0], x[2q+1][blk 0], x[2q][blk 1],
// x[2q+1][blk 1]} of: the K scale, the V scale times 2^ev (the P' factor), and,
// for types with a min, the centred K and V mins.
struct Smem {
    int pref, slen, bars, misc, tasks, scl, scl_warp, ring0, stage, vofs, pair_stride, total;
    __host__ __device__ Smem(int rowK, int rowV, int pairs, bool k_min, bool v_min) {
        int o = 0;
        pref = o;  o += rup((kMaxSeq + 1) * 4, 16);
        slen = o;  o += kMaxSeq * 4;
        bars = o;  o += rup(kMaxPairs * kStages * 2 * 8, 16);
        misc = o;  o += 16;                     // error flag, merge task count
        tasks = o; o += kMaxTasks * 16;         // merge tasks of the CTA (MergeTask)
        scl = o;
        scl_warp = 32 * 16 * (2 + (k_min ? 1 : 0) + (v_min ? 1 : 0));
        o += 2 * pairs * scl_warp;
        o = rup(o, 128);
        ring0 = o;
        vofs = kC * rowK;                       // V rows follow the K rows of a slot
        stage = rup(kC * (rowK + rowV), 128);
        pair_stride = kStages * stage;
        o += pairs * pair_stride;
        total = o;
    }
};

// ------------------------------------------------------------------ helpers

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t ld_u16(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }

// 32 bits from shared memory at an address whose offset from a 4-byte boundary
// is A (0 or 2), known at compile time: the ring slots are 128-byte aligned and
// every row, head and 4-lane offset is a multiple of 4 bytes, so the alignment of
// a field depends only on its block's offset in the row.
template <int A>
__device__ __forceinline__ uint32_t ld32(const uint8_t* p) {
    static_assert(A == 0 || A == 2, "2-byte aligned fields only");
    if constexpr (A == 0) return *reinterpret_cast<const uint32_t*>(p);
    else return ld_u16(p) | (ld_u16(p + 2) << 16);
}

using dtc::hsub2_u32;
using dtc::kF16x2_1032;
using dtc::kF16x2_1040;
using dtc::kF16x2_1152;
using dtc::pow2f;

// x = hi + lo packed as f16x2 pairs (hi: x truncated to 11 significant bits).
__device__ __forceinline__ void split2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
    const float h0 = __uint_as_float(__float_as_uint(x0) & 0xFFFFE000u);
    const float h1 = __uint_as_float(__float_as_uint(x1) & 0xFFFFE000u);
    hi = tc::pack_f16x2(h0, h1);
    lo = tc::pack_f16x2(x0 - h0, x1 - h1);
}

// K operand of one (position, block): the 8 quants of thread tig as 4 f16x2
// registers (k-step 0: r0, r1; k-step 1: r2, r3).  Element order E_tig (Q is
// loaded in the same):
//   q8_0    8 tig + [0 .. 7]
//   4/5-bit [4t, 4t+1, 16+4t, 17+4t, 4t+2, 4t+3, 18+4t, 19+4t]  (t = tig)
template <int T, int BLK>
__device__ __forceinline__ void kfrag(const uint8_t* g, int tig, uint32_t (&r)[4]) {
    using B = BlockTraits<T>;
    constexpr int GB = group_bytes(T);
    if constexpr (T == kQ8_0) {
        constexpr int A = (BLK * GB + 2) & 3;
        const uint32_t w0 = ld32<A>(g + 2 + 8 * tig) ^ 0x80808080u;
        const uint32_t w1 = ld32<A>(g + 6 + 8 * tig) ^ 0x80808080u;
        r[0] = hsub2_u32(__byte_perm(w0, 0x6464u, 0x5140u), kF16x2_1152);
        r[1] = hsub2_u32(__byte_perm(w0, 0x6464u, 0x5342u), kF16x2_1152);
        r[2] = hsub2_u32(__byte_perm(w1, 0x6464u, 0x5140u), kF16x2_1152);
        r[3] = hsub2_u32(__byte_perm(w1, 0x6464u, 0x5342u), kF16x2_1152);
    } else {
        const uint32_t w = ld32<(BLK * GB + B::OFF_QS) & 3>(g + B::OFF_QS + 4 * tig);
        const uint32_t x01 = __byte_perm(w, 0u, 0x4140u);  // [b0, 0, b1, 0]
        const uint32_t x23 = __byte_perm(w, 0u, 0x4342u);  // [b2, 0, b3, 0]
        uint32_t lo01 = (x01 & 0x000F000Fu) | 0x64006400u, hi01 = ((x01 >> 4) & 0x000F000Fu) | 0x64006400u;
        uint32_t lo23 = (x23 & 0x000F000Fu) | 0x64006400u, hi23 = ((x23 >> 4) & 0x000F000Fu) | 0x64006400u;
        if constexpr (B::OFF_QH >= 0) {  // 5th bit of element e: bit e of qh, to bit 4 / 20 of its pair
            const uint32_t qh = ld32<(BLK * GB + B::OFF_QH) & 3>(g + B::OFF_QH);
            lo01 |= (((qh >> (4 * tig)) & 3u) * 0x80010u) & 0x00100010u;
            hi01 |= (((qh >> (16 + 4 * tig)) & 3u) * 0x80010u) & 0x00100010u;
            lo23 |= (((qh >> (4 * tig + 2)) & 3u) * 0x80010u) & 0x00100010u;
            hi23 |= (((qh >> (18 + 4 * tig)) & 3u) * 0x80010u) & 0x00100010u;
        }
        constexpr uint32_t bias = B::OFF_QH >= 0 ? kF16x2_1040 : kF16x2_1032;
        r[0] = hsub2_u32(lo01, bias);
        r[1] = hsub2_u32(hi01, bias);
        r[2] = hsub2_u32(lo23, bias);
        r[3] = hsub2_u32(hi23, bias);
    }
}

// Element index (0..31 in the block) of Q value i (0..7) of thread tig: the
// same order as kfrag.
template <int T>
__device__ __forceinline__ int kelem(int tig, int i) {
    if constexpr (T == kQ8_0) return 8 * tig + i;
    else return 4 * tig + (i & 1) + ((i & 2) ? 16 : 0) + ((i & 4) ? 2 : 0);
}

// V operand registers of one position pair (pos0, pos1) and one block for
// thread gid: for tile jj (0..3) {V[pos0][F(jj)], V[pos1][F(jj)]} as f16x2,
// where F(jj) is the V element order of lane group gid:
//   q8_0    4 gid + jj
//   4/5-bit [2g, 2g+1, 16+2g, 17+2g][jj]  (g = gid)
template <int T, int BLK>
__device__ __forceinline__ void vfrag(const uint8_t* g0, const uint8_t* g1, int gid, uint32_t (&r)[4]) {
    using B = BlockTraits<T>;
    constexpr int GB = group_bytes(T);
    if constexpr (T == kQ8_0) {
        constexpr int A = (BLK * GB + 2) & 3;
        const uint32_t w0 = ld32<A>(g0 + 2 + 4 * gid) ^ 0x80808080u;
        const uint32_t w1 = ld32<A>(g1 + 2 + 4 * gid) ^ 0x80808080u;
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
            const uint32_t t = __byte_perm(w0, w1, (uint32_t)(jj | ((4 + jj) << 8)));
            r[jj] = hsub2_u32((t & 0x00FF00FFu) | 0x64006400u, kF16x2_1152);
        }
    } else {
        const uint32_t u = ld_u16(g0 + B::OFF_QS + 2 * gid) | (ld_u16(g1 + B::OFF_QS + 2 * gid) << 16);
        uint32_t x[4] = {u & 0x000F000Fu, (u >> 8) & 0x000F000Fu, (u >> 4) & 0x000F000Fu, (u >> 12) & 0x000F000Fu};
        if constexpr (B::OFF_QH >= 0) {
            constexpr int A = (BLK * GB + B::OFF_QH) & 3;
            const uint32_t s0 = ld32<A>(g0 + B::OFF_QH) >> (2 * gid), s1 = ld32<A>(g1 + B::OFF_QH) >> (2 * gid);
            // bits k = 0, 1, 16, 17 of s are the elements F(0..3); position 0 -> bit 4, position 1 -> bit 20
            const int ks[4] = {0, 1, 16, 17};
#pragma unroll
            for (int jj = 0; jj < 4; ++jj)
                x[jj] |= (((s0 >> ks[jj]) & 1u) << 4) | (((s1 >> ks[jj]) & 1u) << 20);
        }
        constexpr uint32_t bias = B::OFF_QH >= 0 ? kF16x2_1040 : kF16x2_1032;
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) r[jj] = hsub2_u32(x[jj] | 0x64006400u, bias);
    }
}

// Element index (0..31 in the block) of V tile jj for lane group n.
template <int T>
__device__ __forceinline__ int velem(int n, int jj) {
    if constexpr (T == kQ8_0) return 4 * n + jj;
    else return 2 * n + (jj & 1) + ((jj & 2) ? 16 : 0);
}

// Centred scale and min of a V block (min 0 without one).
template <int T>
__device__ __forceinline__ void vscale(const uint8_t* g, float& d, float& m) {
    using B = BlockTraits<T>;
    d = h2f((uint16_t)ld_u16(g));
    if constexpr (B::HAS_MIN) {
        constexpr float kCentre = B::OFF_QH >= 0 ? 16.0f : 8.0f;
        m = fmaf(kCentre, d, h2f((uint16_t)ld_u16(g + B::OFF_M)));
    } else {
        m = 0.0f;
    }
}

__device__ __forceinline__ float quad_max(float v) {
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
    return fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
}
__device__ __forceinline__ float quad_sum(float v) {
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    return v + __shfl_xor_sync(0xffffffffu, v, 2);
}

// Bounded wait of one lane on an mbarrier phase; gives up when another warp of
// the CTA has flagged an error.
__device__ __forceinline__ bool lwait(uint64_t* bar, uint32_t parity, volatile int* err, int* status, int site) {
    return dpipe::pwait(bar, parity, err, status, site);
}

// Pair holding item i under the cut of n items over P pairs.
__device__ __forceinline__ int pair_of(long long i, long long n, long long P) {
    const unsigned long long x = (unsigned long long)((i + 1) * P - 1);
    if ((x >> 32) == 0 && (n >> 32) == 0) return (int)((uint32_t)x / (uint32_t)n);  // 32-bit division
    return (int)(x / (unsigned long long)n);
}
// First item of pair bb under the cut of n items over P pairs: bb n / P.
__device__ __forceinline__ long long cut_at(long long bb, long long n, long long P) {
    const unsigned long long x = (unsigned long long)(bb * n);
    if ((x >> 32) == 0 && (P >> 32) == 0) return (long long)((uint32_t)x / (uint32_t)P);
    return (long long)(x / (unsigned long long)P);
}

// One batch of a log-sum-exp merge: fold the first n (<= K) of the runs' (max, sum) and
// outputs into the running (M, Ls, acc), rescaling them to the batch's new max.
template <int K>
__device__ __forceinline__ void lse_batch(const float2 (&ml)[K], const float4 (&v)[K], int n, float& M, float& Ls,
                                          float4& acc) {
    if (n <= 0) return;
    float bm = M;
#pragma unroll
    for (int j = 0; j < K; ++j)
        if (j < n) bm = fmaxf(bm, ml[j].x);
    const float rs = (M == -INFINITY) ? 0.0f : fast_exp2(M - bm);
    Ls *= rs;
    acc.x *= rs; acc.y *= rs; acc.z *= rs; acc.w *= rs;
    M = bm;
#pragma unroll
    for (int j = 0; j < K; ++j) {
        if (j >= n) break;
        const float wj = ml[j].x == -INFINITY ? 0.0f : fast_exp2(ml[j].x - M);
        Ls = fmaf(wj, ml[j].y, Ls);
        acc.x = fmaf(wj, v[j].x, acc.x); acc.y = fmaf(wj, v[j].y, acc.y);
        acc.z = fmaf(wj, v[j].z, acc.z); acc.w = fmaf(wj, v[j].w, acc.w);
    }
}

// Log-sum-exp merge of the runs of (sequence seq, KV head group qh0 / G) by one
// warp: the runs are the non-empty intersections of the sequence's items with
// the pairs' item ranges, each written to the workspace slot of its first
// chunk.  Lanes take 32 pairs at a time; pass 1 finds the max of every head,
// pass 2 weighs the runs (lane r holds run r's weights, broadcast by shuffles)
// while lanes cover the G x 64 outputs as float4s, four runs' loads in flight.
__device__ __forceinline__ void merge_runs(const Args& a, int seq, long long ps, int nchunks, long long n_items,
                                           long long P, int qh0, int lane, float* out) {
    const int G = a.G, Hq = a.Hq;
    const bool emit_partial = (a.flags & CVATTN_DECODE_EMIT_PARTIAL) != 0;
    const int b0 = pair_of(ps, n_items, P), b1 = pair_of(ps + nchunks - 1, n_items, P);
    const float* seq_ml = a.ws_ml + ((int64_t)seq * a.ws_chunks) * Hq * 2;
    const float* seq_o = a.ws_o + ((int64_t)seq * a.ws_chunks) * Hq * kD;
    auto run_slot = [&](int bb, bool& valid) {
        const long long blo = cut_at(bb, n_items, P), bhi = cut_at(bb + 1, n_items, P);
        valid = bb <= b1 && bhi > blo;  // a pair without items writes nothing
        return valid ? (int)((blo > ps ? blo : ps) - ps) : 0;
    };
    float M[kHP];
#pragma unroll
    for (int h = 0; h < kHP; ++h) M[h] = -INFINITY;
    for (int base = b0; base <= b1; base += 32) {
        bool valid;
        const int c = run_slot(base + lane, valid);
#pragma unroll
        for (int h = 0; h < kHP; ++h)
            if (h < G && valid) M[h] = fmaxf(M[h], __ldcg(seq_ml + ((int64_t)c * Hq + qh0 + h) * 2));
    }
#pragma unroll
    for (int h = 0; h < kHP; ++h) M[h] = dec::warp_max(M[h]);
    float Ls[kHP];
    float4 acc[4];
#pragma unroll
    for (int h = 0; h < kHP; ++h) Ls[h] = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    const int hsel = lane >> 4;  // output float4 k of this lane: head 2k + hsel, dims 4 (lane & 15) ..
    for (int base = b0; base <= b1; base += 32) {
        bool valid;
        const int c = run_slot(base + lane, valid);
        float w[kHP];
#pragma unroll
        for (int h = 0; h < kHP; ++h) {
            w[h] = 0.0f;
            if (h < G && valid) {
                const float2 ml = __ldcg(reinterpret_cast<const float2*>(seq_ml + ((int64_t)c * Hq + qh0 + h) * 2));
                w[h] = ml.x == -INFINITY ? 0.0f : fast_exp2(ml.x - M[h]);
                Ls[h] = fmaf(w[h], ml.y, Ls[h]);
            }
        }
        const uint32_t vm = __ballot_sync(0xffffffffu, valid);
        for (int r0 = 0; r0 < 32; r0 += 4) {
            if (!((vm >> r0) & 0xFu)) continue;
            float4 o[4][4];
            float ww[4][4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int rr = r0 + u;
                const bool on = (vm >> rr) & 1u;
                const int cr = __shfl_sync(0xffffffffu, c, rr);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float wa = __shfl_sync(0xffffffffu, w[2 * k], rr);
                    const float wb = __shfl_sync(0xffffffffu, w[2 * k + 1], rr);
                    const int h = 2 * k + hsel;
                    ww[u][k] = hsel ? wb : wa;
                    o[u][k] = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (on && h < G)
                        o[u][k] = dpipe::ldcg_f4(seq_o + ((int64_t)cr * Hq + qh0 + h) * kD + 4 * (lane & 15));
                }
            }
#pragma unroll
            for (int u = 0; u < 4; ++u)
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    acc[k].x = fmaf(ww[u][k], o[u][k].x, acc[k].x);
                    acc[k].y = fmaf(ww[u][k], o[u][k].y, acc[k].y);
                    acc[k].z = fmaf(ww[u][k], o[u][k].z, acc[k].z);
                    acc[k].w = fmaf(ww[u][k], o[u][k].w, acc[k].w);
                }
        }
    }
#pragma unroll
    for (int h = 0; h < kHP; ++h) Ls[h] = dec::warp_sum(Ls[h]);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int h = 2 * k + hsel;
        if (h < G) {
            const float l = hsel ? Ls[2 * k + 1] : Ls[2 * k];
            const float inv = emit_partial ? 1.0f : 1.0f / l;
            *reinterpret_cast<float4*>(out + (qh0 + h) * kD + 4 * (lane & 15)) =
                make_float4(acc[k].x * inv, acc[k].y * inv, acc[k].z * inv, acc[k].w * inv);
        }
    }
    if (emit_partial && lane < G) {
        float m = M[0], l = Ls[0];
#pragma unroll
        for (int h = 1; h < kHP; ++h)
            if (lane == h) { m = M[h]; l = Ls[h]; }
        a.partial_ml[((int64_t)seq * Hq + qh0 + lane) * 2] = m;
        a.partial_ml[((int64_t)seq * Hq + qh0 + lane) * 2 + 1] = l;
    }
}

// ------------------------------------------------------------------ kernel

template <int KT, int VT>
__global__ void __launch_bounds__(kMaxThreads, 1) decode_mma_kernel(const Args a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int gid = lane >> 2, tig = lane & 3;
    const int n_pairs = (int)(blockDim.x >> 6);
    const int G = a.G, Hq = a.Hq, n_seq = a.n_seq;
    constexpr int GBK = group_bytes(KT), GBV = group_bytes(VT);
    constexpr int headK = 2 * GBK, headV = 2 * GBV, rowK = 2 * headK, rowV = 2 * headV;
    constexpr bool K_MIN = BlockTraits<KT>::HAS_MIN, V_MIN = BlockTraits<VT>::HAS_MIN;
    const Smem L(rowK, rowV, n_pairs, K_MIN, V_MIN);
    const bool emit_partial = (a.flags & CVATTN_DECODE_EMIT_PARTIAL) != 0;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
    volatile int* err = reinterpret_cast<volatile int*>(smem + L.misc);
    int* pref = reinterpret_cast<int*>(smem + L.pref);
    int* slen = reinterpret_cast<int*>(smem + L.slen);
    griddep_launch_dependents();

    if (tid == 0) {
        for (int i = 0; i < n_pairs * kStages; ++i) {
            mbar_init(&bars[2 * i], 1u);      // full: the producer's arrive + transaction bytes
            mbar_init(&bars[2 * i + 1], 2u);  // empty: one arrive per warp of the pair
        }
        *err = 0;
        reinterpret_cast<int*>(smem + L.misc)[1] = 0;  // merge tasks posted
        fence_mbar_init();
    }
    // With CVATTN_DECODE_INPUTS_READY the lengths and cached rows are final: the
    // chunk scan and the first bulk loads run before griddepcontrol.wait; Q, the
    // new rows and every write wait.
    const bool early = (a.flags & CVATTN_DECODE_INPUTS_READY) != 0;
    if (!early) griddep_wait();
    if (warp == 0) {  // exclusive scan of chunk counts; invalid or empty sequences get none
        int carry = 0;
        for (int base = 0; base < n_seq; base += 32) {
            const int s = base + lane;
            int nc = 0;
            if (s < n_seq) {
                const int len = a.kv_len[s];
                const bool ok = len > 0 && len <= a.capacity && len <= a.max_kv_len;
                if (ok) nc = (len + kC - 1) / kC;
                slen[s] = ok ? len : 0;
            }
            int incl = nc;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            if (s < n_seq) pref[s] = carry + incl - nc;
            carry += __shfl_sync(0xffffffffu, incl, 31);
        }
        if (lane == 0) pref[n_seq] = carry;
        if (blockIdx.x == 0) {  // block 0 zeroes the outputs of empty / invalid sequences
            if (early) griddep_wait();
            for (int base = 0; base < n_seq; base += 32) {
                const int s = base + lane;
                const int len = s < n_seq ? a.kv_len[s] : 0;
                const bool bad_len = s < n_seq && !(len > 0 && len <= a.capacity && len <= a.max_kv_len);
                if (bad_len && len != 0) record_status(a.status, kStatusBadLength);
                uint32_t bad = __ballot_sync(0xffffffffu, bad_len);
                while (bad) {
                    const int z = base + __ffs(bad) - 1;
                    bad &= bad - 1;
                    float* out = a.out + (int64_t)z * a.out_seq_stride;
                    for (int i = lane; i < Hq * kD; i += 32) out[i] = 0.0f;
                    if (emit_partial)
                        for (int i = lane; i < Hq; i += 32) {
                            a.partial_ml[((int64_t)z * Hq + i) * 2] = -INFINITY;
                            a.partial_ml[((int64_t)z * Hq + i) * 2 + 1] = 0.0f;
                        }
                }
            }
        }
    }
    __syncthreads();

    const int pair = warp >> 1, g = warp & 1;
    const long long n_items = pref[n_seq];
    const long long P = (long long)gridDim.x * n_pairs;
    const int gp = blockIdx.x * n_pairs + pair;
    const int lo = (int)(gp * n_items / P);
    const int n_local = (int)((gp + 1) * n_items / P) - lo;
    uint8_t* ring = smem + L.ring0 + pair * L.pair_stride;
    float4* sK = reinterpret_cast<float4*>(smem + L.scl + warp * L.scl_warp);  // this warp's scale table
    float4* sV = sK + 32;
    float4* sKm = sV + 32;                  // K mins (types with a min)
    float4* sVm = sKm + (K_MIN ? 32 : 0);   // V mins (types with a min)
    uint64_t* pbars = bars + pair * kStages * 2;
    const bool producer = g == 0 && lane == 0;

    // producer cursor (lane 0 of the pair's first warp): the next item to load
    int pseq = 0, pchunk = 0, issued = 0;
    auto issue = [&](int t) {  // raw rows of local item t into slot t % kStages
        const int s = t % kStages;
        if (t >= kStages && !lwait(&pbars[2 * s + 1], ((t / kStages) - 1) & 1, err, a.status, 21)) return false;
        const uint8_t* kb = a.k_seq_ptrs ? reinterpret_cast<const uint8_t*>(a.k_seq_ptrs[pseq]) : a.k_base + pseq * a.k_nb2;
        const uint8_t* vb = a.v_seq_ptrs ? reinterpret_cast<const uint8_t*>(a.v_seq_ptrs[pseq]) : a.v_base + pseq * a.v_nb2;
        const int p0 = pchunk * kC, n = min(kC, slen[pseq] - p0);
        const uint8_t* ksrc = kb + (int64_t)p0 * rowK;
        const uint8_t* vsrc = vb + (int64_t)p0 * rowV;
        uint8_t* kdst = ring + s * L.stage;
        uint8_t* vdst = kdst + L.vofs;
        const uint32_t kbytes = (uint32_t)(n * rowK), vbytes = (uint32_t)(n * rowV);
        const uint32_t kbulk = ((reinterpret_cast<uintptr_t>(ksrc) & 15) == 0) ? (kbytes & ~15u) : 0u;
        const uint32_t vbulk = ((reinterpret_cast<uintptr_t>(vsrc) & 15) == 0) ? (vbytes & ~15u) : 0u;
        // tails (and unaligned rows) by plain 2-byte copies; the arrive below releases them
        for (uint32_t i = kbulk / 2; i < kbytes / 2; ++i)
            reinterpret_cast<uint16_t*>(kdst)[i] = reinterpret_cast<const uint16_t*>(ksrc)[i];
        for (uint32_t i = vbulk / 2; i < vbytes / 2; ++i)
            reinterpret_cast<uint16_t*>(vdst)[i] = reinterpret_cast<const uint16_t*>(vsrc)[i];
        mbar_arrive_expect_tx(&pbars[2 * s], kbulk + vbulk);
        if (kbulk) bulk_g2s(kdst, ksrc, kbulk, &pbars[2 * s]);
        if (vbulk) bulk_g2s(vdst, vsrc, vbulk, &pbars[2 * s]);
        dstream::next_item(slen, n_seq, pseq, pchunk);
        ++issued;
        return true;
    };
    if (producer && n_local > 0) {
        dpipe::item_of(pref, n_seq, lo, pseq, pchunk);
        for (int t = 0; t < kStages && t < n_local; ++t)
            if (!issue(t)) break;
    }
    if (early) griddep_wait();

    // ---- per-warp state
    const int qh0 = g * G;  // first query head of this KV head
    const bool head_ok = gid < G;
    uint32_t qa[2][2][4];   // Q A fragments [block][k-step]
    float esc = 0.0f;       // 2^-e_Q * scale (log2 units) of head gid
    float qsum[2] = {0.0f, 0.0f};
    float O[8][4];
    float mref = -INFINITY, lsum = 0.0f, pmv[2] = {0.0f, 0.0f};
    int ev[2] = {0, 0};
    int run_n = 0, run_c0 = 0;
    // sequences this warp must merge: only the first and the last run of a range can be partial
    int n_merge = 0, mseq0 = 0, mn0 = 0, mseq1 = 0, mn1 = 0;
    int cseq = 0, cchunk = 0;
    if (n_local > 0) dpipe::item_of(pref, n_seq, lo, cseq, cchunk);
    int qseq = -1;
    float xk_new[2] = {0.0f, 0.0f}, xv_new[2] = {0.0f, 0.0f};

    // RoPE fused into the step (cvattn_decode_rope; n_dims = head_dim = 64): Q and the new K row
    // turn by the new token's position, as ggml_rope_ext (src/cosyvoice-llm.cpp:56-57); the
    // (cos, sin) of pair k comes from lane k (one sincosf per lane and sequence).
    const RopeDev rope{a.rope_mode, a.rope_n_dims, kD, a.rope_theta_scale, a.rope_freq_scale, a.rope_attn_factor};
    auto load_q = [&](int sq, float2 rcs) {
        float x[2][8];
        float am = 0.0f;
        if (head_ok) {
            const float* qr = a.q + (int64_t)sq * a.q_seq_stride + (qh0 + gid) * kD;
#pragma unroll
            for (int b = 0; b < 2; ++b) {
                if constexpr (KT == kQ8_0) {
                    const float4 f0 = *reinterpret_cast<const float4*>(qr + 32 * b + 8 * tig);
                    const float4 f1 = *reinterpret_cast<const float4*>(qr + 32 * b + 8 * tig + 4);
                    x[b][0] = f0.x; x[b][1] = f0.y; x[b][2] = f0.z; x[b][3] = f0.w;
                    x[b][4] = f1.x; x[b][5] = f1.y; x[b][6] = f1.z; x[b][7] = f1.w;
                } else {
                    const float4 f0 = *reinterpret_cast<const float4*>(qr + 32 * b + 4 * tig);
                    const float4 f1 = *reinterpret_cast<const float4*>(qr + 32 * b + 16 + 4 * tig);
                    x[b][0] = f0.x; x[b][1] = f0.y; x[b][2] = f1.x; x[b][3] = f1.y;
                    x[b][4] = f0.z; x[b][5] = f0.w; x[b][6] = f1.z; x[b][7] = f1.w;
                }
            }
        } else {
#pragma unroll
            for (int b = 0; b < 2; ++b)
#pragma unroll
                for (int i = 0; i < 8; ++i) x[b][i] = 0.0f;
        }
        if (rope.n_dims > 0) {
            if (rope.mode & 2) {  // NEOX: element e of block 0 pairs with element e of block 1 (pair k = e)
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int k = kelem<KT>(tig, i);
                    const float2 cs = make_float2(__shfl_sync(0xffffffffu, rcs.x, k), __shfl_sync(0xffffffffu, rcs.y, k));
                    const float a0 = x[0][i], a1 = x[1][i];
                    x[0][i] = rope_rotate(a0, a1, cs, true);
                    x[1][i] = rope_rotate(a1, a0, cs, false);
                }
            } else {  // NORMAL: elements 2k and 2k + 1 are this lane's entries i and i + 1 (i even)
#pragma unroll
                for (int b = 0; b < 2; ++b)
#pragma unroll
                    for (int i = 0; i < 8; i += 2) {
                        const int k = (32 * b + kelem<KT>(tig, i)) >> 1;
                        const float2 cs = make_float2(__shfl_sync(0xffffffffu, rcs.x, k), __shfl_sync(0xffffffffu, rcs.y, k));
                        const float a0 = x[b][i], a1 = x[b][i + 1];
                        x[b][i] = rope_rotate(a0, a1, cs, true);
                        x[b][i + 1] = rope_rotate(a1, a0, cs, false);
                    }
            }
        }
#pragma unroll
        for (int b = 0; b < 2; ++b)
#pragma unroll
            for (int i = 0; i < 8; ++i) am = fmaxf(am, fabsf(x[b][i]));
        am = quad_max(am);
        const int ex = dtc::norm_exp(am);
        const float sc = pow2f(ex);
        esc = pow2f(-ex) * a.scale_log2;
#pragma unroll
        for (int b = 0; b < 2; ++b) {
            float part = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; ++i) part += x[b][i];
            qsum[b] = quad_sum(part) * a.scale_log2;
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                split2(x[b][4 * j] * sc, x[b][4 * j + 1] * sc, qa[b][j][0], qa[b][j][1]);
                split2(x[b][4 * j + 2] * sc, x[b][4 * j + 3] * sc, qa[b][j][2], qa[b][j][3]);
            }
        }
    };

    for (int t = 0; t < n_local; ++t) {
        const int s = t % kStages;
        const int seq = cseq, chunk = cchunk;
        dstream::next_item(slen, n_seq, cseq, cchunk);
        const int len = slen[seq];
        const int p0 = chunk * kC, n = min(kC, len - p0);
        const int nchunks = (len + kC - 1) / kC;
        const uint8_t* Kst = ring + s * L.stage + g * headK;
        const uint8_t* Vst = ring + s * L.stage + L.vofs + g * headV;
        if (seq != qseq) {
            float2 rcs = make_float2(1.0f, 0.0f);  // (cos, sin) of pair k = lane at position len - 1
            if (rope.n_dims > 0) rcs = rope_cs(rope, rope_theta(rope, len - 1, lane));
            // the step's new K/V row of this sequence and KV head (fused append), loaded with Q
            // so its latency is not paid at the sequence's last chunk
            if (a.k_new) {
#pragma unroll
                for (int b = 0; b < 2; ++b) {
                    xk_new[b] = a.k_new[(int64_t)seq * 2 * kD + g * kD + b * 32 + lane];
                    xv_new[b] = a.v_new[(int64_t)seq * 2 * kD + g * kD + b * 32 + lane];
                }
                if (rope.n_dims > 0) {  // the new K row turns by position len - 1
                    if (rope.mode & 2) {  // NEOX: element lane of block 0 pairs with element lane of block 1
                        const float a0 = xk_new[0], a1 = xk_new[1];
                        xk_new[0] = rope_rotate(a0, a1, rcs, true);
                        xk_new[1] = rope_rotate(a1, a0, rcs, false);
                    } else {  // NORMAL: elements lane and lane ^ 1 of block b, pair 16 b + lane / 2
#pragma unroll
                        for (int b = 0; b < 2; ++b) {
                            const float partner = __shfl_xor_sync(0xffffffffu, xk_new[b], 1);
                            const int k = 16 * b + (lane >> 1);
                            const float2 cs = make_float2(__shfl_sync(0xffffffffu, rcs.x, k), __shfl_sync(0xffffffffu, rcs.y, k));
                            xk_new[b] = rope_rotate(xk_new[b], partner, cs, (lane & 1) == 0);
                        }
                    }
                }
            }
            load_q(seq, rcs);
            qseq = seq;
        }
        // raw rows of item t have landed (lane 0 waits, the warp follows)
        {
            bool ok = true;
            if (lane == 0) ok = lwait(&pbars[2 * s], (t / kStages) & 1, err, a.status, 22);
            if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
        }
        if (a.k_new && chunk == nchunks - 1) {
            // update_cache of the step's row (position len - 1): this warp's head, into the slot and the cache
            const uint8_t* kb = a.k_seq_ptrs ? reinterpret_cast<const uint8_t*>(a.k_seq_ptrs[seq]) : a.k_base + seq * a.k_nb2;
            const uint8_t* vb = a.v_seq_ptrs ? reinterpret_cast<const uint8_t*>(a.v_seq_ptrs[seq]) : a.v_base + seq * a.v_nb2;
            const int rr = len - 1 - p0;
#pragma unroll
            for (int b = 0; b < 2; ++b) {  // one quantization, stored into the slot and the cache
                quantize_block_warp<KT>(xk_new[b], const_cast<uint8_t*>(Kst) + rr * rowK + b * GBK, lane,
                                        const_cast<uint8_t*>(kb) + (int64_t)(len - 1) * rowK + g * headK + b * GBK);
                quantize_block_warp<VT>(xv_new[b], const_cast<uint8_t*>(Vst) + rr * rowV + b * GBV, lane,
                                        const_cast<uint8_t*>(vb) + (int64_t)(len - 1) * rowV + g * headV + b * GBV);
            }
            fence_proxy_async_smem();  // the slot is later overwritten by the bulk copies
            __syncwarp();
        }
        // Scale table of the item (this warp's KV head): lane q converts the block scales
        // (and mins) of positions 2q and 2q + 1 once, for the four lanes that read them in
        // the sub-steps below.  Positions past n get zero V weight (P' = 0, no min term),
        // so only the scores of a partial item need a mask.  The V exponent of each block
        // for this run comes from max |d_V| over the item's positions.
        int evn[2];
        {
            float dk[2][2], dvv[2][2], mk[2][2], mvv[2][2];  // [position of the pair][block]
            float vm[2] = {0.0f, 0.0f};
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int pos = 2 * lane + u;
                const bool valid = pos < n;
#pragma unroll
                for (int b = 0; b < 2; ++b) {
                    dk[u][b] = mk[u][b] = dvv[u][b] = mvv[u][b] = 0.0f;
                    if (valid) {
                        const uint8_t* kr = Kst + pos * rowK + b * GBK;
                        dk[u][b] = h2f((uint16_t)ld_u16(kr));
                        if constexpr (K_MIN) {
                            constexpr float kCentre = BlockTraits<KT>::OFF_QH >= 0 ? 16.0f : 8.0f;
                            mk[u][b] = fmaf(kCentre, dk[u][b], h2f((uint16_t)ld_u16(kr + BlockTraits<KT>::OFF_M)));
                        }
                        vscale<VT>(Vst + pos * rowV + b * GBV, dvv[u][b], mvv[u][b]);
                        vm[b] = fmaxf(vm[b], fabsf(dvv[u][b]));
                    }
                }
            }
#pragma unroll
            for (int b = 0; b < 2; ++b) {
                vm[b] = dec::warp_max(vm[b]);
                if (run_n == 0) {
                    evn[b] = dstream::v_exp_target(vm[b]);
                } else {
                    const int x = vm[b] > 0.0f ? dstream::ilog2f(vm[b]) + ev[b] : 0;
                    evn[b] = (x < kEvMin || x > kEvMax) ? dstream::v_exp_target(vm[b]) : ev[b];
                }
            }
            const float f0 = pow2f(evn[0]), f1 = pow2f(evn[1]);
            sK[lane] = make_float4(dk[0][0], dk[1][0], dk[0][1], dk[1][1]);
            sV[lane] = make_float4(dvv[0][0] * f0, dvv[1][0] * f0, dvv[0][1] * f1, dvv[1][1] * f1);
            if constexpr (K_MIN) sKm[lane] = make_float4(mk[0][0], mk[1][0], mk[0][1], mk[1][1]);
            if constexpr (V_MIN) sVm[lane] = make_float4(mvv[0][0], mvv[1][0], mvv[0][1], mvv[1][1]);
            __syncwarp();
        }
        if (run_n == 0) {
#pragma unroll
            for (int j = 0; j < 8; ++j)
#pragma unroll
                for (int i = 0; i < 4; ++i) O[j][i] = 0.0f;
            mref = -INFINITY;
            lsum = 0.0f;
            pmv[0] = pmv[1] = 0.0f;
            run_c0 = chunk;
        } else {
#pragma unroll
            for (int b = 0; b < 2; ++b)
                if (evn[b] != ev[b]) {  // uniform per warp
                    const float f = pow2f(evn[b] - ev[b]);
#pragma unroll
                    for (int j = 4 * b; j < 4 * b + 4; ++j)
#pragma unroll
                        for (int i = 0; i < 4; ++i) O[j][i] *= f;
                }
        }
        ev[0] = evn[0];
        ev[1] = evn[1];

        // One 16-position sub-step: S = Q.K^T for two 8-position tiles, the scores of head gid
        // at this lane's 4 positions (log2 units), the lazy reference max, P' = P d_V 2^ev split
        // into the A fragments of P.V, and O += P'.V over 8 dim tiles.  kFull: all 64 positions
        // of the item are valid, no score needs a mask.  (Lanes of a padding head, gid >= G, run
        // on zero Q rows: finite scores whose rows of O are never written.)
        auto sub_step = [&](auto full_tag, int sub) {
            constexpr bool kFull = decltype(full_tag)::value;
            float acc[2][2][4];
#pragma unroll
            for (int b = 0; b < 2; ++b)
#pragma unroll
                for (int tt = 0; tt < 2; ++tt)
#pragma unroll
                    for (int i = 0; i < 4; ++i) acc[b][tt][i] = 0.0f;
#pragma unroll
            for (int tt = 0; tt < 2; ++tt) {
                const int pos = 16 * sub + 8 * tt + gid;  // the B column of this lane group
                uint32_t r[4];
                kfrag<KT, 0>(Kst + pos * rowK, tig, r);
                mma16816(acc[0][tt], qa[0][0], r[0], r[1]);
                mma16816(acc[0][tt], qa[0][1], r[2], r[3]);
                kfrag<KT, 1>(Kst + pos * rowK + GBK, tig, r);
                mma16816(acc[1][tt], qa[1][0], r[0], r[1]);
                mma16816(acc[1][tt], qa[1][1], r[2], r[3]);
            }
            float sc[4];
            float4 dvq[2], mvq[2];
            (void)mvq;
#pragma unroll
            for (int tt = 0; tt < 2; ++tt) {
                const int q = 8 * sub + 4 * tt + tig;  // positions 2q, 2q + 1
                const float4 dk = sK[q];
                dvq[tt] = sV[q];
                float4 mk = make_float4(0.f, 0.f, 0.f, 0.f);
                if constexpr (K_MIN) mk = sKm[q];
                if constexpr (V_MIN) mvq[tt] = sVm[q];
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    const float d0 = i ? dk.y : dk.x, d1 = i ? dk.w : dk.z;
                    float v = d0 * (acc[0][tt][i] + acc[0][tt][2 + i]) + d1 * (acc[1][tt][i] + acc[1][tt][2 + i]);
                    v *= esc;
                    if constexpr (K_MIN) v += (i ? mk.y : mk.x) * qsum[0] + (i ? mk.w : mk.z) * qsum[1];
                    if constexpr (!kFull) v = (2 * q + i < n) ? v : -INFINITY;
                    sc[2 * tt + i] = v;
                }
            }
            // ---- lazy reference max of head gid (uniform decision per warp)
            {
                const float mx = quad_max(fmaxf(fmaxf(sc[0], sc[1]), fmaxf(sc[2], sc[3])));
                const bool big = mx > mref + kLazyLog2;  // a run's first scores: mref = -inf
                if (__any_sync(0xffffffffu, big || (emit_partial && mx > mref))) {
                    const float mn = fmaxf(mref, mx);
                    const float alpha = (mn == -INFINITY || mref == -INFINITY) ? (mref == -INFINITY ? 0.0f : 1.0f)
                                                                               : fast_exp2(mref - mn);
                    if (mn != -INFINITY) {
#pragma unroll
                        for (int j = 0; j < 8; ++j)
#pragma unroll
                            for (int i = 0; i < 4; ++i) O[j][i] *= alpha;
                        lsum *= alpha;
                        pmv[0] *= alpha;
                        pmv[1] *= alpha;
                        mref = mn;
                    }
                }
            }
            // ---- P = 2^(s - mref) <= 2^8, P' = P d_V 2^ev split into the A fragments of P.V
            float p[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                if constexpr (kFull) p[k] = fast_exp2(sc[k] - mref);
                else p[k] = sc[k] == -INFINITY ? 0.0f : fast_exp2(sc[k] - mref);
            }
            lsum += (p[0] + p[1]) + (p[2] + p[3]);
            uint32_t pa[2][4];
#pragma unroll
            for (int b = 0; b < 2; ++b) {
                const float x0 = p[0] * (b ? dvq[0].z : dvq[0].x), x1 = p[1] * (b ? dvq[0].w : dvq[0].y);
                const float x2 = p[2] * (b ? dvq[1].z : dvq[1].x), x3 = p[3] * (b ? dvq[1].w : dvq[1].y);
                if constexpr (V_MIN) {
                    pmv[b] = fmaf(p[0], b ? mvq[0].z : mvq[0].x, pmv[b]);
                    pmv[b] = fmaf(p[1], b ? mvq[0].w : mvq[0].y, pmv[b]);
                    pmv[b] = fmaf(p[2], b ? mvq[1].z : mvq[1].x, pmv[b]);
                    pmv[b] = fmaf(p[3], b ? mvq[1].w : mvq[1].y, pmv[b]);
                }
                split2(x0, x1, pa[b][0], pa[b][1]);
                split2(x2, x3, pa[b][2], pa[b][3]);
            }
            // ---- O += P' . V, 8 dim tiles (4 per V block)
            {
                uint32_t v0[4], v1[4];
                const uint8_t* vr = Vst + (16 * sub + 2 * tig) * rowV;
                vfrag<VT, 0>(vr, vr + rowV, gid, v0);
                vfrag<VT, 0>(vr + 8 * rowV, vr + 9 * rowV, gid, v1);
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) mma16816(O[jj], pa[0], v0[jj], v1[jj]);
                vfrag<VT, 1>(vr + GBV, vr + rowV + GBV, gid, v0);
                vfrag<VT, 1>(vr + 8 * rowV + GBV, vr + 9 * rowV + GBV, gid, v1);
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) mma16816(O[4 + jj], pa[1], v0[jj], v1[jj]);
            }
        };
        if (n == kC) {
#pragma unroll 1
            for (int sub = 0; sub < kC / 16; ++sub) sub_step(std::true_type{}, sub);
        } else {
#pragma unroll 1
            for (int sub = 0; sub < kC / 16 && 16 * sub < n; ++sub) sub_step(std::false_type{}, sub);
        }
        // slot s may be refilled once both warps are done with it
        __syncwarp();
        if (lane == 0) mbar_arrive(&pbars[2 * s + 1]);
        if (producer && issued < n_local) {
            if (!issue(issued)) *err = 1;
        }
        if (run_n == 0) run_c0 = chunk;
        ++run_n;
        if (t + 1 < n_local && cseq == seq) continue;

        // ------------------------------------------------ end of the run
        const float l = quad_sum(lsum);
        float pm[2] = {0.0f, 0.0f};
        if constexpr (V_MIN) {
            pm[0] = quad_sum(pmv[0]);
            pm[1] = quad_sum(pmv[1]);
        }
        const float ie0 = pow2f(-ev[0]), ie1 = pow2f(-ev[1]);
        float* out = a.out + (int64_t)seq * a.out_seq_stride;
        const int qh = qh0 + gid;
        if (run_n == nchunks) {  // the whole sequence went through this warp
            if (head_ok) {
                const float inv = emit_partial ? 1.0f : 1.0f / l;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int b = j >> 2;
#pragma unroll
                    for (int i = 0; i < 2; ++i) {
                        const int dim = 32 * b + velem<VT>(2 * tig + i, j & 3);
                        out[qh * kD + dim] = ((O[j][i] + O[j][2 + i]) * (b ? ie1 : ie0) + pm[b]) * inv;
                    }
                }
                if (emit_partial && tig == 0) {
                    a.partial_ml[((int64_t)seq * Hq + qh) * 2] = mref;
                    a.partial_ml[((int64_t)seq * Hq + qh) * 2 + 1] = l;
                }
            }
        } else {
            float* wso = a.ws_o + (((int64_t)seq * a.ws_chunks + run_c0) * Hq) * kD;
            float* wsml = a.ws_ml + (((int64_t)seq * a.ws_chunks + run_c0) * Hq) * 2;
            if (head_ok) {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int b = j >> 2;
#pragma unroll
                    for (int i = 0; i < 2; ++i) {
                        const int dim = 32 * b + velem<VT>(2 * tig + i, j & 3);
                        wso[qh * kD + dim] = (O[j][i] + O[j][2 + i]) * (b ? ie1 : ie0) + pm[b];
                    }
                }
                if (tig == 0) *reinterpret_cast<float2*>(wsml + qh * 2) = make_float2(mref, l);
            }
            __syncwarp();  // orders the warp's partial stores before lane 0's release
            uint32_t last = 0;
            if (lane == 0) {  // the release publishes the warp's partial; acquire sees the others'
                const uint32_t prev = dstream::atom_add_acq_rel(&a.ws_cnt[(int64_t)seq * 2 + g], (uint32_t)run_n);
                last = (prev + (uint32_t)run_n == (uint32_t)nchunks) ? 1u : 0u;
            }
            last = __shfl_sync(0xffffffffu, last, 0);
            if (last) {  // merged after the loop, when the Q and O registers are free
                if (n_merge == 0) { mseq0 = seq; mn0 = nchunks; } else { mseq1 = seq; mn1 = nchunks; }
                ++n_merge;
            }
        }
        run_n = 0;
    }

    // ---- The merges this CTA's warps were elected for (the last writer of a sequence's runs for
    // one KV head), done by every thread of the CTA: the elected warp lists the run slots in its
    // scale table (free after the loop) and posts a task; after one CTA barrier, thread =
    // (task, head, 4 dims) loads up to kMergeBatch runs' (max, sum) and outputs at once, for two items together, so a sequence
    // split over many pairs costs a round or two of L2 loads instead of one warp's many.  (A
    // sequence over more than kMaxMergeRuns pairs, and every merge of a one-pair CTA, whose two
    // warps would otherwise share 64 threads, is merged by its warp alone.)
    int* mcount = reinterpret_cast<int*>(smem + L.misc) + 1;
    MergeTask* tasks = reinterpret_cast<MergeTask*>(smem + L.tasks);
    int* slot_tab = reinterpret_cast<int*>(smem + L.scl);
    __syncwarp();  // the lanes' partial loads follow lane 0's acquire
    for (int i = 0; i < n_merge && i < 2; ++i) {
        const int sq = i ? mseq1 : mseq0, nch = i ? mn1 : mn0;
        const long long ps = pref[sq];
        const int b0 = pair_of(ps, n_items, P), b1 = pair_of(ps + nch - 1, n_items, P);
        if (b1 - b0 + 1 > kMaxMergeRuns || n_pairs < 2) {  // (one pair: its two warps merge in parallel)
            merge_runs(a, sq, ps, nch, n_items, P, qh0, lane, a.out + (int64_t)sq * a.out_seq_stride);
            if (lane == 0) a.ws_cnt[(int64_t)sq * 2 + g] = 0u;
            continue;
        }
        const int off = (warp * L.scl_warp) / 4 + i * kMaxMergeRuns;
        int nr = 0;  // the slots of the pairs' runs, listed 32 pairs at a time (a pair without items has none)
        for (int base = 0; base <= b1 - b0; base += 32) {
            int c = -1;
            if (base + lane <= b1 - b0) {
                const long long blo = cut_at(b0 + base + lane, n_items, P), bhi = cut_at(b0 + base + lane + 1, n_items, P);
                if (bhi > blo) c = (int)((blo > ps ? blo : ps) - ps);
            }
            const uint32_t vm = __ballot_sync(0xffffffffu, c >= 0);
            if (c >= 0) slot_tab[off + nr + __popc(vm & ((1u << lane) - 1u))] = c;
            nr += __popc(vm);
        }
        if (lane == 0) tasks[atomicAdd(mcount, 1)] = MergeTask{sq, g, nr, off};
    }
    __syncthreads();  // tasks posted; the electing acquires precede every thread's partial loads
    {
        const int n_tasks = *mcount;
        // thread = two merge items (task, head, 4 dims) at once, so the loads of both are in flight
        // together: a CTA elected for several sequences pays half the rounds of L2 loads
        const int n_work = n_tasks * G * (kD / 4);
        auto item_of = [&](int w, MergeTask& T, int& h, int& dq) {
            T = tasks[w / (G * (kD / 4))];
            h = (w / (kD / 4)) % G;
            dq = (w % (kD / 4)) * 4;
        };
        for (int w0 = tid; w0 < n_work; w0 += 2 * blockDim.x) {
            const int w1 = w0 + blockDim.x;
            const bool two = w1 < n_work;
            MergeTask TA, TB;
            int hA, dqA, hB, dqB;
            item_of(w0, TA, hA, dqA);
            item_of(two ? w1 : w0, TB, hB, dqB);
            const int qhA = TA.g * G + hA, qhB = TB.g * G + hB;
            const float* mlA = a.ws_ml + ((int64_t)TA.seq * a.ws_chunks) * Hq * 2 + qhA * 2;
            const float* oA = a.ws_o + ((int64_t)TA.seq * a.ws_chunks) * Hq * kD + qhA * kD + dqA;
            const float* mlB = a.ws_ml + ((int64_t)TB.seq * a.ws_chunks) * Hq * 2 + qhB * 2;
            const float* oB = a.ws_o + ((int64_t)TB.seq * a.ws_chunks) * Hq * kD + qhB * kD + dqB;
            float MA = -INFINITY, LA = 0.0f, MB = -INFINITY, LB = 0.0f;
            float4 accA = make_float4(0.f, 0.f, 0.f, 0.f), accB = accA;
            const int RR = TA.nruns > TB.nruns ? TA.nruns : TB.nruns;
            for (int r0 = 0; r0 < RR; r0 += kMergeBatch) {
                float2 ma[kMergeBatch], mb[kMergeBatch];
                float4 va[kMergeBatch], vb[kMergeBatch];
#pragma unroll
                for (int j = 0; j < kMergeBatch; ++j) {
                    const int ca = slot_tab[TA.slots + min(r0 + j, TA.nruns - 1)];
                    const int cb = slot_tab[TB.slots + min(r0 + j, TB.nruns - 1)];
                    ma[j] = __ldcg(reinterpret_cast<const float2*>(mlA + (int64_t)ca * Hq * 2));
                    va[j] = dpipe::ldcg_f4(oA + (int64_t)ca * Hq * kD);
                    mb[j] = __ldcg(reinterpret_cast<const float2*>(mlB + (int64_t)cb * Hq * 2));
                    vb[j] = dpipe::ldcg_f4(oB + (int64_t)cb * Hq * kD);
                }
                lse_batch<kMergeBatch>(ma, va, TA.nruns - r0, MA, LA, accA);
                lse_batch<kMergeBatch>(mb, vb, TB.nruns - r0, MB, LB, accB);
            }
            for (int k = 0; k < (two ? 2 : 1); ++k) {
                const MergeTask& T = k ? TB : TA;
                const int h = k ? hB : hA, dq = k ? dqB : dqA, qh = k ? qhB : qhA;
                const float Mk = k ? MB : MA, Lk = k ? LB : LA;
                const float4 acc = k ? accB : accA;
                float* out = a.out + (int64_t)T.seq * a.out_seq_stride;
                const float inv = emit_partial ? 1.0f : 1.0f / Lk;
                *reinterpret_cast<float4*>(out + qh * kD + dq) = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
                if (dq == 0) {
                    if (emit_partial) {
                        a.partial_ml[((int64_t)T.seq * Hq + qh) * 2] = Mk;
                        a.partial_ml[((int64_t)T.seq * Hq + qh) * 2 + 1] = Lk;
                    }
                    if (h == 0) a.ws_cnt[(int64_t)T.seq * 2 + T.g] = 0u;  // the ticket is not read again in this launch
                }
            }
        }
    }

    // copies still in flight into this pair's ring (an early exit) complete before the CTA ends
    if (producer) {
        int done = 0;
        for (int t = max(0, issued - kStages); t < issued; ++t) {
            const int s = t % kStages;
            if (!mbar_wait(&pbars[2 * s], (t / kStages) & 1, nullptr, 0)) break;
            ++done;
        }
        (void)done;
    }
}

template <int KT>
cudaError_t launch_for_k(cudaStream_t s, const Args& a, int v_type, int n_sms);
template <> cudaError_t launch_for_k<kQ4_0>(cudaStream_t, const Args&, int, int);
template <> cudaError_t launch_for_k<kQ4_1>(cudaStream_t, const Args&, int, int);
template <> cudaError_t launch_for_k<kQ5_0>(cudaStream_t, const Args&, int, int);
template <> cudaError_t launch_for_k<kQ5_1>(cudaStream_t, const Args&, int, int);
template <> cudaError_t launch_for_k<kQ8_0>(cudaStream_t, const Args&, int, int);

inline bool supported_type(int t) { return t == kQ4_0 || t == kQ4_1 || t == kQ5_0 || t == kQ5_1 || t == kQ8_0; }

// Warp pairs per CTA for this type pair: as many as fit the shared-memory budget.
inline int max_pairs(int k_type, int v_type) {
    const int rowK = (int)type_row_bytes(k_type, 2 * kD), rowV = (int)type_row_bytes(v_type, 2 * kD);
    const bool k_min = k_type == kQ4_1 || k_type == kQ5_1, v_min = v_type == kQ4_1 || v_type == kQ5_1;
    int p = kMaxPairs;
    while (p > 1 && Smem(rowK, rowV, p, k_min, v_min).total > kSmemLimit) --p;
    return p;
}

// Launch shape for `items` 64-position items: warp pairs per CTA and CTAs.  As many pairs as
// fit (at most one per item per SM); latency-bound launches (at most kLatencyItemsPerSm items
// per SM) take at most kLatencyPairs: with more, a sequence splits into more runs and the pairs
// contend for issue slots, and with fewer the CTA is small enough to share its SM with the next
// launch's (measured on the 24-layer decode step, 7.7 items per SM: 6 pairs 24.7 us per layer,
// 4 pairs 22.7, 3 or 2 pairs 28-29).
inline void launch_shape(int k_type, int v_type, long items, int n_sms, int& pairs, int& grid) {
    pairs = max_pairs(k_type, v_type);
    const long per_sm = (items + n_sms - 1) / n_sms;
    if (per_sm < pairs) pairs = (int)(per_sm > 0 ? per_sm : 1);
    if (per_sm <= kLatencyItemsPerSm && pairs > kLatencyPairs) pairs = kLatencyPairs;
    const long ctas_needed = (items + pairs - 1) / pairs;
    grid = (int)(ctas_needed < n_sms ? (ctas_needed > 0 ? ctas_needed : 1) : n_sms);
}

// Whether the warp-MMA kernel should take a launch of n_seq sequences and `items` items (the
// host bound): throughput-bound launches (kMmaItemsPerSm items per SM or more), and every
// launch of at least one item per SM whose sequences span at most 2 kMaxMergeRuns pairs each.
// (Measured, one layer, per launch, against the streaming kernel: the 64-sequence decode
// mix 20.9 vs 22.9 us, 148 x 64 6.9 vs 8.2, 64 x 256 10.3 vs 11.7, 3 x 4096 29.1 vs 43.3,
// 8 x 4096 26.4 vs 30.7, 16 x 4096 22.0 vs 24.8; below one item per SM the streaming kernel
// wins: 1 x 4096 50.9 vs 42.8, 2 x 4096 51.2 vs 45.5, 1 x 8192 93.6 vs 80.8.)
constexpr long kMmaItemsPerSm = 32;
inline bool mma_pays(int k_type, int v_type, long n_seq, long items, int n_sms) {
    if (items >= kMmaItemsPerSm * n_sms) return true;
    if (n_seq <= 0 || items < n_sms) return false;
    int pairs = 1, grid = 1;
    launch_shape(k_type, v_type, items, n_sms, pairs, grid);
    return (long)grid * pairs / n_seq + 1 <= 2 * kMaxMergeRuns;
}

}  // namespace dmma
}  // namespace cvattn
