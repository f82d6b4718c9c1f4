// decode_pipe.cuh -- persistent, warp-specialized tensor-core split-KV decode.
//
// Same contract as decode.cuh / decode_tc.cuh (one query row per sequence,
// ggml_flash_attn_ext semantics with f32 precision, src/cosyvoice-kv-cache.cpp:
// 379-386; optional fused update_cache append :316,322; split partials merged
// by the last chunk to finish) and the same exact-integer tensor-core math as
// decode_tc.cuh, organised so that HBM never idles:
//
//   one CTA per SM; the (sequence, 128-position chunk) work items are cut
//   into one contiguous range per CTA, and item t of a CTA alternates between
//   the two halves of its range (t even: first half) and uses slot s = t & 1
//   of every double-buffered resource;
//   warp 16     producer: cp.async.bulk of item t+2's raw K/V rows into raw
//               slot s as soon as item t's converters release it;
//   warps 0-7   two converter groups (group s takes the items of slot s):
//               raw ggml blocks -> 128B-swizzled f16 tiles of exact integer
//               quants + fp32 scales, and the item's Q hi/lo tile;
//   warp 17     MMA issuer polling both stages: S^T(t) = K.Q^T once tiles
//               are ready, O^T(t) = V^T.P' once P' is ready;
//   warps 8-15  two softmax groups (group s takes the items of slot s):
//               scores from TMEM, chunk max / sum, P' rows, then the chunk's
//               output merged into the group's running partial of the
//               sequence (consecutive chunks of one half of the range).
// A run that covers a whole sequence writes the output directly; otherwise
// the run's partial lands in the workspace slot of its first chunk, the
// run's other slots are marked empty, and a ticket counting chunks elects the
// last writer, which merges the written partials (log-sum-exp).  A converter
// group reuses its slot once the O MMA of two items back has completed, so
// conversion of item t+2 overlaps softmax and epilogue of items t and t+1.
// mbarriers hand each stage from role to role; every wait is bounded and a
// failed wait stops all roles through a shared error flag.
#pragma once

#include "decode_tc.cuh"

namespace cvattn {
namespace dpipe {

using dec::Args;
using dtc::convert_group;
using dtc::norm_exp;
using dtc::pow2f;

constexpr int kD = 64;
constexpr int kC = 128;
constexpr int kHP = 8;
constexpr int kGroup = 128;          // threads per converter / softmax group
constexpr int kThreads = 576;        // 8 converter + 8 softmax + producer + MMA warps
constexpr int kSoftWarp0 = 8;
constexpr int kProdWarp = 16;
constexpr int kMmaWarp = 17;
constexpr uint32_t kTmemCols = 512;  // S stages at columns 0 / 64, O stages at 128 / 192, running O at 256 / 264
constexpr uint32_t kRunCol = 256;
constexpr int kMaxSeq = 512;         // prefix-sum table in shared memory
constexpr int kBarConv = 1;          // named barriers: converter group s uses 1 + s,
constexpr int kBarSoft = 3;          //                 softmax group s uses 3 + s
constexpr int kRedFloats = 1024;     // per softmax group: reductions (256), or the combine's chunk weights

enum { B_RAW_FULL = 0, B_RAW_EMPTY = 2, B_TILE_FULL = 4, B_S_FULL = 6, B_P_FULL = 8, B_O_FULL = 10, B_COUNT = 12 };

struct Smem {
    int raw[2], ktile[2], vtile[2], qtile[2];
    int dk[2], mk[2], dv[2], mv[2], qsum[2], esc[2], wmax[2];  // written by converters
    int red[2], stat[2];                                      // written by softmax group s
    int pref, bars, misc, total;
    __host__ __device__ Smem(int rowK, int rowV, bool k_min, bool v_min) {
        int o = 0;
        const int rawb = dtc::round_up(kC * (rowK + rowV), 1024);
        for (int s = 0; s < 2; ++s) { raw[s] = o; o += rawb; }
        for (int s = 0; s < 2; ++s) { ktile[s] = o; o += 2 * 16384; }  // K tiles; P' (16 KB) once S is done
        for (int s = 0; s < 2; ++s) { vtile[s] = o; o += 2 * 16384; }
        for (int s = 0; s < 2; ++s) { qtile[s] = o; o += 2 * 2048; }
        for (int s = 0; s < 2; ++s) {
            dk[s] = o;   o += 2 * 2 * kC * 4;
            mk[s] = o;   o += k_min ? 2 * 2 * kC * 4 : 0;
            dv[s] = o;   o += 2 * 2 * kC * 4;
            mv[s] = o;   o += v_min ? 2 * 2 * kC * 4 : 0;
            qsum[s] = o; o += 2 * 2 * kHP * 4;   // sum of Q over each group, times scale (log2 units)
            esc[s] = o;  o += 2 * kHP * 4;       // 2^-e_Q times scale (log2 units)
            wmax[s] = o; o += 4 * 4 * 4;         // [converter warp][g*2+blk] max |d_V|
        }
        for (int s = 0; s < 2; ++s) { red[s] = o; o += kRedFloats * 4; }  // [warp][max 16 | sum 16 | p*m_V 32]; combine scratch
        for (int s = 0; s < 2; ++s) { stat[s] = o; o += 96 * 4; }     // chunk max [16], 1/V scale [4], run (max, sum) [2][16][2]
        pref = o; o += dtc::round_up((kMaxSeq + 1) * 4, 16);
        bars = o; o += dtc::round_up(B_COUNT * 8 + 8, 16);  // mbarriers (8-byte aligned) + TMEM address slot
        misc = o; o += 16;                                  // ticket flags [2], error flag
        total = dtc::round_up(o, 128);
    }
};

// Slot offset without indexing a runtime array (which would go to local memory).
__device__ __forceinline__ int pick(const int (&v)[2], int s) { return s ? v[1] : v[0]; }

__device__ __forceinline__ void named_sync(int id, int n) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// AND of v over the n threads of named barrier id (all of them must call it):
// makes a wait result uniform across a role before any later named barrier.
__device__ __forceinline__ bool bar_and(int id, int n, bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r) : "r"((uint32_t)v), "r"(id), "r"(n) : "memory");
    return r != 0;
}

// Bounded wait that also gives up once another role has flagged an error.
__device__ __forceinline__ bool pwait(uint64_t* bar, uint32_t parity, volatile int* err, int* status, int site) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (;;) {
        if (mbar_try_wait_hint(bar, parity, 1000u)) return true;
        if (*err) return false;
        if (global_timer_ns() - t0 > kWaitBudgetNs) {
            record_status(status, kStatusTimeout | (site << 8));
            *err = 1;
            return false;
        }
    }
}

// Work item -> (sequence, chunk) through the prefix table of chunk counts.
__device__ __forceinline__ void item_of(const int* pref, int n_seq, int item, int& seq, int& chunk) {
    int lo = 0, hi = n_seq;  // largest s with pref[s] <= item
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (pref[mid] <= item) lo = mid; else hi = mid;
    }
    seq = lo;
    chunk = item - pref[lo];
}

// Warp-wide reduction of 16 values per lane ("transpose" butterfly: 16
// shuffles instead of 16 x 5).  Returns the reduction over all 32 lanes of
// value index xpose_index(lane); lanes l and l ^ 1 hold the same index.
__device__ __forceinline__ int xpose_index(int lane) {
    return ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
}
template <bool kMax>
__device__ __forceinline__ float op2(float a, float b) { return kMax ? fmaxf(a, b) : a + b; }
template <bool kMax>
__device__ __forceinline__ float xpose_reduce16(const float (&v)[16], int lane) {
    float a[8], b[4], c[2];
    const bool u16 = lane & 16, u8 = lane & 8, u4 = lane & 4, u2 = lane & 2;
#pragma unroll
    for (int i = 0; i < 8; ++i)
        a[i] = op2<kMax>(u16 ? v[8 + i] : v[i], __shfl_xor_sync(0xffffffffu, u16 ? v[i] : v[8 + i], 16));
#pragma unroll
    for (int i = 0; i < 4; ++i)
        b[i] = op2<kMax>(u8 ? a[4 + i] : a[i], __shfl_xor_sync(0xffffffffu, u8 ? a[i] : a[4 + i], 8));
#pragma unroll
    for (int i = 0; i < 2; ++i)
        c[i] = op2<kMax>(u4 ? b[2 + i] : b[i], __shfl_xor_sync(0xffffffffu, u4 ? b[i] : b[2 + i], 4));
    float d = op2<kMax>(u2 ? c[1] : c[0], __shfl_xor_sync(0xffffffffu, u2 ? c[0] : c[1], 2));
    return op2<kMax>(d, __shfl_xor_sync(0xffffffffu, d, 1));
}

// Log-sum-exp merge of one sequence's chunk partials by the nt threads of a
// group, straight from the (L2-resident) workspace: every thread derives the
// per-head max and weights for the outputs it owns, so no shared scratch is
// needed and the chunk count is unbounded.
__device__ __forceinline__ void combine_direct(const Args& a, int seq, int nchunks, float* out, int tid, int nt) {
    const int Hq = a.Hq;
    const bool emit_partial = (a.flags & CVATTN_DECODE_EMIT_PARTIAL) != 0;
    const float* seq_ml = a.ws_ml + ((int64_t)seq * a.ws_chunks) * Hq * 2;
    const float* seq_o = a.ws_o + ((int64_t)seq * a.ws_chunks) * Hq * kD;
    for (int it = tid; it < Hq * (kD / 4); it += nt) {
        const int h = it / (kD / 4), dd = (it % (kD / 4)) * 4;
        // pass 1: running max and rescaled sum together (one sweep of independent loads)
        float M = -INFINITY, Ls = 0.0f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int c0 = 0; c0 < nchunks; c0 += 8) {
            float2 ml[8];
            float4 v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int c = min(c0 + j, nchunks - 1);
                ml[j] = __ldcg(reinterpret_cast<const float2*>(seq_ml + ((int64_t)c * Hq + h) * 2));
                v[j] = __ldcg(reinterpret_cast<const float4*>(seq_o + ((int64_t)c * Hq + h) * kD + dd));
            }
            float bm = M;
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (c0 + j < nchunks) bm = fmaxf(bm, ml[j].x);
            const float r = (M == -INFINITY) ? 0.0f : fast_exp2(M - bm);
            Ls *= r;
            acc.x *= r; acc.y *= r; acc.z *= r; acc.w *= r;
            M = bm;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (c0 + j >= nchunks) break;
                if (ml[j].x == -INFINITY) continue;  // empty slot (merged into another chunk's partial)
                const float w = fast_exp2(ml[j].x - M);
                Ls = fmaf(w, ml[j].y, Ls);
                acc.x = fmaf(w, v[j].x, acc.x); acc.y = fmaf(w, v[j].y, acc.y);
                acc.z = fmaf(w, v[j].z, acc.z); acc.w = fmaf(w, v[j].w, acc.w);
            }
        }
        const float inv = emit_partial ? 1.0f : 1.0f / Ls;
        *reinterpret_cast<float4*>(out + h * kD + dd) = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
        if (emit_partial && dd == 0) {
            a.partial_ml[((int64_t)seq * Hq + h) * 2] = M;
            a.partial_ml[((int64_t)seq * Hq + h) * 2 + 1] = Ls;
        }
    }
}

// Raw rows of one chunk -> swizzled f16 tiles [g][128 keys x 64 dims] + scales
// [g*2+blk][key] (+ mins); thread = key.  For V, also the per-warp max |d|.
template <int T, bool kIsV>
__device__ __forceinline__ void convert_rows(const uint8_t* raw, int row, int head, int n, int key, int cw, int lane,
                                             uint8_t* tiles, float* dsc, float* msc, float* wmax) {
    constexpr int GB = group_bytes(T);
#pragma unroll
    for (int it = 0; it < 4; ++it) {
        const int g = it >> 1, blk = it & 1;
        uint32_t w[16];
        float d = 0.0f, m = 0.0f;
        if (key < n) {
            convert_group<T>(raw + key * row + g * head + blk * GB, w, d, m);
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) w[i] = 0u;
        }
        uint8_t* tile = tiles + g * 16384;
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4)
            *reinterpret_cast<uint4*>(tile + tc::sw128_offset(key, blk * 4 + c4)) =
                make_uint4(w[4 * c4], w[4 * c4 + 1], w[4 * c4 + 2], w[4 * c4 + 3]);
        dsc[(g * 2 + blk) * kC + key] = d;
        if constexpr (BlockTraits<T>::HAS_MIN) msc[(g * 2 + blk) * kC + key] = m;
        if constexpr (kIsV) {
            const float dm = dec::warp_max(fabsf(d));
            if (lane == 0) wmax[cw * 4 + g * 2 + blk] = dm;
        }
    }
}

// q8_0 variant without shared-memory bank conflicts: a half-warp takes one
// 32-element block of 16 consecutive keys, the other half-warp the other
// block of the same head.  The two blocks start 9 words apart (34-byte
// blocks), so the 32 lanes of every load hit 32 different banks; a funnel
// shift realigns the 2-byte aligned quants.
template <bool kIsV>
__device__ __forceinline__ void convert_q8_half_warps(const uint8_t* raw, int row, int head, int n, int cw, int lane,
                                                      uint8_t* tiles, float* dsc, float* wmax) {
    const int blk = lane >> 4;
    float dmax[2] = {0.0f, 0.0f};
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int key = r * 64 + cw * 16 + (lane & 15);
#pragma unroll
        for (int g = 0; g < 2; ++g) {
            uint32_t w[16];
            float d = 0.0f;
            if (key < n) {
                const uint8_t* grp = raw + key * row + g * head + blk * 34;
                d = h2f(*reinterpret_cast<const uint16_t*>(grp));
                const uintptr_t qa = reinterpret_cast<uintptr_t>(grp + 2);
                const uint32_t* wp = reinterpret_cast<const uint32_t*>(qa & ~uintptr_t(3));
                const uint32_t sh = (uint32_t)(qa & 3) * 8u;  // 0 or 16
                uint32_t x[9];
#pragma unroll
                for (int j = 0; j < 9; ++j) x[j] = wp[j];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint32_t y = __funnelshift_r(x[j], x[j + 1], sh) ^ 0x80808080u;
                    w[2 * j] = dtc::hsub2_u32(__byte_perm(y, 0x6464u, 0x5140u), dtc::kF16x2_1152);
                    w[2 * j + 1] = dtc::hsub2_u32(__byte_perm(y, 0x6464u, 0x5342u), dtc::kF16x2_1152);
                }
            } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) w[i] = 0u;
            }
            uint8_t* tile = tiles + g * 16384;
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4)
                *reinterpret_cast<uint4*>(tile + tc::sw128_offset(key, blk * 4 + c4)) =
                    make_uint4(w[4 * c4], w[4 * c4 + 1], w[4 * c4 + 2], w[4 * c4 + 3]);
            dsc[(g * 2 + blk) * kC + key] = d;
            dmax[g] = fmaxf(dmax[g], fabsf(d));
        }
    }
    if constexpr (kIsV) {
#pragma unroll
        for (int g = 0; g < 2; ++g) {
            float v = dmax[g];
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
            if ((lane & 15) == 0) wmax[cw * 4 + g * 2 + blk] = v;
        }
    }
}

// 16-byte L2 load issued as its own instruction (so a batch stays in flight together).
__device__ __forceinline__ float4 ldcg_f4(const float* p) {
    float4 v;
    asm volatile("ld.global.cg.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
    return v;
}

// Merge of one sequence's partials by the nt threads of a group.  A chunk
// slot whose max is -inf is empty (its chunk was merged into the partial of
// an earlier slot), so only the written partials are read: each warp
// derives, for its heads, the max / sum over all slots with the lanes
// walking the slots, and the weights of the non-empty ones; then thread =
// (head, 4 dims) x 2 streams those partials.  scr: kRedFloats floats.
__device__ __forceinline__ void combine_sparse(const Args& a, int seq, int nchunks, float* out, int tid, int nt,
                                               int bar_id, float* scr) {
    const int Hq = a.Hq;
    if (nchunks > 64 || nchunks * (Hq + 1) + 1 > kRedFloats) {
        combine_direct(a, seq, nchunks, out, tid, nt);
        return;
    }
    const bool emit_partial = (a.flags & CVATTN_DECODE_EMIT_PARTIAL) != 0;
    const float* seq_ml = a.ws_ml + ((int64_t)seq * a.ws_chunks) * Hq * 2;
    const float* seq_o = a.ws_o + ((int64_t)seq * a.ws_chunks) * Hq * kD;
    int* idx = reinterpret_cast<int*>(scr);             // [P] chunk slot of the p-th partial
    int* pcount = reinterpret_cast<int*>(scr + nchunks);
    float* wt = scr + nchunks + 1;                       // [P][Hq] weight (1/sum folded in)
    const int lane = tid & 31, nw = nt >> 5;
    const uint32_t below = (1u << lane) - 1u;
    for (int h = tid >> 5; h < Hq; h += nw) {
        const int c0 = lane, c1 = lane + 32;
        const float2 e2 = make_float2(-INFINITY, 0.0f);
        const float2 ml0 = c0 < nchunks ? __ldcg(reinterpret_cast<const float2*>(seq_ml + ((int64_t)c0 * Hq + h) * 2)) : e2;
        const float2 ml1 = c1 < nchunks ? __ldcg(reinterpret_cast<const float2*>(seq_ml + ((int64_t)c1 * Hq + h) * 2)) : e2;
        const float M = dec::warp_max(fmaxf(ml0.x, ml1.x));
        const bool v0 = ml0.x != -INFINITY, v1 = ml1.x != -INFINITY;
        const float w0 = v0 ? fast_exp2(ml0.x - M) : 0.0f, w1 = v1 ? fast_exp2(ml1.x - M) : 0.0f;
        const float Ls = dec::warp_sum(w0 * ml0.y + w1 * ml1.y);
        const float inv = emit_partial ? 1.0f : 1.0f / Ls;
        const uint32_t b0 = __ballot_sync(0xffffffffu, v0), b1 = __ballot_sync(0xffffffffu, v1);
        const int r0 = __popc(b0 & below), r1 = __popc(b0) + __popc(b1 & below);
        if (v0) wt[r0 * Hq + h] = w0 * inv;
        if (v1) wt[r1 * Hq + h] = w1 * inv;
        if (h == 0) {  // the set of written slots is the same for every head
            if (v0) idx[r0] = c0;
            if (v1) idx[r1] = c1;
            if (lane == 0) *pcount = __popc(b0) + __popc(b1);
        }
        if (emit_partial && lane == 0) {
            a.partial_ml[((int64_t)seq * Hq + h) * 2] = M;
            a.partial_ml[((int64_t)seq * Hq + h) * 2 + 1] = Ls;
        }
    }
    named_sync(bar_id, nt);
    const int P = *pcount;
    const int n_out = Hq * (kD / 4);
    for (int it0 = tid; it0 < n_out; it0 += 2 * nt) {
        const int it1 = it0 + nt;
        const bool has1 = it1 < n_out;
        const int h0 = it0 / (kD / 4), dd0 = (it0 % (kD / 4)) * 4;
        const int h1 = has1 ? it1 / (kD / 4) : h0, dd1 = has1 ? (it1 % (kD / 4)) * 4 : dd0;
        float4 acc0 = make_float4(0.f, 0.f, 0.f, 0.f), acc1 = acc0;
        for (int p0 = 0; p0 < P; p0 += 8) {
            float4 u0[8], u1[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int c = idx[min(p0 + j, P - 1)];
                u0[j] = ldcg_f4(seq_o + ((int64_t)c * Hq + h0) * kD + dd0);
                u1[j] = ldcg_f4(seq_o + ((int64_t)c * Hq + h1) * kD + dd1);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (p0 + j >= P) break;
                const float w0 = wt[(p0 + j) * Hq + h0], w1 = wt[(p0 + j) * Hq + h1];
                acc0.x = fmaf(w0, u0[j].x, acc0.x); acc0.y = fmaf(w0, u0[j].y, acc0.y);
                acc0.z = fmaf(w0, u0[j].z, acc0.z); acc0.w = fmaf(w0, u0[j].w, acc0.w);
                acc1.x = fmaf(w1, u1[j].x, acc1.x); acc1.y = fmaf(w1, u1[j].y, acc1.y);
                acc1.z = fmaf(w1, u1[j].z, acc1.z); acc1.w = fmaf(w1, u1[j].w, acc1.w);
            }
        }
        *reinterpret_cast<float4*>(out + h0 * kD + dd0) = acc0;
        if (has1) *reinterpret_cast<float4*>(out + h1 * kD + dd1) = acc1;
    }
}

template <int KT, int VT>
__global__ void __launch_bounds__(kThreads, 1) decode_pipe_kernel(const Args a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = a.G, Hq = a.Hq, n_seq = a.n_seq;
    constexpr int GBK = group_bytes(KT), GBV = group_bytes(VT);
    constexpr int headK = 2 * GBK, headV = 2 * GBV, rowK = 2 * headK, rowV = 2 * headV;
    constexpr bool K_MIN = BlockTraits<KT>::HAS_MIN, V_MIN = BlockTraits<VT>::HAS_MIN;
    const Smem L(rowK, rowV, K_MIN, V_MIN);
    const bool emit_partial = (a.flags & CVATTN_DECODE_EMIT_PARTIAL) != 0;
    if (smem_addr(smem) & 1023u) {
        if (tid == 0) record_status(a.status, kStatusTimeout | (9 << 8));
        return;
    }
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.bars + B_COUNT * 8);
    volatile int* flags = reinterpret_cast<volatile int*>(smem + L.misc);
    volatile int* err = reinterpret_cast<volatile int*>(smem + L.misc + 8);
    int* pref = reinterpret_cast<int*>(smem + L.pref);
    griddep_launch_dependents();  // the next layer's launch may start its prologue on SMs this grid frees

    // ---- setup: barriers, TMEM, per-sequence chunk prefix sums
    if (tid == 0) {
        for (int i = 0; i < B_COUNT; ++i) {
            const bool by_threads = (i >= B_RAW_EMPTY && i < B_RAW_EMPTY + 2) || (i >= B_TILE_FULL && i < B_TILE_FULL + 2) ||
                                    (i >= B_P_FULL && i < B_P_FULL + 2);
            mbar_init(&bars[i], by_threads ? (uint32_t)kGroup : 1u);
        }
        *err = 0;
        fence_mbar_init();
    }
    if (warp == kMmaWarp) {
        tc::tmem_alloc(tmem_slot, kTmemCols);
        tc::tmem_relinquish();
    }
    // Inputs (Q, new rows, lengths, cache) and the workspace belong to the previous
    // kernel until griddepcontrol.wait.  With CVATTN_DECODE_INPUTS_READY the lengths
    // and cached rows are already final: the chunk scan and the producer's K/V
    // streaming run before the wait; everything that reads Q / new rows or writes
    // anything waits.
    const bool early = (a.flags & CVATTN_DECODE_INPUTS_READY) != 0;
    if (!early) griddep_wait();
    if (warp == 0) {  // exclusive scan of chunk counts; invalid or empty sequences get none
        int carry = 0;
        for (int base = 0; base < n_seq; base += 32) {
            const int s = base + lane;
            int nc = 0;
            if (s < n_seq) {
                const int len = a.kv_len[s];
                if (len > 0 && len <= a.capacity && len <= a.max_kv_len) nc = (len + kC - 1) / kC;
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
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tmem = *tmem_slot;
    const int n_items = pref[n_seq];
    // contiguous item range per CTA; local item t alternates between its two halves
    // (t even: first half, t odd: second half), so each softmax group walks
    // consecutive chunks and merges them before anything leaves the SM
    const int lo = (int)(((long long)blockIdx.x * n_items) / gridDim.x);
    const int n_local = (int)(((long long)(blockIdx.x + 1) * n_items) / gridDim.x) - lo;
    const int n_half0 = (n_local + 1) >> 1;
    auto item_at = [&](int t) { return (t & 1) ? lo + n_half0 + (t >> 1) : lo + (t >> 1); };

    if (warp == kProdWarp) {
        // ===================================================== producer
        if (lane == 0) {
            for (int t = 0; t < n_local; ++t) {
                const int s = t & 1;
                if (t >= 2 && !pwait(&bars[B_RAW_EMPTY + s], ((t >> 1) - 1) & 1, err, a.status, 1)) break;
                int seq, chunk;
                item_of(pref, n_seq, item_at(t), seq, chunk);
                const int len = a.kv_len[seq];
                const int p0 = chunk * kC, n = min(kC, len - p0);
                const uint8_t* kb = a.k_seq_ptrs ? reinterpret_cast<const uint8_t*>(a.k_seq_ptrs[seq]) : a.k_base + seq * a.k_nb2;
                const uint8_t* vb = a.v_seq_ptrs ? reinterpret_cast<const uint8_t*>(a.v_seq_ptrs[seq]) : a.v_base + seq * a.v_nb2;
                const uint8_t* ksrc = kb + (int64_t)p0 * rowK;
                const uint8_t* vsrc = vb + (int64_t)p0 * rowV;
                uint8_t* kdst = smem + pick(L.raw, s);
                uint8_t* vdst = kdst + kC * rowK;
                const uint32_t kbytes = (uint32_t)(n * rowK), vbytes = (uint32_t)(n * rowV);
                const uint32_t kbulk = ((reinterpret_cast<uintptr_t>(ksrc) & 15) == 0) ? (kbytes & ~15u) : 0u;
                const uint32_t vbulk = ((reinterpret_cast<uintptr_t>(vsrc) & 15) == 0) ? (vbytes & ~15u) : 0u;
                // tails first: the arrive below releases these generic stores
                for (uint32_t i = kbulk / 2; i < kbytes / 2; ++i)
                    reinterpret_cast<uint16_t*>(kdst)[i] = reinterpret_cast<const uint16_t*>(ksrc)[i];
                for (uint32_t i = vbulk / 2; i < vbytes / 2; ++i)
                    reinterpret_cast<uint16_t*>(vdst)[i] = reinterpret_cast<const uint16_t*>(vsrc)[i];
                mbar_arrive_expect_tx(&bars[B_RAW_FULL + s], kbulk + vbulk);
                if (kbulk) bulk_g2s(kdst, ksrc, kbulk, &bars[B_RAW_FULL + s]);
                if (vbulk) bulk_g2s(vdst, vsrc, vbulk, &bars[B_RAW_FULL + s]);
            }
        }
    } else if (warp == kMmaWarp) {
        // ===================================================== MMA issuer
        if (lane == 0) {
            const uint32_t idesc_s = tc::idesc_f16_f32(128, 16, false);
            const uint32_t idesc_o = tc::idesc_f16_f32(128, 64, true, true);
            int ns = 0, no = 0;  // next item whose S / O is to be issued
            uint64_t t_idle = 0;
            uint32_t spins = 0;
            while (no < n_local) {
                bool progressed = false;
                // S(ns) reuses the TMEM stage of S(ns - 2): its softmax is over once O(ns - 2) is issued
                if (ns < n_local && ns <= no + 1 && mbar_test(&bars[B_TILE_FULL + (ns & 1)], (ns >> 1) & 1)) {
                    tc::fence_after();
                    const int s = ns & 1;
                    const uint32_t kaddr = smem_addr(smem + pick(L.ktile, s)), qaddr = smem_addr(smem + pick(L.qtile, s));
#pragma unroll
                    for (int g = 0; g < 2; ++g)
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk) {
                            const uint64_t ad = tc::sdesc_sw128(kaddr + g * 16384 + kk * 32, 16, 1024);
                            const uint64_t bd = tc::sdesc_sw128(qaddr + g * 2048 + kk * 32, 16, 1024);
                            tc::mma_ss(tmem + s * 64 + (g * 2 + (kk >> 1)) * 16, ad, bd, idesc_s, (kk & 1) ? 1u : 0u);
                        }
                    tc::mma_commit(&bars[B_S_FULL + s]);
                    ++ns;
                    progressed = true;
                }
                if (no < ns && mbar_test(&bars[B_P_FULL + (no & 1)], (no >> 1) & 1)) {
                    tc::fence_after();
                    const int s = no & 1;
                    const uint32_t vaddr = smem_addr(smem + pick(L.vtile, s)), paddr = smem_addr(smem + pick(L.ktile, s));
#pragma unroll
                    for (int kk = 0; kk < kC / 16; ++kk) {
                        const uint64_t ad = tc::sdesc_sw128(vaddr + kk * 2048, 16384, 1024);
                        const uint64_t bd = tc::sdesc_sw128(paddr + kk * 2048, 16, 1024);
                        tc::mma_ss(tmem + 128 + s * 64, ad, bd, idesc_o, kk > 0 ? 1u : 0u);
                    }
                    tc::mma_commit(&bars[B_O_FULL + s]);
                    ++no;
                    progressed = true;
                }
                if (progressed) {
                    t_idle = 0;
                    spins = 0;
                    continue;
                }
                // nothing ready: sleep briefly on one of the two pending barriers (alternating), so the
                // issuer neither burns issue slots of its sub-partition nor reacts late to either stage
                if ((spins & 1u) == 0 && ns < n_local && ns <= no + 1)
                    mbar_try_wait_hint(&bars[B_TILE_FULL + (ns & 1)], (ns >> 1) & 1, 100u);
                else if (no < ns)
                    mbar_try_wait_hint(&bars[B_P_FULL + (no & 1)], (no >> 1) & 1, 100u);
                if ((++spins & 63u) == 0) {  // the clock and the error flag are slow to read: poll them rarely
                    if (*err) break;
                    const uint64_t now = global_timer_ns();
                    if (t_idle == 0) {
                        t_idle = now;
                    } else if (now - t_idle > kWaitBudgetNs) {
                        record_status(a.status, kStatusTimeout | (4 << 8));
                        *err = 1;
                        break;
                    }
                }
            }
        }
    } else if (warp < kSoftWarp0) {
        // ===================================================== converters (group s: items of slot s)
        if (early) griddep_wait();
        const int s = warp >> 2;
        const int bar_id = kBarConv + s;
        const int key = tid & (kGroup - 1);  // key row of the chunk
        const int cw = warp & 3;
        uint8_t* Kraw = smem + pick(L.raw, s);
        uint8_t* Vraw = Kraw + kC * rowK;
        float* dk = reinterpret_cast<float*>(smem + pick(L.dk, s));
        float* mk = reinterpret_cast<float*>(smem + pick(L.mk, s));
        float* dv = reinterpret_cast<float*>(smem + pick(L.dv, s));
        float* mv = reinterpret_cast<float*>(smem + pick(L.mv, s));
        float* wmax = reinterpret_cast<float*>(smem + pick(L.wmax, s));
        float* esc = reinterpret_cast<float*>(smem + pick(L.esc, s));
        float* qsum = reinterpret_cast<float*>(smem + pick(L.qsum, s));
        for (int t = s; t < n_local; t += 2) {
            int seq, chunk;
            item_of(pref, n_seq, item_at(t), seq, chunk);
            const int len = a.kv_len[seq];
            const int p0 = chunk * kC, n = min(kC, len - p0);
            const int nchunks = (len + kC - 1) / kC;
            {   // tiles of slot s are free once O(t - 2) has completed; raw data of item t has landed
                bool ok = t < 2 || pwait(&bars[B_O_FULL + s], ((t >> 1) - 1) & 1, err, a.status, 5);
                ok = ok && pwait(&bars[B_RAW_FULL + s], (t >> 1) & 1, err, a.status, 6);
                if (!bar_and(bar_id, kGroup, ok)) break;
            }
            if (a.k_new && chunk == nchunks - 1) {
                const uint8_t* kb = a.k_seq_ptrs ? reinterpret_cast<const uint8_t*>(a.k_seq_ptrs[seq]) : a.k_base + seq * a.k_nb2;
                const uint8_t* vb = a.v_seq_ptrs ? reinterpret_cast<const uint8_t*>(a.v_seq_ptrs[seq]) : a.v_base + seq * a.v_nb2;
                const int r = len - 1 - p0;
                for (int gi = cw; gi < 8; gi += 4) {
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
                named_sync(bar_id, kGroup);
            }
            // this thread's two 8-float pieces of Q, loaded now so the latency hides under the conversion
            float4 qv[2][2];
#pragma unroll
            for (int qi = 0; qi < 2; ++qi) {
                const int item = key + qi * 128;
                const int g = item >> 7, row = (item >> 3) & 15, c = item & 7;
                const int h = row & 7;
                if (h < G) {
                    const float* qr = a.q + (int64_t)seq * a.q_seq_stride + (g * G + h) * kD + 8 * c;
                    qv[qi][0] = *reinterpret_cast<const float4*>(qr);
                    qv[qi][1] = *reinterpret_cast<const float4*>(qr + 4);
                } else {
                    qv[qi][0] = qv[qi][1] = make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
            if constexpr (KT == kQ8_0) convert_q8_half_warps<false>(Kraw, rowK, headK, n, cw, lane, smem + pick(L.ktile, s), dk, nullptr);
            else convert_rows<KT, false>(Kraw, rowK, headK, n, key, cw, lane, smem + pick(L.ktile, s), dk, mk, nullptr);
            if constexpr (VT == kQ8_0) convert_q8_half_warps<true>(Vraw, rowV, headV, n, cw, lane, smem + pick(L.vtile, s), dv, wmax);
            else convert_rows<VT, true>(Vraw, rowV, headV, n, key, cw, lane, smem + pick(L.vtile, s), dv, mv, wmax);
            mbar_arrive(&bars[B_RAW_EMPTY + s]);  // raw slot s may be refilled
            // Q hi/lo tile of this item's sequence
#pragma unroll
            for (int qi = 0; qi < 2; ++qi) {
                const int item = key + qi * 128;
                const int g = item >> 7, row = (item >> 3) & 15, c = item & 7;
                const int h = row & 7;
                const bool lo_row = row >= 8;
                const float4 u = qv[qi][0], v = qv[qi][1];
                const float x[8] = {u.x, u.y, u.z, u.w, v.x, v.y, v.z, v.w};
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
                    if (!lo_row) wv[e / 2] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
                    else wv[e / 2] = tc::pack_f16x2(y0 - __half2float(h0), y1 - __half2float(h1));
                }
                *reinterpret_cast<uint4*>(smem + pick(L.qtile, s) + g * 2048 + tc::sw128_offset(row, c)) =
                    make_uint4(wv[0], wv[1], wv[2], wv[3]);
                if (!lo_row && c == 0) esc[g * kHP + h] = pow2f(-ex) * a.scale_log2;
                if constexpr (K_MIN) {
                    part += __shfl_xor_sync(0xffffffffu, part, 1);
                    part += __shfl_xor_sync(0xffffffffu, part, 2);
                    if (!lo_row && (c & 3) == 0) qsum[(g * 2 + (c >> 2)) * kHP + h] = part * a.scale_log2;
                }
            }
            fence_proxy_async_smem();
            mbar_arrive(&bars[B_TILE_FULL + s]);
        }
    } else {
        // ===================================================== softmax + epilogue (group s: items of slot s)
        if (early) griddep_wait();
        const int s = (warp - kSoftWarp0) >> 2;
        const int bar_id = kBarSoft + s;
        const int stid = tid & (kGroup - 1);     // 0..127 = TMEM lane
        const int sw = warp & 3;                 // TMEM lane quarter of this warp
        const uint32_t lane_base = (uint32_t)(sw * 32) << 16;
        float* red = reinterpret_cast<float*>(smem + pick(L.red, s));
        float* stat = reinterpret_cast<float*>(smem + pick(L.stat, s));
        const float* dk = reinterpret_cast<const float*>(smem + pick(L.dk, s));
        const float* mk = reinterpret_cast<const float*>(smem + pick(L.mk, s));
        const float* dv = reinterpret_cast<const float*>(smem + pick(L.dv, s));
        const float* mv = reinterpret_cast<const float*>(smem + pick(L.mv, s));
        const float* esc = reinterpret_cast<const float*>(smem + pick(L.esc, s));
        const float* qsum = reinterpret_cast<const float*>(smem + pick(L.qsum, s));
        const float* wmax = reinterpret_cast<const float*>(smem + pick(L.wmax, s));
        uint8_t* ptile = smem + pick(L.ktile, s);  // the K tiles are dead once S is complete
        const int xi = xpose_index(lane);
        // running partial of the sequence this group is walking: O in TMEM (lane = (kv head, dim),
        // 8 columns = heads), its per-head (max, sum) in shared memory, double-buffered by run position
        int run_n = 0, run_c0 = 0;
        const uint32_t run_taddr = tmem + lane_base + kRunCol + s * 8;
        float* runml = stat + 32;

        for (int t = s; t < n_local; t += 2) {
            int seq, chunk;
            item_of(pref, n_seq, item_at(t), seq, chunk);
            const int len = a.kv_len[seq];
            const int n = min(kC, len - chunk * kC);
            const int nchunks = (len + kC - 1) / kC;
            // ------------------------------------------------ softmax
            if (!bar_and(bar_id, kGroup, pwait(&bars[B_S_FULL + s], (t >> 1) & 1, err, a.status, 8))) break;
            tc::fence_after();
            const int key = stid;
            float p[16];  // index g * 8 + h
#pragma unroll
            for (int g = 0; g < 2; ++g) {
                uint32_t sv[32];
                tc::tmem_ld32(tmem + lane_base + s * 64 + g * 32, sv);
                tc::tmem_ld_wait();
                const float d0 = dk[(g * 2) * kC + key], d1 = dk[(g * 2 + 1) * kC + key];
                float m0 = 0.0f, m1 = 0.0f;
                if constexpr (K_MIN) { m0 = mk[(g * 2) * kC + key]; m1 = mk[(g * 2 + 1) * kC + key]; }
#pragma unroll
                for (int h = 0; h < kHP; ++h) {
                    float tt = d0 * (__uint_as_float(sv[h]) + __uint_as_float(sv[8 + h])) +
                               d1 * (__uint_as_float(sv[16 + h]) + __uint_as_float(sv[24 + h]));
                    tt *= esc[g * kHP + h];
                    if constexpr (K_MIN) tt += m0 * qsum[(g * 2) * kHP + h] + m1 * qsum[(g * 2 + 1) * kHP + h];
                    p[g * 8 + h] = (key < n && h < G) ? tt : -INFINITY;  // scores in log2 units for now
                }
            }
            tc::fence_before();
            {
                const float wm = xpose_reduce16<true>(p, lane);
                if (!(lane & 1)) red[sw * 64 + xi] = wm;
            }
            named_sync(bar_id, kGroup);
            float M[16];
#pragma unroll
            for (int i = 0; i < 16; i += 4) {
                float4 r = *reinterpret_cast<const float4*>(red + i);
#pragma unroll
                for (int w2 = 1; w2 < 4; ++w2) {
                    const float4 q = *reinterpret_cast<const float4*>(red + w2 * 64 + i);
                    r.x = fmaxf(r.x, q.x); r.y = fmaxf(r.y, q.y); r.z = fmaxf(r.z, q.z); r.w = fmaxf(r.w, q.w);
                }
                M[i] = r.x; M[i + 1] = r.y; M[i + 2] = r.z; M[i + 3] = r.w;
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) p[i] = (p[i] == -INFINITY) ? 0.0f : fast_exp2(p[i] - M[i]);
            {
                const float ws = xpose_reduce16<false>(p, lane);
                if (!(lane & 1)) red[sw * 64 + 16 + xi] = ws;
            }
            if constexpr (V_MIN) {
#pragma unroll
                for (int b2 = 0; b2 < 2; ++b2) {
                    float pm[16];
#pragma unroll
                    for (int g = 0; g < 2; ++g) {
                        const float mvk = mv[(g * 2 + b2) * kC + key];
#pragma unroll
                        for (int h = 0; h < kHP; ++h) pm[g * 8 + h] = p[g * 8 + h] * mvk;
                    }
                    const float r = xpose_reduce16<false>(pm, lane);
                    if (!(lane & 1)) red[sw * 64 + 32 + b2 * 16 + xi] = r;  // index b2 * 16 + g * 8 + h
                }
            }
            // P' row of this key: chunk (g*4 + blk*2 + {hi, lo}) holds 8 heads
            float ivs[4];
#pragma unroll
            for (int g = 0; g < 2; ++g)
#pragma unroll
                for (int b2 = 0; b2 < 2; ++b2) {
                    float vmx = wmax[g * 2 + b2];
#pragma unroll
                    for (int w2 = 1; w2 < 4; ++w2) vmx = fmaxf(vmx, wmax[w2 * 4 + g * 2 + b2]);
                    const int ev = norm_exp(vmx);
                    ivs[g * 2 + b2] = pow2f(-ev);
                    const float dvk = dv[(g * 2 + b2) * kC + key] * pow2f(ev);
                    uint32_t hi[4], lo[4];
#pragma unroll
                    for (int h = 0; h < kHP; h += 2) {
                        const float x0 = p[g * 8 + h] * dvk, x1 = p[g * 8 + h + 1] * dvk;
                        const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
                        hi[h / 2] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
                        lo[h / 2] = tc::pack_f16x2(x0 - __half2float(h0), x1 - __half2float(h1));
                    }
                    *reinterpret_cast<uint4*>(ptile + tc::sw128_offset(key, g * 4 + b2 * 2)) =
                        make_uint4(hi[0], hi[1], hi[2], hi[3]);
                    *reinterpret_cast<uint4*>(ptile + tc::sw128_offset(key, g * 4 + b2 * 2 + 1)) =
                        make_uint4(lo[0], lo[1], lo[2], lo[3]);
                }
            if (stid == 0) {
#pragma unroll
                for (int i = 0; i < 16; i += 4)
                    *reinterpret_cast<float4*>(stat + i) = make_float4(M[i], M[i + 1], M[i + 2], M[i + 3]);
                *reinterpret_cast<float4*>(stat + 16) = make_float4(ivs[0], ivs[1], ivs[2], ivs[3]);
            }
            fence_proxy_async_smem();
            mbar_arrive(&bars[B_P_FULL + s]);

            // ------------------------------------------------ epilogue
            // (the barrier inside bar_and also publishes red / stat to the whole group)
            if (!bar_and(bar_id, kGroup, pwait(&bars[B_O_FULL + s], (t >> 1) & 1, err, a.status, 9))) break;
            tc::fence_after();
            float* out = a.out + (int64_t)seq * a.out_seq_stride;
            const int g = stid >> 6, dim = stid & 63, blk = dim >> 5;
            uint32_t ov[16];
            tc::tmem_ld16(tmem + lane_base + 128 + s * 64 + g * 32 + blk * 16, ov);
            tc::tmem_ld_wait();
            tc::fence_before();
            const float inv_vs = stat[16 + g * 2 + blk];
            float lsum[kHP], pmv[kHP];
#pragma unroll
            for (int h = 0; h < kHP; h += 4) {
                float4 r = *reinterpret_cast<const float4*>(red + 16 + g * 8 + h);
                float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
                if constexpr (V_MIN) q = *reinterpret_cast<const float4*>(red + 32 + blk * 16 + g * 8 + h);
#pragma unroll
                for (int w2 = 1; w2 < 4; ++w2) {
                    const float4 u = *reinterpret_cast<const float4*>(red + w2 * 64 + 16 + g * 8 + h);
                    r.x += u.x; r.y += u.y; r.z += u.z; r.w += u.w;
                    if constexpr (V_MIN) {
                        const float4 v = *reinterpret_cast<const float4*>(red + w2 * 64 + 32 + blk * 16 + g * 8 + h);
                        q.x += v.x; q.y += v.y; q.z += v.z; q.w += v.w;
                    }
                }
                lsum[h] = r.x; lsum[h + 1] = r.y; lsum[h + 2] = r.z; lsum[h + 3] = r.w;
                pmv[h] = q.x; pmv[h + 1] = q.y; pmv[h + 2] = q.z; pmv[h + 3] = q.w;
            }
            // merge this chunk into the group's running partial of the sequence
            const float* ml_old = runml + (run_n & 1) * 32;
            float* ml_new = runml + ((run_n + 1) & 1) * 32;
            float run_m[kHP], run_l[kHP], run_o[kHP];
            {
                uint32_t ro[8];
                if (run_n > 0) {
                    tc::tmem_ld8(run_taddr, ro);
                    tc::tmem_ld_wait();
                }
#pragma unroll
                for (int h = 0; h < kHP; ++h) run_o[h] = run_n > 0 ? __uint_as_float(ro[h]) : 0.0f;
            }
#pragma unroll
            for (int h = 0; h < kHP; ++h) {
                if (h >= G) break;
                float o = (__uint_as_float(ov[h]) + __uint_as_float(ov[8 + h])) * inv_vs;
                if constexpr (V_MIN) o += pmv[h];
                const float m = stat[g * 8 + h], l = lsum[h];
                if (run_n == 0) {
                    run_o[h] = o; run_m[h] = m; run_l[h] = l;
                } else {
                    const float2 pm = *reinterpret_cast<const float2*>(ml_old + (g * 8 + h) * 2);
                    const float mx = fmaxf(pm.x, m);
                    const float ra = fast_exp2(pm.x - mx), rb = fast_exp2(m - mx);
                    run_o[h] = run_o[h] * ra + o * rb;
                    run_l[h] = pm.y * ra + l * rb;
                    run_m[h] = mx;
                }
                if (dim == 0) *reinterpret_cast<float2*>(ml_new + (g * 8 + h) * 2) = make_float2(run_m[h], run_l[h]);
            }
            {
                uint32_t ro[8];
#pragma unroll
                for (int h = 0; h < kHP; ++h) ro[h] = __float_as_uint(run_o[h]);
                tc::tmem_st8(run_taddr, ro);
                tc::tmem_st_wait();
            }
            if (run_n == 0) run_c0 = chunk;
            ++run_n;
            bool flush = t + 2 >= n_local;
            if (!flush) {
                int seq2, chunk2;
                item_of(pref, n_seq, item_at(t + 2), seq2, chunk2);
                flush = seq2 != seq;
            }
            if (flush) {
                if (run_n == nchunks) {  // the whole sequence went through this group
#pragma unroll
                    for (int h = 0; h < kHP; ++h) {
                        if (h >= G) break;
                        const int qh = g * G + h;
                        out[qh * kD + dim] = emit_partial ? run_o[h] : run_o[h] / run_l[h];
                        if (emit_partial && dim == 0) {
                            a.partial_ml[((int64_t)seq * Hq + qh) * 2] = run_m[h];
                            a.partial_ml[((int64_t)seq * Hq + qh) * 2 + 1] = run_l[h];
                        }
                    }
                } else {
                    // partial into the slot of the run's first chunk; the run's other chunk slots are marked empty
                    float* wso = a.ws_o + (((int64_t)seq * a.ws_chunks + run_c0) * Hq) * kD;
                    float* wsml = a.ws_ml + (((int64_t)seq * a.ws_chunks + run_c0) * Hq) * 2;
#pragma unroll
                    for (int h = 0; h < kHP; ++h) {
                        if (h >= G) break;
                        const int qh = g * G + h;
                        wso[qh * kD + dim] = run_o[h];
                        if (dim == 0) *reinterpret_cast<float2*>(wsml + qh * 2) = make_float2(run_m[h], run_l[h]);
                    }
                    for (int i = stid; i < (run_n - 1) * Hq; i += kGroup) {
                        float* e = a.ws_ml + (((int64_t)seq * a.ws_chunks + run_c0 + 1 + i / Hq) * Hq + i % Hq) * 2;
                        *reinterpret_cast<float2*>(e) = make_float2(-INFINITY, 0.0f);
                    }
                    named_sync(bar_id, kGroup);
                    if (stid == 0) {  // the fence after the barrier releases the whole group's writes
                        __threadfence();
                        const uint32_t prev = atomicAdd(&a.ws_cnt[seq], (uint32_t)run_n);
                        flags[s] = (prev + (uint32_t)run_n == (uint32_t)nchunks) ? 1 : 0;
                        if (flags[s]) __threadfence();
                    }
                    named_sync(bar_id, kGroup);
                    if (flags[s]) {
                        combine_sparse(a, seq, nchunks, out, stid, kGroup, bar_id, red);
                        if (stid == 0) a.ws_cnt[seq] = 0u;
                    }
                }
                run_n = 0;
            }
            // red / stat are rewritten by this group's next softmax: all reads above must be done
            named_sync(bar_id, kGroup);
        }
    }

    tc::fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc::fence_after();
        tc::tmem_dealloc(tmem, kTmemCols);
    }
}

template <int KT>
cudaError_t launch_for_k(cudaStream_t s, const Args& a, int v_type, dim3 grid);
template <> cudaError_t launch_for_k<kQ4_0>(cudaStream_t, const Args&, int, dim3);
template <> cudaError_t launch_for_k<kQ4_1>(cudaStream_t, const Args&, int, dim3);
template <> cudaError_t launch_for_k<kQ5_0>(cudaStream_t, const Args&, int, dim3);
template <> cudaError_t launch_for_k<kQ5_1>(cudaStream_t, const Args&, int, dim3);
template <> cudaError_t launch_for_k<kQ8_0>(cudaStream_t, const Args&, int, dim3);

inline bool supported_type(int t) { return t == kQ4_0 || t == kQ4_1 || t == kQ5_0 || t == kQ5_1 || t == kQ8_0; }

inline int smem_bytes(int k_type, int v_type) {
    const int rowK = (int)type_row_bytes(k_type, 2 * kD), rowV = (int)type_row_bytes(v_type, 2 * kD);
    return Smem(rowK, rowV, k_type == kQ4_1 || k_type == kQ5_1, v_type == kQ4_1 || v_type == kQ5_1).total;
}

}  // namespace dpipe
}  // namespace cvattn
