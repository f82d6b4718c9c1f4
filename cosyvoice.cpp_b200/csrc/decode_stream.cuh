// decode_stream.cuh -- persistent, warp-specialized tensor-core split-KV decode
// that streams 64-position items through a 4-deep ring and keeps each
// sequence's running output in TMEM.
//
// Same contract and exact-integer tensor-core math as decode_pipe.cuh (one
// query row per sequence, ggml_flash_attn_ext with f32 precision,
// src/cosyvoice-kv-cache.cpp:379-386; optional fused update_cache append
// :316,322; split partials merged by the last writer).  What changes:
//
//   * an item is (sequence, 64-position chunk) for both KV heads.  S^T = K.Q^T
//     is one M=128 MMA per K block over rows (kv head, position) against both
//     heads' Q columns (N = 32: kv head x {hi, lo} x 8 heads); the cross-head
//     quarter of S is computed and ignored.  O^T = V^T.P' is M=128 rows
//     (kv head, dim) x N=64 (kv head x V block x {hi, lo} x 8 heads);
//   * tiles live in 4 slots (item t uses slot t & 3) and raw rows in 3 slots
//     (t % 3), so the conversion of item t waits only for the O MMA of item
//     t - 4, never for the softmax of the item before it; K and Q are handed
//     to the S MMA before V is converted;
//   * each softmax group keeps the running output of the sequence it walks
//     in its own TMEM columns: the MMA accumulates O(t) onto O(t - 2).  The
//     scores of an item are exponentiated against a per-head reference max
//     that is raised only when a score exceeds it by more than 2^8 (then O,
//     the per-thread sums and the min terms are rescaled once O(t - 2) has
//     landed), and P' = P * d_V carries a power-of-two factor per (kv head,
//     V block) that changes only when an item's V scales leave [2^-3, 2^7) of
//     it (again with a rescale).  P <= 2^8 and |d_V| 2^e < 2^7 keep P' < 2^15,
//     inside f16, and the hi + lo split keeps 22 bits of it;
//   * row sums, min terms and the output are formed once per run (a run is
//     the consecutive chunks of one sequence that a softmax group walks).
//
// Roles (608 threads, one CTA per SM):
//   warps 0-7    two converter groups (group c takes items t = c mod 2):
//                raw ggml blocks -> 128B-swizzled f16 tiles of exact integer
//                quants + fp32 scales, and the item's Q hi/lo tile (built
//                once per sequence and kept in registers);
//   warps 8-15   two softmax groups (group s takes items t = s mod 2);
//   warp 16      producer: cp.async.bulk of raw K/V rows;
//   warp 17      S issuer: S(t) once K and Q of t are converted and the
//                softmax of t - 4 has left its TMEM stage;
//   warp 18      O issuer: O(t) once P'(t) is ready.
// Each issuer blocks on its own barrier sequence, so it reacts as soon as a
// stage completes.
// mbarriers hand each stage from role to role; every wait is bounded and a
// failed wait stops all roles through a shared error flag.
#pragma once

#include "decode_pipe.cuh"
#include "rope.cuh"

namespace cvattn {
namespace dstream {

using dec::Args;
using dtc::convert_group;
using dtc::pow2f;
using dpipe::bar_and;
using dpipe::item_of;
using dpipe::named_sync;
using dpipe::pwait;
using dpipe::xpose_index;
using dpipe::xpose_reduce16;

constexpr int kD = 64;
constexpr int kC = 64;               // positions per item
constexpr int kHP = 8;               // query heads per KV head, padded
constexpr int kGroup = 128;          // threads per converter / softmax group
constexpr int kThreads = 608;        // 8 converter + 8 softmax + producer + 2 MMA warps
constexpr int kSoftWarp0 = 8;
constexpr int kProdWarp = 16;
constexpr int kMmaWarp = 17;         // S issuer (and TMEM owner)
constexpr int kMmaOWarp = 18;        // O issuer
constexpr int kSlots = 4;            // tile ring (item t -> slot t & 3)
constexpr int kRawSlots = 3;         // raw-row ring (item t -> slot t % 3)
constexpr uint32_t kTmemCols = 512;  // S stages at columns 64 s, running O of group g at 256 + 64 g
constexpr uint32_t kOCol = 256;
constexpr int kMaxSeq = 512;         // prefix-sum table in shared memory
constexpr int kBarConv = 1;          // named barriers: converter group c uses 1 + c,
constexpr int kBarSoft = 3;          //                 softmax group s uses 3 + s
constexpr int kTileK = 16384, kTileV = 16384, kTileQ = 4096;
constexpr int kSlotBytes = kTileK + kTileV + kTileQ;
constexpr float kLazyLog2 = 8.0f;    // P = 2^(score - reference) stays <= 2^8
constexpr int kEvMin = -3, kEvMax = 6;  // floor(log2(max |d_V| 2^e)) kept in [-3, 6]

enum { B_RAW_FULL = 0, B_RAW_EMPTY = 3, B_K_FULL = 6, B_V_FULL = 10, B_S_FULL = 14, B_P_FULL = 18, B_O_DONE = 22, B_COUNT = 26 };

struct Smem {
    int raw0, raw_stride, tile0;
    int sc0, sc_stride, dk, mk, dv, mv, qsum, esc, wmax, ofirst;  // per tile slot, relative to sc0 + s * sc_stride
    int grp0, grp_stride, redmax, redsum, scr;                     // per softmax group
    int pref, slen, bars, misc, total;
    __host__ __device__ Smem(int rowK, int rowV, bool k_min, bool v_min) {
        int o = 0;
        raw0 = o;
        raw_stride = dtc::round_up(kC * (rowK + rowV), 1024);
        o += kRawSlots * raw_stride;
        tile0 = o;  // [K 16 KB (P' once S is done) | V 16 KB | Q 4 KB] per slot
        o += kSlots * kSlotBytes;
        int r = 0;
        dk = r;     r += 4 * kC * 4;              // [kv head * 2 + block][position]
        mk = r;     r += k_min ? 4 * kC * 4 : 0;
        dv = r;     r += 4 * kC * 4;
        mv = r;     r += v_min ? 4 * kC * 4 : 0;
        qsum = r;   r += 2 * 2 * kHP * 4;         // sum of Q over each K block, times scale (log2 units)
        esc = r;    r += 2 * kHP * 4;             // 2^-e_Q times scale (log2 units)
        wmax = r;   r += 4 * 4 * 4;               // [kv head * 2 + block][4] partial max |d_V|
        ofirst = r; r += 16;                      // O(t) starts a run: no accumulation onto O(t - 2)
        sc0 = o;
        sc_stride = dtc::round_up(r, 16);
        o += kSlots * sc_stride;
        r = 0;
        redmax = r; r += 2 * 4 * 8 * 4;           // [item parity][warp][head] score max
        redsum = r; r += 4 * 32 * 4;              // [warp][sum 8 | min terms 16]
        scr = r;    r += dpipe::kRedFloats * 4;   // the last writer's merge
        grp0 = o;
        grp_stride = dtc::round_up(r, 16);
        o += 2 * grp_stride;
        pref = o;   o += dtc::round_up((kMaxSeq + 1) * 4, 16);
        slen = o;   o += kMaxSeq * 4;                          // lengths (0 for empty / invalid sequences)
        bars = o;   o += dtc::round_up(B_COUNT * 8 + 8, 16);  // mbarriers + TMEM address slot
        misc = o;   o += 16;                                   // ticket flags [2], error flag
        total = dtc::round_up(o, 128);
    }
};

// OR of v over the n threads of named barrier id (all of them must call it).
__device__ __forceinline__ bool bar_or(int id, int n, bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r) : "r"((uint32_t)v), "r"(id), "r"(n) : "memory");
    return r != 0;
}

// Warp-wide reduction of 8 values per lane (transpose butterfly, 9 shuffles).
// Returns the reduction over all 32 lanes of value index xpose_index8(lane);
// the 4 lanes that differ only in bits 0-1 hold the same index.
__device__ __forceinline__ int xpose_index8(int lane) {
    return ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);
}
template <bool kMax>
__device__ __forceinline__ float xpose_reduce8(const float (&v)[8], int lane) {
    float a[4], b[2];
    const bool u16 = lane & 16, u8 = lane & 8, u4 = lane & 4;
#pragma unroll
    for (int i = 0; i < 4; ++i)
        a[i] = dpipe::op2<kMax>(u16 ? v[4 + i] : v[i], __shfl_xor_sync(0xffffffffu, u16 ? v[i] : v[4 + i], 16));
#pragma unroll
    for (int i = 0; i < 2; ++i)
        b[i] = dpipe::op2<kMax>(u8 ? a[2 + i] : a[i], __shfl_xor_sync(0xffffffffu, u8 ? a[i] : a[2 + i], 8));
    float c = dpipe::op2<kMax>(u4 ? b[1] : b[0], __shfl_xor_sync(0xffffffffu, u4 ? b[0] : b[1], 4));
    c = dpipe::op2<kMax>(c, __shfl_xor_sync(0xffffffffu, c, 2));
    return dpipe::op2<kMax>(c, __shfl_xor_sync(0xffffffffu, c, 1));
}

// Next work item after (seq, chunk) in item order: the next chunk, or the
// first chunk of the next sequence that has any (lengths from shared memory).
__device__ __forceinline__ void next_item(const int* slen, int n_seq, int& seq, int& chunk) {
    ++chunk;
    while (seq < n_seq && chunk * kC >= slen[seq]) {
        ++seq;
        chunk = 0;
    }
}

// x = hi + lo for a pair of floats, packed as f16x2 (hi) and f16x2 (lo): hi is
// x truncated to 11 significant bits (exact in f16 for normal magnitudes), lo
// the exact remainder rounded to f16, so hi + lo carries 21+ bits of x.  Bit
// masks and packed conversions only (no single-value conversions).
__device__ __forceinline__ void split_f16x2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
    const float h0 = __uint_as_float(__float_as_uint(x0) & 0xFFFFE000u);
    const float h1 = __uint_as_float(__float_as_uint(x1) & 0xFFFFE000u);
    hi = tc::pack_f16x2(h0, h1);
    lo = tc::pack_f16x2(x0 - h0, x1 - h1);
}

// Runs of one sequence: the non-empty intersections of its item range
// [p_seq, p_seq + nchunks) with the two halves of every CTA's item range (the
// cut of the main loop).  Each run leaves its partial in the workspace slot of
// its first chunk; writes those slots to idx and returns their count (at most
// two per CTA).
__device__ __forceinline__ int run_slots(int p_seq, int nchunks, int n_items, int grid, int* idx) {
    const int first = p_seq, end = p_seq + nchunks;
    // CTA b holds items [b n / grid, (b + 1) n / grid): item i is in CTA ((i + 1) grid - 1) / n
    const int b0 = (int)(((long long)(first + 1) * grid - 1) / n_items);
    const int b1 = (int)(((long long)end * grid - 1) / n_items);
    int r = 0;
    for (int b = b0; b <= b1; ++b) {
        const int lo = (int)(((long long)b * n_items) / grid);
        const int hi = (int)(((long long)(b + 1) * n_items) / grid);
        const int mid = lo + ((hi - lo + 1) >> 1);
        const int a0 = max(lo, first), a1 = min(mid, end);
        if (a0 < a1) idx[r++] = a0 - first;
        const int c0 = max(mid, first), c1 = min(hi, end);
        if (c0 < c1) idx[r++] = c0 - first;
    }
    return r;
}

// Log-sum-exp merge of one sequence's run partials by the nt threads of a
// softmax group: the run slots are known from the cut (no empty slots are
// read or marked), and each thread = (head, 4 dims) loads the (max, sum) and
// output of up to 8 runs at once, so a sequence split a few ways takes one
// round of L2 loads.  idx: dpipe::kRedFloats ints of scratch.
__device__ __forceinline__ void combine_runs(const Args& a, int seq, int p_seq, int nchunks, int n_items, int grid,
                                             float* out, int tid, int nt, int bar_id, int* idx) {
    if (tid == 0) idx[dpipe::kRedFloats - 1] = run_slots(p_seq, nchunks, n_items, grid, idx);
    named_sync(bar_id, nt);
    const int R = idx[dpipe::kRedFloats - 1];
    const int Hq = a.Hq;
    const bool emit_partial = (a.flags & CVATTN_DECODE_EMIT_PARTIAL) != 0;
    const float* seq_ml = a.ws_ml + ((int64_t)seq * a.ws_chunks) * Hq * 2;
    const float* seq_o = a.ws_o + ((int64_t)seq * a.ws_chunks) * Hq * kD;
    for (int it = tid; it < Hq * (kD / 4); it += nt) {
        const int h = it / (kD / 4), dd = (it % (kD / 4)) * 4;
        float M = -INFINITY, Ls = 0.0f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int r0 = 0; r0 < R; r0 += 8) {
            float2 ml[8];
            float4 v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int c = idx[min(r0 + j, R - 1)];
                ml[j] = __ldcg(reinterpret_cast<const float2*>(seq_ml + ((int64_t)c * Hq + h) * 2));
                v[j] = dpipe::ldcg_f4(seq_o + ((int64_t)c * Hq + h) * kD + dd);
            }
            float bm = M;
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (r0 + j < R) bm = fmaxf(bm, ml[j].x);
            const float rs = (M == -INFINITY) ? 0.0f : fast_exp2(M - bm);
            Ls *= rs;
            acc.x *= rs; acc.y *= rs; acc.z *= rs; acc.w *= rs;
            M = bm;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (r0 + j >= R) break;
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

// Atomic add with acquire-release semantics at GPU scope: publishes this
// thread's (and, after a CTA barrier, its group's) earlier writes and sees
// those of every earlier add on the same counter.
__device__ __forceinline__ uint32_t atom_add_acq_rel(uint32_t* p, uint32_t v) {
    uint32_t old;
    asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// floor(log2(x)) of a positive normal float.
__device__ __forceinline__ int ilog2f(float x) { return ((__float_as_int(x) >> 23) & 0xff) - 127; }

// Exponent e with max |d_V| 2^e in [16, 32); 0 for an all-zero block.
__device__ __forceinline__ int v_exp_target(float vmax) {
    if (!(vmax > 0.0f)) return 0;
    const int e = 4 - ilog2f(vmax);
    return e > 60 ? 60 : (e < -60 ? -60 : e);
}

// Raw rows of one item -> swizzled f16 tiles [kv head][64 positions x 64 dims]
// + scales [kv head * 2 + block][position] (+ mins).  Converter warp cw takes
// kv head cw / 2 and block cw % 2 for positions lane and lane + 32, so the
// alignment of the quants (2-byte or 4-byte, by block) is uniform per warp
// and each lane stores whole 16-byte chunks of distinct rows (no bank
// conflicts).  For V also max |d| of that column of blocks (wmax row
// [kv head * 2 + block]: the max, then three zeros).
template <int T, bool kIsV>
__device__ __forceinline__ void convert_item(const uint8_t* raw, int row, int head, int n, int cw, int lane,
                                             uint8_t* tiles, float* dsc, float* msc, float* wmax) {
    constexpr int GB = group_bytes(T);
    const int g = cw >> 1, blk = cw & 1;
    uint8_t* tile = tiles + g * 8192;
    float dm = 0.0f;
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const int key = lane + 32 * u;
        uint32_t w[16];
        float d = 0.0f, m = 0.0f;
        if (key < n) {
            convert_group<T>(raw + key * row + g * head + blk * GB, w, d, m);
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) w[i] = 0u;
        }
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4)
            *reinterpret_cast<uint4*>(tile + tc::sw128_offset(key, blk * 4 + c4)) =
                make_uint4(w[4 * c4], w[4 * c4 + 1], w[4 * c4 + 2], w[4 * c4 + 3]);
        dsc[(g * 2 + blk) * kC + key] = d;
        if constexpr (BlockTraits<T>::HAS_MIN) msc[(g * 2 + blk) * kC + key] = m;
        dm = fmaxf(dm, fabsf(d));
    }
    if constexpr (kIsV) {
        dm = dec::warp_max(dm);
        if (lane == 0) *reinterpret_cast<float4*>(wmax + (g * 2 + blk) * 4) = make_float4(dm, 0.0f, 0.0f, 0.0f);
    }
}

// (bounds of 640 threads cap registers at 96: the SM sub-partition holding five of
// the 19 warps must fit them)
template <int KT, int VT>
__global__ void __launch_bounds__(640, 1) decode_stream_kernel(const Args a) {
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
    int* slen = reinterpret_cast<int*>(smem + L.slen);
    griddep_launch_dependents();  // the next launch may start its prologue on SMs this grid frees

    // ---- setup: barriers, TMEM, per-sequence chunk prefix sums
    if (tid == 0) {
        for (int i = 0; i < B_COUNT; ++i) {
            const bool by_threads = (i >= B_RAW_EMPTY && i < B_RAW_EMPTY + kRawSlots) ||
                                    (i >= B_K_FULL && i < B_V_FULL + kSlots) ||
                                    (i >= B_P_FULL && i < B_P_FULL + kSlots);
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
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tmem = *tmem_slot;
    const int n_items = pref[n_seq];
    // contiguous item range per CTA; local item t alternates between its two halves
    // (t even: first half, t odd: second half), so each softmax group walks
    // consecutive chunks and accumulates them before anything leaves the SM
    const int lo = (int)(((long long)blockIdx.x * n_items) / gridDim.x);
    const int n_local = (int)(((long long)(blockIdx.x + 1) * n_items) / gridDim.x) - lo;
    const int n_half0 = (n_local + 1) >> 1;
    auto item_at = [&](int t) { return (t & 1) ? lo + n_half0 + (t >> 1) : lo + (t >> 1); };

    if (warp == kProdWarp) {
        // ===================================================== producer
        if (lane == 0) {
            int r = 0, k3 = 0;  // raw slot t % 3 and its fill count t / 3
            // one cursor per half of the range (items t even / odd), each with its sequence's rows;
            // (seq, chunk, ...) is the cursor of item t, (seq_o, chunk_o, ...) the other half's
            int seq = 0, chunk = 0, seq_o = 0, chunk_o = 0, cur = -1, cur_o = -1;
            const uint8_t *kb = nullptr, *vb = nullptr, *kb_o = nullptr, *vb_o = nullptr;
            item_of(pref, n_seq, item_at(0), seq, chunk);
            if (n_local > 1) item_of(pref, n_seq, item_at(1), seq_o, chunk_o);
            for (int t = 0; t < n_local; ++t) {
                if (t >= kRawSlots && !pwait(&bars[B_RAW_EMPTY + r], (k3 - 1) & 1, err, a.status, 1)) break;
                if (cur != seq) {
                    cur = seq;
                    kb = a.k_seq_ptrs ? reinterpret_cast<const uint8_t*>(a.k_seq_ptrs[seq]) : a.k_base + seq * a.k_nb2;
                    vb = a.v_seq_ptrs ? reinterpret_cast<const uint8_t*>(a.v_seq_ptrs[seq]) : a.v_base + seq * a.v_nb2;
                }
                const int len = slen[seq];
                const int p0 = chunk * kC, n = min(kC, len - p0);
                const uint8_t* ksrc = kb + (int64_t)p0 * rowK;
                const uint8_t* vsrc = vb + (int64_t)p0 * rowV;
                uint8_t* kdst = smem + L.raw0 + r * L.raw_stride;
                uint8_t* vdst = kdst + kC * rowK;
                const uint32_t kbytes = (uint32_t)(n * rowK), vbytes = (uint32_t)(n * rowV);
                const uint32_t kbulk = ((reinterpret_cast<uintptr_t>(ksrc) & 15) == 0) ? (kbytes & ~15u) : 0u;
                const uint32_t vbulk = ((reinterpret_cast<uintptr_t>(vsrc) & 15) == 0) ? (vbytes & ~15u) : 0u;
                // tails first: the arrive below releases these generic stores
                for (uint32_t i = kbulk / 2; i < kbytes / 2; ++i)
                    reinterpret_cast<uint16_t*>(kdst)[i] = reinterpret_cast<const uint16_t*>(ksrc)[i];
                for (uint32_t i = vbulk / 2; i < vbytes / 2; ++i)
                    reinterpret_cast<uint16_t*>(vdst)[i] = reinterpret_cast<const uint16_t*>(vsrc)[i];
                mbar_arrive_expect_tx(&bars[B_RAW_FULL + r], kbulk + vbulk);
                if (kbulk) bulk_g2s(kdst, ksrc, kbulk, &bars[B_RAW_FULL + r]);
                if (vbulk) bulk_g2s(vdst, vsrc, vbulk, &bars[B_RAW_FULL + r]);
                if (++r == kRawSlots) { r = 0; ++k3; }
                next_item(slen, n_seq, seq, chunk);
                // the next item comes from the other half
                int x = seq; seq = seq_o; seq_o = x;
                x = chunk; chunk = chunk_o; chunk_o = x;
                x = cur; cur = cur_o; cur_o = x;
                const uint8_t* y = kb; kb = kb_o; kb_o = y;
                y = vb; vb = vb_o; vb_o = y;
            }
        }
    } else if (warp == kMmaWarp) {
        // ===================================================== S issuer
        if (lane == 0) {
            const uint32_t idesc_s = tc::idesc_f16_f32(128, 32, false);
            // descriptors of slot 0; slot s4 adds s4 * kSlotBytes / 16 to the address field
            const uint32_t kaddr0 = smem_addr(smem + L.tile0);
            const uint64_t ad0 = tc::sdesc_sw128(kaddr0, 16, 1024);
            const uint64_t bd0 = tc::sdesc_sw128(kaddr0 + kTileK + kTileV, 16, 1024);
            for (int t = 0; t < n_local; ++t) {
                const int s4 = t & 3;
                // S(t) reuses the TMEM stage of S(t - 4): free once the softmax of t - 4 has handed over P'
                if (t >= kSlots && !pwait(&bars[B_P_FULL + s4], ((t >> 2) - 1) & 1, err, a.status, 3)) break;
                if (!pwait(&bars[B_K_FULL + s4], (t >> 2) & 1, err, a.status, 4)) break;
                tc::fence_after();
                const uint64_t so = (uint64_t)(s4 * (kSlotBytes >> 4));
#pragma unroll
                for (int blk = 0; blk < 2; ++blk)
#pragma unroll
                    for (int kk = 0; kk < 2; ++kk) {
                        const uint64_t k16 = (uint64_t)(2 * (blk * 2 + kk));  // 32 bytes per 16 dims
                        tc::mma_ss(tmem + s4 * 64 + blk * 32, ad0 + so + k16, bd0 + so + k16, idesc_s, kk ? 1u : 0u);
                    }
                tc::mma_commit(&bars[B_S_FULL + s4]);
            }
        }
    } else if (warp == kMmaOWarp) {
        // ===================================================== O issuer
        if (lane == 0) {
            const uint32_t idesc_o = tc::idesc_f16_f32(128, 64, true, true);
            const uint32_t paddr0 = smem_addr(smem + L.tile0);
            const uint64_t ad0 = tc::sdesc_sw128(paddr0 + kTileK, 8192, 1024);  // V^T, MN-major
            const uint64_t bd0 = tc::sdesc_sw128(paddr0, 16, 1024);             // P', MN-major
            for (int t = 0; t < n_local; ++t) {
                const int s4 = t & 3;
                if (!pwait(&bars[B_P_FULL + s4], (t >> 2) & 1, err, a.status, 2)) break;
                tc::fence_after();
                const uint64_t so = (uint64_t)(s4 * (kSlotBytes >> 4));
                const bool first = *reinterpret_cast<const volatile int*>(smem + L.sc0 + s4 * L.sc_stride + L.ofirst) != 0;
#pragma unroll
                for (int kk = 0; kk < kC / 16; ++kk) {
                    const uint64_t k16 = (uint64_t)(kk * (2048 >> 4));  // 2 KB per 16 positions
                    tc::mma_ss(tmem + kOCol + (t & 1) * 64, ad0 + so + k16, bd0 + so + k16, idesc_o,
                               (kk > 0 || !first) ? 1u : 0u);
                }
                tc::mma_commit(&bars[B_O_DONE + s4]);
            }
        }
    } else if (warp < kSoftWarp0) {
        // ===================================================== converters (group c: items t = c mod 2)
        if (early) griddep_wait();
        const int c = warp >> 2;
        const int bar_id = kBarConv + c;
        const int ctid = tid & (kGroup - 1);
        const int cw = warp & 3;
        // this thread's two 8-float pieces of Q of a sequence
        float4 qv[2][2];
        auto load_q = [&](int sq) {
#pragma unroll
            for (int qi = 0; qi < 2; ++qi) {
                const int item = ctid + qi * 128;
                const int g = item >> 7, row = (item >> 3) & 15, cc = item & 7;
                const int h = row & 7;
                if (h < G) {
                    const float* qr = a.q + (int64_t)sq * a.q_seq_stride + (g * G + h) * kD + 8 * cc;
                    qv[qi][0] = *reinterpret_cast<const float4*>(qr);
                    qv[qi][1] = *reinterpret_cast<const float4*>(qr + 4);
                } else {
                    qv[qi][0] = qv[qi][1] = make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
        };
        // this thread's two 16-byte pieces of the Q hi/lo tile (row (kv head, {hi, lo},
        // head), 8 dims), with the row's factor 2^-e_Q * scale and (K with mins) its
        // sums over a K block: built once per sequence
        uint4 qw[2];
        float qe[2], qs[2];
        const RopeDev rope{a.rope_mode, a.rope_n_dims, kD, a.rope_theta_scale, a.rope_freq_scale, a.rope_attn_factor};
        int seq = 0, chunk = 0;  // cursor of the group's current item
        auto build_q = [&]() {
            // (cos, sin) of pair k = lane at the new token's position: one sincosf per lane,
            // handed to the elements that need it by shuffles
            float2 qcs = make_float2(1.0f, 0.0f);
            if (rope.n_dims > 0) qcs = rope_cs(rope, rope_theta(rope, slen[seq] - 1, lane));
#pragma unroll
            for (int qi = 0; qi < 2; ++qi) {
                const int item = ctid + qi * 128;
                const int row = (item >> 3) & 15, cc = item & 7;
                const bool lo_row = row >= 8;
                const float4 u = qv[qi][0], v = qv[qi][1];
                float x[8] = {u.x, u.y, u.z, u.w, v.x, v.y, v.z, v.w};
                if (rope.n_dims > 0) {  // Q turns by the new token's position (n_dims = head_dim)
                    float y[8];
                    bool first = true;
                    if (rope.mode & 2) {  // NEOX: partner dims d +- 32 live in lane cc ^ 4
#pragma unroll
                        for (int e = 0; e < 8; ++e) y[e] = __shfl_xor_sync(0xffffffffu, x[e], 4);
                        first = cc < 4;
                    } else {  // NORMAL: partner dim d ^ 1 is in this thread
#pragma unroll
                        for (int e = 0; e < 8; ++e) y[e] = x[e ^ 1];
                    }
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        // pair k: NEOX d mod 32, NORMAL d / 2, with d = 8 cc + e; its (cos, sin) from lane k
                        const int k = (rope.mode & 2) ? 8 * (cc & 3) + e : 4 * cc + (e >> 1);
                        const float2 cs = make_float2(__shfl_sync(0xffffffffu, qcs.x, k), __shfl_sync(0xffffffffu, qcs.y, k));
                        x[e] = rope_rotate(x[e], y[e], cs, (rope.mode & 2) ? first : (e & 1) == 0);
                    }
                }
                float am = 0.0f, part = 0.0f;
#pragma unroll
                for (int e = 0; e < 8; ++e) { am = fmaxf(am, fabsf(x[e])); part += x[e]; }
#pragma unroll
                for (int o = 1; o < 8; o <<= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
                const int ex = dtc::norm_exp(am);
                const float scq = pow2f(ex);
                uint32_t wv[4];
#pragma unroll
                for (int e = 0; e < 8; e += 2) {
                    uint32_t hi, lo;
                    split_f16x2(x[e] * scq, x[e + 1] * scq, hi, lo);
                    wv[e / 2] = lo_row ? lo : hi;
                }
                qw[qi] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
                qe[qi] = pow2f(-ex) * a.scale_log2;
                part += __shfl_xor_sync(0xffffffffu, part, 1);
                part += __shfl_xor_sync(0xffffffffu, part, 2);
                qs[qi] = part * a.scale_log2;
            }
        };
        bool q_dirty = true;  // qv holds a sequence's Q that qw / qe / qs do not reflect yet
        if (c < n_local) {
            item_of(pref, n_seq, item_at(c), seq, chunk);
            load_q(seq);
        }
        for (int t = c; t < n_local; t += 2) {
            const int s4 = t & 3, r = t % kRawSlots, k3 = t / kRawSlots;
            const int len = slen[seq];
            const int p0 = chunk * kC, n = min(kC, len - p0);
            const int nchunks = (len + kC - 1) / kC;
            uint8_t* Kraw = smem + L.raw0 + r * L.raw_stride;
            uint8_t* Vraw = Kraw + kC * rowK;
            uint8_t* tiles = smem + L.tile0 + s4 * kSlotBytes;
            uint8_t* sc = smem + L.sc0 + s4 * L.sc_stride;
            float* dk = reinterpret_cast<float*>(sc + L.dk);
            float* mk = reinterpret_cast<float*>(sc + L.mk);
            float* dv = reinterpret_cast<float*>(sc + L.dv);
            float* mv = reinterpret_cast<float*>(sc + L.mv);
            float* wmax = reinterpret_cast<float*>(sc + L.wmax);
            float* esc = reinterpret_cast<float*>(sc + L.esc);
            float* qsum = reinterpret_cast<float*>(sc + L.qsum);
            {   // tiles of slot s4 are free once O(t - 4) has completed; raw rows of item t have landed
                bool ok = t < kSlots || pwait(&bars[B_O_DONE + s4], ((t >> 2) - 1) & 1, err, a.status, 5);
                ok = ok && pwait(&bars[B_RAW_FULL + r], k3 & 1, err, a.status, 6);
                if (!bar_and(bar_id, kGroup, ok)) break;
            }
            if (q_dirty) {
                build_q();
                q_dirty = false;
            }
            if (a.k_new && chunk == nchunks - 1) {
                const uint8_t* kb = a.k_seq_ptrs ? reinterpret_cast<const uint8_t*>(a.k_seq_ptrs[seq]) : a.k_base + seq * a.k_nb2;
                const uint8_t* vb = a.v_seq_ptrs ? reinterpret_cast<const uint8_t*>(a.v_seq_ptrs[seq]) : a.v_base + seq * a.v_nb2;
                const int rr = len - 1 - p0;
                // (cos, sin) of pair k = lane at position len - 1 (NEOX pairs element `lane` of
                // both 32-element halves of a head; NORMAL takes pair d / 2 from its lane)
                float2 kcs = make_float2(1.0f, 0.0f);
                if (rope.n_dims > 0) kcs = rope_cs(rope, rope_theta(rope, len - 1, lane));
                for (int gi = cw; gi < 8; gi += 4) {
                    const bool isv = gi >= 4;
                    const int g2 = gi & 3;
                    float xv = (isv ? a.v_new : a.k_new)[(int64_t)seq * 2 * kD + g2 * 32 + lane];
                    if (!isv && rope.n_dims > 0) {  // the new K row turns by position len - 1
                        const float* krow = a.k_new + (int64_t)seq * 2 * kD + (g2 >> 1) * kD;  // its head
                        const int d = (g2 & 1) * 32 + lane;
                        int k;
                        bool first;
                        const int pd = rope_pair(rope, d, k, first);
                        const float2 cs = make_float2(__shfl_sync(0xffffffffu, kcs.x, k), __shfl_sync(0xffffffffu, kcs.y, k));
                        xv = rope_rotate(xv, krow[pd], cs, first);
                    }
                    if (!isv) {
                        quantize_block_warp<KT>(xv, Kraw + rr * rowK + g2 * GBK, lane);
                        quantize_block_warp<KT>(xv, const_cast<uint8_t*>(kb) + (int64_t)(len - 1) * rowK + g2 * GBK, lane);
                    } else {
                        quantize_block_warp<VT>(xv, Vraw + rr * rowV + g2 * GBV, lane);
                        quantize_block_warp<VT>(xv, const_cast<uint8_t*>(vb) + (int64_t)(len - 1) * rowV + g2 * GBV, lane);
                    }
                }
                named_sync(bar_id, kGroup);
            }
            convert_item<KT, false>(Kraw, rowK, headK, n, cw, lane, tiles, dk, mk, nullptr);
            // Q hi/lo tile of this item's sequence
#pragma unroll
            for (int qi = 0; qi < 2; ++qi) {
                const int item = ctid + qi * 128;
                const int g = item >> 7, row = (item >> 3) & 15, cc = item & 7;
                const int h = row & 7;
                const bool lo_row = row >= 8;
                *reinterpret_cast<uint4*>(tiles + kTileK + kTileV + g * 2048 + tc::sw128_offset(row, cc)) = qw[qi];
                if (!lo_row && cc == 0) esc[g * kHP + h] = qe[qi];
                if constexpr (K_MIN)
                    if (!lo_row && (cc & 3) == 0) qsum[(g * 2 + (cc >> 2)) * kHP + h] = qs[qi];
            }
            fence_proxy_async_smem();
            mbar_arrive(&bars[B_K_FULL + s4]);  // S(t) may start while V converts
            convert_item<VT, true>(Vraw, rowV, headV, n, cw, lane, tiles + kTileK, dv, mv, wmax);
            mbar_arrive(&bars[B_RAW_EMPTY + r]);  // raw slot r may be refilled
            // Q of the next item, loaded now so the latency hides under the waits and the conversion
            const int prev = seq;
            next_item(slen, n_seq, seq, chunk);
            if (t + 2 < n_local && seq != prev) {
                load_q(seq);
                q_dirty = true;
            }
            fence_proxy_async_smem();
            mbar_arrive(&bars[B_V_FULL + s4]);
        }
    } else {
        // ===================================================== softmax (group s: items t = s mod 2)
        if (early) griddep_wait();
        const int s = (warp - kSoftWarp0) >> 2;
        const int bar_id = kBarSoft + s;
        const int stid = tid & (kGroup - 1);     // 0..127 = TMEM lane
        const int sw = warp & 3;                 // TMEM lane quarter of this warp
        const int g = stid >> 6;                 // kv head of this lane: rows (g, position) of S, (g, dim) of O
        const int key = stid & 63;               // position within the item; the dim in O
        const int oblk = key >> 5;               // V block of that dim (uniform per warp)
        const uint32_t lane_base = (uint32_t)(sw * 32) << 16;
        uint8_t* gbase = smem + L.grp0 + s * L.grp_stride;
        float* redmax = reinterpret_cast<float*>(gbase + L.redmax);
        float* redsum = reinterpret_cast<float*>(gbase + L.redsum);
        float* scr = reinterpret_cast<float*>(gbase + L.scr);
        const uint32_t o_taddr = tmem + lane_base + kOCol + s * 64 + g * 32 + oblk * 16;
        // running state of the sequence this group walks
        float mref[kHP], lsum[kHP], pmv[V_MIN ? 16 : 1];
        int ev0 = 0, ev1 = 0;  // power-of-two factor of P' for V blocks 0 / 1 of this lane's kv head
#pragma unroll
        for (int h = 0; h < kHP; ++h) { mref[h] = -INFINITY; lsum[h] = 0.0f; }
#pragma unroll
        for (int i = 0; i < (V_MIN ? 16 : 1); ++i) pmv[i] = 0.0f;
        int run_n = 0, run_c0 = 0;
        int seq_n = 0, chunk_n = 0;  // cursor of the group's next item
        if (s < n_local) item_of(pref, n_seq, item_at(s), seq_n, chunk_n);

        for (int t = s; t < n_local; t += 2) {
            const int seq = seq_n, chunk = chunk_n;
            next_item(slen, n_seq, seq_n, chunk_n);
            const int len = slen[seq];
            const int n = min(kC, len - chunk * kC);
            const int nchunks = (len + kC - 1) / kC;
            const int s4 = t & 3;
            uint8_t* sc = smem + L.sc0 + s4 * L.sc_stride;
            const float* dk = reinterpret_cast<const float*>(sc + L.dk);
            const float* mk = reinterpret_cast<const float*>(sc + L.mk);
            const float* dv = reinterpret_cast<const float*>(sc + L.dv);
            const float* mv = reinterpret_cast<const float*>(sc + L.mv);
            const float* esc = reinterpret_cast<const float*>(sc + L.esc);
            const float* qsum = reinterpret_cast<const float*>(sc + L.qsum);
            const float4* wmax4 = reinterpret_cast<const float4*>(sc + L.wmax);
            // S(t) has landed and the V tile, scales and max |d_V| of item t are written
            if (!bar_and(bar_id, kGroup, pwait(&bars[B_S_FULL + s4], (t >> 2) & 1, err, a.status, 8) &&
                                         pwait(&bars[B_V_FULL + s4], (t >> 2) & 1, err, a.status, 7)))
                break;
            tc::fence_after();
            uint32_t sa[16], sb[16];  // S of K blocks 0 / 1: [hi 8 heads | lo 8 heads]
            tc::tmem_ld16(tmem + lane_base + s4 * 64 + g * 16, sa);
            tc::tmem_ld16(tmem + lane_base + s4 * 64 + 32 + g * 16, sb);
            // per-position scales and the per-sequence Q factors while the loads are in flight
            const float d0 = dk[(g * 2) * kC + key], d1 = dk[(g * 2 + 1) * kC + key];
            const float dv0 = dv[(g * 2) * kC + key], dv1 = dv[(g * 2 + 1) * kC + key];
            float m0 = 0.0f, m1 = 0.0f, mv0 = 0.0f, mv1 = 0.0f;
            if constexpr (K_MIN) { m0 = mk[(g * 2) * kC + key]; m1 = mk[(g * 2 + 1) * kC + key]; }
            if constexpr (V_MIN) { mv0 = mv[(g * 2) * kC + key]; mv1 = mv[(g * 2 + 1) * kC + key]; }
            float e8[kHP];
            {
                const float4 e0 = *reinterpret_cast<const float4*>(esc + g * kHP);
                const float4 e1 = *reinterpret_cast<const float4*>(esc + g * kHP + 4);
                e8[0] = e0.x; e8[1] = e0.y; e8[2] = e0.z; e8[3] = e0.w;
                e8[4] = e1.x; e8[5] = e1.y; e8[6] = e1.z; e8[7] = e1.w;
            }
            // V scale exponents of this item for this lane's kv head (identical across its 64 lanes)
            int evn0, evn1;
            bool evchg = false;
            {
                const float4 w0 = wmax4[g * 2], w1 = wmax4[g * 2 + 1];
                const float vm0 = fmaxf(fmaxf(w0.x, w0.y), fmaxf(w0.z, w0.w));
                const float vm1 = fmaxf(fmaxf(w1.x, w1.y), fmaxf(w1.z, w1.w));
                if (run_n == 0) {
                    evn0 = v_exp_target(vm0);
                    evn1 = v_exp_target(vm1);
                } else {
                    const int x0 = vm0 > 0.0f ? ilog2f(vm0) + ev0 : 0, x1 = vm1 > 0.0f ? ilog2f(vm1) + ev1 : 0;
                    evn0 = (x0 < kEvMin || x0 > kEvMax) ? v_exp_target(vm0) : ev0;
                    evn1 = (x1 < kEvMin || x1 > kEvMax) ? v_exp_target(vm1) : ev1;
                    evchg = evn0 != ev0 || evn1 != ev1;
                }
            }
            tc::tmem_ld_wait();
            float sc8[kHP];  // scores in log2 units
            bool big = false;
#pragma unroll
            for (int h = 0; h < kHP; ++h) {
                float tt = d0 * (__uint_as_float(sa[h]) + __uint_as_float(sa[8 + h])) +
                           d1 * (__uint_as_float(sb[h]) + __uint_as_float(sb[8 + h]));
                tt *= e8[h];
                if constexpr (K_MIN) tt += m0 * qsum[(g * 2) * kHP + h] + m1 * qsum[(g * 2 + 1) * kHP + h];
                sc8[h] = (key < n && h < G) ? tt : -INFINITY;
                big |= sc8[h] - mref[h] > kLazyLog2;  // always true on a run's first item (reference -inf)
            }
            // a score above the reference by more than 2^8 or a V scale out of range anywhere in the
            // group sends the whole group through the max path and the rescale; emitted partials
            // carry the true max, so then every item takes the max path
            const bool need_max = bar_or(bar_id, kGroup, big || evchg || emit_partial);
            float alpha[kHP];
#pragma unroll
            for (int h = 0; h < kHP; ++h) alpha[h] = 1.0f;
            if (need_max) {
                float* rm = redmax + ((t >> 1) & 1) * 32;
                const float wm = xpose_reduce8<true>(sc8, lane);
                if ((lane & 3) == 0) rm[sw * 8 + xpose_index8(lane)] = wm;
                named_sync(bar_id, kGroup);
#pragma unroll
                for (int h = 0; h < kHP; ++h) {
                    const float M = fmaxf(rm[(2 * g) * 8 + h], rm[(2 * g + 1) * 8 + h]);
                    float mn = fmaxf(mref[h], M);
                    if (mn == -INFINITY) mn = 0.0f;  // a padding head: every score is -inf
                    alpha[h] = fast_exp2(mref[h] - mn);
                    mref[h] = mn;
                }
            }
            if (need_max && run_n > 0) {
                // O holds the run so far once O(t - 2) has completed
                if (!bar_and(bar_id, kGroup, pwait(&bars[B_O_DONE + ((t - 2) & 3)], ((t - 2) >> 2) & 1, err, a.status, 9)))
                    break;
                tc::fence_after();
                const float fe = pow2f(oblk ? evn1 - ev1 : evn0 - ev0);
                bool rescale = fe != 1.0f;
#pragma unroll
                for (int h = 0; h < kHP; ++h) rescale |= alpha[h] != 1.0f;
                if (rescale) {  // uniform per warp: g and oblk are
                    uint32_t ov[16];
                    tc::tmem_ld16(o_taddr, ov);
                    tc::tmem_ld_wait();
#pragma unroll
                    for (int h = 0; h < kHP; ++h) {
                        const float f = alpha[h] * fe;
                        ov[h] = __float_as_uint(__uint_as_float(ov[h]) * f);
                        ov[8 + h] = __float_as_uint(__uint_as_float(ov[8 + h]) * f);
                    }
                    tc::tmem_st16(o_taddr, ov);
                    tc::tmem_st_wait();
                }
#pragma unroll
                for (int h = 0; h < kHP; ++h) lsum[h] *= alpha[h];
                if constexpr (V_MIN) {
#pragma unroll
                    for (int h = 0; h < kHP; ++h) { pmv[h] *= alpha[h]; pmv[8 + h] *= alpha[h]; }
                }
                tc::fence_before();
            }
            ev0 = evn0;
            ev1 = evn1;
            // P = 2^(score - reference) <= 2^8; P' = P d_V 2^e split into f16 hi + lo
            float p[kHP];
#pragma unroll
            for (int h = 0; h < kHP; ++h) {
                p[h] = sc8[h] == -INFINITY ? 0.0f : fast_exp2(sc8[h] - mref[h]);
                lsum[h] += p[h];
            }
            uint8_t* ptile = smem + L.tile0 + s4 * kSlotBytes;  // the K tile is dead once S is complete
#pragma unroll
            for (int b2 = 0; b2 < 2; ++b2) {
                const float f = (b2 ? dv1 : dv0) * pow2f(b2 ? ev1 : ev0);
                uint32_t hi[4], lo4[4];
#pragma unroll
                for (int h = 0; h < kHP; h += 2) split_f16x2(p[h] * f, p[h + 1] * f, hi[h / 2], lo4[h / 2]);
                *reinterpret_cast<uint4*>(ptile + tc::sw128_offset(key, g * 4 + b2 * 2)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                *reinterpret_cast<uint4*>(ptile + tc::sw128_offset(key, g * 4 + b2 * 2 + 1)) =
                    make_uint4(lo4[0], lo4[1], lo4[2], lo4[3]);
                if constexpr (V_MIN) {
                    const float mvk = b2 ? mv1 : mv0;
#pragma unroll
                    for (int h = 0; h < kHP; ++h) pmv[b2 * 8 + h] += p[h] * mvk;
                }
            }
            if (stid == 0) *reinterpret_cast<volatile int*>(sc + L.ofirst) = run_n == 0 ? 1 : 0;
            fence_proxy_async_smem();
            mbar_arrive(&bars[B_P_FULL + s4]);
            if (run_n == 0) run_c0 = chunk;
            ++run_n;

            if (t + 2 < n_local && seq_n == seq) continue;
            // ------------------------------------------------ end of the run: O(t) holds all of it
            if (!bar_and(bar_id, kGroup, pwait(&bars[B_O_DONE + s4], (t >> 2) & 1, err, a.status, 10))) break;
            tc::fence_after();
            uint32_t ov[16];
            tc::tmem_ld16(o_taddr, ov);
            {
                const float ls = xpose_reduce8<false>(lsum, lane);
                if ((lane & 3) == 0) redsum[sw * 32 + xpose_index8(lane)] = ls;
                if constexpr (V_MIN) {
                    const float pv = xpose_reduce16<false>(pmv, lane);
                    if (!(lane & 1)) redsum[sw * 32 + 8 + xpose_index(lane)] = pv;
                }
            }
            tc::tmem_ld_wait();
            tc::fence_before();
            named_sync(bar_id, kGroup);
            float* out = a.out + (int64_t)seq * a.out_seq_stride;
            const int dim = key;
            const float inv_e = pow2f(oblk ? -ev1 : -ev0);
            float run_o[kHP], run_l[kHP];
#pragma unroll
            for (int h = 0; h < kHP; ++h) {
                run_l[h] = redsum[(2 * g) * 32 + h] + redsum[(2 * g + 1) * 32 + h];
                float o = (__uint_as_float(ov[h]) + __uint_as_float(ov[8 + h])) * inv_e;
                if constexpr (V_MIN) o += redsum[(2 * g) * 32 + 8 + oblk * 8 + h] + redsum[(2 * g + 1) * 32 + 8 + oblk * 8 + h];
                run_o[h] = o;
            }
            if (run_n == nchunks) {  // the whole sequence went through this group
#pragma unroll
                for (int h = 0; h < kHP; ++h) {
                    if (h >= G) break;
                    const int qh = g * G + h;
                    out[qh * kD + dim] = emit_partial ? run_o[h] : run_o[h] / run_l[h];
                    if (emit_partial && dim == 0) {
                        a.partial_ml[((int64_t)seq * Hq + qh) * 2] = mref[h];
                        a.partial_ml[((int64_t)seq * Hq + qh) * 2 + 1] = run_l[h];
                    }
                }
            } else {
                // partial into the slot of the run's first chunk
                float* wso = a.ws_o + (((int64_t)seq * a.ws_chunks + run_c0) * Hq) * kD;
                float* wsml = a.ws_ml + (((int64_t)seq * a.ws_chunks + run_c0) * Hq) * 2;
#pragma unroll
                for (int h = 0; h < kHP; ++h) {
                    if (h >= G) break;
                    const int qh = g * G + h;
                    wso[qh * kD + dim] = run_o[h];
                    if (dim == 0) *reinterpret_cast<float2*>(wsml + qh * 2) = make_float2(mref[h], run_l[h]);
                }
                named_sync(bar_id, kGroup);
                if (stid == 0) {  // the release after the barrier publishes the whole group's writes
                    const uint32_t prev = atom_add_acq_rel(&a.ws_cnt[seq], (uint32_t)run_n);
                    flags[s] = (prev + (uint32_t)run_n == (uint32_t)nchunks) ? 1 : 0;
                }
                named_sync(bar_id, kGroup);
                if (flags[s]) {  // the last run to finish merges all of them
                    combine_runs(a, seq, pref[seq], nchunks, n_items, (int)gridDim.x, out, stid, kGroup, bar_id,
                                 reinterpret_cast<int*>(scr));
                    if (stid == 0) a.ws_cnt[seq] = 0u;
                }
            }
            run_n = 0;
#pragma unroll
            for (int h = 0; h < kHP; ++h) { mref[h] = -INFINITY; lsum[h] = 0.0f; }
#pragma unroll
            for (int i = 0; i < (V_MIN ? 16 : 1); ++i) pmv[i] = 0.0f;
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

}  // namespace dstream
}  // namespace cvattn
