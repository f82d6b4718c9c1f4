// flash_pipe.cuh -- persistent tcgen05 flash attention with two query tiles
// per CTA for the multi-query paths: Qwen2 causal prefill
// (src/cosyvoice-llm.cpp:62 with the mask of :20-29 / :101-108) and DiT
// attention, cached (src/cosyvoice-graph.cpp:363-366) or uncached (:373-377),
// with the streaming chunk mask of src/cosyvoice-token2wav.cpp:285-298 and an
// explicit f16 mask.  Same semantics, parameters and numerics as
// flash_tc.cuh (ggml_flash_attn_ext, scale 1/sqrt(D), f16 operands, fp32
// accumulation, softmax statistics and output).
//
// One CTA per SM walks work items.  An item is a pair of 128-row query tiles
// that read the same K/V: two query heads of one KV group (G >= 2), or two
// consecutive query tiles of one head (G = 1).  Every K/V tile (64 keys) is
// loaded once for both.
//   warps 0-3   softmax group 0 (query tile 0), thread = row = TMEM lane
//   warps 4-7   softmax group 1 (query tile 1)
//   warps 8-11  producer: K/V tiles of any ggml type -> f16 128B-swizzled
//               shared memory (6 stages); an f16 cache uses TMA tensor loads
//   warps 12-13 MMA issuers, one per query tile x: S_x = Q_x K^T into TMEM
//               (M128 N64 K64); P_x is written to TMEM by its softmax group as
//               f16 and feeds O_x += P_x V directly from TMEM (M128 N64 K64).
//               (One thread issues an MMA in ~30 ns, so the two tiles get an
//               issuer each.)
// TMEM (512 columns): per group x two S buffers (64 columns each), two P
// buffers (32 each) and O (64).  Tile T of a group uses buffer T & 1, so the
// MMA computes S(T+1) while the softmax works on S(T) and O(T-1) reads the
// other P buffer: the softmax never waits for an MMA round trip.  The softmax
// keeps a reference max per row and rescales O in TMEM only when a tile
// raises it by more than 2^8 (so P <= 256 stays exact in f16).  Fully masked
// key tiles are never loaded.
#pragma once

#include "decode_tc.cuh"
#include "flash_tc.cuh"

namespace cvattn {
namespace fp {

using fa::BM;
using fa::D;
using fa::Params;

constexpr int kBN = 64;  // keys per tile
constexpr int kStages = 6;
// The kernel's shape for H softmax warpgroups per query tile (1 or 2).  With 2
// (the default), warps w and w + 4 of a query tile share TMEM lane quarter w and
// take 32 of the tile's 64 key columns each: twice the independent softmax
// chains per sub-partition, at the cost of one vote per tile between the two
// halves of a row.  It pays where items are short (DiT: ~12 key tiles per query
// tile, with Q loads and epilogues between them) and breaks even on long
// causal prefill.
template <int H>
struct Shape {
    static_assert(H == 1 || H == 2, "one or two softmax warpgroups per query tile");
    static constexpr int kSoftWarps = 8 * H;      // softmax warps of both query tiles
    static constexpr int kSoftThreads = 128 * H;  // softmax threads of one query tile
    static constexpr int kChunks = kBN / 32 / H;  // 32-column chunks of a tile per softmax thread
    static constexpr int kProdWarp0 = kSoftWarps;
    static constexpr int kMmaWarp = kSoftWarps + 4;  // MMA issuer of query tile 0 / 1
    static constexpr int kThreads = (kMmaWarp + 2) * 32;
};
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kSCol = 0, kPCol = 256, kOCol = 384;  // S: x*128 + b*64, P: 256 + x*64 + b*32, O: 384 + x*64
constexpr float kRescaleThreshold = 8.0f;
// The optimistic pass of a tile is redone against the tile's own max when a thread's sum of P
// over its columns exceeds kRedoSum (some P > 2^7: the row's max rose by more than 7 since
// the reference was set); without a redo every P <= kRedoSum, far inside f16.  (Starting
// the prefix masks' rows from the reference max 0, so that the first tile needs no redo,
// measured slower: causal prefill 462 -> 444 TFLOP/s, DiT 292 -> 289.)
constexpr float kRedoSum = 4096.0f;
#ifndef CVATTN_FLASH_EXP_POLY
#define CVATTN_FLASH_EXP_POLY 0
#endif
constexpr bool kExpPoly = CVATTN_FLASH_EXP_POLY != 0;  // part of the exponentials on the FMA pipe


// shared memory (offsets from a 1024-aligned base)
constexpr int kTileBytes = kBN * D * 2;              // 8 KB
constexpr int kQOff = 0;                             // 2 x 16 KB
constexpr int kKOff = 32 * 1024;                     // kStages x 8 KB
constexpr int kVOff = kKOff + kStages * kTileBytes;  // kStages x 8 KB
constexpr int kBarOff = kVOff + kStages * kTileBytes;  // 128 KB
constexpr int kXchOff = kBarOff + 512;               // row statistics the two column halves exchange
constexpr int kXchBytes = 2048 * 4;
constexpr int kSmemBytes = kXchOff + kXchBytes;      // one CTA per SM (TMEM: 512 columns)
constexpr int kRawOff = kSmemBytes;                  // staged producer: raw rows of two tiles

__host__ __device__ constexpr bool is_block_quant(int t) {
    return t == kQ4_0 || t == kQ4_1 || t == kQ5_0 || t == kQ5_1 || t == kQ8_0;
}
// Width in bytes of the TMA box that holds one raw head row of type t (staged
// producer, TMA form): the row starts 4-byte aligned, the box at the 16-byte
// boundary at or below it, so it spans the row plus up to 12 leading bytes.
__host__ __device__ constexpr int raw_box_bytes(int t) {
    return (2 * group_bytes(t) + ((2 * group_bytes(t)) % 16 ? 12 : 0) + 15) / 16 * 16;
}
// Bytes of the raw K and V head rows of one 64-key tile (staged producer): the
// larger of the packed cp.async layout and the TMA box layout.
__host__ __device__ constexpr int raw_tile_bytes(int kt, int vt) {
    return kBN * (raw_box_bytes(kt) + raw_box_bytes(vt));
}
// Dynamic shared memory of flash_pipe_kernel<KT, VT>.
__host__ __device__ constexpr int smem_bytes(int kt, int vt) {
    return (is_block_quant(kt) && is_block_quant(vt)) ? kRawOff + 2 * raw_tile_bytes(kt, vt) : kSmemBytes;
}

struct Bars {
    uint64_t kv_full[kStages];
    uint64_t kv_empty[kStages];
    uint64_t q_full[2];
    uint64_t s_full[2][2];   // [group][buffer]
    uint64_t p_ready[2][2];
    uint64_t o_done[2][2];   // O(T) commits o_done[x][T & 1]
    uint64_t o_free[2];
    uint64_t raw_full[2];    // staged producer, TMA form: raw tile n landed in buffer n & 1
    uint32_t tmem_base;
    int err;
};

// Bounded wait shared by the roles: gives up after kWaitBudgetNs or once another
// role has flagged an error, so every thread reaches teardown.
__device__ __forceinline__ bool wait_or_err(uint64_t* bar, uint32_t parity, int* err, int* status, int site) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (;;) {
        if (mbar_try_wait_hint(bar, parity, 1000u)) return true;
        if (*reinterpret_cast<volatile int*>(err)) return false;
        if (global_timer_ns() - t0 > kWaitBudgetNs) {
            record_status(status, kStatusTimeout | (site << 8));
            *reinterpret_cast<volatile int*>(err) = 1;
            return false;
        }
    }
}

// A work item: batch entry, KV head, and per query tile x its head and row
// tile (active[x] = 0 when the pair has only one tile).
struct Item {
    int b, g;
    int h[2], qt[2];
    bool active[2];
};

// Pairing: for an even G, two query heads of one KV group at the same query
// tile; for G = 1 and odd G, two consecutive query tiles of one head (an odd G
// paired by heads would leave one item in (G + 1) / 2 half empty: 1 in 4 for
// Qwen2's G = 7).  Items are ordered longest first (query tile index
// descending) so the causal / chunk-masked tail finishes together; for G = 1 the
// pairs of one head stay adjacent instead (they read the same K/V).
__device__ __forceinline__ bool heads_paired(const Params& p) { return p.G >= 2 && (p.G & 1) == 0; }

__device__ __forceinline__ Item item_at(const Params& p, int idx) {
    Item it;
    const int n_qt = (p.n_q + BM - 1) / BM;
    const int Hkv = p.Hq / p.G;
    if (!heads_paired(p) && p.G >= 3) {
        // consecutive query tiles of one head; pairs longest first, every head at a pair index
        // next to each other, so the G heads of a KV group share its K/V through L2
        const int qpairs = (n_qt + 1) / 2;
        const int per_qp = p.batch * p.Hq;
        const int qp = qpairs - 1 - idx / per_qp;
        const int r = idx % per_qp;
        it.h[0] = it.h[1] = r % p.Hq;
        it.g = it.h[0] / p.G;
        it.b = r / p.Hq;
        it.qt[0] = 2 * qp;
        it.qt[1] = 2 * qp + 1;
        it.active[0] = true;
        it.active[1] = it.qt[1] < n_qt;
        return it;
    }
    if (p.G >= 2) {
        const int pairs = (p.G + 1) / 2;
        const int per_qt = p.batch * Hkv * pairs;
        const int qt = n_qt - 1 - idx / per_qt;
        int r = idx % per_qt;
        const int pi = r % pairs; r /= pairs;
        it.g = r % Hkv;
        it.b = r / Hkv;
        it.h[0] = it.g * p.G + 2 * pi;
        it.h[1] = it.h[0] + 1;
        it.active[0] = true;
        it.active[1] = 2 * pi + 1 < p.G;
        it.qt[0] = it.qt[1] = qt;
    } else {
        // the query-tile pairs of one head are neighbours, so the CTAs that run them at
        // the same time share that head's K/V through L2
        const int qpairs = (n_qt + 1) / 2;
        const int qp = qpairs - 1 - idx % qpairs;
        const int r = idx / qpairs;
        it.h[0] = it.h[1] = r % p.Hq;
        it.g = it.h[0];
        it.b = r / p.Hq;
        it.qt[0] = 2 * qp;
        it.qt[1] = 2 * qp + 1;
        it.active[0] = true;
        it.active[1] = it.qt[1] < n_qt;
    }
    return it;
}

__device__ __forceinline__ int n_items(const Params& p) {
    const int n_qt = (p.n_q + BM - 1) / BM;
    const int Hkv = p.Hq / p.G;
    if (heads_paired(p)) return n_qt * p.batch * Hkv * ((p.G + 1) / 2);
    return ((n_qt + 1) / 2) * p.batch * p.Hq;
}

// Key tiles query tile qt needs (0 for an inactive tile).
__device__ __forceinline__ int tiles_of(const Params& p, bool active, int qt) {
    if (!active) return 0;
    return (fa::key_limit(p, qt * BM) + kBN - 1) / kBN;
}

// 2^x for a pair on the FMA pipe (offloads the MUFU, which caps D = 64
// attention): Cody-Waite reduction x = n + f with n = round(x) (adding
// 1.5 * 2^23 rounds to an integer in the low mantissa bits), f in [-1/2, 1/2];
// 2^f by a degree-4 polynomial fitted here (least squares on the relative
// error over Chebyshev nodes, Lawson-reweighted toward minimax: max relative
// error 2.7e-6 in fp32, far below the f16 rounding P receives); 2^n added
// into the exponent field.  x is clamped to [-126, 127] so the exponent
// arithmetic stays in range (2^-126 rounds to 0 in f16).
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
    x.x = fminf(fmaxf(x.x, -126.0f), 127.0f);
    x.y = fminf(fmaxf(x.y, -126.0f), 127.0f);
    const float2 one = make_float2(1.0f, 1.0f), magic = make_float2(12582912.0f, 12582912.0f);
    const float2 t = ffma2(x, one, magic);
    const float2 r = ffma2(t, one, make_float2(-12582912.0f, -12582912.0f));
    const float2 f = ffma2(r, make_float2(-1.0f, -1.0f), x);
    float2 q = make_float2(0.009570101276040077f, 0.009570101276040077f);
    q = ffma2(q, f, make_float2(0.05591785907745361f, 0.05591785907745361f));
    q = ffma2(q, f, make_float2(0.240247443318367f, 0.240247443318367f));
    q = ffma2(q, f, make_float2(0.6931217908859253f, 0.6931217908859253f));
    q = ffma2(q, f, make_float2(0.9999992847442627f, 0.9999992847442627f));
    const int n0 = __float_as_int(t.x) - 0x4B400000, n1 = __float_as_int(t.y) - 0x4B400000;
    return make_float2(__int_as_float(__float_as_int(q.x) + (n0 << 23)), __int_as_float(__float_as_int(q.y) + (n1 << 23)));
}

// The mask of one softmax row.  The causal and chunk masks (and n_kv) are a
// prefix of the keys: key j is visible iff j < lim (causal: j <= causal_offset
// + i, src/cosyvoice-llm.cpp:20-29; chunk: j < key_offset or j - key_offset <
// the row's block end, src/cosyvoice-token2wav.cpp:285-298, i.e. j <
// key_offset + block end).  An explicit f16 mask adds mrow[j] (times log2 e)
// to the visible keys j < lim = n_kv.  A chunk of 32 columns whose keys all lie
// below wlim, the smallest lim of the warp's 32 rows, needs no mask, and one
// that starts at or past wmax, the largest, has no visible entry (warp-uniform
// tests).
struct RowMask {
    int lim;
    int wlim;
    int wmax;               // the largest lim of the warp's rows: chunks at or past it are fully masked
    bool explicit_mask;     // uniform over the CTA
    const uint16_t* mrow;   // explicit mask row (read only below lim)
};

// Scores of the 32 columns of a chunk whose first key is jc: log2 units, -inf
// past the row's limit (plus the explicit mask).
__device__ __forceinline__ void mask_chunk(const uint32_t (&sv)[32], int jc, const RowMask& rm, float (&sc)[32]) {
    const int rem = rm.lim - jc;  // columns e < rem are visible
    if (rm.explicit_mask) {
#pragma unroll
        for (int e = 0; e < 32; ++e)
            sc[e] = e < rem ? __uint_as_float(sv[e]) + h2f(rm.mrow[jc + e]) * 1.4426950408889634f : -INFINITY;
    } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) sc[e] = e < rem ? __uint_as_float(sv[e]) : -INFINITY;
    }
}

__device__ __forceinline__ bool chunk_unmasked(int jc, const RowMask& rm) {
    return !rm.explicit_mask && jc + 32 <= rm.wlim;
}

// Row max of this thread's kChunks x 32 columns of an S tile (key j0 onward), 4 independent chains.
template <int kChunks>
__device__ __forceinline__ void max_pass(uint32_t s_taddr, int j0, const RowMask& rm, float& mt) {
    float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
    for (int c = 0; c < kChunks; ++c) {
        const int jc = j0 + 32 * c;
        if (jc >= rm.wmax) continue;  // no visible entry in the warp's rows (warp-uniform)
        uint32_t sv[32];
        tc::tmem_ld32(s_taddr + 32 * c, sv);
        tc::tmem_ld_wait();
        if (chunk_unmasked(jc, rm)) {
#pragma unroll
            for (int e = 0; e < 32; ++e) m4[e & 3] = fmaxf(m4[e & 3], __uint_as_float(sv[e]));
        } else {
            float sc[32];
            mask_chunk(sv, jc, rm, sc);
#pragma unroll
            for (int e = 0; e < 32; ++e) m4[e & 3] = fmaxf(m4[e & 3], sc[e]);
        }
    }
    mt = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
}

// P = 2^(s - mu) of 32 scores (f16 pairs into pw), with the running sum (two
// chains).  kPoly: one pair in four is exponentiated on the FMA pipe.
template <bool kPoly>
__device__ __forceinline__ void exp_chunk(const float (&sc)[32], float mu, float2 (&acc)[2], uint32_t (&pw)[16]) {
    const float2 neg_mu = make_float2(-mu, -mu), one = make_float2(1.0f, 1.0f);
#pragma unroll
    for (int e = 0; e < 32; e += 2) {
        const float2 xx = ffma2(make_float2(sc[e], sc[e + 1]), one, neg_mu);
        const float2 pp = (kPoly && ((e >> 1) & 3) == 3) ? exp2_poly2(xx) : make_float2(fast_exp2(xx.x), fast_exp2(xx.y));
        acc[(e >> 1) & 1] = ffma2(pp, one, acc[(e >> 1) & 1]);
        pw[e / 2] = tc::pack_f16x2(pp.x, pp.y);
    }
}

// P = 2^(s - mu) of this thread's columns of one S tile into the tile's TMEM P
// columns; returns their sum.  Chunks with no masked entry in the warp's rows skip
// the mask; chunks with no visible entry in the warp's rows write zeros without
// reading S.  (Double-buffering the four TMEM loads measured slower: the larger
// unrolled body costs more than the load latency it hides.)
template <int kChunks>
__device__ __forceinline__ float exp_pass(uint32_t s_taddr, uint32_t p_taddr, float mu, int j0, const RowMask& rm) {
    float2 acc[2] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f)};
    for (int c = 0; c < kChunks; ++c) {
        uint32_t pw[16];
        const int jc = j0 + 32 * c;
        if (jc >= rm.wmax) {  // warp-uniform
#pragma unroll
            for (int i = 0; i < 16; ++i) pw[i] = 0u;
        } else {
            uint32_t sv[32];
            tc::tmem_ld32(s_taddr + 32 * c, sv);
            tc::tmem_ld_wait();
            float sc[32];
            if (chunk_unmasked(jc, rm)) {
#pragma unroll
                for (int e = 0; e < 32; ++e) sc[e] = __uint_as_float(sv[e]);
                exp_chunk<kExpPoly>(sc, mu, acc, pw);
            } else {
                mask_chunk(sv, jc, rm, sc);
                exp_chunk<false>(sc, mu, acc, pw);
            }
        }
        tc::tmem_st16(p_taddr + 16 * c, pw);
    }
    return (acc[0].x + acc[0].y) + (acc[1].x + acc[1].y);
}


// ------------------------------------------------- staged producer (quantized K/V)
//
// The 128 producer threads copy a tile's raw K and V head rows into shared
// memory with coalesced 4-byte cp.async (one tile ahead, two raw buffers), then
// convert them there: thread r takes row r & 63 and block r >> 6 of K, then of
// V (the block is uniform per warp), builds the block's 32 quants as exact f16
// integers (centred for the 4/5-bit types) and scales them in f16 with one
// rounding (hmul2, or hfma2 with the centred min), i.e. the same f16 value the
// dequantize-then-round path gives for the _0 types.

__device__ __forceinline__ void prod_bar(int id, int n) { asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(n) : "memory"); }

__device__ __forceinline__ bool prod_bar_and(int id, int n, bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r) : "r"((uint32_t)v), "r"(id), "r"(n) : "memory");
    return r != 0;
}

// Number of the n threads at barrier `id` whose v is true (bar.red.popc).
__device__ __forceinline__ int prod_bar_count(int id, int n, bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.popc.u32 %0, %2, %3, p;\n\t}"
        : "=r"(r) : "r"((uint32_t)v), "r"(id), "r"(n) : "memory");
    return (int)r;
}

__device__ __forceinline__ void cp_async4(void* smem_dst, const void* gmem_src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" :: "r"(smem_addr(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" :: "n"(N) : "memory"); }

// Block `blk` of raw head row g (2-byte aligned in shared memory) -> f16 chunks
// blk * 4 .. blk * 4 + 3 of row `row` of a 128B-swizzled tile; zeros past n_kv.
template <int T>
__device__ __forceinline__ void convert_block_f16(const uint8_t* g, bool valid, uint8_t* tile, int row, int blk) {
    uint32_t w[16];
    if (valid) {
        float d, m;
        dtc::convert_group<T>(g, w, d, m);
        const __half2 d2 = __float2half2_rn(d);
        if constexpr (BlockTraits<T>::HAS_MIN) {
            const __half2 m2 = __float2half2_rn(m);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const __half2 x = __hfma2(*reinterpret_cast<const __half2*>(&w[i]), d2, m2);
                w[i] = *reinterpret_cast<const uint32_t*>(&x);
            }
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const __half2 x = __hmul2(*reinterpret_cast<const __half2*>(&w[i]), d2);
                w[i] = *reinterpret_cast<const uint32_t*>(&x);
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) w[i] = 0u;
    }
#pragma unroll
    for (int c = 0; c < 4; ++c)
        *reinterpret_cast<uint4*>(tile + tc::sw128_offset(row, blk * 4 + c)) =
            make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
}

// Forms of the staged producer (Params::staged).
constexpr int kStagedCpAsync = 1;  // 4-byte cp.async of each head row by all 128 threads
constexpr int kStagedBoxes = 2;    // rows 16-byte aligned: TMA byte boxes around the head's row
constexpr int kStagedChunk = 3;    // contiguous rows: one bulk copy of the tile's whole rows
// Largest raw tile of the chunk form (whole K and V rows of 64 keys).
constexpr int kChunkRawMax = 44 * 1024;

// The producer role for block-quantized K and V (128 threads, r = 0..127).
// Tiles are produced in the order the MMA issuers consume them, one raw tile
// ahead in two raw buffers.  The raw rows arrive in one of three forms:
//   kStagedCpAsync: coalesced 4-byte cp.async of the head rows by all 128 threads;
//   kStagedBoxes:   two TMA tensor loads by one thread (byte maps, boxes of
//                   raw_box_bytes x 64 rows from the 16-byte boundary below the head);
//   kStagedChunk:   the tile's 64 rows are contiguous in memory, so one thread
//                   copies them whole (all KV heads) with cp.async.bulk, and the
//                   last <= 12 bytes of a ragged tile with 4-byte cp.async.
template <int KT, int VT, int kForm>
__device__ __forceinline__ void produce_staged(const Params& p, uint8_t* smem, Bars* B, int total, int r,
                                               const CUtensorMap* kmap, const CUtensorMap* vmap) {
    constexpr int HBK = 2 * group_bytes(KT), HBV = 2 * group_bytes(VT);  // bytes of one head row
    constexpr int WK = HBK / 4, WV = HBV / 4;
    constexpr bool kBoxes = kForm == kStagedBoxes, kChunk = kForm == kStagedChunk;
    // raw buffer size, K part size, and the row pitch of the raw tile in shared memory
    const int RB = kChunk ? p.raw_bytes : raw_tile_bytes(KT, VT);
    const int KB = kChunk ? p.raw_k_bytes : kBN * (kBoxes ? raw_box_bytes(KT) : HBK);
    const int PK = kChunk ? (int)p.k_nb1 : (kBoxes ? raw_box_bytes(KT) : HBK);
    const int PV = kChunk ? (int)p.v_nb1 : (kBoxes ? raw_box_bytes(VT) : HBV);
    constexpr int kBar = 1;  // named barrier of the 128 producer threads
    uint8_t* raw0 = smem + kRawOff;
    // tile cursor: item idx (its batch entry, KV head and key-tile count) and tile j;
    // item_at / tiles_of run once per item, not once per tile
    struct Cursor {
        int idx, j, nt, b, g;
    };
    auto find_item = [&](Cursor& c) -> bool {  // the first item at or after c.idx with a key tile
        while (c.idx < total) {
            const Item it = item_at(p, c.idx);
            c.nt = max(tiles_of(p, it.active[0], it.qt[0]), tiles_of(p, it.active[1], it.qt[1]));
            if (c.nt > 0) {
                c.b = it.b;
                c.g = it.g;
                c.j = 0;
                return true;
            }
            c.idx += gridDim.x;
        }
        return false;
    };
    auto advance = [&](Cursor& c) -> bool {
        if (++c.j < c.nt) return true;
        c.idx += gridDim.x;
        return find_item(c);
    };
    auto issue = [&](const Cursor& c, uint8_t* dst, int buf) {
        const int rows = min(kBN, p.n_kv - c.j * kBN);
        if constexpr (kBoxes) {
            if (r == 0) {
                mbar_arrive_expect_tx(&B->raw_full[buf], (uint32_t)RB);
                tc::tma_load_3d(dst, kmap, (c.g * HBK) & ~15, c.j * kBN, c.b, &B->raw_full[buf]);
                tc::tma_load_3d(dst + KB, vmap, (c.g * HBV) & ~15, c.j * kBN, c.b, &B->raw_full[buf]);
            }
        } else if constexpr (kChunk) {
            if (r == 0) {
                const uint8_t* ks = p.k + (int64_t)c.b * p.k_nb2 + (int64_t)c.j * kBN * p.k_nb1;
                const uint8_t* vs = p.v + (int64_t)c.b * p.v_nb2 + (int64_t)c.j * kBN * p.v_nb1;
                const uint32_t kbytes = (uint32_t)rows * (uint32_t)p.k_nb1, vbytes = (uint32_t)rows * (uint32_t)p.v_nb1;
                const uint32_t kb16 = kbytes & ~15u, vb16 = vbytes & ~15u;
                mbar_arrive_expect_tx(&B->raw_full[buf], kb16 + vb16);
                bulk_g2s(dst, ks, kb16, &B->raw_full[buf]);
                bulk_g2s(dst + KB, vs, vb16, &B->raw_full[buf]);
                for (uint32_t o = kb16; o < kbytes; o += 4) cp_async4(dst + o, ks + o);
                for (uint32_t o = vb16; o < vbytes; o += 4) cp_async4(dst + KB + o, vs + o);
            }
            cp_async_commit();
        } else {
            const uint8_t* kb = p.k + (int64_t)c.b * p.k_nb2 + (int64_t)c.g * HBK + (int64_t)c.j * kBN * p.k_nb1;
            const uint8_t* vb = p.v + (int64_t)c.b * p.v_nb2 + (int64_t)c.g * HBV + (int64_t)c.j * kBN * p.v_nb1;
#pragma unroll 4
            for (int w = r; w < kBN * WK; w += 128) {
                const int row = w / WK, wi = w - row * WK;
                if (row < rows) cp_async4(dst + row * HBK + 4 * wi, kb + (int64_t)row * p.k_nb1 + 4 * wi);
            }
            uint8_t* vdst = dst + kBN * HBK;
#pragma unroll 4
            for (int w = r; w < kBN * WV; w += 128) {
                const int row = w / WV, wi = w - row * WV;
                if (row < rows) cp_async4(vdst + row * HBV + 4 * wi, vb + (int64_t)row * p.v_nb1 + 4 * wi);
            }
            cp_async_commit();
        }
    };
    if constexpr (kBoxes) {
        if (r == 0) {
            tc::prefetch_tmap(kmap);
            tc::prefetch_tmap(vmap);
        }
    }
    constexpr bool kMbar = kBoxes || kChunk;  // raw tiles land on raw_full[buf]
    uint32_t issued = 0, landed = 0;          // raw_full forms: tiles issued / seen landed (thread 0's count)
    Cursor cur{(int)blockIdx.x, 0, 0, 0, 0};
    bool have = find_item(cur);
    if (have) {
        issue(cur, raw0, 0);
        ++issued;
    }
    const int row = r & (kBN - 1), blk = r >> 6;
    for (uint32_t n = 0; have; ++n) {
        Cursor nxt = cur;
        const bool have2 = advance(nxt);
        prod_bar(kBar, 128);  // tile n - 1 is converted: its raw buffer takes tile n + 1
        bool ok = true;
        if (have2) {
            if (kMbar && r == 0) fence_proxy_async_smem();  // the generic reads of tile n - 1 precede the async writes
            issue(nxt, raw0 + ((n + 1) & 1) * RB, (int)((n + 1) & 1));
            ++issued;
        }
        if constexpr (kMbar) {
            ok = wait_or_err(&B->raw_full[n & 1], (n >> 1) & 1, &B->err, p.status, 14);
            if (ok) ++landed;
        }
        if constexpr (!kBoxes) {  // this thread's cp.async of tile n (the chunk form's tail)
            if (have2) cp_async_wait<1>();
            else cp_async_wait<0>();
        }
        const int s = n % kStages;
        const uint32_t use = n / kStages;
        ok = ok && (use == 0 || wait_or_err(&B->kv_empty[s], (use - 1) & 1, &B->err, p.status, 5));
        // every thread's copies of tile n have landed and stage s is free (or all stop together)
        if (!prod_bar_and(kBar, 128, ok)) break;
        const uint8_t* raw = raw0 + (n & 1) * RB;
        const bool valid = cur.j * kBN + row < p.n_kv;
        // the head's first byte in a raw row
        const int hk = kChunk ? cur.g * HBK : (kBoxes ? ((cur.g * HBK) & 15) : 0);
        const int hv = kChunk ? cur.g * HBV : (kBoxes ? ((cur.g * HBV) & 15) : 0);
        convert_block_f16<KT>(raw + row * PK + hk + blk * group_bytes(KT), valid, smem + kKOff + s * kTileBytes, row,
                              blk);
        convert_block_f16<VT>(raw + KB + row * PV + hv + blk * group_bytes(VT), valid,
                              smem + kVOff + s * kTileBytes, row, blk);
        fence_proxy_async_smem();
        mbar_arrive(&B->kv_full[s]);
        cur = nxt;
        have = have2;
    }
    if constexpr (kMbar) {
        // no async write into shared memory outlives the CTA: thread 0 waits (bounded) for the
        // tiles it issued that were not seen landing (at most two, in different buffers)
        if (r == 0) {
            for (uint32_t t = landed; t < issued; ++t) {
                const uint64_t t0 = global_timer_ns();
                while (!mbar_try_wait_hint(&B->raw_full[t & 1], (t >> 1) & 1, 1000u))
                    if (global_timer_ns() - t0 > kWaitBudgetNs) break;
            }
        }
    }
    if constexpr (!kBoxes) cp_async_wait<0>();  // no copy into shared memory outlives the CTA
}

template <int KT, int VT, int H>
__global__ void __launch_bounds__(Shape<H>::kThreads, 1)
    flash_pipe_kernel(const __grid_constant__ Params p, const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap) {
    constexpr int kHalves = H, kSoftWarps = Shape<H>::kSoftWarps, kSoftThreads = Shape<H>::kSoftThreads;
    constexpr int kChunks = Shape<H>::kChunks, kProdWarp0 = Shape<H>::kProdWarp0, kMmaWarp = Shape<H>::kMmaWarp;
    extern __shared__ __align__(1024) uint8_t smem[];
    Bars* B = reinterpret_cast<Bars*>(smem + kBarOff);
    if (smem_addr(smem) & 1023u) {
        if (threadIdx.x == 0) record_status(p.status, kStatusTimeout);
        return;
    }
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int total = n_items(p);

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&B->kv_full[s], p.use_tma ? 1 : 128);
            mbar_init(&B->kv_empty[s], 2);  // one arrival per MMA issuer
        }
        for (int x = 0; x < 2; ++x) {
            mbar_init(&B->q_full[x], kSoftThreads);
            mbar_init(&B->o_free[x], kSoftThreads);
            mbar_init(&B->raw_full[x], 1);
            for (int b = 0; b < 2; ++b) {
                mbar_init(&B->s_full[x][b], 1);
                mbar_init(&B->p_ready[x][b], kSoftThreads);
                mbar_init(&B->o_done[x][b], 1);
            }
        }
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

    if (warp < kSoftWarps) {
        // ====================================================== softmax of query tile x
        // warp = x * 4 * kHalves + hf * 4 + quad: rows quad * 32 .. + 31 (the warp's TMEM
        // lane quarter), key columns hf * 32 * kChunks .. + 32 * kChunks - 1 of each tile
        const int x = warp / (4 * kHalves);
        const int hf = (warp >> 2) & (kHalves - 1);
        const int quad = warp & 3;
        const int r = quad * 32 + lane;  // query row in the tile = TMEM lane
        const int col0 = hf * 32 * kChunks;
        const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
        const uint32_t s_tbase = tmem + lane_base + kSCol + x * 128 + col0;   // + buffer * 64
        const uint32_t p_tbase = tmem + lane_base + kPCol + x * 64 + col0 / 2;  // + buffer * 32
        const uint32_t o_taddr = tmem + lane_base + kOCol + x * 64 + col0;    // O columns = output dims
        uint8_t* qtile = smem + kQOff + x * 16384;
        // Row statistics the two halves of a row exchange (kHalves == 2): the tile max of a
        // redone tile and the row sum, each [half][row].  Every exchange is one bar.red.and
        // over the row's two warps, which also ANDs their `ok`, so both leave together;
        // consecutive exchanges never share a slot (a vote barrier separates two tile maxima).
        float* xch = reinterpret_cast<float*>(smem + kXchOff);
        float* x_mt = xch + 1024 + x * 256;   // [half][128]
        float* x_l = xch + 1536 + x * 256;    // [half][128]
        const int bar_pair = 2 + x * 4 + quad;
        auto exchange = [&](float* slots, float v, bool ok_in, float& other) -> bool {
            if constexpr (kHalves == 2) {
                slots[hf * 128 + r] = v;
                const bool all = prod_bar_and(bar_pair, 64, ok_in);
                other = slots[(hf ^ 1) * 128 + r];
                return all;
            } else {
                other = v;
                return ok_in;
            }
        };
        uint32_t T = 0;  // tiles of this group so far (all items): tile T uses buffer T & 1
        bool ok = true;
        for (int idx = blockIdx.x; ok && idx < total; idx += gridDim.x) {
            const Item it = item_at(p, idx);
            // (selects, not it.h[x]: x is not a compile-time index)
            if (!(x ? it.active[1] : it.active[0])) continue;
            const int qt = x ? it.qt[1] : it.qt[0];
            const int nt = tiles_of(p, true, qt);
            const int h = x ? it.h[1] : it.h[0], b = it.b;
            const int i0 = qt * BM, i = i0 + r;
            const bool row_ok = i < p.n_q;
            float* orow = p.out + (((int64_t)b * p.n_q + i) * p.Hq + h) * D + col0;
            if (nt == 0) {  // no visible key for any row of the tile: zero output
                if (row_ok) {
#pragma unroll
                    for (int c = 0; c < 16 / kHalves; ++c)
                        *reinterpret_cast<float4*>(orow + 4 * c) = make_float4(0.f, 0.f, 0.f, 0.f);
                }
                continue;
            }
            {   // this thread's dims of the Q row -> f16 (scaled into log2 units) swizzled; the
                // previous item's S MMAs are done
                const float* qrow = p.q + (int64_t)b * p.q_nb_batch + (int64_t)i * p.q_nb_tok + (int64_t)h * p.q_nb_head + col0;
                uint32_t w[32 / kHalves];
#pragma unroll
                for (int c = 0; c < 16 / kHalves; ++c) {
                    const float4 v = row_ok ? *reinterpret_cast<const float4*>(qrow + 4 * c) : make_float4(0.f, 0.f, 0.f, 0.f);
                    const float sc = p.scale_log2;
                    w[2 * c] = tc::pack_f16x2(v.x * sc, v.y * sc);
                    w[2 * c + 1] = tc::pack_f16x2(v.z * sc, v.w * sc);
                }
#pragma unroll
                for (int c = 0; c < 8 / kHalves; ++c)
                    *reinterpret_cast<uint4*>(qtile + tc::sw128_offset(r, col0 / 8 + c)) =
                        make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
                fence_proxy_async_smem();
                mbar_arrive(&B->q_full[x]);
            }
            RowMask rm;
            {
                rm.explicit_mask = p.mask_mode == CVATTN_MASK_EXPLICIT;
                rm.mrow = (rm.explicit_mask && row_ok) ? p.mask + (int64_t)b * p.mask_nb2 + (int64_t)i * p.mask_nb1
                                                      : p.mask;
                int lim = p.n_kv;
                if (p.mask_mode == CVATTN_MASK_CAUSAL) {
                    lim = min(lim, p.causal_offset + i + 1);
                } else if (p.mask_mode == CVATTN_MASK_CHUNK) {
                    const int be = fa::block_end(p, i + p.row_offset);
                    if (be != 0x7fffffff) lim = min(lim, p.key_offset + max(be, 0));
                }
                // A row past n_q is never written out: its scores (zero Q) stay unmasked so the
                // warp's other rows keep the unmasked path (with an explicit mask: nothing visible).
                rm.lim = row_ok ? lim : (rm.explicit_mask ? 0 : 0x7fffffff);
                rm.wlim = __reduce_min_sync(0xffffffffu, rm.lim);
                rm.wmax = __reduce_max_sync(0xffffffffu, rm.lim);
            }
            float m_ref = -INFINITY, l = 0.0f;  // the same m_ref in both halves of a row
            for (int jt = 0; jt < nt; ++jt, ++T) {
                const int buf = T & 1;
                const uint32_t s_taddr = s_tbase + buf * 64, p_taddr = p_tbase + buf * 32;
                const int j0 = jt * kBN + col0;
                ok = __all_sync(0xffffffffu, wait_or_err(&B->s_full[x][buf], (T >> 1) & 1, &B->err, p.status, 1));
                if (ok) tc::fence_after();
                if (ok && T >= 2) {  // P buffer `buf` is free once O(T-2) has read it
                    ok = __all_sync(0xffffffffu, wait_or_err(&B->o_done[x][buf], ((T - 2) >> 1) & 1, &B->err, p.status, 2));
                    if (ok) tc::fence_after();
                }
                // One pass against the running reference max: P = 2^(s - m_ref) and its sum.  Only
                // when a thread's sum exceeds kRedoSum (the row's max rose), and on a row's first
                // visible tile, is the tile redone against the tile's own max.
                float lt = 0.0f;
                if (ok && __any_sync(0xffffffffu, m_ref != -INFINITY))
                    lt = exp_pass<kChunks>(s_taddr, p_taddr, m_ref == -INFINITY ? 0.0f : m_ref, j0, rm);
                bool redo = m_ref == -INFINITY || !(lt <= kRedoSum);
                if constexpr (kHalves == 2) {
                    // one vote over the row's two warps: nothing to do (the common case), or some
                    // thread failed a wait or needs the tile redone -- then both halves redo every
                    // row (rows whose max did not rise keep their reference max, alpha = 1)
                    if (prod_bar_count(bar_pair, 64, !ok || redo) != 0) {
                        if (!prod_bar_and(bar_pair, 64, ok)) {
                            ok = false;
                            break;
                        }
                        redo = true;
                    }
                } else if (!ok) {
                    break;
                }
                if (__any_sync(0xffffffffu, redo)) {  // the same decision in both halves of a row
                    tc::tmem_st_wait();  // the optimistic P stores land before they are overwritten
                    float mt = -INFINITY, mt_other;
                    max_pass<kChunks>(s_taddr, j0, rm, mt);
                    exchange(x_mt, mt, true, mt_other);
                    mt = fmaxf(mt, mt_other);
                    float alpha = 1.0f;
                    if (mt > m_ref + kRescaleThreshold) {
                        alpha = (m_ref == -INFINITY) ? 0.0f : fast_exp2(m_ref - mt);
                        m_ref = mt;
                        l *= alpha;
                    }
                    if (jt > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
                        // O(T-1) (the other P buffer) accumulates with the old reference first
                        bool w_ok = __all_sync(0xffffffffu, wait_or_err(&B->o_done[x][buf ^ 1], ((T - 1) >> 1) & 1, &B->err, p.status, 11));
                        if constexpr (kHalves == 2) w_ok = prod_bar_and(bar_pair, 64, w_ok);  // both halves agree
                        if (!w_ok) {
                            ok = false;
                            break;
                        }
                        tc::fence_after();
                        for (int c = 0; c < kChunks; ++c) {  // this thread's O columns
                            uint32_t ov[32];
                            tc::tmem_ld32(o_taddr + 32 * c, ov);
                            tc::tmem_ld_wait();
#pragma unroll
                            for (int e = 0; e < 32; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
                            tc::tmem_st32(o_taddr + 32 * c, ov);
                        }
                    }
                    lt = exp_pass<kChunks>(s_taddr, p_taddr, m_ref == -INFINITY ? 0.0f : m_ref, j0, rm);
                }
                l += lt;
                tc::tmem_st_wait();
                tc::fence_before();
                mbar_arrive(&B->p_ready[x][buf]);
            }
            if (!ok) break;
            // epilogue: O_x of the item's last tile (T - 1) complete; the row sum of both halves
            ok = __all_sync(0xffffffffu, wait_or_err(&B->o_done[x][(T - 1) & 1], ((T - 1) >> 1) & 1, &B->err, p.status, 3));
            float l_other;
            if (!exchange(x_l, l, ok, l_other)) {
                ok = false;
                break;
            }
            if constexpr (kHalves == 2) l += l_other;
            tc::fence_after();
            float o[64 / kHalves];
            for (int c = 0; c < kChunks; ++c) {
                uint32_t ov[32];
                tc::tmem_ld32(o_taddr + 32 * c, ov);
                tc::tmem_ld_wait();
#pragma unroll
                for (int e = 0; e < 32; ++e) o[32 * c + e] = __uint_as_float(ov[e]);
            }
            tc::fence_before();
            mbar_arrive(&B->o_free[x]);
            if (row_ok) {
                const float inv = l > 0.0f ? 1.0f / l : 0.0f;
#pragma unroll
                for (int c = 0; c < 16 / kHalves; ++c)
                    *reinterpret_cast<float4*>(orow + 4 * c) =
                        make_float4(o[4 * c] * inv, o[4 * c + 1] * inv, o[4 * c + 2] * inv, o[4 * c + 3] * inv);
            }
        }
    } else if (warp < kMmaWarp) {
        // ====================================================== producer
        const int r = tid - kProdWarp0 * 32;  // 0..127 = key row of the tile
        if constexpr (is_block_quant(KT) && is_block_quant(VT)) {
            if (p.staged) {
                if (p.staged == kStagedBoxes) produce_staged<KT, VT, kStagedBoxes>(p, smem, B, total, r, &kmap, &vmap);
                else if (p.staged == kStagedChunk) produce_staged<KT, VT, kStagedChunk>(p, smem, B, total, r, &kmap, &vmap);
                else produce_staged<KT, VT, kStagedCpAsync>(p, smem, B, total, r, &kmap, &vmap);
                goto producer_done;
            }
        }
        {
        uint32_t n_kv_tiles = 0;
        for (int idx = blockIdx.x; idx < total; idx += gridDim.x) {
            const Item it = item_at(p, idx);
            const int nt = max(tiles_of(p, it.active[0], it.qt[0]), tiles_of(p, it.active[1], it.qt[1]));
            const int b = it.b, g = it.g;
            bool ok = true;
            for (int jt = 0; jt < nt; ++jt, ++n_kv_tiles) {
                const int s = n_kv_tiles % kStages;
                const uint32_t use = n_kv_tiles / kStages;
                if (p.use_tma) {
                    if (r == 0) {
                        if (use > 0 && !wait_or_err(&B->kv_empty[s], (use - 1) & 1, &B->err, p.status, 4)) {
                            ok = false;
                        } else {
                            mbar_arrive_expect_tx(&B->kv_full[s], 2 * kTileBytes);
                            tc::tma_load_3d(smem + kKOff + s * kTileBytes, &kmap, g * D, jt * kBN, b, &B->kv_full[s]);
                            tc::tma_load_3d(smem + kVOff + s * kTileBytes, &vmap, g * D, jt * kBN, b, &B->kv_full[s]);
                        }
                    }
                } else {
                    if (use > 0 && !wait_or_err(&B->kv_empty[s], (use - 1) & 1, &B->err, p.status, 5)) {
                        ok = false;
                    } else {
                        const uint8_t* kbase = p.k + (int64_t)b * p.k_nb2 + (int64_t)g * p.k_head_bytes;
                        const uint8_t* vbase = p.v + (int64_t)b * p.v_nb2 + (int64_t)g * p.v_head_bytes;
                        // threads 0-63 convert the tile's K rows, 64-127 its V rows
                        const int row = r & (kBN - 1);
                        const int key = jt * kBN + row;
                        const bool valid = key < p.n_kv;
                        if (r < kBN) fa::store_row_f16<KT>(kbase + (int64_t)key * p.k_nb1, valid, smem + kKOff + s * kTileBytes, row);
                        else fa::store_row_f16<VT>(vbase + (int64_t)key * p.v_nb1, valid, smem + kVOff + s * kTileBytes, row);
                        fence_proxy_async_smem();
                        mbar_arrive(&B->kv_full[s]);
                    }
                }
                if (p.use_tma ? (r == 0 && !ok) : !__all_sync(0xffffffffu, ok)) break;
            }
            if (!ok || *reinterpret_cast<volatile int*>(&B->err)) break;
        }
        }
    producer_done:;
    } else if (warp >= kMmaWarp && lane == 0) {
        // ====================================================== MMA issuer of query tile x
        const int x = warp - kMmaWarp;
        const uint32_t idesc_s = tc::idesc_f16_f32(128, kBN, false);
        const uint32_t idesc_o = tc::idesc_f16_f32(128, 64, true);
        const uint32_t sq = smem_addr(smem + kQOff + x * 16384);
        uint32_t n_kv_tiles = 0;
        uint32_t Ts = 0, To = 0;  // S / O issued (all items): buffers Ts & 1, To & 1
        uint32_t n_q = 0, n_items_x = 0;
        bool ok = true;
        auto issue_s = [&](int stage) {
            const uint32_t buf = Ts & 1;
            const uint32_t kaddr = smem_addr(smem + kKOff + stage * kTileBytes);
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
                const uint64_t a = tc::sdesc_sw128(sq + kk * 32, 16, 1024);
                const uint64_t bb = tc::sdesc_sw128(kaddr + kk * 32, 16, 1024);
                tc::mma_ss(tmem + kSCol + x * 128 + buf * 64, a, bb, idesc_s, kk > 0 ? 1u : 0u);
            }
            tc::mma_commit(&B->s_full[x][buf]);
            ++Ts;
        };
        auto issue_o = [&](int stage, bool first) {
            const uint32_t buf = To & 1;
            const uint32_t vaddr = smem_addr(smem + kVOff + stage * kTileBytes);
#pragma unroll
            for (int kk = 0; kk < kBN / 16; ++kk) {
                const uint64_t bb = tc::sdesc_sw128(vaddr + kk * 2048, 16, 1024);
                tc::mma_ts(tmem + kOCol + x * 64, tmem + kPCol + x * 64 + buf * 32 + kk * 8, bb, idesc_o,
                           (!first || kk > 0) ? 1u : 0u);
            }
            tc::mma_commit(&B->o_done[x][buf]);
            ++To;
        };
        auto kv_wait = [&](uint32_t u, int site) {
            const bool r = wait_or_err(&B->kv_full[u % kStages], (u / kStages) & 1, &B->err, p.status, site);
            if (r) tc::fence_after();
            return r;
        };
        for (int idx = blockIdx.x; ok && idx < total; idx += gridDim.x) {
            const Item it = item_at(p, idx);
            const int n0 = tiles_of(p, it.active[0], it.qt[0]), n1 = tiles_of(p, it.active[1], it.qt[1]);
            const int mine = x ? n1 : n0;
            const int nt = max(n0, n1);
            const uint32_t base = n_kv_tiles;
            if (mine > 0) {
                // S(0), S(1): the two S buffers run ahead of the softmax
                ok = kv_wait(base, 7) && wait_or_err(&B->q_full[x], n_q & 1, &B->err, p.status, 6);
                ++n_q;
                if (ok) {
                    tc::fence_after();
                    issue_s((int)(base % kStages));
                }
                if (ok && mine > 1) {
                    ok = kv_wait(base + 1, 10);
                    if (ok) issue_s((int)((base + 1) % kStages));
                }
            }
            for (int jt = 0; ok && jt < nt; ++jt) {
                const int s = (int)((base + jt) % kStages);
                if (jt >= mine) {
                    // this tile's K/V is not read by query tile x; arrive only once the tile has
                    // landed, so this issuer never arrives twice on a stage in one phase
                    ok = kv_wait(base + jt, 13);
                    if (!ok) break;
                    mbar_arrive(&B->kv_empty[s]);
                    continue;
                }
                // O_x(jt) once P_x(jt) is in TMEM (and, for the item's first O, once the
                // previous item's epilogue has read O_x)
                ok = wait_or_err(&B->p_ready[x][To & 1], (To >> 1) & 1, &B->err, p.status, 8);
                if (ok && jt == 0 && n_items_x > 0)
                    ok = wait_or_err(&B->o_free[x], (n_items_x - 1) & 1, &B->err, p.status, 9);
                if (!ok) break;
                tc::fence_after();
                issue_o(s, jt == 0);
                if (jt + 2 < mine) {  // S_x(jt+2) into the buffer the softmax just released
                    ok = kv_wait(base + jt + 2, 12);
                    if (!ok) break;
                    issue_s((int)((base + jt + 2) % kStages));
                }
                tc::mma_commit(&B->kv_empty[s]);  // this issuer is done with stage s once its MMAs complete
            }
            n_kv_tiles += nt;
            if (mine > 0) ++n_items_x;
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

}  // namespace fp
}  // namespace cvattn
