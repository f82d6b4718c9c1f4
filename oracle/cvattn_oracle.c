/*
 * cvattn_oracle.c -- CPU restatement of the cosyvoice.cpp attention path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA engine in
 * cosyvoice.cpp_b200/csrc.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py load it.  The product
 * library (libcvattn.so) never links, calls or falls back to it.
 *
 * What it restates (reference paths are relative to the cosyvoice.cpp tree):
 *   - KV block codecs used by ggml_set_rows on the KV cache
 *     (src/cosyvoice-kv-cache.cpp:316,322).  The arithmetic lives in upstream
 *     ggml (un-vendored, unpinned: cmake/Dependencies.cmake:98-106), so the
 *     restatement follows gguf-py 0.19.0 gguf/quants.py, which documents
 *     itself as bit-exact with ggml's reference quantizers:
 *       Q4_0 quants.py:220-252, Q4_1 :254-289, Q5_0 :291-331,
 *       Q5_1 :333-376, Q8_0 :378-401, np_roundf :41-47.
 *     Pinned against golden vectors produced by gguf-py itself
 *     (tests/golden/make_golden.py).
 *   - ggml_flash_attn_ext semantics as called at
 *     src/cosyvoice-kv-cache.cpp:383 and src/cosyvoice-graph.cpp:375:
 *     softmax(scale * q.k + mask) . v, GQA head h -> kv head h / (Hq/Hkv),
 *     max_bias = 0, softcap = 0, additive f16 mask with -inf entries.
 *     Attention outputs are "parity unpinned" against ggml itself (ggml is
 *     not available to run); the fp64 restatement is the numeric oracle.
 *   - build_causal_mask (src/cosyvoice-llm.cpp:20-29) and the DiT chunk mask
 *     fill (src/cosyvoice-token2wav.cpp:285-298).
 *   - ggml_rope_ext as the reference calls it before the KV append and the
 *     attention (src/cosyvoice-llm.cpp:56-57,180 NEOX per head;
 *     src/cosyvoice-graph.cpp:354-355 NORMAL on the first head_dim elements
 *     of the whole row), restated from ggml's CPU backend (parity unpinned:
 *     ggml is not available to run).
 *   - A ggml-CPU-style single-pass fp32 flash attention (online max / sum per
 *     query row, K/V rows dequantized on the fly) used as the timed CPU
 *     baseline because ggml's own CPU kernel cannot be built here.
 *
 * Build with -ffp-contract=off: the codecs must not fuse x*id + c into an
 * FMA, exactly as numpy evaluates them as two rounded float32 operations.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

enum {
    T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q4_1 = 3, T_Q5_0 = 6, T_Q5_1 = 7, T_Q8_0 = 8
};

/* ---------------------------------------------------------------- fp16 -- */

/* IEEE-754 binary32 -> binary16, round to nearest, ties to even (the
 * conversion numpy's astype(np.float16) performs).  Written from the format
 * definitions: 1 sign, 5 exponent (bias 15), 10 fraction bits. */
uint16_t oracle_f32_to_f16(float f)
{
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t absx = x & 0x7fffffffu;
    if (absx >= 0x7f800000u) {                       /* inf or NaN */
        if (absx > 0x7f800000u) return (uint16_t)(sign | 0x7e00u | ((absx >> 13) & 0x3ffu));
        return (uint16_t)(sign | 0x7c00u);
    }
    int32_t e = (int32_t)(absx >> 23) - 127;         /* unbiased exponent */
    uint32_t mant = absx & 0x7fffffu;
    if (e > 15) return (uint16_t)(sign | 0x7c00u);   /* overflow -> inf */
    if (e >= -14) {                                  /* normal half */
        uint32_t h = ((uint32_t)(e + 15) << 10) | (mant >> 13);
        uint32_t rem = mant & 0x1fffu;                /* 13 dropped bits */
        if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1u; /* may carry into exponent: correct */
        return (uint16_t)(sign | h);
    }
    /* subnormal half (or zero): value = m * 2^-24 */
    if (e < -25) return (uint16_t)sign;              /* below half of smallest subnormal */
    uint32_t full = mant | 0x800000u;                /* 24-bit significand, value = full * 2^(e-23) */
    int shift = -e - 1;                              /* full * 2^(e-23) / 2^-24 = full >> (-1-e) */
    uint32_t h = full >> shift;
    uint32_t rem = full & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (h & 1u))) h += 1u;
    return (uint16_t)(sign | h);
}

float oracle_f16_to_f32(uint16_t h)
{
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu;
    uint32_t m = h & 0x3ffu;
    uint32_t x;
    if (e == 0) {
        if (m == 0) x = sign;
        else {                                       /* subnormal: normalise */
            int k = 0;
            while (!(m & 0x400u)) { m <<= 1; k++; }
            m &= 0x3ffu;
            x = sign | ((uint32_t)(127 - 15 - k + 1) << 23) | (m << 13);
        }
    } else if (e == 31) {
        x = sign | 0x7f800000u | (m << 13);
    } else {
        x = sign | ((e - 15 + 127) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

/* ------------------------------------------------------- block sizes -- */

int oracle_block_elems(int type) { return (type == T_F32 || type == T_F16) ? 1 : 32; }

int oracle_block_bytes(int type)
{
    switch (type) {
    case T_F32: return 4;
    case T_F16: return 2;
    case T_Q4_0: return 18;
    case T_Q4_1: return 20;
    case T_Q5_0: return 22;
    case T_Q5_1: return 24;
    case T_Q8_0: return 34;
    default: return 0;
    }
}

/* ggml_row_size: bytes of n elements (n a multiple of the block size). */
int64_t oracle_row_bytes(int type, int64_t n)
{
    return n / oracle_block_elems(type) * oracle_block_bytes(type);
}

static void put_f16(uint8_t* p, float v)
{
    uint16_t h = oracle_f32_to_f16(v);
    p[0] = (uint8_t)(h & 0xff);
    p[1] = (uint8_t)(h >> 8);
}

static float get_f16(const uint8_t* p) { return oracle_f16_to_f32((uint16_t)(p[0] | (p[1] << 8))); }

/* -------------------------------------------------------- quantizers -- */

/* quants.py:378-401 (Q8_0): d = amax/127, id = 1/d (0 when d == 0),
 * q = round-half-away(x*id), d stored as f16 of the fp32 d. */
static void quant_block_q8_0(const float* x, uint8_t* y)
{
    float amax = 0.0f;
    for (int j = 0; j < 32; j++) { float a = fabsf(x[j]); if (a > amax) amax = a; }
    float d = amax / 127.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    put_f16(y, d);
    for (int j = 0; j < 32; j++) {
        float v = x[j] * id;
        y[2 + j] = (uint8_t)(int8_t)roundf(v);      /* roundf: ties away from zero (np_roundf) */
    }
}

/* Signed value of largest magnitude, first occurrence (argmax semantics). */
static float signed_absmax(const float* x)
{
    float amax = 0.0f, max = 0.0f;
    for (int j = 0; j < 32; j++) { float a = fabsf(x[j]); if (a > amax) { amax = a; max = x[j]; } }
    return max;
}

/* quants.py:220-252 (Q4_0): d = max/-8, q = min(15, trunc(x*id + 8.5)),
 * byte j = q[j] | q[j+16] << 4. */
static void quant_block_q4_0(const float* x, uint8_t* y)
{
    float max = signed_absmax(x);
    float d = max / -8.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    put_f16(y, d);
    for (int j = 0; j < 16; j++) {
        float a = x[j] * id, b = x[j + 16] * id;
        int q0 = (int)truncf(a + 8.5f), q1 = (int)truncf(b + 8.5f);
        if (q0 > 15) q0 = 15; if (q1 > 15) q1 = 15;
        if (q0 < 0) q0 = 0; if (q1 < 0) q1 = 0;
        y[2 + j] = (uint8_t)(q0 | (q1 << 4));
    }
}

/* quants.py:254-289 (Q4_1): d = (max-min)/15, m = min,
 * q = min(15, trunc((x-min)*id + 0.5)). */
static void quant_block_q4_1(const float* x, uint8_t* y)
{
    float mn = x[0], mx = x[0];
    for (int j = 1; j < 32; j++) { if (x[j] < mn) mn = x[j]; if (x[j] > mx) mx = x[j]; }
    float d = (mx - mn) / 15.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    put_f16(y, d);
    put_f16(y + 2, mn);
    for (int j = 0; j < 16; j++) {
        float a = (x[j] - mn) * id, b = (x[j + 16] - mn) * id;
        int q0 = (int)truncf(a + 0.5f), q1 = (int)truncf(b + 0.5f);
        if (q0 > 15) q0 = 15; if (q1 > 15) q1 = 15;
        if (q0 < 0) q0 = 0; if (q1 < 0) q1 = 0;
        y[4 + j] = (uint8_t)(q0 | (q1 << 4));
    }
}

/* quants.py:291-331 (Q5_0): d = max/-16, q = min(31, trunc(x*id + 16.5)),
 * qs byte j = (q[j] & 15) | (q[j+16] & 15) << 4, qh bit j = q[j] >> 4. */
static void quant_block_q5_0(const float* x, uint8_t* y)
{
    float max = signed_absmax(x);
    float d = max / -16.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    put_f16(y, d);
    uint32_t qh = 0;
    for (int j = 0; j < 16; j++) {
        float a = x[j] * id, b = x[j + 16] * id;
        int q0 = (int)truncf(a + 16.5f), q1 = (int)truncf(b + 16.5f);
        if (q0 > 31) q0 = 31; if (q1 > 31) q1 = 31;
        if (q0 < 0) q0 = 0; if (q1 < 0) q1 = 0;
        y[6 + j] = (uint8_t)((q0 & 15) | ((q1 & 15) << 4));
        qh |= (uint32_t)((q0 >> 4) & 1) << j;
        qh |= (uint32_t)((q1 >> 4) & 1) << (j + 16);
    }
    y[2] = (uint8_t)qh; y[3] = (uint8_t)(qh >> 8); y[4] = (uint8_t)(qh >> 16); y[5] = (uint8_t)(qh >> 24);
}

/* quants.py:333-376 (Q5_1): d = (max-min)/31, m = min,
 * q = min(31, trunc((x-min)*id + 0.5)). */
static void quant_block_q5_1(const float* x, uint8_t* y)
{
    float mn = x[0], mx = x[0];
    for (int j = 1; j < 32; j++) { if (x[j] < mn) mn = x[j]; if (x[j] > mx) mx = x[j]; }
    float d = (mx - mn) / 31.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    put_f16(y, d);
    put_f16(y + 2, mn);
    uint32_t qh = 0;
    for (int j = 0; j < 16; j++) {
        float a = (x[j] - mn) * id, b = (x[j + 16] - mn) * id;
        int q0 = (int)truncf(a + 0.5f), q1 = (int)truncf(b + 0.5f);
        if (q0 > 31) q0 = 31; if (q1 > 31) q1 = 31;
        if (q0 < 0) q0 = 0; if (q1 < 0) q1 = 0;
        y[8 + j] = (uint8_t)((q0 & 15) | ((q1 & 15) << 4));
        qh |= (uint32_t)((q0 >> 4) & 1) << j;
        qh |= (uint32_t)((q1 >> 4) & 1) << (j + 16);
    }
    y[4] = (uint8_t)qh; y[5] = (uint8_t)(qh >> 8); y[6] = (uint8_t)(qh >> 16); y[7] = (uint8_t)(qh >> 24);
}

/* Quantize one row of n elements (n a multiple of the block size) into dst. */
int oracle_quantize_row(int type, const float* x, int64_t n, void* dst)
{
    uint8_t* y = (uint8_t*)dst;
    if (type == T_F32) { memcpy(y, x, (size_t)n * 4); return 0; }
    if (type == T_F16) { for (int64_t i = 0; i < n; i++) put_f16(y + 2 * i, x[i]); return 0; }
    if (n % 32) return -1;
    int bb = oracle_block_bytes(type);
    for (int64_t b = 0; b < n / 32; b++) {
        const float* xb = x + 32 * b;
        uint8_t* yb = y + bb * b;
        switch (type) {
        case T_Q8_0: quant_block_q8_0(xb, yb); break;
        case T_Q4_0: quant_block_q4_0(xb, yb); break;
        case T_Q4_1: quant_block_q4_1(xb, yb); break;
        case T_Q5_0: quant_block_q5_0(xb, yb); break;
        case T_Q5_1: quant_block_q5_1(xb, yb); break;
        default: return -1;
        }
    }
    return 0;
}

/* ------------------------------------------------------ dequantizers -- */

/* One block -> 32 floats, following the dequantize_blocks methods of
 * quants.py (d*q for the symmetric types, d*q + m for the _1 types). */
static void dequant_block(int type, const uint8_t* p, float* out)
{
    switch (type) {
    case T_Q8_0: {
        float d = get_f16(p);
        for (int j = 0; j < 32; j++) out[j] = (float)(int8_t)p[2 + j] * d;
        break;
    }
    case T_Q4_0: {
        float d = get_f16(p);
        for (int j = 0; j < 16; j++) {
            out[j] = d * (float)((int)(p[2 + j] & 15) - 8);
            out[j + 16] = d * (float)((int)(p[2 + j] >> 4) - 8);
        }
        break;
    }
    case T_Q4_1: {
        float d = get_f16(p), m = get_f16(p + 2);
        for (int j = 0; j < 16; j++) {
            out[j] = d * (float)(p[4 + j] & 15) + m;
            out[j + 16] = d * (float)(p[4 + j] >> 4) + m;
        }
        break;
    }
    case T_Q5_0: {
        float d = get_f16(p);
        uint32_t qh = (uint32_t)p[2] | ((uint32_t)p[3] << 8) | ((uint32_t)p[4] << 16) | ((uint32_t)p[5] << 24);
        for (int j = 0; j < 16; j++) {
            int q0 = (p[6 + j] & 15) | (int)(((qh >> j) & 1) << 4);
            int q1 = (p[6 + j] >> 4) | (int)(((qh >> (j + 16)) & 1) << 4);
            out[j] = d * (float)(q0 - 16);
            out[j + 16] = d * (float)(q1 - 16);
        }
        break;
    }
    case T_Q5_1: {
        float d = get_f16(p), m = get_f16(p + 2);
        uint32_t qh = (uint32_t)p[4] | ((uint32_t)p[5] << 8) | ((uint32_t)p[6] << 16) | ((uint32_t)p[7] << 24);
        for (int j = 0; j < 16; j++) {
            int q0 = (p[8 + j] & 15) | (int)(((qh >> j) & 1) << 4);
            int q1 = (p[8 + j] >> 4) | (int)(((qh >> (j + 16)) & 1) << 4);
            out[j] = d * (float)q0 + m;
            out[j + 16] = d * (float)q1 + m;
        }
        break;
    }
    }
}

int oracle_dequantize_row(int type, const void* src, int64_t n, float* out)
{
    const uint8_t* p = (const uint8_t*)src;
    if (type == T_F32) { memcpy(out, p, (size_t)n * 4); return 0; }
    if (type == T_F16) { for (int64_t i = 0; i < n; i++) out[i] = get_f16(p + 2 * i); return 0; }
    if (n % 32) return -1;
    int bb = oracle_block_bytes(type);
    if (!bb) return -1;
    for (int64_t b = 0; b < n / 32; b++) dequant_block(type, p + bb * b, out + 32 * b);
    return 0;
}

/* Quantize / dequantize many rows (row strides in elements / bytes). */
int oracle_quantize_rows(int type, const float* x, int64_t n_rows, int64_t n, void* dst)
{
    int64_t rb = oracle_row_bytes(type, n);
    for (int64_t r = 0; r < n_rows; r++)
        if (oracle_quantize_row(type, x + r * n, n, (uint8_t*)dst + r * rb)) return -1;
    return 0;
}

int oracle_dequantize_rows(int type, const void* src, int64_t n_rows, int64_t n, float* out)
{
    int64_t rb = oracle_row_bytes(type, n);
    for (int64_t r = 0; r < n_rows; r++)
        if (oracle_dequantize_row(type, (const uint8_t*)src + r * rb, n, out + r * n)) return -1;
    return 0;
}

/* ------------------------------------------------------------- masks -- */

/* src/cosyvoice-llm.cpp:20-29: n_batch new rows over seq_len keys; row i
 * sees key j iff j <= seq_len - n_batch + i.  Writes f16 bits 0 / 0xFC00. */
void oracle_causal_mask(uint16_t* mask, int32_t n_batch, int32_t seq_len)
{
    int32_t visible_prefix_end = seq_len - n_batch;
    for (int32_t i = 0; i < n_batch; i++) {
        for (int32_t j = 0; j < seq_len; j++) *mask++ = j > visible_prefix_end ? 0xFC00u : 0u;
        visible_prefix_end++;
    }
}

/* src/cosyvoice-token2wav.cpp:285-298: row i sees column j iff
 * j < (first boundary > i, else n).  bounds sorted ascending. */
void oracle_chunk_mask(uint16_t* mask, int32_t n, const int32_t* bounds, int32_t n_bounds)
{
    for (int32_t i = 0; i < n; i++) {
        int32_t block_end = n;
        for (int32_t b = 0; b < n_bounds; b++) if (bounds[b] > i) { block_end = bounds[b]; break; }
        for (int32_t j = 0; j < n; j++) mask[(int64_t)i * n + j] = j < block_end ? 0u : 0xFC00u;
    }
}

/* --------------------------------------------------------- attention -- */

/*
 * fp64 attention over already-dequantized rows (one batch entry).
 *   q   [n_q][Hq][D]      f32    (ggml q->data order for a permuted [D,Hq,n_q] view)
 *   k,v [n_kv][Hkv][D]    f32    (cache rows: one position holds all heads)
 *   mask [n_q][mask_stride] f32 additive or NULL (-inf entries skipped)
 *   out [n_q][Hq][D]      f32    (ggml flash_attn_ext result order)
 * q head h reads kv head h / (Hq / Hkv).  A row with every key masked
 * produces zeros.
 */
void oracle_attention_f64(const float* q, int32_t n_q, int32_t Hq, int32_t D,
                          const float* k, const float* v, int32_t n_kv, int32_t Hkv,
                          const float* mask, int64_t mask_stride, double scale, float* out)
{
    int32_t G = Hq / Hkv;
    double* s = (double*)malloc(sizeof(double) * (size_t)(n_kv > 0 ? n_kv : 1));
    double* o = (double*)malloc(sizeof(double) * (size_t)D);
    for (int32_t t = 0; t < n_q; t++) {
        for (int32_t h = 0; h < Hq; h++) {
            int32_t g = h / G;
            const float* qr = q + ((int64_t)t * Hq + h) * D;
            double m = -INFINITY;
            for (int32_t j = 0; j < n_kv; j++) {
                double mv = mask ? (double)mask[(int64_t)t * mask_stride + j] : 0.0;
                if (mv == -INFINITY) { s[j] = -INFINITY; continue; }
                const float* kr = k + ((int64_t)j * Hkv + g) * D;
                double acc = 0.0;
                for (int32_t d = 0; d < D; d++) acc += (double)qr[d] * (double)kr[d];
                s[j] = acc * scale + mv;
                if (s[j] > m) m = s[j];
            }
            for (int32_t d = 0; d < D; d++) o[d] = 0.0;
            double l = 0.0;
            if (m != -INFINITY) {
                for (int32_t j = 0; j < n_kv; j++) {
                    if (s[j] == -INFINITY) continue;
                    double p = exp(s[j] - m);
                    l += p;
                    const float* vr = v + ((int64_t)j * Hkv + g) * D;
                    for (int32_t d = 0; d < D; d++) o[d] += p * (double)vr[d];
                }
            }
            float* orow = out + ((int64_t)t * Hq + h) * D;
            for (int32_t d = 0; d < D; d++) orow[d] = l > 0.0 ? (float)(o[d] / l) : 0.0f;
        }
    }
    free(s);
    free(o);
}

/*
 * ggml-CPU-style fp32 flash attention, used as the timed CPU baseline.
 * One pass per (sequence, query row, head) with an online running max M and
 * sum S; each key row is dequantized from the typed cache as it is visited
 * (the V row accumulation follows the same order).  Work is spread over
 * OpenMP threads by (sequence, head).
 *
 *   q      [n_seq][n_q][Hq][D] f32
 *   k_rows per-sequence base pointers of typed cache rows (row = all heads)
 *   v_rows the same for V
 *   kv_len [n_seq]  keys per sequence
 *   causal nonzero: query t of n_q sees keys j <= kv_len - n_q + t
 *   out    [n_seq][n_q][Hq][D] f32
 */
void oracle_flash_cpu(const float* q, int32_t n_seq, int32_t n_q, int32_t Hq, int32_t Hkv, int32_t D,
                      int32_t k_type, const void* const* k_rows, int64_t k_nb1,
                      int32_t v_type, const void* const* v_rows, int64_t v_nb1,
                      const int32_t* kv_len, int32_t causal, float scale, float* out, int32_t n_threads)
{
    int32_t G = Hq / Hkv;
    int64_t k_head_bytes = k_nb1 / Hkv, v_head_bytes = v_nb1 / Hkv;
    int64_t total = (int64_t)n_seq * Hq;
#ifdef _OPENMP
    if (n_threads > 0) omp_set_num_threads(n_threads);
#pragma omp parallel
#endif
    {
        float* kbuf = (float*)malloc(sizeof(float) * (size_t)D);
        float* vbuf = (float*)malloc(sizeof(float) * (size_t)D);
        float* acc = (float*)malloc(sizeof(float) * (size_t)D);
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (int64_t w = 0; w < total; w++) {
            int32_t sidx = (int32_t)(w / Hq), h = (int32_t)(w % Hq), g = h / G;
            int32_t L = kv_len[sidx];
            for (int32_t t = 0; t < n_q; t++) {
                const float* qr = q + (((int64_t)sidx * n_q + t) * Hq + h) * D;
                int32_t last = causal ? L - n_q + t : L - 1;
                float M = -INFINITY, S = 0.0f;
                for (int32_t d = 0; d < D; d++) acc[d] = 0.0f;
                for (int32_t j = 0; j <= last; j++) {
                    const uint8_t* kr = (const uint8_t*)k_rows[sidx] + (int64_t)j * k_nb1 + g * k_head_bytes;
                    oracle_dequantize_row(k_type, kr, D, kbuf);
                    float s = 0.0f;
                    for (int32_t d = 0; d < D; d++) s += qr[d] * kbuf[d];
                    s *= scale;
                    float Mold = M, ms = 1.0f, vs = 1.0f;
                    if (s > M) { M = s; ms = expf(Mold - M); } else { vs = expf(s - M); }
                    const uint8_t* vr = (const uint8_t*)v_rows[sidx] + (int64_t)j * v_nb1 + g * v_head_bytes;
                    oracle_dequantize_row(v_type, vr, D, vbuf);
                    if (ms != 1.0f) for (int32_t d = 0; d < D; d++) acc[d] *= ms;
                    for (int32_t d = 0; d < D; d++) acc[d] += vbuf[d] * vs;
                    S = S * ms + vs;
                }
                float inv = S == 0.0f ? 0.0f : 1.0f / S;
                float* orow = out + (((int64_t)sidx * n_q + t) * Hq + h) * D;
                for (int32_t d = 0; d < D; d++) orow[d] = acc[d] * inv;
            }
        }
        free(kbuf);
        free(vbuf);
        free(acc);
    }
}

/* ---------------------------------------------------------------- RoPE -- */

/* Rotary position embedding, ggml_rope_ext with ext_factor 0 and no frequency
 * factors (the only form the reference uses: freq_scale 1, attn_factor 1).
 * ggml's CPU backend forms theta_scale = powf(freq_base, -2/n_dims) and, per
 * position p, the angle of pair k as p * theta_scale^k by k sequential float
 * products, then freq_scale * angle; cos / sin are cosf / sinf times
 * attn_factor.  Rows are cut into units of unit_len elements (a head for the
 * LLM, the whole row for the DiT); in each unit the first n_dims elements
 * rotate in pairs -- NEOX: element i with i + n_dims/2; NORMAL: 2k with
 * 2k + 1 -- as out_a = a cos - b sin, out_b = a sin + b cos (two rounded
 * products and one rounded sum each), and the rest is copied.
 * x and out: n_rows rows of row_len floats (row r at x + r * row_len). */
void oracle_rope(const float* x, float* out, const int32_t* pos, int32_t n_rows, int32_t row_len, int32_t unit_len,
                 int32_t n_dims, int32_t mode, float freq_base, float freq_scale, float attn_factor)
{
    const int neox = (mode & 2) != 0;
    const int half = n_dims / 2;
    const float theta_scale = powf(freq_base, -2.0f / (float)n_dims);
    float* cs = (float*)malloc(sizeof(float) * 2 * (half > 0 ? half : 1));
    for (int32_t r = 0; r < n_rows; ++r) {
        float theta = (float)pos[r];
        for (int k = 0; k < half; ++k) {
            const float th = freq_scale * theta;
            cs[2 * k] = cosf(th) * attn_factor;
            cs[2 * k + 1] = sinf(th) * attn_factor;
            theta *= theta_scale;
        }
        const float* xr = x + (int64_t)r * row_len;
        float* orow = out + (int64_t)r * row_len;
        for (int32_t u = 0; u + unit_len <= row_len; u += unit_len) {
            for (int k = 0; k < half; ++k) {
                const int i0 = neox ? k : 2 * k, i1 = neox ? k + half : 2 * k + 1;
                const float a = xr[u + i0], b = xr[u + i1], c = cs[2 * k], sn = cs[2 * k + 1];
                orow[u + i0] = a * c - b * sn;
                orow[u + i1] = a * sn + b * c;
            }
            for (int i = n_dims; i < unit_len; ++i) orow[u + i] = xr[u + i];
        }
    }
    free(cs);
}

int oracle_max_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
