/*
 * cvattn.h -- C ABI of the B200 attention engine for cosyvoice.cpp.
 *
 * The engine replaces the ggml_flash_attn_ext attention path of cosyvoice.cpp
 * (KV append/quantize, Qwen2 decode and prefill attention, DiT attention with
 * fixed / offloadable / uncached KV slots).  Every entry point is plain C:
 * device pointers, sizes and ggml type ids; no C++ or torch types.
 *
 * Conventions
 *   - KV memory follows ggml's cache tensor layout (src/cosyvoice-kv-cache.cpp:104-119):
 *     a tensor of type T with ne = {n_heads*head_dim, ne1 positions, ne2 batch};
 *     one row (one position) holds every KV head, block-quantized for the
 *     32-element types; nb1 = bytes between positions, nb2 = between batch entries.
 *   - Streams are passed as void* (a cudaStream_t / CUstream); 0 = legacy default.
 *   - Calls are asynchronous on the stream and never abort the process: bad
 *     arguments return a status; bad device-resident indices are skipped and
 *     recorded in the context's status word (cvattn_context_sync_status).
 *   - Type ids are ggml's: F32=0, F16=1, Q4_0=2, Q4_1=3, Q5_0=6, Q5_1=7, Q8_0=8.
 *   - Each worker thread uses its own cvattn_context and stream
 *     (src/cosyvoice-model.cpp:82-107 gives each worker its own backend).
 */
#ifndef CVATTN_H
#define CVATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CVATTN_ABI_VERSION 2

/* ------------------------------------------------------------------ status */

typedef enum cvattn_status {
    CVATTN_OK = 0,
    CVATTN_ERR_INVALID_ARGUMENT = 1,
    CVATTN_ERR_UNSUPPORTED = 2,   /* type pair / head shape the engine does not implement */
    CVATTN_ERR_LENGTH = 3,        /* sequence longer than the cache (src/cosyvoice-llm.cpp:98-99,207) */
    CVATTN_ERR_ALLOC = 4,
    CVATTN_ERR_CUDA = 5,          /* a CUDA runtime call failed */
    CVATTN_ERR_DEVICE = 6,        /* a kernel skipped work on a bad device-resident index */
    CVATTN_ERR_NO_DEVICE = 7,
    CVATTN_ERR_TIMEOUT = 8        /* a bounded in-kernel wait gave up */
} cvattn_status;

/* Human-readable status text. */
const char* cvattn_status_string(cvattn_status s);

/* Maps a status onto enum ggml_status (SUCCESS 0, FAILED -1, ALLOC_FAILED -2),
 * the value cosyvoice_worker_context::status holds (src/cosyvoice-model.cpp:522-525). */
int32_t cvattn_status_to_ggml(cvattn_status s);

/* ABI version and struct sizes, so bindings can verify their mirrors.
 * which: 0 cvattn_tensor, 1 cvattn_decode_params, 2 cvattn_flash_params,
 *        3 cvattn_kv_cache_params, 4 cvattn_dit_step, 5 cvattn_rope_params. */
int32_t cvattn_abi_version(void);
size_t cvattn_abi_sizeof(int32_t which);

/* ------------------------------------------------------------------- types */

enum {
    CVATTN_TYPE_F32 = 0, CVATTN_TYPE_F16 = 1, CVATTN_TYPE_Q4_0 = 2, CVATTN_TYPE_Q4_1 = 3,
    CVATTN_TYPE_Q5_0 = 6, CVATTN_TYPE_Q5_1 = 7, CVATTN_TYPE_Q8_0 = 8
};

/* A ggml KV tensor (or an uncached K/V activation in the same row layout). */
typedef struct cvattn_tensor {
    void*   data;      /* device address of position 0, batch 0 */
    int32_t type;      /* ggml type id */
    int32_t n_heads;   /* heads packed in one row */
    int32_t head_dim;  /* elements per head */
    int32_t reserved;  /* 0 */
    int64_t ne1;       /* positions (capacity) */
    int64_t ne2;       /* batch entries */
    int64_t nb1;       /* bytes between positions */
    int64_t nb2;       /* bytes between batch entries */
} cvattn_tensor;

/* ggml_row_size(type, n): bytes of n elements; 0 for an unknown type or a
 * count that is not a multiple of the block size. */
size_t cvattn_row_size(int32_t type, int64_t n);

/* ---------------------------------------------------- capability and types */

/* Replaces the ggml_backend_supports_op probes on set_rows + flash_attn_ext
 * (src/cosyvoice-loader.cpp:543-567).  True for every pair of
 * {F32, F16, Q8_0, Q5_1, Q5_0, Q4_1, Q4_0} when head_dim == 64 and
 * n_q_heads is a multiple of n_kv_heads with a ratio of at most 8. */
int32_t cvattn_supports(int32_t k_type, int32_t v_type, int32_t head_dim,
                        int32_t n_q_heads, int32_t n_kv_heads);

/* The loader's fallback chain q4_0 -> q4_1 -> q5_0 -> q5_1 -> q8_0 -> f16 -> f32
 * on ggml ids (src/cosyvoice-loader.cpp:498-510); -1 past f32. */
int32_t cvattn_kv_fallback_type(int32_t ggml_type);

/* cosyvoice_kv_cache_type_t (include/cosyvoice.h:32-42) <-> ggml type id
 * (src/cosyvoice-loader.cpp:468-496); -1 for an unknown value. */
int32_t cvattn_kv_cache_type_to_ggml(int32_t cosyvoice_kv_cache_type);
int32_t cvattn_ggml_to_kv_cache_type(int32_t ggml_type);

/* Flash-attention branch of cosyvoice_check_kv_cache_types
 * (src/cosyvoice-loader.cpp:533-632) with cvattn_supports as the probe.
 * kv_type_union is the packed value of include/cosyvoice.h:193-221
 * (bit 31 = separate K/V; K bits 0-4, V 5-9, fallback 10-14).
 * Outputs the resolved ggml K/V types, the rewritten union and whether
 * flash attention is on. */
cvattn_status cvattn_negotiate_kv_types(uint32_t kv_type_union, int32_t kv_fallback,
                                        int32_t head_dim, int32_t n_q_heads, int32_t n_kv_heads,
                                        int32_t* k_type, int32_t* v_type,
                                        uint32_t* resolved_union, int32_t* fattn);

/* ----------------------------------------------------------------- context */

typedef struct cvattn_context cvattn_context;

/* One per worker.  Holds the device status word and per-device state. */
cvattn_status cvattn_context_create(int32_t device, cvattn_context** out);
void          cvattn_context_destroy(cvattn_context* ctx);

/* Synchronizes the stream, then reads and clears the device status word.
 * Returns CVATTN_ERR_DEVICE if a kernel skipped a bad index since the last
 * call; *detail (optional) receives the first recorded code. */
cvattn_status cvattn_context_sync_status(cvattn_context* ctx, void* stream, int32_t* detail);

/* -------------------------------------------------------------- KV append */

/* Quantize-on-write of new K or V rows: the ggml_set_rows of
 * cosyvoice_kv_cache::update_cache (src/cosyvoice-kv-cache.cpp:315-316,321-322).
 *   src    f32 rows of cache->n_heads*cache->head_dim elements:
 *          row (t, b) at src + t*src_nb1 + b*src_nb2 (bytes)
 *   pos    device int32 positions: pos[t + b*pos_nb1/4] (pos_nb1 = 0: shared by
 *          every batch entry, the LLM's 1-D position_ids; otherwise the DiT's
 *          [S, batch] position tensor, src/cosyvoice-graph.cpp:447-449)
 * Blocks are bit-identical to ggml's reference quantizers.  A position outside
 * [0, cache->ne1) is skipped and recorded in the status word. */
cvattn_status cvattn_kv_append(cvattn_context* ctx, void* stream, const cvattn_tensor* cache,
                               const float* src, int64_t src_nb1, int64_t src_nb2,
                               const int32_t* pos, int64_t pos_nb1,
                               int32_t n_new, int32_t batch);

/* ------------------------------------------------------------------- RoPE */

/* Rotary position embedding as ggml_rope_ext applies it in the reference, with
 * ext_factor 0 and no frequency factors (the only form it uses):
 *   LLM  src/cosyvoice-llm.cpp:56-57,180  NEOX, n_dims = unit_len = head_dim,
 *        freq_base = rope_theta, freq_scale 1, attn_factor 1;
 *   DiT  src/cosyvoice-graph.cpp:354-355  NORMAL, n_dims = head_dim on the
 *        whole 1024-wide row (unit_len = row length), freq_base 10000.
 * Angles follow ggml's CPU backend: theta_scale = powf(freq_base, -2/n_dims)
 * (formed on the host), pair k at position p turns by p * theta_scale^k built
 * by k sequential float products, times freq_scale. */
enum {
    CVATTN_ROPE_NORMAL = 0,  /* pairs (2k, 2k + 1)          (GGML_ROPE_TYPE_NORMAL) */
    CVATTN_ROPE_NEOX = 2     /* pairs (k, k + n_dims / 2)   (GGML_ROPE_TYPE_NEOX)   */
};

typedef struct cvattn_rope_params {
    int32_t mode;         /* CVATTN_ROPE_NORMAL or CVATTN_ROPE_NEOX */
    int32_t n_dims;       /* rotated prefix of each unit: even, 2..unit_len */
    int32_t unit_len;     /* elements per rotation unit: head_dim, or the whole row */
    float   freq_base;    /* rope_theta */
    float   freq_scale;
    float   attn_factor;  /* scales cos and sin */
} cvattn_rope_params;

/* out = RoPE(x) for n_rows rows of row_len f32 (row r at x + r*x_nb1 and
 * out + r*out_nb1 bytes; out may equal x), row r at position pos[r] (device
 * int32).  row_len must be a multiple of unit_len. */
cvattn_status cvattn_rope(void* stream, const cvattn_rope_params* rope,
                          const float* x, int64_t x_nb1, float* out, int64_t out_nb1,
                          const int32_t* pos, int32_t n_rows, int32_t row_len);

/* cvattn_kv_append with the K rows rotated on the way in: the ggml_rope_ext of
 * the keys fused with update_cache (src/cosyvoice-llm.cpp:57-59,180-182;
 * src/cosyvoice-graph.cpp:355,365).  Row (t, b) turns by its cache position
 * pos[t + b*pos_nb1/4].  The bytes equal cvattn_rope followed by
 * cvattn_kv_append. */
cvattn_status cvattn_kv_append_rope(cvattn_context* ctx, void* stream, const cvattn_tensor* cache,
                                    const float* src, int64_t src_nb1, int64_t src_nb2,
                                    const int32_t* pos, int64_t pos_nb1,
                                    int32_t n_new, int32_t batch, const cvattn_rope_params* rope);

/* Dequantize rows [0, n_rows) of every batch entry to f32
 * (dst row (t, b) at dst + (b*n_rows + t)*n_heads*head_dim).  Used for the
 * offload of a slot to f32 and by tests. */
cvattn_status cvattn_kv_dequantize(cvattn_context* ctx, void* stream, const cvattn_tensor* cache,
                                   int32_t n_rows, float* dst);

/* ------------------------------------------------------------------ decode */

enum {
    CVATTN_DECODE_EMIT_PARTIAL = 1,  /* write unnormalized O and (max, sum) instead of O/sum */
    CVATTN_DECODE_CUDA_CORES = 2,    /* use the CUDA-core kernel even where the tensor-core one applies */
    CVATTN_DECODE_NOT_PERSISTENT = 4, /* use the one-chunk-per-CTA tensor-core kernel, not a persistent one */
    /* The caller guarantees that kv_len and the cached rows this call reads (all
     * but the row it appends itself) are not written by the kernels just before it
     * on the stream -- e.g. one model step that decodes every layer with the
     * append fused, its lengths uploaded by the host.  The pipelined kernel then
     * starts streaming K/V while the previous kernel is still finishing
     * (programmatic dependent launch); Q, the new rows and all outputs still wait
     * for it. */
    CVATTN_DECODE_INPUTS_READY = 8,
    /* use the persistent kernel with 128-position items and a per-chunk merge
     * instead of the default streaming one (64-position items, running output) */
    CVATTN_DECODE_WIDE_CHUNKS = 16,
    /* Block-quantized K and V (2 KV heads, head_dim 64) have two persistent
     * tensor-core kernels: the tcgen05 streaming kernel (tiles in shared memory,
     * running output in tensor memory; shorter per-item pipeline) and the
     * register-resident warp-MMA kernel (fewer instructions per item).  By
     * default a launch with at least 32 64-position items per SM (counted from
     * n_seq and max_kv_len) runs the warp-MMA kernel, smaller ones the streaming
     * kernel; these flags force one.  cvattn_decode_rope always runs on the
     * streaming kernel. */
    CVATTN_DECODE_TMEM_STREAM = 32,
    CVATTN_DECODE_WARP_MMA = 64
};

/* One decode token per sequence: ggml_flash_attn_ext with n_q = 1 and no mask
 * (src/cosyvoice-kv-cache.cpp:379-386 via src/cosyvoice-llm.cpp:62), batched
 * over sequences, optionally fused with the append of that token's K/V row
 * (src/cosyvoice-kv-cache.cpp:316,322). */
typedef struct cvattn_decode_params {
    const float*    q;               /* device f32 [n_seq][n_q_heads][head_dim] */
    int64_t         q_seq_stride;    /* floats between sequences */
    float*          out;             /* device f32 [n_seq][n_q_heads][head_dim] */
    int64_t         out_seq_stride;  /* floats between sequences */
    cvattn_tensor   k;               /* type/heads/dims/nb1 shared by all sequences;   */
    cvattn_tensor   v;               /* sequence s rows at data + s*nb2 unless *_seq_ptrs */
    const uint64_t* k_seq_ptrs;      /* optional device [n_seq]: row-0 address per sequence */
    const uint64_t* v_seq_ptrs;      /* (separate worker caches); NULL = data + s*nb2 */
    const int32_t*  kv_len;          /* device [n_seq]: visible keys incl. an appended row */
    const float*    k_new;           /* optional device f32 [n_seq][n_heads*head_dim]: row */
    const float*    v_new;           /* written at position kv_len-1 before attending      */
    float*          partial_ml;      /* EMIT_PARTIAL: device f32 [n_seq][n_q_heads][2] (max, sum) */
    int32_t         n_seq;
    int32_t         n_q_heads;
    int32_t         max_kv_len;      /* host bound on kv_len[] (sizes the grid) */
    int32_t         flags;
    float           scale;           /* 1/sqrt(head_dim) in the reference */
    int32_t         reserved;
    void*           workspace;       /* device scratch of cvattn_decode_workspace_size bytes, */
    size_t          workspace_size;  /* zeroed before first use (cvattn_workspace_init)        */
} cvattn_decode_params;

/* Workspace bytes for cvattn_decode with this type pair and shape (chunk
 * partials plus one ticket counter per sequence); 0 if unsupported. */
size_t cvattn_decode_workspace_size(int32_t k_type, int32_t v_type, int32_t n_seq, int32_t max_kv_len,
                                    int32_t n_q_heads, int32_t n_kv_heads, int32_t head_dim);

/* Zero a workspace: once after allocation, and again after
 * cvattn_context_sync_status has reported CVATTN_ERR_TIMEOUT or
 * CVATTN_ERR_DEVICE for a decode that used it.  A completed decode leaves its
 * ticket counters at zero; a decode whose kernel gave up early can leave them
 * counting, and later decodes through that workspace would then not merge
 * their split partials. */
cvattn_status cvattn_workspace_init(void* stream, void* workspace, size_t bytes);

cvattn_status cvattn_decode(cvattn_context* ctx, void* stream, const cvattn_decode_params* p);

/* cvattn_decode for callers that cannot allocate device memory.  This entry
 * point has no counterpart in the reference.  Examples of such callers: a
 * ggml custom-op callback that runs inside a scheduled graph compute and
 * receives only its tensors, or a real-time worker that must not block on
 * the driver's allocator.
 * Inputs and outputs are the caller's, as for cvattn_decode; the workspace
 * fields of p are ignored.  The split-KV partials and ticket counters live
 * instead in a static device array of CVATTN_DECODE_NOALLOC_SCRATCH_BYTES,
 * which every GPU that loads the library holds until the process exits.
 *   - Requests needing more than that (cvattn_decode_workspace_size) return
 *     CVATTN_ERR_LENGTH and launch nothing.
 *   - No cudaMalloc/cudaFree is called.  The first call on a device, made
 *     with that device current, looks up the array's device address; make
 *     that first call before any stream capture.
 *   - All calls on a device share the array: calls whose kernels overlap on
 *     the GPU race and must be serialized.  The ticket counters are zeroed on
 *     the stream at the start of every call; partials from the previous call
 *     remain in the array. */
#define CVATTN_DECODE_NOALLOC_SCRATCH_BYTES (8u * 1024u * 1024u)
cvattn_status cvattn_decode_noalloc(cvattn_context* ctx, void* stream, const cvattn_decode_params* p);

/* cvattn_decode with the RoPE of the decode step fused in: Q and the appended
 * K row of sequence s turn by position kv_len[s] - 1 (the ggml_rope_ext calls
 * of src/cosyvoice-llm.cpp:56-57 before update_cache and attention_forward).
 * Runs on either persistent decode kernel (warp-MMA or streaming, the
 * dispatcher's choice), so it needs block-quantized K and V, 2 KV heads,
 * head_dim 64, at most 512 sequences, no flag that selects another kernel,
 * and a per-head rope (unit_len = n_dims = head_dim); otherwise
 * CVATTN_ERR_UNSUPPORTED (use cvattn_rope, then cvattn_decode). */
cvattn_status cvattn_decode_rope(cvattn_context* ctx, void* stream, const cvattn_decode_params* p,
                                 const cvattn_rope_params* rope);

/* Log-sum-exp combine of split partials (cross-GPU split-KV):
 *   partial_o  f32 [n_parts][n_rows][head_dim] unnormalized
 *   partial_ml f32 [n_parts][n_rows][2] (max in log2 units, sum)
 *   out        f32 [n_rows][head_dim] */
cvattn_status cvattn_combine(void* stream, const float* partial_o, const float* partial_ml,
                             int32_t n_parts, int32_t n_rows, int32_t head_dim, float* out);

/* ------------------------------------------------- prefill / DiT attention */

enum {
    CVATTN_MASK_NONE = 0,      /* every key visible (uncached DiT without mask) */
    CVATTN_MASK_EXPLICIT = 1,  /* additive f16 mask rows (ggml semantics) */
    CVATTN_MASK_CAUSAL = 2,    /* query i sees key j iff j <= causal_offset + i (src/cosyvoice-llm.cpp:20-29) */
    CVATTN_MASK_CHUNK = 3      /* DiT streaming chunk mask (src/cosyvoice-token2wav.cpp:285-298) */
};

#define CVATTN_MAX_CHUNK_BOUNDS 64

/* Multi-query attention: Qwen2 prefill (src/cosyvoice-llm.cpp:62, mask
 * :101-108) and DiT attention, cached (src/cosyvoice-graph.cpp:363-366) or
 * uncached (:373-377).  Q is f32 as ggml passes it; K/V are typed cache rows
 * or uncached f32 activations in the same row layout. */
typedef struct cvattn_flash_params {
    const float*    q;            /* device f32; element (d, i, h, b) at          */
    int64_t         q_nb_tok;     /* q + i*q_nb_tok + h*q_nb_head + b*q_nb_batch + d */
    int64_t         q_nb_head;    /* (strides in floats)                          */
    int64_t         q_nb_batch;
    float*          out;          /* device f32 [batch][n_q][n_q_heads][head_dim] */
    cvattn_tensor   k;            /* positions [0, n_kv) of batch b at data + b*nb2 */
    cvattn_tensor   v;
    int32_t         n_q;
    int32_t         n_kv;
    int32_t         n_q_heads;
    int32_t         batch;
    float           scale;
    int32_t         mask_mode;    /* CVATTN_MASK_* */
    const uint16_t* mask;         /* EXPLICIT: device f16 bits, row i at mask + i*mask_nb1 + b*mask_nb2 */
    int64_t         mask_nb1;     /* (elements) */
    int64_t         mask_nb2;
    int32_t         causal_offset;                 /* CAUSAL: n_kv - n_q for llm_prefill */
    int32_t         n_chunk_bounds;                /* CHUNK */
    int32_t         chunk_bounds[CVATTN_MAX_CHUNK_BOUNDS]; /* ascending chunk ends (host values) */
    int32_t         chunk_key_offset;  /* CHUNK: keys below this are always visible (cached prompt) */
    int32_t         chunk_row_offset;  /* CHUNK: query i uses mask row i + chunk_row_offset */
    int32_t         flags;             /* CVATTN_FLASH_*; 0 for the default kernel */
} cvattn_flash_params;

enum {
    /* one query tile per CTA, shared-memory P (the first tensor-core kernel);
       the default is the persistent two-tile kernel with P in tensor memory */
    CVATTN_FLASH_ONE_TILE = 1,
    /* persistent kernel: two softmax warpgroups per query tile, each taking half
       of every key tile's columns (the default) */
    CVATTN_FLASH_SPLIT_COLUMNS = 2,
    /* persistent kernel: one softmax warpgroup per query tile, a thread per row */
    CVATTN_FLASH_WHOLE_ROWS = 4
};

cvattn_status cvattn_flash(cvattn_context* ctx, void* stream, const cvattn_flash_params* p);

/* ------------------------------------------------------- offload and load */

/* Copy positions [0, n_tokens) of every batch entry of a KV tensor to host
 * memory, batch-major and contiguous (the per-layer K or V part of
 * cosyvoice_kv_cache::offload_cache, src/cosyvoice-kv-cache.cpp:160-172),
 * and back (load_cache, :233-243).  host may be pageable or pinned. */
cvattn_status cvattn_kv_copy_to_host(void* stream, const cvattn_tensor* t, int32_t n_tokens, void* host);
cvattn_status cvattn_kv_copy_from_host(void* stream, const cvattn_tensor* t, int32_t n_tokens,
                                       const void* host);

/* -------------------------------------------------- KV cache host object */

/* Host-side mirror of class cosyvoice_kv_cache (src/cosyvoice-kv-cache.h:10-69)
 * in the flash-attention mode the reference uses by default. */
typedef struct cvattn_kv_cache cvattn_kv_cache;

typedef struct cvattn_kv_cache_params {
    int32_t  layers;
    int32_t  k_head_dim;
    int32_t  v_head_dim;
    int32_t  n_kv_heads;
    uint32_t max_seq;
    int32_t  k_type;             /* ggml ids */
    int32_t  v_type;
    int32_t  batch;
    int32_t  n_slots;
    int32_t  n_offloaded_slots;
} cvattn_kv_cache_params;

/* build_kv_cache (src/cosyvoice-kv-cache.cpp:45-102): one device allocation
 * holding K then V for every (slot, layer), each 256-byte aligned. */
cvattn_status cvattn_kv_cache_create(cvattn_context* ctx, const cvattn_kv_cache_params* p,
                                     cvattn_kv_cache** out);
void          cvattn_kv_cache_destroy(cvattn_kv_cache* c);

/* The K (which = 0) or V (which = 1) tensor of (layer, slot). */
cvattn_status cvattn_kv_cache_tensor(cvattn_kv_cache* c, int32_t layer, int32_t slot, int32_t which,
                                     cvattn_tensor* out);
size_t        cvattn_kv_cache_device_bytes(const cvattn_kv_cache* c);

/* cur_len and the view length seen by attention. */
uint32_t      cvattn_kv_cache_get_len(const cvattn_kv_cache* c);
void          cvattn_kv_cache_set_len(cvattn_kv_cache* c, uint32_t len);

/* update_cache (src/cosyvoice-kv-cache.cpp:309-355): append n_new rows of f32
 * K and V ([n_heads*head_dim] per row, token-major, batch-major) at device
 * positions pos (pos_nb1 as in cvattn_kv_append) into the bound slot; the
 * attention view becomes cur_len + n_new long. */
cvattn_status cvattn_kv_cache_update(cvattn_kv_cache* c, void* stream, int32_t layer,
                                     const float* k, const float* v, const int32_t* pos,
                                     int64_t pos_nb1, int32_t n_new);

/* attention_forward (src/cosyvoice-kv-cache.cpp:379-386) over the current view
 * of (layer, bound slot).  q f32 [batch][n_q][n_q_heads][head_dim]; scale
 * 1/sqrt(head_dim); n_q == 1 without a mask runs the decode kernel, anything
 * else the tensor-core flash kernel.  mask semantics as cvattn_flash_params.
 * The call neither allocates nor synchronizes: the decode workspace is sized
 * at creation, and the view length reaches the device through a small kernel
 * on the stream (which also clears the workspace's ticket counters). */
cvattn_status cvattn_kv_cache_attention(cvattn_kv_cache* c, void* stream, int32_t layer,
                                        const float* q, int32_t n_q, int32_t n_q_heads,
                                        int32_t mask_mode, const uint16_t* mask, int64_t mask_nb1,
                                        float* out);

/* shift_kv_node_pos (src/cosyvoice-kv-cache.cpp:398-408): cur_len += n. */
void          cvattn_kv_cache_shift(cvattn_kv_cache* c, uint32_t n);

/* bind_slot / slide_kv_slot (src/cosyvoice-kv-cache.cpp:415-467). */
int32_t       cvattn_kv_cache_bind_slot(cvattn_kv_cache* c, int32_t slot);
cvattn_status cvattn_kv_cache_slide_slot(cvattn_kv_cache* c);
int32_t       cvattn_kv_cache_current_slot(const cvattn_kv_cache* c);

/* offload_slot / load_slot (src/cosyvoice-kv-cache.cpp:148-246,276-290).
 * offload copies positions [0, n_tokens) of every layer of device slot 0 --
 * the slot the reference's offload_cache reads (kv_cache_layers[i], :163-172),
 * which every offloadable DiT step binds (src/cosyvoice-token2wav.cpp:390) --
 * to host slot `offloaded_slot`; load copies a host slot into the bound
 * device slot (:233-243) and sets cur_len to its length.  The host layout is
 * the reference's: per layer, K of every batch entry, then V.
 * Unlike the reference, which synchronizes after every transfer, both calls
 * only enqueue copies on the stream (one strided copy per layer and tensor,
 * from or into pinned host memory) and return, so the copies overlap the next
 * step's kernels.  Stream order covers later kernels on the same stream; a
 * load or offload on another stream first waits for the slot's last copy. */
cvattn_status cvattn_kv_cache_offload_slot(cvattn_kv_cache* c, void* stream, int32_t offloaded_slot,
                                           uint32_t n_tokens);
cvattn_status cvattn_kv_cache_load_slot(cvattn_kv_cache* c, void* stream, int32_t offloaded_slot);
/* The bytes of host slot `offloaded_slot` (struct offloaded_kv_cache's buffer
 * and len, src/cosyvoice-kv-cache.cpp:19-32): waits on the host until the
 * slot's last copy has completed, then returns its address, its byte count
 * and (optional) its length in positions.  The pointer stays valid until the
 * slot grows, is cleared or the cache is destroyed. */
cvattn_status cvattn_kv_cache_offloaded_slot(cvattn_kv_cache* c, int32_t offloaded_slot, const void** data,
                                             size_t* bytes, uint32_t* n_tokens);
size_t        cvattn_kv_cache_offloaded_size(const cvattn_kv_cache* c);
void          cvattn_kv_cache_clear_offloaded(cvattn_kv_cache* c);

/* ------------------------------------------------------- DiT step plan */

/* One ODE step of dit_sched_config (src/cosyvoice-token2wav.cpp:100-167). */
typedef struct cvattn_dit_step {
    uint8_t rebuild, cache_kv, load, offload, slide, slice, mask, reserved;
    int64_t cut_len;
} cvattn_dit_step;

cvattn_status cvattn_dit_sched_plan(int32_t n_steps, int32_t n_offloadable_slots, int32_t n_fixed_slots,
                                    int64_t cut_len, uint32_t offset, int32_t streaming,
                                    int32_t kv_slidable, cvattn_dit_step* out);

#ifdef __cplusplus
}
#endif

#endif /* CVATTN_H */
