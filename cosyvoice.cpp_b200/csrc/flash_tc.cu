// flash_tc.cu -- host side of the tcgen05 flash-attention kernel
// (flash_tc.cuh): TMA tensor maps for f16 caches and the type dispatch.
#include <cuda.h>

#include <cstring>

#include "flash_pipe.cuh"
#include "internal.h"

namespace cvattn {
namespace fa {

// ------------------------------------------------------------------ host

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    }
    return fn;
}

// f16 KV tensor as a 3-D map {row elements, n_kv positions, batch}; box of
// 64 elements x box_rows positions, 128B swizzle; positions >= n_kv read as zero.
static bool make_kv_map(CUtensorMap* map, const cvattn_tensor& t, int n_kv, int batch, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[3] = {(cuuint64_t)t.n_heads * t.head_dim, (cuuint64_t)n_kv, (cuuint64_t)batch};
    const cuuint64_t strides[2] = {(cuuint64_t)t.nb1, (cuuint64_t)t.nb2};
    const cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
    const cuuint32_t estride[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, t.data, dims, strides, box, estride,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Block-quantized KV tensor as raw bytes for the staged producer's TMA form:
// a 3-D byte map {row bytes, n_kv positions, batch}, box of box_bytes x 64
// positions, no swizzle; positions >= n_kv and bytes past the row read as zero.
static bool make_raw_map(CUtensorMap* map, const cvattn_tensor& t, int n_kv, int batch, int box_bytes) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[3] = {(cuuint64_t)t.n_heads * type_row_bytes(t.type, t.head_dim), (cuuint64_t)n_kv,
                                (cuuint64_t)batch};
    const cuuint64_t strides[2] = {(cuuint64_t)t.nb1, (cuuint64_t)t.nb2};
    const cuuint32_t box[3] = {(cuuint32_t)box_bytes, (cuuint32_t)fp::kBN, 1};
    const cuuint32_t estride[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, t.data, dims, strides, box, estride,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace fa

bool flash_supported(int k_type, int v_type, int head_dim, int n_q_heads, int n_kv_heads) {
    if (!type_known(k_type) || !type_known(v_type) || head_dim != fa::D) return false;
    if (n_kv_heads <= 0 || n_q_heads <= 0 || n_q_heads % n_kv_heads) return false;
    return n_q_heads / n_kv_heads <= 8;
}

cudaError_t launch_flash(cudaStream_t stream, const cvattn_flash_params& a, int* status) {
    using namespace fa;
    Params p{};
    p.q = a.q;
    p.q_nb_tok = a.q_nb_tok;
    p.q_nb_head = a.q_nb_head;
    p.q_nb_batch = a.q_nb_batch;
    p.out = a.out;
    p.k = static_cast<const uint8_t*>(a.k.data);
    p.v = static_cast<const uint8_t*>(a.v.data);
    p.k_nb1 = a.k.nb1;
    p.k_nb2 = a.k.nb2;
    p.v_nb1 = a.v.nb1;
    p.v_nb2 = a.v.nb2;
    p.k_head_bytes = (int)type_row_bytes(a.k.type, a.k.head_dim);
    p.v_head_bytes = (int)type_row_bytes(a.v.type, a.v.head_dim);
    p.n_q = a.n_q;
    p.n_kv = a.n_kv;
    p.Hq = a.n_q_heads;
    p.G = a.n_q_heads / a.k.n_heads;
    p.batch = a.batch;
    p.scale_log2 = a.scale * 1.4426950408889634f;
    p.mask_mode = a.mask_mode;
    p.mask = a.mask;
    p.mask_nb1 = a.mask_nb1;
    p.mask_nb2 = a.mask_nb2;
    p.causal_offset = a.causal_offset;
    p.n_bounds = a.mask_mode == CVATTN_MASK_CHUNK ? a.n_chunk_bounds : 0;
    for (int i = 0; i < p.n_bounds; ++i) p.bounds[i] = a.chunk_bounds[i];
    p.key_offset = a.chunk_key_offset;
    p.row_offset = a.chunk_row_offset;
    p.status = status;
    // Q rows are read as float4: the head row must be 16-byte aligned
    if ((reinterpret_cast<uintptr_t>(a.q) & 15) || (a.q_nb_tok & 3) || (a.q_nb_head & 3) || (a.q_nb_batch & 3))
        return cudaErrorInvalidValue;
    CUtensorMap km, vm;
    memset(&km, 0, sizeof(km));
    memset(&vm, 0, sizeof(vm));
    // TMA path: both caches f16, 16-byte aligned rows and strides
    const bool aligned = ((reinterpret_cast<uintptr_t>(a.k.data) | reinterpret_cast<uintptr_t>(a.v.data)) & 15) == 0 &&
                         ((a.k.nb1 | a.k.nb2 | a.v.nb1 | a.v.nb2) & 15) == 0;
    p.use_tma = 0;
    if (a.k.type == kF16 && a.v.type == kF16 && aligned && a.n_kv > 0) {
        // key tiles: 64 keys for the persistent kernel, 128 for the one-tile kernel
        const int rows = (a.flags & CVATTN_FLASH_ONE_TILE) ? BN : fp::kBN;
        if (make_kv_map(&km, a.k, a.n_kv, a.batch, rows) && make_kv_map(&vm, a.v, a.n_kv, a.batch, rows)) p.use_tma = 1;
    }
    if (!p.use_tma) {
        // plain-load path reads 16-byte chunks of f16/f32 rows
        if ((a.k.type == kF16 || a.k.type == kF32) &&
            ((reinterpret_cast<uintptr_t>(a.k.data) & 15) || (a.k.nb1 & 15) || (a.k.nb2 & 15)))
            return cudaErrorInvalidValue;
        if ((a.v.type == kF16 || a.v.type == kF32) &&
            ((reinterpret_cast<uintptr_t>(a.v.data) & 15) || (a.v.nb1 & 15) || (a.v.nb2 & 15)))
            return cudaErrorInvalidValue;
    }
    // block-quantized K and V with 4-byte aligned rows go through the staged producer
    // (raw rows into shared memory, conversion there); default form: coalesced cp.async
    const bool staged = fp::is_block_quant(a.k.type) && fp::is_block_quant(a.v.type) &&
                        ((reinterpret_cast<uintptr_t>(a.k.data) | reinterpret_cast<uintptr_t>(a.v.data)) & 3) == 0 &&
                        ((a.k.nb1 | a.k.nb2 | a.v.nb1 | a.v.nb2) & 3) == 0;
    p.staged = staged ? fp::kStagedCpAsync : 0;
    if (staged && a.n_kv > 0 && !(a.flags & CVATTN_FLASH_ONE_TILE)) {
        const long k_row = (long)a.k.n_heads * p.k_head_bytes, v_row = (long)a.v.n_heads * p.v_head_bytes;
        const int bk = fp::raw_box_bytes(a.k.type), bv = fp::raw_box_bytes(a.v.type);
        const long chunk_k = (64 * k_row + 127) / 128 * 128, chunk_v = (64 * v_row + 127) / 128 * 128;
        if (aligned && k_row >= bk && v_row >= bv && make_raw_map(&km, a.k, a.n_kv, a.batch, bk) &&
            make_raw_map(&vm, a.v, a.n_kv, a.batch, bv)) {
            // TMA boxes: 16-byte aligned bases and strides (the box x coordinate is the
            // 16-byte boundary below the head's row), rows at least one box wide
            p.staged = fp::kStagedBoxes;
        } else if (((reinterpret_cast<uintptr_t>(a.k.data) | reinterpret_cast<uintptr_t>(a.v.data)) & 15) == 0 &&
                   (a.batch == 1 || ((a.k.nb2 | a.v.nb2) & 15) == 0) && (long)a.k.nb1 == k_row &&
                   (long)a.v.nb1 == v_row && chunk_k + chunk_v <= fp::kChunkRawMax) {
            // bulk copies of whole rows: contiguous rows, 16-byte aligned tile starts
            // (64 rows of a multiple of 4 bytes are a multiple of 256 bytes)
            p.staged = fp::kStagedChunk;
            p.raw_k_bytes = (int)chunk_k;
            p.raw_bytes = (int)(chunk_k + chunk_v);
        }
    }
    if (!(a.flags & CVATTN_FLASH_ONE_TILE)) {
        // persistent kernel: one CTA per SM over the query-tile pairs; the softmax columns
        // split over two warpgroups per query tile unless CVATTN_FLASH_WHOLE_ROWS
        p.halves = (a.flags & CVATTN_FLASH_WHOLE_ROWS) ? 1 : 2;
        const int num_sms = current_sm_count();
        if (num_sms <= 0) return cudaErrorInvalidDevice;
        // the item count of fp::n_items: head pairs for an even G, query-tile pairs otherwise
        const long n_qt = (a.n_q + BM - 1) / BM;
        const bool heads_paired = p.G >= 2 && (p.G & 1) == 0;
        const long items = heads_paired ? n_qt * a.batch * (a.n_q_heads / p.G) * ((p.G + 1) / 2)
                                        : ((n_qt + 1) / 2) * a.batch * a.n_q_heads;
        if (items <= 0) return cudaSuccess;
        const dim3 grid_p((unsigned)(items < num_sms ? items : num_sms));
        switch (a.k.type) {
        case kF32: return fp::launch_for_k<kF32>(stream, a.v.type, p, km, vm, grid_p);
        case kF16: return fp::launch_for_k<kF16>(stream, a.v.type, p, km, vm, grid_p);
        case kQ4_0: return fp::launch_for_k<kQ4_0>(stream, a.v.type, p, km, vm, grid_p);
        case kQ4_1: return fp::launch_for_k<kQ4_1>(stream, a.v.type, p, km, vm, grid_p);
        case kQ5_0: return fp::launch_for_k<kQ5_0>(stream, a.v.type, p, km, vm, grid_p);
        case kQ5_1: return fp::launch_for_k<kQ5_1>(stream, a.v.type, p, km, vm, grid_p);
        case kQ8_0: return fp::launch_for_k<kQ8_0>(stream, a.v.type, p, km, vm, grid_p);
        default: return cudaErrorInvalidValue;
        }
    }
    const dim3 grid((unsigned)((a.n_q + BM - 1) / BM), (unsigned)a.n_q_heads, (unsigned)a.batch);
    switch (a.k.type) {
    case kF32: return launch_for_k<kF32>(stream, a.v.type, p, km, vm, grid);
    case kF16: return launch_for_k<kF16>(stream, a.v.type, p, km, vm, grid);
    case kQ4_0: return launch_for_k<kQ4_0>(stream, a.v.type, p, km, vm, grid);
    case kQ4_1: return launch_for_k<kQ4_1>(stream, a.v.type, p, km, vm, grid);
    case kQ5_0: return launch_for_k<kQ5_0>(stream, a.v.type, p, km, vm, grid);
    case kQ5_1: return launch_for_k<kQ5_1>(stream, a.v.type, p, km, vm, grid);
    case kQ8_0: return launch_for_k<kQ8_0>(stream, a.v.type, p, km, vm, grid);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace cvattn
