// decode.cu -- host side of the split-KV decode kernel (decode.cuh) and the
// standalone log-sum-exp combine used for cross-GPU split-KV partials.
#include "decode.cuh"
#include "decode_mma.cuh"
#include "decode_pipe.cuh"
#include "decode_stream.cuh"
#include "decode_tc.cuh"
#include "internal.h"
#include "rope.cuh"

namespace cvattn {

using namespace dec;

static int smem_for(int C, int k_type, int v_type, int Hkv) {
    const int rowK = (int)type_row_bytes(k_type, (int64_t)Hkv * kD);
    const int rowV = (int)type_row_bytes(v_type, (int64_t)Hkv * kD);
    const bool vmin = v_type == kQ4_1 || v_type == kQ5_1;
    return Smem(C, Hkv, rowK, rowV, vmin).total;
}

// Positions per CTA: 128 while the chunk fits the shared-memory budget, else
// halved (f16/f32 rows are 2-4x larger than q8_0 rows).
int decode_chunk_positions(int k_type, int v_type, int n_kv_heads, int head_dim) {
    if (head_dim != kD) return 0;
    for (int C = 128; C >= 32; C >>= 1)
        if (smem_for(C, k_type, v_type, n_kv_heads) <= 160 * 1024) return C;
    return 0;
}

bool decode_supported(int k_type, int v_type, int head_dim, int n_q_heads, int n_kv_heads) {
    if (!type_known(k_type) || !type_known(v_type) || head_dim != kD) return false;
    if (n_kv_heads <= 0 || n_q_heads <= 0 || n_q_heads % n_kv_heads) return false;
    if (n_q_heads / n_kv_heads > kHP) return false;
    return decode_chunk_positions(k_type, v_type, n_kv_heads, head_dim) > 0;
}

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

size_t decode_ticket_bytes(int n_seq, int n_kv_heads) {
    return align256((size_t)n_seq * (size_t)(n_kv_heads > 2 ? n_kv_heads : 2) * 4);
}

size_t decode_workspace_bytes(int k_type, int v_type, int n_seq, int max_kv_len, int n_q_heads, int n_kv_heads,
                              int head_dim) {
    int C = decode_chunk_positions(k_type, v_type, n_kv_heads, head_dim);
    if (C == 0 || n_seq <= 0 || max_kv_len < 0) return 0;
    if (C > dstream::kC) C = dstream::kC;  // partial slots for the 64-position items
    const size_t chunks = (size_t)((max_kv_len + C - 1) / C);
    return decode_ticket_bytes(n_seq, n_kv_heads) + align256((size_t)n_seq * chunks * n_q_heads * 2 * 4) +
           align256((size_t)n_seq * chunks * n_q_heads * kD * 4);
}

bool decode_rope_supported(const cvattn_decode_params& p) {
    const int Hkv = p.k.n_heads;
    const int G = Hkv > 0 ? p.n_q_heads / Hkv : 0;
    return !(p.flags & (CVATTN_DECODE_CUDA_CORES | CVATTN_DECODE_NOT_PERSISTENT | CVATTN_DECODE_WIDE_CHUNKS)) &&
           Hkv == 2 && p.k.head_dim == kD && G >= 1 && G <= dtc::kHP && dstream::supported_type(p.k.type) &&
           dstream::supported_type(p.v.type) && p.n_seq <= dstream::kMaxSeq &&
           dstream::smem_bytes(p.k.type, p.v.type) <= 227 * 1024;
}

cudaError_t launch_decode(cudaStream_t stream, const cvattn_decode_params& p, int* status, const RopeDev* rope) {
    const int Hkv = p.k.n_heads;
    const int C = decode_chunk_positions(p.k.type, p.v.type, Hkv, p.k.head_dim);
    const int chunks = (p.max_kv_len + C - 1) / C;
    Args a{};
    a.q = p.q;
    a.q_seq_stride = p.q_seq_stride;
    a.out = p.out;
    a.out_seq_stride = p.out_seq_stride;
    a.k_base = static_cast<const uint8_t*>(p.k.data);
    a.v_base = static_cast<const uint8_t*>(p.v.data);
    a.k_nb2 = p.k.nb2;
    a.v_nb2 = p.v.nb2;
    a.capacity = p.k.ne1 < p.v.ne1 ? p.k.ne1 : p.v.ne1;
    a.k_seq_ptrs = p.k_seq_ptrs;
    a.v_seq_ptrs = p.v_seq_ptrs;
    a.kv_len = p.kv_len;
    a.k_new = p.k_new;
    a.v_new = p.v_new;
    a.partial_ml = p.partial_ml;
    a.n_seq = p.n_seq;
    a.Hq = p.n_q_heads;
    a.Hkv = Hkv;
    a.G = p.n_q_heads / Hkv;
    a.C = C;
    a.flags = p.flags;
    a.max_kv_len = p.max_kv_len;
    a.scale_log2 = p.scale * 1.4426950408889634f;
    if (rope) {
        a.rope_mode = rope->mode;
        a.rope_n_dims = rope->n_dims;
        a.rope_theta_scale = rope->theta_scale;
        a.rope_freq_scale = rope->freq_scale;
        a.rope_attn_factor = rope->attn_factor;
    }
    uint8_t* ws = static_cast<uint8_t*>(p.workspace);
    const size_t cnt_bytes = decode_ticket_bytes(p.n_seq, Hkv);
    const size_t ml_bytes = align256((size_t)p.n_seq * chunks * p.n_q_heads * 2 * 4);
    a.ws_cnt = reinterpret_cast<uint32_t*>(ws);
    a.ws_ml = reinterpret_cast<float*>(ws + cnt_bytes);
    a.ws_o = reinterpret_cast<float*>(ws + cnt_bytes + ml_bytes);
    a.ws_chunks = chunks;
    a.status = status;
    // tensor-core paths: Qwen2 shape (2 KV heads, D 64), block-quantized or f16 K/V
    if (!(p.flags & CVATTN_DECODE_CUDA_CORES) && Hkv == 2 && p.k.head_dim == kD && a.G <= dtc::kHP &&
        dtc::supported_type(p.k.type) && dtc::supported_type(p.v.type)) {
        const int chunks_tc = (p.max_kv_len + dtc::kC - 1) / dtc::kC;
        a.C = dtc::kC;
        a.ws_chunks = chunks_tc;
        a.ws_ml = reinterpret_cast<float*>(ws + cnt_bytes);
        a.ws_o = reinterpret_cast<float*>(ws + cnt_bytes + align256((size_t)p.n_seq * chunks_tc * p.n_q_heads * 2 * 4));
        // persistent pipelined kernel when its ring of stages fits one SM
        const int num_sms = current_sm_count();
        const bool persistent = !(p.flags & CVATTN_DECODE_NOT_PERSISTENT) && num_sms > 0;
        // The register-resident warp-MMA kernel takes every launch of at least one
        // 64-position item per SM (for the host bound max_kv_len) whose sequences split over
        // at most 128 warp pairs each, and every throughput-bound launch (dmma::mma_pays);
        // smaller launches (one to a few long sequences) run the TMEM streaming kernel, whose
        // per-item pipeline is shorter.  CVATTN_DECODE_WARP_MMA / CVATTN_DECODE_TMEM_STREAM force
        // either.  Both apply the RoPE of the fused step.
        const long items_bound = (long)p.n_seq * ((p.max_kv_len + dmma::kC - 1) / dmma::kC);
        const bool want_mma = (p.flags & CVATTN_DECODE_WARP_MMA) ||
                              (!(p.flags & CVATTN_DECODE_TMEM_STREAM) &&
                               dmma::mma_pays(p.k.type, p.v.type, p.n_seq, items_bound, num_sms));
        if (persistent && want_mma && !(p.flags & CVATTN_DECODE_WIDE_CHUNKS) &&
            dmma::supported_type(p.k.type) && dmma::supported_type(p.v.type) && p.n_seq <= dmma::kMaxSeq) {
            const int chunks_s = (p.max_kv_len + dmma::kC - 1) / dmma::kC;
            Args b = a;
            b.C = dmma::kC;
            b.ws_chunks = chunks_s;
            b.ws_ml = reinterpret_cast<float*>(ws + cnt_bytes);
            b.ws_o = reinterpret_cast<float*>(ws + cnt_bytes + align256((size_t)p.n_seq * chunks_s * p.n_q_heads * 2 * 4));
            switch (p.k.type) {
            case kQ4_0: return dmma::launch_for_k<kQ4_0>(stream, b, p.v.type, num_sms);
            case kQ4_1: return dmma::launch_for_k<kQ4_1>(stream, b, p.v.type, num_sms);
            case kQ5_0: return dmma::launch_for_k<kQ5_0>(stream, b, p.v.type, num_sms);
            case kQ5_1: return dmma::launch_for_k<kQ5_1>(stream, b, p.v.type, num_sms);
            case kQ8_0: return dmma::launch_for_k<kQ8_0>(stream, b, p.v.type, num_sms);
            default: break;
            }
        }
        if (persistent && !(p.flags & CVATTN_DECODE_WIDE_CHUNKS) && dstream::supported_type(p.k.type) &&
            dstream::supported_type(p.v.type) && p.n_seq <= dstream::kMaxSeq &&
            dstream::smem_bytes(p.k.type, p.v.type) <= 227 * 1024) {
            // streaming kernel: 64-position items, partial slots per 64 positions
            const int chunks_s = (p.max_kv_len + dstream::kC - 1) / dstream::kC;
            Args b = a;
            b.C = dstream::kC;
            b.ws_chunks = chunks_s;
            b.ws_ml = reinterpret_cast<float*>(ws + cnt_bytes);
            b.ws_o = reinterpret_cast<float*>(ws + cnt_bytes + align256((size_t)p.n_seq * chunks_s * p.n_q_heads * 2 * 4));
            const long items = (long)p.n_seq * (chunks_s > 0 ? chunks_s : 1);
            const dim3 grid_s((unsigned)(items < num_sms ? items : num_sms));
            switch (p.k.type) {
            case kQ4_0: return dstream::launch_for_k<kQ4_0>(stream, b, p.v.type, grid_s);
            case kQ4_1: return dstream::launch_for_k<kQ4_1>(stream, b, p.v.type, grid_s);
            case kQ5_0: return dstream::launch_for_k<kQ5_0>(stream, b, p.v.type, grid_s);
            case kQ5_1: return dstream::launch_for_k<kQ5_1>(stream, b, p.v.type, grid_s);
            case kQ8_0: return dstream::launch_for_k<kQ8_0>(stream, b, p.v.type, grid_s);
            default: break;
            }
        }
        if (a.rope_n_dims > 0) return cudaErrorNotSupported;  // only the two kernels above apply a RoPE
        if (persistent && dpipe::supported_type(p.k.type) &&
            dpipe::supported_type(p.v.type) && p.n_seq <= dpipe::kMaxSeq &&
            dpipe::smem_bytes(p.k.type, p.v.type) <= 227 * 1024) {
            const long items = (long)p.n_seq * (chunks_tc > 0 ? chunks_tc : 1);
            const dim3 grid_p((unsigned)(items < num_sms ? items : num_sms));
            switch (p.k.type) {
            case kQ4_0: return dpipe::launch_for_k<kQ4_0>(stream, a, p.v.type, grid_p);
            case kQ4_1: return dpipe::launch_for_k<kQ4_1>(stream, a, p.v.type, grid_p);
            case kQ5_0: return dpipe::launch_for_k<kQ5_0>(stream, a, p.v.type, grid_p);
            case kQ5_1: return dpipe::launch_for_k<kQ5_1>(stream, a, p.v.type, grid_p);
            case kQ8_0: return dpipe::launch_for_k<kQ8_0>(stream, a, p.v.type, grid_p);
            default: break;
            }
        }
        const dim3 grid_tc((unsigned)(chunks_tc > 0 ? chunks_tc : 1), (unsigned)p.n_seq);
        switch (p.k.type) {
        case kF16: return dtc::launch_for_k<kF16>(stream, a, p.v.type, grid_tc);
        case kQ4_0: return dtc::launch_for_k<kQ4_0>(stream, a, p.v.type, grid_tc);
        case kQ4_1: return dtc::launch_for_k<kQ4_1>(stream, a, p.v.type, grid_tc);
        case kQ5_0: return dtc::launch_for_k<kQ5_0>(stream, a, p.v.type, grid_tc);
        case kQ5_1: return dtc::launch_for_k<kQ5_1>(stream, a, p.v.type, grid_tc);
        case kQ8_0: return dtc::launch_for_k<kQ8_0>(stream, a, p.v.type, grid_tc);
        default: return cudaErrorInvalidValue;
        }
    }
    const int smem = smem_for(C, p.k.type, p.v.type, Hkv);
    const dim3 grid((unsigned)(chunks > 0 ? chunks : 1), (unsigned)p.n_seq);
    switch (p.k.type) {
    case kF32: return launch_for_k<kF32>(stream, a, p.v.type, grid, smem);
    case kF16: return launch_for_k<kF16>(stream, a, p.v.type, grid, smem);
    case kQ4_0: return launch_for_k<kQ4_0>(stream, a, p.v.type, grid, smem);
    case kQ4_1: return launch_for_k<kQ4_1>(stream, a, p.v.type, grid, smem);
    case kQ5_0: return launch_for_k<kQ5_0>(stream, a, p.v.type, grid, smem);
    case kQ5_1: return launch_for_k<kQ5_1>(stream, a, p.v.type, grid, smem);
    case kQ8_0: return launch_for_k<kQ8_0>(stream, a, p.v.type, grid, smem);
    default: return cudaErrorInvalidValue;
    }
}

// ---------------------------------------------------------------- combine --
// out[r] = sum_p 2^(m_p - M) O_p[r] / sum_p 2^(m_p - M) l_p, M = max_p m_p.
// One warp per row; lanes cover head_dim in pairs.
__global__ void __launch_bounds__(256) combine_kernel(const float* __restrict__ po, const float* __restrict__ pml,
                                                      int n_parts, int n_rows, int D, float* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (row >= n_rows) return;
    float M = -INFINITY;
    for (int pp = 0; pp < n_parts; ++pp) M = fmaxf(M, pml[((int64_t)pp * n_rows + row) * 2]);
    float Ls = 0.0f;
    for (int pp = 0; pp < n_parts; ++pp) {
        const float m = pml[((int64_t)pp * n_rows + row) * 2];
        if (m != -INFINITY) Ls += fast_exp2(m - M) * pml[((int64_t)pp * n_rows + row) * 2 + 1];
    }
    const float inv = Ls > 0.0f ? 1.0f / Ls : 0.0f;
    for (int d = lane; d < D; d += 32) {
        float acc = 0.0f;
        for (int pp = 0; pp < n_parts; ++pp) {
            const float m = pml[((int64_t)pp * n_rows + row) * 2];
            if (m != -INFINITY) acc = fmaf(fast_exp2(m - M), po[((int64_t)pp * n_rows + row) * D + d], acc);
        }
        out[(int64_t)row * D + d] = acc * inv;
    }
}

cudaError_t launch_combine(cudaStream_t stream, const float* partial_o, const float* partial_ml, int n_parts,
                           int n_rows, int head_dim, float* out) {
    if (n_rows == 0) return cudaSuccess;
    combine_kernel<<<(n_rows + 7) / 8, 256, 0, stream>>>(partial_o, partial_ml, n_parts, n_rows, head_dim, out);
    return cudaGetLastError();
}

}  // namespace cvattn
