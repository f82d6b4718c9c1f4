// internal.h -- launchers shared between the kernel files and the C-ABI layer.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/cvattn.h"

namespace cvattn {

// Device form of a RoPE (csrc/rope.cuh): theta_scale = powf(freq_base, -2 / n_dims).
struct RopeDev {
    int mode;        // 0 NORMAL (pairs 2k, 2k + 1), 2 NEOX (pairs k, k + n_dims / 2)
    int n_dims;      // rotated prefix of each unit; 0 = no rotation
    int unit_len;    // elements per rotation unit (a head, or the whole row)
    float theta_scale, freq_scale, attn_factor;
};

// kv_append.cu (rope: null for none)
cudaError_t launch_kv_append(cudaStream_t stream, const cvattn_tensor& cache, const float* src, int64_t src_nb1,
                             int64_t src_nb2, const int32_t* pos, int64_t pos_stride, int n_new, int batch,
                             int* status, const RopeDev* rope = nullptr);
cudaError_t launch_rope(cudaStream_t stream, const RopeDev& rope, const float* x, int64_t x_nb1f, float* out,
                        int64_t out_nb1f, const int32_t* pos, int n_rows, int row_len);
cudaError_t launch_kv_dequant(cudaStream_t stream, const cvattn_tensor& cache, int n_rows, float* dst);

// kv_append.cu: per-device SM count (looked up once per device, thread-safe)
int device_sm_count(int device);
// The current device's SM count (0 if the runtime cannot say).
int current_sm_count();
// Fill n int32 lengths with one value and zero n_tickets 32-bit ticket counters
// (one launch; either count may be 0).
cudaError_t launch_fill_lengths(cudaStream_t stream, int32_t* lens, int n, int32_t value, uint32_t* tickets,
                                int n_tickets);

// decode.cu
int decode_chunk_positions(int k_type, int v_type, int n_kv_heads, int head_dim);
// Bytes of the ticket block that leads a decode workspace: one 32-bit counter
// per (sequence, KV head), 256-byte aligned.
size_t decode_ticket_bytes(int n_seq, int n_kv_heads);
size_t decode_workspace_bytes(int k_type, int v_type, int n_seq, int max_kv_len, int n_q_heads, int n_kv_heads, int head_dim);
bool decode_supported(int k_type, int v_type, int head_dim, int n_q_heads, int n_kv_heads);
cudaError_t launch_decode(cudaStream_t stream, const cvattn_decode_params& p, int* status,
                          const RopeDev* rope = nullptr);
// whether launch_decode can apply a RoPE to Q and the appended K row (the streaming kernel)
bool decode_rope_supported(const cvattn_decode_params& p);
cudaError_t launch_combine(cudaStream_t stream, const float* partial_o, const float* partial_ml, int n_parts,
                           int n_rows, int head_dim, float* out);

// flash_tc.cu
bool flash_supported(int k_type, int v_type, int head_dim, int n_q_heads, int n_kv_heads);
cudaError_t launch_flash(cudaStream_t stream, const cvattn_flash_params& p, int* status);

}  // namespace cvattn
