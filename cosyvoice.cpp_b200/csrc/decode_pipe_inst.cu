// decode_pipe_inst.cu -- instantiates decode_pipe_kernel for one K type
// (CVATTN_KT) and every block-quantized V type; compiled once per K type.
#include "decode_pipe.cuh"

#ifndef CVATTN_KT
#error "compile with -DCVATTN_KT=<ggml type id>"
#endif

namespace cvattn {
namespace dpipe {

template <int KT, int VT>
static cudaError_t run(cudaStream_t s, const Args& a, dim3 grid) {
    auto fn = decode_pipe_kernel<KT, VT>;
    const int smem = smem_bytes(KT, VT);
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    fn<<<grid, kThreads, smem, s>>>(a);
    return cudaGetLastError();
}

template <>
cudaError_t launch_for_k<CVATTN_KT>(cudaStream_t s, const Args& a, int vt, dim3 grid) {
    switch (vt) {
    case kQ4_0: return run<CVATTN_KT, kQ4_0>(s, a, grid);
    case kQ4_1: return run<CVATTN_KT, kQ4_1>(s, a, grid);
    case kQ5_0: return run<CVATTN_KT, kQ5_0>(s, a, grid);
    case kQ5_1: return run<CVATTN_KT, kQ5_1>(s, a, grid);
    case kQ8_0: return run<CVATTN_KT, kQ8_0>(s, a, grid);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace dpipe
}  // namespace cvattn
