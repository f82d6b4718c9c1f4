// decode_inst.cu -- instantiates decode_kernel for one K type (CVATTN_KT) and
// every V type; compiled once per K type so the 49 type pairs build in parallel.
#include "decode.cuh"

#ifndef CVATTN_KT
#error "compile with -DCVATTN_KT=<ggml type id>"
#endif

namespace cvattn {
namespace dec {

template <int KT, int VT, int GT>
static cudaError_t run(cudaStream_t s, const Args& a, dim3 grid, int smem) {
    auto fn = decode_kernel<KT, VT, GT>;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    fn<<<grid, kThreads, smem, s>>>(a);
    return cudaGetLastError();
}

template <>
cudaError_t launch_for_k<CVATTN_KT>(cudaStream_t s, const Args& a, int v_type, dim3 grid, int smem) {
    const bool g7 = a.G == 7;
#define CVATTN_V_CASE(VT) \
    case VT: return g7 ? run<CVATTN_KT, VT, 7>(s, a, grid, smem) : run<CVATTN_KT, VT, 8>(s, a, grid, smem);
    switch (v_type) {
        CVATTN_V_CASE(kF32)
        CVATTN_V_CASE(kF16)
        CVATTN_V_CASE(kQ4_0)
        CVATTN_V_CASE(kQ4_1)
        CVATTN_V_CASE(kQ5_0)
        CVATTN_V_CASE(kQ5_1)
        CVATTN_V_CASE(kQ8_0)
    default: return cudaErrorInvalidValue;
    }
#undef CVATTN_V_CASE
}

}  // namespace dec
}  // namespace cvattn
