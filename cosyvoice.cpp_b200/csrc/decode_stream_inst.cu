// decode_stream_inst.cu -- instantiates decode_stream_kernel for one K type
// (CVATTN_KT) and every block-quantized V type; compiled once per K type.
#include "decode_stream.cuh"

#ifndef CVATTN_KT
#error "compile with -DCVATTN_KT=<ggml type id>"
#endif

namespace cvattn {
namespace dstream {

template <int KT, int VT>
static cudaError_t run(cudaStream_t s, const Args& a, dim3 grid) {
    auto fn = decode_stream_kernel<KT, VT>;
    const int smem = smem_bytes(KT, VT);
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    // programmatic stream serialization: the launch may begin while the previous kernel
    // finishes; the kernel waits (griddepcontrol.wait) before it touches any input
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, fn, a);
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

}  // namespace dstream
}  // namespace cvattn
