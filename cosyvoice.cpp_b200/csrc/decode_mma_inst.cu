// decode_mma_inst.cu -- instantiates decode_mma_kernel for one K type
// (CVATTN_KT) and every block-quantized V type; compiled once per K type.
#include "decode_mma.cuh"

#ifndef CVATTN_KT
#error "compile with -DCVATTN_KT=<ggml type id>"
#endif

namespace cvattn {
namespace dmma {

// Launch over min(sm_count, ceil(items / pairs)) CTAs of `pairs` warp pairs, with
// programmatic stream serialization: the kernel waits (griddepcontrol.wait)
// before it reads an input the previous kernel may still write.
template <int KT, int VT>
static cudaError_t run(cudaStream_t s, const Args& a, int n_sms) {
    auto fn = decode_mma_kernel<KT, VT>;
    const int rowK = (int)type_row_bytes(KT, 2 * kD), rowV = (int)type_row_bytes(VT, 2 * kD);
    const long items = (long)a.n_seq * ((a.max_kv_len + kC - 1) / kC);
    int pairs = 1, grid = 1;
    launch_shape(KT, VT, items, n_sms, pairs, grid);
    const int smem = Smem(rowK, rowV, pairs, BlockTraits<KT>::HAS_MIN, BlockTraits<VT>::HAS_MIN).total;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3((unsigned)(64 * pairs));
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
cudaError_t launch_for_k<CVATTN_KT>(cudaStream_t s, const Args& a, int vt, int n_sms) {
    switch (vt) {
    case kQ4_0: return run<CVATTN_KT, kQ4_0>(s, a, n_sms);
    case kQ4_1: return run<CVATTN_KT, kQ4_1>(s, a, n_sms);
    case kQ5_0: return run<CVATTN_KT, kQ5_0>(s, a, n_sms);
    case kQ5_1: return run<CVATTN_KT, kQ5_1>(s, a, n_sms);
    case kQ8_0: return run<CVATTN_KT, kQ8_0>(s, a, n_sms);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace dmma
}  // namespace cvattn
