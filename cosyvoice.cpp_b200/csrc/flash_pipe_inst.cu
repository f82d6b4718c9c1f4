// flash_pipe_inst.cu -- instantiates flash_pipe_kernel for one K type (CVATTN_KT) and
// every V type; compiled once per K type so the 49 type pairs build in parallel.
#include "flash_pipe.cuh"

#ifndef CVATTN_KT
#error "compile with -DCVATTN_KT=<ggml type id>"
#endif

namespace cvattn {
namespace fp {

template <int KT, int VT, int H>
static cudaError_t run_h(cudaStream_t s, const Params& p, const CUtensorMap& km, const CUtensorMap& vm, dim3 grid) {
    auto fn = flash_pipe_kernel<KT, VT, H>;
    int smem = smem_bytes(KT, VT);
    if (p.staged == kStagedChunk && kRawOff + 2 * p.raw_bytes > smem) smem = kRawOff + 2 * p.raw_bytes;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    fn<<<grid, Shape<H>::kThreads, smem, s>>>(p, km, vm);
    return cudaGetLastError();
}

template <int KT, int VT>
static cudaError_t run(cudaStream_t s, const Params& p, const CUtensorMap& km, const CUtensorMap& vm, dim3 grid) {
    return p.halves == 2 ? run_h<KT, VT, 2>(s, p, km, vm, grid) : run_h<KT, VT, 1>(s, p, km, vm, grid);
}

template <>
cudaError_t launch_for_k<CVATTN_KT>(cudaStream_t s, int vt, const Params& p, const CUtensorMap& km,
                                    const CUtensorMap& vm, dim3 grid) {
    switch (vt) {
    case kF32: return run<CVATTN_KT, kF32>(s, p, km, vm, grid);
    case kF16: return run<CVATTN_KT, kF16>(s, p, km, vm, grid);
    case kQ4_0: return run<CVATTN_KT, kQ4_0>(s, p, km, vm, grid);
    case kQ4_1: return run<CVATTN_KT, kQ4_1>(s, p, km, vm, grid);
    case kQ5_0: return run<CVATTN_KT, kQ5_0>(s, p, km, vm, grid);
    case kQ5_1: return run<CVATTN_KT, kQ5_1>(s, p, km, vm, grid);
    case kQ8_0: return run<CVATTN_KT, kQ8_0>(s, p, km, vm, grid);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace fp
}  // namespace cvattn
