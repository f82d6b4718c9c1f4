// flash_tc.cu -- placeholder until the tcgen05 flash-attention kernel lands.
#include "internal.h"

namespace cvattn {
bool flash_supported(int, int, int, int, int) { return false; }
cudaError_t launch_flash(cudaStream_t, const cvattn_flash_params&, int*) { return cudaErrorNotSupported; }
}  // namespace cvattn
