// FMT_B 4-bit instantiations of the LUT matmul (table blocks 32/64/128).
#include "blut_mm_inst.cuh"

namespace blut {

cudaError_t launch_mm_b4(int group, bool pair, const MMParams& p, int sms, cudaStream_t stream) {
  return launch_by_group<PolB4>(group, pair, p, sms, stream);
}

}  // namespace blut
