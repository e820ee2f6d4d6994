// FMT_B 2-bit instantiations of the LUT matmul (table blocks 32/64/128).
#include "blut_mm_inst.cuh"

namespace blut {

cudaError_t launch_mm_b2(int group, bool pair, const MMParams& p, int sms, cudaStream_t stream) {
  return launch_by_group<PolB2>(group, pair, p, sms, stream);
}

}  // namespace blut
