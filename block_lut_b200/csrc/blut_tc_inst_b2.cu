// tcgen05 LUT matmul and TC-layout dequantisation for FMT_B 2-bit codes (and the NestedLUT coarse tier).
#include "blut_internal.h"
#include "blut_tc.cuh"

namespace blut {

cudaError_t launch_tc_b2(int group, int group_tokens, const TcParams& p, int sms, cudaStream_t stream) {
  return launch_tc_family<TcDecB2>(group, group_tokens, p, sms, stream);
}

cudaError_t dequant_tc_b2(int group, const TcDequantArgs& a, int64_t nblocks, cudaStream_t stream) {
  return tc_dequant_family<TcDecB2>(group, a, nblocks, stream);
}

}  // namespace blut
