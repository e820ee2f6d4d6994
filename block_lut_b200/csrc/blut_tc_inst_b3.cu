// tcgen05 LUT matmul and TC-layout dequantisation for FMT_B 3-bit codes.
#include "blut_internal.h"
#include "blut_tc.cuh"

namespace blut {

cudaError_t launch_tc_b3(int group, int group_tokens, const TcParams& p, int sms, cudaStream_t stream) {
  return launch_tc_family<TcDecB3>(group, group_tokens, p, sms, stream);
}

cudaError_t dequant_tc_b3(int group, const TcDequantArgs& a, int64_t nblocks, cudaStream_t stream) {
  return tc_dequant_family<TcDecB3>(group, a, nblocks, stream);
}

}  // namespace blut
