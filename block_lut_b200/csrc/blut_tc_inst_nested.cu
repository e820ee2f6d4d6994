// tcgen05 LUT matmul and TC-layout dequantisation for NestedLUT, full tier.
#include "blut_internal.h"
#include "blut_tc.cuh"

namespace blut {

cudaError_t launch_tc_nested(int group, int group_tokens, const TcParams& p, int sms, cudaStream_t stream) {
  return launch_tc_family<TcDecNested>(group, group_tokens, p, sms, stream);
}

cudaError_t dequant_tc_nested(int group, const TcDequantArgs& a, int64_t nblocks, cudaStream_t stream) {
  return tc_dequant_family<TcDecNested>(group, a, nblocks, stream);
}

}  // namespace blut
