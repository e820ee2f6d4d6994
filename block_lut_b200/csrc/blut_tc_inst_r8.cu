// tcgen05 LUT matmul and TC-layout dequantisation for FMT_R8 (the
// reference's BlockLUT: uint8 indices, bf16 table, bf16 absmax).
#include "blut_internal.h"
#include "blut_tc.cuh"

namespace blut {

cudaError_t launch_tc_r8(int group_tokens, const TcParams& p, int sms, cudaStream_t stream) {
  if (group_tokens == 1) return launch_tc_gemv<TcDecR8>(p, p.gemv_groups, stream);
  if (group_tokens == 32) return launch_tc<TcDecR8, 32>(p, sms, stream);
  if (group_tokens == 128) return launch_tc<TcDecR8, 128>(p, sms, stream);
  return cudaErrorInvalidValue;
}

cudaError_t dequant_tc_r8(const TcDequantArgs& a, int64_t nblocks, cudaStream_t stream) {
  return tc_dequant_launch<TcDecR8>(a, nblocks, stream);
}

}  // namespace blut
