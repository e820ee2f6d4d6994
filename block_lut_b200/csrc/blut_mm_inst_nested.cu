// NestedLUT instantiations: full tier (coarse + residual codes, combined
// 16-entry tables) and coarse-only tier (the 2-bit lookup on coarse planes).
#include "blut_mm_inst.cuh"

namespace blut {

cudaError_t launch_mm_nested(int group, bool pair, const MMParams& p, int sms, cudaStream_t stream) {
  return launch_by_group<PolNestedFull>(group, pair, p, sms, stream);
}

}  // namespace blut
