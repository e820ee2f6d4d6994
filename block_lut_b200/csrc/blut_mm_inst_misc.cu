// FMT_R8 (reference format) and dense (shared expert) instantiations, and
// the format dispatch of the LUT matmul.
#include "blut_mm_inst.cuh"

namespace blut {

cudaError_t launch_mm_r8(bool pair, const MMParams& p, int sms, cudaStream_t stream) {
  return launch_pair_or_single<PolR8>(pair, p, sms, stream);
}

cudaError_t launch_mm_dense(bool bf16, bool pair, const MMParams& p, int sms, cudaStream_t stream) {
  return bf16 ? launch_pair_or_single<PolDense<true>>(pair, p, sms, stream)
              : launch_pair_or_single<PolDense<false>>(pair, p, sms, stream);
}

cudaError_t launch_lut_mm(const blut_mat_desc& d, bool pair, const MMParams& p, int sms, cudaStream_t stream) {
  switch (d.format) {
    case BLUT_FMT_R8: return launch_mm_r8(pair, p, sms, stream);
    case BLUT_FMT_DENSE: return launch_mm_dense(d.dtype == BLUT_BF16, pair, p, sms, stream);
    case BLUT_FMT_NESTED:
      return d.tier == 0 ? launch_mm_nested(d.group, pair, p, sms, stream)
                         : launch_mm_b2(d.group, pair, p, sms, stream);
    case BLUT_FMT_B:
      if (d.bits == 4) return launch_mm_b4(d.group, pair, p, sms, stream);
      if (d.bits == 3) return launch_mm_b3(d.group, pair, p, sms, stream);
      if (d.bits == 2) return launch_mm_b2(d.group, pair, p, sms, stream);
      return cudaErrorInvalidValue;
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace blut
