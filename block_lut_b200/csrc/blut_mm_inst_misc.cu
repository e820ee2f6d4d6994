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

namespace blut {

int dequant_tiled(const blut_mat_desc& d, const void* tiled, const void* table, void* out, cudaStream_t stream) {
  if (!tiled || !out) return BLUT_ERR_INVALID;
  if (d.layout & BLUT_LAYOUT_TC) return dequant_tiled_tc(d, tiled, table, out, stream);
  MMParams p{};
  if (!mm_planes(d, false, p)) return BLUT_ERR_UNSUPPORTED;
  if (d.format == BLUT_FMT_R8 && !table) return BLUT_ERR_INVALID;
  p.w = static_cast<const uint8_t*>(tiled);
  p.r8_table = static_cast<const uint16_t*>(table);
  uint16_t* o = static_cast<uint16_t*>(out);
  const int pr = (d.layout & BLUT_LAYOUT_PAIRED) ? 1 : 0;
  cudaError_t e;
  switch (d.format) {
    case BLUT_FMT_R8: e = launch_tiled_dequant<PolR8>(p, o, d.cols, pr, stream); break;
    case BLUT_FMT_DENSE:
      e = d.dtype == BLUT_BF16 ? launch_tiled_dequant<PolDense<true>>(p, o, d.cols, pr, stream)
                               : launch_tiled_dequant<PolDense<false>>(p, o, d.cols, pr, stream);
      break;
    case BLUT_FMT_NESTED:
      e = d.tier == 0 ? tiled_dequant_by_group<PolNestedFull>(d.group, p, o, d.cols, pr, stream)
                      : tiled_dequant_by_group<PolB2>(d.group, p, o, d.cols, pr, stream);
      break;
    case BLUT_FMT_B:
      e = d.bits == 4   ? tiled_dequant_by_group<PolB4>(d.group, p, o, d.cols, pr, stream)
          : d.bits == 3 ? tiled_dequant_by_group<PolB3>(d.group, p, o, d.cols, pr, stream)
                        : tiled_dequant_by_group<PolB2>(d.group, p, o, d.cols, pr, stream);
      break;
    default: return BLUT_ERR_UNSUPPORTED;
  }
  return e == cudaSuccess ? BLUT_OK : BLUT_ERR_LAUNCH;
}

}  // namespace blut
