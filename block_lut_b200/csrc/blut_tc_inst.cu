// Instantiations of the tcgen05 LUT matmul for FMT_B 4-bit and dense
// weights, the dispatch over every format of the TC layout, and the
// diagnostic dequantisation of that layout through the same decode.  The
// 2-bit, 3-bit, NestedLUT and FMT_R8 families are instantiated in their own
// translation units (blut_tc_inst_{b2,b3,nested,r8}.cu).
#include "blut_internal.h"
#include "blut_tc.cuh"

namespace blut {

bool tc_planes(const blut_mat_desc& d, bool pair, TcParams& p) {
  TiledLayout L;
  if (!make_layout(d, L) || !L.tc) return false;
  int idx[3];
  const int np = plane_select(d, L, idx);
  p.nplanes = np;
  p.tile_bytes = 0;
  for (int q = 0; q < 3; ++q) {
    p.plane_off[q] = q < np ? L.off[idx[q]] : 0;
    p.piece[q] = q < np ? (int)L.piece[idx[q]] : 0;
    p.tile_bytes += p.piece[q];
  }
  p.ntiles = (int)L.ntiles;
  p.nblocks = (int)L.nchunks;
  p.units = (p.ntiles + 1) / 2;
  p.pair = pair ? 1 : 0;
  p.mul = tc_mul_consts(d.format == BLUT_FMT_R8 ? d.tier : 0);
  return true;
}

template <int MT>
static cudaError_t launch_tc_dense(const blut_mat_desc& d, const TcParams& p, int sms, cudaStream_t stream) {
  return d.dtype == BLUT_BF16 ? launch_tc<TcDecDense<true>, MT>(p, sms, stream)
                              : launch_tc<TcDecDense<false>, MT>(p, sms, stream);
}

// Column blocks per small-batch GEMV item: the blocks holding the pieces a
// thread keeps in flight (tc_gemv_pf), at least one.
int tc_gemv_blocks(const blut_mat_desc& d) {
  int pf = 4, kb = tc_block_cols(d.format, d.group);
  switch (d.format) {
    case BLUT_FMT_DENSE: return 4;
    case BLUT_FMT_R8: pf = tc_gemv_pf<TcDecR8>(); break;
    case BLUT_FMT_NESTED:
      pf = d.tier == 1 ? tc_gemv_pf<TcDecB2<64>>()
                       : (d.group == 32 ? tc_gemv_pf<TcDecNested<32>>() : tc_gemv_pf<TcDecNested<64>>());
      break;
    case BLUT_FMT_B:
      pf = d.bits == 4 ? (d.group == 32 ? tc_gemv_pf<TcDecB4<32>>() : tc_gemv_pf<TcDecB4<64>>())
         : d.bits == 3 ? (d.group == 32 ? tc_gemv_pf<TcDecB3<32>>() : tc_gemv_pf<TcDecB3<64>>())
                       : tc_gemv_pf<TcDecB2<64>>();
      break;
  }
  return std::max(1, pf * 64 / kb);
}

// group_tokens: 32 or 128 (tcgen05 matmul), 1 (small-batch GEMV).
cudaError_t launch_tc_mm(const blut_mat_desc& d, const TcParams& p, int group_tokens, int sms, cudaStream_t stream) {
  if (group_tokens != 32 && group_tokens != 128 && group_tokens != 1) return cudaErrorInvalidValue;
  switch (d.format) {
    case BLUT_FMT_DENSE:
      if (group_tokens == 1)
        return d.dtype == BLUT_BF16 ? launch_tc_gemv<TcDecDense<true>>(p, p.gemv_groups, stream)
                                    : launch_tc_gemv<TcDecDense<false>>(p, p.gemv_groups, stream);
      return group_tokens == 32 ? launch_tc_dense<32>(d, p, sms, stream) : launch_tc_dense<128>(d, p, sms, stream);
    case BLUT_FMT_B:
      if (d.bits == 4) return launch_tc_family<TcDecB4>(d.group, group_tokens, p, sms, stream);
      if (d.bits == 3) return launch_tc_b3(d.group, group_tokens, p, sms, stream);
      if (d.bits == 2) return launch_tc_b2(d.group, group_tokens, p, sms, stream);
      break;
    case BLUT_FMT_NESTED:  // the coarse tier is a 2-bit lookup of planes 0, 1
      return d.tier == 1 ? launch_tc_b2(d.group, group_tokens, p, sms, stream)
                         : launch_tc_nested(d.group, group_tokens, p, sms, stream);
    case BLUT_FMT_R8:
      return p.r8_table ? launch_tc_r8(group_tokens, p, sms, stream) : cudaErrorInvalidValue;
  }
  return cudaErrorInvalidValue;
}

int dequant_tiled_tc(const blut_mat_desc& d, const void* tiled, const void* r8_table, void* out,
                     cudaStream_t stream) {
  TiledLayout L;
  if (!make_layout(d, L) || !L.tc) return BLUT_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(tiled) | reinterpret_cast<uintptr_t>(out)) & 15) return BLUT_ERR_INVALID;
  TcDequantArgs a{};
  a.w = static_cast<const uint8_t*>(tiled);
  int idx[3];
  const int np = plane_select(d, L, idx);
  for (int q = 0; q < 3; ++q) {
    a.off[q] = q < np ? L.off[idx[q]] : 0;
    a.piece[q] = q < np ? (int)L.piece[idx[q]] : 0;
  }
  a.ntiles = (int)L.ntiles;
  a.cols = d.cols;
  a.paired = (d.layout & BLUT_LAYOUT_PAIRED) ? 1 : 0;
  a.out = static_cast<uint16_t*>(out);
  a.mul = tc_mul_consts(d.format == BLUT_FMT_R8 ? d.tier : 0);
  a.r8_table = static_cast<const uint16_t*>(r8_table);
  cudaError_t e = cudaErrorInvalidValue;
  switch (d.format) {
    case BLUT_FMT_DENSE:
      e = d.dtype == BLUT_BF16 ? tc_dequant_launch<TcDecDense<true>>(a, L.nchunks, stream)
                               : tc_dequant_launch<TcDecDense<false>>(a, L.nchunks, stream);
      break;
    case BLUT_FMT_B:
      if (d.bits == 4) e = tc_dequant_family<TcDecB4>(d.group, a, L.nchunks, stream);
      else if (d.bits == 3) e = dequant_tc_b3(d.group, a, L.nchunks, stream);
      else if (d.bits == 2) e = dequant_tc_b2(d.group, a, L.nchunks, stream);
      else return BLUT_ERR_UNSUPPORTED;
      break;
    case BLUT_FMT_NESTED:
      e = d.tier == 1 ? dequant_tc_b2(d.group, a, L.nchunks, stream) : dequant_tc_nested(d.group, a, L.nchunks, stream);
      break;
    case BLUT_FMT_R8:
      if (!r8_table) return BLUT_ERR_INVALID;
      e = dequant_tc_r8(a, L.nchunks, stream);
      break;
    default:
      return BLUT_ERR_UNSUPPORTED;
  }
  return e == cudaSuccess ? BLUT_OK : BLUT_ERR_LAUNCH;
}

}  // namespace blut
