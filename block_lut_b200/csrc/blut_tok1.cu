// Instantiations of the single-token pass (blut_tok1.cuh) for every format
// of the TC layout, with a dense shared expert of the same dtype.
#include "blut_internal.h"
#include "blut_tok1.cuh"

namespace blut {
namespace {

template <template <int> class DecT, bool PAIR>
cudaError_t tok1_family(int group, const Tok1Args& a, double rb, double sb, cudaStream_t s) {
  switch (group) {
    case 32: return launch_tok1_dec<DecT<32>, PAIR>(a, rb, sb, s);
    case 64: return launch_tok1_dec<DecT<64>, PAIR>(a, rb, sb, s);
    case 128: return launch_tok1_dec<DecT<128>, PAIR>(a, rb, sb, s);
  }
  return cudaErrorInvalidValue;
}

template <bool PAIR>
cudaError_t tok1_dispatch(const blut_mat_desc& d, const Tok1Args& a, double rb, double sb, cudaStream_t s) {
  switch (d.format) {
    case BLUT_FMT_DENSE:
      return d.dtype == BLUT_BF16 ? launch_tok1_dec<TcDecDense<true>, PAIR>(a, rb, sb, s)
                                  : launch_tok1_dec<TcDecDense<false>, PAIR>(a, rb, sb, s);
    case BLUT_FMT_B:
      if (d.bits == 4) return tok1_family<TcDecB4, PAIR>(d.group, a, rb, sb, s);
      if (d.bits == 3) return tok1_family<TcDecB3, PAIR>(d.group, a, rb, sb, s);
      if (d.bits == 2) return tok1_family<TcDecB2, PAIR>(d.group, a, rb, sb, s);
      break;
    case BLUT_FMT_NESTED:  // the coarse tier is a 2-bit lookup of planes 0, 1
      return d.tier == 1 ? tok1_family<TcDecB2, PAIR>(d.group, a, rb, sb, s)
                         : tok1_family<TcDecNested, PAIR>(d.group, a, rb, sb, s);
    case BLUT_FMT_R8:
      return a.m[0].p.r8_table ? launch_tok1_dec<TcDecR8, PAIR>(a, rb, sb, s) : cudaErrorInvalidValue;
  }
  return cudaErrorInvalidValue;
}

}  // namespace

cudaError_t launch_tok1(const blut_mat_desc& d, const Tok1Args& a, bool pair, double routed_bytes,
                        double shared_bytes, cudaStream_t stream) {
  return pair ? tok1_dispatch<true>(d, a, routed_bytes, shared_bytes, stream)
              : tok1_dispatch<false>(d, a, routed_bytes, shared_bytes, stream);
}

}  // namespace blut
