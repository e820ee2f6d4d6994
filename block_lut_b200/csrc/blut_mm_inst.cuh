// Helper for the per-format instantiation units.
#pragma once

#include "blut_internal.h"
#include "blut_mm.cuh"

namespace blut {

template <class Pol>
inline cudaError_t launch_pair_or_single(bool pair, const MMParams& p, int sms, cudaStream_t stream) {
  return pair ? launch_mm<Pol, true>(p, sms, stream) : launch_mm<Pol, false>(p, sms, stream);
}

template <template <int> class Pol>
inline cudaError_t launch_by_group(int group, bool pair, const MMParams& p, int sms, cudaStream_t stream) {
  switch (group) {
    case 32: return launch_pair_or_single<Pol<32>>(pair, p, sms, stream);
    case 64: return launch_pair_or_single<Pol<64>>(pair, p, sms, stream);
    case 128: return launch_pair_or_single<Pol<128>>(pair, p, sms, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace blut
