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

namespace blut {

// Diagnostic: one warp per (tile, chunk) copies the piece into shared memory,
// runs the policy's fragment lookups and scatters the A fragments back to a
// dense [rows][cols] matrix.
template <class Pol>
__global__ void __launch_bounds__(32) tiled_dequant_kernel(const MMParams p, uint16_t* __restrict__ out, int64_t cols,
                                                           int paired) {
  extern __shared__ __align__(16) uint8_t sm[];
  uint32_t* r8tab = reinterpret_cast<uint32_t*>(sm);
  uint8_t* piece = sm + mm_r8_smem<Pol>();
  const int pt = blockIdx.x, c = blockIdx.y, lane = threadIdx.x;
  const int tile = (int)logical_tile(pt, p.ntiles, paired != 0);
  if constexpr (Pol::kR8) {
    for (int i = lane; i < 256 * 32; i += 32) r8tab[i] = p.r8_table[i >> 5];
  }
  const uint8_t* planes[3];
  int off = 0;
  for (int q = 0; q < Pol::kNumPlanes; ++q) {
    const uint4* src = reinterpret_cast<const uint4*>(p.w + p.plane_off[q] + ((int64_t)c * p.ntiles + pt) * p.piece[q]);
    uint4* dst = reinterpret_cast<uint4*>(piece + off);
    for (int i = lane; i < p.piece[q] / 16; i += 32) dst[i] = src[i];
    planes[q] = piece + off;
    off += p.piece[q];
  }
  __syncwarp();
  PolExtra ex;
  ex.r8_table = r8tab;
  ex.r8_mask = p.r8_mask;
  Pol P;
  P.begin(planes, lane, ex);
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int s = 0; s < 8; ++s) {
    if (s % Pol::kSlabsPerBlock == 0) P.block(s / Pol::kSlabsPerBlock);
    uint32_t a[4];
    P.frag(s, a);
    const int64_t r0 = (int64_t)tile * kTileRows + g;
    const int64_t k0 = (int64_t)c * kChunk + 16 * s + 2 * t;
    uint32_t* o = reinterpret_cast<uint32_t*>(out);
    o[(r0 * cols + k0) >> 1] = a[0];
    o[((r0 + 8) * cols + k0) >> 1] = a[1];
    o[(r0 * cols + k0 + 8) >> 1] = a[2];
    o[((r0 + 8) * cols + k0 + 8) >> 1] = a[3];
  }
}

template <class Pol>
inline cudaError_t launch_tiled_dequant(const MMParams& p, uint16_t* out, int64_t cols, int paired,
                                        cudaStream_t stream) {
  int smem = mm_r8_smem<Pol>() + p.tile_bytes;
  auto kern = tiled_dequant_kernel<Pol>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  kern<<<dim3(p.ntiles, p.nchunks), 32, smem, stream>>>(p, out, cols, paired);
  return cudaGetLastError();
}

template <template <int> class Pol>
inline cudaError_t tiled_dequant_by_group(int group, const MMParams& p, uint16_t* out, int64_t cols, int paired,
                                          cudaStream_t stream) {
  switch (group) {
    case 32: return launch_tiled_dequant<Pol<32>>(p, out, cols, paired, stream);
    case 64: return launch_tiled_dequant<Pol<64>>(p, out, cols, paired, stream);
    case 128: return launch_tiled_dequant<Pol<128>>(p, out, cols, paired, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace blut
