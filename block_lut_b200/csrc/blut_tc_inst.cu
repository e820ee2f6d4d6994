// Instantiations of the tcgen05 LUT matmul (FMT_B 4-bit, dense) and the
// diagnostic dequantisation of the TC tiled layout through the same decode.
#include "blut_internal.h"
#include "blut_tc.cuh"

namespace blut {

bool tc_planes(const blut_mat_desc& d, bool pair, TcParams& p) {
  TiledLayout L;
  if (!make_layout(d, L) || !L.tc || L.nplanes > 2) return false;
  p.nplanes = L.nplanes;
  p.tile_bytes = 0;
  for (int q = 0; q < 2; ++q) {
    p.plane_off[q] = q < L.nplanes ? L.off[q] : 0;
    p.piece[q] = q < L.nplanes ? (int)L.piece[q] : 0;
    p.tile_bytes += p.piece[q];
  }
  p.ntiles = (int)L.ntiles;
  p.nblocks = (int)L.nchunks;
  p.units = (p.ntiles + 1) / 2;
  p.pair = pair ? 1 : 0;
  p.mul = TcMul{1u << 31, 1u << 16};
  return true;
}

template <int MT>
static cudaError_t launch_tc_mt(const blut_mat_desc& d, const TcParams& p, int sms, cudaStream_t stream) {
  if (d.format == BLUT_FMT_DENSE)
    return d.dtype == BLUT_BF16 ? launch_tc<TcDecDense<true>, MT>(p, sms, stream)
                                : launch_tc<TcDecDense<false>, MT>(p, sms, stream);
  if (d.format == BLUT_FMT_B && d.bits == 4) {
    switch (d.group) {
      case 32: return launch_tc<TcDecB4<32>, MT>(p, sms, stream);
      case 64: return launch_tc<TcDecB4<64>, MT>(p, sms, stream);
      case 128: return launch_tc<TcDecB4<128>, MT>(p, sms, stream);
    }
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_tc_mm(const blut_mat_desc& d, const TcParams& p, int group_tokens, int sms, cudaStream_t stream) {
  if (group_tokens == 32) return launch_tc_mt<32>(d, p, sms, stream);
  if (group_tokens == 128) return launch_tc_mt<128>(d, p, sms, stream);
  return cudaErrorInvalidValue;
}

// One CTA per (physical tile, block), one thread per row: decode the row's
// block straight from global memory with the matmul's decode policy and
// write it to out[rows][cols].
template <class Dec>
__global__ void __launch_bounds__(kTcRows) tc_dequant_kernel(const uint8_t* __restrict__ w, int64_t off0,
                                                             int64_t off1, int piece0, int piece1, int ntiles,
                                                             int64_t cols, int paired, uint16_t* __restrict__ out,
                                                             TcMul mul) {
  const int pt = blockIdx.x, b = blockIdx.y, row = threadIdx.x;
  const int64_t r = logical_tile(pt, ntiles, paired != 0) * kTcRows + row;
  const uint8_t* cp = w + off0 + ((int64_t)b * ntiles + pt) * piece0;
  uint4* dst = reinterpret_cast<uint4*>(out + r * cols + (int64_t)b * Dec::KB);
  if constexpr (Dec::kDense) {
#pragma unroll
    for (int u = 0; u < Dec::KB / 8; ++u) dst[u] = *reinterpret_cast<const uint4*>(cp + (u * kTcRows + row) * 16);
  } else {
    const uint8_t* tp = w + off1 + ((int64_t)b * ntiles + pt) * piece1;
#pragma unroll
    for (int h = 0; h < Dec::kHalves; ++h) {
      uint32_t a[32];
      Dec::decode(cp, tp, row, h, a, mul);
#pragma unroll
      for (int i = 0; i < 8; ++i) dst[h * 8 + i] = make_uint4(a[4 * i], a[4 * i + 1], a[4 * i + 2], a[4 * i + 3]);
    }
  }
}

template <class Dec>
static cudaError_t tc_dequant(const TiledLayout& L, const uint8_t* w, int64_t cols, int paired, uint16_t* out,
                              cudaStream_t stream) {
  dim3 grid((unsigned)L.ntiles, (unsigned)L.nchunks);
  tc_dequant_kernel<Dec><<<grid, kTcRows, 0, stream>>>(w, L.off[0], L.nplanes > 1 ? L.off[1] : 0, (int)L.piece[0],
                                                       L.nplanes > 1 ? (int)L.piece[1] : 0, (int)L.ntiles, cols,
                                                       paired, out, TcMul{1u << 31, 1u << 16});
  return cudaGetLastError();
}

int dequant_tiled_tc(const blut_mat_desc& d, const void* tiled, void* out, cudaStream_t stream) {
  TiledLayout L;
  if (!make_layout(d, L)) return BLUT_ERR_UNSUPPORTED;
  const uint8_t* w = static_cast<const uint8_t*>(tiled);
  uint16_t* o = static_cast<uint16_t*>(out);
  const int pr = (d.layout & BLUT_LAYOUT_PAIRED) ? 1 : 0;
  if ((reinterpret_cast<uintptr_t>(tiled) | reinterpret_cast<uintptr_t>(out)) & 15) return BLUT_ERR_INVALID;
  cudaError_t e = cudaErrorInvalidValue;
  if (d.format == BLUT_FMT_DENSE) {
    e = d.dtype == BLUT_BF16 ? tc_dequant<TcDecDense<true>>(L, w, d.cols, pr, o, stream)
                             : tc_dequant<TcDecDense<false>>(L, w, d.cols, pr, o, stream);
  } else if (d.format == BLUT_FMT_B && d.bits == 4) {
    switch (d.group) {
      case 32: e = tc_dequant<TcDecB4<32>>(L, w, d.cols, pr, o, stream); break;
      case 64: e = tc_dequant<TcDecB4<64>>(L, w, d.cols, pr, o, stream); break;
      case 128: e = tc_dequant<TcDecB4<128>>(L, w, d.cols, pr, o, stream); break;
    }
  } else {
    return BLUT_ERR_UNSUPPORTED;
  }
  return e == cudaSuccess ? BLUT_OK : BLUT_ERR_LAUNCH;
}

}  // namespace blut
