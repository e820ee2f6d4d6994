// Format-R LUT GEMV on the canonical layout (the reference's lut_gemv API):
//   y[r] = sum_c x[c] * cb[idx[r, c]] * absmax[min((r*K + c) / 128, nb - 1)]
// One warp per row, 16 codes per 16-byte load, a per-lane replicated fp32
// codebook in shared memory (conflict-free gathers), fp32 accumulation.
#include <algorithm>

#include "blut_common.cuh"
#include "blut_internal.h"

namespace blut {

namespace {

constexpr int kRowsPerCta = 8;

__global__ void __launch_bounds__(256) lut_gemv_kernel(const uint16_t* __restrict__ x, const uint8_t* __restrict__ idx,
                                                       const uint16_t* __restrict__ cb,
                                                       const uint16_t* __restrict__ absmax, uint16_t* __restrict__ y,
                                                       int64_t m, int64_t k, int64_t nb, bool vec) {
  extern __shared__ float sm[];
  float* tab = sm;              // [256][32]
  float* xs = sm + 256 * 32;    // [k]
  for (int i = threadIdx.x; i < 256 * 32; i += blockDim.x) tab[i] = __uint_as_float(uint32_t(cb[i >> 5]) << 16);
  for (int64_t i = threadIdx.x; i < k; i += blockDim.x) xs[i] = __uint_as_float(uint32_t(x[i]) << 16);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * kRowsPerCta + warp;
  if (r >= m) return;
  const float* tl = tab + lane;
  float acc = 0.f;
  const int64_t base = r * k;
  if (vec) {
    for (int64_t c = lane * 16; c < k; c += 32 * 16) {
      const uint4 v = *reinterpret_cast<const uint4*>(idx + base + c);
      const uint8_t* b = reinterpret_cast<const uint8_t*>(&v);
      const float s = __uint_as_float(uint32_t(absmax[std::min<int64_t>((base + c) >> 7, nb - 1)]) << 16);
      float part = 0.f;
#pragma unroll
      for (int q = 0; q < 16; ++q) part = fmaf(xs[c + q], tl[b[q] * 32], part);
      acc = fmaf(part, s, acc);
    }
  } else {
    for (int64_t c = lane; c < k; c += 32) {
      const float s = __uint_as_float(uint32_t(absmax[std::min<int64_t>((base + c) >> 7, nb - 1)]) << 16);
      acc = fmaf(xs[c] * tl[idx[base + c] * 32], s, acc);
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) y[r] = __bfloat16_as_ushort(__float2bfloat16_rn(acc));
}

}  // namespace

int lut_gemv(const void* x, const void* idx, const void* cb, const void* absmax, void* y, int64_t m, int64_t k,
             int64_t nb, cudaStream_t stream) {
  if (!x || !idx || !cb || !absmax || !y || m <= 0 || k <= 0 || nb <= 0) return BLUT_ERR_INVALID;
  const size_t smem = (256 * 32 + (size_t)k) * sizeof(float);
  if (smem > 220 * 1024) return BLUT_ERR_UNSUPPORTED;
  const bool vec = k % 16 == 0 && ((uintptr_t)idx & 15) == 0;
  if (cudaFuncSetAttribute(lut_gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return BLUT_ERR_CUDA;
  const unsigned grid = (unsigned)((m + kRowsPerCta - 1) / kRowsPerCta);
  lut_gemv_kernel<<<grid, 32 * kRowsPerCta, smem, stream>>>((const uint16_t*)x, (const uint8_t*)idx,
                                                            (const uint16_t*)cb, (const uint16_t*)absmax,
                                                            (uint16_t*)y, m, k, nb, vec);
  return cudaGetLastError() == cudaSuccess ? BLUT_OK : BLUT_ERR_LAUNCH;
}

}  // namespace blut
