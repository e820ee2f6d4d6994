// Router top-k shared by the MoE orchestration (blut_moe.cu) and the
// single-token GEMV (blut_tok1.cuh).
#pragma once

#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "blut_internal.h"

namespace blut {

// Softmax over E logits (fp32) and top-k with the lowest expert index winning
// ties, optional renormalisation; one warp per token.  Row R-1 of a logits
// row with a gate entry yields sigmoid(logit) in *sg.
template <int kPer>  // expert logits per lane: E <= 32 * kPer
__device__ __forceinline__ void warp_topk_n(const float* __restrict__ lg, int E, int K, int renorm, int32_t* ids,
                                            float* tw) {
  const int lane = threadIdx.x & 31;
  float v[kPer];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < E ? lg[e] : -INFINITY;
    mx = fmaxf(mx, v[i]);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < E ? expf(v[i] - mx) : -1.f;
    sum += e < E ? v[i] : 0.f;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float inv = 1.f / sum;
  float wsum = 0.f, myw = 0.f;
  int myid = 0;
  for (int j = 0; j < K; ++j) {
    float best = -1.f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      if (v[i] > best) { best = v[i]; bi = lane + 32 * i; }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
    }
    const float p = best * inv;
    wsum += p;
    if (lane == j) { myw = p; myid = bi; }
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      if (lane + 32 * i == bi) v[i] = -2.f;  // taken
    }
  }
  if (lane < K) {
    ids[lane] = myid;
    tw[lane] = renorm ? myw / wsum : myw;
  }
}

__device__ __forceinline__ void warp_topk(const float* __restrict__ lg, int E, int K, int renorm, int32_t* ids, float* tw,
                          float* sg_out, bool has_gate) {
  if (has_gate && (threadIdx.x & 31) == 0) *sg_out = 1.f / (1.f + expf(-lg[E]));
  if (K <= 0) return;
  if (E <= 64) warp_topk_n<2>(lg, E, K, renorm, ids, tw);
  else if (E <= 128) warp_topk_n<4>(lg, E, K, renorm, ids, tw);
  else if (E <= 256) warp_topk_n<8>(lg, E, K, renorm, ids, tw);
  else warp_topk_n<kMaxExperts / 32>(lg, E, K, renorm, ids, tw);
}

}  // namespace blut
