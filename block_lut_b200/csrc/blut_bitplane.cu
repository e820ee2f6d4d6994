// Progressive bit-plane storage of Format R indices, and the fused tier
// recover that reads a prefix of it.
//
// The planes follow runtime/model_offload.py:751-758. For n indices (n a
// multiple of 4) the buffer holds three sections, [low4 | mid2 | high2]:
//   low4   n/2 bytes  byte q: element 2q in bits 0-3, element 2q+1 in bits 4-7
//   mid2   n/4 bytes  byte q: bits 4-5 of element 4q+j in bits 2j..2j+1
//   high2  n/4 bytes  byte q: bits 6-7 of element 4q+j in bits 2j..2j+1
// Tier t reads a prefix of the buffer (csrc/tensor_engine/tensor_engine.cpp:
// 505-509): tier 2 the low section (n/2 bytes), tier 1 low + mid (3n/4), tier
// 0 all n bytes. Its index is low | mid << 4 | high << 6, where the sections
// it did not read count as zero: idx & 0x0F, idx & 0x3F, idx.
//
// The reference rebuilds a tier's indices first, in place on the GPU with two
// kernels (tier 2, csrc/kernels/tensor_recover.cu:166-192) or on the host
// (tier 1, tensor_engine.cpp:535-547), and then recovers bf16 in a third pass
// (csrc/topology/model_topology.cpp:597-618). Here one pass reads only the
// tier's sections and the absmax, and writes
//   out[i] = bf16(table[index(i)] * absmax[min(i / bs, nb - 1)]).
// The kernel is HBM-bound: per element it moves 0.5 / 0.75 / 1 byte of planes,
// 2 / bs bytes of absmax and 2 bytes of output.
#include <algorithm>

#include "blut_common.cuh"
#include "blut_internal.h"

namespace blut {

namespace {

constexpr int kBpThreads = 256;
constexpr int kBpGroup = 32;    // elements per thread and step of the packer's vector path
constexpr int kBpChunk = 1024;  // elements per warp and step of the recover's vector path

inline unsigned bp_grid(int64_t work, int per_sm) {
  const int64_t want = std::max<int64_t>((work + kBpThreads - 1) / kBpThreads, 1);
  return (unsigned)std::min<int64_t>(want, (int64_t)num_sms() * per_sm);
}

// Vector path: thread step v covers elements [32v, 32v + 32). Its low section
// is 16 bytes at 16v, its mid and high sections 8 bytes at n/2 + 8v and
// 3n/4 + 8v, so with n % 32 == 0 and 16-byte aligned buffers every access is
// aligned. Element k of the step sits at bits 4(k & 7) of low word k >> 3 and
// at bits 2(k & 15) of mid / high word k >> 4.
__global__ void __launch_bounds__(kBpThreads) bitplane_pack_kernel(uint8_t* __restrict__ planes,
                                                                   const uint8_t* __restrict__ idx, int64_t n,
                                                                   bool vec) {
  uint8_t* lo = planes;
  uint8_t* mi = planes + n / 2;
  uint8_t* hi = planes + n / 2 + n / 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nv = vec ? n / kBpGroup : 0;
  for (int64_t v = tid; v < nv; v += stride) {
    const uint4 c0 = *reinterpret_cast<const uint4*>(idx + v * kBpGroup);
    const uint4 c1 = *reinterpret_cast<const uint4*>(idx + v * kBpGroup + 16);
    const uint32_t w[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    uint32_t l[4] = {0, 0, 0, 0}, m[2] = {0, 0}, h[2] = {0, 0};
#pragma unroll
    for (int k = 0; k < kBpGroup; ++k) {
      const uint32_t x = (w[k >> 2] >> (8 * (k & 3))) & 0xFFu;
      l[k >> 3] |= (x & 0xFu) << (4 * (k & 7));
      m[k >> 4] |= ((x >> 4) & 3u) << (2 * (k & 15));
      h[k >> 4] |= (x >> 6) << (2 * (k & 15));
    }
    *reinterpret_cast<uint4*>(lo + v * 16) = make_uint4(l[0], l[1], l[2], l[3]);
    *reinterpret_cast<uint2*>(mi + v * 8) = make_uint2(m[0], m[1]);
    *reinterpret_cast<uint2*>(hi + v * 8) = make_uint2(h[0], h[1]);
  }
  // the quads after the vector steps (all of them without the vector path)
  for (int64_t q = nv * (kBpGroup / 4) + tid; q < n / 4; q += stride) {
    const uint8_t* x = idx + 4 * q;
    lo[2 * q] = uint8_t((x[0] & 0xFu) | ((x[1] & 0xFu) << 4));
    lo[2 * q + 1] = uint8_t((x[2] & 0xFu) | ((x[3] & 0xFu) << 4));
    uint32_t m = 0, h = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      m |= ((uint32_t(x[j]) >> 4) & 3u) << (2 * j);
      h |= (uint32_t(x[j]) >> 6) << (2 * j);
    }
    mi[q] = uint8_t(m);
    hi[q] = uint8_t(h);
  }
}

// The tier's table is replicated per lane in shared memory: entry e for lane l
// at word 32e + l (the bf16 in the low half), so the 32 lookups of a warp hit
// 32 different banks whatever the indices.
//
// Vector path: warp w takes chunks of 1024 elements, c = w, w + warps, ...;
// lane l handles the four runs of 8 elements at 1024c + 256r + 8l (r < 4).
// A run's indices are a u32 of the low section and a u16 of the mid and high
// sections (element k at bits 4k, 2k), and its output is one 16-byte store,
// so every load and store instruction of the warp covers one contiguous span.
// With n % 8 == 0, bs % 8 == 0, 4-byte aligned planes and a 16-byte aligned
// output, every access is aligned and a run never crosses an absmax block.
// The elements after the last whole chunk go through the per-quad path.
template <int kTier>
__global__ void __launch_bounds__(kBpThreads) bitplane_recover_kernel(uint16_t* __restrict__ out,
                                                                      const uint8_t* __restrict__ planes,
                                                                      const uint16_t* __restrict__ absmax,
                                                                      const uint16_t* __restrict__ table, int64_t n,
                                                                      int64_t nb, int bs, bool vec) {
  constexpr int kEntries = kTier == 2 ? 16 : kTier == 1 ? 64 : 256;
  extern __shared__ uint32_t bp_tab[];
  for (int w = threadIdx.x; w < kEntries * 32; w += blockDim.x) bp_tab[w] = table[w >> 5];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const uint32_t* tab = bp_tab + lane;
  const uint8_t* lo = planes;
  const uint8_t* mi = planes + n / 2;
  const uint8_t* hi = planes + n / 2 + n / 4;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t nchunk = vec ? n / kBpChunk : 0;
  for (int64_t c = tid >> 5; c < nchunk; c += stride >> 5) {
    const int64_t e0 = c * kBpChunk + 8 * lane;
    uint32_t L[4], M[4] = {0, 0, 0, 0}, H[4] = {0, 0, 0, 0}, S[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int64_t e = e0 + 256 * r;
      L[r] = *reinterpret_cast<const uint32_t*>(lo + e / 2);
      if (kTier <= 1) M[r] = *reinterpret_cast<const uint16_t*>(mi + e / 4);
      if (kTier == 0) H[r] = *reinterpret_cast<const uint16_t*>(hi + e / 4);
      S[r] = absmax[std::min<int64_t>(e / bs, nb - 1)];
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const uint32_t s2 = S[r] | (S[r] << 16);
      uint32_t o[4];
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        uint32_t t = 0;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int k = 2 * p + u;
          uint32_t x = (L[r] >> (4 * k)) & 0xFu;
          if (kTier <= 1) x |= ((M[r] >> (2 * k)) & 3u) << 4;
          if (kTier == 0) x |= ((H[r] >> (2 * k)) & 3u) << 6;
          t |= tab[32 * x] << (16 * u);
        }
        o[p] = bf16x2_mul(t, s2);
      }
      *reinterpret_cast<uint4*>(out + e0 + 256 * r) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  for (int64_t q = nchunk * (kBpChunk / 4) + tid; q < n / 4; q += stride) {
    const uint32_t l = uint32_t(lo[2 * q]) | (uint32_t(lo[2 * q + 1]) << 8);
    const uint32_t m = kTier <= 1 ? mi[q] : 0u;
    const uint32_t h = kTier == 0 ? hi[q] : 0u;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t i = 4 * q + j;
      const uint32_t x = ((l >> (4 * j)) & 0xFu) | (((m >> (2 * j)) & 3u) << 4) | (((h >> (2 * j)) & 3u) << 6);
      const uint32_t s = absmax[std::min<int64_t>(i / bs, nb - 1)];
      out[i] = uint16_t(bf16x2_mul(tab[32 * x], s) & 0xFFFFu);
    }
  }
}

constexpr size_t recover_smem(int tier) { return size_t(tier == 2 ? 16 : tier == 1 ? 64 : 256) * 32 * sizeof(uint32_t); }

// Resident blocks per SM (registers and the replicated table decide it); the
// grid is that many blocks per SM, so no block waits for a second wave.
template <int kTier>
int recover_blocks_per_sm() {
  static const int b = [] {
    int v = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, bitplane_recover_kernel<kTier>, kBpThreads,
                                                      recover_smem(kTier)) != cudaSuccess || v < 1)
      v = 1;
    return v;
  }();
  return b;
}

int pack_blocks_per_sm() {
  static const int b = [] {
    int v = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, bitplane_pack_kernel, kBpThreads, 0) != cudaSuccess || v < 1)
      v = 1;
    return v;
  }();
  return b;
}

}  // namespace

int64_t bitplane_bytes(int64_t n, int tier) {
  if (n <= 0 || n % 4 || tier < 0 || tier > 2) return BLUT_ERR_INVALID;
  return tier == 2 ? n / 2 : tier == 1 ? n / 2 + n / 4 : n;
}

int bitplane_pack(void* planes, const void* idx, int64_t n, cudaStream_t stream) {
  if (!planes || !idx || n <= 0) return BLUT_ERR_INVALID;
  if (n % 4) return BLUT_ERR_UNSUPPORTED;
  const bool vec = n % kBpGroup == 0 && ((uintptr_t)planes & 15) == 0 && ((uintptr_t)idx & 15) == 0;
  const int64_t work = vec ? n / kBpGroup : n / 4;
  bitplane_pack_kernel<<<bp_grid(work, pack_blocks_per_sm()), kBpThreads, 0, stream>>>((uint8_t*)planes, (const uint8_t*)idx, n,
                                                                     vec);
  return cudaGetLastError() == cudaSuccess ? BLUT_OK : BLUT_ERR_LAUNCH;
}

int bitplane_recover(void* out, const void* planes, const void* absmax, const void* table, int64_t n, int tier,
                     int bs, cudaStream_t stream) {
  if (!out || !planes || !absmax || !table || n <= 0 || bs <= 0 || tier < 0 || tier > 2) return BLUT_ERR_INVALID;
  if (n % 4) return BLUT_ERR_UNSUPPORTED;
  const int64_t nb = (n + bs - 1) / bs;
  const bool vec = n % 8 == 0 && bs % 8 == 0 && ((uintptr_t)planes & 3) == 0 && ((uintptr_t)out & 15) == 0;
  const int64_t work = vec ? std::max<int64_t>(n / kBpChunk * 32, n / 4 - n / kBpChunk * (kBpChunk / 4)) : n / 4;
  const size_t smem = recover_smem(tier);
  const auto* pl = (const uint8_t*)planes;
  const auto* am = (const uint16_t*)absmax;
  const auto* tb = (const uint16_t*)table;
  if (tier == 2)
    bitplane_recover_kernel<2><<<bp_grid(work, recover_blocks_per_sm<2>()), kBpThreads, smem, stream>>>(
        (uint16_t*)out, pl, am, tb, n, nb, bs, vec);
  else if (tier == 1)
    bitplane_recover_kernel<1><<<bp_grid(work, recover_blocks_per_sm<1>()), kBpThreads, smem, stream>>>(
        (uint16_t*)out, pl, am, tb, n, nb, bs, vec);
  else
    bitplane_recover_kernel<0><<<bp_grid(work, recover_blocks_per_sm<0>()), kBpThreads, smem, stream>>>(
        (uint16_t*)out, pl, am, tb, n, nb, bs, vec);
  return cudaGetLastError() == cudaSuccess ? BLUT_OK : BLUT_ERR_LAUNCH;
}

}  // namespace blut
