// LUT matmul mainloop: every (token group, weight tile) of a layer in one launch.
//
// Work item = (group of <= 32 tokens routed to one expert, 16-row tile of
// the expert's matrix; a gate tile and its up tile together for the gate/up
// projection).  A CTA of 4 warps owns an item; the K chunks are split among
// the warps (split-K), each warp streams its chunks through its own ring of
// shared-memory stages filled by bulk TMA copies (cp.async.bulk, one per
// plane per tile, completing on an mbarrier), looks codes up into A
// fragments and runs mma.m16n8k16 against the tokens' B fragments.  The
// ring runs ahead across items, so a CTA's stream of chunks never drains
// between items.  Partial sums meet in shared memory; the epilogue applies
// SiLU(gate) * up and writes the next projection's B fragments, or writes
// fp32 rows of the expert outputs.
#pragma once

#include <mutex>

#include "blut_policies.cuh"

namespace blut {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kWarpRingBytes = 20 * 1024;

struct GroupTab {
  const int* n_groups;  // device scalar
  const int* expert;
  const int* slot0;
  const int* ntok;
  const int* nt0;
};

struct MMParams {
  const uint8_t* w;        // tiled matrices of all experts
  int64_t wstride;         // bytes between experts
  int64_t plane_off[3];    // matrix-relative offsets of the planes this kernel reads
  int piece[3];            // bytes per (tile, chunk) piece of those planes
  int tile_bytes;          // sum of piece[] (one tile's share of a stage)
  int stages;              // ring stages per warp
  int ntiles;              // 16-row tiles of the matrix
  int nchunks;             // 128-column chunks (K / 128)
  GroupTab gt;
  const uint8_t* bin;      // B fragments of the input, [n-tile][chunk][2 KB]
  // pair epilogue: B fragments of SiLU(gate) * up, [n-tile][out_nchunks][2 KB]
  uint8_t* act_out;
  int out_nchunks;
  // single epilogue: fp32 rows y[slot][y_ld]
  float* y_out;
  int y_ld;
  const uint16_t* r8_table;  // global bf16 [256], FMT_R8 only
  uint32_t r8_mask;
  int* status;
};

__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + expf(-v)); }

template <class Pol>
__host__ __device__ constexpr int mm_r8_smem() {
  return Pol::kR8 ? 256 * 32 * 4 : 0;
}

template <class Pol, bool kPair>
__host__ __device__ constexpr int mm_red_bytes() {
  return kWarps * (kPair ? 2 : 1) * kMaxNT * 32 * 16;
}

template <class Pol, bool kPair>
__global__ void __launch_bounds__(kThreads) lut_mm_kernel(const MMParams p) {
  constexpr int NTL = kPair ? 2 : 1;
  constexpr int kR8Bytes = mm_r8_smem<Pol>();
  extern __shared__ __align__(128) uint8_t smem[];
  uint32_t* r8tab = reinterpret_cast<uint32_t*>(smem);
  float4* red = reinterpret_cast<float4*>(smem + kR8Bytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kR8Bytes + mm_red_bytes<Pol, kPair>());
  uint8_t* ring = smem + kR8Bytes + mm_red_bytes<Pol, kPair>() + kWarps * 8 * 8;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int S = p.stages;
  const int stage_bytes = NTL * p.tile_bytes;
  uint8_t* my_ring = ring + warp * S * stage_bytes;
  const uint32_t my_bar0 = smem_u32(bars + warp * 8);

  if constexpr (kR8Bytes > 0) {
    for (int i = threadIdx.x; i < 256 * 32; i += kThreads) r8tab[i] = p.r8_table[i >> 5];
  }
  if (lane == 0) {
    for (int s = 0; s < S; ++s) mbar_init(my_bar0 + 8 * s, 1);
    fence_mbar_init();
  }
  __syncthreads();

  PolExtra ex;
  ex.r8_table = r8tab;
  ex.r8_mask = p.r8_mask;

  const int tiles_per_item = kPair ? p.ntiles / 2 : p.ntiles;
  const int n_items = *p.gt.n_groups * tiles_per_item;
  const int c0 = warp * p.nchunks / kWarps;
  const int cpw = (warp + 1) * p.nchunks / kWarps - c0;
  const int my_items = n_items > (int)blockIdx.x ? (n_items - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int total = my_items * cpw;

  // Producer side (lane 0): issue the copies of step n into stage n % S.
  auto issue = [&](int n) {
    const int item = blockIdx.x + (n / cpw) * gridDim.x;
    const int c = c0 + n % cpw;
    const int gi = item / tiles_per_item;
    const int ti = item - gi * tiles_per_item;
    const uint8_t* base = p.w + (int64_t)p.gt.expert[gi] * p.wstride;
    const int slot = n % S;
    const uint32_t bar = my_bar0 + 8 * slot;
    uint8_t* dst = my_ring + slot * stage_bytes;
    mbar_expect_tx(bar, stage_bytes);
#pragma unroll
    for (int t = 0; t < NTL; ++t) {
      const int tile = t == 0 ? ti : ti + tiles_per_item;
      int doff = t * p.tile_bytes;
#pragma unroll
      for (int q = 0; q < Pol::kNumPlanes; ++q) {
        const uint8_t* src = base + p.plane_off[q] + ((int64_t)tile * p.nchunks + c) * p.piece[q];
        bulk_g2s(smem_u32(dst + doff), src, p.piece[q], bar);
        doff += p.piece[q];
      }
    }
  };

  int issued = 0;
  if (lane == 0) {
    for (; issued < total && issued < S; ++issued) issue(issued);
  }
  bool ok = true;
  int n = 0;
  for (int j = 0; j < my_items; ++j) {
    const int item = blockIdx.x + j * gridDim.x;
    const int gi = item / tiles_per_item;
    const int ti = item - gi * tiles_per_item;
    const int ntok = p.gt.ntok[gi];
    const int ntv = (ntok + kNTile - 1) / kNTile;
    const int nt0 = p.gt.nt0[gi];

    float acc[NTL][kMaxNT][4];
#pragma unroll
    for (int t = 0; t < NTL; ++t)
#pragma unroll
      for (int i = 0; i < kMaxNT; ++i)
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[t][i][r] = 0.f;

    for (int cc = 0; cc < cpw; ++cc, ++n) {
      const int slot = n % S;
      if (ok) {
        bool w_ok = mbar_wait_bounded(my_bar0 + 8 * slot, (n / S) & 1, p.status);
        ok = __shfl_sync(0xffffffffu, w_ok ? 1 : 0, 0) != 0;
      }
      if (ok) {
        const int c = c0 + cc;
        const uint8_t* st = my_ring + slot * stage_bytes;
        Pol P[NTL];
#pragma unroll
        for (int t = 0; t < NTL; ++t) {
          const uint8_t* planes[3];
          int off = t * p.tile_bytes;
#pragma unroll
          for (int q = 0; q < Pol::kNumPlanes; ++q) {
            planes[q] = st + off;
            off += p.piece[q];
          }
          P[t].begin(planes, lane, ex);
        }
        const uint8_t* bsrc = p.bin + ((int64_t)nt0 * p.nchunks + c) * kBfragChunkBytes + lane * 64;
        const int64_t bstep = (int64_t)p.nchunks * kBfragChunkBytes;
#pragma unroll
        for (int sp = 0; sp < 4; ++sp) {
          uint4 b[kMaxNT];
#pragma unroll
          for (int i = 0; i < kMaxNT; ++i) {
            if (i < ntv) b[i] = __ldg(reinterpret_cast<const uint4*>(bsrc + i * bstep + sp * 16));
          }
#pragma unroll
          for (int s2 = 0; s2 < 2; ++s2) {
            const int s = 2 * sp + s2;
            if (s % Pol::kSlabsPerBlock == 0) {
#pragma unroll
              for (int t = 0; t < NTL; ++t) P[t].block(s / Pol::kSlabsPerBlock);
            }
#pragma unroll
            for (int t = 0; t < NTL; ++t) {
              uint32_t a[4];
              P[t].frag(s, a);
#pragma unroll
              for (int i = 0; i < kMaxNT; ++i) {
                if (i < ntv) mma16816<Pol::kBF16>(acc[t][i], a, s2 ? b[i].z : b[i].x, s2 ? b[i].w : b[i].y);
              }
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0 && ok && issued < total) {
        fence_proxy_async();
        issue(issued++);
      }
    }

    // split-K reduction across the warps
#pragma unroll
    for (int t = 0; t < NTL; ++t)
#pragma unroll
      for (int i = 0; i < kMaxNT; ++i)
        red[((warp * NTL + t) * kMaxNT + i) * 32 + lane] = make_float4(acc[t][i][0], acc[t][i][1], acc[t][i][2], acc[t][i][3]);
    __syncthreads();
    if (warp < ntv) {
      const int i = warp;
      float v[NTL][4];
#pragma unroll
      for (int t = 0; t < NTL; ++t) {
        float4 s4 = red[((0 * NTL + t) * kMaxNT + i) * 32 + lane];
#pragma unroll
        for (int w = 1; w < kWarps; ++w) {
          const float4 o = red[((w * NTL + t) * kMaxNT + i) * 32 + lane];
          s4.x += o.x; s4.y += o.y; s4.z += o.z; s4.w += o.w;
        }
        v[t][0] = s4.x; v[t][1] = s4.y; v[t][2] = s4.z; v[t][3] = s4.w;
      }
      const int g = lane >> 2, tq = lane & 3;
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int row = g + 8 * (r >> 1);     // tile row
        const int tok = 2 * tq + (r & 1);     // token inside the n-tile
        const bool valid = i * kNTile + tok < ntok;
        if constexpr (kPair) {
          const float val = valid ? silu_f(v[0][r]) * v[1][r] : 0.f;
          const int col = ti * kTileRows + row;  // column of the next projection's K
          uint8_t* dst = p.act_out + ((int64_t)(nt0 + i) * p.out_nchunks + (col >> 7)) * kBfragChunkBytes +
                         bfrag_byte(tok, col & 127);
          *reinterpret_cast<uint16_t*>(dst) = f32_to_act<Pol::kBF16>(val);
        } else {
          if (valid) {
            const int slot = p.gt.slot0[gi] + i * kNTile + tok;
            p.y_out[(int64_t)slot * p.y_ld + ti * kTileRows + row] = v[0][r];
          }
        }
      }
    }
    __syncthreads();
  }

  // After a timed-out wait, let copies still in flight land before exiting.
  if (!ok && lane == 0) {
    for (int m = n; m < issued; ++m) mbar_wait_bounded(my_bar0 + 8 * (m % S), (m / S) & 1, p.status);
  }
}

// Host-side launch helper: dynamic smem and grid for one instantiation.
template <class Pol, bool kPair>
inline int mm_smem_bytes(int stages, int tile_bytes) {
  return mm_r8_smem<Pol>() + mm_red_bytes<Pol, kPair>() + kWarps * 8 * 8 +
         kWarps * stages * (kPair ? 2 : 1) * tile_bytes;
}

template <class Pol, bool kPair>
inline cudaError_t launch_mm(MMParams p, int num_sms, cudaStream_t stream) {
  const int smem = mm_smem_bytes<Pol, kPair>(p.stages, p.tile_bytes);
  auto kern = lut_mm_kernel<Pol, kPair>;
  // attribute + occupancy per (instantiation, smem size), computed once
  static std::mutex mu;
  static int cached_smem = -1, cached_per_sm = 1;
  int per_sm;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (cached_smem != smem) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return e;
      int n = 0;
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kThreads, smem);
      if (e != cudaSuccess) return e;
      cached_per_sm = n < 1 ? 1 : n;
      cached_smem = smem;
    }
    per_sm = cached_per_sm;
  }
  kern<<<num_sms * per_sm, kThreads, smem, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace blut
