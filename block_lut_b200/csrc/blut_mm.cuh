// LUT matmul mainloop: every (token group, weight tile) of a layer in one launch.
//
// Work item = (group of <= 32 tokens routed to one expert, W consecutive
// tile units of that expert's matrix); a unit is a gate tile plus its up tile
// for the gate/up projection (paired layout), or one 16-row tile for the
// down projection.  A CTA has one producer warp and W consumer warps:
//
//  * the producer's elected lane streams, chunk by chunk (128 columns), the
//    code/table planes of the item's W units -- one bulk TMA copy
//    (cp.async.bulk) per plane, contiguous thanks to the chunk-major tiled
//    layout -- plus the group's B fragments of that chunk, into a ring of
//    shared-memory stages (full barrier: transaction bytes; empty barrier:
//    one arrival per consumer warp);
//  * each consumer warp owns one unit for the whole K loop: it looks codes
//    up into mma.m16n8k16 A fragments, multiplies them against the shared
//    B fragments of up to 4 n-tiles (8 tokens each), accumulates in fp32
//    registers and finishes with the epilogue -- SiLU(gate) * up written as
//    the down projection's B fragments, or fp32 expert-output rows.
//
// Every wait is bounded: a wait that runs out sets a CTA-wide abort flag and
// the device status word, all warps skip the remaining work, and the
// producer lets the copies it still has in flight land before exiting.
#pragma once

#include <mutex>

#include "blut_policies.cuh"

namespace blut {

constexpr int kMaxConsumers = 6;
constexpr int kRingBudget = 96 * 1024;       // shared-memory ring bytes per CTA
constexpr uint64_t kWaitLimitNs = 2000000000ull;
constexpr uint32_t kWaitSleepNs = 20000;  // longest hardware sleep of one try (woken early on completion)

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
  int tile_bytes;          // sum of piece[]
  int ntiles;              // physical 16-row tiles of the matrix
  int nchunks;             // 128-column chunks (K / 128)
  int units;               // pairs (gate/up) or tiles (down)
  int W;                   // units per work item = consumer warps
  int b_ntiles;            // B n-tiles reserved per stage (max over groups)
  int stages;              // ring stages
  GroupTab gt;
  const uint8_t* bin;      // B fragments of the input, [n-tile][chunk][2 KB]
  uint8_t* act_out;        // pair epilogue: B fragments of SiLU(gate)*up
  int out_nchunks;
  float* y_out;            // single epilogue: fp32 rows y[slot][y_ld]
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

__host__ __device__ inline int mm_stage_bytes(const MMParams& p, int ntl) {
  return ((p.W * ntl * p.tile_bytes + p.b_ntiles * kBfragChunkBytes) + 127) & ~127;
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Bounded wait that also gives up as soon as another warp aborted, or after
// `limit_ns` of wall time.  With the default limit each poll may sleep up to
// kWaitSleepNs and the clock is read every 16 polls; a limit shorter than one
// sleep (a test forcing the abort path) polls without sleeping and reads the
// clock every time, so such a wait gives up as soon as its first poll fails.
__device__ __forceinline__ bool wait_or_abort(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                              int* status, uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  if (*abort_flag) return false;
  const bool short_limit = limit_ns < kWaitSleepNs;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1; i < (1u << 31); ++i) {
    if (short_limit ? mbar_try_wait(bar, parity) : mbar_try_wait_sleep(bar, parity, kWaitSleepNs)) return true;
    if (short_limit || (i & 15) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > limit_ns) break;
    }
  }
  *abort_flag = 1;
  atomicOr(status, kDevTimeout);
  return false;
}

// Bounded wait that ignores the abort flag (used to drain copies in flight).
__device__ __forceinline__ void wait_drain(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0; i < (1u << 31); ++i) {
    if (mbar_try_wait(bar, parity)) return;
    if ((i & 63) == 63 && globaltimer_ns() - t0 > kWaitLimitNs) return;
  }
}

// Per-CTA state a consumer warp needs for the ring.
struct ConsumerCtx {
  uint8_t* ring;
  int stage_bytes;
  int S;
  int boff;
  int qoff[3];
  uint64_t* full;
  uint64_t* empty;
  volatile int* abort_flag;
  int cw;
  int lane;
  PolExtra ex;
};

// One work item of one consumer warp: the whole K loop for its unit with NTV
// n-tiles of tokens, then the epilogue.  n is the ring step of the item's
// first chunk.
template <class Pol, bool kPair, int NTV>
__device__ __forceinline__ void consume_item(const MMParams& p, const ConsumerCtx& x, int64_t item, int ipg,
                                             int64_t n) {
  constexpr int NTL = kPair ? 2 : 1;
  const int gi = (int)(item / ipg);
  const int u0 = (int)(item % ipg) * p.W;
  const int nu = min(p.W, p.units - u0);
  const int ntok = p.gt.ntok[gi];
  const int nt0 = p.gt.nt0[gi];
  const bool mine = x.cw < nu;
  const int lane = x.lane;
  // byte offsets of this warp's tile planes inside a stage (fixed for the item)
  int toff[NTL][3];
#pragma unroll
  for (int t = 0; t < NTL; ++t)
#pragma unroll
    for (int q = 0; q < 3; ++q) toff[t][q] = x.qoff[q] + (x.cw * NTL + t) * p.piece[q];
  const int boff = x.boff + lane * 64;

  float acc[NTL][NTV][4];
#pragma unroll
  for (int t = 0; t < NTL; ++t)
#pragma unroll
    for (int i = 0; i < NTV; ++i)
#pragma unroll
      for (int r = 0; r < 4; ++r) acc[t][i][r] = 0.f;

  for (int c = 0; c < p.nchunks; ++c, ++n) {
    const int slot = (int)(n % x.S);
    bool ok = wait_or_abort(smem_u32(x.full + slot), (uint32_t)((n / x.S) & 1), x.abort_flag, p.status);
    ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    if (ok && mine) {
      const uint8_t* st = x.ring + (int64_t)slot * x.stage_bytes;
      Pol P[NTL];
#pragma unroll
      for (int t = 0; t < NTL; ++t) {
        const uint8_t* planes[3] = {st + toff[t][0], st + toff[t][1], st + toff[t][2]};
        P[t].begin(planes, lane, x.ex);
      }
#pragma unroll
      for (int sp = 0; sp < 4; ++sp) {
        uint4 b[NTV];
#pragma unroll
        for (int i = 0; i < NTV; ++i) b[i] = lds128(st + boff + i * kBfragChunkBytes + sp * 16);
        if ((2 * sp) % Pol::kSlabsPerBlock == 0) {
#pragma unroll
          for (int t = 0; t < NTL; ++t) P[t].block((2 * sp) / Pol::kSlabsPerBlock);
        }
#pragma unroll
        for (int t = 0; t < NTL; ++t) {
          uint32_t a0[4], a1[4];
          P[t].frag2(sp, a0, a1);
#pragma unroll
          for (int i = 0; i < NTV; ++i) mma16816<Pol::kBF16>(acc[t][i], a0, b[i].x, b[i].y);
#pragma unroll
          for (int i = 0; i < NTV; ++i) mma16816<Pol::kBF16>(acc[t][i], a1, b[i].z, b[i].w);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(x.empty + slot));
  }

  if (!mine) return;
  const int u = u0 + x.cw;  // logical unit: I-tile of the pair, or H-tile
  const int g = lane >> 2, tq = lane & 3;
#pragma unroll
  for (int i = 0; i < NTV; ++i) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int row = g + 8 * (r >> 1);
      const int tok = 2 * tq + (r & 1);
      const bool valid = i * kNTile + tok < ntok;
      if constexpr (kPair) {
        const float val = valid ? silu_f(acc[0][i][r]) * acc[1][i][r] : 0.f;
        const int col = u * kTileRows + row;  // K index of the next projection
        uint8_t* dst = p.act_out + ((int64_t)(nt0 + i) * p.out_nchunks + (col >> 7)) * kBfragChunkBytes +
                       bfrag_byte(tok, col & 127);
        *reinterpret_cast<uint16_t*>(dst) = f32_to_act<Pol::kBF16>(val);
      } else {
        if (valid) {
          const int slot = p.gt.slot0[gi] + i * kNTile + tok;
          p.y_out[(int64_t)slot * p.y_ld + u * kTileRows + row] = acc[0][i][r];
        }
      }
    }
  }
}

template <class Pol, bool kPair>
__global__ void __launch_bounds__(32 * (kMaxConsumers + 1), 2) lut_mm_kernel(const MMParams p) {
  constexpr int NTL = kPair ? 2 : 1;
  constexpr int kR8Bytes = mm_r8_smem<Pol>();
  extern __shared__ __align__(128) uint8_t smem[];
  const int S = p.stages;
  uint32_t* r8tab = reinterpret_cast<uint32_t*>(smem);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kR8Bytes);
  uint64_t* empty = full + 8;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(full + 16);
  uint8_t* ring = smem + kR8Bytes + 256;
  const int stage_bytes = mm_stage_bytes(p, NTL);
  const int W = p.W;
  // stage layout: plane q of the W*NTL tiles at qoff[q], then the B n-tiles at boff
  int qoff[3];
  {
    int o = 0;
#pragma unroll
    for (int q = 0; q < 3; ++q) {
      qoff[q] = o;
      o += q < Pol::kNumPlanes ? W * NTL * p.piece[q] : 0;
    }
  }
  const int boff = W * NTL * p.tile_bytes;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if constexpr (kR8Bytes > 0) {
    for (int i = threadIdx.x; i < 256 * 32; i += blockDim.x) r8tab[i] = p.r8_table[i >> 5];
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_u32(full + s), 1);
      mbar_init(smem_u32(empty + s), W);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  const int ipg = (p.units + W - 1) / W;  // items per group
  const int64_t n_items = (int64_t)(*p.gt.n_groups) * ipg;
  const int64_t i0 = n_items * blockIdx.x / gridDim.x;
  const int64_t i1 = n_items * (blockIdx.x + 1) / gridDim.x;
  const int64_t total = (i1 - i0) * p.nchunks;

  if (warp == 0) {
    // ------------------------------------------------------------ producer --
    if (lane != 0) return;
    int64_t n = 0;
    for (; n < total; ++n) {
      const int slot = (int)(n % S);
      const int64_t use = n / S;
      if (use > 0 && !wait_or_abort(smem_u32(empty + slot), (uint32_t)((use - 1) & 1), abort_flag, p.status))
        break;
      if (*abort_flag) break;
      const int64_t item = i0 + n / p.nchunks;
      const int c = (int)(n % p.nchunks);
      const int gi = (int)(item / ipg);
      const int u0 = (int)(item % ipg) * W;
      const int nu = min(W, p.units - u0);
      const int ntv = (p.gt.ntok[gi] + kNTile - 1) / kNTile;
      const int nt0 = p.gt.nt0[gi];
      const uint8_t* base = p.w + (int64_t)p.gt.expert[gi] * p.wstride;
      uint8_t* dst = ring + (int64_t)slot * stage_bytes;
      const uint32_t bar = smem_u32(full + slot);
      mbar_expect_tx(bar, (uint32_t)(nu * NTL * p.tile_bytes + ntv * kBfragChunkBytes));
      const int64_t pt0 = (int64_t)u0 * NTL;
#pragma unroll
      for (int q = 0; q < Pol::kNumPlanes; ++q) {
        const uint8_t* src = base + p.plane_off[q] + ((int64_t)c * p.ntiles + pt0) * p.piece[q];
        bulk_g2s(smem_u32(dst + qoff[q]), src, (uint32_t)(nu * NTL * p.piece[q]), bar);
      }
      for (int i = 0; i < ntv; ++i) {
        const uint8_t* src = p.bin + ((int64_t)(nt0 + i) * p.nchunks + c) * kBfragChunkBytes;
        bulk_g2s(smem_u32(dst + boff + i * kBfragChunkBytes), src, kBfragChunkBytes, bar);
      }
    }
    if (*abort_flag) {
      // let the copies already issued land before the CTA's shared memory goes away
      for (int64_t m = n - S > 0 ? n - S : 0; m < n; ++m) wait_drain(smem_u32(full + m % S), (uint32_t)((m / S) & 1));
    }
    return;
  }

  // -------------------------------------------------------------- consumers --
  const int cw = warp - 1;
  PolExtra ex;
  ex.r8_table = r8tab;
  ex.r8_mask = p.r8_mask;
  ConsumerCtx ctx{ring, stage_bytes, S, boff, {qoff[0], qoff[1], qoff[2]}, full, empty, abort_flag, cw, lane, ex};
  int64_t n = 0;
  for (int64_t item = i0; item < i1; ++item) {
    const int gi = (int)(item / ipg);
    const int ntv = (p.gt.ntok[gi] + kNTile - 1) / kNTile;
    switch (ntv) {  // the n-tile count is fixed per item: one branch-free instance each
      case 1: consume_item<Pol, kPair, 1>(p, ctx, item, ipg, n); break;
      case 2: consume_item<Pol, kPair, 2>(p, ctx, item, ipg, n); break;
      case 3: consume_item<Pol, kPair, 3>(p, ctx, item, ipg, n); break;
      default: consume_item<Pol, kPair, 4>(p, ctx, item, ipg, n); break;
    }
    n += p.nchunks;
  }
}

// Host-side launch: ring depth from the shared-memory budget, grid from occupancy.
template <class Pol, bool kPair>
inline int mm_smem_bytes(const MMParams& p) {
  return mm_r8_smem<Pol>() + 256 + p.stages * mm_stage_bytes(p, kPair ? 2 : 1);
}

template <class Pol, bool kPair>
inline cudaError_t launch_mm(MMParams p, int num_sms, cudaStream_t stream) {
  const int stage = mm_stage_bytes(p, kPair ? 2 : 1);
  p.stages = std::max(3, std::min(8, kRingBudget / stage));
  const int smem = mm_smem_bytes<Pol, kPair>(p);
  const int threads = 32 * (p.W + 1);
  auto kern = lut_mm_kernel<Pol, kPair>;
  // attribute + occupancy per (instantiation, device, smem size, block size),
  // computed once (zero: not yet computed)
  static std::mutex mu;
  static int cached_smem[kMaxDevices], cached_threads[kMaxDevices], cached_per_sm[kMaxDevices];
  const int dev = cache_device();
  int per_sm;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 0 || cached_smem[dev] != smem || cached_threads[dev] != threads) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return e;
      int nb = 0;
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, threads, smem);
      if (e != cudaSuccess) return e;
      per_sm = nb < 1 ? 1 : nb;
      if (dev >= 0) {
        cached_per_sm[dev] = per_sm;
        cached_smem[dev] = smem;
        cached_threads[dev] = threads;
      }
    } else {
      per_sm = cached_per_sm[dev];
    }
  }
  kern<<<num_sms * per_sm, threads, smem, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace blut
