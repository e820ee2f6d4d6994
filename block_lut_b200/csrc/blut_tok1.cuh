// Single-token MoE layer (one token per call, the decode regime the
// reference's GEMV targets): three launches instead of the general path's
// router / plan / gather / gate-up / slice-sum / down / combine chain.
//
//   tok1_logits_kernel (blut_moe.cu)  the router logits, the shared-expert
//       gate, zeroed counters and status;
//   tok1_kernel<Dec, pair = true>    the top-k (in every routed CTA), then
//       gate/up of every routed group and of the shared expert in one
//       persistent launch; the last CTA to finish a 128-row unit (both of
//       its tiles, every K slice) sums the slices and writes SiLU(gate) * up
//       for that unit;
//   tok1_kernel<Dec, pair = false>   down of every group and the shared
//       expert; the last CTA to finish an output tile sums, for its rows,
//       every group's slices weighted by the routing weight plus the shared
//       expert's slices weighted by its gate, and rounds once.
//
// The GEMV is the one of tc_gemv_kernel (one thread per weight row, the
// format's decode, fp32 FMAs) made persistent: the CTAs of the routed part
// walk the routed items and those of the shared part the shared items, and
// while one item is computed the thread's register ring already holds the
// next item's weights.  Activations are read row-major (the token row for
// gate/up, a group's SiLU * up row for down), so no gather is needed.
#pragma once

#include "blut_route.cuh"
#include "blut_tc.cuh"

namespace blut {

constexpr int kTok1Threads = kTcRows;
// Pieces of its row a thread keeps in flight, and CTAs per SM: a two-piece
// ring leaves registers for five CTAs (20 warps) per SM, which hides the
// per-item latencies better than a four-piece ring at four CTAs (measured
// on config 2 at batch 1: 876 -> 946 tokens/s).
constexpr int kTok1Ring = 2;
constexpr int kTok1CtasPerSm = 5;

// One matrix of a single-token pass.
struct Tok1Mat {
  TcParams p;          // planes, tiles, blocks, K slices (ks, bps), decode constants, weights
  int64_t n_items;     // group bound * ntiles * ks
  int ctas;            // CTAs of the persistent grid that work on this matrix
  const uint16_t* xin; // activation rows; group g reads xin + g * x_ld
  int64_t x_ld;
  float* part;         // gate/up: [group][unit][ks][gate | up][128]; down: [ks][group bound][hidden]
  uint16_t* act;       // gate/up: SiLU * up rows, [group][rows / 2]
  int cnt0;            // gate/up: first completion counter of this matrix ([group][unit])
};

// Experts of at most this many: the gate/up CTAs take the top-k themselves.
constexpr int kTok1MaxExperts = 256;

struct Tok1Args {
  Tok1Mat m[2];        // routed experts, shared expert (m[1].ctas == 0: none)
  int* groups;         // [0] routed groups, [1 + g] expert of group g (written by the gate/up launch)
  float* gw;           // [g] routing weight of group g
  const float* sg;     // shared expert gate (nullptr: 1)
  int* cnt;            // completion counters (zeroed by the logits kernel)
  int gbound;          // routed group bound (the top-k)
  void* out;           // the layer output [hidden], fp16 / bf16 or fp32
  int out_f32;
  int hidden;
  // routing, used by the gate/up launch
  const float* logits;     // router logits of the token [num_experts]; nullptr: the caller's ids
  const int32_t* ids_in;   // the caller's top-k ids and weights [gbound]
  const float* tw_in;
  int num_experts, renorm;
  int* status;
  int has_shared;
};

// Warp 0 of a routed gate/up CTA: the token's top-k (softmax over the
// logits, lowest index on ties, optional renormalisation) or the caller's
// ids, as the group table in shared memory (one group per valid slot, in slot
// order).  CTA 0 also publishes the table for the down launch, flags ids out
// of range (-1 is an empty slot) and, when the token has no expert and there
// is no shared expert, writes the zero output no GEMV item will write.
__device__ __forceinline__ void tok1_route_warp(const Tok1Args& a, int* s_groups, float* s_gw, bool publish) {
  __shared__ int32_t sids[32];
  __shared__ float stw[32];
  const int lane = threadIdx.x & 31;
  const int K = a.gbound, E = a.num_experts;
  if (a.logits) {
    if (E <= 64) warp_topk_n<2>(a.logits, E, K, a.renorm, sids, stw);
    else if (E <= 128) warp_topk_n<4>(a.logits, E, K, a.renorm, sids, stw);
    else warp_topk_n<8>(a.logits, E, K, a.renorm, sids, stw);
  } else if (lane < K) {
    sids[lane] = a.ids_in[lane];
    stw[lane] = a.tw_in[lane];
  }
  __syncwarp();
  const int id = lane < K ? sids[lane] : -1;
  const bool ok = lane < K && id >= 0 && id < E;
  const unsigned msk = __ballot_sync(0xffffffffu, ok);
  if (ok) {
    const int g = __popc(msk & ((1u << lane) - 1u));
    s_groups[1 + g] = id;
    s_gw[g] = stw[lane];
    if (publish) {
      a.groups[1 + g] = id;
      a.gw[g] = stw[lane];
    }
  }
  if (lane == 0) s_groups[0] = __popc(msk);
  if (!publish) return;
  if (lane == 0) a.groups[0] = __popc(msk);
  if (lane < K && !ok && id != -1) atomicOr(a.status, kDevBadExpert);
  if (msk == 0 && !a.has_shared) {
    for (int h = lane; h < a.hidden; h += 32) {
      if (a.out_f32)
        static_cast<float*>(a.out)[h] = 0.f;
      else
        static_cast<uint16_t*>(a.out)[h] = 0;
    }
  }
}

struct Tok1Item {
  int gi, pt, s, b0, n;
  const uint8_t* base;
};

// Item `it` of matrix m (ordered (group, tile, slice)); false past the last
// item or at a group that does not exist (every later item's group is larger).
template <class Dec>
__device__ __forceinline__ bool tok1_resolve(const int* groups, const Tok1Mat& m, bool shared, int ng, int64_t it,
                                             Tok1Item& r) {
  const TcParams& p = m.p;
  if (it >= m.n_items) return false;
  r.s = (int)(it % p.ks);
  r.pt = (int)((it / p.ks) % p.ntiles);
  r.gi = (int)(it / ((int64_t)p.ks * p.ntiles));
  if (r.gi >= ng) return false;
  r.b0 = r.s * p.bps;
  const int b1 = min(p.nblocks, r.b0 + p.bps);
  r.n = r.b0 < b1 ? (b1 - r.b0) * (Dec::kDense ? 1 : Dec::kHalves) : 0;
  const int e = shared ? 0 : groups[1 + r.gi];
  r.base = p.w + (int64_t)e * p.wstride;
  return true;
}

// Columns of one item's activation slice a thread stages: an item is 256
// columns (tok1_slices), two to four rounds of the thread's register ring.
constexpr int kTok1XPer = 2;
constexpr int kTok1MaxCols = kTok1XPer * kTok1Threads;

// Sum of n fp32 values at p, p + stride, ... in index order, eight loads in
// flight at a time (L2: other CTAs wrote them in this launch).
__device__ __forceinline__ float tok1_sum(const float* p, int n, int64_t stride) {
  // eight loads in flight per round, the ragged last round included
  float s = 0.f;
  for (int i = 0; i < n; i += 8) {
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = i + k < n ? __ldcg(p + (i + k) * stride) : 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (i + k < n) s += v[k];
  }
  return s;
}

// The epilogue of item `it`, run by the CTA whose completion of it was the
// last of its unit (gate/up) or output tile (down).
template <class Dec, bool PAIR>
__device__ __forceinline__ void tok1_epilogue(const Tok1Args& a, const Tok1Mat& m, const Tok1Item& it,
                                              const int* groups, const float* gw) {
  const TcParams& p = m.p;
  const int row = threadIdx.x;
  if constexpr (PAIR) {
    // every slice of both tiles of this unit is in: SiLU(gate) * up
    const int unit = it.pt >> 1;
    const float* src = m.part + (((int64_t)it.gi * p.units + unit) * p.ks) * (2 * kTcRows) + row;
    const float g = tok1_sum(src, p.ks, 2 * kTcRows);
    const float u = tok1_sum(src + kTcRows, p.ks, 2 * kTcRows);
    m.act[(int64_t)it.gi * (p.ntiles / 2) * kTcRows + unit * kTcRows + row] = f32_to_act<Dec::kBF16>(silu_f(g) * u);
  } else {
    // every contribution to this output tile is in: the weighted combine
    const int h = it.pt * kTcRows + row;
    const Tok1Mat& r = a.m[0];
    const int ngr = min(groups[0], a.gbound);
    float o = 0.f;
#pragma unroll 2
    for (int g = 0; g < ngr; ++g)
      o = fmaf(gw[g], tok1_sum(r.part + (int64_t)g * a.hidden + h, r.p.ks, (int64_t)a.gbound * a.hidden), o);
    if (a.m[1].ctas > 0) {
      const Tok1Mat& sm = a.m[1];
      o = fmaf(a.sg ? *a.sg : 1.f, tok1_sum(sm.part + h, sm.p.ks, a.hidden), o);
    }
    if (a.out_f32)
      static_cast<float*>(a.out)[h] = o;
    else
      static_cast<uint16_t*>(a.out)[h] = f32_to_act<Dec::kBF16>(o);
  }
}

// Loop of one CTA over its items.  Per item: the activation slice staged
// from registers loaded during the previous item, the weights already in the
// register ring, the dot products with the next item's loads in flight, the
// fp32 result stored, then one thread counts the item done (fence + atomic)
// and reads that count only after the next item's compute, so neither the
// atomic's round trip nor the staging loads sit on the critical path.  The
// CTA that completes a unit or output tile runs its epilogue one item later.
template <class Dec, bool PAIR>
__device__ __forceinline__ void tok1_run(const Tok1Args& a, const Tok1Mat& m, const int* groups, const float* gw,
                                         bool shared, int cta, int nctas, uint8_t* smem) {
  constexpr int KB = Dec::KB;
  constexpr int PF = kTok1Ring;
  constexpr int W = Dec::kDense ? Dec::KB : 64;  // columns per piece
  using U = typename std::conditional<Dec::kDense, TcDenseBlk<Dec::kBF16>, typename Dec::Half>::type;
  static_assert(kTok1MaxCols % (PF * W) == 0, "an item is whole rounds of the register ring");
  const TcParams& p = m.p;
  const int row = threadIdx.x;
  const int ng = shared ? 1 : min(groups[0], a.gbound);
  __shared__ int s_last;
  uint32_t tab = 0;
  if constexpr (Dec::kR8) tab = smem_u32(smem) + (row & 31) * 4;
  float* xs = reinterpret_cast<float*>(smem + tc_table_bytes<Dec>());
  int64_t item = cta;
  Tok1Item cur, nxt, prev{};
  if (!tok1_resolve<Dec>(groups, m, shared, ng, item, cur)) return;  // uniform over the CTA
  if constexpr (Dec::kR8) tc_fill_r8_table(reinterpret_cast<uint32_t*>(smem), p.r8_table);
  U ring[PF];
#pragma unroll
  for (int j = 0; j < PF; ++j)
    if (j < cur.n) tc_gemv_load<Dec>(p, cur.base, cur.pt, cur.b0, j, row, tab, ring[j]);
  auto load_x = [&](const Tok1Item& it, uint16_t (&xr)[kTok1XPer]) {
    const uint16_t* xrow = m.xin + (int64_t)it.gi * m.x_ld + it.b0 * KB;
#pragma unroll
    for (int k = 0; k < kTok1XPer; ++k) {
      const int col = threadIdx.x + k * kTok1Threads;
      xr[k] = col < it.n * W ? xrow[col] : uint16_t(0);
    }
  };
  uint16_t xr[kTok1XPer];
  load_x(cur, xr);
  int prev_old = 0, prev_target = 0;  // thread 0: the count before the previous item's increment, and its goal
  bool have_prev = false;
  const int down_target = PAIR ? 0 : min(groups[0], a.gbound) * a.m[0].p.ks + (a.m[1].ctas > 0 ? a.m[1].p.ks : 0);
  for (;;) {
    const bool more = tok1_resolve<Dec>(groups, m, shared, ng, item + nctas, nxt);
    __syncthreads();  // the previous item's reads of xs are done (and the R8 table is complete)
#pragma unroll
    for (int k = 0; k < kTok1XPer; ++k) xs[threadIdx.x + k * kTok1Threads] = act_to_f32<Dec::kBF16>(xr[k]);
    __syncthreads();  // xs complete
    if (more) load_x(nxt, xr);
    float2 acc[1] = {make_float2(0.f, 0.f)};
    // the item's pieces in rounds of PF: a slot's next content is the piece
    // PF further on in this item, or in the last round the same slot's piece
    // of the CTA's next item
    for (int i0 = 0; i0 < cur.n; i0 += PF) {
#pragma unroll
      for (int j = 0; j < PF; ++j) {
        const int i = i0 + j;
        if (i < cur.n) {
          if constexpr (Dec::kDense) {
            uint32_t o[16];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              o[4 * k] = ring[j].v[k].x; o[4 * k + 1] = ring[j].v[k].y;
              o[4 * k + 2] = ring[j].v[k].z; o[4 * k + 3] = ring[j].v[k].w;
            }
            tc_gemv_fma32<Dec::kBF16, 1>(o, xs, 0, i * W, acc);
          } else {
#pragma unroll
            for (int qq = 0; qq < 2; ++qq) {
              uint32_t o[16];
              Dec::lookup_q(ring[j], qq, o, p.mul);
              tc_gemv_fma32<Dec::kBF16, 1>(o, xs, 0, i * W + 32 * qq, acc);
            }
          }
        }
        if (i + PF < cur.n)
          tc_gemv_load<Dec>(p, cur.base, cur.pt, cur.b0, i + PF, row, tab, ring[j]);
        else if (i0 + PF >= cur.n && more && j < nxt.n)
          tc_gemv_load<Dec>(p, nxt.base, nxt.pt, nxt.b0, j, row, tab, ring[j]);
      }
    }
    const float v = acc[0].x + acc[0].y;
    int* counter;
    int target;
    if constexpr (PAIR) {
      const int unit = cur.pt >> 1;
      float* mine = m.part + (((int64_t)cur.gi * p.units + unit) * p.ks) * (2 * kTcRows);
      mine[cur.s * (2 * kTcRows) + (cur.pt & 1) * kTcRows + row] = v;
      counter = a.cnt + m.cnt0 + cur.gi * p.units + unit;
      target = 2 * p.ks;  // both tiles of the unit, every slice
    } else {
      m.part[((int64_t)cur.s * (shared ? 1 : a.gbound) + cur.gi) * a.hidden + cur.pt * kTcRows + row] = v;
      counter = a.cnt + cur.pt;  // one counter per output tile, over both matrices
      target = down_target;
    }
    __syncthreads();  // this item's results are stored (the fence below publishes them for the whole CTA)
    if (threadIdx.x == 0) {
      s_last = have_prev && prev_old == prev_target - 1;  // the previous item's count is back by now
      __threadfence();
      prev_old = atomicAdd(counter, 1);
      prev_target = target;
    }
    __syncthreads();  // s_last visible
    if (s_last) {
      __threadfence();
      tok1_epilogue<Dec, PAIR>(a, m, prev, groups, gw);
    }
    prev = cur;
    have_prev = true;
    if (!more) break;
    cur = nxt;
    item += nctas;
  }
  if (threadIdx.x == 0) s_last = prev_old == prev_target - 1;
  __syncthreads();
  if (s_last) {
    __threadfence();
    tok1_epilogue<Dec, PAIR>(a, m, prev, groups, gw);
  }
}

// CTAs [0, m[0].ctas) work on the routed experts, the rest on the shared one.
// In the gate/up launch every routed CTA takes the token's top-k first (the
// shared expert's CTAs need none); the down launch reads the table CTA 0 of
// the gate/up launch published.
// A down-mode launch with no group table (groups == nullptr) is a single
// matrix: one group, expert 0, weight 1 (blut_matmul at one token).
template <class Dec, bool PAIR>
__global__ void __launch_bounds__(kTok1Threads, kTok1CtasPerSm) tok1_kernel(const Tok1Args a) {
  extern __shared__ __align__(16) uint8_t tsm[];
  __shared__ int s_groups[33];
  __shared__ float s_gw[32];
  if ((int)blockIdx.x < a.m[0].ctas) {
    const int* groups = a.groups;
    const float* gw = a.gw;
    if (PAIR || !a.groups) {
      if (PAIR) {
        if (threadIdx.x < 32) tok1_route_warp(a, s_groups, s_gw, blockIdx.x == 0);
      } else if (threadIdx.x == 0) {
        s_groups[0] = 1;
        s_groups[1] = 0;
        s_gw[0] = 1.f;
      }
      __syncthreads();
      groups = s_groups;
      gw = s_gw;
    }
    tok1_run<Dec, PAIR>(a, a.m[0], groups, gw, false, blockIdx.x, a.m[0].ctas, tsm);
  } else {
    tok1_run<TcDecDense<Dec::kBF16>, PAIR>(a, a.m[1], a.groups, a.gw, true, blockIdx.x - a.m[0].ctas, a.m[1].ctas,
                                           tsm);
  }
}

// Shared-memory bytes of a tok1 launch: the FMT_R8 table, then the staged
// activation slice (every thread writes its kTok1XPer columns).
template <class Dec>
inline int tok1_smem(const Tok1Args&) {
  return tc_table_bytes<Dec>() + kTok1MaxCols * 4;
}

// A routed weight byte counts as kTok1RoutedCost shared (dense) bytes when
// the CTAs are split: the routed CTAs also take the top-k and decode the
// format.  Measured on Qwen1.5-MoE at one token (bf16 shared expert, 4-bit
// g64 experts): 1054 tokens/s at 1.0, 1075 at 1.5, 1117 at 2.0.
constexpr double kTok1RoutedCost = 2.0;

// CTAs of the routed and shared parts: the resident CTAs of the GPU, split
// in proportion to the weight bytes each part reads (routed bytes weighted).
template <class Dec, bool PAIR>
inline cudaError_t launch_tok1_dec(Tok1Args a, double routed_bytes, double shared_bytes, cudaStream_t stream) {
  const int smem = tok1_smem<Dec>(a);
  auto kern = tok1_kernel<Dec, PAIR>;
  static std::mutex mu;
  static int cached_smem[kMaxDevices], cached_per_sm[kMaxDevices];
  const int dev = cache_device();
  int per_sm = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && cached_smem[dev] >= smem) {
      per_sm = cached_per_sm[dev];
    } else {
      const int attr = std::max(smem, 48 * 1024);
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, attr);
      if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kTok1Threads, smem);
      if (e != cudaSuccess) return e;
      per_sm = std::max(1, per_sm);
      if (dev >= 0) {
        cached_smem[dev] = attr;
        cached_per_sm[dev] = per_sm;
      }
    }
  }
  const int64_t total = (int64_t)num_sms() * per_sm;
  const bool sh = a.m[1].n_items > 0;
  int64_t cr = total, cs = 0;
  if (sh) {
    const double rw = kTok1RoutedCost * routed_bytes;
    cs = std::max<int64_t>(1, (int64_t)(total * shared_bytes / std::max(1.0, rw + shared_bytes) + 0.5));
    cs = std::min<int64_t>(cs, total - 1);
    cr = total - cs;
  }
  // a part with fewer items than its share of the CTAs hands the rest to the other
  cs = std::min<int64_t>(cs, a.m[1].n_items);
  cr = std::max<int64_t>(1, std::min<int64_t>(total - cs, a.m[0].n_items));
  if (sh) cs = std::max<int64_t>(1, std::min<int64_t>(total - cr, a.m[1].n_items));
  a.m[0].ctas = (int)cr;
  a.m[1].ctas = (int)cs;
  kern<<<(unsigned)(cr + cs), kTok1Threads, smem, stream>>>(a);
  return cudaGetLastError();
}

// Per-format dispatch (blut_tok1.cu).
cudaError_t launch_tok1(const blut_mat_desc& d, const Tok1Args& a, bool pair, double routed_bytes,
                        double shared_bytes, cudaStream_t stream);

}  // namespace blut
