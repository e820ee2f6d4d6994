// MoE layer orchestration: router, routing plan, B-fragment gather, the LUT
// matmul launches and the weighted combine.  All launches go on the caller's
// stream; nothing synchronises the host and nothing allocates.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "blut_internal.h"
#include "blut_route.cuh"
#include "blut_tc.cuh"
#include "blut_tok1.cuh"

namespace blut {

// --------------------------------------------------------------- router ---
// Router logits, fp32 accumulation: one warp per (row, token) dot product,
// 8 warps per CTA; each lane issues all of its 16-byte loads before the FMAs
// (4 independent accumulators).  Row r < E reads w_main[r]; row E (when
// w_gate is set) reads the shared-expert gate vector.
// One warp's fp32 dot product of x and w (H elements).  Lane l takes the
// 8-element chunks l, l + 32, ...; chunk c accumulates into acc[c % 4], in
// chunk order, and the four sums are added pairwise, then across the warp.
// Each lane issues eight chunks' weight and activation loads before their
// FMAs.
template <bool BF16>
__device__ __forceinline__ float router_dot(const uint16_t* xr, const uint16_t* __restrict__ wr, int H, int lane) {
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int k0 = lane * 8; k0 < H; k0 += 32 * 8 * 8) {
    uint4 wv[8], xv[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int k = k0 + q * 256;
      wv[q] = k < H ? *reinterpret_cast<const uint4*>(wr + k) : make_uint4(0, 0, 0, 0);
      xv[q] = k < H ? *reinterpret_cast<const uint4*>(xr + k) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int k = k0 + q * 256;
      if (k >= H) break;
      const uint16_t* xs = reinterpret_cast<const uint16_t*>(&xv[q]);
      const uint16_t* ws = reinterpret_cast<const uint16_t*>(&wv[q]);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[q & 3] = fmaf(act_to_f32<BF16>(xs[e]), act_to_f32<BF16>(ws[e]), acc[q & 3]);
    }
  }
  float s = (acc[0] + acc[1]) + (acc[2] + acc[3]);
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  return s;
}

template <bool BF16>
__global__ void __launch_bounds__(256) router_logits_kernel(const uint16_t* __restrict__ x,
                                                            const uint16_t* __restrict__ w_main,
                                                            const uint16_t* __restrict__ w_gate, int T, int H,
                                                            int E, float* __restrict__ logits) {
  const int lane = threadIdx.x & 31;
  const int R = E + (w_gate ? 1 : 0);
  const int64_t task = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (task >= (int64_t)R * T) return;
  const int t = (int)(task / R), r = (int)(task % R);
  const uint16_t* wr = r < E ? w_main + (int64_t)r * H : w_gate;
  const float s = router_dot<BF16>(x + (int64_t)t * H, wr, H, lane);
  if (lane == 0) logits[(int64_t)t * R + r] = s;
}

// Standalone top-k over router logits (the blut_router entry point).
__global__ void __launch_bounds__(256) topk_kernel(const float* __restrict__ logits, int T, int E, int K,
                                                   int renorm, int has_gate, int32_t* __restrict__ ids,
                                                   float* __restrict__ tw, float* __restrict__ sg) {
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= T) return;
  const int R = E + (has_gate ? 1 : 0);
  warp_topk(logits + (int64_t)t * R, E, K, renorm, ids + (int64_t)t * K, tw + (int64_t)t * K,
            has_gate ? sg + t : nullptr, has_gate != 0);
}

// Single-token path (blut_tok1.cuh), launch 1 of 3: the token's router
// logits (experts, then the shared-expert gate row, whose sigmoid goes to
// *sg), a warp per row, eight rows per CTA; CTA 0 also zeroes the status word
// and the completion counters of the two GEMV launches.  The top-k runs in
// the gate/up launch, in every CTA that needs it.
template <bool BF16>
__global__ void __launch_bounds__(256) tok1_logits_kernel(const uint16_t* __restrict__ x,
                                                          const uint16_t* __restrict__ w_main,
                                                          const uint16_t* __restrict__ w_gate, int H, int e_main,
                                                          float* __restrict__ logits, float* __restrict__ sg,
                                                          int* __restrict__ cnt, int ncnt, int* __restrict__ status) {
  const int lane = threadIdx.x & 31;
  const int R = e_main + (w_gate ? 1 : 0);
  if (blockIdx.x == 0) {
    for (int i = threadIdx.x; i < ncnt; i += blockDim.x) cnt[i] = 0;
    if (threadIdx.x == 0) *status = 0;  // the status word reports this call only, as the plan kernel's does
  }
  const int r = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (r >= R) return;
  const float v = router_dot<BF16>(x, r < e_main ? w_main + (int64_t)r * H : w_gate, H, lane);
  if (lane == 0) {
    logits[r] = v;
    if (r == e_main) *sg = 1.f / (1.f + expf(-v));
  }
}

// ----------------------------------------------------------------- plan ---
// Single CTA.  (1) With router logits: top-k per token (a warp per token)
// and the shared-expert gate.  (2) Per-expert counts; parallel exclusive
// scans give each expert its slot range, its groups of <= 32 tokens and their
// 8-token n-tiles (ceil(count / 8) of them).  (3) Slots are taken with
// per-expert atomic counters: which slot a (token, k) pair gets inside its
// expert does not change any result, because every token is its own MMA
// column.  (4) The shared expert's groups cover the tokens in order.
__global__ void __launch_bounds__(1024) plan_kernel(const int32_t* __restrict__ ids_in,
                                                    const float* __restrict__ logits, int topk_e, int R,
                                                    int num_tokens, int top_k, int num_experts, int renorm,
                                                    int has_gate, int has_shared, int gtok, int sgtok,
                                                    PlanPtrs pp, int32_t* __restrict__ ids_out,
                                                    float* __restrict__ tw_out, float* __restrict__ sg_out) {
  __shared__ int cnt[kMaxExperts];
  __shared__ int off[kMaxExperts];
  __shared__ int goff[kMaxExperts];
  __shared__ int toff[kMaxExperts];
  __shared__ int fill[kMaxExperts];
  __shared__ int tot[3];
  const int S = num_tokens * top_k;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) *pp.status = 0;
  if (threadIdx.x < kNumCounters) pp.counters[threadIdx.x] = 0;
  if (logits) {  // row t: topk_e expert logits, then the gate logit when has_gate
    for (int t = warp; t < num_tokens; t += 32) {
      warp_topk(logits + (int64_t)t * R, topk_e, ids_in ? 0 : top_k, renorm, ids_out + (int64_t)t * top_k,
                tw_out + (int64_t)t * top_k, sg_out + t, has_gate != 0);
    }
  }
  for (int e = threadIdx.x; e < num_experts; e += blockDim.x) {
    cnt[e] = 0;
    fill[e] = 0;
  }
  __syncthreads();
  const int32_t* ids = ids_in ? ids_in : ids_out;
  for (int q = threadIdx.x; q < S; q += blockDim.x) {
    const int e = ids[q];
    if (e >= 0 && e < num_experts) atomicAdd(&cnt[e], 1);
    else if (e != -1) atomicOr(pp.status, kDevBadExpert);  // -1 = empty slot
  }
  __syncthreads();
  if (warp == 0) {  // exclusive scans of tokens, groups and n-tiles over the experts
    int run_t = 0, run_g = 0, run_n = 0;
    for (int base = 0; base < num_experts; base += 32) {
      const int e = base + lane;
      const int c = e < num_experts ? cnt[e] : 0;
      int vt = c, vg = (c + gtok - 1) / gtok, vn = (c + kNTile - 1) / kNTile;
      int st = vt, sgp = vg, sn = vn;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int a = __shfl_up_sync(0xffffffffu, st, o);
        const int b = __shfl_up_sync(0xffffffffu, sgp, o);
        const int d = __shfl_up_sync(0xffffffffu, sn, o);
        if (lane >= o) { st += a; sgp += b; sn += d; }
      }
      if (e < num_experts) {
        off[e] = run_t + st - vt;
        goff[e] = run_g + sgp - vg;
        toff[e] = run_n + sn - vn;
      }
      run_t += __shfl_sync(0xffffffffu, st, 31);
      run_g += __shfl_sync(0xffffffffu, sgp, 31);
      run_n += __shfl_sync(0xffffffffu, sn, 31);
    }
    if (lane == 0) {
      tot[0] = run_t;
      tot[1] = run_g;
      tot[2] = run_n;
    }
  }
  __syncthreads();
  // groups and n-tiles of each expert (a thread per expert)
  for (int e = threadIdx.x; e < num_experts; e += blockDim.x) {
    const int c = cnt[e];
    int gi = goff[e], nt = toff[e];
    for (int q = 0; q * gtok < c; ++q, ++gi) {
      const int ntok = min(gtok, c - q * gtok);
      pp.g_expert[gi] = e;
      pp.g_slot0[gi] = off[e] + q * gtok;
      pp.g_ntok[gi] = ntok;
      pp.g_nt0[gi] = nt;
      for (int i = 0; i * kNTile < ntok; ++i, ++nt) {
        pp.nt_slot0[nt] = off[e] + q * gtok + i * kNTile;
        pp.nt_cnt[nt] = min(kNTile, ntok - i * kNTile);
      }
    }
  }
  if (threadIdx.x == 0) {
    pp.meta[0] = tot[1];
    pp.meta[1] = tot[2];
    int sng = 0, snt = 0;
    if (has_shared) {
      for (int q = 0; q * sgtok < num_tokens; ++q) {
        const int ntok = min(sgtok, num_tokens - q * sgtok);
        pp.sg_expert[sng] = 0;
        pp.sg_slot0[sng] = q * sgtok;
        pp.sg_ntok[sng] = ntok;
        pp.sg_nt0[sng] = snt;
        snt += (ntok + kNTile - 1) / kNTile;
        ++sng;
      }
    }
    pp.meta[2] = sng;
    pp.meta[3] = snt;
  }
  for (int q = threadIdx.x; q < S; q += blockDim.x) {
    const int e = ids[q];
    if (e < 0 || e >= num_experts) {
      pp.tk_slot[q] = -1;
      continue;
    }
    const int slot = off[e] + atomicAdd(&fill[e], 1);
    pp.tk_slot[q] = slot;
    pp.slot_tok[slot] = q / top_k;
  }
}

// --------------------------------------------------------------- gather ---
// Activations of one (n-tile, 128-column chunk) block, 32 threads.  z = 0:
// routed n-tiles (token of slot via slot_tok), z = 1: shared expert (slot =
// token).  Bit z of tc_mask selects the tcgen05 operand order
// (tc_bact_byte) for that destination instead of mma.sync B fragments.
__global__ void __launch_bounds__(32) gather_bfrag_kernel(const uint16_t* __restrict__ x, int hidden, PlanPtrs pp,
                                                          uint8_t* __restrict__ xf, uint8_t* __restrict__ xfs,
                                                          int tc_mask, int kb_r, int kb_s, int64_t ntstride_r,
                                                          int64_t ntstride_s) {
  const bool shared = blockIdx.z == 1;
  const int nt = blockIdx.x;
  const int c = blockIdx.y;
  const int n_nt = shared ? pp.meta[3] : pp.meta[1];
  if (nt >= n_nt) return;
  const int nchunks = hidden / kChunk;
  const int lane = threadIdx.x;
  const int g = lane >> 2, tq = lane & 3;
  int cntv, slot0;
  if (shared) {
    slot0 = nt * kNTile;  // shared groups and their n-tiles are 8-aligned
    cntv = 0;
    // count tokens of this n-tile: the last group may be partial
    const int sng = pp.meta[2];
    for (int q = 0; q < sng; ++q) {
      const int nt0 = pp.sg_nt0[q];
      const int ntok = pp.sg_ntok[q];
      if (nt >= nt0 && nt < nt0 + (ntok + kNTile - 1) / kNTile) {
        slot0 = pp.sg_slot0[q] + (nt - nt0) * kNTile;
        cntv = min(kNTile, ntok - (nt - nt0) * kNTile);
      }
    }
  } else {
    slot0 = pp.nt_slot0[nt];
    cntv = pp.nt_cnt[nt];
  }
  if ((tc_mask >> blockIdx.z) & 1) {
    // 16 column groups x 8 tokens of 16 bytes: lane -> token lane & 7, groups (lane >> 3) + 4i
    const int tok = lane & 7;
    const uint16_t* row = nullptr;
    if (tok < cntv) {
      const int slot = slot0 + tok;
      row = x + (int64_t)(shared ? slot : pp.slot_tok[slot]) * hidden + c * kChunk;
    }
    uint8_t* dst = shared ? xfs : xf;
    const int kb = shared ? kb_s : kb_r;
    const int64_t nts = shared ? ntstride_s : ntstride_r;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int kg = (lane >> 3) + 4 * i;
      const uint4 v = row ? *reinterpret_cast<const uint4*>(row + kg * 8) : make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(dst + tc_bact_off((int64_t)nt * kNTile + tok, c * kChunk + kg * 8, kb, nts)) = v;
    }
    return;
  }
  uint32_t wv[16];
  if (g < cntv) {
    const int slot = slot0 + g;
    const int tok = shared ? slot : pp.slot_tok[slot];
    const uint32_t* row = reinterpret_cast<const uint32_t*>(x + (int64_t)tok * hidden + c * kChunk);
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      wv[2 * s] = row[(16 * s + 2 * tq) >> 1];
      wv[2 * s + 1] = row[(16 * s + 2 * tq + 8) >> 1];
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) wv[i] = 0;
  }
  uint8_t* dst = (shared ? xfs : xf) + ((int64_t)nt * nchunks + c) * kBfragChunkBytes + lane * 64;
  uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int i = 0; i < 4; ++i) d4[i] = make_uint4(wv[4 * i], wv[4 * i + 1], wv[4 * i + 2], wv[4 * i + 3]);
}

// ------------------------------------------------------ split-K epilogue ---
// Gate/up passes computed in K slices: for unit ku = group * units + u and
// each of its (row, token), sum the slices' fp32 partials in slice order and
// write SiLU(gate) * up into the down projection's activations.  Block
// (ku, j): 256 threads = 8 rows x 32 tokens, rows 8j .. 8j + 7 of the unit.
template <bool BF16>
__global__ void __launch_bounds__(256) splitk_silu_kernel(const float* __restrict__ part, int ks, int units,
                                                          GroupTab gt, uint8_t* __restrict__ act, int out_kb,
                                                          int64_t ntstride) {
  const int ku = blockIdx.x;
  const int gi = ku / units, u = ku % units;
  if (gi >= *gt.n_groups) return;
  const int ntok = gt.ntok[gi], nt0 = gt.nt0[gi];
  const int idx = blockIdx.y * 256 + threadIdx.x;  // row * 32 + token
  const int row = idx >> 5, n = idx & 31;
  if (row >= kTcRows || n >= ntok) return;
  const float* src = part + (int64_t)ku * ks * (2 * kTcRows * 32) + idx;
  float g = 0.f, v = 0.f;
  // four slices' loads in flight, the ragged last round included, added in slice order
  for (int s = 0; s < ks; s += 4) {
    float gs[4], vs[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const bool in = s + i < ks;
      gs[i] = in ? src[(int64_t)(s + i) * (2 * kTcRows * 32)] : 0.f;
      vs[i] = in ? src[(int64_t)(s + i) * (2 * kTcRows * 32) + kTcRows * 32] : 0.f;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (s + i < ks) {
        g += gs[i];
        v += vs[i];
      }
    }
  }
  const int col = u * kTcRows + row;
  uint8_t* dst = act + tc_bact_off((int64_t)nt0 * kNTile + n, col, out_kb, ntstride);
  *reinterpret_cast<uint16_t*>(dst) = f32_to_act<BF16>(silu_f(g) * v);
}

// -------------------------------------------------------------- combine ---
// out[t] = sum_j w[t,j] * y[slot(t,j)] (+ g_t * y_shared[t]), fp32, one
// rounding to the output type.
__device__ __forceinline__ void add4(float4& v, const float4& w) {
  v.x += w.x; v.y += w.y; v.z += w.z; v.w += w.w;
}
// One CTA per (token, 128 columns).  The rows to add are
// the routed slots' split-K slices (weighted by the slot's routing weight)
// and the shared expert's slices (weighted by its gate, or 1); eight warps
// take every eighth row, one float4 column per lane, with four rows' loads
// in flight per warp, and the warps' sums are added in warp order.  Every
// call adds the same rows in the same order, so results are deterministic.
constexpr int kCombineWarps = 8;
constexpr int kCombineCols = 128;
template <bool BF16>
__global__ void __launch_bounds__(kCombineWarps * 32) combine_kernel(
    const float* __restrict__ y, const float* __restrict__ ys, const float* __restrict__ tw,
    const int* __restrict__ tk_slot, const float* __restrict__ sg, int top_k, int hidden, int shared_mode,
    void* __restrict__ out_v, int out_f32, int ks_r, int64_t ystride, int ks_s, int64_t ysstride) {
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y * kCombineCols + lane * 4;
  const int nr = top_k * ks_r;
  const int rows = nr + (shared_mode >= 0 ? ks_s : 0);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (h < hidden) {
    for (int r0 = warp; r0 < rows; r0 += 4 * kCombineWarps) {
      float4 v[4];
      float w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = r0 + i * kCombineWarps;
        w[i] = 0.f;
        v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (r >= rows) continue;
        if (r < nr) {
          const int j = r / ks_r, sl = r - j * ks_r;
          const int slot = tk_slot[(int64_t)t * top_k + j];
          if (slot < 0) continue;
          w[i] = tw[(int64_t)t * top_k + j];
          v[i] = *reinterpret_cast<const float4*>(y + sl * ystride + (int64_t)slot * hidden + h);
        } else {
          const int sl = r - nr;
          w[i] = shared_mode == 1 ? sg[t] : 1.f;
          v[i] = *reinterpret_cast<const float4*>(ys + sl * ysstride + (int64_t)t * hidden + h);
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        acc.x = fmaf(w[i], v[i].x, acc.x);
        acc.y = fmaf(w[i], v[i].y, acc.y);
        acc.z = fmaf(w[i], v[i].z, acc.z);
        acc.w = fmaf(w[i], v[i].w, acc.w);
      }
    }
  }
  __shared__ float4 part[kCombineWarps][32];
  part[warp][lane] = acc;
  __syncthreads();
  if (warp != 0 || h >= hidden) return;
  acc = part[0][lane];
#pragma unroll
  for (int i = 1; i < kCombineWarps; ++i) add4(acc, part[i][lane]);
  if (out_f32) {
    *reinterpret_cast<float4*>(static_cast<float*>(out_v) + (int64_t)t * hidden + h) = acc;
  } else {
    uint2 o;
    o.x = uint32_t(f32_to_act<BF16>(acc.x)) | (uint32_t(f32_to_act<BF16>(acc.y)) << 16);
    o.y = uint32_t(f32_to_act<BF16>(acc.z)) | (uint32_t(f32_to_act<BF16>(acc.w)) << 16);
    *reinterpret_cast<uint2*>(static_cast<uint16_t*>(out_v) + (int64_t)t * hidden + h) = o;
  }
}

// ------------------------------------------------------------ host side ---
// SM count of the current device (cached per device).
int num_sms() {
  static std::atomic<int> cache[kMaxDevices];
  const int dev = cache_device();
  int sms = dev >= 0 ? cache[dev].load(std::memory_order_relaxed) : 0;
  if (sms > 0) return sms;
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, d) != cudaSuccess ||
      sms <= 0)
    sms = 148;
  if (dev >= 0) cache[dev].store(sms, std::memory_order_relaxed);
  return sms;
}

static bool same_format(const blut_mat_desc& a, const blut_mat_desc& b) {
  return a.format == b.format && a.bits == b.bits && a.group == b.group && a.tier == b.tier && a.dtype == b.dtype;
}

// Expected number of experts hit by T tokens choosing k of E uniformly
// (every expert once k >= E, which caller routing allows).
static double expected_active(int T, int k, int E) {
  const double keep = std::max(0.0, 1.0 - (double)k / E);
  double miss = 1.0;
  for (int t = 0; t < T; ++t) miss *= keep;
  return E * (1.0 - miss);
}

// Non-empty routed slots to plan for.  Expert parallelism passes every
// received row with all k slots, most of them empty (experts of other
// ranks); the caller's expected count (blut_moe_args.expected_slots) then
// stands in for T*k in the grouping and split choices.  Buffer sizes still
// allow for all T*k slots.
static int64_t expected_slots(const blut_moe_args& a) {
  const int64_t S = (int64_t)a.num_tokens * a.top_k;
  return a.num_experts > 0 && a.expected_slots > 0 && a.expected_slots < S ? (int64_t)a.expected_slots : S;
}

// Expected routed token groups of gtok tokens: the experts hit plus the
// slots over gtok.  Experts hit: T tokens choosing k of E, or, with the
// caller's slot count, that many slots each landing on one of E experts.
static double expected_groups(const blut_moe_args& a, int gtok) {
  const int64_t S = (int64_t)a.num_tokens * a.top_k, Sx = expected_slots(a);
  const double E = (double)a.num_experts;
  const double active = Sx < S ? E * (1.0 - std::pow(1.0 - 1.0 / E, (double)Sx))
                               : expected_active(a.num_tokens, a.top_k, a.num_experts);
  return active + (double)Sx / gtok;
}

// K slices per tcgen05 pass, every slice keeping at least two column blocks;
// gate/up passes split at most 8 ways (their partial sums go through
// memory), down passes 16.  Routed and shared passes split while the
// (expected) work items are fewer than two per resident CTA (two CTAs per
// SM): the shared expert's side-stream passes finish sooner split, which
// measured 2212 -> 2602 tokens/s at batch 8 and 7322 -> 7489 at batch 32 on
// Qwen1.5-MoE.  The small-batch GEMV sizes its slices by the pieces a thread
// keeps in flight.
void moe_split(const blut_moe_args& a, MoESplit& s) {
  const int sms = num_sms();
  const int64_t T = a.num_tokens, K = a.top_k, E = a.num_experts, S = T * K;
  // Prefill: on the tcgen05 path, with at least 64 tokens per expert on
  // average, tokens go in groups of kWideGroupTok so one decoded weight tile
  // feeds wide MMAs.
  const int64_t Sx = expected_slots(a);
  const bool tc_r = (a.w13.layout & BLUT_LAYOUT_TC) != 0;
  const bool tc_s = a.shared_inter > 0 && (a.s13.layout & BLUT_LAYOUT_TC) != 0;
  s.gtok[0] = tc_r && Sx >= 64 * E ? kWideGroupTok : kGroupTok;
  s.gtok[1] = tc_s && T >= 64 ? kWideGroupTok : kGroupTok;
  s.gemv[0] = tc_r && T <= kGemvMaxTokens;
  s.gemv[1] = tc_s && T <= kGemvMaxTokens;
  const double est_r = expected_groups(a, s.gtok[0]);
  const int64_t gmax_r = std::min(E, S) + (S + s.gtok[0] - 1) / s.gtok[0] + 1;
  const int64_t gmax_s = (T + s.gtok[1] - 1) / s.gtok[1];
  const blut_mat_desc* d[4] = {&a.w13, &a.w2, &a.s13, &a.s2};
  for (int i = 0; i < 4; ++i) {
    s.ks[i] = 1;
    s.bps[i] = 0;
    s.units[i] = 0;
    s.groups[i] = i < 2 ? gmax_r : gmax_s;
    TiledLayout L;
    if ((i >= 2 && a.shared_inter <= 0) || !make_layout(*d[i], L)) continue;
    s.bps[i] = (int)L.nchunks;
    if (!L.tc) continue;
    s.units[i] = (int)((L.ntiles + 1) / 2);
    if (s.gemv[i / 2]) {
      // small-batch GEMV, one CTA per (group, tile, K slice): a slice is
      // the blocks a thread keeps in flight, halved while that leaves fewer
      // than four CTAs per SM
      const double tiles = (i < 2 ? est_r : (double)gmax_s) * L.ntiles;
      int64_t bps = tc_gemv_blocks(*d[i]);
      while (bps > 1 && tiles * ((L.nchunks + bps - 1) / bps) < 4.0 * sms) bps = (bps + 1) / 2;
      s.ks[i] = (int)((L.nchunks + bps - 1) / bps);
      s.bps[i] = (int)bps;
      continue;
    }
    if (s.gtok[i / 2] != kGroupTok) continue;  // wide groups have enough items
    const double est = (i < 2 ? est_r : (double)gmax_s) * s.units[i];
    const int max_ks = (i % 2 == 0) ? 8 : 16;
    int ks = 1;
    // split while the items (for routed passes the expected count) are
    // fewer than two per resident CTA
    while (ks * 2 <= max_ks && L.nchunks / (ks * 2) >= 2 && est * ks < 4.0 * sms) ks *= 2;
    const int bps = (int)((L.nchunks + ks - 1) / ks);
    s.ks[i] = (int)((L.nchunks + bps - 1) / bps);
    s.bps[i] = bps;
  }
}

bool tok1_applies(const blut_moe_args& a, const MoESplit& s) {
  return a.num_tokens == 1 && s.gemv[0] && (a.shared_inter <= 0 || s.gemv[1]) && a.num_experts <= kTok1MaxExperts;
}

// K slices of a single-token GEMV pass: a slice is the 256 columns a
// thread stages (kTok1MaxCols), one or two rounds of its register ring.
static void tok1_slices(const blut_mat_desc& d, int& bps, int& ks) {
  TiledLayout L;
  bps = ks = 0;
  if (!make_layout(d, L)) return;
  bps = std::max(1, kTok1MaxCols / (int)L.kb);
  ks = (int)((L.nchunks + bps - 1) / bps);
}

// Workspace carve-up; returns total bytes, fills pointers when base != null.
size_t moe_workspace(const blut_moe_args& a, uint8_t* base, MoEWs* ws) {
  const int64_t T = a.num_tokens, K = a.top_k, E = a.num_experts, H = a.hidden, I = a.inter;
  const int64_t S = T * K;
  MoESplit sp;
  moe_split(a, sp);
  const int64_t gmax = E + (S + sp.gtok[0] - 1) / sp.gtok[0] + 1;
  const int64_t ntmax = (S + kNTile - 1) / kNTile + gmax;
  const int64_t sgmax = (T + sp.gtok[1] - 1) / sp.gtok[1] + 1;
  const int64_t sntmax = (T + kNTile - 1) / kNTile + 1;
  const bool sh = a.shared_inter > 0;
  size_t off = 0;
  auto take = [&](int64_t bytes) {
    const size_t o = off;
    off = (size_t)align256(off + bytes);
    return o;
  };
  MoEWs w{};
  size_t o_status = take(256);
  size_t o_ids = take(S * 4), o_tw = take(S * 4), o_sg = take(T * 4);
  size_t o_lg = take(T * (E + 1) * 4);
  size_t o_meta = take(64);
  size_t o_g = take(gmax * 4 * 4), o_nt = take(ntmax * 4 * 2), o_sgp = take(sgmax * 4 * 4);
  size_t o_tk = take(S * 4), o_st = take(S * 4);
  size_t o_xf = take(ntmax * (H / kChunk) * kBfragChunkBytes);
  size_t o_af = take(ntmax * (I / kChunk) * kBfragChunkBytes);
  size_t o_y = take(S * H * 4 * sp.ks[1]);
  size_t o_xfs = sh ? take(sntmax * (H / kChunk) * kBfragChunkBytes) : 0;
  size_t o_afs = sh ? take(sntmax * (a.shared_inter / kChunk) * kBfragChunkBytes) : 0;
  size_t o_ys = sh ? take(T * H * 4 * sp.ks[3]) : 0;
  // split-K partial sums of the gate/up passes: [item][gate|up][128 rows][32 tokens] fp32
  const int64_t ku_r = sp.ks[0] > 1 || sp.gemv[0] ? sp.groups[0] * sp.units[0] : 0;
  const int64_t ku_s = sp.ks[2] > 1 || sp.gemv[1] ? sp.groups[2] * sp.units[2] : 0;
  size_t o_part_r = take(ku_r * sp.ks[0] * 2 * kTcRows * 32 * 4);
  size_t o_part_s = take(ku_s * sp.ks[2] * 2 * kTcRows * 32 * 4);
  // single-token path
  const bool t1 = tok1_applies(a, sp);
  int t1_bps[4] = {0, 0, 0, 0}, t1_ks[4] = {0, 0, 0, 0};
  size_t o_t1g = 0, o_t1w = 0, o_t1c = 0, o_t1pr = 0, o_t1ps = 0, o_t1ar = 0, o_t1as = 0, o_t1yr = 0, o_t1ys = 0;
  int t1_ncnt_pair = 0, t1_ncnt = 0;
  if (t1) {
    const blut_mat_desc* d[4] = {&a.w13, &a.w2, &a.s13, &a.s2};
    for (int i = 0; i < (sh ? 4 : 2); ++i) tok1_slices(*d[i], t1_bps[i], t1_ks[i]);
    const int64_t units_r = a.inter / kTcRows, units_s = sh ? a.shared_inter / kTcRows : 0;
    t1_ncnt_pair = (int)(K * units_r + units_s);
    t1_ncnt = t1_ncnt_pair + (int)((H + kTcRows - 1) / kTcRows);
    o_t1g = take((1 + K) * 4);
    o_t1w = take(K * 4);
    o_t1c = take((int64_t)t1_ncnt * 4);
    o_t1pr = take(K * units_r * t1_ks[0] * 2 * kTcRows * 4);
    o_t1ps = sh ? take(units_s * t1_ks[2] * 2 * kTcRows * 4) : 0;
    o_t1ar = take(K * I * 2);
    o_t1as = sh ? take(a.shared_inter * 2) : 0;
    o_t1yr = take((int64_t)t1_ks[1] * K * H * 4);
    o_t1ys = sh ? take((int64_t)t1_ks[3] * H * 4) : 0;
  }
  if (base && ws) {
    w.tok1 = t1;
    if (t1) {
      for (int i = 0; i < 4; ++i) {
        w.t1_ks[i] = t1_ks[i];
        w.t1_bps[i] = t1_bps[i];
      }
      w.t1_groups = reinterpret_cast<int*>(base + o_t1g);
      w.t1_gw = reinterpret_cast<float*>(base + o_t1w);
      w.t1_cnt = reinterpret_cast<int*>(base + o_t1c);
      w.t1_ncnt_pair = t1_ncnt_pair;
      w.t1_ncnt = t1_ncnt;
      w.t1_part_r = reinterpret_cast<float*>(base + o_t1pr);
      w.t1_part_s = sh ? reinterpret_cast<float*>(base + o_t1ps) : nullptr;
      w.t1_act_r = reinterpret_cast<uint16_t*>(base + o_t1ar);
      w.t1_act_s = sh ? reinterpret_cast<uint16_t*>(base + o_t1as) : nullptr;
      w.t1_y_r = reinterpret_cast<float*>(base + o_t1yr);
      w.t1_y_s = sh ? reinterpret_cast<float*>(base + o_t1ys) : nullptr;
    }
    w.split = sp;
    w.y_sstride = S * H;
    w.ys_sstride = T * H;
    w.part_r = reinterpret_cast<float*>(base + o_part_r);
    w.part_s = reinterpret_cast<float*>(base + o_part_s);

    w.status = reinterpret_cast<int*>(base + o_status);
    w.ids = reinterpret_cast<int32_t*>(base + o_ids);
    w.tw = reinterpret_cast<float*>(base + o_tw);
    w.sg = reinterpret_cast<float*>(base + o_sg);
    w.logits = reinterpret_cast<float*>(base + o_lg);
    int* g = reinterpret_cast<int*>(base + o_g);
    int* nt = reinterpret_cast<int*>(base + o_nt);
    int* sg = reinterpret_cast<int*>(base + o_sgp);
    w.pp.status = w.status;
    w.pp.counters = w.status + 16;  // inside the 256-byte status block
    w.pp.meta = reinterpret_cast<int*>(base + o_meta);
    w.pp.g_expert = g;
    w.pp.g_slot0 = g + gmax;
    w.pp.g_ntok = g + 2 * gmax;
    w.pp.g_nt0 = g + 3 * gmax;
    w.pp.nt_slot0 = nt;
    w.pp.nt_cnt = nt + ntmax;
    w.pp.sg_expert = sg;
    w.pp.sg_slot0 = sg + sgmax;
    w.pp.sg_ntok = sg + 2 * sgmax;
    w.pp.sg_nt0 = sg + 3 * sgmax;
    w.pp.tk_slot = reinterpret_cast<int*>(base + o_tk);
    w.pp.slot_tok = reinterpret_cast<int*>(base + o_st);
    w.xf = base + o_xf;
    w.af = base + o_af;
    w.y = reinterpret_cast<float*>(base + o_y);
    w.xfs = sh ? base + o_xfs : nullptr;
    w.afs = sh ? base + o_afs : nullptr;
    w.ys = sh ? reinterpret_cast<float*>(base + o_ys) : nullptr;
    w.ntmax = ntmax;
    w.sntmax = sntmax;
    *ws = w;
  }
  return off;
}

int validate_moe(const blut_moe_args& a) {
  if (a.num_tokens <= 0 || a.hidden <= 0 || a.inter <= 0 || a.num_experts <= 0 || a.top_k <= 0) return BLUT_ERR_INVALID;
  // The router picks k distinct experts, so it needs k <= E.  Caller routing
  // does not: under expert parallelism a rank may own fewer experts than k,
  // the other slots of its rows being empty (-1).
  if (a.num_experts > kMaxExperts || a.top_k > 32 || (!a.topk_ids && a.top_k > a.num_experts))
    return BLUT_ERR_UNSUPPORTED;
  if ((int64_t)a.num_tokens * a.top_k > kMaxSlots) return BLUT_ERR_UNSUPPORTED;
  if (a.hidden % kChunk || a.inter % kChunk) return BLUT_ERR_UNSUPPORTED;
  if (a.dtype != BLUT_F16 && a.dtype != BLUT_BF16) return BLUT_ERR_INVALID;
  if (!a.x || !a.out || !a.w13_tiled || !a.w2_tiled) return BLUT_ERR_INVALID;
  if (!a.topk_ids && !a.router_w) return BLUT_ERR_INVALID;
  if (a.topk_ids && !a.topk_weights) return BLUT_ERR_INVALID;
  if (!same_format(a.w13, a.w2)) return BLUT_ERR_UNSUPPORTED;
  if (a.w13.rows != 2LL * a.inter || a.w13.cols != a.hidden || a.w2.rows != a.hidden || a.w2.cols != a.inter)
    return BLUT_ERR_INVALID;
  if (a.w13.dtype != a.dtype) return BLUT_ERR_UNSUPPORTED;
  // gate/up tiles must be paired in the tiled layout, the down projection not
  if (!(a.w13.layout & BLUT_LAYOUT_PAIRED) || (a.w2.layout & BLUT_LAYOUT_PAIRED)) return BLUT_ERR_INVALID;
  if (a.shared_inter > 0 && (!(a.s13.layout & BLUT_LAYOUT_PAIRED) || (a.s2.layout & BLUT_LAYOUT_PAIRED)))
    return BLUT_ERR_INVALID;
  // a projection pair runs on one matmul path: both tcgen05 or both mma.sync
  if ((a.w13.layout ^ a.w2.layout) & BLUT_LAYOUT_TC) return BLUT_ERR_INVALID;
  if (a.shared_inter > 0 && ((a.s13.layout ^ a.s2.layout) & BLUT_LAYOUT_TC)) return BLUT_ERR_INVALID;
  if (a.w13.format == BLUT_FMT_R8 && !a.lut_table) return BLUT_ERR_INVALID;
  TiledLayout L13, L2;
  if (!make_layout(a.w13, L13) || !make_layout(a.w2, L2)) return BLUT_ERR_UNSUPPORTED;
  if (a.w13_stride < L13.total || a.w2_stride < L2.total) return BLUT_ERR_INVALID;
  if ((a.w13_stride | a.w2_stride) & 255) return BLUT_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(a.w13_tiled) | reinterpret_cast<uintptr_t>(a.w2_tiled) |
       reinterpret_cast<uintptr_t>(a.x) | reinterpret_cast<uintptr_t>(a.out)) & 15)
    return BLUT_ERR_INVALID;
  if (a.shared_inter > 0) {
    if (a.shared_inter % kChunk || !a.s13_tiled || !a.s2_tiled) return BLUT_ERR_INVALID;
    if (a.s13.format != BLUT_FMT_DENSE || a.s2.format != BLUT_FMT_DENSE) return BLUT_ERR_UNSUPPORTED;
    if (a.s13.dtype != a.dtype || a.s2.dtype != a.dtype) return BLUT_ERR_UNSUPPORTED;
    if (a.s13.rows != 2LL * a.shared_inter || a.s13.cols != a.hidden || a.s2.rows != a.hidden ||
        a.s2.cols != a.shared_inter)
      return BLUT_ERR_INVALID;
    if (a.shared_gate_mode == 1 && !a.shared_gate_w && !(a.router_w && !a.topk_ids)) return BLUT_ERR_INVALID;
  }
  return BLUT_OK;
}

// Fills the plane part of MMParams for matrix `d`.
bool mm_planes(const blut_mat_desc& d, bool pair, MMParams& p) {
  TiledLayout L;
  if (!make_layout(d, L)) return false;
  int idx[3];
  const int np = plane_select(d, L, idx);
  int tb = 0;
  for (int q = 0; q < 3; ++q) {
    p.plane_off[q] = q < np ? L.off[idx[q]] : 0;
    p.piece[q] = q < np ? (int)L.piece[idx[q]] : 0;
    tb += p.piece[q];
  }
  p.tile_bytes = tb;
  p.ntiles = (int)L.ntiles;
  p.nchunks = (int)L.nchunks;
  p.units = pair ? p.ntiles / 2 : p.ntiles;
  p.W = 1;
  p.b_ntiles = kMaxNT;
  p.stages = 2;
  p.r8_mask = d.tier == 1 ? 0x3Fu : d.tier == 2 ? 0x0Fu : 0xFFu;
  return true;
}

// Units per work item: as many consumer warps per CTA as keeps at least two
// items per SM for the expected number of token groups.
int choose_units_per_item(double est_groups, int units, int sms) {
  int w = kMaxConsumers;
  while (w > 1 && est_groups * ((units + w - 1) / w) < 2.0 * sms) w /= 2;
  return w;
}

// Error check after a stage.  With BLUT_DEBUG_SYNC set, every stage also
// synchronises the stream, so a failing kernel is named by its own stage.
static bool debug_sync() {
  static const bool on = std::getenv("BLUT_DEBUG_SYNC") != nullptr;
  return on;
}

int stage_done(const char* stage, cudaStream_t s) {
  cudaError_t e = cudaGetLastError();
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (e == cudaSuccess && debug_sync() && cudaStreamIsCapturing(s, &cap) == cudaSuccess &&
      cap == cudaStreamCaptureStatusNone) {
    e = cudaStreamSynchronize(s);
    if (e == cudaSuccess) e = cudaGetLastError();
  }
  if (e != cudaSuccess) {
    std::fprintf(stderr, "libblut: %s: %s\n", stage, cudaGetErrorString(e));
    return BLUT_ERR_LAUNCH;
  }
  return BLUT_OK;
}

// A side stream and its fork / join events per device and host thread, made
// on first use.  They are not made while `stream` is being captured into a
// CUDA graph (the forward then runs on `stream` alone), so a capture that
// wants the concurrency follows one ordinary call on that thread.
struct SideStream {
  cudaStream_t s = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
};
static SideStream* side_stream(cudaStream_t stream) {
  constexpr int kMaxDevices = 64;
  thread_local SideStream per_device[kMaxDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  SideStream& ss = per_device[dev];
  if (ss.s) return &ss;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) return nullptr;
  SideStream n;
  if (cudaStreamCreateWithFlags(&n.s, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&n.fork, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&n.join, cudaEventDisableTiming) != cudaSuccess) {
    if (n.join) cudaEventDestroy(n.join);
    if (n.fork) cudaEventDestroy(n.fork);
    if (n.s) cudaStreamDestroy(n.s);
    cudaGetLastError();
    return nullptr;
  }
  ss = n;
  return &ss;
}

// Single-token layer in three launches (blut_tok1.cuh): route, gate/up with
// the SiLU * up epilogue, down with the weighted combine.
static int moe_forward_tok1(const blut_moe_args& a, const MoEWs& ws, cudaStream_t stream) {
  const bool bf16 = a.dtype == BLUT_BF16;
  const bool sh = a.shared_inter > 0;
  const int K = a.top_k, E = a.num_experts, H = a.hidden;
  const bool route = a.topk_ids == nullptr;
  const bool gate = sh && a.shared_gate_mode == 1;
  const uint16_t* w_main = route ? (const uint16_t*)a.router_w : nullptr;
  const uint16_t* w_gate =
      !gate ? nullptr : a.shared_gate_w ? (const uint16_t*)a.shared_gate_w : (const uint16_t*)a.router_w + (int64_t)E * H;
  const int e_main = route ? E : 0;
  const int R = e_main + (gate ? 1 : 0);
  auto lk = bf16 ? tok1_logits_kernel<true> : tok1_logits_kernel<false>;
  lk<<<std::max(1, (R + 7) / 8), 256, 0, stream>>>((const uint16_t*)a.x, w_main, w_gate, H, e_main, ws.logits, ws.sg,
                                                     ws.t1_cnt, ws.t1_ncnt, ws.status);
  int rc = stage_done("single-token router logits", stream);
  if (rc != BLUT_OK) return rc;

  // the two projections: routed matrices in part 0, the shared expert in part 1
  auto mat = [&](const blut_mat_desc& d, const void* w, int64_t stride, bool pair, int i, Tok1Mat& m) -> bool {
    m = Tok1Mat{};
    if (!tc_planes(d, pair, m.p)) return false;
    m.p.w = (const uint8_t*)w;
    m.p.wstride = stride;
    m.p.r8_table = (const uint16_t*)a.lut_table;
    m.p.status = ws.status;
    m.p.ks = ws.t1_ks[i];
    m.p.bps = ws.t1_bps[i];
    m.n_items = (int64_t)(i < 2 ? K : 1) * m.p.ntiles * m.p.ks;
    return m.p.ks > 0;
  };
  TiledLayout L13, L2, Ls13, Ls2;
  make_layout(a.w13, L13);
  make_layout(a.w2, L2);
  double rb13 = (double)K * L13.total, rb2 = (double)K * L2.total, sb13 = 0, sb2 = 0;
  if (sh) {
    make_layout(a.s13, Ls13);
    make_layout(a.s2, Ls2);
    sb13 = (double)Ls13.total;
    sb2 = (double)Ls2.total;
  }
  Tok1Args g{};
  g.groups = ws.t1_groups;
  g.gw = ws.t1_gw;
  g.sg = gate ? ws.sg : nullptr;
  g.gbound = K;
  g.hidden = H;
  g.logits = route ? ws.logits : nullptr;
  g.ids_in = a.topk_ids;
  g.tw_in = a.topk_weights;
  g.num_experts = E;
  g.renorm = a.renorm;
  g.status = ws.status;
  g.has_shared = sh ? 1 : 0;
  g.out = a.out;
  g.out_f32 = a.out_f32;
  if (!mat(a.w13, a.w13_tiled, a.w13_stride, true, 0, g.m[0])) return BLUT_ERR_UNSUPPORTED;
  g.m[0].xin = (const uint16_t*)a.x;
  g.m[0].part = ws.t1_part_r;
  g.m[0].act = ws.t1_act_r;
  if (sh) {
    if (!mat(a.s13, a.s13_tiled, 0, true, 2, g.m[1])) return BLUT_ERR_UNSUPPORTED;
    g.m[1].xin = (const uint16_t*)a.x;
    g.m[1].part = ws.t1_part_s;
    g.m[1].act = ws.t1_act_s;
    g.m[1].cnt0 = K * g.m[0].p.units;
  }
  g.cnt = ws.t1_cnt;
  cudaEvent_t* ev = a.prof_events ? (cudaEvent_t*)a.prof_events : nullptr;
  if (ev && cudaEventRecord(ev[0], stream) != cudaSuccess) return BLUT_ERR_INVALID;
  if (launch_tok1(a.w13, g, true, rb13, sb13, stream) != cudaSuccess) return BLUT_ERR_LAUNCH;
  if ((rc = stage_done("single-token gate/up", stream)) != BLUT_OK) return rc;
  if (ev && cudaEventRecord(ev[1], stream) != cudaSuccess) return BLUT_ERR_INVALID;

  Tok1Args d = g;
  if (!mat(a.w2, a.w2_tiled, a.w2_stride, false, 1, d.m[0])) return BLUT_ERR_UNSUPPORTED;
  d.m[0].xin = ws.t1_act_r;
  d.m[0].x_ld = a.inter;
  d.m[0].part = ws.t1_y_r;
  if (sh) {
    if (!mat(a.s2, a.s2_tiled, 0, false, 3, d.m[1])) return BLUT_ERR_UNSUPPORTED;
    d.m[1].xin = ws.t1_act_s;
    d.m[1].part = ws.t1_y_s;
  }
  d.cnt = ws.t1_cnt + ws.t1_ncnt_pair;
  d.out = a.out;
  d.out_f32 = a.out_f32;
  if (ev && cudaEventRecord(ev[2], stream) != cudaSuccess) return BLUT_ERR_INVALID;
  if (launch_tok1(a.w2, d, false, rb2, sb2, stream) != cudaSuccess) return BLUT_ERR_LAUNCH;
  if ((rc = stage_done("single-token down", stream)) != BLUT_OK) return rc;
  if (ev && cudaEventRecord(ev[3], stream) != cudaSuccess) return BLUT_ERR_INVALID;
  return BLUT_OK;
}

int moe_forward(const blut_moe_args& a, void* workspace, size_t ws_bytes, cudaStream_t stream) {
  int rc = validate_moe(a);
  if (rc != BLUT_OK) return rc;
  if (!workspace) return BLUT_ERR_INVALID;
  const size_t need = moe_workspace(a, nullptr, nullptr);
  if (ws_bytes < need) return BLUT_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) & 255) return BLUT_ERR_INVALID;
  MoEWs ws;
  moe_workspace(a, static_cast<uint8_t*>(workspace), &ws);
  if (ws.tok1) return moe_forward_tok1(a, ws, stream);
  const bool bf16 = a.dtype == BLUT_BF16;
  const bool sh = a.shared_inter > 0;
  const int T = a.num_tokens, K = a.top_k, E = a.num_experts, H = a.hidden;
  const int sms = num_sms();
  const double est_groups = expected_groups(a, ws.split.gtok[0]);
  const double est_sgroups = (T + ws.split.gtok[1] - 1) / ws.split.gtok[1];
  const int b_ntiles = (std::min(T, kGroupTok) + kNTile - 1) / kNTile;

  // 1. routing (or the caller's routing) and the shared-expert gate
  const bool route = a.topk_ids == nullptr;
  const bool gate = sh && a.shared_gate_mode == 1;
  const float* tw = route ? ws.tw : a.topk_weights;
  if (route || gate) {
    // logits of the experts (when routing) and of the shared-expert gate row
    const uint16_t* w_main = route ? (const uint16_t*)a.router_w : nullptr;
    const uint16_t* w_gate =
        !gate ? nullptr : a.shared_gate_w ? (const uint16_t*)a.shared_gate_w : (const uint16_t*)a.router_w + (int64_t)E * H;
    const int e_main = route ? E : 0;
    const int R = e_main + (gate ? 1 : 0);
    const unsigned grid = (unsigned)(((int64_t)R * T + 7) / 8);
    if (bf16)
      router_logits_kernel<true><<<grid, 256, 0, stream>>>((const uint16_t*)a.x, w_main, w_gate, T, H, e_main,
                                                           ws.logits);
    else
      router_logits_kernel<false><<<grid, 256, 0, stream>>>((const uint16_t*)a.x, w_main, w_gate, T, H, e_main,
                                                            ws.logits);
    if ((rc = stage_done("router logits", stream)) != BLUT_OK) return rc;
  }
  // 2. top-k (when routing) + plan.  Long prompts take the top-k in a
  // separate launch, a warp per token over the whole GPU; the plan kernel is
  // one CTA.
  const bool wide_topk = (route || gate) && T > kPlanTopkTokens;
  if (wide_topk) {
    topk_kernel<<<(T + 7) / 8, 256, 0, stream>>>(ws.logits, T, route ? E : 0, route ? K : 0, a.renorm, gate ? 1 : 0,
                                                 ws.ids, ws.tw, ws.sg);
    if ((rc = stage_done("top-k", stream)) != BLUT_OK) return rc;
  }
  plan_kernel<<<1, 1024, 0, stream>>>(wide_topk && route ? ws.ids : a.topk_ids,
                                      (route || gate) && !wide_topk ? ws.logits : nullptr, route ? E : 0,
                                      (route ? E : 0) + (gate ? 1 : 0), T, K, E, a.renorm, gate ? 1 : 0,
                                      sh ? 1 : 0, ws.split.gtok[0], ws.split.gtok[1], ws.pp, ws.ids, ws.tw, ws.sg);
  if ((rc = stage_done("plan", stream)) != BLUT_OK) return rc;
  // 3. activations of x in the operand order of each matmul path
  const bool tc = (a.w13.layout & BLUT_LAYOUT_TC) != 0;
  const bool stc = sh && (a.s13.layout & BLUT_LAYOUT_TC) != 0;
  {
    dim3 grid((unsigned)std::max<int64_t>(ws.ntmax, sh ? ws.sntmax : 0), (unsigned)(H / kChunk), sh ? 2 : 1);
    gather_bfrag_kernel<<<grid, 32, 0, stream>>>((const uint16_t*)a.x, H, ws.pp, ws.xf, ws.xfs,
                                                 (tc ? 1 : 0) | (stc ? 2 : 0), tc_block_cols(a.w13.format, a.w13.group),
                                                 sh ? tc_block_cols(a.s13.format, a.s13.group) : 0, ws.ntmax,
                                                 ws.sntmax);
  }
  if ((rc = stage_done("gather", stream)) != BLUT_OK) return rc;

  // One projection of all groups: gate/up (pair) writes the down projection's
  // activations, down writes fp32 rows.
  const GroupTab routed{ws.pp.meta + 0, ws.pp.g_expert, ws.pp.g_slot0, ws.pp.g_ntok, ws.pp.g_nt0};
  const GroupTab shared{ws.pp.meta + 2, ws.pp.sg_expert, ws.pp.sg_slot0, ws.pp.sg_ntok, ws.pp.sg_nt0};
  cudaStream_t cur = stream;  // stream of the pass being launched
  auto pass = [&](const blut_mat_desc& d, const void* w, int64_t stride, const GroupTab& gt, double est,
                  const uint8_t* bin, uint8_t* act, int out_k, float* y, int counter, float* part,
                  int64_t y_sstride, const blut_mat_desc* next) -> int {
    const bool pair = act != nullptr;
    if (d.layout & BLUT_LAYOUT_TC) {
      TcParams t{};
      if (!tc_planes(d, pair, t)) return BLUT_ERR_UNSUPPORTED;
      t.w = (const uint8_t*)w;
      t.wstride = stride;
      t.gt = gt;
      t.bin = bin;
      t.ntstride = counter < 2 ? ws.ntmax : ws.sntmax;
      t.act_out = act;
      t.out_kb = next ? tc_block_cols(next->format, next->group) : 0;
      t.y_out = y;
      t.y_ld = H;
      t.counter = ws.pp.counters + counter;
      t.status = ws.status;
      t.r8_table = (const uint16_t*)a.lut_table;
      t.ks = ws.split.ks[counter];
      t.bps = ws.split.bps[counter];
      t.part = part;
      t.y_sstride = y_sstride;
      const bool gemv = ws.split.gemv[counter / 2];
      // the GEMV grid covers every group the plan can form: an expert with c
      // tokens forms ceil(c / gtok) groups, so the A active experts of S
      // slots form at most A + (S - A) / gtok <= min(E, S) + S / gtok
      const int64_t slots = (int64_t)a.num_tokens * a.top_k;
      t.gemv_groups = counter < 2 ? std::min<int64_t>(a.num_experts, slots) + slots / ws.split.gtok[0]
                                  : ws.split.groups[counter];
      if (launch_tc_mm(d, t, gemv ? 1 : ws.split.gtok[counter / 2], sms, cur) != cudaSuccess)
        return BLUT_ERR_LAUNCH;
      if (pair && (t.ks > 1 || gemv)) {
        // sum the gate/up slices in order, SiLU(gate) * up into the down projection's activations
        const dim3 grid((unsigned)(ws.split.groups[counter] * t.units), (unsigned)(kTcRows * 32 / 256));
        if (a.dtype == BLUT_BF16)
          splitk_silu_kernel<true><<<grid, 256, 0, cur>>>(part, t.ks, t.units, gt, act, t.out_kb, t.ntstride);
        else
          splitk_silu_kernel<false><<<grid, 256, 0, cur>>>(part, t.ks, t.units, gt, act, t.out_kb, t.ntstride);
      }
      return cudaGetLastError() == cudaSuccess ? BLUT_OK : BLUT_ERR_LAUNCH;
    }
    MMParams m{};
    if (!mm_planes(d, pair, m)) return BLUT_ERR_UNSUPPORTED;
    m.status = ws.status;
    m.r8_table = (const uint16_t*)a.lut_table;
    m.gt = gt;
    m.w = (const uint8_t*)w;
    m.wstride = stride;
    m.bin = bin;
    m.act_out = act;
    m.out_nchunks = out_k / kChunk;
    m.y_out = y;
    m.y_ld = H;
    m.W = choose_units_per_item(est, m.units, sms);
    m.b_ntiles = b_ntiles;
    return launch_lut_mm(d, pair, m, sms, cur) == cudaSuccess ? BLUT_OK : BLUT_ERR_LAUNCH;
  };
  cudaEvent_t* ev = a.prof_events ? (cudaEvent_t*)a.prof_events : nullptr;

  // 4. The shared expert depends only on the gathered activations, so its
  // gate/up and down passes run on a side stream beside the routed passes
  // (when one is available, see side_stream); the combine waits for both.
  SideStream* side = sh ? side_stream(stream) : nullptr;
  // Once the side stream is forked, every return joins it back into `stream`
  // (recording the join event first if the shared passes stopped early), so
  // an error never leaves a capture with an unjoined fork or side-stream
  // kernels unordered with the caller's next use of the workspace.
  struct JoinGuard {
    SideStream* side = nullptr;
    cudaStream_t stream = nullptr;
    bool recorded = false;
    ~JoinGuard() {
      if (!side) return;
      if (!recorded) cudaEventRecord(side->join, side->s);
      cudaStreamWaitEvent(stream, side->join, 0);
    }
  } join_guard;
  auto shared_passes = [&]() -> int {
    int r;
    if ((r = pass(a.s13, a.s13_tiled, 0, shared, est_sgroups, ws.xfs, ws.afs, a.shared_inter, nullptr, 2,
                  ws.part_s, 0, &a.s2)) != BLUT_OK)
      return r;
    if ((r = stage_done("shared gate/up", cur)) != BLUT_OK) return r;
    if ((r = pass(a.s2, a.s2_tiled, 0, shared, est_sgroups, ws.afs, nullptr, 0, ws.ys, 3, nullptr,
                  ws.ys_sstride, nullptr)) != BLUT_OK)
      return r;
    return stage_done("shared down", cur);
  };
  if (side) {
    if (cudaEventRecord(side->fork, stream) != cudaSuccess) return BLUT_ERR_CUDA;
    if (cudaStreamWaitEvent(side->s, side->fork, 0) != cudaSuccess) return BLUT_ERR_CUDA;
    join_guard.side = side;
    join_guard.stream = stream;
    cur = side->s;
    if ((rc = shared_passes()) != BLUT_OK) return rc;
    if (cudaEventRecord(side->join, side->s) != cudaSuccess) return BLUT_ERR_CUDA;
    join_guard.recorded = true;
    cur = stream;
  }
  // 5. routed gate/up + SiLU*up, then down
  if (ev && cudaEventRecord(ev[0], stream) != cudaSuccess) return BLUT_ERR_INVALID;
  if ((rc = pass(a.w13, a.w13_tiled, a.w13_stride, routed, est_groups, ws.xf, ws.af, a.inter, nullptr, 0,
                 ws.part_r, 0, &a.w2)) != BLUT_OK)
    return rc;
  if ((rc = stage_done("routed gate/up", stream)) != BLUT_OK) return rc;
  if (ev && cudaEventRecord(ev[1], stream) != cudaSuccess) return BLUT_ERR_INVALID;
  if (ev && cudaEventRecord(ev[2], stream) != cudaSuccess) return BLUT_ERR_INVALID;
  if ((rc = pass(a.w2, a.w2_tiled, a.w2_stride, routed, est_groups, ws.af, nullptr, 0, ws.y, 1, nullptr,
                 ws.y_sstride, nullptr)) != BLUT_OK)
    return rc;
  if ((rc = stage_done("routed down", stream)) != BLUT_OK) return rc;
  if (ev && cudaEventRecord(ev[3], stream) != cudaSuccess) return BLUT_ERR_INVALID;
  if (side) {
    join_guard.side = nullptr;  // joined here, with the error checked
    if (cudaStreamWaitEvent(stream, side->join, 0) != cudaSuccess) return BLUT_ERR_CUDA;
  } else if (sh) {
    if ((rc = shared_passes()) != BLUT_OK) return rc;
  }

  // 6. combine
  const int smode = sh ? a.shared_gate_mode : -1;
  const dim3 cgrid(T, (H + kCombineCols - 1) / kCombineCols);
  auto kern = bf16 ? combine_kernel<true> : combine_kernel<false>;
  kern<<<cgrid, kCombineWarps * 32, 0, stream>>>(ws.y, ws.ys, tw, ws.pp.tk_slot, ws.sg, K, H, smode, a.out, a.out_f32,
                                                 ws.split.ks[1], ws.y_sstride, ws.split.ks[3], ws.ys_sstride);
  return stage_done("combine", stream);
}

int moe_launch_count(const blut_moe_args& a) {
  const bool sh = a.shared_inter > 0;
  int n = 0;
  {
    MoESplit sp;
    moe_split(a, sp);
    if (tok1_applies(a, sp)) return 3;  // route, gate/up, down
  }
  if (!a.topk_ids || (sh && a.shared_gate_mode == 1)) {
    ++n;                                                   // router / gate logits
    if (a.num_tokens > kPlanTopkTokens) ++n;               // separate top-k
  }
  n += 2;                                                  // top-k + plan, gather
  n += 2;                                                  // routed gate/up, down
  if (sh) n += 2;                                          // shared gate/up, down
  n += 1;                                                  // combine
  MoESplit sp;
  moe_split(a, sp);
  n += (sp.ks[0] > 1 || sp.gemv[0]) + (sh && (sp.ks[2] > 1 || sp.gemv[1]));  // gate/up slice sums
  return n;
}

int router(const void* x, const void* w, int T, int H, int E, int K, int renorm, int has_sg, int dtype,
           int32_t* ids, float* tw, float* sg, float* logits, cudaStream_t stream) {
  if (!x || !w || !ids || !tw || !logits || T <= 0 || H <= 0 || E <= 0 || K <= 0 || K > 32 || K > E)
    return BLUT_ERR_INVALID;
  if (H % 8 || (has_sg && !sg) || (dtype != BLUT_BF16 && dtype != BLUT_F16)) return BLUT_ERR_INVALID;
  if (E > kMaxExperts) return BLUT_ERR_UNSUPPORTED;
  const uint16_t* wm = (const uint16_t*)w;
  const uint16_t* wg = has_sg ? wm + (int64_t)E * H : nullptr;
  const unsigned grid = (unsigned)(((int64_t)(E + (has_sg ? 1 : 0)) * T + 7) / 8);
  if (dtype == BLUT_BF16)
    router_logits_kernel<true><<<grid, 256, 0, stream>>>((const uint16_t*)x, wm, wg, T, H, E, logits);
  else
    router_logits_kernel<false><<<grid, 256, 0, stream>>>((const uint16_t*)x, wm, wg, T, H, E, logits);
  topk_kernel<<<(T + 7) / 8, 256, 0, stream>>>(logits, T, E, K, renorm, has_sg, ids, tw, sg);
  return cudaGetLastError() == cudaSuccess ? BLUT_OK : BLUT_ERR_LAUNCH;
}

}  // namespace blut
