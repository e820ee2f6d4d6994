// Single-matrix LUT matmul y = W x, x [M][K] and y [M][N], on the matmul
// path of the matrix's tiled layout (tcgen05 for BLUT_LAYOUT_TC, mma.sync
// otherwise).  One token on the TC layout is one launch of the single-token
// GEMV (blut_tok1.cuh), after a memset of its counters.  Otherwise three
// launches: a gather kernel puts x into the path's operand order and writes
// the token groups (one "expert", groups of 32 tokens, or 128 on the tcgen05
// path from 128 tokens on), the matmul writes fp32 rows (in K slices when
// the tcgen05 path has too few work items to fill the GPU), and a reduce
// kernel sums the slices in slice order into y.  This is the single-matrix
// LUT GEMV/GEMM of the reference (vllm_lut/cuda_lut_gemv.py:153-169,
// fused_kernel.py:13-46) for every format of this library and every token
// count.
#include <algorithm>

#include "blut_internal.h"
#include "blut_mm.cuh"
#include "blut_tc.cuh"
#include "blut_tok1.cuh"

namespace blut {

namespace {

constexpr int64_t kMatmulMaxTokens = 1 << 20;

struct MatmulPlan {
  bool tc;
  bool gemv;        // tcgen05 layout, at most kGemvMaxTokens tokens: small-batch GEMV
  int gtok;         // tokens per group
  int64_t groups;   // token groups
  int64_t nt8;      // n-tiles of 8 tokens
  int ks, bps;      // K slices and column blocks per slice
  int units;        // tcgen05 units (pairs of 128-row tiles)
};

struct MatmulWs {
  int* status;      // status word (the first word of the workspace)
  int* counter;     // tcgen05 work-item counter
  int* n_groups;
  int *expert, *slot0, *ntok, *nt0;
  uint8_t* bin;     // x in the operand order of the path
  float* ys;        // ks slices of fp32 y
};

bool matmul_plan(const blut_mat_desc& d, int64_t m, MatmulPlan& p, TiledLayout& L) {
  if (!make_layout(d, L)) return false;
  p.tc = L.tc != 0;
  p.gtok = p.tc && m >= kWideGroupTok ? kWideGroupTok : kGroupTok;
  p.groups = (m + p.gtok - 1) / p.gtok;
  p.nt8 = (m + kNTile - 1) / kNTile;
  p.ks = 1;
  p.bps = (int)L.nchunks;
  p.units = 0;
  p.gemv = p.tc && m <= kGemvMaxTokens;
  if (p.gemv) {  // the single-token GEMV: K slices of the 256 columns a thread stages
    p.bps = std::max(1, kTok1MaxCols / (int)L.kb);
    p.ks = (int)((L.nchunks + p.bps - 1) / p.bps);
    p.units = (int)((L.ntiles + 1) / 2);
  } else if (p.tc) {
    p.units = (int)((L.ntiles + 1) / 2);
    if (p.gtok == kGroupTok) {  // split K while the items are fewer than four per SM
      const int sms = num_sms();
      int ks = 1;
      while (ks * 2 <= 16 && L.nchunks / (ks * 2) >= 2 && (double)p.groups * p.units * ks < 4.0 * sms) ks *= 2;
      p.bps = (int)((L.nchunks + ks - 1) / ks);
      p.ks = (int)((L.nchunks + p.bps - 1) / p.bps);
    }
  }
  return true;
}

size_t matmul_carve(const blut_mat_desc& d, int64_t m, const MatmulPlan& p, uint8_t* base, MatmulWs* w) {
  size_t off = 0;
  auto take = [&](int64_t bytes) {
    const size_t o = off;
    off = (size_t)align256(off + bytes);
    return o;
  };
  // status word; the single-token GEMV's completion counters (one per
  // 128-row tile) follow it, so one memset clears both
  const size_t o_status = take(256 + (p.gemv ? (d.rows + kTcRows - 1) / kTcRows * 4 : 0));
  const size_t o_groups = take(4 * p.groups * 4);
  const size_t o_bin = take(p.nt8 * kNTile * d.cols * 2);
  const size_t o_ys = take((int64_t)p.ks * m * d.rows * 4);
  if (base && w) {
    w->status = reinterpret_cast<int*>(base + o_status);
    w->counter = w->status + 4;
    w->n_groups = w->status + 8;
    int* g = reinterpret_cast<int*>(base + o_groups);
    w->expert = g;
    w->slot0 = g + p.groups;
    w->ntok = g + 2 * p.groups;
    w->nt0 = g + 3 * p.groups;
    w->bin = base + o_bin;
    w->ys = reinterpret_cast<float*>(base + o_ys);
  }
  return off;
}

int validate_matmul(const blut_mat_desc& d, int64_t m) {
  if (m <= 0 || m > kMatmulMaxTokens) return BLUT_ERR_UNSUPPORTED;
  if (d.layout & BLUT_LAYOUT_PAIRED) return BLUT_ERR_INVALID;  // a single projection
  if (d.cols % kChunk) return BLUT_ERR_UNSUPPORTED;
  if (d.dtype != BLUT_F16 && d.dtype != BLUT_BF16) return BLUT_ERR_INVALID;
  TiledLayout L;
  if (!make_layout(d, L)) return BLUT_ERR_UNSUPPORTED;
  return BLUT_OK;
}

}  // namespace

struct MatmulGroups {
  int64_t groups;   // token groups: group g holds tokens g * gtok .. (one expert)
  int gtok;
  int *n_groups, *expert, *slot0, *ntok, *nt0;
  int *status, *counter;
};

// x of one (n-tile of 8 tokens, 128-column chunk), 32 threads: the tcgen05
// operand order (tc_bact_off) or mma.sync B fragments.  The CTAs of chunk 0
// also write the token groups, and the first clears the status word (it
// reports this call) and the work counter.
__global__ void __launch_bounds__(32) matmul_gather_kernel(const uint16_t* __restrict__ x, int64_t m, int k,
                                                           uint8_t* __restrict__ bin, int tc, int kb,
                                                           int64_t ntstride, MatmulGroups gp) {
  const int64_t nt = blockIdx.x;
  const int c = blockIdx.y;
  const int lane = threadIdx.x;
  if (c == 0) {
    for (int64_t g = nt * 32 + lane; g < gp.groups && g < (nt + 1) * 32; g += 32) {
      gp.expert[g] = 0;
      gp.slot0[g] = (int)(g * gp.gtok);
      gp.ntok[g] = (int)std::min<int64_t>(gp.gtok, m - g * gp.gtok);
      gp.nt0[g] = (int)(g * gp.gtok / kNTile);
    }
    if (nt == 0 && lane == 0) {
      *gp.n_groups = (int)gp.groups;
      *gp.status = 0;
      *gp.counter = 0;
    }
  }
  const int64_t t0 = nt * kNTile;
  const int cnt = (int)std::min<int64_t>(kNTile, m - t0);
  if (tc) {
    const int tok = lane & 7;
    const uint16_t* row = tok < cnt ? x + (t0 + tok) * k + c * kChunk : nullptr;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int kg = (lane >> 3) + 4 * i;
      const uint4 v = row ? *reinterpret_cast<const uint4*>(row + kg * 8) : make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(bin + tc_bact_off(t0 + tok, c * kChunk + kg * 8, kb, ntstride)) = v;
    }
    return;
  }
  const int g = lane >> 2, tq = lane & 3;
  uint32_t wv[16];
  if (g < cnt) {
    const uint32_t* row = reinterpret_cast<const uint32_t*>(x + (t0 + g) * k + c * kChunk);
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      wv[2 * s] = row[(16 * s + 2 * tq) >> 1];
      wv[2 * s + 1] = row[(16 * s + 2 * tq + 8) >> 1];
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) wv[i] = 0;
  }
  uint4* d4 = reinterpret_cast<uint4*>(bin + (nt * (k / kChunk) + c) * kBfragChunkBytes + lane * 64);
#pragma unroll
  for (int i = 0; i < 4; ++i) d4[i] = make_uint4(wv[4 * i], wv[4 * i + 1], wv[4 * i + 2], wv[4 * i + 3]);
}

// y = sum of the ks fp32 slices in slice order, four values per thread;
// four slices' loads are in flight at a time, the ragged last round included.
template <bool BF16>
__global__ void __launch_bounds__(256) matmul_reduce_kernel(const float* __restrict__ ys, int ks, int64_t sstride,
                                                            int64_t n4, void* __restrict__ y, int y_f32) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const float* p = ys + 4 * i;
    float4 v = *reinterpret_cast<const float4*>(p);
    for (int s = 1; s < ks; s += 4) {
      float4 u[4];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        u[q] = s + q < ks ? *reinterpret_cast<const float4*>(p + (s + q) * sstride) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (s + q < ks) {
          v.x += u[q].x; v.y += u[q].y; v.z += u[q].z; v.w += u[q].w;
        }
      }
    }
    if (y_f32) {
      reinterpret_cast<float4*>(y)[i] = v;
    } else {
      uint2 o;
      o.x = uint32_t(f32_to_act<BF16>(v.x)) | (uint32_t(f32_to_act<BF16>(v.y)) << 16);
      o.y = uint32_t(f32_to_act<BF16>(v.z)) | (uint32_t(f32_to_act<BF16>(v.w)) << 16);
      reinterpret_cast<uint2*>(y)[i] = o;
    }
  }
}

size_t matmul_workspace(const blut_mat_desc& d, int64_t m) {
  if (validate_matmul(d, m) != BLUT_OK) return 0;
  MatmulPlan p;
  TiledLayout L;
  if (!matmul_plan(d, m, p, L)) return 0;
  return matmul_carve(d, m, p, nullptr, nullptr);
}

int matmul_launch_count(const blut_mat_desc& d, int64_t m) {
  const int rc = validate_matmul(d, m);
  if (rc != BLUT_OK) return rc;
  MatmulPlan p;
  TiledLayout L;
  if (!matmul_plan(d, m, p, L)) return BLUT_ERR_UNSUPPORTED;
  return p.gemv ? 1 : 3;  // single-token GEMV (after a memset); else gather (+ token groups), matmul, reduce
}

int matmul(const blut_mat_desc& d, const void* w, const void* lut_table, const void* x, int64_t m, void* y,
           int y_f32, void* workspace, size_t ws_bytes, cudaStream_t stream) {
  int rc = validate_matmul(d, m);
  if (rc != BLUT_OK) return rc;
  if (!w || !x || !y || !workspace) return BLUT_ERR_INVALID;
  if (d.format == BLUT_FMT_R8 && !lut_table) return BLUT_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15)
    return BLUT_ERR_INVALID;
  if (reinterpret_cast<uintptr_t>(workspace) & 255) return BLUT_ERR_INVALID;
  MatmulPlan p;
  TiledLayout L;
  if (!matmul_plan(d, m, p, L)) return BLUT_ERR_UNSUPPORTED;
  if (ws_bytes < matmul_carve(d, m, p, nullptr, nullptr)) return BLUT_ERR_WORKSPACE;
  MatmulWs ws;
  matmul_carve(d, m, p, static_cast<uint8_t*>(workspace), &ws);
  const int sms = num_sms();
  const int64_t N = d.rows, K = d.cols;

  if (p.gemv) {
    // one token: the single-token GEMV (blut_tok1.cuh) as one matrix; the
    // last CTA to finish a 128-row tile sums its K slices into y
    int* cnt = ws.status + 64;  // after the 256-byte status block
    if (cudaMemsetAsync(ws.status, 0, 256 + (N + kTcRows - 1) / kTcRows * 4, stream) != cudaSuccess)
      return BLUT_ERR_CUDA;
    Tok1Args a{};
    if (!tc_planes(d, false, a.m[0].p)) return BLUT_ERR_UNSUPPORTED;
    a.m[0].p.w = static_cast<const uint8_t*>(w);
    a.m[0].p.wstride = 0;
    a.m[0].p.r8_table = static_cast<const uint16_t*>(lut_table);
    a.m[0].p.status = ws.status;
    a.m[0].p.ks = p.ks;
    a.m[0].p.bps = p.bps;
    a.m[0].n_items = (int64_t)a.m[0].p.ntiles * p.ks;
    a.m[0].xin = static_cast<const uint16_t*>(x);
    a.m[0].part = ws.ys;
    a.cnt = cnt;
    a.gbound = 1;
    a.out = y;
    a.out_f32 = y_f32;
    a.hidden = (int)N;
    a.status = ws.status;
    if (launch_tok1(d, a, false, (double)L.total, 0.0, stream) != cudaSuccess) return BLUT_ERR_LAUNCH;
    return stage_done("matmul (single token)", stream);
  }

  // n-tile nt of chunk 0 writes groups 32 nt .. 32 nt + 31: there are at
  // most nt8 / 4 + 1 groups (32-token groups, 4 n-tiles each), so nt8
  // n-tiles cover them
  const MatmulGroups gp{p.groups, p.gtok, ws.n_groups, ws.expert, ws.slot0, ws.ntok, ws.nt0, ws.status,
                        ws.counter};
  matmul_gather_kernel<<<dim3((unsigned)p.nt8, (unsigned)(K / kChunk)), 32, 0, stream>>>(
      static_cast<const uint16_t*>(x), m, (int)K, ws.bin, p.tc ? 1 : 0, p.tc ? L.kb : 0, p.nt8, gp);
  if ((rc = stage_done("matmul gather", stream)) != BLUT_OK) return rc;

  const GroupTab gt{ws.n_groups, ws.expert, ws.slot0, ws.ntok, ws.nt0};
  if (p.tc) {
    TcParams t{};
    if (!tc_planes(d, false, t)) return BLUT_ERR_UNSUPPORTED;
    t.w = static_cast<const uint8_t*>(w);
    t.wstride = 0;
    t.gt = gt;
    t.bin = ws.bin;
    t.ntstride = p.nt8;
    t.y_out = ws.ys;
    t.y_ld = (int)N;
    t.y_sstride = m * N;
    t.counter = ws.counter;
    t.status = ws.status;
    t.r8_table = static_cast<const uint16_t*>(lut_table);
    t.ks = p.ks;
    t.bps = p.bps;
    t.gemv_groups = p.groups;
    if (launch_tc_mm(d, t, p.gemv ? 1 : p.gtok, sms, stream) != cudaSuccess) return BLUT_ERR_LAUNCH;
  } else {
    MMParams mp{};
    if (!mm_planes(d, false, mp)) return BLUT_ERR_UNSUPPORTED;
    mp.status = ws.status;
    mp.r8_table = static_cast<const uint16_t*>(lut_table);
    mp.gt = gt;
    mp.w = static_cast<const uint8_t*>(w);
    mp.wstride = 0;
    mp.bin = ws.bin;
    mp.y_out = ws.ys;
    mp.y_ld = (int)N;
    mp.W = choose_units_per_item((double)p.groups, mp.units, sms);
    mp.b_ntiles = (int)((std::min<int64_t>(m, kGroupTok) + kNTile - 1) / kNTile);
    if (launch_lut_mm(d, false, mp, sms, stream) != cudaSuccess) return BLUT_ERR_LAUNCH;
  }
  if ((rc = stage_done("matmul", stream)) != BLUT_OK) return rc;

  const int64_t n4 = m * N / 4;
  const unsigned grid = (unsigned)std::min<int64_t>((n4 + 255) / 256, 8 * sms);
  if (d.dtype == BLUT_BF16)
    matmul_reduce_kernel<true><<<grid, 256, 0, stream>>>(ws.ys, p.ks, m * N, n4, y, y_f32);
  else
    matmul_reduce_kernel<false><<<grid, 256, 0, stream>>>(ws.ys, p.ks, m * N, n4, y, y_f32);
  return stage_done("matmul reduce", stream);
}

}  // namespace blut
