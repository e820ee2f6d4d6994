// Common definitions of libblut: PTX wrappers for sm_100a and the tiled
// (MMA-fragment-ordered) device layout of LUT weight matrices.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/blut.h"

namespace blut {

// Device-side status bits (stored in the first word of a workspace).
constexpr int kDevTimeout = 1;

constexpr int kTileRows = 16;   // rows per MMA tile (m16)
constexpr int kChunk = 128;     // K columns per chunk (8 slabs of k16)
constexpr int kNTile = 8;       // tokens per MMA n-tile (n8)
constexpr int kMaxNT = 4;       // n-tiles per work group (32 tokens)
constexpr int kGroupTok = kMaxNT * kNTile;
constexpr int kBfragChunkBytes = 32 * 64;  // one (n-tile, chunk) of B fragments

// ------------------------------------------------------------------------
// Tiled layout of one matrix.  The matrix is cut into 16-row tiles and
// 128-column chunks; each "plane" (a code plane or a table plane) stores its
// (tile, chunk) pieces chunk-major (all tiles of chunk 0, then of chunk 1,
// ...), so that one bulk copy per plane fetches one chunk of W consecutive
// tiles.  With BLUT_LAYOUT_PAIRED, gate tile t sits at physical tile 2t and
// up tile t at 2t + 1, so a gate/up pair is one contiguous run.  Inside a
// piece, data sits in the
// order the mma.m16n8k16 A fragment consumes it (lane = 4 * (row & 7) +
// ((k & 7) >> 1)), see the *_pos helpers below.
// ------------------------------------------------------------------------
enum PlaneKind : int {
  kPlaneCodes4 = 1,   // 4-bit codes: 1024 B per piece
  kPlaneCodes2 = 2,   // 2-bit codes:  512 B
  kPlaneCodes1 = 3,   // 1-bit codes (bit 2 of a 3-bit code): 256 B
  kPlaneCodes8 = 4,   // 8-bit codes (FMT_R8): 2048 B
  kPlaneTables = 5,   // per (row, block) tables as hi/lo byte planes
  kPlaneScales = 6,   // FMT_R8 absmax per (row, chunk): 32 B
  kPlaneDense = 7,    // fp16/bf16 weights: 4096 B
  kPlaneCombined = 8  // NESTED (TC layout): 16-entry tables fp16(coarse[c] + refine[c][r])
};

struct TiledLayout {
  int nplanes;
  int kind[4];
  int entries[4];       // table planes: entries per table (2^bits)
  int64_t piece[4];     // bytes per (tile, chunk) piece
  int64_t off[4];       // plane byte offset inside the matrix buffer
  int64_t total;        // matrix bytes (256-aligned)
  int64_t ntiles, nchunks;
  // BLUT_LAYOUT_TC: tiles of kTcRows rows, "chunks" are blocks of kb columns,
  // and bpr[p] is the bytes one row holds per block in plane p.
  int tc, kb;
  int bpr[4];
};

__host__ __device__ inline int64_t align256(int64_t x) { return (x + 255) & ~int64_t(255); }

// Host: the current device, for caches of per-device launch set-up (function
// attributes and occupancy are per device).  Devices at or beyond
// kMaxDevices are not cached (-1).
constexpr int kMaxDevices = 64;
__host__ inline int cache_device() {
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= kMaxDevices) return -1;
  return d;
}

// ------------------------------------------------------------------------
// TC layout (BLUT_LAYOUT_TC): 128-row tiles for the tcgen05 matmuls, where
// one thread decodes one weight row into tensor memory.  A (tile, block)
// piece of a plane holds bpr bytes per row, cut into units of
// u = min(16, bpr) bytes and stored unit-major: byte o of row r sits at
// (o / u) * 128 * u + r * u + o % u.  A warp's 32 rows reading one unit
// touch one contiguous 32 * u byte range (no bank conflicts), and for dense
// weights the piece is exactly the canonical no-swizzle K-major operand
// layout of tcgen05.mma (8-row x 16-byte core matrices).  Per plane and row,
// the block's bytes are:
//   codes4  the row's canonical 4-bit code bytes of the block (LSB first)
//   codes2  32-bit words of 16 two-bit codes: bits 2i..2i+1 of byte j of
//           word w hold weight 16w + 4i + j (so that masking the word with
//           0x03030303 after a shift by 2i yields four consecutive codes)
//   codes1  32-bit words of 32 one-bit codes (bit 2 of a 3-bit code): bit
//           4n + s of word w holds weight 32w + 16(s >> 1) + 8(n & 1) +
//           (n >> 1) + 4(s & 1), the nibble order that codes2 words take
//           when masked with 0x33333333
//   tables  per table of the block: 2^b high bytes, then 2^b low bytes
//   combined (NESTED) per table: 16 high bytes, then 16 low bytes of
//           fp16(f32(coarse[c]) + f32(refine[c][r])) at entry 4c + r
//   dense   the row's fp16 / bf16 values of the block
// B 4-bit: codes4 + tables.  B 3-bit: codes2 (low bits) + codes1 + tables.
// B 2-bit: codes2 + tables.  NESTED: coarse codes2 + coarse tables +
// residual codes2 + combined tables (the full tier reads planes 0, 2, 3,
// the coarse tier planes 0, 1).  R8 (blocks of 64 columns): codes8, the
// row's uint8 indices of the block, + scales, the bf16 absmax of the
// 128-weight block holding these 64 columns (stored once per 64 columns).
// ------------------------------------------------------------------------
constexpr int kTcRows = 128;

__host__ __device__ inline int tc_unit(int bpr) { return bpr < 16 ? bpr : 16; }
__host__ __device__ inline int tc_pos(int bpr, int row, int o) {
  const int u = tc_unit(bpr);
  return (o / u) * (kTcRows * u) + row * u + o % u;
}
// Columns per block: dense 32 (two k16 MMA slabs per pipeline stage), LUT
// formats max(64, group) so that a block holds whole tables.
__host__ __device__ inline int tc_block_cols(int format, int group) {
  return format == BLUT_FMT_DENSE ? 32 : format == BLUT_FMT_R8 ? 64 : (group > 64 ? group : 64);
}

__host__ inline bool make_tc_layout(const blut_mat_desc& d, TiledLayout& L) {
  const bool paired = (d.layout & BLUT_LAYOUT_PAIRED) != 0;
  if (d.rows <= 0 || d.cols <= 0 || d.rows % (paired ? 2 * kTcRows : kTcRows)) return false;
  L = TiledLayout{};
  L.tc = 1;
  L.kb = tc_block_cols(d.format, d.group);
  if (d.cols % L.kb) return false;
  L.ntiles = d.rows / kTcRows;
  L.nchunks = d.cols / L.kb;
  auto add = [&](int kind, int bpr, int entries) {
    L.kind[L.nplanes] = kind;
    L.bpr[L.nplanes] = bpr;
    L.piece[L.nplanes] = (int64_t)kTcRows * bpr;
    L.entries[L.nplanes] = entries;
    L.nplanes++;
  };
  const bool g_ok = d.group == 32 || d.group == 64 || d.group == 128;
  switch (d.format) {
    case BLUT_FMT_B:
      if (d.dtype != BLUT_F16 || !g_ok) return false;
      if (d.bits == 4) {
        add(kPlaneCodes4, L.kb / 2, 0);
        add(kPlaneTables, (L.kb / d.group) * 32, 16);
      } else if (d.bits == 3) {
        add(kPlaneCodes2, L.kb / 4, 0);
        add(kPlaneCodes1, L.kb / 8, 0);
        add(kPlaneTables, (L.kb / d.group) * 16, 8);
      } else if (d.bits == 2) {
        add(kPlaneCodes2, L.kb / 4, 0);
        add(kPlaneTables, (L.kb / d.group) * 8, 4);
      } else {
        return false;
      }
      break;
    case BLUT_FMT_NESTED:
      if (d.dtype != BLUT_F16 || !g_ok) return false;
      add(kPlaneCodes2, L.kb / 4, 0);                  // coarse codes
      add(kPlaneTables, (L.kb / d.group) * 8, 4);      // coarse tables
      add(kPlaneCodes2, L.kb / 4, 0);                  // residual codes
      add(kPlaneCombined, (L.kb / d.group) * 32, 16);  // combined tables
      break;
    case BLUT_FMT_R8:  // absmax blocks of 128 weights lie in one row when cols % 128 == 0
      if (d.group != 128 || d.dtype != BLUT_BF16 || d.cols % 128) return false;
      add(kPlaneCodes8, L.kb, 0);
      add(kPlaneScales, 2, 0);
      break;
    case BLUT_FMT_DENSE:
      if (d.dtype != BLUT_F16 && d.dtype != BLUT_BF16) return false;
      add(kPlaneDense, L.kb * 2, 0);
      break;
    default:
      return false;
  }
  int64_t off = 0;
  for (int p = 0; p < L.nplanes; ++p) {
    L.off[p] = off;
    off = align256(off + L.piece[p] * L.ntiles * L.nchunks);
  }
  L.total = off;
  return true;
}

__host__ __device__ inline int64_t table_piece_bytes(int entries, int group) {
  return int64_t(kChunk / group) * kTileRows * entries * 2;
}

// Fills `L` for `d`.  Returns false if the shape/format has no tiled layout.
__host__ inline bool make_layout(const blut_mat_desc& d, TiledLayout& L) {
  if ((d.layout & ~(BLUT_LAYOUT_PAIRED | BLUT_LAYOUT_TC)) != 0) return false;
  if (d.layout & BLUT_LAYOUT_TC) return make_tc_layout(d, L);
  if (d.rows <= 0 || d.cols <= 0 || d.rows % kTileRows || d.cols % kChunk) return false;
  if ((d.layout & BLUT_LAYOUT_PAIRED) && d.rows % (2 * kTileRows)) return false;
  L = TiledLayout{};
  L.ntiles = d.rows / kTileRows;
  L.nchunks = d.cols / kChunk;
  auto add = [&](int kind, int64_t piece, int entries) {
    L.kind[L.nplanes] = kind;
    L.piece[L.nplanes] = piece;
    L.entries[L.nplanes] = entries;
    L.nplanes++;
  };
  const bool g_ok = d.group == 32 || d.group == 64 || d.group == 128;
  switch (d.format) {
    case BLUT_FMT_R8:
      if (d.group != 128 || d.dtype != BLUT_BF16) return false;
      add(kPlaneCodes8, 2048, 0);
      add(kPlaneScales, 32, 0);
      break;
    case BLUT_FMT_B:
      if (!g_ok || d.dtype != BLUT_F16) return false;
      if (d.bits == 4) {
        add(kPlaneCodes4, 1024, 0);
        add(kPlaneTables, table_piece_bytes(16, d.group), 16);
      } else if (d.bits == 3) {
        add(kPlaneCodes2, 512, 0);
        add(kPlaneCodes1, 256, 0);
        add(kPlaneTables, table_piece_bytes(8, d.group), 8);
      } else if (d.bits == 2) {
        add(kPlaneCodes2, 512, 0);
        add(kPlaneTables, table_piece_bytes(4, d.group), 4);
      } else {
        return false;
      }
      break;
    case BLUT_FMT_NESTED:
      if (!g_ok || d.dtype != BLUT_F16) return false;
      add(kPlaneCodes2, 512, 0);                              // coarse codes
      add(kPlaneTables, table_piece_bytes(4, d.group), 4);    // coarse tables
      add(kPlaneCodes2, 512, 0);                              // residual codes
      add(kPlaneTables, table_piece_bytes(16, d.group), 16);  // combined tables
      break;
    case BLUT_FMT_DENSE:
      if (d.dtype != BLUT_F16 && d.dtype != BLUT_BF16) return false;
      add(kPlaneDense, 4096, 0);
      break;
    default:
      return false;
  }
  int64_t off = 0;
  for (int p = 0; p < L.nplanes; ++p) {
    L.off[p] = off;
    off = align256(off + L.piece[p] * L.ntiles * L.nchunks);
  }
  L.total = off;
  return true;
}

// Planes a matmul of `d` reads, in the order its decode takes them: every
// plane, except NESTED, whose full tier reads the coarse codes, residual
// codes and combined tables (planes 0, 2, 3) and whose coarse tier reads the
// coarse codes and tables (planes 0, 1).  Returns their number.
__host__ inline int plane_select(const blut_mat_desc& d, const TiledLayout& L, int (&idx)[3]) {
  idx[0] = 0; idx[1] = 1; idx[2] = 2;
  if (d.format == BLUT_FMT_NESTED) {
    if (d.tier == 0) {
      idx[1] = 2; idx[2] = 3;
      return 3;
    }
    return 2;
  }
  return L.nplanes < 3 ? L.nplanes : 3;
}

// Pieces are stored chunk-major inside each plane: piece (chunk c, physical
// tile pt) sits at plane_off + (c * ntiles + pt) * piece, so the tiles a CTA
// streams together at one chunk are one contiguous range.  With
// BLUT_LAYOUT_PAIRED, logical tile t of the first half of the rows (gate) is
// physical tile 2t and tile t of the second half (up) is physical tile 2t+1.
__host__ __device__ inline int64_t piece_off(const TiledLayout& L, int plane, int64_t chunk, int64_t pt) {
  return L.off[plane] + (chunk * L.ntiles + pt) * L.piece[plane];
}
__host__ __device__ inline int64_t phys_tile(int64_t t, int64_t ntiles, bool paired) {
  if (!paired) return t;
  const int64_t half = ntiles / 2;
  return t < half ? 2 * t : 2 * (t - half) + 1;
}
__host__ __device__ inline int64_t logical_tile(int64_t pt, int64_t ntiles, bool paired) {
  if (!paired) return pt;
  return (pt & 1) ? ntiles / 2 + pt / 2 : pt / 2;
}

// Position of element (r, k) of a (tile, chunk) piece: r in [0,16), k in [0,128).
// Fragment coordinates: slab s = k / 16, half h = r / 8, lane = 4 * (r & 7) + t,
// t = (k & 7) >> 1, quad q = (k & 1) | ((k >> 3) & 1) << 1 selects one of the
// lane's four elements {2t, 2t+1, 2t+8, 2t+9} of the slab.
struct FragPos {
  int h, lane, s, q;
};
__host__ __device__ inline FragPos frag_pos(int r, int k) {
  FragPos p;
  p.h = r >> 3;
  const int kk = k & 15;
  p.lane = 4 * (r & 7) + ((kk & 7) >> 1);
  p.s = k >> 4;
  p.q = (kk & 1) | (((kk >> 3) & 1) << 1);
  return p;
}
// 32-bit word index and bit offset of element (r, k) in each code plane.
__host__ __device__ inline void codes4_pos(int r, int k, int& word, int& bit) {
  FragPos p = frag_pos(r, k);
  word = (p.h * 512 + p.lane * 16 + (p.s >> 1) * 4) >> 2;
  bit = 16 * (p.s & 1) + 4 * p.q;
}
__host__ __device__ inline void codes2_pos(int r, int k, int& word, int& bit) {
  FragPos p = frag_pos(r, k);
  word = (p.lane * 16 + p.h * 8 + (p.s >> 2) * 4) >> 2;
  bit = 4 * p.q + 2 * (p.s & 1) + 16 * ((p.s >> 1) & 1);
}
__host__ __device__ inline void codes1_pos(int r, int k, int& word, int& bit) {
  FragPos p = frag_pos(r, k);
  word = (p.lane * 8 + p.h * 4) >> 2;
  bit = 4 * p.q + (p.s & 3) + 16 * (p.s >> 2);
}
__host__ __device__ inline void codes8_pos(int r, int k, int& word, int& bit) {
  FragPos p = frag_pos(r, k);
  word = (p.h * 1024 + p.lane * 32 + p.s * 4) >> 2;
  bit = 8 * p.q;
}
// Byte offset of the (hi, lo) bytes of entry e of row r's table of chunk-block jb.
__host__ __device__ inline int table_hi_byte(int r, int jb, int e, int entries) {
  return (jb * kTileRows + r) * (2 * entries) + e;
}
// Byte offset of element (r, k) in a dense piece (2-byte elements).
__host__ __device__ inline int dense_byte(int r, int k) {
  FragPos p = frag_pos(r, k);
  const int kk = k & 15;
  return p.h * 2048 + p.lane * 64 + p.s * 8 + (kk >> 3) * 4 + (kk & 1) * 2;
}
// Byte offset of element (token n in [0,8), k in [0,128)) inside one
// (n-tile, chunk) block of B fragments (mma B operand, "col" layout).
__host__ __device__ inline int bfrag_byte(int n, int k) {
  const int kk = k & 15;
  const int lane = 4 * n + ((kk & 7) >> 1);
  const int word = 2 * (k >> 4) + (kk >> 3);
  return lane * 64 + word * 4 + (kk & 1) * 2;
}

// ------------------------------------------------------------------------
// PTX wrappers
// ------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// As mbar_try_wait, but a thread whose phase is not complete yet may sleep in
// hardware for up to `ns` nanoseconds (it wakes as soon as the phase
// completes) instead of returning at once to spin.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait: gives up after ~2 s of wall time and reports it in *status.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1; i < (1u << 30); ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63) == 0 && globaltimer_ns() - t0 > 2000000000ull) break;
  }
  atomicOr(status, kDevTimeout);
  return false;
}
// Bulk (non-tensor) TMA copy global -> shared, completing on an mbarrier.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

template <bool kBF16>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (kBF16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

template <bool kBF16>
__device__ __forceinline__ uint16_t f32_to_act(float v) {
  if constexpr (kBF16) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(v));
  } else {
    return __half_as_ushort(__float2half_rn(v));
  }
}
template <bool kBF16>
__device__ __forceinline__ float act_to_f32(uint16_t v) {
  if constexpr (kBF16) {
    return __bfloat162float(__ushort_as_bfloat16(v));
  } else {
    return __half2float(__ushort_as_half(v));
  }
}

}  // namespace blut
