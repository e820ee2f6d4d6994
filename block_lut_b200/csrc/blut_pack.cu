// Canonical-layout kernels: bit-exact dequantisation, repacking into the
// tiled layout, and the encoders.
#include <algorithm>

#include "blut_common.cuh"
#include "blut_internal.h"

namespace blut {

namespace {

inline unsigned grid1d(int64_t n, int threads) {
  const int64_t g = (n + threads - 1) / threads;
  return (unsigned)std::min<int64_t>(std::max<int64_t>(g, 1), 1 << 30);
}

__device__ __forceinline__ uint16_t bf16_mul_bits(uint16_t a, uint16_t b) {
  // exact float product of two bf16 values, one RNE rounding to bf16
  const float p = __fmul_rn(__uint_as_float(uint32_t(a) << 16), __uint_as_float(uint32_t(b) << 16));
  return __bfloat16_as_ushort(__float2bfloat16_rn(p));
}

// Code of element k of a row stored as a little-endian bit stream.
__device__ __forceinline__ uint32_t stream_code(const uint8_t* row, int64_t k, int bits) {
  const int64_t bit = k * bits;
  const int64_t byte = bit >> 3;
  const int sh = int(bit & 7);
  uint32_t v = row[byte];
  if (sh + bits > 8) v |= uint32_t(row[byte + 1]) << 8;
  return (v >> sh) & ((1u << bits) - 1u);
}

// ------------------------------------------------------------ FMT_R8 ----
// out[e][i] = bf16(table[idx & mask] * absmax[e][min(i / bs, nb - 1)]); one
// thread per 16 elements (uint4 of codes) when aligned, else per element.
__global__ void r8_dequant_kernel(uint16_t* __restrict__ out, const uint8_t* __restrict__ idx,
                                  const uint16_t* __restrict__ absmax, const uint16_t* __restrict__ table,
                                  int64_t n, int64_t nb, int bs, uint32_t mask, bool vec) {
  __shared__ uint16_t tab[256];
  for (int i = threadIdx.x; i < 256; i += blockDim.x) tab[i] = table[i];
  __syncthreads();
  const int64_t e = blockIdx.y;
  const uint8_t* ip = idx + e * n;
  const uint16_t* ap = absmax + e * nb;
  uint16_t* op = out + e * n;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if (vec) {
    for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < n / 16; v += stride) {
      const uint4 c = *reinterpret_cast<const uint4*>(ip + v * 16);
      const uint8_t* cb = reinterpret_cast<const uint8_t*>(&c);
      const int64_t i0 = v * 16;
      const uint16_t s = ap[std::min<int64_t>(i0 / bs, nb - 1)];
      // a 16-element group never crosses a block boundary when bs % 16 == 0
      uint32_t w[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const uint16_t lo = bf16_mul_bits(tab[cb[2 * q] & mask], s);
        const uint16_t hi = bf16_mul_bits(tab[cb[2 * q + 1] & mask], s);
        w[q] = uint32_t(lo) | (uint32_t(hi) << 16);
      }
      uint4* o = reinterpret_cast<uint4*>(op + i0);
      o[0] = make_uint4(w[0], w[1], w[2], w[3]);
      o[1] = make_uint4(w[4], w[5], w[6], w[7]);
    }
  } else {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
      op[i] = bf16_mul_bits(tab[ip[i] & mask], ap[std::min<int64_t>(i / bs, nb - 1)]);
    }
  }
}

// ------------------------------------------------------- FMT_B / NESTED ----
__global__ void b_dequant_kernel(uint16_t* __restrict__ out, const uint8_t* __restrict__ codes,
                                 const uint16_t* __restrict__ tables, int64_t rows, int64_t cols, int bits,
                                 int group) {
  const int64_t n = rows * cols;
  const int64_t row_bytes = cols * bits / 8;
  const int64_t nb = cols / group;
  const int ent = 1 << bits;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols, k = i - r * cols;
    const uint32_t c = stream_code(codes + r * row_bytes, k, bits);
    out[i] = tables[(r * nb + k / group) * ent + c];
  }
}

__global__ void nested_dequant_kernel(uint16_t* __restrict__ out, const uint8_t* __restrict__ cc,
                                      const uint8_t* __restrict__ rc, const uint16_t* __restrict__ ct,
                                      const uint16_t* __restrict__ rt, int64_t rows, int64_t cols, int group,
                                      bool coarse_only) {
  const int64_t n = rows * cols;
  const int64_t row_bytes = cols / 4;
  const int64_t nb = cols / group;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols, k = i - r * cols;
    const int64_t blk = r * nb + k / group;
    const uint32_t c = stream_code(cc + r * row_bytes, k, 2);
    const float cv = __half2float(__ushort_as_half(ct[blk * 4 + c]));
    if (coarse_only) {
      out[i] = ct[blk * 4 + c];
    } else {
      const uint32_t q = stream_code(rc + r * row_bytes, k, 2);
      const float rv = __half2float(__ushort_as_half(rt[blk * 16 + c * 4 + q]));
      out[i] = __half_as_ushort(__float2half_rn(__fadd_rn(cv, rv)));
    }
  }
}

__global__ void lut_recover_kernel(uint16_t* __restrict__ out, const uint8_t* __restrict__ idx,
                                   const uint16_t* __restrict__ lut, int64_t n) {
  __shared__ uint16_t tab[256];
  for (int i = threadIdx.x; i < 256; i += blockDim.x) tab[i] = lut[i];
  __syncthreads();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = tab[idx[i]];
}

// --------------------------------------------------------- tiled repack ----
// One thread per element: places its code / value at its fragment position.
// Code planes narrower than a byte are assembled with atomicOr into the
// zeroed tiled buffer (whose planes are 256-byte aligned and padded).
struct PackArgs {
  TiledLayout L;
  int format, bits, group, tier, layout;
  int64_t rows, cols;
  uint8_t* dst;
  const uint8_t* codes;
  const uint8_t* codes2;
  const uint16_t* tables;
  const uint16_t* tables2;
  const uint16_t* scales;
};

__device__ __forceinline__ uint8_t* piece_ptr(const PackArgs& a, int plane, int64_t r, int64_t k) {
  const int64_t pt = phys_tile(r / kTileRows, a.L.ntiles, (a.layout & BLUT_LAYOUT_PAIRED) != 0);
  return a.dst + piece_off(a.L, plane, k / kChunk, pt);
}

__device__ __forceinline__ void or_code(uint8_t* piece, int word, int bit, uint32_t v) {
  if (v) atomicOr(reinterpret_cast<unsigned int*>(piece) + word, v << bit);
}

__global__ void pack_codes_kernel(PackArgs a) {
  const int64_t n = a.rows * a.cols;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / a.cols, k = i - r * a.cols;
    const int rr = int(r % kTileRows), kc = int(k % kChunk);
    int word, bit;
    switch (a.format) {
      case BLUT_FMT_R8: {
        codes8_pos(rr, kc, word, bit);
        piece_ptr(a, 0, r, k)[word * 4 + bit / 8] = a.codes[i];
        break;
      }
      case BLUT_FMT_DENSE: {
        *reinterpret_cast<uint16_t*>(piece_ptr(a, 0, r, k) + dense_byte(rr, kc)) =
            reinterpret_cast<const uint16_t*>(a.codes)[i];
        break;
      }
      case BLUT_FMT_B: {
        const uint32_t c = stream_code(a.codes + r * (a.cols * a.bits / 8), k, a.bits);
        if (a.bits == 4) {
          codes4_pos(rr, kc, word, bit);
          or_code(piece_ptr(a, 0, r, k), word, bit, c);
        } else if (a.bits == 2) {
          codes2_pos(rr, kc, word, bit);
          or_code(piece_ptr(a, 0, r, k), word, bit, c);
        } else {
          codes2_pos(rr, kc, word, bit);
          or_code(piece_ptr(a, 0, r, k), word, bit, c & 3u);
          codes1_pos(rr, kc, word, bit);
          or_code(piece_ptr(a, 1, r, k), word, bit, c >> 2);
        }
        break;
      }
      case BLUT_FMT_NESTED: {
        codes2_pos(rr, kc, word, bit);
        or_code(piece_ptr(a, 0, r, k), word, bit, stream_code(a.codes + r * (a.cols / 4), k, 2));
        or_code(piece_ptr(a, 2, r, k), word, bit, stream_code(a.codes2 + r * (a.cols / 4), k, 2));
        break;
      }
    }
  }
}

// One thread per (row, block, entry) for tables; per (row, chunk) for R8 scales.
__global__ void pack_tables_kernel(PackArgs a) {
  if (a.format == BLUT_FMT_R8) {
    const int64_t n = a.rows * a.L.nchunks;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
      const int64_t r = i / a.L.nchunks, ch = i - r * a.L.nchunks;
      const uint16_t s = a.scales[(r * a.cols + ch * kChunk) / a.group];
      *reinterpret_cast<uint16_t*>(piece_ptr(a, 1, r, ch * kChunk) + (r % kTileRows) * 2) = s;
    }
    return;
  }
  // One thread per table byte: (row, block, plane byte b) with b < 2 * entries;
  // byte b holds the high byte of entry b (b < entries) or the low byte of
  // entry b - entries.  FMT_B: one table plane; NESTED: the coarse plane
  // (4 entries, bytes 0..7) and the combined plane (16 entries, bytes 8..39).
  const int64_t nb = a.cols / a.group;
  const int per_block = a.format == BLUT_FMT_NESTED ? 8 + 32 : 2 * (1 << a.bits);
  const int64_t n = a.rows * nb * per_block;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    int b = int(i % per_block);
    const int64_t rb = i / per_block;
    const int64_t r = rb / nb, j = rb - r * nb;
    const int64_t k0 = j * a.group;
    const int rr = int(r % kTileRows);
    const int jb = int((k0 % kChunk) / a.group);
    int plane, ent;
    uint16_t v;
    if (a.format == BLUT_FMT_B) {
      plane = a.L.nplanes - 1;
      ent = 1 << a.bits;
      v = a.tables[rb * ent + (b % ent)];
    } else if (b < 8) {  // NESTED coarse table
      plane = 1;
      ent = 4;
      v = a.tables[rb * 4 + (b % 4)];
    } else {             // NESTED combined table: fp16(coarse[c] + refine[c * 4 + r])
      b -= 8;
      plane = 3;
      ent = 16;
      const int e = b % 16;
      const float cv = __half2float(__ushort_as_half(a.tables[rb * 4 + (e >> 2)]));
      const float rv = __half2float(__ushort_as_half(a.tables2[rb * 16 + e]));
      v = __half_as_ushort(__float2half_rn(__fadd_rn(cv, rv)));
    }
    const int e = b % ent;
    const bool hi = b < ent;
    uint8_t* p = piece_ptr(a, plane, r, k0);
    p[table_hi_byte(rr, jb, e, ent) + (hi ? 0 : ent)] = hi ? uint8_t(v >> 8) : uint8_t(v & 0xFF);
  }
}

// Code of element k of row r in a canonical b-bit stream (element k at bits
// k*b .. k*b+b-1 of the row's little-endian bit stream).
__device__ __forceinline__ uint32_t canon_code(const uint8_t* codes, int64_t cols, int b, int64_t r, int64_t k) {
  const int64_t bit = k * b;
  const uint8_t* q = codes + r * (cols * b / 8) + (bit >> 3);
  uint32_t v = q[0];
  if ((bit & 7) + b > 8) v |= uint32_t(q[1]) << 8;
  return (v >> (bit & 7)) & ((1u << b) - 1u);
}

// TC layout: one thread per byte of plane `plane` (block-major, then physical
// tile, then the unit-major piece), fetching that byte from the canonical
// arrays.
__global__ void pack_tc_kernel(PackArgs a, int plane) {
  const TiledLayout& L = a.L;
  const int bpr = L.bpr[plane];
  const int unit = tc_unit(bpr);
  const int64_t piece = L.piece[plane];
  const int64_t n = piece * L.ntiles * L.nchunks;
  const bool paired = (a.layout & BLUT_LAYOUT_PAIRED) != 0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t blk = i / (piece * L.ntiles);
    const int64_t rem = i - blk * piece * L.ntiles;
    const int64_t pt = rem / piece;
    const int x = (int)(rem - pt * piece);
    const int rr = (x / unit) % kTcRows;
    const int o = (x / (kTcRows * unit)) * unit + x % unit;  // byte of the row's block data
    const int64_t r = logical_tile(pt, L.ntiles, paired) * kTcRows + rr;
    uint8_t v = 0;
    switch (L.kind[plane]) {
      case kPlaneCodes4:
        v = a.codes[r * (a.cols / 2) + blk * (L.kb / 2) + o];
        break;
      case kPlaneCodes2: {  // byte j of word w: weights 16w + 4i + j at bits 2i
        const bool resid = a.format == BLUT_FMT_NESTED && plane == 2;
        const uint8_t* src = resid ? a.codes2 : a.codes;
        const int b = a.format == BLUT_FMT_NESTED ? 2 : a.bits;
        const int64_t k0 = blk * L.kb + (o >> 2) * 16 + (o & 3);
        uint32_t acc = 0;
        for (int i = 0; i < 4; ++i) acc |= (canon_code(src, a.cols, b, r, k0 + 4 * i) & 3u) << (2 * i);
        v = uint8_t(acc);
        break;
      }
      case kPlaneCodes1: {  // bit 4n + s of word w: bit 2 of weight 32w + 16(s>>1) + 8(n&1) + (n>>1) + 4(s&1)
        uint32_t acc = 0;
        for (int bb = 0; bb < 8; ++bb) {
          const int pos = 8 * (o & 3) + bb, n = pos >> 2, sb = pos & 3;
          const int64_t k = blk * L.kb + (o >> 2) * 32 + 16 * (sb >> 1) + 8 * (n & 1) + (n >> 1) + 4 * (sb & 1);
          acc |= ((canon_code(a.codes, a.cols, 3, r, k) >> 2) & 1u) << bb;
        }
        v = uint8_t(acc);
        break;
      }
      case kPlaneCodes8:  // FMT_R8 indices, row-major canonical
        v = a.codes[r * a.cols + blk * L.kb + o];
        break;
      case kPlaneScales: {  // FMT_R8 absmax of the 128-weight block holding columns blk * kb ..
        const uint16_t e = a.scales[(r * a.cols + blk * L.kb) / 128];
        v = o ? uint8_t(e >> 8) : uint8_t(e & 0xFF);
        break;
      }
      case kPlaneCombined: {  // entry e = 4c + r: fp16(coarse[c] + refine[c][r])
        const int m = o / 32, wb = o % 32, e = wb % 16;
        const int64_t tb = r * (a.cols / a.group) + blk * (L.kb / a.group) + m;
        const float cv = __half2float(__ushort_as_half(a.tables[tb * 4 + (e >> 2)]));
        const float rv = __half2float(__ushort_as_half(a.tables2[tb * 16 + e]));
        const uint16_t x = __half_as_ushort(__float2half_rn(__fadd_rn(cv, rv)));
        v = wb < 16 ? uint8_t(x >> 8) : uint8_t(x & 0xFF);
        break;
      }
      case kPlaneTables: {
        const int ent = L.entries[plane];
        const int m = o / (2 * ent), wb = o % (2 * ent);
        const int64_t tb = r * (a.cols / a.group) + blk * (L.kb / a.group) + m;
        const uint16_t e = a.tables[tb * ent + (wb % ent)];
        v = wb < ent ? uint8_t(e >> 8) : uint8_t(e & 0xFF);
        break;
      }
      case kPlaneDense: {
        const uint16_t e = reinterpret_cast<const uint16_t*>(a.codes)[r * a.cols + blk * L.kb + o / 2];
        v = (o & 1) ? uint8_t(e >> 8) : uint8_t(e & 0xFF);
        break;
      }
    }
    a.dst[L.off[plane] + i] = v;
  }
}

// ------------------------------------------------------------- encoders ----
// Per (row, block) Lloyd k-means, one warp per block, g / 32 values per lane
// (lane l holds elements l, l + 32, ...).  Every floating-point step is an
// explicitly rounded float op in the order of the CPU restatement, so the
// tables and codes are bit-identical to it.
template <int PER>
struct WarpBlock {
  float v[PER];
  bool m[PER];
};

template <int PER>
__device__ __forceinline__ int nearest(float v, const float* c, int K) {
  int best = 0;
  float bd = fabsf(__fsub_rn(v, c[0]));
#pragma unroll
  for (int i = 1; i < 16; ++i) {
    if (i < K) {
      const float d = fabsf(__fsub_rn(v, c[i]));
      if (d < bd) { bd = d; best = i; }
    }
  }
  return best;
}

template <int PER>
__device__ void warp_lloyd(const WarpBlock<PER>& b, int K, float (&c)[16]) {
  const float big = 3.0e38f;
  float lo = big, hi = -big;
  bool any = false;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    if (b.m[j]) { lo = fminf(lo, b.v[j]); hi = fmaxf(hi, b.v[j]); any = true; }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  if (!__any_sync(0xffffffffu, any)) { lo = 0.f; hi = 0.f; }
  const float span = __fsub_rn(hi, lo);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float frac = float(2 * i + 1) / float(2 * K);  // exact (power-of-two denominator)
    c[i] = __fadd_rn(lo, __fmul_rn(span, frac));
  }
  for (int it = 0; it < 10; ++it) {
    int a[PER];
#pragma unroll
    for (int j = 0; j < PER; ++j) a[j] = nearest<PER>(b.v[j], c, K);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      if (i >= K) continue;
      float p = (b.m[0] && a[0] == i) ? b.v[0] : 0.f;
      int cnt = __popc(__ballot_sync(0xffffffffu, b.m[0] && a[0] == i));
#pragma unroll
      for (int j = 1; j < PER; ++j) {
        const bool s = b.m[j] && a[j] == i;
        p = __fadd_rn(p, s ? b.v[j] : 0.f);
        cnt += __popc(__ballot_sync(0xffffffffu, s));
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) p = __fadd_rn(p, __shfl_xor_sync(0xffffffffu, p, o));
      if (cnt > 0) c[i] = __fdiv_rn(p, float(cnt));
    }
  }
}

// Sorted fp16 table (stable insertion sort on values) as float, and as bits.
__device__ __forceinline__ void sort_table(float (&c)[16], int K, uint16_t (&h)[16]) {
#pragma unroll
  for (int i = 0; i < 16; ++i) h[i] = __half_as_ushort(__float2half_rn(c[i]));
  for (int i = 1; i < K; ++i) {
    const uint16_t x = h[i];
    const float xv = __half2float(__ushort_as_half(x));
    int j = i - 1;
    while (j >= 0 && __half2float(__ushort_as_half(h[j])) > xv) {
      h[j + 1] = h[j];
      --j;
    }
    h[j + 1] = x;
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) c[i] = __half2float(__ushort_as_half(h[i]));
}

// Writes the g codes of a warp's block (staged in shared memory) as bytes.
__device__ __forceinline__ void write_block_codes(uint8_t* sm, uint8_t* dst, int group, int bits, int lane) {
  __syncwarp();
  const int nbytes = group * bits / 8;
  for (int m = lane; m < nbytes; m += 32) {
    uint32_t byte = 0;
    for (int bpos = 0; bpos < 8; ++bpos) {
      const int bit = 8 * m + bpos;
      const int el = bit / bits, sh = bit % bits;
      byte |= ((uint32_t(sm[el]) >> sh) & 1u) << bpos;
    }
    dst[m] = uint8_t(byte);
  }
  __syncwarp();
}

template <int PER>
__global__ void __launch_bounds__(256) encode_kernel(const float* __restrict__ w, int64_t rows, int64_t cols,
                                                     int bits, int nested, uint8_t* __restrict__ codes,
                                                     uint16_t* __restrict__ tables, uint8_t* __restrict__ codes2,
                                                     uint16_t* __restrict__ tables2) {
  constexpr int G = PER * 32;
  __shared__ uint8_t sm[8][G];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t nb = cols / G;
  const int64_t blk = (int64_t)blockIdx.x * 8 + warp;
  if (blk >= rows * nb) return;
  const int64_t r = blk / nb, j = blk - r * nb;
  WarpBlock<PER> b;
#pragma unroll
  for (int q = 0; q < PER; ++q) {
    b.v[q] = w[r * cols + j * G + lane + 32 * q];
    b.m[q] = true;
  }
  const int K = nested ? 4 : (1 << bits);
  const int cbits = nested ? 2 : bits;
  float c[16];
  uint16_t h[16];
  warp_lloyd<PER>(b, K, c);
  sort_table(c, K, h);
  int code[PER];
#pragma unroll
  for (int q = 0; q < PER; ++q) code[q] = nearest<PER>(b.v[q], c, K);
  if (lane < K) tables[blk * K + lane] = h[lane];
#pragma unroll
  for (int q = 0; q < PER; ++q) sm[warp][lane + 32 * q] = uint8_t(code[q]);
  const int64_t row_bytes = cols * cbits / 8;
  write_block_codes(sm[warp], codes + r * row_bytes + j * G * cbits / 8, G, cbits, lane);
  if (!nested) return;

  // refinement: per coarse code ci, Lloyd over the residuals of its values
  WarpBlock<PER> e;
  float comb[4][4];
#pragma unroll
  for (int q = 0; q < PER; ++q) e.v[q] = __fsub_rn(b.v[q], c[code[q]]);
  for (int ci = 0; ci < 4; ++ci) {
#pragma unroll
    for (int q = 0; q < PER; ++q) e.m[q] = code[q] == ci;
    float rc[16];
    uint16_t rh[16];
    warp_lloyd<PER>(e, 4, rc);
    bool mine = false;
#pragma unroll
    for (int q = 0; q < PER; ++q) mine |= e.m[q];
    if (!__any_sync(0xffffffffu, mine)) {
#pragma unroll
      for (int i = 0; i < 16; ++i) rc[i] = 0.f;
    }
    sort_table(rc, 4, rh);
    if (lane < 4) tables2[blk * 16 + ci * 4 + lane] = rh[lane];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      comb[ci][i] = __half2float(__float2half_rn(__fadd_rn(c[ci], rc[i])));
  }
#pragma unroll
  for (int q = 0; q < PER; ++q) {
    const int ci = code[q];
    int best = 0;
    float bd = fabsf(__fsub_rn(b.v[q], comb[ci][0]));
#pragma unroll
    for (int i = 1; i < 4; ++i) {
      const float d = fabsf(__fsub_rn(b.v[q], comb[ci][i]));
      if (d < bd) { bd = d; best = i; }
    }
    sm[warp][lane + 32 * q] = uint8_t(best);
  }
  write_block_codes(sm[warp], codes2 + r * row_bytes + j * G / 4, G, 2, lane);
}

// Reference BlockLUT encoders on bf16 input: one warp per flat block of
// bs values (bs / 32 per lane), zero padding past n.
//   F32 = false: LUTQuantizer.quantize (quantizer.py:243-306): absmax floored
//     at bf16(1e-10) and rounded to bf16, the normalised value rounded to
//     bf16, the table bf16.
//   F32 = true: fast_encode.encode_lut (fast_encode.py:22-102): absmax
//     floored at 1e-10 in fp32, the normalised value w / absmax kept in fp32,
//     the table fp32 (the absmax is stored rounded to bf16).
// Both take the first index of the smallest |v - table[e]|.
template <bool F32>
__global__ void __launch_bounds__(256) encode_r_kernel(const uint16_t* __restrict__ w, int64_t n,
                                                       const void* __restrict__ cb_v, int bs,
                                                       uint8_t* __restrict__ idx, uint16_t* __restrict__ absmax) {
  __shared__ float tab[256];
  for (int i = threadIdx.x; i < 256; i += blockDim.x)
    tab[i] = F32 ? static_cast<const float*>(cb_v)[i]
                 : __uint_as_float(uint32_t(static_cast<const uint16_t*>(cb_v)[i]) << 16);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t nb = (n + bs - 1) / bs;
  const int64_t blk = (int64_t)blockIdx.x * 8 + warp;
  if (blk >= nb) return;
  const int per = bs / 32;
  float v[8];
  float am = 0.f;
  for (int q = 0; q < per; ++q) {
    const int64_t i = blk * bs + lane + 32 * q;
    v[q] = i < n ? __uint_as_float(uint32_t(w[i]) << 16) : 0.f;
    am = fmaxf(am, fabsf(v[q]));
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
  const float floor_v =
      F32 ? 1e-10f : __uint_as_float(uint32_t(__bfloat16_as_ushort(__float2bfloat16_rn(1e-10f))) << 16);
  am = fmaxf(am, floor_v);
  const uint16_t amb = __bfloat16_as_ushort(__float2bfloat16_rn(am));
  const float amf = F32 ? am : __uint_as_float(uint32_t(amb) << 16);
  if (lane == 0) absmax[blk] = amb;
  for (int q = 0; q < per; ++q) {
    const int64_t i = blk * bs + lane + 32 * q;
    if (i >= n) continue;
    const float x = __fdiv_rn(v[q], amf);
    const float nv = F32 ? x : __bfloat162float(__float2bfloat16_rn(x));
    int best = 0;
    float bd = fabsf(__fsub_rn(nv, tab[0]));
    for (int e = 1; e < 256; ++e) {
      const float d = fabsf(__fsub_rn(nv, tab[e]));
      if (d < bd) { bd = d; best = e; }
    }
    idx[i] = uint8_t(best);
  }
}

}  // namespace

int dequant(const blut_mat_desc& d, const blut_canon& c, void* out, cudaStream_t stream) {
  if (!out || d.rows <= 0 || d.cols <= 0) return BLUT_ERR_INVALID;
  const int64_t n = d.rows * d.cols;
  const int threads = 256;
  switch (d.format) {
    case BLUT_FMT_R8: {
      if (!c.codes || !c.tables || !c.scales || d.group <= 0) return BLUT_ERR_INVALID;
      if (d.tier < 0 || d.tier > 2) return BLUT_ERR_INVALID;
      const uint32_t mask = d.tier == 1 ? 0x3Fu : d.tier == 2 ? 0x0Fu : 0xFFu;
      const int64_t nb = (n + d.group - 1) / d.group;
      const bool vec = n % 16 == 0 && d.group % 16 == 0 && ((uintptr_t)c.codes & 15) == 0 && ((uintptr_t)out & 15) == 0;
      const int64_t work = vec ? n / 16 : n;
      r8_dequant_kernel<<<dim3(std::min<unsigned>(grid1d(work, threads), 65535u), 1), threads, 0, stream>>>(
          (uint16_t*)out, (const uint8_t*)c.codes, (const uint16_t*)c.scales, (const uint16_t*)c.tables, n, nb,
          d.group, mask, vec);
      break;
    }
    case BLUT_FMT_B: {
      if (!c.codes || !c.tables || (d.bits < 2 || d.bits > 4)) return BLUT_ERR_INVALID;
      if (d.group <= 0 || d.cols % d.group || (d.cols * d.bits) % 8) return BLUT_ERR_UNSUPPORTED;
      b_dequant_kernel<<<std::min<unsigned>(grid1d(n, threads), 65535u), threads, 0, stream>>>(
          (uint16_t*)out, (const uint8_t*)c.codes, (const uint16_t*)c.tables, d.rows, d.cols, d.bits, d.group);
      break;
    }
    case BLUT_FMT_NESTED: {
      if (!c.codes || !c.tables || (d.tier == 0 && (!c.codes2 || !c.tables2))) return BLUT_ERR_INVALID;
      if (d.group <= 0 || d.cols % d.group || d.cols % 4) return BLUT_ERR_UNSUPPORTED;
      nested_dequant_kernel<<<std::min<unsigned>(grid1d(n, threads), 65535u), threads, 0, stream>>>(
          (uint16_t*)out, (const uint8_t*)c.codes, (const uint8_t*)c.codes2, (const uint16_t*)c.tables,
          (const uint16_t*)c.tables2, d.rows, d.cols, d.group, d.tier != 0);
      break;
    }
    case BLUT_FMT_DENSE:
      if (!c.codes) return BLUT_ERR_INVALID;
      if (cudaMemcpyAsync(out, c.codes, n * 2, cudaMemcpyDeviceToDevice, stream) != cudaSuccess) return BLUT_ERR_CUDA;
      break;
    default:
      return BLUT_ERR_UNSUPPORTED;
  }
  return cudaGetLastError() == cudaSuccess ? BLUT_OK : BLUT_ERR_LAUNCH;
}

int blocklut_decompress(void* out, const void* idx, const void* absmax, const void* cb, int64_t num_experts,
                        int64_t elems, int64_t blocks_per_expert, int block_size, cudaStream_t stream) {
  if (!out || !idx || !absmax || !cb || num_experts <= 0 || elems <= 0 || blocks_per_expert <= 0 || block_size <= 0)
    return BLUT_ERR_INVALID;
  if (num_experts > 65535) return BLUT_ERR_UNSUPPORTED;
  const bool vec = elems % 16 == 0 && block_size % 16 == 0 && ((uintptr_t)idx & 15) == 0 && ((uintptr_t)out & 15) == 0;
  const int64_t work = vec ? elems / 16 : elems;
  r8_dequant_kernel<<<dim3(std::min<unsigned>(grid1d(work, 256), 65535u), (unsigned)num_experts), 256, 0, stream>>>(
      (uint16_t*)out, (const uint8_t*)idx, (const uint16_t*)absmax, (const uint16_t*)cb, elems, blocks_per_expert,
      block_size, 0xFFu, vec);
  return cudaGetLastError() == cudaSuccess ? BLUT_OK : BLUT_ERR_LAUNCH;
}

int lut_recover(void* out, const void* idx, const void* lut, int64_t n, cudaStream_t stream) {
  if (!out || !idx || !lut || n <= 0) return BLUT_ERR_INVALID;
  lut_recover_kernel<<<std::min<unsigned>(grid1d(n, 256), 65535u), 256, 0, stream>>>(
      (uint16_t*)out, (const uint8_t*)idx, (const uint16_t*)lut, n);
  return cudaGetLastError() == cudaSuccess ? BLUT_OK : BLUT_ERR_LAUNCH;
}

int pack_tiled(const blut_mat_desc& d, const blut_canon& c, void* tiled, cudaStream_t stream) {
  TiledLayout L;
  if (!tiled) return BLUT_ERR_INVALID;
  if (!make_layout(d, L)) return BLUT_ERR_UNSUPPORTED;
  if (((uintptr_t)tiled & 255) != 0) return BLUT_ERR_INVALID;
  if (!c.codes) return BLUT_ERR_INVALID;
  if (d.format == BLUT_FMT_R8 && !c.scales) return BLUT_ERR_INVALID;
  if ((d.format == BLUT_FMT_B || d.format == BLUT_FMT_NESTED) && !c.tables) return BLUT_ERR_INVALID;
  if (d.format == BLUT_FMT_NESTED && (!c.codes2 || !c.tables2)) return BLUT_ERR_INVALID;
  PackArgs a;
  a.L = L;
  a.format = d.format;
  a.bits = d.bits;
  a.group = d.group;
  a.tier = d.tier;
  a.layout = d.layout;
  a.rows = d.rows;
  a.cols = d.cols;
  a.dst = (uint8_t*)tiled;
  a.codes = (const uint8_t*)c.codes;
  a.codes2 = (const uint8_t*)c.codes2;
  a.tables = (const uint16_t*)c.tables;
  a.tables2 = (const uint16_t*)c.tables2;
  a.scales = (const uint16_t*)c.scales;
  if (cudaMemsetAsync(tiled, 0, L.total, stream) != cudaSuccess) return BLUT_ERR_CUDA;
  if (L.tc) {
    for (int p = 0; p < L.nplanes; ++p) {
      const int64_t nb = L.piece[p] * L.ntiles * L.nchunks;
      pack_tc_kernel<<<std::min<unsigned>(grid1d(nb, 256), 1u << 20), 256, 0, stream>>>(a, p);
    }
    return cudaGetLastError() == cudaSuccess ? BLUT_OK : BLUT_ERR_LAUNCH;
  }
  const int64_t n = d.rows * d.cols;
  pack_codes_kernel<<<std::min<unsigned>(grid1d(n, 256), 1u << 20), 256, 0, stream>>>(a);
  if (d.format != BLUT_FMT_DENSE) {
    const int per_block = d.format == BLUT_FMT_NESTED ? 8 + 32 : 2 * (1 << d.bits);
    const int64_t nt = d.format == BLUT_FMT_R8 ? d.rows * L.nchunks : d.rows * (d.cols / d.group) * per_block;
    pack_tables_kernel<<<std::min<unsigned>(grid1d(nt, 256), 1u << 20), 256, 0, stream>>>(a);
  }
  return cudaGetLastError() == cudaSuccess ? BLUT_OK : BLUT_ERR_LAUNCH;
}

int encode(const blut_mat_desc& d, const float* w, void* codes, void* tables, void* codes2, void* tables2,
           cudaStream_t stream) {
  if (!w || !codes || !tables || d.rows <= 0 || d.cols <= 0) return BLUT_ERR_INVALID;
  const bool nested = d.format == BLUT_FMT_NESTED;
  if (!nested && d.format != BLUT_FMT_B) return BLUT_ERR_UNSUPPORTED;
  if (nested && (!codes2 || !tables2)) return BLUT_ERR_INVALID;
  if (!nested && (d.bits < 2 || d.bits > 4)) return BLUT_ERR_UNSUPPORTED;
  if (d.group != 32 && d.group != 64 && d.group != 128) return BLUT_ERR_UNSUPPORTED;
  if (d.cols % d.group) return BLUT_ERR_UNSUPPORTED;
  const int64_t nblk = d.rows * (d.cols / d.group);
  const unsigned grid = (unsigned)((nblk + 7) / 8);
  auto go = [&](auto kern) {
    kern<<<grid, 256, 0, stream>>>(w, d.rows, d.cols, d.bits, nested ? 1 : 0, (uint8_t*)codes, (uint16_t*)tables,
                                   (uint8_t*)codes2, (uint16_t*)tables2);
  };
  if (d.group == 32) go(encode_kernel<1>);
  else if (d.group == 64) go(encode_kernel<2>);
  else go(encode_kernel<4>);
  return cudaGetLastError() == cudaSuccess ? BLUT_OK : BLUT_ERR_LAUNCH;
}

int encode_r(const void* w, int64_t n, const void* cb, int block_size, void* idx, void* absmax, bool f32,
             cudaStream_t stream) {
  if (!w || !cb || !idx || !absmax || n <= 0) return BLUT_ERR_INVALID;
  if (block_size % 32 || block_size > 256 || block_size <= 0) return BLUT_ERR_UNSUPPORTED;
  const int64_t nb = (n + block_size - 1) / block_size;
  auto kern = f32 ? encode_r_kernel<true> : encode_r_kernel<false>;
  kern<<<(unsigned)((nb + 7) / 8), 256, 0, stream>>>((const uint16_t*)w, n, cb, block_size, (uint8_t*)idx,
                                                     (uint16_t*)absmax);
  return cudaGetLastError() == cudaSuccess ? BLUT_OK : BLUT_ERR_LAUNCH;
}

}  // namespace blut
