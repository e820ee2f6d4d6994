// Lookup policies: turn one 16-row x 128-column (tile, chunk) piece of a LUT
// weight matrix, resident in shared memory, into mma.m16n8k16 A fragments.
//
// A lane (g = lane / 4, t = lane % 4) owns rows g and g + 8 and, in slab s
// (16 columns), the four columns {2t, 2t+1, 2t+8, 2t+9}.  Code planes store
// exactly those four codes of a row next to each other (nibbles / bit pairs /
// bytes), so a whole quad is looked up at once:
//
//  * Per-(row, block) tables of 2^b fp16 entries are stored as a plane of
//    high bytes and a plane of low bytes.  `prmt` selects up to 4 bytes out
//    of 8 with 3-bit selectors, so the quad's codes are the selector: one
//    prmt per byte plane for b <= 3, a 3-prmt tree for b = 4.  Two more
//    prmt interleave low/high bytes into the two fp16x2 A registers.  No
//    shared-memory gathers, no bank conflicts.
//  * FMT_R8 (the reference format: 256-entry global table) looks codes up in
//    a shared-memory table replicated once per lane (bank = lane, so the
//    gather is conflict-free), then multiplies by the row's bf16 absmax with
//    mul.rn.bf16x2 -- bit-exact with the reference's bf16 dequant.
#pragma once

#include "blut_common.cuh"

namespace blut {

struct PolExtra {
  const uint32_t* r8_table;  // shared memory, [256][32] replicated table
  uint32_t r8_mask;          // tier mask applied to 8-bit codes
};

__device__ __forceinline__ uint4 lds128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ uint2 lds64(const uint8_t* p) { return *reinterpret_cast<const uint2*>(p); }

// Interleave 4 low bytes and 4 high bytes into two fp16x2 registers:
// lo = [l0 l1 l2 l3], hi = [h0 h1 h2 h3]  ->  {l0 h0 l1 h1}, {l2 h2 l3 h3}.
__device__ __forceinline__ void interleave(uint32_t lo, uint32_t hi, uint32_t& a01, uint32_t& a23) {
  a01 = prmt(lo, hi, 0x5140);
  a23 = prmt(lo, hi, 0x7362);
}

// 16-entry byte-plane lookup of 4 codes given their selectors: sel holds the
// low three code bits per nibble, sel2 picks the half (code bit 3) per byte.
__device__ __forceinline__ void lookup16s(uint32_t sel, uint32_t sel2, const uint32_t (&H)[4],
                                          const uint32_t (&L)[4], uint32_t& a01, uint32_t& a23) {
  const uint32_t hi = prmt(prmt(H[0], H[1], sel), prmt(H[2], H[3], sel), sel2);
  const uint32_t lo = prmt(prmt(L[0], L[1], sel), prmt(L[2], L[3], sel), sel2);
  interleave(lo, hi, a01, a23);
}

// 16-entry byte-plane lookup of 4 codes held in the low 16 bits of f (nibbles).
__device__ __forceinline__ void lookup16(uint32_t f, const uint32_t (&H)[4], const uint32_t (&L)[4],
                                         uint32_t& a01, uint32_t& a23) {
  lookup16s(f & 0x7777u, ((f >> 1) & 0x4444u) | 0x3210u, H, L, a01, a23);
}

// ---------------------------------------------------------------- FMT_B 4-bit
template <int GROUP>
struct PolB4 {
  static constexpr bool kBF16 = false;
  static constexpr bool kR8 = false;
  static constexpr int kSlabsPerBlock = GROUP / 16;
  static constexpr int kNumPlanes = 2;
  const uint8_t* tab;
  uint32_t c[2][4];
  uint32_t H[2][4], L[2][4];
  __device__ __forceinline__ void begin(const uint8_t* const* planes, int lane, const PolExtra&) {
    const uint4 v0 = lds128(planes[0] + lane * 16);
    const uint4 v1 = lds128(planes[0] + 512 + lane * 16);
    c[0][0] = v0.x; c[0][1] = v0.y; c[0][2] = v0.z; c[0][3] = v0.w;
    c[1][0] = v1.x; c[1][1] = v1.y; c[1][2] = v1.z; c[1][3] = v1.w;
    tab = planes[1] + (lane >> 2) * 32;
  }
  __device__ __forceinline__ void block(int jb) {
    const uint8_t* p0 = tab + jb * (16 * 32);
    const uint4 h0 = lds128(p0), l0 = lds128(p0 + 16);
    const uint4 h1 = lds128(p0 + 8 * 32), l1 = lds128(p0 + 8 * 32 + 16);
    H[0][0] = h0.x; H[0][1] = h0.y; H[0][2] = h0.z; H[0][3] = h0.w;
    L[0][0] = l0.x; L[0][1] = l0.y; L[0][2] = l0.z; L[0][3] = l0.w;
    H[1][0] = h1.x; H[1][1] = h1.y; H[1][2] = h1.z; H[1][3] = h1.w;
    L[1][0] = l1.x; L[1][1] = l1.y; L[1][2] = l1.z; L[1][3] = l1.w;
  }
  __device__ __forceinline__ void frag(int s, uint32_t (&a)[4]) const {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t f = c[h][s >> 1] >> (16 * (s & 1));
      lookup16(f, H[h], L[h], a[h], a[2 + h]);
    }
  }
  // Slabs 2sp and 2sp+1 share one code word: their selectors come from one
  // mask (and one shift for the odd slab's half).
  __device__ __forceinline__ void frag2(int sp, uint32_t (&a0)[4], uint32_t (&a1)[4]) const {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t w = c[h][sp];
      const uint32_t sel = w & 0x77777777u;
      const uint32_t sel2 = ((w >> 1) & 0x44444444u) | 0x32103210u;
      lookup16s(sel, sel2, H[h], L[h], a0[h], a0[2 + h]);
      lookup16s(sel >> 16, sel2 >> 16, H[h], L[h], a1[h], a1[2 + h]);
    }
  }
};

// ---------------------------------------------------------------- FMT_B 2-bit
// Also the coarse-only tier of FMT_NESTED (coarse codes + coarse tables).
template <int GROUP>
struct PolB2 {
  static constexpr bool kBF16 = false;
  static constexpr bool kR8 = false;
  static constexpr int kSlabsPerBlock = GROUP / 16;
  static constexpr int kNumPlanes = 2;
  const uint8_t* tab;
  uint32_t c[2][2];
  uint32_t H[2], L[2];
  __device__ __forceinline__ void begin(const uint8_t* const* planes, int lane, const PolExtra&) {
    const uint4 v = lds128(planes[0] + lane * 16);
    c[0][0] = v.x; c[0][1] = v.y; c[1][0] = v.z; c[1][1] = v.w;
    tab = planes[1] + (lane >> 2) * 8;
  }
  __device__ __forceinline__ void block(int jb) {
    const uint8_t* p0 = tab + jb * (16 * 8);
    const uint2 r0 = lds64(p0), r1 = lds64(p0 + 8 * 8);
    H[0] = r0.x; L[0] = r0.y; H[1] = r1.x; L[1] = r1.y;
  }
  __device__ __forceinline__ void frag(int s, uint32_t (&a)[4]) const {
    const int sh = 2 * (s & 1) + 16 * ((s >> 1) & 1);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t sel = (c[h][s >> 2] >> sh) & 0x3333u;
      interleave(prmt(L[h], L[h], sel), prmt(H[h], H[h], sel), a[h], a[2 + h]);
    }
  }
  __device__ __forceinline__ void frag2(int sp, uint32_t (&a0)[4], uint32_t (&a1)[4]) const {
    frag(2 * sp, a0);
    frag(2 * sp + 1, a1);
  }
};

// ---------------------------------------------------------------- FMT_B 3-bit
// Low two bits in a 2-bit plane, bit 2 in a 1-bit plane; 8-entry tables.
template <int GROUP>
struct PolB3 {
  static constexpr bool kBF16 = false;
  static constexpr bool kR8 = false;
  static constexpr int kSlabsPerBlock = GROUP / 16;
  static constexpr int kNumPlanes = 3;
  const uint8_t* tab;
  uint32_t c[2][2];
  uint32_t b2[2];
  uint32_t H[2][2], L[2][2];
  __device__ __forceinline__ void begin(const uint8_t* const* planes, int lane, const PolExtra&) {
    const uint4 v = lds128(planes[0] + lane * 16);
    c[0][0] = v.x; c[0][1] = v.y; c[1][0] = v.z; c[1][1] = v.w;
    const uint2 w = lds64(planes[1] + lane * 8);
    b2[0] = w.x; b2[1] = w.y;
    tab = planes[2] + (lane >> 2) * 16;
  }
  __device__ __forceinline__ void block(int jb) {
    const uint8_t* p0 = tab + jb * (16 * 16);
    const uint4 r0 = lds128(p0), r1 = lds128(p0 + 8 * 16);
    H[0][0] = r0.x; H[0][1] = r0.y; L[0][0] = r0.z; L[0][1] = r0.w;
    H[1][0] = r1.x; H[1][1] = r1.y; L[1][0] = r1.z; L[1][1] = r1.w;
  }
  __device__ __forceinline__ void frag(int s, uint32_t (&a)[4]) const {
    const int sh = 2 * (s & 1) + 16 * ((s >> 1) & 1);
    const int sb = (s & 3) + 16 * (s >> 2);  // bit of quad 0 in the 1-bit word
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t hb = sb >= 2 ? (b2[h] >> (sb - 2)) : (b2[h] << (2 - sb));
      const uint32_t sel = ((c[h][s >> 2] >> sh) & 0x3333u) | (hb & 0x4444u);
      interleave(prmt(L[h][0], L[h][1], sel), prmt(H[h][0], H[h][1], sel), a[h], a[2 + h]);
    }
  }
  __device__ __forceinline__ void frag2(int sp, uint32_t (&a0)[4], uint32_t (&a1)[4]) const {
    frag(2 * sp, a0);
    frag(2 * sp + 1, a1);
  }
};

// ------------------------------------------------------ FMT_NESTED full tier
// Coarse 2-bit plane + residual 2-bit plane; the 16-entry table of a block is
// fp16(coarse[c] + refine[c][r]) at index c * 4 + r (precomputed at pack
// time), so the lookup is the 4-bit one with code = c << 2 | r.
template <int GROUP>
struct PolNestedFull {
  static constexpr bool kBF16 = false;
  static constexpr bool kR8 = false;
  static constexpr int kSlabsPerBlock = GROUP / 16;
  static constexpr int kNumPlanes = 3;  // coarse codes, residual codes, combined tables
  const uint8_t* tab;
  uint32_t cc[2][2], rc[2][2];
  uint32_t H[2][4], L[2][4];
  __device__ __forceinline__ void begin(const uint8_t* const* planes, int lane, const PolExtra&) {
    const uint4 v = lds128(planes[0] + lane * 16);
    cc[0][0] = v.x; cc[0][1] = v.y; cc[1][0] = v.z; cc[1][1] = v.w;
    const uint4 r = lds128(planes[1] + lane * 16);
    rc[0][0] = r.x; rc[0][1] = r.y; rc[1][0] = r.z; rc[1][1] = r.w;
    tab = planes[2] + (lane >> 2) * 32;
  }
  __device__ __forceinline__ void block(int jb) {
    const uint8_t* p0 = tab + jb * (16 * 32);
    const uint4 h0 = lds128(p0), l0 = lds128(p0 + 16);
    const uint4 h1 = lds128(p0 + 8 * 32), l1 = lds128(p0 + 8 * 32 + 16);
    H[0][0] = h0.x; H[0][1] = h0.y; H[0][2] = h0.z; H[0][3] = h0.w;
    L[0][0] = l0.x; L[0][1] = l0.y; L[0][2] = l0.z; L[0][3] = l0.w;
    H[1][0] = h1.x; H[1][1] = h1.y; H[1][2] = h1.z; H[1][3] = h1.w;
    L[1][0] = l1.x; L[1][1] = l1.y; L[1][2] = l1.z; L[1][3] = l1.w;
  }
  __device__ __forceinline__ void frag(int s, uint32_t (&a)[4]) const {
    const int sh = 2 * (s & 1) + 16 * ((s >> 1) & 1);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t cf = cc[h][s >> 2] >> sh;
      const uint32_t rf = rc[h][s >> 2] >> sh;
      const uint32_t sel = (rf & 0x3333u) | ((cf << 2) & 0x4444u);
      const uint32_t sel2 = ((cf << 1) & 0x4444u) | 0x3210u;
      const uint32_t hi = prmt(prmt(H[h][0], H[h][1], sel), prmt(H[h][2], H[h][3], sel), sel2);
      const uint32_t lo = prmt(prmt(L[h][0], L[h][1], sel), prmt(L[h][2], L[h][3], sel), sel2);
      interleave(lo, hi, a[h], a[2 + h]);
    }
  }
  __device__ __forceinline__ void frag2(int sp, uint32_t (&a0)[4], uint32_t (&a1)[4]) const {
    frag(2 * sp, a0);
    frag(2 * sp + 1, a1);
  }
};

// ------------------------------------------------------------------- FMT_R8
struct PolR8 {
  static constexpr bool kBF16 = true;
  static constexpr bool kR8 = true;
  static constexpr int kSlabsPerBlock = 8;
  static constexpr int kNumPlanes = 2;  // codes8, scales
  const uint8_t* codes;
  const uint32_t* tbl;
  uint32_t mask;
  uint32_t sc[2];  // row absmax as bf16x2 (same value twice)
  __device__ __forceinline__ void begin(const uint8_t* const* planes, int lane, const PolExtra& ex) {
    codes = planes[0] + lane * 32;
    const uint16_t* s = reinterpret_cast<const uint16_t*>(planes[1]);
    const uint32_t s0 = s[lane >> 2], s1 = s[8 + (lane >> 2)];
    sc[0] = s0 | (s0 << 16);
    sc[1] = s1 | (s1 << 16);
    tbl = ex.r8_table + (lane & 31);
    mask = ex.r8_mask;
  }
  __device__ __forceinline__ void block(int) {}
  __device__ __forceinline__ void frag(int s, uint32_t (&a)[4]) const {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t w = *reinterpret_cast<const uint32_t*>(codes + h * 1024 + s * 4);
      const uint32_t v0 = tbl[(w & mask) * 32];
      const uint32_t v1 = tbl[((w >> 8) & mask) * 32];
      const uint32_t v2 = tbl[((w >> 16) & mask) * 32];
      const uint32_t v3 = tbl[((w >> 24) & mask) * 32];
      a[h] = bf16x2_mul(prmt(v0, v1, 0x5410), sc[h]);
      a[2 + h] = bf16x2_mul(prmt(v2, v3, 0x5410), sc[h]);
    }
  }
  __device__ __forceinline__ void frag2(int sp, uint32_t (&a0)[4], uint32_t (&a1)[4]) const {
    frag(2 * sp, a0);
    frag(2 * sp + 1, a1);
  }
};

// ---------------------------------------------------------------- FMT_DENSE
template <bool BF16>
struct PolDense {
  static constexpr bool kBF16 = BF16;
  static constexpr bool kR8 = false;
  static constexpr int kSlabsPerBlock = 8;
  static constexpr int kNumPlanes = 1;
  const uint8_t* p;
  __device__ __forceinline__ void begin(const uint8_t* const* planes, int lane, const PolExtra&) {
    p = planes[0] + lane * 64;
  }
  __device__ __forceinline__ void block(int) {}
  __device__ __forceinline__ void frag(int s, uint32_t (&a)[4]) const {
    const uint2 r0 = lds64(p + s * 8);
    const uint2 r1 = lds64(p + 2048 + s * 8);
    a[0] = r0.x; a[2] = r0.y; a[1] = r1.x; a[3] = r1.y;
  }
  __device__ __forceinline__ void frag2(int sp, uint32_t (&a0)[4], uint32_t (&a1)[4]) const {
    frag(2 * sp, a0);
    frag(2 * sp + 1, a1);
  }
};

}  // namespace blut
