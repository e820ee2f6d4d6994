// tcgen05 LUT matmul: every (token group, 256-row unit) of a layer in one
// persistent launch, with the tensor core's accumulators in tensor memory.
//
// A work item is a group of <= 32 tokens routed to one expert times one unit
// of two 128-row tiles of that expert's matrix (the gate tile and the up tile
// of a BLUT_LAYOUT_PAIRED gate/up matrix, or two consecutive tiles of a down
// matrix).  Items are handed out by a global atomic counter, so CTAs that
// finish early take more.  A CTA has ten warps:
//
//  * warp 0 (producer): takes items from the counter, posts them to a small
//    shared-memory queue and streams each item's planes, block by block,
//    with one bulk copy (cp.async.bulk) per plane and per 8-token n-tile of
//    activations into a ring of shared-memory stages;
//  * warp 1 (MMA): allocates the tensor memory and issues, from one thread,
//    tcgen05.mma M=128 x N=16|32 x K=16 per tile and slab, fp32 accumulators
//    in tensor memory;
//  * warps 2..9 (decode): one thread per weight row.  For LUT formats each
//    thread looks its row's codes up in its row's tables (byte permutes in
//    registers) and writes the fp16 A operand of a 64-column half-block to
//    tensor memory (tcgen05.st), which the MMA reads directly
//    (A-from-tensor-memory form).  Dense weights skip this: the MMA reads
//    them from shared memory.  After the K loop the same warps run the
//    epilogue from tensor memory: SiLU(gate) * up written as the down
//    projection's activations, or fp32 expert-output rows.
//
// Every wait is bounded (2 s); one that runs out sets the CTA's abort flag
// and the device status word, the roles leave their loops, the producer lets
// the copies it has in flight land, the MMA thread waits for its last MMAs,
// and the tensor memory is released before the CTA exits.
#pragma once

#include <type_traits>

#include "blut_internal.h"
#include "blut_mm.cuh"

namespace blut {

constexpr int kTcDecodeWarps = 8;  // one decode set: 2 tiles x 4 tensor-memory lane quarters
// Decode sets per CTA, taking turns over the column blocks of an item.
// Decode (MT = 32) runs two CTAs per SM with one set each (one producer and
// one MMA thread per 8 decode warps).  That measured faster than one CTA with
// two or three sets (4 or 6 A slots) and than three CTAs with one A slot
// each.  Prefill (MT = 128) runs one CTA per SM with two sets.
template <int MT>
constexpr int tc_sets() {
  return MT == 32 ? 1 : 2;
}
template <int MT>
constexpr int tc_ctas_per_sm() {
  return MT == 32 ? 2 : 1;
}
template <int MT>
constexpr int tc_threads() {
  return 32 * (2 + kTcDecodeWarps * tc_sets<MT>());
}
constexpr int kTcRingBudget = 104 * 1024;       // per CTA, two CTAs per SM (MT = 32)
constexpr int kTcRingBudgetWide = 200 * 1024;   // one CTA per SM (MT = 128)
constexpr int kTcMaxStages = 16;                // barrier slots per ring
constexpr int kTcHeader = 1024;                 // barriers, queue and flags before the rings
constexpr int kTcQueue = 4;          // depth of the shared-memory item queue
// Token groups hold up to MT tokens: MT = 32 for decode (two CTAs per SM,
// 256 tensor-memory columns each) and MT = 128 for prefill (one CTA per SM,
// 512 columns), so that one decoded weight tile feeds MMAs of N up to MT.
// An accumulator buffer is 2 tiles x MT fp32 columns.  LUT formats keep one
// buffer and a ring of three A slots of 64 columns (2 tiles x 64 fp16
// columns of K) after it; dense weights need no A slots and double-buffer
// the accumulators so the MMA runs one item ahead of the epilogue.
template <int MT>
constexpr int tc_aslots() {  // A slots: three at two CTAs per SM, two per decode set at one
  return tc_ctas_per_sm<MT>() == 2 ? 3 : 2 * tc_sets<MT>();
}
template <int MT>
constexpr int tc_cols(bool dense) {
  return tc_ctas_per_sm<MT>() == 2 ? (dense ? 4 * MT : 256) : 512;
}

// Multipliers handed to the decode (see tc_mulhi): shifts and selector
// arithmetic run as integer multiplies on the FMA pipe, and values the
// compiler cannot see keep it from folding them back into shifts on the
// integer ALU, the pipe the byte permutes already load.
struct TcMul {
  uint32_t k31, k30, k28, k26, k16;  // mul.hi by 2^n: right shift by 32 - n
  uint32_t k4, k2;                   // mul.lo by 4, 2: left shift by 2, 1
  uint32_t k11, k11h;                // 0x11, 0x110000: selector nibble doubling (tc_lut4x4)
  uint32_t k128;                     // bytes between table entries of one lane (TcDecR8)
  uint32_t r8mask;                   // FMT_R8 tier mask of four indices (0xFFFFFFFF, 0x3F3F3F3F, 0x0F0F0F0F)
};
__host__ inline TcMul tc_mul_consts(int r8_tier = 0) {
  return TcMul{1u << 31, 1u << 30, 1u << 28, 1u << 26, 1u << 16, 4u, 2u, 0x11u, 0x110000u, 128u,
               r8_tier == 1 ? 0x3F3F3F3Fu : r8_tier == 2 ? 0x0F0F0F0Fu : 0xFFFFFFFFu};
}

struct TcParams {
  const uint8_t* w;        // tiled (BLUT_LAYOUT_TC) matrices of all experts
  int64_t wstride;         // bytes between experts
  int64_t plane_off[3];    // offsets inside one matrix of the planes the decode reads
  int piece[3];            // bytes of one (tile, block) piece per plane
  int nplanes;
  int tile_bytes;          // sum of piece[]
  int ntiles;              // 128-row tiles of the matrix
  int nblocks;             // column blocks (K / kb)
  int units;               // ceil(ntiles / 2)
  int pair;                // 1: gate/up epilogue (SiLU(gate) * up); 0: fp32 rows
  GroupTab gt;
  const uint8_t* bin;      // activations in the tcgen05 operand order (tc_bact_off), blocks of KB columns
  int64_t ntstride;        // n-tiles between column blocks of bin and act_out
  uint8_t* act_out;        // pair epilogue: down-projection activations, blocks of out_kb columns
  int out_kb;
  float* y_out;            // single epilogue: y[slot][y_ld] (slice s of split K at y_out + s * y_sstride)
  int y_ld;
  int64_t y_sstride;
  // Split K: each (group, unit) is cut into ks slices of bps blocks.  Gate/up
  // slices write fp32 partials (part, [item][gate|up][128 rows][32 tokens])
  // that splitk_silu_kernel sums in slice order; down slices write separate
  // output rows that the combine sums in slice order.
  int ks, bps;
  float* part;
  int* counter;            // item counter (zeroed by the plan kernel)
  TcMul mul;               // tc_mul_consts()
  const uint16_t* r8_table;  // FMT_R8: the tier's bf16 [256] table
  int64_t gemv_groups;     // small-batch GEMV: bound on the token groups (the grid is sized by it)
  int* status;
  int stages;              // weight stages (LUT formats) or weight + activation stages (dense)
  int xstages;             // activation stages (LUT formats)
  uint64_t wait_ns;        // limit of every bounded wait (wait_limit_ns())
};

// Activations for the tcgen05 matmuls: blocks of kb columns (the consumer's
// column block), each block holding every n-tile of 8 tokens in order
// (ntstride of them), each (block, n-tile) piece kb / 8 core matrices of 8
// tokens x 8 columns, K-major, as tcgen05.mma reads its B operand without
// swizzle.  A token group's n-tiles are consecutive, so one bulk copy moves
// a group's block.  Byte offset of (token n, column k):
__host__ __device__ inline int64_t tc_bact_off(int64_t n, int k, int kb, int64_t ntstride) {
  return ((int64_t)(k / kb) * ntstride + (n >> 3)) * (kb * 16) + ((k % kb) >> 3) * 128 + (n & 7) * 16 + (k & 7) * 2;
}

// ------------------------------------------------------------ PTX helpers --
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// Shared-memory matrix descriptor, no swizzle, K-major: lbo = bytes between
// core matrices adjacent in K, sbo = bytes between 8-row groups.
__device__ __forceinline__ uint64_t tc_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// Instruction descriptor of kind::f16: fp32 accumulate, A and B K-major,
// M = 128, N = n.
__host__ __device__ inline uint32_t tc_idesc(bool bf16, int n) {
  const uint32_t ab = bf16 ? 1u : 0u;
  return (1u << 4) | (ab << 7) | (ab << 10) | ((uint32_t)(n >> 3) << 17) | ((128u >> 4) << 24);
}

__device__ __forceinline__ void tc_mma_ts(uint32_t d, uint32_t a, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void tc_mma_ss(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}

// The MMAs of one 64-column half-block (4 slabs of K = 16) for one tile
// (NT = 1) or both tiles (NT = 2) of a unit, issued from one straight-line
// block so that the single issuing thread spends few instructions per half
// (it shares its sub-partition with ALU-bound decode warps, so every
// instruction it issues waits for a slot): slab sl of tile t reads A from
// tensor-memory column a + 32 t + 8 sl and B through the descriptor
// {b_lo + 16 sl, b_hi} (the low word's bits 0-13 are the activations'
// shared address >> 4, and slab sl starts 256 sl bytes further).
// Accumulators: d0 (tile 0) and d1 (tile 1).  `acc` = 0 starts them fresh
// at slab 0; later slabs always accumulate.
template <int NT>
__device__ __forceinline__ void tc_mma_half(uint32_t d0, uint32_t d1, uint32_t a, uint32_t b_lo, uint32_t b_hi,
                                            uint32_t idesc, uint32_t acc) {
  if constexpr (NT == 2) {
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t.reg .b64 bd;\n\t.reg .b32 bl, a0, a1;\n\t"
        "setp.ne.b32 p, %6, 0;\n\t"
        "setp.eq.b32 q, %6, %6;\n\t"
        "mov.b64 bd, {%3, %4};\n\t"
        "add.u32 a1, %2, 32;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%2], bd, %5, p;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [a1], bd, %5, p;\n\t"
        "add.u32 bl, %3, 16;\n\tmov.b64 bd, {bl, %4};\n\tadd.u32 a0, %2, 8;\n\tadd.u32 a1, %2, 40;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a0], bd, %5, q;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [a1], bd, %5, q;\n\t"
        "add.u32 bl, %3, 32;\n\tmov.b64 bd, {bl, %4};\n\tadd.u32 a0, %2, 16;\n\tadd.u32 a1, %2, 48;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a0], bd, %5, q;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [a1], bd, %5, q;\n\t"
        "add.u32 bl, %3, 48;\n\tmov.b64 bd, {bl, %4};\n\tadd.u32 a0, %2, 24;\n\tadd.u32 a1, %2, 56;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a0], bd, %5, q;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [a1], bd, %5, q;\n\t}" ::"r"(d0),
        "r"(d1), "r"(a), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(acc)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t.reg .b64 bd;\n\t.reg .b32 bl, a0;\n\t"
        "setp.ne.b32 p, %5, 0;\n\t"
        "setp.eq.b32 q, %5, %5;\n\t"
        "mov.b64 bd, {%2, %3};\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], bd, %4, p;\n\t"
        "add.u32 bl, %2, 16;\n\tmov.b64 bd, {bl, %3};\n\tadd.u32 a0, %1, 8;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a0], bd, %4, q;\n\t"
        "add.u32 bl, %2, 32;\n\tmov.b64 bd, {bl, %3};\n\tadd.u32 a0, %1, 16;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a0], bd, %4, q;\n\t"
        "add.u32 bl, %2, 48;\n\tmov.b64 bd, {bl, %3};\n\tadd.u32 a0, %1, 24;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a0], bd, %4, q;\n\t}" ::"r"(d0),
        "r"(a), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(acc)
        : "memory");
    (void)d1;
  }
}

// 32 consecutive 32-bit columns of this thread's lane.
__device__ __forceinline__ void tc_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31]));
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 16 consecutive 32-bit columns of this thread's lane.
__device__ __forceinline__ void tc_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]));
}
// 16 consecutive 32-bit columns, then the wait; the registers are tied to the
// wait so that no use is scheduled before it.
__device__ __forceinline__ void tc_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tc_wait_ld16(uint32_t (&v)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                 "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15])
               :
               : "memory");
}

__device__ __forceinline__ uint4 tc_lds128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }

// ------------------------------------------------------- decode policies --
// One thread decodes one weight row.  A policy reads the row's codes and
// tables for 64 columns (a "half" of a block of KB columns) from the stage's
// planes (load_half) and turns them into 16 fp16 pairs per 32 columns
// (lookup_q, quarter qq of the half): out[i] = (weight 2i, weight 2i + 1).
//
// The lookups are byte permutes (prmt) on the integer ALU, the kernel's
// limiting pipe.  Tables sit as a plane of high bytes and a plane of low
// bytes, so a permute picks one byte of up to 8 entries per output byte.
// Shifts run as multiplies (mul.hi by 2^n for right shifts, mul.lo for left
// ones) on the otherwise idle FMA pipe; the multipliers come from the kernel
// parameters (TcMul) so that the compiler cannot fold them back into shifts.
__device__ __forceinline__ uint32_t tc_mulhi(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.hi.u32 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t tc_mullo(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.lo.u32 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Per-stage pointers to this tile's piece of each plane the decode reads;
// tab is the shared-memory address of this lane's column of the replicated
// FMT_R8 table.
struct TcPtrs {
  const uint8_t* p[3];
  uint32_t tab;
};

// 16-entry tables (4-bit codes): `w` holds 8 codes, one per nibble.  Permutes
// pick entries 0-7 and 8-15 with the low three code bits, a third picks
// between them with bit 3, for the high and the low bytes; two more (SA, SB)
// interleave the bytes of nibbles into fp16 pairs.  o0 / o1 come from nibbles
// 0-3, o2 / o3 from nibbles 4-7.
template <uint32_t SA, uint32_t SB>
__device__ __forceinline__ void tc_lut16(uint32_t w, const uint4& th, const uint4& tl, const TcMul& m,
                                         uint32_t& o0, uint32_t& o1, uint32_t& o2, uint32_t& o3) {
  const uint32_t s1 = w & 0x77777777u;
  const uint32_t s2 = (tc_mulhi(w, m.k31) & 0x44444444u) | 0x32103210u;  // bit 3 of each code to bit 2
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint32_t a = h ? tc_mulhi(s1, m.k16) : s1;
    const uint32_t b = h ? tc_mulhi(s2, m.k16) : s2;
    const uint32_t hi = prmt(prmt(th.x, th.y, a), prmt(th.z, th.w, a), b);
    const uint32_t lo = prmt(prmt(tl.x, tl.y, a), prmt(tl.z, tl.w, a), b);
    (h ? o2 : o0) = prmt(lo, hi, SA);
    (h ? o3 : o1) = prmt(lo, hi, SB);
  }
}
// Canonical 4-bit codes (nibble j = weight j): out[0..3] = pairs (0,1) .. (6,7).
__device__ __forceinline__ void tc_lut16x8(uint32_t w, const uint4& th, const uint4& tl, uint32_t* out,
                                           const TcMul& m) {
  tc_lut16<0x5140u, 0x7362u>(w, th, tl, m, out[0], out[1], out[2], out[3]);
}

// 8-entry tables (3-bit codes): `a` holds 8 codes with bit 3 of every nibble
// clear, nibbles 0-7 = weights (x, x+8, x+1, x+9, x+2, x+10, x+3, x+11) of a
// 16-weight run; t = {high bytes 0-3, 4-7, low bytes 0-3, 4-7}.  Gives the
// pairs (x, x+1), (x+8, x+9), (x+2, x+3), (x+10, x+11).
__device__ __forceinline__ void tc_lut8x8(uint32_t a, const uint4& t, const TcMul& m, uint32_t& o0, uint32_t& o1,
                                          uint32_t& o2, uint32_t& o3) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint32_t s = h ? tc_mulhi(a, m.k16) : a;
    const uint32_t lo = prmt(t.z, t.w, s);
    const uint32_t hi = prmt(t.x, t.y, s);
    (h ? o2 : o0) = prmt(lo, hi, 0x6240u);
    (h ? o3 : o1) = prmt(lo, hi, 0x7351u);
  }
}

// 4-entry tables (2-bit codes): x holds the codes of 4 consecutive weights in
// bits 0-1 of its bytes; th / tl are the table's high / low bytes.  One
// multiply-add turns x into the selector nibbles (c0, c0 + 4, c1, c1 + 4, ...)
// and one permute then yields an fp16 pair: out[0] = (0, 1), out[1] = (2, 3).
__device__ __forceinline__ void tc_lut4x4(uint32_t x, uint32_t th, uint32_t tl, uint32_t* out, const TcMul& m) {
  uint32_t s0, s1;
  asm("mad.lo.u32 %0, %1, %2, 0x40404040;" : "=r"(s0) : "r"(x), "r"(m.k11));
  asm("mad.hi.u32 %0, %1, %2, 0x4040;" : "=r"(s1) : "r"(x), "r"(m.k11h));
  out[0] = prmt(tl, th, s0);
  out[1] = prmt(tl, th, s1);
}
// 16 weights of a codes2 word into out[0..7].
__device__ __forceinline__ void tc_lut4x16(uint32_t w, uint32_t th, uint32_t tl, uint32_t* out, const TcMul& m) {
  tc_lut4x4(w & 0x03030303u, th, tl, out + 0, m);
  tc_lut4x4(tc_mulhi(w, m.k30) & 0x03030303u, th, tl, out + 2, m);
  tc_lut4x4(tc_mulhi(w, m.k28) & 0x03030303u, th, tl, out + 4, m);
  tc_lut4x4(tc_mulhi(w, m.k26) & 0x03030303u, th, tl, out + 6, m);
}

__device__ __forceinline__ uint2 tc_lds64(const uint8_t* p) { return *reinterpret_cast<const uint2*>(p); }

// FMT_B, 4-bit codes, tables per `G` columns.  Planes: codes4, tables.
template <int G>
struct TcDecB4 {
  static constexpr bool kDense = false;
  static constexpr bool kBF16 = false;
  static constexpr bool kR8 = false;
  static constexpr int kHalfBytes = G == 32 ? 96 : 64;  // bytes of a half's codes and tables a thread holds
  static constexpr int KB = G > 64 ? G : 64;  // columns per block
  static constexpr int kHalves = KB / 64;     // 64-column halves per block
  static constexpr int kNumPlanes = 2;
  struct Half {
    uint4 c[2], th[2], tl[2];
  };
  __device__ __forceinline__ static void load_half(const TcPtrs& pp, int row, int h, Half& d) {
#pragma unroll
    for (int qq = 0; qq < 2; ++qq) d.c[qq] = tc_lds128(pp.p[0] + ((2 * h + qq) * kTcRows + row) * 16);
#pragma unroll
    for (int qq = 0; qq < (G == 32 ? 2 : 1); ++qq) {
      const int tb = G == 32 ? 2 * h + qq : (G == 64 ? h : 0);  // table of these columns
      d.th[qq] = tc_lds128(pp.p[1] + ((2 * tb) * kTcRows + row) * 16);
      d.tl[qq] = tc_lds128(pp.p[1] + ((2 * tb + 1) * kTcRows + row) * 16);
    }
  }
  __device__ __forceinline__ static void lookup_q(const Half& d, int qq, uint32_t (&out)[16], const TcMul& m) {
    const int tq = G == 32 ? qq : 0;
    tc_lut16x8(d.c[qq].x, d.th[tq], d.tl[tq], out + 0, m);
    tc_lut16x8(d.c[qq].y, d.th[tq], d.tl[tq], out + 4, m);
    tc_lut16x8(d.c[qq].z, d.th[tq], d.tl[tq], out + 8, m);
    tc_lut16x8(d.c[qq].w, d.th[tq], d.tl[tq], out + 12, m);
  }
};

// FMT_B, 2-bit codes (and the NESTED coarse tier).  Planes: codes2, tables
// (8 bytes per table).
template <int G>
struct TcDecB2 {
  static constexpr bool kDense = false;
  static constexpr bool kBF16 = false;
  static constexpr bool kR8 = false;
  static constexpr int kHalfBytes = G == 32 ? 32 : 24;
  static constexpr int KB = G > 64 ? G : 64;
  static constexpr int kHalves = KB / 64;
  static constexpr int kNumPlanes = 2;
  struct Half {
    uint4 c;
    uint32_t th[2], tl[2];
  };
  __device__ __forceinline__ static void load_half(const TcPtrs& pp, int row, int h, Half& d) {
    d.c = tc_lds128(pp.p[0] + (h * kTcRows + row) * 16);
    if constexpr (G == 32) {  // two tables in one 16-byte unit
      const uint4 t = tc_lds128(pp.p[1] + row * 16);
      d.th[0] = t.x; d.tl[0] = t.y; d.th[1] = t.z; d.tl[1] = t.w;
    } else {
      const uint2 t = tc_lds64(pp.p[1] + row * 8);
      d.th[0] = t.x; d.tl[0] = t.y; d.th[1] = t.x; d.tl[1] = t.y;
    }
  }
  __device__ __forceinline__ static void lookup_q(const Half& d, int qq, uint32_t (&out)[16], const TcMul& m) {
    const int tq = G == 32 ? qq : 0;
    tc_lut4x16(qq ? d.c.z : d.c.x, d.th[tq], d.tl[tq], out + 0, m);
    tc_lut4x16(qq ? d.c.w : d.c.y, d.th[tq], d.tl[tq], out + 8, m);
  }
};

// FMT_B, 3-bit codes.  Planes: codes2 (bits 0-1), codes1 (bit 2), tables
// (16 bytes per table).
template <int G>
struct TcDecB3 {
  static constexpr bool kDense = false;
  static constexpr bool kBF16 = false;
  static constexpr bool kR8 = false;
  static constexpr int kHalfBytes = G == 32 ? 56 : 40;
  static constexpr int KB = G > 64 ? G : 64;
  static constexpr int kHalves = KB / 64;
  static constexpr int kNumPlanes = 3;
  struct Half {
    uint4 c2;
    uint2 c1;
    uint4 t[G == 32 ? 2 : 1];
  };
  __device__ __forceinline__ static void load_half(const TcPtrs& pp, int row, int h, Half& d) {
    d.c2 = tc_lds128(pp.p[0] + (h * kTcRows + row) * 16);
    d.c1 = tc_lds64(pp.p[1] + row * (KB / 8) + h * 8);
#pragma unroll
    for (int i = 0; i < (G == 32 ? 2 : 1); ++i) d.t[i] = tc_lds128(pp.p[2] + (i * kTcRows + row) * 16);
  }
  // 16 weights: codes2 word w2, the codes1 bits at nibble bit 2 of y (bit 3 clear)
  __device__ __forceinline__ static void run16(uint32_t w2, uint32_t ya, uint32_t yb, const uint4& t, uint32_t* out,
                                               const TcMul& m) {
    const uint32_t a = (w2 & 0x33333333u) | ya;                   // weights 0, 8, 1, 9, 2, 10, 3, 11
    const uint32_t b = (tc_mulhi(w2, m.k30) & 0x33333333u) | yb;  // weights 4, 12, 5, 13, 6, 14, 7, 15
    tc_lut8x8(a, t, m, out[0], out[4], out[1], out[5]);
    tc_lut8x8(b, t, m, out[2], out[6], out[3], out[7]);
  }
  __device__ __forceinline__ static void lookup_q(const Half& d, int qq, uint32_t (&out)[16], const TcMul& m) {
    const uint4& t = d.t[G == 32 ? qq : 0];
    const uint32_t w1 = qq ? d.c1.y : d.c1.x;
    run16(qq ? d.c2.z : d.c2.x, tc_mullo(w1, m.k4) & 0x44444444u, tc_mullo(w1, m.k2) & 0x44444444u, t, out + 0, m);
    run16(qq ? d.c2.w : d.c2.y, w1 & 0x44444444u, tc_mulhi(w1, m.k31) & 0x44444444u, t, out + 8, m);
  }
};

// FMT_NESTED, full tier: the coarse and residual codes form the 4-bit index
// 4c + r into the combined table.  Planes: coarse codes2, residual codes2,
// combined tables (32 bytes per table).
template <int G>
struct TcDecNested {
  static constexpr bool kDense = false;
  static constexpr bool kBF16 = false;
  static constexpr bool kR8 = false;
  static constexpr int kHalfBytes = G == 32 ? 96 : 64;
  static constexpr int KB = G > 64 ? G : 64;
  static constexpr int kHalves = KB / 64;
  static constexpr int kNumPlanes = 3;
  struct Half {
    uint4 cc, cr;
    uint4 th[G == 32 ? 2 : 1], tl[G == 32 ? 2 : 1];
  };
  __device__ __forceinline__ static void load_half(const TcPtrs& pp, int row, int h, Half& d) {
    d.cc = tc_lds128(pp.p[0] + (h * kTcRows + row) * 16);
    d.cr = tc_lds128(pp.p[1] + (h * kTcRows + row) * 16);
#pragma unroll
    for (int i = 0; i < (G == 32 ? 2 : 1); ++i) {
      d.th[i] = tc_lds128(pp.p[2] + ((2 * i) * kTcRows + row) * 16);
      d.tl[i] = tc_lds128(pp.p[2] + ((2 * i + 1) * kTcRows + row) * 16);
    }
  }
  // 16 weights of one coarse word wc and residual word wr into out[0..7]
  __device__ __forceinline__ static void run16(uint32_t wc, uint32_t wr, const uint4& th, const uint4& tl,
                                               uint32_t* out, const TcMul& m) {
    const uint32_t a = (wr & 0x33333333u) | (tc_mullo(wc, m.k4) & 0xCCCCCCCCu);  // weights 0, 8, 1, 9, ...
    const uint32_t b = (tc_mulhi(wr, m.k30) & 0x33333333u) | (wc & 0xCCCCCCCCu);  // weights 4, 12, 5, 13, ...
    tc_lut16<0x6240u, 0x7351u>(a, th, tl, m, out[0], out[4], out[1], out[5]);
    tc_lut16<0x6240u, 0x7351u>(b, th, tl, m, out[2], out[6], out[3], out[7]);
  }
  __device__ __forceinline__ static void lookup_q(const Half& d, int qq, uint32_t (&out)[16], const TcMul& m) {
    const int tq = G == 32 ? qq : 0;
    run16(qq ? d.cc.z : d.cc.x, qq ? d.cr.z : d.cr.x, d.th[tq], d.tl[tq], out + 0, m);
    run16(qq ? d.cc.w : d.cc.y, qq ? d.cr.w : d.cr.y, d.th[tq], d.tl[tq], out + 8, m);
  }
};

// FMT_R8, the reference's BlockLUT: uint8 indices into one 256-entry bf16
// table (masked to the tier's 64 or 16 entries), times the bf16 absmax of
// the weight's 128-weight block.  The table sits in shared memory once per
// CTA, replicated across the 32 banks (entry e of lane l at word 32 e + l),
// so the 32 lanes' lookups never conflict.  Each looked-up pair is scaled by
// one bf16x2 multiply: the product of two bf16 values is exact in fp32, so
// its single rounding to nearest even equals bf16(f32(table) * f32(absmax)).
// Planes: codes8, scales (blocks of 64 columns).
__device__ __forceinline__ uint32_t tc_lds32(uint32_t addr) {
  uint32_t v;
  asm("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint32_t tc_mad(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t tc_bmul2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
constexpr int kTcR8TableBytes = 256 * 32 * 4;

struct TcDecR8 {
  static constexpr bool kDense = false;
  static constexpr bool kBF16 = true;
  static constexpr bool kR8 = true;
  static constexpr int kHalfBytes = 72;
  static constexpr int KB = 64;
  static constexpr int kHalves = 1;
  static constexpr int kNumPlanes = 2;
  struct Half {
    uint4 c[4];
    uint32_t s2, tab;
  };
  __device__ __forceinline__ static void load_half(const TcPtrs& pp, int row, int, Half& d) {
#pragma unroll
    for (int u = 0; u < 4; ++u) d.c[u] = tc_lds128(pp.p[0] + (u * kTcRows + row) * 16);
    const uint32_t s = *reinterpret_cast<const uint16_t*>(pp.p[1] + row * 2);
    d.s2 = s | (s << 16);
    d.tab = pp.tab;
  }
  // four weights of index word w into out[0..1]
  __device__ __forceinline__ static void run4(uint32_t w, uint32_t s2, uint32_t tab, uint32_t* out,
                                              const TcMul& m) {
    w &= m.r8mask;
    const uint32_t v0 = tc_lds32(tc_mad(prmt(w, 0u, 0x4440u), m.k128, tab));
    const uint32_t v1 = tc_lds32(tc_mad(prmt(w, 0u, 0x4441u), m.k128, tab));
    const uint32_t v2 = tc_lds32(tc_mad(prmt(w, 0u, 0x4442u), m.k128, tab));
    const uint32_t v3 = tc_lds32(tc_mad(prmt(w, 0u, 0x4443u), m.k128, tab));
    out[0] = tc_bmul2(prmt(v0, v1, 0x5410u), s2);
    out[1] = tc_bmul2(prmt(v2, v3, 0x5410u), s2);
  }
  __device__ __forceinline__ static void lookup_q(const Half& d, int qq, uint32_t (&out)[16], const TcMul& m) {
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const uint4& c = d.c[2 * qq + u];
      run4(c.x, d.s2, d.tab, out + 8 * u + 0, m);
      run4(c.y, d.s2, d.tab, out + 8 * u + 2, m);
      run4(c.z, d.s2, d.tab, out + 8 * u + 4, m);
      run4(c.w, d.s2, d.tab, out + 8 * u + 6, m);
    }
  }
};

// Fills the replicated FMT_R8 table (entry e of lane l at word 32 e + l).
__device__ __forceinline__ void tc_fill_r8_table(uint32_t* tab, const uint16_t* __restrict__ src) {
  for (int i = threadIdx.x; i < 256 * 32; i += blockDim.x) tab[i] = src[i >> 5];
}

// Dense fp16 / bf16 weights: the MMA reads them from shared memory.
template <bool BF16>
struct TcDecDense {
  static constexpr bool kDense = true;
  static constexpr bool kBF16 = BF16;
  static constexpr bool kR8 = false;
  static constexpr int kHalfBytes = 64;
  static constexpr int KB = 32;
  static constexpr int kHalves = 0;
  static constexpr int kNumPlanes = 1;
  struct Half {};
  __device__ __forceinline__ static void load_half(const TcPtrs&, int, int, Half&) {}
  __device__ __forceinline__ static void lookup_q(const Half&, int, uint32_t (&)[16], const TcMul&) {}
};

// Position in a ring of n barrier-guarded slots: slot index, the parity of
// the slot's current phase, and whether the ring has wrapped (a slot being
// reused must first see its previous phase released).
struct TcRing {
  int i = 0;
  uint32_t ph = 0;
  bool wrapped = false;
  __device__ __forceinline__ void next(int n) {
    if (++i == n) {
      i = 0;
      ph ^= 1u;
      wrapped = true;
    }
  }
};

// ------------------------------------------------------------------ kernel --
// Shared-memory rings.  Dense weights and their activations are both read by
// the MMA, so one stage holds both and the MMA's commit frees it.  For LUT
// formats the weight stage is read only by the decode warps, which free it
// as soon as their loads are done; the activations, read by the MMA, sit in
// a separate small ring freed by the MMA's commit.  Weight stages therefore
// recycle without waiting for the tensor core.
template <class Dec, int MT>
__host__ __device__ inline int tc_stage_bytes(const TcParams& p) {
  return (2 * p.tile_bytes + (Dec::kDense ? (MT / kNTile) * Dec::KB * 16 : 0) + 127) & ~127;
}
template <class Dec, int MT>
__host__ __device__ constexpr int tc_xstage_bytes() {
  return Dec::kDense ? 0 : (MT / kNTile) * Dec::KB * 16;
}

// Barriers, queue and flags take the first kTcHeader bytes, then the FMT_R8
// table (TcDecR8 only), then the rings.
template <class Dec>
__host__ __device__ constexpr int tc_table_bytes() {
  return Dec::kR8 ? kTcR8TableBytes : 0;
}
template <class Dec, int MT>
__host__ inline int tc_smem_bytes(const TcParams& p) {
  return kTcHeader + tc_table_bytes<Dec>() + p.stages * tc_stage_bytes<Dec, MT>(p) +
         p.xstages * tc_xstage_bytes<Dec, MT>();
}

// Waits for this thread's tcgen05.st; `v` (the registers of the store in
// flight) is tied to the wait so the compiler keeps them unchanged until then.
__device__ __forceinline__ void tc_wait_st_keep(uint32_t (&v)[16]) {
  asm volatile("tcgen05.wait::st.sync.aligned;"
               : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                 "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15])
               :
               : "memory");
}

template <class Dec, int MT>
__global__ void __launch_bounds__(tc_threads<MT>(), tc_ctas_per_sm<MT>()) tc_mm_kernel(const TcParams p) {
  constexpr bool kDense = Dec::kDense;
  constexpr int KB = Dec::KB;
  constexpr uint32_t kCols = tc_cols<MT>(kDense);  // tensor-memory columns of this CTA
  constexpr int kDBufs = kDense ? 2 : 1;           // accumulator buffers
  constexpr int kDCols = 2 * MT;                   // columns of one accumulator buffer
  constexpr int kACol0 = kDCols;                   // first A slot (LUT formats)
  constexpr int kSets = tc_sets<MT>();
  constexpr int kTcASlots = tc_aslots<MT>();
  constexpr int kEpiWarps = kTcDecodeWarps * kSets;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);  // [kTcMaxStages] weight stage loaded
  uint64_t* empty = full + 16;                         // [kTcMaxStages] weight stage read
  uint64_t* afull = full + 32;                         // [kTcASlots <= 8] A slot written (decode warps)
  uint64_t* aempty = full + 40;                        // [kTcASlots] A slot read (MMA commit)
  uint64_t* dfull = full + 48;                         // [kDBufs] accumulators complete (MMA commit)
  uint64_t* dempty = full + 50;                        // [kDBufs] accumulators read (epilogue warps)
  uint64_t* qfull = full + 52;                         // [kTcQueue] item posted
  uint64_t* qempty = full + 56;                        // [kTcQueue] item taken by every role
  uint64_t* fin = full + 60;                           // last MMAs complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(full + 61);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(full + 62);
  volatile int* qitem = reinterpret_cast<volatile int*>(full + 63);  // [kTcQueue]
  uint64_t* xfull = full + 66;                         // [kTcMaxStages] activation stage loaded (LUT formats)
  uint64_t* xempty = full + 82;                        // [kTcMaxStages] activation stage read (MMA commit)
  uint32_t* r8tab = reinterpret_cast<uint32_t*>(smem + kTcHeader);  // barriers end at full + 98 (784 bytes)
  uint8_t* ring = smem + kTcHeader + tc_table_bytes<Dec>();
  const int S = p.stages, SX = p.xstages;
  const int stage_bytes = tc_stage_bytes<Dec, MT>(p);
  constexpr int xstage_bytes = tc_xstage_bytes<Dec, MT>();
  uint8_t* xring = ring + (int64_t)S * stage_bytes;
  const int boff = 2 * p.tile_bytes;  // activations inside a dense stage
  // planes inside a stage: each holds the pieces of the unit's two tiles
  const int qoff[3] = {0, 2 * p.piece[0], 2 * (p.piece[0] + p.piece[1])};

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_u32(full + s), 1);
      mbar_init(smem_u32(empty + s), kDense ? 1 : kTcDecodeWarps);
    }
    for (int s = 0; s < SX; ++s) {
      mbar_init(smem_u32(xfull + s), 1);
      mbar_init(smem_u32(xempty + s), 1);
    }
    for (int j = 0; j < kTcASlots; ++j) {
      mbar_init(smem_u32(afull + j), kTcDecodeWarps);
      mbar_init(smem_u32(aempty + j), 1);
    }
    for (int j = 0; j < kDBufs; ++j) {
      mbar_init(smem_u32(dfull + j), 1);
      mbar_init(smem_u32(dempty + j), kEpiWarps);
    }
    for (int j = 0; j < kTcQueue; ++j) {
      mbar_init(smem_u32(qfull + j), 1);
      mbar_init(smem_u32(qempty + j), 1 + kEpiWarps);
    }
    mbar_init(smem_u32(fin), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if constexpr (Dec::kR8) tc_fill_r8_table(r8tab, p.r8_table);
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int n_items = *p.gt.n_groups * p.units * p.ks;

  if (warp == 0) {
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      TcRing r, rx, rq;
      uint32_t issued = 0, lastph = 0;    // per weight stage: issued at least once, parity of the last issue
      uint32_t xissued = 0, xlastph = 0;  // the same per activation stage
      for (;; rq.next(kTcQueue)) {
        const int qs = rq.i;
        if (rq.wrapped && !wait_or_abort(smem_u32(qempty + qs), rq.ph ^ 1u, abort_flag, p.status, p.wait_ns)) break;
        int item = atomicAdd(p.counter, 1);
        if (item >= n_items || *abort_flag) item = -1;
        qitem[qs] = item;
        mbar_arrive(smem_u32(qfull + qs));
        if (item < 0) break;
        const int ku = item / p.ks, gi = ku / p.units, u = ku % p.units;
        const int b0 = (item % p.ks) * p.bps, b1 = min(p.nblocks, b0 + p.bps);
        const int nnt = (p.gt.ntok[gi] + kNTile - 1) / kNTile;
        const int nt0 = p.gt.nt0[gi];
        const int ntl = min(2, p.ntiles - 2 * u);
        const uint8_t* base = p.w + (int64_t)p.gt.expert[gi] * p.wstride;
        bool ok = true;
        for (int b = b0; b < b1; ++b, r.next(S)) {
          const int s = r.i;
          if (r.wrapped && !wait_or_abort(smem_u32(empty + s), r.ph ^ 1u, abort_flag, p.status, p.wait_ns)) {
            ok = false;
            break;
          }
          issued |= 1u << s;
          lastph = (lastph & ~(1u << s)) | (r.ph << s);
          uint8_t* dst = ring + (int64_t)s * stage_bytes;
          uint32_t bar = smem_u32(full + s);
          mbar_expect_tx(bar, (uint32_t)(ntl * p.tile_bytes + (kDense ? nnt * KB * 16 : 0)));
          const int64_t pt = (int64_t)b * p.ntiles + 2 * u;
#pragma unroll
          for (int k = 0; k < Dec::kNumPlanes; ++k)
            bulk_g2s(smem_u32(dst + qoff[k]), base + p.plane_off[k] + pt * p.piece[k], (uint32_t)(ntl * p.piece[k]),
                     bar);
          uint8_t* xdst = dst + boff;
          if constexpr (!kDense) {
            const int sx = rx.i;
            if (rx.wrapped && !wait_or_abort(smem_u32(xempty + sx), rx.ph ^ 1u, abort_flag, p.status, p.wait_ns)) {
              ok = false;
              break;
            }
            xissued |= 1u << sx;
            xlastph = (xlastph & ~(1u << sx)) | (rx.ph << sx);
            xdst = xring + sx * xstage_bytes;
            bar = smem_u32(xfull + sx);
            mbar_expect_tx(bar, (uint32_t)(nnt * KB * 16));
            rx.next(SX);
          }
          bulk_g2s(smem_u32(xdst), p.bin + ((int64_t)b * p.ntstride + nt0) * (KB * 16), (uint32_t)(nnt * KB * 16),
                   bar);
        }
        if (!ok) break;
      }
      if (*abort_flag) {
        // let the copies already issued land before the CTA's shared memory goes away
        for (int st = 0; st < S; ++st)
          if ((issued >> st) & 1u) wait_drain(smem_u32(full + st), (lastph >> st) & 1u);
        for (int st = 0; st < SX; ++st)
          if ((xissued >> st) & 1u) wait_drain(smem_u32(xfull + st), (xlastph >> st) & 1u);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA --
    if (lane == 0) {
      TcRing r, ra, rd, rq;
      for (;; rq.next(kTcQueue)) {
        const int qs = rq.i;
        if (!wait_or_abort(smem_u32(qfull + qs), rq.ph, abort_flag, p.status, p.wait_ns)) break;
        const int item = qitem[qs];
        mbar_arrive(smem_u32(qempty + qs));
        if (item < 0) break;
        const int ku = item / p.ks, gi = ku / p.units, u = ku % p.units;
        const int b0 = (item % p.ks) * p.bps, b1 = min(p.nblocks, b0 + p.bps);
        const int nnt = (p.gt.ntok[gi] + kNTile - 1) / kNTile;
        const int ntl = min(2, p.ntiles - 2 * u);
        const uint32_t idesc = tc_idesc(Dec::kBF16, min(MT, (nnt + 1) / 2 * 16));
        const int db = rd.i;
        if (rd.wrapped && !wait_or_abort(smem_u32(dempty + db), rd.ph ^ 1u, abort_flag, p.status, p.wait_ns)) break;
        tc_fence_after();
        const uint32_t dcol = tmem + db * kDCols;
        bool ok = true;
        // dense: r walks the combined stages; LUT formats: r walks the activation stages
        for (int b = b0; b < b1 && ok; ++b, r.next(kDense ? S : SX)) {
          const int s = r.i;
          if (!wait_or_abort(smem_u32((kDense ? full : xfull) + s), r.ph, abort_flag, p.status, p.wait_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = smem_u32(kDense ? ring + (int64_t)s * stage_bytes : xring + s * xstage_bytes);
          if constexpr (kDense) {
#pragma unroll
            for (int sl = 0; sl < KB / 16; ++sl) {
              const uint64_t bd = tc_desc(st + boff + sl * 256, 128, KB * 16);
              for (int t = 0; t < ntl; ++t) {
                const uint64_t ad = tc_desc(st + t * p.piece[0] + sl * 2 * 2048, 2048, 128);
                tc_mma_ss(dcol + t * MT, ad, bd, idesc, ((b - b0) | sl) != 0);
              }
            }
          } else {
            const uint64_t bd0 = tc_desc(st, 128, KB * 16);  // slab 0 of half 0; later slabs add to the low word
            const uint32_t b_lo = (uint32_t)bd0, b_hi = (uint32_t)(bd0 >> 32);
#pragma unroll
            for (int h = 0; h < Dec::kHalves; ++h, ra.next(kTcASlots)) {
              const int j = ra.i;
              if (!wait_or_abort(smem_u32(afull + j), ra.ph, abort_flag, p.status, p.wait_ns)) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint32_t a = tmem + kACol0 + j * 64;
              const uint32_t acc = ((b - b0) | h) != 0;
              if (ntl == 2)
                tc_mma_half<2>(dcol, dcol + MT, a, b_lo + h * 64, b_hi, idesc, acc);
              else
                tc_mma_half<1>(dcol, dcol + MT, a, b_lo + h * 64, b_hi, idesc, acc);
              tc_commit(smem_u32(aempty + j));
            }
          }
          tc_commit(smem_u32((kDense ? empty : xempty) + s));
        }
        if (!ok) break;
        tc_commit(smem_u32(dfull + db));
        rd.next(kDBufs);
      }
      // all MMAs this thread issued are complete before the memory goes away
      tc_commit(smem_u32(fin));
      wait_drain(smem_u32(fin), 0);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------- decode and epilogue --
    const int dw = warp - 2;
    const int set = dw / kTcDecodeWarps;      // decode set: takes blocks b0 + set, b0 + set + kSets, ...
    const int t = (dw % kTcDecodeWarps) >> 2;  // tile of the unit
    const int q = warp & 3;            // tensor-memory lane quarter this warp may access
    const int row = 32 * q + lane;     // row inside the 128-row tile
    const uint32_t lane_base = (uint32_t)(32 * q) << 16;
    TcRing r, ra, rd, rq;
    for (;; rq.next(kTcQueue)) {
      const int qs = rq.i;
      bool ok = wait_or_abort(smem_u32(qfull + qs), rq.ph, abort_flag, p.status, p.wait_ns);
      if (__shfl_sync(0xffffffffu, ok ? 1 : 0, 0) == 0) break;
      const int item = qitem[qs];
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(qempty + qs));
      if (item < 0) break;
      const int ku = item / p.ks, gi = ku / p.units, u = ku % p.units;
      const int b0 = (item % p.ks) * p.bps, b1 = min(p.nblocks, b0 + p.bps);
      const int ntok = p.gt.ntok[gi];
      const int ntl = min(2, p.ntiles - 2 * u);
      if constexpr (!kDense) {
        const bool active = t < ntl;
        bool aborted = false;
        // A half is decoded as two quarters (qa, qb): the store of the first
        // runs while the second is decoded.
        for (int b = b0; b < b1 && !aborted; ++b, r.next(S)) {
          if (kSets > 1 && (b - b0) % kSets != set) {  // the other decode set's block
#pragma unroll
            for (int h = 0; h < Dec::kHalves; ++h) ra.next(kTcASlots);
            continue;
          }
          const int s = r.i;
          ok = wait_or_abort(smem_u32(full + s), r.ph, abort_flag, p.status, p.wait_ns);
          if (__shfl_sync(0xffffffffu, ok ? 1 : 0, 0) == 0) {
            aborted = true;
            break;
          }
          const uint8_t* st = ring + (int64_t)s * stage_bytes;
          TcPtrs pp;
#pragma unroll
          for (int k = 0; k < 3; ++k) pp.p[k] = st + qoff[k] + t * p.piece[k];
          pp.tab = smem_u32(r8tab) + lane * 4;
#pragma unroll
          for (int h = 0; h < Dec::kHalves; ++h, ra.next(kTcASlots)) {
            const int j = ra.i;
            uint32_t qa[16], qb[16];
            typename Dec::Half hd;
            if (active) {  // the first quarter's lookups run before the slot is known free
              Dec::load_half(pp, row, h, hd);
              Dec::lookup_q(hd, 0, qa, p.mul);
            }
            if (ra.wrapped) {
              ok = wait_or_abort(smem_u32(aempty + j), ra.ph ^ 1u, abort_flag, p.status, p.wait_ns);
              if (__shfl_sync(0xffffffffu, ok ? 1 : 0, 0) == 0) {
                aborted = true;
                break;
              }
            }
            tc_fence_after();
            const uint32_t aslot = tmem + lane_base + kACol0 + j * 64 + t * 32;
            if (active) {
              tc_st16(aslot, qa);  // the first quarter's store overlaps the second's lookups
              Dec::lookup_q(hd, 1, qb, p.mul);
              tc_st16(aslot + 16, qb);
              tc_wait_st_keep(qa);
              tc_wait_st_keep(qb);
            }
            if (h == Dec::kHalves - 1) {  // this stage's shared memory is no longer read
              __syncwarp();
              if (lane == 0) mbar_arrive(smem_u32(empty + s));
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(afull + j));
          }
        }
        if (aborted) break;
      }
      // epilogue
      const int db = rd.i;
      ok = wait_or_abort(smem_u32(dfull + db), rd.ph, abort_flag, p.status, p.wait_ns);
      if (__shfl_sync(0xffffffffu, ok ? 1 : 0, 0) == 0) break;
      tc_fence_after();
      const uint32_t dcol = tmem + lane_base + db * kDCols;
      if (p.pair) {
        // chunks of 16 tokens of unit row `row`, chunk c to the warp pair
        // (set, t) with c % (2 kSets) == 2 set + t; gate tile at columns
        // 0 .. MT-1, up tile at MT .. 2MT-1
        const int col = u * kTcRows + row;  // K index of the down projection
        const int nt0 = p.gt.nt0[gi];
        uint8_t* dst = p.act_out + tc_bact_off((int64_t)nt0 * kNTile, col, p.out_kb, p.ntstride);
#pragma unroll 1
        for (int c = 2 * set + t; c < MT / 16; c += 2 * kSets) {
          const int tok0 = 16 * c;
          if (tok0 >= ntok) break;  // warp-uniform
          uint32_t g[16], v[16];
          tc_ld16(dcol + tok0, g);
          tc_wait_ld16(g);
          tc_ld16(dcol + MT + tok0, v);
          tc_wait_ld16(v);
          if (p.ks > 1) {
            // partial sums of this slice (MT = 32); splitk_silu_kernel adds
            // the slices up after this launch (a kernel boundary orders them
            // without fences)
            float* mine = p.part + (int64_t)item * (2 * kTcRows * 32) + row * 32 + tok0;
#pragma unroll
            for (int n = 0; n < 16; n += 4) {
              *reinterpret_cast<float4*>(mine + n) =
                  make_float4(__uint_as_float(g[n]), __uint_as_float(g[n + 1]), __uint_as_float(g[n + 2]),
                              __uint_as_float(g[n + 3]));
              *reinterpret_cast<float4*>(mine + kTcRows * 32 + n) =
                  make_float4(__uint_as_float(v[n]), __uint_as_float(v[n + 1]), __uint_as_float(v[n + 2]),
                              __uint_as_float(v[n + 3]));
            }
            continue;
          }
#pragma unroll
          for (int n = 0; n < 16; ++n) {
            const int tok = tok0 + n;
            if (tok < ntok) {
              const float val = silu_f(__uint_as_float(g[n])) * __uint_as_float(v[n]);
              *reinterpret_cast<uint16_t*>(dst + (int64_t)(tok >> 3) * (p.out_kb * 16) + (tok & 7) * 16) =
                  f32_to_act<Dec::kBF16>(val);
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(dempty + db));
      } else {
        // tile t of the unit, chunks of 16 tokens c with c % kSets == set
        if (t < ntl) {
          const int hrow = (2 * u + t) * kTcRows + row;
          float* y = p.y_out + (item % p.ks) * p.y_sstride + (int64_t)p.gt.slot0[gi] * p.y_ld + hrow;
#pragma unroll 1
          for (int c = set; c < MT / 16; c += kSets) {
            const int tok0 = 16 * c;
            if (tok0 >= ntok) break;  // warp-uniform
            uint32_t v[16];
            tc_ld16(dcol + t * MT + tok0, v);
            tc_wait_ld16(v);
#pragma unroll
            for (int n = 0; n < 16; ++n)
              if (tok0 + n < ntok) y[(int64_t)(tok0 + n) * p.y_ld] = __uint_as_float(v[n]);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(dempty + db));
      }
      rd.next(kDBufs);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols));
  }
}

// Host-side launch: ring depth from the shared-memory budget, one persistent
// CTA per resident slot.
template <class Dec, int MT>
inline cudaError_t launch_tc(TcParams p, int num_sms, cudaStream_t stream) {
  const int budget = (tc_ctas_per_sm<MT>() == 2 ? kTcRingBudget : kTcRingBudgetWide) - tc_table_bytes<Dec>();
  const int stage = tc_stage_bytes<Dec, MT>(p);
  const int xstage = tc_xstage_bytes<Dec, MT>();
  // LUT formats: as many activation stages as weight stages.  The producer
  // issues a block's activations right after its weights and an activation
  // stage is freed only by the block's MMAs, so the activation ring bounds
  // the weight bytes in flight; with small (2- and 3-bit) weight stages a
  // shallow activation ring would starve the loads.
  const int depth = std::min(kTcMaxStages, budget / (stage + xstage));
  p.stages = std::max(2, depth);
  if (p.wait_ns == 0) p.wait_ns = wait_limit_ns();
  p.xstages = xstage ? p.stages : 0;
  const int smem = tc_smem_bytes<Dec, MT>(p);
  auto kern = tc_mm_kernel<Dec, MT>;
  // per (instantiation, device): shared-memory attribute and CTAs per SM
  // (zero: not yet computed)
  static std::mutex mu;
  static int cached_smem[kMaxDevices], cached_per_sm[kMaxDevices];
  const int dev = cache_device();
  int per_sm;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 0 || cached_smem[dev] != smem) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return e;
      // Two CTAs per SM share its 512 tensor-memory columns when their shared
      // memory fits (the occupancy query can answer one here, as it models a
      // smaller shared-memory carveout); a CTA that finds no SM slot free just
      // starts later and finds the work counter exhausted.
      int dev = 0, smem_sm = 0, nb = 0;
      e = cudaGetDevice(&dev);
      if (e == cudaSuccess) e = cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
      if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, tc_threads<MT>(), smem);
      if (e != cudaSuccess) return e;
      const int want = tc_ctas_per_sm<MT>();
      per_sm = want > 1 && (nb >= want || want * (smem + 1024) <= smem_sm) ? want : 1;
      e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
      if (e != cudaSuccess) return e;
      if (dev >= 0) {
        cached_per_sm[dev] = per_sm;
        cached_smem[dev] = smem;
      }
    } else {
      per_sm = cached_per_sm[dev];
    }
  }
  kern<<<num_sms * per_sm, tc_threads<MT>(), smem, stream>>>(p);
  return cudaGetLastError();
}

// ------------------------------------------------------ small-batch GEMV --
// A single-token batch (kGemvMaxTokens) leaves the tensor core nothing to
// amortise: every weight is used once, and the tcgen05 pipeline's fill and
// drain dominate.  tc_gemv_kernel reads the same TC-layout buffer straight
// from global memory, one thread per weight row, decodes it with the
// format's policy and accumulates in fp32 on the FMA pipe.  A CTA is one
// (token group, 128-row tile, K slice); each thread keeps a ring of
// tc_gemv_pf() pieces of its row in flight.  It writes exactly what
// tc_mm_kernel writes (gate/up partial sums for splitk_silu_kernel, or fp32
// output rows per K slice), so the kernels around it are unchanged.
constexpr int kGemvMaxCols = 2048;  // columns per CTA (K slice): bounds the staged fp32 activations

template <bool BF16>
__device__ __forceinline__ float2 tc_unpack2(uint32_t v) {
  if constexpr (BF16) {
    return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xFFFF0000u));
  } else {
    return __half22float2(*reinterpret_cast<const __half2*>(&v));
  }
}

// Accumulates 16 pairs (32 consecutive columns starting at column c of the
// slice) into acc[NT]; xs holds the chunk's tokens as fp32 [token][column].
template <bool BF16, int NT>
__device__ __forceinline__ void tc_gemv_fma32(const uint32_t (&o)[16], const float* __restrict__ xs, int ldx, int c,
                                              float2 (&acc)[NT]) {
#pragma unroll
  for (int i = 0; i < 16; i += 2) {
    const float2 w0 = tc_unpack2<BF16>(o[i]);
    const float2 w1 = tc_unpack2<BF16>(o[i + 1]);
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const float4 x = *reinterpret_cast<const float4*>(xs + t * ldx + c + 2 * i);
      acc[t].x = fmaf(w0.x, x.x, acc[t].x);
      acc[t].y = fmaf(w0.y, x.y, acc[t].y);
      acc[t].x = fmaf(w1.x, x.z, acc[t].x);
      acc[t].y = fmaf(w1.y, x.w, acc[t].y);
    }
  }
}

template <class Dec>
__device__ __forceinline__ void tc_gemv_ptrs(const TcParams& p, const uint8_t* base, int b, int pt, uint32_t tab,
                                             TcPtrs& pp) {
#pragma unroll
  for (int k = 0; k < 3; ++k) pp.p[k] = base + p.plane_off[k] + ((int64_t)b * p.ntiles + pt) * p.piece[k];
  pp.tab = tab;
}

// Halves (64-column pieces; dense: 32-column blocks) a GEMV thread keeps in
// flight: four, or two when a half's registers exceed 64 bytes.
template <class Dec>
__host__ __device__ constexpr int tc_gemv_pf() {
  return Dec::kDense ? 4 : (Dec::kHalfBytes <= 64 ? 4 : 2);
}
template <bool BF16>
struct TcDenseBlk {
  uint4 v[4];
};

// Loads piece i (half i % kHalves of block b0 + i / kHalves; dense: block
// b0 + i) of this thread's row.
template <class Dec, class U>
__device__ __forceinline__ void tc_gemv_load(const TcParams& p, const uint8_t* base, int pt, int b0, int i, int row,
                                             uint32_t tab, U& u) {
  const int kh = Dec::kDense ? 1 : Dec::kHalves;
  TcPtrs pp;
  tc_gemv_ptrs<Dec>(p, base, b0 + i / kh, pt, tab, pp);
  if constexpr (Dec::kDense) {
#pragma unroll
    for (int k = 0; k < 4; ++k) u.v[k] = *reinterpret_cast<const uint4*>(pp.p[0] + (k * kTcRows + row) * 16);
  } else {
    Dec::load_half(pp, row, i % kh, u);
  }
}

// One pass over the slice's n pieces for NT tokens of the chunk: a register
// ring of PF pieces, refilled as each is consumed, so a thread has PF loads
// in flight.  ring[] arrives with pieces 0 .. PF-1 already requested.
template <class Dec, int NT, class U>
__device__ __forceinline__ void tc_gemv_pass(const TcParams& p, const uint8_t* base, int pt, int b0, int n, int row,
                                             uint32_t tab, const float* xs, int ldx, U (&ring)[tc_gemv_pf<Dec>()],
                                             float (&out)[NT]) {
  constexpr int PF = tc_gemv_pf<Dec>();
  constexpr int W = Dec::kDense ? Dec::KB : 64;  // columns per piece
  float2 acc[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) acc[t] = make_float2(0.f, 0.f);
  for (int i0 = 0; i0 < n; i0 += PF) {
#pragma unroll
    for (int j = 0; j < PF; ++j) {
      const int i = i0 + j;
      if (i < n) {
        if constexpr (Dec::kDense) {
          uint32_t o[16];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            o[4 * k] = ring[j].v[k].x; o[4 * k + 1] = ring[j].v[k].y;
            o[4 * k + 2] = ring[j].v[k].z; o[4 * k + 3] = ring[j].v[k].w;
          }
          tc_gemv_fma32<Dec::kBF16, NT>(o, xs, ldx, i * W, acc);
        } else {
#pragma unroll
          for (int qq = 0; qq < 2; ++qq) {
            uint32_t o[16];
            Dec::lookup_q(ring[j], qq, o, p.mul);
            tc_gemv_fma32<Dec::kBF16, NT>(o, xs, ldx, i * W + 32 * qq, acc);
          }
        }
        if (i + PF < n) tc_gemv_load<Dec>(p, base, pt, b0, i + PF, row, tab, ring[j]);
      }
    }
  }
#pragma unroll
  for (int t = 0; t < NT; ++t) out[t] = acc[t].x + acc[t].y;
}

// NT: tokens accumulated per pass over the weights; a group of more tokens
// takes several passes.
template <class Dec, int NT>
__global__ void __launch_bounds__(kTcRows, 4) tc_gemv_kernel(const TcParams p) {
  constexpr int KB = Dec::KB;
  constexpr int PF = tc_gemv_pf<Dec>();
  using U = typename std::conditional<Dec::kDense, TcDenseBlk<Dec::kBF16>, typename Dec::Half>::type;
  const int64_t cta = blockIdx.x;
  const int s = (int)(cta % p.ks);
  const int pt = (int)((cta / p.ks) % p.ntiles);
  const int gi = (int)(cta / ((int64_t)p.ks * p.ntiles));
  // the group's entries are in bounds for every gi below the group bound, so
  // they load together with the group count
  const int ng = *p.gt.n_groups;
  const int ntok = p.gt.ntok[gi], nt0 = p.gt.nt0[gi], ex = p.gt.expert[gi], slot0 = p.gt.slot0[gi];
  if (gi >= ng) return;
  const int b0 = s * p.bps, b1 = min(p.nblocks, b0 + p.bps);
  if (b0 >= b1) return;
  const int row = threadIdx.x;
  const uint8_t* base = p.w + (int64_t)ex * p.wstride;
  const int n = (b1 - b0) * (Dec::kDense ? 1 : Dec::kHalves);  // pieces of the slice
  extern __shared__ __align__(16) uint8_t gsm[];
  uint32_t tab = 0;
  if constexpr (Dec::kR8) tab = smem_u32(gsm) + (row & 31) * 4;
  float* xs = reinterpret_cast<float*>(gsm + tc_table_bytes<Dec>());  // [NT][ldx]
  const int ncols = (b1 - b0) * KB, ldx = ncols;
  for (int c0 = 0; c0 < ntok; c0 += NT) {
    const int nc = min(NT, ntok - c0);
    // the slice's first pieces are in flight while the activations are staged
    U ring[PF];
#pragma unroll
    for (int j = 0; j < PF; ++j)
      if (j < n) tc_gemv_load<Dec>(p, base, pt, b0, j, row, tab, ring[j]);
    if (c0 == 0) {
      if constexpr (Dec::kR8) tc_fill_r8_table(reinterpret_cast<uint32_t*>(gsm), p.r8_table);
    }
    __syncthreads();  // the previous pass's reads of xs are done
    for (int i = threadIdx.x; i < NT * ncols; i += blockDim.x) {
      const int t = i / ncols, col = i - t * ncols;
      float v = 0.f;
      if (t < nc) {
        const uint16_t h = *reinterpret_cast<const uint16_t*>(
            p.bin + tc_bact_off((int64_t)nt0 * kNTile + c0 + t, b0 * KB + col, KB, p.ntstride));
        v = act_to_f32<Dec::kBF16>(h);
      }
      xs[t * ldx + col] = v;
    }
    __syncthreads();  // xs (and the R8 table) complete
    float out[NT];
    tc_gemv_pass<Dec, NT>(p, base, pt, b0, n, row, tab, xs, ldx, ring, out);
    if (p.pair) {
      // partial sums [item = (group, unit, slice)][gate | up][row][token]
      const int64_t item = ((int64_t)gi * p.units + (pt >> 1)) * p.ks + s;
      float* dst = p.part + item * (2 * kTcRows * 32) + (pt & 1) * (kTcRows * 32) + row * 32 + c0;
#pragma unroll
      for (int t = 0; t < NT; ++t)
        if (t < nc) dst[t] = out[t];
    } else {
      float* y = p.y_out + (int64_t)s * p.y_sstride + (int64_t)(slot0 + c0) * p.y_ld + pt * kTcRows + row;
#pragma unroll
      for (int t = 0; t < NT; ++t)
        if (t < nc) y[(int64_t)t * p.y_ld] = out[t];
    }
  }
}

// Host launch of the GEMV: one CTA per (group bound, tile, K slice), one
// token per pass (the GEMV serves single-token batches).
template <class Dec, int NT>
inline cudaError_t launch_tc_gemv_nt(const TcParams& p, int64_t group_bound, cudaStream_t stream) {
  const int64_t ctas = group_bound * p.ntiles * p.ks;
  const int smem = tc_table_bytes<Dec>() + NT * p.bps * Dec::KB * 4;
  if (p.bps * Dec::KB > kGemvMaxCols || ctas <= 0 || ctas > (1LL << 31) - 1) return cudaErrorInvalidValue;
  auto kern = tc_gemv_kernel<Dec, NT>;
  static std::mutex mu;
  static int cached[kMaxDevices];  // shared-memory attribute set per device (zero: not yet)
  const int dev = cache_device();
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 0 || cached[dev] < smem) {
      const int attr = std::max(smem, 48 * 1024);
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, attr);
      if (e != cudaSuccess) return e;
      if (dev >= 0) cached[dev] = attr;
    }
  }
  kern<<<(unsigned)ctas, kTcRows, smem, stream>>>(p);
  return cudaGetLastError();
}
template <class Dec>
inline cudaError_t launch_tc_gemv(const TcParams& p, int64_t group_bound, cudaStream_t stream) {
  return launch_tc_gemv_nt<Dec, 1>(p, group_bound, stream);
}

// One CTA per (physical tile, block), one thread per row: decode the row's
// block straight from global memory with the matmul's decode policy and
// write it to out[rows][cols] (the diagnostic dequantisation of the layout).
struct TcDequantArgs {
  const uint8_t* w;
  int64_t off[3];
  int piece[3];
  int ntiles;
  int64_t cols;
  int paired;
  uint16_t* out;
  TcMul mul;
  const uint16_t* r8_table;
};

template <class Dec>
__global__ void __launch_bounds__(kTcRows) tc_dequant_kernel(const TcDequantArgs a) {
  const int pt = blockIdx.x, b = blockIdx.y, row = threadIdx.x;
  const int64_t r = logical_tile(pt, a.ntiles, a.paired != 0) * kTcRows + row;
  uint4* dst = reinterpret_cast<uint4*>(a.out + r * a.cols + (int64_t)b * Dec::KB);
  TcPtrs pp;
#pragma unroll
  for (int k = 0; k < 3; ++k) pp.p[k] = a.w + a.off[k] + ((int64_t)b * a.ntiles + pt) * a.piece[k];
  pp.tab = 0;
  if constexpr (Dec::kR8) {
    __shared__ uint32_t tab[256 * 32];
    tc_fill_r8_table(tab, a.r8_table);
    __syncthreads();
    pp.tab = smem_u32(tab) + (threadIdx.x & 31) * 4;
  }
  if constexpr (Dec::kDense) {
#pragma unroll
    for (int u = 0; u < Dec::KB / 8; ++u)
      dst[u] = *reinterpret_cast<const uint4*>(pp.p[0] + (u * kTcRows + row) * 16);
  } else {
#pragma unroll
    for (int h = 0; h < Dec::kHalves; ++h) {
      typename Dec::Half d;
      Dec::load_half(pp, row, h, d);
#pragma unroll
      for (int qq = 0; qq < 2; ++qq) {
        uint32_t o[16];
        Dec::lookup_q(d, qq, o, a.mul);
#pragma unroll
        for (int i = 0; i < 4; ++i) dst[h * 8 + qq * 4 + i] = make_uint4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
      }
    }
  }
}

// Launchers of a decode family over its table blocks (32, 64, 128 columns)
// and token-group widths (32, 128).
// group_tokens: 32 or 128 for the tcgen05 matmul with that token-group
// width, 1 for the small-batch GEMV (groups of up to 32 tokens).
template <template <int> class DecT>
inline cudaError_t launch_tc_family(int group, int group_tokens, const TcParams& p, int sms, cudaStream_t stream) {
  if (group_tokens == 1) {
    switch (group) {
      case 32: return launch_tc_gemv<DecT<32>>(p, p.gemv_groups, stream);
      case 64: return launch_tc_gemv<DecT<64>>(p, p.gemv_groups, stream);
      case 128: return launch_tc_gemv<DecT<128>>(p, p.gemv_groups, stream);
    }
    return cudaErrorInvalidValue;
  }
  const bool wide = group_tokens == 128;
  if (group_tokens != 32 && !wide) return cudaErrorInvalidValue;
  switch (group) {
    case 32: return wide ? launch_tc<DecT<32>, 128>(p, sms, stream) : launch_tc<DecT<32>, 32>(p, sms, stream);
    case 64: return wide ? launch_tc<DecT<64>, 128>(p, sms, stream) : launch_tc<DecT<64>, 32>(p, sms, stream);
    case 128: return wide ? launch_tc<DecT<128>, 128>(p, sms, stream) : launch_tc<DecT<128>, 32>(p, sms, stream);
  }
  return cudaErrorInvalidValue;
}
template <class Dec>
inline cudaError_t tc_dequant_launch(const TcDequantArgs& a, int64_t nblocks, cudaStream_t stream) {
  tc_dequant_kernel<Dec><<<dim3((unsigned)a.ntiles, (unsigned)nblocks), kTcRows, 0, stream>>>(a);
  return cudaGetLastError();
}
template <template <int> class DecT>
inline cudaError_t tc_dequant_family(int group, const TcDequantArgs& a, int64_t nblocks, cudaStream_t stream) {
  switch (group) {
    case 32: return tc_dequant_launch<DecT<32>>(a, nblocks, stream);
    case 64: return tc_dequant_launch<DecT<64>>(a, nblocks, stream);
    case 128: return tc_dequant_launch<DecT<128>>(a, nblocks, stream);
  }
  return cudaErrorInvalidValue;
}

// Per-family entry points, each in its own translation unit.
cudaError_t launch_tc_b2(int group, int group_tokens, const TcParams& p, int sms, cudaStream_t stream);
cudaError_t launch_tc_b3(int group, int group_tokens, const TcParams& p, int sms, cudaStream_t stream);
cudaError_t launch_tc_nested(int group, int group_tokens, const TcParams& p, int sms, cudaStream_t stream);
cudaError_t launch_tc_r8(int group_tokens, const TcParams& p, int sms, cudaStream_t stream);
cudaError_t dequant_tc_b2(int group, const TcDequantArgs& a, int64_t nblocks, cudaStream_t stream);
cudaError_t dequant_tc_b3(int group, const TcDequantArgs& a, int64_t nblocks, cudaStream_t stream);
cudaError_t dequant_tc_nested(int group, const TcDequantArgs& a, int64_t nblocks, cudaStream_t stream);
cudaError_t dequant_tc_r8(const TcDequantArgs& a, int64_t nblocks, cudaStream_t stream);

}  // namespace blut
