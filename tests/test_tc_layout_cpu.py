"""Host-side check of the tcgen05 (BLUT_LAYOUT_TC) bit arrangements.

Random codes are packed into one 64-column half by the layout's documented
rules (csrc/blut_common.cuh: codes4, codes2, codes1, combined tables).  The
byte-permute lookups of each decode policy (csrc/blut_tc.cuh: tc_lut16,
tc_lut8x8, tc_lut4x4) are then emulated, and every fp16 pair they produce
must equal a direct table lookup of its two weights.  This checks, without a
GPU, that the packing rules and the decoders agree.  The GPU tests check the
CUDA packer and decoders themselves bit for bit.
"""
import numpy as np
import pytest

M32 = 0xFFFFFFFF


def prmt(a, b, sel):
    """PTX prmt.b32 default mode, selector nibbles without the sign bit."""
    src = [(a >> (8 * i)) & 0xFF for i in range(4)] + [(b >> (8 * i)) & 0xFF for i in range(4)]
    out = 0
    for k in range(4):
        n = (sel >> (4 * k)) & 0xF
        assert n < 8, "decoders never set the sign-replicate bit"
        out |= src[n] << (8 * k)
    return out


def mulhi(a, b):
    return ((a * b) >> 32) & M32


def words_of(bs):
    return [int.from_bytes(bytes(bs[i:i + 4]), "little") for i in range(0, len(bs), 4)]


def split_table(vals):
    """fp16 table -> (high-byte words, low-byte words) as the tables plane stores them."""
    u = np.asarray(vals, dtype=np.float16).view(np.uint16).astype(np.int64)
    return words_of([int(v) >> 8 for v in u]), words_of([int(v) & 0xFF for v in u])


def pair_ok(word, table, codes, i):
    lo = np.uint16(word & 0xFFFF).view(np.float16)
    hi = np.uint16(word >> 16).view(np.float16)
    t = np.asarray(table, dtype=np.float16)
    return lo.view(np.uint16) == t[codes[2 * i]].view(np.uint16) and hi.view(np.uint16) == t[codes[2 * i + 1]].view(np.uint16)


# ----------------------------------------------------------------- packing --
def pack_codes2(c):
    """codes2: bits 2i..2i+1 of byte j of word w hold weight 16w + 4i + j."""
    out = []
    for w in range(len(c) // 16):
        for j in range(4):
            out.append(sum((int(c[16 * w + 4 * i + j]) & 3) << (2 * i) for i in range(4)))
    return words_of(out)


def pack_codes1(c):
    """codes1: bit 4n + s of word w holds bit 2 of weight
    32w + 16(s >> 1) + 8(n & 1) + (n >> 1) + 4(s & 1)."""
    words = []
    for w in range(len(c) // 32):
        v = 0
        for n in range(8):
            for s in range(4):
                k = 32 * w + 16 * (s >> 1) + 8 * (n & 1) + (n >> 1) + 4 * (s & 1)
                v |= ((int(c[k]) >> 2) & 1) << (4 * n + s)
        words.append(v)
    return words


# -------------------------------------------------------------- decoders ----
def lut16(w, th, tl, sa, sb):
    """tc_lut16: 16-entry lookup of the 8 nibbles of w -> (o0, o1, o2, o3)."""
    s1 = w & 0x77777777
    s2 = (mulhi(w, 1 << 31) & 0x44444444) | 0x32103210
    res = []
    for h in range(2):
        a = mulhi(s1, 1 << 16) if h else s1
        b = mulhi(s2, 1 << 16) if h else s2
        hi = prmt(prmt(th[0], th[1], a), prmt(th[2], th[3], a), b)
        lo = prmt(prmt(tl[0], tl[1], a), prmt(tl[2], tl[3], a), b)
        res += [prmt(lo, hi, sa), prmt(lo, hi, sb)]
    return res  # o0, o1 from nibbles 0-3, o2, o3 from nibbles 4-7


def lut8x8(a, t):
    res = []
    for h in range(2):
        s = mulhi(a, 1 << 16) if h else a
        lo = prmt(t[2], t[3], s)
        hi = prmt(t[0], t[1], s)
        res += [prmt(lo, hi, 0x6240), prmt(lo, hi, 0x7351)]
    return res


def lut4x4(x, th, tl):
    s0 = (x * 0x11 + 0x40404040) & M32
    s1 = (mulhi(x, 0x110000) + 0x4040) & M32
    return [prmt(tl, th, s0), prmt(tl, th, s1)]


def decode_b4(codes, table):
    w = words_of([int(codes[2 * o]) | (int(codes[2 * o + 1]) << 4) for o in range(32)])
    th, tl = split_table(table)
    out = []
    for x in w:
        o = lut16(x, th, tl, 0x5140, 0x7362)
        out += [o[0], o[1], o[2], o[3]]
    return out


def decode_b2(codes, table):
    th, tl = split_table(table)
    out = []
    for x in pack_codes2(codes):
        for g in range(4):
            out += lut4x4((mulhi(x, 1 << (32 - 2 * g)) if g else x) & 0x03030303, th[0], tl[0])
    return out


def decode_b3(codes, table):
    th, tl = split_table(table)
    t = [th[0], th[1], tl[0], tl[1]]
    c2, c1 = pack_codes2(codes), pack_codes1(codes)
    out = [0] * 32
    for q in range(2):  # quarters of 32 weights
        w1 = c1[q]
        ys = [((w1 * 4) & M32) & 0x44444444, ((w1 * 2) & M32) & 0x44444444, w1 & 0x44444444,
              mulhi(w1, 1 << 31) & 0x44444444]
        for half in range(2):
            w2 = c2[2 * q + half]
            a = (w2 & 0x33333333) | ys[2 * half]
            b = (mulhi(w2, 1 << 30) & 0x33333333) | ys[2 * half + 1]
            base = 16 * q + 8 * half
            ra, rb = lut8x8(a, t), lut8x8(b, t)
            for o, idx in zip(ra, (0, 4, 1, 5)):
                out[base + idx] = o
            for o, idx in zip(rb, (2, 6, 3, 7)):
                out[base + idx] = o
    return out


def decode_nested(cc, cr, comb):
    th, tl = split_table(comb)
    wc, wr = pack_codes2(cc), pack_codes2(cr)
    out = [0] * 32
    for v in range(4):
        a = (wr[v] & 0x33333333) | (((wc[v] * 4) & M32) & 0xCCCCCCCC)
        b = (mulhi(wr[v], 1 << 30) & 0x33333333) | (wc[v] & 0xCCCCCCCC)
        for o, idx in zip(lut16(a, th, tl, 0x6240, 0x7351), (0, 4, 1, 5)):
            out[8 * v + idx] = o
        for o, idx in zip(lut16(b, th, tl, 0x6240, 0x7351), (2, 6, 3, 7)):
            out[8 * v + idx] = o
    return out


# ------------------------------------------------------------------- tests --
def _table(rng, n):
    return np.sort(rng.standard_normal(n).astype(np.float16))


@pytest.mark.parametrize("seed", range(4))
def test_b4_b3_b2_lookups_match_the_tables(seed):
    rng = np.random.Generator(np.random.PCG64(seed))
    for bits, dec in ((4, decode_b4), (3, decode_b3), (2, decode_b2)):
        codes = rng.integers(0, 1 << bits, 64)
        table = _table(rng, 1 << bits)
        out = dec(codes, table)
        assert len(out) == 32
        assert all(pair_ok(out[i], table, codes, i) for i in range(32)), f"{bits}-bit decode"


@pytest.mark.parametrize("seed", range(4))
def test_nested_full_tier_lookup_matches_combined_table(seed):
    rng = np.random.Generator(np.random.PCG64(100 + seed))
    cc, cr = rng.integers(0, 4, 64), rng.integers(0, 4, 64)
    coarse, refine = _table(rng, 4), (rng.standard_normal(16) * 0.1).astype(np.float16)
    # combined entry 4c + r = fp16(f32(coarse[c]) + f32(refine[4c + r]))
    comb = (coarse.astype(np.float32).repeat(4) + refine.astype(np.float32)).astype(np.float16)
    out = decode_nested(cc, cr, comb)
    idx = 4 * cc + cr
    assert all(pair_ok(out[i], comb, idx, i) for i in range(32))


def test_codes1_and_codes2_arrangements_are_bijective():
    # every weight of a 32-weight word appears exactly once in codes1, and
    # every weight of a 16-weight word once in codes2
    seen = sorted(16 * (s >> 1) + 8 * (n & 1) + (n >> 1) + 4 * (s & 1) for n in range(8) for s in range(4))
    assert seen == list(range(32))
    assert sorted(4 * i + j for i in range(4) for j in range(4)) == list(range(16))


def test_bf16_products_are_exact_in_fp32():
    """The Format R decode scales each table entry by its absmax with one
    bf16x2 multiply (one rounding of the exact product).  The reference
    computes bf16(f32(t) * f32(s)).  Both agree because the product of two
    bf16 values (8 significant bits each) is exact in fp32 (24 bits), away
    from the fp32 subnormal range."""
    rng = np.random.Generator(np.random.PCG64(7))
    t = rng.standard_normal(200000).astype(np.float32)
    s = (10.0 ** rng.uniform(-12, 4, 200000)).astype(np.float32)
    to_bf16 = lambda v: (np.asarray(v, dtype=np.float32).view(np.uint32) & 0xFFFF0000).view(np.float32)  # noqa: E731
    tb, sb = to_bf16(t), to_bf16(s)
    p32 = tb * sb
    p64 = tb.astype(np.float64) * sb.astype(np.float64)
    normal = np.abs(p64) >= np.finfo(np.float32).tiny
    assert np.array_equal(p32[normal].astype(np.float64), p64[normal])
