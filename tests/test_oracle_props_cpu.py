"""Properties of the oracle's per-block formats (Format B and NestedLUT 2+2).

The reference has no implementation, test or vector for these formats, so
their oracle cannot be pinned to reference outputs.  These tests pin it to
what the format's definition requires instead, at any size:

* the code stream is LSB-first per row (two 4-bit indices per byte, element
  0 in the low nibble, the convention of the reference's bit-plane files,
  runtime/model_offload.py:753-756) and packs/unpacks losslessly;
* every (row, block) table is fp16 and sorted, and every code is the first
  nearest entry of its block's table;
* the Lloyd iterations never do worse than the uniform grid they start from;
* NestedLUT's coarse tier is exactly the 2-bit Format B encoding, its full
  tier looks up fp16(coarse[c] + refine[c][r]) with the residual code the
  first nearest of the four candidates, and it has a smaller error than the
  coarse tier.
"""
import numpy as np
import pytest

from oracle import blut_oracle as O


def _weights(seed, n=8, k=512):
    rng = np.random.Generator(np.random.PCG64(seed))
    return O.student_t_weights(rng, (n, k)).astype(np.float32)


@pytest.mark.parametrize("bits", [2, 3, 4])
def test_pack_codes_round_trip_and_bit_order(bits):
    rng = np.random.Generator(np.random.PCG64(bits))
    codes = rng.integers(0, 1 << bits, size=(5, 64), dtype=np.uint8)
    packed = O.pack_codes(codes, bits)
    assert packed.shape == (5, 64 * bits // 8)
    assert np.array_equal(O.unpack_codes(packed, bits, 64), codes)
    # element k occupies bits [k*bits, (k+1)*bits) of the row, LSB first
    stream = np.unpackbits(packed, axis=1, bitorder="little")
    for k in (0, 1, 2, 63):
        val = sum(int(stream[0, k * bits + j]) << j for j in range(bits))
        assert val == codes[0, k]
    if bits == 4:  # two indices per byte, element 0 in the low nibble
        assert np.array_equal(packed & 0xF, codes[:, 0::2]) and np.array_equal(packed >> 4, codes[:, 1::2])


def _check_tables_and_codes(v, tables, codes):
    """tables sorted fp16; each code the first index of the minimum |v - t| (float32)."""
    assert tables.dtype == np.float16
    assert np.all(np.diff(tables.astype(np.float32), axis=-1) >= 0)
    t = tables.astype(np.float32)
    d = np.abs(v[..., :, None] - t[..., None, :]).astype(np.float32)
    dmin = d.min(axis=-1)
    picked = np.take_along_axis(d, codes[..., None].astype(np.int64), axis=-1)[..., 0]
    assert np.array_equal(picked, dmin)
    # no lower index reaches the same distance
    first = np.argmax(d == dmin[..., None], axis=-1)
    assert np.array_equal(first, codes)


def _uniform_grid_mse(v, n_cent):
    """Error of the Lloyd start: the uniform grid over each block's range, in fp16."""
    lo, hi = v.min(axis=-1), v.max(axis=-1)
    frac = ((2 * np.arange(n_cent) + 1) / np.float32(2 * n_cent)).astype(np.float32)
    grid = (lo[..., None] + ((hi - lo)[..., None] * frac)).astype(np.float16).astype(np.float32)
    q = np.take_along_axis(grid, O._nearest(v, grid), axis=-1)
    return ((v - q) ** 2).mean(axis=-1)


@pytest.mark.parametrize("group", [32, 64, 128])
@pytest.mark.parametrize("bits", [2, 3, 4])
def test_encode_b_tables_codes_and_lloyd_gain(bits, group):
    w = _weights(10 * bits + group)
    n, k = w.shape
    packed, tables = O.encode_b(w, bits, group)
    assert tables.shape == (n, k // group, 1 << bits)
    v = w.reshape(n, k // group, group)
    codes = O.unpack_codes(packed, bits, k).reshape(v.shape)
    _check_tables_and_codes(v, tables, codes)
    deq = O.dequant_b(packed, tables, bits, group).astype(np.float32)
    assert np.array_equal(deq.reshape(v.shape), np.take_along_axis(tables.astype(np.float32), codes.astype(np.int64), -1))
    mse = ((v - deq.reshape(v.shape)) ** 2).mean(axis=-1)
    start = _uniform_grid_mse(v, 1 << bits)
    # Lloyd does not increase a block's error (fp32 arithmetic, fp16 tables: a tiny slack)
    assert np.all(mse <= start * (1 + 1e-3) + 1e-12)
    assert mse.mean() < start.mean()
    # the quantiser's error falls as the code grows
    if bits > 2:
        p2, t2 = O.encode_b(w, bits - 1, group)
        assert mse.mean() < ((w - O.dequant_b(p2, t2, bits - 1, group).astype(np.float32)) ** 2).mean()


@pytest.mark.parametrize("bits", [2, 4])
def test_encode_b_constant_and_zero_blocks_are_exact(bits):
    w = _weights(3, n=3, k=192)
    w[0, 64:128] = 0.0
    w[1, :64] = np.float32(np.float16(0.0123))
    w[2, 128:] = np.float32(np.float16(-3.5))
    packed, tables = O.encode_b(w, bits, 64)
    deq = O.dequant_b(packed, tables, bits, 64).astype(np.float32)
    assert np.array_equal(deq[0, 64:128], w[0, 64:128])
    assert np.array_equal(deq[1, :64], w[1, :64])
    assert np.array_equal(deq[2, 128:], w[2, 128:])


def test_lloyd_ignores_masked_values():
    v = _weights(4, n=4, k=128).reshape(4, 2, 64)
    rng = np.random.Generator(np.random.PCG64(5))
    mask = rng.random(v.shape) < 0.6
    a = O.lloyd_blocks(v, 4, mask=mask)
    b = O.lloyd_blocks(np.where(mask, v, np.float32(7.0)), 4, mask=mask)
    assert np.array_equal(a, b)


@pytest.mark.parametrize("group", [32, 64, 128])
def test_encode_nested_tiers(group):
    w = _weights(20 + group)
    n, k = w.shape
    nb = k // group
    cp, rp, ct, rt = O.encode_nested(w, group)
    # the coarse tier is the 2-bit Format B encoding of the same weights
    p2, t2 = O.encode_b(w, 2, group)
    assert np.array_equal(cp, p2) and np.array_equal(ct, t2)
    v = w.reshape(n, nb, group)
    c = O.unpack_codes(cp, 2, k).reshape(v.shape).astype(np.int64)
    r = O.unpack_codes(rp, 2, k).reshape(v.shape).astype(np.int64)
    _check_tables_and_codes(v, ct, c)
    # refinement tables: fp16, sorted per coarse code, zero for coarse codes no value took
    rt4 = rt.reshape(n, nb, 4, 4)
    assert rt.dtype == np.float16 and np.all(np.diff(rt4.astype(np.float32), axis=-1) >= 0)
    used = np.stack([(c == i).any(axis=-1) for i in range(4)], axis=-1)
    assert np.all(rt4[~used] == 0)
    # full tier: fp16(coarse[c] + refine[c][r]), the residual code the first nearest candidate
    comb = O.nested_combined_table(ct, rt).astype(np.float32).reshape(n, nb, 4, 4)
    cand = comb[np.arange(n)[:, None, None], np.arange(nb)[None, :, None], c]  # [n, nb, g, 4]
    d = np.abs(v[..., None] - cand).astype(np.float32)
    dmin = d.min(axis=-1)
    assert np.array_equal(np.argmax(d == dmin[..., None], axis=-1), r)
    full = O.dequant_nested(cp, rp, ct, rt, group).astype(np.float32).reshape(v.shape)
    assert np.array_equal(full, np.take_along_axis(cand, r[..., None], axis=-1)[..., 0])
    coarse = O.dequant_nested(cp, rp, ct, rt, group, coarse_only=True).astype(np.float32).reshape(v.shape)
    assert np.array_equal(coarse, np.take_along_axis(ct.astype(np.float32), c, axis=-1))
    assert ((v - full) ** 2).mean() < 0.5 * ((v - coarse) ** 2).mean()
