"""Host-side check of the bit-plane recover kernel's index arithmetic
(csrc/blut_bitplane.cu, bitplane_recover_kernel).

The kernel's vector path gives warp c (of n // 1024 chunks) the four runs of
8 indices at 1024c + 256r + 8l for lane l, loading a run as a u32 of the low
section at byte e/2 and a u16 of the mid and high sections at n/2 + e/4 and
3n/4 + e/4; the indices after the last whole chunk go through a per-quad
path. This test rebuilds exactly those loads in numpy and checks four
things: every index is produced once, every load stays inside the tier's
prefix, every vector access is aligned, and the values equal the oracle's
Format R dequant. The GPU test checks the kernel itself."""
import numpy as np
import pytest

from oracle import blut_oracle as O

CHUNK = 1024


def emulate(planes, am, table, n, tier, bs, planes_addr=0, out_addr=0):
    need = {2: n // 2, 1: 3 * n // 4, 0: n}[tier]
    pl = planes[:need]                       # only the tier's prefix exists
    nb = (n + bs - 1) // bs
    vec = n % 8 == 0 and bs % 8 == 0 and planes_addr % 4 == 0 and out_addr % 16 == 0
    nchunk = n // CHUNK if vec else 0
    idx = np.full(n, -1, dtype=np.int64)
    seen = np.zeros(n, dtype=np.int64)
    scale = np.zeros(n, dtype=np.uint16)
    if nchunk:
        c, r, lane = np.meshgrid(np.arange(nchunk), np.arange(4), np.arange(32), indexing="ij")
        e = (c * CHUNK + 256 * r + 8 * lane).reshape(-1)
        lo_off, mid_off, hi_off = e // 2, n // 2 + e // 4, 3 * n // 4 + e // 4
        assert ((planes_addr + lo_off) % 4 == 0).all() and ((2 * e + out_addr) % 16 == 0).all()
        assert (lo_off + 4 <= n // 2).all()
        L = pl[lo_off[:, None] + np.arange(4)].astype(np.uint32) @ (1 << (8 * np.arange(4, dtype=np.uint32)))
        M = np.zeros_like(L)
        H = np.zeros_like(L)
        if tier <= 1:
            assert ((planes_addr + mid_off) % 2 == 0).all() and (mid_off + 2 <= need).all()
            M = pl[mid_off[:, None] + np.arange(2)].astype(np.uint32) @ np.array([1, 256], dtype=np.uint32)
        if tier == 0:
            assert ((planes_addr + hi_off) % 2 == 0).all() and (hi_off + 2 <= need).all()
            H = pl[hi_off[:, None] + np.arange(2)].astype(np.uint32) @ np.array([1, 256], dtype=np.uint32)
        blk = np.minimum(e // bs, nb - 1)
        assert (np.minimum((e + 7) // bs, nb - 1) == blk).all()   # a run never crosses an absmax block
        k = np.arange(8, dtype=np.uint32)
        x = ((L[:, None] >> (4 * k)) & 0xF) | (((M[:, None] >> (2 * k)) & 3) << 4) | \
            (((H[:, None] >> (2 * k)) & 3) << 6)
        pos = e[:, None] + k
        idx[pos] = x
        seen[pos.reshape(-1)] += 1
        scale[pos] = am[blk][:, None]
    q = np.arange(nchunk * (CHUNK // 4), n // 4)
    if q.size:
        assert (2 * q + 1 < n // 2).all()
        l = pl[2 * q].astype(np.uint32) | (pl[2 * q + 1].astype(np.uint32) << 8)
        m = pl[n // 2 + q].astype(np.uint32) if tier <= 1 else np.zeros_like(l)
        h = pl[3 * n // 4 + q].astype(np.uint32) if tier == 0 else np.zeros_like(l)
        for j in range(4):
            i = 4 * q + j
            idx[i] = ((l >> (4 * j)) & 0xF) | (((m >> (2 * j)) & 3) << 4) | (((h >> (2 * j)) & 3) << 6)
            seen[i] += 1
            scale[i] = am[np.minimum(i // bs, nb - 1)]
    assert (seen == 1).all()
    # bf16(table[x] * scale): one rounding of the exact product, as the oracle
    prod = O.bf16_to_f32(table[idx.astype(np.int64)]).astype(np.float64) * O.bf16_to_f32(scale)
    return O.f32_to_bf16(prod.astype(np.float32))


@pytest.mark.parametrize("n,bs", [(4100, 128), (1 << 16, 128), (3088, 96), (2048 + 8, 32), (96, 32), (4, 128),
                                  (65536, 100), (1 << 20, 128)])
@pytest.mark.parametrize("tier", [0, 1, 2])
def test_recover_mapping_covers_bounds_and_values(n, bs, tier):
    rng = np.random.Generator(np.random.PCG64(n + bs + tier))
    idx = rng.integers(0, 256, n, dtype=np.uint8)
    am = O.f32_to_bf16(rng.uniform(0.01, 0.1, (n + bs - 1) // bs).astype(np.float32))
    table = O.f32_to_bf16(rng.uniform(-1, 1, 256).astype(np.float32))
    out = emulate(O.bitplane_pack(idx), am, table, n, tier, bs)
    assert np.array_equal(out, O.dequant_r(idx, am, table, bs, tier))


def test_unaligned_buffers_take_the_quad_path():
    n = 8192
    rng = np.random.Generator(np.random.PCG64(5))
    idx = rng.integers(0, 256, n, dtype=np.uint8)
    am = O.f32_to_bf16(np.full(n // 128, 0.05, dtype=np.float32))
    table = O.f32_to_bf16(rng.uniform(-1, 1, 256).astype(np.float32))
    for planes_addr, out_addr in ((2, 0), (0, 6)):
        out = emulate(O.bitplane_pack(idx), am, table, n, 0, 128, planes_addr, out_addr)
        assert np.array_equal(out, O.dequant_r(idx, am, table, 128, 0))
