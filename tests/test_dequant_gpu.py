"""Bit-exact dequantisation and encoding on the GPU against the oracle and the
reference's golden vectors."""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import blut_oracle as O
from tests._helpers import bf16_tensor, cuda, qm_from_numpy, to_u16

from block_lut_b200 import _lib
from block_lut_b200.formats import LUTFormat, QuantizedMatrix, dequant, encode, encode_r
from block_lut_b200.quantizer import LUTQuantizer, decompress_blocklut

pytestmark = pytest.mark.gpu


def test_decompress_kat_golden(golden):
    d = golden("dequant_kat.npz")
    out = decompress_blocklut(cuda(d["idx"]), bf16_tensor(d["absmax"]), bf16_tensor(d["table"]), 128)
    assert np.array_equal(to_u16(out), d["expected"])


def test_quantizer_api_golden(golden):
    e = golden("encode_r.npz")
    q = LUTQuantizer("BLOCKLUT", 128)
    res = q.quantize(bf16_tensor(e["w"]).reshape(96, 384), bf16_tensor(e["table"]))
    assert np.array_equal(res["indices"].numpy(), e["idx"].reshape(-1))
    assert np.array_equal(to_u16(res["absmax"]), e["absmax"].reshape(-1))
    deq = q.decompress(res["indices"], res["absmax"], res["codebook"])
    assert np.array_equal(to_u16(deq), e["dequant"].reshape(-1))


@pytest.mark.parametrize("tier,table", [(1, "mapped64"), (2, "mapped16")])
def test_r8_tiers_golden(golden, tier, table):
    t = golden("tiers.npz")
    n = t["idx"].size
    qm = QuantizedMatrix(LUTFormat("r8", 8, 128, tier), 1, n, cuda(t["idx"].reshape(-1)), bf16_tensor(t[table]),
                         scales=bf16_tensor(t["absmax"]))
    assert np.array_equal(to_u16(dequant(qm)).reshape(-1), t[f"tier{tier}"].reshape(-1))


@pytest.mark.parametrize("n,bs", [(1, 128), (15, 128), (16, 128), (4097, 128), (128 * 33, 128), (1000, 64),
                                  (2048, 32)])
def test_r8_random_shapes(n, bs):
    rng = np.random.Generator(np.random.PCG64(n))
    idx = rng.integers(0, 256, n, dtype=np.uint8)
    am = O.f32_to_bf16(rng.uniform(0.01, 0.1, (n + bs - 1) // bs).astype(np.float32))
    tab = O.f32_to_bf16(rng.uniform(-1, 1, 256).astype(np.float32))
    out = decompress_blocklut(cuda(idx), bf16_tensor(am), bf16_tensor(tab), bs)
    assert np.array_equal(to_u16(out), O.dequant_r(idx, am, tab, bs))


def test_batch_decompress_and_recover():
    rng = np.random.Generator(np.random.PCG64(3))
    E, n = 5, 4096 + 16
    nb = (n + 127) // 128
    idx = rng.integers(0, 256, (E, n), dtype=np.uint8)
    am = O.f32_to_bf16(rng.uniform(0.01, 0.1, (E, nb)).astype(np.float32))
    tab = O.f32_to_bf16(rng.uniform(-1, 1, 256).astype(np.float32))
    out = torch.empty(E, n, dtype=torch.bfloat16, device="cuda")
    ti, ta, tt = cuda(idx), bf16_tensor(am), bf16_tensor(tab)
    _lib.check(_lib.lib().blut_batch_blocklut_decompress(out.data_ptr(), ti.data_ptr(), ta.data_ptr(), tt.data_ptr(),
                                                         E, n, nb, 128, _lib.stream_ptr()))
    ref = np.stack([O.dequant_r(idx[e], am[e], tab, 128) for e in range(E)])
    assert np.array_equal(to_u16(out), ref)
    rec = torch.empty(E * n, dtype=torch.int16, device="cuda")
    _lib.check(_lib.lib().blut_lut_recover(rec.data_ptr(), ti.data_ptr(), tt.data_ptr(), E * n, _lib.stream_ptr()))
    assert np.array_equal(rec.cpu().numpy().view(np.uint16), tab[idx.reshape(-1)])


@pytest.mark.parametrize("bits", [2, 3, 4])
@pytest.mark.parametrize("group", [32, 64, 128])
def test_format_b_dequant_bit_exact(bits, group):
    rng = np.random.Generator(np.random.PCG64(bits * 1000 + group))
    rows, cols = 48, 384
    w = O.student_t_weights(rng, (rows, cols))
    packed, tables = O.encode_b(w, bits, group)
    fmt = LUTFormat("b", bits, group)
    qm = qm_from_numpy(fmt, rows, cols, {"codes": packed, "tables": tables})
    out = dequant(qm).cpu().numpy()
    assert np.array_equal(out.view(np.uint16), O.dequant_b(packed, tables, bits, group).view(np.uint16))


@pytest.mark.parametrize("tier", [0, 1])
@pytest.mark.parametrize("group", [32, 64, 128])
def test_nested_dequant_bit_exact(tier, group):
    rng = np.random.Generator(np.random.PCG64(77 + group))
    rows, cols = 32, 256
    w = O.student_t_weights(rng, (rows, cols))
    cp, rp, ct, rt = O.encode_nested(w, group)
    fmt = LUTFormat("nested", 4, group, tier)
    qm = qm_from_numpy(fmt, rows, cols, {"codes": cp, "codes2": rp, "tables": ct, "tables2": rt})
    out = dequant(qm).cpu().numpy()
    ref = O.dequant_nested(cp, rp, ct, rt, group, coarse_only=tier == 1)
    assert np.array_equal(out.view(np.uint16), ref.view(np.uint16))


@pytest.mark.parametrize("bits", [2, 3, 4])
@pytest.mark.parametrize("group", [32, 64, 128])
def test_gpu_encoder_bit_identical_to_oracle(bits, group):
    rng = np.random.Generator(np.random.PCG64(5 + bits + group))
    rows, cols = 24, 512
    w = O.student_t_weights(rng, (rows, cols))
    qm = encode(cuda(w), LUTFormat("b", bits, group))
    packed, tables = O.encode_b(w, bits, group)
    assert np.array_equal(qm.tables.cpu().numpy().view(np.uint16), tables.view(np.uint16))
    assert np.array_equal(qm.codes.cpu().numpy(), packed)


@pytest.mark.parametrize("group", [32, 64, 128])
def test_gpu_nested_encoder_bit_identical_to_oracle(group):
    rng = np.random.Generator(np.random.PCG64(9 + group))
    rows, cols = 16, 256
    w = O.student_t_weights(rng, (rows, cols))
    qm = encode(cuda(w), LUTFormat("nested", 4, group))
    cp, rp, ct, rt = O.encode_nested(w, group)
    assert np.array_equal(qm.tables.cpu().numpy().view(np.uint16), ct.view(np.uint16))
    assert np.array_equal(qm.tables2.cpu().numpy().view(np.uint16), rt.view(np.uint16))
    assert np.array_equal(qm.codes.cpu().numpy(), cp)
    assert np.array_equal(qm.codes2.cpu().numpy(), rp)


def test_encode_r_padding_tail():
    rng = np.random.Generator(np.random.PCG64(11))
    n = 1000  # not a multiple of the block
    w = O.f32_to_bf16(O.student_t_weights(rng, (n,)))
    tab = O.f32_to_bf16(np.sort(rng.uniform(-1, 1, 256)).astype(np.float32))
    idx, am = encode_r(bf16_tensor(w), bf16_tensor(tab), 128)
    ridx, ram = O.encode_r(w, tab, 128)
    assert np.array_equal(idx.cpu().numpy(), ridx)
    assert np.array_equal(to_u16(am), ram)


def test_dequant_rejects_bad_args():
    fmt = LUTFormat("b", 4, 64)
    d = fmt.desc(16, 100)  # cols not a multiple of the group
    c = _lib.Canon(1 << 20, None, 1 << 20, None, None)
    assert _lib.lib().blut_dequant(C.byref(d), C.byref(c), 1 << 20, None) == _lib.BLUT_ERR_UNSUPPORTED


TILED_FORMATS = [LUTFormat("b", b, g) for b in (2, 3, 4) for g in (32, 64, 128)] + \
    [LUTFormat("nested", 4, g, t) for g in (32, 64, 128) for t in (0, 1)]


@pytest.mark.parametrize("paired", [False, True])
@pytest.mark.parametrize("fmt", TILED_FORMATS, ids=lambda f: f"{f.kind}{f.bits}g{f.group}t{f.tier}")
def test_tiled_layout_lookup_bit_exact(fmt, paired):
    """pack_tiled + the MoE kernels' fragment lookups reproduce the canonical dequant exactly."""
    from block_lut_b200.formats import dequant_tiled, pack_tiled
    rng = np.random.Generator(np.random.PCG64(fmt.bits * 100 + fmt.group + fmt.tier))
    rows, cols = 64, 384
    w = O.student_t_weights(rng, (rows, cols))
    qm = encode(cuda(w), fmt)
    ref = dequant(qm)
    buf, _ = pack_tiled([qm], paired=paired)
    out = dequant_tiled(fmt, rows, cols, buf, paired=paired)
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))


@pytest.mark.parametrize("paired", [False, True])
@pytest.mark.parametrize("group", [32, 64, 128])
@pytest.mark.parametrize("kind,bits,tier", [("b", 4, 0), ("b", 3, 0), ("b", 2, 0), ("nested", 4, 0),
                                            ("nested", 4, 1)])
def test_tc_layout_lookup_bit_exact(kind, bits, tier, group, paired):
    """BLUT_LAYOUT_TC: pack + the tcgen05 matmul's per-row decode reproduce the canonical dequant."""
    from block_lut_b200.formats import dequant_tiled, pack_tiled
    fmt = LUTFormat(kind, bits, group, tier)
    rng = np.random.Generator(np.random.PCG64(500 + group + 7 * bits + tier))
    rows, cols = 512, 384
    qm = encode(cuda(O.student_t_weights(rng, (rows, cols))), fmt)
    buf, _ = pack_tiled([qm], paired=paired, tc=True)
    out = dequant_tiled(fmt, rows, cols, buf, paired=paired, tc=True)
    assert torch.equal(out.view(torch.int16), dequant(qm).view(torch.int16))


@pytest.mark.parametrize("paired", [False, True])
@pytest.mark.parametrize("tier", [0, 1, 2])
def test_tc_layout_r8_lookup_bit_exact(tier, paired):
    """FMT_R8 in the tcgen05 layout: the shared-memory table lookup and the
    bf16x2 absmax multiply reproduce bf16(f32(table[tier(idx)]) * f32(absmax))
    bit for bit, with absmax spanning 1e-12 .. 1e4 and a table holding zeros,
    signed tiny and large values (products stay above the fp32 subnormal
    range, where the reference's fp32-then-bf16 rounding could differ from one
    bf16 rounding)."""
    from block_lut_b200.formats import dequant_tiled, pack_tiled
    rng = np.random.Generator(np.random.PCG64(70 + tier))
    rows, cols = 512, 384
    idx = rng.integers(0, 256, rows * cols, dtype=np.uint8)
    am = O.f32_to_bf16((10.0 ** rng.uniform(-12, 4, rows * cols // 128)).astype(np.float32))
    t = rng.uniform(-1, 1, 256).astype(np.float32)
    t[:8] = [0.0, -0.0, 1e-20, -1e-20, 3e4, -3e4, 1.0, -1.0]
    tab = bf16_tensor(O.f32_to_bf16(t))
    fmt = LUTFormat("r8", 8, 128, tier)
    qm = QuantizedMatrix(fmt, rows, cols, cuda(idx), tab, scales=bf16_tensor(am))
    assert fmt.has_tc_layout(rows, cols, paired)
    buf, _ = pack_tiled([qm], paired=paired, tc=True)
    out = dequant_tiled(fmt, rows, cols, buf, tab, paired=paired, tc=True)
    assert torch.equal(out.view(torch.int16), dequant(qm).view(torch.int16))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_tc_layout_dense_round_trip(dtype):
    from block_lut_b200.formats import dense_matrix, dequant_tiled, pack_tiled
    rng = np.random.Generator(np.random.PCG64(77))
    w = torch.from_numpy(rng.standard_normal((256, 160)).astype(np.float32)).to("cuda", dtype)
    dm = dense_matrix(w)
    for paired in (False, True):
        buf, _ = pack_tiled([dm], paired=paired, tc=True)
        assert torch.equal(dequant_tiled(dm.fmt, 256, 160, buf, paired=paired, tc=True), w)


@pytest.mark.parametrize("tier", [0, 1, 2])
def test_tiled_layout_r8_and_dense(tier):
    from block_lut_b200.formats import dense_matrix, dequant_tiled, pack_tiled
    rng = np.random.Generator(np.random.PCG64(40 + tier))
    rows, cols = 32, 256
    idx = rng.integers(0, 256, rows * cols, dtype=np.uint8)
    am = O.f32_to_bf16(rng.uniform(0.01, 0.1, rows * cols // 128).astype(np.float32))
    tab = bf16_tensor(O.f32_to_bf16(rng.uniform(-1, 1, 256).astype(np.float32)))
    fmt = LUTFormat("r8", 8, 128, tier)
    qm = QuantizedMatrix(fmt, rows, cols, cuda(idx), tab, scales=bf16_tensor(am))
    buf, _ = pack_tiled([qm])
    out = dequant_tiled(fmt, rows, cols, buf, tab)
    assert torch.equal(out.view(torch.int16), dequant(qm).view(torch.int16))
    dm = dense_matrix(torch.from_numpy(rng.standard_normal((rows, cols)).astype(np.float16)).cuda())
    dbuf, _ = pack_tiled([dm])
    assert torch.equal(dequant_tiled(dm.fmt, rows, cols, dbuf), dm.codes)
