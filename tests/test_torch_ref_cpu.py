"""The torch CPU restatement that bench.py times as the reference arm
(``oracle/blut_torch_ref.py``), pinned to the reference's own ``apply`` goldens
(Format R) and to the numpy oracle (Format B, NestedLUT dequantisation)."""
import numpy as np
import pytest
import torch

from oracle import blut_oracle as O
from oracle import blut_torch_ref as R
from tests.golden.make_golden import sha, small_layer_indices


def _bf16(u16):
    return torch.from_numpy(np.ascontiguousarray(u16).view(np.int16)).view(torch.bfloat16)


@pytest.mark.parametrize("T", [2, 8])
def test_apply_format_r_equals_reference_golden(golden, T):
    s = golden("apply_small.npz")
    w13, w2 = small_layer_indices(int(s["idx_seed"]), 8, 256, 128)
    assert sha(w13, w2) == str(s["sha"])
    cb = _bf16(s["table"])
    a13, a2 = _bf16(s["a13"]), _bf16(s["a2"])
    out = R.apply(_bf16(s[f"x{T}"]), _bf16(s[f"tw{T}"]), torch.from_numpy(s[f"ti{T}"]).long(),
                  lambda e: R.dequant_r(torch.from_numpy(w13[e]), a13[e], cb, 256, 256),
                  lambda e: R.dequant_r(torch.from_numpy(w2[e]), a2[e], cb, 256, 128))
    assert out.dtype == torch.bfloat16
    ref = O.bf16_to_f32(s[f"out{T}"])
    o = out.float().numpy()
    # the same torch ops as the reference's apply; oneDNN's blocked sums may
    # flip the last bf16 rounding of a few outputs
    ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(ref), 1e-30))) - 7)
    assert (np.abs(o - ref) <= ulp).all()
    assert (o != ref).mean() < 0.01


@pytest.mark.parametrize("bits", [2, 3, 4])
@pytest.mark.parametrize("group", [32, 64, 128])
def test_dequant_b_matches_oracle(bits, group):
    rng = np.random.Generator(np.random.PCG64(bits * 1000 + group))
    rows, cols = 16, 256
    w = O.student_t_weights(rng, (rows, cols))
    packed, tables = O.encode_b(w, bits, group)
    want = O.dequant_b(packed, tables, bits, group).astype(np.float32)
    got = R.dequant_b(torch.from_numpy(packed), torch.from_numpy(tables).reshape(rows, cols // group, -1), bits,
                      group, rows, cols)
    assert np.array_equal(got.numpy(), want)


@pytest.mark.parametrize("coarse_only", [False, True])
def test_dequant_nested_matches_oracle(coarse_only):
    rng = np.random.Generator(np.random.PCG64(9))
    rows, cols, group = 8, 256, 64
    w = O.student_t_weights(rng, (rows, cols))
    cp, rp, ct, rt = O.encode_nested(w, group)
    want = O.dequant_nested(cp, rp, ct, rt, group, coarse_only=coarse_only).astype(np.float32)
    got = R.dequant_nested(torch.from_numpy(cp), torch.from_numpy(rp),
                           torch.from_numpy(ct).reshape(rows, cols // group, 4),
                           torch.from_numpy(rt).reshape(rows, cols // group, 16), group, rows, cols,
                           coarse_only=coarse_only)
    assert np.array_equal(got.numpy(), want)


def test_apply_format_b_matches_oracle():
    rng = np.random.Generator(np.random.PCG64(3))
    E, H, I, T, k = 4, 128, 64, 6, 2
    mats = []
    for _ in range(E):
        m = {}
        for name, (rows, cols) in (("w13", (2 * I, H)), ("w2", (H, I))):
            packed, tables = O.encode_b(O.student_t_weights(rng, (rows, cols)), 4, 64)
            m[name] = (packed, tables, rows, cols)
        mats.append(m)

    def deq_t(e, name):
        p, t, rows, cols = mats[e][name]
        return R.dequant_b(torch.from_numpy(p), torch.from_numpy(t).reshape(rows, cols // 64, 16), 4, 64, rows, cols)
    x = O.rms_activations(rng, T, H).astype(np.float32)
    ids, tw = O.routing(rng.standard_normal((T, E)).astype(np.float32), k)
    out = R.apply(torch.from_numpy(x), torch.from_numpy(tw), torch.from_numpy(ids).long(),
                  lambda e: deq_t(e, "w13"), lambda e: deq_t(e, "w2"))
    W13 = [deq_t(e, "w13").numpy() for e in range(E)]
    W2 = [deq_t(e, "w2").numpy() for e in range(E)]
    ref = O.moe_forward(x, ids, tw, W13, W2, act_dtype="f32")
    assert np.abs(out.numpy() - ref).max() < 1e-5


@pytest.mark.parametrize("kind", ["b2g128", "b3g32", "b4g64", "nested0", "nested1"])
def test_dequant_on_random_codes_matches_oracle(kind):
    """Uniform random codes and sorted random tables (what the config-shape GPU tests use)."""
    rng = np.random.Generator(np.random.PCG64(7))
    rows, cols = 96, 512

    def tables(group, ent, scale=0.02):
        return np.sort((rng.standard_normal((rows, cols // group, ent)) * scale).astype(np.float16), axis=-1)
    if kind.startswith("nested"):
        coarse_only = kind.endswith("1")
        cc = rng.integers(0, 256, size=(rows, cols // 4), dtype=np.uint8)
        cr = rng.integers(0, 256, size=(rows, cols // 4), dtype=np.uint8)
        ct, rt = tables(64, 4), tables(64, 16, 0.004)
        want = O.dequant_nested(cc, cr, ct, rt, 64, coarse_only=coarse_only).astype(np.float32)
        got = R.dequant_nested(*map(torch.from_numpy, (cc, cr, ct, rt)), 64, rows, cols, coarse_only=coarse_only)
    else:
        bits, group = int(kind[1]), int(kind[3:])
        packed = rng.integers(0, 256, size=(rows, cols * bits // 8), dtype=np.uint8)
        t = tables(group, 1 << bits)
        want = O.dequant_b(packed, t, bits, group).astype(np.float32)
        got = R.dequant_b(torch.from_numpy(packed), torch.from_numpy(t), bits, group, rows, cols)
    assert np.array_equal(got.numpy(), want)
