"""The CPU oracle against golden vectors recorded from the reference's own code.

Every fixture in tests/golden was produced by tests/golden/make_golden.py,
which runs the reference's ``vllm_lut`` functions on seeded inputs.
"""
import numpy as np
import pytest

from oracle import blut_oracle as O
from tests.golden.make_golden import qwen_layer_weights, sha, small_layer_indices


def test_dequant_kat_bit_exact(golden):
    # vllm_lut/cuda/build_lut_kernel.py:142-198 known-answer test (reference tolerance 0.01; we need exact)
    d = golden("dequant_kat.npz")
    out = O.dequant_r(d["idx"], d["absmax"], d["table"], int(d["block_size"]))
    assert np.array_equal(out, d["expected"])


def test_encode_r_bit_exact(golden):
    # LUTQuantizer.quantize (quantizer.py:243-306) with the shipped Qwen codebook
    e = golden("encode_r.npz")
    idx, am = O.encode_r(e["w"], e["table"], 128)
    assert np.array_equal(idx, e["idx"].reshape(-1))
    assert np.array_equal(am, e["absmax"].reshape(-1))
    deq = O.dequant_r(e["idx"], e["absmax"], e["table"], 128)
    assert np.array_equal(deq.reshape(-1), e["dequant"].reshape(-1))


def test_encode_r_matches_reference_converter(golden):
    # convert_checkpoint.quantize_weight (convert_checkpoint.py:61-104): flat
    # blocks over the whole tensor, zero-padded tail, absmax clamp at 1e-10
    e = golden("convert_r.npz")
    idx, am = O.encode_r(e["w"], e["table"], 128)
    assert e["w"].size % 128 != 0 and int(e["absmax"][0]) == int(O.f32_to_bf16(np.float32(1e-10)))
    assert np.array_equal(idx, e["idx"])
    assert np.array_equal(am, e["absmax"])


def test_nested_reconstruction_matches_reference_additive_rule(golden):
    # evaluation/explore_additive_lut.py:266-276 reconstructs coarse[c] + fine[f]
    # (times absmax, 1 here). The NestedLUT table with refine[c][r] = fine[r]
    # for every c must give the same values from the same two code streams.
    d = golden("additive.npz")
    n, group = d["ic"].size, 64
    coarse_t = np.tile(d["coarse"].astype(np.float16), (1, n // group, 1))
    refine_t = np.tile(np.tile(d["fine"].astype(np.float16), 4), (1, n // group, 1))
    cp = O.pack_codes(d["ic"].reshape(1, n), 2)
    rp = O.pack_codes(d["ifn"].reshape(1, n), 2)
    out = O.dequant_nested(cp, rp, coarse_t, refine_t, group)
    assert np.array_equal(out.astype(np.float32).reshape(-1), d["x"])


def test_bitplane_pack_matches_reference(golden):
    # runtime/model_offload.py:751-758, run from the reference's source
    d = golden("bitplane.npz")
    n = d["idx"].size
    assert n % 32 != 0 and int(d["chunk_sizes"].sum()) == n
    assert np.array_equal(O.bitplane_pack(d["idx"]), d["planes"])
    # each tier's prefix reads back the tier's index (tensor_engine.cpp:505-509,535-547)
    for tier, need in ((2, n // 2), (1, 3 * n // 4), (0, n)):
        assert np.array_equal(O.bitplane_index(d["planes"][:need], n, tier), O.tier_index(d["idx"], tier))


@pytest.mark.parametrize("tier,table", [(1, "mapped64"), (2, "mapped16")])
def test_nested_tiers_bit_exact(golden, tier, table):
    t = golden("tiers.npz")
    out = O.dequant_r(t["idx"], t["absmax"], t[table], 128, tier=tier)
    assert np.array_equal(out, t[f"tier{tier}"])


def test_routing_matches_reference(golden):
    r = golden("routing.npz")
    ids, w = O.routing(r["logits_f32"], 4)
    assert np.array_equal(ids, r["ids_f32"])
    np.testing.assert_allclose(w, r["w_f32"], rtol=0, atol=1e-6)
    # bf16 logits contain exact ties; torch.topk orders tied experts arbitrarily,
    # so compare the selected weights exactly and the id sets per weight value.
    lg = O.bf16_to_f32(r["logits_bf16"])
    ids, w = O.routing(lg, 8)
    ref_w = O.bf16_to_f32(r["w_bf16"])
    assert np.array_equal(O.round_to(w, "bf16"), ref_w)
    for t in range(lg.shape[0]):
        ours = sorted(zip(np.round(lg[t, ids[t]], 6), ids[t]))
        theirs = sorted(zip(np.round(lg[t, r["ids_bf16"][t]], 6), r["ids_bf16"][t]))
        assert [v for v, _ in ours] == [v for v, _ in theirs]
        # the id sets may differ only among experts whose logits tie with the k-th value
        kth = min(v for v, _ in ours)
        assert {i for v, i in ours if v > kth} == {i for v, i in theirs if v > kth}


def _r8_experts(w13, w2, a13, a2, table):
    e_n, two_i, h = w13.shape
    W13 = np.stack([O.bf16_to_f32(O.dequant_r(w13[e].reshape(-1), a13[e], table)).reshape(two_i, h)
                    for e in range(e_n)])
    W2 = np.stack([O.bf16_to_f32(O.dequant_r(w2[e].reshape(-1), a2[e], table)).reshape(h, two_i // 2)
                   for e in range(e_n)])
    return W13, W2


@pytest.mark.parametrize("T", [2, 8])
def test_apply_small_bit_exact(golden, T):
    s = golden("apply_small.npz")
    w13, w2 = small_layer_indices(int(s["idx_seed"]), 8, 256, 128)
    assert sha(w13, w2) == str(s["sha"])
    W13, W2 = _r8_experts(w13, w2, s["a13"], s["a2"], s["table"])
    x = O.bf16_to_f32(s[f"x{T}"])
    tw = O.bf16_to_f32(s[f"tw{T}"])
    out = O.moe_forward_reference_bf16(x, s[f"ti{T}"], tw, W13, W2)
    assert np.array_equal(out, O.bf16_to_f32(s[f"out{T}"]))
    # the fp64 oracle (the CUDA path's rounding points) stays within the bf16 budget of the reference
    ex = O.moe_forward(x, s[f"ti{T}"], tw, W13, W2, act_dtype="bf16")
    assert np.abs(ex - O.bf16_to_f32(s[f"out{T}"])).max() < 2e-3


def test_apply_qwen_shape_bit_exact(golden):
    q = golden("apply_qwen.npz")
    w13, w2, a13, a2, _ = qwen_layer_weights(int(q["seed"]), 60, 2048, 1408)
    assert sha(w13, w2, a13, a2) == str(q["sha"])
    ids = q["ti"]
    W13 = lambda e: O.bf16_to_f32(O.dequant_r(w13[e].reshape(-1), a13[e], q["table"])).reshape(2816, 2048)  # noqa
    W2 = lambda e: O.bf16_to_f32(O.dequant_r(w2[e].reshape(-1), a2[e], q["table"])).reshape(2048, 1408)  # noqa
    out = O.moe_forward_reference_bf16(O.bf16_to_f32(q["x"]), ids, O.bf16_to_f32(q["tw"]), W13, W2)
    ref = O.bf16_to_f32(q["out"])
    # At K=2048 the reference's bf16 F.linear (oneDNN) sums in its own blocked
    # fp32 order, which flips the final bf16 rounding of a few outputs: allow
    # a 1-ulp difference on at most 0.1% of the elements, nothing more.
    ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(ref), 1e-30))) - 7)
    diff = np.abs(out - ref)
    assert (diff <= ulp).all()
    assert (diff > 0).mean() < 1e-3


def _reference_fast_encode_check(w_bf16_u16, codebook_f32, block_size=128):
    """The rule the reference checks its fast GPU encoder against, restated
    with torch on the CPU as fast_encode.py:205-221 writes it: zero-padded
    flat blocks, absmax clamped at 1e-10, normalised = blocks / absmax in
    fp32, argmin over the fp32 codebook."""
    import torch
    w = torch.from_numpy(O.bf16_to_f32(w_bf16_u16))
    n = w.numel()
    nb = (n + block_size - 1) // block_size
    padded = torch.zeros(nb * block_size)
    padded[:n] = w
    blocks = padded.reshape(-1, block_size)
    block_max = blocks.abs().max(dim=1, keepdim=True)[0].clamp(min=1e-10)
    normalized = (blocks / block_max).reshape(-1)[:n]
    cb = torch.from_numpy(np.asarray(codebook_f32, dtype=np.float32))
    idx = (normalized.unsqueeze(1) - cb.unsqueeze(0)).abs().argmin(dim=1).to(torch.uint8)
    return idx.numpy(), block_max.reshape(-1).numpy()


def test_encode_lut_f32_follows_the_reference_fast_encoder_rule():
    # fast_encode.encode_lut (fast_encode.py:22-102) as convert_model.py calls
    # it: a bf16 codebook cast to fp32 (convert_model.py:53-55); a ragged tail
    # and an all-zero block (absmax floor)
    rng = np.random.Generator(np.random.PCG64(11))
    table = O.f32_to_bf16(np.sort(rng.standard_normal(256).astype(np.float32)) / 3.0)
    cb = O.bf16_to_f32(table)
    w = O.f32_to_bf16((rng.standard_t(5, 128 * 37 + 45) * 0.02).astype(np.float32))
    w[128 * 3:128 * 4] = 0
    idx, am = O.encode_lut_f32(w, cb, 128)
    ridx, rmax = _reference_fast_encode_check(w, cb, 128)
    assert np.array_equal(idx, ridx)
    assert np.array_equal(am, O.f32_to_bf16(rmax))
    assert O.bf16_to_f32(am[3]) == O.bf16_to_f32(O.f32_to_bf16(np.float32(1e-10)))


def test_encode_lut_f32_and_quantize_differ_only_by_the_bf16_rounding():
    # The two reference encoders differ where bf16 rounding of the normalised
    # value w / absmax moves it onto a codebook midpoint.  Entries 0.1015625
    # and 0.10253906 are two bf16 steps apart, so their midpoint is itself a
    # bf16 value: a quotient just above it rounds onto it (a tie, which the
    # first index wins) while in fp32 it is nearer the second entry.  Find
    # such a weight for absmax 3.0 and check each oracle's rule there.
    cb = np.array([0.1015625, 0.1015625 + 2 * 2.0 ** -11] + [4.0] * 254, dtype=np.float32)
    cb = O.bf16_to_f32(O.f32_to_bf16(cb))
    table = O.f32_to_bf16(cb)
    amax = np.float32(3.0)
    cand = O.f32_to_bf16(np.linspace(0.29, 0.32, 4000).astype(np.float32))
    q = (O.bf16_to_f32(cand) / amax).astype(np.float32)
    qb = O.bf16_to_f32(O.f32_to_bf16(q))
    near = lambda v: (np.abs(v - cb[1]) < np.abs(v - cb[0])).astype(int)  # noqa: E731
    differ = np.nonzero(near(q) != near(qb))[0]
    assert differ.size > 0
    x = cand[differ[0]]
    w = np.zeros(128, dtype=np.uint16)
    w[0], w[1] = O.f32_to_bf16(amax), x
    f_idx = O.encode_lut_f32(w, cb, 128)[0][1]
    q_idx = O.encode_r(w, table, 128)[0][1]
    assert f_idx == near(q[differ[0:1]])[0] and q_idx == near(qb[differ[0:1]])[0] and f_idx != q_idx
