"""Parity at the full shapes of the named benchmark configurations, against the
float64 oracle on the same quantised weights (tolerances in
tests/_helpers.check_layer: max-abs 2e-3 and rel-L2 1e-3 for fp16 outputs).

* config 5: ``blut_matmul`` for every N x K of the sweep, b in {2, 3, 4},
  g in {32, 64, 128}, M in {1, 16, 256, 4096} (for M = 4096 a fixed sample of
  output rows is checked);
* config 3: a Qwen3-30B-A3B MoE layer (E 128, I 768, top-8 renormalised)
  routed by the library's router (the top-k over more than 64 experts),
  NestedLUT 2+2 g64, full and coarse-only tiers, batch 64;
* config 4: a DeepSeek-V2-Lite MoE layer (E 64, I 1408, top-6, two shared
  experts as one dense MLP of I 2816, added ungated) over 4096 tokens, which
  runs the 128-token grouped (prefill) matmuls; a fixed sample of tokens is
  checked.

The codes are uniform random and the tables sorted random fp16 per (row,
block): the encoder has its own bit-exact tests, and these check the matmul
and MoE paths at the shapes the configs name.  The oracle's torch
dequantisation used here is checked against the numpy oracle on such random
data in tests/test_torch_ref_cpu.py.
"""
import os

import numpy as np
import pytest
import torch

from oracle import blut_oracle as O
from oracle import blut_torch_ref as R
from tests._helpers import check_layer, cuda, qm_from_numpy

from block_lut_b200.formats import LUTFormat
from block_lut_b200.linear import LUTLinear
from block_lut_b200.moe import LUTExperts, LUTMoELayer, SharedExpert

pytestmark = pytest.mark.gpu

THREADS = os.cpu_count() or 1


def _tables(rng, rows, cols, group, ent, scale=0.02):
    return np.sort((rng.standard_normal((rows, cols // group, ent)) * scale).astype(np.float16), axis=-1)


def _random_b(rng, rows, cols, bits, group):
    packed = rng.integers(0, 256, size=(rows, cols * bits // 8), dtype=np.uint8)
    return {"codes": packed, "tables": _tables(rng, rows, cols, group, 1 << bits)}


def _random_nested(rng, rows, cols, group):
    return {"codes": rng.integers(0, 256, size=(rows, cols // 4), dtype=np.uint8),
            "codes2": rng.integers(0, 256, size=(rows, cols // 4), dtype=np.uint8),
            "tables": _tables(rng, rows, cols, group, 4),
            "tables2": _tables(rng, rows, cols, group, 16, scale=0.004)}


def _deq(fmt, d):
    """Dequantised fp32 weights through the oracle's torch restatement (multi-threaded;
    bit-exact with the numpy oracle's dequant_b / dequant_nested, tests/test_torch_ref_cpu.py)."""
    t = {key: torch.from_numpy(v) for key, v in d.items()}
    rows = d["codes"].shape[0]
    if fmt.kind == "nested":
        cols = d["codes"].shape[1] * 4
        return R.dequant_nested(t["codes"], t["codes2"], t["tables"], t["tables2"], fmt.group, rows, cols,
                                coarse_only=fmt.tier == 1).numpy()
    cols = d["codes"].shape[1] * 8 // fmt.bits
    return R.dequant_b(t["codes"], t["tables"], fmt.bits, fmt.group, rows, cols).numpy()


SWEEP_SHAPES = [(1408, 2048), (2048, 1408), (768, 2048), (2048, 768), (5632, 2048)]


@pytest.mark.parametrize("group", [32, 64, 128])
@pytest.mark.parametrize("bits", [2, 3, 4])
@pytest.mark.parametrize("nk", SWEEP_SHAPES, ids=lambda v: f"{v[0]}x{v[1]}")
def test_config5_matmul_sweep(nk, bits, group):
    n, k = nk
    fmt = LUTFormat("b", bits, group)
    rng = np.random.Generator(np.random.PCG64(n + k + 10 * bits + group))
    d = _random_b(rng, n, k, bits, group)
    lin = LUTLinear(qm_from_numpy(fmt, n, k, d))
    W = _deq(fmt, d).astype(np.float64)
    for m in (1, 16, 256, 4096):
        x = cuda(O.rms_activations(rng, m, k).astype(np.float16))
        y = lin(x)
        rows = np.arange(m) if m <= 256 else np.unique(np.r_[0:32, m - 32:m, rng.integers(0, m, 64)])
        ref = x[torch.from_numpy(rows).cuda()].double().cpu().numpy() @ W.T
        check_layer(y[torch.from_numpy(rows).cuda()], ref, torch.float16, f"{fmt} {n}x{k} m={m}")
    lin.check_status()


def _layer_experts(rng, fmts, E, H, I, make):
    """One set of canonical random experts, tiled once per format (tier)."""
    canon13 = [make(rng, 2 * I, H) for _ in range(E)]
    canon2 = [make(rng, H, I) for _ in range(E)]
    out = {}
    for f in fmts:
        q13 = [qm_from_numpy(f, 2 * I, H, c) for c in canon13]
        q2 = [qm_from_numpy(f, H, I, c) for c in canon2]
        out[f] = LUTExperts.from_quantized(q13, q2)
        del q13, q2
    return out, canon13, canon2


def test_config3_qwen3_layer_router_renorm_nested_tiers():
    E, H, I, k, T, g = 128, 2048, 768, 8, 64, 64
    fmts = [LUTFormat("nested", 4, g, 0), LUTFormat("nested", 4, g, 1)]
    rng = np.random.Generator(np.random.PCG64(3030))
    experts, c13, c2 = _layer_experts(rng, fmts, E, H, I, lambda r, a, b: _random_nested(r, a, b, g))
    rw = (rng.standard_normal((E, H)) * 0.05).astype(np.float16)
    x = cuda(O.rms_activations(rng, T, H).astype(np.float16))
    xn = x.float().cpu().numpy().astype(np.float64)
    logits = xn @ rw.astype(np.float64).T
    ids, tw = O.routing(logits, k, renorm=True)
    srt = np.sort(logits, axis=1)
    keep = srt[:, -k] - srt[:, -k - 1] > 1e-4  # tokens without a near-tie at the k-th expert
    assert keep.sum() >= T * 3 // 4
    for f in fmts:
        assert experts[f].tc, "config 3 runs the tcgen05 path"
        layer = LUTMoELayer(experts[f], k, router_w=cuda(rw), renorm=True)
        out = layer.forward(x)
        layer.check_status()
        ref = O.moe_forward_threaded(xn, ids, tw, lambda e: _deq(f, c13[e]), lambda e: _deq(f, c2[e]),
                                     "f16", THREADS)
        check_layer(out[torch.from_numpy(keep).cuda()], ref[keep], torch.float16,
                    f"qwen3 layer tier {f.tier}")
        # one token at a time: the single-token path, with the top-8 of 128
        # experts and its renormalisation taken inside the gate/up launch
        assert layer.launch_count(1, caller_routing=False) == 3
        for i in np.flatnonzero(keep)[:3]:
            out1 = layer.forward(x[i:i + 1])
            layer.check_status()
            ref1 = O.moe_forward_threaded(xn[i:i + 1], ids[i:i + 1], tw[i:i + 1], lambda e: _deq(f, c13[e]),
                                          lambda e: _deq(f, c2[e]), "f16", THREADS)
            check_layer(out1, ref1, torch.float16, f"qwen3 layer tier {f.tier}, single token {i}")


def test_config4_dsv2_lite_prefill_wide_groups():
    E, H, I, k, T, Is = 64, 2048, 1408, 6, 4096, 2816
    fmt = LUTFormat("b", 4, 64)
    rng = np.random.Generator(np.random.PCG64(4040))
    experts, c13, c2 = _layer_experts(rng, [fmt], E, H, I, lambda r, a, b: _random_b(r, a, b, 4, 64))
    s13 = O.student_t_weights(rng, (2 * Is, H)).astype(np.float16)
    s2 = O.student_t_weights(rng, (H, Is)).astype(np.float16)
    rw = (rng.standard_normal((E, H)) * 0.05).astype(np.float16)
    layer = LUTMoELayer(experts[fmt], k, router_w=cuda(rw), shared=SharedExpert.from_dense(cuda(s13), cuda(s2)),
                        shared_gate_mode=0)
    x = cuda(O.rms_activations(rng, T, H).astype(np.float16))
    out = layer.forward(x)
    layer.check_status()
    # 128-token groups: every expert averages 384 tokens
    assert T * k >= 64 * E
    sample = np.unique(np.r_[0:64, T - 64:T, rng.integers(0, T, 256)])
    xn = x.float().cpu().numpy().astype(np.float64)[sample]
    logits = xn @ rw.astype(np.float64).T
    ids, tw = O.routing(logits, k)
    srt = np.sort(logits, axis=1)
    keep = srt[:, -k] - srt[:, -k - 1] > 1e-4
    assert keep.sum() >= len(sample) * 3 // 4
    ref = O.moe_forward_threaded(xn, ids, tw, lambda e: _deq(fmt, c13[e]), lambda e: _deq(fmt, c2[e]),
                                 "f16", THREADS)
    h = xn @ s13.astype(np.float64).T
    a = O.round_to((O.silu(h[:, :Is]) * h[:, Is:]).astype(np.float32), "f16").astype(np.float64)
    ref += a @ s2.astype(np.float64).T
    rows = torch.from_numpy(sample[keep]).cuda()
    check_layer(out[rows], ref[keep], torch.float16, "dsv2-lite prefill")
