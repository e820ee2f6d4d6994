"""The reference-facing operator API on the GPU: LUTFusedMoEMethod (vLLM plugin),
fused_lut_moe, lut_gemv, DeepseekV2MoE_LUT and the fused router."""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import blut_oracle as O
from tests._helpers import bf16_tensor, check_layer, cuda, routing_inputs, to_u16
from tests.golden.make_golden import small_layer_indices

from block_lut_b200.cuda_lut_gemv import lut_gemv
from block_lut_b200.fast_moe import fused_lut_moe
from block_lut_b200.fused_kernel import fused_lut_gemv
from block_lut_b200.moe import router

pytestmark = pytest.mark.gpu


def _small_r8_layer(golden):
    s = golden("apply_small.npz")
    w13, w2 = small_layer_indices(int(s["idx_seed"]), 8, 256, 128)
    layer = SimpleNamespace(w13_weight=cuda(w13), w2_weight=cuda(w2), w13_absmax=bf16_tensor(s["a13"]),
                            w2_absmax=bf16_tensor(s["a2"]), _codebook=bf16_tensor(s["table"]))
    return s, layer


def test_quant_method_apply_matches_reference_golden(golden):
    from block_lut_b200.quant_method import LUTConfig, LUTFusedMoEMethod
    s, layer = _small_r8_layer(golden)
    method = LUTFusedMoEMethod(LUTConfig(code_type="BLOCKLUT"))
    for T in (2, 8):
        out = method.apply(layer, bf16_tensor(s[f"x{T}"]), bf16_tensor(s[f"tw{T}"]), cuda(s[f"ti{T}"]).long())
        assert out.dtype == torch.bfloat16 and out.shape == (T, 256)
        ref = O.bf16_to_f32(s[f"out{T}"])
        o = out.float().cpu().numpy()
        assert np.abs(o - ref).max() <= 2e-3 and O.rel_l2(o, ref) <= 1e-2
        # same call through fused_lut_moe (fast_moe.py:30) gives the same bits
        f = fused_lut_moe(bf16_tensor(s[f"x{T}"]), cuda(s[f"ti{T}"]), bf16_tensor(s[f"tw{T}"]), layer.w13_weight,
                          layer.w13_absmax, layer.w2_weight, layer.w2_absmax, layer._codebook)
        assert torch.equal(f, out)


def test_fused_expert_compute_one_expert(golden):
    # fast_moe._fused_expert_compute (fast_moe.py:14-27): one expert, one token
    from block_lut_b200.fast_moe import _fused_expert_compute
    s, layer = _small_r8_layer(golden)
    table, a13, a2 = s["table"], s["a13"], s["a2"]
    w13, w2 = layer.w13_weight.cpu().numpy(), layer.w2_weight.cpu().numpy()
    e = 3
    x = bf16_tensor(s["x2"])[0]
    y = _fused_expert_compute(x, layer.w13_weight[e], layer.w2_weight[e], layer._codebook, layer.w13_absmax[e],
                              layer.w2_absmax[e])
    assert y.dtype == torch.bfloat16 and tuple(y.shape) == (256,)
    W13 = [O.bf16_to_f32(O.dequant_r(w13[e].reshape(-1), a13[e], table, 128)).reshape(256, 256)]
    W2 = [O.bf16_to_f32(O.dequant_r(w2[e].reshape(-1), a2[e], table, 128)).reshape(256, 128)]
    ref = O.moe_forward(x.float().cpu().numpy()[None], np.zeros((1, 1), dtype=np.int64),
                        np.ones((1, 1), dtype=np.float32), W13, W2, act_dtype="bf16")
    check_layer(y[None], ref, torch.bfloat16, "_fused_expert_compute")


def test_expert_wrapper_on_lut_linear():
    # moe_layer.LUTMoEExpertWrapper (moe_layer.py:32-143)
    from block_lut_b200.moe_layer import LUTMoEExpertWrapper
    from block_lut_b200.quantizer import LUTQuantizer
    H, I = 256, 128
    rng = np.random.Generator(np.random.PCG64(31))
    w13 = O.f32_to_bf16(O.student_t_weights(rng, (2 * I, H)))
    w2 = O.f32_to_bf16(O.student_t_weights(rng, (H, I)))
    tab = O.f32_to_bf16(np.sort(rng.uniform(-1, 1, 256)).astype(np.float32))
    wr = LUTMoEExpertWrapper(H, I, LUTQuantizer(block_size=128))
    wr.set_weights(bf16_tensor(w13), bf16_tensor(w2), bf16_tensor(tab))
    x = cuda(O.f32_to_bf16(O.rms_activations(rng, 5, H))).view(torch.bfloat16)
    for name, w, rows, cols in (("w13", w13, 2 * I, H), ("w2", w2, H, I)):
        idx, am = O.encode_r(w.reshape(-1), tab, 128)
        W = O.bf16_to_f32(O.dequant_r(idx, am, tab, 128)).reshape(rows, cols)
        assert np.array_equal(to_u16(wr.get_weight(name)), O.f32_to_bf16(W))
        xin = x if name == "w13" else x[:, :I].contiguous()
        y = wr(xin, name)
        assert tuple(y.shape) == (5, rows) and wr._linear[name] is not None
        check_layer(y, xin.double().cpu().numpy() @ W.astype(np.float64).T, torch.bfloat16, f"wrapper {name}")
    wr.set_decompressed(wr.get_weight("w13"), wr.get_weight("w2"))
    assert wr.has_decompressed() and tuple(wr(x, "w13").shape) == (5, 2 * I)
    wr.clear_decompressed()
    assert not wr.has_decompressed()


def test_quant_method_decompress_helpers():
    # _decompress_one / _batch_decompress (quant_method.py:281-308), bit-exact
    from block_lut_b200.quant_method import LUTConfig, LUTFusedMoEMethod
    method = LUTFusedMoEMethod(LUTConfig(code_type="BLOCKLUT"))
    rng = np.random.Generator(np.random.PCG64(12))
    E, rows, cols = 3, 64, 256
    nb = rows * cols // 128
    idx = rng.integers(0, 256, (E, rows, cols), dtype=np.uint8)
    am = O.f32_to_bf16(rng.uniform(0.01, 0.1, (E, nb)).astype(np.float32))
    tab = O.f32_to_bf16(rng.uniform(-1, 1, 256).astype(np.float32))
    one = method._decompress_one(cuda(idx[1]), bf16_tensor(am[1]), bf16_tensor(tab))
    assert tuple(one.shape) == (rows * cols,)
    assert np.array_equal(to_u16(one), O.dequant_r(idx[1].reshape(-1), am[1], tab, 128))
    every = method._batch_decompress(cuda(idx), bf16_tensor(am), bf16_tensor(tab))
    assert tuple(every.shape) == idx.shape
    ref = np.stack([O.dequant_r(idx[e].reshape(-1), am[e], tab, 128).reshape(rows, cols) for e in range(E)])
    assert np.array_equal(to_u16(every), ref)


def test_quant_method_create_weights_format_b():
    from block_lut_b200.formats import LUTFormat, encode
    from block_lut_b200.quant_method import LUTConfig, LUTFusedMoEMethod
    cfg = LUTConfig.from_config({"quant_method": "lut", "code_type": "BLOCKLUT", "codebook_scope": "row_block",
                                 "index_bits": 4, "lut_block": 64})
    assert cfg.lut_format() == LUTFormat("b", 4, 64)
    method = LUTFusedMoEMethod(cfg)
    layer = torch.nn.Module()
    E, H, I = 3, 256, 128
    method.create_weights(layer, E, H, I, torch.float16)
    assert layer.w13_weight.shape == (E, 2 * I, H // 2) and layer.w13_weight.dtype == torch.uint8
    assert layer.w13_tables.shape == (E, 2 * I, H // 64, 16) and layer.w13_tables.dtype == torch.float16
    rng = np.random.Generator(np.random.PCG64(4))
    W13, W2 = [], []
    for e in range(E):
        a, b = O.student_t_weights(rng, (2 * I, H)), O.student_t_weights(rng, (H, I))
        qa, qb = encode(cuda(a), cfg.lut_format()), encode(cuda(b), cfg.lut_format())
        layer.w13_weight.data[e].copy_(qa.codes)
        layer.w13_tables.data[e].copy_(qa.tables)
        layer.w2_weight.data[e].copy_(qb.codes)
        layer.w2_tables.data[e].copy_(qb.tables)
        W13.append(O.dequant_b(qa.codes.cpu().numpy(), qa.tables.cpu().numpy(), 4, 64).astype(np.float32))
        W2.append(O.dequant_b(qb.codes.cpu().numpy(), qb.tables.cpu().numpy(), 4, 64).astype(np.float32))
    method.process_weights_after_loading(layer)
    x = cuda(O.rms_activations(rng, 5, H).astype(np.float16))
    ids, tw = routing_inputs(rng, 5, E, 2)
    out = method.apply(layer, x, cuda(tw), cuda(ids))
    ref = O.moe_forward(x.float().cpu().numpy(), ids, tw, W13, W2, act_dtype="f16")
    check_layer(out, ref, torch.float16, "quant_method format b")

    # release_canonical: the same layer, its canonical parameters freed once tiled
    cfg2 = LUTConfig.from_config({"quant_method": "lut", "code_type": "BLOCKLUT", "codebook_scope": "row_block",
                                  "index_bits": 4, "lut_block": 64, "release_canonical": True})
    m2, layer2 = LUTFusedMoEMethod(cfg2), torch.nn.Module()
    m2.create_weights(layer2, E, H, I, torch.float16)
    for name in ("w13_weight", "w13_tables", "w2_weight", "w2_tables"):
        getattr(layer2, name).data.copy_(getattr(layer, name).data)
    m2.process_weights_after_loading(layer2)
    out2 = m2.apply(layer2, x, cuda(tw), cuda(ids))
    assert torch.equal(out2, out)
    assert layer2.w13_weight.numel() == 0 and layer2.w2_tables.numel() == 0
    # another top-k is served from the kept tiled experts
    ids1, tw1 = routing_inputs(rng, 5, E, 1)
    out1 = m2.apply(layer2, x, cuda(tw1), cuda(ids1))
    check_layer(out1, O.moe_forward(x.float().cpu().numpy(), ids1, tw1, W13, W2, act_dtype="f16"), torch.float16,
                "quant_method released, top-1")


@pytest.mark.parametrize("m,k", [(2816, 2048), (2048, 1408), (64, 1000)])
def test_lut_gemv(m, k):
    rng = np.random.Generator(np.random.PCG64(m + k))
    idx = rng.integers(0, 256, (m, k), dtype=np.uint8)
    nb = (m * k + 127) // 128
    am = O.f32_to_bf16(rng.uniform(0.01, 0.1, nb).astype(np.float32))
    tab = O.f32_to_bf16(np.sort(rng.uniform(-1, 1, 256)).astype(np.float32))
    x = O.f32_to_bf16(rng.standard_normal(k).astype(np.float32))
    y = lut_gemv(bf16_tensor(x), cuda(idx), bf16_tensor(tab), bf16_tensor(am))
    # cuda_lut_gemv.py:48-58 keeps the fp32 product (no bf16 rounding of the weight)
    blk = np.minimum(np.arange(m * k) // 128, nb - 1).reshape(m, k)
    w = O.bf16_to_f32(tab)[idx].astype(np.float64) * O.bf16_to_f32(am)[blk].astype(np.float64)
    ref = w @ O.bf16_to_f32(x).astype(np.float64)
    rb = O.round_to(ref.astype(np.float32), "bf16")
    o = y.float().cpu().numpy()
    ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(rb), 1e-30))) - 7)
    assert (np.abs(o - rb) <= ulp).all()
    # fused_kernel.fused_lut_gemv (fused_kernel.py:13-46) is the same kernel
    f = fused_lut_gemv(bf16_tensor(x), cuda(idx), bf16_tensor(tab), bf16_tensor(am))
    assert torch.equal(f.view(torch.int16), y.view(torch.int16))


def test_router_kernel_against_oracle(golden):
    rng = np.random.Generator(np.random.PCG64(13))
    T, H, E, k = 32, 2048, 60, 4
    x = cuda(O.rms_activations(rng, T, H).astype(np.float16))
    w = cuda((rng.standard_normal((E + 1, H)) * 0.02).astype(np.float16))
    ids, tw, sg = router(x, w, k, shared_gate=True)
    logits = x.float().cpu().numpy().astype(np.float64) @ w.float().cpu().numpy().astype(np.float64).T
    rids, rtw = O.routing(logits[:, :E], k)
    srt = np.sort(logits[:, :E], axis=1)
    keep = srt[:, -k] - srt[:, -k - 1] > 1e-4
    assert np.array_equal(ids.cpu().numpy()[keep], rids[keep])
    np.testing.assert_allclose(tw.cpu().numpy()[keep], rtw[keep], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(sg.cpu().numpy(), 1 / (1 + np.exp(-logits[:, E])), rtol=1e-5, atol=1e-6)


def test_deepseek_v2_moe_lut_forward():
    """A per-block format named by the LUT config (Format B 4-bit g64)."""
    from block_lut_b200.formats import LUTFormat
    from block_lut_b200.moe_layer import DeepseekV2MoE_LUT, _routing
    cfg = SimpleNamespace(hidden_size=256, moe_intermediate_size=128, n_routed_experts=6, num_experts_per_tok=2,
                          n_shared_experts=1, norm_topk_prob=False)
    lut_cfg = SimpleNamespace(lut_format=lambda: LUTFormat("b", 4, 64))
    m = DeepseekV2MoE_LUT(cfg, lut_config=lut_cfg, dtype=torch.float16)
    rng = np.random.Generator(np.random.PCG64(6))
    w13 = torch.from_numpy(O.student_t_weights(rng, (6, 256, 256)))
    w2 = torch.from_numpy(O.student_t_weights(rng, (6, 256, 128)))
    sgu = torch.from_numpy(O.student_t_weights(rng, (256, 256))).half()
    sd = torch.from_numpy(O.student_t_weights(rng, (256, 128))).half()
    with torch.no_grad():
        m.gate.weight.copy_(torch.from_numpy((rng.standard_normal((6, 256)) * 0.1).astype(np.float16)))
        m.shared_gate_up.weight.copy_(sgu)
        m.shared_down.weight.copy_(sd)
    m.quantize_expert_weights(w13, w2)
    x = cuda(O.rms_activations(rng, 10, 256).astype(np.float16)).reshape(2, 5, 256)
    out = m(x)
    assert out.shape == x.shape
    # oracle: same encoded weights, the reference's _routing on fp64 logits
    xn = x.reshape(10, 256).float().cpu().numpy().astype(np.float64)
    logits = xn @ m.gate.weight.detach().float().cpu().numpy().astype(np.float64).T
    ids, tw = O.routing(logits, 2)
    tw_ref, ids_ref = _routing(torch.from_numpy(logits), 2)
    assert np.array_equal(ids_ref.numpy(), ids)
    ex = m._moe.experts
    from block_lut_b200.formats import encode
    W13 = [O.dequant_b(*[t.cpu().numpy() for t in (q.codes, q.tables)], 4, 64).astype(np.float32)
           for q in (encode(w13[e].cuda(), LUTFormat("b", 4, 64)) for e in range(6))]
    W2 = [O.dequant_b(*[t.cpu().numpy() for t in (q.codes, q.tables)], 4, 64).astype(np.float32)
          for q in (encode(w2[e].cuda(), LUTFormat("b", 4, 64)) for e in range(6))]
    h = xn @ sgu.double().numpy().T
    a = O.round_to((O.silu(h[:, :128]) * h[:, 128:]).astype(np.float32), "f16").astype(np.float64)
    ref = O.moe_forward(xn, ids, tw, W13, W2, act_dtype="f16") + a @ sd.double().numpy().T
    assert ex.num_experts == 6
    check_layer(out.reshape(10, 256), ref, torch.float16, "DeepseekV2MoE_LUT")


@pytest.mark.parametrize("codebook", ["loaded", "trained"])
def test_deepseek_v2_moe_lut_blocklut_as_patched(codebook, tmp_path):
    """The reference's own format, driven the way vllm_lut/patcher.py drives
    the block: a LUT_MoE_vLLMConfig-like config (code_type, lut_path,
    lut_tier), the codebook loaded from ``blocklut_256.npy`` or trained on the
    expert weights, then ``quantize_expert_weights(w13, w2)`` and a forward.
    Checked against the float64 oracle on the experts' own BlockLUT weights."""
    from block_lut_b200.moe_layer import DeepseekV2MoE_LUT
    E, H, I, ns, k, T = 6, 256, 128, 2, 2, 12
    cfg = SimpleNamespace(hidden_size=H, moe_intermediate_size=I, n_routed_experts=E, num_experts_per_tok=k,
                          n_shared_experts=ns, norm_topk_prob=False, num_hidden_layers=27)
    lut_cfg = SimpleNamespace(code_type="BLOCKLUT", lut_path=str(tmp_path), lut_tier=0,
                              enable_progressive_loading=False)
    rng = np.random.Generator(np.random.PCG64(41))
    if codebook == "loaded":
        np.save(tmp_path / "blocklut_256.npy", np.sort(rng.uniform(-1, 1, 256)).astype(np.float32))
    m = DeepseekV2MoE_LUT(cfg, lut_config=lut_cfg)
    assert m.load_codebook(str(tmp_path)) == (codebook == "loaded")
    w13 = torch.from_numpy(O.student_t_weights(rng, (E, 2 * I, H))).to(torch.bfloat16)
    w2 = torch.from_numpy(O.student_t_weights(rng, (E, H, I))).to(torch.bfloat16)
    si = I * ns
    sgu = torch.from_numpy(O.student_t_weights(rng, (2 * si, H))).to(torch.bfloat16)
    sd = torch.from_numpy(O.student_t_weights(rng, (H, si))).to(torch.bfloat16)
    with torch.no_grad():
        m.gate.weight.copy_(torch.from_numpy((rng.standard_normal((E, H)) * 0.1).astype(np.float32)))
        m.shared_gate_up.weight.copy_(sgu)
        m.shared_down.weight.copy_(sd)
    assert m.shared_gate_up.weight.shape == (2 * si, H) and m.shared_down.weight.shape == (H, si)
    m.quantize_expert_weights(w13.cuda(), w2.cuda())
    assert len(m.experts) == E and m._codebook.dtype == torch.bfloat16 and m._codebook.numel() == 256
    assert m._moe.experts.fmt.kind == "r8"
    x = torch.from_numpy(O.rms_activations(rng, T, H).astype(np.float32)).to(torch.bfloat16).cuda()
    out = m(x.reshape(2, T // 2, H))
    assert out.shape == (2, T // 2, H) and out.dtype == torch.bfloat16
    # oracle: each expert's BlockLUT weights as stored by its wrapper, dequantised on the CPU
    cb = m._codebook.cpu().view(torch.int16).numpy().view(np.uint16)

    def deq(ex, name, rows, cols):
        idx = getattr(ex, f"{name}_indices").reshape(-1).cpu().numpy()
        am = getattr(ex, f"{name}_absmax").reshape(-1).cpu().view(torch.int16).numpy().view(np.uint16)
        return O.bf16_to_f32(O.dequant_r(idx, am, cb, 128, 0)).reshape(rows, cols)
    W13 = [deq(ex, "w13", 2 * I, H) for ex in m.experts]
    W2 = [deq(ex, "w2", H, I) for ex in m.experts]
    # the wrappers' bf16 weights are the same values (decompress_blocklut on the GPU)
    assert np.array_equal(m.experts[0].get_weight("w13").float().cpu().numpy(), W13[0])
    xn = x.float().cpu().numpy().astype(np.float64)
    gw = m.gate.weight.detach().float().cpu().numpy().astype(np.float64)
    logits = xn @ gw.T
    ids, tw = O.routing(logits, k)
    srt = np.sort(logits, axis=1)
    keep = srt[:, -k] - srt[:, -k - 1] > 1e-4
    assert keep.sum() >= T // 2
    h = xn @ sgu.double().numpy().T
    a = O.round_to((O.silu(h[:, :si]) * h[:, si:]).astype(np.float32), "bf16").astype(np.float64)
    ref = O.moe_forward(xn, ids, tw, W13, W2, act_dtype="bf16") + a @ sd.double().numpy().T
    check_layer(out.reshape(T, H)[torch.from_numpy(keep).cuda()], ref[keep], torch.bfloat16,
                f"DeepseekV2MoE_LUT BlockLUT ({codebook} codebook)")
