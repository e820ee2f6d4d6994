"""The checkpoint converter on the GPU.

A small bf16 Hugging Face checkpoint (2 layers of 4 experts, two shards, with
shared-expert, router and fp32 tensors that must pass through) is converted
to Format R, Format B and NestedLUT. Each encoded tensor must equal the oracle
encoders bit for bit, and everything else must be copied unchanged. The
converted files are then loaded the way vLLM's expert mapping loads them,
through ``LUTFusedMoEMethod`` (absmax from the written ``lut_absmax.npz``),
and the layer runs against the oracle.
"""
import json

import numpy as np
import pytest
import torch
from safetensors.torch import load_file, save_file

from oracle import blut_oracle as O
from tests._helpers import check_layer, cuda, routing_inputs, to_u16

from block_lut_b200 import convert_checkpoint as CC
from block_lut_b200.quant_method import LUTConfig, LUTFusedMoEMethod

pytestmark = pytest.mark.gpu

L, E, H, I = 2, 4, 256, 128
SHARDS = ("model-00001-of-00002.safetensors", "model-00002-of-00002.safetensors")


def _stem(layer, e, proj):
    return f"model.layers.{layer}.mlp.experts.{e}.{proj}_proj"


def _name(layer, e, proj):
    return _stem(layer, e, proj) + ".weight"


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    src = tmp_path_factory.mktemp("src")
    rng = np.random.Generator(np.random.PCG64(21))
    bf = lambda shape: torch.from_numpy(O.student_t_weights(rng, shape)).to(torch.bfloat16)  # noqa: E731
    shards = [{}, {}]
    for layer in range(L):
        s = shards[layer]
        for e in range(E):
            for proj, shape in (("gate", (I, H)), ("up", (I, H)), ("down", (H, I))):
                s[_name(layer, e, proj)] = bf(shape)
        s[f"model.layers.{layer}.mlp.shared_expert.gate_proj.weight"] = bf((64, H))
        s[f"model.layers.{layer}.mlp.gate.weight"] = bf((E, H))
    # routed-expert tensors that are not bf16 ``.weight`` tensors are copied
    shards[0]["model.layers.0.mlp.experts.e_score_correction.weight"] = torch.zeros(E, dtype=torch.float32)
    shards[1]["model.norm.weight"] = torch.ones(H, dtype=torch.float32)
    wm = {}
    for fname, part in zip(SHARDS, shards):
        save_file(part, str(src / fname))
        wm.update({k: fname for k in part})
    (src / CC.INDEX_NAME).write_text(json.dumps({"metadata": {"total_size": 0}, "weight_map": wm}))
    (src / "config.json").write_text(json.dumps({"model_type": "qwen2_moe", "num_experts": E}))
    np.save(src / "blocklut_256.npy", np.linspace(-1, 1, 256, dtype=np.float32))
    tensors = {k: v for part in shards for k, v in part.items()}
    return src, tensors


def _converted(out):
    conv = {}
    for f in sorted(out.glob("model-*_lut.safetensors")):
        conv.update(load_file(str(f)))
    return conv


def _check_index(out, tensors, extra=()):
    index = json.loads((out / CC.INDEX_NAME).read_text())["weight_map"]
    want = set(tensors)
    for k in tensors:
        if CC.should_encode(k, tensors[k].dtype):
            want |= {k[:-len(".weight")] + s for s in extra}
    assert set(index) == want
    assert all(v.endswith("_lut.safetensors") for v in index.values())


def _layer_inputs(seed, dtype):
    rng = np.random.Generator(np.random.PCG64(seed))
    x = O.rms_activations(rng, 6, H)
    xt = cuda(O.f32_to_bf16(x)).view(torch.bfloat16) if dtype == torch.bfloat16 else cuda(x.astype(np.float16))
    ids, tw = routing_inputs(rng, 6, E, 2)
    return xt, ids, tw


def test_format_r_conversion_bit_exact_and_loads(ckpt, tmp_path):
    src, tensors = ckpt
    out = tmp_path / "out"
    assert CC.main(["--model", str(src), "--output", str(out), "--write_quant_config"]) == 0
    table = to_u16(torch.from_numpy(np.load(src / "blocklut_256.npy")).to(torch.bfloat16))
    conv = _converted(out)
    absmax = np.load(out / CC.ABSMAX_NAME)
    assert set(conv) == set(tensors)
    for name, w in tensors.items():
        if CC.should_encode(name, w.dtype):
            idx, am = O.encode_r(to_u16(w), table, 128)
            assert conv[name].dtype == torch.uint8 and conv[name].shape == w.shape
            assert np.array_equal(conv[name].numpy().reshape(-1), idx), name
            assert absmax[name].dtype == np.float32 and np.array_equal(O.f32_to_bf16(absmax[name]), am), name
        else:
            assert conv[name].dtype == w.dtype and torch.equal(conv[name], w), name
    assert sorted(absmax.files) == sorted(k for k in tensors if CC.should_encode(k, tensors[k].dtype))
    _check_index(out, tensors)
    assert (out / "blocklut_256.npy").exists()

    # load layer 1 as vLLM would (gate rows, then up rows) and run it
    cfg = json.loads((out / "config.json").read_text())["quantization_config"]
    method = LUTFusedMoEMethod(LUTConfig.from_config(cfg))
    layer = torch.nn.Module()
    method.create_weights(layer, E, H, I, torch.bfloat16)
    layer.layer_id = 1
    W13, W2 = [], []
    for e in range(E):
        i13 = torch.cat([conv[_name(1, e, "gate")], conv[_name(1, e, "up")]])
        layer.w13_weight.data[e].copy_(i13)
        layer.w2_weight.data[e].copy_(conv[_name(1, e, "down")])
        a13 = np.concatenate([absmax[_name(1, e, "gate")], absmax[_name(1, e, "up")]])
        W13.append(O.bf16_to_f32(O.dequant_r(i13.numpy().reshape(-1), O.f32_to_bf16(a13), table, 128)).reshape(2 * I, H))
        W2.append(O.bf16_to_f32(O.dequant_r(conv[_name(1, e, "down")].numpy().reshape(-1),
                                            O.f32_to_bf16(absmax[_name(1, e, "down")]), table, 128)).reshape(H, I))
    method.process_weights_after_loading(layer)
    assert np.array_equal(to_u16(layer._codebook), table)
    x, ids, tw = _layer_inputs(5, torch.bfloat16)
    y = method.apply(layer, x, cuda(tw), cuda(ids))
    ref = O.moe_forward(x.float().cpu().numpy(), ids, tw, W13, W2, act_dtype="bf16")
    check_layer(y, ref, torch.bfloat16, "converted Format R layer")


@pytest.mark.parametrize("argv", [["--format", "b", "--bits", "4", "--group", "64"],
                                  ["--format", "b", "--bits", "2", "--group", "128"],
                                  ["--format", "nested", "--group", "64"]])
def test_format_b_conversion_bit_exact_and_loads(ckpt, tmp_path, argv):
    src, tensors = ckpt
    out = tmp_path / "out"
    assert CC.main(["--model", str(src), "--output", str(out)] + argv) == 0
    fmt = CC.format_of(CC.parse_args(["--model", str(src)] + argv))
    nested = fmt.kind == "nested"
    extra = (".tables", ".residual", ".refine") if nested else (".tables",)
    conv = _converted(out)
    for name, w in tensors.items():
        if not CC.should_encode(name, w.dtype):
            assert torch.equal(conv[name], w), name
            continue
        stem = name[:-len(".weight")]
        wf = w.float().numpy()
        if nested:
            want = dict(zip(("", ".residual", ".tables", ".refine"), O.encode_nested(wf, fmt.group)))
        else:
            want = dict(zip(("", ".tables"), O.encode_b(wf, fmt.bits, fmt.group)))
        for suffix, ref in want.items():
            got = conv[name if suffix == "" else stem + suffix].numpy()
            assert got.dtype == ref.dtype and np.array_equal(got.view(np.uint8), ref.view(np.uint8)), name + suffix
    _check_index(out, tensors, extra)
    assert not (out / CC.ABSMAX_NAME).exists()

    cfg = json.loads((out / "config.json").read_text())["quantization_config"]
    assert cfg["codebook_scope"] == "row_block"
    method = LUTFusedMoEMethod(LUTConfig.from_config(cfg))
    assert method.fmt == fmt
    layer = torch.nn.Module()
    method.create_weights(layer, E, H, I, torch.float16)
    cat = lambda e, s: torch.cat([conv[_stem(0, e, "gate") + s], conv[_stem(0, e, "up") + s]])  # noqa: E731
    W13, W2 = [], []
    for e in range(E):
        down = _stem(0, e, "down")
        parts = ((".weight", "weight"), (".tables", "tables")) + \
            (((".residual", "residual"), (".refine", "refine")) if nested else ())
        for suffix, p in parts:
            getattr(layer, f"w13_{p}").data[e].copy_(cat(e, suffix))
            getattr(layer, f"w2_{p}").data[e].copy_(conv[down + suffix])
        if nested:
            order = (".weight", ".residual", ".tables", ".refine")
            W13.append(O.dequant_nested(*(cat(e, s).numpy() for s in order), fmt.group).astype(np.float32))
            W2.append(O.dequant_nested(*(conv[down + s].numpy() for s in order), fmt.group).astype(np.float32))
        else:
            W13.append(O.dequant_b(cat(e, ".weight").numpy(), cat(e, ".tables").numpy(), fmt.bits,
                                   fmt.group).astype(np.float32))
            W2.append(O.dequant_b(conv[down + ".weight"].numpy(), conv[down + ".tables"].numpy(), fmt.bits,
                                  fmt.group).astype(np.float32))
    method.process_weights_after_loading(layer)
    x, ids, tw = _layer_inputs(6, torch.float16)
    y = method.apply(layer, x, cuda(tw), cuda(ids))
    ref = O.moe_forward(x.float().cpu().numpy(), ids, tw, W13, W2, act_dtype="f16")
    check_layer(y, ref, torch.float16, f"converted {fmt} layer")


@pytest.mark.parametrize("argv", [["--format", "b", "--bits", "4", "--group", "64"],
                                  ["--format", "nested", "--group", "64"]])
def test_from_lut_reencodes_a_format_r_checkpoint(ckpt, tmp_path, argv):
    """Format R checkpoint -> Format B / NestedLUT: each routed-expert weight is
    the Format R dequant (bf16) re-encoded, bit for bit as the oracle does it."""
    src, tensors = ckpt
    r_out, out = tmp_path / "r", tmp_path / "b"
    assert CC.main(["--model", str(src), "--output", str(r_out)]) == 0
    assert CC.main(["--model", str(r_out), "--output", str(out), "--from_lut"] + argv) == 0
    fmt = CC.format_of(CC.parse_args(["--model", str(src)] + argv))
    assert sorted(p.name for p in out.glob("*.safetensors")) == sorted(CC.lut_name(f) for f in SHARDS)
    r_conv, conv = _converted(r_out), _converted(out)
    absmax = np.load(r_out / CC.ABSMAX_NAME)
    table = to_u16(torch.from_numpy(np.load(src / "blocklut_256.npy")).to(torch.bfloat16))
    for name, w in tensors.items():
        if not CC.should_encode(name, w.dtype):
            assert torch.equal(conv[name], w), name
            continue
        deq = O.bf16_to_f32(O.dequant_r(r_conv[name].numpy().reshape(-1), O.f32_to_bf16(absmax[name]), table,
                                        128)).reshape(w.shape)
        stem = name[:-len(".weight")]
        if fmt.kind == "nested":
            want = dict(zip(("", ".residual", ".tables", ".refine"), O.encode_nested(deq, fmt.group)))
        else:
            want = dict(zip(("", ".tables"), O.encode_b(deq, fmt.bits, fmt.group)))
        for suffix, ref in want.items():
            got = conv[name if suffix == "" else stem + suffix].numpy()
            assert np.array_equal(got.view(np.uint8), ref.view(np.uint8)), name + suffix
    cfg = json.loads((out / "config.json").read_text())["quantization_config"]
    assert cfg["codebook_scope"] == "row_block" and cfg["lut_block"] == fmt.group
    with pytest.raises(ValueError):
        CC.main(["--model", str(r_out), "--output", str(tmp_path / "bad"), "--from_lut"])


@pytest.mark.parametrize("bs", [64, 128, 256])
def test_encode_lut_f32_bit_exact(bs):
    """blut_encode_lut_f32 (fast_encode.encode_lut's rule) against the oracle:
    ragged tail, an all-zero block, and block sizes of 64, 128 and 256."""
    from block_lut_b200.fast_encode import encode_lut
    from block_lut_b200.formats import encode_lut_f32
    rng = np.random.Generator(np.random.PCG64(bs))
    cb = O.bf16_to_f32(O.f32_to_bf16(np.sort(rng.standard_normal(256).astype(np.float32)) / 3.0))
    w = O.f32_to_bf16(O.student_t_weights(rng, (bs * 301 + 77,)))
    w[bs * 5:bs * 6] = 0
    idx, am = encode_lut_f32(cuda(w).view(torch.bfloat16), cuda(cb), bs)
    ridx, ram = O.encode_lut_f32(w, cb, bs)
    assert np.array_equal(idx.cpu().numpy(), ridx)
    assert np.array_equal(to_u16(am), ram)
    if bs == 128:  # the drop-in returns CPU tensors, as the reference's does
        i2, a2 = encode_lut(cuda(w).view(torch.bfloat16), cuda(cb))
        assert i2.device.type == "cpu" and a2.device.type == "cpu" and a2.dtype == torch.bfloat16
        assert np.array_equal(i2.numpy(), ridx) and np.array_equal(to_u16(a2), ram)


def test_format_r_conversion_with_the_fast_encoder(ckpt, tmp_path):
    """--encoder fast: convert_model.py's rule (fp32 normalisation against the
    bf16 codebook cast to fp32), bit-exact with the oracle."""
    src, tensors = ckpt
    out = tmp_path / "out"
    assert CC.main(["--model", str(src), "--output", str(out), "--encoder", "fast"]) == 0
    cb = torch.from_numpy(np.load(src / "blocklut_256.npy")).to(torch.bfloat16).float().numpy()
    conv = _converted(out)
    absmax = np.load(out / CC.ABSMAX_NAME)
    n = 0
    for name, w in tensors.items():
        if CC.should_encode(name, w.dtype):
            idx, am = O.encode_lut_f32(to_u16(w), cb, 128)
            assert np.array_equal(conv[name].numpy().reshape(-1), idx), name
            assert np.array_equal(O.f32_to_bf16(absmax[name]), am), name
            n += 1
    assert n == L * E * 3
