"""Host logic of the checkpoint converter (block_lut_b200/convert_checkpoint.py):
tensor selection, codebook choice, shard discovery, index remapping, side
files and the quantization_config it writes.  Encoding needs the GPU and is
tested in tests/test_convert_gpu.py; here the converter must refuse to run."""
import json
import os

import numpy as np
import pytest
import torch

from block_lut_b200 import convert_checkpoint as CC


def test_tensor_selection_follows_reference():
    # convert_model.py:91-95: routed experts' bf16 .weight tensors only
    assert CC.should_encode("model.layers.3.mlp.experts.7.gate_proj.weight", torch.bfloat16)
    assert not CC.should_encode("model.layers.3.mlp.experts.7.gate_proj.weight", torch.float16)
    assert not CC.should_encode("model.layers.3.mlp.shared_expert.gate_proj.weight", torch.bfloat16)
    assert not CC.should_encode("model.layers.3.mlp.shared_experts.gate_proj.weight", torch.bfloat16)
    assert not CC.should_encode("model.layers.3.mlp.gate.weight", torch.bfloat16)
    assert not CC.should_encode("model.layers.3.mlp.experts.7.gate_proj.bias", torch.bfloat16)


def test_codebook_choice(tmp_path):
    with pytest.raises(FileNotFoundError):
        CC.codebook_file(str(tmp_path), "BLOCKLUT")
    np.save(tmp_path / "blocklut_256.npy", np.linspace(-1, 1, 256, dtype=np.float32))
    assert CC.codebook_file(str(tmp_path), "BLOCKLUT").endswith("blocklut_256.npy")
    # NESTEDLUT falls back to the BlockLUT table (convert_model.py:48-50)
    assert CC.codebook_file(str(tmp_path), "NESTEDLUT").endswith("blocklut_256.npy")
    np.save(tmp_path / "nested_lut_mapped16.npy", np.zeros(256, dtype=np.uint16))
    assert CC.codebook_file(str(tmp_path), "NESTEDLUT").endswith("nested_lut_mapped16.npy")


def test_shards_index_and_side_files(tmp_path):
    for f in ("model-00002-of-00002.safetensors", "model-00001-of-00002.safetensors", "config.json",
              "tokenizer.model", "blocklut_256.npy", "README.md", CC.INDEX_NAME, "modeling_x.py"):
        (tmp_path / f).write_bytes(b"{}")
    shards = [os.path.basename(f) for f in CC.shard_files(str(tmp_path))]
    assert shards == ["model-00001-of-00002.safetensors", "model-00002-of-00002.safetensors"]
    # the index is rewritten, not copied over (the reference copies it last)
    assert CC.side_files(str(tmp_path)) == ["blocklut_256.npy", "config.json", "modeling_x.py", "tokenizer.model"]
    idx = CC.remap_index({"metadata": {"total_size": 1},
                          "weight_map": {"a.weight": "model-00001-of-00002.safetensors"}})
    assert idx == {"metadata": {"total_size": 1}, "weight_map": {"a.weight": "model-00001-of-00002_lut.safetensors"}}


def test_single_file_checkpoint(tmp_path):
    (tmp_path / "model.safetensors").write_bytes(b"")
    assert CC.shard_files(str(tmp_path)) == [str(tmp_path / "model.safetensors")]
    assert CC.lut_name("model.safetensors") == "model_lut.safetensors"


@pytest.mark.parametrize("argv,expect", [
    (["--format", "b", "--bits", "3", "--group", "32"],
     {"codebook_scope": "row_block", "index_bits": 3, "lut_block": 32}),
    (["--format", "nested", "--group", "64", "--tier", "coarse"],
     {"codebook_scope": "row_block", "lut_block": 64,
      "nested": {"coarse_bits": 2, "residual_bits": 2, "tier": "coarse"}}),
    (["--write_quant_config"], {"code_type": "BLOCKLUT", "block_size": 128}),
])
def test_quant_config_selects_the_converted_format(tmp_path, argv, expect):
    from block_lut_b200.quant_method import LUTConfig
    args = CC.parse_args(["--model", str(tmp_path)] + argv)
    cfg = CC.quant_config(args, str(tmp_path / "out"))
    for k, v in expect.items():
        assert cfg[k] == v
    assert cfg["quant_method"] == "lut" and os.path.isabs(cfg["lut_path"])
    # the loader reads it back as the converted format
    fmt = LUTConfig.from_config(json.loads(json.dumps(cfg))).lut_format()
    want = CC.format_of(args)
    assert fmt.kind == (want.kind if want else "r8")
    if want:
        assert (fmt.bits, fmt.group, fmt.tier) == (want.bits, want.group, want.tier)


def test_shard_names_and_in_place_refusal(tmp_path, monkeypatch):
    # a shard already named *_lut keeps its name, so a re-conversion in place is refused
    assert CC.lut_name("model-00001-of-00002_lut.safetensors") == "model-00001-of-00002_lut.safetensors"
    monkeypatch.setattr(torch.cuda, "is_available", lambda: True)
    with pytest.raises(ValueError, match="differ"):
        CC.convert_checkpoint(CC.parse_args(["--model", str(tmp_path), "--output", str(tmp_path)]))


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU refusal")
def test_converter_refuses_without_gpu(tmp_path):
    np.save(tmp_path / "blocklut_256.npy", np.linspace(-1, 1, 256, dtype=np.float32))
    with pytest.raises(RuntimeError, match="GPU"):
        CC.convert_checkpoint(CC.parse_args(["--model", str(tmp_path), "--output", str(tmp_path / "o")]))
    with pytest.raises(Exception):
        CC.quantize_weight(torch.zeros(256, dtype=torch.bfloat16), torch.zeros(256, dtype=torch.bfloat16))


def test_absmax_file_feeds_the_loader(tmp_path):
    """lut_absmax.npz as the converter writes it (float32 copies of bf16, keyed
    by .weight names) loads into w13_absmax (gate blocks, then up blocks) and
    w2_absmax of the right layer (quant_method.py:189-222): by layer_id when
    the layer has one, else in call order."""
    from types import SimpleNamespace
    from block_lut_b200.quant_method import LUTConfig, LUTFusedMoEMethod
    E, nb = 2, 3
    data = {}
    for layer in (0, 1):
        for e in range(E):
            for j, proj in enumerate(("gate", "up", "down")):
                v = torch.tensor([layer * 100 + e * 10 + j + q / 4 for q in range(nb)]).to(torch.bfloat16)
                data[f"model.layers.{layer}.mlp.experts.{e}.{proj}_proj.weight"] = v.float().numpy()
    data["model.layers.0.mlp.shared_expert.gate_proj.weight"] = np.zeros(nb, dtype=np.float32)
    np.savez(tmp_path / CC.ABSMAX_NAME, **data)
    method = LUTFusedMoEMethod(LUTConfig(code_type="BLOCKLUT"))

    def fresh(layer_id=None):
        ns = SimpleNamespace(w13_weight=torch.zeros(E, 4, 4, dtype=torch.uint8),
                             w13_absmax=torch.zeros(E, 2 * nb, dtype=torch.bfloat16),
                             w2_absmax=torch.zeros(E, nb, dtype=torch.bfloat16))
        if layer_id is not None:
            ns.layer_id = layer_id
        return ns

    def want(layer, e, proj):
        return torch.from_numpy(data[f"model.layers.{layer}.mlp.experts.{e}.{proj}_proj.weight"]).to(torch.bfloat16)

    for expect_layer, lay in ((0, fresh()), (1, fresh()), (1, fresh(layer_id=1))):
        method._load_absmax(lay, str(tmp_path / CC.ABSMAX_NAME))
        for e in range(E):
            assert torch.equal(lay.w13_absmax[e], torch.cat([want(expect_layer, e, "gate"), want(expect_layer, e, "up")]))
            assert torch.equal(lay.w2_absmax[e], want(expect_layer, e, "down"))


def test_load_codebooks(tmp_path):
    # convert_checkpoint.py:36-58: BLOCKLUT needs blocklut_256.npy; NESTEDLUT falls back to it
    with pytest.raises(FileNotFoundError):
        CC.load_codebooks(str(tmp_path), "BLOCKLUT")
    np.save(tmp_path / "blocklut_256.npy", np.linspace(-1, 1, 256, dtype=np.float32))
    books = CC.load_codebooks(str(tmp_path), "NESTEDLUT")
    assert set(books) == {"blocklut", "mapped16", "mapped64"}
    assert books["blocklut"].dtype == torch.bfloat16 and torch.equal(books["mapped16"], books["blocklut"])
    m16 = np.arange(256, dtype=np.uint16) | 0x3F00       # bf16 bit patterns of numbers in [0.5, 1)
    np.save(tmp_path / "nested_lut_mapped16.npy", m16)
    books = CC.load_codebooks(str(tmp_path), "NESTEDLUT")
    assert np.array_equal(books["mapped16"].view(torch.int16).numpy().view(np.uint16), m16)
    assert set(CC.load_codebooks(str(tmp_path), "BLOCKLUT")) == {"blocklut", "mapped16"}


def test_moe_layer_host_paths(tmp_path):
    from types import SimpleNamespace
    from block_lut_b200.moe_layer import DeepseekV2MoE_LUT, LUTMoEExpertWrapper
    from block_lut_b200.quantizer import LUTQuantizer
    cfg = SimpleNamespace(hidden_size=64, moe_intermediate_size=32, n_routed_experts=4, num_experts_per_tok=2)
    assert DeepseekV2MoE_LUT(cfg).load_codebook(str(tmp_path)) is False   # no codebook files
    wr = LUTMoEExpertWrapper(64, 32, LUTQuantizer())
    assert not wr.has_decompressed() and "hidden=64" in wr.extra_repr()
    assert wr._shape("w13") == (64, 64) and wr._shape("w2") == (64, 32)
    with pytest.raises(ValueError):
        wr._shape("w3")
