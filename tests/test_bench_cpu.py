"""bench.py's model descriptions without a GPU: the config.json each vLLM
workload writes describes the same MoE shapes as the kernel-level workloads
(configs 2, 3 and 4), and transformers reads them with the routing
fields vLLM's grouped top-k needs (a group count of None would break it)."""
import pytest

import bench
from block_lut_b200.formats import LUTFormat


def test_qwen15_config_matches_the_decode_stack():
    c = bench.qwen15_moe_config(bench.QWEN["LAYERS"], {}, "float16")
    assert c["num_experts"] == bench.QWEN["E"] and c["num_experts_per_tok"] == bench.QWEN["TOPK"]
    assert c["moe_intermediate_size"] == bench.QWEN["I"]
    assert c["shared_expert_intermediate_size"] == bench.QWEN["IS"]
    assert c["num_hidden_layers"] == bench.QWEN["LAYERS"] == 24 and not c["norm_topk_prob"]


def test_qwen3_config_matches_the_decode_stack():
    c = bench.qwen3_moe_config(bench.QWEN3["LAYERS"], {}, "float16")
    assert c["num_experts"] == bench.QWEN3["E"] == 128 and c["num_experts_per_tok"] == bench.QWEN3["TOPK"] == 8
    assert c["moe_intermediate_size"] == bench.QWEN3["I"] and c["norm_topk_prob"] is bench.QWEN3["RENORM"]
    assert c["num_hidden_layers"] == 48


def test_dsv2_lite_config_matches_the_prefill_stack():
    d = bench.DSV2
    c = bench.dsv2_lite_config(d["LAYERS"], bench.lut_quant_config(LUTFormat("b", 4, 64)), "float16")
    assert c["n_routed_experts"] == d["E"] == 64 and c["num_experts_per_tok"] == d["TOPK"] == 6
    assert c["moe_intermediate_size"] == d["I"] and c["n_shared_experts"] * c["moe_intermediate_size"] == d["IS"]
    # 27 layers: the dense first one and the 26 MoE layers of the kernel-level workload
    assert c["num_hidden_layers"] == d["LAYERS"] + 1 == 27 and c["first_k_dense_replace"] == 1
    assert c["kv_lora_rank"] == 512 and c["q_lora_rank"] is None
    q = c["quantization_config"]
    assert q["quant_method"] == "lut" and q["index_bits"] == 4 and q["lut_block"] == 64
    transformers = pytest.importorskip("transformers")
    cfg = transformers.DeepseekV2Config(**{k: v for k, v in c.items()
                                           if k not in ("architectures", "model_type", "quantization_config")})
    assert cfg.n_group == 1 and cfg.topk_group == 1 and cfg.topk_method == "greedy"


def test_vllm_prompt_ids_stay_inside_every_vocabulary():
    """run_vllm draws prompt token ids below min(150000, vocab - 1000): inside
    DeepSeek-V2-Lite's 102400-entry vocabulary as well as Qwen's 151936."""
    import inspect
    src = inspect.getsource(bench.run_vllm)
    assert 'min(150000, cfg["vocab_size"] - 1000)' in src
    for make in (bench.qwen15_moe_config, bench.qwen3_moe_config, bench.dsv2_lite_config):
        v = make(2, {}, "float16")["vocab_size"]
        assert min(150000, v - 1000) <= v
