"""The LUT plugin inside vLLM (config 2's caller): ``LLM(model=<Qwen1.5-
MoE-A2.7B architecture, 2 layers>, quantization="lut", load_format="dummy")``
generates tokens, and the routed experts of every MoE layer run through
``LUTFusedMoEMethod.apply`` (vllm/model_executor/layers/fused_moe/runner/
moe_runner.py calls it with vLLM's own top-k).

vLLM runs in a child process (its engine sets up a process group of its
own).  The child widens vLLM's dummy-weight range so that activations stay
in fp16's normal range, gives the LUT experts random codes and sorted random
tables after loading, records the first decode-step call of the plugin
(input rows, vLLM's top-k ids and weights, the output, and the experts it
used), and saves them.  Here that call is checked against the float64
oracle within the layer tolerance of tests/_helpers.check_layer.
"""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from oracle import blut_oracle as O
from tests._helpers import check_layer

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import json, os, sys, tempfile
os.environ["VLLM_ENABLE_V1_MULTIPROCESSING"] = "0"
sys.path.insert(0, sys.argv[1])
out_path = sys.argv[2]
import numpy as np
import torch
import bench
from block_lut_b200.formats import LUTFormat
from block_lut_b200 import quant_method as QM
import vllm.model_executor.model_loader.dummy_loader as DL

_init = DL.initialize_dummy_weights
DL.initialize_dummy_weights = lambda model, cfg, *a, **k: _init(model, cfg, low=-0.05, high=0.05)

_pwal = QM.LUTFusedMoEMethod.process_weights_after_loading
def pwal(self, layer):
    g = torch.Generator(device=layer.w13_weight.device).manual_seed(7)
    for name in ("w13", "w2"):
        codes = getattr(layer, name + "_weight")
        codes.copy_(torch.randint(0, 256, codes.shape, generator=g, device=codes.device, dtype=torch.uint8))
        t = getattr(layer, name + "_tables")
        t.copy_((torch.randn(t.shape, generator=g, device=t.device) * 0.02).sort(dim=-1).values.to(t.dtype))
    return _pwal(self, layer)
QM.LUTFusedMoEMethod.process_weights_after_loading = pwal

rec = {}
_apply = QM.LUTFusedMoEMethod.apply
def apply(self, layer, x, topk_weights, topk_ids, **kw):
    out = _apply(self, layer, x, topk_weights, topk_ids, **kw)
    if not rec and x.shape[0] <= 4 and not torch.cuda.is_current_stream_capturing():
        torch.cuda.synchronize()
        ids = topk_ids.cpu().numpy().astype(np.int32)
        used = np.unique(ids)
        sel = torch.from_numpy(used).long().cuda()
        rec.update(x=x.float().cpu().numpy(), ids=ids, tw=topk_weights.float().cpu().numpy(),
                   out=out.float().cpu().numpy(), used=used,
                   **{f"{n}_{k}": getattr(layer, f"{n}_{k}")[sel].cpu().numpy()
                      for n in ("w13", "w2") for k in ("weight", "tables")})
    return out
QM.LUTFusedMoEMethod.apply = apply

from vllm import LLM, SamplingParams
d = tempfile.mkdtemp()
fmt = LUTFormat("b", 4, 64)
qc = bench.lut_quant_config(fmt)
qc["release_canonical"] = False  # the recorder reads the experts' parameters after the first calls
with open(os.path.join(d, "config.json"), "w") as f:
    json.dump(bench.qwen15_moe_config(2, qc, "float16"), f)
llm = LLM(model=d, quantization="lut", load_format="dummy", skip_tokenizer_init=True, max_model_len=256,
          gpu_memory_utilization=0.3, max_num_seqs=4, dtype="float16", enforce_eager=True, seed=0)
prompts = [{"prompt_token_ids": list(range(1000 + 17 * i, 1032 + 17 * i))} for i in range(2)]
outs = llm.generate(prompts, SamplingParams(max_tokens=6, min_tokens=6, ignore_eos=True, temperature=0.0,
                                            detokenize=False), use_tqdm=False)
n = [len(o.outputs[0].token_ids) for o in outs]
assert n == [6, 6], n
assert rec, "the lut plugin's apply was not called at a decode step"
np.savez(out_path, **rec)
print("vllm child ok", n)
"""


@pytest.mark.gpu
def test_vllm_generates_through_lut_plugin_and_matches_oracle(tmp_path):
    pytest.importorskip("vllm")
    script = tmp_path / "child.py"
    script.write_text(CHILD)
    out = tmp_path / "rec.npz"
    env = dict(os.environ, PYTHONPATH=ROOT)
    r = subprocess.run([sys.executable, str(script), ROOT, str(out)], capture_output=True, text=True, timeout=900,
                       env=env, cwd=str(tmp_path))
    assert r.returncode == 0 and "vllm child ok" in r.stdout, (r.returncode, r.stdout[-3000:], r.stderr[-6000:])
    d = np.load(out)
    x, ids, tw, got = d["x"], d["ids"], d["tw"], d["out"]
    used = list(d["used"])
    assert 1 <= x.shape[0] <= 4 and ids.shape == (x.shape[0], 4)
    W13 = {e: O.dequant_b(d["w13_weight"][i], d["w13_tables"][i], 4, 64).astype(np.float32)
           for i, e in enumerate(used)}
    W2 = {e: O.dequant_b(d["w2_weight"][i], d["w2_tables"][i], 4, 64).astype(np.float32)
          for i, e in enumerate(used)}
    ref = O.moe_forward(x.astype(np.float64), ids, tw, lambda e: W13[e], lambda e: W2[e], act_dtype="f16")
    # outputs are normal fp16 numbers (the smallest is 6.1e-5), and the oracle
    # rounds SiLU(gate) * up to fp16 where the kernel does
    assert np.abs(ref).max() > 1e-4
    check_layer(torch.from_numpy(got).half(), ref, torch.float16, "vLLM decode step, MoE layer")
