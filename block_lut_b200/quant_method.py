"""vLLM quantisation plugin ``quant_method="lut"`` on libblut kernels.

Drop-in for the reference's ``vllm_lut/quant_method.py``: the same
``LUTConfig`` / ``LUTFusedMoEMethod`` classes, the same ``create_weights``
parameters (``w13_weight``, ``w2_weight``, ``w13_absmax``, ``w2_absmax``,
``_codebook``; names, shapes and dtypes of quant_method.py:117-163), the same
``process_weights_after_loading`` file conventions (``blocklut_256.npy`` and
``lut_absmax.npz`` under ``lut_path``, quant_method.py:169-224) and the same
``apply(layer, x, topk_weights, topk_ids, **kwargs)`` contract
(quant_method.py:230-279).  Importing the module registers ``"lut"`` with
vLLM when vLLM is importable (quant_method.py:322-331).

Besides the reference format (``code_type`` BLOCKLUT / NESTEDLUT with
``codebook_scope`` "global"), ``LUTConfig`` accepts the packed per-block
codebook formats through extra ``quantization_config`` keys:
``codebook_scope: "row_block"``, ``index_bits`` (2, 3, 4), ``lut_block``
(32, 64, 128) and, for NestedLUT 2+2, ``nested: {"coarse_bits": 2,
"residual_bits": 2, "tier": "full" | "coarse"}``.  Their parameters are
``w13_weight`` / ``w2_weight`` (uint8 packed codes), ``w13_tables`` /
``w2_tables`` (fp16 per-block tables) and, for NestedLUT, ``w13_residual`` /
``w2_residual`` and ``w13_refine`` / ``w2_refine``.

``apply`` runs every active (token, expert) pair of the layer through one
``blut_moe_forward`` call; there is no CPU or PyTorch fallback.
"""
from __future__ import annotations

import math
import os
import sys
from types import SimpleNamespace
from typing import Any, Dict

import numpy as np
import torch

from . import _lib
from .formats import LUTFormat, QuantizedMatrix
from .moe import LUTExperts, LUTMoELayer
from .quantizer import LUTQuantizer, decompress_blocklut

try:  # vLLM is the caller; the classes subclass its bases when it is importable
    from vllm.model_executor.layers.quantization.base_config import QuantizationConfig as _QCBase
    from vllm.model_executor.layers.fused_moe.fused_moe_method_base import FusedMoEMethodBase as _MoEBase
    _HAVE_VLLM = True
except Exception:  # pragma: no cover - exercised only without vLLM
    _QCBase = object
    _MoEBase = object
    _HAVE_VLLM = False


def _set_weight_attrs(param, attrs):
    if not attrs:
        return
    try:
        from vllm.model_executor.utils import set_weight_attrs
        set_weight_attrs(param, attrs)
    except Exception:
        for k, v in attrs.items():
            setattr(param, k, v)


class LUTConfig(_QCBase):
    """LUT quantisation config (``quantization_config`` of a LUT checkpoint)."""

    def __init__(self, code_type: str = "BLOCKLUT", lut_path: str = "", block_size: int = 128, **kwargs):
        if _QCBase is not object:
            super().__init__()
        self.code_type = code_type
        self.lut_path = lut_path or kwargs.get("lut_path", "")
        self.block_size = block_size
        self.codebook_scope = kwargs.get("codebook_scope", "global")
        self.index_bits = int(kwargs.get("index_bits", 8 if self.codebook_scope == "global" else 4))
        self.lut_block = int(kwargs.get("lut_block", 64))
        nested = kwargs.get("nested")
        self.nested = dict(nested) if nested else None
        self.tier = int(kwargs.get("tier", 0))
        # free the canonical expert parameters once the kernels' tiled copy exists
        self.release_canonical = bool(kwargs.get("release_canonical", False))
        print(f"[LUT] LUTConfig init: code_type={code_type}, lut_path={self.lut_path}, "
              f"scope={self.codebook_scope}, kwargs keys={list(kwargs.keys())}", file=sys.stderr)

    @classmethod
    def get_name(cls) -> str:
        return "lut"

    @classmethod
    def get_supported_act_dtypes(cls) -> list:
        return [torch.bfloat16, torch.float16]

    @classmethod
    def get_min_capability(cls) -> int:
        return 100  # sm_100a kernels

    @classmethod
    def get_config_filenames(cls) -> list:
        return []

    @classmethod
    def from_config(cls, config: Dict[str, Any]) -> "LUTConfig":
        cfg = dict(config)
        cfg.pop("quant_method", None)
        return cls(**cfg)

    def lut_format(self) -> LUTFormat:
        """The weight format this config describes."""
        if self.codebook_scope == "global":
            return LUTFormat("r8", 8, self.block_size, self.tier)
        if self.nested:
            tier = 1 if str(self.nested.get("tier", "full")) == "coarse" else 0
            return LUTFormat("nested", 4, self.lut_block, tier)
        return LUTFormat("b", self.index_bits, self.lut_block, 0)

    def get_quant_method(self, layer, prefix):
        try:
            from vllm.model_executor.layers.fused_moe.layer import FusedMoE as _Experts
        except Exception:  # pragma: no cover
            _Experts = ()
        try:  # the reference targets a vLLM with RoutedExperts
            from vllm.model_executor.layers.fused_moe.routed_experts import RoutedExperts
            _Experts = (RoutedExperts,) + ((_Experts,) if not isinstance(_Experts, tuple) else _Experts)
        except Exception:
            pass
        from vllm.model_executor.layers.linear import LinearBase, UnquantizedLinearMethod
        if _Experts and isinstance(layer, _Experts):
            return LUTFusedMoEMethod(self)
        if isinstance(layer, LinearBase):
            return UnquantizedLinearMethod()
        return None


class LUTFusedMoEMethod(_MoEBase):
    """LUT experts: packed indices + codebooks in HBM, dequantised inside the kernels."""

    def __init__(self, quant_config: LUTConfig):
        if _MoEBase is not object:
            cfg = SimpleNamespace(is_act_and_mul=True, has_bias=False, is_gated=False, tp_size=1, ep_size=1,
                                  routing_method="default", hidden_dim=1, intermediate_size=1, num_experts=1,
                                  experts_per_token=1, num_local_experts=1, num_logical_experts=1,
                                  moe_parallel_config=SimpleNamespace(tp_size=1, ep_size=1, tp_rank=0, sp_size=1))
            super().__init__(cfg)
        self.quant_config = quant_config
        self.fmt = quant_config.lut_format()
        self.quantizer = LUTQuantizer(code_type=quant_config.code_type, block_size=quant_config.block_size)

    # ----------------------------------------------------------- weights --
    def create_weights(self, layer, num_experts, hidden_size, intermediate_size_per_partition, params_dtype,
                       **extra):
        device = "cuda"
        two_i = 2 * intermediate_size_per_partition
        i_n, h_n = intermediate_size_per_partition, hidden_size

        def reg(name, shape, dtype, attrs=True):
            p = torch.nn.Parameter(torch.zeros(*shape, dtype=dtype, device=device), requires_grad=False)
            layer.register_parameter(name, p)
            if attrs:
                _set_weight_attrs(p, extra)

        f = self.fmt
        if f.kind == "r8":
            bs = self.quant_config.block_size
            reg("w13_weight", (num_experts, two_i, h_n), torch.uint8)
            reg("w2_weight", (num_experts, h_n, i_n), torch.uint8)
            reg("w13_absmax", (num_experts, math.ceil(two_i * h_n / bs)), torch.bfloat16, False)
            reg("w2_absmax", (num_experts, math.ceil(h_n * i_n / bs)), torch.bfloat16, False)
            reg("_codebook", (256,), torch.bfloat16, False)
        else:
            cb = 2 if f.kind == "nested" else f.bits
            ent = f.table_entries
            reg("w13_weight", (num_experts, two_i, h_n * cb // 8), torch.uint8)
            reg("w2_weight", (num_experts, h_n, i_n * cb // 8), torch.uint8)
            reg("w13_tables", (num_experts, two_i, h_n // f.group, ent), torch.float16)
            reg("w2_tables", (num_experts, h_n, i_n // f.group, ent), torch.float16)
            if f.kind == "nested":
                reg("w13_residual", (num_experts, two_i, h_n // 4), torch.uint8)
                reg("w2_residual", (num_experts, h_n, i_n // 4), torch.uint8)
                reg("w13_refine", (num_experts, two_i, h_n // f.group, 16), torch.float16)
                reg("w2_refine", (num_experts, h_n, i_n // f.group, 16), torch.float16)

    def process_weights_after_loading(self, layer):
        if not hasattr(layer, "w13_weight") or getattr(layer, "_lut_codebook_loaded", False):
            return
        cb_path = self.quant_config.lut_path or ""
        if self.fmt.kind == "r8":
            if cb_path and os.path.isdir(cb_path) and self.quantizer.load(cb_path):
                table = self.quantizer.lut_codebook
                if self.fmt.tier == 1 and self.quantizer.nested_mapped64 is not None:
                    table = self.quantizer.nested_mapped64
                elif self.fmt.tier == 2 and self.quantizer.nested_mapped16 is not None:
                    table = self.quantizer.nested_mapped16
                layer._codebook.copy_(table)
            npz_path = os.path.join(cb_path, "lut_absmax.npz") if cb_path else ""
            if npz_path and os.path.exists(npz_path):
                self._load_absmax(layer, npz_path)
        layer._lut_codebook_loaded = True
        layer._blut = None  # built on first apply (after any later weight copies)
        layer._blut_experts = None

    def _load_absmax(self, layer, npz_path):
        """Absmax arrays keyed by HF ``.weight`` names (quant_method.py:189-222)."""
        data = np.load(npz_path)
        keys = [k for k in data.files if "experts." in k and "shared_expert" not in k and k.endswith(".weight")]
        layer_ids = sorted({p[i + 1] for k in keys for p in [k.split(".")] for i, s in enumerate(p) if s == "layers"},
                           key=int)
        if not layer_ids:
            return
        if not hasattr(self, "_pw_moe_idx"):
            self._pw_moe_idx = 0
        lid = getattr(layer, "layer_id", None)
        lid = str(lid) if lid is not None and str(lid) in layer_ids else layer_ids[self._pw_moe_idx % len(layer_ids)]
        self._pw_moe_idx += 1
        for e in range(layer.w13_weight.shape[0]):
            gk, uk, dk = (f"model.layers.{lid}.mlp.experts.{e}.{n}_proj.weight" for n in ("gate", "up", "down"))
            if gk in data and uk in data:
                layer.w13_absmax.data[e] = torch.cat([torch.from_numpy(data[gk]), torch.from_numpy(data[uk])]).to(
                    device=layer.w13_absmax.device, dtype=torch.bfloat16)
            if dk in data:
                layer.w2_absmax.data[e] = torch.from_numpy(data[dk]).to(device=layer.w2_absmax.device,
                                                                        dtype=torch.bfloat16)

    def _layer(self, layer, top_k: int) -> LUTMoELayer:
        cached = getattr(layer, "_blut", None)
        if cached is not None and cached.top_k == top_k:
            return cached
        experts = getattr(layer, "_blut_experts", None)
        if experts is None:
            experts = self._tile_experts(layer)
            layer._blut_experts = experts
            if self.quant_config.release_canonical:
                # the tiled copy is the only one the kernels read: give the
                # canonical parameters' memory back (vLLM cannot reload into
                # them afterwards)
                for name in ("w13_weight", "w2_weight", "w13_absmax", "w2_absmax", "w13_tables", "w2_tables",
                             "w13_residual", "w2_residual", "w13_refine", "w2_refine"):
                    prm = getattr(layer, name, None)
                    if prm is not None:
                        prm.data = torch.empty(0, dtype=prm.dtype, device=prm.device)
        layer._blut = LUTMoELayer(experts, top_k)
        return layer._blut

    def _tile_experts(self, layer) -> LUTExperts:
        """The layer's experts in the tiled layout of the kernels (a copy of the canonical parameters)."""
        f = self.fmt
        e_n, two_i = layer.w13_weight.shape[:2]
        h_n = layer.w2_weight.shape[1]
        i_n = two_i // 2
        if f.kind == "r8":
            cb = layer._codebook.to(torch.bfloat16).contiguous()
            w13 = [QuantizedMatrix(f, two_i, h_n, layer.w13_weight[e].reshape(-1), cb,
                                   scales=layer.w13_absmax[e]) for e in range(e_n)]
            w2 = [QuantizedMatrix(f, h_n, i_n, layer.w2_weight[e].reshape(-1), cb,
                                  scales=layer.w2_absmax[e]) for e in range(e_n)]
            experts = LUTExperts.from_quantized(w13, w2, cb)
        else:
            nested = f.kind == "nested"
            w13 = [QuantizedMatrix(f, two_i, h_n, layer.w13_weight[e], layer.w13_tables[e],
                                   layer.w13_residual[e] if nested else None,
                                   layer.w13_refine[e] if nested else None) for e in range(e_n)]
            w2 = [QuantizedMatrix(f, h_n, i_n, layer.w2_weight[e], layer.w2_tables[e],
                                  layer.w2_residual[e] if nested else None,
                                  layer.w2_refine[e] if nested else None) for e in range(e_n)]
            experts = LUTExperts.from_quantized(w13, w2)
        return experts

    # ----------------------------------------------------------- forward --
    def apply(self, layer, x, topk_weights, topk_ids, **kwargs):
        """MoE over the LUT experts: [T, H] -> [T, H] in x's dtype."""
        moe = self._layer(layer, topk_ids.shape[-1])
        return moe.forward(x, topk_ids, topk_weights)

    # ------------------------------------------------ reference helpers --
    def _decompress_one(self, indices, absmax, codebook, block_size=128):
        """One expert's Format R weights to bf16, flattened (quant_method.py:281-290)."""
        return decompress_blocklut(indices, absmax, codebook, block_size)

    def _batch_decompress(self, indices, absmax, codebook, block_size=128):
        """Every expert at once, expert e scaled by absmax[e], in the shape of
        ``indices`` (quant_method.py:292-308); one ``blut_batch_blocklut_decompress``."""
        n_exp = indices.shape[0]
        dev = indices.device if indices.is_cuda else torch.device("cuda")
        idx = indices.reshape(n_exp, -1).to(dev).contiguous()
        am = absmax.reshape(n_exp, -1).to(device=dev, dtype=torch.bfloat16).contiguous()
        cb = codebook.to(device=dev, dtype=torch.bfloat16).contiguous()
        out = torch.empty(idx.shape, dtype=torch.bfloat16, device=dev)
        with _lib.on_device(out):
            _lib.check(_lib.lib().blut_batch_blocklut_decompress(out.data_ptr(), idx.data_ptr(), am.data_ptr(),
                                                                 cb.data_ptr(), n_exp, idx.shape[1], am.shape[1],
                                                                 block_size, _lib.stream_ptr()), "_batch_decompress")
        return out.reshape(indices.shape)

    def get_fused_moe_quant_config(self, layer=None):
        from vllm.model_executor.layers.fused_moe.config import FusedMoEQuantConfig, FusedMoEQuantDesc
        desc = FusedMoEQuantDesc(dtype=torch.uint8)
        return FusedMoEQuantConfig(_a1=desc, _a2=desc, _w1=desc, _w2=desc)

    def __repr__(self):
        return f"LUTFusedMoEMethod({self.quant_config.code_type}, {self.fmt.kind})"


# Register "lut" with vLLM on import (quant_method.py:322-331).
try:
    from vllm.model_executor.layers.quantization import QUANTIZATION_METHODS, _CUSTOMIZED_METHOD_TO_QUANT_CONFIG
    if "lut" not in QUANTIZATION_METHODS:
        QUANTIZATION_METHODS.append("lut")
    _CUSTOMIZED_METHOD_TO_QUANT_CONFIG["lut"] = LUTConfig
except Exception:
    pass
