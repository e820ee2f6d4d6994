"""``DeepseekV2MoE_LUT`` and ``_routing``, the reference's ``vllm_lut/moe_layer.py`` API.

``DeepseekV2MoE_LUT.forward(hidden_states)`` (moe_layer.py:281-355) runs the
router (fused logits + softmax + top-k kernel), all routed LUT experts in one
``blut_moe_forward`` call and the bf16/fp16 shared experts in the same call,
instead of the reference's Python loop over (k, expert) masks.
``_routing(router_logits, top_k)`` keeps the reference's semantics
(moe_layer.py:358-376): softmax in float32, top-k, weights cast back to the
logits' dtype. ``LUTMoEExpertWrapper`` (moe_layer.py:32-143) holds one
expert's Format R weights and multiplies by them through ``LUTLinear``.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from .formats import LUTFormat, QuantizedMatrix, encode
from .linear import LUTLinear
from .moe import LUTExperts, LUTMoELayer, SharedExpert
from .quantizer import LUTQuantizer, decompress_blocklut


def _routing(router_logits: torch.Tensor, top_k: int) -> Tuple[torch.Tensor, torch.Tensor]:
    routing_weights = torch.softmax(router_logits.float(), dim=-1)
    topk_weights, topk_indices = torch.topk(routing_weights, top_k, dim=-1)
    return topk_weights.to(router_logits.dtype), topk_indices


class LUTMoEExpertWrapper(nn.Module):
    """One expert's Format R weights: uint8 indices, bf16 absmax and the bf16[256]
    codebook for the fused gate/up matrix ``w13`` [2I, H] and the down matrix
    ``w2`` [H, I] (moe_layer.py:32-143).

    ``forward(x, name)`` is ``x @ W^T``. It uses the cached bf16 weights when
    ``set_decompressed`` stored them, as the reference does for hot experts.
    Otherwise it is a ``LUTLinear`` matmul straight from the indices. Shapes
    without a tiled layout, and absmax blocks other than 128, are decompressed
    on the GPU and multiplied with ``F.linear``, which is the reference's own
    path."""

    def __init__(self, hidden_size: int, intermediate_size: int, quantizer: LUTQuantizer,
                 device: Optional[torch.device] = None):
        super().__init__()
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.quantizer = quantizer
        self.device = device or torch.device("cuda")
        for name in ("w13_indices", "w13_absmax", "w2_indices", "w2_absmax", "codebook"):
            self.register_buffer(name, None)
        self._w13_bf16: Optional[torch.Tensor] = None
        self._w2_bf16: Optional[torch.Tensor] = None
        self._linear: dict = {}

    def set_weights(self, w13_weight: torch.Tensor, w2_weight: torch.Tensor, codebook: torch.Tensor) -> None:
        """Quantise bf16 weights with the GPU encoder and keep the result."""
        self.codebook = codebook.to(device=self.device, dtype=torch.bfloat16)
        q13 = self.quantizer.quantize(w13_weight, codebook)
        q2 = self.quantizer.quantize(w2_weight, codebook)
        self.w13_indices, self.w13_absmax = q13["indices"].to(self.device), q13["absmax"].to(self.device)
        self.w2_indices, self.w2_absmax = q2["indices"].to(self.device), q2["absmax"].to(self.device)
        self._linear.clear()

    def set_decompressed(self, w13_bf16: torch.Tensor, w2_bf16: torch.Tensor) -> None:
        self._w13_bf16 = w13_bf16.to(self.device)
        self._w2_bf16 = w2_bf16.to(self.device)

    def has_decompressed(self) -> bool:
        return self._w13_bf16 is not None

    def clear_decompressed(self) -> None:
        self._w13_bf16 = None
        self._w2_bf16 = None

    def _shape(self, name: str) -> Tuple[int, int]:
        if name == "w13":
            return 2 * self.intermediate_size, self.hidden_size
        if name == "w2":
            return self.hidden_size, self.intermediate_size
        raise ValueError(f"Unknown weight name: {name}")

    def get_weight(self, name: str) -> torch.Tensor:
        """bf16 weight: the cached copy, else decompressed on the GPU."""
        rows, cols = self._shape(name)
        cached = self._w13_bf16 if name == "w13" else self._w2_bf16
        if cached is not None:
            return cached
        idx, am = (self.w13_indices, self.w13_absmax) if name == "w13" else (self.w2_indices, self.w2_absmax)
        return decompress_blocklut(idx, am, self.codebook, self.quantizer.block_size).reshape(rows, cols)

    def _lut_linear(self, name: str) -> Optional[LUTLinear]:
        if name not in self._linear:
            rows, cols = self._shape(name)
            idx, am = (self.w13_indices, self.w13_absmax) if name == "w13" else (self.w2_indices, self.w2_absmax)
            lin = None
            if self.quantizer.block_size == 128:
                qm = QuantizedMatrix(LUTFormat("r8", 8, 128), rows, cols, idx.reshape(-1).contiguous(),
                                     self.codebook.contiguous(), scales=am.reshape(-1).to(torch.bfloat16).contiguous())
                try:
                    lin = LUTLinear(qm)
                except ValueError:  # no tiled layout for this shape
                    lin = None
            self._linear[name] = lin
        return self._linear[name]

    def forward(self, x: torch.Tensor, name: str) -> torch.Tensor:
        rows, cols = self._shape(name)
        cached = self._w13_bf16 if name == "w13" else self._w2_bf16
        lin = None if cached is not None else self._lut_linear(name)
        if lin is None:
            return F.linear(x, self.get_weight(name))
        x2 = x.reshape(-1, cols).to(torch.bfloat16)
        return lin(x2).reshape(*x.shape[:-1], rows).to(x.dtype)

    def extra_repr(self) -> str:
        return f"hidden={self.hidden_size}, intermediate={self.intermediate_size}, codebook_size=256"


class DeepseekV2MoE_LUT(nn.Module):
    """LUT-quantised MoE block (moe_layer.py:146-355): routed experts LUT, shared experts dense.

    Built as the reference builds it:

    * ``__init__`` makes the router ``gate`` [E, H], the shared experts
      (``n_shared_experts`` x ``moe_intermediate_size`` columns) as dense
      ``shared_gate_up`` [2 I_s, H] (gate rows, then up rows) and
      ``shared_down`` [H, I_s], and a ``LUTQuantizer`` of ``lut_config.code_type``
      (BLOCKLUT when there is no config).  The reference declares the shared
      gate/up projection I_s wide, which its SiLU-and-mul halves before a
      down projection that expects I_s inputs; here it is 2 I_s wide, so the
      shared MLP has the intermediate size the config names.
    * ``load_codebook(lut_path)`` loads ``blocklut_256.npy``;
      ``quantize_expert_weights(w13, w2)`` trains the codebook on all the
      expert weights when none was loaded, then quantises every expert to
      the reference's BlockLUT format (uint8 index, bf16 absmax per 128,
      the 256-entry codebook) in ``experts`` (one ``LUTMoEExpertWrapper``
      each).  A ``lut_config`` with a ``lut_format()`` that names a per-block
      format (Format B, NestedLUT) encodes that format instead.
    * ``forward(hidden_states)``: router logits, softmax top-k (renormalised
      when ``config.norm_topk_prob``), every routed expert and the shared
      experts (added unscaled, as the reference adds them) in one
      ``blut_moe_forward`` call, where the reference loops over (k, expert)
      masks with a decompression and three matmuls per expert.

    ``config`` needs ``hidden_size``, ``moe_intermediate_size``,
    ``n_routed_experts``, ``num_experts_per_tok`` and optionally
    ``n_shared_experts`` and ``norm_topk_prob``; ``lut_config`` is the
    patcher's ``LUT_MoE_vLLMConfig`` (``code_type``, ``lut_path``, ``lut_tier``)
    or a ``LUTConfig``.
    """

    def __init__(self, config, parallel_config=None, quant_config=None, reduce_results: bool = True,
                 prefix: str = "", lut_config=None, dtype: torch.dtype = torch.bfloat16):
        super().__init__()
        self.config = config
        self.lut_config = lut_config
        self.hidden_size = config.hidden_size
        self.intermediate_size = config.moe_intermediate_size
        self.num_experts = config.n_routed_experts
        self.top_k = config.num_experts_per_tok
        self.n_shared_experts = getattr(config, "n_shared_experts", None)
        self.renorm = bool(getattr(config, "norm_topk_prob", False))
        self.dtype = dtype
        self.gate = nn.Linear(self.hidden_size, self.num_experts, bias=False, dtype=dtype)
        if self.n_shared_experts:
            si = self.intermediate_size * self.n_shared_experts
            self.shared_gate_up = nn.Linear(self.hidden_size, 2 * si, bias=False, dtype=dtype)
            self.shared_down = nn.Linear(si, self.hidden_size, bias=False, dtype=dtype)
        else:
            self.shared_gate_up = None
            self.shared_down = None
        self.quantizer = LUTQuantizer(code_type=getattr(lut_config, "code_type", "BLOCKLUT") if lut_config
                                      else "BLOCKLUT")
        self._codebook_loaded = False
        self.experts: nn.ModuleList = nn.ModuleList()
        self.layer_id: int = 0
        self._moe: Optional[LUTMoELayer] = None

    def load_codebook(self, lut_path: str) -> bool:
        """Load the checkpoint's codebook files (moe_layer.py:229-237); True when
        ``blocklut_256.npy`` was found. The table becomes the ``_codebook`` buffer
        that ``quantize_expert_weights`` quantises with."""
        loaded = self.quantizer.load(lut_path)
        if loaded and self.quantizer.lut_codebook is not None:
            self._codebook_loaded = True
            self.register_buffer("_codebook", self.quantizer.lut_codebook.to("cuda"))
        return loaded

    def lut_format(self) -> LUTFormat:
        """The routed experts' format: the reference's BlockLUT unless the
        config names a per-block format."""
        if self.lut_config is not None and hasattr(self.lut_config, "lut_format"):
            return self.lut_config.lut_format()
        tier = int(getattr(self.lut_config, "lut_tier", 0) or 0) if self.lut_config is not None else 0
        return LUTFormat("r8", 8, self.quantizer.block_size, tier)

    @torch.no_grad()
    def quantize_expert_weights(self, w13_weights: torch.Tensor, w2_weights: torch.Tensor) -> None:
        """Quantise [E, 2I, H] / [E, H, I] expert weights (moe_layer.py:239-279) and build the layer."""
        fmt = self.lut_format()
        E = w13_weights.shape[0]
        self.experts = nn.ModuleList()
        if fmt.kind == "r8":
            if not self._codebook_loaded:  # train on these weights, as the reference does
                self.quantizer.train(torch.cat([w13_weights.reshape(-1), w2_weights.reshape(-1)]))
                self.register_buffer("_codebook", self.quantizer.lut_codebook.to("cuda"))
                self._codebook_loaded = True
            cb = self._codebook.to(device="cuda", dtype=torch.bfloat16).contiguous()
            q13, q2 = [], []
            for e in range(E):
                ex = LUTMoEExpertWrapper(self.hidden_size, self.intermediate_size, self.quantizer)
                ex.set_weights(w13_weights[e], w2_weights[e], cb)
                self.experts.append(ex)
                q13.append(QuantizedMatrix(fmt, 2 * self.intermediate_size, self.hidden_size,
                                           ex.w13_indices.reshape(-1).contiguous(), cb,
                                           scales=ex.w13_absmax.reshape(-1).to(torch.bfloat16).contiguous()))
                q2.append(QuantizedMatrix(fmt, self.hidden_size, self.intermediate_size,
                                          ex.w2_indices.reshape(-1).contiguous(), cb,
                                          scales=ex.w2_absmax.reshape(-1).to(torch.bfloat16).contiguous()))
            experts = LUTExperts.from_quantized(q13, q2, cb)
        else:
            q13 = [encode(w13_weights[e].cuda(), fmt) for e in range(E)]
            q2 = [encode(w2_weights[e].cuda(), fmt) for e in range(E)]
            experts = LUTExperts.from_quantized(q13, q2)
        cdt = fmt.compute_dtype
        shared = None
        if self.shared_gate_up is not None:
            shared = SharedExpert.from_dense(self.shared_gate_up.weight.detach().to(device="cuda", dtype=cdt),
                                             self.shared_down.weight.detach().to(device="cuda", dtype=cdt))
        self._moe = LUTMoELayer(experts, self.top_k, router_w=self.gate.weight.detach().to("cuda"),
                                renorm=self.renorm, shared=shared, shared_gate_mode=0)

    def forward(self, hidden_states: torch.Tensor, **kwargs) -> torch.Tensor:
        if self._moe is None:
            raise RuntimeError("call quantize_expert_weights() first")
        shape = hidden_states.shape
        out = self._moe.forward(hidden_states.reshape(-1, shape[-1]))
        return out.reshape(shape)
