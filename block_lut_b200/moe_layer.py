"""``DeepseekV2MoE_LUT`` and ``_routing``, the reference's ``vllm_lut/moe_layer.py`` API.

``DeepseekV2MoE_LUT.forward(hidden_states)`` (moe_layer.py:281-355) runs the
router (fused logits + softmax + top-k kernel), all routed LUT experts in one
``blut_moe_forward`` call and the bf16/fp16 shared experts in the same call,
instead of the reference's Python loop over (k, expert) masks.
``_routing(router_logits, top_k)`` keeps the reference's semantics
(moe_layer.py:358-376): softmax in float32, top-k, weights cast back to the
logits' dtype.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.nn as nn

from .formats import LUTFormat, encode
from .moe import LUTExperts, LUTMoELayer, SharedExpert


def _routing(router_logits: torch.Tensor, top_k: int) -> Tuple[torch.Tensor, torch.Tensor]:
    routing_weights = torch.softmax(router_logits.float(), dim=-1)
    topk_weights, topk_indices = torch.topk(routing_weights, top_k, dim=-1)
    return topk_weights.to(router_logits.dtype), topk_indices


class DeepseekV2MoE_LUT(nn.Module):
    """LUT-quantised MoE block (routed experts LUT, shared experts dense).

    ``config`` needs ``hidden_size``, ``moe_intermediate_size``,
    ``n_routed_experts``, ``num_experts_per_tok`` and optionally
    ``n_shared_experts`` and ``norm_topk_prob``.  ``lut_config`` is a
    ``LUTConfig`` (its ``lut_format()`` picks the weight format).
    """

    def __init__(self, config, parallel_config=None, quant_config=None, reduce_results: bool = True,
                 prefix: str = "", lut_config=None, dtype: torch.dtype = torch.float16):
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
        self.shared_gate_up: Optional[torch.Tensor] = None
        self.shared_down: Optional[torch.Tensor] = None
        self.layer_id: int = 0
        self._moe: Optional[LUTMoELayer] = None

    def lut_format(self) -> LUTFormat:
        if self.lut_config is not None and hasattr(self.lut_config, "lut_format"):
            return self.lut_config.lut_format()
        return LUTFormat("b", 4, 64)

    @torch.no_grad()
    def quantize_expert_weights(self, w13_weights: torch.Tensor, w2_weights: torch.Tensor,
                                shared_gate_up: Optional[torch.Tensor] = None,
                                shared_down: Optional[torch.Tensor] = None) -> None:
        """Encode [E, 2I, H] / [E, H, I] float weights on the GPU and build the layer."""
        fmt = self.lut_format()
        if fmt.kind == "r8":
            raise ValueError("DeepseekV2MoE_LUT encodes per-block formats; load reference-format "
                             "checkpoints through LUTFusedMoEMethod")
        w13 = [encode(w13_weights[e].cuda(), fmt) for e in range(w13_weights.shape[0])]
        w2 = [encode(w2_weights[e].cuda(), fmt) for e in range(w2_weights.shape[0])]
        shared = None
        if shared_gate_up is not None:
            self.shared_gate_up = shared_gate_up.to(self.dtype).cuda().contiguous()
            self.shared_down = shared_down.to(self.dtype).cuda().contiguous()
            shared = SharedExpert.from_dense(self.shared_gate_up, self.shared_down)
        experts = LUTExperts.from_quantized(w13, w2)
        self._moe = LUTMoELayer(experts, self.top_k, router_w=self.gate.weight.detach().cuda(), renorm=self.renorm,
                                shared=shared, shared_gate_mode=0)

    def forward(self, hidden_states: torch.Tensor, **kwargs) -> torch.Tensor:
        if self._moe is None:
            raise RuntimeError("call quantize_expert_weights() first")
        shape = hidden_states.shape
        out = self._moe.forward(hidden_states.reshape(-1, shape[-1]))
        return out.reshape(shape)
