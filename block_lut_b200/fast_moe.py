"""``fused_lut_moe``, the reference's ``vllm_lut/fast_moe.py`` entry point.

Same arguments as the reference (fast_moe.py:30-80): reference-format
(uint8 index, bf16 absmax, bf16[256] codebook) expert stacks plus the
router's ``topk_ids`` / ``topk_weights``.  Instead of a Python loop over the
unique experts (one GEMV launch and host sync per expert), every active
(token, expert) pair runs in one ``blut_moe_forward`` call.  The first call
on a weight stack repacks it into the tiled layout and caches it, keyed by
the tensors' address, shape and version.  An entry also holds weak
references to the tensors it was built from (their view bases), so a stack
freed and replaced by another at the same address is repacked, not served
from the stale entry (the reference's id-keyed cache can alias that way).
"""
from __future__ import annotations

import weakref
from collections import OrderedDict

import torch

from .formats import LUTFormat, QuantizedMatrix
from .moe import LUTExperts, LUTMoELayer

# Tiled layers by weight stack, least recently used first; a model's layers
# each keep their entry while fewer than _CACHE_MAX stacks are in use.
_CACHE: "OrderedDict" = OrderedDict()
_CACHE_MAX = 256


def _key(*ts):
    return tuple((t.data_ptr(), tuple(t.shape), t._version) for t in ts)


def _root(t: torch.Tensor) -> torch.Tensor:
    """The tensor that owns t's memory: its view base, or t itself."""
    return t._base if t._base is not None else t


def _same_tensors(refs, ts) -> bool:
    return all(r() is _root(t) for r, t in zip(refs, ts))


def r8_layer(w13_weight, w13_absmax, w2_weight, w2_absmax, codebook, top_k: int, tier: int = 0) -> LUTMoELayer:
    """Tiled ``LUTMoELayer`` for reference-format stacks (cached)."""
    ts = (w13_weight, w13_absmax, w2_weight, w2_absmax, codebook)
    key = _key(*ts) + (top_k, tier)
    hit = _CACHE.get(key)
    layer = hit[0] if hit is not None and _same_tensors(hit[1], ts) else None
    if layer is not None:
        _CACHE.move_to_end(key)
    else:
        _CACHE.pop(key, None)
        while len(_CACHE) >= _CACHE_MAX:
            _CACHE.popitem(last=False)
        fmt = LUTFormat("r8", 8, 128, tier)
        e_n, two_i, h = w13_weight.shape
        cb = codebook.to(device=w13_weight.device, dtype=torch.bfloat16).contiguous()
        w13 = QuantizedMatrix(fmt, two_i, h, w13_weight.reshape(e_n, -1), cb,
                              scales=w13_absmax.to(torch.bfloat16).reshape(e_n, -1))
        w2 = QuantizedMatrix(fmt, w2_weight.shape[1], w2_weight.shape[2], w2_weight.reshape(e_n, -1), cb,
                             scales=w2_absmax.to(torch.bfloat16).reshape(e_n, -1))
        experts = LUTExperts.from_quantized([w13.expert(e) for e in range(e_n)],
                                            [w2.expert(e) for e in range(e_n)], cb)
        layer = LUTMoELayer(experts, top_k)
        _CACHE[key] = (layer, [weakref.ref(_root(t)) for t in ts])
    return layer


def _fused_expert_compute(x, w13_slices, w2_slices, cb, a13, a2):
    """One expert on one token (fast_moe.py:14-27): W2 (SiLU(gate) * up) with
    [gate; up] = W13 x. Runs as one ``blut_moe_forward`` over a single-expert
    stack with routing weight 1; returns [hidden] in x's dtype."""
    layer = r8_layer(w13_slices.unsqueeze(0), a13.reshape(1, -1), w2_slices.unsqueeze(0), a2.reshape(1, -1), cb, 1)
    xt = x.reshape(1, -1)
    ids = torch.zeros(1, 1, dtype=torch.int32, device=xt.device)
    w = torch.ones(1, 1, dtype=torch.float32, device=xt.device)
    return layer.forward(xt, ids, w).reshape(-1)


def fused_lut_moe(x, topk_ids, topk_weights, w13_weight, w13_absmax, w2_weight, w2_absmax, codebook):
    """[T, H] (or [H]) activations -> [T, H] MoE output (reference-format experts)."""
    x2 = x.reshape(1, -1) if x.dim() == 1 else x
    ids = topk_ids.reshape(x2.shape[0], -1)
    layer = r8_layer(w13_weight, w13_absmax, w2_weight, w2_absmax, codebook, ids.shape[1])
    return layer.forward(x2, ids, topk_weights.reshape(ids.shape))
