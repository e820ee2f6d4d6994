"""Torch CPU restatement of the reference's LUT-MoE expert forward -- test and
bench infrastructure only.

Nothing in ``block_lut_b200`` imports this file.  ``bench.py`` times it as the
CPU baseline (its ``cpu_baseline`` leg and its ``--impl reference`` arm), on
all host cores, because the reference's own ``LUTFusedMoEMethod.apply`` cannot
travel to the GPU box (the reference has no installable package) and its
Format B / NestedLUT configs have no reference implementation at all.

``apply`` follows the reference's T > 1 path step for step
(``vllm_lut/quant_method.py:230-279``): for every distinct expert id it
dequantises the whole expert (the reference: ``cb[idx] * absmax[i // 128]``,
``quant_method.py:262-266``), runs ``F.linear`` over all T tokens,
``F.silu(gate) * up``, ``F.linear`` again, and scatter-adds the rows of the
tokens that chose the expert, weighted.  Format R runs in bf16 as the
reference does; Format B and NestedLUT (per-(row, block) fp16 tables, no
reference code) gather their tables into fp32 weights and accumulate in fp32
(a table gather, then F.linear with fp32 accumulation).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def dequant_r(idx_u8: torch.Tensor, absmax_bf16: torch.Tensor, cb_bf16: torch.Tensor, rows: int, cols: int,
              block: int = 128) -> torch.Tensor:
    """Format R: ``cb[idx] * absmax[i // block]`` in bf16 (quant_method.py:262-266)."""
    flat = idx_u8.reshape(-1).long()
    bid = (torch.arange(flat.numel()) // block).clamp(max=absmax_bf16.numel() - 1)
    return (cb_bf16[flat] * absmax_bf16.reshape(-1)[bid]).reshape(rows, cols)


def unpack_codes(packed: torch.Tensor, bits: int, cols: int) -> torch.Tensor:
    """LSB-first bit stream per row (uint8 [rows, cols * bits / 8]) -> int64 codes [rows, cols]."""
    rows = packed.shape[0]
    if bits == 4:
        p = packed.long()
        return torch.stack([p & 15, p >> 4], dim=-1).reshape(rows, cols)
    if bits == 2:
        p = packed.long()
        return torch.stack([p & 3, (p >> 2) & 3, (p >> 4) & 3, p >> 6], dim=-1).reshape(rows, cols)
    bit = (packed.long()[..., None] >> torch.arange(8)) & 1           # [rows, nbytes, 8]
    bit = bit.reshape(rows, cols, bits)
    return (bit << torch.arange(bits)).sum(-1)


def dequant_b(packed: torch.Tensor, tables: torch.Tensor, bits: int, group: int, rows: int, cols: int) -> torch.Tensor:
    """Format B: ``tables[row, col // group, code]`` (fp16 tables [rows, cols / group, 2^bits]) as fp32."""
    codes = unpack_codes(packed, bits, cols).reshape(rows, cols // group, group)
    return torch.gather(tables.float(), 2, codes).reshape(rows, cols)


def dequant_nested(coarse: torch.Tensor, resid: torch.Tensor, coarse_t: torch.Tensor, refine_t: torch.Tensor,
                   group: int, rows: int, cols: int, coarse_only: bool = False) -> torch.Tensor:
    """NestedLUT 2+2: ``fp16(coarse[c] + refine[c][r])`` per (row, block), or ``coarse[c]``, as fp32."""
    c = unpack_codes(coarse, 2, cols).reshape(rows, cols // group, group)
    v = torch.gather(coarse_t.float(), 2, c)
    if not coarse_only:
        r = unpack_codes(resid, 2, cols).reshape(rows, cols // group, group)
        v = (v + torch.gather(refine_t.float(), 2, 4 * c + r)).half().float()
    return v.reshape(rows, cols)


def apply(x: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor, w13, w2) -> torch.Tensor:
    """The reference's T > 1 MoE loop (quant_method.py:261-277) on CPU tensors.

    ``w13(e)`` / ``w2(e)`` return expert e's dequantised [2I, H] / [H, I]
    weights in the dtype the products run in (bf16 for Format R, fp32 else).
    """
    out = torch.zeros(x.shape, dtype=x.dtype)
    for eid in torch.unique(topk_ids).tolist():
        a = w13(eid)
        xe = x.to(a.dtype)
        ni = a.shape[0] // 2
        gate_up = F.linear(xe, a)
        activated = F.silu(gate_up[:, :ni]) * gate_up[:, ni:]
        expert_out = F.linear(activated, w2(eid))
        for k in range(topk_ids.shape[-1]):
            m = topk_ids[:, k] == eid
            if not m.any():
                continue
            out[m] += (expert_out[m] * topk_weights[m, k].unsqueeze(-1).to(expert_out.dtype)).to(out.dtype)
    return out
