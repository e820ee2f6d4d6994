"""``fused_lut_gemv``, the reference's ``vllm_lut/fused_kernel.py:13-46`` API.

The reference has torch.compile fuse
``(codebook[indices] * absmax[min(flat // block_size, nb - 1)]) @ input_vec``
into one kernel. Here the call runs the single-launch ``blut_lut_gemv``
kernel that ``cuda_lut_gemv.lut_gemv`` uses: a warp per row, fp32
accumulation, bf16 out. That kernel reads one absmax per 128 flat elements,
saturating at the last one as the reference does. A block of 128 (the
reference's default, and the block of every checkpoint it writes) goes
straight to the kernel. A block of a multiple of 128 is first expanded to
one scale per 128 elements, which gives every element the same scale as the
reference's block index. Smaller blocks cannot be expressed per 128 elements
and raise.
"""
from __future__ import annotations

import torch

from .cuda_lut_gemv import lut_gemv


def absmax_per_128(absmax: torch.Tensor, block_size: int, numel: int) -> torch.Tensor:
    """One scale per 128 flat elements of a ``numel``-element matrix whose
    ``absmax`` has one scale per ``block_size`` elements (a multiple of 128),
    the reference's block index saturating at the last scale:
    ``out[j] = absmax[min(j * 128 // block_size, nb - 1)]``.  For every flat
    index f, ``out[min(f // 128, len(out) - 1)]`` is then
    ``absmax[min(f // block_size, nb - 1)]``."""
    if block_size % 128 or block_size <= 0:
        raise ValueError(f"block_size {block_size} is not a multiple of 128")
    am = absmax.reshape(-1)
    n128 = -(-numel // 128)
    j = torch.arange(n128, device=am.device) * 128 // block_size
    return am[j.clamp(max=am.numel() - 1)]


def fused_lut_gemv(input_vec: torch.Tensor, indices: torch.Tensor, codebook: torch.Tensor, absmax: torch.Tensor,
                   block_size: int = 128) -> torch.Tensor:
    """[K] bf16, [M, K] uint8, [256] bf16, [num_blocks] bf16 -> [M] bf16."""
    if block_size != 128:
        if block_size % 128:
            raise ValueError(f"fused_lut_gemv needs an absmax block of a multiple of 128 elements, not {block_size}")
        absmax = absmax_per_128(absmax.to(indices.device), block_size, indices.numel())
    return lut_gemv(input_vec, indices, codebook, absmax)
