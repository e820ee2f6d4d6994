"""``fused_lut_gemv``, the reference's ``vllm_lut/fused_kernel.py:13-46`` API.

The reference has torch.compile fuse
``(codebook[indices] * absmax[block]) @ input_vec`` into one kernel. Here the
call runs the single-launch ``blut_lut_gemv`` kernel that
``cuda_lut_gemv.lut_gemv`` uses: a warp per row, fp32 accumulation, bf16 out.
That kernel's absmax block is 128 elements, the reference's default and the
block of every checkpoint it writes; other block sizes raise.
"""
from __future__ import annotations

import torch

from .cuda_lut_gemv import lut_gemv


def fused_lut_gemv(input_vec: torch.Tensor, indices: torch.Tensor, codebook: torch.Tensor, absmax: torch.Tensor,
                   block_size: int = 128) -> torch.Tensor:
    """[K] bf16, [M, K] uint8, [256] bf16, [num_blocks] bf16 -> [M] bf16."""
    if block_size != 128:
        raise ValueError(f"fused_lut_gemv supports the reference's absmax block of 128, not {block_size}")
    return lut_gemv(input_vec, indices, codebook, absmax)
