"""Fused LUT-dequant GEMV, the reference's ``vllm_lut/cuda_lut_gemv.py`` API.

``lut_gemv(input_vec, indices, codebook, absmax)`` computes
``y[r] = sum_c x[c] * codebook[indices[r, c]] * absmax[(r*K + c) // 128]``
(cuda_lut_gemv.py:23-81,153-169) with the ``blut_lut_gemv`` kernel: one warp
per row, 16-byte code loads, a conflict-free replicated codebook in shared
memory, fp32 accumulation, and no device synchronisation after the launch.
"""
from __future__ import annotations

import torch

from . import _lib


def lut_gemv(input_vec: torch.Tensor, indices: torch.Tensor, codebook: torch.Tensor,
             absmax: torch.Tensor) -> torch.Tensor:
    """[K] bf16, [M, K] uint8, [256] bf16, [num_blocks] bf16 -> [M] bf16."""
    m, k = indices.shape
    x = input_vec.reshape(-1).to(torch.bfloat16).contiguous()
    idx = indices.contiguous()
    cb = codebook.to(device=idx.device, dtype=torch.bfloat16).contiguous()
    am = absmax.reshape(-1).to(device=idx.device, dtype=torch.bfloat16).contiguous()
    y = torch.empty(m, dtype=torch.bfloat16, device=idx.device)
    with _lib.on_device(idx):
        _lib.check(_lib.lib().blut_lut_gemv(x.data_ptr(), idx.data_ptr(), cb.data_ptr(), am.data_ptr(), y.data_ptr(),
                                            m, k, am.numel(), _lib.stream_ptr()), "lut_gemv")
    return y


def load_kernel():
    """The reference compiled its kernel lazily; libblut is prebuilt, so this just loads it."""
    return _lib.lib()
