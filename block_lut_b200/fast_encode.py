"""Drop-in for ``vllm_lut.fast_encode`` (fast_encode.py:172-180): the fused GPU
BlockLUT encoder that ``convert_model.py`` uses.

``encode_lut(weight, codebook_f, block_size=128)`` takes flat bf16 weights and
an fp32 codebook on the GPU and returns ``(indices uint8 [N], absmax bf16
[num_blocks])`` on the CPU, as the reference does.  The normalised value
``w / absmax`` stays fp32, so near codebook midpoints the indices can differ
from ``LUTQuantizer.quantize``'s, which rounds it to bf16 first.  The kernel is
``blut_encode_lut_f32`` (``include/blut.h``); no module is compiled at import.
"""
from __future__ import annotations

import torch

from .formats import encode_lut_f32


def encode_lut(weight: torch.Tensor, codebook_f: torch.Tensor, block_size: int = 128):
    if not weight.is_cuda:
        raise ValueError("encode_lut encodes on the GPU: pass a CUDA tensor (no CPU path)")
    idx, absmax = encode_lut_f32(weight.reshape(-1), codebook_f, block_size)
    torch.cuda.synchronize(weight.device)
    return idx.cpu(), absmax.cpu()
