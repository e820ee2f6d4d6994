"""Progressive bit-plane tiers of Format R indices, on the GPU.

The HF offload engine stores each expert tensor's uint8 indices as three
sections, low4 | mid2 | high2 (runtime/model_offload.py:751-758). A cold or
warm expert reads only a prefix of them (tier 2: n/2 bytes, tier 1: 3n/4,
csrc/tensor_engine/tensor_engine.cpp:505-509) and recovers bf16 weights with
the tier's table (mapped16, mapped64 or the full table).

``pack_bitplanes`` writes the sections. ``recover_tier`` reads a tier's
sections and the absmax in one kernel and writes bf16. It replaces the
reference's unpack (tensor_recover.cu:166-192 on the GPU for tier 2,
tensor_engine.cpp:535-547 on the host for tier 1) followed by its recover pass
(model_topology.cpp:597-618). There is no CPU path.
"""
from __future__ import annotations

import torch

from . import _lib


def bitplane_bytes(n: int, tier: int) -> int:
    """Bytes of the buffer that ``tier`` reads: n/2 (2), 3n/4 (1) or n (0)."""
    v = int(_lib.lib().blut_bitplane_bytes(n, tier))
    if v < 0:
        raise ValueError(f"bit-plane tiers need n > 0, n % 4 == 0 and tier in 0..2 (n={n}, tier={tier})")
    return v


def _check(t: torch.Tensor, dtype: torch.dtype, name: str):
    if not t.is_cuda or not t.is_contiguous() or t.dtype != dtype:
        raise ValueError(f"{name}: expected a contiguous CUDA {dtype} tensor")


@_lib.stream_ordered
def pack_bitplanes(idx: torch.Tensor, stream=None) -> torch.Tensor:
    """uint8 indices [n] (any shape, n % 4 == 0) -> the n-byte bit-plane buffer."""
    _check(idx, torch.uint8, "idx")
    n = idx.numel()
    bitplane_bytes(n, 0)
    planes = torch.empty(n, dtype=torch.uint8, device=idx.device)
    with _lib.on_device(idx):
        _lib.check(_lib.lib().blut_bitplane_pack(planes.data_ptr(), idx.data_ptr(), n, _lib.stream_ptr(stream)),
                   "bitplane_pack")
    return planes


@_lib.stream_ordered
def recover_tier(planes: torch.Tensor, absmax: torch.Tensor, table: torch.Tensor, n: int, tier: int,
                 block_size: int = 128, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """bf16 [n] = table[index] * absmax[i // block_size] from a tier's sections.

    ``planes`` needs at least ``bitplane_bytes(n, tier)`` bytes (only those are
    read), ``table`` the tier's table (bf16, at least 16 / 64 / 256 entries)."""
    _check(planes, torch.uint8, "planes")
    _check(absmax, torch.bfloat16, "absmax")
    _check(table, torch.bfloat16, "table")
    need = bitplane_bytes(n, tier)
    if planes.numel() < need:
        raise ValueError(f"tier {tier} reads {need} bytes of planes, got {planes.numel()}")
    if absmax.numel() < (n + block_size - 1) // block_size:
        raise ValueError("absmax has fewer blocks than n needs")
    if table.numel() < (16, 64, 256)[2 - tier]:
        raise ValueError(f"tier {tier} table needs {(16, 64, 256)[2 - tier]} entries")
    if out is None:
        out = torch.empty(n, dtype=torch.bfloat16, device=planes.device)
    else:
        _check(out, torch.bfloat16, "out")
        if out.numel() < n:
            raise ValueError("out is smaller than n")
    with _lib.on_device(planes):
        _lib.check(_lib.lib().blut_bitplane_recover(out.data_ptr(), planes.data_ptr(), absmax.data_ptr(),
                                                    table.data_ptr(), n, tier, block_size, _lib.stream_ptr(stream)),
                   "bitplane_recover")
    return out
