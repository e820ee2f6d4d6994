"""Single-matrix LUT matmul: ``LUTLinear(qm)(x) = x @ dequant(W).T``.

The matrix is tiled once (the tcgen05 layout when the format and shape have
one, else the mma.sync layout) and every call is one ``blut_matmul``: three
stream-ordered launches, fp32 accumulation, no allocation beyond the shared
grow-only workspace.  This is the single-matrix LUT GEMV of the reference
(``lut_gemv``, vllm_lut/cuda_lut_gemv.py:153-169; ``fused_lut_gemv``,
vllm_lut/fused_kernel.py:13-46) for every format of the library and any
number of tokens.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional

import torch

from . import _lib
from .formats import QuantizedMatrix, pack_tiled
from .moe import workspace


class LUTLinear:
    """One quantised weight matrix W [rows, cols] (y = x W^T)."""

    def __init__(self, qm: QuantizedMatrix, tc: Optional[bool] = None, stream=None):
        fmt = qm.fmt
        if tc is None:
            tc = fmt.has_tc_layout(qm.rows, qm.cols)
        self.fmt, self.rows, self.cols, self.tc = fmt, qm.rows, qm.cols, bool(tc)
        self.buf, _ = pack_tiled([qm], stream, tc=self.tc)
        self.lut_table = qm.tables if fmt.kind == "r8" else None
        self.desc = fmt.desc(qm.rows, qm.cols, False, self.tc)

    def launch_count(self, m: int) -> int:
        n = _lib.lib().blut_matmul_launch_count(C.byref(self.desc), int(m))
        if n < 0:
            raise RuntimeError(f"blut_matmul rejects m={m} for {self.fmt} [{self.rows}, {self.cols}]")
        return n

    @_lib.stream_ordered
    def forward(self, x: torch.Tensor, out: Optional[torch.Tensor] = None, out_f32: bool = False,
                stream=None) -> torch.Tensor:
        if x.dim() != 2 or x.shape[1] != self.cols:
            raise ValueError(f"x must be [m, {self.cols}]")
        if x.dtype != self.fmt.compute_dtype or not x.is_cuda:
            raise ValueError(f"x must be a CUDA {self.fmt.compute_dtype} tensor")
        x = x.contiguous()
        m = x.shape[0]
        dt = torch.float32 if out_f32 else x.dtype
        if out is None:
            out = torch.empty(m, self.rows, dtype=dt, device=x.device)
        elif tuple(out.shape) != (m, self.rows) or out.dtype != dt or not out.is_contiguous():
            raise ValueError("out has the wrong shape, dtype or layout")
        if m == 0:  # an empty batch: nothing to launch
            return out
        lib = _lib.lib()
        need = lib.blut_matmul_workspace_size(C.byref(self.desc), m)
        if need == 0:
            raise RuntimeError(f"blut_matmul rejects m={m} for {self.fmt} [{self.rows}, {self.cols}]")
        ws = workspace(x.device, need, stream=stream)
        with _lib.on_device(x):
            _lib.check(lib.blut_matmul(C.byref(self.desc), self.buf.data_ptr(),
                                       None if self.lut_table is None else self.lut_table.data_ptr(), x.data_ptr(),
                                       m, out.data_ptr(), 1 if out_f32 else 0, ws.data_ptr(), ws.numel(),
                                       _lib.stream_ptr(stream)), "matmul")
        return out

    __call__ = forward

    def check_status(self, stream=None) -> None:
        """Raise if a device-side wait of the last call timed out."""
        ws = workspace(self.buf.device, 256, 0)
        with _lib.on_device(ws):
            _lib.check(_lib.lib().blut_moe_check_status(ws.data_ptr(), _lib.stream_ptr(stream)), "matmul status")
