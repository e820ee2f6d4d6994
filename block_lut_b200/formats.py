"""LUT weight formats, their canonical tensors and the tiled device layout.

Formats (names follow the reference's ``code_type`` vocabulary):

* ``r8``     -- the reference's BlockLUT: one uint8 index per weight into a
  global 256-entry bf16 codebook, bf16 absmax per 128 flat elements
  (``vllm_lut/quant_method.py:117-163``).  ``tier`` 1 / 2 read the 6-bit /
  4-bit NestedLUT tiers through the mapped64 / mapped16 tables
  (``runtime/model_offload.py:751-758``, ``csrc/tensor_engine/tensor_engine.hpp:287-291``).
* ``b``      -- packed ``bits``-bit codes with one sorted fp16 codebook of
  2**bits entries per (row, block of ``group`` columns).
* ``nested`` -- NestedLUT 2+2: 2-bit coarse code into a 4-entry fp16 table per
  block plus a 2-bit residual code into a 4x4 refinement table;
  ``tier`` 0 = full (coarse + refine), 1 = coarse only.
* ``dense``  -- plain fp16 / bf16 weights (the shared expert).

A matrix is kept in its canonical (checkpoint) layout and, for the MoE
kernels, repacked once into the tiled layout (16-row tiles x 128-column
chunks in MMA-fragment order) by ``pack_tiled``.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib

_KIND = {"r8": _lib.FMT_R8, "b": _lib.FMT_B, "nested": _lib.FMT_NESTED, "dense": _lib.FMT_DENSE}


def _dt_code(dtype: torch.dtype) -> int:
    if dtype == torch.float16:
        return _lib.F16
    if dtype == torch.bfloat16:
        return _lib.BF16
    raise ValueError(f"unsupported dtype {dtype}")


@dataclass(frozen=True)
class LUTFormat:
    kind: str = "b"
    bits: int = 4
    group: int = 64
    tier: int = 0
    dense_dtype: torch.dtype = torch.float16

    def __post_init__(self):
        if self.kind not in _KIND:
            raise ValueError(f"unknown format kind {self.kind!r}")

    @property
    def compute_dtype(self) -> torch.dtype:
        """dtype of weights and activations inside the kernels."""
        if self.kind == "r8":
            return torch.bfloat16
        if self.kind == "dense":
            return self.dense_dtype
        return torch.float16

    @property
    def table_entries(self) -> int:
        return 4 if self.kind == "nested" else (1 << self.bits)

    def desc(self, rows: int, cols: int, paired: bool = False, tc: bool = False) -> _lib.MatDesc:
        """C descriptor; ``paired`` selects the gate/up-paired tiled layout,
        ``tc`` the 128-row layout of the tcgen05 matmuls."""
        bits = {"r8": 8, "b": self.bits, "nested": 4, "dense": 16}[self.kind]
        group = 128 if self.kind == "r8" and self.group not in (128,) else self.group
        layout = (_lib.LAYOUT_PAIRED if paired else 0) | (_lib.LAYOUT_TC if tc else 0)
        return _lib.MatDesc(_KIND[self.kind], bits, group, self.tier, _dt_code(self.compute_dtype),
                            layout, int(rows), int(cols))

    def has_tc_layout(self, rows: int, cols: int, paired: bool = False) -> bool:
        """Whether the tcgen05 (BLUT_LAYOUT_TC) layout exists for this format and shape."""
        d = self.desc(rows, cols, paired, tc=True)
        return _lib.lib().blut_tiled_bytes(C.byref(d)) >= 0

    def bytes_per_weight(self) -> float:
        """Bytes the tiled layout streams per weight element (the roofline basis)."""
        if self.kind == "r8":
            return 1.0 + 2.0 / 128
        if self.kind == "dense":
            return 2.0
        if self.kind == "b":
            return self.bits / 8 + (1 << self.bits) * 2 / self.group
        if self.tier == 1:  # coarse only: coarse plane + coarse tables
            return 0.25 + 8 / self.group
        # full tier streams coarse + residual planes and the combined 16-entry tables
        return 0.5 + 32 / self.group


@dataclass
class QuantizedMatrix:
    """Canonical tensors of one matrix (or a stack along a leading expert dim)."""
    fmt: LUTFormat
    rows: int
    cols: int
    codes: torch.Tensor
    tables: Optional[torch.Tensor] = None
    codes2: Optional[torch.Tensor] = None
    tables2: Optional[torch.Tensor] = None
    scales: Optional[torch.Tensor] = None

    def expert(self, e: int) -> "QuantizedMatrix":
        """Expert ``e`` of a stack (canonical tensors with a leading expert
        dimension; the r8 codebook is shared by all experts)."""
        pick = lambda t: None if t is None else t[e]  # noqa: E731
        if self.fmt.kind == "r8":
            return QuantizedMatrix(self.fmt, self.rows, self.cols, self.codes[e], self.tables, None, None,
                                   self.scales[e])
        return QuantizedMatrix(self.fmt, self.rows, self.cols, pick(self.codes), pick(self.tables),
                               pick(self.codes2), pick(self.tables2), None)

    def canon(self) -> _lib.Canon:
        p = lambda t: None if t is None else t.data_ptr()  # noqa: E731
        return _lib.Canon(p(self.codes), p(self.codes2), p(self.tables), p(self.tables2), p(self.scales))


def _check_cuda(*ts):
    for t in ts:
        if t is not None and (not t.is_cuda or not t.is_contiguous()):
            raise ValueError("libblut expects contiguous CUDA tensors")


@_lib.stream_ordered
def encode(w: torch.Tensor, fmt: LUTFormat, stream=None) -> QuantizedMatrix:
    """Quantise a float matrix [rows, cols] with the GPU Lloyd encoder (formats b / nested)."""
    if fmt.kind not in ("b", "nested"):
        raise ValueError("encode() handles formats 'b' and 'nested'; use encode_r for 'r8'")
    w = w.to(torch.float32).contiguous()
    _check_cuda(w)
    rows, cols = w.shape
    nb = cols // fmt.group
    dev = w.device
    cbits = 2 if fmt.kind == "nested" else fmt.bits
    codes = torch.empty(rows, cols * cbits // 8, dtype=torch.uint8, device=dev)
    tables = torch.empty(rows, nb, fmt.table_entries, dtype=torch.float16, device=dev)
    codes2 = tables2 = None
    if fmt.kind == "nested":
        codes2 = torch.empty_like(codes)
        tables2 = torch.empty(rows, nb, 16, dtype=torch.float16, device=dev)
    d = fmt.desc(rows, cols)
    p = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    with _lib.on_device(w):
        _lib.check(_lib.lib().blut_encode(C.byref(d), w.data_ptr(), codes.data_ptr(), tables.data_ptr(), p(codes2),
                                          p(tables2), _lib.stream_ptr(stream)), "encode")
    return QuantizedMatrix(fmt, rows, cols, codes, tables, codes2, tables2)


@_lib.stream_ordered
def encode_r(w: torch.Tensor, codebook: torch.Tensor, block_size: int = 128, stream=None):
    """Reference BlockLUT quantiser on the GPU: returns (uint8 indices [N], bf16 absmax [nb])."""
    w = w.to(torch.bfloat16).contiguous().reshape(-1)
    cb = codebook.to(device=w.device, dtype=torch.bfloat16).contiguous()
    _check_cuda(w, cb)
    n = w.numel()
    idx = torch.empty(n, dtype=torch.uint8, device=w.device)
    absmax = torch.empty((n + block_size - 1) // block_size, dtype=torch.bfloat16, device=w.device)
    with _lib.on_device(w):
        _lib.check(_lib.lib().blut_encode_r(w.data_ptr(), n, cb.data_ptr(), block_size, idx.data_ptr(),
                                            absmax.data_ptr(), _lib.stream_ptr(stream)), "encode_r")
    return idx, absmax


@_lib.stream_ordered
def encode_lut_f32(w: torch.Tensor, codebook_f: torch.Tensor, block_size: int = 128, stream=None):
    """The fast BlockLUT encoder's rule on the GPU (fp32 normalisation against
    an fp32 codebook): returns (uint8 indices [N], bf16 absmax [nb])."""
    w = w.to(torch.bfloat16).contiguous().reshape(-1)
    cb = codebook_f.to(device=w.device, dtype=torch.float32).contiguous()
    _check_cuda(w, cb)
    n = w.numel()
    idx = torch.empty(n, dtype=torch.uint8, device=w.device)
    absmax = torch.empty((n + block_size - 1) // block_size, dtype=torch.bfloat16, device=w.device)
    with _lib.on_device(w):
        _lib.check(_lib.lib().blut_encode_lut_f32(w.data_ptr(), n, cb.data_ptr(), block_size, idx.data_ptr(),
                                                  absmax.data_ptr(), _lib.stream_ptr(stream)), "encode_lut_f32")
    return idx, absmax


@_lib.stream_ordered
def dequant(qm: QuantizedMatrix, stream=None) -> torch.Tensor:
    """Bit-exact dequantisation of one matrix to [rows, cols] (bf16 for r8, fp16 otherwise)."""
    out_dtype = qm.fmt.compute_dtype
    out = torch.empty(qm.rows, qm.cols, dtype=out_dtype, device=qm.codes.device)
    d = qm.fmt.desc(qm.rows, qm.cols)
    c = qm.canon()
    with _lib.on_device(out):
        _lib.check(_lib.lib().blut_dequant(C.byref(d), C.byref(c), out.data_ptr(), _lib.stream_ptr(stream)),
                   "dequant")
    return out


def tiled_bytes(fmt: LUTFormat, rows: int, cols: int, paired: bool = False, tc: bool = False) -> int:
    d = fmt.desc(rows, cols, paired, tc)
    n = _lib.lib().blut_tiled_bytes(C.byref(d))
    if n < 0:
        need = "rows % 128 (256 paired) == 0, cols % 64, a Format B, NestedLUT or dense format" if tc else \
            "rows % 16 and cols % 128 == 0"
        raise ValueError(f"no tiled layout for {fmt} [{rows}, {cols}]: needs {need}")
    return int(n)


@_lib.stream_ordered
def pack_tiled(mats, stream=None, paired: bool = False, tc: bool = False) -> tuple[torch.Tensor, int]:
    """Repack canonical matrices (a list, all of one format and shape) into one
    tiled buffer; returns (uint8 buffer, per-matrix stride in bytes).
    ``paired`` interleaves the row tiles of the two halves (gate/up); ``tc``
    selects the layout of the tcgen05 matmuls."""
    mats = list(mats)
    fmt, rows, cols = mats[0].fmt, mats[0].rows, mats[0].cols
    stride = tiled_bytes(fmt, rows, cols, paired, tc)
    dev = mats[0].codes.device
    buf = torch.empty(len(mats) * stride, dtype=torch.uint8, device=dev)
    d = fmt.desc(rows, cols, paired, tc)
    with _lib.on_device(buf):
        s = _lib.stream_ptr(stream)
        for i, m in enumerate(mats):
            c = m.canon()
            _lib.check(_lib.lib().blut_pack_tiled(C.byref(d), C.byref(c), buf.data_ptr() + i * stride, s),
                       "pack_tiled")
    return buf, stride


@_lib.stream_ordered
def dequant_tiled(fmt: LUTFormat, rows: int, cols: int, tiled: torch.Tensor, lut_table: Optional[torch.Tensor] = None,
                  stream=None, paired: bool = False, tc: bool = False) -> torch.Tensor:
    """Dense matrix rebuilt from one tiled matrix through the kernels' lookups."""
    out = torch.empty(rows, cols, dtype=fmt.compute_dtype, device=tiled.device)
    d = fmt.desc(rows, cols, paired, tc)
    with _lib.on_device(out):
        _lib.check(_lib.lib().blut_dequant_tiled(C.byref(d), tiled.data_ptr(),
                                                 None if lut_table is None else lut_table.data_ptr(), out.data_ptr(),
                                                 _lib.stream_ptr(stream)), "dequant_tiled")
    return out


def dense_matrix(w: torch.Tensor) -> QuantizedMatrix:
    """A plain fp16 / bf16 matrix wrapped as a ``dense`` QuantizedMatrix."""
    w = w.contiguous()
    return QuantizedMatrix(LUTFormat("dense", 16, 128, 0, w.dtype), w.shape[0], w.shape[1], w)
