"""Shared builders for the GPU parity tests: seeded inputs, oracle-side
references, and the tolerance checks written once."""
from __future__ import annotations

import numpy as np
import torch

from oracle import blut_oracle as O

from block_lut_b200.formats import LUTFormat, QuantizedMatrix
from block_lut_b200.moe import LUTExperts

# Tolerance for layer outputs (fp32 accumulation): max-abs 2e-3, rel-L2 1e-3.
MAX_ABS = 2e-3
REL_L2 = 1e-3


def cuda(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t if dtype is None else t.view(dtype)


def bf16_tensor(u16: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(u16).view(np.int16)).cuda().view(torch.bfloat16)


def to_u16(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def check_layer(out: torch.Tensor, ref64: np.ndarray, dtype: torch.dtype, what: str = ""):
    """GPU layer output vs the float64 oracle.

    fp16 outputs: max-abs <= 2e-3 and rel-L2 <= 1e-3 directly.  bf16 outputs
    carry bf16's own final rounding (2^-9 relative), which alone exceeds that
    rel-L2: they are compared with the oracle rounded to bf16,
    allowing 1 bf16 ulp per element and rel-L2 <= 1e-3.
    """
    o = out.float().cpu().numpy().astype(np.float64)
    if dtype == torch.float16:
        err = np.abs(o - ref64).max()
        rel = O.rel_l2(o, ref64)
        assert err <= MAX_ABS and rel <= REL_L2, f"{what} max-abs {err:.3g} rel-L2 {rel:.3g}"
    else:
        rb = O.round_to(ref64.astype(np.float32), "bf16").astype(np.float64)
        ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(rb), 1e-30))) - 7)
        err = np.abs(o - rb)
        assert (err <= np.maximum(ulp, MAX_ABS)).all(), f"{what} max diff {err.max():.3g}"
        rel = O.rel_l2(o, rb)
        assert rel <= REL_L2, f"{what} rel-L2 {rel:.3g}"


def routing_inputs(rng, T, E, k, renorm=False):
    logits = rng.standard_normal((T, E)).astype(np.float32) * 2
    ids, w = O.routing(logits, k, renorm)
    return ids, w


# ----------------------------------------------------------- quantised experts --
def oracle_quantize(w: np.ndarray, fmt: LUTFormat):
    """CPU encode of one matrix -> (numpy canonical dict, fp32 dequantised matrix)."""
    if fmt.kind == "b":
        packed, tables = O.encode_b(w, fmt.bits, fmt.group)
        deq = O.dequant_b(packed, tables, fmt.bits, fmt.group).astype(np.float32)
        return {"codes": packed, "tables": tables}, deq
    if fmt.kind == "nested":
        cp, rp, ct, rt = O.encode_nested(w, fmt.group)
        deq = O.dequant_nested(cp, rp, ct, rt, fmt.group, coarse_only=fmt.tier == 1).astype(np.float32)
        return {"codes": cp, "codes2": rp, "tables": ct, "tables2": rt}, deq
    raise ValueError(fmt.kind)


def qm_from_numpy(fmt: LUTFormat, rows: int, cols: int, d: dict) -> QuantizedMatrix:
    g = lambda k: None if d.get(k) is None else cuda(d[k])  # noqa: E731
    return QuantizedMatrix(fmt, rows, cols, g("codes"), g("tables"), g("codes2"), g("tables2"), g("scales"))


def build_b_layer(fmt: LUTFormat, E: int, H: int, I: int, seed: int = 0, tc=None):
    """Oracle-encoded experts -> (LUTExperts, W13 list fp32, W2 list fp32).
    ``tc``: tiled layout (None: tcgen05 when available, else mma.sync)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    W13, W2, q13, q2 = [], [], [], []
    for _ in range(E):
        a = O.student_t_weights(rng, (2 * I, H))
        b = O.student_t_weights(rng, (H, I))
        c13, d13 = oracle_quantize(a, fmt)
        c2, d2 = oracle_quantize(b, fmt)
        q13.append(qm_from_numpy(fmt, 2 * I, H, c13))
        q2.append(qm_from_numpy(fmt, H, I, c2))
        W13.append(d13)
        W2.append(d2)
    return LUTExperts.from_quantized(q13, q2, tc=tc), W13, W2


def build_r8_layer(E: int, H: int, I: int, seed: int = 0, tier: int = 0, table_u16=None, tc=None):
    """Random reference-format experts -> (LUTExperts, W13 list, W2 list, table).
    ``tc``: tiled layout (None: tcgen05 when available, else mma.sync)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    if table_u16 is None:
        table_u16 = O.f32_to_bf16(np.sort(rng.uniform(-1, 1, 256)).astype(np.float32))
    fmt = LUTFormat("r8", 8, 128, tier)
    tab = bf16_tensor(table_u16)
    q13, q2, W13, W2 = [], [], [], []
    for _ in range(E):
        for rows, cols, qs, Ws in ((2 * I, H, q13, W13), (H, I, q2, W2)):
            idx = rng.integers(0, 256, size=rows * cols, dtype=np.uint8)
            am = O.f32_to_bf16(rng.uniform(0.02, 0.08, (rows * cols + 127) // 128).astype(np.float32))
            qs.append(QuantizedMatrix(fmt, rows, cols, cuda(idx), tab, scales=bf16_tensor(am)))
            Ws.append(O.bf16_to_f32(O.dequant_r(idx, am, table_u16, 128, tier)).reshape(rows, cols))
    return LUTExperts.from_quantized(q13, q2, tab, tc=tc), W13, W2, table_u16
