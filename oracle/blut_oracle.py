"""CPU oracle for the LUT-dequantised MoE expert forward of block_lut.

TEST INFRASTRUCTURE ONLY.  This module is the checker that the CUDA path is
compared against; it is imported by ``tests/``, ``__graft_entry__.smoke()`` and
the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` and nowhere
else.  The product package (``block_lut_b200``) never imports it and has no CPU
fallback.

It restates, in numpy, the reference algorithm of every function on the hot
path (citations are paths inside the hu-jinzhao/block_lut project):

Format R (the reference's own format, pinned against golden vectors produced
by running the reference's Python code, see ``tests/golden/make_golden.py``):
  * ``dequant_r``      -- ``vllm_lut/quantizer.py:449-477`` (decompress_blocklut),
                          ``vllm_lut/quant_method.py:281-290`` (_decompress_one),
                          ``csrc/kernels/tensor_recover.cu:101-142``.
  * ``encode_r``       -- ``vllm_lut/quantizer.py:243-306`` (quantize: block absmax,
                          bf16 normalisation, first-index argmin).
  * ``tier_index``     -- progressive tiers of ``runtime/model_offload.py:751-758``
                          and ``csrc/tensor_engine/tensor_engine.hpp:287-291``.
  * ``bitplane_pack``, ``bitplane_index`` -- the 3-section bit-plane buffer of
                          ``runtime/model_offload.py:751-758`` and the tier
                          unpacks of ``csrc/kernels/tensor_recover.cu:166-192``
                          and ``csrc/tensor_engine/tensor_engine.cpp:535-547``.
  * ``encode_r`` also equals the reference converter's ``quantize_weight``
                          (``vllm_lut/convert_checkpoint.py:61-104``).
  * ``routing``        -- ``vllm_lut/moe_layer.py:358-376`` and
                          ``customized/qwen.py:44-54`` (softmax -> top-k -> renorm).
  * ``moe_forward``    -- ``vllm_lut/quant_method.py:230-279`` (apply) with the
                          intermediate rounded at the points the CUDA path rounds.

Format B (packed codes into per-(row, block) codebooks) and NestedLUT 2+2 have
no implementation in the reference.  Their definitions here are this build's
restatement of the reference's building blocks -- Lloyd iterations of
``quantizer.py:120-178`` run per (row, block), the argmin assignment of
``quantizer.py:292-296``, the additive coarse+fine value of
``evaluation/explore_additive_lut.py:3-8,72-140`` and the bit-plane packing
convention of ``runtime/model_offload.py:751-758`` (element 0 in the low bits).
PARITY UNPINNED for Format B and for the per-block Lloyd encoders: no
reference test or golden vector exists for them. The NestedLUT reconstruction
rule alone is pinned, by the reference's ``dequantize_additive_lut``
(``evaluation/explore_additive_lut.py:266-276``) run on seeded codes.

bf16 values are carried as uint16 bit patterns (numpy has no bfloat16), fp16
as numpy float16.
"""
from __future__ import annotations

import numpy as np

# ----------------------------------------------------------------------------
# bf16 helpers (round-to-nearest-even, as torch's CPU bf16 arithmetic does)
# ----------------------------------------------------------------------------


def bf16_to_f32(u16: np.ndarray) -> np.ndarray:
    return (np.asarray(u16, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(f: np.ndarray) -> np.ndarray:
    f = np.asarray(f, dtype=np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(f)
    if nan.any():
        r = np.where(nan, np.uint16(0x7FC0), r)
    return r


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to ``dtype`` ('f16' | 'bf16' | 'f32') and back to float32."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "bf16":
        return bf16_to_f32(f32_to_bf16(x))
    return x


# ----------------------------------------------------------------------------
# Format R: uint8 index per weight, global 256-entry bf16 codebook, bf16
# absmax per `block_size` flat elements.
# ----------------------------------------------------------------------------


def tier_index(idx: np.ndarray, tier: int) -> np.ndarray:
    """Index read at a progressive tier (model_offload.py:751-758 planes).

    Tier 0 reads all 8 bits (full table), tier 1 the low4 | mid2 << 4 planes
    (mapped64 table), tier 2 only the low4 plane (mapped16 table).
    """
    idx = np.asarray(idx, dtype=np.uint8)
    if tier == 0:
        return idx
    if tier == 1:
        return idx & np.uint8(0x3F)
    if tier == 2:
        return idx & np.uint8(0x0F)
    raise ValueError(f"tier {tier}")


def bitplane_pack(idx: np.ndarray) -> np.ndarray:
    """Progressive 3-section bit-plane buffer of n uint8 indices, n % 4 == 0
    (runtime/model_offload.py:751-758): [low4 | mid2 | high2], where

    * low4  [n/2]: byte q holds element 2q in bits 0-3 and 2q+1 in bits 4-7;
    * mid2  [n/4]: byte q holds bits 4-5 of element 4q+j in bits 2j..2j+1;
    * high2 [n/4]: the same for bits 6-7.
    """
    quads = np.asarray(idx, dtype=np.uint8).reshape(-1, 4).astype(np.uint32)
    low = (quads[:, 0::2] & 0xF) | ((quads[:, 1::2] & 0xF) << 4)   # 2 bytes per quad
    sh = np.arange(0, 8, 2, dtype=np.uint32)
    mid = (((quads >> 4) & 3) << sh).sum(axis=1)
    high = ((quads >> 6) << sh).sum(axis=1)
    return np.concatenate([low.reshape(-1), mid, high]).astype(np.uint8)


def bitplane_index(planes: np.ndarray, n: int, tier: int) -> np.ndarray:
    """The index a tier reads back from the first bytes of a bit-plane buffer.

    Tier 2 reads the low section (n/2 bytes), tier 1 low + mid (3n/4), tier 0
    all n bytes (tensor_engine.cpp:505-509). The index is low | mid << 4 |
    high << 6 over the sections read. This is the tier-2 GPU unpack of
    tensor_recover.cu:166-192 and the tier-1 host unpack of
    tensor_engine.cpp:535-547, so it equals ``tier_index(idx, tier)``.
    """
    planes = np.asarray(planes, dtype=np.uint8)
    assert n % 4 == 0 and planes.size >= {2: n // 2, 1: 3 * n // 4, 0: n}[tier]
    lo = planes[: n // 2]
    out = np.stack([lo & 0xF, lo >> 4], axis=1).reshape(-1)
    sh = np.arange(0, 8, 2, dtype=np.uint8)
    if tier <= 1:
        out |= (((planes[n // 2: 3 * n // 4, None] >> sh) & 3) << 4).reshape(-1).astype(np.uint8)
    if tier == 0:
        out |= (((planes[3 * n // 4: n, None] >> sh) & 3) << 6).reshape(-1).astype(np.uint8)
    return out


def dequant_r(idx: np.ndarray, absmax_bf16: np.ndarray, table_bf16: np.ndarray,
              block_size: int = 128, tier: int = 0) -> np.ndarray:
    """bf16(f32(table[idx[i]]) * f32(absmax[min(i // bs, nb - 1)])) as bf16 bits.

    quantizer.py:471-477: ``codebook[indices.long()] * absmax[block_id]`` in bf16;
    the product of two bf16 values is exact in float32, so one RNE rounding
    reproduces torch's CPU result.
    """
    flat = tier_index(np.asarray(idx).reshape(-1), tier)
    absmax_bf16 = np.asarray(absmax_bf16, dtype=np.uint16).reshape(-1)
    nb = absmax_bf16.shape[0]
    blk = np.minimum(np.arange(flat.shape[0]) // block_size, nb - 1)
    v = bf16_to_f32(np.asarray(table_bf16, dtype=np.uint16)[flat]) * bf16_to_f32(absmax_bf16[blk])
    return f32_to_bf16(v).reshape(np.asarray(idx).shape)


def encode_r(w_bf16: np.ndarray, table_bf16: np.ndarray, block_size: int = 128):
    """Reference BlockLUT quantiser (quantizer.py:243-306) on bf16 input.

    absmax = max |w| over the flat block (exact in bf16), clamped at
    bf16(1e-10); normalised = bf16(w / absmax); index = first argmin over the
    256 entries of |f32(normalised) - f32(table)|.  Returns (idx u8 [N],
    absmax bf16 [nb]).
    """
    w = np.asarray(w_bf16, dtype=np.uint16).reshape(-1)
    n = w.shape[0]
    nb = (n + block_size - 1) // block_size
    wp = np.zeros(nb * block_size, dtype=np.uint16)
    wp[:n] = w
    wf = bf16_to_f32(wp).reshape(nb, block_size)
    amax = np.abs(wf).max(axis=1)
    amax = np.maximum(amax, bf16_to_f32(f32_to_bf16(np.float32(1e-10))))
    amax_b = f32_to_bf16(amax)
    norm = bf16_to_f32(f32_to_bf16(wf / bf16_to_f32(amax_b)[:, None])).reshape(-1)
    cb = bf16_to_f32(np.asarray(table_bf16, dtype=np.uint16))
    idx = np.empty(norm.shape[0], dtype=np.uint8)
    step = 1 << 16
    for s in range(0, norm.shape[0], step):
        d = np.abs(norm[s:s + step, None] - cb[None, :])
        idx[s:s + step] = np.argmin(d, axis=1).astype(np.uint8)
    return idx[:n], amax_b


def encode_lut_f32(w_bf16: np.ndarray, codebook_f32: np.ndarray, block_size: int = 128):
    """The fast GPU encoder's rule (vllm_lut/fast_encode.py:22-102), with the
    exact division its own check compares against (fast_encode.py:205-221).

    absmax = max(max |w| over the flat block, 1e-10) in fp32; normalised =
    f32(w) / absmax in fp32 (not rounded to bf16); index = first argmin of
    |normalised - codebook| over the fp32 codebook.  The stored absmax is
    bf16(absmax).  Returns (idx u8 [N], absmax bf16 [nb]).
    """
    w = np.asarray(w_bf16, dtype=np.uint16).reshape(-1)
    n = w.shape[0]
    nb = (n + block_size - 1) // block_size
    wp = np.zeros(nb * block_size, dtype=np.uint16)
    wp[:n] = w
    wf = bf16_to_f32(wp).reshape(nb, block_size)
    amax = np.maximum(np.abs(wf).max(axis=1), np.float32(1e-10)).astype(np.float32)
    norm = (wf / amax[:, None]).astype(np.float32).reshape(-1)
    cb = np.asarray(codebook_f32, dtype=np.float32)
    idx = np.empty(norm.shape[0], dtype=np.uint8)
    step = 1 << 16
    for s in range(0, norm.shape[0], step):
        d = np.abs(norm[s:s + step, None] - cb[None, :])
        idx[s:s + step] = np.argmin(d, axis=1).astype(np.uint8)
    return idx[:n], f32_to_bf16(amax)


# ----------------------------------------------------------------------------
# Format B: packed b-bit codes, one sorted fp16 codebook of 2**b entries per
# (row, block of g elements along K).  NestedLUT: 2-bit coarse code into a
# 4-entry per-block table plus a 2-bit residual code into a 4x4 per-block
# refinement table; value = fp16(coarse[c] + refine[c][r]).
# ----------------------------------------------------------------------------


def pack_codes(codes: np.ndarray, bits: int) -> np.ndarray:
    """Pack [N, K] codes (< 2**bits) into a little-endian bit stream per row.

    Element k of a row occupies bits [k*bits, (k+1)*bits) of the row's byte
    string, least significant bit first -- the convention of the reference's
    bit-plane files (model_offload.py:753-756: element 0 in the low nibble /
    low bit pair).  Requires K * bits % 8 == 0.
    """
    codes = np.asarray(codes, dtype=np.uint8)
    n, k = codes.shape
    assert (k * bits) % 8 == 0
    bitarr = ((codes[:, :, None] >> np.arange(bits, dtype=np.uint8)) & 1).reshape(n, k * bits)
    return np.packbits(bitarr, axis=1, bitorder="little")


def unpack_codes(packed: np.ndarray, bits: int, k: int) -> np.ndarray:
    packed = np.asarray(packed, dtype=np.uint8)
    n = packed.shape[0]
    bitarr = np.unpackbits(packed, axis=1, bitorder="little")[:, : k * bits].reshape(n, k, bits)
    w = (1 << np.arange(bits)).astype(np.uint16)
    return (bitarr.astype(np.uint16) * w).sum(axis=2).astype(np.uint8)


def dequant_b(packed: np.ndarray, tables: np.ndarray, bits: int, group: int) -> np.ndarray:
    """w[n, k] = tables[n, k // g, code(n, k)] (fp16, a pure lookup)."""
    tables = np.asarray(tables, dtype=np.float16)
    n, nblk, ent = tables.shape
    assert ent == 1 << bits
    k = nblk * group
    codes = unpack_codes(packed, bits, k).astype(np.int64)
    rows = np.arange(n)[:, None]
    blk = (np.arange(k) // group)[None, :]
    return tables[rows, blk, codes]


def nested_combined_table(coarse_t: np.ndarray, refine_t: np.ndarray) -> np.ndarray:
    """16-entry table t[c * 4 + r] = fp16(f32(coarse[c]) + f32(refine[c][r])).

    float32 holds every fp16 sum with >= 2p+2 bits, so the float add followed
    by one RNE rounding to fp16 equals a correctly rounded fp16 add.
    """
    c = np.asarray(coarse_t, dtype=np.float16).astype(np.float32)
    r = np.asarray(refine_t, dtype=np.float16).astype(np.float32)
    n, nb = c.shape[:2]
    r = r.reshape(n, nb, 4, 4)
    return (c[:, :, :, None] + r).astype(np.float16).reshape(n, nb, 16)


def dequant_nested(coarse_packed, resid_packed, coarse_t, refine_t, group: int,
                   coarse_only: bool = False) -> np.ndarray:
    coarse_t = np.asarray(coarse_t, dtype=np.float16)
    n, nb, _ = coarse_t.shape
    k = nb * group
    c = unpack_codes(coarse_packed, 2, k).astype(np.int64)
    rows = np.arange(n)[:, None]
    blk = (np.arange(k) // group)[None, :]
    if coarse_only:
        return coarse_t[rows, blk, c]
    r = unpack_codes(resid_packed, 2, k).astype(np.int64)
    comb = nested_combined_table(coarse_t, refine_t)
    return comb[rows, blk, c * 4 + r]


# ---------------------------------------------------------------- encoders ---

_LLOYD_ITERS = 10


def _lane_tree_sum(v: np.ndarray) -> np.ndarray:
    """Sum over the last axis (length g in {32, 64, 128}) in the order a warp uses.

    Lane l first adds its elements l, l+32, l+64, ... in order, then the 32
    lane partials are combined by a xor butterfly with offsets 16, 8, 4, 2, 1.
    float32 throughout, so the GPU encoder reproduces the sums bit for bit.
    """
    v = np.asarray(v, dtype=np.float32)
    g = v.shape[-1]
    per = g // 32
    lanes = v.reshape(v.shape[:-1] + (per, 32))
    p = lanes[..., 0, :].copy()
    for j in range(1, per):
        p = (p + lanes[..., j, :]).astype(np.float32)
    lane = np.arange(32)
    for off in (16, 8, 4, 2, 1):
        p = (p + p[..., lane ^ off]).astype(np.float32)
    return p[..., 0]


def _nearest(v: np.ndarray, cent: np.ndarray) -> np.ndarray:
    """First index of the minimum |v - c| (ties -> lowest index), float32."""
    d = np.abs(v[..., :, None] - cent[..., None, :]).astype(np.float32)
    return np.argmin(d, axis=-1)


def lloyd_blocks(v: np.ndarray, n_cent: int, iters: int = _LLOYD_ITERS,
                 mask: np.ndarray | None = None):
    """Per-block 1-D Lloyd k-means (quantizer.py:120-178 run per block).

    ``v``: float32 [..., g].  Initial centroids lie on a uniform grid over
    [min, max] of the block's (masked) values: c_i = lo + (hi - lo) * ((2i+1) /
    (2 n_cent)).  Each iteration assigns every value to its nearest centroid
    (lowest index on ties) and moves each non-empty centroid to the float32
    mean of its values (sum in warp order, then IEEE division).  Returns the
    float32 centroids [..., n_cent] (not yet sorted or rounded).
    """
    v = np.asarray(v, dtype=np.float32)
    if mask is None:
        mask = np.ones(v.shape, dtype=bool)
    big = np.float32(3.0e38)
    lo = np.where(mask, v, big).min(axis=-1)
    hi = np.where(mask, v, -big).max(axis=-1)
    empty = ~mask.any(axis=-1)
    lo = np.where(empty, np.float32(0), lo).astype(np.float32)
    hi = np.where(empty, np.float32(0), hi).astype(np.float32)
    frac = ((2 * np.arange(n_cent) + 1) / np.float32(2 * n_cent)).astype(np.float32)
    span = (hi - lo).astype(np.float32)
    cent = (lo[..., None] + (span[..., None] * frac).astype(np.float32)).astype(np.float32)
    for _ in range(iters):
        a = _nearest(v, cent)
        for i in range(n_cent):
            sel = (a == i) & mask
            s = _lane_tree_sum(np.where(sel, v, np.float32(0)))
            cnt = sel.sum(axis=-1).astype(np.float32)
            upd = cnt > 0
            mean = (s / np.where(upd, cnt, np.float32(1))).astype(np.float32)
            cent[..., i] = np.where(upd, mean, cent[..., i])
    return cent


def encode_b(w: np.ndarray, bits: int, group: int, iters: int = _LLOYD_ITERS):
    """Format B encoder: per (row, block) Lloyd, fp16 sorted table, argmin codes.

    Returns (packed u8 [N, K*bits/8], tables fp16 [N, K/g, 2**bits]).
    """
    w = np.asarray(w, dtype=np.float32)
    n, k = w.shape
    assert k % group == 0 and group % 32 == 0
    v = w.reshape(n, k // group, group)
    cent = lloyd_blocks(v, 1 << bits, iters)
    t16 = np.sort(cent.astype(np.float16), axis=-1, kind="stable")
    codes = _nearest(v, t16.astype(np.float32)).astype(np.uint8).reshape(n, k)
    return pack_codes(codes, bits), t16


def encode_nested(w: np.ndarray, group: int, iters: int = _LLOYD_ITERS):
    """NestedLUT 2+2 encoder.

    Coarse: 4-entry per-block Lloyd table (as ``encode_b`` with bits=2).
    Refinement: for each coarse code c, a 4-entry Lloyd table over the
    residuals v - coarse[c] of the block's values whose coarse code is c
    (zeros when none).  The residual code minimises |v - fp16(coarse[c] +
    refine[c][r])| (lowest r on ties).
    Returns (coarse_packed, resid_packed, coarse_t [N,nb,4], refine_t [N,nb,16]).
    """
    w = np.asarray(w, dtype=np.float32)
    n, k = w.shape
    nb = k // group
    v = w.reshape(n, nb, group)
    cent = lloyd_blocks(v, 4, iters)
    ct = np.sort(cent.astype(np.float16), axis=-1, kind="stable")
    c = _nearest(v, ct.astype(np.float32))
    cv = np.take_along_axis(ct.astype(np.float32), c, axis=-1)
    e = (v - cv).astype(np.float32)
    rt = np.zeros((n, nb, 4, 4), dtype=np.float16)
    for ci in range(4):
        m = c == ci
        rc = lloyd_blocks(e, 4, iters, mask=m)
        rc = np.where(m.any(axis=-1)[..., None], rc, np.float32(0))
        rt[:, :, ci, :] = np.sort(rc.astype(np.float16), axis=-1, kind="stable")
    comb = nested_combined_table(ct, rt.reshape(n, nb, 16)).astype(np.float32).reshape(n, nb, 4, 4)
    # cand[n, b, i, r] = combined value of element i for residual code r
    cand = comb[np.arange(n)[:, None, None], np.arange(nb)[None, :, None], c]
    r = np.argmin(np.abs(v[..., None] - cand).astype(np.float32), axis=-1)
    return (pack_codes(c.reshape(n, k).astype(np.uint8), 2),
            pack_codes(r.reshape(n, k).astype(np.uint8), 2),
            ct, rt.reshape(n, nb, 16))


# ----------------------------------------------------------------------------
# Router and MoE layer
# ----------------------------------------------------------------------------


def routing(logits: np.ndarray, top_k: int, renorm: bool = False):
    """softmax(float32) -> top-k (descending, lowest expert index on ties) -> renorm.

    moe_layer.py:373-376 and customized/qwen.py:44-54.  Weights are returned
    in float32 (the caller rounds to its activation dtype if it wants to).
    """
    z = np.asarray(logits, dtype=np.float64)
    z = z - z.max(axis=-1, keepdims=True)
    p = np.exp(z)
    p = (p / p.sum(axis=-1, keepdims=True)).astype(np.float32)
    order = np.argsort(-p, axis=-1, kind="stable")[:, :top_k]
    w = np.take_along_axis(p, order, axis=-1)
    if renorm:
        w = (w / w.sum(axis=-1, keepdims=True)).astype(np.float32)
    return order.astype(np.int32), w.astype(np.float32)


def silu(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.float64)
    return x / (1.0 + np.exp(-x))


def _expert(w, e):
    """Expert e of a stacked array, or of a callable e -> array (lazy dequant)."""
    return np.asarray(w(e) if callable(w) else w[e], dtype=np.float64)


def moe_forward(x: np.ndarray, topk_ids: np.ndarray, topk_w: np.ndarray,
                w13, w2, act_dtype: str = "f16",
                shared13: np.ndarray | None = None, shared2: np.ndarray | None = None,
                shared_gate: np.ndarray | None = None) -> np.ndarray:
    """Routed-expert MoE forward in float64 with the CUDA path's rounding points.

    For each token t and slot j with expert e = topk_ids[t, j]:
      h = W13[e] x_t ; a = round_act(silu(h[:I]) * h[I:]) ; y = W2[e] a
      out_t += topk_w[t, j] * y
    (quant_method.py:262-277: gate/up projection, SiLU(gate) * up, down
    projection, weighted scatter-add).  ``w13``: [E, 2I, H] dequantised
    weights, ``w2``: [E, H, I] (or callables e -> matrix).  The optional shared expert adds
    sigmoid(x . shared_gate) * W2s(silu(W1s x) * W3s x) (customized/qwen.py:89-100).
    Returns float64 [T, H]; the caller rounds to the output dtype.
    """
    x = np.asarray(x, dtype=np.float64)
    t_n, h_n = x.shape
    out = np.zeros((t_n, h_n), dtype=np.float64)
    ids = np.asarray(topk_ids)
    for e in np.unique(ids):
        tok, slot = np.nonzero(ids == e)
        xe = x[tok]
        w13e = _expert(w13, e)
        inter = w13e.shape[0] // 2
        h = xe @ w13e.T
        a = round_to((silu(h[:, :inter]) * h[:, inter:]).astype(np.float32), act_dtype).astype(np.float64)
        y = a @ _expert(w2, e).T
        # np.add.at: a token that names the same expert in two slots gets both
        np.add.at(out, tok, np.asarray(topk_w, dtype=np.float64)[tok, slot][:, None] * y)
    if shared13 is not None:
        si = shared13.shape[0] // 2
        h = x @ np.asarray(shared13, dtype=np.float64).T
        a = round_to((silu(h[:, :si]) * h[:, si:]).astype(np.float32), act_dtype).astype(np.float64)
        y = a @ np.asarray(shared2, dtype=np.float64).T
        g = 1.0 / (1.0 + np.exp(-(x @ np.asarray(shared_gate, dtype=np.float64).reshape(-1))))
        out += g[:, None] * y
    return out


def moe_forward_threaded(x: np.ndarray, topk_ids: np.ndarray, topk_w: np.ndarray, w13, w2,
                         act_dtype: str = "f16", threads: int = 1) -> np.ndarray:
    """``moe_forward`` with the active experts spread over a thread pool (numpy
    releases the GIL in the gathers and BLAS calls).  The CPU baseline leg of
    bench.py times this: per expert, table-gather dequant then matmuls."""
    from concurrent.futures import ThreadPoolExecutor

    x = np.asarray(x, dtype=np.float64)
    ids = np.asarray(topk_ids)

    def one(e):
        tok, slot = np.nonzero(ids == e)
        w13e = _expert(w13, e)
        inter = w13e.shape[0] // 2
        h = x[tok] @ w13e.T
        a = round_to((silu(h[:, :inter]) * h[:, inter:]).astype(np.float32), act_dtype).astype(np.float64)
        return tok, np.asarray(topk_w, dtype=np.float64)[tok, slot][:, None] * (a @ _expert(w2, e).T)

    out = np.zeros_like(x)
    with ThreadPoolExecutor(max_workers=max(1, threads)) as ex:
        for tok, y in ex.map(one, list(np.unique(ids))):
            np.add.at(out, tok, y)
    return out


def moe_forward_reference_bf16(x: np.ndarray, topk_ids: np.ndarray, topk_w: np.ndarray,
                               w13, w2) -> np.ndarray:
    """The reference's ``apply`` (quant_method.py:262-277) with its bf16 rounding.

    Every torch op of the reference rounds its result to bf16: the gate/up
    ``F.linear`` (float accumulation), ``F.silu(gate)``, ``* up``, the down
    ``F.linear``, ``expert_out * w`` and the ``out[m] +=`` accumulation, in the
    reference's loop order (unique experts ascending, then slot k).  Used to
    pin this oracle bit-exactly against the reference's recorded outputs.
    """
    bf = lambda a: round_to(np.asarray(a, dtype=np.float32), "bf16")  # noqa: E731
    x = np.asarray(x, dtype=np.float32)
    out = np.zeros_like(x)
    ids = np.asarray(topk_ids)
    tw = np.asarray(topk_w, dtype=np.float32)
    for e in np.unique(ids):
        w13e = _expert(w13, e)
        inter = w13e.shape[0] // 2
        gu = bf(x.astype(np.float64) @ w13e.T)
        a = bf(bf(silu(gu[:, :inter])) * gu[:, inter:])
        y = bf(a.astype(np.float64) @ _expert(w2, e).T)
        for k in range(ids.shape[1]):
            m = ids[:, k] == e
            out[m] = bf(out[m] + bf(y[m] * tw[m, k][:, None]))
    return out


# ----------------------------------------------------------------------------
# Synthetic inputs of the benchmark configs: Student-t(df=5) weights scaled to std
# 0.02, N(0,1) activations RMS-normalised per token.
# ----------------------------------------------------------------------------


def student_t_weights(rng: np.random.Generator, shape, std: float = 0.02) -> np.ndarray:
    df = 5.0
    scale = std / np.sqrt(df / (df - 2.0))
    return (rng.standard_t(df, size=shape) * scale).astype(np.float32)


def rms_activations(rng: np.random.Generator, t: int, h: int) -> np.ndarray:
    x = rng.standard_normal((t, h)).astype(np.float32)
    x = x / np.sqrt((x.astype(np.float64) ** 2).mean(axis=1, keepdims=True)).astype(np.float32)
    return x


def rel_l2(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
