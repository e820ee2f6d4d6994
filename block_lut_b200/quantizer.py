"""Reference-compatible quantiser API (``vllm_lut/quantizer.py``) on libblut kernels.

Same names, arguments and file conventions as the reference:

* ``LUTQuantizer(code_type, block_size, lut_size, device)`` with ``train``,
  ``quantize``, ``decompress``, ``save`` and ``load`` (quantizer.py:30-396);
* ``decompress_blocklut(indices, absmax, codebook, block_size)`` (quantizer.py:449-477);
* ``train_lut_codebook`` and ``quantize_expert_weights`` (quantizer.py:403-446).

``quantize`` and ``decompress`` run the bit-exact CUDA encoder / dequantiser.
Codebook training is offline tooling (the reference's mini-batch k-means,
quantizer.py:120-178) and runs as torch tensor ops on the given device.
"""
from __future__ import annotations

import math
import os
from typing import Dict, Optional, Tuple

import numpy as np
import torch

from . import _lib
from .formats import encode_r


class LUTQuantizer:
    """BlockLUT / NestedLUT quantiser (uint8 index, bf16 absmax per block, bf16[256] codebook)."""

    def __init__(self, code_type: str = "BLOCKLUT", block_size: int = 128, lut_size: int = 256,
                 device: str = "cuda"):
        assert code_type in ("LUT", "BLOCKLUT", "NESTEDLUT"), f"Unsupported code_type: {code_type}"
        self.code_type = code_type
        self.block_size = block_size
        self.lut_size = lut_size
        self.device = device
        self.lut_codebook: Optional[torch.Tensor] = None
        self.nested_mapped64: Optional[torch.Tensor] = None
        self.nested_mapped16: Optional[torch.Tensor] = None

    # ---------------------------------------------------------------- train --
    @torch.no_grad()
    def train(self, expert_weights: torch.Tensor, n_iter: int = 50) -> None:
        """Codebook training (quantizer.py:66-117): block-normalise, then k-means.

        NESTEDLUT also trains the K=64 codebook and merges it to 16.  The
        reference's ``_train_kmeans`` stores every codebook it trains in
        ``lut_codebook``, so after its NESTEDLUT training ``lut_codebook``
        holds the 64 entries (quantizer.py:112-113,177); here it keeps the
        ``lut_size`` codebook, the one ``quantize`` needs.  Both consume the
        same random numbers, so ``nested_mapped64`` / ``nested_mapped16`` are
        the reference's.
        """
        flat = expert_weights.reshape(-1)
        if self.code_type == "LUT":
            self._train_kmeans(flat, self.lut_size, n_iter)
            return
        n = flat.shape[0]
        nb = math.ceil(n / self.block_size)
        if nb * self.block_size != n:
            pad = torch.zeros(nb * self.block_size, dtype=flat.dtype, device=flat.device)
            pad[:n] = flat
            flat = pad
        blocks = flat.view(-1, self.block_size)
        amax = blocks.abs().max(dim=1, keepdim=True).values.clamp(min=1e-10)
        data = (blocks / amax).reshape(-1)
        full = self._train_kmeans(data, self.lut_size, n_iter)
        if self.code_type == "NESTEDLUT":
            c64 = self._train_kmeans(data, 64, n_iter)
            c16 = self._greedy_merge(c64.float(), 16)
            self.nested_mapped64 = self._build_mapped_table(c64.float(), 256)
            self.nested_mapped16 = self._build_mapped_table(c16, 256)
            self.lut_codebook = full

    def _train_kmeans(self, data: torch.Tensor, k: int, n_iter: int, max_samples: int = 200000) -> torch.Tensor:
        """1-D Lloyd k-means (quantizer.py:120-178): a random subset of at most
        ``max_samples`` values, random initial centroids, nearest-centroid
        assignment (first minimum), each non-empty cluster's centroid set to
        its members' mean, centroids sorted and rounded to bf16.  Random
        numbers are drawn in the reference's order (subset, then initial
        centroids) and each mean is a ``Tensor.mean`` of the members in data
        order, so a CPU run under the same ``torch.manual_seed`` reproduces
        the reference's codebook."""
        data = data.to(self.device).float()
        if data.shape[0] > max_samples:
            data = data[torch.randperm(data.shape[0], device=data.device)[:max_samples]]
        n_init = min(k, data.shape[0])
        cent = data[torch.randperm(data.shape[0], device=data.device)[:n_init]].clone()
        if n_init < k:
            cent = torch.cat([cent, torch.zeros(k - n_init, device=data.device)])
        chunk = 1 << 16  # rows of the [n, k] distance matrix held at once
        for _ in range(n_iter):
            a = torch.cat([torch.abs(data[s:s + chunk, None] - cent[None, :]).argmin(dim=1)
                           for s in range(0, data.shape[0], chunk)])
            order = torch.argsort(a, stable=True)       # members of each cluster, in data order
            counts = torch.bincount(a, minlength=k).tolist()
            members = torch.split(data[order], counts)
            for c, m in enumerate(members):
                if m.numel():
                    cent[c] = m.mean()
        cent, _ = torch.sort(cent)
        self.lut_codebook = cent.to(torch.bfloat16).cpu()
        return self.lut_codebook

    def _greedy_merge(self, centroids: torch.Tensor, target_k: int) -> torch.Tensor:
        """Merges centroid pairs to ``target_k`` (quantizer.py:202-221), with the
        reference's distance matrix ``|c_i - c_j| + eye * inf``: its zero
        entries times inf are NaN, so the argmin (which returns the first NaN)
        always picks the pair (0, 1)."""
        c = centroids.clone()
        while c.shape[0] > target_k:
            d = torch.abs(c[None, :] - c[:, None]) + torch.eye(c.shape[0], device=c.device) * float("inf")
            i, j = divmod(int(d.argmin()), c.shape[0])
            c[i] = (c[i] + c[j]) / 2
            c = torch.cat([c[:j], c[j + 1:]])
        return torch.sort(c).values

    def _build_mapped_table(self, centroids: torch.Tensor, table_size: int) -> torch.Tensor:
        reps, rem = divmod(table_size, centroids.shape[0])
        t = centroids.repeat(reps)
        if rem:
            t = torch.cat([t, centroids[:rem]])
        return t.to(torch.bfloat16).cpu()

    # ------------------------------------------------------------- quantize --
    @torch.no_grad()
    def quantize(self, weight: torch.Tensor, codebook: Optional[torch.Tensor] = None) -> Dict[str, torch.Tensor]:
        """BlockLUT-quantise ``weight`` on the GPU (bit-exact with the reference quantiser)."""
        codebook = self.lut_codebook if codebook is None else codebook
        if codebook is None:
            raise RuntimeError("LUT codebook not trained or loaded. Call train() or load() first.")
        if self.code_type == "LUT":
            raise NotImplementedError("code_type LUT (global normalisation) is not on the BlockLUT hot path")
        dev = weight.device if weight.is_cuda else torch.device("cuda")
        idx, absmax = encode_r(weight.to(dev), codebook.to(dev), self.block_size)
        return {"indices": idx.cpu(), "absmax": absmax.cpu(), "codebook": codebook.cpu()}

    @torch.no_grad()
    def decompress(self, indices: torch.Tensor, absmax: torch.Tensor, codebook: torch.Tensor,
                   out_shape: Optional[Tuple[int, ...]] = None) -> torch.Tensor:
        w = decompress_blocklut(indices, absmax, codebook, self.block_size)
        return w.reshape(out_shape) if out_shape is not None else w

    # ------------------------------------------------------------------ I/O --
    def save(self, path: str) -> None:
        os.makedirs(path, exist_ok=True)
        for t, name in ((self.lut_codebook, "blocklut_256.npy"), (self.nested_mapped64, "nested_lut_mapped64.npy"),
                        (self.nested_mapped16, "nested_lut_mapped16.npy")):
            if t is not None:
                np.save(os.path.join(path, name), t.float().numpy() if name == "blocklut_256.npy"
                        else t.view(torch.int16).numpy().view(np.uint16))

    def load(self, path: str) -> bool:
        f = os.path.join(path, "blocklut_256.npy")
        if not os.path.exists(f):
            f = os.path.join(path, "full256.npy")
            if not os.path.exists(f):
                return False
        self.lut_codebook = _load_table(f)
        for attr, fname in (("nested_mapped64", "nested_lut_mapped64.npy"),
                            ("nested_mapped16", "nested_lut_mapped16.npy")):
            fp = os.path.join(path, fname)
            if os.path.exists(fp):
                setattr(self, attr, _load_table(fp))
        return True


def _load_table(path: str) -> torch.Tensor:
    """A codebook .npy as bf16: float arrays are rounded, uint16 arrays are bf16 bit patterns."""
    a = np.load(path)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16)
    return torch.from_numpy(a.astype(np.float32)).to(torch.bfloat16)


def decompress_blocklut(indices: torch.Tensor, absmax: torch.Tensor, codebook: torch.Tensor,
                        block_size: int = 128) -> torch.Tensor:
    """[N] uint8 -> [N] bf16: ``codebook[indices] * absmax[i // block_size]`` on the GPU."""
    dev = indices.device if indices.is_cuda else torch.device("cuda")
    idx = indices.reshape(-1).to(dev).contiguous()
    am = absmax.reshape(-1).to(device=dev, dtype=torch.bfloat16).contiguous()
    cb = codebook.to(device=dev, dtype=torch.bfloat16).contiguous()
    out = torch.empty(idx.numel(), dtype=torch.bfloat16, device=dev)
    with _lib.on_device(out):
        _lib.check(_lib.lib().blut_batch_blocklut_decompress(out.data_ptr(), idx.data_ptr(), am.data_ptr(),
                                                             cb.data_ptr(), 1, idx.numel(), am.numel(), block_size,
                                                             _lib.stream_ptr()), "decompress_blocklut")
    return out


def train_lut_codebook(weights: torch.Tensor, code_type: str = "BLOCKLUT", block_size: int = 128,
                       lut_size: int = 256, n_iter: int = 50) -> LUTQuantizer:
    q = LUTQuantizer(code_type=code_type, block_size=block_size, lut_size=lut_size,
                     device=str(weights.device) if weights.is_cuda else "cuda")
    q.train(weights, n_iter=n_iter)
    return q


def quantize_expert_weights(weights: torch.Tensor, quantizer: LUTQuantizer,
                            code_type: str = "BLOCKLUT") -> Dict[str, torch.Tensor]:
    idx, am = [], []
    for i in range(weights.shape[0]):
        r = quantizer.quantize(weights[i])
        idx.append(r["indices"])
        am.append(r["absmax"])
    return {"indices": torch.stack(idx), "absmax": torch.stack(am), "codebook": quantizer.lut_codebook}


__all__ = ["LUTQuantizer", "decompress_blocklut", "train_lut_codebook", "quantize_expert_weights"]
