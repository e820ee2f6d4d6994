"""Checkpoint converter: a bf16 Hugging Face MoE checkpoint -> a LUT checkpoint,
encoded on the GPU.

Drop-in for the reference's ``vllm_lut/convert_checkpoint.py`` and
``vllm_lut/convert_model.py``. It keeps the same:

* command line: ``--model``, ``--output``, ``--code_type BLOCKLUT | NESTEDLUT``
  (convert_checkpoint.py:25-33);
* codebook: ``blocklut_256.npy`` for BLOCKLUT, ``nested_lut_mapped16.npy``
  (falling back to ``blocklut_256.npy``) for NESTEDLUT (convert_model.py:43-52);
* tensor selection: routed-expert ``.weight`` tensors in bf16 are encoded;
  shared experts, dense weights and tensors of other dtypes are copied
  unchanged (convert_model.py:91-108);
* output names: ``<shard>_lut.safetensors``, and the index ``weight_map``
  pointing at them (convert_checkpoint.py:186-201);
* side files copied: ``.json``, ``.py``, ``.txt``, ``.model``, ``.npy``
  (convert_checkpoint.py:203-206, convert_model.py:148-152).

Format R (the reference's format):

* each routed-expert weight is stored under its own name as uint8 indices of
  its original shape (convert_model.py:95-102);
* the per-128 block absmax values, which the reference converters compute
  but never write, go to ``lut_absmax.npz``, keyed by the ``.weight`` names.
  They are stored as float32, exact copies of the bf16 values. This is the
  file ``process_weights_after_loading`` reads (quant_method.py:189-222).

The index file is written after the side files are copied. The reference
copies ``*.json`` last, so there the original index overwrites the remapped
one (convert_checkpoint.py:200-206).

Format B and NestedLUT (``--format b | nested``, ``--bits``, ``--group``):

* each routed-expert weight is stored as packed codes under its name, with
  fp16 tables under ``<proj>.tables``;
* NestedLUT adds ``<proj>.residual`` and ``<proj>.refine``;
* vLLM's expert mapping renames ``experts.<e>.<proj>.`` to ``experts.w13_`` or
  ``experts.w2_``, so these keys load into the ``w13_tables`` / ``w2_tables``
  (…) parameters that ``LUTFusedMoEMethod.create_weights`` registers;
* ``config.json`` gets the ``quantization_config`` that selects the format.

``--from_lut`` starts from a Format R checkpoint instead (this converter's
output or the reference's): each routed-expert weight is dequantised on the
GPU to bf16 and re-encoded to Format B or NestedLUT.

Codebooks stored as uint16 arrays (the NestedLUT ``mapped`` tables) are read as
bf16 bit patterns, as the runtime's tier tables are; the reference converters
cast their integer values instead.

Format R has two encoders, as the two reference scripts do: ``--encoder
quantize`` (the default, ``LUTQuantizer.quantize`` as ``convert_checkpoint.py``
calls it) and ``--encoder fast`` (``fast_encode.encode_lut`` as
``convert_model.py`` calls it: fp32 normalisation against the fp32 codebook).

Encoding runs on the GPU through libblut (``blut_encode_r``,
``blut_encode_lut_f32``, ``blut_encode``).
There is no CPU path: without CUDA the converter raises.
"""
from __future__ import annotations

import argparse
import glob
import json
import os
import shutil
import sys
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch

from .formats import LUTFormat, QuantizedMatrix, dequant, encode, encode_lut_f32, encode_r
from .quantizer import _load_table

SIDE_SUFFIXES = (".json", ".py", ".txt", ".model", ".npy")
INDEX_NAME = "model.safetensors.index.json"
ABSMAX_NAME = "lut_absmax.npz"
BLOCK_SIZE = 128


def parse_args(argv: Optional[List[str]] = None) -> argparse.Namespace:
    p = argparse.ArgumentParser(description="bf16 MoE checkpoint -> LUT checkpoint (GPU encoder)")
    p.add_argument("--model", required=True, help="directory of the bf16 checkpoint")
    p.add_argument("--output", default="", help="output directory (default: <model>_lut)")
    p.add_argument("--code_type", default="BLOCKLUT", choices=["BLOCKLUT", "NESTEDLUT"])
    p.add_argument("--format", default="r", choices=["r", "b", "nested"],
                   help="r: uint8 indices into the global codebook (the reference's format); "
                        "b / nested: packed codes with per-(row, block) fp16 tables")
    p.add_argument("--bits", type=int, default=4, choices=[2, 3, 4], help="Format B index bits")
    p.add_argument("--group", type=int, default=64, choices=[32, 64, 128], help="Format B / NestedLUT block")
    p.add_argument("--tier", default="full", choices=["full", "coarse"], help="NestedLUT tier the config selects")
    p.add_argument("--write_quant_config", action="store_true",
                   help="also write quantization_config for Format R (always written for b / nested)")
    p.add_argument("--from_lut", action="store_true",
                   help="read a Format R checkpoint (uint8 indices, lut_absmax.npz, codebook) instead of a bf16 "
                        "one, and re-encode its routed experts to --format b | nested")
    p.add_argument("--encoder", default="quantize", choices=["quantize", "fast"],
                   help="Format R encoder: quantize = LUTQuantizer.quantize, the rule of convert_checkpoint.py "
                        "(normalised value rounded to bf16); fast = fast_encode.encode_lut, the rule of "
                        "convert_model.py (fp32 normalisation, fp32 codebook)")
    p.add_argument("--device", default="cuda", help="CUDA device of the encoder")
    return p.parse_args(argv)


# ------------------------------------------------------------- host helpers --
def is_routed_expert(name: str) -> bool:
    """Routed-expert tensor names (convert_model.py:91)."""
    return "experts." in name and "shared_expert" not in name


def should_encode(name: str, dtype: torch.dtype) -> bool:
    """Encoded: routed-expert ``.weight`` tensors stored in bf16 (convert_model.py:91-95)."""
    return is_routed_expert(name) and name.endswith(".weight") and dtype == torch.bfloat16


def is_lut_weight(name: str, dtype: torch.dtype, absmax_keys) -> bool:
    """In a Format R checkpoint: a routed-expert ``.weight`` stored as uint8
    indices whose absmax is in ``lut_absmax.npz``."""
    return is_routed_expert(name) and name.endswith(".weight") and dtype == torch.uint8 and name in absmax_keys


def load_codebooks(model_path: str, code_type: str = "BLOCKLUT") -> Dict[str, torch.Tensor]:
    """The codebook files of a checkpoint directory as bf16 tables, keyed
    ``blocklut``, ``mapped16``, ``mapped64`` (convert_checkpoint.py:36-58).
    BLOCKLUT needs ``blocklut_256.npy``. For NESTEDLUT a missing mapped
    table falls back to the BlockLUT table."""
    books: Dict[str, torch.Tensor] = {}
    for fname, key in (("blocklut_256.npy", "blocklut"), ("nested_lut_mapped16.npy", "mapped16"),
                       ("nested_lut_mapped64.npy", "mapped64")):
        path = os.path.join(model_path, fname)
        if os.path.exists(path):
            books[key] = _load_table(path)
    if code_type == "BLOCKLUT" and "blocklut" not in books:
        raise FileNotFoundError(f"blocklut_256.npy not found in {model_path}")
    if code_type == "NESTEDLUT":
        for key in ("blocklut", "mapped16", "mapped64"):
            if key not in books:
                books[key] = books.get("blocklut")
    return books


def codebook_file(model_path: str, code_type: str) -> str:
    """The codebook the reference converter picks (convert_model.py:43-52)."""
    name = "blocklut_256.npy" if code_type == "BLOCKLUT" else "nested_lut_mapped16.npy"
    path = os.path.join(model_path, name)
    if not os.path.exists(path):
        path = os.path.join(model_path, "blocklut_256.npy")
    if not os.path.exists(path):
        raise FileNotFoundError(f"Codebook not found in {model_path}")
    return path


def shard_files(model_path: str) -> List[str]:
    """``model-*.safetensors`` in name order, else ``model.safetensors`` (convert_checkpoint.py:125-131)."""
    files = sorted(glob.glob(os.path.join(model_path, "model-*.safetensors")))
    single = os.path.join(model_path, "model.safetensors")
    if not files and os.path.exists(single):
        files = [single]
    return files


def lut_name(fname: str) -> str:
    """``<shard>_lut.safetensors``; a shard that already has the suffix keeps its name."""
    base = os.path.basename(fname)
    return base if base.endswith("_lut.safetensors") else base.replace(".safetensors", "_lut.safetensors")


def remap_index(index_data: Dict) -> Dict:
    """The index with every shard name replaced by its ``_lut`` file (convert_checkpoint.py:186-194)."""
    return {"metadata": index_data.get("metadata", {}),
            "weight_map": {k: lut_name(v) for k, v in index_data.get("weight_map", {}).items()}}


def side_files(model_path: str) -> List[str]:
    """Files copied beside the shards; the shards and the index are rewritten instead."""
    out = []
    for f in sorted(os.listdir(model_path)):
        if not f.endswith(SIDE_SUFFIXES) or f.startswith("model-") or f in ("model.safetensors", INDEX_NAME):
            continue
        if os.path.isfile(os.path.join(model_path, f)):
            out.append(f)
    return out


def format_of(args: argparse.Namespace) -> Optional[LUTFormat]:
    if args.format == "r":
        return None
    if args.format == "nested":
        return LUTFormat("nested", 4, args.group, 1 if args.tier == "coarse" else 0)
    return LUTFormat("b", args.bits, args.group, 0)


def quant_config(args: argparse.Namespace, output_path: str) -> Dict:
    """``quantization_config`` that makes ``LUTConfig.from_config`` select the converted format."""
    cfg = {"quant_method": "lut", "code_type": args.code_type, "lut_path": os.path.abspath(output_path),
           "block_size": BLOCK_SIZE}
    fmt = format_of(args)
    if fmt is not None:
        cfg.update(codebook_scope="row_block", index_bits=fmt.bits if fmt.kind == "b" else 4, lut_block=fmt.group)
        if fmt.kind == "nested":
            cfg["nested"] = {"coarse_bits": 2, "residual_bits": 2, "tier": args.tier}
    return cfg


def _stem(name: str) -> str:
    return name[:-len(".weight")]


# ---------------------------------------------------------------- encoders --
def quantize_weight(weight: torch.Tensor, codebook: torch.Tensor, device: str = "cuda") -> Tuple[torch.Tensor, torch.Tensor]:
    """Format R encoding of one tensor (convert_checkpoint.py:61-104): returns the
    flat uint8 indices [N] and the bf16 absmax of each flat block of 128 (the
    last one zero-padded), both on the CPU.  Encoded on the GPU."""
    w = weight.to(device=device, dtype=torch.bfloat16)
    idx, absmax = encode_r(w, codebook.to(device), BLOCK_SIZE)
    return idx.cpu(), absmax.cpu()


def fast_encode_weight(weight: torch.Tensor, codebook: torch.Tensor, device: str = "cuda") -> Tuple[torch.Tensor, torch.Tensor]:
    """Format R encoding by convert_model.py's rule (fast_encode.encode_lut with
    the bf16 codebook cast to fp32, convert_model.py:53-61,99): flat uint8
    indices [N] and bf16 absmax per block of 128, on the CPU."""
    w = weight.to(device=device, dtype=torch.bfloat16)
    idx, absmax = encode_lut_f32(w, codebook.to(device=device).float(), BLOCK_SIZE)
    return idx.cpu(), absmax.cpu()


def dequant_lut_weight(idx: torch.Tensor, absmax: np.ndarray, table: torch.Tensor, device: str = "cuda") -> torch.Tensor:
    """A Format R weight (uint8 indices [rows, cols], absmax per flat block of
    128, 256-entry table) back to bf16 [rows, cols] on the GPU, bit-exact
    (quantizer.py:449-477)."""
    rows, cols = idx.shape
    qm = QuantizedMatrix(LUTFormat("r8", 8, BLOCK_SIZE), rows, cols, idx.to(device).contiguous().reshape(-1),
                         table.to(device=device, dtype=torch.bfloat16).contiguous(),
                         scales=torch.from_numpy(np.asarray(absmax, dtype=np.float32)).to(device=device,
                                                                                         dtype=torch.bfloat16))
    return dequant(qm)


def encode_expert(name: str, weight: torch.Tensor, fmt: LUTFormat, device: str = "cuda") -> Dict[str, torch.Tensor]:
    """Format B / NestedLUT encoding of one [rows, cols] expert weight: the
    checkpoint entries (codes under ``name``, tables, NestedLUT residual codes
    and refinement tables under sibling keys)."""
    if weight.dim() != 2 or weight.shape[1] % fmt.group:
        raise ValueError(f"{name}: Format B needs a 2-D weight with cols % {fmt.group} == 0, got {tuple(weight.shape)}")
    qm = encode(weight.to(device=device, dtype=torch.float32), fmt)
    stem = _stem(name)
    out = {name: qm.codes.cpu(), stem + ".tables": qm.tables.cpu()}
    if fmt.kind == "nested":
        out[stem + ".residual"] = qm.codes2.cpu()
        out[stem + ".refine"] = qm.tables2.cpu()
    return out


# -------------------------------------------------------------- converter --
def convert_checkpoint(args: argparse.Namespace) -> Dict:
    """Convert ``args.model`` into ``args.output``; returns counts and sizes."""
    from safetensors import safe_open
    from safetensors.torch import save_file

    if not torch.cuda.is_available():
        raise RuntimeError("convert_checkpoint encodes on the GPU; no CUDA device is available")
    model_path = args.model
    output_path = args.output or (model_path.rstrip("/") + "_lut")
    if os.path.realpath(output_path) == os.path.realpath(model_path):
        raise ValueError("--output must differ from --model: the shards would overwrite their own inputs")
    os.makedirs(output_path, exist_ok=True)
    fmt = format_of(args)
    codebook = _load_table(codebook_file(model_path, args.code_type)) if fmt is None or args.from_lut else None
    src_absmax = None
    if args.from_lut:
        if fmt is None:
            raise ValueError("--from_lut re-encodes a Format R checkpoint: pass --format b or --format nested")
        npz = os.path.join(model_path, ABSMAX_NAME)
        if not os.path.exists(npz):
            raise FileNotFoundError(f"--from_lut needs {ABSMAX_NAME} in {model_path}")
        src_absmax = np.load(npz)
        src_keys = set(src_absmax.files)
    shards = shard_files(model_path)
    if not shards:
        raise FileNotFoundError(f"no safetensors shards in {model_path}")

    stats = {"experts": 0, "copied": 0, "bytes_in": 0, "bytes_out": 0}
    absmax: Dict[str, np.ndarray] = {}
    encoded: List[str] = []
    for ckpt in shards:
        new_state: Dict[str, torch.Tensor] = {}
        with safe_open(ckpt, framework="pt", device="cpu") as f:
            for name in f.keys():
                t = f.get_tensor(name)
                take = is_lut_weight(name, t.dtype, src_keys) if src_absmax is not None else \
                    should_encode(name, t.dtype)
                if not take:
                    new_state[name] = t
                    stats["copied"] += 1
                    continue
                if src_absmax is not None:
                    w = dequant_lut_weight(t, src_absmax[name], codebook, args.device)
                    new_state.update(encode_expert(name, w, fmt, args.device))
                elif fmt is None:
                    enc = fast_encode_weight if getattr(args, "encoder", "quantize") == "fast" else quantize_weight
                    idx, am = enc(t, codebook, args.device)
                    new_state[name] = idx.reshape(t.shape)
                    absmax[name] = am.float().numpy()
                else:
                    new_state.update(encode_expert(name, t, fmt, args.device))
                encoded.append(name)
                stats["experts"] += 1
        out_path = os.path.join(output_path, lut_name(ckpt))
        save_file(new_state, out_path)
        stats["bytes_in"] += os.path.getsize(ckpt)
        stats["bytes_out"] += os.path.getsize(out_path)
        del new_state

    for f in side_files(model_path):
        shutil.copy2(os.path.join(model_path, f), os.path.join(output_path, f))

    index_src = os.path.join(model_path, INDEX_NAME)
    if os.path.exists(index_src):
        with open(index_src) as fh:
            new_index = remap_index(json.load(fh))
        # Format B adds keys (tables, residual codes, refinement tables) beside each encoded weight
        if fmt is not None:
            wm = new_index["weight_map"]
            for k in encoded:
                if k in wm:
                    for suffix in ((".tables", ".residual", ".refine") if fmt.kind == "nested" else (".tables",)):
                        wm[_stem(k) + suffix] = wm[k]
        with open(os.path.join(output_path, INDEX_NAME), "w") as fh:
            json.dump(new_index, fh, indent=2)

    if fmt is None:
        np.savez(os.path.join(output_path, ABSMAX_NAME), **absmax)
    cfg_path = os.path.join(output_path, "config.json")
    if (fmt is not None or args.write_quant_config) and os.path.exists(cfg_path):
        with open(cfg_path) as fh:
            cfg = json.load(fh)
        cfg["quantization_config"] = quant_config(args, output_path)
        with open(cfg_path, "w") as fh:
            json.dump(cfg, fh, indent=2)
    stats["output"] = output_path
    return stats


def main(argv: Optional[List[str]] = None) -> int:
    args = parse_args(argv)
    s = convert_checkpoint(args)
    print(f"converted {s['experts']} expert weights, copied {s['copied']} tensors: "
          f"{s['bytes_in'] / 1e9:.2f} GB -> {s['bytes_out'] / 1e9:.2f} GB in {s['output']}", file=sys.stderr)
    return 0


if __name__ == "__main__":
    sys.exit(main())
