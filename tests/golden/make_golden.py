"""Generate the golden fixtures in this folder by running the reference's code.

Run once, in a container that has the block_lut reference checkout and vLLM
installed (CPU is enough):

    python tests/golden/make_golden.py /path/to/block_lut

It imports the reference's own ``vllm_lut.quantizer`` and
``vllm_lut.quant_method`` and records their outputs on seeded inputs:

* ``dequant_kat.npz``  -- the decompress known-answer test of
  ``vllm_lut/cuda/build_lut_kernel.py:142-198`` (N=4096, seed 42,
  linspace(-3, 3, 256) codebook, block 128), expected values from the
  reference's ``decompress_blocklut`` (``vllm_lut/quantizer.py:449-477``).
* ``encode_r.npz``     -- ``LUTQuantizer.quantize`` (``quantizer.py:243-306``) with
  the shipped Qwen codebook ``models/qwen/blocklut_256.npy`` on Student-t
  weights, and ``LUTQuantizer.decompress`` of the result.
* ``tiers.npz``        -- ``decompress_blocklut`` through the shipped NestedLUT
  tables ``models/qwen/nested_lut_mapped{64,16}.npy`` at the tier indices of
  ``runtime/model_offload.py:751-758``.
* ``routing.npz``      -- ``vllm_lut.moe_layer._routing`` (``moe_layer.py:358-376``).
* ``apply_small.npz``  -- ``LUTFusedMoEMethod.apply`` (``quant_method.py:230-279``)
  on a small layer (E=8, H=256, I=128, top-2) at T=2 and T=8; the uint8
  indices are regenerated from a stored seed, everything else is stored.
* ``convert_r.npz``    -- the reference converter's encoder ``quantize_weight``
  (``vllm_lut/convert_checkpoint.py:61-104``) with the shipped Qwen codebook,
  on a bf16 matrix of 8000 elements (a zero-padded tail block) whose first
  block is all zeros (the absmax clamp).  ``python make_golden.py <ref> convert``
  regenerates only this file.
* ``bitplane.npz``     -- the progressive bit-plane buffer of
  ``runtime/model_offload.py:751-758``. The reference's own
  ``split_and_extract_from_tensor`` is lifted from that file's source with
  ``ast``, because the module imports a compiled extension, and run on seeded
  indices (n = 4100) with three file chunks. ``python make_golden.py <ref>
  bitplane`` regenerates only this file.
* ``additive.npz``     -- ``dequantize_additive_lut``
  (``evaluation/explore_additive_lut.py:266-276``), the reference's additive
  two-table reconstruction (coarse[c] + fine[f]) times absmax, on seeded
  codes. Its tables are dyadic, so every sum is exact in fp16, and its absmax
  is 1. ``python make_golden.py <ref> additive`` regenerates only this file.
* ``apply_qwen.npz``   -- ``apply`` on a Qwen1.5-MoE-shaped layer (E=60, H=2048,
  I=1408, top-4, T=8).  The 519 MB of weights are not stored: they are
  regenerated from the stored seed with numpy's PCG64 integer stream (stable
  across platforms), and their SHA-256 is stored to detect drift.

bf16 tensors are stored as uint16 bit patterns.
"""
from __future__ import annotations

import hashlib
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def bits(t):
    import torch
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def qwen_layer_weights(seed, e, h, i):
    """Deterministic Format-R weights for the Qwen-shaped apply fixture."""
    rng = np.random.Generator(np.random.PCG64(seed))
    w13 = rng.integers(0, 256, size=(e, 2 * i, h), dtype=np.uint8)
    w2 = rng.integers(0, 256, size=(e, h, i), dtype=np.uint8)
    # absmax values: bf16 patterns of numbers in [0.03, 0.12)
    a13 = rng.integers(0, 1 << 16, size=(e, 2 * i * h // 128), dtype=np.uint32)
    a2 = rng.integers(0, 1 << 16, size=(e, h * i // 128), dtype=np.uint32)
    lo, hi = 0.03, 0.12

    def to_absmax(u):
        f = (lo + (hi - lo) * (u.astype(np.float64) / 65536.0)).astype(np.float32)
        return (f.view(np.uint32) >> 16).astype(np.uint16)  # truncation: exact, deterministic

    x_u = rng.integers(0, 1 << 16, size=(8, h), dtype=np.uint32)
    return w13, w2, to_absmax(a13), to_absmax(a2), x_u


def small_layer_indices(seed, e, h, i):
    """uint8 indices of the small apply fixture (regenerated, not stored)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    return (rng.integers(0, 256, size=(e, 2 * i, h), dtype=np.uint8),
            rng.integers(0, 256, size=(e, h, i), dtype=np.uint8))


def sha(*arrs):
    m = hashlib.sha256()
    for a in arrs:
        m.update(np.ascontiguousarray(a).tobytes())
    return m.hexdigest()


def main(ref_root):
    sys.path.insert(0, ref_root)
    import torch
    import torch.nn.functional as F  # noqa: F401
    from types import SimpleNamespace
    from vllm_lut import quantizer as Q
    from vllm_lut.quant_method import LUTConfig, LUTFusedMoEMethod
    from vllm_lut.moe_layer import _routing

    torch.set_num_threads(os.cpu_count() or 1)

    # 1. decompress KAT (build_lut_kernel.py:142-198), CPU generator
    torch.manual_seed(42)
    n, bs = 4096, 128
    orig = torch.randn(n, dtype=torch.bfloat16)
    blocks = orig.reshape(-1, bs)
    absmax, _ = blocks.abs().max(dim=1, keepdim=True)
    absmax = absmax.clamp(min=1e-10)
    normalized = blocks / absmax
    codebook = torch.linspace(-3, 3, 256, dtype=torch.bfloat16)
    dists = torch.abs(normalized.reshape(-1).float().unsqueeze(1) - codebook.float().unsqueeze(0))
    indices = dists.argmin(dim=1).to(torch.uint8)
    expected = Q.decompress_blocklut(indices, absmax.reshape(-1), codebook, bs)
    np.savez_compressed(os.path.join(HERE, "dequant_kat.npz"),
                        idx=indices.numpy(), absmax=bits(absmax.reshape(-1)),
                        table=bits(codebook), expected=bits(expected), block_size=bs)

    # 2. encoder + decompress with the shipped Qwen codebook
    cb = torch.from_numpy(np.load(os.path.join(ref_root, "models/qwen/blocklut_256.npy"))).to(torch.bfloat16)
    rng = np.random.Generator(np.random.PCG64(0))
    df = 5.0
    w = (rng.standard_t(df, size=(96, 384)) * (0.02 / np.sqrt(df / (df - 2)))).astype(np.float32)
    wb = torch.from_numpy(w).to(torch.bfloat16)
    qz = Q.LUTQuantizer(code_type="BLOCKLUT", block_size=128, device="cpu")
    res = qz.quantize(wb, cb)
    deq = qz.decompress(res["indices"], res["absmax"], cb)
    np.savez_compressed(os.path.join(HERE, "encode_r.npz"),
                        w=bits(wb), table=bits(cb), idx=res["indices"].numpy(),
                        absmax=bits(res["absmax"]), dequant=bits(deq))

    # 3. NestedLUT tier tables (bf16 bit patterns shipped as uint16 .npy)
    m64 = np.load(os.path.join(ref_root, "models/qwen/nested_lut_mapped64.npy")).astype(np.uint16)
    m16 = np.load(os.path.join(ref_root, "models/qwen/nested_lut_mapped16.npy")).astype(np.uint16)
    t64 = torch.from_numpy(m64.view(np.int16)).view(torch.bfloat16)
    t16 = torch.from_numpy(m16.view(np.int16)).view(torch.bfloat16)
    idx = res["indices"]
    tier_out = {}
    for tier, (mask, tab) in {1: (0x3F, t64), 2: (0x0F, t16)}.items():
        ti = (idx & mask).to(torch.uint8)
        tier_out[f"tier{tier}"] = bits(Q.decompress_blocklut(ti, res["absmax"], tab, 128))
    np.savez_compressed(os.path.join(HERE, "tiers.npz"), idx=idx.numpy(), absmax=bits(res["absmax"]),
                        full=bits(cb), mapped64=m64, mapped16=m16, **tier_out)

    # 4. routing
    g = torch.Generator().manual_seed(7)
    logits32 = torch.randn(16, 60, generator=g) * 2.0
    w32, i32 = _routing(logits32, 4)
    logits16 = (torch.randn(16, 128, generator=g) * 2.0).to(torch.bfloat16)
    w16, i16 = _routing(logits16, 8)
    np.savez_compressed(os.path.join(HERE, "routing.npz"),
                        logits_f32=logits32.numpy(), w_f32=w32.numpy(), ids_f32=i32.numpy(),
                        logits_bf16=bits(logits16), w_bf16=bits(w16), ids_bf16=i16.numpy())

    method = LUTFusedMoEMethod(LUTConfig(code_type="BLOCKLUT"))

    def run_apply(layer, x, tw, ti):
        LUTFusedMoEMethod._cached = {}
        with torch.no_grad():
            return method.apply(layer, x, tw, ti)

    # 5. small apply (all inputs stored)
    e_n, h_n, i_n, k = 8, 256, 128, 2
    w13, w2 = small_layer_indices(11, e_n, h_n, i_n)
    rng = np.random.Generator(np.random.PCG64(1))
    a13 = torch.from_numpy(rng.uniform(0.03, 0.12, size=(e_n, 2 * i_n * h_n // 128)).astype(np.float32)).to(torch.bfloat16)
    a2 = torch.from_numpy(rng.uniform(0.03, 0.12, size=(e_n, h_n * i_n // 128)).astype(np.float32)).to(torch.bfloat16)
    layer = SimpleNamespace(w13_weight=torch.from_numpy(w13), w2_weight=torch.from_numpy(w2),
                            w13_absmax=a13, w2_absmax=a2, _codebook=cb)
    small = {"idx_seed": 11, "sha": sha(w13, w2), "a13": bits(a13), "a2": bits(a2), "table": bits(cb)}
    for t_n in (2, 8):
        x = torch.from_numpy(rng.standard_normal((t_n, h_n)).astype(np.float32)).to(torch.bfloat16)
        logits = torch.from_numpy(rng.standard_normal((t_n, e_n)).astype(np.float32))
        tw, ti = _routing(logits, k)
        tw = tw.to(torch.bfloat16)
        out = run_apply(layer, x, tw, ti)
        small.update({f"x{t_n}": bits(x), f"tw{t_n}": bits(tw), f"ti{t_n}": ti.numpy().astype(np.int32),
                      f"out{t_n}": bits(out)})
    np.savez_compressed(os.path.join(HERE, "apply_small.npz"), **small)

    # 6. Qwen-shaped apply, weights regenerated from the seed
    seed = 20260101
    e_n, h_n, i_n, k, t_n = 60, 2048, 1408, 4, 8
    w13, w2, a13, a2, x_u = qwen_layer_weights(seed, e_n, h_n, i_n)
    x = torch.from_numpy((np.asarray(x_u, dtype=np.float64) / 65536.0 * 4.0 - 2.0).astype(np.float32)).to(torch.bfloat16)
    logits = torch.from_numpy(np.random.Generator(np.random.PCG64(seed + 1)).standard_normal((t_n, e_n)).astype(np.float32))
    tw, ti = _routing(logits, k)
    tw = tw.to(torch.bfloat16)
    layer = SimpleNamespace(w13_weight=torch.from_numpy(w13), w2_weight=torch.from_numpy(w2),
                            w13_absmax=torch.from_numpy(a13.view(np.int16)).view(torch.bfloat16),
                            w2_absmax=torch.from_numpy(a2.view(np.int16)).view(torch.bfloat16), _codebook=cb)
    t0 = time.time()
    out = run_apply(layer, x, tw, ti)
    print(f"qwen apply T={t_n}: {time.time() - t0:.2f}s")
    np.savez_compressed(os.path.join(HERE, "apply_qwen.npz"), seed=seed, sha=sha(w13, w2, a13, a2),
                        table=bits(cb), x=bits(x), tw=bits(tw), ti=ti.numpy().astype(np.int32), out=bits(out))
    print("wrote fixtures to", HERE)


def convert_fixture(ref_root):
    sys.path.insert(0, ref_root)
    import torch
    from vllm_lut.convert_checkpoint import quantize_weight
    cb = torch.from_numpy(np.load(os.path.join(ref_root, "models/qwen/blocklut_256.npy"))).to(torch.bfloat16)
    rng = np.random.Generator(np.random.PCG64(11))
    df = 5.0
    w = (rng.standard_t(df, size=(40, 200)) * (0.02 / np.sqrt(df / (df - 2)))).astype(np.float32)
    w.reshape(-1)[:128] = 0.0
    wb = torch.from_numpy(w).to(torch.bfloat16)
    idx, absmax = quantize_weight(wb, cb)
    np.savez_compressed(os.path.join(HERE, "convert_r.npz"), w=bits(wb), table=bits(cb), idx=idx.numpy(),
                        absmax=bits(absmax))


def bitplane_fixture(ref_root):
    import ast
    from types import SimpleNamespace
    import torch
    path = os.path.join(ref_root, "runtime/model_offload.py")
    tree = ast.parse(open(path).read())
    fn = next(n for n in ast.walk(tree) if isinstance(n, ast.FunctionDef) and n.name == "split_and_extract_from_tensor")
    ns = {"np": np, "torch": torch}
    exec(compile(ast.Module(body=[fn], type_ignores=[]), path, "exec"), ns)
    rng = np.random.Generator(np.random.PCG64(17))
    n = 4100
    idx = rng.integers(0, 256, size=n, dtype=np.uint8)
    am = rng.integers(0, 1 << 16, size=(n + 127) // 128, dtype=np.uint16)
    fake = SimpleNamespace(lut_moe_config=SimpleNamespace(code_type="BLOCKLUT"),
                           _quantize_weight_to_blocklut=lambda w: (idx, am))
    chunks, _ = ns["split_and_extract_from_tensor"](fake, torch.zeros(1), 3)
    np.savez_compressed(os.path.join(HERE, "bitplane.npz"), idx=idx, planes=np.concatenate(chunks),
                        chunk_sizes=np.array([c.size for c in chunks]))


def additive_fixture(ref_root):
    import importlib.util
    path = os.path.join(ref_root, "evaluation/explore_additive_lut.py")
    spec = importlib.util.spec_from_file_location("explore_additive_lut", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    rng = np.random.Generator(np.random.PCG64(23))
    coarse = np.sort(rng.integers(-64, 64, 4)).astype(np.float32) / 64.0
    fine = np.sort(rng.integers(-16, 16, 4)).astype(np.float32) / 1024.0
    n = 512
    ic = rng.integers(0, 4, n).astype(np.uint8)
    ifn = rng.integers(0, 4, n).astype(np.uint8)
    absmax = np.ones(n // 128, dtype=np.float32)
    x = mod.dequantize_additive_lut(ic, ifn, absmax, coarse, fine, 128, n)
    np.savez_compressed(os.path.join(HERE, "additive.npz"), coarse=coarse, fine=fine, ic=ic, ifn=ifn, x=x)


def train_fixture(ref_root):
    """``train.npz``: the reference's codebook training (``vllm_lut/quantizer.py:66-236``)
    on CPU under fixed ``torch.manual_seed`` values.

    * ``LUTQuantizer("BLOCKLUT", lut_size=64).train`` (block normalisation,
      ``_train_kmeans``) and ``LUTQuantizer("NESTEDLUT", lut_size=64).train``
      (adds the K=64 codebook, ``_greedy_merge`` to 16, ``_build_mapped_table``),
      both seeded with 7, on 8192 Student-t weights with a zero-padded tail block.
    * ``_train_kmeans(data, 16, 4, max_samples=1500)`` (the random-subset path), seed 11.
    * ``_greedy_merge`` of a fixed 24-value array to 6, and ``_build_mapped_table``
      of 12 and 5 values to 256 (the remainder path).
    """
    sys.path.insert(0, ref_root)
    import torch
    from vllm_lut import quantizer as Q

    torch.set_num_threads(1)
    rng = np.random.Generator(np.random.PCG64(31))
    w = (rng.standard_t(5, size=8000) * 0.02 / np.sqrt(5.0 / 3.0)).astype(np.float32)
    out = {"w": w}
    for name in ("BLOCKLUT", "NESTEDLUT"):
        torch.manual_seed(7)
        q = Q.LUTQuantizer(code_type=name, block_size=128, lut_size=64, device="cpu")
        q.train(torch.from_numpy(w), n_iter=6)
        out[f"{name.lower()}_codebook"] = bits(q.lut_codebook)
        if name == "NESTEDLUT":
            out["mapped64"] = bits(q.nested_mapped64)
            out["mapped16"] = bits(q.nested_mapped16)
    torch.manual_seed(11)
    q = Q.LUTQuantizer(code_type="BLOCKLUT", device="cpu")
    data = torch.from_numpy(rng.standard_normal(3000).astype(np.float32))
    out["km_data"] = data.numpy()
    out["km16"] = bits(q._train_kmeans(data, 16, 4, max_samples=1500))
    merge_in = torch.from_numpy(np.sort(rng.standard_normal(24)).astype(np.float32))
    out["merge_in"] = merge_in.numpy()
    out["merge6"] = q._greedy_merge(merge_in, 6).numpy()
    for n in (12, 5):
        c = torch.from_numpy(np.sort(rng.standard_normal(n)).astype(np.float32))
        out[f"map_in{n}"] = c.numpy()
        out[f"map{n}"] = bits(q._build_mapped_table(c, 256))
    np.savez_compressed(os.path.join(HERE, "train.npz"), **out)


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: make_golden.py <block_lut checkout> [convert | bitplane | additive | train]")
    if sys.argv[2:] == ["convert"]:
        convert_fixture(sys.argv[1])
    elif sys.argv[2:] == ["bitplane"]:
        bitplane_fixture(sys.argv[1])
    elif sys.argv[2:] == ["additive"]:
        additive_fixture(sys.argv[1])
    elif sys.argv[2:] == ["train"]:
        train_fixture(sys.argv[1])
    else:
        main(sys.argv[1])
        convert_fixture(sys.argv[1])
        bitplane_fixture(sys.argv[1])
        additive_fixture(sys.argv[1])
        train_fixture(sys.argv[1])
