"""Codebook training (``block_lut_b200.quantizer``) against the reference's own
training run on CPU (``tests/golden/train.npz``, from ``vllm_lut/quantizer.py:66-236``).

Codebook training is offline tooling that the reference runs as torch ops on
whatever device it is given; on CPU under the same ``torch.manual_seed`` the
restatement reproduces the reference's codebooks bit for bit.
"""
import numpy as np
import torch

from block_lut_b200.quantizer import LUTQuantizer


def _bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def test_blocklut_train_matches_reference(golden):
    g = golden("train.npz")
    torch.manual_seed(7)
    q = LUTQuantizer("BLOCKLUT", block_size=128, lut_size=64, device="cpu")
    q.train(torch.from_numpy(g["w"]), n_iter=6)
    assert q.lut_codebook.dtype == torch.bfloat16 and q.lut_codebook.shape == (64,)
    assert np.array_equal(_bits(q.lut_codebook), g["blocklut_codebook"])


def test_nestedlut_train_matches_reference(golden):
    """mapped64 / mapped16 equal the reference's; ``lut_codebook`` keeps the
    full codebook, which the reference replaces by its K=64 one."""
    g = golden("train.npz")
    torch.manual_seed(7)
    q = LUTQuantizer("NESTEDLUT", block_size=128, lut_size=64, device="cpu")
    q.train(torch.from_numpy(g["w"]), n_iter=6)
    assert np.array_equal(_bits(q.nested_mapped64), g["mapped64"])
    assert np.array_equal(_bits(q.nested_mapped16), g["mapped16"])
    assert np.array_equal(_bits(q.lut_codebook), g["blocklut_codebook"])
    # the tier tables hold 64 and 16 distinct values, repeated to 256 entries
    assert len(np.unique(g["mapped64"])) <= 64 and len(np.unique(g["mapped16"])) <= 16


def test_train_kmeans_subset_path_matches_reference(golden):
    g = golden("train.npz")
    torch.manual_seed(11)
    q = LUTQuantizer("BLOCKLUT", device="cpu")
    cb = q._train_kmeans(torch.from_numpy(g["km_data"]), 16, 4, max_samples=1500)
    assert np.array_equal(_bits(cb), g["km16"])
    assert torch.all(cb[1:].float() >= cb[:-1].float())  # sorted


def test_greedy_merge_matches_reference(golden):
    g = golden("train.npz")
    q = LUTQuantizer("BLOCKLUT", device="cpu")
    out = q._greedy_merge(torch.from_numpy(g["merge_in"]), 6)
    assert np.array_equal(out.numpy(), g["merge6"])


def test_build_mapped_table_matches_reference(golden):
    g = golden("train.npz")
    q = LUTQuantizer("BLOCKLUT", device="cpu")
    for n in (12, 5):
        t = q._build_mapped_table(torch.from_numpy(g[f"map_in{n}"]), 256)
        assert t.shape == (256,)
        assert np.array_equal(_bits(t), g[f"map{n}"])


def test_save_load_round_trip(tmp_path, golden):
    g = golden("train.npz")
    torch.manual_seed(7)
    q = LUTQuantizer("NESTEDLUT", block_size=128, lut_size=64, device="cpu")
    q.train(torch.from_numpy(g["w"]), n_iter=2)
    q.save(str(tmp_path))
    r = LUTQuantizer("NESTEDLUT", device="cpu")
    assert r.load(str(tmp_path))
    for a in ("lut_codebook", "nested_mapped64", "nested_mapped16"):
        assert np.array_equal(_bits(getattr(r, a)), _bits(getattr(q, a))), a
    assert not LUTQuantizer(device="cpu").load(str(tmp_path / "missing"))
