"""The repack cache behind fused_lut_moe / _fused_expert_compute, without a GPU.

The tiling itself needs a GPU, so it is stubbed: these tests check which
calls reuse a cached layer.  A stack passed again, or through new views of
it, is a hit.  Different tensors that present the same key (as a stack freed
and replaced at the same address would), or a stack that no longer exists,
are repacked.
"""
import gc

import pytest
import torch

from block_lut_b200 import fast_moe as F


@pytest.fixture
def builds(monkeypatch):
    made = []

    class FakeExperts:
        @classmethod
        def from_quantized(cls, w13, w2, cb):
            made.append(len(w13))
            return object()

    monkeypatch.setattr(F, "LUTExperts", FakeExperts)
    monkeypatch.setattr(F, "LUTMoELayer", lambda experts, top_k: ("layer", len(made)))
    monkeypatch.setattr(F, "_CACHE", F.OrderedDict())
    return made


def _stack(e=3, i=4, h=128):
    return (torch.randint(0, 255, (e, 2 * i, h), dtype=torch.uint8), torch.rand(e, 2 * i * h // 128),
            torch.randint(0, 255, (e, h, i), dtype=torch.uint8), torch.rand(e, h * i // 128),
            torch.rand(256))


def test_same_stack_and_views_of_it_hit(builds):
    s = _stack()
    first = F.r8_layer(*s, top_k=2)
    assert F.r8_layer(*s, top_k=2) is first
    views = tuple(t[:] for t in s)  # new tensor objects over the same memory
    assert F.r8_layer(*views, top_k=2) is first
    assert builds == [3]
    F.r8_layer(*s, top_k=3)  # another top-k is another layer
    assert len(builds) == 2


def test_other_tensors_with_the_same_key_are_repacked(builds, monkeypatch):
    monkeypatch.setattr(F, "_key", lambda *ts: ("same address, shape and version",))
    a = _stack()
    la = F.r8_layer(*a, top_k=2)
    b = _stack()
    lb = F.r8_layer(*b, top_k=2)
    assert lb is not la and len(builds) == 2
    assert F.r8_layer(*b, top_k=2) is lb and len(builds) == 2
    del a, b
    gc.collect()
    c = _stack()
    F.r8_layer(*c, top_k=2)  # the entry's tensors are gone: repacked
    assert len(builds) == 3
