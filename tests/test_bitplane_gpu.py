"""Progressive bit-plane tiers on the GPU (block_lut_b200/bitplanes.py):
the packer against the reference's own output and the oracle, and the fused
tier recover bit for bit against the oracle's Format R dequant. The sections
a tier does not read are filled with 0xFF, so a kernel that touched them
would change the result."""
import numpy as np
import pytest
import torch

from oracle import blut_oracle as O
from tests._helpers import bf16_tensor, cuda, to_u16

from block_lut_b200.bitplanes import bitplane_bytes, pack_bitplanes, recover_tier

pytestmark = pytest.mark.gpu


def test_pack_matches_reference_golden(golden):
    d = golden("bitplane.npz")
    planes = pack_bitplanes(cuda(d["idx"]))
    assert np.array_equal(planes.cpu().numpy(), d["planes"])


@pytest.mark.parametrize("n", [4, 28, 32, 4100, 1 << 20, (1 << 20) + 12])
def test_pack_matches_oracle(n):
    idx = np.random.Generator(np.random.PCG64(n)).integers(0, 256, n, dtype=np.uint8)
    assert np.array_equal(pack_bitplanes(cuda(idx)).cpu().numpy(), O.bitplane_pack(idx))


def test_pack_unaligned_source_takes_the_byte_path():
    n = 4096
    idx = np.random.Generator(np.random.PCG64(3)).integers(0, 256, n + 4, dtype=np.uint8)
    src = cuda(idx)[4:]
    assert src.data_ptr() % 16 != 0
    assert np.array_equal(pack_bitplanes(src).cpu().numpy(), O.bitplane_pack(idx[4:]))


def _case(n, bs, seed):
    rng = np.random.Generator(np.random.PCG64(seed))
    idx = rng.integers(0, 256, n, dtype=np.uint8)
    am = rng.uniform(0.01, 0.1, (n + bs - 1) // bs).astype(np.float32)
    am[::7] = 1e-12
    am[3::11] = 1e4
    table = rng.uniform(-1, 1, 256).astype(np.float32)
    # zeros, signed tiny and large entries; every product stays above the fp32
    # subnormal range, where the reference's fp32-then-bf16 rounding could
    # differ from the kernel's single bf16 rounding
    table[:6] = (0.0, -0.0, 1e-20, -1e-20, 3e4, -3e4)
    return idx, O.f32_to_bf16(am), O.f32_to_bf16(table)


@pytest.mark.parametrize("tier", [0, 1, 2])
# (1 << 20) + 8 and 3088 take the warp-chunk path and then the per-quad tail;
# 4100 and bs 100 only the per-quad path
@pytest.mark.parametrize("n,bs", [(4100, 128), (1 << 20, 128), ((1 << 20) + 8, 96), (3088, 128), (65536, 100),
                                  (96, 32), (4, 128)])
def test_recover_tier_bit_exact(tier, n, bs):
    idx, am, table = _case(n, bs, n + bs + tier)
    planes = O.bitplane_pack(idx)
    planes[bitplane_bytes(n, tier):] = 0xFF
    out = recover_tier(cuda(planes), bf16_tensor(am), bf16_tensor(table), n, tier, bs)
    ref = O.dequant_r(idx, am, table, bs, tier)
    assert np.array_equal(to_u16(out), ref)


@pytest.mark.parametrize("tier", [0, 2])
def test_recover_into_unaligned_output_and_prefix_buffer(tier):
    n, bs = 8192, 128
    idx, am, table = _case(n, bs, 40 + tier)
    # only the tier's prefix is allocated, as the engine reads it from disk
    planes = cuda(O.bitplane_pack(idx)[: bitplane_bytes(n, tier)].copy())
    buf = torch.zeros(n + 8, dtype=torch.bfloat16, device="cuda")
    out = buf[3:3 + n]
    assert out.data_ptr() % 16 != 0
    recover_tier(planes, bf16_tensor(am), bf16_tensor(table), n, tier, bs, out=out)
    assert np.array_equal(to_u16(out), O.dequant_r(idx, am, table, bs, tier))
    assert not buf[:3].any() and not buf[3 + n:].any()


def test_device_round_trip_and_argument_errors():
    n = 1 << 16
    idx, am, table = _case(n, 128, 9)
    d_idx = cuda(idx)
    planes = pack_bitplanes(d_idx)
    out = recover_tier(planes, bf16_tensor(am), bf16_tensor(table), n, 0)
    assert np.array_equal(to_u16(out), O.dequant_r(idx, am, table, 128))
    with pytest.raises(ValueError):
        recover_tier(planes[: n // 2], bf16_tensor(am), bf16_tensor(table), n, 1)
    with pytest.raises(ValueError):
        recover_tier(planes, bf16_tensor(am), bf16_tensor(table)[:32], n, 1)
    with pytest.raises(ValueError):
        pack_bitplanes(d_idx[:6])
