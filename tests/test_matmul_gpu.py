"""Single-matrix LUT matmul (blut_matmul through LUTLinear) against the
float64 oracle y = x W^T on the same quantised weights, on both matmul paths,
for token counts across the decode / wide-group boundary (tolerance in
tests/_helpers.check_layer)."""
import numpy as np
import pytest
import torch

from oracle import blut_oracle as O
from tests._helpers import bf16_tensor, check_layer, cuda, oracle_quantize, qm_from_numpy

from block_lut_b200.formats import LUTFormat, QuantizedMatrix, dense_matrix
from block_lut_b200.linear import LUTLinear

pytestmark = pytest.mark.gpu

N, K = 256, 384
MS = [1, 5, 32, 33, 130, 300]


def _b_matrix(fmt, seed):
    rng = np.random.Generator(np.random.PCG64(seed))
    canon, deq = oracle_quantize(O.student_t_weights(rng, (N, K)), fmt)
    return qm_from_numpy(fmt, N, K, canon), deq


@pytest.mark.parametrize("fmt,tc", [
    (LUTFormat("b", 4, 64), True), (LUTFormat("b", 4, 64), False), (LUTFormat("b", 3, 32), True),
    (LUTFormat("b", 2, 128), True), (LUTFormat("b", 2, 64), False), (LUTFormat("nested", 4, 64, 0), True),
    (LUTFormat("nested", 4, 64, 1), True), (LUTFormat("nested", 4, 128, 0), False)],
    ids=lambda v: f"{v.kind}{v.bits}g{v.group}t{v.tier}" if isinstance(v, LUTFormat) else ("tc" if v else "mma"))
def test_lut_matmul_matches_oracle(fmt, tc):
    qm, W = _b_matrix(fmt, 11 * fmt.bits + fmt.group + fmt.tier)
    lin = LUTLinear(qm, tc=tc)
    assert lin.tc == tc
    for m in MS:
        rng = np.random.Generator(np.random.PCG64(m))
        x = cuda(O.rms_activations(rng, m, K).astype(np.float16))
        ref = x.float().cpu().numpy().astype(np.float64) @ W.astype(np.float64).T
        check_layer(lin(x), ref, torch.float16, f"{fmt} tc={tc} m={m}")
        y32 = lin(x, out_f32=True)
        assert y32.dtype == torch.float32
        assert np.abs(y32.cpu().numpy() - ref).max() <= 1e-3, f"{fmt} m={m} fp32 output"
    lin.check_status()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_dense_matmul_tcgen05(dtype):
    rng = np.random.Generator(np.random.PCG64(3))
    w = torch.from_numpy(O.student_t_weights(rng, (N, K))).to("cuda", dtype)
    lin = LUTLinear(dense_matrix(w))
    assert lin.tc
    for m in (1, 40, 129):
        x = torch.from_numpy(O.rms_activations(rng, m, K)).to("cuda", dtype)
        ref = x.double().cpu().numpy() @ w.double().cpu().numpy().T
        check_layer(lin(x), ref, dtype, f"dense {dtype} m={m}")


@pytest.mark.parametrize("tc", [True, False], ids=["tc", "mma"])
@pytest.mark.parametrize("tier", [0, 2])
def test_r8_matmul(tier, tc):
    rng = np.random.Generator(np.random.PCG64(60 + tier))
    table = O.f32_to_bf16(np.sort(rng.uniform(-1, 1, 256)).astype(np.float32))
    idx = rng.integers(0, 256, size=N * K, dtype=np.uint8)
    am = O.f32_to_bf16(rng.uniform(0.02, 0.08, N * K // 128).astype(np.float32))
    fmt = LUTFormat("r8", 8, 128, tier)
    qm = QuantizedMatrix(fmt, N, K, cuda(idx), bf16_tensor(table), scales=bf16_tensor(am))
    W = O.bf16_to_f32(O.dequant_r(idx, am, table, 128, tier)).reshape(N, K).astype(np.float64)
    lin = LUTLinear(qm, tc=tc)
    assert lin.tc == tc
    for m in (1, 8, 70, 200):
        x = cuda(O.f32_to_bf16(O.rms_activations(rng, m, K))).view(torch.bfloat16)
        check_layer(lin(x), x.double().cpu().numpy() @ W.T, torch.bfloat16, f"r8 tier {tier} m={m}")


def test_matmul_rejects_bad_arguments():
    qm, _ = _b_matrix(LUTFormat("b", 4, 64), 1)
    lin = LUTLinear(qm)
    with pytest.raises(ValueError):
        lin(torch.zeros(3, K + 128, dtype=torch.float16, device="cuda"))
    with pytest.raises(ValueError):
        lin(torch.zeros(3, K, dtype=torch.bfloat16, device="cuda"))
    # an empty batch gives an empty result without a launch, as torch's matmul does
    assert lin(torch.zeros(0, K, dtype=torch.float16, device="cuda")).shape == (0, N)
