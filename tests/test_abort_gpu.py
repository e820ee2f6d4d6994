"""The bounded-wait abort path of the tcgen05 kernels, driven without a fault.

Every device-side wait in ``tc_mm_kernel`` gives up after a time limit, sets
the CTA's abort flag and ``BLUT_ERR_TIMEOUT`` in the workspace status, lets
its bulk copies and MMAs in flight finish and frees its tensor memory.  Here
the limit is cut to 1 ns (``blut_debug_set_wait_limit``), so the first wait
that does not find its barrier complete gives up: the call must report the
timeout through ``check_status`` and leave the context usable, and the next
call with the default limit must produce the right output.
"""
import numpy as np
import pytest
import torch

from oracle import blut_oracle as O

from block_lut_b200 import _lib
from block_lut_b200.formats import LUTFormat
from block_lut_b200.moe import LUTMoELayer
from tests._helpers import build_b_layer, check_layer, cuda, routing_inputs


@pytest.mark.gpu
def test_wait_timeout_reports_and_recovers():
    fmt = LUTFormat("b", 4, 64)
    E, H, I, T, k = 8, 512, 256, 16, 2
    experts, W13, W2 = build_b_layer(fmt, E, H, I, seed=5, tc=True)
    layer = LUTMoELayer(experts, k)
    rng = np.random.Generator(np.random.PCG64(6))
    x = cuda(O.rms_activations(rng, T, H).astype(np.float16))
    ids, w = routing_inputs(rng, T, E, k)
    ids_t, w_t = cuda(ids), cuda(w)
    lib = _lib.lib()
    try:
        assert lib.blut_debug_set_wait_limit(1) == _lib.BLUT_OK
        layer.forward(x, ids_t, w_t)  # launches succeed; the kernels give up on the device
        torch.cuda.synchronize()
        with pytest.raises(RuntimeError, match="timed out"):
            layer.check_status()
    finally:
        lib.blut_debug_set_wait_limit(0)
    # the context is intact: a normal call is correct and its status is clean
    out = layer.forward(x, ids_t, w_t)
    torch.cuda.synchronize()
    layer.check_status()
    ref = O.moe_forward(x.float().cpu().numpy(), ids, w, W13, W2, act_dtype="f16")
    check_layer(out, ref, torch.float16, "after abort")
