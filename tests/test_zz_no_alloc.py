"""blut_moe_forward_noalloc: the MoE layer forward for callers that cannot
allocate device memory when they call -- a plugin that its host framework
hands only input and output pointers, or a serving loop that must not call
cudaMalloc.  Its scratch is a library-owned device array, so the caller
passes just the layer arguments and the stream.

The test runs it twice in a row through the C ABI and checks each output
against blut_moe_forward's with a caller workspace, within the layer
tolerance the other tests use (max-abs 2e-3, rel-L2 1e-3).  The file name
makes pytest collect it last.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import blut_oracle as O
from tests._helpers import MAX_ABS, REL_L2, build_b_layer, cuda

from block_lut_b200 import _lib
from block_lut_b200.formats import LUTFormat, tiled_bytes
from block_lut_b200.moe import LUTMoELayer, SharedExpert

pytestmark = pytest.mark.gpu


def test_noalloc_forward_matches_workspace_forward_on_two_calls():
    E, H, I, Is, T, k = 8, 256, 256, 256, 24, 2
    fmt = LUTFormat("b", 4, 64)
    experts, _, _ = build_b_layer(fmt, E=E, H=H, I=I, seed=21)
    rng = np.random.Generator(np.random.PCG64(22))
    router_w = cuda((rng.standard_normal((E + 1, H)) * 0.1).astype(np.float16))
    s13 = cuda(O.student_t_weights(rng, (2 * Is, H)).astype(np.float16))
    s2 = cuda(O.student_t_weights(rng, (H, Is)).astype(np.float16))
    layer = LUTMoELayer(experts, k, router_w=router_w, shared=SharedExpert.from_dense(s13, s2), shared_gate_mode=1)
    x = cuda(O.rms_activations(rng, T, H).astype(np.float16))

    ref = layer.forward(x)  # the existing entry point, caller workspace
    torch.cuda.synchronize()
    r = ref.float().cpu().numpy()

    args = _lib.MoEArgs.from_buffer_copy(layer._args)
    args.num_tokens = T
    args.x = x.data_ptr()
    args.topk_ids = args.topk_weights = None
    for _ in range(2):
        out = torch.full_like(x, float("nan"))
        args.out = out.data_ptr()
        rc = _lib.lib().blut_moe_forward_noalloc(C.byref(args), _lib.stream_ptr())
        assert rc == _lib.BLUT_OK, _lib.status_string(rc)
        torch.cuda.synchronize()
        o = out.float().cpu().numpy()
        assert np.isfinite(o).all()
        assert np.abs(o - r).max() <= MAX_ABS
        assert O.rel_l2(o, r) <= REL_L2


def test_noalloc_rejects_a_layer_beyond_its_scratch_before_launching():
    # 512 tokens x top-4 at H 2048: the fp32 expert outputs alone need 16 MiB
    fmt = LUTFormat("b", 4, 64)
    a = _lib.MoEArgs()
    a.num_tokens, a.hidden, a.inter, a.num_experts, a.top_k, a.dtype = 512, 2048, 1408, 60, 4, _lib.F16
    a.w13, a.w2 = fmt.desc(2816, 2048, paired=True), fmt.desc(2048, 1408)
    a.w13_tiled = a.w2_tiled = a.x = a.out = 1 << 20
    a.w13_stride, a.w2_stride = tiled_bytes(fmt, 2816, 2048), tiled_bytes(fmt, 2048, 1408)
    a.topk_ids = a.topk_weights = 1 << 21
    assert _lib.lib().blut_moe_workspace_size(C.byref(a)) > 16 << 20
    assert _lib.lib().blut_moe_forward_noalloc(C.byref(a), None) == _lib.BLUT_ERR_WORKSPACE
