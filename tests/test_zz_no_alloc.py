"""blut_moe_forward_noalloc: the MoE layer forward for callers that cannot
allocate device memory when they call -- a plugin that its host framework
hands only input and output pointers, or a serving loop that must not call
cudaMalloc.  Its scratch is a library-owned device array, so the caller
passes just the layer arguments and the stream.

The test runs it twice in a row through the C ABI.  Both calls make the
same deterministic launches as blut_moe_forward with a caller workspace, so
each output must equal that entry point's bit for bit; the first is also
checked against the float64 oracle within the layer tolerance (max-abs 2e-3,
rel-L2 1e-3), and the device status is read back through
blut_moe_check_status(NULL, stream).  The file name makes pytest collect it
last.
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
    experts, W13, W2 = build_b_layer(fmt, E=E, H=H, I=I, seed=21)
    rng = np.random.Generator(np.random.PCG64(22))
    rw = (rng.standard_normal((E + 1, H)) * 0.1).astype(np.float16)
    s13n = O.student_t_weights(rng, (2 * Is, H)).astype(np.float16)
    s2n = O.student_t_weights(rng, (H, Is)).astype(np.float16)
    layer = LUTMoELayer(experts, k, router_w=cuda(rw), shared=SharedExpert.from_dense(cuda(s13n), cuda(s2n)),
                        shared_gate_mode=1)
    x = cuda(O.rms_activations(rng, T, H).astype(np.float16))

    ref = layer.forward(x)  # the existing entry point, caller workspace
    torch.cuda.synchronize()

    # the float64 oracle, routed from the same fp16 inputs
    xn = x.float().cpu().numpy().astype(np.float64)
    logits = xn @ rw[:E].astype(np.float64).T
    ids, tw = O.routing(logits, k)
    srt = np.sort(logits, axis=1)
    keep = srt[:, -k] - srt[:, -k - 1] > 1e-4  # tokens without a near-tie at the k-th expert
    assert keep.sum() >= T // 2
    want = O.moe_forward(xn, ids, tw, W13, W2, act_dtype="f16", shared13=s13n.astype(np.float64),
                         shared2=s2n.astype(np.float64), shared_gate=rw[E].astype(np.float64))

    args = _lib.MoEArgs.from_buffer_copy(layer._args)
    args.num_tokens = T
    args.x = x.data_ptr()
    args.topk_ids = args.topk_weights = None
    lib = _lib.lib()
    for call in range(2):
        out = torch.full_like(x, float("nan"))
        args.out = out.data_ptr()
        rc = lib.blut_moe_forward_noalloc(C.byref(args), _lib.stream_ptr())
        assert rc == _lib.BLUT_OK, _lib.status_string(rc)
        assert lib.blut_moe_check_status(None, _lib.stream_ptr()) == _lib.BLUT_OK  # synchronises
        assert torch.equal(out, ref), f"call {call}: differs from blut_moe_forward"
        if call == 0:
            o = out.float().cpu().numpy()[keep]
            err, rel = float(np.abs(o - want[keep]).max()), O.rel_l2(o, want[keep])
            assert err <= MAX_ABS and rel <= REL_L2, f"vs oracle: max-abs {err:.3g} rel-L2 {rel:.3g}"


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
