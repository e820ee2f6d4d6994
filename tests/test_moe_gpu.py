"""MoE layer parity: blut_moe_forward against the float64 oracle on the same
quantised weights and routing (tolerance in tests/_helpers.check_layer)."""
import numpy as np
import pytest
import torch

from oracle import blut_oracle as O
from tests._helpers import (bf16_tensor, build_b_layer, build_r8_layer, check_layer, cuda, routing_inputs)
from tests.golden.make_golden import qwen_layer_weights, small_layer_indices

from block_lut_b200.formats import LUTFormat, QuantizedMatrix, encode
from block_lut_b200.moe import LUTExperts, LUTMoELayer, SharedExpert

pytestmark = pytest.mark.gpu

# (format, tiled layout): Format B and NestedLUT run on the tcgen05 path by
# default; the mma.sync path is kept for every format.
FORMATS = [(LUTFormat("b", 4, 64), True), (LUTFormat("b", 4, 32), True), (LUTFormat("b", 4, 128), True),
           (LUTFormat("b", 3, 64), True), (LUTFormat("b", 3, 32), True), (LUTFormat("b", 3, 128), True),
           (LUTFormat("b", 2, 64), True), (LUTFormat("b", 2, 32), True), (LUTFormat("b", 2, 128), True),
           (LUTFormat("nested", 4, 64, 0), True), (LUTFormat("nested", 4, 64, 1), True),
           (LUTFormat("nested", 4, 32, 0), True), (LUTFormat("nested", 4, 128, 0), True),
           (LUTFormat("b", 4, 64), False), (LUTFormat("b", 3, 64), False), (LUTFormat("b", 2, 64), False),
           (LUTFormat("b", 2, 128), False), (LUTFormat("nested", 4, 64, 0), False),
           (LUTFormat("nested", 4, 64, 1), False)]


@pytest.fixture(scope="module", params=FORMATS,
                ids=lambda p: f"{p[0].kind}{p[0].bits}g{p[0].group}t{p[0].tier}-{'tc' if p[1] else 'mma'}")
def b_layer(request):
    fmt, tc = request.param
    layer = build_b_layer(fmt, E=6, H=256, I=256, seed=1, tc=tc)
    assert layer[0].tc == tc
    return fmt, layer


@pytest.mark.parametrize("T,k", [(1, 2), (3, 2), (8, 2), (16, 3), (80, 2)])
def test_format_b_layer(b_layer, T, k):
    fmt, (experts, W13, W2) = b_layer
    rng = np.random.Generator(np.random.PCG64(T * 31 + k))
    x = O.rms_activations(rng, T, 256)
    ids, tw = routing_inputs(rng, T, 6, k)
    layer = LUTMoELayer(experts, k)
    xh = cuda(x.astype(np.float16))
    out = layer.forward(xh, cuda(ids), cuda(tw))
    ref = O.moe_forward(xh.float().cpu().numpy(), ids, tw, W13, W2, act_dtype="f16")
    check_layer(out, ref, torch.float16, f"{fmt} T={T}")
    layer.check_status()


@pytest.mark.parametrize("tc", [True, False], ids=["tc", "mma"])
def test_r8_layer_and_tiers(tc):
    for tier in (0, 1, 2):
        experts, W13, W2, _ = build_r8_layer(5, 256, 384, seed=tier, tier=tier, tc=tc)
        assert experts.tc == tc
        rng = np.random.Generator(np.random.PCG64(4 + tier))
        for T in (1, 8, 24):
            x = O.rms_activations(rng, T, 256)
            ids, tw = routing_inputs(rng, T, 5, 2)
            xb = cuda(O.f32_to_bf16(x)).view(torch.bfloat16)
            out = LUTMoELayer(experts, 2).forward(xb, cuda(ids), cuda(tw))
            ref = O.moe_forward(xb.float().cpu().numpy(), ids, tw, W13, W2, act_dtype="bf16")
            check_layer(out, ref, torch.bfloat16, f"r8 tier {tier} T={T}")


@pytest.mark.parametrize("T", [2, 8])
def test_r8_against_reference_apply_golden(golden, T):
    """The reference's own apply() outputs (bf16 per-op rounding) vs this path.

    The reference rounds gate_up, silu, *up, the down projection, *w and the
    accumulation to bf16 (quant_method.py:262-277); this path keeps fp32 until
    one final rounding, so the two agree within the reference's own bf16
    rounding: max-abs 2e-3 (outputs ~0.2) and rel-L2 1e-2.
    """
    s = golden("apply_small.npz")
    w13, w2 = small_layer_indices(int(s["idx_seed"]), 8, 256, 128)
    fmt = LUTFormat("r8", 8, 128)
    tab = bf16_tensor(s["table"])
    q13 = [QuantizedMatrix(fmt, 256, 256, cuda(w13[e].reshape(-1)), tab, scales=bf16_tensor(s["a13"][e]))
           for e in range(8)]
    q2 = [QuantizedMatrix(fmt, 256, 128, cuda(w2[e].reshape(-1)), tab, scales=bf16_tensor(s["a2"][e]))
          for e in range(8)]
    layer = LUTMoELayer(LUTExperts.from_quantized(q13, q2, tab), 2)
    out = layer.forward(bf16_tensor(s[f"x{T}"]), cuda(s[f"ti{T}"]), bf16_tensor(s[f"tw{T}"]).float())
    ref = O.bf16_to_f32(s[f"out{T}"])
    o = out.float().cpu().numpy()
    assert np.abs(o - ref).max() <= 2e-3
    assert O.rel_l2(o, ref) <= 1e-2


def test_r8_qwen_shape_against_reference_golden(golden):
    q = golden("apply_qwen.npz")
    w13, w2, a13, a2, _ = qwen_layer_weights(int(q["seed"]), 60, 2048, 1408)
    fmt = LUTFormat("r8", 8, 128)
    tab = bf16_tensor(q["table"])
    q13 = [QuantizedMatrix(fmt, 2816, 2048, cuda(w13[e].reshape(-1)), tab, scales=bf16_tensor(a13[e]))
           for e in range(60)]
    q2 = [QuantizedMatrix(fmt, 2048, 1408, cuda(w2[e].reshape(-1)), tab, scales=bf16_tensor(a2[e]))
          for e in range(60)]
    layer = LUTMoELayer(LUTExperts.from_quantized(q13, q2, tab), 4)
    x = bf16_tensor(q["x"])
    out = layer.forward(x, cuda(q["ti"]), bf16_tensor(q["tw"]).float())
    ref = O.bf16_to_f32(q["out"])
    o = out.float().cpu().numpy()
    # x spans [-2, 2] here, outputs reach ~2: the reference's bf16 per-op rounding
    # (measured 0.015 max-abs, 5e-3 rel-L2 against float64) dominates
    assert O.rel_l2(o, ref) <= 1e-2
    # strict check against the float64 oracle with this path's rounding points
    W13 = lambda e: O.bf16_to_f32(O.dequant_r(w13[e].reshape(-1), a13[e], q["table"])).reshape(2816, 2048)  # noqa
    W2 = lambda e: O.bf16_to_f32(O.dequant_r(w2[e].reshape(-1), a2[e], q["table"])).reshape(2048, 1408)  # noqa
    ex = O.moe_forward(x.float().cpu().numpy(), q["ti"], O.bf16_to_f32(q["tw"]), W13, W2, act_dtype="bf16")
    check_layer(out, ex, torch.bfloat16, "r8 qwen")


@pytest.mark.parametrize("T", [1, 8, 16])
def test_qwen15_layer_format_b_4bit_g64(T):
    """Config 1: Qwen1.5-MoE layer (H 2048, 60 experts of I 1408, top-4 softmax,
    shared expert I 5632 with sigmoid gate), BlockLUT 4-bit g64, seed 0."""
    H, I, E, k, Is = 2048, 1408, 60, 4, 5632
    fmt = LUTFormat("b", 4, 64)
    g = torch.Generator(device="cuda").manual_seed(0)
    st = torch.distributions.StudentT(torch.tensor(5.0, device="cuda"))
    scale = 0.02 / (5.0 / 3.0) ** 0.5
    torch.manual_seed(0)
    q13, q2 = [], []
    for _ in range(E):
        q13.append(encode(st.sample((2 * I, H)) * scale, fmt))
        q2.append(encode(st.sample((H, I)) * scale, fmt))
    experts = LUTExperts.from_quantized(q13, q2)
    router_w = (st.sample((E + 1, H)) * scale).half()
    s13 = (st.sample((2 * Is, H)) * scale).half()
    s2 = (st.sample((H, Is)) * scale).half()
    layer = LUTMoELayer(experts, k, router_w=router_w, shared=SharedExpert.from_dense(s13, s2), shared_gate_mode=1)
    rng = np.random.Generator(np.random.PCG64(T))
    x = cuda(O.rms_activations(rng, T, H).astype(np.float16))
    out = layer.forward(x)
    layer.check_status()
    # oracle: routing from the same fp16 inputs, dequant from the same canonical tensors
    xn = x.float().cpu().numpy()
    rw = router_w.float().cpu().numpy()
    logits = xn.astype(np.float64) @ rw[:E].T.astype(np.float64)
    ids, tw = O.routing(logits, k)
    srt = np.sort(logits, axis=1)
    assert (srt[:, -k] - srt[:, -k - 1] > 1e-4).all(), "near-tie in routing; pick another seed"
    cache = {}

    def deq(lst, e):
        m = lst[e]
        return O.dequant_b(m.codes.cpu().numpy(), m.tables.cpu().numpy(), 4, 64).astype(np.float32)
    ref = O.moe_forward(xn, ids, tw, lambda e: deq(q13, e), lambda e: deq(q2, e), act_dtype="f16",
                        shared13=s13.float().cpu().numpy(), shared2=s2.float().cpu().numpy(),
                        shared_gate=rw[E])
    check_layer(out, ref, torch.float16, f"qwen1.5 layer T={T}")


def test_single_token_path_edge_slots():
    """The single-token path (route, gate/up, down with the combine): a token
    whose slots are all empty (-1) gives zeros without a shared expert and the
    shared expert alone with one; one empty slot beside a valid one, and the
    same expert chosen twice, count like the general path; fp32 output."""
    fmt = LUTFormat("b", 4, 64)
    experts, W13, W2 = build_b_layer(fmt, E=4, H=256, I=128, seed=7, tc=True)
    rng = np.random.Generator(np.random.PCG64(3))
    x = cuda(O.rms_activations(rng, 1, 256).astype(np.float16))
    xs = x.float().cpu().numpy()
    s13 = O.student_t_weights(rng, (256, 256)).astype(np.float16)
    s2 = O.student_t_weights(rng, (256, 128)).astype(np.float16)
    layer = LUTMoELayer(experts, 2)
    assert layer.launch_count(1, caller_routing=True) == 3
    empty = cuda(np.array([[-1, -1]], dtype=np.int32))
    w = cuda(np.array([[0.6, 0.4]], dtype=np.float32))
    out = layer.forward(x, empty, w)
    # a stale status word (left by anything that used the workspace before)
    # does not outlive the next call: the route kernel clears it
    from block_lut_b200.moe import _WS
    _WS[(x.device.type, x.device.index, 0)][0] = 1
    out = layer.forward(x, empty, w)
    layer.check_status()
    assert torch.count_nonzero(out).item() == 0
    sh = LUTMoELayer(experts, 2, shared=SharedExpert.from_dense(cuda(s13), cuda(s2)), shared_gate_mode=0)
    out = sh.forward(x, empty, w)
    sh.check_status()
    h = xs.astype(np.float64) @ s13.astype(np.float64).T
    a = O.round_to((O.silu(h[:, :128]) * h[:, 128:]).astype(np.float32), "f16").astype(np.float64)
    check_layer(out, a @ s2.astype(np.float64).T, torch.float16, "shared expert only")
    for ids in ([[2, -1]], [[1, 1]]):
        ids = np.array(ids, dtype=np.int32)
        tw = np.array([[0.6, 0.4]], dtype=np.float32)
        out = layer.forward(x, cuda(ids), cuda(tw), out_f32=True)
        layer.check_status()
        assert out.dtype == torch.float32
        ref = O.moe_forward(xs, np.where(ids < 0, 0, ids), np.where(ids < 0, 0, tw), W13, W2, act_dtype="f16")
        err = np.abs(out.cpu().numpy() - ref).max()
        assert err <= 2e-3, (ids.tolist(), err)


@pytest.mark.parametrize("T", [12, 1])  # T = 1: the single-token GEMV on the tcgen05 layout
@pytest.mark.parametrize("tc", [True, False], ids=["tc", "mma"])
def test_shared_expert_modes_and_graph_capture(tc, T):
    """Shared expert (run on the library's side stream) with and without its
    gate, then the whole layer captured in a CUDA graph and replayed."""
    fmt = LUTFormat("b", 4, 64)
    experts, W13, W2 = build_b_layer(fmt, E=4, H=256, I=128, seed=5, tc=tc)
    rng = np.random.Generator(np.random.PCG64(12))
    s13 = O.student_t_weights(rng, (256, 256)).astype(np.float16)
    s2 = O.student_t_weights(rng, (256, 128)).astype(np.float16)
    gate = O.student_t_weights(rng, (256,)).astype(np.float16)
    x = cuda(O.rms_activations(rng, T, 256).astype(np.float16))
    ids, tw = routing_inputs(rng, T, 4, 2)
    for mode in (0, 1):
        sh = SharedExpert.from_dense(cuda(s13), cuda(s2), cuda(gate) if mode else None, tc=tc)
        layer = LUTMoELayer(experts, 2, shared=sh, shared_gate_mode=mode)
        out = layer.forward(x, cuda(ids), cuda(tw))
        if mode == 1:
            ref = O.moe_forward(x.float().cpu().numpy(), ids, tw, W13, W2, act_dtype="f16",
                                shared13=s13.astype(np.float32), shared2=s2.astype(np.float32),
                                shared_gate=gate.astype(np.float32))
        else:  # unscaled shared output
            xs = x.float().cpu().numpy().astype(np.float64)
            h = xs @ s13.astype(np.float64).T
            a = O.round_to((O.silu(h[:, :128]) * h[:, 128:]).astype(np.float32), "f16").astype(np.float64)
            ref = O.moe_forward(xs, ids, tw, W13, W2, act_dtype="f16") + a @ s2.astype(np.float64).T
        check_layer(out, ref, torch.float16, f"shared mode {mode}")
    # CUDA graph capture replays the same result, bit for bit
    ti, tww = cuda(ids), cuda(tw)
    res = layer.forward(x, ti, tww)
    static_out = torch.empty_like(res)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        layer.forward(x, ti, tww, out=static_out)
    torch.cuda.current_stream().wait_stream(s)
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        layer.forward(x, ti, tww, out=static_out)
    static_out.zero_()
    gr.replay()
    torch.cuda.synchronize()
    assert torch.equal(static_out, res)


def test_router_path_matches_oracle_routing():
    fmt = LUTFormat("b", 4, 64)
    E, k = 8, 3
    experts, W13, W2 = build_b_layer(fmt, E=E, H=256, I=128, seed=8)
    rng = np.random.Generator(np.random.PCG64(21))
    rw = (rng.standard_normal((E, 256)) * 0.1).astype(np.float16)
    for renorm in (False, True):
        T = 20
        x = cuda(O.rms_activations(rng, T, 256).astype(np.float16))
        layer = LUTMoELayer(experts, k, router_w=cuda(rw), renorm=renorm)
        out = layer.forward(x)
        xn = x.float().cpu().numpy().astype(np.float64)
        logits = xn @ rw.astype(np.float64).T
        ids, tw = O.routing(logits, k, renorm)
        srt = np.sort(logits, axis=1)
        keep = srt[:, -k] - srt[:, -k - 1] > 1e-4  # skip tokens with near-ties at the k-th expert
        ref = O.moe_forward(xn, ids, tw, W13, W2, act_dtype="f16")
        check_layer(out[torch.from_numpy(keep).cuda()], ref[keep], torch.float16, f"router renorm={renorm}")


def test_deterministic_and_invalid_ids_reported():
    fmt = LUTFormat("b", 2, 64)
    experts, W13, W2 = build_b_layer(fmt, E=4, H=256, I=128, seed=2)
    rng = np.random.Generator(np.random.PCG64(2))
    x = cuda(O.rms_activations(rng, 9, 256).astype(np.float16))
    ids, tw = routing_inputs(rng, 9, 4, 2)
    layer = LUTMoELayer(experts, 2)
    a = layer.forward(x, cuda(ids), cuda(tw))
    b = layer.forward(x, cuda(ids), cuda(tw))
    assert torch.equal(a, b)
    bad = ids.copy()
    bad[0, 0] = 17  # out of range: skipped on the device and reported
    layer.forward(x, cuda(bad), cuda(tw))
    with pytest.raises(RuntimeError, match="invalid"):
        layer.check_status()
    layer.check_status()  # the status word was cleared by the read


def test_empty_batch_returns_empty():
    """A rank or a scheduler step with no tokens: empty outputs, no launch, no error."""
    fmt = LUTFormat("b", 4, 64)
    experts, _, _ = build_b_layer(fmt, E=4, H=256, I=128, seed=3)
    layer = LUTMoELayer(experts, 2)
    x = torch.zeros(0, 256, dtype=torch.float16, device="cuda")
    ids = torch.zeros(0, 2, dtype=torch.int32, device="cuda")
    tw = torch.zeros(0, 2, dtype=torch.float32, device="cuda")
    assert layer.forward(x, ids, tw).shape == (0, 256)
    assert layer.forward(x, ids, tw, out_f32=True).dtype == torch.float32
    layer.check_status()


def test_qwen15_layer_decode_batch32_bench_shape():
    """The bench's layer at its decode batch (config 2: batch 32), router + shared expert."""
    H, I, E, k, Is, T = 2048, 1408, 60, 4, 5632, 32
    fmt = LUTFormat("b", 4, 64)
    torch.manual_seed(1)
    st = torch.distributions.StudentT(torch.tensor(5.0, device="cuda"))
    scale = 0.02 / (5.0 / 3.0) ** 0.5
    q13 = [encode(st.sample((2 * I, H)) * scale, fmt) for _ in range(E)]
    q2 = [encode(st.sample((H, I)) * scale, fmt) for _ in range(E)]
    g = torch.Generator(device="cuda").manual_seed(3)
    router_w = (torch.randn(E + 1, H, generator=g, device="cuda") * 0.02).half()
    s13 = (torch.randn(2 * Is, H, generator=g, device="cuda") * 0.02).half()
    s2 = (torch.randn(H, Is, generator=g, device="cuda") * 0.02).half()
    layer = LUTMoELayer(LUTExperts.from_quantized(q13, q2), k, router_w=router_w,
                        shared=SharedExpert.from_dense(s13, s2), shared_gate_mode=1)
    x = torch.randn(T, H, generator=g, device="cuda")
    x = (x / x.pow(2).mean(dim=1, keepdim=True).sqrt()).half()
    out = torch.empty_like(x)
    layer.forward(x, out=out)
    torch.cuda.synchronize()
    layer.check_status()
    xn = x.float().cpu().numpy()
    rw = router_w.float().cpu().numpy()
    logits = xn.astype(np.float64) @ rw[:E].T.astype(np.float64)
    ids, tw = O.routing(logits, k)
    srt = np.sort(logits, axis=1)
    keep = srt[:, -k] - srt[:, -k - 1] > 1e-4

    def deq(lst, e):
        m = lst[e]
        return O.dequant_b(m.codes.cpu().numpy(), m.tables.cpu().numpy(), 4, 64).astype(np.float32)
    ref = O.moe_forward(xn, ids, tw, lambda e: deq(q13, e), lambda e: deq(q2, e), act_dtype="f16",
                        shared13=s13.float().cpu().numpy(), shared2=s2.float().cpu().numpy(), shared_gate=rw[E])
    check_layer(out[torch.from_numpy(keep).cuda()], ref[keep], torch.float16, "bench-shaped layer")


@pytest.mark.parametrize("T,with_shared,fmt", [
    (1024, False, LUTFormat("b", 4, 64)), (2048, True, LUTFormat("b", 4, 64)),
    (1024, False, LUTFormat("b", 3, 64)), (1024, False, LUTFormat("nested", 4, 64, 0)),
    (1024, False, LUTFormat("b", 2, 128))], ids=lambda v: str(v) if not isinstance(v, LUTFormat) else
    f"{v.kind}{v.bits}g{v.group}t{v.tier}")
def test_prefill_wide_groups(T, with_shared, fmt):
    """Prefill regime (tcgen05 path, >= 64 tokens per expert): 128-token groups,
    the separate top-k launch, and (with the shared expert) wide shared groups."""
    E, H, I, k, Is = 8, 512, 256, 2, 256
    experts, W13, W2 = build_b_layer(fmt, E=E, H=H, I=I, seed=31, tc=True)
    rng = np.random.Generator(np.random.PCG64(T))
    rw = (rng.standard_normal((E + 1, H)) * 0.05).astype(np.float16)
    sh = None
    if with_shared:
        s13 = O.student_t_weights(rng, (2 * Is, H)).astype(np.float16)
        s2 = O.student_t_weights(rng, (H, Is)).astype(np.float16)
        sh = SharedExpert.from_dense(cuda(s13), cuda(s2), tc=True)
    layer = LUTMoELayer(experts, k, router_w=cuda(rw), shared=sh, shared_gate_mode=1)
    x = cuda(O.rms_activations(rng, T, H).astype(np.float16))
    out = layer.forward(x)
    layer.check_status()
    xn = x.float().cpu().numpy().astype(np.float64)
    logits = xn @ rw[:E].astype(np.float64).T
    ids, tw = O.routing(logits, k)
    srt = np.sort(logits, axis=1)
    keep = srt[:, -k] - srt[:, -k - 1] > 1e-4
    kw = {}
    if with_shared:
        kw = dict(shared13=s13.astype(np.float32), shared2=s2.astype(np.float32), shared_gate=rw[E].astype(np.float32))
    ref = O.moe_forward(xn, ids, tw, W13, W2, act_dtype="f16", **kw)
    check_layer(out[torch.from_numpy(keep).cuda()], ref[keep], torch.float16, f"prefill T={T}")
    # the same layer at decode size still matches (both regimes in one process)
    xd = x[:5].contiguous()
    check_layer(layer.forward(xd)[torch.from_numpy(keep[:5]).cuda()], ref[:5][keep[:5]], torch.float16, "decode")


@pytest.mark.parametrize("T", [1, 8])
def test_decode_step_graph_with_host_io(T):
    """LUTMoEStep: one CUDA graph per step that copies every layer's input
    from pinned host memory, runs the layers and copies the outputs back;
    replays give the eager layers' outputs bit for bit, and new host inputs
    flow through a replay."""
    from block_lut_b200.moe import LUTMoEStep
    fmt = LUTFormat("b", 4, 64)
    layers = []
    for seed in (3, 4):
        experts, _, _ = build_b_layer(fmt, E=6, H=256, I=256, seed=seed, tc=True)
        rng = np.random.Generator(np.random.PCG64(seed))
        rw = cuda((rng.standard_normal((7, 256)) * 0.05).astype(np.float16))
        s13 = O.student_t_weights(rng, (256, 256)).astype(np.float16)
        s2 = O.student_t_weights(rng, (256, 128)).astype(np.float16)
        layers.append(LUTMoELayer(experts, 2, router_w=rw, shared=SharedExpert.from_dense(cuda(s13), cuda(s2)),
                                  shared_gate_mode=1))
    step = LUTMoEStep(layers, T)
    for it in range(2):
        rng = np.random.Generator(np.random.PCG64(50 + it))
        xs = [O.rms_activations(rng, T, 256).astype(np.float16) for _ in layers]
        for h, x in zip(step.host_in, xs):
            h.copy_(torch.from_numpy(x))
        step.run()
        torch.cuda.synchronize()
        for m, h, x in zip(layers, step.host_out, xs):
            assert torch.equal(h, m.forward(cuda(x)).cpu())
    step.check_status()
