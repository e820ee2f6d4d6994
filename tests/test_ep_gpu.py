"""Expert parallelism on GPUs over NCCL: two ranks, one per GPU, each owning
half of the routed experts, must reproduce the single-GPU layer (same
quantised weights, router and shared expert) on every rank's own tokens.
Needs two GPUs; skipped otherwise."""
import multiprocessing as mp
import os
import socket
import traceback

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

E, H, I, K, T, IS = 8, 256, 256, 2, 24, 256


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, q):
    try:
        import sys
        from datetime import timedelta
        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path.insert(0, root)
        import torch.distributed as dist
        from oracle import blut_oracle as O
        from tests._helpers import check_layer, cuda, build_b_layer
        from block_lut_b200.ep import EPMoELayer, expert_ranges
        from block_lut_b200.formats import LUTFormat
        from block_lut_b200.moe import LUTExperts, LUTMoELayer, SharedExpert

        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, init_method=f"tcp://127.0.0.1:{port}",
                                timeout=timedelta(seconds=60), device_id=torch.device("cuda", rank))
        fmt = LUTFormat("b", 4, 64)
        full, _, _ = build_b_layer(fmt, E=E, H=H, I=I, seed=41)  # identical on both ranks
        s, c = expert_ranges(E, world)[rank]
        mine = LUTExperts(full.fmt, c, H, I, full.w13[s * full.w13_stride:(s + c) * full.w13_stride],
                          full.w13_stride, full.w2[s * full.w2_stride:(s + c) * full.w2_stride], full.w2_stride,
                          None, full.tc)
        rng = np.random.Generator(np.random.PCG64(5))
        rw = cuda((rng.standard_normal((E + 1, H)) * 0.05).astype(np.float16))
        s13 = cuda(O.student_t_weights(rng, (2 * IS, H)).astype(np.float16))
        s2 = cuda(O.student_t_weights(rng, (H, IS)).astype(np.float16))
        x = cuda(O.rms_activations(np.random.Generator(np.random.PCG64(100 + rank)), T, H).astype(np.float16))
        ep = EPMoELayer(mine, E, K, rw, shared=(s13, s2))
        out = ep.forward(x)
        ref = LUTMoELayer(full, K, router_w=rw, shared=SharedExpert.from_dense(s13, s2), shared_gate_mode=1)
        want = ref.forward(x)
        torch.cuda.synchronize()
        check_layer(out, want.float().cpu().numpy().astype(np.float64), torch.float16, f"ep rank {rank}")
        ep.local.check_status()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok", ""))
    except BaseException:  # report every failure to the parent
        q.put((rank, "error", traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="expert parallelism over NCCL needs two GPUs")
def test_ep_nccl_two_gpus_matches_single_gpu():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, status, msg in sorted(results):
        assert status == "ok", f"rank {rank}:\n{msg}"


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_one_process_drives_two_devices():
    """Launch set-up (shared-memory attributes, occupancy, SM count, the side
    stream) is per device: the same layer built on cuda:0 and cuda:1 in one
    process gives the same result on both."""
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from oracle import blut_oracle as O
    from block_lut_b200.formats import LUTFormat, QuantizedMatrix
    from block_lut_b200.moe import LUTExperts, LUTMoELayer, SharedExpert
    fmt = LUTFormat("b", 4, 64)
    rng = np.random.Generator(np.random.PCG64(9))
    mats = []
    for _ in range(E):
        for rows, cols in ((2 * I, H), (H, I)):
            packed, tables = O.encode_b(O.student_t_weights(rng, (rows, cols)), 4, 64)
            mats.append((rows, cols, packed, tables))
    s13 = O.student_t_weights(rng, (2 * IS, H)).astype(np.float16)
    s2 = O.student_t_weights(rng, (H, IS)).astype(np.float16)
    x = O.rms_activations(rng, T, H).astype(np.float16)
    ids, tw = O.routing(rng.standard_normal((T, E)).astype(np.float32), K)
    outs = []
    for dev in ("cuda:0", "cuda:1"):
        q = [QuantizedMatrix(fmt, r, c, torch.from_numpy(p).to(dev), torch.from_numpy(t).to(dev)) for r, c, p, t in mats]
        ex = LUTExperts.from_quantized(q[0::2], q[1::2])
        sh = SharedExpert.from_dense(torch.from_numpy(s13).to(dev), torch.from_numpy(s2).to(dev))
        layer = LUTMoELayer(ex, K, shared=sh, shared_gate_mode=0)
        with torch.cuda.device(dev):
            out = layer.forward(torch.from_numpy(x).to(dev), torch.from_numpy(ids).to(dev),
                                torch.from_numpy(tw).to(dev))
            torch.cuda.synchronize()
            layer.check_status()
        outs.append(out.cpu())
    assert torch.equal(outs[0], outs[1])
