"""Expert parallelism on GPUs over peer memory: two ranks, one per GPU, each
owning half of the routed experts, exchange token rows with blut_ep_dispatch /
blut_ep_combine (direct stores and loads in the other GPU's memory).  Every
rank's output must match the float64 oracle on its own tokens (router ids
and weights from the same router kernel) and the single-GPU layer, over
several exchanges of varying batch size, two layers sharing one exchange
window, and a CUDA graph replay.  A rank that never dispatches makes the
other rank's bounded wait give up with BLUT_ERR_TIMEOUT (no hang, no fault).
Needs two GPUs; skipped otherwise.  NVLS is off (NCCL carries only the set-up
and barriers here)."""
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


def _rank_main(rank, world, port, q, mode):
    """GPU work first, checks after: a rank leaves only through the
    collective close of the exchange window, so no rank exits (freeing its
    window) while another may still store into it."""
    try:
        import sys
        from datetime import timedelta
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path.insert(0, root)
        import torch.distributed as dist
        from oracle import blut_oracle as O
        from tests._helpers import check_layer, cuda, build_b_layer
        from block_lut_b200 import _lib
        from block_lut_b200.ep import EPMoELayer, PeerExchange, expert_ranges
        from block_lut_b200.formats import LUTFormat
        from block_lut_b200.moe import LUTExperts, LUTMoELayer, SharedExpert, router

        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, init_method=f"tcp://127.0.0.1:{port}",
                                timeout=timedelta(seconds=60), device_id=torch.device("cuda", rank))
        fmt = LUTFormat("b", 4, 64)
        full, W13, W2 = build_b_layer(fmt, E=E, H=H, I=I, seed=41)  # identical on both ranks
        s, c = expert_ranges(E, world)[rank]
        mine = LUTExperts(full.fmt, c, H, I, full.w13[s * full.w13_stride:(s + c) * full.w13_stride],
                          full.w13_stride, full.w2[s * full.w2_stride:(s + c) * full.w2_stride], full.w2_stride,
                          None, full.tc)
        rng = np.random.Generator(np.random.PCG64(5))
        rw = cuda((rng.standard_normal((E + 1, H)) * 0.05).astype(np.float16))
        rw2 = cuda((rng.standard_normal((E, H)) * 0.05).astype(np.float16))
        s13 = cuda(O.student_t_weights(rng, (2 * IS, H)).astype(np.float16))
        s2 = cuda(O.student_t_weights(rng, (H, IS)).astype(np.float16))
        xchg = PeerExchange(T, H, K, torch.float16, f"cuda:{rank}")
        layers = [EPMoELayer(mine, E, K, rw, xchg, shared=(s13, s2)), EPMoELayer(mine, E, K, rw2, xchg)]
        refs = [LUTMoELayer(full, K, router_w=rw, shared=SharedExpert.from_dense(s13, s2), shared_gate_mode=1),
                LUTMoELayer(full, K, router_w=rw2)]
        records, err, status = [], None, None
        try:
            dist.barrier()
            if mode == "timeout":
                # rank 1 never dispatches: rank 0's wait for its rows runs out
                _lib.lib().blut_debug_set_wait_limit(50_000_000)
                if rank == 0:
                    x = cuda(O.rms_activations(np.random.Generator(np.random.PCG64(1)), T, H).astype(np.float16))
                    ids, tw, _ = router(x, rw2, K)
                    xchg.dispatch(x, ids, tw, layers[1].owner, layers[1].local_id)
                    try:
                        xchg.check_status()
                        status = "no timeout"
                    except RuntimeError as exc:
                        status = str(exc)
                _lib.lib().blut_debug_set_wait_limit(0)
            else:
                xs, eager = None, None
                for it, n in enumerate((T, T, T // 2 + 1, 1, T)):  # every exchange advances the epoch
                    # each layer gets its own RMS-normalised rows (outputs of a
                    # layer are far smaller, and fp16 quantises them coarsely)
                    xs = [cuda(O.rms_activations(np.random.Generator(np.random.PCG64(100 + 10 * rank + 2 * it + li)),
                                                 n, H).astype(np.float16)) for li in range(2)]
                    eager = []
                    for li, (lay, ref, h) in enumerate(zip(layers, refs, xs)):
                        out = lay.forward(h)
                        want = ref.forward(h)
                        ids, tw, _ = router(h, lay.router_w, K, shared_gate=li == 0)
                        records.append((it, li, h.float().cpu().numpy(), out.float().cpu(),
                                        want.float().cpu().numpy().astype(np.float64), ids.cpu().numpy(),
                                        tw.cpu().numpy()))
                        eager.append(out)
                xchg.check_status()
                # the two layers as one CUDA graph: replays give the eager result
                side = torch.cuda.Stream()
                side.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(side):
                    for lay, h in zip(layers, xs):
                        lay.forward(h)
                torch.cuda.current_stream().wait_stream(side)
                torch.cuda.synchronize()
                dist.barrier()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    gout = [lay.forward(h) for lay, h in zip(layers, xs)]
                for _ in range(3):
                    g.replay()
                torch.cuda.synchronize()
                same = all(torch.equal(a_, b_) for a_, b_ in zip(gout, eager))
                status = "graph equal" if same else "graph replay differs from the eager exchange"
                xchg.check_status()
                for lay in layers:
                    lay.local.check_status()
                del g
        except BaseException:
            err = traceback.format_exc()
        xchg.close()
        dist.destroy_process_group()
        if err:
            raise RuntimeError(err)
        if mode == "timeout":
            if rank == 0:
                assert "timed out" in status.lower() or "timeout" in status.lower(), status
        else:
            assert status == "graph equal", status
            s13n, s2n, gate = s13.float().cpu().numpy(), s2.float().cpu().numpy(), rw[E].float().cpu().numpy()
            for it, li, hn, out, want, ids, tw in records:
                kw = dict(shared13=s13n, shared2=s2n, shared_gate=gate) if li == 0 else {}
                ref64 = O.moe_forward(hn, ids, tw, W13, W2, act_dtype="f16", **kw)
                check_layer(out, ref64, torch.float16, f"ep rank {rank} step {it} layer {li}")
                check_layer(out, want, torch.float16, f"ep vs single gpu, rank {rank} step {it} layer {li}")
        q.put((rank, "ok", ""))
    except BaseException:  # report every failure to the parent
        q.put((rank, "error", traceback.format_exc()))


def _run_two(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q, mode)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    for rank, status, msg in sorted(results):
        assert status == "ok", f"rank {rank}:\n{msg}"


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="expert parallelism over peer memory needs two GPUs")
def test_ep_peer_exchange_two_gpus_matches_oracle_and_single_gpu():
    _run_two("parity")


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_ep_silent_rank_times_out_cleanly():
    _run_two("timeout")


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
