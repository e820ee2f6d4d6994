"""Expert parallelism over the GPUs of one box (torch.distributed, NCCL).

Experts shard naturally: rank r owns the contiguous expert range
``expert_ranges(E, world)[r]`` of every layer (E=60 on 8 ranks -> 8,8,8,8,7,7,7,7),
dense weights are replicated, and every rank routes its own decode batch.
One layer:

1. router on the rank's own tokens (global expert ids, weights, shared gate);
2. dispatch: every token travels to every rank with its k slots rewritten to
   that rank's local expert ids, -1 where the expert lives elsewhere
   (fixed T rows per destination, so no count exchange is needed);
   three ``all_to_all_single`` calls (activations, ids, weights);
3. each rank runs its local experts on the N*T received tokens in one
   ``blut_moe_forward`` (empty slots are skipped) with fp32 partial sums;
4. combine: ``all_to_all_single`` sends the partials back; the owner sums the
   N partials and adds its shared expert, which ran on a side stream beside
   the exchanges and the local experts (it needs only the rank's own tokens).

These are the message shapes of the reference's only EP code (the DeepSeek
remote code's dispatch/combine all_to_all, models/deepseek/modeling_deepseek.py:604-660).
The exchange functions are device-agnostic (CPU tensors under gloo in the
tests); the expert compute is the CUDA path.
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import torch
import torch.distributed as dist

from .formats import dense_matrix
from .moe import LUTExperts, LUTMoELayer, SharedExpert, router


def expert_ranges(num_experts: int, world: int) -> List[Tuple[int, int]]:
    """Contiguous (start, count) per rank; the first E % world ranks get one more."""
    base, extra = divmod(num_experts, world)
    out, s = [], 0
    for r in range(world):
        c = base + (1 if r < extra else 0)
        out.append((s, c))
        s += c
    return out


def owner_tables(num_experts: int, world: int, device) -> Tuple[torch.Tensor, torch.Tensor]:
    """owner[e] = rank of expert e, local[e] = e - start(owner)."""
    owner = torch.empty(num_experts, dtype=torch.int32)
    local = torch.empty(num_experts, dtype=torch.int32)
    for r, (s, c) in enumerate(expert_ranges(num_experts, world)):
        owner[s:s + c] = r
        local[s:s + c] = torch.arange(c, dtype=torch.int32)
    return owner.to(device), local.to(device)


def build_dispatch(x: torch.Tensor, ids: torch.Tensor, tw: torch.Tensor, owner: torch.Tensor,
                   local: torch.Tensor, world: int):
    """Send buffers [world, T, ...]: x replicated, per-destination local ids (-1 elsewhere), weights."""
    T, k = ids.shape
    ids_l = ids.long()
    own = owner[ids_l]                                             # [T, k]
    loc = local[ids_l]                                             # [T, k]
    dest = torch.arange(world, device=ids.device, dtype=own.dtype).view(world, 1, 1)
    send_ids = torch.where(own.unsqueeze(0) == dest, loc.unsqueeze(0), torch.full_like(loc, -1).unsqueeze(0))
    send_x = x.unsqueeze(0).expand(world, T, x.shape[1]).contiguous()
    send_w = tw.float().unsqueeze(0).expand(world, T, k).contiguous()
    return send_x, send_ids.to(torch.int32).contiguous(), send_w


def exchange(send_x, send_ids, send_w, group=None):
    """Dispatch all-to-all (equal splits): row block d of each buffer goes to rank d."""
    recv_x, recv_ids, recv_w = torch.empty_like(send_x), torch.empty_like(send_ids), torch.empty_like(send_w)
    dist.all_to_all_single(recv_x, send_x, group=group)
    dist.all_to_all_single(recv_ids, send_ids, group=group)
    dist.all_to_all_single(recv_w, send_w, group=group)
    return recv_x, recv_ids, recv_w


def combine(partials: torch.Tensor, group=None) -> torch.Tensor:
    """Combine all-to-all: partials [world, T, H] (block d = tokens of rank d) -> summed [T, H]."""
    back = torch.empty_like(partials)
    dist.all_to_all_single(back, partials, group=group)
    return back.sum(dim=0)


class EPMoELayer:
    """One MoE layer, expert-parallel: this rank's experts + replicated router and shared expert."""

    def __init__(self, local_experts: LUTExperts, num_experts: int, top_k: int, router_w: torch.Tensor,
                 shared: Optional[Tuple[torch.Tensor, torch.Tensor]] = None, renorm: bool = False, group=None):
        self.world = dist.get_world_size(group)
        self.group = group
        self.top_k = top_k
        self.renorm = renorm
        self.local = LUTMoELayer(local_experts, top_k)
        self.router_w = router_w.to(local_experts.fmt.compute_dtype).contiguous()
        self.num_experts = num_experts
        self.owner, self.local_id = owner_tables(num_experts, self.world, router_w.device)
        self.shared = None
        if shared is not None:
            s13, s2 = shared
            ex = LUTExperts.from_quantized([dense_matrix(s13)], [dense_matrix(s2)])
            self.shared = LUTMoELayer(ex, 1)
            self.shared.ws_slot = 1  # runs concurrently with self.local: its own workspace
            self._zero_ids = None
            self._side = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        T, H = x.shape
        ids, tw, sg = router(x, self.router_w, self.top_k, self.renorm, shared_gate=self.shared is not None)
        shared_out = None
        if self.shared is not None:
            # the shared expert needs only this rank's tokens: it runs on a side
            # stream while the tokens are exchanged and the local experts run;
            # every tensor it touches was made on the main stream, which waits
            # for the side stream before returning
            if self._zero_ids is None or self._zero_ids.shape[0] != T:
                self._zero_ids = torch.zeros(T, 1, dtype=torch.int32, device=x.device)
            if self._side is None:
                self._side = torch.cuda.Stream(device=x.device)
            main = torch.cuda.current_stream(x.device)
            shared_out = torch.empty(T, H, dtype=torch.float32, device=x.device)
            self._side.wait_stream(main)
            with torch.cuda.stream(self._side):
                self.shared.forward(x, self._zero_ids, sg.view(T, 1), out=shared_out, out_f32=True)
        sx, si, sw = build_dispatch(x, ids, tw, self.owner, self.local_id, self.world)
        rx, ri, rw = exchange(sx, si, sw, self.group)
        part = self.local.forward(rx.view(-1, H), ri.view(-1, self.top_k), rw.view(-1, self.top_k), out_f32=True)
        out = combine(part.view(self.world, T, H), self.group)
        if shared_out is not None:
            main.wait_stream(self._side)
            out += shared_out
        return out.to(x.dtype)

    __call__ = forward


def run_bench_ep(a, rank, world, dev, build_layers, make_inputs, Clocks, peaks, metric, shp, fmt, format_name):
    """bench.py --gpus N: every rank owns E/N experts of each layer and a decode
    batch of its own; value = total tokens of all ranks / max step time."""
    import json

    H, E, I, TOPK, IS = shp["H"], shp["E"], shp["I"], shp["TOPK"], shp["IS"]
    s, c = expert_ranges(E, world)[rank]
    fmt, layers = build_layers(a.layers, c, s, fmt, dev, shape=dict(shp, IS=0))
    eps = []
    g = torch.Generator(device=dev).manual_seed(99)
    for ex, rw, _ in layers:
        shared = None
        if IS > 0:
            s13 = (torch.randn(2 * IS, H, generator=g, device=dev) * 0.02).to(fmt.compute_dtype)
            s2 = (torch.randn(H, IS, generator=g, device=dev) * 0.02).to(fmt.compute_dtype)
            shared = (s13, s2)
        eps.append(EPMoELayer(ex, E, TOPK, rw if shared is not None else rw[:E].contiguous(),
                              shared=shared, renorm=shp["RENORM"]))
    xs = make_inputs(a.layers, a.batch, rank, dev, H, fmt.compute_dtype)

    outs = [None] * len(eps)

    def step():
        for i, (m, x) in enumerate(zip(eps, xs)):
            outs[i] = m.forward(x)

    for _ in range(max(2, a.warmup)):
        step()
    torch.cuda.synchronize()
    for m in eps:
        m.local.check_status()
    # the whole step (routing, exchanges, expert kernels) as one CUDA graph;
    # every rank captures the same collectives in the same order
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    dist.barrier()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(max(1, a.warmup)):
        graph.replay()
    torch.cuda.synchronize()
    dist.barrier()
    clk = Clocks(torch.cuda.current_device())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    dist.barrier()
    e0.record()
    for _ in range(a.steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    dist.barrier()
    del graph  # a graph holding NCCL work is released before the process group
    clocks = clk.stop()
    ms = torch.tensor([e0.elapsed_time(e1) / a.steps], device=dev)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms.item())
    total_tokens = a.batch * world
    peak, _ = peaks()
    # e2e through EPMoELayer.forward: each rank's tokens from pinned host
    # memory to the device and its layer outputs back, every step
    xh = [x.cpu().pin_memory() for x in xs]
    oh = [torch.empty_like(x, device="cpu").pin_memory() for x in xs]
    xd = [torch.empty_like(x) for x in xs]

    def e2e_step():
        for m, h_in, d_in, h_out in zip(eps, xh, xd, oh):
            d_in.copy_(h_in, non_blocking=True)
            h_out.copy_(m.forward(d_in), non_blocking=True)
    e2e_step()
    torch.cuda.synchronize()
    dist.barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for _ in range(a.steps):
        e2e_step()
    f1.record()
    torch.cuda.synchronize()
    e_ms = torch.tensor([f0.elapsed_time(f1) / a.steps], device=dev)
    dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
    e_ms = float(e_ms.item())
    # this library's kernels per step: router (logits + top-k), local experts
    # on all ranks' tokens, shared expert on the rank's own tokens
    m0 = eps[0]
    per_layer = 2 + m0.local.launch_count(world * a.batch, caller_routing=True) + (
        m0.shared.launch_count(a.batch, caller_routing=True) if m0.shared is not None else 0)
    if rank == 0:
        res = {"metric": metric, "value": total_tokens / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
               "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True,
               "scaling": "weak", "vs_baseline": None, "dtype": "bf16" if fmt.kind == "r8" else "f16",
               "data": "synthetic: Student-t(df=5) std 0.02 weights, GPU Lloyd-encoded; N(0,1) RMS-normalised fp16",
               "config": {"workload": f"{shp['NAME']}, decode batch {a.batch} per rank",
                          "layers": a.layers, "global_batch": total_tokens, "experts": E, "top_k": TOPK,
                          "format": format_name(fmt), "parallelism": f"ep{world}",
                          "exchange": "NCCL all_to_all_single dispatch (x, ids, w) + combine (fp32 partials)"},
               "graph": f"CUDA graph of the {a.layers}-layer step, NCCL collectives included",
               "roofline": None, "cpu_baseline": None,
               "e2e": {"value": total_tokens / (e_ms / 1e3), "unit": "tokens/s", "ms_per_step": e_ms,
                       "h2d_bytes_per_step": sum(x.numel() * 2 for x in xs) * world,
                       "d2h_bytes_per_step": sum(x.numel() * 2 for x in xs) * world,
                       "path": "EPMoELayer.forward per layer with pinned host I/O on every rank"},
               "gpu_launches": a.steps * a.layers * per_layer, "clocks": clocks}
        print(json.dumps(res), flush=True)
    dist.barrier()
    dist.destroy_process_group()
