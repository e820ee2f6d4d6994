#!/usr/bin/env python
"""LUT-MoE decode throughput on B200 (config 2's MoE stack: Qwen1.5-MoE-A2.7B).

Workload: the 24 MoE layers of Qwen1.5-MoE-A2.7B at decode -- per layer a
softmax top-4 router over 60 routed experts (SwiGLU, I=1408) quantised to
BlockLUT 4-bit with one 16-entry fp16 codebook per (row, 64-column block),
plus the dense fp16 shared expert (I=5632) gated by sigmoid(x . g).  One
step = one decode step of a batch through all 24 MoE layers (attention and
the dense projections are outside the LUT path and are not run).  Weights are
synthetic Student-t(df=5) scaled to std 0.02 (seed 0), GPU-encoded with the
Lloyd encoder; activations are N(0,1) fp16, RMS-normalised.  Per step the
expert weights streamed (~12.7 GB) exceed the 126 MB L2, so no flush is needed.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Rank 0 prints one JSON line.  Under torchrun (N > 1) the layers run expert
parallel: each rank owns E/N experts of every layer and its own decode batch,
tokens are exchanged with NCCL all-to-all (dispatch and combine).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

H, E, I, TOPK, IS, LAYERS = 2048, 60, 1408, 4, 5632, 24
QWEN = dict(H=H, E=E, I=I, IS=IS, TOPK=TOPK, LAYERS=LAYERS, RENORM=False, BATCH=32,
            NAME="Qwen1.5-MoE-A2.7B MoE stack", KIND="b")
# Config 3: the 48 MoE layers of Qwen3-30B-A3B at decode -- 128 routed
# experts of I 768, top-8 softmax renormalised, no shared expert, batch 64,
# NestedLUT 2+2 with g 64 (full tier, or coarse only with --tier 1).
QWEN3 = dict(H=2048, E=128, I=768, IS=0, TOPK=8, LAYERS=48, RENORM=True, BATCH=64,
             NAME="Qwen3-30B-A3B MoE stack", KIND="nested")
# DRAM read + write over algorithmic bytes of the routed tcgen05 launches, from
# one ncu capture per format (profiles/: tc_mm_kernel_qwen15_decode_b32.md,
# tc_mm_kernel_qwen15_formatR_decode_b32.md,
# tc_mm_kernel_qwen3_nested_coarse_b64.md); formats without a capture report
# no traffic
TRAFFIC_RATIOS = {("b", 4, 64, 0): 1.024, ("r8", 8, 128, 0): 1.035, ("nested", 4, 64, 1): 1.06}
METRIC = "LUT-MoE decode tokens/s; expert LUT-GEMV HBM GB/s vs ~8 TB/s peak"
# Config 4: DeepSeek-V2-Lite MoE layers (26 of 27; layer 0 is dense),
# 64 routed experts of I 1408, top-6 softmax, two shared experts (one MLP of
# I 2816), prefill of 8 x 4096 tokens.
DSV2 = dict(H=2048, E=64, I=1408, IS=2816, TOPK=6, LAYERS=26, TOKENS=8 * 4096, RENORM=False,
            NAME="DeepSeek-V2-Lite MoE stack", KIND="b")
PREFILL_METRIC = "LUT-MoE prefill tokens/s; grouped LUT-GEMM tensor TFLOP/s"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=None,
                   help="timed steps (default: 200 decode, 100 qwen3, 5 prefill / sweep; about a second each)")
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--batch", type=int, default=None, help="decode tokens per rank (workload default)")
    p.add_argument("--layers", type=int, default=None, help="MoE layers (workload default)")
    p.add_argument("--kind", choices=["b", "nested", "r8"], default=None,
                   help="expert format (workload default): Format B, NestedLUT, or the reference's Format R")
    p.add_argument("--bits", type=int, default=4, help="Format B code bits")
    p.add_argument("--group", type=int, default=64)
    p.add_argument("--tier", type=int, default=0, help="NestedLUT tier (0 full, 1 coarse only) or Format R tier")
    p.add_argument("--path", choices=["auto", "tc", "mma"], default="auto",
                   help="matmul path of the experts: tcgen05 where the format has it (auto), or forced")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu", action="store_true")
    p.add_argument("--workload", choices=["decode", "qwen3", "prefill", "sweep", "tiers", "vllm"], default="decode",
                   help="decode: the headline metric (config 2); qwen3: config 3's MoE stack at decode; "
                        "prefill: config 4's MoE layers; sweep: config 5's single-matrix kernel sweep; "
                        "tiers: Format R progressive bit-plane tier recover; vllm: config 2 end to end "
                        "through vLLM with the lut plugin")
    p.add_argument("--vllm-model", choices=["qwen15", "qwen3", "dsv2lite"], default="qwen15",
                   help="--workload vllm: config 2's Qwen1.5-MoE-A2.7B, config 3's Qwen3-30B-A3B, or config 4's "
                        "DeepSeek-V2-Lite architecture (prefill of 8 x 4096 tokens)")
    p.add_argument("--sweep-bits", default="2,3,4")
    p.add_argument("--sweep-groups", default="32,64,128")
    p.add_argument("--sweep-m", default="1,2,4,8,16,64,256,1024,4096")
    a = p.parse_args()
    if a.steps is None:
        a.steps = {"decode": 200, "qwen3": 100}.get(a.workload, 5)
    qwen3 = a.workload == "qwen3" or (a.workload == "vllm" and a.vllm_model == "qwen3")
    dsv2 = a.workload == "prefill" or (a.workload == "vllm" and a.vllm_model == "dsv2lite")
    a.shape = QWEN3 if qwen3 else DSV2 if dsv2 else QWEN
    a.batch = a.batch if a.batch is not None else a.shape.get("BATCH", 32)
    a.layers = a.layers if a.layers is not None else a.shape["LAYERS"]
    a.kind = a.kind or a.shape.get("KIND", "b")
    return a


def bench_format(a):
    from block_lut_b200.formats import LUTFormat
    if a.kind == "r8":
        return LUTFormat("r8", 8, 128, a.tier)
    return LUTFormat("nested", 4, a.group, a.tier) if a.kind == "nested" else LUTFormat("b", a.bits, a.group)


def bench_path(a):
    return None if a.path == "auto" else a.path == "tc"


def format_name(fmt):
    if fmt.kind == "r8":
        return f"Format R (reference BlockLUT): uint8 index, bf16 256-entry table (tier {fmt.tier}), " \
               "bf16 absmax per 128 weights"
    if fmt.kind == "nested":
        return f"NestedLUT 2+2 g{fmt.group} {'coarse-only' if fmt.tier == 1 else 'full'} tier fp16 tables"
    return f"BlockLUT {fmt.bits}-bit g{fmt.group} fp16 tables"


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ---------------------------------------------------------------- clocks --
class Clocks:
    """nvidia-smi sampler running during the timed region."""

    def __init__(self, index: int):
        self.path = tempfile.mktemp(suffix=".csv")
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.f = open(self.path, "w")
            self.p = subprocess.Popen(["nvidia-smi", f"--id={index}", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                       "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self):
        if self.p is None:
            return None
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except Exception:
            self.p.kill()
        self.f.close()
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [s.strip() for s in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------ workload ---
def build_layers(n_layers, experts_local, e0, fmt, device, seed=0, shape=None, tc=None):
    """Synthetic MoE layers (experts [e0, e0 + experts_local) of each) in
    format `fmt`; shape {H, E, I, IS} defaults to Qwen1.5-MoE-A2.7B's (IS 0:
    no shared expert)."""
    import torch
    from block_lut_b200.formats import QuantizedMatrix, encode, encode_r
    from block_lut_b200.moe import LUTExperts, SharedExpert
    H, E, I, IS = (shape or QWEN)["H"], (shape or QWEN)["E"], (shape or QWEN)["I"], (shape or QWEN)["IS"]
    dt = fmt.compute_dtype
    # Format R: one 256-entry table for every matrix (evenly spaced over the
    # absmax-normalised range [-1, 1]), uint8 nearest-entry indices
    cb = torch.linspace(-1.0, 1.0, 256, device=device).to(torch.bfloat16)

    def quantise(w, rows, cols):
        if fmt.kind == "r8":
            idx, am = encode_r(w, cb)
            return QuantizedMatrix(fmt, rows, cols, idx, cb, scales=am)
        return encode(w, fmt)

    torch.manual_seed(seed)
    st = torch.distributions.StudentT(torch.tensor(5.0, device=device))
    scale = 0.02 / (5.0 / 3.0) ** 0.5
    layers = []
    for li in range(n_layers):
        gen = torch.Generator(device=device).manual_seed(seed * 1000 + li)
        q13, q2 = [], []
        for e in range(E):
            if e0 <= e < e0 + experts_local:
                torch.manual_seed(seed * 100000 + li * 100 + e)
                q13.append(quantise(st.sample((2 * I, H)) * scale, 2 * I, H))
                q2.append(quantise(st.sample((H, I)) * scale, H, I))
        experts = LUTExperts.from_quantized(q13, q2, tc=tc)
        del q13, q2
        router_w = (torch.randn(E + 1, H, generator=gen, device=device) * 0.02).to(dt)
        shared = None
        if IS > 0:
            s13 = (torch.randn(2 * IS, H, generator=gen, device=device) * 0.02).to(dt)
            s2 = (torch.randn(H, IS, generator=gen, device=device) * 0.02).to(dt)
            shared = SharedExpert.from_dense(s13, s2)
        layers.append((experts, router_w, shared))
    torch.cuda.synchronize()
    return fmt, layers


def make_inputs(n_layers, batch, rank, device, hidden=H, dtype=None):
    import torch
    dtype = dtype or torch.float16
    g = torch.Generator(device=device).manual_seed(7 + rank)
    xs = []
    for _ in range(n_layers):
        x = torch.randn(batch, hidden, generator=g, device=device)
        x = x / x.pow(2).mean(dim=1, keepdim=True).sqrt()
        xs.append(x.to(dtype).contiguous())
    return xs


def cpu_model() -> str:
    """The host CPU's model name (lscpu's "Model name", from /proc/cpuinfo)."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


class CpuLayer:
    """Bounded CPU sample of the workload: one MoE layer at the bench batch,
    run by the torch restatement of the reference's apply
    (``oracle/blut_torch_ref.py``: per active expert, dequantise the whole
    expert, F.linear over all tokens, SiLU * up, F.linear, weighted
    scatter-add) on all host cores.  Its experts carry random codes of the
    workload's format (Format R: uint8 indices, bf16 absmax, a bf16 table;
    Format B / NestedLUT: packed codes and sorted fp16 tables per (row,
    block)); dequantisation is timed, as it is part of every reference call."""

    def __init__(self, batch, fmt, shape=None, seed=0):
        import torch
        from oracle import blut_oracle as O
        from oracle import blut_torch_ref as R
        torch.set_num_threads(os.cpu_count() or 1)
        self.threads = torch.get_num_threads()
        sh = shape or QWEN
        h_, e_, i_, is_, k_ = sh["H"], sh["E"], sh["I"], sh["IS"], sh["TOPK"]
        rng = np.random.Generator(np.random.PCG64(seed))
        g = torch.Generator().manual_seed(seed)
        x = O.rms_activations(rng, batch, h_).astype(np.float32)
        ids, tw = O.routing(rng.standard_normal((batch, e_)).astype(np.float32), k_, renorm=sh["RENORM"])
        self.active = sorted(set(ids.reshape(-1).tolist()))
        bf16 = fmt.kind == "r8"
        self.x = torch.from_numpy(x).to(torch.bfloat16 if bf16 else torch.float16)
        self.ids = torch.from_numpy(ids).long()
        self.tw = torch.from_numpy(tw).to(self.x.dtype)

        def tables(rows, cols, ent):
            t = torch.randn(rows, cols // fmt.group, ent, generator=g) * 0.02
            return t.sort(dim=-1).values.half()

        def expert(rows, cols):
            if fmt.kind == "r8":
                idx = torch.randint(0, 256, (rows * cols,), generator=g, dtype=torch.uint8)
                am = (torch.rand(rows * cols // 128, generator=g) * 0.06 + 0.02).to(torch.bfloat16)
                return lambda: R.dequant_r(idx, am, self.cb, rows, cols)  # noqa: E731
            if fmt.kind == "nested":
                cc = torch.randint(0, 256, (rows, cols // 4), generator=g, dtype=torch.uint8)
                cr = torch.randint(0, 256, (rows, cols // 4), generator=g, dtype=torch.uint8)
                ct, rt = tables(rows, cols, 4), tables(rows, cols, 16)
                return lambda: R.dequant_nested(cc, cr, ct, rt, fmt.group, rows, cols,  # noqa: E731
                                                coarse_only=fmt.tier == 1)
            codes = torch.randint(0, 256, (rows, cols * fmt.bits // 8), generator=g, dtype=torch.uint8)
            t = tables(rows, cols, 1 << fmt.bits)
            return lambda: R.dequant_b(codes, t, fmt.bits, fmt.group, rows, cols)  # noqa: E731

        self.cb = torch.linspace(-1.0, 1.0, 256).to(torch.bfloat16)
        self.w13 = {e: expert(2 * i_, h_) for e in self.active}
        self.w2 = {e: expert(h_, i_) for e in self.active}
        self.shared = None
        if is_ > 0:
            dt = self.x.dtype if bf16 else torch.float32
            self.shared = ((torch.randn(2 * is_, h_, generator=g) * 0.02).to(dt),
                           (torch.randn(h_, is_, generator=g) * 0.02).to(dt),
                           (torch.randn(h_, generator=g) * 0.02).to(dt))
        self.desc = (f"1 of {sh['LAYERS']} MoE layers at batch {batch} ({len(self.active)} active experts"
                     f"{' + shared expert' if is_ > 0 else ''}), torch CPU restatement of the reference's "
                     f"LUTFusedMoEMethod.apply (quant_method.py:261-277): per active expert whole-expert "
                     f"dequant + F.linear over all tokens, {'bf16' if bf16 else 'fp32'}; "
                     f"{self.threads} threads, {cpu_model()}")

    def run(self) -> float:
        """Seconds for one layer forward."""
        import torch
        import torch.nn.functional as F
        from oracle import blut_torch_ref as R
        t0 = time.perf_counter()
        out = R.apply(self.x, self.tw, self.ids, lambda e: self.w13[e](), lambda e: self.w2[e]())
        if self.shared is not None:
            s13, s2, sg = self.shared
            xs = self.x.to(s13.dtype)
            h = F.linear(xs, s13)
            si = s13.shape[0] // 2
            y = F.linear(F.silu(h[:, :si]) * h[:, si:], s2)
            out = out + (torch.sigmoid(xs @ sg)[:, None] * y).to(out.dtype)
        return time.perf_counter() - t0


def cpu_sample(batch, fmt, shape=None, seed=0, reps=2):
    """(seconds per layer: the faster of ``reps`` runs after one warm-up, CpuLayer)."""
    c = CpuLayer(batch, fmt, shape, seed)
    c.run()
    return min(c.run() for _ in range(reps)), c


# ------------------------------------------------------------------ ours --
def run_ours(a):
    import torch
    import torch.distributed as dist
    from block_lut_b200.moe import LUTMoELayer, LUTMoEStep, router

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
        return run_ep(a, rank, world, dev)

    W = a.shape
    Hh, Ee, Ii, ISs, K = W["H"], W["E"], W["I"], W["IS"], W["TOPK"]
    fmt, layers = build_layers(a.layers, Ee, 0, bench_format(a), dev, shape=W, tc=bench_path(a))
    moes = [LUTMoELayer(ex, K, router_w=rw if sh is not None else rw[:Ee].contiguous(), renorm=W["RENORM"],
                        shared=sh, shared_gate_mode=1) for ex, rw, sh in layers]
    xs = make_inputs(a.layers, a.batch, rank, dev, Hh, fmt.compute_dtype)
    outs = [torch.empty_like(x) for x in xs]

    def step():
        for m, x, o in zip(moes, xs, outs):
            m.forward(x, out=o)

    for _ in range(2):
        step()
    torch.cuda.synchronize()
    for m in moes:
        m.check_status()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(a.warmup):
        graph.replay()
    torch.cuda.synchronize()

    clk = Clocks(local)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(a.steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    clocks = clk.stop()
    ms = e0.elapsed_time(e1) / a.steps
    tokens_s = a.batch / (ms / 1e3)

    # dominant kernel: routed LUT matmuls (gate/up + down), per-launch CUDA events
    def routed_times(xs_, outs_):
        """(mean gate/up ms, mean down ms, active experts per layer) over the layers."""
        import ctypes as C
        n_act = []
        for m, x in zip(moes, xs_):
            ids, _, _ = router(x, m.router_w, K, renorm=W["RENORM"], shared_gate=m.shared is not None)
            n_act.append(int(torch.unique(ids).numel()))
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in moes]
        for ev in evs:  # torch creates the CUDA event on its first record
            for e in ev:
                e.record()
        torch.cuda.synchronize()
        gu, dn, reps = 0.0, 0.0, 5
        for _ in range(reps):
            for m, x, o, ev in zip(moes, xs_, outs_, evs):
                handles = (C.c_void_p * 4)(*[e.cuda_event for e in ev])
                m._args.prof_events = C.cast(handles, C.c_void_p)
                m.forward(x, out=o)
                m._args.prof_events = None
            torch.cuda.synchronize()
            for ev in evs:
                gu += ev[0].elapsed_time(ev[1])
                dn += ev[2].elapsed_time(ev[3])
        return gu / (reps * len(moes)), dn / (reps * len(moes)), n_act

    t_gu, t_dn, n_active = routed_times(xs, outs)
    bpw = fmt.bytes_per_weight()
    key = (fmt.kind, fmt.bits, fmt.group, fmt.tier if fmt.kind != "b" else 0)
    na = sum(n_active) / len(n_active)
    b_gu = na * 2 * Ii * Hh * bpw
    b_dn = na * Hh * Ii * bpw
    # at batch 1 the single-token path streams the dense shared expert inside
    # the same two launches as the routed experts
    tok1 = a.batch == 1 and moes[0].launch_count(1, caller_routing=False) == 3
    if tok1 and moes[0].shared is not None:
        sb = moes[0].shared.weight_bytes()
        b_gu += sb * 2 / 3
        b_dn += sb / 3
    achieved = (b_gu + b_dn) / ((t_gu + t_dn) / 1e3) / 1e9
    peak, peak_kind = peaks()

    # config 2's other decode point: batch 1, the same stack as its own CUDA graph
    batch1 = None
    if a.batch != 1:
        x1 = make_inputs(a.layers, 1, rank, dev, Hh, fmt.compute_dtype)
        o1 = [torch.empty_like(x) for x in x1]

        def step1():
            for m, x, o in zip(moes, x1, o1):
                m.forward(x, out=o)
        step1()
        torch.cuda.synchronize()
        g1 = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g1):
            step1()
        for _ in range(a.warmup):
            g1.replay()
        n1 = max(10, min(a.steps, 100))
        e0.record()
        for _ in range(n1):
            g1.replay()
        e1.record()
        torch.cuda.synchronize()
        ms1 = e0.elapsed_time(e1) / n1
        gu1, dn1, act1 = routed_times(x1, o1)
        na1 = sum(act1) / len(act1)
        shared_b = moes[0].shared.weight_bytes() if moes[0].shared is not None else 0.0
        # the single-token path (3 launches) runs the shared expert inside the
        # same gate/up and down launches as the routed experts
        fused = moes[0].launch_count(1, caller_routing=False) == 3
        b1 = na1 * 3 * Ii * Hh * bpw + (shared_b if fused else 0.0)
        what = ("single-token GEMV launches (routed experts + dense shared expert), per layer" if fused
                else "routed LUT matmuls (single-token GEMV), per layer")
        batch1 = {"value": 1.0 / (ms1 / 1e3), "unit": "tokens/s", "ms_per_step": ms1, "steps": n1,
                  "launches_per_layer": moes[0].launch_count(1, caller_routing=False),
                  "roofline": {"kernel": what, "bound": "hbm",
                               "achieved": b1 / ((gu1 + dn1) / 1e3) / 1e9, "peak": peak,
                               "frac": b1 / ((gu1 + dn1) / 1e3) / 1e9 / peak, "ms_gateup": gu1, "ms_down": dn1,
                               "bytes_per_layer": b1},
                  "layer_roofline": {"what": "whole layer step time against its weight bytes (routed experts, "
                                             "dense shared expert, router)",
                                     "bytes_per_layer": na1 * 3 * Ii * Hh * bpw + shared_b + (Ee + 1) * Hh * 2,
                                     "frac": (na1 * 3 * Ii * Hh * bpw + shared_b + (Ee + 1) * Hh * 2)
                                     / (ms1 / a.layers / 1e3) / 1e9 / peak}}

    # e2e through the public API: pinned host inputs -> device -> layers ->
    # host, every step.  The serving path is LUTMoEStep (one CUDA graph per
    # step, both transfers included); the same step through per-layer eager
    # LUTMoELayer.forward calls with per-layer copies is reported beside it.
    e2e = None
    if not a.no_e2e:
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        stepg = LUTMoEStep(moes, a.batch, dev)
        for h, x in zip(stepg.host_in, xs):
            h.copy_(x.cpu())
        for _ in range(max(1, a.warmup)):
            stepg.run()
        torch.cuda.synchronize()
        f0.record()
        for _ in range(a.steps):
            stepg.run()
        f1.record()
        torch.cuda.synchronize()
        g_ms = f0.elapsed_time(f1) / a.steps
        # the host copies of the outputs equal the device-timed graph's
        same = all(torch.equal(h, o.cpu()) for h, o in zip(stepg.host_out, outs))
        del stepg

        xh = [x.cpu().pin_memory() for x in xs]
        oh = [torch.empty_like(x, device="cpu").pin_memory() for x in xs]
        xd = [torch.empty_like(x) for x in xs]

        def e2e_step():
            for m, h_in, d_in, h_out in zip(moes, xh, xd, oh):
                d_in.copy_(h_in, non_blocking=True)
                h_out.copy_(m.forward(d_in), non_blocking=True)
        for _ in range(max(1, a.warmup)):
            e2e_step()
        torch.cuda.synchronize()
        f0.record()
        for _ in range(a.steps):
            e2e_step()
        f1.record()
        torch.cuda.synchronize()
        e_ms = f0.elapsed_time(f1) / a.steps
        e2e = {"value": a.batch / (g_ms / 1e3), "unit": "tokens/s", "ms_per_step": g_ms,
               "h2d_bytes_per_step": sum(x.numel() * 2 for x in xs),
               "d2h_bytes_per_step": sum(x.numel() * 2 for x in xs),
               "path": "LUTMoEStep.run: one CUDA graph per step that copies every layer's input from pinned "
                       "host memory in one transfer, runs LUTMoELayer.forward (router + experts + shared) per "
                       "layer and copies every output back to pinned host memory in one transfer",
               "outputs_match_device_graph": same,
               "eager": {"value": a.batch / (e_ms / 1e3), "ms_per_step": e_ms,
                         "path": "LUTMoELayer.forward per layer from Python with pinned host I/O"}}

    cpu = None
    if not a.no_cpu:
        dt, c = cpu_sample(a.batch, fmt, W)
        cpu = {"value": a.batch / (dt * a.layers), "unit": "tokens/s", "cores": c.threads, "kind": "port",
               "sample": c.desc, "ms_per_layer": dt * 1e3}

    per_layer_launches = moes[0].launch_count(a.batch, caller_routing=False)
    res = {
        "metric": METRIC, "value": tokens_s, "unit": "tokens/s", "n_gpus": 1, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16" if fmt.kind == "r8" else "f16",
        "data": "synthetic: Student-t(df=5) std 0.02 weights, GPU-encoded (Lloyd tables, or Format R nearest "
                "entry of an evenly spaced table); N(0,1) RMS-normalised tokens",
        "config": {"workload": f"{W['NAME']}, decode batch {a.batch}", "layers": a.layers,
                   "global_batch": a.batch, "experts": Ee, "top_k": K, "renorm": W["RENORM"], "hidden": Hh,
                   "inter": Ii, "shared_inter": ISs, "format": format_name(fmt),
                   "parallelism": "single GPU", "graph": f"CUDA graph of the {a.layers}-layer step",
                   "l2": f"inputs larger than L2: {sum(n_active) * 3 * Ii * Hh * bpw / 1e9:.1f} GB of expert "
                         f"weights streamed per step"},
        "roofline": {"kernel": "tok1_kernel (single-token GEMV launches: routed experts + dense shared expert, "
                               "per layer)" if tok1 else
                               ("tc_mm_kernel (tcgen05" if moes[0].experts.tc else "lut_mm_kernel (mma.sync") +
                               "; routed gate/up+SiLU*up and down, per layer)", "bound": "hbm",
                     "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                     else "fallback 6650 GB/s",
                     # DRAM read + write per layer: the algorithmic bytes times the ratio an
                     # ncu capture of this format's routed launches measured (TRAFFIC_RATIOS)
                     "traffic": (b_gu + b_dn) * TRAFFIC_RATIOS[key] if moes[0].experts.tc and key in
                     TRAFFIC_RATIOS and not tok1 else None,
                     "bytes_per_layer": b_gu + b_dn, "ms_gateup": t_gu, "ms_down": t_dn,
                     "active_experts": na, "active_experts_per_layer": n_active[:4]},
        "cpu_baseline": cpu, "e2e": e2e, "batch1": batch1,
        "gpu_launches": a.steps * a.layers * per_layer_launches,
        "clocks": clocks,
    }
    print(json.dumps(res), flush=True)


def run_ep(a, rank, world, dev):
    from block_lut_b200.ep import run_bench_ep
    return run_bench_ep(a, rank, world, dev, build_layers, make_inputs, Clocks, peaks, METRIC, a.shape,
                        bench_format(a), format_name)


# ------------------------------------------------------------- reference --
def run_reference(a):
    """The reference arm: the torch CPU restatement of the reference's apply
    (CpuLayer) on the host cores.  A step is one MoE layer of the workload at
    the bench batch (the bounded sample); ``ms_per_step`` is that layer's
    time and ``value`` scales it to the whole stack (batch / (layers x
    time)).  Timing stops after about a minute of steps, so that the run
    ends within a few minutes whatever ``--steps`` asks for."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    fmt = bench_format(a)
    c = CpuLayer(a.batch, fmt, a.shape, seed=0)
    for _ in range(a.warmup):
        c.run()
    times = []
    for _ in range(a.steps):
        times.append(c.run())
        if sum(times) > 60:
            break
    dt = statistics.median(times)
    val = a.batch / (dt * a.layers)
    res = {"impl": "reference", "metric": METRIC, "value": val, "unit": "tokens/s", "n_gpus": world,
           "steps": len(times), "steps_requested": a.steps, "warmup": a.warmup, "ms_per_step": dt * 1e3,
           "step": f"one of the {a.layers} MoE layers (value = batch / ({a.layers} x median step time))",
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
           "dtype": "bf16" if fmt.kind == "r8" else "f32",
           "data": "synthetic random codes, absmax and sorted fp16 tables of the workload's shapes",
           "config": {"workload": f"{a.shape['NAME']}, decode batch {a.batch}", "layers": a.layers,
                      "global_batch": a.batch, "format": format_name(fmt), "cpu": cpu_model()},
           "cpu_baseline": {"value": val, "unit": "tokens/s", "cores": c.threads, "kind": "port",
                            "sample": c.desc},
           "e2e": {"value": val, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(res), flush=True)


def run_prefill(a):
    """Config 4 prefill: every MoE layer of the stack over one 8 x 4096-token
    batch, on one GPU.  Reported as tokens/s of the whole stack and, for the
    routed matmuls, as tensor TFLOP/s against the measured bf16 peak."""
    import ctypes as C
    import torch
    from block_lut_b200.moe import LUTMoELayer
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    n_layers = a.layers
    T, k = DSV2["TOKENS"], DSV2["TOPK"]
    fmt, layers = build_layers(n_layers, DSV2["E"], 0, bench_format(a), dev, shape=DSV2)
    moes = [LUTMoELayer(ex, k, router_w=rw[:DSV2["E"]].contiguous(), shared=sh, shared_gate_mode=0)
            for ex, rw, sh in layers]
    g = torch.Generator(device=dev).manual_seed(7)
    x = torch.randn(T, DSV2["H"], generator=g, device=dev)
    x = (x / x.pow(2).mean(dim=1, keepdim=True).sqrt()).half().contiguous()
    out = torch.empty_like(x)

    def step():
        for m in moes:
            m.forward(x, out=out)
    for _ in range(max(1, a.warmup)):
        step()
    torch.cuda.synchronize()
    for m in moes:
        m.check_status()
    clk = Clocks(0)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    clocks = clk.stop()
    ms = e0.elapsed_time(e1) / a.steps
    # routed matmul time per layer through the library's profiling events
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    for e in evs:
        e.record()
    torch.cuda.synchronize()
    handles = (C.c_void_p * 4)(*[e.cuda_event for e in evs])
    t_mm = 0.0
    for m in moes:
        m._args.prof_events = C.cast(handles, C.c_void_p)
        m.forward(x, out=out)
        m._args.prof_events = None
        torch.cuda.synchronize()
        t_mm += evs[0].elapsed_time(evs[1]) + evs[2].elapsed_time(evs[3])
    t_mm /= len(moes)
    H, I, IS = DSV2["H"], DSV2["I"], DSV2["IS"]
    flops_routed = 2.0 * T * k * 3 * I * H
    flops_shared = 2.0 * T * 3 * IS * H
    pk = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))) if os.path.exists(
        os.path.join(ROOT, "MEASURED_PEAKS.json")) else {}
    peak = pk.get("bf16_tflops_sustained", 1400.0)
    achieved = flops_routed / (t_mm / 1e3) / 1e12
    res = {"metric": PREFILL_METRIC, "value": T / (ms / 1e3), "unit": "tokens/s", "n_gpus": 1, "steps": a.steps,
           "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
           "dtype": "f16", "data": "synthetic: Student-t(df=5) std 0.02 weights, GPU Lloyd-encoded; N(0,1) tokens",
           "config": {"workload": f"DeepSeek-V2-Lite MoE stack, prefill {T} tokens", "layers": n_layers,
                      "tokens": T, "experts": DSV2["E"], "top_k": k, "hidden": H, "inter": I, "shared_inter": IS,
                      "format": format_name(fmt), "parallelism": "single GPU"},
           "roofline": {"kernel": "tc_mm_kernel (tcgen05, 128-token groups; routed gate/up+SiLU*up and down)",
                        "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                        "frac": achieved / peak,
                        "peak_source": "measured (MEASURED_PEAKS.json bf16_tflops_sustained)" if pk else "fallback",
                        "traffic": None, "ms_routed_mm_per_layer": t_mm,
                        "tflop_per_layer": (flops_routed + flops_shared) / 1e12},
           "gpu_launches": a.steps * n_layers * moes[0].launch_count(T, caller_routing=False),
           "clocks": clocks}
    print(json.dumps(res), flush=True)


# Config 5: single-matrix LUT GEMV/GEMM sweep, N x K of the MoE
# projections, M tokens, Format B b bits and table block g.
SWEEP_NK = [(1408, 2048), (2048, 1408), (768, 2048), (2048, 768), (5632, 2048)]
SWEEP_METRIC = "LUT GEMV/GEMM kernel sweep: fraction of the attainable roofline (geometric mean)"


def run_sweep(a):
    """Config 5: y = x W^T through blut_matmul (LUTLinear) for every (N x K,
    M, b, g).  Each case is timed as a CUDA graph of its four launches, L2
    flushed (a 256 MB write) before every timed call; attainable time =
    max(bytes / HBM peak, 2MNK / bf16 peak) with bytes = N K bpe + 2 M K +
    2 M N; frac = attainable / measured."""
    import torch
    from block_lut_b200.formats import LUTFormat, QuantizedMatrix
    from block_lut_b200.linear import LUTLinear
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    bw, _ = peaks()
    pk = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))) if os.path.exists(
        os.path.join(ROOT, "MEASURED_PEAKS.json")) else {}
    tf = pk.get("bf16_tflops", 1590.0)
    bits_l = [int(v) for v in a.sweep_bits.split(",")]
    groups_l = [int(v) for v in a.sweep_groups.split(",")]
    ms_l = [int(v) for v in a.sweep_m.split(",")]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    flush_sum = None
    g = torch.Generator(device=dev).manual_seed(5)
    rows, fracs, launches = [], [], 0
    reps = max(3, a.steps)
    clk = Clocks(0)
    for (n, k) in SWEEP_NK:
        for b in bits_l:
            for grp in groups_l:
                fmt = LUTFormat("b", b, grp)
                codes = torch.randint(0, 256, (n, k * b // 8), generator=g, device=dev, dtype=torch.uint8)
                tables = torch.sort((torch.randn(n, k // grp, 1 << b, generator=g, device=dev) * 0.02).half(),
                                    dim=-1).values.contiguous()
                lin = LUTLinear(QuantizedMatrix(fmt, n, k, codes, tables))
                for m in ms_l:
                    x = torch.randn(m, k, generator=g, device=dev).half()
                    out = torch.empty(m, n, dtype=torch.float16, device=dev)
                    for _ in range(2):
                        lin(x, out=out)
                    s_ = torch.cuda.Stream()
                    s_.wait_stream(torch.cuda.current_stream())
                    with torch.cuda.stream(s_):
                        lin(x, out=out)
                    torch.cuda.current_stream().wait_stream(s_)
                    graph = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(graph):
                        lin(x, out=out)
                    ts = []
                    for _ in range(reps):
                        # write the 256 MB buffer, then read it back: L2 ends up
                        # holding only clean lines of it, so no write-back of
                        # flush data lands inside the timed call
                        flush.fill_(1)
                        flush_sum = flush.sum()
                        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                        e0.record()
                        graph.replay()
                        e1.record()
                        torch.cuda.synchronize()
                        ts.append(e0.elapsed_time(e1) / 1e3)
                    launches += reps * lin.launch_count(m)
                    t = statistics.median(ts)
                    byt = n * k * fmt.bytes_per_weight() + 2 * m * k + 2 * m * n
                    fl = 2.0 * m * n * k
                    t_att = max(byt / (bw * 1e9), fl / (tf * 1e12))
                    frac = t_att / t
                    fracs.append(frac)
                    rows.append([n, k, m, b, grp, round(t * 1e6, 2), round(byt / t / 1e9, 1),
                                 round(fl / t / 1e12, 2), "hbm" if byt / (bw * 1e9) >= fl / (tf * 1e12) else "tensor",
                                 round(frac, 3)])
                    del graph
                lin.check_status()
    clocks = clk.stop()
    geo = float(np.exp(np.mean(np.log(np.maximum(fracs, 1e-9)))))
    res = {"metric": SWEEP_METRIC, "value": geo, "unit": "fraction", "n_gpus": 1, "steps": reps,
           "warmup": 2, "ms_per_step": None, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
           "dtype": "f16", "data": "synthetic random codes and sorted random fp16 tables; N(0,1) fp16 tokens",
           "config": {"workload": "config 5 single-matrix LUT GEMV/GEMM sweep (blut_matmul, tcgen05 path)",
                      "nk": SWEEP_NK, "m": ms_l, "bits": bits_l, "groups": groups_l,
                      "l2": "256 MB write + read-back before every timed call (clean L2, no dirty write-back "
                            "in the timed region)",
                      "timing": "median of the per-call CUDA-event times of a CUDA graph of the call's 3 launches"},
           "roofline": {"kernel": "blut_matmul (plan + gather + tc_mm_kernel + reduce)", "bound": "per case",
                        "peak_hbm_gbs": bw, "peak_bf16_tflops": tf,
                        "frac_min": min(fracs), "frac_max": max(fracs), "traffic": None},
           "sweep_columns": ["N", "K", "M", "bits", "group", "us", "GB/s", "TFLOP/s", "bound", "frac"],
           "sweep": rows, "cpu_baseline": None, "e2e": None, "gpu_launches": launches, "clocks": clocks}
    print(json.dumps(res), flush=True)


TIERS_METRIC = "Format R progressive-tier recover: fraction of HBM bandwidth (geometric mean over tiers 0-2)"
# DRAM read + write over algorithmic bytes of bitplane_recover_kernel<0> on this
# workload, from one ncu capture: reads match exactly; writes come out short by
# the output still dirty in L2 when the launch ends.
TIERS_TRAFFIC_RATIO = 0.965


def run_tiers(a):
    """Progressive bit-plane tiers of the HF offload engine
    (runtime/model_offload.py:751-758): blut_bitplane_recover over the routed
    experts of one Qwen1.5-MoE layer as one buffer (60 x 3 x 1408 x 2048 =
    519 M indices). Per tier, algorithmic bytes = the planes the tier reads
    (n/2, 3n/4, n) + 2 n / 128 of absmax + 2 n of bf16 output; the planes
    (>= 260 MB) and the output (1 GB) are larger than L2. e2e: the cold tier
    (2) from pinned host memory, with the H2D copy of its planes and absmax in
    the timed region; the bf16 output stays on the device for the expert
    matmul, so nothing is read back."""
    import torch
    from block_lut_b200.bitplanes import bitplane_bytes, pack_bitplanes, recover_tier
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    bw, src = peaks()
    n = E * 3 * I * H
    g = torch.Generator(device=dev).manual_seed(7)
    idx = torch.randint(0, 256, (n,), generator=g, dtype=torch.uint8, device=dev)
    planes = pack_bitplanes(idx)
    del idx
    am = (torch.rand(n // 128, generator=g, device=dev) * 0.05 + 0.01).to(torch.bfloat16)
    table = torch.randn(256, generator=g, device=dev).to(torch.bfloat16)
    out = torch.empty(n, dtype=torch.bfloat16, device=dev)
    steps = max(1, a.steps)
    clk = Clocks(0)
    rows, fracs = [], []
    for tier in (0, 1, 2):
        for _ in range(max(3, a.warmup)):
            recover_tier(planes, am, table, n, tier, out=out)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            recover_tier(planes, am, table, n, tier, out=out)
        e1.record()
        torch.cuda.synchronize()
        t = e0.elapsed_time(e1) / 1e3 / steps
        byt = bitplane_bytes(n, tier) + 2 * (n // 128) + 2 * n
        fracs.append(byt / t / 1e9 / bw)
        rows.append([tier, bitplane_bytes(n, tier), round(t * 1e6, 1), round(byt / t / 1e9, 1), round(fracs[-1], 3),
                     round(n / t / 1e9, 1)])
    # e2e, cold tier: pinned host planes + absmax -> device -> bf16
    nb2 = bitplane_bytes(n, 2)
    h_planes = planes[:nb2].cpu().pin_memory()
    h_am = am.cpu().pin_memory()
    d_planes = torch.empty(nb2, dtype=torch.uint8, device=dev)
    d_am = torch.empty_like(am)
    for _ in range(3):
        d_planes.copy_(h_planes, non_blocking=True)
        d_am.copy_(h_am, non_blocking=True)
        recover_tier(d_planes, d_am, table, n, 2, out=out)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        d_planes.copy_(h_planes, non_blocking=True)
        d_am.copy_(h_am, non_blocking=True)
        recover_tier(d_planes, d_am, table, n, 2, out=out)
    e1.record()
    torch.cuda.synchronize()
    t_e2e = e0.elapsed_time(e1) / 1e3 / steps
    clocks = clk.stop()
    cpu = None
    if not a.no_cpu:
        from oracle import blut_oracle as O
        ns = 1 << 24
        idx_s = np.random.Generator(np.random.PCG64(1)).integers(0, 256, ns, dtype=np.uint8)
        p_np = O.bitplane_pack(idx_s)
        am_np = O.f32_to_bf16(np.full(ns // 128, 0.03, dtype=np.float32))
        tab_np = O.f32_to_bf16(np.linspace(-1, 1, 256, dtype=np.float32))
        t0 = time.perf_counter()
        O.dequant_r(O.bitplane_index(p_np[: ns // 2], ns, 2), am_np, tab_np, 128, 2)
        tc = time.perf_counter() - t0
        cpu = {"value": round((ns // 2 + 2 * (ns // 128) + 2 * ns) / tc / 1e9, 3), "unit": "GB/s", "cores": 1,
               "kind": "port", "sample": f"tier 2, {ns} indices through the numpy oracle (unpack + dequant)"}
    res = {"metric": TIERS_METRIC, "value": float(np.exp(np.mean(np.log(fracs)))), "unit": "fraction", "n_gpus": 1,
           "steps": steps,
           "warmup": max(3, a.warmup), "ms_per_step": None, "higher_is_better": True, "scaling": "weak",
           "vs_baseline": None, "dtype": "u8->bf16", "data": "synthetic uniform indices, random absmax and table",
           "config": {"workload": "bit-plane tier recover, one Qwen1.5-MoE layer's routed experts",
                      "elements": n, "block_size": 128,
                      "l2": "planes (>= 260 MB) and output (1 GB) larger than L2, no flush"},
           "tiers_columns": ["tier", "plane bytes", "us", "GB/s", "frac", "G elements/s"], "tiers": rows,
           "roofline": {"bound": "hbm", "achieved": rows[0][3], "peak": bw, "unit": "GB/s", "frac": rows[0][4],
                        "traffic": round(TIERS_TRAFFIC_RATIO * (bitplane_bytes(n, 0) + 2 * (n // 128) + 2 * n)),
                        "kernel": "bitplane_recover_kernel<0>", "peak_source": src},
           "cpu_baseline": cpu,
           "e2e": {"value": round(n / t_e2e / 1e9, 2), "unit": "G elements/s (tier 2 from pinned host memory)",
                   "h2d_bytes_per_step": nb2 + 2 * (n // 128), "d2h_bytes_per_step": 0},
           "gpu_launches": 4 * steps, "clocks": clocks}
    print(json.dumps(res), flush=True)


# --------------------------------------------------------------- vllm ---
VLLM_METRIC = "vLLM decode tokens/s, full model, LUT experts"
VLLM_PREFILL_METRIC = "vLLM prefill tokens/s, full model, LUT experts"


def qwen15_moe_config(layers: int, quant: dict, dtype: str) -> dict:
    """config.json of the Qwen1.5-MoE-A2.7B architecture (config 2)."""
    return {
        "architectures": ["Qwen2MoeForCausalLM"], "model_type": "qwen2_moe",
        "hidden_size": 2048, "intermediate_size": 5632, "moe_intermediate_size": 1408,
        "shared_expert_intermediate_size": 5632, "num_experts": 60, "num_experts_per_tok": 4,
        "norm_topk_prob": False, "num_hidden_layers": layers, "num_attention_heads": 16,
        "num_key_value_heads": 16, "vocab_size": 151936, "max_position_embeddings": 8192,
        "rope_theta": 1000000.0, "rms_norm_eps": 1e-6, "hidden_act": "silu", "decoder_sparse_step": 1,
        "mlp_only_layers": [], "tie_word_embeddings": False, "torch_dtype": dtype, "use_sliding_window": False,
        "sliding_window": None, "attention_dropout": 0.0, "initializer_range": 0.02,
        "bos_token_id": 151643, "eos_token_id": 151643, "quantization_config": quant,
    }


def qwen3_moe_config(layers: int, quant: dict, dtype: str) -> dict:
    """config.json of the Qwen3-30B-A3B architecture (config 3): 128
    experts of I 768, top-8 renormalised, no shared expert, 32 query and 4
    key/value heads of 128."""
    return {
        "architectures": ["Qwen3MoeForCausalLM"], "model_type": "qwen3_moe",
        "hidden_size": 2048, "intermediate_size": 6144, "moe_intermediate_size": 768, "num_experts": 128,
        "num_experts_per_tok": 8, "norm_topk_prob": True, "num_hidden_layers": layers,
        "num_attention_heads": 32, "num_key_value_heads": 4, "head_dim": 128, "vocab_size": 151936,
        "max_position_embeddings": 40960, "rope_theta": 1000000.0, "rms_norm_eps": 1e-6, "hidden_act": "silu",
        "decoder_sparse_step": 1, "mlp_only_layers": [], "tie_word_embeddings": False, "torch_dtype": dtype,
        "use_sliding_window": False, "sliding_window": None, "attention_bias": False, "attention_dropout": 0.0,
        "initializer_range": 0.02, "bos_token_id": 151643, "eos_token_id": 151645, "quantization_config": quant,
    }


def dsv2_lite_config(layers: int, quant: dict, dtype: str) -> dict:
    """config.json of the DeepSeek-V2-Lite architecture (config 4):
    27 layers, the first a dense MLP (I 10944); 64 routed experts of I 1408,
    top-6 softmax without renormalisation, 2 shared experts; MLA attention
    with kv_lora_rank 512, no query compression, 16 heads of 128 + 64 rope
    dims.  ``layers`` counts MoE layers; the dense first layer comes on top."""
    return {
        "architectures": ["DeepseekV2ForCausalLM"], "model_type": "deepseek_v2",
        "hidden_size": 2048, "intermediate_size": 10944, "moe_intermediate_size": 1408,
        "n_routed_experts": 64, "n_shared_experts": 2, "num_experts_per_tok": 6, "first_k_dense_replace": 1,
        "moe_layer_freq": 1, "num_hidden_layers": layers + 1, "num_attention_heads": 16,
        "num_key_value_heads": 16, "kv_lora_rank": 512, "q_lora_rank": None, "qk_nope_head_dim": 128,
        "qk_rope_head_dim": 64, "v_head_dim": 128, "topk_method": "greedy", "n_group": 1, "topk_group": 1,
        "norm_topk_prob": False, "routed_scaling_factor": 1.0, "scoring_func": "softmax",
        "vocab_size": 102400, "max_position_embeddings": 163840, "rope_theta": 10000.0, "rms_norm_eps": 1e-6,
        "hidden_act": "silu", "tie_word_embeddings": False, "attention_bias": False, "attention_dropout": 0.0,
        "initializer_range": 0.02, "torch_dtype": dtype, "bos_token_id": 100000, "eos_token_id": 100001,
        "quantization_config": quant,
    }


def lut_quant_config(fmt) -> dict:
    """The checkpoint's quantization_config for the LUT plugin (block_lut_b200.quant_method.LUTConfig)."""
    q = {"quant_method": "lut", "code_type": "BLOCKLUT", "release_canonical": True}
    if fmt.kind == "b":
        q.update({"codebook_scope": "row_block", "index_bits": fmt.bits, "lut_block": fmt.group})
    elif fmt.kind == "nested":
        q.update({"codebook_scope": "row_block", "lut_block": fmt.group,
                  "nested": {"coarse_bits": 2, "residual_bits": 2, "tier": "coarse" if fmt.tier else "full"}})
    return q


def run_vllm(a):
    """Config 2 end to end: the full Qwen1.5-MoE-A2.7B architecture (24
    layers, attention and dense layers in the model dtype, experts through
    the lut plugin) in vLLM with CUDA graphs, weights from vLLM's dummy
    loader (there is no checkpoint here); with --vllm-model qwen3, config 3's
    Qwen3-30B-A3B (48 layers, NestedLUT experts, prompt 1024); with
    --vllm-model dsv2lite, config 4's DeepSeek-V2-Lite (26 MoE layers after
    a dense one, MLA attention) on 8 prompts of 4096 tokens in one prefill
    step, reported as prefill tokens/s = 8 x 4096 / time of prefill + 1
    token.  Per batch
    size: a prompt of random token ids per sequence, then 128 generated tokens; decode tokens/s
    = batch x 128 / (time of prefill + 128 tokens - time of prefill + 1
    token).  The engine runs in this process (VLLM_ENABLE_V1_MULTIPROCESSING=0)
    so that the plugin registered on import is the one it uses."""
    os.environ.setdefault("VLLM_ENABLE_V1_MULTIPROCESSING", "0")
    import random
    import torch
    import block_lut_b200.quant_method  # noqa: F401  registers "lut" with vLLM
    from vllm import LLM, SamplingParams
    fmt = bench_format(a)
    dtype = "bfloat16" if fmt.kind == "r8" else "float16"
    layers = a.layers
    qwen3, dsv2 = a.vllm_model == "qwen3", a.vllm_model == "dsv2lite"
    d = tempfile.mkdtemp(prefix="blut_vllm_")
    make_config = qwen3_moe_config if qwen3 else dsv2_lite_config if dsv2 else qwen15_moe_config
    cfg = make_config(layers, lut_quant_config(fmt), dtype)
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(cfg, f)
    prompt = 1024 if qwen3 else 4096 if dsv2 else 512
    batches = [8] if dsv2 else sorted({1, a.batch})
    extra = {"max_num_batched_tokens": prompt * max(batches)} if dsv2 else {}  # the whole batch in one prefill
    t0 = time.time()
    llm = LLM(model=d, quantization="lut", load_format="dummy", skip_tokenizer_init=True, max_model_len=prompt + 512,
              gpu_memory_utilization=0.8, max_num_seqs=max(batches), dtype=dtype, enforce_eager=False, seed=0,
              **extra)
    init_s = time.time() - t0
    rng = random.Random(0)
    res_b = {}
    for bs in batches:
        # token ids inside the model's vocabulary (102400 for DeepSeek-V2-Lite, 151936 for the Qwen models)
        hi = min(150000, cfg["vocab_size"] - 1000)
        prompts = [{"prompt_token_ids": [rng.randrange(1000, hi) for _ in range(prompt)]} for _ in range(bs)]

        def gen(n):
            sp = SamplingParams(max_tokens=n, min_tokens=n, ignore_eos=True, temperature=0.0, detokenize=False)
            torch.cuda.synchronize()
            t = time.perf_counter()
            outs = llm.generate(prompts, sp, use_tqdm=False)
            torch.cuda.synchronize()
            assert all(len(o.outputs[0].token_ids) == n for o in outs)
            return time.perf_counter() - t
        for _ in range(max(1, a.warmup)):
            gen(2)
        t1 = min(gen(1) for _ in range(3))
        t129 = min(gen(129) for _ in range(max(1, min(a.steps, 3))))
        res_b[bs] = {"decode_tokens_s": bs * 128 / (t129 - t1), "ms_per_token_step": (t129 - t1) / 128 * 1e3,
                     "prefill_s": t1, "prefill_tokens_s": bs * prompt / t1}
    top = res_b[max(batches)]
    model_name = "Qwen3-30B-A3B" if qwen3 else "DeepSeek-V2-Lite" if dsv2 else "Qwen1.5-MoE-A2.7B"
    res = {"metric": VLLM_PREFILL_METRIC if dsv2 else VLLM_METRIC,
           "value": top["prefill_tokens_s"] if dsv2 else top["decode_tokens_s"], "unit": "tokens/s", "n_gpus": 1,
           "steps": 1 if dsv2 else 128, "warmup": a.warmup,
           "ms_per_step": top["prefill_s"] * 1e3 if dsv2 else top["ms_per_token_step"], "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "f16" if dtype == "float16" else "bf16",
           "data": "vLLM dummy weights (random), random prompt token ids",
           "config": {"workload": f"{model_name} ({layers} MoE layers{' + 1 dense' if dsv2 else ''}) in vLLM, "
                                  f"prompt {prompt}, generate 128",
                      "format": format_name(fmt), "engine": "vLLM LLM(quantization='lut', load_format='dummy'), "
                      "CUDA graphs on", "init_s": round(init_s, 1)},
           "batches": {str(k): v for k, v in res_b.items()}}
    print(json.dumps(res), flush=True)


if __name__ == "__main__":
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "vllm":
        run_vllm(args)
    elif args.workload == "prefill":
        run_prefill(args)
    elif args.workload == "sweep":
        run_sweep(args)
    elif args.workload == "tiers":
        run_tiers(args)
    else:
        run_ours(args)
