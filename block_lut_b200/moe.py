"""One MoE layer of LUT-quantised routed experts (+ optional shared expert).

``LUTMoELayer.forward`` is a single call into ``blut_moe_forward`` (router or
caller routing -> plan -> B-fragment gather -> gate/up + SiLU*up -> down ->
weighted combine), all stream-ordered on the caller's stream with a
caller-owned workspace, so it can be captured in a CUDA graph.
"""
from __future__ import annotations

import ctypes as C
import math
import threading
from dataclasses import dataclass
from typing import Optional, Sequence

import torch

from . import _lib
from .formats import LUTFormat, QuantizedMatrix, dense_matrix, pack_tiled


@dataclass
class LUTExperts:
    """E routed experts of one layer, tiled: w13 [E][2I, H] and w2 [E][H, I]."""
    fmt: LUTFormat
    num_experts: int
    hidden: int
    inter: int
    w13: torch.Tensor
    w13_stride: int
    w2: torch.Tensor
    w2_stride: int
    lut_table: Optional[torch.Tensor] = None  # r8: bf16 [256] tier table
    tc: bool = False  # tiled for the tcgen05 matmuls (BLUT_LAYOUT_TC)

    @classmethod
    def from_quantized(cls, w13: Sequence[QuantizedMatrix], w2: Sequence[QuantizedMatrix],
                       lut_table: Optional[torch.Tensor] = None, stream=None,
                       tc: Optional[bool] = None) -> "LUTExperts":
        """Tile the experts.  ``tc`` None picks the tcgen05 layout whenever the
        format and shapes have one, else the mma.sync layout."""
        w13, w2 = list(w13), list(w2)
        fmt = w13[0].fmt
        if tc is None:
            tc = fmt.has_tc_layout(w13[0].rows, w13[0].cols, paired=True) and \
                fmt.has_tc_layout(w2[0].rows, w2[0].cols)
        b13, s13 = pack_tiled(w13, stream, paired=True, tc=tc)
        b2, s2 = pack_tiled(w2, stream, tc=tc)
        if fmt.kind == "r8":
            if lut_table is None:
                lut_table = w13[0].tables
            lut_table = lut_table.to(device=b13.device, dtype=torch.bfloat16).contiguous()
        return cls(fmt, len(w13), w13[0].cols, w13[0].rows // 2, b13, s13, b2, s2, lut_table, bool(tc))

    def weight_bytes(self, experts: int = 1) -> float:
        """Bytes streamed for ``experts`` experts (gate/up/down), per the format."""
        return experts * 3 * self.inter * self.hidden * self.fmt.bytes_per_weight()


@dataclass
class SharedExpert:
    """Dense shared expert: s13 [2 I_s, H], s2 [H, I_s] tiled, optional gate vector [H]."""
    inter: int
    s13: torch.Tensor
    s2: torch.Tensor
    desc13: _lib.MatDesc
    desc2: _lib.MatDesc
    gate: Optional[torch.Tensor] = None

    @classmethod
    def from_dense(cls, w13: torch.Tensor, w2: torch.Tensor, gate: Optional[torch.Tensor] = None,
                   stream=None, tc: Optional[bool] = None) -> "SharedExpert":
        """Tile the shared expert; ``tc`` as in ``LUTExperts.from_quantized``."""
        m13, m2 = dense_matrix(w13), dense_matrix(w2)
        if tc is None:
            tc = m13.fmt.has_tc_layout(*w13.shape, paired=True) and m2.fmt.has_tc_layout(*w2.shape)
        b13, _ = pack_tiled([m13], stream, paired=True, tc=tc)
        b2, _ = pack_tiled([m2], stream, tc=tc)
        g = None if gate is None else gate.reshape(-1).to(w13.dtype).contiguous()
        return cls(w13.shape[0] // 2, b13, b2, m13.fmt.desc(*w13.shape, paired=True, tc=tc),
                   m2.fmt.desc(*w2.shape, tc=tc), g)

    def weight_bytes(self) -> float:
        """Bytes of the dense shared expert (gate, up and down, 2 bytes per weight)."""
        return 2.0 * (self.desc13.rows * self.desc13.cols + self.desc2.rows * self.desc2.cols)


_WS: dict = {}
_WS_LOCK = threading.Lock()


def workspace(device: torch.device, nbytes: int, slot: int = 0, stream=None) -> torch.Tensor:
    """Grow-only workspace per (device, slot).  Layers whose calls run in one
    stream's order share a slot; a layer that runs concurrently with others
    on another stream takes a slot of its own (``LUTMoELayer.ws_slot``): the
    lock only keeps the table consistent across host threads, it does not
    order their kernels.  ``stream``: the stream the caller launches on, when
    it is not torch's current one; a buffer outgrown there is marked as used
    by that stream, so the caching allocator does not hand its memory out
    while the stream's kernels may still read it."""
    key = (device.type, device.index, slot)
    with _WS_LOCK:
        buf = _WS.get(key)
        if buf is None or buf.numel() < nbytes:
            if buf is not None and stream is not None:
                buf.record_stream(stream)
            buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            _WS[key] = buf
    return buf


class LUTMoELayer:
    """Routed LUT experts of one layer, optionally with a router and a shared expert.

    ``router_w``: [E (+1)] x H gate weights; when the shared expert is gated by
    ``sigmoid(x . g)`` and no separate gate vector is given, row E of
    ``router_w`` is that gate (the Qwen2-MoE ``shared_expert_gate``).
    """

    def __init__(self, experts: LUTExperts, top_k: int, router_w: Optional[torch.Tensor] = None,
                 renorm: bool = False, shared: Optional[SharedExpert] = None, shared_gate_mode: int = 1):
        self.experts = experts
        self.top_k = int(top_k)
        self.router_w = None if router_w is None else router_w.to(experts.fmt.compute_dtype).contiguous()
        self.renorm = bool(renorm)
        self.shared = shared
        self.ws_slot = 0  # workspace slot (see workspace); 1 for a layer run beside others on a side stream
        # expected share of the T*k slots that name an expert of this layer:
        # below 1 when most slots are empty (-1), as for the rows expert
        # parallelism hands to one rank; it steers only the work split
        self.slot_fraction = 1.0
        self.shared_gate_mode = int(shared_gate_mode)
        self.dtype = experts.fmt.compute_dtype
        self._args = self._make_args()
        self._ws_need = {}  # workspace bytes per (token count, expected slots): nothing else of the args changes

    def _make_args(self) -> _lib.MoEArgs:
        ex = self.experts
        a = _lib.MoEArgs()
        a.hidden, a.inter, a.num_experts, a.top_k = ex.hidden, ex.inter, ex.num_experts, self.top_k
        a.dtype = _lib.BF16 if self.dtype == torch.bfloat16 else _lib.F16
        a.w13 = ex.fmt.desc(2 * ex.inter, ex.hidden, paired=True, tc=ex.tc)
        a.w2 = ex.fmt.desc(ex.hidden, ex.inter, tc=ex.tc)
        a.w13_tiled, a.w2_tiled = ex.w13.data_ptr(), ex.w2.data_ptr()
        a.w13_stride, a.w2_stride = ex.w13_stride, ex.w2_stride
        a.lut_table = None if ex.lut_table is None else ex.lut_table.data_ptr()
        a.router_w = None if self.router_w is None else self.router_w.data_ptr()
        a.renorm = int(self.renorm)
        if self.shared is not None:
            sh = self.shared
            a.shared_inter = sh.inter
            a.shared_gate_mode = self.shared_gate_mode
            a.s13, a.s2 = sh.desc13, sh.desc2
            a.s13_tiled, a.s2_tiled = sh.s13.data_ptr(), sh.s2.data_ptr()
            a.shared_gate_w = None if sh.gate is None else sh.gate.data_ptr()
        return a

    def launch_count(self, num_tokens: int, caller_routing: bool) -> int:
        """Kernel launches one forward issues (the count only tests pointers for NULL)."""
        a = _lib.MoEArgs.from_buffer_copy(self._args)
        a.num_tokens = num_tokens
        a.expected_slots = self._expected_slots(num_tokens)
        a.topk_ids = 1 if caller_routing else None
        return int(_lib.lib().blut_moe_launch_count(C.byref(a)))

    def _expected_slots(self, num_tokens: int) -> int:
        """blut_moe_args.expected_slots for a call on ``num_tokens`` rows (0: all slots may be used)."""
        if self.slot_fraction >= 1.0:
            return 0
        return max(1, math.ceil(num_tokens * self.top_k * self.slot_fraction))

    def forward(self, x: torch.Tensor, topk_ids: Optional[torch.Tensor] = None,
                topk_weights: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                stream=None, out_f32: bool = False) -> torch.Tensor:
        """out[t] = sum_j w[t,j] * expert_{ids[t,j]}(x_t) (+ shared(x_t)); x [T, H].

        ``out_f32`` returns the unrounded float32 sums (expert-parallel partials).
        ``stream``: launch there instead of on torch's current stream; the
        input conversions, the output allocation and the copies after the
        launch then run on it too, in order with the kernels.
        """
        if stream is not None:
            with torch.cuda.stream(stream):
                return self._forward(x, topk_ids, topk_weights, out, stream, out_f32)
        return self._forward(x, topk_ids, topk_weights, out, None, out_f32)

    def _forward(self, x, topk_ids, topk_weights, out, stream, out_f32):
        if not x.is_cuda:
            raise ValueError("LUTMoELayer.forward expects CUDA tensors (no CPU path)")
        if x.numel() == 0:  # an empty batch (as torch's ops return for the reference): nothing to launch
            dt = torch.float32 if out_f32 else x.dtype
            res = out if out is not None else torch.empty(x.shape, dtype=dt, device=x.device)
            return res
        if out_f32:
            return self._forward_f32(x, topk_ids, topk_weights, out, stream)
        in_dtype = x.dtype
        x2, a, keep = self._prepare(x, topk_ids, topk_weights)
        T = x2.shape[0]
        if out is None or out.dtype != self.dtype:
            res = torch.empty(T, x2.shape[1], dtype=self.dtype, device=x2.device)
        else:
            res = out.reshape(T, -1)
        a.out = res.data_ptr()
        self._launch(a, x2, stream)
        if out is not None and res.data_ptr() != out.data_ptr():
            out.copy_(res.reshape(out.shape))
            return out
        res = res.reshape(x.shape)
        return res if in_dtype == self.dtype else res.to(in_dtype)

    __call__ = forward

    def _launch(self, a: _lib.MoEArgs, x2: torch.Tensor, stream) -> None:
        """blut_moe_forward with this call's arguments ``a`` on the layer's workspace."""
        lib = _lib.lib()
        key = (int(a.num_tokens), int(a.expected_slots))  # the split, hence the size, depends on both
        need = self._ws_need.get(key)
        if need is None:
            need = lib.blut_moe_workspace_size(C.byref(a))
            if need == 0:
                raise RuntimeError("blut_moe_forward rejected the layer arguments (see blut_moe_workspace_size)")
            self._ws_need[key] = need
        ws = workspace(x2.device, need, self.ws_slot, stream)
        with _lib.on_device(x2):
            _lib.check(lib.blut_moe_forward(C.byref(a), ws.data_ptr(), ws.numel(), _lib.stream_ptr(stream)),
                       "moe_forward")

    def _prepare(self, x, topk_ids, topk_weights):
        """Input rows, a per-call copy of the layer's argument block (so calls
        from several host threads never share one), and the tensors it points
        to (kept alive until the launch)."""
        x2 = x.reshape(-1, x.shape[-1])
        if x2.dtype != self.dtype:
            x2 = x2.to(self.dtype)
        x2 = x2.contiguous()
        T = x2.shape[0]
        a = _lib.MoEArgs.from_buffer_copy(self._args)
        a.num_tokens = T
        a.expected_slots = self._expected_slots(T)
        a.x = x2.data_ptr()
        keep = [x2]
        if topk_ids is not None:
            ids = topk_ids.reshape(T, -1)
            ids = (ids if ids.dtype == torch.int32 else ids.to(torch.int32)).contiguous()
            tw = topk_weights.reshape(T, -1)
            tw = (tw if tw.dtype == torch.float32 else tw.to(torch.float32)).contiguous()
            keep += [ids, tw]
            a.topk_ids, a.topk_weights = ids.data_ptr(), tw.data_ptr()
        else:
            if self.router_w is None:
                raise ValueError("no routing given and the layer has no router weights")
            a.topk_ids = a.topk_weights = None
        return x2, a, keep

    def _forward_f32(self, x, topk_ids, topk_weights, out, stream):
        x2, a, keep = self._prepare(x, topk_ids, topk_weights)
        if out is None:
            res = torch.empty(x2.shape[0], x2.shape[1], dtype=torch.float32, device=x2.device)
        else:
            res = out
        if res.dtype != torch.float32 or not res.is_contiguous():
            raise ValueError("out_f32 needs a contiguous float32 output")
        a.out = res.data_ptr()
        a.out_f32 = 1
        self._launch(a, x2, stream)
        return res

    def check_status(self, stream=None) -> None:
        """Synchronise and raise if a kernel reported a device-side error."""
        ws = _WS.get((self.experts.w13.device.type, self.experts.w13.device.index, self.ws_slot))
        if ws is not None:
            with _lib.on_device(ws):
                _lib.check(_lib.lib().blut_moe_check_status(ws.data_ptr(), _lib.stream_ptr(stream)),
                           "device status")


class LUTMoEStep:
    """A decode step over several MoE layers, replayed as one CUDA graph per
    batch size: the shape in which a serving engine runs the layers (vLLM
    captures its decode step the same way).

    ``LUTMoEStep(layers, batch)`` needs layers of one hidden size and dtype.
    It builds a pinned host input buffer ``host_in`` [layers, batch, H] (one
    [batch, H] input per layer, ``host_in[i]``) and a pinned host output
    buffer ``host_out`` of the same shape. It then captures one graph that
    copies all inputs to the device in one transfer, runs every layer on its
    own input (``layer.forward``: this library's routing and experts) and
    copies all outputs back in one transfer.  ``run()`` replays it on the
    current stream; the caller fills ``host_in`` before and reads
    ``host_out`` after a ``torch.cuda.synchronize()`` (or an event).  The
    layers run one after another on one stream, so they share their
    workspace as in eager calls; a later call that grows that workspace (a
    larger batch on the same layers) invalidates the graph, so capture a
    step per batch size after the largest eager call.
    """

    def __init__(self, layers: Sequence[LUTMoELayer], batch: int, device=None):
        if not layers:
            raise ValueError("LUTMoEStep needs at least one layer")
        self.layers = list(layers)
        H = {m.experts.hidden for m in self.layers}
        dt = {m.dtype for m in self.layers}
        if len(H) != 1 or len(dt) != 1:
            raise ValueError("LUTMoEStep stacks layers of one hidden size and dtype")
        H, dt = H.pop(), dt.pop()
        self.batch = int(batch)
        dev = torch.device(device) if device is not None else self.layers[0].experts.w13.device
        self.device = dev
        n = len(self.layers)
        self.host_in = torch.zeros(n, self.batch, H, dtype=dt).pin_memory()
        self.host_out = torch.zeros(n, self.batch, H, dtype=dt).pin_memory()
        self._dev_in = torch.zeros(n, self.batch, H, dtype=dt, device=dev)
        self._dev_out = torch.empty_like(self._dev_in)
        with torch.cuda.device(dev):
            side = torch.cuda.Stream(device=dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):  # first calls: workspaces and the library's side stream
                for _ in range(2):
                    self._body()
            torch.cuda.current_stream(dev).wait_stream(side)
            torch.cuda.synchronize(dev)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self._body()
        torch.cuda.synchronize(dev)

    def _body(self) -> None:
        self._dev_in.copy_(self.host_in, non_blocking=True)
        for i, m in enumerate(self.layers):
            m.forward(self._dev_in[i], out=self._dev_out[i])
        self.host_out.copy_(self._dev_out, non_blocking=True)

    def run(self) -> None:
        """Replays the step on the current stream (asynchronous)."""
        self.graph.replay()

    def check_status(self) -> None:
        for m in self.layers:
            m.check_status()


@_lib.stream_ordered
def router(x: torch.Tensor, w_router: torch.Tensor, top_k: int, renorm: bool = False,
           shared_gate: bool = False, stream=None):
    """Fused router on the GPU: (topk_ids int32 [T,k], topk_weights f32 [T,k], gate f32 [T] | None)."""
    x = x.contiguous()
    w = w_router.to(x.dtype).contiguous()
    T, H = x.shape
    E = w.shape[0] - (1 if shared_gate else 0)
    ids = torch.empty(T, top_k, dtype=torch.int32, device=x.device)
    tw = torch.empty(T, top_k, dtype=torch.float32, device=x.device)
    sg = torch.empty(T, dtype=torch.float32, device=x.device) if shared_gate else None
    logits = torch.empty(T, w.shape[0], dtype=torch.float32, device=x.device)
    dt = _lib.BF16 if x.dtype == torch.bfloat16 else _lib.F16
    with _lib.on_device(x):
        _lib.check(_lib.lib().blut_router(x.data_ptr(), w.data_ptr(), T, H, E, top_k, int(renorm), int(shared_gate),
                                          dt, ids.data_ptr(), tw.data_ptr(), None if sg is None else sg.data_ptr(),
                                          logits.data_ptr(), _lib.stream_ptr(stream)), "router")
    return ids, tw, sg
