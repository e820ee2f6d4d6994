"""ctypes binding of ``libblut.so`` (the C ABI declared in ``include/blut.h``).

There is no CPU fallback: if the library is missing or a GPU is absent the
calls fail loudly.  Build the library with ``python -m block_lut_b200._build``.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libblut.so")

# status codes (blut.h)
BLUT_OK = 0
BLUT_ERR_INVALID = -1
BLUT_ERR_UNSUPPORTED = -2
BLUT_ERR_WORKSPACE = -3
BLUT_ERR_LAUNCH = -4
BLUT_ERR_TIMEOUT = -5
BLUT_ERR_CUDA = -6

# formats / dtypes
FMT_R8, FMT_B, FMT_NESTED, FMT_DENSE = 1, 2, 3, 4
LAYOUT_PAIRED, LAYOUT_TC = 1, 2
F16, BF16, F32 = 0, 1, 2


class MatDesc(C.Structure):
    _fields_ = [("format", C.c_int32), ("bits", C.c_int32), ("group", C.c_int32), ("tier", C.c_int32),
                ("dtype", C.c_int32), ("layout", C.c_int32), ("rows", C.c_int64), ("cols", C.c_int64)]


class Canon(C.Structure):
    _fields_ = [("codes", C.c_void_p), ("codes2", C.c_void_p), ("tables", C.c_void_p),
                ("tables2", C.c_void_p), ("scales", C.c_void_p)]


class MoEArgs(C.Structure):
    _fields_ = [("num_tokens", C.c_int32), ("hidden", C.c_int32), ("inter", C.c_int32),
                ("num_experts", C.c_int32), ("top_k", C.c_int32), ("dtype", C.c_int32),
                ("w13", MatDesc), ("w2", MatDesc),
                ("w13_tiled", C.c_void_p), ("w2_tiled", C.c_void_p),
                ("w13_stride", C.c_int64), ("w2_stride", C.c_int64),
                ("lut_table", C.c_void_p), ("x", C.c_void_p),
                ("topk_ids", C.c_void_p), ("topk_weights", C.c_void_p), ("router_w", C.c_void_p),
                ("renorm", C.c_int32), ("shared_inter", C.c_int32), ("shared_gate_mode", C.c_int32),
                ("reserved", C.c_int32),
                ("s13", MatDesc), ("s2", MatDesc),
                ("s13_tiled", C.c_void_p), ("s2_tiled", C.c_void_p),
                ("shared_gate_w", C.c_void_p), ("out", C.c_void_p), ("prof_events", C.c_void_p),
                ("out_f32", C.c_int32), ("expected_slots", C.c_int32)]


EP_MAX_RANKS = 8
EP_HANDLE_BYTES = 64


class EpDesc(C.Structure):
    _fields_ = [("world", C.c_int32), ("rank", C.c_int32), ("capacity", C.c_int32), ("hidden", C.c_int32),
                ("top_k", C.c_int32), ("dtype", C.c_int32), ("windows", C.c_void_p * EP_MAX_RANKS)]


# (name, restype, argtypes) of every exported entry point, in blut.h order.
_VP, _I32, _I64 = C.c_void_p, C.c_int32, C.c_int64
SIGNATURES = [
    ("blut_status_string", C.c_char_p, [C.c_int]),
    ("blut_dequant", C.c_int, [C.POINTER(MatDesc), C.POINTER(Canon), _VP, _VP]),
    ("blut_blocklut_decompress", C.c_int, [_VP, _VP, _VP, _VP, _I64, _I32, _VP]),
    ("blut_batch_blocklut_decompress", C.c_int, [_VP, _VP, _VP, _VP, _I64, _I64, _I64, _I32, _VP]),
    ("blut_lut_recover", C.c_int, [_VP, _VP, _VP, _I64, _VP]),
    ("blut_bitplane_bytes", C.c_int64, [_I64, _I32]),
    ("blut_bitplane_pack", C.c_int, [_VP, _VP, _I64, _VP]),
    ("blut_bitplane_recover", C.c_int, [_VP, _VP, _VP, _VP, _I64, _I32, _I32, _VP]),
    ("blut_tiled_bytes", C.c_int64, [C.POINTER(MatDesc)]),
    ("blut_pack_tiled", C.c_int, [C.POINTER(MatDesc), C.POINTER(Canon), _VP, _VP]),
    ("blut_dequant_tiled", C.c_int, [C.POINTER(MatDesc), _VP, _VP, _VP, _VP]),
    ("blut_matmul_workspace_size", C.c_size_t, [C.POINTER(MatDesc), _I64]),
    ("blut_matmul", C.c_int, [C.POINTER(MatDesc), _VP, _VP, _VP, _I64, _VP, _I32, _VP, C.c_size_t, _VP]),
    ("blut_matmul_launch_count", C.c_int, [C.POINTER(MatDesc), _I64]),
    ("blut_encode", C.c_int, [C.POINTER(MatDesc), _VP, _VP, _VP, _VP, _VP, _VP]),
    ("blut_encode_r", C.c_int, [_VP, _I64, _VP, _I32, _VP, _VP, _VP]),
    ("blut_encode_lut_f32", C.c_int, [_VP, _I64, _VP, _I32, _VP, _VP, _VP]),
    ("blut_lut_gemv", C.c_int, [_VP, _VP, _VP, _VP, _VP, _I64, _I64, _I64, _VP]),
    ("blut_router", C.c_int, [_VP, _VP, _I32, _I32, _I32, _I32, _I32, _I32, _I32, _VP, _VP, _VP, _VP, _VP]),
    ("blut_moe_workspace_size", C.c_size_t, [C.POINTER(MoEArgs)]),
    ("blut_moe_forward", C.c_int, [C.POINTER(MoEArgs), _VP, C.c_size_t, _VP]),
    ("blut_moe_forward_noalloc", C.c_int, [C.POINTER(MoEArgs), _VP]),
    ("blut_moe_check_status", C.c_int, [_VP, _VP]),
    ("blut_moe_launch_count", C.c_int, [C.POINTER(MoEArgs)]),
    ("blut_debug_set_wait_limit", C.c_int, [C.c_uint64]),
    ("blut_ep_window_bytes", C.c_size_t, [_I32, _I32, _I32, _I32]),
    ("blut_ep_alloc", C.c_int, [C.c_size_t, C.POINTER(C.c_void_p)]),
    ("blut_ep_free", C.c_int, [_VP]),
    ("blut_ep_ipc_handle", C.c_int, [_VP, _VP]),
    ("blut_ep_ipc_open", C.c_int, [_VP, C.POINTER(C.c_void_p)]),
    ("blut_ep_ipc_close", C.c_int, [_VP]),
    ("blut_ep_views", C.c_int, [C.POINTER(EpDesc), C.POINTER(C.c_void_p), C.POINTER(C.c_void_p),
                                C.POINTER(C.c_void_p), C.POINTER(C.c_void_p)]),
    ("blut_ep_dispatch", C.c_int, [C.POINTER(EpDesc), _VP, _VP, _VP, _I32, _VP, _VP, _I32, _VP]),
    ("blut_ep_combine", C.c_int, [C.POINTER(EpDesc), _I32, _VP, _VP, _I32, _VP]),
    ("blut_ep_check_status", C.c_int, [C.POINTER(EpDesc), _VP]),
]

_lib = None
_lock = threading.Lock()


def lib() -> C.CDLL:
    """Load ``libblut.so`` once (raises if it was not built)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m block_lut_b200._build`")
                L = C.CDLL(LIB_PATH)
                for name, res, args in SIGNATURES:
                    fn = getattr(L, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = L
    return _lib


def status_string(rc: int) -> str:
    return lib().blut_status_string(int(rc)).decode()


def check(rc: int, what: str = "") -> None:
    if rc != BLUT_OK:
        raise RuntimeError(f"libblut {what}: {status_string(rc)} (status {rc})")


def stream_ptr(stream=None) -> int:
    """cudaStream_t of ``stream`` (default: torch's current stream)."""
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


def stream_ordered(fn):
    """Decorator for wrappers with a ``stream`` argument: the body runs with
    that stream (when given) as torch's current stream, so the tensors the
    wrapper converts or allocates belong to the stream its kernels run on.
    Otherwise a converted input freed on return could be handed out again by
    the caching allocator while the kernel on ``stream`` still reads it."""
    import contextlib
    import functools
    import inspect
    import torch
    sig = inspect.signature(fn)

    @functools.wraps(fn)
    def wrapper(*args, **kwargs):
        s = sig.bind_partial(*args, **kwargs).arguments.get("stream")
        with torch.cuda.stream(s) if s is not None else contextlib.nullcontext():
            return fn(*args, **kwargs)
    return wrapper


def on_device(t):
    """Context making the device of CUDA tensor ``t`` current.  The library
    launches on the current device, so every call runs under the device of
    its tensors (a kernel launched on another device than its buffers' would
    access peer memory)."""
    import contextlib
    import torch
    if isinstance(t, torch.Tensor) and t.is_cuda:
        return torch.cuda.device(t.device)
    return contextlib.nullcontext()
