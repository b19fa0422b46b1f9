"""Binding of the sm_100a C-ABI library (``librqb200.so``, include/rq_b200.h).

Every compute entry point of the package goes through here.  There is no
other implementation: if the library is missing, or no sm_100 (B200) CUDA
device is present, these functions raise ``NativeUnavailable`` -- the
package never silently computes on the CPU.

Tensors stay where the caller keeps them.  Inputs on the CPU are staged to
the current CUDA device for the kernel and the results copied back, which is
what the reference's device-agnostic quantize/dequantize calls promise
(``tests/test_quant_ops.py::test_device_agnostic`` in the reference).
"""
from __future__ import annotations

import ctypes
import os
import threading
from typing import Dict, Optional, Tuple

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
_DEFAULT_LIB = os.path.join(_HERE, "librqb200.so")
LIB_PATH = os.environ.get("RQ_B200_LIB", _DEFAULT_LIB)
# the thin torch extension over the same library (csrc/torch_ops.cpp)
OPS_PATH = os.path.join(_HERE, "librq_torch_ops.so")

RQ_OK = 0
RQ_ERR_UNSUPPORTED = -8
F32, BF16, F16 = 0, 1, 2
W_NF4, W_NF4_DQ_FP8, W_NF4_DQ_INT8, W_INT8, W_INT8_ROW = 0, 1, 2, 3, 4

_DT_CODE = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16}


class RqGather(ctypes.Structure):
    """struct RqGather of include/rq_b200.h (device pointers)."""
    _fields_ = [("outs", ctypes.c_void_p), ("flags", ctypes.c_void_p), ("my_flags", ctypes.c_void_p),
                ("ctrl", ctypes.c_void_p), ("ld", ctypes.c_int64), ("col", ctypes.c_int64),
                ("world", ctypes.c_int), ("rank", ctypes.c_int)]


class NativeUnavailable(RuntimeError):
    """The sm_100a kernels cannot run here (library or B200 GPU missing)."""


class NativeError(RuntimeError):
    """A kernel entry point returned an error status."""


_lib = None
_lib_lock = threading.Lock()


def _bind(L: ctypes.CDLL) -> None:
    P, I, I64, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
    sig = {
        "rq_abi_version": ([], I),
        "rq_status_string": ([I], ctypes.c_char_p),
        "rq_last_cuda_error": ([], I),
        "rq_last_status": ([], I),
        "rq_last_path": ([], I),
        "rq_set_decode_exact": ([I], None),
        "rq_merge_lora": ([I, P, P, I, P, P, I64, I64, I, P, P, I, F, I, P, I, P], I),
        "rq_weight_absmax": ([I, P, P, I, P, P, I64, I64, I, I, P, P], I),
        "rq_weight_to_fp8": ([I, P, P, I, P, P, I64, I64, I, I, F, P, P], I),
        "rq_take_kernel_timeouts": ([P], I),
        "rq_nf4_quantize": ([P, I, I64, I, P, P, P], I),
        "rq_nf4_dequantize": ([P, I64, P, I, I, P, I, P], I),
        "rq_int8_quantize": ([P, I, I64, I, P, P, P], I),
        "rq_int8_quantize_rows": ([P, I, I64, I64, P, P, P], I),
        "rq_int8_dequantize": ([P, I64, P, I, I, I64, P, I, P], I),
        "rq_dq_quantize_scales": ([P, I64, I, I, P, P, P], I),
        "rq_dq_dequantize": ([P, I64, P, P, I, I, I, P, I, P], I),
        "rq_linear_workspace_bytes": ([I64, I64, I64, I], I64),
        "rq_linear_forward": ([I, P, P, I, P, P, I64, I64, I, P, I, I64, P, P, I, P, P, I, F, P, P, I64, P], I),
        "rq_linear_dx": ([I, P, P, I, P, P, I64, I64, I, P, I, I64, P, P, I, F, P, P, I64, P], I),
        "rq_linear_forward_noalloc": ([I, P, P, I, P, P, I64, I64, I, P, I, I64, P, P, I, P, P, I, F, P, P], I),
        "rq_linear_forward_gather": ([I, P, P, I, P, P, I64, I64, I, P, I, I64, P, I, P, P, I, F,
                                      ctypes.POINTER(RqGather), P, I64, P], I),
        "rq_peer_alloc": ([I64, ctypes.POINTER(ctypes.c_void_p)], I),
        "rq_peer_free": ([P], I),
        "rq_peer_handle": ([P, P], I),
        "rq_peer_open": ([P, ctypes.POINTER(ctypes.c_void_p)], I),
        "rq_peer_close": ([P], I),
        "launch_int4_dequant_matmul": ([P, P, P, P, P, I, I, I, I], None),
        "launch_int8_dequant_matmul": ([P, P, P, P, P, I, I, I, I], None),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res


def exported_symbols() -> Tuple[str, ...]:
    """Names of the C entry points this binding declares."""
    return ("rq_abi_version", "rq_status_string", "rq_last_cuda_error", "rq_last_status", "rq_last_path",
            "rq_set_decode_exact", "rq_merge_lora", "rq_weight_absmax", "rq_weight_to_fp8",
            "rq_take_kernel_timeouts",
            "rq_nf4_quantize", "rq_nf4_dequantize", "rq_int8_quantize", "rq_int8_quantize_rows",
            "rq_int8_dequantize", "rq_dq_quantize_scales", "rq_dq_dequantize",
            "rq_linear_workspace_bytes", "rq_linear_forward", "rq_linear_dx", "rq_linear_forward_noalloc",
            "rq_linear_forward_gather", "rq_peer_alloc", "rq_peer_free", "rq_peer_handle", "rq_peer_open",
            "rq_peer_close",
            "launch_int4_dequant_matmul", "launch_int8_dequant_matmul")


def load_library() -> ctypes.CDLL:
    """Load librqb200.so (no device needed).  Raises NativeUnavailable."""
    global _lib
    if _lib is not None:
        return _lib
    with _lib_lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise NativeUnavailable(
                    f"rocm_qlora B200 library not built: {LIB_PATH} is missing "
                    "(run `make -C rocm-qlora_b200` or __graft_entry__.build())")
            L = ctypes.CDLL(LIB_PATH)
            _bind(L)
            _lib = L
    return _lib


_ops_state: Optional[bool] = None


def ops() -> bool:
    """Whether torch.ops.rocm_qlora.{linear_forward, linear_dx} are loaded:
    the layer then calls the library through one dispatcher call instead of
    ctypes.  Only with the in-tree library (the extension links it), so a
    library chosen through RQ_B200_LIB is always called directly."""
    global _ops_state
    if _ops_state is None:
        with _lib_lock:
            if _ops_state is None:
                ok = False
                if os.path.abspath(LIB_PATH) == _DEFAULT_LIB and os.path.exists(OPS_PATH):
                    try:
                        torch.ops.load_library(OPS_PATH)
                        ok = hasattr(torch.ops.rocm_qlora, "linear_forward")
                    except (OSError, RuntimeError):
                        ok = False
                _ops_state = ok
    return _ops_state


def device_supported(device: Optional[torch.device] = None) -> bool:
    if not torch.cuda.is_available():
        return False
    idx = torch.cuda.current_device() if device is None or device.index is None else device.index
    return torch.cuda.get_device_capability(idx) == (10, 0)


def is_available() -> bool:
    """True when the library loads and the current CUDA device is sm_100."""
    try:
        load_library()
    except (NativeUnavailable, OSError):
        return False
    return device_supported()


def _lib_for_compute() -> ctypes.CDLL:
    L = load_library()
    if not torch.cuda.is_available():
        raise NativeUnavailable("rocm_qlora (B200 build) needs a CUDA device; none is visible")
    if not device_supported():
        cap = torch.cuda.get_device_capability()
        raise NativeUnavailable(f"rocm_qlora (B200 build) needs an sm_100 GPU; current device is sm_{cap[0]}{cap[1]}")
    return L


def check(rc: int, what: str) -> None:
    if rc != RQ_OK:
        L = load_library()
        msg = L.rq_status_string(rc).decode()
        extra = f" (cudaError {L.rq_last_cuda_error()})" if rc == -4 else ""
        raise NativeError(f"{what} failed: {msg}{extra}")


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DT_CODE[dt]
    except KeyError:
        raise TypeError(f"unsupported dtype {dt}; rocm_qlora kernels take float32, bfloat16 or float16") from None


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def to_cuda(t: torch.Tensor) -> torch.Tensor:
    """Contiguous CUDA view of t (copied to the current device if on CPU)."""
    if not t.is_cuda:
        t = t.to(torch.device("cuda", torch.cuda.current_device()))
    return t.contiguous()


def compute_device(*ts: Optional[torch.Tensor]) -> torch.device:
    for t in ts:
        if t is not None and t.is_cuda:
            return t.device
    return torch.device("cuda", torch.cuda.current_device())


# ----------------------------------------------------------- workspaces
# One zero-initialised buffer per (device, stream); calls that may overlap on
# the GPU must not share one, and the counter area must start at zero.
_ws: Dict[Tuple[int, int], torch.Tensor] = {}
_ws_lock = threading.Lock()


def workspace(device: torch.device, nbytes: int, stream: Optional[int] = None) -> torch.Tensor:
    """The library workspace of (device, stream), at least nbytes; `stream`
    is the stream's handle when the caller has it already."""
    key = (device.index, stream_ptr(device) if stream is None else stream)
    with _ws_lock:
        buf = _ws.get(key)
        if buf is None or buf.numel() < nbytes:
            size = max(nbytes, 1 << 20)
            if buf is not None:
                size = max(size, 2 * buf.numel())
            buf = torch.zeros(size, dtype=torch.uint8, device=device)
            _ws[key] = buf
    return buf


def lib() -> ctypes.CDLL:
    return _lib_for_compute()


def set_decode_exact(exact: bool) -> None:
    """Decode GEMV numerics for later calls: False (default) rounds each NF4
    level once to the activation dtype and applies the block scale to fp32
    partial sums; True forms the reference's own weights (level x scale,
    rounded per weight), so only the summation order separates the results
    (slower).  Same as RQ_DECODE_EXACT=1 in the environment."""
    load_library().rq_set_decode_exact(1 if exact else 0)
