"""ctypes boundary to libtileops_b200.so (the C ABI declared in include/tileops_b200.h).

This replaces the reference's plugin layer (tileops/runtime/_infra.py:161 BACKEND_PACKAGES,
:492 dispatch_compile_quant and the invoke_* wrappers in tileops/runtime/__init__.py:446-641):
instead of JIT-compiling TileLang kernels per target, every op calls one precompiled sm_100a
entry point with raw device pointers, sizes and the current torch stream. There is no other
backend and no CPU path: a missing library or a non-CUDA tensor is an error.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).with_name("libtileops_b200.so")

TO_OK = 0
TO_EINVAL = -1
TO_EUNSUPPORTED = -2
TO_ECUDA = -3
TO_ETIMEOUT = -4
TO_ENOSPACE = -5

DTYPE_CODES = {
    torch.float32: 0,
    torch.float16: 1,
    torch.bfloat16: 2,
    torch.int8: 3,
    torch.float8_e4m3fn: 4,
    torch.int32: 5,
    torch.int64: 6,
}

_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_int64
_F = ctypes.c_float
_S = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/tileops_b200.h one for one.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "to_version": (ctypes.c_char_p, []),
    "to_last_error_string": (ctypes.c_char_p, []),
    "to_device_check": (_I, [_I]),
    "to_device_error_word": (_I, [ctypes.POINTER(_I), _I]),
    "to_wait_limit_selftest": (_I, [_I, _I, _P, _P]),
    "to_set_launch_overlap": (_I, [_I]),
    "to_quant_per_tensor_i8": (_I, [_P, _I, _P, _P, _L, _P]),
    "to_dequant_per_tensor_i8": (_I, [_P, _P, _P, _I, _L, _P]),
    "to_quant_per_channel_i8": (_I, [_P, _I, _P, _P, _L, _L, _L, _P]),
    "to_dequant_per_channel_i8": (_I, [_P, _P, _P, _I, _L, _L, _L, _P]),
    "to_input_quant_workspace_size": (_S, []),
    "to_input_to_int8": (_I, [_P, _I, _L, _P, _P, _P, _S, _P]),
    "to_input_to_fp8": (_I, [_P, _I, _L, _P, _P, _P, _S, _P]),
    "to_input_to_fp8_fnuz": (_I, [_P, _I, _L, _P, _P, _P, _S, _P]),
    "to_input_to_fp8_noalloc": (_I, [_P, _I, _L, _P, _P, _P]),
    "to_per_token_group_quant_i8": (_I, [_P, _I, _L, _L, _F, _P, _P, _P]),
    "to_per_token_group_quant_fp8": (_I, [_P, _I, _L, _L, _F, _I, _L, _L, _P, _P, _P]),
    "to_per_token_group_quant_fp8_fnuz": (_I, [_P, _I, _L, _L, _F, _I, _L, _L, _P, _P, _P]),
    "to_per_token_group_quant_fp8_tma": (_I, [_P, _I, _L, _L, _L, _F, _I, _P, _P, _L, _P]),
    "to_block_dequant_i8": (_I, [_P, _P, _P, _L, _L, _L, _L, _P]),
    "to_block_dequant_fp8": (_I, [_P, _P, _P, _L, _L, _L, _L, _P]),
    "to_block_dequant_fp8_fnuz": (_I, [_P, _P, _P, _L, _L, _L, _L, _P]),
    "to_awq_pack": (_I, [_P, _I, _P, _L, _L, _P]),
    "to_awq_unpack": (_I, [_P, _I, _P, _L, _L, _P]),
    "to_awq_dequant": (_I, [_P, _P, _I, _P, _P, _L, _L, _L, _P]),
    "to_awq_gemm_workspace_size": (_S, [_L, _L, _L, _L]),
    "to_awq_gemm": (_I, [_P, _P, _P, _I, _P, _P, _L, _L, _L, _L, _P, _S, _P]),
    "to_awq_gemm_strided": (_I, [_P, _L, _P, _P, _I, _P, _P, _L, _L, _L, _L, _P, _S, _P]),
    "to_awq_gemm_gather": (_I, [_P, _P, _P, _I, _P, ctypes.POINTER(_P), _I, _I, _L, _L, _L, _L,
                                _P, _S, _P]),
    "to_awq_gemm_act_workspace_size": (_S, [_L, _L, _L, _L]),
    "to_awq_gemm_act": (_I, [_P, _P, _P, _I, _P, _P, _L, _L, _L, _L, _I, _P, _S, _P]),
    "to_awq_gemm_act_gather": (_I, [_P, _P, _P, _I, _P, ctypes.POINTER(_P), _I, _I, _L, _L, _L,
                                    _L, _I, _P, _S, _P]),
    "to_act_and_mul_group_quant": (_I, [_P, _P, _I, _L, _L, _L, _L, _I, _L, _F, _I, _I, _I, _P,
                                        _P, _P]),
    "to_peer_flags_bytes": (_S, []),
    "to_peer_barrier": (_I, [ctypes.POINTER(_P), _I, _I, _P, _P]),
    "to_ipc_alloc": (_I, [_S, ctypes.POINTER(_P), _P]),
    "to_ipc_open": (_I, [_P, ctypes.POINTER(_P)]),
    "to_ipc_close": (_I, [_P]),
    "to_ipc_free": (_I, [_P]),
    "to_w8a8_i8_gemm": (_I, [_P, _P, _P, _P, _P, _I, _P, _P, _L, _L, _L, _L, _L, _P]),
    "to_w8a8_fp8_gemm": (_I, [_P, _P, _P, _P, _P, _I, _P, _L, _L, _L, _L, _L, _P]),
    "to_gemm": (_I, [_P, _P, _P, _I, _L, _L, _L, _P]),
    "to_gemv": (_I, [_P, _P, _P, _I, _L, _L, _P]),
    "to_silu_and_mul": (_I, [_P, _P, _P, _I, _L, _L, _L, _L, _L, _P]),
    "to_gelu_and_mul": (_I, [_P, _P, _P, _I, _L, _L, _L, _L, _L, _P]),
}

_lib: ctypes.CDLL | None = None
_lock = threading.Lock()
_checked_devices: set[int] = set()


def load() -> ctypes.CDLL:
    """Loads the library once per process and declares every entry point's signature."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH.name} is not built; run `python -m tileops_b200.build` "
                    "(tileops_b200 has no CPU or fallback path)"
                )
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def last_error() -> str:
    msg = load().to_last_error_string()
    return msg.decode() if msg else ""


def check(rc: int, op: str) -> None:
    """Maps a TO_E* status to the exception type the reference raises for that failure."""
    if rc == TO_OK:
        return
    msg = last_error() or f"{op} failed with status {rc}"
    if rc == TO_EINVAL:
        raise ValueError(msg)
    if rc == TO_EUNSUPPORTED:
        raise NotImplementedError(msg)
    raise RuntimeError(msg)


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)


# torch's raw accessors of the current device and stream: the public torch.cuda.current_device()
# and current_stream() re-run their lazy-initialisation and index checks on every call, which
# costs several microseconds per library call in a decode loop. The public forms stand in where
# a torch build lacks them.
_get_device = getattr(torch._C, "_cuda_getDevice", None) or torch.cuda.current_device
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def ensure_device(t: torch.Tensor, op: str) -> int:
    """Requires a CUDA tensor on an sm_100 device and makes that device current."""
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        dev = t.device if isinstance(t, torch.Tensor) else type(t).__name__
        raise TypeError(f"{op}: tileops_b200 runs on CUDA tensors only (got {dev})")
    idx = t.get_device()
    if idx not in _checked_devices:
        check(load().to_device_check(idx), op)
        _checked_devices.add(idx)
    if _get_device() != idx:
        torch.cuda.set_device(idx)
    return idx


def same_device(op: str, ref: torch.Tensor, *others: torch.Tensor | None) -> None:
    dev = ref.get_device()
    for o in others:
        if o is not None and o.get_device() != dev:
            raise TypeError(f"{op}: all tensors must be on {ref.device} (got {o.device})")


_WORKSPACES: dict[tuple[int, int], torch.Tensor] = {}
_WS_LOCK = threading.Lock()
_WS_BYTES: dict[tuple, int] = {}


def workspace_bytes(query: str, *shape: int) -> int:
    """The library's workspace size for these shapes (a pure function of them), queried once."""
    key = (query, *shape)
    v = _WS_BYTES.get(key)
    if v is None:
        v = int(getattr(load(), query)(*shape))
        _WS_BYTES[key] = v
    return v


def workspace(nbytes: int, device: int, stream: int | None = None) -> torch.Tensor | None:
    """Scratch of at least `nbytes` for a call about to be queued on the current stream of
    `device`. One buffer per (device, stream) serves consecutive calls: every kernel that takes a
    workspace touches it only after the previous kernel in its stream has completed (the
    decode kernel waits on griddepcontrol.wait first, the others are ordinary launches), and
    its flags are per-launch epochs left at zero once consumed. While the stream is being
    captured into a CUDA graph each call gets its own buffer from the graph's memory pool.
    `stream` is that current stream (stream_ptr(device)) when the caller has it already."""
    if nbytes <= 0:
        return None
    if torch.cuda.is_current_stream_capturing():
        return torch.empty(nbytes, dtype=torch.uint8, device=torch.device("cuda", device))
    key = (device, stream_ptr(device) if stream is None else stream)
    ws = _WORKSPACES.get(key)
    if ws is None or ws.numel() < nbytes:
        with _WS_LOCK:
            ws = _WORKSPACES.get(key)
            if ws is None or ws.numel() < nbytes:
                ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8,
                                 device=torch.device("cuda", device))
                _WORKSPACES[key] = ws
    return ws


def stream_ptr(device: int | None = None) -> int:
    """The current stream of `device` (default: the current device) as a cudaStream_t."""
    if _raw_stream is not None:
        return _raw_stream(_get_device() if device is None else device)
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def dtype_code(dt: torch.dtype, op: str) -> int:
    try:
        return DTYPE_CODES[dt]
    except KeyError:
        raise TypeError(f"{op}: unsupported dtype {dt}") from None


def device_error_word(clear: bool = True) -> int:
    """Reads the device error word set by kernels whose bounded waits expired (0 = none)."""
    v = ctypes.c_int(0)
    check(load().to_device_error_word(ctypes.byref(v), 1 if clear else 0), "device_error_word")
    return v.value


def wait_limit_selftest(limit_us: int, arrive: bool, out_ptr: int, stream: int = 0) -> None:
    """Launches the bounded-wait self-test: one warp waits on an mbarrier for at most
    `limit_us` microseconds; with `arrive` False nothing arrives and the wait gives up, setting
    the device error word to 1. `out_ptr` is a device buffer of two u64 that receives
    {completed, nanoseconds waited}."""
    check(load().to_wait_limit_selftest(int(limit_us), 1 if arrive else 0, out_ptr, stream),
          "wait_limit_selftest")


IPC_HANDLE_BYTES = 64


def ipc_alloc(nbytes: int) -> tuple[int, bytes]:
    """Allocates `nbytes` on the current device; returns (device pointer, CUDA IPC handle)."""
    p = _P(0)
    h = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    check(load().to_ipc_alloc(int(nbytes), ctypes.byref(p), h), "ipc_alloc")
    return int(p.value), h.raw


def ipc_open(handle: bytes) -> int:
    """Maps a peer process's buffer (its IPC handle) into this process; returns the pointer."""
    if len(handle) != IPC_HANDLE_BYTES:
        raise ValueError(f"ipc_open: a handle has {IPC_HANDLE_BYTES} bytes (got {len(handle)})")
    p = _P(0)
    h = ctypes.create_string_buffer(handle, IPC_HANDLE_BYTES)
    check(load().to_ipc_open(h, ctypes.byref(p)), "ipc_open")
    return int(p.value)


def ipc_close(ptr_value: int) -> None:
    check(load().to_ipc_close(ptr_value), "ipc_close")


def ipc_free(ptr_value: int) -> None:
    check(load().to_ipc_free(ptr_value), "ipc_free")


def version() -> str:
    return load().to_version().decode()


def set_launch_overlap(enable: bool) -> bool:
    """Turns programmatic dependent launch on or off for the small-M AWQ streaming kernels, the
    2-CTA W8A8 kernel and the dense GEMV, and returns the previous setting. With it on, a call may read its weights while the previous
    kernel in the stream is still running, so no kernel that writes those weights may be the
    launch immediately before it (a decode loop over fixed weights is the intended use)."""
    return bool(load().to_set_launch_overlap(1 if enable else 0))
