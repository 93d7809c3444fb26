"""ctypes binding of the C ABI in include/nsa_b200.h.

The shared library is loaded from this package directory only; if it is
missing the first call raises (there is no CPU fallback).  Status codes from
the library become Python exceptions: argument problems ValueError, anything
from the CUDA runtime RuntimeError.
"""
from __future__ import annotations

import contextlib
import ctypes
import os
import threading

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libnsa_b200.so")

NSA_OK = 0
NSA_ERR_INVALID = 1
NSA_ERR_ALIGN = 2
NSA_ERR_UNSUPPORTED = 3
NSA_ERR_WORKSPACE = 4
NSA_ERR_CUDA = 5
NSA_ERR_TIMEOUT = 6

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32
_F = ctypes.c_float
_SZ = ctypes.c_size_t
_INT = ctypes.c_int

# name -> (restype, argtypes); the C declarations are in include/nsa_b200.h
PROTOTYPES = {
    "nsa_error_string": (ctypes.c_char_p, [_INT]),
    "nsa_last_error_message": (ctypes.c_char_p, []),
    "nsa_device_error": (_INT, [ctypes.POINTER(_INT), _P]),
    "nsa_selftest_wait_timeout": (_INT, [_I64, _P]),
    "nsa_version": (ctypes.c_char_p, []),
    "nsa_dense_workspace_bytes": (_SZ, [_I64, _I64, _I64]),
    "nsa_dense_decode": (_INT, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _F, _P, _SZ, _P]),
    "nsa_sparse_workspace_bytes": (_SZ, [_I64, _I64, _I64, _I64]),
    "nsa_sparse_decode": (_INT, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P, _F, _P, _SZ,
                                 _P]),
    "nsa_sparse_decode_noalloc": (_INT, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P, _F, _P]),
    "nsa_kivi_quantize_k": (_INT, [_P, _INT, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _P]),
    "nsa_kivi_quantize_v": (_INT, [_P, _INT, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _P]),
    "nsa_kivi_dequant_k": (_INT, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _P]),
    "nsa_kivi_dequant_v": (_INT, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _P]),
    "nsa_kivi_workspace_bytes": (_SZ, [_I64, _I64, _I64, _I64]),
    "nsa_kivi_decode": (_INT, [_P] * 16 + [_I64] * 10 + [_F, _P, _SZ, _P]),
    "nsa_kivi_append": (_INT, [_P, _P, _P, _P]),
    "nsa_kivi_stream_workspace_bytes": (_SZ, [_P]),
    "nsa_kivi_stream_step_launches": (_INT, [_P]),
    "nsa_kivi_stream_decode": (_INT, [_P, _P, _P, _F, _P, _SZ, _P]),
    "nsa_kivi_stream_decode_step": (_INT, [_P, _P, _P, _P, _P, _F, _P, _SZ, _P]),
    "nsa_kivi_stream_decode_step_layers": (_INT, [_P, _I64, _P, _P, _P, _P, _F, _P, _SZ, _P]),
    "nsa_ring_append": (_INT, [_P, _P, _P, _P, _P] + [_I64] * 5 + [_P]),
    "nsa_ring_decode": (_INT, [_P, _P, _P, _P] + [_I64] * 6 + [_P, _F, _P, _SZ, _P]),
    "nsa_ring_decode_step": (_INT, [_P, _P, _P, _P] + [_I64] * 6 + [_P, _P, _P, _F, _P, _SZ, _P]),
    "nsa_host_pipe_create": (_P, [_SZ, _SZ, _INT]),
    "nsa_host_pipe_destroy": (None, [_P]),
    "nsa_host_pipe_begin": (_INT, [_P, _P]),
    "nsa_host_pipe_end": (_INT, [_P, _P]),
    "nsa_kivi_stream_decode_step_host": (_INT, [_P, _P, _P, _P, _F, _P, _SZ, _P]),
    "nsa_sparse_decode_host": (_INT, [_P, _P, _P, _P, _P] + [_I64] * 7 + [_P, _P, _F, _P, _SZ, _P]),
    "nsa_dense_decode_host": (_INT, [_P, _P, _P, _P, _P] + [_I64] * 6 + [_F, _P, _SZ, _P]),
}

_lock = threading.Lock()
_lib = None


class NativeError(RuntimeError):
    """A CUDA-level failure reported by the native library."""


def load() -> ctypes.CDLL:
    """Load libnsa_b200.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"native library {LIB_PATH} is not built; run "
                    "`python numerics-and-sparse-attn_b200/build.py` (or __graft_entry__.build())")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in PROTOTYPES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(status: int) -> None:
    """Raise the Python exception matching a C status code."""
    if status == NSA_OK:
        return
    lib = load()
    msg = lib.nsa_last_error_message().decode(errors="replace")
    name = lib.nsa_error_string(status).decode()
    if status in (NSA_ERR_INVALID, NSA_ERR_ALIGN, NSA_ERR_UNSUPPORTED):
        raise ValueError(f"{name}: {msg}")
    raise NativeError(f"{name}: {msg}")


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def device_error(device: torch.device | None = None) -> int:
    """Synchronize the current stream and return (and clear) the device error
    word (NSA_OK when no kernel recorded a timeout)."""
    dev = device or torch.device("cuda", torch.cuda.current_device())
    code = _INT(0)
    with torch.cuda.device(dev):
        check(load().nsa_device_error(ctypes.byref(code), stream_handle(dev)))
    return code.value


_ws_lock = threading.Lock()
_workspaces: dict = {}


def on_device(device: torch.device):
    """torch.cuda.device(device), or no context when it is already current."""
    if device.index is None or torch.cuda.current_device() == device.index:
        return contextlib.nullcontext()
    return torch.cuda.device(device)


def workspace(device: torch.device, nbytes: int, stream: int | None = None) -> torch.Tensor:
    """Zero-initialised scratch buffer for split-K partials and tickets, one
    per (device, stream); the kernels leave its counters zeroed again."""
    key = (device.index, stream_handle(device) if stream is None else stream)
    with _ws_lock:
        ws = _workspaces.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
            _workspaces[key] = ws
    return ws


class HostPipe:
    """Device staging slots and copy streams for the host-buffer entry points
    (nsa_host_pipe in include/nsa_b200.h): ``depth`` slots of ``in_bytes`` of
    input and ``out_bytes`` of output on ``device``.  Consecutive host-buffer
    calls through one pipe overlap their copies with each other's decode;
    ``begin()`` / ``end()`` order the pipe's copies after / before the current
    stream's work (the outputs are in host memory once the stream passes
    ``end()``)."""

    def __init__(self, in_bytes: int, out_bytes: int, device=None, depth: int = 2):
        dev = torch.device(device) if device is not None else torch.device("cuda")
        self.device = dev if dev.index is not None else torch.device("cuda", torch.cuda.current_device())
        self.in_bytes, self.out_bytes, self.depth = int(in_bytes), int(out_bytes), int(depth)
        lib = load()
        with on_device(self.device):
            h = lib.nsa_host_pipe_create(self.in_bytes, self.out_bytes, self.depth)
        if not h:
            raise NativeError("nsa_host_pipe_create: " + lib.nsa_last_error_message().decode(errors="replace"))
        self.handle = h

    def begin(self, stream: int | None = None) -> None:
        with on_device(self.device):
            check(load().nsa_host_pipe_begin(self.handle, stream_handle(self.device) if stream is None else stream))

    def end(self, stream: int | None = None) -> None:
        with on_device(self.device):
            check(load().nsa_host_pipe_end(self.handle, stream_handle(self.device) if stream is None else stream))

    def close(self) -> None:
        h, self.handle = getattr(self, "handle", None), None
        if h:
            load().nsa_host_pipe_destroy(h)

    def __del__(self):
        try:
            self.close()
        except Exception:  # interpreter shutdown
            pass
