"""B200 (sm_100a) decode attention: dense GQA, StreamingLLM sink+window and
KIVI 2-bit, as a drop-in for the reference's dense_kernel.py,
sparse_kernel.py and quant_kernel.py entry points.

The kernels live in ``libnsa_b200.so`` (C ABI: include/nsa_b200.h), built by
``build.py``; this package is the thin Python host side over it.
"""
from . import _lib
from ._lib import HostPipe
from .constants import *  # noqa: F401,F403
from .decode import (RingCache, dense_decode_attention, dense_decode_attention_host, sparse_decode_attention,
                     sparse_decode_attention_host)
from .kivi import (KiviCache, build_quantized_kv_cache, decode_step_layers, dequantize_k, dequantize_v,
                   quantize_k_cache, quantize_v_cache, sparse_decode_attention_quantized)

__all__ = [
    "dense_decode_attention",
    "sparse_decode_attention",
    "quantize_k_cache",
    "quantize_v_cache",
    "build_quantized_kv_cache",
    "sparse_decode_attention_quantized",
    "dequantize_k",
    "dequantize_v",
    "KiviCache",
    "decode_step_layers",
    "RingCache",
    "HostPipe",
    "dense_decode_attention_host",
    "sparse_decode_attention_host",
    "native_library_path",
    "device_error",
]


def native_library_path() -> str:
    return _lib.LIB_PATH


def device_error(device=None) -> int:
    """Read and clear the device error word (0 when no kernel timed out)."""
    return _lib.device_error(device)
