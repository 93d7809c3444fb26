"""Drop-in for the reference's quant_kernel.py: the KIVI quantizers, the
quantized-cache builder and the quantized sink+window attention run the
sm_100a kernels of numerics-and-sparse-attn_b200.  ``dequantize_k`` /
``dequantize_v`` are host-callable forms of the reference's Triton-only
``_dequantize_k_tile`` / ``_dequantize_v_tile``."""
import importlib as _importlib

_pkg = _importlib.import_module("numerics-and-sparse-attn_b200")

quantize_k_cache = _pkg.quantize_k_cache
quantize_v_cache = _pkg.quantize_v_cache
build_quantized_kv_cache = _pkg.build_quantized_kv_cache
sparse_decode_attention_quantized = _pkg.sparse_decode_attention_quantized
dequantize_k = _pkg.dequantize_k
dequantize_v = _pkg.dequantize_v
KiviCache = _pkg.KiviCache

__all__ = ["quantize_k_cache", "quantize_v_cache", "build_quantized_kv_cache", "sparse_decode_attention_quantized",
           "dequantize_k", "dequantize_v", "KiviCache"]
