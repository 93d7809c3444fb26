"""Drop-in for the reference's sparse_kernel.py: ``sparse_decode_attention``
runs the sm_100a sink+window kernel of numerics-and-sparse-attn_b200."""
import importlib as _importlib

_pkg = _importlib.import_module("numerics-and-sparse-attn_b200")

sparse_decode_attention = _pkg.sparse_decode_attention

__all__ = ["sparse_decode_attention"]
