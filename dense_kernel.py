"""Drop-in for the reference's dense_kernel.py: ``dense_decode_attention``
runs the sm_100a split-K kernel of numerics-and-sparse-attn_b200."""
import importlib as _importlib

_pkg = _importlib.import_module("numerics-and-sparse-attn_b200")

dense_decode_attention = _pkg.dense_decode_attention

__all__ = ["dense_decode_attention"]
