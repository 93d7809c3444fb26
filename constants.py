"""Drop-in for the reference's constants.py: the same names and values, taken
from the B200 package (numerics-and-sparse-attn_b200/constants.py)."""
import importlib as _importlib

_c = _importlib.import_module("numerics-and-sparse-attn_b200.constants")

BATCH = _c.BATCH
N_HEADS = _c.N_HEADS
N_KV_HEADS = _c.N_KV_HEADS
GQA_GROUP = _c.GQA_GROUP
D_HEAD = _c.D_HEAD
BLOCK_N = _c.BLOCK_N
SINK_SIZE = _c.SINK_SIZE
RESIDUAL_SIZE = _c.RESIDUAL_SIZE
GROUP_SIZE = _c.GROUP_SIZE
QUANT_BITS = _c.QUANT_BITS
CONTEXT_LENGTHS = _c.CONTEXT_LENGTHS
WINDOW_SIZES = _c.WINDOW_SIZES
