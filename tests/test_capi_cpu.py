"""CPU-only checks of the boundary: the C-ABI library builds, loads and
exports every function declared in include/*.h; the Python binding declares
a prototype for each; host-side argument checks raise before any GPU work."""
import ctypes
import glob
import importlib
import os
import re

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = importlib.import_module("numerics-and-sparse-attn_b200")
LIBMOD = importlib.import_module("numerics-and-sparse-attn_b200._lib")


def _declared():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names.update(re.findall(r"\b(nsa_[a-z0-9_]+)\s*\(", src))
    return sorted(names)


@pytest.fixture(scope="module")
def lib():
    build = importlib.import_module("numerics-and-sparse-attn_b200.build")
    build.build()
    return ctypes.CDLL(LIBMOD.LIB_PATH)


def test_header_declares_entry_points():
    names = _declared()
    assert "nsa_dense_decode" in names and "nsa_sparse_decode" in names
    assert len(names) >= 8


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in _declared() if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"


def test_python_binding_covers_header():
    assert sorted(LIBMOD.PROTOTYPES) == _declared()


def test_status_strings(lib):
    L = LIBMOD.load()
    assert L.nsa_error_string(0) == b"NSA_OK"
    assert L.nsa_error_string(6) == b"NSA_ERR_TIMEOUT"
    assert b"sm_100a" in L.nsa_version()


def test_workspace_queries_without_gpu(lib):
    L = LIBMOD.load()
    # queries are pure host arithmetic (SM count falls back when no device)
    assert L.nsa_dense_workspace_bytes(32, 8, 8192) > 0
    assert L.nsa_sparse_workspace_bytes(32, 8, 256, 4) > 0
    assert L.nsa_dense_workspace_bytes(-1, 8, 10) == 0
    # an empty batch is a valid (no-op) call: its queries return without work
    assert L.nsa_dense_workspace_bytes(0, 8, 8192) < 4096
    assert L.nsa_sparse_workspace_bytes(0, 8, 256, 4) < 4096
    assert L.nsa_kivi_workspace_bytes(0, 8, 256, 128) < 4096


def test_host_validation_rejects_cpu_tensors():
    q = torch.zeros(2, 64, 128, dtype=torch.float16)
    k = torch.zeros(2, 8, 16, 128, dtype=torch.float16)
    with pytest.raises(ValueError, match="CUDA"):
        PKG.dense_decode_attention(q, k, k, seq_len=16)
    with pytest.raises(ValueError, match="CUDA"):
        PKG.sparse_decode_attention(q, k, k, seq_len=16, window=12)


def test_drop_in_modules_mirror_reference_names():
    import constants
    import dense_kernel
    import sparse_kernel

    assert (constants.BATCH, constants.N_HEADS, constants.N_KV_HEADS, constants.GQA_GROUP, constants.D_HEAD) == \
        (32, 64, 8, 8, 128)
    assert (constants.SINK_SIZE, constants.RESIDUAL_SIZE, constants.GROUP_SIZE, constants.QUANT_BITS) == \
        (4, 128, 32, 2)
    assert callable(dense_kernel.dense_decode_attention)
    assert callable(sparse_kernel.sparse_decode_attention)
