"""The allocation-free sink+window entry point, nsa_sparse_decode_noalloc.

It is for callers that cannot allocate device memory where they decode (a
host runtime that owns all device memory through its own pool, a plain C
caller without an allocator): its split-K scratch is a static 4 MiB device
array inside the library instead of a caller-provided workspace.  These tests
call it through the C ABI and compare it with the workspace entry point
(nsa_sparse_decode, via sparse_decode_attention) on two calls in a row, in
shapes that use the split-K scratch, and check that oversized shapes are
refused.  This file is collected last so that a failure here does not hide
the results of the other tests.
"""
import ctypes
import importlib

import pytest
import torch

import sparse_kernel

pytestmark = pytest.mark.gpu
TOL = 2e-3  # the fp16 paths' tolerance (tests/test_gpu_fp16_decode.py)
DEV = "cuda"
_lib = importlib.import_module("numerics-and-sparse-attn_b200._lib")


def _noalloc(q, k, v, seq_len, window, sink=4, ring_heads=None):
    b, h, d = q.shape
    o = torch.empty_like(q)
    heads_ptr = ring_heads.data_ptr() if ring_heads is not None else None
    status = _lib.load().nsa_sparse_decode_noalloc(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), b, h, k.shape[1], d, window, sink, seq_len,
        None, heads_ptr, 128 ** -0.5, torch.cuda.current_stream().cuda_stream)
    return status, o


@pytest.mark.parametrize("B,W,L", [(2, 256, 5000), (32, 4096, 10_000), (3, 1024, 600)])
def test_noalloc_matches_workspace_entry_point_twice(B, W, L):
    """Split-K shapes (fewer units than SMs, or long windows): the static
    scratch holds tickets and partials; two calls in a row with different
    inputs both match the workspace entry point."""
    g = torch.Generator(device=DEV).manual_seed(B * 7 + W)
    for call in range(2):
        q = torch.randn(B, 64, 128, device=DEV, generator=g).half()
        k = torch.randn(B, 8, 4 + W, 128, device=DEV, generator=g).half()
        v = torch.randn(B, 8, 4 + W, 128, device=DEV, generator=g).half()
        status, o = _noalloc(q, k, v, L, W)
        assert status == 0, _lib.load().nsa_last_error_message()
        ref = sparse_kernel.sparse_decode_attention(q, k, v, seq_len=L, window=W)
        err = (o.float() - ref.float()).abs().max().item()
        assert err < TOL, (call, err)


def test_noalloc_ring_layout_twice():
    B, W, S, L = 4, 256, 4, 163_840
    head = (L - S) % W
    heads = torch.full((B,), head, dtype=torch.int32, device=DEV)
    g = torch.Generator(device=DEV).manual_seed(3)
    for _ in range(2):
        q = torch.randn(B, 64, 128, device=DEV, generator=g).half()
        k = torch.randn(B, 8, S + W, 128, device=DEV, generator=g).half()
        v = torch.randn(B, 8, S + W, 128, device=DEV, generator=g).half()
        status, o = _noalloc(q, k, v, L, W, S, heads)
        assert status == 0
        ref = sparse_kernel.sparse_decode_attention(q, k, v, seq_len=L, window=W, ring_head=heads)
        assert (o.float() - ref.float()).abs().max().item() < TOL


def test_noalloc_rejects_scratch_beyond_its_maximum(monkeypatch):
    """A shape whose split-K scratch exceeds the 4 MiB array is refused with
    NSA_ERR_UNSUPPORTED and a message, before anything is launched."""
    monkeypatch.setenv("NSA_SPLIT_MODE", "stream")  # force split-K partials for every unit
    B, W = 128, 4096
    q = torch.zeros(B, 64, 128, device=DEV, dtype=torch.float16)
    k = torch.zeros(B, 8, 4 + W, 128, device=DEV, dtype=torch.float16)
    status, _ = _noalloc(q, k, k, 8000, W)
    assert status == _lib.NSA_ERR_UNSUPPORTED
    assert b"4194304" in _lib.load().nsa_last_error_message()
    assert importlib.import_module("numerics-and-sparse-attn_b200").device_error() == 0
