"""The allocation-free sink+window entry point, nsa_sparse_decode_noalloc.

It is for callers that cannot allocate device memory where they decode (a
host runtime that owns all device memory through its own pool, a plain C
caller without an allocator): its split-K scratch is a static 4 MiB device
array inside the library instead of a caller-provided workspace.  These tests
call it through the C ABI, on two calls in a row with fresh inputs, and check
its output against the fp32 oracle (oracle/attention.py, run on the CPU for
the first sequences of the batch) and against the workspace entry point
(nsa_sparse_decode, via sparse_decode_attention) for the whole batch.  The
shapes cover every launch plan: split units (the static scratch holds tickets
and partials), the one-CTA-per-unit window kernel of the benchmark shape, and
whole-unit plans with B * Hkv >= 1024, which need no scratch and so have no
size limit.  Oversized split plans are refused.  This file is collected last
so that a failure here does not hide the results of the other tests.
"""
import importlib

import pytest
import torch

import sparse_kernel
from oracle import attention as oa

pytestmark = pytest.mark.gpu
TOL = 2e-3  # the fp16 paths' tolerance against the fp32 oracle (north_star)
DEV = "cuda"
_lib = importlib.import_module("numerics-and-sparse-attn_b200._lib")
ORACLE_ROWS = 4  # sequences checked against the CPU oracle (all rows against the workspace path)


def _noalloc(q, k, v, seq_len, window, sink=4, ring_heads=None):
    b, h, d = q.shape
    o = torch.empty_like(q)
    heads_ptr = ring_heads.data_ptr() if ring_heads is not None else None
    status = _lib.load().nsa_sparse_decode_noalloc(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), b, h, k.shape[1], d, window, sink, seq_len,
        None, heads_ptr, 128 ** -0.5, torch.cuda.current_stream().cuda_stream)
    return status, o


def _check_twice(B, W, L, seed, S=4, ring=False):
    g = torch.Generator(device=DEV).manual_seed(seed)
    head = (L - S) % W if ring and W > 0 and L > S else 0
    heads = torch.full((B,), head, dtype=torch.int32, device=DEV) if ring else None
    for call in range(2):
        q = torch.randn(B, 64, 128, device=DEV, generator=g).half()
        k = torch.randn(B, 8, S + W, 128, device=DEV, generator=g).half()
        v = torch.randn(B, 8, S + W, 128, device=DEV, generator=g).half()
        status, o = _noalloc(q, k, v, L, W, S, heads)
        assert status == 0, _lib.load().nsa_last_error_message()
        torch.cuda.synchronize()
        n = min(B, ORACLE_ROWS)
        ref = oa.sparse_attention_slots(q[:n].cpu().float(), k[:n].cpu().float(), v[:n].cpu().float(), L, W, S,
                                        ring_head=head)
        err = (o[:n].cpu().float() - ref).abs().max().item()
        assert err < TOL, ("oracle", call, err)
        ws = sparse_kernel.sparse_decode_attention(q, k, v, seq_len=L, window=W, sink=S, ring_head=heads)
        err = (o.float() - ws.float()).abs().max().item()
        assert err < TOL, ("workspace entry point", call, err)
    assert importlib.import_module("numerics-and-sparse-attn_b200").device_error() == 0


@pytest.mark.parametrize("B,W,L", [(2, 512, 5000), (3, 1024, 600), (4, 4096, 10_000)])
def test_noalloc_split_units_twice(B, W, L):
    """Fewer units than SMs and windows beyond the window kernel's 384 slots:
    each unit is split over several CTAs, whose tickets and partials live in
    the static scratch."""
    _check_twice(B, W, L, seed=B * 7 + W)


def test_noalloc_forced_stream_k_twice(monkeypatch):
    """Stream-K over 256 units with a long window (forced): every unit is
    split, so the scratch and its ticket reset are reused across both calls."""
    monkeypatch.setenv("NSA_SPLIT_MODE", "stream")
    _check_twice(32, 4096, 10_000, seed=11)


def test_noalloc_benchmark_shape_ring_twice():
    """The benchmark's sink+window shape (B=32, 8 KV heads, S=4, W=256, ring
    after L=163,840 tokens): one CTA per unit (window kernel), no scratch."""
    _check_twice(32, 256, 163_840, seed=3, ring=True)


@pytest.mark.parametrize("W", [256, 1024])
def test_noalloc_many_units_without_scratch_twice(W):
    """B * Hkv = 1024 units: W=256 takes the window kernel and W=1024 the
    whole-unit persistent plan.  Neither touches the scratch, so neither is
    bound by its 4 MiB (the split-K size of this shape would exceed it)."""
    assert _lib.load().nsa_sparse_workspace_bytes(128, 8, W, 4) > 4 * 1024 * 1024
    _check_twice(128, W, 50_000, seed=W)


def test_noalloc_empty_batch_is_a_no_op():
    z = torch.empty(0, 64, 128, device=DEV, dtype=torch.float16)
    kz = torch.empty(0, 8, 260, 128, device=DEV, dtype=torch.float16)
    status, _ = _noalloc(z, kz, kz, 1000, 256)
    assert status == 0


def test_noalloc_rejects_scratch_beyond_its_maximum(monkeypatch):
    """A split plan whose scratch exceeds the 4 MiB array is refused with
    NSA_ERR_UNSUPPORTED and a message, before anything is launched."""
    monkeypatch.setenv("NSA_SPLIT_MODE", "stream")  # force split-K partials for every unit
    B, W = 128, 4096
    q = torch.zeros(B, 64, 128, device=DEV, dtype=torch.float16)
    k = torch.zeros(B, 8, 4 + W, 128, device=DEV, dtype=torch.float16)
    status, _ = _noalloc(q, k, k, 8000, W)
    assert status == _lib.NSA_ERR_UNSUPPORTED
    assert b"4194304" in _lib.load().nsa_last_error_message()
    assert importlib.import_module("numerics-and-sparse-attn_b200").device_error() == 0
