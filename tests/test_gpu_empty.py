"""Empty batches: every entry point accepts B = 0 (zero-size tensors, whose
data pointers are NULL), does no work and returns correctly shaped empty
outputs, and a following non-empty call on the same device is unaffected.
(The reference derives its grid from constants, not from the tensors --
dense_kernel.py:75, sparse_kernel.py:110, quant_kernel.py:567 -- so it has no
empty case of its own; this is the superset behaviour of the C ABI.)"""
import importlib

import pytest
import torch

import dense_kernel
import quant_kernel
import sparse_kernel

pytestmark = pytest.mark.gpu
DEV = "cuda"
pkg = importlib.import_module("numerics-and-sparse-attn_b200")


def _h(*shape):
    return torch.empty(*shape, dtype=torch.float16, device=DEV)


def test_dense_and_sparse_empty_batch():
    q, k = _h(0, 64, 128), _h(0, 8, 300, 128)
    o = dense_kernel.dense_decode_attention(q, k, k, 300)
    assert o.shape == (0, 64, 128) and o.dtype == torch.float16
    kc = _h(0, 8, 4 + 256, 128)
    o = sparse_kernel.sparse_decode_attention(q, kc, kc, 163_840, 256)
    assert o.shape == (0, 64, 128)
    o = sparse_kernel.sparse_decode_attention(q, kc, kc, 163_840, 256, ring_head=3)
    assert o.shape == (0, 64, 128)
    torch.cuda.synchronize()
    assert pkg.device_error(torch.device(DEV)) == 0


def test_kivi_empty_batch():
    k = torch.empty(0, 8, 256, 128, dtype=torch.float32, device=DEV)
    for fn in (quant_kernel.quantize_k_cache, quant_kernel.quantize_v_cache):
        packed, scale, zero = fn(k)
        assert packed.shape[0] == 0 and scale.shape[0] == 0 and zero.shape[0] == 0
    cache = quant_kernel.build_quantized_kv_cache(_h(0, 8, 4 + 256, 128), _h(0, 8, 4 + 256, 128))
    q = _h(0, 64, 128)
    o = quant_kernel.sparse_decode_attention_quantized(
        q, cache["k_residual"], cache["v_residual"], cache["k_sink_packed"], cache["k_sink_scale"],
        cache["k_sink_zero"], cache["v_sink_packed"], cache["v_sink_scale"], cache["v_sink_zero"],
        cache["k_win_packed"], cache["k_win_scale"], cache["k_win_zero"], cache["v_win_packed"],
        cache["v_win_scale"], cache["v_win_zero"], seq_len=163_840, window=256)
    assert o.shape == (0, 64, 128)
    sc = quant_kernel.KiviCache(0, 8, 256, device=DEV)
    tok = _h(0, 8, 128)
    assert sc.decode_step(q, tok, tok).shape == (0, 64, 128)
    sc.append(tok, tok)
    assert sc.attend(q).shape == (0, 64, 128)
    torch.cuda.synchronize()
    assert pkg.device_error(torch.device(DEV)) == 0


def test_ring_empty_batch_then_nonempty():
    ring = pkg.RingCache(0, 8, 256, device=DEV)
    q, tok = _h(0, 64, 128), _h(0, 8, 128)
    assert ring.decode_step(q, tok, tok).shape == (0, 64, 128)
    ring.append(tok, tok)
    assert ring.attend(q).shape == (0, 64, 128)
    # the device is untouched: a normal call afterwards still matches its own append + attend
    g = torch.Generator(device=DEV).manual_seed(7)
    r1, r2 = pkg.RingCache(2, 8, 64, device=DEV), pkg.RingCache(2, 8, 64, device=DEV)
    for _ in range(5):
        q = torch.randn(2, 64, 128, device=DEV, generator=g).half()
        nk = torch.randn(2, 8, 128, device=DEV, generator=g).half()
        nv = torch.randn(2, 8, 128, device=DEV, generator=g).half()
        a = r1.decode_step(q, nk, nv)
        r2.append(nk, nv)
        b = r2.attend(q)
        assert torch.equal(a, b)
    torch.cuda.synchronize()
    assert pkg.device_error(torch.device(DEV)) == 0
