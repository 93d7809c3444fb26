"""The fp16 ring cache with per-unit lengths (RingCache / nsa_ring_*): the
cache contents after every append are the history's positions in their ring
slots, and attention equals the oracle's sink+window attention over the same
slots (sparse_kernel.py:15-46 slot rule with the ring head), through the sink
phase, the first window fill and wrap-around; the one-launch step (B=32: every
unit has its own CTA) leaves the cache of append + decode bit for bit and the
same outputs up to the last rounding (the window kernel's warps claim a unit's
jobs as they free up, so the accumulation order varies between launches)."""
import importlib

import pytest
import torch

from oracle import attention as oa

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 2e-3  # fp16 paths (north_star)
pkg = importlib.import_module("numerics-and-sparse-attn_b200")


def _err(a, b):
    return (a.float().cpu() - torch.as_tensor(b).float().cpu()).abs().max().item()


def _expected_cache(k_hist, L, S, W):
    """Ring slots after appending positions [0, L) (zeros where never written)."""
    B, H, _, D = k_hist.shape
    out = torch.zeros(B, H, S + W, D, dtype=k_hist.dtype, device=k_hist.device)
    for p in range(L):
        if p < S:
            out[:, :, p] = k_hist[:, :, p]
        elif W > 0:
            out[:, :, S + (p - S) % W] = k_hist[:, :, p]
    return out


@pytest.mark.parametrize("B,W", [(32, 256), (32, 60), (2, 256), (2, 0)])
def test_ring_from_empty_matches_oracle(B, W):
    S, Hkv = 4, 8
    n = S + 2 * W + 9
    g = torch.Generator(device=DEV).manual_seed(B * 1000 + W)
    k_hist = torch.randn(B, Hkv, n, 128, device=DEV, generator=g).half()
    v_hist = torch.randn(B, Hkv, n, 128, device=DEV, generator=g).half()
    cache = pkg.RingCache(B, Hkv, W, sink=S, device=DEV)
    check = {1, 2, S, S + 1, S + W - 1, S + W, S + W + 1, n} | set(range(3, n + 1, 97))
    for L in range(1, n + 1):
        q = torch.randn(B, 8 * Hkv, 128, device=DEV, generator=g).half()
        o = cache.decode_step(q, k_hist[:, :, L - 1].contiguous(), v_hist[:, :, L - 1].contiguous())
        if L in check:
            assert (cache.unit_lens == L).all()
            assert torch.equal(cache.k, _expected_cache(k_hist, L, S, W)), L
            assert torch.equal(cache.v, _expected_cache(v_hist, L, S, W)), L
            head = cache.ring_head()
            ref = oa.sparse_attention_slots(q.float(), cache.k.float(), cache.v.float(), L, W, S, ring_head=head)
            assert _err(o, ref) < TOL, L


def test_ring_fused_step_equals_append_then_attend():
    B, Hkv, S, W = 32, 8, 4, 256
    g = torch.Generator(device=DEV).manual_seed(9)
    fused = pkg.RingCache(B, Hkv, W, sink=S, device=DEV)
    split = pkg.RingCache(B, Hkv, W, sink=S, device=DEV)
    for L in range(1, S + W + 40):
        q = torch.randn(B, 64, 128, device=DEV, generator=g).half()
        nk = torch.randn(B, Hkv, 128, device=DEV, generator=g).half()
        nv = torch.randn(B, Hkv, 128, device=DEV, generator=g).half()
        o_f = fused.decode_step(q, nk, nv)
        split.append(nk, nv)
        o_s = split.attend(q)
        assert (o_f.float() - o_s.float()).abs().max().item() < 2e-3, L  # rounding-level
    assert torch.equal(fused.k, split.k) and torch.equal(fused.v, split.v)
    assert torch.equal(fused.unit_lens, split.unit_lens)


def test_ring_load_history_then_steps():
    """load_history at L=163,840 (the benchmark state) equals the ring of the
    history, and further one-launch steps match the oracle."""
    B, Hkv, S, W, L = 32, 8, 4, 256, 163_840
    g = torch.Generator(device=DEV).manual_seed(4)
    k_tail = torch.randn(B, Hkv, W + 4, 128, device=DEV, generator=g).half()  # positions L-W-4 .. L-1
    v_tail = torch.randn(B, Hkv, W + 4, 128, device=DEV, generator=g).half()
    k_sink = torch.randn(B, Hkv, S, 128, device=DEV, generator=g).half()
    v_sink = torch.randn(B, Hkv, S, 128, device=DEV, generator=g).half()
    k_hist = torch.zeros(B, Hkv, L, 128, device=DEV, dtype=torch.float16)
    v_hist = torch.zeros_like(k_hist)
    k_hist[:, :, :S], v_hist[:, :, :S] = k_sink, v_sink
    k_hist[:, :, L - W - 4:], v_hist[:, :, L - W - 4:] = k_tail, v_tail
    cache = pkg.RingCache(B, Hkv, W, sink=S, device=DEV)
    cache.load_history(k_hist, v_hist, L)
    del k_hist, v_hist
    for step in range(3):
        q = torch.randn(B, 64, 128, device=DEV, generator=g).half()
        nk = torch.randn(B, Hkv, 128, device=DEV, generator=g).half()
        nv = torch.randn(B, Hkv, 128, device=DEV, generator=g).half()
        o = cache.decode_step(q, nk, nv)
        Lc = L + step + 1
        ref = oa.sparse_attention_slots(q.float(), cache.k.float(), cache.v.float(), Lc, W, S,
                                        ring_head=cache.ring_head())
        assert _err(o, ref) < TOL, step
        # the newest token sits at its ring slot
        assert torch.equal(cache.k[:, :, S + (Lc - 1 - S) % W], nk)
