"""Host-buffer entry points (HostPipe + *_host calls): the query and output in
pinned host memory, copies and decode pipelined on a two-slot pipe.  Every
output equals the device-tensor call on the same inputs (bit for bit on the
dense path; up to the last rounding for sink+window and KIVI, whose warps take
a unit's jobs in whichever order they free up), over enough calls that each slot is reused
(and, for KIVI, across a group flush), and the KIVI cache state after
host-buffer steps equals that after device steps bit for bit."""
import importlib

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"
pkg = importlib.import_module("numerics-and-sparse-attn_b200")


def _pinned(t):
    return t.cpu().contiguous().pin_memory()


def test_kivi_step_host_equals_device_step():
    B, Hkv, W, L = 32, 8, 256, 163_840
    g1 = torch.Generator(device=DEV).manual_seed(7)
    g2 = torch.Generator(device=DEV).manual_seed(7)
    dev_cache = pkg.KiviCache.synthetic(B, Hkv, W, L, device=DEV, generator=g1)
    host_cache = pkg.KiviCache.synthetic(B, Hkv, W, L, device=DEV, generator=g2)
    n_steps = 40  # crosses a group flush (every 32 steps)
    g = torch.Generator(device=DEV).manual_seed(8)
    qs = [torch.randn(B, 8 * Hkv, 128, device=DEV, generator=g).half() for _ in range(n_steps)]
    ks = [torch.randn(B, Hkv, 128, device=DEV, generator=g).half() for _ in range(n_steps)]
    vs = [torch.randn(B, Hkv, 128, device=DEV, generator=g).half() for _ in range(n_steps)]
    xs = [_pinned(torch.cat([q.flatten(), k.flatten(), v.flatten()])) for q, k, v in zip(qs, ks, vs)]
    outs = [torch.empty(B, 8 * Hkv, 128, dtype=torch.float16).pin_memory() for _ in range(n_steps)]
    pipe = pkg.HostPipe(xs[0].numel() * 2, outs[0].numel() * 2, device=DEV, depth=2)
    pipe.begin()
    for i in range(n_steps):
        host_cache.decode_step_host(pipe, xs[i], outs[i])
    pipe.end()
    ref = [dev_cache.decode_step(qs[i], ks[i], vs[i]).cpu() for i in range(n_steps)]
    torch.cuda.synchronize()
    for i in range(n_steps):
        assert (outs[i].float() - ref[i].float()).abs().max().item() < 2e-3, f"step {i}"
    a, b = dev_cache.state(), host_cache.state()
    for key in a:
        assert torch.equal(a[key], b[key]), key
    pipe.close()


@pytest.mark.parametrize("path", ["sparse", "dense"])
def test_fp16_host_equals_device(path):
    B, Hkv, S, W, L = 32, 8, 4, 256, 163_840
    g = torch.Generator(device=DEV).manual_seed(11)
    slots = S + W if path == "sparse" else 2048
    k = torch.randn(B, Hkv, slots, 128, device=DEV, generator=g).half()
    v = torch.randn(B, Hkv, slots, 128, device=DEV, generator=g).half()
    heads = torch.full((B,), (L - S) % W, dtype=torch.int32, device=DEV)
    n = 6
    qs = [torch.randn(B, 8 * Hkv, 128, device=DEV, generator=g).half() for _ in range(n)]
    q_h = [_pinned(q) for q in qs]
    o_h = [torch.empty(B, 8 * Hkv, 128, dtype=torch.float16).pin_memory() for _ in range(n)]
    pipe = pkg.HostPipe(q_h[0].numel() * 2, o_h[0].numel() * 2, device=DEV, depth=2)
    pipe.begin()
    for i in range(n):
        if path == "sparse":
            pkg.sparse_decode_attention_host(pipe, q_h[i], o_h[i], k, v, L, W, S, ring_head=heads)
        else:
            pkg.dense_decode_attention_host(pipe, q_h[i], o_h[i], k, v, slots - 5)
    pipe.end()
    torch.cuda.synchronize()
    for i in range(n):
        if path == "sparse":
            ref = pkg.sparse_decode_attention(qs[i], k, v, L, W, S, ring_head=heads)
        else:
            ref = pkg.dense_decode_attention(qs[i], k, v, slots - 5)
        if path == "dense":
            assert torch.equal(o_h[i], ref.cpu()), f"call {i}"
        else:
            assert (o_h[i].float() - ref.cpu().float()).abs().max().item() < 2e-3, f"call {i}"
    pipe.close()


def test_pipe_rejects_small_slots_and_device_buffers():
    B, Hkv = 32, 8
    g = torch.Generator(device=DEV).manual_seed(3)
    k = torch.randn(B, Hkv, 260, 128, device=DEV, generator=g).half()
    q_h = torch.zeros(B, 8 * Hkv, 128, dtype=torch.float16).pin_memory()
    o_h = torch.empty_like(q_h).pin_memory()
    small = pkg.HostPipe(1024, 1024, device=DEV)
    with pytest.raises(pkg._lib.NativeError, match="pipe slots"):
        pkg.sparse_decode_attention_host(small, q_h, o_h, k, k, 1000, 256, 4)
    small.close()
    pipe = pkg.HostPipe(q_h.numel() * 2, o_h.numel() * 2, device=DEV)
    with pytest.raises(ValueError, match="host tensor"):
        pkg.sparse_decode_attention_host(pipe, q_h.to(DEV), o_h, k, k, 1000, 256, 4)
    pipe.close()
    with pytest.raises(pkg._lib.NativeError, match="non-zero slot sizes"):
        pkg.HostPipe(0, 16, device=DEV)
