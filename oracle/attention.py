"""Decode-attention oracles (PyTorch, fp32).  TEST INFRASTRUCTURE ONLY.

Plain-PyTorch restatements of the reference's own oracles.  Like the
reference's, they follow the device of their inputs (CPU in the CPU suite; the
GPU parity tests may run them on CUDA tensors as the fp32 checker).

* ``dense_attention``          test_dense_correctness.py:13-30
* ``sparse_attention_full``    test_sparse_correctness.py:22-48, with the GQA
                               group derived from the shapes instead of the
                               module constant GQA_GROUP (the reference's
                               version raises on 8 query / 2 KV heads).
* ``build_compacted_cache``    test_sparse_correctness.py:51-72, shape-generic.
* ``slot_validity``            sparse_kernel.py:15-46 (``_kv_indices``) plus the
                               ring-buffer head offset used by the ring layout.
* ``sparse_attention_slots``   what sparse_kernel.py:67-102 computes: softmax
                               over the valid physical slots of a cache.
* ``quantized_attention``      test_quantized_attention_correctness.py:32-61.
"""
from __future__ import annotations

import numpy as np
import torch

from . import kivi as _kivi

GARBAGE_VALUE = 1e4  # test_sparse_correctness.py:15


def _attend(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, sm_scale: float,
            mask: torch.Tensor | None = None) -> torch.Tensor:
    """GQA by reshape + einsum broadcast (test_dense_correctness.py:23-30).

    q [B, H, D]; k, v [B, KV, N, D]; mask [B or 1, N] bool (True = attend)."""
    b, h, d = q.shape
    kv = k.shape[1]
    g = h // kv
    qf = q.float().reshape(b, kv, g, d)
    qk = torch.einsum("bkgd,bknd->bkgn", qf, k.float()) * sm_scale
    if mask is not None:
        qk = qk.masked_fill(~mask[:, None, None, :], float("-inf"))
    p = torch.softmax(qk, dim=-1)
    o = torch.einsum("bkgn,bknd->bkgd", p, v.float())
    return o.reshape(b, h, d)


def dense_attention(q, k, v, sm_scale=None):
    """Dense causal GQA decode over all cached tokens (test_dense_correctness.py:13-30)."""
    if sm_scale is None:
        sm_scale = q.shape[-1] ** -0.5
    return _attend(q, k, v, sm_scale)


def sparse_attention_full(q, k_full, v_full, seq_len: int, window: int, sink: int, sm_scale=None):
    """StreamingLLM mask over the full un-evicted context
    (test_sparse_correctness.py:22-48): dense until seq_len > sink+window,
    then ``pos < sink | pos >= seq_len - window``."""
    if sm_scale is None:
        sm_scale = q.shape[-1] ** -0.5
    pos = torch.arange(seq_len, device=q.device)
    if seq_len <= sink + window:
        mask = torch.ones(seq_len, dtype=torch.bool, device=q.device)
    else:
        mask = (pos < sink) | (pos >= seq_len - window)
    return _attend(q, k_full[:, :, :seq_len], v_full[:, :, :seq_len], sm_scale, mask[None])


def build_compacted_cache(k_full, v_full, seq_len: int, window: int, sink: int,
                          garbage: float = GARBAGE_VALUE):
    """[B, KV, sink+window, D] compacted cache (test_sparse_correctness.py:51-72):
    slot i < sink holds position i; slot sink+i holds position
    seq_len-window+i; slots whose position does not exist hold ``garbage``."""
    b, kv, _, d = k_full.shape
    kc = torch.full((b, kv, sink + window, d), garbage, dtype=k_full.dtype, device=k_full.device)
    vc = torch.full_like(kc, garbage)
    ns = min(sink, seq_len)
    kc[:, :, :ns] = k_full[:, :, :ns]
    vc[:, :, :ns] = v_full[:, :, :ns]
    start = seq_len - window
    for i in range(window):
        pos = start + i
        if 0 <= pos < seq_len:
            kc[:, :, sink + i] = k_full[:, :, pos]
            vc[:, :, sink + i] = v_full[:, :, pos]
    return kc, vc


def build_ring_cache(k_full, v_full, seq_len: int, window: int, sink: int,
                     garbage: float = GARBAGE_VALUE):
    """Ring layout of the same cache: position p < sink at slot p, position
    p >= sink at slot ``sink + (p - sink) % window``; returns (k, v, ring_head)
    with ``ring_head = (seq_len - sink) % window`` (0 when window == 0)."""
    b, kv, _, d = k_full.shape
    kc = torch.full((b, kv, sink + window, d), garbage, dtype=k_full.dtype, device=k_full.device)
    vc = torch.full_like(kc, garbage)
    ns = min(sink, seq_len)
    kc[:, :, :ns] = k_full[:, :, :ns]
    vc[:, :, :ns] = v_full[:, :, :ns]
    for pos in range(max(sink, seq_len - window), seq_len):
        s = sink + (pos - sink) % window
        kc[:, :, s] = k_full[:, :, pos]
        vc[:, :, s] = v_full[:, :, pos]
    head = (seq_len - sink) % window if window > 0 and seq_len > sink else 0
    return kc, vc, head


def slot_validity(seq_len: int, window: int, sink: int, ring_head: int = 0) -> np.ndarray:
    """Validity of each physical slot [sink+window] (sparse_kernel.py:15-46).

    Sink slot s is valid iff s < seq_len.  Window slot s maps to logical
    window index ``i = (s - sink - ring_head) mod window`` and position
    ``seq_len - window + i``; it is valid iff that position is >= sink.
    ring_head = 0 is the reference's compacted layout."""
    n = sink + window
    valid = np.zeros(n, bool)
    for s in range(n):
        if s < sink:
            valid[s] = s < seq_len
        else:
            i = (s - sink - ring_head) % window
            valid[s] = (seq_len - window + i) >= sink
    return valid


def sparse_attention_slots(q, k_cache, v_cache, seq_len: int, window: int, sink: int,
                           ring_head: int = 0, sm_scale=None):
    """Softmax over the valid physical slots of a compacted or ring cache."""
    if sm_scale is None:
        sm_scale = q.shape[-1] ** -0.5
    mask = torch.from_numpy(slot_validity(seq_len, window, sink, ring_head)).to(q.device)
    return _attend(q, k_cache, v_cache, sm_scale, mask[None])


def quantized_attention(q, win_old_len: int, cache: dict, sink: int = 4, sm_scale=None):
    """KIVI oracle (test_quantized_attention_correctness.py:32-61): dequantize
    sink[:sink] + window-old + residual from the same packed tensors and run
    fp32 attention over their concatenation."""
    d = q.shape[-1]
    if sm_scale is None:
        sm_scale = d ** -0.5
    def _np(x):
        return x.detach().cpu().numpy() if hasattr(x, "detach") else np.asarray(x)

    g = _np(cache["k_sink_packed"]).shape[2] * 4  # the padded sink group's token count

    ks = _kivi.unpack_dequant(_np(cache["k_sink_packed"]), _np(cache["k_sink_scale"]), _np(cache["k_sink_zero"]), g, 2)[:, :, :sink]
    vs = _kivi.unpack_dequant(_np(cache["v_sink_packed"]), _np(cache["v_sink_scale"]), _np(cache["v_sink_zero"]), d, 3)[:, :, :sink]
    kw = _kivi.unpack_dequant(_np(cache["k_win_packed"]), _np(cache["k_win_scale"]), _np(cache["k_win_zero"]), win_old_len, 2)
    vw = _kivi.unpack_dequant(_np(cache["v_win_packed"]), _np(cache["v_win_scale"]), _np(cache["v_win_zero"]), d, 3)
    kr = torch.as_tensor(_np(cache["k_residual"])).float().numpy()
    vr = torch.as_tensor(_np(cache["v_residual"])).float().numpy()
    k = torch.from_numpy(np.concatenate([ks, kw, kr], axis=2))
    v = torch.from_numpy(np.concatenate([vs, vw, vr], axis=2))
    return _attend(q.detach().cpu().float(), k, v, sm_scale)


def stream_attention(q, st: dict, seq_len: int, geom, sm_scale=None):
    """Attention over a streaming KIVI cache state (``kivi.stream_state``)."""
    if sm_scale is None:
        sm_scale = q.shape[-1] ** -0.5
    k, v = _kivi.stream_dequant_tokens(st, seq_len, geom)
    return _attend(q.detach().cpu().float(), torch.from_numpy(k), torch.from_numpy(v), sm_scale)
