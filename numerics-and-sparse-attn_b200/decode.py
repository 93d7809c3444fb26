"""Host side of the fp16-cache decode paths (dense, sink+window).

Mirrors the reference's Python entry points -- same names, argument meaning
and defaults -- and forwards to the C ABI (include/nsa_b200.h).  Differences,
all strict supersets:

* shapes come from the tensors, not from module constants, so any batch size
  and any number of KV heads (with 8 query heads each) work;
* ``dense_decode_attention`` accepts ``seq_len <= k.shape[2]`` (a cache with
  spare capacity) instead of requiring equality;
* ``sparse_decode_attention`` also reads a ring-buffer cache (``ring_head``)
  and per-sequence lengths (``seq_lens``).

Inputs must be contiguous float16 CUDA tensors with head_dim 128; anything
else raises ValueError / TypeError.  There is no CPU fallback.
"""
from __future__ import annotations

import torch

from . import _lib
from .constants import D_HEAD, SINK_SIZE


def _require(cond: bool, msg: str, exc=ValueError):
    if not cond:
        raise exc(msg)


def _check_fp16_cuda(name: str, t: torch.Tensor, ndim: int):
    _require(isinstance(t, torch.Tensor), f"{name} must be a torch.Tensor", TypeError)
    _require(t.is_cuda, f"{name} must be a CUDA tensor (no CPU fallback)")
    _require(t.dtype == torch.float16, f"{name} must be float16, got {t.dtype}", TypeError)
    _require(t.dim() == ndim, f"{name} must have {ndim} dims, got shape {tuple(t.shape)}")
    _require(t.is_contiguous(), f"{name} must be contiguous")


def _check_qkv(q, k, v):
    _check_fp16_cuda("q", q, 3)
    _check_fp16_cuda("k", k, 4)
    _check_fp16_cuda("v", v, 4)
    b, h, d = q.shape
    _require(k.shape == v.shape, f"k and v shapes differ: {tuple(k.shape)} vs {tuple(v.shape)}")
    _require(k.shape[0] == b and k.shape[3] == d, f"q {tuple(q.shape)} and k {tuple(k.shape)} disagree")
    _require(d == D_HEAD, f"head_dim must be {D_HEAD}, got {d}")
    _require(k.device == q.device and v.device == q.device, "q, k and v must be on the same device")
    return b, h, k.shape[1], d


def dense_decode_attention(q, k, v, seq_len, sm_scale=None):
    """Dense causal GQA decode (dense_kernel.py:70-82).

    q: [B, H, 128] fp16.  k/v: [B, H/8, L, 128] fp16, L >= seq_len.
    Attends cache slots [0, seq_len).  Returns o shaped and typed like q.
    """
    b, h, hkv, d = _check_qkv(q, k, v)
    seq_len = int(seq_len)
    if sm_scale is None:
        sm_scale = D_HEAD ** -0.5
    o = torch.empty_like(q)
    lib = _lib.load()
    ws_bytes = lib.nsa_dense_workspace_bytes(b, hkv, seq_len)
    with _lib.on_device(q.device):
        stream = _lib.stream_handle(q.device)
        ws = _lib.workspace(q.device, ws_bytes, stream)
        _lib.check(lib.nsa_dense_decode(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), b, h, hkv, d,
                                        k.shape[2], seq_len, float(sm_scale), ws.data_ptr(), ws.numel(), stream))
    return o


def _check_host(name, t, shape):
    _require(isinstance(t, torch.Tensor) and not t.is_cuda and t.dtype == torch.float16 and t.is_contiguous()
             and tuple(t.shape) == tuple(shape),
             f"{name} must be a contiguous float16 host tensor of shape {tuple(shape)} (pinned for overlap)")


def dense_decode_attention_host(pipe, q_host, o_host, k, v, seq_len, sm_scale=None):
    """dense_decode_attention with the query and the output in host memory
    (``pipe``: a _lib.HostPipe on k's device): copy in, decode and copy out
    are queued on the pipe's streams and the current stream; o_host holds the
    result once the stream passes ``pipe.end()``."""
    _check_fp16_cuda("k", k, 4)
    _check_fp16_cuda("v", v, 4)
    b, hkv, cache_len, d = k.shape
    _require(k.shape == v.shape and d == D_HEAD and v.device == k.device, "k and v must match, head_dim 128")
    _check_host("q_host", q_host, (b, 8 * hkv, d))
    _check_host("o_host", o_host, (b, 8 * hkv, d))
    seq_len = int(seq_len)
    lib = _lib.load()
    with _lib.on_device(k.device):
        stream = _lib.stream_handle(k.device)
        ws = _lib.workspace(k.device, lib.nsa_dense_workspace_bytes(b, hkv, seq_len), stream)
        _lib.check(lib.nsa_dense_decode_host(pipe.handle, q_host.data_ptr(), k.data_ptr(), v.data_ptr(),
                                             o_host.data_ptr(), b, 8 * hkv, hkv, d, cache_len, seq_len,
                                             float(D_HEAD ** -0.5 if sm_scale is None else sm_scale),
                                             ws.data_ptr(), ws.numel(), stream))


def sparse_decode_attention_host(pipe, q_host, o_host, k_cache, v_cache, seq_len, window, sink=SINK_SIZE,
                                 sm_scale=None, *, ring_head=None, seq_lens=None):
    """sparse_decode_attention with the query and the output in host memory
    (``pipe``: a _lib.HostPipe on the cache's device); ring_head / seq_lens as
    there (device tensors).  o_host holds the result once the stream passes
    ``pipe.end()``."""
    _check_fp16_cuda("k_cache", k_cache, 4)
    _check_fp16_cuda("v_cache", v_cache, 4)
    b, hkv, slots, d = k_cache.shape
    window, sink, seq_len = int(window), int(sink), int(seq_len)
    _require(k_cache.shape == v_cache.shape and d == D_HEAD and slots == sink + window,
             "k_cache / v_cache must be [B, Hkv, sink+window, 128] and match")
    _check_host("q_host", q_host, (b, 8 * hkv, d))
    _check_host("o_host", o_host, (b, 8 * hkv, d))
    heads_ptr = lens_ptr = None
    if ring_head is not None:
        _require(isinstance(ring_head, torch.Tensor) and ring_head.dtype == torch.int32 and ring_head.is_cuda
                 and ring_head.numel() == b, "ring_head must be an int32 CUDA tensor of length B")
        heads_ptr = ring_head.data_ptr()
    if seq_lens is not None:
        _require(isinstance(seq_lens, torch.Tensor) and seq_lens.dtype == torch.int64 and seq_lens.is_cuda
                 and seq_lens.numel() == b, "seq_lens must be an int64 CUDA tensor of length B")
        lens_ptr = seq_lens.data_ptr()
    lib = _lib.load()
    with _lib.on_device(k_cache.device):
        stream = _lib.stream_handle(k_cache.device)
        ws = _lib.workspace(k_cache.device, lib.nsa_sparse_workspace_bytes(b, hkv, window, sink), stream)
        _lib.check(lib.nsa_sparse_decode_host(pipe.handle, q_host.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                                              o_host.data_ptr(), b, 8 * hkv, hkv, d, window, sink, seq_len, lens_ptr,
                                              heads_ptr, float(D_HEAD ** -0.5 if sm_scale is None else sm_scale),
                                              ws.data_ptr(), ws.numel(), stream))


def sparse_decode_attention(q, k_cache, v_cache, seq_len, window, sink=SINK_SIZE, sm_scale=None, *,
                            ring_head=None, seq_lens=None):
    """StreamingLLM sink + sliding-window decode (sparse_kernel.py:105-118).

    k_cache/v_cache: [B, H/8, sink+window, 128] fp16.  With ``ring_head``
    None the cache is the reference's compacted layout (slot sink+i holds
    position seq_len-window+i); an int or an int32 [B] CUDA tensor selects the
    ring layout (position p >= sink at slot sink + (p-sink) % window, head =
    (seq_len-sink) % window).  ``seq_lens`` (int64 [B] CUDA) overrides
    ``seq_len`` per sequence.
    """
    b, h, hkv, d = _check_qkv(q, k_cache, v_cache)
    window, sink, seq_len = int(window), int(sink), int(seq_len)
    _require(k_cache.shape[2] == sink + window,
             f"k_cache must hold sink+window = {sink + window} slots, got {k_cache.shape[2]}")
    if sm_scale is None:
        sm_scale = D_HEAD ** -0.5
    heads_ptr = 0
    heads = None
    if ring_head is not None:
        if isinstance(ring_head, torch.Tensor):
            heads = ring_head
        else:
            heads = torch.full((b,), int(ring_head), dtype=torch.int32, device=q.device)
        _require(heads.dtype == torch.int32 and heads.is_cuda and heads.numel() == b and heads.is_contiguous(),
                 "ring_head tensor must be a contiguous int32 CUDA tensor of length B")
        heads_ptr = heads.data_ptr()
    lens_ptr = 0
    if seq_lens is not None:
        _require(isinstance(seq_lens, torch.Tensor) and seq_lens.dtype == torch.int64 and seq_lens.is_cuda
                 and seq_lens.numel() == b and seq_lens.is_contiguous(),
                 "seq_lens must be a contiguous int64 CUDA tensor of length B")
        lens_ptr = seq_lens.data_ptr()
    o = torch.empty_like(q)
    lib = _lib.load()
    ws_bytes = lib.nsa_sparse_workspace_bytes(b, hkv, window, sink)
    with _lib.on_device(q.device):
        stream = _lib.stream_handle(q.device)
        ws = _lib.workspace(q.device, ws_bytes, stream)
        _lib.check(lib.nsa_sparse_decode(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), o.data_ptr(), b, h,
                                         hkv, d, window, sink, seq_len, lens_ptr or None, heads_ptr or None,
                                         float(sm_scale), ws.data_ptr(), ws.numel(), stream))
    return o


class RingCache:
    """fp16 sink + sliding-window KV cache managed on the device (no reference
    counterpart: the reference rebuilds a compacted cache on the host,
    test_sparse_correctness.py:51-72).

    k/v: [B, Hkv, sink + window, 128] fp16; unit_lens: int64 [B*Hkv], the
    tokens appended per (batch row, kv head).  Position p < sink lives in slot
    p, position p >= sink in slot sink + (p - sink) % window (dropped when
    window is 0): the ring layout of ``sparse_decode_attention`` with head
    (len - sink) % window, whose attended set this cache reproduces exactly.
    ``decode_step`` appends one token per unit and attends in one launch when
    every unit gets its own CTA (see nsa_ring_decode_step)."""

    def __init__(self, batch, n_kv_heads, window, sink=SINK_SIZE, device=None):
        self.batch, self.n_kv_heads, self.window, self.sink = int(batch), int(n_kv_heads), int(window), int(sink)
        _require(self.batch >= 0 and self.n_kv_heads > 0 and self.window >= 0 and self.sink >= 0
                 and self.window + self.sink >= 1, "need batch >= 0, n_kv_heads > 0, window, sink >= 0")
        self.device = torch.device(device if device is not None else "cuda")
        _require(self.device.type == "cuda", "RingCache lives on a CUDA device (no CPU fallback)")
        shape = (self.batch, self.n_kv_heads, self.sink + self.window, D_HEAD)
        self.k = torch.zeros(shape, dtype=torch.float16, device=self.device)
        self.v = torch.zeros(shape, dtype=torch.float16, device=self.device)
        self.unit_lens = torch.zeros(self.batch * self.n_kv_heads, dtype=torch.int64, device=self.device)
        self._ws_bytes = _lib.load().nsa_sparse_workspace_bytes(self.batch, self.n_kv_heads, self.window, self.sink)

    def _check_token(self, new_k, new_v):
        for name, t in (("new_k", new_k), ("new_v", new_v)):
            _check_fp16_cuda(name, t, 3)
            _require(tuple(t.shape) == (self.batch, self.n_kv_heads, D_HEAD),
                     f"{name} must be [B, Hkv, {D_HEAD}], got {tuple(t.shape)}")

    def _check_q(self, q):
        _check_fp16_cuda("q", q, 3)
        _require(tuple(q.shape) == (self.batch, 8 * self.n_kv_heads, D_HEAD),
                 f"q must be [B, 8*Hkv, {D_HEAD}], got {tuple(q.shape)}")

    def append(self, new_k, new_v):
        """Store one token per (batch row, kv head): new_k/new_v [B, Hkv, 128] fp16."""
        self._check_token(new_k, new_v)
        with torch.cuda.device(self.device):
            _lib.check(_lib.load().nsa_ring_append(
                self.k.data_ptr(), self.v.data_ptr(), self.unit_lens.data_ptr(), new_k.data_ptr(), new_v.data_ptr(),
                self.batch, self.n_kv_heads, D_HEAD, self.window, self.sink, _lib.stream_handle(self.device)))

    def attend(self, q, sm_scale=None):
        """Decode q [B, 8*Hkv, 128] fp16 against the cache -> o like q."""
        self._check_q(q)
        o = torch.empty_like(q)
        with torch.cuda.device(self.device):
            ws = _lib.workspace(self.device, self._ws_bytes)
            _lib.check(_lib.load().nsa_ring_decode(
                q.data_ptr(), self.k.data_ptr(), self.v.data_ptr(), o.data_ptr(), self.batch, 8 * self.n_kv_heads,
                self.n_kv_heads, D_HEAD, self.window, self.sink, self.unit_lens.data_ptr(),
                float(D_HEAD ** -0.5 if sm_scale is None else sm_scale), ws.data_ptr(), ws.numel(),
                _lib.stream_handle(self.device)))
        return o

    def decode_step(self, q, new_k, new_v, sm_scale=None):
        """Append new_k/new_v, then attend q (one launch when possible)."""
        self._check_token(new_k, new_v)
        self._check_q(q)
        o = torch.empty_like(q)
        with torch.cuda.device(self.device):
            ws = _lib.workspace(self.device, self._ws_bytes)
            _lib.check(_lib.load().nsa_ring_decode_step(
                q.data_ptr(), self.k.data_ptr(), self.v.data_ptr(), o.data_ptr(), self.batch, 8 * self.n_kv_heads,
                self.n_kv_heads, D_HEAD, self.window, self.sink, self.unit_lens.data_ptr(), new_k.data_ptr(),
                new_v.data_ptr(), float(D_HEAD ** -0.5 if sm_scale is None else sm_scale), ws.data_ptr(),
                ws.numel(), _lib.stream_handle(self.device)))
        return o

    def load_history(self, k_hist, v_hist, seq_len):
        """Set the cache to its state after appending positions [0, seq_len) of
        k_hist/v_hist [B, Hkv, >= seq_len, 128] fp16 (one gather, no per-token
        launches)."""
        _check_fp16_cuda("k_hist", k_hist, 4)
        _check_fp16_cuda("v_hist", v_hist, 4)
        L, S, W = int(seq_len), self.sink, self.window
        _require(k_hist.shape[2] >= L, "history shorter than seq_len")
        self.unit_lens.fill_(L)
        ns = min(L, S)
        self.k[:, :, :ns] = k_hist[:, :, :ns]
        self.v[:, :, :ns] = v_hist[:, :, :ns]
        if W > 0 and L > S:
            pos = torch.arange(max(S, L - W), L, device=self.device)
            slots = S + (pos - S) % W
            self.k[:, :, slots] = k_hist[:, :, pos]
            self.v[:, :, slots] = v_hist[:, :, pos]

    def ring_head(self) -> int:
        """Ring head of a cache whose units all hold the same length."""
        L = int(self.unit_lens[0].item())
        return (L - self.sink) % self.window if (self.window > 0 and L > self.sink) else 0
