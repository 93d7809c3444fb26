"""Host side of the KIVI 2-bit paths.

Reference-shaped entry points (same names, arguments and return values as
quant_kernel.py): ``quantize_k_cache``, ``quantize_v_cache``,
``build_quantized_kv_cache``, ``sparse_decode_attention_quantized``, plus
host-callable ``dequantize_k`` / ``dequantize_v`` (the reference's
``_dequantize_k_tile`` / ``_dequantize_v_tile`` are Triton-only helpers).

``KiviCache`` is the streaming cache the reference lacks: one new token per
sequence per step is appended and quantized on the GPU (quantize-on-append),
then attention reads sink + quantized window + fp16 residual.  Its layout and
semantics are documented with ``nsa_kivi_stream_cache`` in include/nsa_b200.h.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .constants import D_HEAD, GROUP_SIZE, QUANT_BITS, RESIDUAL_SIZE, SINK_SIZE


def _req(cond, msg, exc=ValueError):
    if not cond:
        raise exc(msg)


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return 0
    if t.dtype == torch.float16:
        return 1
    raise TypeError(f"quantizer input must be float32 or float16, got {t.dtype}")


def _check_cuda4(name, t):
    _req(isinstance(t, torch.Tensor), f"{name} must be a torch.Tensor", TypeError)
    _req(t.is_cuda, f"{name} must be a CUDA tensor (no CPU fallback)")
    _req(t.dim() == 4, f"{name} must be [batch, kv_heads, seq, head_dim], got {tuple(t.shape)}")


def quantize_k_cache(k, group_size=GROUP_SIZE, bits=QUANT_BITS):
    """quant_kernel.py:106-126.  k: [B, Hkv, T, D] float32 (or float16),
    T % group_size == 0.  Returns (packed u8 [B,Hkv,T/4,D], scale f16
    [B,Hkv,T/G,D], zero_point f16 [B,Hkv,T/G,D]), bit-exact with the reference."""
    _check_cuda4("k", k)
    b, h, t, d = k.shape
    # the reference asserts this (quant_kernel.py:110)
    assert t % group_size == 0, "this simple version assumes seq_len is a multiple of group_size"
    k = k.contiguous()
    packed = torch.empty((b, h, t // 4, d), dtype=torch.uint8, device=k.device)
    scale = torch.empty((b, h, t // group_size, d), dtype=torch.float16, device=k.device)
    zero = torch.empty_like(scale)
    with torch.cuda.device(k.device):
        _lib.check(_lib.load().nsa_kivi_quantize_k(k.data_ptr(), _dtype_code(k), packed.data_ptr(), scale.data_ptr(),
                                                   zero.data_ptr(), b, h, t, d, group_size, bits,
                                                   _lib.stream_handle(k.device)))
    return packed, scale, zero


def quantize_v_cache(v, group_size=GROUP_SIZE, bits=QUANT_BITS):
    """quant_kernel.py:193-214.  v: [B, Hkv, T, D] float32 (or float16),
    D % group_size == 0.  Returns (packed u8 [B,Hkv,T,D/4], scale f16
    [B,Hkv,T,D/G], zero_point f16 [B,Hkv,T,D/G]), bit-exact with the reference."""
    _check_cuda4("v", v)
    b, h, t, d = v.shape
    assert d % group_size == 0, "this simple version assumes D_HEAD is a multiple of group_size"
    v = v.contiguous()
    packed = torch.empty((b, h, t, d // 4), dtype=torch.uint8, device=v.device)
    scale = torch.empty((b, h, t, d // group_size), dtype=torch.float16, device=v.device)
    zero = torch.empty_like(scale)
    with torch.cuda.device(v.device):
        _lib.check(_lib.load().nsa_kivi_quantize_v(v.data_ptr(), _dtype_code(v), packed.data_ptr(), scale.data_ptr(),
                                                   zero.data_ptr(), b, h, t, d, group_size, bits,
                                                   _lib.stream_handle(v.device)))
    return packed, scale, zero


def dequantize_k(packed, scale, zero_point, seq_len, tok_start=0, n_tokens=None):
    """Dequantize K tokens [tok_start, tok_start + n_tokens) (positions clamped
    to [0, seq_len)) -> float32 [B, Hkv, n_tokens, D]: ``s * (code - z)``."""
    b, h, _, d = packed.shape
    n = seq_len - tok_start if n_tokens is None else n_tokens
    out = torch.empty((b, h, n, d), dtype=torch.float32, device=packed.device)
    with torch.cuda.device(packed.device):
        _lib.check(_lib.load().nsa_kivi_dequant_k(packed.contiguous().data_ptr(), scale.contiguous().data_ptr(),
                                                  zero_point.contiguous().data_ptr(), out.data_ptr(), b, h, seq_len, d,
                                                  tok_start, n, _lib.stream_handle(packed.device)))
    return out


def dequantize_v(packed, scale, zero_point, seq_len=None, tok_start=0, n_tokens=None):
    """Dequantize V tokens [tok_start, tok_start + n_tokens) -> float32 [B, Hkv, n, D]."""
    b, h, t, dp = packed.shape
    seq_len = t if seq_len is None else seq_len
    n = seq_len - tok_start if n_tokens is None else n_tokens
    out = torch.empty((b, h, n, dp * 4), dtype=torch.float32, device=packed.device)
    with torch.cuda.device(packed.device):
        _lib.check(_lib.load().nsa_kivi_dequant_v(packed.contiguous().data_ptr(), scale.contiguous().data_ptr(),
                                                  zero_point.contiguous().data_ptr(), out.data_ptr(), b, h, seq_len,
                                                  dp * 4, tok_start, n, _lib.stream_handle(packed.device)))
    return out


def build_quantized_kv_cache(k_compacted, v_compacted, residual_size=RESIDUAL_SIZE, sink=SINK_SIZE):
    """quant_kernel.py:584-622: slice a compacted [B, Hkv, S+W, D] cache into
    the fp16 residual (last ``residual_size`` slots), the sink padded to one
    group by repeating slot 0, and window-old [S, S+W-R); quantize the last two
    on the GPU.  Returns the reference's 14-key dict."""
    _check_cuda4("k_compacted", k_compacted)
    n = k_compacted.shape[2]
    win_end = n - residual_size
    out = {
        "k_residual": k_compacted[:, :, win_end:, :].contiguous(),
        "v_residual": v_compacted[:, :, win_end:, :].contiguous(),
    }
    pad = GROUP_SIZE - sink

    def _pad(x):
        real = x[:, :, :sink, :]
        return torch.cat([real, real[:, :, :1, :].expand(-1, -1, pad, -1)], dim=2).contiguous()

    out["k_sink_packed"], out["k_sink_scale"], out["k_sink_zero"] = quantize_k_cache(_pad(k_compacted))
    out["v_sink_packed"], out["v_sink_scale"], out["v_sink_zero"] = quantize_v_cache(_pad(v_compacted))
    kw = k_compacted[:, :, sink:win_end, :].contiguous()
    vw = v_compacted[:, :, sink:win_end, :].contiguous()
    out["k_win_packed"], out["k_win_scale"], out["k_win_zero"] = quantize_k_cache(kw)
    out["v_win_packed"], out["v_win_scale"], out["v_win_zero"] = quantize_v_cache(vw)
    return out


_KIVI_ORDER = ["k_sink_packed", "k_sink_scale", "k_sink_zero", "v_sink_packed", "v_sink_scale", "v_sink_zero",
               "k_win_packed", "k_win_scale", "k_win_zero", "v_win_packed", "v_win_scale", "v_win_zero"]


def sparse_decode_attention_quantized(q, k_cache, v_cache,
                                      k_sink_packed, k_sink_scale, k_sink_zero,
                                      v_sink_packed, v_sink_scale, v_sink_zero,
                                      k_win_packed, k_win_scale, k_win_zero,
                                      v_win_packed, v_win_scale, v_win_zero,
                                      seq_len, window, sink=SINK_SIZE, residual_size=RESIDUAL_SIZE,
                                      group_size=GROUP_SIZE, bits=QUANT_BITS, sm_scale=None):
    """quant_kernel.py:551-581.  k_cache/v_cache are the fp16 RESIDUAL
    [B, Hkv, residual_size, D]; the other 12 tensors as built by
    build_quantized_kv_cache.  Requires window >= residual_size."""
    _req(isinstance(q, torch.Tensor) and q.is_cuda, "q must be a CUDA tensor (no CPU fallback)")
    _req(q.dtype == torch.float16, f"q must be float16, got {q.dtype}", TypeError)
    _req(q.dim() == 3 and q.is_contiguous(), "q must be a contiguous [B, H, D] tensor")
    b, h, d = q.shape
    _req(d == D_HEAD, f"head_dim must be {D_HEAD}")
    _req(k_cache.dtype == torch.float16 and v_cache.dtype == torch.float16, "residual caches must be float16",
         TypeError)
    hkv = k_cache.shape[1]
    _req(tuple(k_cache.shape) == (b, hkv, residual_size, d) and v_cache.shape == k_cache.shape,
         f"k_cache/v_cache must be [B, Hkv, residual_size={residual_size}, D]")
    window, sink, seq_len = int(window), int(sink), int(seq_len)
    tensors = [k_sink_packed, k_sink_scale, k_sink_zero, v_sink_packed, v_sink_scale, v_sink_zero,
               k_win_packed, k_win_scale, k_win_zero, v_win_packed, v_win_scale, v_win_zero]
    nw = window - residual_size
    expect = [(b, hkv, GROUP_SIZE // 4, d), (b, hkv, 1, d), (b, hkv, 1, d),
              (b, hkv, GROUP_SIZE, d // 4), (b, hkv, GROUP_SIZE, d // GROUP_SIZE), (b, hkv, GROUP_SIZE, d // GROUP_SIZE),
              (b, hkv, max(nw, 0) // 4, d), (b, hkv, max(nw, 0) // GROUP_SIZE, d), (b, hkv, max(nw, 0) // GROUP_SIZE, d),
              (b, hkv, max(nw, 0), d // 4), (b, hkv, max(nw, 0), d // GROUP_SIZE),
              (b, hkv, max(nw, 0), d // GROUP_SIZE)]
    for name, t, shp in zip(_KIVI_ORDER, tensors, expect):
        _req(isinstance(t, torch.Tensor) and t.is_cuda and t.is_contiguous(), f"{name} must be a contiguous CUDA tensor")
        _req(tuple(t.shape) == shp, f"{name} must have shape {shp}, got {tuple(t.shape)}")
        _req(t.dtype == (torch.uint8 if name.endswith("packed") else torch.float16), f"{name} has wrong dtype {t.dtype}",
             TypeError)
    if sm_scale is None:
        sm_scale = D_HEAD ** -0.5
    o = torch.empty_like(q)
    lib = _lib.load()
    ws_bytes = lib.nsa_kivi_workspace_bytes(b, hkv, window, residual_size)
    with torch.cuda.device(q.device):
        ws = _lib.workspace(q.device, ws_bytes)
        ptrs = [t.data_ptr() if t.numel() else None for t in tensors]
        _lib.check(lib.nsa_kivi_decode(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), *ptrs, o.data_ptr(),
                                       b, h, hkv, d, seq_len, window, sink, residual_size, group_size, bits,
                                       float(sm_scale), ws.data_ptr(), ws.numel(), _lib.stream_handle(q.device)))
    return o


# --------------------------------------------------------------------------
# streaming cache
# --------------------------------------------------------------------------

class KiviStreamCacheDesc(ctypes.Structure):
    """ctypes mirror of nsa_kivi_stream_cache (include/nsa_b200.h)."""
    _fields_ = [(n, ctypes.c_int64) for n in ("batch", "n_kv_heads", "head_dim", "window", "sink", "residual",
                                              "n_groups")] + \
               [(n, ctypes.c_void_p) for n in ("unit_lens", "sink_k", "sink_v", "groups", "k_res", "v_res")]


# Group records of the streaming cache (csrc/kivi_format.cuh): one group's
# share of the reference's six quantized tensors, 3 KiB.
REC_BYTES = 3072
_QUANT_NAMES = ("k_{}_packed", "k_{}_scale", "k_{}_zero", "v_{}_packed", "v_{}_scale", "v_{}_zero")


def _record(kp, ks, kz, vp, vs, vz):
    """Records u8 [..., 3072] from one group's tensors in the reference layouts
    (kp u8 [..., 8, D], ks / kz f16 [..., 1, D], vp u8 [..., 32, D/4],
    vs / vz f16 [..., 32, D/32])."""
    lead = kp.shape[:-2]
    return torch.cat([t.contiguous().view(torch.uint8).reshape(*lead, -1) for t in (kp, ks, kz, vp, vs, vz)], dim=-1)


def _unrecord(rec):
    """Records u8 [..., n, 3072] -> the six tensors in the reference layouts,
    the n groups one after another along the token axis (copies)."""
    lead, n = rec.shape[:-2], rec.shape[-2]

    def f16(a, b, rows, cols):
        return rec[..., a:b].contiguous().view(torch.float16).reshape(*lead, rows, cols)

    return (rec[..., 0:1024].reshape(*lead, n * 8, D_HEAD), f16(1024, 1280, n, D_HEAD), f16(1280, 1536, n, D_HEAD),
            rec[..., 1536:2560].reshape(*lead, n * GROUP_SIZE, D_HEAD // 4),
            f16(2560, 2816, n * GROUP_SIZE, D_HEAD // 32), f16(2816, 3072, n * GROUP_SIZE, D_HEAD // 32))


def _res_perm(n_slots, device):
    """[n_slots, D] element order of the residual ring: slot s stores channel
    c at perm[s, c], and perm[s] is its own inverse (16-byte chunk ch of the
    row sits at chunk (ch & 8) | ((ch & 7) ^ (s & 7)))."""
    s = torch.arange(n_slots, device=device)[:, None]
    c = torch.arange(D_HEAD, device=device)[None, :]
    ch = c >> 3
    return (((ch & 8) | ((ch & 7) ^ (s & 7))) << 3) | (c & 7)


def decode_step_layers(caches, qs, new_ks, new_vs, sm_scale=None):
    """KiviCache.decode_step for several layers' caches (one geometry) at once:
    returns the list of outputs.  Up to 64 layers share one kernel launch
    (nsa_kivi_stream_decode_step_layers) when the step fits one launch per layer."""
    n = len(caches)
    _req(len(qs) == n and len(new_ks) == n and len(new_vs) == n, "one q, new_k and new_v per cache")
    if n == 0:
        return []
    c0 = caches[0]
    for c, q, nk, nv in zip(caches, qs, new_ks, new_vs):
        _req(isinstance(c, KiviCache) and c.device == c0.device, "caches must be KiviCaches on one device")
        for name, t, shape in (("q", q, (c.batch, 8 * c.n_kv_heads, c.head_dim)),
                               ("new_k", nk, (c.batch, c.n_kv_heads, c.head_dim)),
                               ("new_v", nv, (c.batch, c.n_kv_heads, c.head_dim))):
            _req(isinstance(t, torch.Tensor) and t.is_cuda and t.dtype == torch.float16 and t.is_contiguous()
                 and tuple(t.shape) == shape, f"{name} must be a contiguous float16 CUDA tensor of shape {shape}")
    if sm_scale is None:
        sm_scale = c0.head_dim ** -0.5
    outs = [torch.empty_like(q) for q in qs]
    descs = (KiviStreamCacheDesc * n)(*[c._desc for c in caches])
    ptrs = lambda ts: (ctypes.c_void_p * n)(*[t.data_ptr() for t in ts])  # noqa: E731
    with torch.cuda.device(c0.device):
        ws = _lib.workspace(c0.device, c0._ws_bytes)
        _lib.check(_lib.load().nsa_kivi_stream_decode_step_layers(
            descs, n, ptrs(new_ks), ptrs(new_vs), ptrs(qs), ptrs(outs), float(sm_scale), ws.data_ptr(), ws.numel(),
            _lib.stream_handle(c0.device)))
    return outs


class KiviCache:
    """Streaming KIVI cache for one attention layer (see nsa_kivi_stream_cache).

    Usage per decode step:  ``o = cache.decode_step(q, new_k, new_v)``
    (append then attend), or ``cache.append(new_k, new_v)`` / ``cache.attend(q)``.
    """

    def __init__(self, batch, n_kv_heads, window, sink=SINK_SIZE, residual=RESIDUAL_SIZE, head_dim=D_HEAD,
                 device=None):
        _req(head_dim == D_HEAD, f"head_dim must be {D_HEAD}")
        _req(1 <= sink <= GROUP_SIZE, "sink must be in [1, 32]")
        _req(residual >= GROUP_SIZE and residual % GROUP_SIZE == 0, "residual must be a positive multiple of 32")
        _req(window >= 0 and (window < residual or (window - residual) % GROUP_SIZE == 0),
             "window - residual must be a multiple of 32")
        device = torch.device(device if device is not None else "cuda")
        _req(device.type == "cuda", "KiviCache lives on a CUDA device")
        self.batch, self.n_kv_heads, self.window, self.sink, self.residual = batch, n_kv_heads, window, sink, residual
        self.head_dim = head_dim
        self.n_groups = (window - residual) // GROUP_SIZE if window >= residual else 0
        self.res_cap = residual + GROUP_SIZE
        self.device = device
        b, h, d, ng = batch, n_kv_heads, head_dim, self.n_groups
        f16, u8 = torch.float16, torch.uint8

        def z(shape, dt):
            return torch.zeros(shape, dtype=dt, device=device)

        self.unit_lens = z((b, h), torch.int64)
        self.sink_k, self.sink_v = z((b, h, sink, d), f16), z((b, h, sink, d), f16)
        # record 0: the sink group; record 1 + s: window-group slot s
        self.groups = z((b, h, 1 + ng, REC_BYTES), u8)
        # residual ring, slots chunk-permuted (_res_perm)
        self.k_res, self.v_res = z((b, h, self.res_cap, d), f16), z((b, h, self.res_cap, d), f16)
        self._perm = _res_perm(self.res_cap, device)
        self._desc = self._make_desc()
        lib = _lib.load()
        self._ws_bytes = lib.nsa_kivi_stream_workspace_bytes(ctypes.byref(self._desc))

    # ---------------------------------------------------------------- plumbing
    def _make_desc(self):
        dsc = KiviStreamCacheDesc()
        for n in ("batch", "n_kv_heads", "head_dim", "window", "sink", "residual", "n_groups"):
            setattr(dsc, n, int(getattr(self, n)))
        for n in ("unit_lens", "sink_k", "sink_v", "groups", "k_res", "v_res"):
            setattr(dsc, n, getattr(self, n).data_ptr())
        return dsc

    def _logical_rows(self, t):
        """Residual ring in channel order (copy)."""
        return t.gather(-1, self._perm.expand_as(t))

    def state(self) -> dict:
        """The cache in the reference's tensor layouts (copies): unit_lens,
        sink_k / sink_v, k_/v_{sink,win}_{packed,scale,zero} as
        build_quantized_kv_cache lays them out (window groups in slot order),
        and k_res / v_res [B, Hkv, R + 32, D] in channel order."""
        st = {"unit_lens": self.unit_lens.clone(), "sink_k": self.sink_k.clone(), "sink_v": self.sink_v.clone()}
        for where, recs in (("sink", self.groups[:, :, :1]), ("win", self.groups[:, :, 1:])):
            for name, t in zip(_QUANT_NAMES, _unrecord(recs)):
                st[name.format(where)] = t
        st["k_res"], st["v_res"] = self._logical_rows(self.k_res), self._logical_rows(self.v_res)
        return st

    @property
    def seq_len(self) -> int:
        return int(self.unit_lens[0, 0].item())

    # ---------------------------------------------------------------- steps
    def append(self, new_k, new_v):
        """Append one token per sequence: new_k/new_v [B, Hkv, D] float16."""
        shape = (self.batch, self.n_kv_heads, self.head_dim)
        for name, t in (("new_k", new_k), ("new_v", new_v)):
            _req(isinstance(t, torch.Tensor) and t.is_cuda and t.dtype == torch.float16 and t.is_contiguous()
                 and tuple(t.shape) == shape, f"{name} must be a contiguous float16 CUDA tensor of shape {shape}")
        with torch.cuda.device(self.device):
            _lib.check(_lib.load().nsa_kivi_append(ctypes.byref(self._desc), new_k.data_ptr(), new_v.data_ptr(),
                                                   _lib.stream_handle(self.device)))

    def attend(self, q, sm_scale=None):
        """Decode q [B, 8*Hkv, D] float16 against the cache -> o like q."""
        _req(isinstance(q, torch.Tensor) and q.is_cuda and q.dtype == torch.float16 and q.is_contiguous()
             and tuple(q.shape) == (self.batch, 8 * self.n_kv_heads, self.head_dim),
             "q must be a contiguous float16 CUDA tensor [B, 8*Hkv, 128]")
        if sm_scale is None:
            sm_scale = self.head_dim ** -0.5
        o = torch.empty_like(q)
        with torch.cuda.device(self.device):
            ws = _lib.workspace(self.device, self._ws_bytes)
            _lib.check(_lib.load().nsa_kivi_stream_decode(ctypes.byref(self._desc), q.data_ptr(), o.data_ptr(),
                                                          float(sm_scale), ws.data_ptr(), ws.numel(),
                                                          _lib.stream_handle(self.device)))
        return o

    def step_launches(self) -> int:
        """Kernel launches of one decode_step, as the library plans it on this
        cache's device: 1 when every unit is decoded by its own CTA (more units
        than half the CTA slots, or units whose groups and residual all fit the
        kernel's stages), else 2."""
        with torch.cuda.device(self.device):
            return int(_lib.load().nsa_kivi_stream_step_launches(ctypes.byref(self._desc)))

    def decode_step(self, q, new_k, new_v, sm_scale=None, out=None):
        """One decode step: quantize-on-append of the new token, then attend
        (one launch when every unit gets its own CTA, else append + attend).
        ``out`` (optional): preallocated output like q."""
        shape = (self.batch, self.n_kv_heads, self.head_dim)
        for name, t in (("new_k", new_k), ("new_v", new_v)):
            _req(isinstance(t, torch.Tensor) and t.is_cuda and t.dtype == torch.float16 and t.is_contiguous()
                 and tuple(t.shape) == shape, f"{name} must be a contiguous float16 CUDA tensor of shape {shape}")
        _req(isinstance(q, torch.Tensor) and q.is_cuda and q.dtype == torch.float16 and q.is_contiguous()
             and tuple(q.shape) == (self.batch, 8 * self.n_kv_heads, self.head_dim),
             "q must be a contiguous float16 CUDA tensor [B, 8*Hkv, 128]")
        if out is None:
            out = torch.empty_like(q)
        else:
            _req(isinstance(out, torch.Tensor) and out.is_cuda and out.dtype == torch.float16
                 and out.is_contiguous() and out.shape == q.shape, "out must be a contiguous float16 CUDA tensor like q")
        if sm_scale is None:
            sm_scale = self.head_dim ** -0.5
        with _lib.on_device(self.device):
            stream = _lib.stream_handle(self.device)
            ws = _lib.workspace(self.device, self._ws_bytes, stream)
            _lib.check(_lib.load().nsa_kivi_stream_decode_step(
                ctypes.byref(self._desc), new_k.data_ptr(), new_v.data_ptr(), q.data_ptr(), out.data_ptr(),
                float(sm_scale), ws.data_ptr(), ws.numel(), stream))
        return out

    def decode_step_host(self, pipe, x_host, o_host, sm_scale=None):
        """decode_step with its inputs and output in host memory: x_host =
        [q | new_k | new_v] packed (float16, B*8*Hkv*D + 2*B*Hkv*D elements),
        o_host like q.  ``pipe``: a _lib.HostPipe on the cache's device; the
        copies overlap other calls' decode, and o_host holds the result once
        the stream passes ``pipe.end()``."""
        n_q = self.batch * 8 * self.n_kv_heads * self.head_dim
        n_x = n_q + 2 * self.batch * self.n_kv_heads * self.head_dim
        for name, t, n in (("x_host", x_host, n_x), ("o_host", o_host, n_q)):
            _req(isinstance(t, torch.Tensor) and not t.is_cuda and t.dtype == torch.float16 and t.is_contiguous()
                 and t.numel() == n, f"{name} must be a contiguous float16 host tensor of {n} elements")
        with _lib.on_device(self.device):
            stream = _lib.stream_handle(self.device)
            ws = _lib.workspace(self.device, self._ws_bytes, stream)
            _lib.check(_lib.load().nsa_kivi_stream_decode_step_host(
                pipe.handle, ctypes.byref(self._desc), x_host.data_ptr(), o_host.data_ptr(),
                float(self.head_dim ** -0.5 if sm_scale is None else sm_scale), ws.data_ptr(), ws.numel(), stream))

    # ---------------------------------------------------------------- filling
    def load_state(self, seq_len, sink_k, sink_v, tail_k=None, tail_v=None, tail_start=None):
        """Set the cache to its state after ``seq_len`` appends.

        sink_k/sink_v: [B, Hkv, min(seq_len, sink), D] float16, positions
        [0, min(seq_len, sink)).  tail_k/tail_v: [B, Hkv, n, D] float16 holding
        positions [tail_start, tail_start + n), tail_start >= sink, covering
        every stream position the state keeps (live window groups and the
        residual).  Uses the GPU quantizers of the append path, so the result
        equals appending the same tokens one by one."""
        S, G, R, NG, C = self.sink, GROUP_SIZE, self.residual, self.n_groups, self.res_cap
        n_stream = max(0, seq_len - S)
        F = max(0, (n_stream - R) // G)
        n_grp = min(F, NG)
        ns = min(seq_len, S)
        self.unit_lens.fill_(seq_len)
        for t in (self.k_res, self.v_res, self.sink_k, self.sink_v):
            t.zero_()
        if ns:
            _req(sink_k.shape[2] >= ns, f"sink_k must hold {ns} tokens")
            kk, vv = sink_k[:, :, :ns], sink_v[:, :, :ns]
            self.sink_k[:, :, :ns] = kk
            self.sink_v[:, :, :ns] = vv
            kp = torch.cat([kk, kk[:, :, :1].expand(-1, -1, G - ns, -1)], dim=2).contiguous()
            vp = torch.cat([vv, vv[:, :, :1].expand(-1, -1, G - ns, -1)], dim=2).contiguous()
            self.groups[:, :, 0] = _record(*quantize_k_cache(kp), *quantize_v_cache(vp))

        def tok(a, b):
            _req(tail_k is not None and a >= tail_start and b <= tail_start + tail_k.shape[2],
                 f"tail must cover positions [{a}, {b})")
            return tail_k[:, :, a - tail_start:b - tail_start], tail_v[:, :, a - tail_start:b - tail_start]

        if n_grp:
            g0 = F - n_grp
            kk, vv = tok(S + G * g0, S + G * F)
            kp, ks, kz = quantize_k_cache(kk.contiguous())
            vp, vs, vz = quantize_v_cache(vv.contiguous())
            for j in range(n_grp):
                slot = (g0 + j) % NG
                t, v = slice(j * G, (j + 1) * G), slice(j, j + 1)
                self.groups[:, :, 1 + slot] = _record(kp[:, :, j * 8:(j + 1) * 8], ks[:, :, v], kz[:, :, v],
                                                      vp[:, :, t], vs[:, :, t], vz[:, :, t])
        if n_stream > G * F:
            kk, vv = tok(S + G * F, seq_len)
            idx = torch.arange(G * F, n_stream, device=self.device) % C
            perm = self._perm[idx].expand_as(kk)
            self.k_res[:, :, idx] = kk.gather(-1, perm)
            self.v_res[:, :, idx] = vv.gather(-1, perm)

    def load_history(self, k_hist, v_hist, seq_len):
        """State after appending positions [0, seq_len) of k_hist/v_hist
        ([B, Hkv, >= seq_len, D] float16)."""
        S = self.sink
        self.load_state(seq_len, k_hist[:, :, :S], v_hist[:, :, :S], k_hist[:, :, S:seq_len], v_hist[:, :, S:seq_len],
                        tail_start=S)

    def kept_positions(self, seq_len):
        """Oldest stream position the state after ``seq_len`` appends keeps."""
        S, G, R, NG = self.sink, GROUP_SIZE, self.residual, self.n_groups
        n_stream = max(0, seq_len - S)
        F = max(0, (n_stream - R) // G)
        return S + G * (F - min(F, NG))

    @classmethod
    def synthetic(cls, batch, n_kv_heads, window, seq_len, sink=SINK_SIZE, residual=RESIDUAL_SIZE, device=None,
                  generator=None, outlier_channels=4, outlier_factor=8.0):
        """A cache in its state after ``seq_len`` appends of seeded N(0,1) fp16
        tokens (K with ``outlier_channels`` of the 128 channels scaled by
        ``outlier_factor``); only the positions the state keeps are drawn."""
        c = cls(batch, n_kv_heads, window, sink, residual, device=device)
        d = c.head_dim
        lo = c.kept_positions(seq_len)
        n_tail = max(0, seq_len - lo)
        ns = min(seq_len, sink)
        kt = torch.randn(batch, n_kv_heads, ns + n_tail, d, device=c.device, generator=generator)
        vt = torch.randn(batch, n_kv_heads, ns + n_tail, d, device=c.device, generator=generator)
        if outlier_channels:
            ch = torch.randperm(d, device=c.device, generator=generator)[:outlier_channels]
            kt[..., ch] *= outlier_factor
        kt, vt = kt.half(), vt.half()
        c.load_state(seq_len, kt[:, :, :ns], vt[:, :, :ns], kt[:, :, ns:], vt[:, :, ns:], tail_start=lo)
        return c
