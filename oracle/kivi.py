"""KIVI 2-bit quantization oracle (numpy, CPU).  TEST INFRASTRUCTURE ONLY.

Restates, in plain float32 numpy, the arithmetic of the reference's Triton
quantizers so that codes, scales and zero points can be compared bit-exactly:

* ``quantize_k``   follows quant_kernel.py:44-103 (``_quantize_k_kernel``) and
                   the wrapper at quant_kernel.py:106-126.
* ``quantize_v``   follows quant_kernel.py:129-190 (``_quantize_v_kernel``) and
                   the wrapper at quant_kernel.py:193-214.
* ``unpack_dequant`` follows test_quantize_correctness.py:16-43.
* ``build_quantized_kv_cache`` follows quant_kernel.py:584-622.
* ``KiviStreamState`` / ``stream_state`` model the streaming (append) cache,
  which the reference does not have; see the class docstring.

Every operation is done in IEEE float32 in the same order as the reference:
``scale = (max - min) / 3``; ``scale == 0 -> 1``; ``zero = floor(-min/scale +
0.5)``; ``code = clamp(floor(x/scale + 0.5) + zero, 0, 3)``.  Scale and zero are
stored as float16 with round-to-nearest-even; codes use the float32 scale.
Pinned against the reference itself by tests/golden (see
tests/test_oracle_golden.py).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

GROUP_SIZE = 32
QUANT_BITS = 2


def _as_f32(x) -> np.ndarray:
    if hasattr(x, "detach"):  # torch tensor
        x = x.detach().cpu().float().numpy()
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32))


def _to_f16(x: np.ndarray) -> np.ndarray:
    """float32 -> float16, round to nearest even; values beyond the float16
    range become +-inf exactly as the reference's fp16 store does."""
    with np.errstate(over="ignore"):
        return x.astype(np.float16)


def _group_params(mn: np.ndarray, mx: np.ndarray, bits: int):
    """Scale and zero point of one group (quant_kernel.py:77-81 / :166-170)."""
    qmax = np.float32((1 << bits) - 1)
    scale = ((mx - mn) / qmax).astype(np.float32)
    scale = np.where(scale == np.float32(0.0), np.float32(1.0), scale).astype(np.float32)
    zero = np.floor((-mn) / scale + np.float32(0.5)).astype(np.float32)
    return scale, zero


def _codes(x: np.ndarray, scale: np.ndarray, zero: np.ndarray, bits: int) -> np.ndarray:
    """quant_kernel.py:96-98 / :181-183: round-half-up, add zero, clamp."""
    qmax = np.float32((1 << bits) - 1)
    q = np.floor(x / scale + np.float32(0.5)).astype(np.float32) + zero
    return np.clip(q, np.float32(0.0), qmax).astype(np.int32)


def quantize_k(k, group_size: int = GROUP_SIZE, bits: int = QUANT_BITS):
    """Per-channel K quantization over groups of ``group_size`` tokens.

    k: [B, H, T, D] float32, T % group_size == 0.
    Returns packed [B, H, T/4, D] uint8 (byte i holds tokens 4i..4i+3 in bits
    0-1, 2-3, 4-5, 6-7), scale and zero [B, H, T/group_size, D] float16.
    """
    k = _as_f32(k)
    b, h, t, d = k.shape
    if t % group_size:
        raise ValueError("seq_len must be a multiple of group_size")
    pf = 8 // bits
    g = k.reshape(b, h, t // group_size, group_size, d)
    scale, zero = _group_params(g.min(axis=3), g.max(axis=3), bits)
    codes = _codes(g, scale[:, :, :, None, :], zero[:, :, :, None, :], bits).reshape(b, h, t // pf, pf, d)
    packed = np.zeros((b, h, t // pf, d), dtype=np.int32)
    for j in range(pf):
        packed |= codes[:, :, :, j, :] << (j * bits)
    return packed.astype(np.uint8), _to_f16(scale), _to_f16(zero)


def quantize_v(v, group_size: int = GROUP_SIZE, bits: int = QUANT_BITS):
    """Per-token V quantization over groups of ``group_size`` channels.

    v: [B, H, T, D] float32, D % group_size == 0.
    Returns packed [B, H, T, D/4] uint8 (byte j holds channels 4j..4j+3 in
    bits 0-1, 2-3, 4-5, 6-7), scale and zero [B, H, T, D/group_size] float16.
    """
    v = _as_f32(v)
    b, h, t, d = v.shape
    if d % group_size:
        raise ValueError("head_dim must be a multiple of group_size")
    pf = 8 // bits
    g = v.reshape(b, h, t, d // group_size, group_size)
    scale, zero = _group_params(g.min(axis=4), g.max(axis=4), bits)
    codes = _codes(g, scale[..., None], zero[..., None], bits).reshape(b, h, t, d // pf, pf)
    packed = np.zeros((b, h, t, d // pf), dtype=np.int32)
    for j in range(pf):
        packed |= codes[..., j] << (j * bits)
    return packed.astype(np.uint8), _to_f16(scale), _to_f16(zero)


def unpack_dequant(packed, scale, zero_point, full_axis_len: int, pack_axis: int,
                   group_size: int = GROUP_SIZE, bits: int = QUANT_BITS) -> np.ndarray:
    """Shift-and-mask unpack plus affine dequant ``s * (code - z)`` in float32.

    Restates test_quantize_correctness.py:16-43: ``pack_axis`` is 2 for K's
    layout (tokens packed) and 3 for V's (channels packed).
    """
    packed = np.asarray(packed.cpu().numpy() if hasattr(packed, "cpu") else packed).astype(np.int32)
    scale = np.asarray(scale.cpu().numpy() if hasattr(scale, "cpu") else scale).astype(np.float32)
    zero_point = np.asarray(zero_point.cpu().numpy() if hasattr(zero_point, "cpu") else zero_point).astype(np.float32)
    pf = 8 // bits
    qmax = (1 << bits) - 1
    shape = list(packed.shape)
    shape[pack_axis] = full_axis_len
    codes = np.zeros(shape, dtype=np.float32)
    for j in range(pf):
        idx = [slice(None)] * len(shape)
        idx[pack_axis] = slice(j, None, pf)
        codes[tuple(idx)] = ((packed >> (j * bits)) & qmax).astype(np.float32)
    gidx = np.arange(full_axis_len) // group_size
    s = np.take(scale, gidx, axis=pack_axis)
    z = np.take(zero_point, gidx, axis=pack_axis)
    return (s * (codes - z)).astype(np.float32)


def build_quantized_kv_cache(k_compacted, v_compacted, residual_size: int = 128, sink: int = 4,
                             group_size: int = GROUP_SIZE, bits: int = QUANT_BITS) -> dict:
    """quant_kernel.py:584-622: split a compacted [B, H, S+W, D] cache into an
    fp16 residual (last ``residual_size`` slots), a sink padded to one group
    by repeating slot 0, and the window-old slots [S, S+W-R); quantize the
    last two.  Returns numpy arrays under the reference's 14 keys."""
    kc = _as_f32(k_compacted)
    vc = _as_f32(v_compacted)
    n_slots = kc.shape[2]
    win_end = n_slots - residual_size
    out = {
        "k_residual": kc[:, :, win_end:, :].astype(np.float16),
        "v_residual": vc[:, :, win_end:, :].astype(np.float16),
    }
    pad = group_size - sink

    def _pad(x):
        real = x[:, :, :sink, :]
        return np.concatenate([real, np.repeat(real[:, :, :1, :], pad, axis=2)], axis=2)

    out["k_sink_packed"], out["k_sink_scale"], out["k_sink_zero"] = quantize_k(_pad(kc), group_size, bits)
    out["v_sink_packed"], out["v_sink_scale"], out["v_sink_zero"] = quantize_v(_pad(vc), group_size, bits)
    out["k_win_packed"], out["k_win_scale"], out["k_win_zero"] = quantize_k(kc[:, :, sink:win_end, :], group_size, bits)
    out["v_win_packed"], out["v_win_scale"], out["v_win_zero"] = quantize_v(vc[:, :, sink:win_end, :], group_size, bits)
    return out


# --------------------------------------------------------------------------
# Streaming (append) KIVI cache: no reference counterpart.
# --------------------------------------------------------------------------

@dataclass
class StreamGeometry:
    """Shape of the streaming KIVI cache for one (window, sink, residual).

    Tokens 0..S-1 are the sink.  Tokens S.. form the stream; stream index
    ``i = pos - S``.  Unflushed stream tokens live in an fp16 residual ring of
    ``R + G`` slots (slot ``i % (R+G)``).  When R+G tokens are unflushed the
    oldest G (one group) are quantized into the window ring of
    ``NG = (W - R) / G`` group slots (group ``gi`` at slot ``gi % NG``),
    evicting the group that was there; with NG == 0 the group is dropped.
    The attention set is exactly StreamingLLM's: the first min(L, S) tokens
    plus stream tokens with ``pos >= L - W``.
    """
    window: int
    sink: int = 4
    residual: int = 128
    group: int = GROUP_SIZE

    def __post_init__(self):
        if self.window >= self.residual and (self.window - self.residual) % self.group:
            raise ValueError("window - residual must be a multiple of the group size")

    @property
    def n_groups(self) -> int:
        return max(0, (self.window - self.residual) // self.group)

    @property
    def res_cap(self) -> int:
        return self.residual + self.group

    def n_flushed(self, seq_len: int) -> int:
        n_stream = max(0, seq_len - self.sink)
        return max(0, (n_stream - self.residual) // self.group)


def stream_state(k_hist, v_hist, seq_len: int, geom: StreamGeometry) -> dict:
    """State of the streaming KIVI cache after ``seq_len`` appends.

    k_hist, v_hist: [B, H, >=seq_len, D] fp16-representable history.
    Returns numpy arrays in the ring layout used by the CUDA cache manager.
    Slots that hold no live token are returned as zeros together with the
    boolean masks ``res_live`` [R+G] and ``grp_live`` [NG] so that callers can
    compare live content only.
    """
    kh = _as_f32(k_hist)[:, :, :seq_len]
    vh = _as_f32(v_hist)[:, :, :seq_len]
    b, h, _, d = kh.shape
    S, G, R = geom.sink, geom.group, geom.residual
    NG, cap = geom.n_groups, geom.res_cap
    st = {}
    n_sink = min(seq_len, S)
    if n_sink > 0:
        def _pad(x):
            real = x[:, :, :n_sink, :]
            return np.concatenate([real, np.repeat(real[:, :, :1, :], G - n_sink, axis=2)], axis=2)
        st["k_sink_packed"], st["k_sink_scale"], st["k_sink_zero"] = quantize_k(_pad(kh), G)
        st["v_sink_packed"], st["v_sink_scale"], st["v_sink_zero"] = quantize_v(_pad(vh), G)
    n_stream = max(0, seq_len - S)
    F = geom.n_flushed(seq_len)
    k_res = np.zeros((b, h, cap, d), np.float16)
    v_res = np.zeros((b, h, cap, d), np.float16)
    res_live = np.zeros(cap, bool)
    for i in range(G * F, n_stream):
        k_res[:, :, i % cap] = kh[:, :, S + i]
        v_res[:, :, i % cap] = vh[:, :, S + i]
        res_live[i % cap] = True
    st["k_res"], st["v_res"], st["res_live"] = k_res, v_res, res_live
    kwp = np.zeros((b, h, NG * G // 4, d), np.uint8)
    kws = np.zeros((b, h, NG, d), np.float16)
    kwz = np.zeros((b, h, NG, d), np.float16)
    vwp = np.zeros((b, h, NG * G, d // 4), np.uint8)
    vws = np.zeros((b, h, NG * G, d // G), np.float16)
    vwz = np.zeros((b, h, NG * G, d // G), np.float16)
    grp_live = np.zeros(NG, bool)
    for gi in range(max(0, F - NG), F):
        slot = gi % NG
        t0 = S + gi * G
        p, s, z = quantize_k(kh[:, :, t0:t0 + G], G)
        kwp[:, :, slot * G // 4:(slot + 1) * G // 4], kws[:, :, slot], kwz[:, :, slot] = p, s[:, :, 0], z[:, :, 0]
        p, s, z = quantize_v(vh[:, :, t0:t0 + G], G)
        vwp[:, :, slot * G:(slot + 1) * G], vws[:, :, slot * G:(slot + 1) * G], vwz[:, :, slot * G:(slot + 1) * G] = p, s, z
        grp_live[slot] = True
    st.update(k_win_packed=kwp, k_win_scale=kws, k_win_zero=kwz,
              v_win_packed=vwp, v_win_scale=vws, v_win_zero=vwz, grp_live=grp_live)
    return st


def stream_dequant_tokens(st: dict, seq_len: int, geom: StreamGeometry):
    """Dequantized K/V [B, H, N, D] float32 of exactly the attended tokens of a
    ``stream_state`` (order: sink, flushed stream tokens, unflushed ones)."""
    S, G, W = geom.sink, geom.group, geom.window
    NG, cap = geom.n_groups, geom.res_cap
    n_stream = max(0, seq_len - S)
    F = geom.n_flushed(seq_len)
    first = max(S, seq_len - W)  # oldest attended stream position
    ks, vs = [], []
    n_sink = min(seq_len, S)
    if n_sink:
        ks.append(unpack_dequant(st["k_sink_packed"], st["k_sink_scale"], st["k_sink_zero"], G, 2)[:, :, :n_sink])
        vs.append(unpack_dequant(st["v_sink_packed"], st["v_sink_scale"], st["v_sink_zero"], st["v_sink_packed"].shape[3] * 4, 3)[:, :, :n_sink])
    for gi in range(max(0, F - NG), F):
        slot = gi % NG
        kd = unpack_dequant(st["k_win_packed"][:, :, slot * G // 4:(slot + 1) * G // 4],
                            st["k_win_scale"][:, :, slot:slot + 1], st["k_win_zero"][:, :, slot:slot + 1], G, 2)
        vd = unpack_dequant(st["v_win_packed"][:, :, slot * G:(slot + 1) * G],
                            st["v_win_scale"][:, :, slot * G:(slot + 1) * G],
                            st["v_win_zero"][:, :, slot * G:(slot + 1) * G], st["v_win_packed"].shape[3] * 4, 3)
        lo = max(0, first - (S + gi * G))
        ks.append(kd[:, :, lo:])
        vs.append(vd[:, :, lo:])
    for i in range(G * F, n_stream):
        if S + i >= first:
            ks.append(st["k_res"][:, :, i % cap][:, :, None].astype(np.float32))
            vs.append(st["v_res"][:, :, i % cap][:, :, None].astype(np.float32))
    return np.concatenate(ks, axis=2), np.concatenate(vs, axis=2)
