"""Parity of the sm_100a KIVI kernels through the C ABI.

* quantizers: codes, scales and zero points bit-exact with the reference's
  golden vectors (and the numpy oracle), float32 and float16 inputs;
* reference-layout attention (sparse_decode_attention_quantized) within the
  2-bit-path tolerance of the fp32 oracle (test_quantized_attention_correctness
  .py:288-317) and of the reference kernel's own outputs;
* streaming cache: state after every append bit-exact with the oracle's model
  (oracle/kivi.py stream_state), attention within tolerance of the oracle.
"""
import numpy as np
import pytest
import torch

import fixtures
import inputs as gi
import quant_kernel
from oracle import attention as oa
from oracle import kivi as ok

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL_2BIT = 1e-2   # north_star tolerance for the 2-bit paths (max |o - o_ref|)


def _err(a, b):
    return (a.float().cpu() - torch.as_tensor(b).float().cpu()).abs().max().item()


def _np(t):
    return t.detach().cpu().numpy()


# ---------------------------------------------------------------- quantizers
def _check_vs_meta(meta, arrays, produced):
    for key, info in meta["arrays"].items():
        if key not in produced:
            continue
        got = np.ascontiguousarray(produced[key])
        assert list(got.shape) == info["shape"], key
        assert gi.sha(got) == info["sha256"], f"{key} differs from the reference's golden vector"


def _k_input(meta):
    shape, seed, kind = tuple(meta["shape"]), meta["seed"], meta["kind"]
    if kind == "degenerate":
        return gi.degenerate_groups(shape, seed, axis=2)
    return {"randn": gi.randn, "kivi_k": gi.kivi_k}[kind](shape, seed)


@pytest.mark.parametrize("name", fixtures.names("quantize_k"))
def test_quantize_k_bit_exact_vs_reference(name):
    meta, arrays = fixtures.load(name)
    x = _k_input(meta)
    p, s, z = quant_kernel.quantize_k_cache(x.to(DEV))
    _check_vs_meta(meta, arrays, {"packed": _np(p), "scale": _np(s), "zero": _np(z)})


@pytest.mark.parametrize("name", fixtures.names("quantize_v"))
def test_quantize_v_bit_exact_vs_reference(name):
    meta, arrays = fixtures.load(name)
    shape, seed = tuple(meta["shape"]), meta["seed"]
    x = gi.randn(shape, seed) if meta["kind"] == "randn" else gi.degenerate_groups(shape, seed, axis=3)
    p, s, z = quant_kernel.quantize_v_cache(x.to(DEV))
    _check_vs_meta(meta, arrays, {"packed": _np(p), "scale": _np(s), "zero": _np(z)})


def test_quantize_fp16_input_matches_float_of_it():
    x = gi.kivi_k((2, 8, 512, 128), 77).half()
    for q_gpu, q_np in ((quant_kernel.quantize_k_cache, ok.quantize_k), (quant_kernel.quantize_v_cache, ok.quantize_v)):
        got = [_np(t) for t in q_gpu(x.to(DEV))]
        ref = q_np(x.float())
        for a, b in zip(got, ref):
            np.testing.assert_array_equal(a, b)


def test_quantize_sink_padding():
    meta, arrays = fixtures.load("quant_sink_pad")
    sink = gi.randn((1, 1, 4, 128), 2)
    padded = torch.cat([sink, sink[:, :, :1].expand(-1, -1, 28, -1)], dim=2).contiguous().to(DEV)
    kp, ks, kz = quant_kernel.quantize_k_cache(padded)
    vp, vs, vz = quant_kernel.quantize_v_cache(padded)
    _check_vs_meta(meta, arrays, {"k_packed": _np(kp), "k_scale": _np(ks), "k_zero": _np(kz),
                                  "v_packed": _np(vp), "v_scale": _np(vs), "v_zero": _np(vz)})


@pytest.mark.parametrize("name,axis", [("dequant_k_tile", 2), ("dequant_v_tile", 3)])
def test_host_dequant_matches_reference_tile(name, axis):
    """test_dequantize_tile_isolated.py:66-120 through the host-callable form."""
    meta, arrays = fixtures.load(name)
    x = gi.randn((1, 1, 256, 128), meta["seed"]).to(DEV)
    if axis == 2:
        p, s, z = quant_kernel.quantize_k_cache(x)
        out = quant_kernel.dequantize_k(p, s, z, 256, 0, 128)
    else:
        p, s, z = quant_kernel.quantize_v_cache(x)
        out = quant_kernel.dequantize_v(p, s, z, 256, 0, 128)
    assert _err(out, arrays["out"]) < 1e-6


# ---------------------------------------------------------------- reference layout
@pytest.mark.parametrize("name", fixtures.names("kivi"))
def test_kivi_attention_matches_reference_golden(name):
    meta, arrays = fixtures.load(name)
    L, W, seed, B = meta["seq_len"], meta["window"], meta["seed"], meta["batch"]
    q = gi.randn((B, 64, 128), seed).half()
    kc = gi.kivi_k((B, 8, 4 + W, 128), seed + 100).half()
    vc = gi.randn((B, 8, 4 + W, 128), seed + 200).half()
    cache = quant_kernel.build_quantized_kv_cache(kc.to(DEV), vc.to(DEV))
    # the GPU cache builder reproduces the reference's quantized tensors bit for bit
    _check_vs_meta(meta, arrays, {"cache_" + k: _np(v) for k, v in cache.items()})
    o = quant_kernel.sparse_decode_attention_quantized(
        q.to(DEV), cache["k_residual"], cache["v_residual"],
        cache["k_sink_packed"], cache["k_sink_scale"], cache["k_sink_zero"],
        cache["v_sink_packed"], cache["v_sink_scale"], cache["v_sink_zero"],
        cache["k_win_packed"], cache["k_win_scale"], cache["k_win_zero"],
        cache["v_win_packed"], cache["v_win_scale"], cache["v_win_zero"],
        seq_len=L, window=W)
    assert _err(o, arrays["o"]) < TOL_2BIT
    assert _err(o, oa.quantized_attention(q, W - 128, {k: v.cpu() for k, v in cache.items()})) < TOL_2BIT


def _ref_layout_call(q, cache, L, W):
    return quant_kernel.sparse_decode_attention_quantized(
        q, cache["k_residual"], cache["v_residual"],
        cache["k_sink_packed"], cache["k_sink_scale"], cache["k_sink_zero"],
        cache["v_sink_packed"], cache["v_sink_scale"], cache["v_sink_zero"],
        cache["k_win_packed"], cache["k_win_scale"], cache["k_win_zero"],
        cache["v_win_packed"], cache["v_win_scale"], cache["v_win_zero"],
        seq_len=L, window=W)


def _masked_quantized_oracle(q, cache, L, W, S=4, R=128):
    """Reference-layout attention with _kv_indices validity (compacted order
    sink | window-old | residual), dequantizing the same tensors."""
    c = {k: v.cpu() for k, v in cache.items()}
    ks = ok.unpack_dequant(c["k_sink_packed"], c["k_sink_scale"], c["k_sink_zero"], 32, 2)[:, :, :S]
    vs = ok.unpack_dequant(c["v_sink_packed"], c["v_sink_scale"], c["v_sink_zero"], 128, 3)[:, :, :S]
    kw = ok.unpack_dequant(c["k_win_packed"], c["k_win_scale"], c["k_win_zero"], W - R, 2)
    vw = ok.unpack_dequant(c["v_win_packed"], c["v_win_scale"], c["v_win_zero"], 128, 3)
    k = torch.from_numpy(np.concatenate([ks, kw, c["k_residual"].float().numpy()], axis=2))
    v = torch.from_numpy(np.concatenate([vs, vw, c["v_residual"].float().numpy()], axis=2))
    mask = torch.from_numpy(oa.slot_validity(L, W, S))
    return oa._attend(q.cpu().float(), k, v, 128 ** -0.5, mask[None])


@pytest.mark.parametrize("W,L", [(128, 5000), (256, 4 + 256 + 1000), (512, 4 + 512 + 1000), (8192, 4 + 8192 + 1000),
                                 (256, 163_840), (256, 2), (256, 100), (256, 200), (512, 300), (160, 261)])
def test_kivi_reference_layout_full_batch(W, L):
    """B=32, 64/8/128 heads; steady state (test_quantized_attention_correctness
    .py:64-103 cases) and ramp-up (slot masks of _kv_indices)."""
    B = 32
    g = torch.Generator(device=DEV).manual_seed(W * 31 + L)
    q = torch.randn(B, 64, 128, device=DEV, generator=g).half()
    kc = torch.randn(B, 8, 4 + W, 128, device=DEV, generator=g)
    kc[..., torch.randperm(128, device=DEV, generator=g)[:4]] *= 8
    kc = kc.half()
    vc = torch.randn(B, 8, 4 + W, 128, device=DEV, generator=g).half()
    cache = quant_kernel.build_quantized_kv_cache(kc, vc)
    o = _ref_layout_call(q, cache, L, W)
    assert _err(o, _masked_quantized_oracle(q, cache, L, W)) < TOL_2BIT


# ---------------------------------------------------------------- streaming cache
def _state_np(cache):
    return {k: _np(v) for k, v in cache.state().items()}


def _compare_state(cache, k_hist, v_hist, L, geom):
    ref = ok.stream_state(k_hist, v_hist, L, geom)
    got = _state_np(cache)
    assert (got["unit_lens"] == L).all()
    if min(L, geom.sink):
        for key in ("k_sink_packed", "k_sink_scale", "k_sink_zero", "v_sink_packed", "v_sink_scale", "v_sink_zero"):
            np.testing.assert_array_equal(got[key], ref[key], err_msg=f"{key} at L={L}")
    live = ref["res_live"]
    for key in ("k_res", "v_res"):
        np.testing.assert_array_equal(got[key][:, :, live], ref[key][:, :, live], err_msg=f"{key} at L={L}")
    gl = ref["grp_live"]
    if gl.any():
        G = geom.group
        for key, per in (("k_win_packed", 8), ("k_win_scale", 1), ("k_win_zero", 1), ("v_win_packed", G),
                         ("v_win_scale", G), ("v_win_zero", G)):
            rows = np.concatenate([np.arange(s * per, (s + 1) * per) for s in np.nonzero(gl)[0]])
            np.testing.assert_array_equal(got[key][:, :, rows], ref[key][:, :, rows], err_msg=f"{key} at L={L}")


@pytest.mark.parametrize("W", [256, 128, 32, 192, 64, 384])
def test_stream_append_from_empty_matches_oracle(W):
    """Appends from an empty cache through the sink re-quantization (steps
    1-4), ramp-up, the first group flushes and window eviction; the state is
    checked bit-exactly and the attention output against the oracle.  B=2:
    one CTA per unit and the append inside the decode launch at every window
    here -- the resident-only kernel at W <= 256, residual copies covering the
    attended rows only at W < 128, two Q-batches at W=384."""
    B, Hkv, S, R = 2, 8, 4, 128
    geom = ok.StreamGeometry(window=W, sink=S, residual=R)
    n_steps = S + W + R + 3 * 32 + 5
    k_hist = gi.kivi_k((B, Hkv, n_steps, 128), 900 + W).half()
    v_hist = gi.randn((B, Hkv, n_steps, 128), 901 + W).half()
    q_all = gi.randn((n_steps, B, 64, 128), 902 + W).half()
    cache = quant_kernel.KiviCache(B, Hkv, W, sink=S, residual=R, device=DEV)
    kd, vd, qd = k_hist.to(DEV), v_hist.to(DEV), q_all.to(DEV)
    check_at = set(range(1, 8)) | {S + R + 31, S + R + 32, S + R + 33, S + W, S + W + 1, S + W + 32, n_steps}
    check_at |= set(range(S + R + 32, n_steps + 1, 29))
    for L in range(1, n_steps + 1):
        o = cache.decode_step(qd[L - 1], kd[:, :, L - 1].contiguous(), vd[:, :, L - 1].contiguous())
        if L in check_at:
            _compare_state(cache, k_hist, v_hist, L, geom)
            st = ok.stream_state(k_hist, v_hist, L, geom)
            ref = oa.stream_attention(q_all[L - 1], st, L, geom)
            assert _err(o, ref) < TOL_2BIT, L


def test_stream_aligned_phase_equals_reference_layout():
    """When (L - S - R) % 32 == 0 and L >= S + W, the streaming state is
    build_quantized_kv_cache of the compacted window, and both kernels agree."""
    B, Hkv, S, R, W = 4, 8, 4, 128, 256
    L = S + W + 32 * 7  # (L - S - R) % 32 == 0
    assert (L - S - R) % 32 == 0
    k_hist = gi.kivi_k((B, Hkv, L, 128), 1234).half().to(DEV)
    v_hist = gi.randn((B, Hkv, L, 128), 1235).half().to(DEV)
    q = gi.randn((B, 64, 128), 1236).half().to(DEV)
    cache = quant_kernel.KiviCache(B, Hkv, W, device=DEV)
    cache.load_history(k_hist, v_hist, L)
    kc, vc = oa.build_compacted_cache(k_hist, v_hist, L, W, S)
    ref_cache = quant_kernel.build_quantized_kv_cache(kc.contiguous(), vc.contiguous())
    o_stream = cache.attend(q)
    o_ref = _ref_layout_call(q, ref_cache, L, W)
    assert _err(o_stream, o_ref) < 2e-3
    # quantized window groups equal, in ring order
    st = _state_np(cache)
    NG = (W - R) // 32
    F = (L - S - R) // 32
    order = [(F - NG + j) % NG for j in range(NG)]
    kwp = np.concatenate([st["k_win_packed"][:, :, s * 8:(s + 1) * 8] for s in order], axis=2)
    np.testing.assert_array_equal(kwp, _np(ref_cache["k_win_packed"]))
    vws = np.concatenate([st["v_win_scale"][:, :, s * 32:(s + 1) * 32] for s in order], axis=2)
    np.testing.assert_array_equal(vws, _np(ref_cache["v_win_scale"]))


def test_stream_full_size_synthetic_against_oracle():
    """B=32, W=256 after L=163,840 appends (the benchmark state), then a few
    decode steps with quantize-on-append, each checked against the oracle
    evaluated on the cache's own tensors."""
    B, Hkv, W, L = 32, 8, 256, 163_840
    g = torch.Generator(device=DEV).manual_seed(5)
    cache = quant_kernel.KiviCache.synthetic(B, Hkv, W, L, device=DEV, generator=g)
    geom = ok.StreamGeometry(window=W)
    for step in range(40):
        q = torch.randn(B, 64, 128, device=DEV, generator=g).half()
        nk = torch.randn(B, Hkv, 128, device=DEV, generator=g).half()
        nv = torch.randn(B, Hkv, 128, device=DEV, generator=g).half()
        o = cache.decode_step(q, nk, nv)
        if step % 13 == 0 or step in (27, 28, 29):  # includes a group flush (p wraps at 32)
            Lc = L + step + 1
            st = _state_np(cache)
            ref = oa.stream_attention(q, st, Lc, geom)
            assert _err(o, ref) < TOL_2BIT, step


@pytest.mark.parametrize("W", [256, 128])
def test_fused_step_equals_append_then_attend(W):
    """B=32 (every unit gets its own CTA): the one-launch decode step --
    store, group flush or sink re-quantization and attention in the decode
    kernel -- gives cache states bit-identical to nsa_kivi_append followed by
    nsa_kivi_stream_decode, and the same outputs up to rounding (a unit's jobs
    go to whichever warp is free first, so the order in which partial sums are
    accumulated varies between launches), from an empty cache through the sink
    phase, the first flushes (dropped groups when W == R) and eviction."""
    B, Hkv, S, R = 32, 8, 4, 128
    n_steps = S + max(W, R + 32) + R + 2 * 32 + 3
    g = torch.Generator(device=DEV).manual_seed(70 + W)
    fused = quant_kernel.KiviCache(B, Hkv, W, sink=S, residual=R, device=DEV)
    split = quant_kernel.KiviCache(B, Hkv, W, sink=S, residual=R, device=DEV)
    assert fused.step_launches() == 1
    check_at = {1, 2, S, S + 1, S + R + 31, S + R + 32, S + R + 33, n_steps}
    for L in range(1, n_steps + 1):
        q = torch.randn(B, 64, 128, device=DEV, generator=g).half()
        nk = (torch.randn(B, Hkv, 128, device=DEV, generator=g) * (1 + (L % 3))).half()
        nv = torch.randn(B, Hkv, 128, device=DEV, generator=g).half()
        o_f = fused.decode_step(q, nk, nv)
        split.append(nk, nv)
        o_s = split.attend(q)
        assert _err(o_f, o_s) < 2e-3, L  # rounding-level (accumulation order); the state is exact
        if L in check_at:
            a, b = _state_np(fused), _state_np(split)
            for key in a:
                np.testing.assert_array_equal(a[key], b[key], err_msg=f"{key} at L={L}")


def test_fused_step_multi_batch_window():
    """W=1024 (28 window groups: six Q-batches refilled through the two-stage
    ring while the warps work): fused decode steps across a group flush match
    the oracle, give append + attend's outputs up to rounding and leave the
    same cache state (bit for bit)."""
    B, Hkv, W, L, S, R = 32, 8, 1024, 163_840, 4, 128
    fused = quant_kernel.KiviCache.synthetic(B, Hkv, W, L, device=DEV,
                                             generator=torch.Generator(device=DEV).manual_seed(9))
    split = quant_kernel.KiviCache.synthetic(B, Hkv, W, L, device=DEV,
                                             generator=torch.Generator(device=DEV).manual_seed(9))
    assert fused.step_launches() == 1
    geom = ok.StreamGeometry(window=W)
    g = torch.Generator(device=DEV).manual_seed(10)
    for step in range(36):
        q = torch.randn(B, 64, 128, device=DEV, generator=g).half()
        nk = torch.randn(B, Hkv, 128, device=DEV, generator=g).half()
        nv = torch.randn(B, Hkv, 128, device=DEV, generator=g).half()
        o_f = fused.decode_step(q, nk, nv)
        split.append(nk, nv)
        o_s = split.attend(q)
        assert _err(o_f, o_s) < 2e-3, step  # rounding-level (accumulation order)
        if step in (0, 27, 28, 35):
            ref = oa.stream_attention(q, _state_np(fused), L + step + 1, geom)
            assert _err(o_f, ref) < TOL_2BIT, step
    a, b = _state_np(fused), _state_np(split)
    for key in a:
        np.testing.assert_array_equal(a[key], b[key], err_msg=key)


@pytest.mark.parametrize("R,W", [(256, 512), (384, 384)])
def test_large_residual_ring_refills_residual_stages(R, W):
    """A residual ring of R + 32 = 288 / 416 slots is four / six F-tiles, more
    than the two F stages: the tiles are refilled into freed stages while the
    warps work (and the job counters reset with them).  Fused steps across a
    group flush match the oracle and append + attend, and the state stays
    bit-exact with append + attend."""
    B, Hkv, L, S = 32, 8, 100_000, 4
    mk = lambda: quant_kernel.KiviCache.synthetic(B, Hkv, W, L, residual=R, device=DEV,  # noqa: E731
                                                  generator=torch.Generator(device=DEV).manual_seed(31))
    fused, split = mk(), mk()
    assert fused.step_launches() == 1
    geom = ok.StreamGeometry(window=W, sink=S, residual=R)
    g = torch.Generator(device=DEV).manual_seed(32)
    for step in range(34):
        q = torch.randn(B, 64, 128, device=DEV, generator=g).half()
        nk = torch.randn(B, Hkv, 128, device=DEV, generator=g).half()
        nv = torch.randn(B, Hkv, 128, device=DEV, generator=g).half()
        o_f = fused.decode_step(q, nk, nv)
        split.append(nk, nv)
        o_s = split.attend(q)
        assert _err(o_f, o_s) < 2e-3, step
        if step in (0, 5, 17, 33) or (L + step + 1 - S - R) % 32 == 0:
            ref = oa.stream_attention(q, _state_np(fused), L + step + 1, geom)
            assert _err(o_f, ref) < TOL_2BIT, step
    a, b = _state_np(fused), _state_np(split)
    for key in a:
        np.testing.assert_array_equal(a[key], b[key], err_msg=key)


@pytest.mark.parametrize("W", [256, 32])
def test_layer_batched_step_equals_per_layer_steps(W):
    """decode_step_layers (3 layers in one launch) gives the same cache
    states, bit for bit, and the same outputs up to rounding (accumulation
    order) as KiviCache.decode_step layer by layer, over steps that include a
    group flush (W=256) or copies of the attended residual rows only (W=32)."""
    import importlib
    kivi = importlib.import_module("numerics-and-sparse-attn_b200.kivi")
    B, Hkv, L, n = 32, 8, 163_840, 3

    def make():
        g = torch.Generator(device=DEV).manual_seed(123)
        return [kivi.KiviCache.synthetic(B, Hkv, W, L, device=DEV, generator=g) for _ in range(n)]

    batched, single = make(), make()
    g = torch.Generator(device=DEV).manual_seed(7)
    for step in range(36):
        qs = [torch.randn(B, 64, 128, device=DEV, generator=g).half() for _ in range(n)]
        nks = [torch.randn(B, Hkv, 128, device=DEV, generator=g).half() for _ in range(n)]
        nvs = [torch.randn(B, Hkv, 128, device=DEV, generator=g).half() for _ in range(n)]
        outs = kivi.decode_step_layers(batched, qs, nks, nvs)
        for layer in range(n):
            ref = single[layer].decode_step(qs[layer], nks[layer], nvs[layer])
            assert _err(outs[layer], ref) < 2e-3, (step, layer)
    for a, b in zip(batched, single):
        sa, sb = _state_np(a), _state_np(b)
        for key in sa:
            np.testing.assert_array_equal(sa[key], sb[key], err_msg=key)


@pytest.mark.parametrize("B,W,launches", [(32, 256, 1), (2, 256, 1), (1, 416, 1), (2, 1024, 2), (32, 1024, 1)])
def test_step_launch_plan(B, W, launches):
    """One launch per decode step when every unit keeps its own CTA: at B=32
    (256 units, more than half the 296 CTA slots), and at any batch when a
    unit's groups and residual all fit the kernel's stages (W <= 416 with
    residual 128); small batches of long windows split their units and
    append in a launch of its own."""
    cache = quant_kernel.KiviCache(B, 8, W, device=DEV)
    assert cache.step_launches() == launches


def test_no_device_error_recorded():
    import importlib
    pkg = importlib.import_module("numerics-and-sparse-attn_b200")
    assert pkg.device_error() == 0
