"""Pin the CPU oracle against golden vectors produced by the reference itself
(tests/golden/make_golden.py: the reference's Triton kernels run under the
Triton interpreter).  CPU only."""
import numpy as np
import pytest
import torch

import fixtures
import inputs as gi
from oracle import attention as oa
from oracle import kivi as ok


def _check_arrays(meta, arrays, produced: dict):
    for key, info in meta["arrays"].items():
        if key not in produced:
            continue
        got = np.ascontiguousarray(produced[key])
        assert list(got.shape) == info["shape"], key
        assert str(got.dtype) == info["dtype"], key
        if info["stored"] == "full":
            np.testing.assert_array_equal(got, arrays[key], err_msg=key)
        else:
            np.testing.assert_array_equal(got.reshape(-1)[:4096], arrays[key + "__head"], err_msg=key)
        assert gi.sha(got) == info["sha256"], f"{key}: digest mismatch"


def _k_input(meta):
    shape, seed, kind = tuple(meta["shape"]), meta["seed"], meta["kind"]
    if kind == "degenerate":
        return gi.degenerate_groups(shape, seed, axis=2)
    return {"randn": gi.randn, "kivi_k": gi.kivi_k}[kind](shape, seed)


@pytest.mark.parametrize("name", fixtures.names("quantize_k"))
def test_quantize_k_bit_exact(name):
    meta, arrays = fixtures.load(name)
    x = _k_input(meta)
    assert gi.sha(x) == meta["input_sha256"], "input generator drifted"
    p, s, z = ok.quantize_k(x)
    _check_arrays(meta, arrays, {"packed": p, "scale": s, "zero": z})


@pytest.mark.parametrize("name", fixtures.names("quantize_v"))
def test_quantize_v_bit_exact(name):
    meta, arrays = fixtures.load(name)
    shape, seed = tuple(meta["shape"]), meta["seed"]
    x = gi.randn(shape, seed) if meta["kind"] == "randn" else gi.degenerate_groups(shape, seed, axis=3)
    assert gi.sha(x) == meta["input_sha256"]
    p, s, z = ok.quantize_v(x)
    _check_arrays(meta, arrays, {"packed": p, "scale": s, "zero": z})


def test_sink_padding_bit_exact():
    meta, arrays = fixtures.load("quant_sink_pad")
    sink = gi.randn((1, 1, 4, 128), 2)
    assert gi.sha(sink) == meta["input_sha256"]
    padded = torch.cat([sink, sink[:, :, :1].expand(-1, -1, 28, -1)], dim=2)
    kp, ks, kz = ok.quantize_k(padded)
    vp, vs, vz = ok.quantize_v(padded)
    _check_arrays(meta, arrays, {"k_packed": kp, "k_scale": ks, "k_zero": kz,
                                 "v_packed": vp, "v_scale": vs, "v_zero": vz})
    # test_quantize_correctness.py:100-125: the 4 real values reconstruct
    # within half the real range
    recon = ok.unpack_dequant(kp, ks, kz, 32, 2)[:, :, :4]
    tol = (sink.amax(2) - sink.amin(2)).max().item() / 2 + 1e-3
    assert np.abs(recon - sink.numpy()).max() < tol


@pytest.mark.parametrize("name,axis", [("dequant_k_tile", 2), ("dequant_v_tile", 3)])
def test_dequant_tile_matches_reference_kernel(name, axis):
    meta, arrays = fixtures.load(name)
    x = gi.randn((1, 1, 256, 128), meta["seed"])
    assert gi.sha(x) == meta["input_sha256"]
    if axis == 2:
        p, s, z = ok.quantize_k(x)
        out = ok.unpack_dequant(p, s, z, 256, 2)[:, :, :128]
    else:
        p, s, z = ok.quantize_v(x)
        out = ok.unpack_dequant(p, s, z, 128, 3)[:, :, :128]
    np.testing.assert_allclose(out, arrays["out"], rtol=0, atol=1e-6)


@pytest.mark.parametrize("name", fixtures.names("dense"))
def test_dense_oracle_matches_reference_kernel(name):
    meta, arrays = fixtures.load(name)
    L, seed, B = meta["seq_len"], meta["seed"], meta["batch"]
    q = gi.randn((B, 64, 128), seed).half()
    k = gi.randn((B, 8, L, 128), seed + 100).half()
    v = gi.randn((B, 8, L, 128), seed + 200).half()
    assert gi.sha(torch.cat([q.reshape(-1), k.reshape(-1), v.reshape(-1)])) == meta["input_sha256"]
    o = oa.dense_attention(q.float(), k.float(), v.float(), 128 ** -0.5)
    ref = torch.from_numpy(arrays["o"]).float()
    assert (o - ref).abs().max().item() < 2e-3


@pytest.mark.parametrize("name", fixtures.names("sparse"))
def test_sparse_oracle_matches_reference_kernel(name):
    meta, arrays = fixtures.load(name)
    L, W, seed, B = meta["seq_len"], meta["window"], meta["seed"], meta["batch"]
    q = gi.randn((B, 64, 128), seed)
    kf = gi.randn((B, 8, L, 128), seed + 100)
    vf = gi.randn((B, 8, L, 128), seed + 200)
    assert gi.sha(torch.cat([q.reshape(-1), kf.reshape(-1), vf.reshape(-1)])) == meta["input_sha256"]
    kc, vc = oa.build_compacted_cache(kf, vf, L, W, 4)
    # the compacted-cache builder restatement reproduces the reference's bytes
    assert gi.sha(torch.cat([kc.half().reshape(-1), vc.half().reshape(-1)])) == meta["cache_sha256"]
    ref = torch.from_numpy(arrays["o"]).float()
    # the masked full-context oracle (test_sparse_correctness.py:22-48) on the
    # fp16-rounded inputs the kernel saw
    o_full = oa.sparse_attention_full(q.half().float(), kf.half().float(), vf.half().float(), L, W, 4)
    assert (o_full - ref).abs().max().item() < 2e-3
    # slot-validity form (sparse_kernel.py:15-46) over the compacted cache
    o_slots = oa.sparse_attention_slots(q.half().float(), kc.half().float(), vc.half().float(), L, W, 4)
    assert (o_slots - ref).abs().max().item() < 2e-3


@pytest.mark.parametrize("name", fixtures.names("kivi"))
def test_kivi_oracle_matches_reference(name):
    meta, arrays = fixtures.load(name)
    L, W, seed, B = meta["seq_len"], meta["window"], meta["seed"], meta["batch"]
    q = gi.randn((B, 64, 128), seed).half()
    kc = gi.kivi_k((B, 8, 4 + W, 128), seed + 100).half()
    vc = gi.randn((B, 8, 4 + W, 128), seed + 200).half()
    assert gi.sha(torch.cat([q.reshape(-1), kc.reshape(-1), vc.reshape(-1)])) == meta["input_sha256"]
    cache = ok.build_quantized_kv_cache(kc, vc)
    _check_arrays(meta, arrays, {"cache_" + k: v for k, v in cache.items()})
    o = oa.quantized_attention(q, W - 128, cache)
    ref = torch.from_numpy(arrays["o"]).float()
    assert (o - ref).abs().max().item() < 2e-3


def test_slot_validity_ring_equals_compacted():
    """A ring cache with head (L-S) mod W attends the same positions as the
    compacted layout of the same context."""
    for L, W in [(2, 256), (100, 256), (5000, 256), (2, 0), (300, 32), (261, 256), (1000, 1)]:
        kf = gi.randn((1, 1, L, 128), L)
        vf = gi.randn((1, 1, L, 128), L + 1)
        q = gi.randn((1, 8, 128), L + 2)
        kc, vc = oa.build_compacted_cache(kf, vf, L, W, 4)
        kr, vr, head = oa.build_ring_cache(kf, vf, L, W, 4)
        a = oa.sparse_attention_slots(q, kc, vc, L, W, 4)
        b = oa.sparse_attention_slots(q, kr, vr, L, W, 4, ring_head=head)
        c = oa.sparse_attention_full(q, kf, vf, L, W, 4)
        assert (a - c).abs().max().item() < 1e-5
        assert (b - c).abs().max().item() < 1e-5
