"""Parity of the sm_100a dense and sink+window decode kernels (through the C
ABI via the drop-in modules) against the reference's golden outputs and the
fp32 oracle.  Tolerance: max |o - o_ref| < 2e-3 on the fp16 paths."""
import pytest
import torch

import dense_kernel
import fixtures
import inputs as gi
import sparse_kernel
from oracle import attention as oa

pytestmark = pytest.mark.gpu
TOL = 2e-3
DEV = "cuda"


def _err(a, b):
    return (a.float().cpu() - b.float().cpu()).abs().max().item()


@pytest.mark.parametrize("name", fixtures.names("dense"))
def test_dense_matches_reference_golden(name):
    meta, arrays = fixtures.load(name)
    L, seed, B = meta["seq_len"], meta["seed"], meta["batch"]
    q = gi.randn((B, 64, 128), seed).half()
    k = gi.randn((B, 8, L, 128), seed + 100).half()
    v = gi.randn((B, 8, L, 128), seed + 200).half()
    o = dense_kernel.dense_decode_attention(q.to(DEV), k.to(DEV), v.to(DEV), seq_len=L, sm_scale=128 ** -0.5)
    assert o.dtype == torch.float16 and o.shape == q.shape
    assert _err(o, torch.from_numpy(arrays["o"])) < TOL
    assert _err(o, oa.dense_attention(q.float(), k.float(), v.float())) < TOL


@pytest.mark.parametrize("seq_len", [1, 2, 63, 64, 65, 1000, 8192, 131_072])
def test_dense_reference_shapes(seq_len):
    """test_dense_correctness.py:33-58 at B=32, 64/8 heads; 131072 crosses the
    int32 offset overflow point the reference hit."""
    B = 32 if seq_len <= 8192 else 8
    g = torch.Generator(device=DEV).manual_seed(seq_len)
    q = torch.randn(B, 64, 128, device=DEV, generator=g)
    k = torch.randn(B, 8, seq_len, 128, device=DEV, generator=g).half()
    v = torch.randn(B, 8, seq_len, 128, device=DEV, generator=g).half()
    o = dense_kernel.dense_decode_attention(q.half(), k, v, seq_len=seq_len)
    ref = oa.dense_attention(q.half().float(), k.float(), v.float())
    assert _err(o, ref) < TOL


def test_dense_int32_crossing_full_batch():
    """B=32 x L=131072: element offsets exceed 2^31 (the reference's bug)."""
    B, L = 32, 131_072
    g = torch.Generator(device=DEV).manual_seed(7)
    q = torch.randn(B, 64, 128, device=DEV, generator=g).half()
    k = torch.randn(B, 8, L, 128, device=DEV, generator=g).half()
    v = torch.randn(B, 8, L, 128, device=DEV, generator=g).half()
    o = dense_kernel.dense_decode_attention(q, k, v, seq_len=L)
    for b in (0, B - 1):  # fp32 reference per batch row keeps the checker's memory small
        ref = oa.dense_attention(q[b:b + 1].float(), k[b:b + 1].float(), v[b:b + 1].float())
        assert _err(o[b:b + 1], ref) < TOL


def test_dense_capacity_larger_than_seq_len():
    B, cap, L = 4, 700, 333
    q = gi.randn((B, 64, 128), 1).half().to(DEV)
    k = gi.randn((B, 8, cap, 128), 2).half().to(DEV)
    v = gi.randn((B, 8, cap, 128), 3).half().to(DEV)
    o = dense_kernel.dense_decode_attention(q, k, v, seq_len=L)
    assert _err(o, oa.dense_attention(q.float(), k[:, :, :L].float(), v[:, :, :L].float())) < TOL


def test_dense_seq_len_zero_is_nan_like_reference():
    q = torch.randn(2, 64, 128, device=DEV).half()
    k = torch.randn(2, 8, 16, 128, device=DEV).half()
    o = dense_kernel.dense_decode_attention(q, k, k, seq_len=0)
    assert torch.isnan(o.float()).all()


@pytest.mark.parametrize("name", fixtures.names("sparse"))
def test_sparse_matches_reference_golden(name):
    meta, arrays = fixtures.load(name)
    L, W, seed, B = meta["seq_len"], meta["window"], meta["seed"], meta["batch"]
    q = gi.randn((B, 64, 128), seed)
    kf = gi.randn((B, 8, L, 128), seed + 100)
    vf = gi.randn((B, 8, L, 128), seed + 200)
    kc, vc = oa.build_compacted_cache(kf, vf, L, W, 4)  # GARBAGE_VALUE in unpopulated slots
    o = sparse_kernel.sparse_decode_attention(q.half().to(DEV), kc.half().to(DEV), vc.half().to(DEV),
                                              seq_len=L, window=W)
    assert _err(o, torch.from_numpy(arrays["o"])) < TOL
    ref = oa.sparse_attention_full(q.half().float(), kf.half().float(), vf.half().float(), L, W, 4)
    assert _err(o, ref) < TOL
    # same context in the ring-buffer layout
    kr, vr, head = oa.build_ring_cache(kf, vf, L, W, 4)
    o2 = sparse_kernel.sparse_decode_attention(q.half().to(DEV), kr.half().to(DEV), vr.half().to(DEV),
                                               seq_len=L, window=W, ring_head=head)
    assert _err(o2, ref) < TOL


@pytest.mark.parametrize("L,W", [(2, 256), (100, 256), (5000, 256), (2, 0), (10_000, 0), (163_840, 256),
                                 (261, 256), (300, 32), (4100, 4096), (20_000, 1024)])
def test_sparse_reference_cases_full_batch(L, W):
    """test_sparse_correctness.py:83-89 cases at B=32 plus wrap-around."""
    B = 32
    g = torch.Generator(device=DEV).manual_seed(L * 7 + W)
    q = torch.randn(B, 64, 128, device=DEV, generator=g).half()
    S = 4
    # attended positions: the sink and the last W tokens (no double counting)
    pos = list(range(min(S, L))) + list(range(max(S, L - W), L))
    kv_pos = torch.randn(B, 8, len(pos), 128, device=DEV, generator=g).half()
    vv_pos = torch.randn(B, 8, len(pos), 128, device=DEV, generator=g).half()
    # compacted and ring caches; every slot not holding an attended position
    # keeps GARBAGE_VALUE (test_sparse_correctness.py:15)
    kc = torch.full((B, 8, S + W, 128), oa.GARBAGE_VALUE, device=DEV).half()
    vc = kc.clone()
    kr, vr = kc.clone(), kc.clone()
    for j, p in enumerate(pos):
        cs = p if p < S else S + p - (L - W)
        rs = p if p < S else S + (p - S) % W
        kc[:, :, cs], vc[:, :, cs] = kv_pos[:, :, j], vv_pos[:, :, j]
        kr[:, :, rs], vr[:, :, rs] = kv_pos[:, :, j], vv_pos[:, :, j]
    ref = oa.dense_attention(q.float(), kv_pos.float(), vv_pos.float())
    o = sparse_kernel.sparse_decode_attention(q, kc, vc, seq_len=L, window=W)
    assert _err(o, ref) < TOL
    head = (L - S) % W if (W > 0 and L > S) else 0
    o2 = sparse_kernel.sparse_decode_attention(q, kr, vr, seq_len=L, window=W, ring_head=head)
    assert _err(o2, ref) < TOL


@pytest.mark.parametrize("B,W", [(6, 1020), (6, 256), (30, 256), (24, 380), (20, 60)])
def test_sparse_ragged_per_sequence_lengths(B, W):
    """Per-sequence seq_lens and ring heads: each row equals a B=1 call
    (W=1020: the persistent kernel, units split over the SMs; W + S <= 384:
    one CTA per unit at any batch, with 260 / 384 / 64 slots in 3 / 4 / 1
    tiles, and 48 units -- fewer than the SMs -- at B=6)."""
    S = 4
    lens = ([1, 3, 100, 260, 261, 5000] * 6)[:B]
    lens = [L + (i // 6) * 7 for i, L in enumerate(lens)]
    q = torch.randn(B, 64, 128, device=DEV).half()
    k = torch.randn(B, 8, S + W, 128, device=DEV).half()
    v = torch.randn(B, 8, S + W, 128, device=DEV).half()
    heads = [((L - S) % W if L > S else 0) for L in lens]
    o = sparse_kernel.sparse_decode_attention(
        q, k, v, seq_len=max(lens), window=W,
        seq_lens=torch.tensor(lens, dtype=torch.int64, device=DEV),
        ring_head=torch.tensor(heads, dtype=torch.int32, device=DEV))
    for b, L in enumerate(lens):
        ref = oa.sparse_attention_slots(q[b:b + 1].float(), k[b:b + 1].float(), v[b:b + 1].float(), L, W, S,
                                        ring_head=heads[b])
        assert _err(o[b:b + 1], ref) < TOL


def test_errors_are_python_exceptions():
    q = torch.randn(2, 64, 128, device=DEV).half()
    k = torch.randn(2, 8, 16, 128, device=DEV).half()
    with pytest.raises(TypeError):
        dense_kernel.dense_decode_attention(q.float(), k, k, seq_len=16)
    with pytest.raises(ValueError):
        dense_kernel.dense_decode_attention(q, k, k, seq_len=17)
    with pytest.raises(ValueError):
        dense_kernel.dense_decode_attention(q[:, :32], k, k, seq_len=16)
    with pytest.raises(ValueError):
        sparse_kernel.sparse_decode_attention(q, k, k, seq_len=16, window=11)


def test_no_device_error_recorded():
    import importlib
    pkg = importlib.import_module("numerics-and-sparse-attn_b200")
    assert pkg.device_error() == 0


@pytest.mark.parametrize("mode", ["stream", "unit", "auto"])
def test_split_modes_and_workspace_reuse(mode, monkeypatch):
    """Stream-K (split units, in-launch combine) and unit-aligned schedules
    give the same answer, and one workspace serves calls of changing shape
    back to back (the combine leaves it zeroed for any later layout)."""
    monkeypatch.setenv("NSA_SPLIT_MODE", mode)
    for kind, B, W, L in [("dense", 2, 0, 1000), ("dense", 32, 0, 4096), ("sparse", 2, 4096, 4100),
                          ("dense", 32, 0, 2049), ("sparse", 32, 2044, 4000), ("sparse", 32, 4096, 4100),
                          ("dense", 32, 0, 4100), ("sparse", 8, 256, 5000)]:
        g = torch.Generator(device=DEV).manual_seed(B * 1000 + L)
        q = torch.randn(B, 64, 128, device=DEV, generator=g).half()
        if kind == "dense":
            k = torch.randn(B, 8, L, 128, device=DEV, generator=g).half()
            v = torch.randn(B, 8, L, 128, device=DEV, generator=g).half()
            o = dense_kernel.dense_decode_attention(q, k, v, seq_len=L)
            ref = oa.dense_attention(q.float(), k.float(), v.float())
        else:
            k = torch.randn(B, 8, 4 + W, 128, device=DEV, generator=g).half()
            v = torch.randn(B, 8, 4 + W, 128, device=DEV, generator=g).half()
            o = sparse_kernel.sparse_decode_attention(q, k, v, seq_len=L, window=W)
            ref = oa.sparse_attention_slots(q.float(), k.float(), v.float(), L, W, 4)
        assert _err(o, ref) < TOL, (mode, kind, B, W, L)
