"""CPU checks of the streaming-KIVI oracle model (oracle/kivi.py): it has no
reference counterpart, so it is pinned to the reference's own builder
(build_quantized_kv_cache, itself pinned by the golden vectors) at the phases
where the two describe the same cache, and to StreamingLLM's attended set."""
import numpy as np
import pytest
import torch

import inputs as gi
from oracle import attention as oa
from oracle import kivi as ok


def _compare_groups(st, ref, order):
    np.testing.assert_array_equal(np.concatenate([st["k_win_packed"][:, :, s * 8:(s + 1) * 8] for s in order], 2),
                                  ref["k_win_packed"])
    np.testing.assert_array_equal(np.concatenate([st["k_win_scale"][:, :, s:s + 1] for s in order], 2),
                                  ref["k_win_scale"])
    np.testing.assert_array_equal(np.concatenate([st["v_win_packed"][:, :, s * 32:(s + 1) * 32] for s in order], 2),
                                  ref["v_win_packed"])
    np.testing.assert_array_equal(np.concatenate([st["v_win_scale"][:, :, s * 32:(s + 1) * 32] for s in order], 2),
                                  ref["v_win_scale"])


@pytest.mark.parametrize("W,extra", [(256, 0), (256, 32 * 3), (512, 32), (128, 64)])
def test_aligned_stream_state_equals_reference_builder(W, extra):
    S, R = 4, 128
    L = S + W + extra
    assert (L - S - R) % 32 == 0
    k = gi.kivi_k((1, 2, L, 128), W + extra).half()
    v = gi.randn((1, 2, L, 128), W + extra + 1).half()
    geom = ok.StreamGeometry(window=W, sink=S, residual=R)
    st = ok.stream_state(k, v, L, geom)
    kc, vc = oa.build_compacted_cache(k, v, L, W, S)
    ref = ok.build_quantized_kv_cache(kc, vc, R, S)
    for key in ("k_sink_packed", "k_sink_scale", "k_sink_zero", "v_sink_packed", "v_sink_scale", "v_sink_zero"):
        np.testing.assert_array_equal(st[key], ref[key])
    NG = (W - R) // 32
    F = geom.n_flushed(L)
    order = [(F - NG + j) % NG for j in range(NG)]
    assert all(st["grp_live"])
    if NG:
        _compare_groups(st, ref, order)
    res_order = [(32 * F + j) % geom.res_cap for j in range(R)]
    np.testing.assert_array_equal(st["k_res"][:, :, res_order], ref["k_residual"])
    q = gi.randn((1, 16, 128), 5).half()
    a = oa.stream_attention(q, st, L, geom)
    b = oa.quantized_attention(q, W - R, ref)
    assert (a - b).abs().max().item() < 1e-5


@pytest.mark.parametrize("W", [256, 32, 160])
def test_stream_attended_set_is_streamingllm(W):
    """With quantization removed (exact fp16 tokens everywhere), the tokens the
    model attends are exactly StreamingLLM's: first min(L, S) and p >= L - W."""
    S, R = 4, 128
    geom = ok.StreamGeometry(window=W, sink=S, residual=R)
    for L in [1, 3, 4, 5, 100, S + W, S + W + 1, S + R + 32, S + R + 33, S + W + 77, 700]:
        n_stream = max(0, L - S)
        F = geom.n_flushed(L)
        kept_res = list(range(S + 32 * F, L))
        kept_grp = [S + 32 * gi_ + j for gi_ in range(max(0, F - geom.n_groups), F) for j in range(32)]
        first = max(S, L - W)
        attended = list(range(min(L, S))) + [p for p in kept_grp + kept_res if p >= first]
        expect = list(range(min(L, S))) + list(range(first, L))
        assert sorted(attended) == expect, L
        assert n_stream - 32 * F <= R + 31
