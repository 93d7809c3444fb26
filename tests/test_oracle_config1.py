"""The CPU-runnable sparse decode configuration: fp32, batch 2, 8 query heads
over 2 KV heads (GQA group 4), head_dim 128, context L=2048, sink S=4,
window W=256, one decode query, Q/K/V ~ N(0,1) from seed 0; the output is
compared against dense causal attention masked to the sink+window positions.

The reference's own oracle (test_sparse_correctness.py:22-48) hard-codes the
group as the module constant GQA_GROUP = 8 (its line 41-42
``repeat_interleave(GQA_GROUP, dim=1)``), so it cannot express a group of 4;
the restatement in oracle/attention.py derives the group from the shapes.
These tests show that it does so correctly at group 4, three ways:

* ``sparse_attention_full`` (the StreamingLLM mask over the full context)
  against dense attention over only the attended positions (gathered first);
* ``sparse_attention_slots`` over the compacted cache
  (test_sparse_correctness.py:51-72) and over the ring layout;
* all of them against a float64 per-(batch, head) loop that maps query head h
  to KV head h // 4 explicitly.  CPU only.
"""
import math

import torch

from oracle import attention as oa

B, H, HKV, D, L, S, W = 2, 8, 2, 128, 2048, 4, 256


def _inputs():
    torch.manual_seed(0)
    q = torch.randn(B, H, D, dtype=torch.float32)
    k = torch.randn(B, HKV, L, D, dtype=torch.float32)
    v = torch.randn(B, HKV, L, D, dtype=torch.float32)
    return q, k, v


def _attended_positions():
    return [p for p in range(L) if p < S or p >= L - W]


def _loop_reference(q, k, v, positions):
    """float64, one (batch, query head) at a time: head h reads KV head h // 4."""
    group = H // HKV
    idx = torch.tensor(positions)
    out = torch.empty(B, H, D, dtype=torch.float64)
    for b in range(B):
        for h in range(H):
            kk = k[b, h // group, idx].double()
            vv = v[b, h // group, idx].double()
            s = kk @ q[b, h].double() / math.sqrt(D)
            p = torch.softmax(s, dim=0)
            out[b, h] = p @ vv
    return out


def test_config1_masked_full_context_equals_dense_over_attended():
    q, k, v = _inputs()
    o_full = oa.sparse_attention_full(q, k, v, L, W, S)
    pos = torch.tensor(_attended_positions())
    assert pos.numel() == S + W
    o_dense = oa.dense_attention(q, k[:, :, pos], v[:, :, pos])
    assert o_full.shape == (B, H, D) and o_full.dtype == torch.float32
    assert (o_full - o_dense).abs().max().item() < 1e-5
    o64 = _loop_reference(q, k, v, pos.tolist())
    assert (o_full.double() - o64).abs().max().item() < 1e-5


def test_config1_slot_forms_equal_the_masked_oracle():
    q, k, v = _inputs()
    o_full = oa.sparse_attention_full(q, k, v, L, W, S)
    kc, vc = oa.build_compacted_cache(k, v, L, W, S)
    assert kc.shape == (B, HKV, S + W, D)
    o_compact = oa.sparse_attention_slots(q, kc, vc, L, W, S)
    assert (o_compact - o_full).abs().max().item() < 1e-5
    kr, vr, head = oa.build_ring_cache(k, v, L, W, S)
    assert head == (L - S) % W
    o_ring = oa.sparse_attention_slots(q, kr, vr, L, W, S, ring_head=head)
    assert (o_ring - o_full).abs().max().item() < 1e-5


def test_config1_group_of_four_is_not_group_of_eight():
    """Query heads 0-3 read KV head 0 and 4-7 read KV head 1: swapping the
    two KV heads moves exactly those halves of the output (a group hard-coded
    at 8 would send all eight query heads to KV head 0)."""
    q, k, v = _inputs()
    o = oa.sparse_attention_full(q, k, v, L, W, S)
    o_sw = oa.sparse_attention_full(q, k.flip(1), v.flip(1), L, W, S)
    assert not torch.allclose(o[:, :4], o_sw[:, :4])
    q_sw = torch.cat([q[:, 4:], q[:, :4]], dim=1)
    o_both = oa.sparse_attention_full(q_sw, k.flip(1), v.flip(1), L, W, S)
    assert (o_both[:, :4] - o[:, 4:]).abs().max().item() < 1e-6
    assert (o_both[:, 4:] - o[:, :4]).abs().max().item() < 1e-6
