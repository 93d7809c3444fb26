"""Multi-process logic of the sharded decode on CPU: 2 gloo ranks each run
the fp32 oracle on their shard of the unit grid, the outputs are assembled
with the same all-gather the GPU path uses, and the MAX-over-ranks timing
reduction is checked; a rank that leaves between steps is detected by the
others as an error of their next collective within the group's timeout, not
a hang.  (The GPU kernels themselves are covered by -m gpu.)"""
import datetime
import importlib
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

shard = importlib.import_module("numerics-and-sparse-attn_b200.shard")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, batch, hkv, ret):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import attention as oa
        g = torch.Generator().manual_seed(11)
        q = torch.randn(batch, hkv * 8, 128, generator=g)
        k = torch.randn(batch, hkv, 40, 128, generator=g)
        v = torch.randn(batch, hkv, 40, 128, generator=g)
        sh = shard.shard_units(batch, hkv, world, rank)
        o_local = oa.dense_attention(sh.q_slice(q), sh.kv_slice(k), sh.kv_slice(v))
        full = shard.gather_outputs(o_local, batch, hkv)
        worst = shard.max_over_ranks(float(rank + 1))
        if rank == 0:
            ref = oa.dense_attention(q, k, v)
            ret["err"] = (full - ref).abs().max().item()
            ret["max"] = worst
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("batch,hkv", [(4, 8), (3, 8), (1, 8)])
def test_sharded_decode_assembles_full_output(batch, hkv):
    world = 2
    with mp.Manager() as m:
        ret = m.dict()
        mp.spawn(_worker, args=(world, _free_port(), batch, hkv, ret), nprocs=world, join=True)
        assert ret["err"] < 1e-6
        assert ret["max"] == world


def test_shard_units_cover_grid_exactly_once():
    for batch, hkv, world in [(32, 8, 1), (32, 8, 2), (32, 8, 8), (256, 8, 8), (5, 8, 2), (1, 8, 8), (2, 8, 8)]:
        seen = torch.zeros(batch, hkv, dtype=torch.int32)
        for r in range(world):
            s = shard.shard_units(batch, hkv, world, r)
            seen[s.b0:s.b1, s.h0:s.h1] += 1
        assert (seen == 1).all(), (batch, hkv, world)
    with pytest.raises(ValueError):
        shard.shard_units(3, 8, 8, 0)


def _dropout_worker(rank, world, port, ret):
    """Step 1 completes on both ranks; rank 1 then leaves (between steps, with
    nothing in flight) and rank 0's step-2 all-gather must fail, not hang."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    o_local = torch.full((1, 8, 128), float(rank))
    full = shard.gather_outputs(o_local, world, 1)
    ret[f"step1_{rank}"] = float(full.sum())
    if rank == 1:
        return  # leaves without destroying the group: its peer sees a lost rank
    t0 = time.monotonic()
    try:
        shard.gather_outputs(o_local, world, 1)
        ret["step2"] = "completed"
    except Exception as e:  # gloo reports the lost peer or the timeout
        ret["step2"] = type(e).__name__
    ret["seconds"] = time.monotonic() - t0


def test_rank_leaving_is_detected_not_hung():
    world = 2
    with mp.Manager() as m:
        ret = m.dict()
        mp.spawn(_dropout_worker, args=(world, _free_port(), ret), nprocs=world, join=True)
        assert ret["step1_0"] == ret["step1_1"] == 8 * 128.0
        assert ret["step2"] != "completed"
        assert ret["seconds"] < 30
