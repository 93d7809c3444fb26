"""Multi-GPU plumbing for decode attention: one process per GPU.

Every (batch row, KV head) unit is independent, so the work shards with no
collective on the decode path.  Rows are split batch-major; when there are
fewer rows than ranks the KV heads of a row are split instead.  Outputs are
assembled with one all-gather only to verify or hand results to a host, and
step times are reduced with a MAX over ranks.  Works with any
torch.distributed backend (NCCL on GPUs; gloo for the CPU tests).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class Shard:
    """Slice of the [batch, kv_heads] unit grid owned by one rank."""
    b0: int
    b1: int
    h0: int
    h1: int

    @property
    def n_rows(self) -> int:
        return self.b1 - self.b0

    @property
    def n_kv_heads(self) -> int:
        return self.h1 - self.h0

    def q_slice(self, q: torch.Tensor, group: int = 8) -> torch.Tensor:
        """Rows and query heads of q [B, H, D] belonging to this shard."""
        return q[self.b0:self.b1, self.h0 * group:self.h1 * group]

    def kv_slice(self, kv: torch.Tensor) -> torch.Tensor:
        """Rows and KV heads of a cache [B, Hkv, ...] belonging to this shard."""
        return kv[self.b0:self.b1, self.h0:self.h1]


def shard_units(batch: int, n_kv_heads: int, world: int, rank: int) -> Shard:
    """Batch-major split of the unit grid over ``world`` ranks.

    batch >= world: contiguous row ranges (sizes differ by at most one),
    all KV heads.  batch < world: ranks are spread over rows first, then the
    KV heads of each row are split among the ranks sharing it."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("need 0 <= rank < world")
    if batch >= world:
        return Shard(rank * batch // world, (rank + 1) * batch // world, 0, n_kv_heads)
    per_row = world // batch
    if per_row > n_kv_heads or world % batch:
        raise ValueError(f"cannot split {batch} rows x {n_kv_heads} kv heads over {world} ranks evenly")
    row, part = divmod(rank, per_row)
    return Shard(row, row + 1, part * n_kv_heads // per_row, (part + 1) * n_kv_heads // per_row)


def max_over_ranks(value: float, device=None) -> float:
    """MAX of a host scalar over all ranks (identity without a process group)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_outputs(o_local: torch.Tensor, batch: int, n_kv_heads: int, group: int = 8) -> torch.Tensor:
    """Assemble the full o [batch, n_kv_heads*group, D] from every rank's shard
    (all ranks receive it).  Shards of unequal size are padded to the largest
    for the collective."""
    world, rank = dist.get_world_size(), dist.get_rank()
    shards = [shard_units(batch, n_kv_heads, world, r) for r in range(world)]
    d = o_local.shape[-1]
    max_rows = max(s.n_rows for s in shards)
    max_heads = max(s.n_kv_heads for s in shards) * group
    buf = torch.zeros(max_rows, max_heads, d, dtype=o_local.dtype, device=o_local.device)
    buf[:o_local.shape[0], :o_local.shape[1]] = o_local
    flat = torch.empty((world * max_rows,) + tuple(buf.shape[1:]), dtype=buf.dtype, device=buf.device)
    dist.all_gather_into_tensor(flat, buf)  # concatenated along dim 0 (gloo and NCCL)
    allb = flat.view((world,) + tuple(buf.shape))
    out = torch.empty(batch, n_kv_heads * group, d, dtype=o_local.dtype, device=o_local.device)
    for r, s in enumerate(shards):
        out[s.b0:s.b1, s.h0 * group:s.h1 * group] = allb[r, :s.n_rows, :s.n_kv_heads * group]
    del rank
    return out
