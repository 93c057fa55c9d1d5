"""Work sharding across GPUs for the prefill path.

(batch, v-head) units are independent, so the path shards with no
communication on the data path:

* ``batch_shard``: rank r of N takes batch rows [r*B/N, (r+1)*B/N) (BASELINE
  config 4), with the matching initial/final states.
* ``head_shard``: rank r takes v-heads [r*HV/N, (r+1)*HV/N) and the qk-heads
  they read under ``hq = h // (HV/HQK)`` (kernels/chunk_delta_cuda.h:12-14),
  which needs (HV/N) to be a multiple of (HV/HQK) so each rank owns whole qk
  groups (4 v-heads and 2 qk-heads per GPU at N=8).

Collectives are used only outside the timed region, to gather outputs for
verification (``gather_shards``).
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class HeadShard:
    v0: int
    v1: int
    q0: int
    q1: int


def batch_shard(B: int, world: int, rank: int) -> tuple[int, int]:
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    if B % world:
        raise ValueError(f"batch {B} does not split evenly over {world} ranks")
    per = B // world
    return rank * per, (rank + 1) * per


def head_shard(HV: int, HQK: int, world: int, rank: int) -> HeadShard:
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    if HV % world:
        raise ValueError(f"{HV} v-heads do not split over {world} ranks")
    group = HV // HQK
    per = HV // world
    if per % group:
        raise ValueError(f"{per} v-heads per rank do not cover whole qk groups of {group}")
    v0, v1 = rank * per, (rank + 1) * per
    return HeadShard(v0, v1, v0 // group, v1 // group)


def slice_heads(shard: HeadShard, q, k, v, g, beta, z=None, s0=None):
    """Slice [B,T,H,*] inputs (and [B,HV,*] state) to one head shard (views)."""
    out = [q[:, :, shard.q0:shard.q1], k[:, :, shard.q0:shard.q1], v[:, :, shard.v0:shard.v1],
           g[:, :, shard.v0:shard.v1], beta[:, :, shard.v0:shard.v1]]
    out.append(None if z is None else z[:, :, shard.v0:shard.v1])
    out.append(None if s0 is None else s0[:, shard.v0:shard.v1])
    return out


def gather_shards(local, world: int, dim: int):
    """all_gather a tensor shard along ``dim`` (verification only, outside timing)."""
    import torch
    import torch.distributed as dist
    parts = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(parts, local.contiguous())
    return torch.cat(parts, dim=dim)
