"""Megatron-style tensor parallelism for compressed linears (one process per
GPU, ``torch.distributed`` over NCCL).

Column-parallel layers (qkv, gate_up) split W by output rows: every rank
packs and multiplies its own [M/tp, K] shard and produces [N, M/tp] with no
collective. Row-parallel layers (o, down) split W by K: every rank packs its
[M, K/tp] shard, multiplies the matching K/tp slice of the activations and the
[N, M] partial outputs are summed with one all-reduce. Every rank packs its
own shard, so each has its own exponent window and packed maxima. Shards
must stay 64-aligned (M/tp and K/tp multiples of 64).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist
from torch import Tensor

from . import runtime

COLUMN, ROW = "column", "row"


def shard_bounds(size: int, world: int, rank: int) -> tuple[int, int]:
    """[begin, end) of rank's equal share of `size`; shares must be 64-aligned."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must lie in [0, world)")
    if size % world or (size // world) % 64:
        raise ValueError(f"{size} does not split into {world} shards that are multiples of 64")
    share = size // world
    return rank * share, (rank + 1) * share


def shard_weight(weight: Tensor, kind: str, world: int, rank: int) -> Tensor:
    """This rank's contiguous shard of an [M, K] weight."""
    m, k = weight.shape
    if kind == COLUMN:
        r0, r1 = shard_bounds(m, world, rank)
        return weight[r0:r1].contiguous()
    if kind == ROW:
        c0, c1 = shard_bounds(k, world, rank)
        return weight[:, c0:c1].contiguous()
    raise ValueError("kind must be 'column' or 'row'")


@dataclass
class ParallelLinear:
    """One rank's part of a tensor-parallel compressed linear."""

    packed: runtime.PackedWeight
    kind: str
    world: int
    rank: int
    group: object = None

    @classmethod
    def from_weight(cls, weight: Tensor, kind: str, world: int, rank: int,
                    device: torch.device | str, group=None) -> "ParallelLinear":
        shard = shard_weight(weight, kind, world, rank)
        return cls(runtime.compress(shard).to(device), kind, world, rank, group)

    def forward(self, x: Tensor, linear=None) -> Tensor:
        """Column: x [.., K] -> [.., M/tp]. Row: x [.., K] (full width; the
        rank takes its K slice) -> [.., M], all-reduced over the group.
        `linear` defaults to runtime.linear."""
        linear = runtime.linear if linear is None else linear
        if self.kind == COLUMN:
            return linear(x, self.packed)
        c0, c1 = shard_bounds(x.shape[-1], self.world, self.rank)
        y = linear(x[..., c0:c1].contiguous(), self.packed)
        if self.world > 1:
            dist.all_reduce(y, group=self.group)
        return y
