"""Splitting one sequence's forward over a group of GPUs by heads and MLP units.

The long-context configuration (one 8192-token sequence per pair of GPUs)
cannot be split by batch alone, so a group of ``size`` ranks shares each
sequence.  Rank ``r`` of the group owns

* the heads ``[r H/size, (r+1) H/size)``: their rows of the QKV projection,
  the QKV post-process and the causal attention of those heads, and the
  matching columns of out_proj (engpt/models.py:142-152);
* the MLP units ``[r W/size, (r+1) W/size)``: their u and gate rows of the
  up/gate projection, their SwiGLU, and the matching columns of down_proj
  (engpt/models.py:163-172).

out_proj and down_proj then give each rank a partial branch (the sum over its
heads or units); one all-reduce (sum) over the group before each carried
residual (engpt/kernels.py:277-324) gives every rank the full branch, so the
carried state ``(Y, rho)``, the embedding and the output head are computed
identically on every rank of the group.  Two all-reduces of ``[tokens, d]``
bf16 per layer are the only communication; every GEMM and the attention are
split evenly.

The group's collectives go through ``torch.distributed`` (NCCL between GPUs).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist


@dataclass
class HeadSplit:
    """This rank's share of the heads and MLP units in a head-split group."""

    rank: int
    size: int
    group: Optional[object] = None     # torch.distributed process group of the ranks sharing the sequences

    def validate(self, n_head: int, mlp_width: int) -> None:
        if self.size < 1 or not 0 <= self.rank < self.size:
            raise ValueError(f"head split rank {self.rank} of {self.size}")
        if n_head % self.size or mlp_width % self.size:
            raise ValueError(f"{n_head} heads and {mlp_width} MLP units do not split {self.size} ways")

    def heads(self, n_head: int):
        k = n_head // self.size
        return self.rank * k, (self.rank + 1) * k

    def units(self, mlp_width: int):
        k = mlp_width // self.size
        return self.rank * k, (self.rank + 1) * k

    def key(self):
        return (self.rank, self.size)

    def all_reduce_(self, t: torch.Tensor) -> None:
        """Sum ``t`` over the group in place (identical result on every rank)."""
        if self.size == 1:
            return
        if dist.get_backend(self.group) == "gloo" and t.is_cuda:
            # the CPU test harness (several processes on one GPU): gloo reduces host tensors
            host = t.cpu()
            dist.all_reduce(host, group=self.group)
            t.copy_(host)
            return
        dist.all_reduce(t, group=self.group)


def pair_groups(world: int, size: int):
    """Head-split groups of ``size`` consecutive ranks and, across them, the data-parallel groups.

    Every rank must call this (``torch.distributed.new_group`` is collective),
    in the same order.  Returns ``(split_groups, dp_groups)``: ``split_groups[i]``
    holds ranks ``[i size, (i+1) size)``; ``dp_groups[j]`` holds the ranks with
    index ``j`` in their split group.
    """
    if world % size:
        raise ValueError(f"world size {world} is not a multiple of the head-split size {size}")
    split_groups = [dist.new_group(list(range(i * size, (i + 1) * size))) for i in range(world // size)]
    dp_groups = [dist.new_group(list(range(j, world, size))) for j in range(size)]
    return split_groups, dp_groups
