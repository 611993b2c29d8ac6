"""Batch shards for the multi-GPU forward: one process per GPU, no collective in the hot path.

Every sequence of the enGPT forward is independent: the embedding, the QKV
epilogue, the carried residual and the cross-entropy are per token, and the
causal attention is per (sequence, head) (engpt/models.py:140-182, 263-292).
A global batch therefore splits over ranks by sequence rows, each rank runs
the whole forward on its rows, and the only communication is after the
forward:

* the loss, a mean over the non-ignored targets (``F.cross_entropy`` with
  ``ignore_index=-100``, engpt/models.py:328-339), is combined as a
  token-weighted mean: one all-reduce of ``(loss * n_valid, n_valid)``;
* logits (or the final ``Y / rho``) are collected with one all-gather,
  padded to the largest shard when the batch does not divide evenly.

The functions take an optional ``group`` and work with any
``torch.distributed`` backend: NCCL on GPUs, gloo for the CPU tests.
"""

from __future__ import annotations

from typing import Callable, Optional, Tuple

import torch
import torch.distributed as dist
from torch import Tensor

IGNORE_INDEX = -100


def _world(group) -> Tuple[int, int]:
    if not dist.is_available() or not dist.is_initialized():
        return 0, 1
    return dist.get_rank(group), dist.get_world_size(group)


def shard_range(batch: int, rank: int, world: int) -> Tuple[int, int]:
    """Rows ``[start, stop)`` of a ``batch``-row global batch owned by ``rank``.

    Contiguous shards; the first ``batch % world`` ranks take one extra row, so
    shard sizes differ by at most one.  A rank may own zero rows.
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} out of range for world size {world}")
    if batch < 0:
        raise ValueError("batch must be >= 0")
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_rows(t: Tensor, rank: int, world: int) -> Tensor:
    """This rank's rows of a global-batch tensor (a view, dim 0 = sequences)."""
    s, e = shard_range(t.shape[0], rank, world)
    return t[s:e]


def valid_targets(targets: Optional[Tensor]) -> Tensor:
    """Number of targets that count toward the mean loss (ignore_index excluded), as a device scalar."""
    if targets is None:
        return torch.zeros((), dtype=torch.int64)
    return (targets != IGNORE_INDEX).sum()


def combine_loss(loss: Optional[Tensor], n_valid, *, device=None, group=None) -> Tensor:
    """Global mean loss over all ranks' valid targets, without a host synchronisation.

    ``loss`` is this rank's mean over its ``n_valid`` targets (an int or a
    scalar tensor; ``loss`` may be None for an empty shard).  Every rank gets
    the same fp32 scalar, NaN when no rank has a valid target; it equals the
    loss of the unsharded batch up to summation order.
    """
    dev = device if device is not None else (loss.device if loss is not None else torch.device("cpu"))
    n = torch.as_tensor(n_valid, dtype=torch.float64, device=dev).reshape(())
    if loss is None:
        num = torch.zeros((), dtype=torch.float64, device=dev)
    else:
        num = torch.where(n > 0, loss.detach().to(device=dev, dtype=torch.float64) * n, 0.0)
    part = torch.stack([num, n])
    _, world = _world(group)
    if world > 1:
        dist.all_reduce(part, op=dist.ReduceOp.SUM, group=group)
    return torch.where(part[1] > 0, part[0] / part[1], float("nan")).to(torch.float32)


def gather_rows(local: Tensor, batch: int, *, group=None) -> Tensor:
    """All-gather per-rank row shards (``shard_range`` layout) into the ``batch``-row tensor on every rank."""
    rank, world = _world(group)
    if world == 1:
        return local
    s, e = shard_range(batch, rank, world)
    if local.shape[0] != e - s:
        raise ValueError(f"rank {rank} holds {local.shape[0]} rows, its shard has {e - s}")
    if batch % world == 0:
        # equal shards: one collective straight into the output
        out = local.new_empty((batch,) + tuple(local.shape[1:]))
        dist.all_gather_into_tensor(out, local.contiguous(), group=group)
        return out
    rows = -(-batch // world)  # largest shard
    buf = local.new_zeros((rows,) + tuple(local.shape[1:]))
    buf[: local.shape[0]].copy_(local)
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf.contiguous(), group=group)
    out = [parts[r][: shard_range(batch, r, world)[1] - shard_range(batch, r, world)[0]] for r in range(world)]
    return torch.cat(out, dim=0)


def forward_sharded(forward: Callable[[Tensor, Optional[Tensor]], Tuple[Tensor, Optional[Tensor]]],
                    idx: Tensor, targets: Optional[Tensor] = None, *, group=None,
                    gather_logits: bool = True) -> Tuple[Optional[Tensor], Optional[Tensor]]:
    """Run ``forward`` (e.g. ``EfficientNGPT.__call__``) on this rank's rows of a global batch.

    ``idx`` / ``targets`` are the global ``[B, T]`` batch, identical on every
    rank.  Returns ``(logits, loss)``: the loss is the global token-weighted
    mean on every rank; the logits are the full ``[B, T, V]`` batch on every
    rank when ``gather_logits`` is true, else this rank's shard.
    """
    rank, world = _world(group)
    B = idx.shape[0]
    if gather_logits and B < world:
        # every rank sees the same global batch, so every rank raises here, before any collective
        raise ValueError(f"gather_logits needs at least one row per rank (batch {B} < world size {world})")
    my_idx = shard_rows(idx, rank, world)
    my_tgt = shard_rows(targets, rank, world) if targets is not None else None
    if my_idx.shape[0] > 0:
        logits, loss = forward(my_idx, my_tgt)
    else:
        logits, loss = None, None
    out_loss = None
    if targets is not None:
        out_loss = combine_loss(loss, valid_targets(my_tgt), device=idx.device, group=group)
    if not gather_logits:
        return logits, out_loss
    return gather_rows(logits, B, group=group), out_loss
