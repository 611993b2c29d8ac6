"""Multi-GPU host logic (batch shards, loss combine, logits gather) on CPU with gloo ranks.

The per-shard forward is the oracle (CPU stand-in for the GPU engine): the
sharded run over world_size 2 must reproduce the unsharded oracle forward of
the whole batch, logits row for row and the loss as the token-weighted mean
over non-ignored targets (F.cross_entropy semantics, engpt/models.py:328-333).
"""

import multiprocessing as mp
import os
import socket
import tempfile

import numpy as np
import pytest
import torch

from engpt_b200 import sharding
from oracle import ngpt_oracle as O

SMALL = dict(vocab_size=32, block_size=12, n_layer=2, n_head=2, n_embd=32, mlp_ratio=2.0, alpha_init=0.1)


def test_shard_range_partitions_every_batch():
    for world in (1, 2, 3, 4, 8):
        for batch in range(0, 19):
            spans = [sharding.shard_range(batch, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == batch
            for (s0, e0), (s1, e1) in zip(spans, spans[1:]):
                assert e0 == s1
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1 and sizes == sorted(sizes, reverse=True)
    with pytest.raises(ValueError):
        sharding.shard_range(4, 2, 2)


def test_single_process_passthrough():
    logits = torch.randn(3, 4, 5)
    assert sharding.gather_rows(logits, 3) is logits
    loss = sharding.combine_loss(torch.tensor(2.5), 7)
    assert loss.item() == pytest.approx(2.5)
    assert torch.isnan(sharding.combine_loss(None, 0))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_forward(weights, cfg):
    def forward(idx, targets):
        logits, loss, _ = O.efficient_ngpt_forward(cfg, weights, idx.numpy(),
                                                   None if targets is None else targets.numpy())
        return torch.from_numpy(logits), (None if loss is None else torch.tensor(loss, dtype=torch.float64))
    return forward


def _worker(rank, world, port, weights, idx, targets, out_dir):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        fwd = _oracle_forward(weights, O.OracleConfig(**SMALL))
        logits, loss = sharding.forward_sharded(fwd, torch.from_numpy(idx), torch.from_numpy(targets))
        # batch 1 < world 2 with a logits gather: every rank raises before any collective (no rank is left
        # waiting in the all-gather), and the group stays usable for the call after it
        try:
            sharding.forward_sharded(fwd, torch.from_numpy(idx[:1]), torch.from_numpy(targets[:1]))
            raised = False
        except ValueError:
            raised = True
        # an empty shard on the last rank: loss only, no gather
        _, loss1 = sharding.forward_sharded(fwd, torch.from_numpy(idx[:1]), torch.from_numpy(targets[:1]),
                                            gather_logits=False)
        # equal shards (2 rows over 2 ranks): the gather goes straight into the output tensor
        logits2, _ = sharding.forward_sharded(fwd, torch.from_numpy(idx[:2]), torch.from_numpy(targets[:2]))
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), logits=logits.numpy(), loss=loss.item(),
                 loss1=loss1.item(), raised=raised, logits2=logits2.numpy())
    finally:
        dist.destroy_process_group()


def test_forward_sharded_world2_matches_unsharded(golden):
    g = golden("model_small.npz")
    weights = {k[2:]: g[k] for k in g if k.startswith("w:")}
    rng = np.random.default_rng(5)
    B, T = 3, SMALL["block_size"]  # 3 rows over 2 ranks: ragged shards (2 + 1)
    idx = rng.integers(0, SMALL["vocab_size"], (B, T))
    targets = rng.integers(0, SMALL["vocab_size"], (B, T))
    targets[0, :5] = -100  # ignored targets make the shards' valid counts unequal
    targets[2, 7] = -100
    cfg = O.OracleConfig(**SMALL)
    ref_logits, ref_loss, _ = O.efficient_ngpt_forward(cfg, weights, idx, targets)
    _, ref_loss1, _ = O.efficient_ngpt_forward(cfg, weights, idx[:1], targets[:1])
    ref_logits2, _, _ = O.efficient_ngpt_forward(cfg, weights, idx[:2], targets[:2])

    ctx = mp.get_context("spawn")
    port = _free_port()
    with tempfile.TemporaryDirectory() as out_dir:
        procs = [ctx.Process(target=_worker, args=(r, 2, port, weights, idx, targets, out_dir)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
        for p in procs:
            if p.is_alive():
                p.kill()
                p.join()
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        res = [dict(np.load(os.path.join(out_dir, f"rank{r}.npz"))) for r in range(2)]
    for r in res:
        np.testing.assert_allclose(r["logits"], ref_logits, rtol=1e-12, atol=1e-12)
        assert abs(float(r["loss"]) - ref_loss) <= 1e-6 * abs(ref_loss)  # combined in fp64, returned fp32
        assert abs(float(r["loss1"]) - ref_loss1) <= 1e-6 * abs(ref_loss1)
        assert bool(r["raised"])
        np.testing.assert_allclose(r["logits2"], ref_logits2, rtol=1e-12, atol=1e-12)
