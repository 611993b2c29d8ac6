"""Head split (engpt_b200.head_split): one sequence's heads and MLP units shared by a group of two ranks.

The group runs as two processes on the one GPU the test has, joined by a
gloo process group (the engine reduces the partial branches through it;
NCCL serves the same collectives between GPUs).  Each rank computes its
heads and units; after the all-reduce of every partial branch both ranks
hold the same carried state.  Checked: both ranks agree exactly, the split
forward matches the unsplit one (bf16: Y/rho 2e-2, loss 1e-3; fp32: 1e-5),
and the long-context configuration (L=24, d=2048, head_dim 128, T=8192)
split over two ranks matches the reference's fp32 forward (the fixture of
tests/golden/cfg5_d2048.npz).
"""

import multiprocessing as mp
import os
import socket
import tempfile

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, port, cfg_kw, batch, bf16_modes, golden_rows, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    import datetime
    import torch
    import torch.distributed as dist
    from engpt_b200 import EfficientNGPT, ModelConfig
    from engpt_b200.head_split import HeadSplit

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=600))
    try:
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        torch.backends.cuda.matmul.allow_tf32 = False
        torch.manual_seed(0)
        model = EfficientNGPT(ModelConfig(**cfg_kw)).to(dev).eval().requires_grad_(False)
        gen = torch.Generator().manual_seed(0)
        idx = torch.randint(0, cfg_kw["vocab_size"], (batch, cfg_kw["block_size"]), generator=gen)
        tgt = torch.roll(idx, -1, dims=1)
        res = {}
        for bf16 in bf16_modes:
            tag = "bf16" if bf16 else "fp32"
            for split in (True, False):
                if not split and rank == 1:
                    continue
                model.set_head_split(HeadSplit(rank, 2, dist.group.WORLD) if split else None)
                with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16, enabled=bf16):
                    _, loss, states = model.forward_with_states(idx.to(dev), tgt.to(dev))
                key = f"{tag}_{'split' if split else 'whole'}"
                res[key + "_loss"] = np.float64(loss.item())
                layers = golden_rows["layers"] if golden_rows else range(len(states))
                rows = golden_rows["rows"] if golden_rows else slice(None)
                for i in layers:
                    y, r = states[i]
                    h = (y[0] / r[0].unsqueeze(-1))[rows]
                    res[f"{key}_h{i}"] = h.float().cpu().numpy()
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **res)
    finally:
        dist.destroy_process_group()


def _run_group(cfg_kw, batch, bf16_modes, golden_rows=None):
    ctx = mp.get_context("spawn")
    port = _free_port()
    with tempfile.TemporaryDirectory() as out_dir:
        procs = [ctx.Process(target=_worker, args=(r, port, cfg_kw, batch, bf16_modes, golden_rows, out_dir))
                 for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=900)
        for p in procs:
            if p.is_alive():
                p.kill()
                p.join()
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        return [dict(np.load(os.path.join(out_dir, f"rank{r}.npz"))) for r in range(2)]


def _row_rel(a, b):
    num = np.sqrt(((np.asarray(a, np.float64) - b) ** 2).sum(-1))
    return float((num / np.maximum(np.sqrt((np.asarray(b, np.float64) ** 2).sum(-1)), 1e-30)).max())


@pytest.mark.parametrize("n_head", [8, 16])   # head_dim 128 and 64
def test_head_split_matches_whole_forward(cuda, n_head):
    cfg_kw = dict(vocab_size=1000, block_size=512, n_layer=3, n_head=n_head, n_embd=1024, mlp_ratio=4.0,
                  dropout=0.0)
    r0, r1 = _run_group(cfg_kw, 2, (True, False))
    for k in r0:
        if "split" in k:
            assert np.array_equal(r0[k], r1[k]), k           # both ranks of the group hold the same state
    for tag, tol, loss_tol in (("bf16", 2e-2, 1e-3), ("fp32", 1e-5, 1e-5)):
        assert abs(float(r0[f"{tag}_split_loss"]) - float(r0[f"{tag}_whole_loss"])) < loss_tol
        for i in range(3):
            assert _row_rel(r0[f"{tag}_split_h{i}"], r0[f"{tag}_whole_h{i}"]) < tol, (tag, i)


def test_head_split_long_context_matches_reference(golden, cuda):
    """L=24, d=2048, H=16 (head_dim 128), T=8192: 8 heads and 4096 MLP units per rank, bf16, against the
    reference's fp32 forward at the fixture's rows and layers: Y/rho within 2e-2, the loss within 1e-3."""
    from tests.helpers import CFG5
    g = golden("cfg5_d2048.npz")
    rows = {"rows": g["state_rows"], "layers": [int(i) for i in g["state_layers"]]}
    r0, r1 = _run_group(CFG5, 1, (True,), golden_rows=rows)
    for res in (r0, r1):
        assert abs(float(res["bf16_split_loss"]) - float(g["loss"])) < 1e-3
        for i in rows["layers"]:
            assert _row_rel(res[f"bf16_split_h{i}"], g[f"h{i}"]) < 2e-2, i
