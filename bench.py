"""Forward-throughput benchmark of the enGPT hot path on B200.

Workload (one "step"): ``EfficientNGPT`` forward + token cross-entropy under
bf16 autocast, L=16, d=1024, H=16 (head_dim 64), T=2048, vocab 50257, a
global batch of 32 sequences, random-init unit-sphere weights (seed 0) and
uniform random token ids (synthetic data).  With N GPUs (one process each)
the batch is split by sequences over the ranks (strong scaling: 4 sequences
per GPU at N=8), with no collective inside the forward; each step ends with
one NCCL all-reduce of the token-weighted loss and an all-gather of every
shard's final represented state Y/rho (``--gather``).  ``--scaling weak``
runs ``--batch`` sequences per rank instead.

Reported (one JSON line from rank 0):
  value      tokens/s over all ranks, inputs resident in HBM, device-timed
             with CUDA events (max over ranks)
  e2e        the same metric through the public API (``model(idx, targets)``)
             with pinned host ids/targets copied in and the loss copied out
             inside the timed region
  roofline   the attention kernel (tcgen05) against bf16 tensor peak
  kernels    per-kernel averages of the CUDA kernels of one forward
  reference_gpu  the reference package's own eager GPU forward at this
             workload and at the shape of its published numbers (N=1)
  cpu_baseline  the oracle's fp32 numpy forward on the host cores (N=1 only)

``--impl reference`` times the reference algorithm's CPU implementation (the
oracle port) on the host cores for the same workload and metric.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time


def _reference_arm(argv):
    return "--impl=reference" in argv or any(x == "--impl" and argv[i + 1:i + 2] == ["reference"]
                                              for i, x in enumerate(argv))


if _reference_arm(sys.argv):
    # the CPU reference arm uses every host core: set the BLAS / OpenMP pools before numpy loads them
    # (torchrun exports OMP_NUM_THREADS=1 to every rank)
    for _var in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[_var] = str(os.cpu_count() or 1)

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

def metric_name(a):
    return f"forward tokens/sec (EfficientNGPT bf16, L={a.layers} d={a.dim} H={a.heads} T={a.seq})"

# The result line goes to the original stdout; everything else written to fd 1 (library banners such as
# NCCL's version line, stray prints) is redirected to stderr so stdout carries exactly one JSON line.
_RESULT_OUT = None


def emit(obj):
    out = _RESULT_OUT if _RESULT_OUT is not None else sys.stdout
    out.write(json.dumps(obj) + "\n")
    out.flush()


def _guard_stdout():
    global _RESULT_OUT
    sys.stdout.flush()
    _RESULT_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
UNIT = "tokens/s"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["engpt_b200", "reference"], default="engpt_b200")
    ap.add_argument("--workload", choices=["forward", "attention"], default="forward",
                    help="forward: the model step (default); attention: the isolated nGPT attention op")
    ap.add_argument("--batch", type=int, default=32, help="sequences per GPU")
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--layers", type=int, default=16)
    ap.add_argument("--heads", type=int, default=16)
    ap.add_argument("--dim", type=int, default=1024)
    ap.add_argument("--vocab", type=int, default=50257)
    ap.add_argument("--qkv-layout", choices=["separate", "packed"], default="separate",
                    help="attention workload: separate [B,T,H,Dh] q/k/v, or views of one [B,T,3,H,Dh] buffer")
    ap.add_argument("--attn-softmax", choices=["bound", "online"], default="bound",
                    help="attention workload: nGPT score-bound offset (the forward's call) or running-max softmax")
    ap.add_argument("--scaling", choices=["strong", "weak"], default="strong",
                    help="strong: --batch sequences in total, split over the ranks; weak: --batch per rank")
    ap.add_argument("--head-split", type=int, default=1,
                    help="ranks per head-split group: each group of this many GPUs shares its sequences' heads and "
                         "MLP units (two all-reduces per layer); the batch is split over the groups")
    ap.add_argument("--gather", choices=["hidden", "logits", "none"], default="hidden",
                    help="N>1: outputs all-gathered over NCCL inside the timed step (final Y/rho, or the logits)")
    ap.add_argument("--overlap-collectives", choices=["on", "off"], default="on",
                    help="N>1: run each step's loss all-reduce and output all-gather on NCCL's stream during the next "
                         "step's forward (equal shards, no head split)")
    ap.add_argument("--cuda-graph", choices=["on", "off"], default="off",
                    help="replay the forward from a CUDA graph (EfficientNGPT.enable_cuda_graphs)")
    ap.add_argument("--cpu-sample-seqs", type=int, default=1)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip timing the reference package's own GPU forward (N=1)")
    return ap.parse_args()


def workload_config(a, world):
    hs = getattr(a, "head_split", 1)
    gb = a.batch if a.scaling == "strong" else a.batch * (world // hs)
    return {
        "workload": (f"EfficientNGPT forward + cross-entropy, bf16 autocast, L={a.layers} d={a.dim} H={a.heads} "
                     f"T={a.seq} V={a.vocab}, {gb} sequences in total"),
        "global_batch": gb,
        "seq_len": a.seq,
        "parallelism": ((f"dp{world // hs} x head split {hs}: groups of {hs} GPUs share each sequence's heads and MLP "
                         f"units (two all-reduces of the partial branch per layer), the batch split over the groups"
                         if hs > 1 else
                         f"dp{world}: the batch split by sequences over the ranks, no collective inside the forward")
                        + f" ({a.scaling} scaling)"
                        + (f"; per step one all-reduce of the loss and an all-gather of the {a.gather} outputs"
                           if world > 1 and a.gather != "none" else "")
                        + ("; the step's collectives overlap the next step's forward (NCCL stream)"
                           if world > 1 and getattr(a, "overlap_collectives", "off") == "on" and hs == 1
                           and a.gather != "logits" and gb % (world // hs) == 0 else "")),
        "l2": "no flush: activations per step (~10 GB at 32 sequences) exceed the 126 MB L2",
    }


def model_config(a):
    from engpt_b200 import ModelConfig
    return ModelConfig(vocab_size=a.vocab, block_size=a.seq, n_layer=a.layers, n_head=a.heads, n_embd=a.dim,
                       mlp_ratio=4.0, dropout=0.0)


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"],
                "bf16_tflops_sustained": p.get("bf16_tflops_sustained", p["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def load_traffic(local_batch=32):
    """Per-launch DRAM bytes of the attention kernel from the committed ncu summary (captured at 32 sequences),
    scaled to this launch's sequences (the traffic is q/k/v/o, proportional to them)."""
    path = os.path.join(ROOT, "profiles", "attn_fwd2_B32_H16_T2048_D64.md")
    if not os.path.exists(path):
        return None
    for line in open(path):
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].split()[0]) * local_batch / 32.0
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clock/throttle sampling during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# -------------------------------------------------------------- CPU baseline
def cpu_baseline(a, n_seqs):
    """The oracle (numpy fp32 restatement of the reference forward) on the host cores."""
    import torch
    from oracle import ngpt_oracle as O
    from engpt_b200 import EfficientNGPT

    torch.manual_seed(0)
    model = EfficientNGPT(model_config(a))
    w = {k: v.detach().numpy() for k, v in model.state_dict().items()}
    del model
    cfg = O.OracleConfig(vocab_size=a.vocab, block_size=a.seq, n_layer=a.layers, n_head=a.heads, n_embd=a.dim)
    gen = torch.Generator().manual_seed(0)
    idx = torch.randint(0, a.vocab, (n_seqs, a.seq), generator=gen).numpy()
    tgt = np.roll(idx, -1, axis=1)
    t0 = time.perf_counter()
    _, loss, _ = O.efficient_ngpt_forward(cfg, w, idx, tgt, dtype=np.float32)
    dt = time.perf_counter() - t0
    return n_seqs * a.seq / dt, dt, loss


def _blas_threads():
    """Threads of the BLAS pool numpy uses (what the CPU legs actually ran with)."""
    try:
        from threadpoolctl import threadpool_info
        n = [p.get("num_threads") for p in threadpool_info() if p.get("user_api") == "blas"]
        return max(n) if n else None
    except Exception:  # pragma: no cover - threadpoolctl missing
        return None


def run_reference(a, world, rank):
    """The reference arm: the oracle port of the reference forward (numpy fp32) on the host cores, rank 0 only.

    It times bounded samples of the workload: --cpu-sample-seqs sequences of --seq tokens per step."""
    if rank != 0:
        return
    import torch
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    from oracle import ngpt_oracle as O
    from engpt_b200 import EfficientNGPT

    torch.manual_seed(0)
    model = EfficientNGPT(model_config(a))
    w = {k: v.detach().numpy() for k, v in model.state_dict().items()}
    del model
    cfg = O.OracleConfig(vocab_size=a.vocab, block_size=a.seq, n_layer=a.layers, n_head=a.heads, n_embd=a.dim)
    gen = torch.Generator().manual_seed(0)
    n = a.cpu_sample_seqs
    idx = torch.randint(0, a.vocab, (n, a.seq), generator=gen).numpy()
    tgt = np.roll(idx, -1, axis=1)
    for _ in range(a.warmup):
        O.efficient_ngpt_forward(cfg, w, idx, tgt, dtype=np.float32)
    times = []
    for _ in range(a.steps):
        t0 = time.perf_counter()
        O.efficient_ngpt_forward(cfg, w, idx, tgt, dtype=np.float32)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = a.steps * n * a.seq / total
    threads = _blas_threads() or cores
    sample = f"{n} x {a.seq}-token sequence(s) of the workload per step, fp32 numpy, {threads} BLAS threads"
    emit({
        "metric": metric_name(a), "value": value, "unit": UNIT, "impl": "reference", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": 1000.0 * total / a.steps, "higher_is_better": True,
        "scaling": a.scaling, "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(a, world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    })


# ------------------------------------------------------------------ GPU arm
# kernels launched per C-ABI call
# kernels launched per C-ABI call (1 unless listed)
LAUNCHES = {"engpt_cross_entropy": 2, "engpt_logits_cross_entropy": 3}


def run_gpu(a, world, rank, local_rank):
    import torch
    import torch.distributed as dist
    from engpt_b200 import EfficientNGPT, _lib, sharding

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    torch.backends.cuda.matmul.allow_tf32 = False
    cfg = model_config(a)
    torch.manual_seed(0)
    model = EfficientNGPT(cfg).to(dev).eval().requires_grad_(False)
    # head-split groups of `hs` ranks share sequences; the batch is split over the world // hs groups
    hs = a.head_split
    replicas, replica = world // hs, rank // hs
    dp_group = None
    if hs > 1:
        from engpt_b200.head_split import HeadSplit, pair_groups
        split_groups, dp_groups = pair_groups(world, hs)
        model.set_head_split(HeadSplit(rank % hs, hs, split_groups[replica]))
        dp_group = dp_groups[rank % hs]
    # the global batch: `batch` sequences split over the replicas (strong scaling), or `batch` per replica (weak)
    global_batch = a.batch if a.scaling == "strong" else a.batch * replicas
    gen = torch.Generator().manual_seed(1000)
    idx_all = torch.randint(0, cfg.vocab_size, (global_batch, a.seq), generator=gen)
    lo, hi = sharding.shard_range(global_batch, replica, replicas)
    if hi - lo == 0:
        raise SystemExit(f"rank {rank}: no sequences (global batch {global_batch} < {world} ranks)")
    idx_h = idx_all[lo:hi].contiguous()
    tgt_h = torch.roll(idx_h, -1, dims=1)
    idx_d, tgt_d = idx_h.to(dev), tgt_h.to(dev)
    local_batch = hi - lo

    # count our kernel launches through the C-ABI
    counter = {"n": 0}
    real_call = _lib.call

    def counting_call(name, *args):
        counter["n"] += LAUNCHES.get(name, 1)
        return real_call(name, *args)

    _lib.call = counting_call

    # this shard's counted targets (device scalar); a head-split group counts its sequences once
    n_valid = sharding.valid_targets(tgt_d) * (1 if rank % hs == 0 else 0)

    # N > 1, batch shards of equal size, the final state gathered: the step's collectives (the loss all-reduce
    # and the all-gather) run on NCCL's stream while the next step's forward runs.  Two buffer sets alternate;
    # a set is rewritten only after the collectives of the step two back that used it completed.
    overlap = (world > 1 and a.overlap_collectives == "on" and hs == 1 and a.gather in ("hidden", "none")
               and global_batch % replicas == 0)
    pend = {"slot": 0, "works": [[], []], "send": [None, None], "recv": [None, None], "part": [None, None]}
    side = torch.cuda.Stream(dev)

    def submit(loss):
        b = pend["slot"] & 1
        pend["slot"] += 1
        for w in pend["works"][b]:
            w.wait()
        torch.cuda.current_stream(dev).wait_stream(side)   # the loss copy that read part[b] two steps back
        nv = n_valid.to(device=dev, dtype=torch.float64)
        part = torch.stack([torch.where(nv > 0, loss.to(torch.float64) * nv, 0.0), nv])
        pend["part"][b] = part
        works = [dist.all_reduce(part, op=dist.ReduceOp.SUM, async_op=True)]
        if a.gather == "hidden":
            hidden = model.last_hidden()
            if pend["send"][b] is None:
                pend["send"][b] = torch.empty_like(hidden)
                pend["recv"][b] = hidden.new_empty((global_batch,) + tuple(hidden.shape[1:]))
            pend["send"][b].copy_(hidden)   # the next forward rewrites the workspace
            works.append(dist.all_gather_into_tensor(pend["recv"][b], pend["send"][b], group=dp_group,
                                                     async_op=True))
        pend["works"][b] = works
        return pend["recv"][b], part

    def drain():
        for ws in pend["works"]:
            for w in ws:
                w.wait()
        torch.cuda.current_stream(dev).wait_stream(side)

    def part_loss(part):
        return torch.where(part[1] > 0, part[0] / part[1], float("nan")).to(torch.float32)

    def step(idx, tgt):
        with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
            logits, loss = model(idx, tgt)
        out = None
        if overlap:
            return submit(loss)
        if world > 1:
            # token-weighted mean over all shards (one all-reduce of 2 doubles), then the outputs of every
            # shard gathered over NCCL: the final represented state [B, T, d] bf16, or the logits
            loss = sharding.combine_loss(loss, n_valid)
            if a.gather == "hidden":
                out = sharding.gather_rows(model.last_hidden(), global_batch, group=dp_group)
            elif a.gather == "logits":
                out = sharding.gather_rows(logits, global_batch, group=dp_group)
        return out, loss

    graphs = a.cuda_graph == "on"
    if graphs:
        model.enable_cuda_graphs()
    for _ in range(max(a.warmup, 1)):
        step(idx_d, tgt_d)
    torch.cuda.synchronize()
    # kernels of one forward (a graph replays the launches counted while it was captured)
    counter["n"] = 0
    if graphs:
        model.enable_cuda_graphs(False)
    step(idx_d, tgt_d)
    per_forward = counter["n"]
    if graphs:
        model.enable_cuda_graphs()
        step(idx_d, tgt_d)
    torch.cuda.synchronize()

    # attention launch timing inside the timed region
    attn_events = []

    def attn_timer(kind):
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        attn_events.append(ev)

    model.attn_timer = attn_timer
    sampler = ClockSampler(local_rank) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.5)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    counter["n"] = 0
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(a.steps):
        out, loss = step(idx_d, tgt_d)
        del out
    if overlap:
        drain()
        loss = part_loss(loss)
    ev1.record()
    torch.cuda.synchronize()
    launches = counter["n"] if not graphs else per_forward * a.steps
    if world > 1:
        dist.barrier()
    clocks = sampler.stop() if sampler else None
    if graphs:
        # a replayed graph runs no Python hooks: the attention launches are timed in one eager step after the
        # timed region (same inputs, same kernels)
        model.enable_cuda_graphs(False)
        step(idx_d, tgt_d)
        torch.cuda.synchronize()
        model.enable_cuda_graphs()
    model.attn_timer = None
    ms = ev0.elapsed_time(ev1)
    attn_ms = [attn_events[i].elapsed_time(attn_events[i + 1]) for i in range(0, len(attn_events), 2)]
    attn_avg = sum(attn_ms) / max(len(attn_ms), 1)
    loss_val = float(loss.item())

    # end-to-end through the public API: pinned host inputs in, loss out, every step
    idx_p, tgt_p = idx_h.pin_memory(), tgt_h.pin_memory()
    loss_h = torch.empty((), dtype=torch.float32).pin_memory()
    step(idx_p, tgt_p)
    if overlap:
        drain()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.steps):
        _, loss = step(idx_p, tgt_p)
        if overlap:
            # the step's loss once its all-reduce completed, copied out on a side stream (the forward of the
            # next step does not wait for it)
            work = pend["works"][(pend["slot"] - 1) & 1][0]
            with torch.cuda.stream(side):
                work.wait()
                loss_h.copy_(part_loss(loss), non_blocking=True)
        else:
            loss_h.copy_(loss, non_blocking=True)
    if overlap:
        drain()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)

    # per-kernel averages of the CUDA kernels (one instrumented forward, outside the timed region)
    kern = profile_kernels(model, step, idx_d, tgt_d, cfg, a, local_batch, hs)

    if world > 1:
        t = torch.tensor([ms, e2e_ms, attn_avg], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms, attn_avg = t.tolist()

    ref_gpu = None
    if world == 1 and not a.no_reference_gpu:
        try:
            ref_gpu = reference_gpu_timing(a, dev, model)
        except Exception as exc:  # pragma: no cover - reported, not fatal
            ref_gpu = {"error": repr(exc)}

    if rank != 0:
        return
    tokens = global_batch * a.seq * a.steps
    value = tokens / (ms / 1000.0)
    e2e = tokens / (e2e_ms / 1000.0)
    peaks = load_peaks()
    Dh = a.dim // a.heads
    # causal: QK^T and PV over the lower triangle, this rank's heads
    attn_flops = 2.0 * local_batch * (a.heads // hs) * a.seq * a.seq * Dh
    achieved = attn_flops / (attn_avg / 1000.0) / 1e12
    peak = peaks["bf16_tflops_sustained"]
    out = {
        "metric": metric_name(a), "value": value, "unit": UNIT, "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": ms / a.steps, "higher_is_better": True, "scaling": a.scaling, "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (uniform random ids, seeded random-init unit-sphere weights)",
        "config": {**workload_config(a, world), "cuda_graph": a.cuda_graph},
        "e2e": {"value": e2e, "unit": UNIT,
                "h2d_bytes_per_step": 2 * global_batch * hs * a.seq * idx_h.element_size(),
                "d2h_bytes_per_step": 4 * world},
        "gpu_launches": launches,
        "roofline": {"kernel": "attn_fwd2_kernel (tcgen05, head_dim 64)", "bound": "tensor", "achieved": achieved,
                     "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak, "traffic": load_traffic(local_batch),
                     "peak_source": f"{peaks['source']} bf16 sustained",
                     "avg_launch_ms": attn_avg, "flops_per_launch": attn_flops},
        "kernels": kern,
        "loss": loss_val,
        "clocks": clocks,
    }
    if ref_gpu is not None:
        out["reference_gpu"] = ref_gpu
    if world == 1 and not a.no_cpu_baseline:
        try:
            tps, dt, _ = cpu_baseline(a, a.cpu_sample_seqs)
            out["cpu_baseline"] = {"value": tps, "unit": UNIT, "cores": _blas_threads() or os.cpu_count() or 1,
                                   "kind": "port",
                                   "sample": f"{a.cpu_sample_seqs} x {a.seq}-token sequence(s), fp32 numpy oracle, "
                                             f"{dt:.1f} s"}
        except Exception as exc:  # pragma: no cover - reported, not fatal
            out["cpu_baseline"] = {"error": repr(exc)}
    emit(out)


def _reference_package():
    """The reference package installed from its sources under baseline/_ref (git-ignored), or None."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "engpt")):
        return None
    if ref not in sys.path:
        sys.path.insert(0, ref)
    import engpt
    return engpt


def _time_forward(fn, warmup, steps):
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def reference_gpu_timing(a, dev, model):
    """The reference's own GPU forward beside this one (reported, not the reference arm).

    The reference package's ``EfficientNGPT.forward`` in eager PyTorch under bf16
    autocast and ``torch.no_grad`` (its benchmark flow, scripts/gpu_train_benchmark.py:148-175),
    on the same seeded weights and ids: at this workload, and at the shape of its
    published numbers (L=4, d=256, H=4, T=256, 16 sequences) next to this
    engine at that shape.
    """
    import torch
    from engpt_b200 import EfficientNGPT, ModelConfig
    engpt = _reference_package()
    if engpt is None:
        return {"unavailable": "reference package not installed under baseline/_ref"}
    out = {"how": "reference engpt.EfficientNGPT.forward, eager PyTorch, bf16 autocast, no_grad, CUDA events"}

    def ref_tokps(cfg_kw, batch, seq, ours=None):
        torch.manual_seed(0)
        ref = engpt.EfficientNGPT(engpt.ModelConfig(**cfg_kw)).to(dev).eval()
        gen = torch.Generator().manual_seed(1000)
        idx = torch.randint(0, cfg_kw["vocab_size"], (batch, seq), generator=gen).to(dev)
        tgt = torch.roll(idx, -1, dims=1)

        def run_ref():
            with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
                ref(idx, tgt)

        ms_ref = _time_forward(run_ref, 2, 3)
        rec = {"reference_tok_s": batch * seq / (ms_ref / 1000.0), "reference_ms": ms_ref}
        del ref
        if ours is not None:
            def run_ours():
                with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
                    ours(idx, tgt)
            ms = _time_forward(run_ours, 3, 5)
            rec.update({"engpt_b200_tok_s": batch * seq / (ms / 1000.0), "engpt_b200_ms": ms})
            # the same forward replayed from a CUDA graph (model.enable_cuda_graphs): no per-kernel host launches
            ours.enable_cuda_graphs()
            ms = _time_forward(run_ours, 3, 20)
            ours.enable_cuda_graphs(False)
            rec.update({"engpt_b200_cuda_graph_tok_s": batch * seq / (ms / 1000.0), "engpt_b200_cuda_graph_ms": ms})
        torch.cuda.empty_cache()
        return rec

    cfg_kw = dict(vocab_size=a.vocab, block_size=a.seq, n_layer=a.layers, n_head=a.heads, n_embd=a.dim,
                  mlp_ratio=4.0, dropout=0.0)
    out["workload"] = ref_tokps(cfg_kw, a.batch, a.seq)
    out["workload"]["shape"] = f"L={a.layers} d={a.dim} H={a.heads} T={a.seq}, {a.batch} sequences"
    pub_kw = dict(vocab_size=50257, block_size=256, n_layer=4, n_head=4, n_embd=256, mlp_ratio=4.0, dropout=0.0)
    torch.manual_seed(0)
    small = EfficientNGPT(ModelConfig(**pub_kw)).to(dev).eval().requires_grad_(False)
    out["published_shape"] = ref_tokps(pub_kw, 16, 256, ours=small)
    out["published_shape"].update({"shape": "L=4 d=256 H=4 T=256, 16 sequences",
                                   "published_reference_eager_tok_s": 1247759,
                                   "published_reference_compiled_tok_s": 2818401})
    return out


def profile_kernels(model, step, idx, tgt, cfg, a, local_batch, hs=1):
    """Average device time per launch of each C-ABI entry point over one forward (events around each call)."""
    import torch
    from engpt_b200 import _lib

    per = {}
    real = _lib.call

    def timed(name, *args):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        r = real(name, *args)
        e1.record()
        per.setdefault(name, []).append((e0, e1))
        return r

    _lib.call = timed
    try:
        step(idx, tgt)
        torch.cuda.synchronize()
    finally:
        _lib.call = real
    n = local_batch * a.seq
    d = a.dim
    peaks = load_peaks()
    # algorithmic bytes per launch (dtypes as used by the engine)
    alg = {
        "engpt_carried_residual_gauge": (4 + 2 + 4 + 2) * n * d + 8 * n,   # Y in/out fp32, branch + aux bf16
        "engpt_qkv_postprocess": 12 * n * d // hs + 4 * n,                # qkv bf16 in, q/k/v bf16 out, rho
        "engpt_swiglu": (4 + 2) * n * 4 * d // hs,                        # ug bf16 in (2W), out bf16 (W)
        "engpt_cross_entropy": 2 * n * a.vocab + 12 * n,
        "engpt_embed_carried": (4 + 4 + 2) * n * d + 12 * n,
        # fp32 weights in, bf16 out (a head-split rank casts its QKV and up/gate rows, all of out_proj / down)
        "engpt_cast_f32_bf16_many": 6 * a.layers * d * d * ((3 + 8) / hs + 5),
    }
    W = 4 * d
    flops = {   # tensor-bound fused GEMMs: 2 * M * N * K
        "engpt_qkv_projection": 2.0 * n * 3 * d * d / hs,
        "engpt_up_gate_swiglu": 2.0 * n * 2 * W * d / hs,
        "engpt_logits_cross_entropy": 2.0 * n * a.vocab * d,         # output head (+ log-sum-exp epilogue)
    }
    out = {}
    for name, evs in per.items():
        ms = [e0.elapsed_time(e1) for e0, e1 in evs]
        avg = sum(ms) / len(ms)
        rec = {"launches_per_step": len(ms), "avg_ms": avg}
        if name in alg:
            gbs = alg[name] / (avg / 1000.0) / 1e9
            rec.update({"bound": "hbm", "achieved_gbs": gbs, "frac": gbs / peaks["hbm_gbs"],
                        "bytes_per_launch": alg[name]})
        elif name in flops:
            tf = flops[name] / (avg / 1000.0) / 1e12
            rec.update({"bound": "tensor", "achieved_tflops": tf, "frac": tf / peaks["bf16_tflops_sustained"],
                        "flops_per_launch": flops[name]})
        out[name.replace("engpt_", "")] = rec
    return out


def run_attention(a, world, rank, local_rank):
    """Isolated nGPT attention op: B x H x T x Dh causal, bf16, unit q/k scaled by s ~ U(0.9, 1.1), scale sqrt(Dh).

    Defaults to the BASELINE isolated-attention shape via --batch 8 (B=8, H=16, T=2048, Dh=64).
    Prints tensor-core roofline numbers for the tcgen05 kernel and, for context, torch's bf16 SDPA.
    """
    import torch
    from engpt_b200 import _lib, kernels as K

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    B, H, T = a.batch, a.heads, a.seq
    Dh = a.dim // a.heads
    g = torch.Generator().manual_seed(1)
    q = torch.randn(B, T, H, Dh, generator=g)
    k = torch.randn(B, T, H, Dh, generator=g)
    v = torch.randn(B, T, H, Dh, generator=g)
    s = torch.rand(Dh, generator=g) * 0.2 + 0.9
    q = (q / q.norm(dim=-1, keepdim=True) * s).to(dev, torch.bfloat16)
    k = (k / k.norm(dim=-1, keepdim=True) * s).to(dev, torch.bfloat16)
    v = v.to(dev, torch.bfloat16)
    if a.qkv_layout == "packed":
        # q/k/v as views of one [B, T, 3, H, Dh] buffer, the layout the forward's QKV epilogue leaves
        packed = torch.stack([q, k, v], dim=2).contiguous()
        q, k, v = packed[:, :, 0], packed[:, :, 1], packed[:, :, 2]
    scale = math.sqrt(Dh)

    o_buf = torch.empty(B, T, H, Dh, device=dev, dtype=torch.bfloat16)
    strides = K.attention_strides(q, k, v, o_buf, head_major=False)
    s_heads = s.to(dev).expand(H, Dh).contiguous()
    st = _lib.stream_handle(dev)

    def ours():
        if a.attn_softmax == "bound":
            # the forward's call: softmax offset from the per-head score bound max s^2
            _lib.call("engpt_ngpt_attention", q.data_ptr(), k.data_ptr(), v.data_ptr(), o_buf.data_ptr(), _lib.BF16,
                      B, T, H, Dh, float(scale), strides.data_ptr(), s_heads.data_ptr(), 1.0, st)
        else:
            _lib.call("engpt_causal_attention", q.data_ptr(), k.data_ptr(), v.data_ptr(), o_buf.data_ptr(),
                      _lib.BF16, B, T, H, Dh, float(scale), strides.data_ptr(), _lib.ATTN_TCGEN05, st)
        return o_buf

    def torch_sdpa():
        return torch.nn.functional.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2),
                                                                v.transpose(1, 2), is_causal=True, scale=scale)

    def timeit(fn, steps):
        for _ in range(max(a.warmup, 1)):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    sampler = ClockSampler(local_rank)
    sampler.start()
    time.sleep(0.3)
    ms = timeit(ours, a.steps)
    clocks = sampler.stop()
    ms_torch = timeit(torch_sdpa, a.steps)
    assert _lib.device_status() == 0
    flops = 2.0 * B * H * T * T * Dh
    peaks = load_peaks()
    achieved = flops / (ms / 1000.0) / 1e12
    emit({
        "metric": "isolated nGPT causal attention TFLOP/s", "value": achieved, "unit": "TFLOP/s",
        "n_gpus": 1, "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True,
        "dtype": "bf16", "data": "synthetic (seeded normal q/k/v, unit q/k scaled by U(0.9,1.1))",
        "config": {"workload": f"causal attention B={B} H={H} T={T} Dh={Dh}, scale sqrt(Dh), q/k/v {a.qkv_layout}, "
                               f"softmax {a.attn_softmax}",
                   "l2": "inputs read once per launch; no flush between launches"},
        "roofline": {"kernel": "attn_fwd2_kernel (tcgen05)" if Dh == 64 else f"attn_fwd_kernel<{Dh}> (tcgen05)", "bound": "tensor", "achieved": achieved,
                     "peak": peaks["bf16_tflops"], "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops"],
                     "traffic": None, "peak_source": f"{peaks['source']} bf16 burst"},
        "torch_sdpa_bf16": {"ms": ms_torch, "tflops": flops / (ms_torch / 1000.0) / 1e12},
        "clocks": clocks,
    })


def main():
    a = parse_args()
    _guard_stdout()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if a.gpus != world and world > 1:
        print(f"warning: --gpus {a.gpus} but WORLD_SIZE={world}; using WORLD_SIZE", file=sys.stderr)
    if a.impl == "reference":
        run_reference(a, world, rank)
        return
    if a.workload == "attention":
        run_attention(a, world, rank, local_rank)
        return
    import datetime
    import torch.distributed as dist
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    try:
        run_gpu(a, world, rank, local_rank)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
