"""Generate the golden fixtures in this folder by running the reference package.

Usage (needs the Pi-Willie/enGPT sources, not needed at test time)::

    PYTHONPATH=<enGPT checkout> python tests/golden/make_golden.py [name ...]

With names (ops, small, attn, sphere, optim, cfg1, cfg4, cfg3, cfg5) only those fixtures are
written; with none, all of them.

The reference is run on the CPU (fp64 for the op-level and small-model
vectors, fp32 for the BASELINE-sized configs) with the seeds listed below.
Large tensors are not stored: weights are fingerprinted (they are regenerated
from ``torch.manual_seed`` by ``engpt_b200.EfficientNGPT``, whose parameter
creation order matches the reference), and activations are stored for a
subset of rows.
"""

from __future__ import annotations

import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _ref():
    import engpt  # noqa: F401  (the reference package)
    from engpt import EfficientNGPT, ModelConfig
    from engpt import kernels as K
    return EfficientNGPT, ModelConfig, K


def fingerprint(sd):
    names = sorted(sd.keys())
    fp = np.zeros((len(names), 6), dtype=np.float64)
    for i, n in enumerate(names):
        t = sd[n].detach().double().reshape(-1)
        fp[i, 0] = t.sum().item()
        fp[i, 1] = (t * t).sum().item()
        fp[i, 2:6] = t[:4].numpy() if t.numel() >= 4 else np.pad(t.numpy(), (0, 4 - t.numel()))
    return np.array(names), fp


def ops_vectors(K):
    out = {}
    g = torch.Generator().manual_seed(11)
    # qkv post-process: even head_dim, rho != 1, one near-zero q row to hit the rho*eps guard.
    for tag, (B, T, H, D) in {"even": (2, 5, 2, 8), "odd": (1, 4, 3, 7)}.items():
        qkv = torch.randn(B, T, 3, H, D, generator=g, dtype=torch.float64)
        qkv[0, 1, 0, 0] *= 1e-9
        rho = torch.rand(B, T, generator=g, dtype=torch.float64) + 0.5
        cos, sin = K.rotary_frequencies(T, D, device="cpu", dtype=torch.float64, theta=10000.0)
        qk_scale = torch.rand(H, D, generator=g, dtype=torch.float64) * 0.2 + 0.9
        with torch.no_grad():
            q, k, v = K.qkv_postprocess_from_carried(qkv.clone(), rho, cos, sin, qk_scale, 1e-6)
        out.update({f"qkv_{tag}_in": qkv.numpy(), f"qkv_{tag}_rho": rho.numpy(),
                    f"qkv_{tag}_cos": cos.numpy(), f"qkv_{tag}_sin": sin.numpy(),
                    f"qkv_{tag}_scale": qk_scale.numpy(), f"qkv_{tag}_q": q.numpy(),
                    f"qkv_{tag}_k": k.numpy(), f"qkv_{tag}_v": v.numpy()})
    # rotary tables in fp32 (the model weight dtype) at a BASELINE-like size.
    cos, sin = K.rotary_frequencies(2048, 64, device="cpu", dtype=torch.float32, theta=10000.0)
    out["rope2048_cos"] = cos.numpy()
    out["rope2048_sin"] = sin.numpy()
    # carried residual + gauge: active gauge (0.75), inactive (1024), disabled (0); one zero branch row.
    y = torch.randn(3, 4, 16, generator=g, dtype=torch.float64) * 3.0
    rho = torch.rand(3, 4, generator=g, dtype=torch.float64) + 0.5
    branch = torch.randn(3, 4, 16, generator=g, dtype=torch.float64)
    branch[1, 2].zero_()
    alpha = torch.rand(16, generator=g, dtype=torch.float64) * 0.5
    out.update({"res_y": y.numpy(), "res_rho": rho.numpy(), "res_branch": branch.numpy(),
                "res_alpha": alpha.numpy()})
    for tag, mr in {"g075": 0.75, "g1024": 1024.0, "g0": 0.0}.items():
        yo, ro = K.carried_residual_gauge(y, rho, branch, alpha, 1e-6, 1e-6, mr)
        out[f"res_{tag}_y"] = yo.numpy()
        out[f"res_{tag}_rho"] = ro.numpy()
    # causal SDPA with the nGPT scale, two shapes (one ragged against 128-row tiles).
    for tag, (B, T, H, D) in {"a": (2, 9, 3, 16), "b": (1, 130, 2, 64)}.items():
        q = torch.randn(B, T, H, D, generator=g, dtype=torch.float64)
        k = torch.randn(B, T, H, D, generator=g, dtype=torch.float64)
        v = torch.randn(B, T, H, D, generator=g, dtype=torch.float64)
        q = q / q.norm(dim=-1, keepdim=True)
        k = k / k.norm(dim=-1, keepdim=True)
        o = K.causal_sdpa(q, k, v, scale=K.ngpt_attention_scale(D), dropout_p=0.0)
        out.update({f"sdpa_{tag}_q": q.numpy(), f"sdpa_{tag}_k": k.numpy(),
                    f"sdpa_{tag}_v": v.numpy(), f"sdpa_{tag}_o": o.numpy()})
    np.savez_compressed(os.path.join(HERE, "ops_small.npz"), **out)


def sphere_vectors(K):
    """Retraction and tangent projection (engpt/kernels.py:98-136) on odd and ragged shapes, fp64, and one
    NGPTAdamW step (engpt/optim.py:38-67) of the reference's small model with seeded gradients."""
    out = {}
    g = torch.Generator().manual_seed(13)
    for tag, shape in {"a": (9, 13), "b": (33, 100), "c": (130, 7)}.items():
        w = torch.randn(*shape, generator=g, dtype=torch.float64)
        gr = torch.randn(*shape, generator=g, dtype=torch.float64)
        out[f"sph_{tag}_w"] = w.numpy()
        out[f"sph_{tag}_g"] = gr.numpy()
        out[f"sph_{tag}_rows"] = K.normalize_rows_(w.clone(), 1e-6).numpy()
        out[f"sph_{tag}_cols"] = K.normalize_columns_(w.clone(), 1e-6).numpy()
        wr = K.normalize_rows_(w.clone(), 1e-12)
        wc = K.normalize_columns_(w.clone(), 1e-12)
        pr, pc = gr.clone(), gr.clone()
        K.project_row_grad_(wr, pr)
        K.project_column_grad_(wc, pc)
        out[f"sph_{tag}_wr"] = wr.numpy()
        out[f"sph_{tag}_wc"] = wc.numpy()
        out[f"sph_{tag}_prow"] = pr.numpy()
        out[f"sph_{tag}_pcol"] = pc.numpy()
    np.savez_compressed(os.path.join(HERE, "sphere_small.npz"), **out)


def optimizer_step(EfficientNGPT, ModelConfig):
    """One NGPTAdamW step (engpt/optim.py:38-67) of the reference's small config in fp32 with seeded gradients."""
    from engpt.optim import NGPTAdamW
    cfg = ModelConfig(vocab_size=64, block_size=16, n_layer=2, n_head=2, n_embd=32, mlp_ratio=2.0, dropout=0.0)
    torch.manual_seed(2)
    model = EfficientNGPT(cfg)
    g = torch.Generator().manual_seed(14)
    grads = {n: torch.randn(p.shape, generator=g) * 0.1 for n, p in model.named_parameters()}
    for n, p in model.named_parameters():
        p.grad = grads[n].clone()
    opt = NGPTAdamW(model, lr=1e-2)
    opt.step()
    out = {"g:" + n: v.numpy() for n, v in grads.items()}
    out.update({"w:" + n: p.detach().numpy() for n, p in model.named_parameters()})
    np.savez_compressed(os.path.join(HERE, "optim_step.npz"), **out)


def capture_states(model, fn):
    states = []
    hooks = [b.register_forward_hook(lambda m, i, o: states.append((o[0].detach().clone(), o[1].detach().clone())))
             for b in model.blocks]
    try:
        res = fn()
    finally:
        for h in hooks:
            h.remove()
    return res, states


def model_small(EfficientNGPT, ModelConfig):
    # The reference's own small equivalence config (tests/test_models.py:7-17), seed 1, fp64.
    cfg = ModelConfig(vocab_size=32, block_size=12, n_layer=2, n_head=2, n_embd=32, mlp_ratio=2.0,
                      dropout=0.0, alpha_init=0.1)
    torch.manual_seed(1)
    model = EfficientNGPT(cfg).double()
    idx = torch.randint(0, cfg.vocab_size, (2, cfg.block_size))
    targets = torch.randint(0, cfg.vocab_size, (2, cfg.block_size))
    with torch.no_grad():
        (logits, loss), states = capture_states(model, lambda: model(idx, targets))
        ref_logits, ref_loss = model.forward_reference(idx, targets)
    out = {"idx": idx.numpy(), "targets": targets.numpy(), "logits": logits.numpy(),
           "loss": np.float64(loss.item()), "ref_logits": ref_logits.numpy(),
           "ref_loss": np.float64(ref_loss.item())}
    for n, t in model.state_dict().items():
        out["w:" + n] = t.numpy()
    for i, (y, r) in enumerate(states):
        out[f"y{i}"] = y.numpy()
        out[f"rho{i}"] = r.numpy()
    np.savez_compressed(os.path.join(HERE, "model_small.npz"), **out)


def model_config(EfficientNGPT, ModelConfig, name, *, V, L, H, d, T, B, state_layers, row_stride):
    """A BASELINE-sized config in fp32: weights from torch.manual_seed(0) (CPU), ids from Generator(0).

    Stored: the loss, every token's log-sum-exp and target logit, weight
    fingerprints, and for the listed layers the represented state Y/rho of
    sequence 0 at every row_stride-th token plus rho of every token of
    sequence 0.  The first 64 vocabulary logits of sequence 0 are stored for
    T <= 256 only (they are 32 KB per 128 tokens)."""
    cfg = ModelConfig(vocab_size=V, block_size=T, n_layer=L, n_head=H, n_embd=d, mlp_ratio=4.0, dropout=0.0)
    torch.manual_seed(0)
    model = EfficientNGPT(cfg)
    model.eval()
    gen = torch.Generator().manual_seed(0)
    idx = torch.randint(0, V, (B, T), generator=gen)
    targets = torch.roll(idx, -1, dims=1)
    with torch.no_grad():
        (logits, loss), states = capture_states(model, lambda: model(idx, targets))
    names, fp = fingerprint(model.state_dict())
    rows = np.arange(0, T, row_stride)
    out = {"idx": idx.numpy().astype(np.int32), "targets": targets.numpy().astype(np.int32),
           "loss": np.float64(loss.item()), "w_names": names, "w_fp": fp,
           "lse": torch.logsumexp(logits.double(), dim=-1).numpy().astype(np.float32),
           "state_rows": rows,
           "state_layers": np.array(state_layers, dtype=np.int32)}
    if T <= 256:
        out["logits_b0_v64"] = logits[0, :, :64].numpy()
    # logits at the target positions for every token (what the loss reads).
    out["logits_at_target"] = logits.gather(-1, targets.unsqueeze(-1))[..., 0].numpy()
    for i in state_layers:
        y, r = states[i]
        h = (y / r.unsqueeze(-1))
        out[f"h{i}"] = h[0, rows].numpy().astype(np.float32)
        out[f"rho{i}"] = r[0].numpy().astype(np.float32)
        out[f"rhomax{i}"] = np.float32(r.max().item())
        out[f"finite{i}"] = np.bool_(torch.isfinite(y).all().item() and torch.isfinite(r).all().item())
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
    print(name, "loss", loss.item(), "max rho per stored layer",
          [round(float(out[f'rhomax{i}']), 2) for i in state_layers])


def isolated_attention(K):
    """The isolated nGPT attention op at B=8, H=16, T=2048, Dh=64 (inputs from Generator(1))."""
    B, H, T, D = 8, 16, 2048, 64
    g = torch.Generator().manual_seed(1)
    q = torch.randn(B, T, H, D, generator=g)
    k = torch.randn(B, T, H, D, generator=g)
    v = torch.randn(B, T, H, D, generator=g)
    s = torch.rand(D, generator=g) * 0.2 + 0.9
    q = q / q.norm(dim=-1, keepdim=True) * s
    k = k / k.norm(dim=-1, keepdim=True) * s
    o = K.causal_sdpa(q, k, v, scale=K.ngpt_attention_scale(D), dropout_p=0.0)
    rows = np.array([0, 1, 127, 128, 129, 1000, 2046, 2047])
    np.savez_compressed(os.path.join(HERE, "attn_cfg2.npz"), rows=rows,
                        o_b0_rows=o[0, rows].numpy(), o_b7_rows=o[7, rows].numpy(),
                        o_sum=np.float64(o.double().sum().item()),
                        o_abs_sum=np.float64(o.double().abs().sum().item()))


def main():
    EfficientNGPT, ModelConfig, K = _ref()
    torch.set_num_threads(os.cpu_count() or 1)
    jobs = {
        "ops": lambda: ops_vectors(K),
        "small": lambda: model_small(EfficientNGPT, ModelConfig),
        "attn": lambda: isolated_attention(K),
        "sphere": lambda: sphere_vectors(K),
        "optim": lambda: optimizer_step(EfficientNGPT, ModelConfig),
        "cfg1": lambda: model_config(EfficientNGPT, ModelConfig, "cfg1", V=50257, L=4, H=4, d=256, T=256, B=16,
                                     state_layers=[0, 1, 2, 3], row_stride=16),
        "cfg4": lambda: model_config(EfficientNGPT, ModelConfig, "cfg4_deep", V=50257, L=128, H=4, d=256, T=256,
                                     B=16, state_layers=list(range(0, 128, 8)) + [127], row_stride=32),
        # the benchmarked forward (L=16, d=1024, H=16, T=2048), two of its sequences
        "cfg3": lambda: model_config(EfficientNGPT, ModelConfig, "cfg3_d1024", V=50257, L=16, H=16, d=1024, T=2048,
                                     B=2, state_layers=[0, 3, 7, 11, 15], row_stride=128),
        # the long-context prefill forward (L=24, d=2048, head_dim 128, T=8192), one sequence
        "cfg5": lambda: model_config(EfficientNGPT, ModelConfig, "cfg5_d2048", V=50257, L=24, H=16, d=2048, T=8192,
                                     B=1, state_layers=[0, 5, 11, 17, 23], row_stride=1024),
    }
    for name in (sys.argv[1:] or list(jobs)):
        jobs[name]()


if __name__ == "__main__":
    sys.exit(main())
