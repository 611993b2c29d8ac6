"""Shared helpers for the parity tests (configs, seeded models, error metrics)."""

import numpy as np
import torch

from engpt_b200 import EfficientNGPT, ModelConfig

# BASELINE-sized configurations (EfficientNGPT forward)
CFG1 = dict(vocab_size=50257, block_size=256, n_layer=4, n_head=4, n_embd=256, mlp_ratio=4.0, dropout=0.0)
CFG1_BT = (16, 256)
CFG4 = dict(vocab_size=50257, block_size=256, n_layer=128, n_head=4, n_embd=256, mlp_ratio=4.0, dropout=0.0)
CFG4_BT = (16, 256)
# the benchmarked forward and the long-context prefill forward
CFG3 = dict(vocab_size=50257, block_size=2048, n_layer=16, n_head=16, n_embd=1024, mlp_ratio=4.0, dropout=0.0)
CFG5 = dict(vocab_size=50257, block_size=8192, n_layer=24, n_head=16, n_embd=2048, mlp_ratio=4.0, dropout=0.0)
SMALL = dict(vocab_size=32, block_size=12, n_layer=2, n_head=2, n_embd=32, mlp_ratio=2.0, dropout=0.0,
             alpha_init=0.1)


def seeded_model(cfg_kwargs, seed=0):
    torch.manual_seed(seed)
    model = EfficientNGPT(ModelConfig(**cfg_kwargs))
    model.eval()
    return model


def state_numpy(model):
    return {k: v.detach().cpu().numpy() for k, v in model.state_dict().items()}


def fingerprint(sd):
    names = sorted(sd.keys())
    fp = np.zeros((len(names), 6), dtype=np.float64)
    for i, n in enumerate(names):
        t = sd[n].detach().double().reshape(-1)
        fp[i, 0] = t.sum().item()
        fp[i, 1] = (t * t).sum().item()
        fp[i, 2:6] = t[:4].numpy() if t.numel() >= 4 else np.pad(t.numpy(), (0, 4 - t.numel()))
    return np.array(names), fp


def row_rel_err(a, b):
    """max over rows of |a - b|_2 / |b|_2 (rows = last axis)."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    num = np.sqrt(((a - b) ** 2).sum(-1))
    den = np.sqrt((b ** 2).sum(-1))
    return float(np.max(num / np.maximum(den, 1e-30)))
