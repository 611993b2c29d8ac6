"""CPU oracle for the enGPT forward hot path (test infrastructure only).

This module is the checker, not the product.  It restates, in plain numpy,
the arithmetic of the reference's forward path so that the CUDA kernels in
``engpt_b200`` can be compared against it on the same seeded inputs.  Only
``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import it.

Every function names the reference code it restates (paths are relative to
the Pi-Willie/enGPT project root).  The restatement is pinned against the
reference's own outputs by the golden fixtures in ``tests/golden/`` (made by
``tests/golden/make_golden.py``, which imports the reference package), see
``tests/test_oracle_golden.py``.

All functions accept a ``dtype`` (``np.float64`` by default) and carry out
their arithmetic in that dtype.
"""

from __future__ import annotations

import math
from typing import Dict, List, Optional, Tuple

import numpy as np

Array = np.ndarray


def rotary_frequencies(seq_len: int, head_dim: int, theta: float, dtype=np.float32) -> Tuple[Array, Array]:
    """cos/sin tables ``[T, rd/2]``; engpt/kernels.py:355-374.

    ``inv_freq`` and the angle table are formed in float32 exactly as the
    reference does (``arange(0, rd, 2) / rd``, ``theta ** x`` rounded to
    float32, fp32 reciprocal, fp32 outer product); cos/sin are taken of the
    float32 angle and rounded to float32, then cast to ``dtype``.
    """
    rd = head_dim - (head_dim % 2)
    if rd == 0:
        z = np.zeros((seq_len, 0), dtype=dtype)
        return z, z
    expo = np.arange(0, rd, 2, dtype=np.float32) / np.float32(rd)
    # theta ** expo rounded once to fp32 (as torch's fp32 pow), then an fp32 reciprocal
    powed = np.power(np.float64(theta), expo.astype(np.float64)).astype(np.float32)
    inv_freq = np.float32(1.0) / powed
    pos = np.arange(seq_len, dtype=np.float32)
    freqs = np.outer(pos, inv_freq).astype(np.float32)
    f64 = freqs.astype(np.float64)
    return np.cos(f64).astype(np.float32).astype(dtype), np.sin(f64).astype(np.float32).astype(dtype)


def apply_rope(x: Array, cos: Array, sin: Array) -> Array:
    """Interleaved-pair RoPE on ``[B, T, H, D]``; engpt/kernels.py:377-396.

    Pairs are ``(x[2i], x[2i+1])`` for ``i < rd/2``; a trailing odd lane passes
    through unchanged.
    """
    half = cos.shape[-1]
    rd = 2 * half
    if rd == 0:
        return x.copy()
    out = x.copy()
    ev = x[..., 0:rd:2]
    od = x[..., 1:rd:2]
    c = cos.reshape(1, cos.shape[0], 1, half)
    s = sin.reshape(1, sin.shape[0], 1, half)
    out[..., 0:rd:2] = ev * c - od * s
    out[..., 1:rd:2] = ev * s + od * c
    return out


def qkv_postprocess_from_carried(qkv: Array, rho: Array, cos: Array, sin: Array,
                                 qk_scale: Array, norm_eps: float) -> Tuple[Array, Array, Array]:
    """Raw ``[B,T,3,H,Dh]`` projection of carried ``Y`` -> attention inputs.

    Restates engpt/kernels.py:139-179: per-head L2 norms of raw q/k (taken
    before RoPE, which preserves them), guarded by ``rho * eps`` when
    ``eps > 0``; q/k are rotated, divided by their norms and scaled by the
    effective ``s_qk``; v is divided by ``rho``.
    """
    bsz, seq_len, _, n_head, head_dim = qkv.shape
    q_raw, k_raw, v_raw = qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
    q_den = np.sqrt(np.sum(q_raw * q_raw, axis=-1))
    k_den = np.sqrt(np.sum(k_raw * k_raw, axis=-1))
    if norm_eps > 0:
        guard = rho[:, :, None] * norm_eps
        q_den = np.maximum(q_den, guard)
        k_den = np.maximum(k_den, guard)
    scale = qk_scale.reshape(1, 1, n_head, head_dim)
    q = apply_rope(q_raw, cos, sin) / q_den[..., None] * scale
    k = apply_rope(k_raw, cos, sin) / k_den[..., None] * scale
    v = v_raw / rho.reshape(bsz, seq_len, 1, 1)
    return q, k, v


def causal_attention(q: Array, k: Array, v: Array, scale: float) -> Array:
    """``softmax(scale * q k^T + causal mask) v`` on ``[B,T,H,D]`` inputs.

    The reference delegates this to ``torch.nn.functional.scaled_dot_product_attention``
    with ``is_causal=True`` (engpt/kernels.py:417-431); here it is written out
    as the textbook max-subtracted softmax.
    """
    bsz, seq_len, n_head, head_dim = q.shape
    qh = np.transpose(q, (0, 2, 1, 3))
    kh = np.transpose(k, (0, 2, 1, 3))
    vh = np.transpose(v, (0, 2, 1, 3))
    s = np.matmul(qh, np.transpose(kh, (0, 1, 3, 2))) * q.dtype.type(scale)
    mask = np.triu(np.ones((seq_len, seq_len), dtype=bool), k=1)
    s = np.where(mask[None, None], -np.inf, s)
    m = np.max(s, axis=-1, keepdims=True)
    p = np.exp(s - m)
    p = p / np.sum(p, axis=-1, keepdims=True)
    o = np.matmul(p, vh)
    return np.transpose(o, (0, 2, 1, 3))


def carried_residual(y: Array, rho: Array, branch: Array, alpha: Array,
                     branch_eps: float, residual_eps: float) -> Tuple[Array, Array]:
    """One-reduction carried nGPT residual; engpt/kernels.py:232-274.

    With ``beta = 1 - alpha`` and the four row sums
    ``R0 = sum b^2, R1 = sum beta^2 y^2, R2 = sum alpha^2 b^2, R3 = sum alpha beta y b``,
    ``c_b = max(sqrt R0, eps_b)``, ``|u|^2 = c_b^2 R1 + rho^2 R2 + 2 rho c_b R3``,
    ``rho+ = max(|u|, eps_r rho c_b)`` and ``u = beta c_b y + alpha rho b``.
    """
    alpha = alpha.reshape((1,) * (branch.ndim - 1) + (-1,))
    beta = 1.0 - alpha
    r0 = np.sum(branch * branch, axis=-1)
    r1 = np.sum(beta * beta * y * y, axis=-1)
    r2 = np.sum(alpha * alpha * branch * branch, axis=-1)
    r3 = np.sum(alpha * beta * y * branch, axis=-1)
    cb = np.sqrt(np.maximum(r0, 0.0))
    if branch_eps > 0:
        cb = np.maximum(cb, branch_eps)
    rho_cb = rho * cb
    u_norm_sq = cb * cb * r1 + rho * rho * r2 + 2.0 * rho_cb * r3
    rho_plus = np.sqrt(np.maximum(u_norm_sq, 0.0))
    if residual_eps > 0:
        rho_plus = np.maximum(rho_plus, residual_eps * rho_cb)
    u = beta * cb[..., None] * y + alpha * rho[..., None] * branch
    return u, rho_plus


def gauge_carried_state(y: Array, rho: Array, max_radius: float) -> Tuple[Array, Array]:
    """Exact gauge change ``(y/g, rho/g)``, ``g = max(rho/max_radius, 1)``; engpt/kernels.py:327-338."""
    if max_radius <= 0:
        return y, rho
    g = np.maximum(rho / max_radius, 1.0)
    return y / g[..., None], rho / g


def carried_residual_gauge(y: Array, rho: Array, branch: Array, alpha: Array, branch_eps: float,
                           residual_eps: float, max_radius: float) -> Tuple[Array, Array]:
    """Residual with the gauge folded in; engpt/kernels.py:277-324."""
    u, rho_plus = carried_residual(y, rho, branch, alpha, branch_eps, residual_eps)
    return gauge_carried_state(u, rho_plus, max_radius)


def normalize_last_dim(x: Array, eps: float) -> Array:
    """``x / max(|x|, eps)`` on the last axis; engpt/kernels.py:85-95."""
    den = np.sqrt(np.sum(x * x, axis=-1, keepdims=True))
    if eps > 0:
        den = np.maximum(den, eps)
    return x / den


def reference_residual(h: Array, branch: Array, alpha: Array, branch_eps: float, residual_eps: float) -> Array:
    """Materialised nGPT residual ``N((1-a) h + a N(b))``; engpt/kernels.py:341-352."""
    alpha = alpha.reshape((1,) * (branch.ndim - 1) + (-1,))
    mixed = (1.0 - alpha) * h + alpha * normalize_last_dim(branch, branch_eps)
    return normalize_last_dim(mixed, residual_eps)


def normalize_rows(x: Array, eps: float) -> Array:
    """Rows to unit L2 norm: ``x / max(|x_row|, eps)``; engpt/kernels.py:98-105 (and its Triton kernel 32-42,
    whose ``sqrt(max(ss, eps^2))`` is the same denominator)."""
    return x / np.maximum(np.sqrt(np.sum(x * x, axis=-1, keepdims=True)), eps)


def normalize_columns(x: Array, eps: float) -> Array:
    """Columns to unit L2 norm; engpt/kernels.py:108-116 (Triton kernel 44-55)."""
    return x / np.maximum(np.sqrt(np.sum(x * x, axis=0, keepdims=True)), eps)


def project_row_grad(weight: Array, grad: Array) -> Array:
    """``grad - (grad . w)_row w``: the tangent space of unit rows; engpt/kernels.py:119-125 (Triton 57-67)."""
    return grad - np.sum(grad * weight, axis=-1, keepdims=True) * weight


def project_column_grad(weight: Array, grad: Array) -> Array:
    """``grad - w (grad . w)_column``: the tangent space of unit columns; engpt/kernels.py:128-136 (Triton 69-81)."""
    return grad - weight * np.sum(grad * weight, axis=0, keepdims=True)


def silu(x: Array) -> Array:
    return x / (1.0 + np.exp(-x))


def carried_up_gate_swiglu(y: Array, rho: Array, weight: Array, s_u: Array, s_gate: Array,
                           sqrt_d: float, scale_u_by_sqrt_d: bool) -> Array:
    """MLP up/gate + SwiGLU from carried state; engpt/kernels.py:182-206."""
    h = y / rho[..., None]
    ug = h @ weight.T
    width = ug.shape[-1] // 2
    u = ug[..., :width] * s_u
    if scale_u_by_sqrt_d:
        u = u * sqrt_d
    gate = ug[..., width:] * s_gate * sqrt_d
    return u * silu(gate)


def scaled_logits_from_carried(y: Array, rho: Array, output_emb: Array, logit_scale: Array) -> Array:
    """``<Y, E_out[v]> s_z[v] / rho``; engpt/kernels.py:209-229."""
    return (y / rho[..., None]) @ (output_emb * logit_scale[:, None]).T


def cross_entropy(logits: Array, targets: Array, ignore_index: int = -100) -> float:
    """Mean token cross-entropy (engpt/models.py:328-333 via ``F.cross_entropy``).

    Targets equal to ``ignore_index`` (F.cross_entropy's default -100) are left
    out of the mean; with no valid target the mean is NaN, as in torch.
    """
    flat = logits.reshape(-1, logits.shape[-1]).astype(np.float64)
    t = targets.reshape(-1)
    keep = t != ignore_index
    if not keep.any():
        return float("nan")
    flat, t = flat[keep], t[keep]
    m = flat.max(axis=-1, keepdims=True)
    lse = (m[:, 0] + np.log(np.exp(flat - m).sum(axis=-1)))
    return float(np.mean(lse - flat[np.arange(flat.shape[0]), t]))


def row_logsumexp(logits: Array) -> Array:
    flat = logits.astype(np.float64)
    m = flat.max(axis=-1, keepdims=True)
    return m[..., 0] + np.log(np.exp(flat - m).sum(axis=-1))


class OracleConfig:
    """Minimal mirror of the fields of ``ModelConfig`` (engpt/config.py:6-39) the forward reads."""

    def __init__(self, vocab_size, block_size, n_layer, n_head, n_embd, mlp_ratio=4.0,
                 norm_eps=1e-6, rope_theta=10000.0, alpha_init=0.05, logit_scale_init=8.0,
                 scale_mlp_u_by_sqrt_d=True, carried_gauge_max=1024.0, **_ignored):
        self.vocab_size = vocab_size
        self.block_size = block_size
        self.n_layer = n_layer
        self.n_head = n_head
        self.n_embd = n_embd
        self.mlp_ratio = mlp_ratio
        self.norm_eps = norm_eps
        self.rope_theta = rope_theta
        self.alpha_init = alpha_init
        self.logit_scale_init = logit_scale_init
        self.scale_mlp_u_by_sqrt_d = scale_mlp_u_by_sqrt_d
        self.carried_gauge_max = carried_gauge_max

    @property
    def head_dim(self) -> int:
        return self.n_embd // self.n_head

    @property
    def mlp_width(self) -> int:
        return int(self.mlp_ratio * self.n_embd)


def efficient_ngpt_forward(cfg: OracleConfig, weights: Dict[str, Array], idx: Array,
                           targets: Optional[Array] = None, dtype=np.float64,
                           keep_states: bool = False, state_rows=None):
    """``EfficientNGPT.forward`` (engpt/models.py:263-292) with the block of engpt/models.py:140-182.

    ``weights`` uses the reference's ``state_dict`` names.  Returns
    ``(logits, loss, states)`` where ``states`` is a list of per-layer
    ``(Y, rho)`` pairs when ``keep_states`` (optionally restricted to the batch
    rows in ``state_rows``).
    """
    w = {k: np.asarray(v, dtype=dtype) for k, v in weights.items()}
    d = cfg.n_embd
    base = 1.0 / math.sqrt(float(d))
    bsz, seq_len = idx.shape
    if seq_len > cfg.block_size:
        raise ValueError("sequence length exceeds block_size")
    y = w["token_emb.weight"][idx]
    rho = np.ones((bsz, seq_len), dtype=dtype)
    cos, sin = rotary_frequencies(seq_len, cfg.head_dim, cfg.rope_theta, dtype=dtype)
    attn_scale = math.sqrt(float(cfg.head_dim))
    sqrt_d = math.sqrt(float(d))
    states: List[Tuple[Array, Array]] = []
    for i in range(cfg.n_layer):
        p = f"blocks.{i}."
        alpha_attn = np.abs(w[p + "alpha_attn_raw"]) * (cfg.alpha_init / base)
        alpha_mlp = np.abs(w[p + "alpha_mlp_raw"]) * (cfg.alpha_init / base)
        qk_scale = w[p + "s_qk"] * (1.0 / base)
        qkv = (y @ w[p + "qkv.weight"].T).reshape(bsz, seq_len, 3, cfg.n_head, cfg.head_dim)
        q, k, v = qkv_postprocess_from_carried(qkv, rho, cos, sin, qk_scale, cfg.norm_eps)
        attn = causal_attention(q, k, v, attn_scale)
        branch = attn.reshape(bsz, seq_len, d) @ w[p + "out_proj.weight"].T
        y, rho = carried_residual_gauge(y, rho, branch, alpha_attn, cfg.norm_eps, cfg.norm_eps,
                                        cfg.carried_gauge_max)
        hidden = carried_up_gate_swiglu(y, rho, w[p + "up_gate.weight"], w[p + "s_u"], w[p + "s_gate"],
                                        sqrt_d, cfg.scale_mlp_u_by_sqrt_d)
        branch = hidden @ w[p + "down_proj.weight"].T
        y, rho = carried_residual_gauge(y, rho, branch, alpha_mlp, cfg.norm_eps, cfg.norm_eps,
                                        cfg.carried_gauge_max)
        if keep_states:
            if state_rows is None:
                states.append((y.copy(), rho.copy()))
            else:
                states.append((y[state_rows].copy(), rho[state_rows].copy()))
    logit_scale = w["s_z"] * (cfg.logit_scale_init / base)
    logits = scaled_logits_from_carried(y, rho, w["output_emb"], logit_scale)
    loss = cross_entropy(logits, targets) if targets is not None else None
    return logits, loss, states
