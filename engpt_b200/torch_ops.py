"""The hot-path ops registered as PyTorch operators: ``torch.ops.engpt_b200.*``.

Registering them with ``torch.library`` makes the CUDA kernels first-class
PyTorch operators (visible to ``torch.ops``, to the dispatcher and, through
the fake implementations below, to tracing and shape propagation) while the
computation still runs through the C ABI of ``libengpt_b200.so``.  The
operator signatures are those of the reference ops they replace:

* ``engpt_b200::qkv_postprocess_from_carried(qkv, rho, cos, sin, qk_scale, norm_eps) -> (q, k, v)``
  -- engpt/kernels.py:139-179
* ``engpt_b200::causal_sdpa(q, k, v, *, scale, dropout_p) -> o`` -- engpt/kernels.py:417-431
* ``engpt_b200::carried_residual_gauge(y, rho, branch, alpha, branch_eps, residual_eps, max_radius) -> (y, rho)``
  -- engpt/kernels.py:277-324

Only CUDA implementations are registered: a CPU tensor finds no kernel and
the dispatcher raises (there is no CPU fallback).  Like the underlying ops
they are forward-only.
"""

from __future__ import annotations

from typing import Tuple

import torch
from torch import Tensor

from . import kernels as K

NAMESPACE = "engpt_b200"


@torch.library.custom_op(f"{NAMESPACE}::qkv_postprocess_from_carried", mutates_args=(), device_types="cuda")
def qkv_postprocess_from_carried(qkv: Tensor, rho: Tensor, cos: Tensor, sin: Tensor, qk_scale: Tensor,
                                 norm_eps: float) -> Tuple[Tensor, Tensor, Tensor]:
    return K.qkv_postprocess_from_carried(qkv, rho, cos, sin, qk_scale, norm_eps)


@qkv_postprocess_from_carried.register_fake
def _qkv_fake(qkv, rho, cos, sin, qk_scale, norm_eps):
    bsz, seq_len, _, n_head, head_dim = qkv.shape
    return tuple(qkv.new_empty(bsz, seq_len, n_head, head_dim) for _ in range(3))


@torch.library.custom_op(f"{NAMESPACE}::causal_sdpa", mutates_args=(), device_types="cuda")
def causal_sdpa(q: Tensor, k: Tensor, v: Tensor, *, scale: float, dropout_p: float) -> Tensor:
    return K.causal_sdpa(q, k, v, scale=scale, dropout_p=dropout_p)


@causal_sdpa.register_fake
def _sdpa_fake(q, k, v, *, scale, dropout_p):
    return q.new_empty(q.shape)


@torch.library.custom_op(f"{NAMESPACE}::carried_residual_gauge", mutates_args=(), device_types="cuda")
def carried_residual_gauge(y: Tensor, rho: Tensor, branch: Tensor, alpha: Tensor, branch_eps: float,
                           residual_eps: float, max_radius: float) -> Tuple[Tensor, Tensor]:
    return K.carried_residual_gauge(y, rho, branch, alpha, branch_eps, residual_eps, max_radius)


@carried_residual_gauge.register_fake
def _residual_fake(y, rho, branch, alpha, branch_eps, residual_eps, max_radius):
    dt = torch.promote_types(y.dtype, branch.dtype)
    return y.new_empty(y.shape, dtype=dt), rho.new_empty(rho.shape, dtype=dt)


OPS = ("qkv_postprocess_from_carried", "causal_sdpa", "carried_residual_gauge")
