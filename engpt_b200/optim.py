"""nGPT optimizer step on the B200 sphere kernels -- engpt/optim.py:38-109.

``NGPTAdamW`` is AdamW (no weight decay) whose step first projects the
gradients of the normalised matrices onto the tangent spaces of their unit
rows or columns and, after the AdamW update, retracts the matrices back onto
the sphere (``EfficientNGPT.project_parameters_``).  Which matrices are rows
and which are columns follows engpt/optim.py:86-105 and
engpt/models.py:223-230, 356-361.  The projections and retractions run on
the CUDA kernels of ``engpt_b200.kernels`` for CUDA parameters (the AdamW
update itself is PyTorch's).
"""

from __future__ import annotations

import torch

from . import kernels as K
from .models import EfficientNGPT


def _project_row_grad_(weight: torch.Tensor, grad: torch.Tensor) -> None:
    if weight.is_cuda:
        K.project_row_grad_(weight, grad)
    else:  # the reference's PyTorch expression, engpt/kernels.py:125
        grad.sub_((grad * weight).sum(dim=-1, keepdim=True) * weight)


def _project_col_grad_(weight: torch.Tensor, grad: torch.Tensor) -> None:
    if weight.is_cuda:
        K.project_column_grad_(weight, grad)
    else:  # engpt/kernels.py:136
        grad.sub_(weight * (grad * weight).sum(dim=0, keepdim=True))


@torch.no_grad()
def project_ngpt_gradients_(model: EfficientNGPT) -> None:
    """Tangent projection of every normalised matrix's gradient -- engpt/optim.py:86-104."""
    if model.token_emb.weight.grad is not None:
        _project_row_grad_(model.token_emb.weight, model.token_emb.weight.grad)
    if model.output_emb.grad is not None:
        _project_row_grad_(model.output_emb, model.output_emb.grad)
    for block in model.blocks:
        if block.qkv.weight.grad is not None:
            _project_row_grad_(block.qkv.weight, block.qkv.weight.grad)
        if block.out_proj.weight.grad is not None:
            _project_col_grad_(block.out_proj.weight, block.out_proj.weight.grad)
        if block.up_gate.weight.grad is not None:
            _project_row_grad_(block.up_gate.weight, block.up_gate.weight.grad)
        if block.down_proj.weight.grad is not None:
            _project_col_grad_(block.down_proj.weight, block.down_proj.weight.grad)


@torch.no_grad()
def project_ngpt_parameters_(model: EfficientNGPT, eps: float = 1e-12) -> None:
    """Exact retraction of every normalised matrix -- engpt/optim.py:107-109."""
    model.project_parameters_(eps=eps)


class NGPTAdamW(torch.optim.AdamW):
    """Spherical AdamW -- engpt/optim.py:38-67: project gradients, AdamW step (no weight decay), retract."""

    def __init__(self, model: EfficientNGPT, *, lr: float = 3e-4, betas=(0.9, 0.95), eps: float = 1e-8) -> None:
        self.model = model
        super().__init__(model.parameters(), lr=lr, betas=betas, eps=eps, weight_decay=0.0)

    def step(self, closure=None):  # type: ignore[override]
        project_ngpt_gradients_(self.model)
        loss = super().step(closure=closure)
        project_ngpt_parameters_(self.model)
        return loss


def build_ngpt_adamw(model: EfficientNGPT, *, lr: float = 3e-4, betas=(0.9, 0.95)) -> NGPTAdamW:
    """engpt/optim.py:70-76."""
    return NGPTAdamW(model, lr=lr, betas=betas)
