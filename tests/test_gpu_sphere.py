"""Optimizer-side sphere kernels (retraction and tangent projection, engpt/kernels.py:32-136) on B200.

Against the reference's outputs (fp64 golden vectors, compared at 1e-5 as the
reference's own test does, tests/test_kernels.py:78-106), against the torch
expressions at the model's matrix shapes, and one NGPTAdamW step
(engpt/optim.py:38-67) against the reference's step on the same weights and
gradients.
"""

import numpy as np
import pytest
import torch

from engpt_b200 import EfficientNGPT, ModelConfig, _lib, kernels as K
from engpt_b200.optim import NGPTAdamW

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _clean(cuda):
    _lib.clear_device_status()
    yield
    assert _lib.device_status() == 0


@pytest.mark.parametrize("tag", ["a", "b", "c"])
def test_sphere_ops_match_reference_vectors(golden, cuda, tag):
    g = golden("sphere_small.npz")
    w = torch.as_tensor(g[f"sph_{tag}_w"], dtype=torch.float32, device=cuda)
    gr = torch.as_tensor(g[f"sph_{tag}_g"], dtype=torch.float32, device=cuda)
    np.testing.assert_allclose(K.normalize_rows_(w.clone(), 1e-6).cpu().numpy(), g[f"sph_{tag}_rows"], atol=1e-5,
                               rtol=1e-5)
    np.testing.assert_allclose(K.normalize_columns_(w.clone(), 1e-6).cpu().numpy(), g[f"sph_{tag}_cols"],
                               atol=1e-5, rtol=1e-5)
    for kind, fn in (("row", K.project_row_grad_), ("col", K.project_column_grad_)):
        wn = torch.as_tensor(g[f"sph_{tag}_w{kind[0]}"], dtype=torch.float32, device=cuda)
        p = gr.clone()
        fn(wn, p)
        np.testing.assert_allclose(p.cpu().numpy(), g[f"sph_{tag}_p{kind}"], atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("shape", [(1024, 1024), (1024, 4096), (4096, 1024), (50257, 1024), (3, 5000), (5000, 3)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_sphere_ops_model_shapes_vs_torch(cuda, shape, dtype):
    """The model's normalised matrices: qkv / up_gate / embeddings by rows, out_proj / down_proj by columns."""
    gen = torch.Generator().manual_seed(shape[0] + shape[1])
    w = torch.randn(*shape, generator=gen).to(cuda, dtype)
    gr = torch.randn(*shape, generator=gen).to(cuda, dtype)
    wf, gf = w.float(), gr.float()
    tol = 1e-5 if dtype == torch.float32 else 8e-3
    rows = K.normalize_rows_(w.clone(), 1e-12)
    ref = wf / wf.norm(dim=-1, keepdim=True).clamp_min(1e-12)
    assert ((rows.float() - ref).abs().max() / ref.abs().max()).item() < tol
    cols = K.normalize_columns_(w.clone(), 1e-12)
    ref = wf / wf.norm(dim=0, keepdim=True).clamp_min(1e-12)
    assert ((cols.float() - ref).abs().max() / ref.abs().max()).item() < tol
    p = gr.clone()
    K.project_row_grad_(w, p)
    ref = gf - (gf * wf).sum(dim=-1, keepdim=True) * wf
    assert ((p.float() - ref).abs().max() / ref.abs().max()).item() < (tol if dtype == torch.float32 else 3e-2)
    p = gr.clone()
    K.project_column_grad_(w, p)
    ref = gf - wf * (gf * wf).sum(dim=0, keepdim=True)
    assert ((p.float() - ref).abs().max() / ref.abs().max()).item() < (tol if dtype == torch.float32 else 3e-2)


def test_ngpt_adamw_step_matches_reference(golden, cuda):
    """NGPTAdamW on CUDA parameters (projection and retraction on the kernels) vs the reference's step."""
    g = golden("optim_step.npz")
    cfg = ModelConfig(vocab_size=64, block_size=16, n_layer=2, n_head=2, n_embd=32, mlp_ratio=2.0, dropout=0.0)
    torch.manual_seed(2)
    model = EfficientNGPT(cfg).to(cuda)
    for n, p in model.named_parameters():
        p.grad = torch.as_tensor(g["g:" + n]).to(cuda)
    NGPTAdamW(model, lr=1e-2).step()
    for n, p in model.named_parameters():
        np.testing.assert_allclose(p.detach().cpu().numpy(), g["w:" + n], rtol=1e-5, atol=1e-6)
    assert model.parameter_norm_report()["max_unit_norm_error"] < 1e-5


def test_sphere_ops_reject_cpu_and_bad_shapes(cuda):
    with pytest.raises(RuntimeError, match="CUDA"):
        K.normalize_rows_(torch.zeros(4, 4))
    with pytest.raises(ValueError):
        K.project_row_grad_(torch.zeros(4, 4, device=cuda), torch.zeros(4, 5, device=cuda))
