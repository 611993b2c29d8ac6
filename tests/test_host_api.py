"""Host-side behaviour of the drop-in API (no GPU): config, module tree, error behaviour, patching."""

import types

import numpy as np
import pytest
import torch

from engpt_b200 import EfficientNGPT, ModelConfig, kernels as K, patch_reference
from tests.helpers import SMALL


def test_model_config_validation_matches_reference():
    with pytest.raises(ValueError, match="divisible"):
        ModelConfig(n_embd=30, n_head=4)
    with pytest.raises(ValueError):
        ModelConfig(vocab_size=0)
    with pytest.raises(ValueError):
        ModelConfig(block_size=0)
    with pytest.raises(ValueError):
        ModelConfig(n_layer=0)
    cfg = ModelConfig(n_embd=1024, n_head=16, mlp_ratio=4.0)
    assert cfg.head_dim == 64 and cfg.mlp_width == 4096


def test_state_dict_keys_and_unit_norms():
    torch.manual_seed(0)
    m = EfficientNGPT(ModelConfig(**SMALL))
    keys = list(m.state_dict().keys())
    assert keys[:3] == ["output_emb", "s_z", "token_emb.weight"]
    assert "blocks.1.qkv.weight" in keys and "blocks.0.alpha_attn_raw" in keys
    assert m.parameter_norm_report()["max_unit_norm_error"] < 2e-6


def test_ops_refuse_cpu_tensors():
    x = torch.zeros(1, 4, 3, 2, 8)
    with pytest.raises(RuntimeError, match="CUDA"):
        K.qkv_postprocess_from_carried(x, torch.ones(1, 4), torch.ones(4, 4), torch.zeros(4, 4),
                                       torch.ones(2, 8), 1e-6)
    q = torch.zeros(1, 4, 2, 8)
    with pytest.raises(RuntimeError, match="CUDA"):
        K.causal_sdpa(q, q, q, scale=1.0, dropout_p=0.0)
    with pytest.raises(RuntimeError, match="CUDA"):
        K.carried_residual_gauge(torch.zeros(2, 8), torch.ones(2), torch.zeros(2, 8), torch.zeros(8), 0, 0, 0)


def test_model_refuses_cpu_and_training_mode():
    torch.manual_seed(0)
    m = EfficientNGPT(ModelConfig(**SMALL))
    idx = torch.zeros(1, 4, dtype=torch.long)
    with pytest.raises(NotImplementedError, match="forward-only"):
        m(idx)
    with torch.no_grad():
        with pytest.raises(RuntimeError, match="CUDA"):
            m(idx)


def test_patch_reference_rebinds_model_namespace():
    models = types.ModuleType("fake_engpt.models")
    for n in ("qkv_postprocess_from_carried", "causal_sdpa", "carried_residual_gauge"):
        setattr(models, n, object())
    pkg = types.ModuleType("fake_engpt")
    pkg.models = models
    orig = models.causal_sdpa
    undo = patch_reference(pkg)
    assert models.causal_sdpa is K.causal_sdpa
    assert models.qkv_postprocess_from_carried is K.qkv_postprocess_from_carried
    undo()
    assert models.causal_sdpa is orig


def test_patch_reference_via_torch_ops():
    import torch
    models = types.ModuleType("fake_engpt2.models")
    for n in ("qkv_postprocess_from_carried", "causal_sdpa", "carried_residual_gauge"):
        setattr(models, n, object())
    pkg = types.ModuleType("fake_engpt2")
    pkg.models = models
    undo = patch_reference(pkg, via_torch_ops=True)
    assert models.causal_sdpa is torch.ops.engpt_b200.causal_sdpa
    assert models.carried_residual_gauge is torch.ops.engpt_b200.carried_residual_gauge
    undo()


def test_torch_ops_registered_with_reference_signatures():
    """torch.ops.engpt_b200.* exist with the reference ops' argument lists (engpt/kernels.py:139, 277, 417)."""
    import torch
    import engpt_b200  # noqa: F401  (registers the operators)
    schemas = {n: str(getattr(torch.ops.engpt_b200, n).default._schema) for n in
               ("qkv_postprocess_from_carried", "causal_sdpa", "carried_residual_gauge")}
    assert "(Tensor qkv, Tensor rho, Tensor cos, Tensor sin, Tensor qk_scale, float norm_eps) -> (Tensor, Tensor, Tensor)" \
        in schemas["qkv_postprocess_from_carried"]
    assert "(Tensor q, Tensor k, Tensor v, *, float scale, float dropout_p) -> Tensor" in schemas["causal_sdpa"]
    assert ("(Tensor y, Tensor rho, Tensor branch, Tensor alpha, float branch_eps, float residual_eps, "
            "float max_radius) -> (Tensor, Tensor)") in schemas["carried_residual_gauge"]


def test_torch_ops_fake_shapes_and_no_cpu_kernel():
    """Shape propagation without running a kernel (fake tensors), and no CPU implementation (no fallback)."""
    import torch
    from torch._subclasses.fake_tensor import FakeTensorMode
    import engpt_b200  # noqa: F401
    with FakeTensorMode():
        qkv = torch.empty(2, 9, 3, 4, 16, device="cuda", dtype=torch.bfloat16)
        rho = torch.empty(2, 9, device="cuda")
        q, k, v = torch.ops.engpt_b200.qkv_postprocess_from_carried(
            qkv, rho, torch.empty(9, 8, device="cuda"), torch.empty(9, 8, device="cuda"),
            torch.empty(4, 16, device="cuda"), 1e-6)
        assert q.shape == (2, 9, 4, 16) and q.dtype == torch.bfloat16
        o = torch.ops.engpt_b200.causal_sdpa(q, k, v, scale=4.0, dropout_p=0.0)
        assert o.shape == q.shape
        y, r = torch.ops.engpt_b200.carried_residual_gauge(
            torch.empty(2, 9, 64, device="cuda"), rho, torch.empty(2, 9, 64, device="cuda", dtype=torch.bfloat16),
            torch.empty(64, device="cuda"), 1e-6, 1e-6, 1024.0)
        assert y.shape == (2, 9, 64) and y.dtype == torch.float32 and r.shape == (2, 9)
    x = torch.zeros(1, 4, 1, 64)
    with pytest.raises(NotImplementedError):
        torch.ops.engpt_b200.causal_sdpa(x, x, x, scale=8.0, dropout_p=0.0)
