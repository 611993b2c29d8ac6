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
