"""The reference package's own model with the B200 ops patched in (the drop-in boundary exercised for real).

The reference ``engpt`` package is taken from ``baseline/_ref`` (installed there
from the reference sources; git-ignored).  Its ``EfficientNGPT`` runs on the GPU
under bf16 autocast, first unpatched (PyTorch ops), then with
``patch_reference`` (Python ops, and the registered ``torch.ops.engpt_b200``
operators).  Per-layer ``(y, rho)`` is captured with forward hooks on the
reference's ``EfficientNGPTBlock`` (its output is the ``(y, rho)`` tuple,
engpt/models.py:182): represented state Y/rho within 2e-2 and the loss
within 1e-3 of the unpatched reference.
"""

import os
import sys

import numpy as np
import pytest
import torch

from engpt_b200 import patch_reference
from tests.helpers import row_rel_err

pytestmark = pytest.mark.gpu

REF_DIR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")


def _import_reference():
    if not os.path.isdir(os.path.join(REF_DIR, "engpt")):
        pytest.skip("reference package not installed under baseline/_ref")
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    import engpt
    return engpt


def _run(engpt, model, idx, tgt):
    states = []
    hooks = [b.register_forward_hook(lambda m, i, o: states.append((o[0].detach().float().clone(),
                                                                       o[1].detach().float().clone())))
             for b in model.blocks]
    try:
        with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
            logits, loss = model(idx, tgt)
    finally:
        for h in hooks:
            h.remove()
    return logits, loss, states


@pytest.mark.parametrize("via_torch_ops", [False, True])
def test_reference_model_with_patched_ops_matches_unpatched(cuda, via_torch_ops):
    engpt = _import_reference()
    cfg = engpt.ModelConfig(vocab_size=50257, block_size=512, n_layer=4, n_head=16, n_embd=1024, mlp_ratio=4.0,
                            dropout=0.0)
    torch.manual_seed(0)
    model = engpt.EfficientNGPT(cfg).to(cuda).eval()
    gen = torch.Generator().manual_seed(0)
    idx = torch.randint(0, cfg.vocab_size, (4, 512), generator=gen).to(cuda)
    tgt = torch.roll(idx, -1, dims=1)
    _, loss_ref, st_ref = _run(engpt, model, idx, tgt)
    undo = patch_reference(engpt, via_torch_ops=via_torch_ops)
    try:
        assert engpt.models.causal_sdpa is not None
        _, loss_b200, st_b200 = _run(engpt, model, idx, tgt)
    finally:
        undo()
    assert len(st_ref) == len(st_b200) == cfg.n_layer
    for (y0, r0), (y1, r1) in zip(st_ref, st_b200):
        h0 = (y0 / r0.unsqueeze(-1)).reshape(-1, cfg.n_embd).cpu().numpy()
        h1 = (y1 / r1.unsqueeze(-1)).reshape(-1, cfg.n_embd).cpu().numpy()
        assert row_rel_err(h1, h0) < 2e-2
    assert abs(loss_b200.item() - loss_ref.item()) < 1e-3, (loss_b200.item(), loss_ref.item())
