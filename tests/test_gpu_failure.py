"""Device-side failure reporting on B200, tested without faulting the GPU.

* A bounded wait that runs out (an mbarrier nothing arrives on, with a 50 us
  limit) records ENGPT_ERR_TIMEOUT and its site in the device status word,
  the CTA's other waiting role leaves through the abort word, the kernel
  returns, and the context keeps working: the next attention launch matches
  the oracle.
* A recorded argument error (an out-of-range target) stays in the status
  word until it is cleared but changes nothing that later launches compute:
  a normal forward run while it is set matches the oracle.
"""

import math

import numpy as np
import pytest
import torch

from engpt_b200 import EfficientNGPT, ModelConfig, _lib, kernels as K
from oracle import ngpt_oracle as O

pytestmark = pytest.mark.gpu

ERR_TIMEOUT, ERR_ARG = 5, 7


@pytest.fixture(autouse=True)
def _clean(cuda):
    _lib.clear_device_status()
    yield
    _lib.clear_device_status()


def _attention_matches_oracle(cuda, T=300):
    g = torch.Generator().manual_seed(T)
    q, k, v = (torch.randn(2, T, 2, 64, generator=g) for _ in range(3))
    q = q / q.norm(dim=-1, keepdim=True)
    k = k / k.norm(dim=-1, keepdim=True)
    qb, kb, vb = (x.to(cuda, torch.bfloat16) for x in (q, k, v))
    with torch.no_grad():
        o = K.causal_sdpa(qb, kb, vb, scale=8.0, dropout_p=0.0, impl="tcgen05")
    ref = O.causal_attention(*(x.float().cpu().numpy().astype(np.float64) for x in (qb, kb, vb)), 8.0)
    return float(np.abs(o.float().cpu().numpy() - ref).max())


def test_bounded_wait_runs_out_and_context_survives(cuda):
    flags = torch.zeros(2, dtype=torch.int32, device=cuda)
    _lib.call("engpt_selftest_wait_timeout", 50_000, flags.data_ptr(), _lib.stream_handle(cuda))
    word = _lib.device_status()
    assert word & 0xFF == ERR_TIMEOUT and word >> 8 == 99, hex(word)
    assert flags.tolist() == [1, 1]            # both roles reported failure; neither hung
    with pytest.raises(_lib.EngptError):
        _lib.raise_on_device_status()           # raises and clears
    assert _lib.device_status() == 0
    assert _attention_matches_oracle(cuda) < 1.5e-2
    assert _lib.device_status() == 0


def test_selftest_rejects_bad_limit(cuda):
    flags = torch.zeros(2, dtype=torch.int32, device=cuda)
    with pytest.raises(_lib.EngptError) as ei:
        _lib.call("engpt_selftest_wait_timeout", 0, flags.data_ptr(), _lib.stream_handle(cuda))
    assert ei.value.code == ERR_ARG


def test_recorded_argument_error_does_not_change_later_launches(cuda):
    cfg_kw = dict(vocab_size=512, block_size=256, n_layer=2, n_head=4, n_embd=256, mlp_ratio=4.0, dropout=0.0)
    torch.manual_seed(0)
    model = EfficientNGPT(ModelConfig(**cfg_kw))
    w = {k: v.detach().numpy() for k, v in model.state_dict().items()}
    model = model.to(cuda).eval()
    gen = torch.Generator().manual_seed(4)
    idx = torch.randint(0, 512, (2, 256), generator=gen)
    tgt = torch.roll(idx, -1, dims=1)
    bad = tgt.clone()
    bad[0, 3] = 512                              # outside the vocabulary
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        _, loss_bad = model(idx.to(cuda), bad.to(cuda))
        torch.cuda.synchronize()
        # the status word now holds the argument error; it is deliberately not cleared here
        _, loss = model(idx.to(cuda), tgt.to(cuda))
        o_err = _attention_matches_oracle(cuda)
    word = _lib.device_status()
    assert word & 0xFF == ERR_ARG, hex(word)
    assert math.isnan(loss_bad.item())
    _, ref_loss, _ = O.efficient_ngpt_forward(O.OracleConfig(**cfg_kw), w, idx.numpy(), tgt.numpy())
    assert abs(loss.item() - ref_loss) < 1e-2, (loss.item(), ref_loss)
    assert o_err < 1.5e-2
    with pytest.raises(_lib.EngptError) as ei:
        _lib.raise_on_device_status()
    assert ei.value.code == ERR_ARG
    assert _lib.device_status() == 0
