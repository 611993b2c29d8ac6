"""engpt_cross_entropy_noalloc: the cross-entropy entry point that allocates nothing.

Some callers cannot call cudaMalloc -- a host that only owns the buffers it was
handed (an FFI or embedded runtime without a device allocator), or a serving
loop that must not risk the device synchronisation cudaMalloc can cause.  For
them the library keeps the per-row scratch in a fixed device array instead of
asking for a buffer.  This test calls the entry point through the C ABI and
checks it against the allocating entry point (engpt_cross_entropy with a
caller-provided row buffer) on two calls in a row, the second smaller than the
first, so stale rows from the first call cannot leak into the second.

This file sorts last so that a run stopping at the first failure has already
run every other test.
"""

import ctypes

import numpy as np
import pytest
import torch

from engpt_b200 import _lib

pytestmark = pytest.mark.gpu

# the tolerance the cross-entropy tests use against the oracle
LOSS_TOL = 1e-4


def _inputs(rows, vocab, seed, dev, dtype):
    rng = np.random.default_rng(seed)
    logits = torch.as_tensor(rng.standard_normal((rows, vocab)) * 4.0, dtype=torch.float32).to(dev, dtype)
    tgt = rng.integers(0, vocab, rows)
    tgt[rows // 3] = -100  # ignore_index
    return logits.contiguous(), torch.as_tensor(tgt, dtype=torch.int64).to(dev)


def test_cross_entropy_noalloc_matches_allocating_entry_point(cuda):
    lib = _lib.load()
    stream = torch.cuda.current_stream(cuda).cuda_stream
    cases = [(4099, 50257, 11, torch.bfloat16), (333, 1001, 12, torch.float32)]
    for rows, vocab, seed, dtype in cases:  # two calls in a row
        logits, tgt = _inputs(rows, vocab, seed, cuda, dtype)
        code = _lib.dtype_code(dtype)
        row_loss = torch.empty(rows, device=cuda, dtype=torch.float32)
        loss_ref = torch.empty((), device=cuda, dtype=torch.float32)
        loss_new = torch.full((), float("nan"), device=cuda, dtype=torch.float32)
        rc = lib.engpt_cross_entropy(logits.data_ptr(), code, rows, vocab, vocab, tgt.data_ptr(),
                                     row_loss.data_ptr(), loss_ref.data_ptr(), stream)
        assert rc == 0, lib.engpt_last_error()
        rc = lib.engpt_cross_entropy_noalloc(logits.data_ptr(), code, rows, vocab, vocab, tgt.data_ptr(),
                                             loss_new.data_ptr(), stream)
        assert rc == 0, lib.engpt_last_error()
        torch.cuda.synchronize(cuda)
        assert np.isfinite(loss_new.item())
        assert abs(loss_new.item() - loss_ref.item()) <= LOSS_TOL, (loss_new.item(), loss_ref.item())


def test_cross_entropy_noalloc_rejects_too_many_rows(cuda):
    lib = _lib.load()
    rows = _lib.CE_NOALLOC_MAX_ROWS + 1
    rc = lib.engpt_cross_entropy_noalloc(ctypes.c_void_p(16), _lib.BF16, rows, 8, 8, ctypes.c_void_p(16),
                                         ctypes.c_void_p(16), None)
    assert rc == 1  # ENGPT_ERR_SHAPE, before any device work
    assert b"exceed" in lib.engpt_last_error()
