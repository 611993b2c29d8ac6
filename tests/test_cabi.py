"""The C-ABI library loads and exports every entry point declared in include/engpt_b200.h (no GPU needed)."""

import ctypes
import os
import re

import pytest

from engpt_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "engpt_b200.h")).read()
    return sorted(set(re.findall(r"ENGPT_API\s+[\w\s\*]+?\b(engpt_\w+)\s*\(", text)))


def test_header_declares_the_hot_path_entry_points():
    syms = declared_symbols()
    for name in ("engpt_qkv_postprocess", "engpt_causal_attention", "engpt_carried_residual_gauge",
                 "engpt_last_error", "engpt_device_status"):
        assert name in syms


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_binding_covers_every_declared_symbol():
    assert sorted(_lib.SIGNATURES) == declared_symbols()


def test_host_side_validation_without_gpu():
    lib = _lib.load()
    assert lib.engpt_abi_version() == 101
    # argument checks run on the host before any CUDA call
    rc = lib.engpt_carried_residual_gauge(None, None, None, 1, None, 1.0, 0, 0.0, 0.0, 0.0, 4, 8, None, None,
                                          None, 0, None)
    assert rc == 7 and b"null" in lib.engpt_last_error()
    rc = lib.engpt_qkv_postprocess(None, 5, None, None, None, 0, None, 1.0, 0.0, 1, 1, 1, 8, None, None, None, 0,
                                   None)
    assert rc == 2
    strides = (ctypes.c_int64 * 12)(*([1] * 12))
    rc = lib.engpt_causal_attention(None, None, None, None, 1, 1, 4, 1, 64, 1.0, strides, 9, None)
    assert rc == 7
    # empty inputs are a no-op
    assert lib.engpt_carried_residual_gauge(None, None, None, 1, None, 1.0, 0, 0.0, 0.0, 0.0, 0, 8, None, None,
                                            None, 0, None) == 0
