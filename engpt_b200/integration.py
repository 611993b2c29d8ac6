"""Drop the CUDA hot-path ops into an imported reference ``engpt`` package.

``engpt/models.py:12-26`` imports its ops *by value* (``from .kernels import
...``), so rebinding ``engpt.kernels.X`` does not reach the model; the names
must be rebound in ``engpt.models`` itself.  ``patch_reference`` does that for
the three hot-path ops (and, optionally, the MLP and output-head helpers) and
returns an ``unpatch`` callable that restores the originals.
"""

from __future__ import annotations

from types import ModuleType
from typing import Callable, Dict

from . import kernels as K

HOT_PATH_OPS = ("qkv_postprocess_from_carried", "causal_sdpa", "carried_residual_gauge")
EXTRA_OPS = ("carried_up_gate_swiglu", "scaled_logits_from_carried")


def patch_reference(engpt_pkg: ModuleType, include_extras: bool = False,
                    via_torch_ops: bool = False) -> Callable[[], None]:
    """Rebind the reference model's op names to the engpt_b200 CUDA ops.

    ``engpt_pkg`` is the imported reference package (``import engpt``).  With
    ``via_torch_ops`` the three hot-path names are bound to the registered
    operators ``torch.ops.engpt_b200.*`` (same kernels, called through the
    PyTorch dispatcher) instead of the Python functions.  Returns a function
    that undoes the patch.
    """
    models = getattr(engpt_pkg, "models", None)
    if models is None:
        import importlib
        models = importlib.import_module(engpt_pkg.__name__ + ".models")
    names = HOT_PATH_OPS + (EXTRA_OPS if include_extras else ())
    if via_torch_ops:
        import torch
        from . import torch_ops  # noqa: F401  (registers the operators)
        impl = {n: getattr(torch.ops.engpt_b200, n) for n in HOT_PATH_OPS}
    else:
        impl = {}
    saved: Dict[str, object] = {}
    for name in names:
        if not hasattr(models, name):
            raise AttributeError(f"{models.__name__} has no attribute {name}; not a compatible engpt package")
        saved[name] = getattr(models, name)
        setattr(models, name, impl.get(name, getattr(K, name)))

    def unpatch() -> None:
        for n, fn in saved.items():
            setattr(models, n, fn)

    return unpatch
