"""B200-native (sm_100a) forward hot path of enGPT (carried-radius nGPT).

Drop-in names for the reference package:

* ``ModelConfig`` -- engpt/config.py
* ``EfficientNGPT`` / ``EfficientNGPTBlock`` -- engpt/models.py (same
  ``state_dict`` keys and seeded init; forward runs the fused CUDA engine)
* ``engpt_b200.kernels`` -- the engpt.kernels hot-path ops on CUDA kernels
* ``torch.ops.engpt_b200.*`` -- the three hot-path ops as registered
  PyTorch operators (``engpt_b200.torch_ops``)
* ``patch_reference(engpt_pkg)`` -- rebinds the hot-path ops inside an
  imported reference package so its own model calls the CUDA kernels
"""

__version__ = "0.1.0"

from .config import ModelConfig
from .models import EfficientNGPT, EfficientNGPTBlock
from . import kernels
from . import torch_ops  # registers torch.ops.engpt_b200.{qkv_postprocess_from_carried, causal_sdpa, carried_residual_gauge}
from .integration import patch_reference

__all__ = ["EfficientNGPT", "EfficientNGPTBlock", "ModelConfig", "kernels", "patch_reference", "__version__"]
