"""The sm_100a backend: fused optimizers, single-tensor steps and casts."""

from ._native import load_library
from .adamw import AdamWCuda, cuda_adamw_step_
from .cast import cast, rn_cast_bf16, sr_cast_bf16
from .sgd import SGDMCuda, cuda_sgdm_step_


def is_available() -> bool:
    """True when a CUDA device of compute capability 10.0 is present and the
    kernel library loads."""
    import torch

    if not torch.cuda.is_available():
        return False
    try:
        load_library()
    except (OSError, RuntimeError):
        return False
    return torch.cuda.get_device_capability() == (10, 0)


__all__ = ["AdamWCuda", "SGDMCuda", "cast", "cuda_adamw_step_", "cuda_sgdm_step_",
           "is_available", "rn_cast_bf16", "sr_cast_bf16"]
