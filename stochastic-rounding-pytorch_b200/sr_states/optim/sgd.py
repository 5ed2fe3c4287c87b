"""Momentum SGD with FP32 math and a configurable momentum format, fused on sm_100a.

Same constructor, validation, state name and checkpoint layout as the
reference's SGDMReferenceSR / SGDMReferenceRN (sr_states/optim/sgd.py:12-69).
"""

from __future__ import annotations

import math

from ._state import StateOptimizer


def validate_sgdm(group):
    if not math.isfinite(group["lr"]) or group["lr"] < 0:
        raise ValueError(f"invalid learning rate: {group['lr']}")
    if not 0 <= group["momentum"] < 1:
        raise ValueError(f"invalid momentum value: {group['momentum']}")


class SGDMReferenceSR(StateOptimizer):
    """u' = u*momentum + g; p' = p - lr*u' (one FMA); u' stored with its format
    (BF16 stochastic by default).  Parameters must be CUDA tensors on sm_100a."""

    _state_names = ("momentum_buffer",)
    _uses_step = False
    _rounding_backend = "cuda"

    def __init__(self, params, lr, momentum=0.9, *, state_format=None, state_dtype=None,
                 rounding=None, seed=0):
        super().__init__(params, {"lr": lr, "momentum": momentum}, state_format=state_format,
                         state_dtype=state_dtype, rounding=rounding, seed=seed)

    def _validate_group(self, group):
        validate_sgdm(group)

    def _step_group(self, group, formats, items, rng_step):
        from ..cuda._fused import sgdm_group_step  # the backend imports this module

        sgdm_group_step(self, group, formats, items, rng_step)


class SGDMReferenceRN(SGDMReferenceSR):
    """Momentum SGD storing the momentum with round-to-nearest-even."""

    _forced_rounding = "nearest"
