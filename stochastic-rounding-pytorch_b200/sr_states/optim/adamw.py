"""AdamW with FP32 math and per-moment storage formats, fused on sm_100a.

Same constructor, hyperparameter validation, state names and checkpoint layout
as the reference's AdamWReferenceSR / AdamWReferenceRN
(sr_states/optim/adamw.py:12-79).  The update itself is the fused multi-tensor
kernel: one launch per group and device (sr_states/cuda/_fused.py).
"""

from __future__ import annotations

import math

from ._state import StateOptimizer


def validate_adamw(group):
    for name in ("lr", "eps", "weight_decay"):
        if not math.isfinite(group[name]) or group[name] < 0:
            raise ValueError(f"invalid {name}: {group[name]}")
    betas = group["betas"]
    if len(betas) != 2 or any(not 0 <= beta < 1 for beta in betas):
        raise ValueError(f"invalid beta values: {betas}")


class AdamWReferenceSR(StateOptimizer):
    """AdamW; both moments stochastically rounded to BF16 by default.

    Per element (FP32, PyTorch's CPU operation order): m' = fma(g, 1-b1, m*b1),
    v' = fma((1-b2)*g, g, v*b2), p' = p*(1-lr*wd) + (-lr/bc1 * m') / (sqrt(v')/sqrt(bc2) + eps);
    the parameter update uses the unrounded moments, then each moment is stored
    with its own format.  Parameters must be CUDA tensors on an sm_100a GPU.
    """

    _state_names = ("exp_avg", "exp_avg_sq")
    _uses_step = True
    _rounding_backend = "cuda"

    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-2, *,
                 state_format=None, state_dtype=None, rounding=None, seed=0):
        super().__init__(params, {"lr": lr, "betas": betas, "eps": eps,
                                  "weight_decay": weight_decay},
                         state_format=state_format, state_dtype=state_dtype, rounding=rounding,
                         seed=seed)

    def _validate_group(self, group):
        validate_adamw(group)

    def _step_group(self, group, formats, items, rng_step):
        from ..cuda._fused import adamw_group_step  # the backend imports this module

        adamw_group_step(self, group, formats, items, rng_step)


class AdamWReferenceRN(AdamWReferenceSR):
    """AdamW storing every moment with round-to-nearest-even; ``state_format``,
    group overrides and checkpoints choose only each state's dtype."""

    _forced_rounding = "nearest"
