"""Fused momentum SGD: the ``block_size`` optimizer class and the single-tensor step.

Drop-in for the reference's SGDMTriton and triton_sgdm_step_
(sr_states/triton/sgd.py:115-237); the work runs in libsrs_b200.so.
"""

from __future__ import annotations

import torch

from ..formats import StateFormat, resolve_formats
from ..optim.sgd import SGDMReferenceSR
from ..rounding import native_codes
from . import _native
from ._fused import sgdm_hparams
from ._launch import device_guard, stream_handle
from ._validate import check_block_size, check_nonnegative
from .adamw import single_row, validate_single


@torch.no_grad()
def cuda_sgdm_step_(
    parameter: torch.Tensor,
    gradient: torch.Tensor,
    momentum: torch.Tensor,
    *,
    lr: float,
    momentum_factor: float,
    seed: int,
    offset: int = 0,
    rounding: str | None = None,
    formats: tuple | dict | None = None,
    block_size: int = 256,
) -> None:
    """One momentum-SGD update of one tensor, in place, on the current CUDA stream.

    u' = u*momentum_factor + g and p' = fma(u', -lr, p) in FP32; u' is stored
    with its format using counter base state_key(seed, 0) at ``offset``.
    """
    if formats is None:
        formats = (StateFormat(momentum.dtype, "stochastic" if rounding is None else rounding),)
        rounding = None
    (fmt,) = resolve_formats(("momentum_buffer",), formats, rounding=rounding, backend="cuda")
    check_block_size(block_size)
    if momentum.dtype != fmt.dtype:
        raise ValueError("state dtype does not match its state format")
    check_nonnegative("learning rate", lr)
    if not 0 <= momentum_factor < 1:
        raise ValueError(f"invalid momentum value: {momentum_factor}")
    validate_single(parameter, gradient, momentum)
    if parameter.numel() == 0:
        return
    u_fmt, u_rule = native_codes(fmt.dtype, fmt.rounding)
    row = single_row(parameter, gradient, (momentum,), key=seed, offset=offset)
    with device_guard(parameter.device):
        _native.launcher().sgdm_single(row, u_fmt, u_rule, sgdm_hparams(lr, momentum_factor),
                                       stream_handle(parameter.device))


class SGDMCuda(SGDMReferenceSR):
    """Fused momentum SGD accepting the reference Triton class's ``block_size`` option."""

    def __init__(self, params, lr, momentum=0.9, *, state_format=None, state_dtype=None,
                 rounding=None, seed=0, block_size=256):
        self._initial_block_size = block_size
        super().__init__(params, lr=lr, momentum=momentum, state_format=state_format,
                         state_dtype=state_dtype, rounding=rounding, seed=seed)
        self.defaults["block_size"] = block_size

    def _validate_group(self, group):
        super()._validate_group(group)
        check_block_size(group.get("block_size", self._initial_block_size))

    def add_param_group(self, param_group):
        default = self.defaults.get("block_size", self._initial_block_size)
        super().add_param_group({"block_size": default, **param_group})
