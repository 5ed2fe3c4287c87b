"""Fused AdamW: the ``block_size`` optimizer class and the single-tensor step.

Drop-in for the reference's AdamWTriton and triton_adamw_step_
(sr_states/triton/adamw.py:160-319); the work runs in libsrs_b200.so.
"""

from __future__ import annotations

import torch

from ..formats import StateFormat, resolve_formats
from ..optim.adamw import AdamWReferenceSR
from ..rounding import native_codes
from . import _native
from ._fused import adamw_hparams
from ._launch import device_guard, stream_handle
from ._validate import check_block_size, check_disjoint, check_layout, check_nonnegative, spans_of

_MASK32 = 0xFFFFFFFF


def _check_hyperparameters(lr, betas, eps, weight_decay):
    check_nonnegative("learning rate", lr)
    check_nonnegative("epsilon", eps)
    check_nonnegative("weight_decay", weight_decay)
    if len(betas) != 2 or any(not 0 <= beta < 1 for beta in betas):
        raise ValueError(f"invalid beta values: {betas}")


def single_row(parameter, gradient, states, *, key, offset) -> _native.SrsRow:
    """Host srs_row describing one tensor (param_index field = the update key)."""
    row = _native.SrsRow()
    row.param, row.grad = parameter.data_ptr(), gradient.data_ptr()
    for i, s in enumerate(states):
        row.state[i] = s.data_ptr()
    row.numel = parameter.numel()
    row.param_index, row.offset = int(key) & _MASK32, int(offset) & _MASK32
    flags = _native.ROW_PARAM_BF16 if parameter.dtype == torch.bfloat16 else 0
    flags |= _native.ROW_GRAD_BF16 if gradient.dtype == torch.bfloat16 else 0
    tensors = (parameter, gradient, *states)
    if all(t.data_ptr() % min(16, 8 * t.element_size()) == 0 for t in tensors):
        flags |= _native.ROW_VECTOR_OK
    row.flags = flags
    return row


def validate_single(parameter, gradient, *states):
    _native.launcher().check_device(parameter.device)
    tensors = (parameter, gradient, *states)
    check_layout(tensors)
    if parameter.numel():
        check_disjoint(spans_of(tensors, parameter.numel()))


@torch.no_grad()
def cuda_adamw_step_(
    parameter: torch.Tensor,
    gradient: torch.Tensor,
    exp_avg: torch.Tensor,
    exp_avg_sq: torch.Tensor,
    *,
    lr: float,
    beta1: float,
    beta2: float,
    eps: float,
    weight_decay: float,
    step: int,
    seed: int = 0,
    offset: int = 0,
    rounding: str | None = None,
    formats: tuple | dict | None = None,
    block_size: int = 256,
) -> None:
    """One AdamW update of one tensor, in place, on the current CUDA stream.

    ``seed`` is the update key (``update_key(group seed, rng step, index)``);
    ``offset`` is the flat index of element 0 within the full parameter.  Each
    moment uses its resolved format; the parameter update uses the unrounded
    FP32 moments.  Tensors: contiguous, same shape, disjoint, on one sm_100a
    device; parameter and gradient FP32 or BF16.
    """
    if formats is None:
        rule = "stochastic" if rounding is None else rounding
        formats = (StateFormat(exp_avg.dtype, rule), StateFormat(exp_avg_sq.dtype, rule))
        rounding = None
    resolved = resolve_formats(("exp_avg", "exp_avg_sq"), formats, rounding=rounding,
                               backend="cuda")
    for state, fmt in zip((exp_avg, exp_avg_sq), resolved):
        check_block_size(block_size)
        if state.dtype != fmt.dtype:
            raise ValueError("state dtype does not match its state format")
    _check_hyperparameters(lr, (beta1, beta2), eps, weight_decay)
    if not isinstance(step, int) or isinstance(step, bool) or step < 1:
        raise ValueError("step must be a positive integer")
    validate_single(parameter, gradient, exp_avg, exp_avg_sq)
    if parameter.numel() == 0:
        return
    (m_fmt, m_rule), (v_fmt, v_rule) = (native_codes(f.dtype, f.rounding) for f in resolved)
    row = single_row(parameter, gradient, (exp_avg, exp_avg_sq), key=seed, offset=offset)
    hp = adamw_hparams(lr, (beta1, beta2), eps, weight_decay, (step,))
    with device_guard(parameter.device):
        _native.launcher().adamw_single(row, m_fmt, m_rule, v_fmt, v_rule, hp,
                                        stream_handle(parameter.device))


class AdamWCuda(AdamWReferenceSR):
    """Fused AdamW accepting the reference Triton class's ``block_size`` option.

    ``block_size`` is validated and stored in each group (checkpoint
    compatibility); the kernels pick their own launch configuration, and
    results never depend on it.
    """

    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-2, *,
                 state_format=None, state_dtype=None, rounding=None, seed=0, block_size=256):
        self._initial_block_size = block_size
        super().__init__(params, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay,
                         state_format=state_format, state_dtype=state_dtype, rounding=rounding,
                         seed=seed)
        self.defaults["block_size"] = block_size

    def _validate_group(self, group):
        super()._validate_group(group)
        check_block_size(group.get("block_size", self._initial_block_size))

    def add_param_group(self, param_group):
        default = self.defaults.get("block_size", self._initial_block_size)
        super().add_param_group({"block_size": default, **param_group})
