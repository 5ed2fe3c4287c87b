"""Group-level fused steps: validate the whole group, then one launch per device.

These implement the ``_step_group`` plugin hook (reference:
sr_states/optim/_state.py:172-182, overridden by sr_states/triton/adamw.py:289-319
and sr_states/triton/sgd.py:533-556).  Every error surfaces before the first
launch; after the launches each AdamW state records its new step.
"""

from __future__ import annotations

import numpy as np
import torch

from .._hash import split_words
from ..rounding import native_codes
from . import _native
from ._tables import collect_updates, group_cache

_F32 = np.float32


def adamw_hparams(lr, betas, eps, weight_decay, steps) -> _native.SrsAdamWHparams:
    """Launch scalars, each the FP32 rounding of the double expression PyTorch's
    CPU kernels receive in the reference (sr_states/reference/adamw.py:79-89)."""
    beta1, beta2 = betas
    hp = _native.SrsAdamWHparams()
    hp.beta1, hp.beta2 = _F32(beta1), _F32(beta2)
    hp.one_minus_beta1, hp.one_minus_beta2 = _F32(1.0 - beta1), _F32(1.0 - beta2)
    hp.eps, hp.decay = _F32(eps), _F32(1.0 - lr * weight_decay)
    hp.n_step_classes = max(len(steps), 1)
    for c, step in enumerate(steps):
        hp.neg_step_size[c] = _F32(-lr / (1.0 - beta1**step))
        hp.bias2_sqrt[c] = _F32((1.0 - beta2**step) ** 0.5)
    return hp


def sgdm_hparams(lr, momentum) -> _native.SrsSgdmHparams:
    hp = _native.SrsSgdmHparams()
    hp.momentum, hp.neg_lr = _F32(momentum), _F32(-lr)
    return hp


def rng_words(seed, rng_step, key_mode=_native.KEY_DERIVE) -> _native.SrsRng:
    rng = _native.SrsRng()
    rng.seed_lo, rng.seed_hi = split_words(seed)
    rng.step_lo, rng.step_hi = split_words(rng_step)
    rng.key_mode = key_mode
    return rng


def _prepare(optimizer, group, formats, items, *, uses_step):
    by_device = collect_updates(items, optimizer._state_names, uses_step=uses_step)
    optimizer._validate_group(group)
    codes = [native_codes(fmt.dtype, fmt.rounding) for fmt in formats]
    launcher = _native.launcher()
    for device in by_device:
        launcher.check_device(device)
    launches = group_cache(optimizer, group).prepare(by_device, launcher.tile_elems())
    return launcher, codes, launches


def _stream(device):
    return torch.cuda.current_stream(device).cuda_stream if device.type == "cuda" else None


def adamw_group_step(optimizer, group, formats, items, rng_step) -> None:
    items = list(items)
    if not items:
        return
    launcher, ((m_fmt, m_rule), (v_fmt, v_rule)), launches = _prepare(
        optimizer, group, formats, items, uses_step=True)
    rng = rng_words(group["sr_seed"], rng_step)
    optimizer._srs_launches = getattr(optimizer, "_srs_launches", 0) + len(launches)
    for launch in launches:
        hp = adamw_hparams(group["lr"], group["betas"], group["eps"], group["weight_decay"],
                           launch.steps)
        with torch.cuda.device(launch.device) if launch.device.type == "cuda" else _null():
            launcher.adamw_multi(launch.table, launch.table.n_rows, launch.table.n_tiles, m_fmt,
                                 m_rule, v_fmt, v_rule, hp, rng, _stream(launch.device))
    for _, state, _, step, _ in items:
        state["step"] = step


def sgdm_group_step(optimizer, group, formats, items, rng_step) -> None:
    items = list(items)
    if not items:
        return
    launcher, ((u_fmt, u_rule),), launches = _prepare(optimizer, group, formats, items,
                                                      uses_step=False)
    rng = rng_words(group["sr_seed"], rng_step)
    hp = sgdm_hparams(group["lr"], group["momentum"])
    optimizer._srs_launches = getattr(optimizer, "_srs_launches", 0) + len(launches)
    for launch in launches:
        with torch.cuda.device(launch.device) if launch.device.type == "cuda" else _null():
            launcher.sgdm_multi(launch.table, launch.table.n_rows, launch.table.n_tiles, u_fmt,
                                u_rule, hp, rng, _stream(launch.device))


class _null:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False
