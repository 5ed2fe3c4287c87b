"""Group-level fused steps: validate the whole group, then one launch per device.

These implement the ``_step_group`` plugin hook (reference:
sr_states/optim/_state.py:172-182, overridden by sr_states/triton/adamw.py:289-319
and sr_states/triton/sgd.py:214-237).  Every error surfaces before the first
launch; after the launches each AdamW state records its new step.
"""

from __future__ import annotations

import numpy as np
import torch

from .._hash import split_words
from ..rounding import native_codes
from . import _native
from ._tables import FastStep, Launch, collect_updates, current_streams, fingerprint, group_cache

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


def _peers_of(optimizer) -> dict:
    """Peer replicas of a sharded optimizer that fuses its all-gather into the step."""
    peers = getattr(optimizer, "_srs_peers", None)
    return {"peers": peers} if peers is not None else {}


def _stream(device):
    return torch.cuda.current_stream(device).cuda_stream if device.type == "cuda" else None


# A repeated step of an unchanged group (same tensors at the same addresses and
# sizes, same formats and streams, every AdamW step advanced by one) reuses the
# launches prepared by the last full step instead of rebuilding them from the
# items: the row tables, layout and overlap checks of that step still hold.
# Hyperparameters are validated on every step.


def _fast_step(optimizer, group, formats, uses_step):
    """(cache, key, launches, steps) for a repeated step, or (cache, key, None, None)."""
    cache = group_cache(optimizer, group)
    key = fingerprint(optimizer, group, formats)
    fast = cache.fast
    if (key is None or fast is None or fast.key != key
            or fast.streams != current_streams(fast.launches)):
        return cache, key, None, None
    if not uses_step:
        return cache, key, fast.launches, None
    steps = [state.get("step", 0) + 1 for state in fast.states]
    if any(s != t + 1 for s, t in zip(steps, fast.steps)):
        return cache, key, None, None
    launches = [Launch(l.device, l.table, tuple(s + 1 for s in l.steps)) for l in fast.launches]
    return cache, key, launches, steps


def _remember(cache, optimizer, group, formats, launches, items, uses_step):
    cache.fast = FastStep(fingerprint(optimizer, group, formats), current_streams(launches),
                          launches, [item[1] for item in items] if uses_step else [],
                          [item[3] for item in items] if uses_step else [])


def adamw_group_step(optimizer, group, formats, items, rng_step) -> None:
    optimizer._validate_group(group)
    codes = [native_codes(fmt.dtype, fmt.rounding) for fmt in formats]
    cache, _, launches, steps = _fast_step(optimizer, group, formats, uses_step=True)
    if launches is None:
        items = list(items)
        if not items:
            return
        launcher, codes, launches = _prepare(optimizer, group, formats, items, uses_step=True)
    else:
        launcher = _native.launcher()
    ((m_fmt, m_rule), (v_fmt, v_rule)) = codes
    rng = rng_words(group["sr_seed"], rng_step)
    optimizer._srs_launches = getattr(optimizer, "_srs_launches", 0) + len(launches)
    for launch in launches:
        hp = adamw_hparams(group["lr"], group["betas"], group["eps"], group["weight_decay"],
                           launch.steps)
        exchange = getattr(optimizer, "_srs_exchange", None)
        with torch.cuda.device(launch.device) if launch.device.type == "cuda" else _null():
            def whole(launch=launch, hp=hp):
                launcher.adamw_multi(launch.table, launch.table.n_rows, launch.table.n_tiles,
                                     m_fmt, m_rule, v_fmt, v_rule, hp, rng,
                                     _stream(launch.device), **_peers_of(optimizer))

            if exchange is not None:
                exchange.run(launch, lambda lo, hi, launch=launch, hp=hp: launcher.adamw_multi(
                    launch.table, launch.table.n_rows, launch.table.n_tiles, m_fmt, m_rule,
                    v_fmt, v_rule, hp, rng, _stream(launch.device), tiles=(lo, hi),
                    **_peers_of(optimizer)), whole)
            else:
                whole()
    if steps is None:
        for _, state, _, step, _ in items:
            state["step"] = step
        _remember(cache, optimizer, group, formats, launches, items, True)
    else:
        for state, step in zip(cache.fast.states, steps):
            state["step"] = step
        cache.fast.launches, cache.fast.steps = launches, steps


def sgdm_group_step(optimizer, group, formats, items, rng_step) -> None:
    optimizer._validate_group(group)
    codes = [native_codes(fmt.dtype, fmt.rounding) for fmt in formats]
    cache, _, launches, _ = _fast_step(optimizer, group, formats, uses_step=False)
    fresh = launches is None
    if fresh:
        items = list(items)
        if not items:
            return
        launcher, codes, launches = _prepare(optimizer, group, formats, items, uses_step=False)
    else:
        launcher = _native.launcher()
    ((u_fmt, u_rule),) = codes
    rng = rng_words(group["sr_seed"], rng_step)
    hp = sgdm_hparams(group["lr"], group["momentum"])
    optimizer._srs_launches = getattr(optimizer, "_srs_launches", 0) + len(launches)
    for launch in launches:
        exchange = getattr(optimizer, "_srs_exchange", None)
        with torch.cuda.device(launch.device) if launch.device.type == "cuda" else _null():
            def whole(launch=launch):
                launcher.sgdm_multi(launch.table, launch.table.n_rows, launch.table.n_tiles,
                                    u_fmt, u_rule, hp, rng, _stream(launch.device),
                                    **_peers_of(optimizer))

            if exchange is not None:
                exchange.run(launch, lambda lo, hi, launch=launch: launcher.sgdm_multi(
                    launch.table, launch.table.n_rows, launch.table.n_tiles, u_fmt, u_rule, hp,
                    rng, _stream(launch.device), tiles=(lo, hi), **_peers_of(optimizer)), whole)
            else:
                whole()
    if fresh:
        _remember(cache, optimizer, group, formats, launches, items, False)


class _null:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False
