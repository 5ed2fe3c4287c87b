"""Allocating casts on the sm_100a cast kernel.

Drop-in for the reference's sr_states/triton/cast.py:32-60 (``cast``) and
sr_states/triton/sr_cast.py:89-164 (``sr_cast_bf16``, ``rn_cast_bf16``): every call
returns a fresh output; element i of a stochastic rule uses the hash of
(i + seed + offset) mod 2^32, so results do not depend on how a tensor is split.
``block_size``/``num_warps``/``store_mode`` are validated for compatibility;
the kernel's launch configuration and output bits do not depend on them.
"""

from __future__ import annotations

import torch

from ..rounding import NATIVE_RULES, native_codes, native_format, validate_rounding
from . import _native
from ._launch import device_guard, stream_handle
from ._validate import CAST_BLOCK_SIZES, CAST_NUM_WARPS, CAST_STORE_MODES

_MASK32 = 0xFFFFFFFF


def _launch(x, out, fmt, rule, seed, offset):
    if x.numel():
        with device_guard(x.device):
            _native.launcher().cast(x.data_ptr(), out.data_ptr(), x.numel(), fmt, rule,
                                    int(seed) & _MASK32, int(offset) & _MASK32,
                                    stream_handle(x.device))
    return out


def _check_launch_options(block_size, num_warps):
    if block_size not in CAST_BLOCK_SIZES:
        raise ValueError(f"block_size must be one of {CAST_BLOCK_SIZES}")
    if num_warps not in CAST_NUM_WARPS:
        raise ValueError(f"num_warps must be one of {CAST_NUM_WARPS}")


def cast(x, *, dtype, rounding="stochastic", seed=0, offset=0, block_size=256, num_warps=4):
    """Cast contiguous CUDA FP32 ``x`` with a registered native rule (fresh output)."""
    validate_rounding(dtype, rounding, backend="cuda")
    _native.launcher().check_device(x.device, "casts")
    if x.dtype != torch.float32:
        raise TypeError(f"expected torch.float32 input, got {x.dtype}")
    if not x.is_contiguous():
        raise ValueError("cast requires a contiguous input")
    _check_launch_options(block_size, num_warps)
    fmt, rule = native_codes(dtype, rounding)
    return _launch(x, torch.empty_like(x, dtype=dtype), fmt, rule, seed, offset)


def _cast_bf16(x, *, seed, offset, block_size, num_warps, store_mode, rule):
    _native.launcher().check_device(x.device, "BF16 casts")
    if x.dtype != torch.float32:
        raise TypeError(f"expected torch.float32 input, got {x.dtype}")
    if not x.is_contiguous():
        raise ValueError("BF16 cast requires a contiguous input")
    _check_launch_options(block_size, num_warps)
    if store_mode not in CAST_STORE_MODES:
        raise ValueError(f"store_mode must be one of {CAST_STORE_MODES}")
    return _launch(x, torch.empty_like(x, dtype=torch.bfloat16), 1, rule, seed, offset)


def sr_cast_bf16(x, *, seed, offset=0, block_size=256, num_warps=4, store_mode="convert"):
    """Stochastic FP32 -> BF16 cast of a contiguous CUDA tensor.  Both store modes
    write the same bits (the kernel always stores the selected BF16 encoding)."""
    return _cast_bf16(x, seed=seed, offset=offset, block_size=block_size, num_warps=num_warps,
                      store_mode=store_mode, rule=1)


def rn_cast_bf16(x, *, block_size=256, num_warps=4):
    """Round-to-nearest-even FP32 -> BF16 cast of a contiguous CUDA tensor."""
    return _cast_bf16(x, seed=0, offset=0, block_size=block_size, num_warps=num_warps,
                      store_mode="convert", rule=0)


def cast_any_layout(x, *, dtype, rule, seed, offset):
    """Device rule ``rule`` (a name of NATIVE_RULES) of ``sr_states.cast``: any
    shape/strides, counters in row-major order of the logical tensor, output
    shaped like ``x``."""
    _native.launcher().check_device(x.device, "the built-in rounding rules (sm_100a kernels)")
    fmt, code = native_format(dtype), NATIVE_RULES.index(rule)
    src = x.contiguous()
    out = torch.empty(x.shape, dtype=dtype, device=x.device)
    return _launch(src, out, fmt, code, seed, offset)
