"""Named rounding rules per storage dtype, shared by casts and every optimizer.

Public surface of the reference (sr_states/rounding.py:28-124): ``register_rounding``,
``validate_rounding`` and ``cast`` with the same arguments, error types and
messages.  The built-in rules (nearest and stochastic for FP32, BF16, FP16,
FP8 E4M3/E5M2) execute on the sm_100a kernels of ``libsrs_b200.so``.

Custom rules: the reference runs a custom rule in its fused kernels through a
``@triton.jit`` callback (sr_states/rounding.py:28-66).  Here the kernels hold
a small table of device rules selected by id (``NATIVE_RULES``, the
``SRS_RULE_*`` codes of include/srs_b200.h): nearest, stochastic and
toward_zero.  ``register_rounding(..., native=<id>)`` binds a name to one of
them; ``native_reference(<id>)`` is the kernel-backed callable of that rule,
for registrations without a CPU implementation of their own.

Backends named in validation:
  ``"reference"`` (also ``"compiled"``): any registered rule; ``cast`` calls the
      rule's ``reference`` callable (the built-ins' callable is the native kernel).
  ``"cuda"`` / ``"triton"``: the fused optimizer kernels; a rule must name a
      native implementation.  ``"triton"`` is the reference's name for its
      fused backend and is accepted so existing code keeps working.
"""

from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass

import torch

# Device rules by SRS_RULE_* code.  Only the first two are built-in names;
# "toward_zero" is reachable through register_rounding(..., native=...).
NATIVE_RULES = ("nearest", "stochastic", "toward_zero")
_BUILTIN_RULES = NATIVE_RULES[:2]
_BACKENDS = {"reference": None, "compiled": None, "cuda": "CUDA", "triton": "Triton"}


@dataclass(frozen=True)
class _Rule:
    reference: Callable
    native: str | None  # built-in kernel rule this name executes on the fused path
    triton: Callable | None = None  # accepted for API compatibility; never executed


_RULES: dict[tuple[torch.dtype, str], _Rule] = {}


def register_rounding(
    name: str,
    dtype: torch.dtype,
    *,
    reference: Callable,
    native: str | None = None,
    triton: Callable | None = None,
) -> None:
    """Register a rounding rule for one storage dtype.

    ``reference(x, *, dtype, seed, offset)`` receives an FP32 tensor and returns
    a tensor of ``dtype`` with the same shape and device, without mutating x;
    ``sr_states.cast`` and the per-parameter ``StateOptimizer`` path call it.

    ``native`` names the sm_100a device rule ("nearest", "stochastic" or
    "toward_zero": the format's value of largest magnitude not above |x|, sign
    kept) that the fused optimizers run for this name; rules without one are
    rejected by the fused optimizers.  The caller vouches that ``reference``
    and the device rule agree.  ``triton`` (a ``@triton.jit`` callback in the
    reference) is accepted so registrations keep importing, but no Triton code
    runs here.  Names and dtypes are stored in checkpoints, callables are not;
    an existing registration can never be replaced.
    """
    if not isinstance(name, str) or not name:
        raise ValueError("rounding name must be a nonempty string")
    if not isinstance(dtype, torch.dtype) or not dtype.is_floating_point:
        raise ValueError("dtype must be a floating-point torch.dtype")
    if not callable(reference) or (triton is not None and not callable(triton)):
        raise TypeError("rounding implementations must be callable")
    if native is not None and native not in NATIVE_RULES:
        raise ValueError(f"native must be one of {NATIVE_RULES} or None")
    if native is not None and dtype not in _NATIVE_FORMATS:
        raise ValueError(f"no native kernels store {dtype}")
    if (dtype, name) in _RULES:
        raise ValueError(f"rounding {name!r} is already registered for {dtype}")
    _RULES[dtype, name] = _Rule(reference, native, triton)


def validate_rounding(dtype: torch.dtype, rounding: str, *, backend: str = "reference") -> None:
    """Raise ValueError unless ``rounding`` is registered for ``dtype`` and usable by ``backend``."""
    if backend not in _BACKENDS:
        raise ValueError(f"unknown rounding backend: {backend!r}")
    rule = _RULES.get((dtype, rounding)) if isinstance(rounding, str) else None
    if not isinstance(dtype, torch.dtype) or rule is None:
        raise ValueError(
            f"no rounding {rounding!r} registered for state_dtype={dtype}; "
            "register before loading checkpoints"
        )
    label = _BACKENDS[backend]
    if label is not None and rule.native is None:
        raise ValueError(f"rounding {rounding!r} for {dtype} has no {label} implementation")


# torch dtype -> SRS_FMT_* code of include/srs_b200.h
_NATIVE_FORMATS = {
    torch.float32: 0,
    torch.bfloat16: 1,
    torch.float16: 2,
    torch.float8_e4m3fn: 3,
    torch.float8_e5m2: 4,
}


def native_format(dtype: torch.dtype) -> int:
    """SRS_FMT_* code of a storage dtype the kernels support."""
    if dtype not in _NATIVE_FORMATS:
        raise ValueError(f"no native kernels store {dtype}")
    return _NATIVE_FORMATS[dtype]


def native_codes(dtype: torch.dtype, rounding: str) -> tuple[int, int]:
    """(SRS_FMT_*, SRS_RULE_*) of a rule usable by the fused kernels."""
    validate_rounding(dtype, rounding, backend="cuda")
    return _NATIVE_FORMATS[dtype], NATIVE_RULES.index(_RULES[dtype, rounding].native)


def cast(
    x: torch.Tensor,
    *,
    dtype: torch.dtype,
    rounding: str = "stochastic",
    seed: int = 0,
    offset: int = 0,
) -> torch.Tensor:
    """Round FP32 ``x`` into ``dtype`` with a registered rule, keeping shape and device.

    Element i (in row-major order) of a stochastic rule uses the hash of
    (i + offset + seed) mod 2^32.  FP8 saturates finite overflow and Inf to the
    signed maximum and keeps NaN; FP16/BF16 keep IEEE overflow; signed zero is
    kept.  The built-in FP16/FP8 stochastic rules use a 24-bit probability grid.
    Built-in FP32 rules return ``x`` itself; other built-ins run the sm_100a
    cast kernel and need a CUDA tensor.
    """
    if x.dtype != torch.float32:
        raise TypeError(f"expected torch.float32 input, got {x.dtype}")
    validate_rounding(dtype, rounding)
    result = _RULES[dtype, rounding].reference(x, dtype=dtype, seed=seed, offset=offset)
    if not isinstance(result, torch.Tensor):
        raise TypeError("rounding routine must return a tensor")
    if result.dtype != dtype or result.shape != x.shape or result.device != x.device:
        raise ValueError(
            "rounding routine must preserve shape/device and return the requested dtype"
        )
    return result


def native_reference(rule: str) -> Callable:
    """The ``reference`` callable of device rule ``rule`` (one of NATIVE_RULES):
    ``(x, *, dtype, seed, offset) -> Tensor`` running the sm_100a cast kernel
    (any shape and strides, counters in row-major order; FP32 is the identity).
    Register it together with ``native=rule`` to use a device rule under a
    name of your own."""
    if rule not in NATIVE_RULES:
        raise ValueError(f"rule must be one of {NATIVE_RULES}")

    def run(x, *, dtype, seed, offset):
        if dtype == torch.float32:
            return x.to(torch.float32)
        if dtype not in _NATIVE_FORMATS:
            raise ValueError(f"no native kernels store {dtype}")
        from .cuda.cast import cast_any_layout

        return cast_any_layout(x, dtype=dtype, rule=rule, seed=seed, offset=offset)

    run.__name__ = f"native_{rule}"
    return run


for _dtype in _NATIVE_FORMATS:
    for _rule in _BUILTIN_RULES:
        _RULES[_dtype, _rule] = _Rule(native_reference(_rule), _rule)
del _dtype, _rule
