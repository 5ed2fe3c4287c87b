"""Per-state storage formats of the optimizers.

Public surface kept identical to the reference (sr_states/formats.py:13-83) so
checkpoints and user code carry over: ``StateFormat(dtype, rounding)`` with
``to_dict``/``from_dict`` (the checkpoint schema), ``force_rounding`` and
``resolve_formats`` with the same accepted inputs, error types and messages.
"""

from __future__ import annotations

from collections.abc import Mapping
from dataclasses import dataclass, replace

import torch

from .rounding import validate_rounding

_DEFAULT_DTYPE = torch.bfloat16
_DEFAULT_RULE = "stochastic"
_KEYS = frozenset(("dtype", "rounding"))


@dataclass(frozen=True)
class StateFormat:
    """Storage dtype of one optimizer state plus the name of its rounding rule."""

    dtype: torch.dtype
    rounding: str = _DEFAULT_RULE

    def validate(self, backend: str = "reference") -> None:
        """Raise ValueError unless the rule is registered for the dtype and backend.

        ``"compiled"`` is accepted as an alias of ``"reference"``.
        """
        validate_rounding(self.dtype, self.rounding,
                          backend="reference" if backend == "compiled" else backend)

    def to_dict(self) -> dict:
        return {"dtype": self.dtype, "rounding": self.rounding}

    @classmethod
    def from_dict(cls, d: dict) -> StateFormat:
        if isinstance(d, Mapping) and set(d) == _KEYS:
            return cls(d["dtype"], d["rounding"])
        raise ValueError("a state format must contain exactly dtype and rounding")


def force_rounding(formats, rounding):
    """Same dtypes, every rule replaced by ``rounding`` (``None``: unchanged)."""
    formats = tuple(formats)
    return formats if rounding is None else tuple(replace(f, rounding=rounding) for f in formats)


def _from_user(names, formats) -> tuple:
    if isinstance(formats, StateFormat):
        return tuple(formats for _ in names)
    if isinstance(formats, Mapping):
        if set(formats) == set(names):
            return tuple(formats[name] for name in names)
        raise ValueError(f"state_format keys must be exactly {names}")
    if isinstance(formats, tuple) and len(formats) == len(names):
        return formats  # internal functional interface: one entry per state, in order
    raise TypeError("state_format must be a StateFormat or a dict keyed by state name")


def resolve_formats(
    names,
    formats=None,
    *,
    state_dtype=None,
    rounding=None,
    forced_rounding=None,
    backend="reference",
):
    """Normalize formats (StateFormat, dict by state name, ordered tuple) or the
    ``state_dtype``/``rounding`` shorthand into a validated tuple, one per name.

    ``forced_rounding`` overrides every rule before validation (the RN classes).
    """
    if formats is None:
        shorthand = StateFormat(_DEFAULT_DTYPE if state_dtype is None else state_dtype,
                                _DEFAULT_RULE if rounding is None else rounding)
        result = tuple(shorthand for _ in names)
    elif state_dtype is None and rounding is None:
        result = _from_user(names, formats)
    else:
        raise ValueError("state_format/formats cannot be combined with state_dtype or rounding")
    if not all(isinstance(f, StateFormat) for f in result):
        raise TypeError("each state format must be a StateFormat")
    result = force_rounding(result, forced_rounding)
    for f in result:
        f.validate(backend)
    return result
