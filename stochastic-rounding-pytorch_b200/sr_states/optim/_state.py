"""Optimizer bookkeeping shared by every optimizer of the package.

Observable contract kept from the reference (sr_states/optim/_state.py:21-239),
because user code, plugins and checkpoints depend on it:

* constructor options ``state_format`` / ``state_dtype`` / ``rounding`` /
  ``seed`` and the same per-group overrides; every group carries its formats
  serialized as ``state_format`` (``{name: {"dtype", "rounding"}}``), plus
  ``sr_seed`` and ``sr_step``;
* ``step()`` reserves the next global RNG step for all groups before any
  parameter is touched (a step that fails part-way still consumes it) and
  numbers parameters across all groups in order, grad-less ones included;
* states are created lazily, zero, in their storage dtype; sparse gradients and
  parameters above 2^32 elements are rejected;
* the plugin hook ``_step_group(group, formats, items, rng_step)`` receives a
  lazy iterable of ``(parameter, state, param_index, next_step, offset)``; the
  fused optimizers override it with one kernel launch per device;
* ``load_state_dict`` restores every state in its own format dtype (PyTorch
  would otherwise cast it to the parameter's dtype) and drops the legacy
  ``sr_offset`` field.

How it is organised here: a ``_FormatPolicy`` per optimizer class owns every
question about formats (constructor, group overrides, checkpoints, decoding the
serialized form); ``step`` walks ``_numbered_groups``; states are allocated by
``_ensure_states``; a checkpoint is loaded by taking the format-typed states
out of it, letting PyTorch load the rest, and putting them back typed.

Optimizers that are not fused declare ``_state_names`` and implement
``_compute(p32, g32, states32, group, step) -> (new_p32, proposals)``; the
default ``_step_parameter`` stores each proposal with ``sr_states.cast``.
"""

from __future__ import annotations

import itertools

import torch
from torch.optim import Optimizer

from .._hash import state_key, update_key
from ..formats import StateFormat, force_rounding, resolve_formats
from ..rounding import cast

try:
    from torch.distributed.tensor import DTensor
except ImportError:  # pragma: no cover - builds without torch.distributed
    DTensor = ()

_RNG_LIMIT = 1 << 32
_LEGACY_GROUP_KEYS = ("state_dtype", "rounding", "sr_offset")
_FORMAT_TYPE_ERROR = "state_format must be a StateFormat or a dict keyed by state name"


def _validate_rng_numel(numel: int) -> None:
    if numel > _RNG_LIMIT:
        raise ValueError("optimizer RNG supports at most 2**32 elements per parameter")


class _FormatPolicy:
    """Storage formats of one optimizer class's states: state names, the rule
    every state is forced to (the RN classes) and the rounding backend whose
    registry validates the rules."""

    def __init__(self, names, forced, backend):
        self.names, self.forced, self.backend = tuple(names), forced, backend
        self._decoded: dict = {}

    def resolve(self, formats=None, **shorthand) -> tuple:
        return resolve_formats(self.names, formats, forced_rounding=self.forced,
                               backend=self.backend, **shorthand)

    def encode(self, formats) -> dict:
        return {name: fmt.to_dict() for name, fmt in zip(self.names, formats)}

    def decode(self, serialized) -> tuple:
        """The formats of a group's serialized ``state_format`` (cached)."""
        key = tuple((n, serialized[n]["dtype"], serialized[n]["rounding"]) for n in self.names)
        formats = self._decoded.get(key)
        if formats is None:
            formats = self._decoded[key] = tuple(StateFormat.from_dict(serialized[n])
                                                 for n in self.names)
        return formats

    def for_group(self, group, inherited, from_checkpoint) -> tuple:
        """Formats of a param group: its explicit ``state_format``, else the
        inherited formats (the defaults, or BF16 stochastic) with the group's
        ``state_dtype`` / ``rounding`` shorthand applied."""
        overrides = {k: group[k] for k in ("state_dtype", "rounding") if k in group}
        explicit = group.get("state_format")
        if explicit is None:
            base = (self.decode(inherited["state_format"]) if inherited
                    else (StateFormat(torch.bfloat16),) * len(self.names))
            chosen = tuple(StateFormat(overrides.get("state_dtype", f.dtype),
                                       overrides.get("rounding", f.rounding)) for f in base)
        else:
            if not isinstance(explicit, (StateFormat, dict)):
                raise TypeError(_FORMAT_TYPE_ERROR)
            if overrides:
                raise ValueError("state_format cannot be combined with state_dtype or rounding")
            if from_checkpoint:
                if not isinstance(explicit, dict) or set(explicit) != set(self.names):
                    raise ValueError(f"state_format keys must be exactly {self.names}")
                explicit = {n: StateFormat.from_dict(f) for n, f in explicit.items()}
            chosen = self.resolve(explicit)
        chosen = force_rounding(chosen, self.forced)
        for fmt in chosen:
            fmt.validate(self.backend)
        return chosen


class StateOptimizer(Optimizer):
    """Base for optimizers with FP32 math and one storage format per state."""

    _state_names: tuple[str, ...] = ()
    _rounding_backend = "reference"
    _uses_step = True
    _forced_rounding: str | None = None

    def __init__(self, params, defaults, *, state_format=None, state_dtype=None, rounding=None,
                 seed=0):
        names = self._state_names
        if not names or len(set(names)) != len(names):
            raise ValueError("_state_names must contain unique state names")
        if state_format is not None and not isinstance(state_format, (StateFormat, dict)):
            raise TypeError(_FORMAT_TYPE_ERROR)
        self._policy = _FormatPolicy(names, self._forced_rounding, self._rounding_backend)
        formats = self._policy.resolve(state_format, state_dtype=state_dtype, rounding=rounding)
        super().__init__(params, {**defaults, "state_format": self._policy.encode(formats),
                                  "sr_seed": int(seed), "sr_step": 0})

    # -------------------------------------------------------------- formats --

    def _serialize(self, formats) -> dict:
        return self._policy.encode(formats)

    def _formats(self, group) -> tuple:
        return self._policy.decode(group["state_format"])

    def param_formats(self) -> dict:
        """``{id(parameter): formats}`` over all groups: the storage formats of
        each parameter's states."""
        return {id(p): self._formats(group) for group in self.param_groups
                for p in group["params"]}

    def _validate_group(self, group):
        """Hyperparameter checks of a subclass; run when a group is added or loaded."""

    def _normalize_group(self, group, inherited=None, *, checkpoint=False):
        formats = self._policy.for_group(group, inherited, checkpoint)
        normalized = {k: v for k, v in group.items() if k not in _LEGACY_GROUP_KEYS}
        normalized.setdefault("sr_step", 0)
        normalized["state_format"] = self._policy.encode(formats)
        self._validate_group({**(inherited or {}), **normalized})
        return normalized

    def add_param_group(self, param_group):
        super().add_param_group(self._normalize_group(param_group, self.defaults))

    # ------------------------------------------------------------- updates --

    def _step_parameter(self, parameter, state, group, formats, step, seed, offset):
        """Per-parameter path: ``_compute`` in FP32, then each proposal stored
        with ``cast`` under counter base ``state_key(seed, i)`` at ``offset``."""
        new_parameter, proposals = self._compute(
            parameter.float(), parameter.grad.float(),
            tuple(state[name].float() for name in self._state_names), group, step)
        if len(proposals) != len(self._state_names):
            raise ValueError("_compute must return one tensor per state")
        stored = [cast(value, dtype=fmt.dtype, rounding=fmt.rounding, seed=state_key(seed, i),
                       offset=offset)
                  for i, (value, fmt) in enumerate(zip(proposals, formats))]
        parameter.copy_(new_parameter)
        for name, value in zip(self._state_names, stored):
            state[name].copy_(value)

    def _shard_start(self, parameter) -> int:
        """Flat element index (within the full parameter) of the first local element."""
        if DTensor and isinstance(parameter, DTensor):
            raise NotImplementedError("DTensor optimizer parameters require FSDP2 support")
        return 0

    def _ensure_states(self, parameter, formats) -> dict:
        """The parameter's state dict with every state present in its format."""
        state = self.state[parameter]
        for name, fmt in zip(self._state_names, formats):
            existing = state.get(name)
            if existing is None:
                state[name] = torch.zeros_like(parameter, dtype=fmt.dtype,
                                               memory_format=torch.preserve_format)
            elif existing.dtype != fmt.dtype:
                raise ValueError(f"{name} dtype does not match its state format")
        return state

    def _group_items(self, group, formats, first_index):
        """Lazily yield ``(parameter, state, param_index, next_step, offset)`` for
        the group's parameters that have a gradient."""
        for param_index, parameter in zip(itertools.count(first_index), group["params"]):
            grad = parameter.grad
            if grad is None:
                continue
            if grad.is_sparse:
                raise RuntimeError(f"{type(self).__name__} does not support sparse gradients")
            offset = self._shard_start(parameter)
            _validate_rng_numel(parameter.numel())
            state = self._ensure_states(parameter, formats)
            yield parameter, state, param_index, state.get("step", 0) + 1, offset

    def _step_group(self, group, formats, items, rng_step):
        """Default: one ``_step_parameter`` call per item with its update key.
        Overrides may collect the items first; they record ``state["step"]`` for
        every successful update when ``_uses_step`` is set."""
        for parameter, state, param_index, next_step, offset in items:
            key = update_key(group["sr_seed"], rng_step, param_index)
            self._step_parameter(parameter, state, group, formats, next_step, key, offset)
            if self._uses_step:
                state["step"] = next_step

    def _numbered_groups(self):
        """``(group, index of its first parameter across all groups)``."""
        sizes = [len(group["params"]) for group in self.param_groups]
        return zip(self.param_groups, itertools.accumulate([0] + sizes[:-1]))

    def _rng_step(self) -> int:
        return max((int(group["sr_step"]) for group in self.param_groups), default=0)

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        rng_step = self._rng_step() + 1
        for group in self.param_groups:  # reserved before any update: a retry draws afresh
            group["sr_step"] = rng_step
        for group, first_index in self._numbered_groups():
            formats = self._formats(group)
            self._step_group(group, formats, self._group_items(group, formats, first_index),
                             rng_step)
        return loss

    # ---------------------------------------------------------- checkpoints --

    def load_state_dict(self, state_dict):
        """Load a checkpoint; every state keeps its format dtype.

        The format-typed states are split off a copy of the checkpoint, so
        PyTorch never converts them to the parameter dtype, and PyTorch loads
        the remainder (groups, steps, foreign entries).  The states are put back,
        converted to their groups' formats on the parameters' devices, by a
        post-load hook that runs before any hook of the caller's, so those see
        the loaded optimizer complete."""
        names = set(self._state_names)
        typed = {key: {n: v for n, v in entry.items() if n in names}
                 for key, entry in state_dict["state"].items()}
        remainder = {"param_groups": [self._normalize_group(g, checkpoint=True)
                                      for g in state_dict["param_groups"]],
                     "state": {key: {n: v for n, v in entry.items() if n not in names}
                               for key, entry in state_dict["state"].items()}}

        def put_back(optimizer):
            for group, saved in zip(optimizer.param_groups, remainder["param_groups"]):
                formats = optimizer._formats(group)
                for parameter, key in zip(group["params"], saved["params"]):
                    states = typed.get(key)
                    if not states:
                        continue
                    slot = optimizer.state[parameter]
                    for name, fmt in zip(optimizer._state_names, formats):
                        if name in states:
                            slot[name] = states[name].to(device=parameter.device,
                                                         dtype=fmt.dtype).clone()

        handle = self.register_load_state_dict_post_hook(put_back, prepend=True)
        try:
            return super().load_state_dict(remainder)
        finally:
            handle.remove()
