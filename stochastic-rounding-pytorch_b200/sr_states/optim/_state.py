"""Optimizer bookkeeping shared by every optimizer of the package.

``StateOptimizer`` keeps the reference's contract (sr_states/optim/_state.py:21-239):

* ``state_format`` / ``state_dtype`` / ``rounding`` / ``seed`` constructor
  options and per-group overrides, serialized into each group as
  ``state_format`` (dict of ``{"dtype", "rounding"}``), ``sr_seed`` and ``sr_step``;
* ``step()`` reserves the global RNG step before touching any parameter (a
  failed step still consumes it) and numbers parameters across all groups;
* lazily zero-initialized states in their storage dtype; sparse gradients and
  parameters above 2^32 elements are rejected;
* ``_step_group(group, formats, items, rng_step)`` is the plugin hook: ``items``
  yields ``(parameter, state, param_index, next_step, offset)`` and the fused
  optimizers override it with one kernel launch per device;
* ``load_state_dict`` restores each state in its own format dtype (PyTorch
  would otherwise cast it to the parameter's dtype) and drops the legacy
  ``sr_offset`` field, restarting such checkpoints at RNG step 0.

Subclasses that are not fused declare ``_state_names`` and implement
``_compute(p32, g32, states32, group, step) -> (new_p32, proposals)``; the
base rounds each proposal with ``sr_states.cast``.
"""

from __future__ import annotations

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


def _validate_rng_numel(numel: int) -> None:
    if numel > _RNG_LIMIT:
        raise ValueError("optimizer RNG supports at most 2**32 elements per parameter")


def _default_formats(count: int) -> tuple:
    return (StateFormat(torch.bfloat16),) * count


class StateOptimizer(Optimizer):
    """Base for optimizers with FP32 math and per-state storage formats."""

    _state_names: tuple[str, ...] = ()
    _rounding_backend = "reference"
    _uses_step = True
    _forced_rounding: str | None = None

    def __init__(
        self, params, defaults, *, state_format=None, state_dtype=None, rounding=None, seed=0
    ):
        names = self._state_names
        if not names or len(set(names)) != len(names):
            raise ValueError("_state_names must contain unique state names")
        if state_format is not None and not isinstance(state_format, (StateFormat, dict)):
            raise TypeError("state_format must be a StateFormat or a dict keyed by state name")
        formats = resolve_formats(
            names, state_format, state_dtype=state_dtype, rounding=rounding,
            forced_rounding=self._forced_rounding, backend=self._rounding_backend)
        super().__init__(params, {**defaults, "state_format": self._serialize(formats),
                                  "sr_seed": int(seed), "sr_step": 0})

    # -------------------------------------------------------------- formats --

    def _serialize(self, formats) -> dict:
        return {name: fmt.to_dict() for name, fmt in zip(self._state_names, formats)}

    def _formats(self, group) -> tuple:
        return tuple(StateFormat.from_dict(group["state_format"][n]) for n in self._state_names)

    def _validate_group(self, group):
        """Subclass hook for hyperparameter checks; runs on construction, add and load."""

    def _group_formats(self, group, inherited, checkpoint) -> tuple:
        explicit = group.get("state_format")
        if explicit is not None:
            if not isinstance(explicit, (StateFormat, dict)):
                raise TypeError("state_format must be a StateFormat or a dict keyed by state name")
            if "state_dtype" in group or "rounding" in group:
                raise ValueError("state_format cannot be combined with state_dtype or rounding")
            if checkpoint:
                if not isinstance(explicit, dict) or set(explicit) != set(self._state_names):
                    raise ValueError(f"state_format keys must be exactly {self._state_names}")
                explicit = {n: StateFormat.from_dict(f) for n, f in explicit.items()}
            return resolve_formats(self._state_names, explicit,
                                   forced_rounding=self._forced_rounding,
                                   backend=self._rounding_backend)
        base = self._formats(inherited) if inherited else _default_formats(
            len(self._state_names))
        if "state_dtype" in group or "rounding" in group:
            base = tuple(StateFormat(group.get("state_dtype", f.dtype),
                                     group.get("rounding", f.rounding)) for f in base)
        return base

    def _normalize_group(self, group, inherited=None, *, checkpoint=False):
        group = dict(group)
        formats = force_rounding(self._group_formats(group, inherited, checkpoint),
                                 self._forced_rounding)
        for fmt in formats:
            fmt.validate(self._rounding_backend)
        for legacy in ("state_dtype", "rounding", "sr_offset"):
            group.pop(legacy, None)
        group.setdefault("sr_step", 0)
        group["state_format"] = self._serialize(formats)
        self._validate_group({**(inherited or {}), **group})
        return group

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

    def _group_items(self, group, formats, first_index):
        """Lazily yield ``(parameter, state, param_index, next_step, offset)``."""
        names = self._state_names
        for param_index, parameter in enumerate(group["params"], start=first_index):
            grad = parameter.grad
            if grad is None:
                continue
            if grad.is_sparse:
                raise RuntimeError(f"{type(self).__name__} does not support sparse gradients")
            offset = self._shard_start(parameter)
            _validate_rng_numel(parameter.numel())
            state = self.state[parameter]
            for name, fmt in zip(names, formats):
                if name not in state:
                    state[name] = torch.zeros_like(parameter, dtype=fmt.dtype,
                                                   memory_format=torch.preserve_format)
                elif state[name].dtype != fmt.dtype:
                    raise ValueError(f"{name} dtype does not match its state format")
            yield parameter, state, param_index, state.get("step", 0) + 1, offset

    def _step_group(self, group, formats, items, rng_step):
        """Default: one ``_step_parameter`` call per item, with its update key.
        Overrides may collect the items first; they record ``state["step"]``
        for every successful update when ``_uses_step`` is set."""
        for parameter, state, param_index, next_step, offset in items:
            key = update_key(group["sr_seed"], rng_step, param_index)
            self._step_parameter(parameter, state, group, formats, next_step, key, offset)
            if self._uses_step:
                state["step"] = next_step

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        # The step is reserved before any update, so a retry after a partial
        # failure draws fresh random numbers.
        rng_step = self._rng_step() + 1
        for group in self.param_groups:
            group["sr_step"] = rng_step
        first_index = 0
        for group in self.param_groups:
            formats = self._formats(group)
            self._step_group(group, formats, self._group_items(group, formats, first_index),
                             rng_step)
            first_index += len(group["params"])
        return loss

    def _rng_step(self) -> int:
        return max((int(group["sr_step"]) for group in self.param_groups), default=0)

    # ---------------------------------------------------------- checkpoints --

    def load_state_dict(self, state_dict):
        checkpoint = dict(state_dict)  # never mutate the caller's checkpoint
        checkpoint["param_groups"] = [self._normalize_group(g, checkpoint=True)
                                      for g in state_dict["param_groups"]]
        originals: dict = {}

        def keep_originals(optimizer, source):
            # Runs before PyTorch casts floating-point state to the parameter dtype.
            for group, saved in zip(optimizer.param_groups, source["param_groups"]):
                for parameter, key in zip(group["params"], saved["params"]):
                    entry = source["state"].get(key, {})
                    originals[parameter] = {n: entry[n] for n in self._state_names if n in entry}

        def restore_formats(optimizer):
            for group in optimizer.param_groups:
                formats = self._formats(group)
                for parameter in group["params"]:
                    kept = originals.get(parameter, {})
                    for name, fmt in zip(self._state_names, formats):
                        if name in kept:
                            optimizer.state[parameter][name] = kept[name].to(
                                device=parameter.device, dtype=fmt.dtype).clone()

        pre = self.register_load_state_dict_pre_hook(keep_originals)
        post = self.register_load_state_dict_post_hook(restore_formats, prepend=True)
        try:
            return super().load_state_dict(checkpoint)
        finally:
            pre.remove()
            post.remove()
