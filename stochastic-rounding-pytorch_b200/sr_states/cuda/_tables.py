"""Row tables of the fused multi-tensor steps and their per-group device cache.

One optimizer group becomes, per device, ONE kernel launch over a table of
``srs_row`` entries (include/srs_b200.h): every parameter with a gradient is a
row, whatever its parameter/gradient dtype and AdamW bias-correction step.
Rows carry their step class; the per-class scalars travel as launch
arguments, so a table stays valid while every parameter's step advances.

The table is rebuilt and re-uploaded only when the rows' layout (sizes, RNG
coordinates, dtypes, step classes), their addresses or the launch stream
change; the overlap check runs on every rebuild.  This mirrors the reference's
bucketing and cache semantics (sr_states/triton/_multi_tensor.py:22-156) with
a single launch per device instead of one per bucket.
"""

from __future__ import annotations

import collections
from dataclasses import dataclass

import numpy as np
import torch

from . import _native
from ._validate import check_disjoint, check_layout, spans_of

_MASK32 = 0xFFFFFFFF


@dataclass(frozen=True)
class Update:
    """One parameter's update: tensors = (param, grad, *states)."""

    tensors: tuple
    param_index: int
    numel: int
    offset: int
    step: int | None


def _positive_step(step, uses_step):
    """The AdamW bias-correction step of an item (None for optimizers without one)."""
    if not uses_step:
        return None
    if isinstance(step, bool) or not isinstance(step, int) or step < 1:
        raise ValueError("step must be a positive integer")
    return step


def collect_updates(items, state_names, *, uses_step):
    """{device: [Update, ...]} of a group's items, in item order.

    The tensors of every item are validated on every full preparation: the
    row-table cache keys on addresses, and an in-place resize or restride keeps
    those.  Empty parameters are validated too but add no row (their device
    still gets an entry, so its capability is checked)."""
    per_device = collections.defaultdict(list)
    for parameter, state, param_index, step, offset in items:
        tensors = (parameter, parameter.grad) + tuple(state[name] for name in state_names)
        check_layout(tensors)
        update = Update(tensors, int(param_index), parameter.numel(), int(offset) & _MASK32,
                        _positive_step(step, uses_step))
        rows = per_device[parameter.device]
        if update.numel > 0:
            rows.append(update)
    return dict(per_device)


@dataclass
class DeviceTable:
    host: np.ndarray  # ROW_DTYPE records
    storage: torch.Tensor  # the same bytes on the launch device
    n_rows: int
    n_tiles: int

    @property
    def device_ptr(self) -> int:
        return self.storage.data_ptr()

    @property
    def uniform_kind(self) -> int:
        """Parameter/gradient dtype bits shared by every row, or KIND_MIXED."""
        kinds = np.unique(self.host["flags"] & (_native.ROW_PARAM_BF16 | _native.ROW_GRAD_BF16))
        return int(kinds[0]) if kinds.size == 1 else _native.KIND_MIXED


@dataclass(frozen=True)
class Launch:
    device: torch.device
    table: DeviceTable
    steps: tuple  # bias-correction step of each class (AdamW); () for SGDM


@dataclass
class _Entry:
    layout: tuple
    addresses: tuple
    stream: object
    launches: list


def _vector_ok(tensors) -> bool:
    for t in tensors:
        need = min(16, 8 * t.element_size())
        if t.data_ptr() % need:
            return False
    return True


def _row_flags(u: Update, step_class: int) -> int:
    p, g = u.tensors[0], u.tensors[1]
    flags = (_native.ROW_PARAM_BF16 if p.dtype == torch.bfloat16 else 0)
    flags |= (_native.ROW_GRAD_BF16 if g.dtype == torch.bfloat16 else 0)
    flags |= (_native.ROW_VECTOR_OK if _vector_ok(u.tensors) else 0)
    return flags | (step_class << _native.ROW_CLASS_SHIFT)


def build_table(updates, classes, tile_elems: int) -> np.ndarray:
    """Host row table (ROW_DTYPE) with tile_begin prefix sums."""
    host = np.zeros(len(updates), dtype=_native.ROW_DTYPE)
    tile = 0
    for i, (u, cls) in enumerate(zip(updates, classes)):
        states = [t.data_ptr() for t in u.tensors[2:]] + [0, 0]
        host[i] = (u.tensors[0].data_ptr(), u.tensors[1].data_ptr(), states[:2], u.numel, tile,
                   u.param_index & _MASK32, u.offset, _row_flags(u, cls), 0)
        tile += -(-u.numel // tile_elems)
    return host


def upload(host: np.ndarray, device: torch.device) -> torch.Tensor:
    src = torch.from_numpy(host.view(np.uint8))
    if device.type == "cuda":
        # Asynchronous copy on the current stream; the pinned staging block is
        # kept by PyTorch's host allocator until the copy has completed.
        return src.pin_memory().to(device, non_blocking=True)
    return src.clone()


def _step_classes(updates):
    """Class of each row = rank of its step among the distinct steps; chunks of
    MAX_STEP_CLASSES classes become separate launches."""
    steps = sorted({u.step for u in updates if u.step is not None})
    rank = {s: i for i, s in enumerate(steps)}
    return [rank.get(u.step, 0) for u in updates], steps


@dataclass
class FastStep:
    """What a repeated step of an unchanged group needs: the launches of the last
    full preparation and, for AdamW, the state dicts and steps they were built for."""

    key: tuple
    streams: tuple
    launches: list  # Launch objects; AdamW step tuples advance with every step
    states: list  # state dict of every updated parameter (AdamW)
    steps: list  # next step of every updated parameter at the last step (AdamW)


def fingerprint(optimizer, group, formats) -> tuple | None:
    """Identity, storage and layout of every tensor a step of ``group`` touches.

    Two equal fingerprints mean the same parameter, gradient, state dict and
    state objects, at the same addresses, sizes, dtypes, shapes and
    contiguity, so the row tables, the layout checks and the overlap check of
    the first of the two steps still hold.  None (a tensor without strided
    storage, e.g. a sparse gradient) sends the step down the full path, which
    raises the proper error.  The per-tensor work runs in the _srs_host module
    (one call instead of a Python loop over the tensors)."""
    sig = _native.host_module().signature(group["params"], optimizer.state,
                                           tuple(optimizer._state_names))
    return None if sig is None else (tuple(formats), sig)


def current_streams(launches) -> tuple:
    return tuple(torch.cuda.current_stream(launch.device) if launch.device.type == "cuda"
                 else None for launch in launches)


class GroupTableCache:
    """Device row tables of one parameter group, reused across steps."""

    def __init__(self):
        self._entries: dict[torch.device, _Entry] = {}
        self.fast: FastStep | None = None

    def prepare(self, by_device, tile_elems: int) -> list[Launch]:
        entries, launches = {}, []
        for device, updates in by_device.items():
            if not updates:
                continue
            classes, steps = _step_classes(updates)
            layout = (tile_elems, tuple(
                (u.numel, u.param_index & _MASK32, u.offset, u.tensors[0].dtype,
                 u.tensors[1].dtype, tuple(t.dtype for t in u.tensors[2:]), c)
                for u, c in zip(updates, classes)))
            addresses = tuple(tuple(t.data_ptr() for t in u.tensors) for u in updates)
            stream = torch.cuda.current_stream(device) if device.type == "cuda" else None
            old = self._entries.get(device)
            if old is None or (old.layout, old.addresses) != (layout, addresses):
                check_disjoint([s for u in updates for s in spans_of(u.tensors, u.numel)])
            if old is not None and (old.layout, old.addresses, old.stream) == (
                    layout, addresses, stream):
                entry = old
            else:
                entry = _Entry(layout, addresses, stream, [])
                for lo in range(0, max(len(steps), 1), _native.MAX_STEP_CLASSES):
                    chunk = [(u, c - lo) for u, c in zip(updates, classes)
                             if lo <= c < lo + _native.MAX_STEP_CLASSES]
                    host = build_table([u for u, _ in chunk], [c for _, c in chunk], tile_elems)
                    n_tiles = int(host["tile_begin"][-1] + -(-host["numel"][-1] // tile_elems))
                    entry.launches.append((DeviceTable(host, upload(host, device), len(host),
                                                       n_tiles), lo))
            entries[device] = entry
            for table, lo in entry.launches:
                launches.append(Launch(device, table,
                                       tuple(steps[lo:lo + _native.MAX_STEP_CLASSES])))
        self._entries = entries
        return launches


def group_cache(optimizer, group) -> GroupTableCache:
    """The table cache of ``group`` (caches of groups no longer present are dropped)."""
    caches = getattr(optimizer, "_srs_table_caches", None)
    if caches is None or id(group) not in caches:
        live = {id(g) for g in optimizer.param_groups}
        caches = {k: v for k, v in (caches or {}).items() if k in live}
        caches[id(group)] = GroupTableCache()
        optimizer._srs_table_caches = caches
    return caches[id(group)]
