"""ZeRO-1 sharding of the fused optimizer steps across the GPUs of one node.

The parameters of all groups, in order, are laid out in one flat buffer per
dtype, padded so that it splits into ``world`` equal shards of a multiple of
64 elements.  Rank r updates only the elements of shard r: every intersection
of the shard with a parameter becomes one row of the fused step, with the
parameter's global index and, as RNG offset, the index of the row's first
element within that parameter.  The counter-hash RNG therefore gives exactly
the bytes of an unsharded step, whatever the world size.  Optimizer states
exist only for the local shard.

The updated parameters are then reassembled on every rank.  With
``gather="fused"`` this happens inside the step: at construction every rank
maps its peers' flat buffers into its address space (CUDA IPC through
libsrs_b200.so), and the fused kernel stores each updated parameter vector
both locally and at the same offset of every peer's buffer, so the exchange
over NVLink overlaps the arithmetic and no separate all-gather runs.  A step
is then: barrier (no peer still reads its replica), fused launch, barrier
(every replica complete), each barrier a one-element NCCL all-reduce on the
current stream.  If any rank cannot export its buffers (for example memory
from the virtual-memory allocator), all ranks fall back to one in-place NCCL
all-gather per flat buffer after the update (``gather="nccl"`` selects it).
``gather="multicast"`` allocates the flat buffers from PyTorch's symmetric
memory and binds them to an NVLink multicast object: the kernel then writes
each updated vector once (``multimem.st``) and NVSwitch delivers it to every
replica; without multicast support it falls back to the peer stores.
``gather="hybrid"`` splits the peers: the step's tile ranges store to all
but ``copy_peers`` of them, and the copy engines send each finished range to
the rest, so the kernel's stores and the copy engines share the exchange.
``gather="copy"`` instead runs the step over ``chunks`` tile ranges and lets
the copy engines send each finished range to the peers while the next one is
updated.  The default, ``"auto"``, takes ``"copy"`` with one peer and
``"fused"`` with more (the faster of the two on B200 in each case).

Gradients must be complete on every rank (already all-reduced), as in ZeRO-1,
unless the optimizer is built with ``grads="reduce_scatter"``: then every
``p.grad`` is a view into a flat gradient buffer laid out like the parameters,
backward accumulates into it, and ``reduce_scatter_grads()`` reduces each
rank's shard in place (one reduce-scatter per buffer) so that the step reads
only its own reduced gradients; ``zero_grad()`` zeroes the buffers in place.

Checkpoints: ``state_dict()`` gathers the shards into the unsharded layout of
AdamWReferenceSR / SGDMReferenceSR (every state in its parameter's shape), so
a checkpoint resumes at any world size or in the unsharded optimizer, and
``load_state_dict`` accepts that layout and keeps the local runs.  Both are
collectives; ``state_dict(to_rank=r)`` delivers the runs to rank r only (a
gather, in bounded buckets).  ``sharded_state_dict()`` /
``load_sharded_state_dict()`` save and restore each rank's own runs without
communication (same world size and parameters required).
"""

from __future__ import annotations

import collections

import torch

from .optim._state import _validate_rng_numel
from .optim.adamw import AdamWReferenceSR
from .optim.sgd import SGDMReferenceSR

SHARD_ALIGN = 64  # elements; keeps every shard boundary 16-byte aligned for 2/4-byte dtypes


class _Piece:
    """A rank's contiguous run of one parameter, presented to the fused step like
    a parameter: the 1-D view of the run plus the matching gradient run."""

    __slots__ = ("tensor", "grad")

    def __init__(self, tensor, grad):
        self.tensor = tensor
        self.grad = grad

    def __getattr__(self, name):
        return getattr(self.tensor, name)


class FlatLayout:
    """Where every parameter lives in its dtype's flat buffer and which run is local."""

    def __init__(self, params, world: int, rank: int, allocate=None):
        """``allocate(numel, dtype, device)`` makes the flat buffers (zeroed);
        without it they are ordinary allocations, or the parameters' own
        storage when that already holds exactly the layout."""
        self.world, self.rank = world, rank
        self.buffers: dict[torch.dtype, torch.Tensor] = {}
        self.place: dict[int, tuple[torch.dtype, int]] = {}  # id(param) -> (dtype, flat offset)
        by_dtype: dict[torch.dtype, list] = {}
        for p in params:
            by_dtype.setdefault(p.dtype, []).append(p)
        self.numel: dict[torch.dtype, int] = {}  # parameter elements (unpadded) per dtype
        for dtype, plist in by_dtype.items():
            total = sum(p.numel() for p in plist)
            self.numel[dtype] = total
            padded = shard_sizes(total, world) * world
            buffer = None if allocate is not None else self._adopt(plist, padded)
            if buffer is None:
                buffer = (allocate(padded, dtype, plist[0].device) if allocate is not None
                          else torch.zeros(padded, dtype=dtype, device=plist[0].device))
                offset = 0
                for p in plist:
                    n = p.numel()
                    buffer[offset:offset + n].copy_(p.detach().reshape(-1))
                    p.data = buffer[offset:offset + n].view(p.shape)
                    offset += n
            offset = 0
            for p in plist:
                self.place[id(p)] = (dtype, offset)
                offset += p.numel()
            self.buffers[dtype] = buffer

    @staticmethod
    def _adopt(plist, padded):
        """The existing storage, if the parameters fill it exactly, back to back
        from its start, and the layout needs no padding.  Anything else in the
        storage (a frozen tensor stored after the parameters, say) would be
        overwritten by the padding's all-gather, so such storage is never
        adopted and the parameters move into a fresh buffer instead."""
        storage = plist[0].untyped_storage()
        offset = 0
        for p in plist:
            if (p.untyped_storage().data_ptr() != storage.data_ptr() or not p.is_contiguous()
                    or p.storage_offset() != offset):
                return None
            offset += p.numel()
        if offset != padded or storage.nbytes() != padded * plist[0].element_size():
            return None
        base = torch.empty(0, dtype=plist[0].dtype, device=plist[0].device).set_(
            storage, 0, (padded,), (1,))
        return base

    def shard(self, dtype, rank=None) -> tuple[int, int]:
        size = self.buffers[dtype].numel() // self.world
        rank = self.rank if rank is None else rank
        return rank * size, (rank + 1) * size

    def run_on(self, p, rank) -> tuple[int, int] | None:
        """[lo, hi) of p's flattened elements that ``rank`` updates, or None."""
        dtype, offset = self.place[id(p)]
        start, stop = self.shard(dtype, rank)
        lo, hi = max(start, offset) - offset, min(stop, offset + p.numel()) - offset
        return (lo, hi) if lo < hi else None

    def local_run(self, p) -> tuple[int, int] | None:
        """[lo, hi) of p's flattened elements that this rank updates, or None."""
        return self.run_on(p, self.rank)


def peer_order(rank: int, world: int) -> list[int]:
    """The other ranks in rotated order (rank+1, rank+2, ... mod world): the
    kernel's peer stores and the copy streams of every rank then start at a
    different destination, so no GPU receives everyone's first writes at once."""
    return [(rank + k) % world for k in range(1, world)]


class _HostIO:
    """The pinned host buffers of one ``step_host`` call."""

    __slots__ = ("grads", "params", "grad_buffers")

    def __init__(self, grads, params, grad_buffers):
        self.grads, self.params, self.grad_buffers = grads, params, grad_buffers


class _ChunkedExchange:
    """Pipelined copies around a sharded step.  Each launch of the step runs over
    ``chunks`` consecutive tile ranges of its row table, and after each range
    the copy engines move the range's updated parameters while the next range
    is updated:

    * ``gather="copy"``: to every peer (one stream per peer, device-to-device
      copies into the peers' mapped buffers);
    * ``step_host``: to pinned host memory (one device-to-host stream), while a
      host-to-device stream loads each range's gradients ahead of its launch.

    A tile range covers one contiguous run of the flat buffer per parameter
    dtype, because the rows follow the flat buffer's order.  ``chunks=1``
    with ``whole=True`` keeps one full launch (the fused peer stores need it)
    and only brackets it with the host copies."""

    def __init__(self, layout, peer_starts, device, chunks=32, whole=False, copy_streams=None):
        self._layout = layout
        self._peer_starts = peer_starts or {}  # dtype -> start of each peer's buffer, here
        self._chunks = 1 if whole else chunks
        self._whole = whole
        n_peers = len(next(iter(peer_starts.values()))) if peer_starts else 0
        # Copy streams: one per peer by default; fewer serialise the peers of a
        # chunk on each stream (peer w goes to stream w % copy_streams).
        n_streams = n_peers if copy_streams is None else max(1, min(int(copy_streams), n_peers))
        self._streams = [torch.cuda.Stream(device) for _ in range(n_streams if n_peers else 0)]
        self._n_peers = n_peers
        self._device = device
        self._host_streams = None
        self.host: _HostIO | None = None  # set for the duration of a step_host call

    def _plan(self, table):
        """[(tile_lo, tile_hi, [(dtype, address, bytes), ...]), ...] for a table."""
        cached = getattr(table, "_srs_exchange_plan", None)
        if cached is not None and cached[0] == self._chunks:
            return cached[1]
        from .cuda import _native

        host, tile = table.host, 2048
        bounds = [table.n_tiles * k // self._chunks for k in range(self._chunks + 1)]
        plan = []
        for lo, hi in zip(bounds, bounds[1:]):
            if lo == hi:
                continue
            runs = []
            for row in host:
                begin, numel = int(row["tile_begin"]), int(row["numel"])
                end_tile = begin + -(-numel // tile)
                if end_tile <= lo or begin >= hi:
                    continue
                bf16 = bool(int(row["flags"]) & _native.ROW_PARAM_BF16)
                dtype, size = (torch.bfloat16, 2) if bf16 else (torch.float32, 4)
                first = max(lo - begin, 0) * tile
                last = min((hi - begin) * tile, numel)
                start = int(row["param"]) + first * size
                nbytes = (last - first) * size
                if runs and runs[-1][0] == dtype and runs[-1][1] + runs[-1][2] == start:
                    runs[-1] = (dtype, runs[-1][1], runs[-1][2] + nbytes)
                else:
                    runs.append((dtype, start, nbytes))
            plan.append((lo, hi, runs))
        table._srs_exchange_plan = (self._chunks, plan)
        return plan

    def _flat(self, dtype, start, nbytes):
        """[a, b) flat element range of a run of the dtype's parameter buffer."""
        buffer = self._layout.buffers[dtype]
        size = buffer.element_size()
        a = (start - buffer.data_ptr()) // size
        return a, a + nbytes // size

    def run(self, launch, launch_tiles, launch_whole=None):
        """launch_tiles(lo, hi) enqueues the step over tiles [lo, hi) on the
        current stream; launch_whole() the full launch (``whole=True``)."""
        from .cuda import _native

        launcher = _native.launcher()
        compute = torch.cuda.current_stream(launch.device)
        plan = self._plan(launch.table)
        host = self.host
        loaded = []
        if host is not None:
            if self._host_streams is None:
                self._host_streams = (torch.cuda.Stream(self._device),
                                      torch.cuda.Stream(self._device))
            h2d, d2h = self._host_streams
            # Gradient loads overwrite what earlier work on the stream may read.
            h2d.wait_stream(compute)
            d2h.wait_stream(compute)
            with torch.cuda.stream(h2d):
                for _, _, runs in plan:
                    for dtype, start, nbytes in runs:
                        a, b = self._flat(dtype, start, nbytes)
                        host.grad_buffers[dtype][a:b].copy_(host.grads[dtype][a:b],
                                                            non_blocking=True)
                    event = torch.cuda.Event()
                    event.record(h2d)
                    loaded.append(event)
        for i, (lo, hi, runs) in enumerate(plan):
            if loaded:
                compute.wait_event(loaded[i])
            if self._whole:
                launch_whole()
            else:
                launch_tiles(lo, hi)
            done = torch.cuda.Event()
            done.record(compute)
            for stream in self._streams:
                stream.wait_event(done)
            for w in range(self._n_peers):
                stream = self._streams[w % len(self._streams)]
                for dtype, start, nbytes in runs:
                    local = self._layout.buffers[dtype].data_ptr()
                    launcher.copy_async(self._peer_starts[dtype][w] + (start - local), start,
                                        nbytes, stream.cuda_stream)
            if host is not None and host.params is not None:
                d2h.wait_event(done)
                with torch.cuda.stream(d2h):
                    for dtype, start, nbytes in runs:
                        a, b = self._flat(dtype, start, nbytes)
                        host.params[dtype][a:b].copy_(self._layout.buffers[dtype][a:b],
                                                      non_blocking=True)
        for stream in self._streams:
            compute.wait_stream(stream)
        if host is not None:
            compute.wait_stream(self._host_streams[1])


class _ZeroMixin:
    """ZeRO-1 behaviour for a fused StateOptimizer subclass (see module docstring)."""

    def __init__(self, params, *args, process_group=None, gather="auto", chunks=32,
                 grads="full", record_timings=False, copy_peers=1, copy_streams=None,
                 **kwargs):
        if gather not in ("auto", "fused", "copy", "nccl", "multicast", "hybrid"):
            raise ValueError("gather must be 'auto', 'fused', 'copy', 'nccl', 'multicast' or "
                             f"'hybrid', got {gather!r}")
        if grads not in ("full", "reduce_scatter"):
            raise ValueError(f"grads must be 'full' or 'reduce_scatter', got {grads!r}")
        super().__init__(params, *args, **kwargs)
        self._group = process_group
        initialized = torch.distributed.is_available() and torch.distributed.is_initialized()
        self._world = torch.distributed.get_world_size(process_group) if initialized else 1
        self._rank = torch.distributed.get_rank(process_group) if initialized else 0
        ordered = [p for g in self.param_groups for p in g["params"]]
        symmetric = (gather == "multicast" and self._world > 1
                     and all(p.device.type == "cuda" for p in ordered))
        if gather == "multicast" and not symmetric:
            gather = "auto"  # one rank or host tensors: no multicast to bind
        self._layout = FlatLayout(ordered, self._world, self._rank,
                                  allocate=_symmetric_zeros if symmetric else None)
        self._symm_handles: dict = {}
        # CUDA events of the last steps (record_timings=True); bounded, so a run
        # that never reads `timings` keeps at most this many steps' events.
        self._record_timings = bool(record_timings)
        self._events: collections.deque = collections.deque(maxlen=4096)
        self._timed: list = []
        self._grad_buffers: dict[torch.dtype, torch.Tensor] = {}
        if grads == "reduce_scatter":
            for dtype, buffer in self._layout.buffers.items():
                self._grad_buffers[dtype] = torch.zeros_like(buffer)
            for p in ordered:
                p.grad = self._grad_slot(p)
        self._peer_bases: list[int] = []
        self._srs_peers = None
        self._srs_exchange = None
        self._host_pipeline = None
        self._chunks = chunks
        self._sync = None
        if self._world > 1:
            device = next(iter(self._layout.buffers.values())).device
            self._sync = torch.zeros(1, device=device)
            if gather == "auto":
                # Measured on B200 (8B parameters): with one peer the copy engines
                # beat the kernel's own peer stores (12.1 vs 13.4 ms per step); with
                # three, concurrent peer copies fell to ~400 GB/s (33.6 vs 18.4 ms).
                gather = "copy" if self._world == 2 else "fused"
            multicast = self._connect_multicast() if gather == "multicast" else None
            if multicast is not None:
                self._srs_peers = multicast
            elif gather in ("fused", "copy", "multicast", "hybrid"):
                connected = self._connect_peers()
                if connected is not None and gather in ("fused", "multicast"):
                    self._srs_peers = connected[0]
                elif connected is not None and gather == "hybrid" and self._world > 2:
                    kernel_peers, copy_starts = _split_peers(*connected, copy_peers)
                    self._srs_peers = kernel_peers
                    self._srs_exchange = _ChunkedExchange(self._layout, copy_starts, device,
                                                          chunks, copy_streams=copy_streams)
                elif connected is not None:  # "copy", or "hybrid" with a single peer
                    self._srs_exchange = _ChunkedExchange(self._layout, connected[1], device,
                                                          chunks, copy_streams=copy_streams)
        if self._world == 1:
            self._gather = "none"
        elif self._srs_peers is not None and self._srs_exchange is not None:
            self._gather = "hybrid"
        elif self._srs_peers is not None:
            self._gather = ("multicast" if self._srs_peers.mode == _peers_multicast()
                            else "fused")
        else:
            self._gather = "copy" if self._srs_exchange is not None else "nccl"
        self._connected_gather = self._gather
        self._connected = (self._srs_peers, self._srs_exchange)

    @property
    def gather_mode(self) -> str:
        """'fused' (peer stores inside the step), 'multicast' (one NVLink
        multicast store per vector inside the step), 'copy' (copy engines
        pipelined with the step), 'hybrid' (the step's tile ranges store to
        some peers, the copy engines serve the others), 'nccl' (all-gather
        after it) or 'none' (one rank)."""
        return self._gather

    def set_gather_mode(self, mode: str) -> None:
        """Switch between the exchange chosen at construction and the NCCL
        all-gather, for the following steps (every rank must switch together).
        Both deliver the same parameters; the NCCL form runs the update as a
        launch of its own, which is how the update alone is timed."""
        if self._world == 1:
            if mode != "none":
                raise ValueError("a single rank has no exchange (gather mode 'none')")
            return
        if mode not in ("nccl", self._connected_gather):
            raise ValueError(f"gather mode must be 'nccl' or {self._connected_gather!r}, "
                             f"got {mode!r}")
        self._gather = mode
        self._srs_peers, self._srs_exchange = (
            self._connected if mode == self._connected_gather else (None, None))

    def _agree(self, value):
        """Every rank's ``value`` (a collective: all ranks call it together)."""
        everyone = [None] * self._world
        torch.distributed.all_gather_object(everyone, value, group=self._group)
        return everyone

    def _connect_peers(self):
        """Map every peer's flat buffers into this process: (peer deltas for the
        fused kernel, {dtype: start of each peer's buffer here}); None on every
        rank if any rank cannot (then the step ends with an NCCL all-gather)."""
        from .cuda import _native

        buffers = self._layout.buffers
        mine = None
        if (self._world - 1 <= _native.MAX_PEERS
                and all(d in (torch.float32, torch.bfloat16) for d in buffers)
                and all(b.device.type == "cuda" for b in buffers.values())):
            launcher = _native.launcher()
            try:
                mine = {str(d): launcher.ipc_export(b.data_ptr()) for d, b in buffers.items()}
            except (ValueError, RuntimeError):
                mine = None
        everyone = self._agree(mine)
        if any(entry is None for entry in everyone):
            return None
        peers, starts, ok = _native.SrsPeers(), {d: [] for d in buffers}, True
        try:
            n = 0
            for r in peer_order(self._rank, self._world):
                for dtype, buf in buffers.items():
                    handle, offset = everyone[r][str(dtype)]
                    base = launcher.ipc_import(handle)
                    self._peer_bases.append(base)
                    deltas = peers.delta_bf16 if dtype == torch.bfloat16 else peers.delta_f32
                    deltas[n] = base + offset - buf.data_ptr()
                    starts[dtype].append(base + offset)
                n += 1
            peers.n_peers = n
        except (ValueError, RuntimeError):
            ok = False
        if not all(self._agree(ok)):
            self._close_peers()
            return None
        return peers, starts

    def _connect_multicast(self):
        """Bind every rank's flat buffers (symmetric allocations) to NVLink
        multicast objects: SrsPeers in multicast mode, with the peers' own
        addresses for the element-wise tails; None on every rank if any rank
        lacks multicast support (then peer stores are tried)."""
        from .cuda import _native

        group = self._group if self._group is not None else torch.distributed.group.WORLD
        handles, mapped, multicast = {}, False, False
        try:
            import torch.distributed._symmetric_memory as symm_mem

            for dtype, buffer in self._layout.buffers.items():
                handles[dtype] = symm_mem.rendezvous(buffer, group)
            mapped = all(len(h.buffer_ptrs) == self._world for h in handles.values())
            multicast = mapped and all(h.multicast_ptr != 0 for h in handles.values())
        except (RuntimeError, ValueError, AttributeError, ImportError):
            mapped = multicast = False
        everyone = self._agree((mapped, multicast))
        if not all(m for m, _ in everyone):
            return None
        peers = _native.SrsPeers()
        # Without multicast support on every rank: plain peer stores through the
        # symmetric mappings.
        peers.mode = (_native.PEERS_MULTICAST if all(mc for _, mc in everyone)
                      else _native.PEERS_STORE)
        peers.n_peers = self._world - 1
        for dtype, buffer in self._layout.buffers.items():
            h = handles[dtype]
            offset = buffer.data_ptr() - int(h.buffer_ptrs[self._rank])
            mc = int(h.multicast_ptr) + offset - buffer.data_ptr() if h.multicast_ptr else 0
            deltas = peers.delta_bf16 if dtype == torch.bfloat16 else peers.delta_f32
            for n, r in enumerate(peer_order(self._rank, self._world)):
                deltas[n] = int(h.buffer_ptrs[r]) + offset - buffer.data_ptr()
            if peers.mode != _native.PEERS_MULTICAST:
                continue
            if dtype == torch.bfloat16:
                peers.mc_delta_bf16 = mc
            else:
                peers.mc_delta_f32 = mc
        self._symm_handles = handles
        return peers

    def _close_peers(self):
        if self._peer_bases:
            from .cuda import _native

            for base in self._peer_bases:
                _native.launcher().ipc_close(base)
        self._peer_bases = []

    def _barrier(self):
        torch.distributed.all_reduce(self._sync, group=self._group)

    # ------------------------------------------------------------ gradients --

    def _grad_slot(self, p):
        dtype, offset = self._layout.place[id(p)]
        return self._grad_buffers[dtype][offset:offset + p.numel()].view(p.shape)

    @torch.no_grad()
    def zero_grad(self, set_to_none: bool = True):
        """With ``grads="reduce_scatter"`` the flat gradient buffers are zeroed in
        place (the gradients stay views into them); otherwise as in PyTorch."""
        if not self._grad_buffers:
            return super().zero_grad(set_to_none)
        for buffer in self._grad_buffers.values():
            buffer.zero_()
        for g in self.param_groups:
            for p in g["params"]:
                p.grad = self._grad_slot(p)

    @torch.no_grad()
    def reduce_scatter_grads(self, op: str = "mean"):
        """Reduce every rank's gradients (``"mean"`` or ``"sum"``) into this rank's
        shard of the flat gradient buffers, in place.  A collective; requires
        ``grads="reduce_scatter"``.  Gradients that backward placed outside the
        buffers (after ``zero_grad(set_to_none=True)`` elsewhere) are copied in."""
        if not self._grad_buffers:
            raise RuntimeError("reduce_scatter_grads requires grads='reduce_scatter'")
        if op not in ("mean", "sum"):
            raise ValueError(f"op must be 'mean' or 'sum', got {op!r}")
        for g in self.param_groups:
            for p in g["params"]:
                slot = self._grad_slot(p)
                if p.grad is None:
                    slot.zero_()
                elif p.grad.data_ptr() != slot.data_ptr() or p.grad.shape != slot.shape:
                    slot.copy_(p.grad)
                p.grad = slot
        if self._world == 1:
            return
        dist = torch.distributed
        gloo = dist.get_backend(self._group) == "gloo"
        for dtype, buffer in self._grad_buffers.items():
            lo, hi = self._layout.shard(dtype)
            if gloo:  # gloo has no reduce-scatter of a flat tensor: reduce everything
                self._collective(dist.all_reduce, buffer)
            else:
                dist.reduce_scatter_tensor(buffer[lo:hi], buffer, group=self._group)
            if op == "mean":
                buffer[lo:hi].div_(self._world)

    # ---------------------------------------------------------- checkpoints --

    def _ordered_params(self):
        return [p for g in self.param_groups for p in g["params"]]

    def state_dict(self, *, to_rank: int | None = None, bucket_bytes: int = 1 << 28):
        """The unsharded state dict: every state in its parameter's shape, the
        layout of the unsharded optimizer, so it resumes at any world size or
        in that optimizer.  A collective: call it on every rank.

        Each rank contributes only its runs.  ``to_rank=None``: every rank
        receives the others' runs (an all-gather) and returns the whole dict;
        ``to_rank=r``: only rank r receives them (a gather) and returns the
        dict, the other ranks return ``{}``.  The runs travel in buckets of
        about ``bucket_bytes`` of states, so the transient memory beyond the
        result stays bounded."""
        local = super().state_dict()
        if self._world > 1 and to_rank is not None and not 0 <= to_rank < self._world:
            raise ValueError(f"to_rank must be a rank of the group, got {to_rank}")
        receive = to_rank is None or to_rank == self._rank
        params = self._ordered_params()
        names = self._state_names
        formats = self.param_formats()
        device = next(iter(self._layout.buffers.values())).device
        # Which parameters have states on any rank, and their AdamW steps.
        present = torch.zeros(len(params), dtype=torch.int64, device=device)
        steps = torch.zeros(len(params), dtype=torch.int64, device=device)
        for i, p in enumerate(params):
            st = self.state.get(p, {})
            if any(n in st for n in names):
                present[i] = 1
                steps[i] = int(st.get("step", 0))
        if self._world > 1:
            for flags in (present, steps):
                self._collective(torch.distributed.all_reduce, flags,
                                 op=torch.distributed.ReduceOp.MAX)
        present, steps = present.tolist(), steps.tolist()
        wanted = [(i, name, fmt) for i, p in enumerate(params) if present[i]
                  for name, fmt in zip(names, formats[id(p)])]
        full = {}
        for bucket in _buckets(wanted, params, bucket_bytes):
            full.update(self._gather_runs(bucket, params, to_rank, receive, device))
        if not receive:
            return {}
        state = {}
        for i, p in enumerate(params):
            if not present[i]:
                continue
            entry = {name: full[i, name].view(p.shape) for name in names}
            if self._uses_step:
                entry["step"] = int(steps[i])
            state[i] = entry
        local["state"] = state
        return local

    def _collective(self, fn, tensor, *args, **kwargs):
        """Run a collective on ``tensor``; with gloo, device tensors go through
        host memory (gloo moves host buffers)."""
        dist = torch.distributed
        if tensor.device.type == "cuda" and dist.get_backend(self._group) == "gloo":
            host = tensor.cpu()
            fn(host, *args, group=self._group, **kwargs)
            tensor.copy_(host)
        else:
            fn(tensor, *args, group=self._group, **kwargs)

    def _gather_runs(self, bucket, params, to_rank, receive, device):
        """{(param index, state name): full-size state} of one bucket, assembled
        from every rank's runs (on the receiving ranks; {} elsewhere)."""
        layout, world = self._layout, self._world

        def runs(rank):
            out = []
            for i, name, fmt in bucket:
                run = layout.run_on(params[i], rank)
                if run is not None:
                    out.append((i, name, fmt, run))
            return out

        def nbytes(rank):
            return sum((hi - lo) * _itemsize(fmt.dtype) for _, _, fmt, (lo, hi) in runs(rank))

        width = max(nbytes(r) for r in range(world))
        mine = torch.zeros(width, dtype=torch.uint8, device=device)
        at = 0
        for i, name, fmt, (lo, hi) in runs(self._rank):
            size = (hi - lo) * _itemsize(fmt.dtype)
            held = self.state.get(params[i], {}).get(name)
            if held is not None:
                mine[at:at + size].copy_(held.reshape(-1).view(torch.uint8))
            at += size
        if world == 1:
            everyone = [mine]
        else:
            everyone = self._exchange(mine, to_rank, receive)
        if not receive:
            return {}
        full = {(i, name): torch.zeros(params[i].numel(), dtype=fmt.dtype, device=device)
                for i, name, fmt in bucket}
        for rank, chunk in enumerate(everyone):
            at = 0
            for i, name, fmt, (lo, hi) in runs(rank):
                size = (hi - lo) * _itemsize(fmt.dtype)
                full[i, name][lo:hi].view(torch.uint8).copy_(chunk[at:at + size])
                at += size
        return full

    def _exchange(self, mine, to_rank, receive):
        """Every rank's equally sized byte buffer: [rank 0's, rank 1's, ...] on the
        receiving ranks (None elsewhere)."""
        dist, world = torch.distributed, self._world
        gloo = dist.get_backend(self._group) == "gloo"
        send = mine.cpu() if gloo and mine.is_cuda else mine
        if to_rank is None:
            out = torch.empty(world * send.numel(), dtype=torch.uint8, device=send.device)
            dist.all_gather_into_tensor(out, send, group=self._group)
            chunks = list(out.view(world, -1))
        else:
            dst = dist.get_global_rank(self._group, to_rank) if self._group is not None else to_rank
            chunks = [torch.empty_like(send) for _ in range(world)] if receive else None
            dist.gather(send, chunks, dst=dst, group=self._group)
        if not receive:
            return None
        return [c.to(mine.device) for c in chunks]

    def load_state_dict(self, state_dict):
        """Load the unsharded layout (from ``state_dict()`` here or from the
        unsharded optimizer) and keep this rank's runs."""
        super().load_state_dict(state_dict)
        self._keep_local_runs()

    def _keep_local_runs(self):
        for p in self._ordered_params():
            st = self.state.get(p)
            if not st:
                continue
            run = self._layout.local_run(p)
            if run is None:
                del self.state[p]
                continue
            for name in self._state_names:
                if name in st and st[name].numel() == p.numel():
                    st[name] = st[name].reshape(-1)[run[0]:run[1]].clone()

    def sharded_state_dict(self):
        """This rank's runs of the states plus the layout they belong to."""
        return {"zero1": {"world": self._world, "rank": self._rank,
                          "numels": [p.numel() for p in self._ordered_params()]},
                "optimizer": super().state_dict()}

    def load_sharded_state_dict(self, sharded):
        """Restore this rank's runs saved by ``sharded_state_dict()`` on the same
        rank of a run with the same world size and parameters."""
        meta = sharded["zero1"]
        if (meta["world"], meta["rank"]) != (self._world, self._rank):
            raise ValueError(
                f"sharded checkpoint of rank {meta['rank']} of {meta['world']} cannot be "
                f"loaded on rank {self._rank} of {self._world}; use state_dict() instead")
        if meta["numels"] != [p.numel() for p in self._ordered_params()]:
            raise ValueError("sharded checkpoint parameters do not match this optimizer")
        super().load_state_dict(sharded["optimizer"])

    def local_numel(self) -> int:
        total = 0
        for g in self.param_groups:
            for p in g["params"]:
                run = self._layout.local_run(p)
                total += (run[1] - run[0]) if run else 0
        return total

    def launches_per_step(self) -> int:
        return getattr(self, "_srs_launches_last_step", 0)

    def _group_items(self, group, formats, first_index):
        names = self._state_names
        for param_index, parameter in enumerate(group["params"], start=first_index):
            grad = parameter.grad
            if grad is None:
                continue
            if grad.is_sparse:
                raise RuntimeError(f"{type(self).__name__} does not support sparse gradients")
            _validate_rng_numel(parameter.numel())
            run = self._layout.local_run(parameter)
            if run is None:
                continue
            lo, hi = run
            piece = _Piece(parameter.detach().view(-1)[lo:hi], grad.reshape(-1)[lo:hi])
            state = self.state[parameter]
            for name, fmt in zip(names, formats):
                if name not in state:
                    state[name] = torch.zeros(hi - lo, dtype=fmt.dtype, device=parameter.device)
                elif state[name].dtype != fmt.dtype:
                    raise ValueError(f"{name} dtype does not match its state format")
            yield piece, state, param_index, state.get("step", 0) + 1, lo + self._shard_start(
                parameter)

    @torch.no_grad()
    def step(self, closure=None):
        stream = (torch.cuda.current_stream()
                  if self._record_timings and torch.cuda.is_available() else None)
        marks = [torch.cuda.Event(enable_timing=True) for _ in range(4)] if stream else None
        fused = self._gather in ("fused", "copy", "multicast", "hybrid")
        if marks:
            marks[0].record(stream)
        if fused:
            self._barrier()
        if marks:
            marks[1].record(stream)
        self._srs_launches = 0
        loss = super().step(closure)
        self._srs_launches_last_step = self._srs_launches
        if marks:
            marks[2].record(stream)
        if fused:
            self._barrier()
        elif self._world > 1:
            for dtype, buffer in self._layout.buffers.items():
                lo, hi = self._layout.shard(dtype)
                if buffer.is_cuda and torch.distributed.get_backend(self._group) == "gloo":
                    host = buffer.cpu()  # gloo moves host buffers
                    torch.distributed.all_gather_into_tensor(host, host[lo:hi].clone(),
                                                             group=self._group)
                    buffer.copy_(host)
                else:
                    torch.distributed.all_gather_into_tensor(buffer, buffer[lo:hi],
                                                             group=self._group)
        if marks:
            marks[3].record(stream)
            self._events.append(marks)
        return loss

    def local_run(self, p) -> tuple[int, int] | None:
        """[lo, hi) of p's flattened elements that this rank updates (its states
        hold exactly these elements), or None."""
        return self._layout.local_run(p)

    def flat_params(self, dtype):
        """This rank's replica of the flat parameter buffer of a dtype (padded
        to equal shards; element i is flat parameter element i)."""
        return self._layout.buffers[dtype]

    def flat_grads(self, dtype):
        """The flat gradient buffer of a parameter dtype (``grads="reduce_scatter"``;
        None otherwise): element i is the gradient of flat parameter element i."""
        return self._grad_buffers.get(dtype)

    def flat_numel(self, dtype) -> int:
        """Parameter elements of a dtype, all ranks (the unpadded flat length)."""
        return self._layout.numel[dtype]

    @torch.no_grad()
    def step_host(self, grads, params=None):
        """One step whose gradients come from pinned host memory and whose updated
        parameters go back to it, the copies pipelined with the update: the step
        runs over ``chunks`` tile ranges, a host-to-device stream loads each
        range's gradients ahead of its launch and a device-to-host stream sends
        each finished range back, so both directions of PCIe and the kernel work
        at the same time.  (With ``gather="fused"`` and more than one rank the
        update stays one launch, bracketed by the two copies.)

        ``grads`` / ``params``: {dtype: pinned CPU tensor} (a tensor alone when
        all parameters share one dtype), laid out like the flat parameter
        buffer of that dtype: element i belongs to flat element i, parameters in
        optimizer order, back to back.  Each rank loads only its shard's
        gradients and writes back only its shard's parameters.  Needs
        ``grads="reduce_scatter"`` (the gradients are loaded into the flat
        gradient buffers the parameters' ``.grad`` views).  The host buffers
        are in use until the current stream has passed the step.
        """
        if not self._grad_buffers:
            raise RuntimeError("step_host requires grads='reduce_scatter' (flat gradient buffers)")
        grads = self._host_tensors(grads, "grads")
        params = None if params is None else self._host_tensors(params, "params")
        for group in self.param_groups:
            for p in group["params"]:
                if p.grad is None or p.grad.data_ptr() != self._grad_slot(p).data_ptr():
                    raise RuntimeError("step_host: every p.grad must be its flat gradient view "
                                       "(set by the optimizer and zero_grad())")
        pipeline = self._srs_exchange
        restore = pipeline
        if pipeline is None:
            # One full launch when the kernel itself stores to the peers; tile
            # ranges otherwise.  One cached pipeline per kind.
            whole = self._srs_peers is not None
            if self._host_pipeline is None:
                self._host_pipeline = {}
            if whole not in self._host_pipeline:
                device = next(iter(self._layout.buffers.values())).device
                self._host_pipeline[whole] = _ChunkedExchange(self._layout, None, device,
                                                              self._chunks, whole=whole)
            pipeline = self._srs_exchange = self._host_pipeline[whole]
        pipeline.host = _HostIO(grads, params, self._grad_buffers)
        try:
            return self.step()
        finally:
            pipeline.host = None
            self._srs_exchange = restore

    def _host_tensors(self, tensors, what):
        if isinstance(tensors, torch.Tensor):
            if len(self._layout.buffers) != 1:
                raise ValueError(f"{what}: one tensor per parameter dtype is needed")
            tensors = {next(iter(self._layout.buffers)): tensors}
        out = {}
        for dtype, buffer in self._layout.buffers.items():
            t = tensors.get(dtype) if isinstance(tensors, dict) else None
            if t is None:
                raise ValueError(f"{what}: no host tensor for {dtype}")
            need = self._layout.numel[dtype]
            if (t.device.type != "cpu" or t.dtype != dtype or not t.is_contiguous()
                    or t.dim() != 1 or t.numel() < need or not t.is_pinned()):
                raise ValueError(f"{what}[{dtype}] must be a contiguous pinned 1-D CPU tensor of "
                                 f"{dtype} with at least {need} elements")
            out[dtype] = t
        return out

    @property
    def timings(self):
        """Per step since the last clear (only with ``record_timings=True``):
        update_ms (the fused launches, including their peer stores when the
        gather is fused) and gather_ms (the barriers around a fused step, or the
        NCCL all-gather); reading it synchronizes on the recorded events."""
        for marks in self._events:
            marks[3].synchronize()
            self._timed.append({"update_ms": marks[1].elapsed_time(marks[2]),
                                "gather_ms": marks[0].elapsed_time(marks[1])
                                + marks[2].elapsed_time(marks[3])})
        self._events.clear()
        return _TimingList(self._timed)

    def close(self):
        """Drop recorded timings and unmap the peers' buffers (call after the last
        step, on every rank, while the process group still exists)."""
        self._events.clear()
        self._timed = []
        if self._srs_exchange is not None or self._symm_handles:
            torch.cuda.current_stream().synchronize()
        if self._symm_handles and self._gather == "multicast":
            self._barrier()  # no rank still stores through the multicast objects
            torch.cuda.current_stream().synchronize()
        self._close_peers()
        self._srs_peers = None
        self._srs_exchange = None
        self._host_pipeline = None
        if self._gather in ("fused", "copy", "multicast", "hybrid"):
            self._gather = "nccl"  # a later step all-gathers
        # The multicast bindings (self._symm_handles) stay: the parameters live in
        # those buffers.  They are released with the buffers, normally at exit.
        self._connected_gather = self._gather if self._world > 1 else "none"
        self._connected = (None, None)


class _TimingList(list):
    def __init__(self, backing):
        super().__init__(backing)
        self._backing = backing

    def clear(self):
        super().clear()
        self._backing.clear()


class ZeroAdamW(_ZeroMixin, AdamWReferenceSR):
    """AdamW (fused, sm_100a) with ZeRO-1 sharded states; see the module docstring."""


class ZeroSGDM(_ZeroMixin, SGDMReferenceSR):
    """Momentum SGD (fused, sm_100a) with ZeRO-1 sharded states."""


def _split_peers(peers, starts, copy_peers):
    """(kernel peers, {dtype: copy-engine peer starts}) from the connected
    peers in rotated order: the last ``copy_peers`` of them (at least one, at
    most all but one) go to the copy engines, the rest to the kernel's stores."""
    from .cuda import _native

    n = peers.n_peers
    k = min(max(int(copy_peers), 1), n - 1)
    kernel = _native.SrsPeers()
    kernel.mode = peers.mode
    kernel.n_peers = n - k
    for i in range(n - k):
        kernel.delta_f32[i] = peers.delta_f32[i]
        kernel.delta_bf16[i] = peers.delta_bf16[i]
    return kernel, {dtype: list(s[n - k:]) for dtype, s in starts.items()}


def _symmetric_zeros(numel, dtype, device):
    """A zeroed flat buffer from PyTorch's symmetric-memory allocator (each rank's
    buffer mappable by the others and bindable to an NVLink multicast object)."""
    import torch.distributed._symmetric_memory as symm_mem

    return symm_mem.empty(numel, dtype=dtype, device=device).zero_()


def _peers_multicast() -> int:
    from .cuda import _native

    return _native.PEERS_MULTICAST


def _itemsize(dtype) -> int:
    return torch.empty((), dtype=dtype).element_size()


def _buckets(wanted, params, limit):
    """Split [(param index, state name, format), ...] into lists of about
    ``limit`` bytes of full-size states each (at least one entry per list)."""
    bucket, size = [], 0
    for item in wanted:
        i, _, fmt = item
        nbytes = params[i].numel() * _itemsize(fmt.dtype)
        if bucket and size + nbytes > limit:
            yield bucket
            bucket, size = [], 0
        bucket.append(item)
        size += nbytes
    if bucket:
        yield bucket


def shard_sizes(numel_total: int, world: int) -> int:
    """Elements per shard of a flat buffer of ``numel_total`` elements (the
    buffer is padded to a multiple of ``world * SHARD_ALIGN``)."""
    unit = world * SHARD_ALIGN
    return -(-numel_total // unit) * unit // world
