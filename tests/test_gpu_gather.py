"""The fused all-gather of the sharded steps: the step kernel stores every
updated parameter vector locally and at the same offset of each peer replica.

On one GPU the peers are emulated by extra buffers of this device (the kernel
sees only address deltas), which checks the stores themselves: replicas get
exactly the updated rows, nothing else is written, and the local results are
bit-identical to the launch without peers.  The two-rank test maps real peer
GPUs through CUDA IPC and needs two GPUs."""

import os

import numpy as np
import pytest
import torch

from sr_states.cuda import _native
from sr_states.cuda._fused import adamw_hparams, rng_words, sgdm_hparams
from sr_states.cuda._tables import DeviceTable, Update, build_table, upload

pytestmark = pytest.mark.gpu

SIZES = [70001, 2048, 1, 4099, 300000]


def _workload(device, p_dtype, states):
    gen = torch.Generator().manual_seed(3)
    total = sum(SIZES) + 517  # padding after the rows that must stay untouched
    flat = torch.randn(total, generator=gen).to(device, p_dtype)
    grads = [torch.randn(n, generator=gen).to(device, torch.bfloat16) * 1e-2 for n in SIZES]
    updates, offset = [], 0
    for i, (n, g) in enumerate(zip(SIZES, grads)):
        st = [torch.zeros(n, dtype=d, device=device) for d in states]
        updates.append(Update((flat[offset:offset + n], g, *st), i, n, 0, 1))
        offset += n
    return flat, updates


def _table(updates, device):
    host = build_table(updates, [0] * len(updates), 2048)
    n_tiles = int(host["tile_begin"][-1] + -(-host["numel"][-1] // 2048))
    return DeviceTable(host, upload(host, device), len(host), n_tiles)


def _clone(updates, flat):
    new_flat = flat.clone()
    out, offset = [], 0
    for u in updates:
        n = u.numel
        out.append(Update((new_flat[offset:offset + n], u.tensors[1],
                           *(s.clone() for s in u.tensors[2:])), u.param_index, n, 0, 1))
        offset += n
    return new_flat, out


def _bits(t):
    return t.view(torch.uint8).cpu().numpy()


@pytest.mark.parametrize("kind", ["adamw", "sgdm"])
@pytest.mark.parametrize("p_dtype", [torch.bfloat16, torch.float32], ids=["bf16", "fp32"])
def test_peer_stores_fill_replicas_and_leave_results_unchanged(cuda_device, kind, p_dtype):
    launcher = _native.launcher()
    states = ((torch.float8_e4m3fn, torch.bfloat16) if kind == "adamw" else (torch.bfloat16,))
    flat, updates = _workload(cuda_device, p_dtype, states)
    flat_ref, updates_ref = _clone(updates, flat)
    replicas = [torch.full_like(flat, 7.0) for _ in range(3)]
    peers = _native.SrsPeers()
    peers.n_peers = len(replicas)
    for i, r in enumerate(replicas):
        deltas = peers.delta_bf16 if p_dtype == torch.bfloat16 else peers.delta_f32
        deltas[i] = r.data_ptr() - flat.data_ptr()
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    rng = rng_words(11, 4)
    for ups, extra in ((updates, {"peers": peers}), (updates_ref, {})):
        table = _table(ups, cuda_device)
        if kind == "adamw":
            hp = adamw_hparams(1e-3, (0.9, 0.999), 1e-8, 0.01, (1,))
            launcher.adamw_multi(table, table.n_rows, table.n_tiles, 3, 1, 1, 1, hp, rng, stream,
                                 **extra)
        else:
            hp = sgdm_hparams(1e-2, 0.9)
            launcher.sgdm_multi(table, table.n_rows, table.n_tiles, 1, 1, hp, rng, stream,
                                **extra)
    torch.cuda.synchronize(cuda_device)
    rows = sum(SIZES)
    assert np.array_equal(_bits(flat), _bits(flat_ref))
    for u, r in zip(updates, updates_ref):
        for a, b in zip(u.tensors[2:], r.tensors[2:]):
            assert np.array_equal(_bits(a), _bits(b))
    for rep in replicas:
        assert np.array_equal(_bits(rep[:rows]), _bits(flat[:rows]))
        assert torch.all(rep[rows:] == 7.0)


@pytest.mark.parametrize("kind", ["adamw", "sgdm"])
def test_tile_range_launches_equal_one_launch(cuda_device, kind):
    """A table launched as consecutive tile ranges (the chunks of a pipelined
    exchange) gives the bits of one launch over the whole table."""
    launcher = _native.launcher()
    states = ((torch.float8_e4m3fn, torch.bfloat16) if kind == "adamw" else (torch.bfloat16,))
    flat, updates = _workload(cuda_device, torch.bfloat16, states)
    flat_ref, updates_ref = _clone(updates, flat)
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    rng = rng_words(5, 9)
    for ups, ranged in ((updates, True), (updates_ref, False)):
        table = _table(ups, cuda_device)
        cuts = [0, 1, 7, 40, table.n_tiles] if ranged else [0, table.n_tiles]
        for lo, hi in zip(cuts, cuts[1:]):
            extra = {"tiles": (lo, hi)} if ranged else {}
            if kind == "adamw":
                hp = adamw_hparams(1e-3, (0.9, 0.999), 1e-8, 0.01, (1,))
                launcher.adamw_multi(table, table.n_rows, table.n_tiles, 3, 1, 1, 1, hp, rng,
                                     stream, **extra)
            else:
                launcher.sgdm_multi(table, table.n_rows, table.n_tiles, 1, 1,
                                    sgdm_hparams(1e-2, 0.9), rng, stream, **extra)
    torch.cuda.synchronize(cuda_device)
    assert np.array_equal(_bits(flat), _bits(flat_ref))
    for u, r in zip(updates, updates_ref):
        for a, b in zip(u.tensors[2:], r.tensors[2:]):
            assert np.array_equal(_bits(a), _bits(b))
    dst = torch.zeros_like(flat)
    launcher.copy_async(dst.data_ptr(), flat.data_ptr(), 1000 * 2, stream)
    torch.cuda.synchronize(cuda_device)
    assert torch.equal(dst[:1000], flat[:1000]) and torch.all(dst[1000:] == 0)
    with pytest.raises(ValueError, match="tile range"):
        launcher.sgdm_multi(table, table.n_rows, table.n_tiles, 1, 1, sgdm_hparams(1e-2, 0.9),
                            rng, stream, tiles=(3, table.n_tiles + 1))


def test_peer_count_is_checked(cuda_device):
    launcher = _native.launcher()
    flat, updates = _workload(cuda_device, torch.bfloat16, (torch.bfloat16,))
    table = _table(updates, cuda_device)
    peers = _native.SrsPeers()
    peers.n_peers = _native.MAX_PEERS + 1
    with pytest.raises(ValueError, match="n_peers"):
        launcher.sgdm_multi(table, table.n_rows, table.n_tiles, 1, 1, sgdm_hparams(1e-2, 0.9),
                            rng_words(1, 1), torch.cuda.current_stream().cuda_stream,
                            peers=peers)


def _two_rank_worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    import datetime

    import torch.distributed as dist

    from sr_states import StateFormat
    from sr_states.distributed import ZeroAdamW

    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        fmt = {"exp_avg": StateFormat(torch.float8_e4m3fn, "stochastic"),
               "exp_avg_sq": StateFormat(torch.bfloat16, "stochastic")}
        runs = {}
        for mode in ("fused", "copy", "nccl", "single", "multicast"):
            gen = torch.Generator().manual_seed(5)
            params = []
            for n in SIZES:
                p = torch.nn.Parameter(torch.randn(n, generator=gen).to("cuda", torch.bfloat16))
                p.grad = (torch.randn(n, generator=gen) * 1e-2).to("cuda", torch.bfloat16)
                params.append(p)
            if mode == "single":
                from sr_states import AdamWReferenceSR

                opt = AdamWReferenceSR(params, lr=1e-3, state_format=fmt, seed=9)
            else:
                opt = ZeroAdamW(params, lr=1e-3, state_format=fmt, seed=9, gather=mode)
                runs[mode + "_mode"] = opt.gather_mode
            for _ in range(3):
                opt.step()
            torch.cuda.synchronize()
            runs[mode] = [p.detach().view(torch.uint16).cpu().numpy().copy() for p in params]
            if mode != "single":
                opt.close()
        same = {m: all(np.array_equal(a, b) for a, b in zip(runs[m], runs["single"]))
                for m in ("fused", "copy", "nccl", "multicast")}
        # Gradients reduce-scattered by NCCL (small integers times 2^-10 summed exactly)
        # equal the unsharded step on the mean gradients.
        outs = {}
        for mode in ("rs", "single"):
            gen = torch.Generator().manual_seed(6)
            params = [torch.nn.Parameter(torch.randn(n, generator=gen).to("cuda", torch.bfloat16))
                      for n in SIZES]
            if mode == "rs":
                opt = ZeroAdamW(params, lr=1e-3, state_format=fmt, seed=9, grads="reduce_scatter")
                opt.zero_grad()
                for i, p in enumerate(params):
                    g = torch.Generator().manual_seed(100 * rank + i)
                    p.grad.copy_((torch.randint(-8, 9, (p.numel(),), generator=g) / 1024.0)
                                 .to("cuda", torch.bfloat16))
                opt.reduce_scatter_grads("mean")
            else:
                from sr_states import AdamWReferenceSR

                opt = AdamWReferenceSR(params, lr=1e-3, state_format=fmt, seed=9)
                for i, p in enumerate(params):
                    total = sum(torch.randint(-8, 9, (p.numel(),),
                                              generator=torch.Generator().manual_seed(100 * r + i))
                                / 1024.0 for r in range(world))
                    p.grad = (total / world).to("cuda", torch.bfloat16)
            opt.step()
            torch.cuda.synchronize()
            outs[mode] = [p.detach().view(torch.uint16).cpu().numpy().copy() for p in params]
            if mode == "rs":
                opt.close()
        same["reduce_scatter"] = all(np.array_equal(a, b) for a, b in zip(outs["rs"], outs["single"]))
        # step_host in every gather mode: each rank loads its gradient shard from
        # the host and writes back its parameter shard; the replicas equal the
        # unsharded steps of the first block.
        for mode in ("fused", "copy", "nccl"):
            gen = torch.Generator().manual_seed(5)
            params, grads = [], []
            for n in SIZES:
                params.append(torch.nn.Parameter(torch.randn(n, generator=gen)
                                                 .to("cuda", torch.bfloat16)))
                grads.append((torch.randn(n, generator=gen) * 1e-2).to(torch.bfloat16))
            opt = ZeroAdamW(params, lr=1e-3, state_format=fmt, seed=9, gather=mode,
                            grads="reduce_scatter")
            host_g = torch.cat(grads).pin_memory()
            host_p = torch.zeros(host_g.numel(), dtype=torch.bfloat16, pin_memory=True)
            for _ in range(3):
                opt.step_host(host_g, host_p)
            torch.cuda.synchronize()
            ok = all(np.array_equal(p.detach().view(torch.uint16).cpu().numpy(), b)
                     for p, b in zip(params, runs["single"]))
            lo, hi = opt._layout.shard(torch.bfloat16)
            hi = min(hi, host_g.numel())
            device = torch.cat([p.detach().reshape(-1) for p in params])
            ok = ok and torch.equal(host_p[lo:hi], device[lo:hi].cpu())
            same["host_" + mode] = ok
            opt.close()
        results[rank] = ((runs["fused_mode"], runs["copy_mode"], runs["nccl_mode"],
                          runs["multicast_mode"]), same)
        del opt, params
        import gc

        gc.collect()
        torch.cuda.synchronize()
        dist.barrier()  # every rank releases its multicast-bound buffers before any exits
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_fused_and_copy_gathers_equal_nccl_and_unsharded_steps():
    import torch.multiprocessing as mp

    manager = mp.get_context("spawn").Manager()  # no fork after CUDA is initialised
    results = manager.dict()
    mp.spawn(_two_rank_worker, args=(2, 29533, results), nprocs=2, join=True)
    for rank in range(2):
        modes, same = results[rank]
        assert modes[:3] == ("fused", "copy", "nccl")
        assert modes[3] in ("multicast", "fused")  # peer stores where NVLS is unavailable
        assert same == {"fused": True, "copy": True, "nccl": True, "multicast": True,
                        "reduce_scatter": True, "host_fused": True, "host_copy": True,
                        "host_nccl": True}
