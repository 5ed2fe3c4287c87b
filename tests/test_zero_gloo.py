"""ZeRO-1 on CPU ranks (gloo, world size 2 and 3): sharded fused steps plus the
all-gather reproduce the unsharded step byte for byte, and each rank holds
exactly its slice of the states.  Kernel launches run the oracle stand-in."""

import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem():
    from sr_states import StateFormat

    torch.manual_seed(1234)
    shapes = [(37, 5), (129,), (1000,), (3,), (2049,), (64, 64)]
    params = [torch.nn.Parameter(torch.randn(s).to(torch.bfloat16 if i % 2 else torch.float32))
              for i, s in enumerate(shapes)]
    grads = [[torch.randn(s).to(p.dtype) for p, s in zip(params, shapes)] for _ in range(3)]
    grads[1][2] = None  # a skipped gradient still consumes its parameter index
    fmt = {"exp_avg": StateFormat(torch.float8_e4m3fn), "exp_avg_sq": StateFormat(torch.bfloat16)}
    return params, grads, fmt


def _run(cls, params, grads, fmt, **kw):
    opt = cls([{"params": params[:3]}, {"params": params[3:], "weight_decay": 0.0}], lr=1e-2,
              state_format=fmt, seed=2**40 + 3, **kw)
    for step_grads in grads:
        for p, g in zip(params, step_grads):
            p.grad = None if g is None else g.clone()
        opt.step()
    return opt


def _worker(rank, world, port, queue):
    sys.path[:0] = [str(ROOT), str(ROOT / "stochastic-rounding-pytorch_b200"), str(ROOT / "tests")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import torch.distributed as dist

    from _support import FakeLauncher
    from sr_states import AdamWReferenceSR
    from sr_states.cuda import _native
    from sr_states.distributed import ZeroAdamW

    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        _native.set_launcher(FakeLauncher())
        params, grads, fmt = _problem()
        reference = [torch.nn.Parameter(p.detach().clone()) for p in params]
        ref_opt = _run(AdamWReferenceSR, reference, grads, fmt)
        sharded = _run(ZeroAdamW, params, grads, fmt)
        for p, q in zip(params, reference):
            assert torch.equal(p.detach().view(torch.uint8), q.detach().view(torch.uint8))
        covered = 0
        for p, q in zip(params, reference):
            run = sharded._layout.local_run(p)
            if run is None:
                assert "exp_avg" not in sharded.state[p]
                continue
            lo, hi = run
            covered += hi - lo
            for name in ("exp_avg", "exp_avg_sq"):
                mine = sharded.state[p][name].view(torch.uint8)
                full = ref_opt.state[q][name].reshape(-1)[lo:hi].view(torch.uint8)
                assert torch.equal(mine, full), (rank, name)
            assert sharded.state[p]["step"] == ref_opt.state[q]["step"]
        total = torch.tensor([covered])
        dist.all_reduce(total)
        assert total.item() == sum(p.numel() for p in params)
        queue.put((rank, "ok"))
    except BaseException as exc:  # report, never hang the parent
        queue.put((rank, repr(exc)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_zero1_sharded_steps_equal_unsharded(world):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert results == {r: "ok" for r in range(world)}, results


def _checkpoint_worker(rank, world, port, queue):
    sys.path[:0] = [str(ROOT), str(ROOT / "stochastic-rounding-pytorch_b200"), str(ROOT / "tests")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import torch.distributed as dist

    from _support import FakeLauncher
    from sr_states import AdamWReferenceSR
    from sr_states.cuda import _native
    from sr_states.distributed import ZeroAdamW

    def resume(cls, checkpoint, values, grads, fmt, sharded=False):
        params = [torch.nn.Parameter(v.clone()) for v in values]
        opt = cls([{"params": params[:3]}, {"params": params[3:], "weight_decay": 0.0}],
                  lr=1e-2, state_format=fmt, seed=2**40 + 3)
        if sharded:
            opt.load_sharded_state_dict(checkpoint)
        else:
            opt.load_state_dict(checkpoint)
        for step_grads in grads:
            for p, g in zip(params, step_grads):
                p.grad = None if g is None else g.clone()
            opt.step()
        return params

    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        _native.set_launcher(FakeLauncher())
        params, grads, fmt = _problem()
        reference = [torch.nn.Parameter(p.detach().clone()) for p in params]
        ref_opt = _run(AdamWReferenceSR, reference, grads[:2], fmt)
        sharded = _run(ZeroAdamW, params, grads[:2], fmt)
        full = sharded.state_dict()
        expected = ref_opt.state_dict()
        # Gathered to one rank, in many small buckets: the same dict there, {} elsewhere.
        last = world - 1
        one = sharded.state_dict(to_rank=last, bucket_bytes=64)
        if rank == last:
            assert set(one["state"]) == set(full["state"]) and one["param_groups"] == full["param_groups"]
            for key, entry in full["state"].items():
                assert one["state"][key].keys() == entry.keys()
                for name in ("exp_avg", "exp_avg_sq"):
                    assert torch.equal(one["state"][key][name].view(torch.uint8),
                                       entry[name].view(torch.uint8))
        else:
            assert one == {}
        assert set(full["state"]) == set(expected["state"])
        for key, entry in expected["state"].items():
            mine = full["state"][key]
            assert mine["step"] == entry["step"]
            for name in ("exp_avg", "exp_avg_sq"):
                assert mine[name].shape == entry[name].shape and mine[name].dtype == entry[name].dtype
                assert torch.equal(mine[name].view(torch.uint8), entry[name].view(torch.uint8))
        assert full["param_groups"] == expected["param_groups"]
        values = [p.detach().clone() for p in reference]
        tail = grads[2:] + grads[:1]
        ref_tail = resume(AdamWReferenceSR, expected, values, tail, fmt)
        for cls, ckpt, kw in ((ZeroAdamW, full, {}), (AdamWReferenceSR, full, {}),
                              (ZeroAdamW, sharded.sharded_state_dict(), {"sharded": True})):
            got = resume(cls, ckpt, values, tail, fmt, **kw)
            for p, q in zip(got, ref_tail):
                assert torch.equal(p.detach().view(torch.uint8), q.detach().view(torch.uint8)), cls
        queue.put((rank, "ok"))
    except BaseException as exc:  # report, never hang the parent
        import traceback
        queue.put((rank, traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_zero1_checkpoints_gather_to_the_unsharded_layout_and_resume(world):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_checkpoint_worker, args=(r, world, port, queue))
             for r in range(world)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert results == {r: "ok" for r in range(world)}, results


def _reduce_scatter_worker(rank, world, port, queue):
    sys.path[:0] = [str(ROOT), str(ROOT / "stochastic-rounding-pytorch_b200"), str(ROOT / "tests")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import torch.distributed as dist

    from _support import FakeLauncher
    from sr_states import AdamWReferenceSR
    from sr_states.cuda import _native
    from sr_states.distributed import ZeroAdamW

    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        _native.set_launcher(FakeLauncher())
        params, _, fmt = _problem()
        reference = [torch.nn.Parameter(p.detach().clone()) for p in params]
        ref_opt = AdamWReferenceSR(reference, lr=1e-2, state_format=fmt, seed=11)
        opt = ZeroAdamW(params, lr=1e-2, state_format=fmt, seed=11, grads="reduce_scatter")

        def rank_grad(p, r, step):
            # small integers times 2^-10: sums over ranks are exact in any order
            gen = torch.Generator().manual_seed(1000 * step + 10 * r + p.numel())
            return (torch.randint(-8, 9, p.shape, generator=gen).float() / 1024).to(p.dtype)

        for step in range(2):
            opt.zero_grad()
            for i, p in enumerate(params):
                if i == 1:
                    p.grad = rank_grad(p, rank, step)  # a fresh tensor: copied into the buffer
                else:
                    p.grad.copy_(rank_grad(p, rank, step))
            opt.reduce_scatter_grads("mean")
            opt.step()
            for q, p in zip(reference, params):
                total = sum(rank_grad(p, r, step).float() for r in range(world)).to(p.dtype)
                q.grad = total.div_(world)
            ref_opt.step()
        for p, q in zip(params, reference):
            assert torch.equal(p.detach().view(torch.uint8), q.detach().view(torch.uint8))
        queue.put((rank, "ok"))
    except BaseException:  # report, never hang the parent
        import traceback
        queue.put((rank, traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_zero_reduce_scattered_gradients_equal_unsharded_mean_gradients(world):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_reduce_scatter_worker, args=(r, world, port, queue))
             for r in range(world)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert results == {r: "ok" for r in range(world)}, results


def test_peer_order_rotates_destinations():
    from sr_states.distributed import peer_order

    for world in (2, 3, 4, 8):
        orders = [peer_order(r, world) for r in range(world)]
        for r, order in enumerate(orders):
            assert sorted(order) == [q for q in range(world) if q != r]
        # At every position each rank is the destination of exactly one rank.
        for k in range(world - 1):
            assert sorted(order[k] for order in orders) == list(range(world))


def _spawn(worker, world):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return results


def _shared_storage_worker(rank, world, port, queue):
    sys.path[:0] = [str(ROOT), str(ROOT / "stochastic-rounding-pytorch_b200"), str(ROOT / "tests")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import torch.distributed as dist

    from _support import FakeLauncher
    from sr_states import AdamWReferenceSR
    from sr_states.cuda import _native
    from sr_states.distributed import ZeroAdamW

    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        _native.set_launcher(FakeLauncher())
        # Two parameters back to back, then a frozen tensor in the same storage,
        # different on every rank (as rank-local data would be).
        storage = torch.randn(1000 + 200, generator=torch.Generator().manual_seed(5))
        storage[1000:] = float(rank + 1)
        params = [torch.nn.Parameter(storage[:600].view(20, 30)),
                  torch.nn.Parameter(storage[600:1000])]
        frozen = storage[1000:]
        before = frozen.clone()
        reference = [torch.nn.Parameter(p.detach().clone()) for p in params]
        opt = ZeroAdamW(params, lr=1e-2, seed=3)
        ref_opt = AdamWReferenceSR(reference, lr=1e-2, seed=3)
        assert opt.gather_mode == "nccl"
        opt.set_gather_mode("nccl")
        try:
            opt.set_gather_mode("fused")
            raise AssertionError("a mode that was never connected must be refused")
        except ValueError:
            pass
        for step in range(2):
            for p, q in zip(params, reference):
                g = torch.randn(p.shape, generator=torch.Generator().manual_seed(step))
                p.grad, q.grad = g.clone(), g.clone()
            opt.step()
            ref_opt.step()
        assert torch.equal(frozen, before), "the frozen tensor after the parameters changed"
        for p, q in zip(params, reference):
            assert torch.equal(p.detach(), q.detach())
        queue.put((rank, "ok"))
    except BaseException:  # report, never hang the parent
        import traceback
        queue.put((rank, traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_zero_never_adopts_storage_shared_with_other_tensors():
    """Parameters that share their storage with a tensor stored after them move to
    a fresh flat buffer, so the padding's all-gather cannot overwrite that tensor."""
    results = _spawn(_shared_storage_worker, 2)
    assert results == {0: "ok", 1: "ok"}, results


def _verify_worker(rank, world, port, queue):
    sys.path[:0] = [str(ROOT), str(ROOT / "stochastic-rounding-pytorch_b200"), str(ROOT / "tests")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    import importlib.util
    import math

    import torch.distributed as dist

    from _support import FakeLauncher
    from sr_states import StateFormat
    from sr_states.cuda import _native
    from sr_states.distributed import ZeroAdamW
    from sr_states.shapes import _llama

    class CorruptingLauncher(FakeLauncher):
        """The oracle stand-in, plus one wrong first-moment byte on rank 1: a
        planted mistake that the bench's verification must report."""

        def adamw_multi(self, table, *args, **kwargs):
            super().adamw_multi(table, *args, **kwargs)
            if rank == 1:
                address = int(table.host[0]["state"][0])
                byte = (ctypes.c_uint8 * 1).from_address(address)
                byte[0] ^= 0x01

    import ctypes

    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
        bench = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(bench)
        named = _llama(2, 64, 16, 128, vocab=300)
        names, shapes = [n for n, _ in named], [s for _, s in named]
        results = []
        for launcher in (FakeLauncher(), CorruptingLauncher()):
            _native.set_launcher(launcher)
            gen = torch.Generator().manual_seed(7)
            params = [torch.nn.Parameter((torch.randn(math.prod(s), generator=gen) * 0.02)
                                         .to(torch.bfloat16).view(s)) for s in shapes]
            fmt = {"exp_avg": StateFormat(torch.float8_e4m3fn, "stochastic"),
                   "exp_avg_sq": StateFormat(torch.bfloat16, "stochastic")}
            opt = ZeroAdamW(params, lr=bench.LR, betas=bench.BETAS, eps=bench.EPS,
                            weight_decay=bench.WEIGHT_DECAY, state_format=fmt, seed=bench.SEED,
                            grads="reduce_scatter")
            opt.flat_grads(torch.bfloat16).copy_(
                torch.randn(opt.flat_grads(torch.bfloat16).numel(), generator=gen) * 1e-4)
            for _ in range(2):
                opt.step()
            results.append(bench.verify_step(opt, names, params, world, rank))
        if rank == 0:
            clean, corrupt = results
            assert clean["replicas_equal"] and clean["mismatched_bytes"] == 0, clean
            assert clean["elements"] > 0 and clean["rng_step"] == 3, clean
            assert corrupt["mismatched_bytes"] > 0, corrupt
        else:
            assert results == [None, None]
        queue.put((rank, "ok"))
    except BaseException:  # report, never hang the parent
        import traceback
        queue.put((rank, traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_bench_verification_passes_sharded_steps_and_reports_a_planted_mistake():
    """bench.py's post-run check (replica digests plus oracle windows gathered
    from the owners of the states) on two gloo ranks: clean steps verify, and a
    wrong state byte on one rank is reported."""
    results = _spawn(_verify_worker, 2)
    assert results == {0: "ok", 1: "ok"}, results


def test_hybrid_split_gives_the_last_peers_to_the_copy_engines():
    from sr_states.cuda import _native
    from sr_states.distributed import _split_peers

    peers = _native.SrsPeers()
    peers.n_peers = 7
    for i in range(7):
        peers.delta_bf16[i] = 1000 * (i + 1)
        peers.delta_f32[i] = -1000 * (i + 1)
    starts = {torch.bfloat16: [10 * (i + 1) for i in range(7)]}
    for k, kept in ((1, 6), (3, 4), (0, 6), (9, 1)):
        kernel, copies = _split_peers(peers, starts, k)
        assert kernel.n_peers == kept
        assert [kernel.delta_bf16[i] for i in range(kept)] == [1000 * (i + 1) for i in range(kept)]
        assert [kernel.delta_f32[i] for i in range(kept)] == [-1000 * (i + 1) for i in range(kept)]
        assert copies[torch.bfloat16] == [10 * (i + 1) for i in range(kept, 7)]
