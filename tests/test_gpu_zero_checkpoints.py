"""Sharded checkpoints and reduce-scattered gradients with the real kernels on one
GPU: two ranks, as two processes on cuda:0 over gloo (the parameter exchange is
the collective all-gather, staged through host memory as gloo requires), each
compared byte for byte with the unsharded optimizer stepping on the mean
gradients in the same process.

Covered: ``reduce_scatter_grads`` (every rank's own gradients, reduced into its
shard), ``state_dict()`` on every rank and ``state_dict(to_rank=...)`` in small
buckets (equal to the unsharded optimizer's, reference layout:
sr_states/optim/_state.py:202-236 of the reference), resuming from it in a
fresh sharded optimizer and in the unsharded one, and
``sharded_state_dict()`` / ``load_sharded_state_dict()``.  Tolerance: exact.
"""

import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, port, queue):
    sys.path[:0] = [str(ROOT), str(ROOT / "stochastic-rounding-pytorch_b200"), str(ROOT / "tests")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import torch.distributed as dist

    from sr_states import AdamWReferenceSR, StateFormat
    from sr_states.distributed import ZeroAdamW

    def bits(t):
        return t.detach().reshape(-1).view(torch.uint8).cpu()

    try:
        torch.cuda.set_device(0)
        device = torch.device("cuda", 0)
        dist.init_process_group("gloo", rank=rank, world_size=WORLD,
                                timeout=datetime.timedelta(seconds=120))
        shapes = [(300, 7), (129,), (4096,), (3,), (2049,), (64, 33)]
        gen = torch.Generator().manual_seed(5)
        init = [(torch.randn(s, generator=gen) * 0.02).to(
            torch.bfloat16 if i % 2 else torch.float32) for i, s in enumerate(shapes)]
        fmt = {"exp_avg": StateFormat(torch.float8_e4m3fn), "exp_avg_sq": StateFormat(torch.bfloat16)}
        kw = dict(lr=1e-2, weight_decay=0.1, state_format=fmt, seed=2**33 + 9)

        def make(cls, values, **extra):
            params = [torch.nn.Parameter(v.clone().to(device)) for v in values]
            groups = [{"params": params[:3]}, {"params": params[3:], "weight_decay": 0.0}]
            return params, cls(groups, **kw, **extra)

        def rank_grad(p, r, step):
            # small integers times 2^-12: sums over ranks are exact in any order
            g = torch.Generator().manual_seed(1000 * step + 10 * r + p.numel())
            return (torch.randint(-8, 9, p.shape, generator=g).float() / 4096).to(device, p.dtype)

        def run(params, opt, ref_params, ref_opt, steps):
            for step in steps:
                opt.zero_grad()
                for p in params:
                    p.grad.copy_(rank_grad(p, rank, step))
                opt.reduce_scatter_grads("mean")
                opt.step()
                for p, q in zip(params, ref_params):
                    total = sum(rank_grad(p, r, step).float() for r in range(WORLD))
                    q.grad = (total / WORLD).to(q.dtype)
                ref_opt.step()
            for p, q in zip(params, ref_params):
                assert torch.equal(bits(p), bits(q)), "parameters differ from the unsharded step"

        params, opt = make(ZeroAdamW, init, gather="nccl", grads="reduce_scatter")
        ref_params, ref_opt = make(AdamWReferenceSR, init)
        run(params, opt, ref_params, ref_opt, range(3))

        expected = ref_opt.state_dict()
        for full in (opt.state_dict(), opt.state_dict(to_rank=0, bucket_bytes=1000)):
            if not full:
                assert rank != 0
                continue
            assert full["param_groups"] == expected["param_groups"]
            assert set(full["state"]) == set(expected["state"])
            for key, entry in expected["state"].items():
                assert full["state"][key]["step"] == entry["step"]
                for name in ("exp_avg", "exp_avg_sq"):
                    assert full["state"][key][name].shape == entry[name].shape
                    assert torch.equal(bits(full["state"][key][name]), bits(entry[name]))
        checkpoint = opt.state_dict()
        sharded = opt.sharded_state_dict()
        values = [p.detach().clone() for p in params]

        # Resume three ways and continue in step with the unsharded optimizer.
        resumed_params, resumed = make(ZeroAdamW, values, gather="nccl", grads="reduce_scatter")
        resumed.load_state_dict(checkpoint)
        again_params, again = make(ZeroAdamW, values, gather="nccl", grads="reduce_scatter")
        again.load_sharded_state_dict(sharded)
        plain_params, plain = make(AdamWReferenceSR, values)
        plain.load_state_dict(checkpoint)
        ref_copy_params, ref_copy = make(AdamWReferenceSR, values)
        ref_copy.load_state_dict(expected)
        for p_list, o in ((resumed_params, resumed), (again_params, again)):
            ref_p, ref_o = make(AdamWReferenceSR, values)
            ref_o.load_state_dict(expected)
            run(p_list, o, ref_p, ref_o, range(3, 5))
        for step in range(3, 5):
            for q, r in zip(plain_params, ref_copy_params):
                total = sum(rank_grad(q, k, step).float() for k in range(WORLD))
                q.grad = (total / WORLD).to(q.dtype)
                r.grad = q.grad.clone()
            plain.step()
            ref_copy.step()
        for q, r in zip(plain_params, ref_copy_params):
            assert torch.equal(bits(q), bits(r)), "unsharded resume from the gathered checkpoint"
        for o in (opt, resumed, again):
            o.close()
        torch.cuda.synchronize()
        queue.put((rank, "ok"))
    except BaseException:  # report, never hang the parent
        import traceback
        queue.put((rank, traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_sharded_checkpoints_and_reduce_scatter_on_one_gpu(cuda_device):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, queue)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    assert results == {r: "ok" for r in range(WORLD)}, results
