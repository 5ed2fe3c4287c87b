"""ZeroAdamW / ZeroSGDM.step_host: gradients streamed in from pinned host memory
and updated parameters streamed back, pipelined with tile-range launches.

The step must give the bits of an ordinary step on the same gradients
(tolerance: exact), for any chunk count, with parameters of two dtypes (two
flat buffers), and the host parameter buffer must then hold the updated
parameters.  Validation (no flat gradient buffers, unpinned or short host
tensors) is checked on CPU.
"""

import numpy as np
import pytest
import torch

from sr_states import AdamWReferenceSR, SGDMReferenceSR, StateFormat
from sr_states.distributed import ZeroAdamW, ZeroSGDM

SIZES = [(70001, torch.bfloat16), (4099, torch.float32), (1, torch.bfloat16),
         (300000, torch.bfloat16), (2048, torch.float32), (5, torch.float32)]


def _bits(t):
    return t.detach().contiguous().view(torch.int16 if t.element_size() == 2 else torch.int32
                                        ).cpu().numpy()


def _params(device, seed):
    gen = torch.Generator().manual_seed(seed)
    return [torch.nn.Parameter(torch.randn(n, generator=gen).to(device, dtype))
            for n, dtype in SIZES]


def _grads(step):
    gen = torch.Generator().manual_seed(100 + step)
    return [(torch.randn(n, generator=gen) * 1e-2).to(dtype) for n, dtype in SIZES]


def _make(kind, params, zero, chunks=32):
    if kind == "adamw":
        fmt = {"exp_avg": StateFormat(torch.float8_e4m3fn),
               "exp_avg_sq": StateFormat(torch.bfloat16)}
        if zero:
            return ZeroAdamW(params, lr=1e-3, state_format=fmt, seed=9, grads="reduce_scatter",
                             chunks=chunks)
        return AdamWReferenceSR(params, lr=1e-3, state_format=fmt, seed=9)
    fmt = StateFormat(torch.bfloat16)
    if zero:
        return ZeroSGDM(params, lr=0.05, momentum=0.9, state_format=fmt, seed=9,
                        grads="reduce_scatter", chunks=chunks)
    return SGDMReferenceSR(params, lr=0.05, momentum=0.9, state_format=fmt, seed=9)


def _host_buffers(opt, grads):
    """{dtype: pinned flat tensor} of the gradients, and empty pinned parameter buffers."""
    host_g, host_p = {}, {}
    for dtype in (torch.bfloat16, torch.float32):
        flat = torch.cat([g.reshape(-1) for g, (_, d) in zip(grads, SIZES) if d == dtype])
        assert flat.numel() == opt.flat_numel(dtype)
        host_g[dtype] = flat.pin_memory()
        host_p[dtype] = torch.empty(flat.numel(), dtype=dtype, pin_memory=True)
    return host_g, host_p


@pytest.mark.gpu
@pytest.mark.parametrize("chunks", [1, 5, 32])
@pytest.mark.parametrize("kind", ["adamw", "sgdm"])
def test_step_host_equals_step_on_device_gradients(cuda_device, kind, chunks):
    ours, theirs = _params(cuda_device, 1), _params(cuda_device, 1)
    opt, ref = _make(kind, ours, True, chunks), _make(kind, theirs, False)
    for step in range(3):
        grads = _grads(step)
        host_g, host_p = _host_buffers(opt, grads)
        for p, g in zip(theirs, grads):
            p.grad = g.to(cuda_device)
        opt.step_host(host_g, host_p)
        ref.step()
        torch.cuda.synchronize()
        for i, (a, b) in enumerate(zip(ours, theirs)):
            assert np.array_equal(_bits(a), _bits(b)), f"step {step} param {i}"
        for dtype in (torch.bfloat16, torch.float32):
            device = torch.cat([p.detach().reshape(-1) for p, (_, d) in zip(ours, SIZES)
                                if d == dtype])
            assert np.array_equal(_bits(host_p[dtype]), _bits(device)), f"host {dtype}"
            # The gradients the step read are the host's.
            assert torch.equal(opt.flat_grads(dtype)[:host_g[dtype].numel()].cpu(),
                               host_g[dtype])
    opt.close()


@pytest.mark.gpu
def test_step_host_without_parameter_readback_and_plain_steps_between(cuda_device):
    ours, theirs = _params(cuda_device, 2), _params(cuda_device, 2)
    opt, ref = _make("adamw", ours, True), _make("adamw", theirs, False)
    for step in range(2):
        grads = _grads(step)
        host_g, _ = _host_buffers(opt, grads)
        for p, g in zip(theirs, grads):
            p.grad = g.to(cuda_device)
        if step == 0:
            opt.step_host(host_g)
        else:  # an ordinary step on gradients already in the flat buffers
            for p, g in zip(ours, grads):
                p.grad.copy_(g)
            opt.step()
        ref.step()
    torch.cuda.synchronize()
    assert all(np.array_equal(_bits(a), _bits(b)) for a, b in zip(ours, theirs))


def test_step_host_validates_its_buffers():
    params = [torch.nn.Parameter(torch.ones(10)), torch.nn.Parameter(torch.ones(3))]
    opt = ZeroAdamW(params, lr=1e-3)
    with pytest.raises(RuntimeError, match="grads='reduce_scatter'"):
        opt.step_host(torch.ones(13))
    opt = ZeroAdamW(params, lr=1e-3, grads="reduce_scatter")
    assert opt.flat_numel(torch.float32) == 13
    assert opt.flat_grads(torch.float32).numel() >= 13
    with pytest.raises(ValueError, match="pinned"):
        opt.step_host(torch.ones(13))  # pageable memory
    with pytest.raises(ValueError, match="no host tensor"):
        opt.step_host({torch.bfloat16: torch.ones(13)})
