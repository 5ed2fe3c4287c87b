"""Host logic of the fused optimizers on CPU: bookkeeping, row tables, caches and
validation, with kernel launches executed by the oracle stand-in."""

import copy

import pytest
import torch

import _scenarios
from _support import FakeLauncher
from sr_states import AdamWReferenceRN, AdamWReferenceSR, SGDMReferenceSR, StateFormat
from sr_states._hash import update_key
from sr_states.cuda import AdamWCuda, SGDMCuda, cuda_adamw_step_, cuda_sgdm_step_


@pytest.mark.parametrize("spec", _scenarios.scenarios(), ids=lambda s: s["name"])
def test_reference_scenarios_replay_on_host_tables(spec, fake_launcher):
    compared, mismatched = _scenarios.replay(spec, torch.device("cpu"))
    assert compared > 0
    if spec["kind"] == "sgdm":
        assert mismatched == 0


@pytest.mark.parametrize("cls", [AdamWCuda, SGDMCuda])
def test_block_size_classes_match_reference_scenario(cls, fake_launcher):
    kind = "adamw" if cls is AdamWCuda else "sgdm"
    spec = next(s for s in _scenarios.scenarios() if s["kind"] == kind)
    _scenarios.replay(spec, torch.device("cpu"), cls=cls)


def _param(n, dtype=torch.float32):
    p = torch.nn.Parameter(torch.ones(n, dtype=dtype))
    p.grad = torch.ones_like(p)
    return p


@pytest.mark.parametrize("cls", [AdamWReferenceSR, SGDMReferenceSR])
def test_one_launch_per_group_and_device_whatever_the_dtypes_and_steps(cls, fake_launcher):
    p, q, r, empty, second = _param(1), _param(4097), _param(3, torch.bfloat16), _param(0), _param(31)
    opt = cls([{"params": [p, q, r, empty]}, {"params": [second]}], lr=0.01)
    opt.step()
    multi = [c for c in fake_launcher.calls]
    assert len(multi) == 2  # one per group; FP32 and BF16 rows share the launch
    assert multi[0][1:3] == (3, 1 + 3 + 1)  # rows, tiles (4097 elements = 3 tiles of 2048)
    fake_launcher.calls.clear()
    q.grad = None
    opt.step()
    q.grad = torch.ones_like(q)
    fake_launcher.calls.clear()
    opt.step()  # AdamW: q is one step behind -> two step classes, still one launch
    assert len(fake_launcher.calls) == 2
    if cls is AdamWReferenceSR:
        assert opt.state[q]["step"] == 2 and opt.state[p]["step"] == 3


@pytest.mark.parametrize("cls", [AdamWReferenceSR, SGDMReferenceSR])
def test_no_launch_when_a_later_parameter_is_invalid(cls, fake_launcher):
    p, r = _param(5), _param(3, torch.bfloat16)
    opt = cls([p, r], lr=0.01)
    opt.step()
    before = p.detach().clone()
    fake_launcher.calls.clear()
    opt.state[r][opt._state_names[0]] = torch.zeros(4, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="shapes"):
        opt.step()
    assert not fake_launcher.calls
    assert torch.equal(p, before)


def test_tables_are_reused_until_addresses_layout_or_steps_change(fake_launcher):
    from sr_states.cuda._tables import group_cache

    p = _param(17)
    opt = AdamWReferenceSR([p], lr=0.01)
    opt.step()
    cache = group_cache(opt, opt.param_groups[0])
    first = cache._entries[p.device]
    opt.step()
    assert cache._entries[p.device] is first  # the step advanced, the table did not change
    keep = p.grad
    p.grad = torch.ones_like(p)  # new address
    opt.step()
    assert cache._entries[p.device] is not first
    assert keep is not None


def test_more_step_classes_than_one_launch_holds(fake_launcher):
    params = [_param(3) for _ in range(40)]
    opt = AdamWReferenceSR(params, lr=0.01)
    for i, p in enumerate(params):
        opt.state[p]["exp_avg"] = torch.zeros(3, dtype=torch.bfloat16)
        opt.state[p]["exp_avg_sq"] = torch.zeros(3, dtype=torch.bfloat16)
        opt.state[p]["step"] = i
    opt.step()
    assert len(fake_launcher.calls) == 2  # 40 distinct AdamW steps -> 32 + 8 classes
    assert [opt.state[p]["step"] for p in params] == list(range(1, 41))


def test_overlapping_writes_are_rejected_even_across_dtypes(fake_launcher):
    shared = torch.ones(12)
    a = torch.nn.Parameter(shared[:8])
    b = torch.nn.Parameter(shared[4:])
    a.grad, b.grad = torch.ones(8), torch.ones(8)
    opt = SGDMReferenceSR([a, b], lr=0.1)
    with pytest.raises(ValueError, match="overlap"):
        opt.step()
    assert not fake_launcher.calls


def test_shared_gradients_are_allowed(fake_launcher):
    a, b = _param(8), _param(8)
    b.grad = a.grad
    SGDMReferenceSR([a, b], lr=0.1).step()


def test_rng_step_is_reserved_even_when_the_step_fails(fake_launcher):
    p = _param(4)
    opt = AdamWReferenceSR([p], lr=0.01)
    opt.step()
    p.grad = torch.sparse_coo_tensor([[0]], [1.0], size=(4,), check_invariants=True)
    with pytest.raises(RuntimeError, match="sparse"):
        opt.step()
    assert opt._rng_step() == 2


def test_rn_class_forces_nearest(fake_launcher):
    p, q = _param(17), _param(17)
    rn = AdamWReferenceRN([p], lr=0.01, state_format={"exp_avg": StateFormat(torch.float8_e4m3fn),
                                                      "exp_avg_sq": StateFormat(torch.float16)})
    sr = AdamWReferenceSR([q], lr=0.01, state_format={
        "exp_avg": StateFormat(torch.float8_e4m3fn, "nearest"),
        "exp_avg_sq": StateFormat(torch.float16, "nearest")})
    for _ in range(3):
        p.grad = q.grad = torch.sin(torch.arange(17.0))
        rn.step()
        sr.step()
    assert torch.equal(p, q)
    for n in rn._state_names:
        assert torch.equal(rn.state[p][n].view(torch.uint8 if n == "exp_avg" else torch.int16),
                           sr.state[q][n].view(torch.uint8 if n == "exp_avg" else torch.int16))


@pytest.mark.parametrize("cls", [AdamWReferenceSR, SGDMReferenceSR])
def test_checkpoint_resume_is_identical(cls, fake_launcher):
    initial = torch.linspace(-1, 1, 1003)
    p = torch.nn.Parameter(initial.clone())
    opt = cls([p], lr=0.01, seed=77)
    p.grad = torch.cos(initial)
    opt.step()
    q = torch.nn.Parameter(p.detach().clone())
    resumed = cls([q], lr=0.1, seed=12)
    resumed.load_state_dict(copy.deepcopy(opt.state_dict()))
    for step in range(1, 4):
        p.grad = torch.sin(initial * step)
        q.grad = p.grad.clone()
        opt.step()
        resumed.step()
        assert torch.equal(p, q)
        for name in opt._state_names:
            assert torch.equal(opt.state[p][name], resumed.state[q][name])


def test_functional_steps_use_the_given_update_key_and_offset(fake_launcher):
    g = 1.0 + torch.arange(1031, dtype=torch.float32) / 2048
    key = update_key(0xFEDCBA9876543210, (1 << 32) + 1, 7)
    offset = (1 << 32) - 211
    full = [torch.ones_like(g), g, torch.zeros_like(g, dtype=torch.float16),
            torch.zeros_like(g, dtype=torch.float16)]
    parts = [t.clone() for t in full]
    options = dict(lr=0.01, beta1=0.5, beta2=0.5, eps=0.125, weight_decay=0.0, step=1, seed=key)
    cuda_adamw_step_(*full, offset=offset, **options)
    for lo, hi in ((0, 11), (11, 227), (227, 728), (728, g.numel())):
        cuda_adamw_step_(*(t[lo:hi] for t in parts), offset=offset + lo, **options)
    for a, b in zip(full, parts):
        assert torch.equal(a.view(torch.uint8), b.view(torch.uint8))
    u = torch.zeros_like(g, dtype=torch.float8_e5m2)
    cuda_sgdm_step_(torch.ones_like(g), g, u, lr=0.1, momentum_factor=0.5, seed=key, offset=3)
    assert fake_launcher.calls[-1] == ("sgdm_single", 1031)
