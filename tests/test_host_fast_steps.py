"""Repeated steps of an unchanged group reuse the prepared launches (CPU, oracle
launcher).  Every case runs beside a twin optimizer whose cache is dropped
before each step, so the twin always takes the full preparation; the two must
stay bit-identical, and the fast path must notice every change that the full
preparation would react to."""

import pytest
import torch

from sr_states import AdamWReferenceSR, SGDMReferenceSR, StateFormat
from sr_states.cuda._tables import group_cache


def _params(seed, sizes=(5, 4097, 3), dtype=torch.float32):
    gen = torch.Generator().manual_seed(seed)
    out = []
    for n in sizes:
        p = torch.nn.Parameter(torch.randn(n, generator=gen).to(dtype))
        p.grad = (torch.randn(n, generator=gen) * 1e-2).to(dtype)
        out.append(p)
    return out


def _twins(cls, **kwargs):
    fmt = ({"exp_avg": StateFormat(torch.float8_e4m3fn, "stochastic"),
            "exp_avg_sq": StateFormat(torch.bfloat16, "stochastic")}
           if cls is AdamWReferenceSR else StateFormat(torch.bfloat16, "stochastic"))
    a, b = _params(1), _params(1)
    return (cls(a, lr=0.01, state_format=fmt, seed=5, **kwargs), a,
            cls(b, lr=0.01, state_format=fmt, seed=5, **kwargs), b)


def _full_step(opt):
    for group in opt.param_groups:
        group_cache(opt, group).fast = None
    opt.step()


def _same(opt_a, a, opt_b, b):
    for p, q in zip(a, b):
        assert torch.equal(p.detach().view(torch.uint8), q.detach().view(torch.uint8))
        for name in opt_a._state_names:
            assert torch.equal(opt_a.state[p][name].view(torch.uint8),
                               opt_b.state[q][name].view(torch.uint8))
        assert opt_a.state[p].get("step") == opt_b.state[q].get("step")


def _kwargs(cls):
    return {"momentum": 0.9} if cls is SGDMReferenceSR else {}


@pytest.mark.parametrize("cls", [AdamWReferenceSR, SGDMReferenceSR])
def test_repeated_steps_take_the_fast_path_and_match_full_preparation(cls, fake_launcher):
    fast, a, full, b = _twins(cls, **_kwargs(cls))
    for _ in range(4):
        fast.step()
        _full_step(full)
        _same(fast, a, full, b)
    assert group_cache(fast, fast.param_groups[0]).fast is not None


@pytest.mark.parametrize("change", ["new_grad", "grad_none", "resize", "state_replaced",
                                    "param_data", "lr", "step_edit"])
@pytest.mark.parametrize("cls", [AdamWReferenceSR, SGDMReferenceSR])
def test_changes_are_noticed(cls, change, fake_launcher):
    if change == "step_edit" and cls is SGDMReferenceSR:
        pytest.skip("momentum SGD keeps no step")
    fast, a, full, b = _twins(cls, **_kwargs(cls))
    for opt in (fast, full):
        opt.step()
        opt.step()
    for opt, ps in ((fast, a), (full, b)):
        p = ps[1]
        if change == "new_grad":
            p.grad = p.grad.clone() * 2
        elif change == "grad_none":
            p.grad = None
        elif change == "resize":
            # Same gradient object and storage, fewer elements: the full
            # preparation rejects the shape mismatch, so the fast path must too.
            p.grad.resize_(2048)
        elif change == "state_replaced":
            opt.load_state_dict(opt.state_dict())
        elif change == "param_data":
            p.data = p.data.clone() + 1
        elif change == "lr":
            opt.param_groups[0]["lr"] = 0.02
        elif change == "step_edit":
            opt.state[p]["step"] = 7
    if change == "resize":
        calls = len(fake_launcher.calls)
        with pytest.raises(ValueError, match="identical shapes"):
            fast.step()
        with pytest.raises(ValueError, match="identical shapes"):
            _full_step(full)
        assert len(fake_launcher.calls) == calls
        return
    fast.step()
    _full_step(full)
    _same(fast, a, full, b)
    fast.step()
    _full_step(full)
    _same(fast, a, full, b)


def test_invalid_hyperparameters_still_raise_on_the_fast_path(fake_launcher):
    opt, a, _, _ = _twins(AdamWReferenceSR)
    opt.step()
    opt.step()
    opt.param_groups[0]["lr"] = -1.0
    calls = len(fake_launcher.calls)
    with pytest.raises(ValueError, match="invalid lr"):
        opt.step()
    assert len(fake_launcher.calls) == calls


def test_sparse_gradient_after_fast_steps_raises_the_reference_error(fake_launcher):
    p = torch.nn.Parameter(torch.ones(4))
    p.grad = torch.ones(4)
    opt = AdamWReferenceSR([p], lr=0.01)
    opt.step()
    opt.step()
    p.grad = torch.sparse_coo_tensor([[0]], [1.0], size=(4,))
    with pytest.raises(RuntimeError, match="sparse"):
        opt.step()


@pytest.mark.parametrize("change", ["grad_transposed_in_place", "param_dtype_view",
                                    "state_transposed_in_place", "param_reshaped"])
@pytest.mark.parametrize("cls", [AdamWReferenceSR, SGDMReferenceSR])
def test_in_place_layout_and_dtype_changes_are_noticed(cls, change, fake_launcher):
    """Changes that keep every object and address (in-place transposes, a dtype
    view of the same storage, a reshape) must still reach the full preparation:
    both twins raise the same error or take the same step."""
    fmt = ({"exp_avg": StateFormat(torch.bfloat16), "exp_avg_sq": StateFormat(torch.bfloat16)}
           if cls is AdamWReferenceSR else StateFormat(torch.bfloat16))
    twins = []
    for _ in range(2):
        gen = torch.Generator().manual_seed(3)
        ps = [torch.nn.Parameter(torch.randn(4, 4, generator=gen).bfloat16()),
              torch.nn.Parameter(torch.randn(7, generator=gen).bfloat16())]
        for p in ps:
            p.grad = (torch.randn(p.shape, generator=gen) * 1e-2).bfloat16()
        opt = cls(ps, lr=0.01, state_format=fmt, seed=5, **_kwargs(cls))
        opt.step()
        opt.step()
        twins.append((opt, ps))
    outcomes = []
    for i, (opt, ps) in enumerate(twins):
        p = ps[0]
        if change == "grad_transposed_in_place":
            p.grad.t_()
        elif change == "param_dtype_view":
            p.data = p.data.view(torch.float16)  # same bytes, another dtype
        elif change == "state_transposed_in_place":
            opt.state[p][opt._state_names[0]].t_()
        elif change == "param_reshaped":
            p.data = p.data.view(2, 8)
        try:
            opt.step() if i == 0 else _full_step(opt)
            outcomes.append(None)
        except (ValueError, TypeError, RuntimeError) as exc:
            outcomes.append((type(exc), str(exc)))
    assert outcomes[0] == outcomes[1]
    if change != "param_reshaped":
        assert outcomes[0] is not None  # the full preparation rejects these
    if outcomes[0] is None:
        _same(twins[0][0], twins[0][1], twins[1][0], twins[1][1])
