"""sm_100a fused optimizer steps vs the reference's golden bytes and the CPU oracle.

Against the oracle (same operation order, correctly rounded sqrt on both sides)
every byte must match, parameters included.  Against the reference's bytes the
states must match exactly, and AdamW parameters must equal the reference's own
update formula evaluated with a correctly rounded square root
(_support.explain_adamw_param, from the reference's recorded intermediates): the
reference's CPU sqrt is not correctly rounded, and that is the only difference.
"""

import hashlib

import numpy as np
import pytest
import torch

import _scenarios
import oracle
from _support import (DTYPE, FMT, assert_bits_or_nan, explain_adamw_param, from_bits, load_json,
                      load_npz, tbits, ulp_distance)

pytestmark = pytest.mark.gpu

FORMATS = [torch.float32, torch.bfloat16, torch.float16, torch.float8_e4m3fn, torch.float8_e5m2]


@pytest.mark.parametrize("spec", _scenarios.scenarios(), ids=lambda s: s["name"])
def test_reference_scenarios_on_gpu(spec, cuda_device):
    compared, mismatched = _scenarios.replay(spec, cuda_device)
    assert compared > 0
    if spec["kind"] == "sgdm":
        assert mismatched == 0


@pytest.mark.parametrize("case", load_json("functional.json")["cases"], ids=lambda c: c["name"])
def test_functional_steps_match_reference(case, cuda_device):
    from sr_states.cuda import cuda_adamw_step_, cuda_sgdm_step_

    arrays = load_npz("functional.npz")
    g = from_bits(arrays["grad"], torch.float32, cuda_device)
    p = torch.linspace(-1, 1, g.numel()).to(cuda_device)
    dtype, name = DTYPE[case["format"]], case["name"]
    rounding = ["nearest", "stochastic"][case["rule"]]
    if case["kind"] == "adamw":
        states = [torch.zeros_like(g, dtype=dtype) for _ in range(2)]
        cuda_adamw_step_(p, g, *states, lr=0.01, beta1=0.5, beta2=0.5, eps=0.125,
                         weight_decay=0.0, step=1, seed=case["key"], offset=case["offset"],
                         rounding=rounding)
    else:
        states = [torch.zeros_like(g, dtype=dtype)]
        cuda_sgdm_step_(p, g, *states, lr=0.01, momentum_factor=0.5, seed=case["key"],
                        offset=case["offset"], rounding=rounding)
    assert np.array_equal(tbits(p), arrays[f"{name}__param"])  # dyadic inputs: exact
    for i, s in enumerate(states):
        assert_bits_or_nan(tbits(s), arrays[f"{name}__state{i}"], case["format"])


def test_config1_matches_reference_every_step(cuda_device):
    """BASELINE config 1 (n = 2^13 golden, 10 steps, teacher-forced): states exact;
    the FP32 parameter byte-exact wherever the reference's CPU sqrt is correctly
    rounded, and everywhere equal to the reference's formula with the correctly
    rounded root (so every difference is that root's)."""
    import oracle
    from sr_states import AdamWReferenceSR

    a = load_npz("config1.npz")
    inter = load_npz("config1_intermediates.npz")
    p = torch.nn.Parameter(from_bits(a["param_init"], torch.float32, cuda_device))
    opt = AdamWReferenceSR([p], lr=3e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01,
                           seed=7)
    roots, params, worst = 0, 0, 0
    for step in range(1, 11):
        previous = tbits(p).view(np.float32).copy()
        p.grad = from_bits(a[f"grad_{step}"], torch.float32, cuda_device)
        opt.step()
        assert np.array_equal(tbits(opt.state[p]["exp_avg"]), a[f"exp_avg_{step}"])
        assert np.array_equal(tbits(opt.state[p]["exp_avg_sq"]), a[f"exp_avg_sq_{step}"])
        scalars = oracle.adamw_scalars(3e-4, 0.9, 0.999, 1e-8, 0.01, step)
        r, d, w = explain_adamw_param(
            tbits(p), a[f"param_{step}"], previous,
            *(inter[f"{k}_{step}"].view(np.float32) for k in ("v32", "sqrt", "m32")),
            scalars, 32)
        roots, params, worst = roots + r, params + d, max(worst, w)
        with torch.no_grad():
            p.copy_(from_bits(a[f"param_{step}"], torch.float32, cuda_device))
    rate = params / (10 * p.numel())
    print(f"config 1 parameters vs the reference: {roots} roots of its CPU sqrt are not "
          f"correctly rounded; {params} parameters differ (rate {rate:.2e}, max {worst} ulp), "
          "each explained by its root")


def test_config1_full_size_state_digests(cuda_device):
    """BASELINE config 1 at 2^20 elements, 10 untouched steps: state SHA-256s equal the
    reference's (states do not depend on the parameter)."""
    from sr_states import AdamWReferenceSR

    spec = load_json("config1_full.json")
    gen = torch.Generator().manual_seed(spec["seed_generator"])
    p = torch.nn.Parameter((torch.randn(spec["n"], generator=gen) * 0.02).to(cuda_device))
    opt = AdamWReferenceSR([p], lr=3e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01,
                           seed=7)
    for entry in spec["steps"]:
        p.grad = (torch.randn(spec["n"], generator=gen) * 1e-3).to(cuda_device)
        opt.step()
        st = opt.state[p]
        assert hashlib.sha256(tbits(st["exp_avg"]).tobytes()).hexdigest() == entry["exp_avg_sha256"]
        assert (hashlib.sha256(tbits(st["exp_avg_sq"]).tobytes()).hexdigest()
                == entry["exp_avg_sq_sha256"])


# ------------------------------------------------------- oracle parity --

SIZES = [1, 7, 8, 9, 2047, 2048, 2049, 3 * 2048 + 5, 40_001]


class _MixedGradParameter(torch.nn.Parameter):
    """Parameter whose gradient may have another dtype (PyTorch forbids that on
    .grad; the fused step supports FP32/BF16 in any combination)."""

    @property
    def grad(self):
        return getattr(self, "_mixed_grad", None)

    @grad.setter
    def grad(self, value):
        self._mixed_grad = value


def _make_rows(device, pdtypes, gen, state_dtypes, n_states, unaligned=True):
    """Rows of every size class; every third row is a view starting one element into
    its allocation, so its addresses are unaligned and it takes the scalar path."""
    host, dev = [], []
    for i, n in enumerate(SIZES):
        pd, gd = pdtypes[i % len(pdtypes)]
        start = 1 if (unaligned and i % 3 == 2) else 0
        full = [(torch.randn(n + start, generator=gen) * 0.5).to(pd),
                (torch.randn(n + start, generator=gen) * 0.1).to(gd)]
        for k in range(n_states):
            s = torch.randn(n + start, generator=gen) * (0.01 if k == 0 else 1e-3)
            full.append((s.abs() if k == 1 else s).to(state_dtypes[k]))
        on_device = [t.to(device)[start:] for t in full]
        host.append((full[0][start:].clone(), full[1][start:].clone(),
                     [t[start:].clone() for t in full[2:]]))
        dev.append((_MixedGradParameter(on_device[0]), on_device[1], on_device[2:]))
    return host, dev


def _np(t):
    return t.numpy() if t.dtype == torch.float32 else tbits(t).copy()


@pytest.mark.parametrize("m_dtype", FORMATS, ids=str)
@pytest.mark.parametrize("v_dtype", FORMATS, ids=str)
def test_adamw_multi_tensor_matches_oracle_bit_exact(m_dtype, v_dtype, cuda_device):
    from sr_states import AdamWReferenceSR, StateFormat
    from sr_states._hash import update_key

    gen = torch.Generator().manual_seed(FMT[m_dtype] * 5 + FMT[v_dtype])
    pdt = [(torch.float32, torch.float32), (torch.bfloat16, torch.bfloat16),
           (torch.float32, torch.bfloat16), (torch.bfloat16, torch.float32)]
    host, dev = _make_rows(cuda_device, pdt, gen, (m_dtype, v_dtype), 2)
    rules = ("stochastic", "nearest") if FMT[m_dtype] % 2 else ("nearest", "stochastic")
    fmt = {"exp_avg": StateFormat(m_dtype, rules[0]), "exp_avg_sq": StateFormat(v_dtype, rules[1])}
    params = [p for p, _, _ in dev]
    seed, rng0 = 2**64 - 3, 2**32 - 1
    opt = AdamWReferenceSR(params, lr=1e-3, betas=(0.8, 0.99), eps=1e-6, weight_decay=0.1,
                           state_format=fmt, seed=seed)
    opt.param_groups[0]["sr_step"] = rng0
    for i, (p, g, st) in enumerate(dev):
        p.grad = g
        opt.state[p]["exp_avg"], opt.state[p]["exp_avg_sq"] = st
        opt.state[p]["step"] = 3 + (i % 2)  # two bias-correction step classes
    opt.step()
    for i, (p, g, (m, v)) in enumerate(host):
        pn, gn, mn, vn = _np(p), _np(g), tbits(m).copy(), tbits(v).copy()
        oracle.adamw_(pn, gn, mn, vn, m_fmt=FMT[m_dtype], m_rule=["nearest", "stochastic"].index(rules[0]),
                      v_fmt=FMT[v_dtype], v_rule=["nearest", "stochastic"].index(rules[1]),
                      lr=1e-3, beta1=0.8, beta2=0.99, eps=1e-6, weight_decay=0.1,
                      step=4 + (i % 2), update_key=update_key(seed, rng0 + 1, i), offset=0)
        dp = dev[i][0]
        assert np.array_equal(tbits(dp), pn.view(tbits(dp).dtype)), f"param row {i}"
        assert_bits_or_nan(tbits(opt.state[dp]["exp_avg"]), mn, FMT[m_dtype], f"m row {i}")
        assert_bits_or_nan(tbits(opt.state[dp]["exp_avg_sq"]), vn, FMT[v_dtype], f"v row {i}")


@pytest.mark.parametrize("u_dtype", FORMATS, ids=str)
@pytest.mark.parametrize("rule", ["nearest", "stochastic"])
def test_sgdm_multi_tensor_matches_oracle_bit_exact(u_dtype, rule, cuda_device):
    from sr_states import SGDMReferenceSR, StateFormat
    from sr_states._hash import update_key

    gen = torch.Generator().manual_seed(40 + FMT[u_dtype])
    pdt = [(torch.float32, torch.float32), (torch.bfloat16, torch.bfloat16)]
    host, dev = _make_rows(cuda_device, pdt, gen, (u_dtype,), 1)
    opt = SGDMReferenceSR([p for p, _, _ in dev], lr=0.05, momentum=0.9,
                          state_format=StateFormat(u_dtype, rule), seed=11)
    for p, g, (u,) in dev:
        p.grad = g
        opt.state[p]["momentum_buffer"] = u
    opt.step()
    for i, (p, g, (u,)) in enumerate(host):
        pn, gn, un = _np(p), _np(g), tbits(u).copy()
        oracle.sgdm_(pn, gn, un, u_fmt=FMT[u_dtype], u_rule=["nearest", "stochastic"].index(rule),
                     lr=0.05, momentum=0.9, update_key=update_key(11, 1, i), offset=0)
        dp = dev[i][0]
        assert np.array_equal(tbits(dp), pn.view(tbits(dp).dtype)), f"param row {i}"
        assert_bits_or_nan(tbits(opt.state[dp]["momentum_buffer"]), un, FMT[u_dtype])


def test_sharded_launches_equal_one_launch_and_grid_size_is_irrelevant(cuda_device, monkeypatch):
    """Shard invariance of the RNG contract: the same parameter updated as 1 row or
    as 5 flat shards (offset = shard start) gives identical bytes; so do grids of
    any size."""
    from sr_states.cuda import _native, cuda_adamw_step_

    gen = torch.Generator().manual_seed(3)
    n = 5 * 2048 * 7 + 333
    base = [(torch.randn(n, generator=gen) * 0.1).to(torch.bfloat16),
            (torch.randn(n, generator=gen) * 1e-2).to(torch.bfloat16),
            (torch.randn(n, generator=gen) * 1e-2).to(torch.float8_e4m3fn),
            (torch.rand(n, generator=gen) * 1e-4).to(torch.bfloat16)]
    options = dict(lr=3e-4, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.1, step=7,
                   seed=0xABCDEF, offset=2**32 - 1000)
    whole = [t.to(cuda_device) for t in base]
    cuda_adamw_step_(*whole, **options)
    shards = [t.to(cuda_device) for t in base]
    cuts = [0, 11, 2048 * 3, 2048 * 3 + 8, n // 2, n]
    for lo, hi in zip(cuts[:-1], cuts[1:]):
        cuda_adamw_step_(*(t[lo:hi] for t in shards),
                         **{**options, "offset": options["offset"] + lo})
    for a, b in zip(whole, shards):
        assert torch.equal(a.view(torch.uint8), b.view(torch.uint8))
    for grid in (1, 5, 1000):
        monkeypatch.setattr(_native.NativeLauncher, "adamw_single",
                            _with_grid(_native.NativeLauncher.adamw_single, grid))
        again = [t.to(cuda_device) for t in base]
        cuda_adamw_step_(*again, **options)
        for a, b in zip(whole, again):
            assert torch.equal(a.view(torch.uint8), b.view(torch.uint8))
        monkeypatch.undo()


def _with_grid(method, grid):
    def call(self, *args, **kwargs):
        kwargs["grid_ctas"] = grid
        return method(self, *args, **kwargs)

    return call


def test_step_on_a_side_stream(cuda_device):
    from sr_states import SGDMReferenceSR

    p, q = (torch.nn.Parameter(torch.linspace(-1, 1, 4099, device=cuda_device)) for _ in range(2))
    p.grad = q.grad = torch.cos(torch.arange(4099.0, device=cuda_device))
    a, b = SGDMReferenceSR([p], lr=0.01, seed=5), SGDMReferenceSR([q], lr=0.01, seed=5)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    for _ in range(3):
        with torch.cuda.stream(side):
            a.step()
        b.step()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    assert torch.equal(p, q)
    assert torch.equal(a.state[p]["momentum_buffer"], b.state[q]["momentum_buffer"])


@pytest.mark.parametrize("seed,step", [(1, 16), (-1, 2**32 + 1), (2**87 + 7, 2**64 + 2**63 + 16),
                                       (-(2**48) + 15, 2**32 - 1)])
def test_device_keys_match_host(seed, step, cuda_device):
    from sr_states._hash import state_key, update_key
    from sr_states.cuda import _native
    from sr_states.cuda._fused import rng_words

    index = torch.tensor([0, 1, 2**31 + 1, 2**32 - 1], dtype=torch.int64).to(torch.int32)
    index = index.to(cuda_device)
    out = torch.empty(3 * index.numel(), dtype=torch.int32, device=cuda_device)
    _native.launcher().derive_keys(index.data_ptr(), out.data_ptr(), index.numel(),
                                   rng_words(seed, step), torch.cuda.current_stream().cuda_stream)
    got = tbits(out).reshape(-1, 3).tolist()
    for i, idx in enumerate([0, 1, 2**31 + 1, 2**32 - 1]):
        k = update_key(seed, step, idx)
        assert got[i] == [k, state_key(k, 0), state_key(k, 1)]


@pytest.mark.parametrize("beta2,step", [(0.999, 1), (0.999, 1000), (0.95, 3), (0.0, 1),
                                        (1 - 2.0**-40, 2)])
def test_adamw_denominator_over_every_exponent_matches_oracle(beta2, step, cuda_device):
    """v' spans every FP32 exponent (plus 0, Inf, NaN), so sqrt(v')/sqrt(bc2) takes
    both the reciprocal-division path and the IEEE fallback; bit-exact vs the oracle."""
    from sr_states.cuda import cuda_adamw_step_

    exps = torch.arange(-149, 128, dtype=torch.float64)
    mant = torch.linspace(1.0, 1.999, 37, dtype=torch.float64)
    v = (torch.exp2(exps)[:, None] * mant[None, :]).reshape(-1).float()
    v = torch.cat((v, torch.tensor([0.0, float("inf"), float("nan"), 3.4e38])))
    n = v.numel()
    gen = torch.Generator().manual_seed(int(step))
    g = torch.randn(n, generator=gen) * torch.exp2(torch.randint(-60, 60, (n,), generator=gen))
    g[::5] = 0.0
    m = torch.randn(n, generator=gen)
    p = torch.randn(n, generator=gen)
    opts = dict(lr=1e-3, beta1=0.9, beta2=beta2, eps=1e-8, weight_decay=0.01, step=step)
    host = [t.numpy().copy() for t in (p, g, m, v)]
    oracle.adamw_(host[0], host[1], host[2].view(np.uint32), host[3].view(np.uint32),
                  m_fmt=oracle.F32, m_rule=0, v_fmt=oracle.F32, v_rule=0, update_key=9,
                  offset=0, **opts)
    dev = [t.to(cuda_device) for t in (p, g, m, v)]
    cuda_adamw_step_(*dev, seed=9, rounding="nearest", **opts)
    for got, want in zip(dev, host):
        assert_bits_or_nan(tbits(got), want.view(np.uint32), oracle.F32)


@pytest.mark.parametrize("case", _scenarios.regression_cases(), ids=lambda c: c["key"])
def test_regression_scenario_matches_reference(case, cuda_device):
    """The reference's own optimizer regression scenario on the sm_100a kernels:
    every byte after seven steps equals the reference's, AdamW FP32 parameters
    included (the scenario's square roots are all correctly rounded on the CPU)."""
    assert _scenarios.replay_regression(case, cuda_device) == []
