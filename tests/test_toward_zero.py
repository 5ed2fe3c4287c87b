"""The toward_zero device rule: the third entry of the kernels' rule table,
reachable through register_rounding(..., native="toward_zero").

It has no reference counterpart as a built-in; the reference runs custom rules
as Triton callbacks and its own tests register one such rule, "toward_zero"
for BF16 (tests/test_rounding_registry.py:15-17: clear the low 16 bits of the
FP32 encoding).  The oracle's rule is pinned here independently: for every
format, the result must be the representable value of largest magnitude not
above |x| (found by searching the format's sorted finite values), sign kept.
The kernels must then give the oracle's bytes (exact, no tolerance).
"""

import copy

import numpy as np
import pytest
import torch

import oracle
import sr_states.rounding as rounding_module
from _support import DTYPE, FMT, assert_bits_or_nan, isnan_bits, tbits
from sr_states import AdamWReferenceSR, SGDMReferenceSR, register_rounding
from sr_states.rounding import NATIVE_RULES, native_codes, native_reference

TZ = NATIVE_RULES.index("toward_zero")
FORMATS = [oracle.BF16, oracle.F16, oracle.E4M3, oracle.E5M2]


@pytest.fixture(autouse=True)
def isolated_registry(monkeypatch):
    monkeypatch.setattr(rounding_module, "_RULES", rounding_module._RULES.copy())


def reference_test_toward_zero(x, *, dtype, seed, offset):
    """The rule the reference's registry tests register (see module docstring)."""
    bits = x.contiguous().view(torch.int32) & -65536
    return bits.view(torch.float32).to(dtype)


def _inputs(n, seed):
    rng = np.random.default_rng(seed)
    raw = rng.integers(0, 2**32, n, dtype=np.uint64).astype(np.uint32)
    specials = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 448.0, 449.0, 464.0, 57344.0,
                         61440.0, 65504.0, 65519.0, 65520.0, 65535.99, 65536.0, 1e30,
                         np.finfo(np.float32).max, np.finfo(np.float32).tiny, 1e-45, 2.0**-9,
                         2.0**-10, 2.0**-17, 2.0**-16, 2.0**-24, 2.0**-25, 1.0, 1.0 - 2.0**-24],
                        dtype=np.float32)
    specials = np.concatenate((specials, -specials))
    mags = np.exp2(rng.uniform(-30, 20, n)).astype(np.float32) * rng.choice([-1, 1], n)
    return np.concatenate((specials, raw.view(np.float32), mags.astype(np.float32)))


def _finite_nonnegative(fmt):
    """(bits, values) of the format's finite non-negative encodings, ascending."""
    width = 16 if fmt in (oracle.BF16, oracle.F16) else 8
    bits = np.arange(1 << (width - 1), dtype=np.uint32)
    with np.errstate(invalid="ignore"):  # NaN encodings
        values = oracle.decode(bits.astype(oracle.BITS_DTYPE[fmt]), fmt).astype(np.float64)
    keep = np.isfinite(values)
    return bits[keep], values[keep]


@pytest.mark.parametrize("fmt", FORMATS)
def test_oracle_rule_is_the_largest_magnitude_not_above_x(fmt):
    x = _inputs(1 << 18, fmt)
    got = oracle.cast(x, fmt, TZ).astype(np.uint32)
    width = 16 if fmt in (oracle.BF16, oracle.F16) else 8
    sign = np.signbit(x).astype(np.uint32) << (width - 1)
    bits, values = _finite_nonnegative(fmt)
    assert np.all(np.diff(values) > 0)
    with np.errstate(invalid="ignore"):  # signalling NaN inputs
        a = np.abs(x.astype(np.float64))
    finite = np.isfinite(a)
    idx = np.searchsorted(values, np.where(finite, a, 0.0), side="right") - 1
    expected = bits[idx] | sign
    inf = np.isinf(a)
    if fmt in (oracle.BF16, oracle.F16):  # infinities stay infinite
        expected = np.where(inf, (0x7F80 if fmt == oracle.BF16 else 0x7C00) | sign, expected)
    else:  # FP8 saturates
        expected = np.where(inf, bits[-1] | sign, expected)
    nan = np.isnan(x)
    assert np.array_equal(got[~nan], expected[~nan])
    assert np.all(isnan_bits(got[nan].astype(oracle.BITS_DTYPE[fmt]), fmt))


def test_oracle_bf16_rule_equals_the_reference_tests_rule():
    x = _inputs(1 << 18, 3)
    expected = tbits(reference_test_toward_zero(torch.from_numpy(x), dtype=torch.bfloat16,
                                                seed=0, offset=0))
    got = oracle.cast(x, oracle.BF16, TZ)
    # Equal everywhere except NaNs whose payload sits only in the low 16 bits,
    # which the test's rule turns into infinities.
    u = x.view(np.uint32)
    low_payload_nan = np.isnan(x) & ((u & 0x007F0000) == 0)
    assert low_payload_nan.any()
    assert np.array_equal(got[~low_payload_nan], expected[~low_payload_nan])
    assert np.all(got[low_payload_nan] == 0xFFFF)


def test_native_rule_table_and_registration():
    assert NATIVE_RULES == ("nearest", "stochastic", "toward_zero")
    # toward_zero is not a built-in name: the reference's tests register it.
    register_rounding("toward_zero", torch.bfloat16, reference=reference_test_toward_zero,
                      native="toward_zero")
    assert native_codes(torch.bfloat16, "toward_zero") == (1, 2)
    register_rounding("rz", torch.float8_e5m2, reference=native_reference("toward_zero"),
                      native="toward_zero")
    assert native_codes(torch.float8_e5m2, "rz") == (4, 2)
    with pytest.raises(ValueError, match="native must be one of"):
        register_rounding("bad", torch.float16, reference=reference_test_toward_zero,
                          native="up")
    with pytest.raises(ValueError, match="rule must be one of"):
        native_reference("up")
    x = torch.tensor([1.5, -2.25])
    assert native_reference("toward_zero")(x, dtype=torch.float32, seed=0, offset=0).equal(x)


def _state_only_and_resume(cls, device):
    """The reference's test_custom_rounding_changes_state_only_and_resumes
    (tests/test_rounding_registry.py:52-71) on the fused path: one step with
    toward-zero BF16 states leaves the parameters of an FP32-state run and
    stores toward_zero(FP32 states); a restored copy then steps identically."""
    register_rounding("toward_zero", torch.bfloat16, reference=reference_test_toward_zero,
                      native="toward_zero")
    p = torch.nn.Parameter(torch.ones(17, device=device))
    q = torch.nn.Parameter(p.detach().clone())
    custom = cls([p], lr=0.01, rounding="toward_zero")
    baseline = cls([q], lr=0.01, state_dtype=torch.float32)
    p.grad = torch.linspace(-1.987, 1.987, 17, device=device)
    q.grad = p.grad.clone()
    custom.step()
    baseline.step()
    assert torch.equal(p, q)
    for name in custom._state_names:
        expected = reference_test_toward_zero(baseline.state[q][name].cpu(),
                                              dtype=torch.bfloat16, seed=0, offset=0)
        assert torch.equal(custom.state[p][name].cpu(), expected), name
    restored_p = torch.nn.Parameter(p.detach().clone())
    restored = cls([restored_p], lr=0.7)
    checkpoint = copy.deepcopy(custom.state_dict())
    assert (checkpoint["param_groups"][0]["state_format"][custom._state_names[0]]["rounding"]
            == "toward_zero")
    restored.load_state_dict(checkpoint)
    for step in range(3):
        p.grad = torch.sin(torch.arange(17, device=device, dtype=torch.float32) + step)
        restored_p.grad = p.grad.clone()
        custom.step()
        restored.step()
        assert torch.equal(p, restored_p)
        for name in custom._state_names:
            assert torch.equal(custom.state[p][name], restored.state[restored_p][name])


@pytest.mark.parametrize("cls", [SGDMReferenceSR, AdamWReferenceSR])
def test_custom_rule_changes_state_only_and_resumes_host(cls, fake_launcher):
    _state_only_and_resume(cls, "cpu")
    launches = [call for call in fake_launcher.calls if call[0].endswith("_multi")]
    assert any(call[4] == TZ and call[-1] == TZ for call in launches)  # the custom run


# ---------------------------------------------------------------- GPU parity --

@pytest.mark.gpu
@pytest.mark.parametrize("cls", [SGDMReferenceSR, AdamWReferenceSR])
def test_custom_rule_changes_state_only_and_resumes(cls, cuda_device):
    _state_only_and_resume(cls, cuda_device)


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", FORMATS)
def test_cast_kernel_matches_oracle(fmt, cuda_device):
    from sr_states.cuda import _native

    x = torch.from_numpy(_inputs((1 << 21) + 5, 11 + fmt))
    dtype = DTYPE[fmt]
    register_rounding("tz", dtype, reference=native_reference("toward_zero"),
                      native="toward_zero")
    expected = oracle.cast(x.numpy(), fmt, TZ, threads=8)
    for start in (0, 1):  # aligned vector path, unaligned scalar path
        xs = x[start:].to(cuda_device)
        y = torch.empty(xs.shape, dtype=dtype, device=cuda_device)
        _native.launcher().cast(xs.data_ptr(), y.data_ptr(), xs.numel(), fmt, TZ, 0, 0,
                                torch.cuda.current_stream(cuda_device).cuda_stream)
        assert_bits_or_nan(tbits(y), expected[start:], fmt, f"start {start}")
        public = rounding_module.cast(xs, dtype=dtype, rounding="tz", seed=5, offset=9)
        assert_bits_or_nan(tbits(public), expected[start:], fmt, f"public, start {start}")


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", FORMATS)
def test_cast_kernel_fp32_encoding_sweep(fmt, cuda_device):
    """Every FP32 encoding in 1/32 of the 2^32 space (2^20-element chunks spread
    evenly over it) against the oracle."""
    from sr_states.cuda import _native

    chunk = 1 << 20
    for c in range(0, 4096, 32):
        first = c * chunk
        bits = torch.arange(first, first + chunk, dtype=torch.int64, device=cuda_device)
        x = bits.to(torch.int32).view(torch.float32)
        y = torch.empty(chunk, dtype=DTYPE[fmt], device=cuda_device)
        _native.launcher().cast(x.data_ptr(), y.data_ptr(), chunk, fmt, TZ, 0, 0,
                                torch.cuda.current_stream(cuda_device).cuda_stream)
        expected = oracle.cast_bits_range(first, chunk, fmt, TZ, threads=8)
        assert_bits_or_nan(tbits(y), expected, fmt, f"chunk {c}")


def _host(t):
    return t.numpy().copy() if t.dtype == torch.float32 else tbits(t).copy()


@pytest.mark.gpu
@pytest.mark.parametrize("m_fmt,v_fmt", [(oracle.BF16, oracle.BF16), (oracle.E4M3, oracle.F16),
                                         (oracle.E5M2, oracle.BF16)])
@pytest.mark.parametrize("mixed", [False, True], ids=["tz-both", "tz-m-sr-v"])
def test_adamw_states_toward_zero_match_oracle(m_fmt, v_fmt, mixed, cuda_device):
    """Multi-tensor AdamW with toward-zero state rules against the oracle,
    bit-exact for parameters and states.  Such launches skip the screened
    arithmetic: every vector takes the per-element IEEE path."""
    from sr_states import StateFormat
    from sr_states._hash import update_key

    register_rounding("tz_m", DTYPE[m_fmt], reference=native_reference("toward_zero"),
                      native="toward_zero")
    if not mixed:
        register_rounding("tz_v", DTYPE[v_fmt], reference=native_reference("toward_zero"),
                          native="toward_zero")
    fmt = {"exp_avg": StateFormat(DTYPE[m_fmt], "tz_m"),
           "exp_avg_sq": StateFormat(DTYPE[v_fmt], "stochastic" if mixed else "tz_v")}
    m_rule, v_rule = TZ, (oracle.STOCHASTIC if mixed else TZ)
    gen = torch.Generator().manual_seed(m_fmt * 10 + v_fmt)
    rows = []
    for n, pdt in ((300_007, torch.bfloat16), (4099, torch.float32), (1, torch.bfloat16)):
        p = torch.randn(n, generator=gen).to(pdt)
        g = (torch.randn(n, generator=gen) * 1e-2).to(pdt)
        m = (torch.randn(n, generator=gen) * 1e-2).to(DTYPE[m_fmt])
        v = (torch.rand(n, generator=gen) * 1e-4).to(DTYPE[v_fmt])
        rows.append((p, g, m, v))
    dev = [tuple(t.to(cuda_device) for t in row) for row in rows]
    params = [torch.nn.Parameter(p) for p, _, _, _ in dev]
    seed, rng0 = 21, 7
    opt = AdamWReferenceSR(params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01,
                           state_format=fmt, seed=seed)
    opt.param_groups[0]["sr_step"] = rng0
    for param, (_, g, m, v) in zip(params, dev):
        param.grad = g
        opt.state[param]["exp_avg"], opt.state[param]["exp_avg_sq"] = m, v
        opt.state[param]["step"] = 3
    opt.step()
    for i, ((p, g, m, v), param) in enumerate(zip(rows, params)):
        pn, gn, mn, vn = _host(p), _host(g), tbits(m).copy(), tbits(v).copy()
        oracle.adamw_(pn, gn, mn, vn, m_fmt=m_fmt, m_rule=m_rule, v_fmt=v_fmt, v_rule=v_rule,
                      lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.01, step=4,
                      update_key=update_key(seed, rng0 + 1, i), threads=8)
        assert np.array_equal(tbits(param), pn.view(tbits(param).dtype)), f"param row {i}"
        assert_bits_or_nan(tbits(opt.state[param]["exp_avg"]), mn, m_fmt, f"m row {i}")
        assert_bits_or_nan(tbits(opt.state[param]["exp_avg_sq"]), vn, v_fmt, f"v row {i}")


@pytest.mark.gpu
@pytest.mark.parametrize("u_fmt", FORMATS)
def test_sgdm_state_toward_zero_matches_oracle(u_fmt, cuda_device):
    from sr_states import StateFormat
    from sr_states._hash import update_key

    register_rounding("tz_u", DTYPE[u_fmt], reference=native_reference("toward_zero"),
                      native="toward_zero")
    gen = torch.Generator().manual_seed(u_fmt)
    rows = []
    for n, pdt in ((200_003, torch.float32), (2049, torch.bfloat16)):
        rows.append((torch.randn(n, generator=gen).to(pdt), torch.randn(n, generator=gen).to(pdt),
                     torch.randn(n, generator=gen).to(DTYPE[u_fmt])))
    dev = [tuple(t.to(cuda_device) for t in row) for row in rows]
    params = [torch.nn.Parameter(p) for p, _, _ in dev]
    opt = SGDMReferenceSR(params, lr=0.1, momentum=0.9,
                          state_format=StateFormat(DTYPE[u_fmt], "tz_u"), seed=5)
    for param, (_, g, u) in zip(params, dev):
        param.grad = g
        opt.state[param]["momentum_buffer"] = u
    opt.step()
    for i, ((p, g, u), param) in enumerate(zip(rows, params)):
        pn, gn, un = _host(p), _host(g), tbits(u).copy()
        oracle.sgdm_(pn, gn, un, u_fmt=u_fmt, u_rule=TZ, lr=0.1, momentum=0.9,
                     update_key=update_key(5, 1, i), threads=8)
        assert np.array_equal(tbits(param), pn.view(tbits(param).dtype)), f"param row {i}"
        assert_bits_or_nan(tbits(opt.state[param]["momentum_buffer"]), un, u_fmt, f"u row {i}")
