"""Properties the reference's own tests assert, checked on the sm_100a kernels.

Each test names the reference test it mirrors (path:line inside the reference
project).  The bit-exact oracle comparisons elsewhere already imply these;
here they are stated directly, on the kernel path, with the reference's
tolerances: statistical bounds of 6 standard errors, the two-neighbour rule,
exact values and specials, seed/offset periodicity, FP32-state optimizers
against torch.optim (rtol 1e-5, atol 1e-6), and the FP8 subnormal tie.
"""

import math

import numpy as np
import pytest
import torch

import oracle
from _support import DTYPE, tbits

pytestmark = pytest.mark.gpu

GRIDS = [(oracle.BF16, 2.0**-7), (oracle.F16, 2.0**-10), (oracle.E4M3, 2.0**-3),
         (oracle.E5M2, 2.0**-2)]  # format, ulp of [1, 2)


def _cast(x, fmt, seed, offset=0, rounding="stochastic"):
    import sr_states

    return sr_states.cast(x, dtype=DTYPE[fmt], rounding=rounding, seed=seed, offset=offset)


def _neighbours(x, fmt):
    """(lower, upper) values of the format around |x| (sign applied), as float64."""
    width = 16 if fmt in (oracle.BF16, oracle.F16) else 8
    bits = np.arange(1 << (width - 1), dtype=np.uint32)
    with np.errstate(invalid="ignore"):
        values = oracle.decode(bits.astype(oracle.BITS_DTYPE[fmt]), fmt).astype(np.float64)
    values = np.sort(values[np.isfinite(values)])
    a = np.abs(x.astype(np.float64))
    i = np.searchsorted(values, a, side="right") - 1
    lower = values[i]
    upper = np.where(values[i] == a, values[i], values[np.minimum(i + 1, values.size - 1)])
    sign = np.where(np.signbit(x), -1.0, 1.0)
    return sign * lower, sign * upper


@pytest.mark.parametrize("fmt,ulp", GRIDS)
def test_empirical_up_probability_and_mean(fmt, ulp, cuda_device):
    """tests/test_sr_statistics.py:10-26 (BF16 there; every grid here)."""
    n, p_up = 200_000, 0.25
    x_value = 1.0 + p_up * ulp
    x = torch.full((n,), x_value, dtype=torch.float32, device=cuda_device)
    out = _cast(x, fmt, seed=2026).float()
    probability = (out > 1.0).float().mean().item()
    se = math.sqrt(p_up * (1 - p_up) / n)
    assert abs(probability - p_up) < 6 * se
    assert abs(out.mean().item() - x_value) < 6 * se * ulp


@pytest.mark.parametrize("fmt,lo,hi", [(oracle.BF16, -20, 21), (oracle.F16, -12, 15),
                                       (oracle.E4M3, -4, 8), (oracle.E5M2, -12, 15)])
def test_distribution_stress_is_unbiased_in_aggregate(fmt, lo, hi, cuda_device):
    """tests/test_sr_statistics.py:28-36, over each format's normal range."""
    base = torch.pow(2.0, torch.arange(lo, hi, dtype=torch.float32))
    inputs = (base[:, None] * (1.0 + torch.linspace(0.01, 0.99, 1024)[None, :])).flatten()
    reps = 64 if fmt in (oracle.E4M3, oracle.E5M2) else 1  # coarse grids: more samples
    x = inputs.repeat(reps).to(cuda_device)
    rounded = _cast(x, fmt, seed=91).float()
    error = ((rounded - x) / x.abs()).mean().abs().item()
    assert error < (1e-4 if reps == 1 else 1e-3)


@pytest.mark.parametrize("fmt", [f for f, _ in GRIDS])
def test_output_is_one_of_the_two_neighbours(fmt, cuda_device):
    """tests/test_sr_edge_cases.py:9-14, 31-54 (random values, the smallest FP32
    subnormal, the FP32 subnormal grid and BF16 midpoint boundaries)."""
    gen = torch.Generator().manual_seed(123)
    scale = 100.0 if fmt in (oracle.BF16, oracle.F16) else 10.0
    x = torch.randn(20_000, generator=gen) * scale
    boundary = torch.tensor([0x00000001, 0x00008000, 0x0000FFFF, 0x00010000, 0x3F807FFF,
                             0x3F808000, 0x3F808001], dtype=torch.int32).view(torch.float32)
    x = torch.cat((x, boundary, -boundary))
    out = _cast(x.to(cuda_device), fmt, seed=7).float().cpu().numpy().astype(np.float64)
    lower, upper = _neighbours(x.numpy(), fmt)
    assert np.all((out == lower) | (out == upper))


@pytest.mark.parametrize("fmt", [f for f, _ in GRIDS])
def test_exact_and_exceptional_values_are_preserved(fmt, cuda_device):
    """tests/test_sr_edge_cases.py:17-28: exact values and signed zero stay, NaN
    (also with its payload only in the discarded bits) stays NaN, infinities
    stay (BF16/FP16) or saturate (FP8)."""
    values = torch.tensor([0.0, -0.0, 1.5, -2.0, math.inf, -math.inf, math.nan])
    low_nan = torch.tensor([0x7F800001, 0x7F800100], dtype=torch.int32).view(torch.float32)
    out = _cast(torch.cat((values, low_nan)).to(cuda_device), fmt, seed=999).cpu()
    expected = values[:4].to(DTYPE[fmt])
    assert torch.equal(out[:4], expected) and torch.signbit(out[1].float())
    top = out[4:6].float()
    if fmt in (oracle.BF16, oracle.F16):
        assert torch.equal(top, torch.tensor([math.inf, -math.inf]))
    else:
        biggest = torch.finfo(DTYPE[fmt]).max
        assert torch.equal(top, torch.tensor([biggest, -biggest]))
    assert torch.isnan(out[6:].float()).all()


def test_seed_offset_reproducibility_partitioning_and_periodicity(cuda_device):
    """tests/test_seed_reproducibility.py:6-36."""
    x = torch.linspace(-10, 10, 10_003, device=cuda_device)
    first = _cast(x, oracle.BF16, seed=1234, offset=77)
    assert torch.equal(first, _cast(x, oracle.BF16, seed=1234, offset=77))
    whole = _cast(x, oracle.BF16, seed=99, offset=1000)
    split = 4096
    parts = torch.cat((_cast(x[:split], oracle.BF16, seed=99, offset=1000),
                       _cast(x[split:], oracle.BF16, seed=99, offset=1000 + split)))
    assert torch.equal(whole, parts)
    y = torch.full((4096,), 1.0 + 2.0**-9, device=cuda_device)
    assert not torch.equal(_cast(y, oracle.BF16, seed=1), _cast(y, oracle.BF16, seed=2))
    z = torch.linspace(-1, 1, 1003, device=cuda_device)
    expected = _cast(z, oracle.BF16, seed=7, offset=31)
    for periods in (-(2**60), -1, 1, 2**60):
        actual = _cast(z, oracle.BF16, seed=7 + periods * 2**32, offset=31 + periods * 2**32)
        assert torch.equal(actual, expected)


@pytest.mark.parametrize("kind", ["sgdm", "adamw"])
def test_fp32_state_optimizer_matches_pytorch(kind, cuda_device):
    """tests/test_triton_states.py:237-259: FP32 states against torch.optim."""
    from sr_states.triton import AdamWTriton, SGDMTriton

    p = torch.nn.Parameter(torch.linspace(-1, 1, 1003, device=cuda_device))
    q = torch.nn.Parameter(p.detach().clone())
    if kind == "adamw":
        options = {"lr": 0.01, "betas": (0.8, 0.95), "eps": 1e-6, "weight_decay": 0.1}
        optimizer = AdamWTriton([p], state_dtype=torch.float32, **options)
        native = torch.optim.AdamW([q], foreach=False, **options)
    else:
        options = {"lr": 0.01, "momentum": 0.8}
        optimizer = SGDMTriton([p], state_dtype=torch.float32, **options)
        native = torch.optim.SGD([q], foreach=False, **options)
    for step in range(1, 21):
        p.grad = torch.sin(torch.arange(1003, device=cuda_device) * 0.001 + step)
        q.grad = p.grad.clone()
        optimizer.step()
        native.step()
        torch.testing.assert_close(p, q, rtol=1e-5, atol=1e-6)
        for name in optimizer._state_names:
            torch.testing.assert_close(optimizer.state[p][name], native.state[q][name],
                                       rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("betas", [(0.0, 0.0), (0.9, 0.999)])
def test_adamw_zero_gradient_only_decays(betas, cuda_device):
    """tests/test_triton_states.py:262-285."""
    from sr_states.triton import triton_adamw_step_

    p = torch.linspace(-1, 1, 1003, device=cuda_device)
    expected = p * (1.0 - 0.01 * 0.1)
    g = torch.zeros_like(p)
    m = torch.zeros_like(p, dtype=torch.bfloat16)
    v = torch.zeros_like(m)
    triton_adamw_step_(p, g, m, v, lr=0.01, beta1=betas[0], beta2=betas[1], eps=1e-8,
                       weight_decay=0.1, step=1, seed=7)
    torch.testing.assert_close(p, expected, rtol=0, atol=0)
    assert torch.count_nonzero(m) == 0 and torch.count_nonzero(v) == 0


@pytest.mark.parametrize("parameter_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("n", [1, 1003])
def test_fp8_sgdm_subnormal_tie_uses_separate_multiply_and_add(parameter_dtype, n,
                                                               cuda_device):
    """tests/test_triton_states.py:85-116: u' = u*0.9 + g lands exactly on the
    E4M3 subnormal tie 5.5/512 when the multiply and add round separately (as
    in the reference's CPU order), and the nearest rule stores the even 6/512.
    An FMA would give 5.49999.../512 and store 5/512."""
    from sr_states import StateFormat
    from sr_states.triton import triton_sgdm_step_

    signs = (1 - 2 * (torch.arange(n, device=cuda_device) % 2)).float()
    p = torch.ones(n, device=cuda_device, dtype=parameter_dtype)
    g = (-signs * (8 / 512)).to(parameter_dtype)
    u = (signs * (15 / 512)).to(torch.float8_e4m3fn)
    triton_sgdm_step_(p, g, u, lr=0.01, momentum_factor=0.9, seed=3,
                      formats=(StateFormat(torch.float8_e4m3fn, "nearest"),))
    assert torch.equal(u.float(), signs * (6 / 512))
    assert tbits(u).size == n
