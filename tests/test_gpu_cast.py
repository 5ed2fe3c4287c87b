"""sm_100a cast kernel vs the reference's golden bytes and the CPU oracle."""

import numpy as np
import pytest
import torch

import oracle
from _support import DTYPE, FMT, assert_bits_or_nan, from_bits, load_json, load_npz, tbits

pytestmark = pytest.mark.gpu

FORMATS = [torch.float32, torch.bfloat16, torch.float16, torch.float8_e4m3fn, torch.float8_e5m2]
RULES = ["nearest", "stochastic"]


@pytest.mark.parametrize("case", load_json("casts.json")["cases"], ids=lambda c: c["key"])
def test_cast_matches_reference_golden_bytes(case, cuda_device):
    from sr_states.cuda import cast

    arrays = load_npz("casts.npz")
    x = from_bits(arrays[case["input"]], torch.float32, cuda_device)
    dtype = DTYPE[case["format"]]
    y = cast(x, dtype=dtype, rounding=RULES[case["rule"]], seed=case["seed"],
             offset=case["offset"])
    assert_bits_or_nan(tbits(y), arrays[case["key"]], case["format"], case["key"])


def _random_inputs(n, seed):
    gen = torch.Generator().manual_seed(seed)
    raw = torch.randint(-(2**31), 2**31, (n // 2,), generator=gen, dtype=torch.int32)
    mags = torch.exp2(torch.rand(n - n // 2, generator=gen, dtype=torch.float64) * 300 - 150)
    mags = (mags * torch.where(torch.rand(mags.shape, generator=gen) < 0.5, -1.0, 1.0)).float()
    return torch.cat((raw.view(torch.float32), mags))


@pytest.mark.parametrize("dtype", FORMATS, ids=str)
@pytest.mark.parametrize("rule", RULES)
def test_cast_matches_oracle_on_random_bits_and_magnitudes(dtype, rule, cuda_device):
    from sr_states.cuda import cast

    x = _random_inputs((1 << 22) + 13, 5)
    seed, offset = 2**32 + 977, 2**32 - 5000
    expected = oracle.cast(x.numpy(), FMT[dtype], RULES.index(rule), seed, offset, threads=8)
    y = cast(x.to(cuda_device), dtype=dtype, rounding=rule, seed=seed, offset=offset)
    assert_bits_or_nan(tbits(y), expected, FMT[dtype])


@pytest.mark.parametrize("dtype", FORMATS[1:], ids=str)
def test_cast_is_invariant_to_grid_and_split(dtype, cuda_device, monkeypatch):
    from sr_states.cuda import _native, cast

    x = _random_inputs(100_003, 9).to(cuda_device)
    whole = tbits(cast(x, dtype=dtype, seed=77, offset=2**32 - 19))
    for grid in (1, 3, 149):
        monkeypatch.setattr(_native.NativeLauncher, "cast",
                            _with_grid(_native.NativeLauncher.cast, grid))
        assert np.array_equal(tbits(cast(x, dtype=dtype, seed=77, offset=2**32 - 19)), whole)
    monkeypatch.undo()
    split = 4101
    parts = [cast(x[:split], dtype=dtype, seed=77, offset=2**32 - 19),
             cast(x[split:], dtype=dtype, seed=77, offset=2**32 - 19 + split)]
    assert np.array_equal(np.concatenate([tbits(p) for p in parts]), whole)


def _with_grid(method, grid):
    def call(self, *args, **kwargs):
        kwargs["grid_ctas"] = grid
        return method(self, *args, **kwargs)

    return call


@pytest.mark.parametrize("n", [0, 1, 7, 8, 9, 2047, 2048, 2049, 100_003])
def test_cast_sizes_and_unaligned_views(n, cuda_device):
    from sr_states.cuda import cast

    base = _random_inputs(n + 3, n)
    for start in (0, 1, 3):  # 0: aligned vector path, 1/3: unaligned scalar path
        x = base[start:start + n]
        expected = oracle.cast(x.numpy(), oracle.E4M3, 1, 5, 11)
        y = cast(x.to(cuda_device), dtype=torch.float8_e4m3fn, seed=5, offset=11)
        assert y.shape == (n,) and y.dtype == torch.float8_e4m3fn
        assert_bits_or_nan(tbits(y), expected, oracle.E4M3)


@pytest.mark.parametrize("dtype", FORMATS[1:], ids=str)
@pytest.mark.parametrize("rule", RULES)
def test_public_cast_any_layout_uses_row_major_counters(dtype, rule, cuda_device):
    import sr_states

    x = torch.linspace(-3, 7, 35 * 9).reshape(35, 9).T  # non-contiguous
    expected = oracle.cast(x.contiguous().numpy(), FMT[dtype], RULES.index(rule), 913,
                           2**32 - 17)
    y = sr_states.cast(x.to(cuda_device), dtype=dtype, rounding=rule, seed=913,
                       offset=2**32 - 17)
    assert y.shape == x.shape and y.device.type == "cuda"
    assert_bits_or_nan(tbits(y), expected.reshape(-1), FMT[dtype])


def test_bf16_cast_variants(cuda_device):
    from sr_states.cuda import rn_cast_bf16, sr_cast_bf16

    x = torch.linspace(-10, 10, 100_003).to(cuda_device)
    expected = oracle.cast(x.cpu().numpy(), oracle.BF16, 1, 991, 17)
    for mode in ("convert", "bits"):
        out = sr_cast_bf16(x, seed=991, offset=17, store_mode=mode)
        assert out.data_ptr() != x.data_ptr()
        assert np.array_equal(tbits(out), expected)
    assert torch.equal(rn_cast_bf16(x), x.to(torch.bfloat16))
    assert sr_cast_bf16(torch.empty(0, device=cuda_device), seed=1).shape == (0,)


def _chunk_starts(total_chunks, every):
    return range(0, total_chunks, every)


@pytest.mark.parametrize("dtype", FORMATS[1:], ids=str)
@pytest.mark.parametrize("rule", RULES)
def test_cast_fp32_encoding_sweep(dtype, rule, cuda_device):
    """Every FP32 encoding in 1/16 of the 2^32 space (2^20-element chunks spread
    evenly over it) against the oracle, counters wrapping past 2^32."""
    from sr_states.cuda import cast

    chunk = 1 << 20
    seed, offset = 0x9E3779B9, 2**32 - 3 * chunk
    for c in _chunk_starts(4096, 16):
        first = c * chunk
        bits = torch.arange(first, first + chunk, dtype=torch.int64, device=cuda_device)
        x = bits.to(torch.int32).view(torch.float32)  # wraps to the FP32 encoding
        y = cast(x, dtype=dtype, rounding=rule, seed=seed, offset=offset + first)
        expected = oracle.cast_bits_range(first, chunk, FMT[dtype], RULES.index(rule), seed,
                                          offset + first, threads=8)
        assert_bits_or_nan(tbits(y), expected, FMT[dtype], f"chunk {c}")
