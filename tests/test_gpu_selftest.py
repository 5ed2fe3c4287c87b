"""Device building blocks of the kernels checked element by element on the GPU
(libsrs_selftest.so compiles the same headers as libsrs_b200.so)."""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

SELFTEST = "stochastic-rounding-pytorch_b200/sr_states/_native/libsrs_selftest.so"


@pytest.fixture(scope="module")
def selftest(cuda_device):
    from pathlib import Path

    lib = ctypes.CDLL(str(Path(__file__).resolve().parents[1] / SELFTEST))
    lib.srs_selftest_packed_math.argtypes = [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_void_p,
                                             ctypes.c_void_p]
    lib.srs_selftest_sr_fast.argtypes = [ctypes.c_int, ctypes.c_uint32, ctypes.c_void_p,
                                         ctypes.c_void_p]
    lib.srs_selftest_cr_facts.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    lib.srs_selftest_adamw_fast.argtypes = [ctypes.c_uint64, ctypes.c_uint32] + [
        ctypes.c_float] * 6 + [ctypes.c_void_p, ctypes.c_void_p]
    return lib


def test_packed_fp32_operations_round_each_operation_once(selftest, cuda_device):
    """mul/add/fma .f32x2 (inline PTX with .rn) equal the scalar _rn intrinsics on
    2^26 random input pairs, and the kernels' multiply-then-add (mul_add_rn2,
    single-use product) rounds the product before the addition.  Counts 4 and 5
    record the hazard that rule avoids: a single-use packed product feeding a
    packed add is fused."""
    counts = torch.zeros(6, dtype=torch.int64, device=cuda_device)
    for seed in (1, 2):
        assert selftest.srs_selftest_packed_math(1 << 25, seed, counts.data_ptr(),
                                                 torch.cuda.current_stream().cuda_stream) == 0
    got = counts.tolist()
    assert got[:4] == [0, 0, 0, 0], got
    print("single-use packed mul->add fused (mismatches): inline PTX", got[4], "CUDA", got[5])


@pytest.mark.parametrize("fmt", [1, 2, 3, 4], ids=["bf16", "f16", "e4m3", "e5m2"])
def test_screened_stochastic_rounding_equals_per_element_rule(selftest, cuda_device, fmt):
    """The screened fast path of the stochastic encoders (FP32 arithmetic with
    round-toward-zero FMAs for the FP16/FP8 grids) gives the per-element rule's
    bytes for every FP32 bit pattern that passes the screen, at two hash seeds."""
    for seed in (0x2545F491, 7):
        counts = torch.zeros(3, dtype=torch.int64, device=cuda_device)
        assert selftest.srs_selftest_sr_fast(fmt, seed, counts.data_ptr(),
                                             torch.cuda.current_stream().cuda_stream) == 0
        compared, differ, screened_out = counts.tolist()
        assert compared + screened_out == 1 << 29
        assert differ == 0, (fmt, seed, differ)
        # NaN patterns (and, for the grids, |x| >= 2^63) are the only ones screened out.
        assert screened_out < (1 << 29) // 3


def test_square_root_and_reciprocal_facts_of_the_screened_arithmetic(selftest, cuda_device):
    """For every FP32 input: the corrected rsqrt square root equals __fsqrt_rn
    from 2^-102 up, and the refined negated reciprocal equals -__frcp_rn on
    [2^-126, 2^126)."""
    counts = torch.zeros(2, dtype=torch.int64, device=cuda_device)
    assert selftest.srs_selftest_cr_facts(counts.data_ptr(),
                                          torch.cuda.current_stream().cuda_stream) == 0
    assert counts.tolist() == [0, 0]


def _rn_reciprocal(c):
    # Division of floats: rounding the double quotient to float is correct rounding.
    return float(np.float32(1.0 / np.float64(np.float32(c))))


def _numerator_floor(nss):
    s = abs(float(np.float32(nss)))
    if s == 0.0:
        return float("inf")
    f = np.float32(2.0 ** -90 / s)
    while float(f) * s < 2.0 ** -90:
        f = np.nextafter(f, np.float32(np.inf))
    return float(f)


@pytest.mark.parametrize("c", [1.0, 0.0316227766, 0.001, 0.5, 0.99949987])
@pytest.mark.parametrize("nss", [-1e-3, -3e-3, -1.0, -1e-6])
@pytest.mark.parametrize("eps", [1e-8, 0.0, 1.0])
def test_screened_adamw_arithmetic_equals_ieee_operations(selftest, cuda_device, c, nss, eps):
    """The screened update p*decay + (nss*m')/(sqrt(v')/c + eps) gives the bits
    of the per-element IEEE operations for every random vector that passes the
    screen (2^21 vectors; a quarter of them with extreme exponents)."""
    counts = torch.zeros(3, dtype=torch.int64, device=cuda_device)
    c32 = float(np.float32(c))
    assert selftest.srs_selftest_adamw_fast(
        1 << 21, 0xC0FFEE, c32, _rn_reciprocal(c32), float(np.float32(nss)),
        _numerator_floor(nss), float(np.float32(eps)), float(np.float32(1 - 1e-5)),
        counts.data_ptr(), torch.cuda.current_stream().cuda_stream) == 0
    compared, differ, screened_out = counts.tolist()
    assert differ == 0, (compared, differ)
    assert compared > (1 << 21) // 2
