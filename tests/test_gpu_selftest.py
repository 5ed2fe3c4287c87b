"""Device building blocks of the kernels checked element by element on the GPU
(libsrs_selftest.so compiles the same headers as libsrs_b200.so)."""

import ctypes

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
