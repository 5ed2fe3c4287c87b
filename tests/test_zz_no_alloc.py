"""srs_adamw_multi_noalloc, the multi-tensor AdamW step that allocates no device
memory (its row table lives in a fixed table of the library's device image),
against srs_adamw_multi, whose row table the caller allocates.

Both entry points launch the same kernel on the same rows, so two steps in a
row must leave bit-identical parameters and states (tolerance: exact).  This
file is named to be collected last, so the GPU test runs both alone in a fresh
process and after every other test has used the library.
"""

import ctypes

import numpy as np
import pytest
import torch

from sr_states.cuda import _native

SEED = 1234
LR, WEIGHT_DECAY, BETA1, BETA2, EPS = 1e-3, 0.01, 0.9, 0.999, 1e-8
# (numel, param dtype, grad dtype, step class): tails, a one-element row, rows
# of every dtype pair and two bias-correction step classes.
ROWS = [(70001, torch.bfloat16, torch.bfloat16, 0), (1, torch.float32, torch.bfloat16, 1),
        (2048, torch.float32, torch.float32, 0), (4099, torch.bfloat16, torch.float32, 1),
        (300000, torch.bfloat16, torch.bfloat16, 0)]
UNIFORM = [(n, torch.bfloat16, torch.bfloat16, c) for n, _, _, c in ROWS]
BF16, E4M3 = 1, 3  # SRS_FMT_BF16, SRS_FMT_E4M3
SR = 1  # SRS_RULE_STOCHASTIC


def hparams(steps):
    hp = _native.SrsAdamWHparams()
    hp.beta1, hp.beta2 = BETA1, BETA2
    hp.one_minus_beta1, hp.one_minus_beta2 = 1.0 - BETA1, 1.0 - BETA2
    hp.eps, hp.decay = EPS, 1.0 - LR * WEIGHT_DECAY
    hp.n_step_classes = len(steps)
    for c, t in enumerate(steps):
        hp.neg_step_size[c] = -LR / (1.0 - BETA1 ** t)
        hp.bias2_sqrt[c] = (1.0 - BETA2 ** t) ** 0.5
    return hp


def rng(step):
    return _native.SrsRng(SEED, 0, step, 0, _native.KEY_DERIVE)


def make_rows(spec, device, generator):
    """Parameters, gradients and (E4M3 m, BF16 v) states of every row."""
    rows = []
    for numel, p_dtype, g_dtype, _ in spec:
        p = torch.randn(numel, generator=generator).to(device, p_dtype)
        g = torch.randn(numel, generator=generator).to(device, g_dtype)
        m = torch.zeros(numel, dtype=torch.float8_e4m3fn, device=device)
        v = torch.zeros(numel, dtype=torch.bfloat16, device=device)
        rows.append([p, g, m, v])
    return rows


def host_table(spec, rows, tile):
    table = np.zeros(len(rows), dtype=_native.ROW_DTYPE)
    begin = 0
    for i, ((numel, p_dtype, g_dtype, cls), (p, g, m, v)) in enumerate(zip(spec, rows)):
        flags = (_native.ROW_PARAM_BF16 if p_dtype == torch.bfloat16 else 0)
        flags |= (_native.ROW_GRAD_BF16 if g_dtype == torch.bfloat16 else 0)
        flags |= _native.ROW_VECTOR_OK | (cls << _native.ROW_CLASS_SHIFT)
        table[i] = (p.data_ptr(), g.data_ptr(), (m.data_ptr(), v.data_ptr()), numel, begin,
                    i, 0, flags, 0)
        begin += -(-numel // tile)
    return table, begin


def uniform_kind(table):
    kinds = np.unique(table["flags"] & 3)
    return int(kinds[0]) if kinds.size == 1 else _native.KIND_MIXED


def bits(t):
    return t.view(torch.uint8).cpu().numpy()


def check(lib, rc):
    assert rc == _native.SRS_OK, lib.srs_last_error().decode()


@pytest.mark.gpu
@pytest.mark.parametrize("spec", [ROWS, UNIFORM], ids=["mixed-dtypes", "bf16"])
def test_noalloc_matches_allocating_entry_point_two_steps_in_a_row(cuda_device, spec):
    lib = _native.load_library()
    tile = int(lib.srs_tile_elems())
    generator = torch.Generator().manual_seed(7)
    ours = make_rows(spec, cuda_device, generator)
    theirs = [[t.clone() for t in row] for row in ours]
    table_ours, n_tiles = host_table(spec, ours, tile)
    table_theirs, _ = host_table(spec, theirs, tile)
    device_table = torch.from_numpy(table_theirs.view(np.uint8)).to(cuda_device)
    stream = torch.cuda.current_stream(cuda_device).cuda_stream

    for call, steps in enumerate([(1, 2), (2, 3)]):
        hp, words = hparams(steps), rng(call + 1)
        check(lib, lib.srs_adamw_multi(device_table.data_ptr(), len(spec), n_tiles, E4M3, SR,
                                       BF16, SR, ctypes.byref(hp), ctypes.byref(words),
                                       uniform_kind(table_theirs), 0, stream))
        allocated = torch.cuda.memory_stats(cuda_device).get("allocation.all.allocated", 0)
        check(lib, lib.srs_adamw_multi_noalloc(table_ours.ctypes.data, len(spec), n_tiles, E4M3,
                                               SR, BF16, SR, ctypes.byref(hp),
                                               ctypes.byref(words), 0, stream))
        assert torch.cuda.memory_stats(cuda_device).get("allocation.all.allocated", 0) == allocated
        torch.cuda.synchronize(cuda_device)
        for r, (a_row, b_row) in enumerate(zip(ours, theirs)):
            for name, a, b in zip(("param", "grad", "m", "v"), a_row, b_row):
                assert np.array_equal(bits(a), bits(b)), f"call {call}: row {r} {name} differs"
        assert any(bool(row[2].float().abs().sum() > 0) for row in ours)  # the step ran
        # Fresh gradients, identical for both sets, before the next call.
        for a_row, b_row in zip(ours, theirs):
            a_row[1].copy_(torch.randn(a_row[1].numel(), generator=generator).to(a_row[1]))
            b_row[1].copy_(a_row[1])


def test_noalloc_rejects_oversized_and_inconsistent_tables_before_any_device_call():
    lib = _native.load_library()
    hp, words = hparams((1,)), rng(1)
    big = np.zeros(_native.NOALLOC_MAX_ROWS + 1, dtype=_native.ROW_DTYPE)
    rc = lib.srs_adamw_multi_noalloc(big.ctypes.data, len(big), 0, 3, 1, 1, 1, ctypes.byref(hp),
                                     ctypes.byref(words), 0, None)
    assert rc == _native.SRS_ERR_INVALID_ARGUMENT
    assert b"at most 4096 rows" in lib.srs_last_error()
    table = np.zeros(2, dtype=_native.ROW_DTYPE)
    table["numel"] = [10, 10]
    table["param"] = table["grad"] = 0x1000
    table["state"] = 0x1000
    table["tile_begin"] = [0, 0]  # row 1 must begin at tile 1
    rc = lib.srs_adamw_multi_noalloc(table.ctypes.data, 2, 2, 3, 1, 1, 1, ctypes.byref(hp),
                                     ctypes.byref(words), 0, None)
    assert rc == _native.SRS_ERR_INVALID_ARGUMENT and b"tile_begin" in lib.srs_last_error()
    table["tile_begin"] = [0, 1]
    rc = lib.srs_adamw_multi_noalloc(table.ctypes.data, 2, 3, 3, 1, 1, 1, ctypes.byref(hp),
                                     ctypes.byref(words), 0, None)
    assert rc == _native.SRS_ERR_INVALID_ARGUMENT and b"n_tiles" in lib.srs_last_error()
    table["flags"] = [0, 1 << _native.ROW_CLASS_SHIFT]  # class 1 with one class
    rc = lib.srs_adamw_multi_noalloc(table.ctypes.data, 2, 2, 3, 1, 1, 1, ctypes.byref(hp),
                                     ctypes.byref(words), 0, None)
    assert rc == _native.SRS_ERR_INVALID_ARGUMENT and b"step class" in lib.srs_last_error()
    assert lib.srs_adamw_multi_noalloc(None, 0, 0, 3, 1, 1, 1, ctypes.byref(hp),
                                       ctypes.byref(words), 0, None) == _native.SRS_OK
