"""srs_adamw_multi_noalloc, the multi-tensor AdamW step that allocates no device
memory (its row table lives in a fixed table of the library's device image),
against srs_adamw_multi, whose row table the caller allocates, and against the
CPU oracle.

Some callers cannot allocate device memory while they step: a runtime that
hands all of HBM to its own arena up front, or code that must not enter an
allocator at step time.  This entry point serves them.  Both entry points
launch the same kernel on the same rows, so two steps in a row must leave
bit-identical parameters and states (tolerance: exact), and the oracle, which
follows the same operation order with a correctly rounded square root, must
agree byte for byte too.  This file is named to be collected last, so the GPU
test runs both alone in a fresh process and after every other test has used
the library.
"""

import ctypes

import numpy as np
import pytest
import torch

import oracle
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


def host_copy(row):
    """CPU numpy copies of a row's (param, grad, m, v) in the oracle's bit layouts."""
    out = []
    for t in row:
        if t.dtype == torch.float32:
            out.append(t.cpu().numpy().copy())
        else:
            size = t.element_size()
            raw = t.view(torch.int16 if size == 2 else torch.uint8).cpu().numpy()
            out.append(raw.view(np.uint16 if size == 2 else np.uint8).copy())
    return out


def oracle_step(spec, cpu_rows, hp, step):
    """The same multi-tensor step on the CPU oracle, row by row."""
    for index, ((numel, p_dtype, g_dtype, cls), (p, g, m, v)) in enumerate(zip(spec, cpu_rows)):
        scalars = [hp.beta1, hp.beta2, hp.one_minus_beta1, hp.one_minus_beta2, hp.eps, hp.decay,
                   hp.neg_step_size[cls], hp.bias2_sqrt[cls]]
        oracle.adamw_core_at(p.ctypes.data, int(p_dtype == torch.bfloat16), g.ctypes.data,
                             int(g_dtype == torch.bfloat16), m.ctypes.data, oracle.E4M3,
                             oracle.STOCHASTIC, v.ctypes.data, oracle.BF16, oracle.STOCHASTIC,
                             numel, scalars, oracle.update_key(SEED, step, index), 0)


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

    expected = [host_copy(row) for row in ours]

    for call, steps in enumerate([(1, 2), (2, 3)]):
        hp, words = hparams(steps), rng(call + 1)
        check(lib, lib.srs_adamw_multi(device_table.data_ptr(), len(spec), n_tiles, E4M3, SR,
                                       BF16, SR, ctypes.byref(hp), ctypes.byref(words),
                                       uniform_kind(table_theirs), 0, stream))
        torch.cuda.synchronize(cuda_device)
        allocated = torch.cuda.memory_stats(cuda_device).get("allocation.all.allocated", 0)
        free_before = torch.cuda.mem_get_info(cuda_device)[0]
        check(lib, lib.srs_adamw_multi_noalloc(table_ours.ctypes.data, len(spec), n_tiles, E4M3,
                                               SR, BF16, SR, ctypes.byref(hp),
                                               ctypes.byref(words), 0, stream))
        torch.cuda.synchronize(cuda_device)
        assert torch.cuda.memory_stats(cuda_device).get("allocation.all.allocated", 0) == allocated
        if call > 0:  # the first call may load the module that holds the table
            assert torch.cuda.mem_get_info(cuda_device)[0] == free_before
        oracle_step(spec, expected, hp, call + 1)
        for r, (a_row, b_row, e_row) in enumerate(zip(ours, theirs, expected)):
            for name, a, b, e in zip(("param", "grad", "m", "v"), a_row, b_row, e_row):
                assert np.array_equal(bits(a), bits(b)), f"call {call}: row {r} {name} differs"
                assert np.array_equal(bits(a), e.view(np.uint8)), (
                    f"call {call}: row {r} {name} differs from the oracle")
        assert any(bool(row[2].float().abs().sum() > 0) for row in ours)  # the step ran
        # Fresh gradients, identical for both sets, before the next call.
        for a_row, b_row in zip(ours, theirs):
            a_row[1].copy_(torch.randn(a_row[1].numel(), generator=generator).to(a_row[1]))
            b_row[1].copy_(a_row[1])
        for a_row, e_row in zip(ours, expected):
            e_row[1] = host_copy(a_row)[1]


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


def test_noalloc_rejects_a_vector_flag_on_misaligned_rows():
    """A row flagged SRS_ROW_VECTOR_OK whose addresses lack the promised alignment
    is refused on the host.  Every table here also carries a wrong n_tiles (the
    row holds 2 tiles, 3 are claimed), which the host check reports after the
    rows, so no call can reach the GPU even if a row check were missing."""
    lib = _native.load_library()
    hp, words = hparams((1,)), rng(1)
    table = np.zeros(1, dtype=_native.ROW_DTYPE)
    table["numel"] = 4096
    table["param"], table["grad"] = 0x10000, 0x20000
    table["state"] = (0x30000, 0x40000)
    table["flags"] = _native.ROW_VECTOR_OK | _native.ROW_PARAM_BF16 | _native.ROW_GRAD_BF16

    def message(rows):
        rc = lib.srs_adamw_multi_noalloc(rows.ctypes.data, 1, 3, E4M3, SR, BF16, SR,
                                         ctypes.byref(hp), ctypes.byref(words), 0, None)
        assert rc == _native.SRS_ERR_INVALID_ARGUMENT
        return lib.srs_last_error()

    for field, index, address in (("param", None, 0x10002), ("grad", None, 0x20008),
                                  ("state", 0, 0x30004), ("state", 1, 0x40008)):
        bad = table.copy()
        if index is None:
            bad[field] = address
        else:
            bad[field][0, index] = address
        assert b"SRS_ROW_VECTOR_OK" in message(bad), (field, index)
    # An FP8 state needs only 8 bytes, and without the flag any alignment passes
    # the row check: these tables fail on n_tiles only.
    fp8_ok = table.copy()
    fp8_ok["state"][0, 0] = 0x30008
    unflagged = table.copy()
    unflagged["param"] = 0x10002
    unflagged["flags"] = _native.ROW_PARAM_BF16 | _native.ROW_GRAD_BF16
    for good in (table, fp8_ok, unflagged):
        assert b"n_tiles" in message(good)


@pytest.mark.gpu
def test_noalloc_captured_into_a_graph_needs_page_locked_rows(cuda_device):
    """Under stream capture the row copy becomes a graph node that reads
    host_rows at every replay, so pageable rows are refused (nothing is
    enqueued and the capture stays usable) and page-locked rows are accepted.
    One replay of the captured step must equal the same step called directly
    (tolerance: exact).  The refusal needs a device to ask whether the stream
    captures, so it is checked here, not in the CPU tests."""
    lib = _native.load_library()
    tile = int(lib.srs_tile_elems())
    generator = torch.Generator().manual_seed(11)
    captured = make_rows(UNIFORM, cuda_device, generator)
    direct = [[t.clone() for t in row] for row in captured]
    table_captured, n_tiles = host_table(UNIFORM, captured, tile)
    table_direct, _ = host_table(UNIFORM, direct, tile)
    pinned = torch.from_numpy(table_captured.view(np.uint8).copy()).pin_memory()
    hp, words = hparams((1, 2)), rng(1)

    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    check(lib, lib.srs_adamw_multi_noalloc(table_direct.ctypes.data, len(UNIFORM), n_tiles,
                                           E4M3, SR, BF16, SR, ctypes.byref(hp),
                                           ctypes.byref(words), 0, stream))
    torch.cuda.synchronize(cuda_device)

    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        stream = torch.cuda.current_stream(cuda_device).cuda_stream
        rc = lib.srs_adamw_multi_noalloc(table_captured.ctypes.data, len(UNIFORM), n_tiles,
                                         E4M3, SR, BF16, SR, ctypes.byref(hp),
                                         ctypes.byref(words), 0, stream)
        refusal = lib.srs_last_error()
        accepted = lib.srs_adamw_multi_noalloc(pinned.data_ptr(), len(UNIFORM), n_tiles, E4M3,
                                               SR, BF16, SR, ctypes.byref(hp),
                                               ctypes.byref(words), 0, stream)
        message = lib.srs_last_error()
    assert rc == _native.SRS_ERR_INVALID_ARGUMENT and b"page-locked" in refusal, refusal
    assert accepted == _native.SRS_OK, message.decode()
    for row in captured:  # capturing ran nothing
        assert not bool(row[2].float().abs().sum() > 0)
    graph.replay()
    torch.cuda.synchronize(cuda_device)
    for r, (a_row, b_row) in enumerate(zip(captured, direct)):
        for name, a, b in zip(("param", "grad", "m", "v"), a_row, b_row):
            assert np.array_equal(bits(a), bits(b)), f"row {r} {name}: replay differs"
    del graph
