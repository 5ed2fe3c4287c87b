"""Shared test helpers: bit views, ULP distances, golden loaders, and a launcher
stand-in that executes the CPU oracle on the row tables the host code builds."""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import torch

import oracle

GOLDEN = Path(__file__).resolve().parent / "golden"

FMT = {torch.float32: oracle.F32, torch.bfloat16: oracle.BF16, torch.float16: oracle.F16,
       torch.float8_e4m3fn: oracle.E4M3, torch.float8_e5m2: oracle.E5M2}
DTYPE = {v: k for k, v in FMT.items()}
_TORCH_BITS = {4: torch.int32, 2: torch.int16, 1: torch.uint8}
_NP_BITS = {4: np.uint32, 2: np.uint16, 1: np.uint8}


def tbits(t: torch.Tensor) -> np.ndarray:
    """Raw bits of a tensor (any device) as an unsigned numpy array."""
    size = t.element_size()
    return t.detach().contiguous().view(_TORCH_BITS[size]).cpu().numpy().view(_NP_BITS[size])


def from_bits(a: np.ndarray, dtype: torch.dtype, device="cpu") -> torch.Tensor:
    size = torch.empty((), dtype=dtype).element_size()
    signed = {4: np.int32, 2: np.int16, 1: np.uint8}[size]
    raw = torch.from_numpy(np.ascontiguousarray(a).view(signed).copy())
    return raw.view(_TORCH_BITS[size]).view(dtype).to(device)


def isnan_bits(bits: np.ndarray, fmt: int) -> np.ndarray:
    return np.isnan(oracle.decode(bits, fmt))


def assert_bits_or_nan(actual: np.ndarray, expected: np.ndarray, fmt: int, context=""):
    """Bit-exact except NaN, which only has to be NaN (the reference's policy)."""
    actual, expected = np.asarray(actual).reshape(-1), np.asarray(expected).reshape(-1)
    assert actual.shape == expected.shape, context
    an, en = isnan_bits(actual, fmt), isnan_bits(expected, fmt)
    assert np.array_equal(an, en), f"{context}: NaN positions differ"
    bad = np.flatnonzero((actual != expected) & ~en)
    assert bad.size == 0, (f"{context}: {bad.size} mismatches, first at {bad[:5]}: "
                           f"{actual[bad[:5]]} vs {expected[bad[:5]]}")


def ulp_distance(a_bits: np.ndarray, b_bits: np.ndarray, width: int) -> np.ndarray:
    """|ordinal(a) - ordinal(b)| of same-width float encodings (sign-magnitude order)."""
    def ordinal(x):
        x = np.asarray(x).astype(np.int64)
        sign = np.int64(1) << (width - 1)
        return np.where(x & sign, -(x & (sign - 1)), x)
    return np.abs(ordinal(a_bits) - ordinal(b_bits))


def load_json(name):
    return json.loads((GOLDEN / name).read_text())


def load_npz(name):
    return np.load(GOLDEN / name)


class FakeLauncher:
    """Stand-in for sr_states.cuda._native.NativeLauncher that runs the oracle on
    CPU tensors, checking the row-table invariants the kernels rely on."""

    def __init__(self):
        self.calls = []
        from sr_states.cuda import _native

        self._native = _native
        self._tile = int(_native.load_library().srs_tile_elems())

    def check_device(self, device, what="fused state updates"):
        if device.type != "cpu":
            raise ValueError(f"{what}: the fake launcher runs on CPU tensors only")

    def tile_elems(self):
        return self._tile

    def _check_table(self, table, n_rows, n_tiles):
        host = table.host
        assert len(host) == n_rows and n_rows > 0
        tiles = -(-host["numel"] // self._tile)
        assert host["tile_begin"][0] == 0
        assert np.array_equal(host["tile_begin"][1:], np.cumsum(tiles)[:-1])
        assert host["tile_begin"][-1] + tiles[-1] == n_tiles
        assert np.all(host["numel"] > 0)
        assert bytes(table.storage.numpy()) == host.tobytes()

    def _key(self, rng, row):
        if rng.key_mode == self._native.KEY_GIVEN:
            return int(row["param_index"])
        return oracle.update_key(rng.seed_lo | (rng.seed_hi << 32),
                                 rng.step_lo | (rng.step_hi << 32), int(row["param_index"]))

    def adamw_multi(self, table, n_rows, n_tiles, m_fmt, m_rule, v_fmt, v_rule, hp, rng, stream,
                    grid_ctas=0):
        self._check_table(table, n_rows, n_tiles)
        self.calls.append(("adamw_multi", n_rows, n_tiles, m_fmt, m_rule, v_fmt, v_rule))
        for row in table.host:
            cls = (int(row["flags"]) >> self._native.ROW_CLASS_SHIFT) & 0xFF
            assert cls < hp.n_step_classes
            scalars = [hp.beta1, hp.beta2, hp.one_minus_beta1, hp.one_minus_beta2, hp.eps,
                       hp.decay, hp.neg_step_size[cls], hp.bias2_sqrt[cls]]
            flags = int(row["flags"])
            oracle.adamw_core_at(int(row["param"]), flags & 1, int(row["grad"]), (flags >> 1) & 1,
                                 int(row["state"][0]), m_fmt, m_rule, int(row["state"][1]),
                                 v_fmt, v_rule, int(row["numel"]), scalars, self._key(rng, row),
                                 int(row["offset"]))

    def sgdm_multi(self, table, n_rows, n_tiles, u_fmt, u_rule, hp, rng, stream, grid_ctas=0):
        self._check_table(table, n_rows, n_tiles)
        self.calls.append(("sgdm_multi", n_rows, n_tiles, u_fmt, u_rule))
        for row in table.host:
            flags = int(row["flags"])
            oracle.sgdm_core_at(int(row["param"]), flags & 1, int(row["grad"]), (flags >> 1) & 1,
                                int(row["state"][0]), u_fmt, u_rule, int(row["numel"]),
                                hp.momentum, hp.neg_lr, self._key(rng, row), int(row["offset"]))

    def adamw_single(self, row, m_fmt, m_rule, v_fmt, v_rule, hp, stream, grid_ctas=0):
        self.calls.append(("adamw_single", row.numel))
        scalars = [hp.beta1, hp.beta2, hp.one_minus_beta1, hp.one_minus_beta2, hp.eps, hp.decay,
                   hp.neg_step_size[0], hp.bias2_sqrt[0]]
        oracle.adamw_core_at(row.param, row.flags & 1, row.grad, (row.flags >> 1) & 1,
                             row.state[0], m_fmt, m_rule, row.state[1], v_fmt, v_rule, row.numel,
                             scalars, row.param_index, row.offset)

    def sgdm_single(self, row, u_fmt, u_rule, hp, stream, grid_ctas=0):
        self.calls.append(("sgdm_single", row.numel))
        oracle.sgdm_core_at(row.param, row.flags & 1, row.grad, (row.flags >> 1) & 1,
                            row.state[0], u_fmt, u_rule, row.numel, hp.momentum, hp.neg_lr,
                            row.param_index, row.offset)

    def cast(self, x_ptr, y_ptr, n, fmt, rule, seed, offset, stream, grid_ctas=0):
        self.calls.append(("cast", n, fmt, rule))
        oracle.cast_at(x_ptr, y_ptr, n, fmt, rule, seed, offset)


def _bf16_rne(bits32: np.ndarray) -> np.ndarray:
    """FP32 encodings -> BF16 encodings, round to nearest even (NaN -> quiet NaN)."""
    b = bits32.astype(np.uint64)
    rounded = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16) & 0xFFFF
    nan = (bits32 & 0x7FFFFFFF) > 0x7F800000
    return np.where(nan, ((bits32 >> 16) | 0x40) & 0xFFFF, rounded).astype(np.uint16)


def adamw_param_formula(previous, m32, root, scalars, width) -> np.ndarray:
    """The reference's parameter update from its own intermediates, each FP32
    operation rounded once (numpy float32 arithmetic, no contraction):
        d = root / sqrt(bc2) + eps;  p' = p * decay + (-lr/bc1 * m') / d
    (sr_states/reference/adamw.py:86-89), then RNE to the parameter's width.
    ``scalars`` are the eight FP32 launch scalars of oracle.adamw_scalars."""
    _, _, _, _, eps, decay, nss, c = (np.float32(x) for x in scalars)
    prev = np.asarray(previous, dtype=np.float32).reshape(-1)
    d = (np.asarray(root, dtype=np.float32).reshape(-1) / c) + eps
    u = (nss * np.asarray(m32, dtype=np.float32).reshape(-1)) / d
    out = (prev * decay + u).view(np.uint32)
    return _bf16_rne(out) if width == 16 else out


def correctly_rounded_sqrt(v32) -> np.ndarray:
    """IEEE FP32 square root (the double-precision root of an FP32 value rounded
    to FP32 is correctly rounded: 53 >= 2 * 24 + 2)."""
    return np.sqrt(np.asarray(v32, dtype=np.float32).astype(np.float64)).astype(np.float32)


def explain_adamw_param(actual_bits, reference_bits, previous, v32, root, m32, scalars, width):
    """Account for every AdamW parameter difference from the reference.

    PyTorch's CPU ``sqrt`` is not correctly rounded (one ulp off on ~0.7% of
    inputs); this package's kernels and oracle use the IEEE square root.  Given
    the reference's own intermediates of the step (its ``v32``, ``v32.sqrt()``
    and ``m32``), check that
      * the update formula with the reference's root reproduces the reference's
        parameter bytes exactly (the formula is pinned), and
      * ``actual`` equals the same formula with the correctly rounded root of the
        same ``v32``, byte for byte.
    So parameters are byte-exact wherever the two roots agree, and every other
    difference is the propagation of that one-ulp root difference.  Returns
    (elements whose roots differ, elements whose parameters differ, max ulp)."""
    reference_bits = np.asarray(reference_bits).reshape(-1)
    actual_bits = np.asarray(actual_bits).reshape(-1)
    pinned = adamw_param_formula(previous, m32, root, scalars, width)
    assert np.array_equal(pinned, reference_bits), "the update formula does not reproduce the reference"
    ieee_root = correctly_rounded_sqrt(v32).reshape(-1)
    expected = adamw_param_formula(previous, m32, ieee_root, scalars, width)
    bad = np.flatnonzero(actual_bits != expected)
    assert bad.size == 0, (f"{bad.size} parameters differ from the reference's formula with a "
                           f"correctly rounded sqrt, first at {bad[:5]}")
    roots_differ = (np.asarray(root, dtype=np.float32).reshape(-1).view(np.uint32)
                    != ieee_root.view(np.uint32))
    assert np.array_equal(actual_bits[~roots_differ], reference_bits[~roots_differ])
    distance = ulp_distance(actual_bits, reference_bits, width)
    return int(roots_differ.sum()), int(np.count_nonzero(distance)), int(distance.max(initial=0))
