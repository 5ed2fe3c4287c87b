"""CPU oracle of the sr_states hot path — TEST INFRASTRUCTURE ONLY.

ctypes/numpy bindings of ``oracle/srs_oracle.c``, a plain-C restatement of the
reference algorithms (each C function cites the reference file:line it
follows).  Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of
``bench.py`` may import this package, and only as the checker or the timed CPU
baseline; the product path (``sr_states`` and ``libsrs_b200.so``) never does.

Parity of this oracle with the reference is pinned by the golden vectors in
``tests/golden/`` that ``tests/golden/make_golden.py`` produced by running the
reference itself.

Arrays are numpy.  Stored values are raw bits: FP32 as uint32 (or float32 for
parameters), BF16/FP16 as uint16, FP8 as uint8.
"""

from __future__ import annotations

import ctypes
import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np

from .build_oracle import LIBRARY, build

F32, BF16, F16, E4M3, E5M2 = 0, 1, 2, 3, 4
NEAREST, STOCHASTIC, TOWARD_ZERO = 0, 1, 2
BITS_DTYPE = {F32: np.uint32, BF16: np.uint16, F16: np.uint16, E4M3: np.uint8, E5M2: np.uint8}
_MASK32 = 0xFFFFFFFF

_lib = None


def lib() -> ctypes.CDLL:
    """Load (building first if needed) the oracle shared library."""
    global _lib
    if _lib is None:
        path = LIBRARY if LIBRARY.exists() else build()
        handle = ctypes.CDLL(str(path))
        u32, i64, i32, vp = ctypes.c_uint32, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p
        handle.srs_o_h32.argtypes, handle.srs_o_h32.restype = [u32], u32
        handle.srs_o_update_key.argtypes = [ctypes.c_uint64, ctypes.c_uint64, u32]
        handle.srs_o_update_key.restype = u32
        handle.srs_o_state_key.argtypes, handle.srs_o_state_key.restype = [u32, u32], u32
        handle.srs_o_hash.argtypes, handle.srs_o_hash.restype = [vp, vp, i64], None
        handle.srs_o_round.argtypes = [ctypes.c_float, i32, i32, u32]
        handle.srs_o_round.restype = u32
        handle.srs_o_decode.argtypes, handle.srs_o_decode.restype = [u32, i32], ctypes.c_float
        handle.srs_o_cast.argtypes = [vp, vp, i64, i32, i32, u32, u32]
        handle.srs_o_cast.restype = None
        handle.srs_o_cast_bits_range.argtypes = [u32, i64, vp, i32, i32, u32, u32]
        handle.srs_o_cast_bits_range.restype = None
        handle.srs_o_adamw.argtypes = [vp, i32, vp, i32, vp, i32, i32, vp, i32, i32, i64, vp,
                                       i64, u32, u32]
        handle.srs_o_adamw.restype = None
        handle.srs_o_sgdm.argtypes = [vp, i32, vp, i32, vp, i32, i32, i64, ctypes.c_double,
                                      ctypes.c_double, u32, u32]
        handle.srs_o_sgdm.restype = None
        handle.srs_o_adamw_scalars.argtypes = [vp, i64, vp]
        handle.srs_o_adamw_scalars.restype = None
        handle.srs_o_adamw_core.argtypes = [vp, i32, vp, i32, vp, i32, i32, vp, i32, i32, i64,
                                            vp, u32, u32]
        handle.srs_o_adamw_core.restype = None
        handle.srs_o_sgdm_core.argtypes = [vp, i32, vp, i32, vp, i32, i32, i64, ctypes.c_float,
                                           ctypes.c_float, u32, u32]
        handle.srs_o_sgdm_core.restype = None
        handle.srs_o_check_uniform_division.argtypes = [ctypes.c_float, ctypes.c_float, u32, u32,
                                                         u32, u32, u32, vp]
        handle.srs_o_check_uniform_division.restype = ctypes.c_uint64
        _lib = handle
    return _lib


def _ptr(a: np.ndarray, start: int = 0) -> int:
    return a.ctypes.data + start * a.itemsize


def _chunks(n: int, threads: int, align: int = 64):
    if n <= 0:
        return [(0, 0)]
    threads = max(1, min(threads, (n + align - 1) // align))
    step = ((n + threads - 1) // threads + align - 1) // align * align
    return [(lo, min(n, lo + step)) for lo in range(0, n, step)] or [(0, 0)]


def _run(n: int, threads: int, fn) -> None:
    parts = _chunks(n, threads)
    if len(parts) == 1:
        fn(*parts[0])
        return
    # ctypes releases the GIL for the duration of each foreign call.
    with ThreadPoolExecutor(len(parts)) as pool:
        list(pool.map(lambda part: fn(*part), parts))


def cpu_threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()


# ---------------------------------------------------------------- keys ----

def h32(counters) -> np.ndarray:
    c = np.ascontiguousarray(counters, dtype=np.uint32)
    out = np.empty_like(c)
    lib().srs_o_hash(_ptr(c), _ptr(out), c.size)
    return out


def update_key(seed: int, step: int, param_index: int) -> int:
    """sr_states/_hash.py:18-23 (low 64 bits of seed and step)."""
    return lib().srs_o_update_key(int(seed) & (2**64 - 1), int(step) & (2**64 - 1),
                                  int(param_index) & _MASK32)


def state_key(key: int, index: int) -> int:
    return lib().srs_o_state_key(int(key) & _MASK32, int(index) & _MASK32)


# --------------------------------------------------------------- casts ----

def decode(bits: np.ndarray, fmt: int) -> np.ndarray:
    """Stored bits -> float32 values (exact)."""
    bits = np.asarray(bits)
    if fmt == F32:
        return bits.astype(np.uint32).view(np.float32)
    if fmt == BF16:
        return (bits.astype(np.uint32) << 16).view(np.float32)
    if fmt == F16:
        return bits.astype(np.uint16).view(np.float16).astype(np.float32)
    table = np.array([lib().srs_o_decode(b, fmt) for b in range(256)], dtype=np.float32)
    return table[bits.astype(np.uint8)]


def cast(x, fmt: int, rule: int, seed: int = 0, offset: int = 0, threads: int = 1) -> np.ndarray:
    """sr_states.cast: counter of element i is (i + offset + seed) mod 2^32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    flat = x.reshape(-1)
    out = np.empty(flat.size, dtype=BITS_DTYPE[fmt])
    seed, offset = int(seed) & _MASK32, int(offset) & _MASK32

    def part(lo, hi):
        lib().srs_o_cast(_ptr(flat, lo), _ptr(out, lo), hi - lo, fmt, rule, seed,
                         (offset + lo) & _MASK32)

    _run(flat.size, threads, part)
    return out.reshape(x.shape)


def cast_bits_range(first_bits: int, n: int, fmt: int, rule: int, seed: int = 0,
                    offset: int = 0, threads: int = 1) -> np.ndarray:
    """Cast of the FP32 encodings first_bits, first_bits+1, ... (mod 2^32)."""
    out = np.empty(n, dtype=BITS_DTYPE[fmt])
    seed, offset = int(seed) & _MASK32, int(offset) & _MASK32

    def part(lo, hi):
        lib().srs_o_cast_bits_range((first_bits + lo) & _MASK32, hi - lo, _ptr(out, lo), fmt,
                                    rule, seed, (offset + lo) & _MASK32)

    _run(n, threads, part)
    return out


# ---------------------------------------------------------- optimizers ----

def _param_bf16(a: np.ndarray) -> int:
    if a.dtype == np.float32:
        return 0
    if a.dtype == np.uint16:
        return 1
    raise TypeError("parameters/gradients are float32 arrays or uint16 BF16 bits")


def adamw_(p, g, m, v, *, m_fmt, m_rule, v_fmt, v_rule, lr, beta1, beta2, eps, weight_decay,
           step, update_key, offset=0, threads=1) -> None:
    """In place, like sr_states.reference.adamw.adamw_step_ with seed=update_key."""
    n = p.size
    assert g.size == m.size == v.size == n
    for a in (p, g, m, v):
        assert a.flags.c_contiguous
    assert m.dtype == BITS_DTYPE[m_fmt] and v.dtype == BITS_DTYPE[v_fmt]
    hp = np.array([lr, beta1, beta2, eps, weight_decay], dtype=np.float64)
    pb, gb = _param_bf16(p), _param_bf16(g)
    key, offset = int(update_key) & _MASK32, int(offset) & _MASK32

    def part(lo, hi):
        lib().srs_o_adamw(_ptr(p, lo), pb, _ptr(g, lo), gb, _ptr(m, lo), m_fmt, m_rule,
                          _ptr(v, lo), v_fmt, v_rule, hi - lo, _ptr(hp), int(step), key,
                          (offset + lo) & _MASK32)

    _run(n, threads, part)


def sgdm_(p, g, u, *, u_fmt, u_rule, lr, momentum, update_key, offset=0, threads=1) -> None:
    """In place, like sr_states.reference.sgd.sgdm_step_ with seed=update_key."""
    n = p.size
    assert g.size == u.size == n and u.dtype == BITS_DTYPE[u_fmt]
    pb, gb = _param_bf16(p), _param_bf16(g)
    key, offset = int(update_key) & _MASK32, int(offset) & _MASK32

    def part(lo, hi):
        lib().srs_o_sgdm(_ptr(p, lo), pb, _ptr(g, lo), gb, _ptr(u, lo), u_fmt, u_rule, hi - lo,
                         float(lr), float(momentum), key, (offset + lo) & _MASK32)

    _run(n, threads, part)


def adamw_scalars(lr, beta1, beta2, eps, weight_decay, step) -> np.ndarray:
    """The eight FP32 launch scalars (b1, b2, 1-b1, 1-b2, eps, 1-lr*wd, -lr/bc1, sqrt(bc2))."""
    hp = np.array([lr, beta1, beta2, eps, weight_decay], dtype=np.float64)
    out = np.empty(8, dtype=np.float32)
    lib().srs_o_adamw_scalars(_ptr(hp), int(step), _ptr(out))
    return out


def adamw_core_at(p_addr, p_bf16, g_addr, g_bf16, m_addr, m_fmt, m_rule, v_addr, v_fmt, v_rule,
                  n, scalars, update_key, offset) -> None:
    """AdamW on raw CPU addresses with explicit FP32 scalars (launcher stand-in in tests)."""
    s = np.ascontiguousarray(scalars, dtype=np.float32)
    lib().srs_o_adamw_core(p_addr, p_bf16, g_addr, g_bf16, m_addr, m_fmt, m_rule, v_addr, v_fmt,
                           v_rule, n, _ptr(s), int(update_key) & _MASK32, int(offset) & _MASK32)


def sgdm_core_at(p_addr, p_bf16, g_addr, g_bf16, u_addr, u_fmt, u_rule, n, momentum_f32,
                 neg_lr_f32, update_key, offset) -> None:
    lib().srs_o_sgdm_core(p_addr, p_bf16, g_addr, g_bf16, u_addr, u_fmt, u_rule, n,
                          float(momentum_f32), float(neg_lr_f32), int(update_key) & _MASK32,
                          int(offset) & _MASK32)


def cast_at(x_addr, y_addr, n, fmt, rule, seed, offset) -> None:
    lib().srs_o_cast(x_addr, y_addr, n, fmt, rule, int(seed) & _MASK32, int(offset) & _MASK32)


def check_uniform_division(c, y, first, last, stride, lo, hi):
    """(mismatches, numerators checked) of the reciprocal division; see srs_oracle.c."""
    checked = np.zeros(1, dtype=np.uint64)
    bad = lib().srs_o_check_uniform_division(float(c), float(y), first, last, stride, lo, hi,
                                             _ptr(checked))
    return int(bad), int(checked[0])
