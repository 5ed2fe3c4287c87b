"""Optimizer RNG keys (host side) for the counter-hash stochastic rounding.

Same contract as the reference (sr_states/_hash.py:5-28): a 32-bit avalanche
hash, an update key folded from the low 64 bits of the group seed and of the
global RNG step plus the 32-bit parameter index, and a per-state key.  The
per-element hashes are computed on the GPU inside the fused kernels; the host
needs only these scalar keys (and tests use them as known answers).
"""

from __future__ import annotations

_U32_MASK = 0xFFFFFFFF
_HASH_MUL_1 = 0x7FEB352D
_HASH_MUL_2 = 0x846CA68B


def _h32(value: int) -> int:
    value &= _U32_MASK
    value ^= value >> 16
    value = (value * _HASH_MUL_1) & _U32_MASK
    value ^= value >> 15
    value = (value * _HASH_MUL_2) & _U32_MASK
    return value ^ (value >> 16)


def update_key(seed: int, step: int, param_index: int) -> int:
    """32-bit key of one parameter update (seed and step: low 64 bits)."""
    key = _h32((int(seed) & _U32_MASK) ^ 0x9E3779B9)
    for word in (int(seed) >> 32, int(step), int(step) >> 32, int(param_index)):
        key = _h32(key ^ (word & _U32_MASK))
    return key


def state_key(key: int, state_index: int) -> int:
    """Counter base of one stored state within an update."""
    return _h32((int(key) ^ int(state_index)) & _U32_MASK)


def split_words(value: int) -> tuple[int, int]:
    """Low and high 32-bit words (unsigned) of the low 64 bits of ``value``."""
    value = int(value)
    return value & _U32_MASK, (value >> 32) & _U32_MASK
