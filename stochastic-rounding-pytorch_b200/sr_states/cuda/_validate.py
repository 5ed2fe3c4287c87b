"""Host-side validation of fused-update inputs, done before anything is launched.

Error types and messages follow the reference (sr_states/triton/_optimizer.py:9-59)
because user code and tests match on them.
"""

from __future__ import annotations

import math

import torch

BLOCK_SIZES = (128, 256, 512, 1024)
CAST_BLOCK_SIZES = (128, 256, 512, 1024, 2048, 4096)
CAST_NUM_WARPS = (1, 2, 4, 8)
CAST_STORE_MODES = ("convert", "bits")
PARAMETER_DTYPES = (torch.float32, torch.bfloat16)
_OVERLAP = "parameter, gradient, and state must not overlap optimizer writes"


def check_nonnegative(name: str, value) -> None:
    if not math.isfinite(value) or value < 0:
        raise ValueError(f"invalid {name}: {value}")


def check_block_size(block_size) -> None:
    """The launch configuration is the library's own; the option is kept for API parity."""
    if block_size not in BLOCK_SIZES:
        raise ValueError(f"block_size must be one of {BLOCK_SIZES}")


def check_layout(tensors) -> None:
    """Same device, identical shapes, contiguous; parameter/gradient FP32 or BF16."""
    first = tensors[0]
    for t in tensors:
        if t.device != first.device:
            raise ValueError("all tensors must be on the same CUDA device")
        if t.shape != first.shape:
            raise ValueError("all tensors must have identical shapes")
        if not t.is_contiguous():
            raise ValueError("fused state updates require contiguous tensors")
    if first.dtype not in PARAMETER_DTYPES or tensors[1].dtype not in PARAMETER_DTYPES:
        raise TypeError("parameter and gradient must be FP32 or BF16")


def check_disjoint(spans) -> None:
    """Byte spans (start, end, written) of one device.  Anything the update writes
    must be disjoint from every other span; read-only spans (gradients) may share."""
    reach_any = reach_written = 0
    for start, end, written in sorted(spans):
        if start < (reach_any if written else reach_written):
            raise ValueError(_OVERLAP)
        reach_any = max(reach_any, end)
        if written:
            reach_written = max(reach_written, end)


def spans_of(tensors, numel: int):
    """(start, end, written) byte spans of one update's tensors; index 1 is the gradient."""
    return [(t.data_ptr(), t.data_ptr() + numel * t.element_size(), role != 1)
            for role, t in enumerate(tensors)]
