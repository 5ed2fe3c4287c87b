"""Small helpers shared by the functional entry points."""

from __future__ import annotations

import contextlib

import torch


def device_guard(device):
    return torch.cuda.device(device) if device.type == "cuda" else contextlib.nullcontext()


def stream_handle(device):
    """cudaStream_t of the current stream of ``device`` (None off-GPU)."""
    return torch.cuda.current_stream(device).cuda_stream if device.type == "cuda" else None
