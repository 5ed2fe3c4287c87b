"""Import-compatible names for code written against the reference's Triton backend.

Every name here is the sm_100a CUDA implementation from ``sr_states.cuda``;
no Triton code is imported or run.  ``from sr_states.triton import AdamWTriton``
therefore keeps working unchanged.
"""

from ..cuda import AdamWCuda, SGDMCuda, cast, rn_cast_bf16, sr_cast_bf16
from ..cuda import cuda_adamw_step_ as triton_adamw_step_
from ..cuda import cuda_sgdm_step_ as triton_sgdm_step_
from ..cuda import is_available as is_triton_available


class AdamWTriton(AdamWCuda):
    """AdamWCuda under the reference's name (sr_states/triton/adamw.py); rule
    validation names the Triton backend, as the reference's messages do."""

    _rounding_backend = "triton"


class SGDMTriton(SGDMCuda):
    """SGDMCuda under the reference's name (sr_states/triton/sgd.py); rule
    validation names the Triton backend, as the reference's messages do."""

    _rounding_backend = "triton"


__all__ = [
    "AdamWTriton",
    "SGDMTriton",
    "cast",
    "is_triton_available",
    "rn_cast_bf16",
    "sr_cast_bf16",
    "triton_adamw_step_",
    "triton_sgdm_step_",
]
