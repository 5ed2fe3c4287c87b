"""sr_states on B200: stochastic-rounding optimizer states and casts on sm_100a.

Drop-in for the public API of KristiTopollai/stochastic-rounding-pytorch
(package ``sr_states``).  Optimizer steps and casts run on hand-written sm_100a
CUDA kernels in ``libsrs_b200.so``; Python keeps the bookkeeping (formats,
registry, RNG step, checkpoints) and calls the kernels through a C ABI.
"""

from .formats import StateFormat
from .optim._state import StateOptimizer
from .optim.adamw import AdamWReferenceRN, AdamWReferenceSR
from .optim.sgd import SGDMReferenceRN, SGDMReferenceSR
from .rounding import cast, register_rounding

__all__ = [
    "AdamWReferenceRN",
    "AdamWReferenceSR",
    "SGDMReferenceRN",
    "SGDMReferenceSR",
    "StateFormat",
    "StateOptimizer",
    "cast",
    "register_rounding",
]

__version__ = "0.1.0+b200"
