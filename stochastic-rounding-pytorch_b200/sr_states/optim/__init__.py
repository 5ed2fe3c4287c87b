"""Optimizers: the bookkeeping base and the fused AdamW / momentum-SGD classes."""

from ._state import StateOptimizer
from .adamw import AdamWReferenceRN, AdamWReferenceSR
from .sgd import SGDMReferenceRN, SGDMReferenceSR

__all__ = ["AdamWReferenceRN", "AdamWReferenceSR", "SGDMReferenceRN", "SGDMReferenceSR",
           "StateOptimizer"]
