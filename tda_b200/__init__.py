"""tda_b200: B200-native (sm_100a) Threshold (Differential) Attention (forward and backward).

Drop-in for the public API of snap-research/TDA's ``triton_threshold_attention``
module; see ``tda_b200.triton_threshold_attention`` for the same module name.
"""
from . import torch_ops  # noqa: F401  (registers the tda:: torch operators)
from .ops import (  # noqa: F401
    DifferentialThresholdRelaFunction,
    ThresholdRelaFunction,
    check_status,
    diff_forward,
    differential_threshold_rela_triton,
    rect_backward,
    rect_forward,
    threshold_rela_triton,
)

__all__ = [
    "threshold_rela_triton",
    "differential_threshold_rela_triton",
    "ThresholdRelaFunction",
    "DifferentialThresholdRelaFunction",
    "rect_forward",
    "rect_backward",
    "diff_forward",
    "check_status",
]
