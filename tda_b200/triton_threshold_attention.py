"""Same module name and public names as the reference's
``triton_threshold_attention.py`` (snap-research/TDA), so callers can switch
with one import change:

    from tda_b200.triton_threshold_attention import (
        threshold_rela_triton, differential_threshold_rela_triton)

No Triton is involved; the calls go to the tda_b200 CUDA library.
"""
from .ops import (  # noqa: F401
    ThresholdRelaFunction,
    differential_threshold_rela_triton,
    threshold_rela_triton,
)

__all__ = ["threshold_rela_triton", "differential_threshold_rela_triton", "ThresholdRelaFunction"]
