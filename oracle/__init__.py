"""CPU oracle for the TDA forward pass -- test infrastructure, not product code.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import it.
"""
from .tda_oracle import (  # noqa: F401
    bf16_round,
    diff_fwd,
    flops,
    l2_normalize,
    rect_fwd,
    rel_l2,
    relu_power,
    tau_vector,
)
