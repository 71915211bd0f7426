"""The tensor-core forward's P.V slab counters (tda_debug_stats), which the
bench uses to report executed tensor-core work beside the algorithmic count.

Cases whose counts follow from the sizes alone:
  * beta = 100: tau exceeds every normalized score, P is zero everywhere, and
    each CTA multiplies only the slab that initialises its O accumulator;
  * beta < 0: every key tile of every query tile is processed (no causal
    skip) and relu(-tau)^p > 0 makes every slab nonzero, so issued == dense.
"""
import pytest
import torch

import tda_b200
from tda_b200 import _lib

pytestmark = pytest.mark.gpu


def _count(fn):
    lib = _lib.load()
    cnt = torch.zeros(2, dtype=torch.int64, device="cuda")
    _lib.check(lib.tda_debug_stats(cnt.data_ptr()))
    try:
        fn()
        torch.cuda.synchronize()
    finally:
        _lib.check(lib.tda_debug_stats(None))
    return [int(x) for x in cnt.tolist()]


@pytest.mark.parametrize("op", ["diff", "rect"])
def test_pv_slab_counters(op):
    B, H, S, D = 1, 2, 640, 128  # 5 query tiles per (batch, head)
    g = torch.Generator().manual_seed(5)
    xs = [torch.randn((B, H, S, D), generator=g).to(torch.bfloat16).cuda() for _ in range(5)]
    n_qt, n_bh = 5, B * H

    def run(beta):
        if op == "diff":
            return lambda: tda_b200.diff_forward(*xs, beta, 0.5, 2.0, True)
        return lambda: tda_b200.rect_forward(xs[0], xs[1], xs[2], beta, 2.0, True)

    issued, dense = _count(run(100.0))
    assert dense == n_bh * (n_qt * (n_qt + 1) // 2) * 8  # causal: key tiles 0..qt per query tile
    assert issued == n_bh * n_qt                          # one slab per CTA
    issued, dense = _count(run(-1.0))
    assert dense == n_bh * n_qt * n_qt * 8                 # beta < 0: every key tile
    assert issued == dense
    # counters off again: a later call leaves them untouched
    lib = _lib.load()
    cnt = torch.zeros(2, dtype=torch.int64, device="cuda")
    run(1.0)()
    torch.cuda.synchronize()
    assert cnt.tolist() == [0, 0]
    tda_b200.check_status()
