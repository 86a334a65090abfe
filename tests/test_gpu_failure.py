"""Device-side failure paths, exercised without faulting, trapping or hanging
the GPU.

Every wait of the pipelined tensor-core kernels (tc_select.cu: operand
stages, accumulators, histograms) is bounded; when one runs out, the waiting
role sets the device error flag, the kernel drains and returns, and the host
turns the flag into an error status.  vg_selftest_bounded_wait runs that path
on its own -- a wait on a barrier phase nothing completes, with a limit of
milliseconds -- and the device must still answer searches afterwards.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle as orc
from vicinity_b200 import FlatIndex, VicinityError, selftest_bounded_wait

pytestmark = pytest.mark.gpu


def test_bounded_wait_expires_and_reports():
    assert selftest_bounded_wait(20_000) is True
    # the context stays usable: a tensor-core search right after it is exact
    g = np.random.default_rng(1)
    db = orc.normalize(g.standard_normal((5_000, 64)).astype(np.float32))
    q = orc.normalize(g.standard_normal((50, 64)).astype(np.float32))
    ids, dist = FlatIndex(db).search(q, 10)
    ri, rd, _ = orc.flat_search_ip(db, q, 10)
    assert np.array_equal(ids, ri.astype(np.int64))
    assert np.array_equal(dist.view(np.uint32), rd.view(np.uint32))


def test_bounded_wait_limit_is_validated():
    for bad in (0, 2_000_000):
        with pytest.raises((ValueError, VicinityError)):
            selftest_bounded_wait(bad)
