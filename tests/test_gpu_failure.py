"""The failure path of the in-kernel waits, exercised without a GPU fault: a kernel's bounded mbarrier wait that
nothing completes gives up after a short limit, records its code in the context's error word and returns; p0_done
reports P0_ETIMEOUT (the reference surfaces device failures at done(), engine/core/gpu.js:141-147) and the same
context then runs GEMV calls that match the oracle.
"""
import numpy as np
import pytest

import p0pc0rn_b200 as p0
from p0pc0rn_b200 import _lib as L
from oracle import ref

from .test_gpu_parity import assert_close, nan_buf, wview

pytestmark = pytest.mark.gpu


def _gemv_ok(g, seed):
    N, K = 256, 2048
    b, _ = ref.pack_q4(ref.randn(N * K, seed, 0.02), N, K)
    X = ref.randn(K, seed + 1)
    yb = nan_buf(g, N * 4)
    p0.gemv(g, {"w": wview(g.upload(b), N, K), "x": {"buf": g.upload(X)}, "N": N, "K": K, "y": {"buf": yb}})
    g.done()
    want, _, _ = ref.gemv(b, X, N, K)
    assert_close(g.read(yb, 0, N * 4, np.float32), want)


def test_bounded_wait_gives_up_and_context_stays_usable(g):
    _gemv_ok(g, 500)
    g.wait_selftest(4096)
    with pytest.raises(p0.P0Error) as ei:
        g.done(10000)
    assert ei.value.status == L.P0_ETIMEOUT
    assert "0x7e1" in str(ei.value)
    # the error word was cleared by the report: the next done() is clean, and the kernels still compute
    g.done()
    _gemv_ok(g, 510)
    # twice in a row behaves the same
    g.wait_selftest(1)
    with pytest.raises(p0.P0Error):
        g.done(10000)
    _gemv_ok(g, 520)


def test_wait_selftest_rejects_bad_limits(g):
    for polls in (0, (1 << 20) + 1):
        with pytest.raises(p0.P0Error, match="polls"):
            g.wait_selftest(polls)
