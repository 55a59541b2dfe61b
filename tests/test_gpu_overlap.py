"""GEMV calls that overlap on the GPU (programmatic dependent launch, and with p0_set_overlap the weight fetch ahead
of the call in front): a chain in which every call reads the output of the call before it, and one call overwrites
the input of an earlier one. Every link is checked against the CPU oracle (lops.js / lops_spec.js restated) fed the
link's actual input, so a call that read its input before the call ahead had written it, or wrote its output while
the call ahead still read it, fails. The chain mixes the kernels the dispatch picks (cluster, whole-tile, fallback)."""
import numpy as np
import pytest

import p0pc0rn_b200 as p0
from oracle import ref

from .test_gpu_parity import assert_close, nan_buf, wview

pytestmark = pytest.mark.gpu

# (M, N, K): each link reads the previous link's output (the M = 4 links as [4][K] rows)
LINKS = [(1, 2048, 2048), (1, 3072, 2048), (1, 2048, 3072), (4, 2048, 512), (4, 16384, 2048), (4, 2048, 16384)]


@pytest.mark.parametrize("overlap", [False, True])
def test_dependent_chain(g, overlap):
    g.set_overlap(overlap)
    try:
        ws = []
        for i, (M, N, K) in enumerate(LINKS):
            b, _ = ref.pack_q4(ref.randn(N * K, 600 + i, 0.02), N, K)
            ws.append((b, g.upload(b)))
        g.done()
        x0 = ref.randn(2048, 610)
        cur = g.upload(x0)
        bufs = [cur]
        for (M, N, K), (b, wb) in zip(LINKS, ws):
            yb = nan_buf(g, M * N * 4)
            a = {"w": wview(wb, N, K), "x": {"buf": cur, "ldx": K}, "N": N, "K": K, "y": {"buf": yb}}
            if M == 1:
                p0.gemv(g, a)
            else:
                p0.gemvM(g, dict(a, M=M))
            bufs.append(yb)
            cur = yb
        # overwrite the first link's input with a call that reads the last output (a write after an earlier read)
        No, Ko = 2048, 2048
        bo, _ = ref.pack_q4(ref.randn(No * Ko, 620, 0.02), No, Ko)
        wbo = g.upload(bo)
        g.done()
        p0.gemv(g, {"w": wview(wbo, No, Ko), "x": {"buf": bufs[-1]}, "N": No, "K": Ko, "y": {"buf": bufs[0]}})
        outs = [g.read(bb, 0, None, np.float32) for bb in bufs]
        xin = x0
        for (M, N, K), (b, _), out in zip(LINKS, ws, outs[1:]):
            X = np.ascontiguousarray(xin[:M * K], np.float32)
            want = ref.gemv(b, X, N, K)[0] if M == 1 else ref.gemvM(b, X, M, N, K)[0]
            assert_close(out[:M * N], want)
            xin = out
        assert_close(outs[0][:No], ref.gemv(bo, outs[-1][:Ko], No, Ko)[0])
    finally:
        g.set_overlap(False)
