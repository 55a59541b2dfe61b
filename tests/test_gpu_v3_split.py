"""The whole-tile streaming GEMV (v3) on calls with fewer tiles than the grid has warps: the column-split vocabulary
head of 2 / 4 / 8 ranks (2048 / 1024 / 512 tiles per rank at K = 2048) and odd group counts. Below 13 tiles per SM (and
at M > 4 below one tile per warp) tiles are cut into k-parts summed in shared memory before the epilogue; the results must match the oracle (lops_spec.js:44-157 restated) within
the parity tolerance, with the per-tile argmax rows equal or tied within 1e-5 (kshipped.js:41-43). P0MM_GEMV=v3 makes
the dispatch take v3 wherever it fits, so the parts path runs whatever the default choice for the shape is.
"""
import numpy as np
import pytest

import p0pc0rn_b200 as p0
from oracle import ref

from .test_gpu_parity import assert_close, nan_buf, wview

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K,parts", [(1, 32768, 2048, None), (8, 32768, 2048, None), (4, 65536, 2048, None),
                                         (2, 24576, 2016, None), (1, 131072, 2048, None), (1, 131072, 2048, "2")])
def test_v3_parts_head(g, monkeypatch, M, N, K, parts):
    # (1, 131072): whole tiles by default (13+ tiles per SM at M <= 4: one tile per warp, some warps idle), k-parts forced
    monkeypatch.setenv("P0MM_GEMV", "v3")
    if parts:
        monkeypatch.setenv("P0MM_V3_PARTS", parts)
    b, _ = ref.pack_q4(ref.randn(N * K, 820 + M, 0.02), N, K)
    X = ref.round_f16(ref.randn(M * K, 821))
    nw = ref.randn(K, 822, 0.1) + 1
    st = np.array([0.9, 1.1, 0.8, 1.0, 0.95, 1.05, 0.85, 1.2][:M], np.float32)
    NT = N // 64
    yb, mxb = nan_buf(g, M * N * 4), nan_buf(g, M * NT * 8, "mx")
    p0.gemvM(g, {"w": wview(g.upload(b), N, K), "x": {"buf": g.upload(X)}, "M": M, "N": N, "K": K, "pro": "rms", "epi": "softcap",
                 "cap": 30.0, "norm": {"buf": g.upload(nw), "off": 0}, "stat": {"buf": g.upload(st), "off": 0, "ld": 1},
                 "y": {"buf": yb}, "mx": {"buf": mxb}})
    g.done()
    y, mx = g.read(yb, 0, M * N * 4, np.float32), g.read(mxb, 0, M * NT * 8, np.float32)
    wy, wmx, _ = ref.gemvM(b, X, M, N, K, pro="rms", epi="softcap", norm=nw, stat=st, stat_ld=1)
    assert_close(y, wy)
    assert_close(mx[0::2], wmx[0::2])
    gi, wi = mx.view(np.uint32)[1::2].astype(np.int64), wmx.view(np.uint32)[1::2].astype(np.int64)
    for t in np.nonzero(gi != wi)[0]:
        m = t // NT
        assert abs(float(wy[m * N + gi[t]]) - float(wy[m * N + wi[t]])) <= 1e-5


def test_v3_parts_store(g, monkeypatch):
    # raw / store, the plain projection form, 512 tiles (8 parts per tile)
    monkeypatch.setenv("P0MM_GEMV", "v3")
    M, N, K = 3, 32768, 1024
    b, _ = ref.pack_q4(ref.randn(N * K, 830, 0.02), N, K)
    X = ref.randn(M * K, 831)
    yb = nan_buf(g, M * N * 4)
    p0.gemvM(g, {"w": wview(g.upload(b), N, K), "x": {"buf": g.upload(X)}, "M": M, "N": N, "K": K, "y": {"buf": yb}})
    g.done()
    want, _, _ = ref.gemvM(b, X, M, N, K)
    assert_close(g.read(yb, 0, M * N * 4, np.float32), want)
