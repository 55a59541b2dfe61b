"""GPU parity of the cluster GEMV (v5): one output unit per thread-block cluster, each CTA a k-slice of the unit, the
CTAs' partials summed by rank 0 through distributed shared memory. Every call here is pinned to v5 and compared with
the CPU oracle (lops.js:30-106 / lops_spec.js:44-157 restated); a repeated call must give the same bits.
"""
import numpy as np
import pytest

import p0pc0rn_b200 as p0
from oracle import ref

from .test_gpu_parity import assert_close, check_mx, nan_buf, wview
from .test_gpu_streamk import gemvM_call

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _prefer_cluster(monkeypatch):
    monkeypatch.setenv("P0MM_GEMV", "v5")


@pytest.mark.parametrize("M", [1, 2, 4, 8])
@pytest.mark.parametrize("N,K", [(2048, 2048), (16384, 2048), (2560, 2048), (64, 2048), (1024, 96), (4096, 32)])
def test_cluster_shapes(g, M, N, K):
    # clusters of 8 (N = 64: one unit), 4 (N = 2048 / 2560), 1-2 (N = 16384); odd group counts (G = 3, 1)
    b, _ = ref.pack_q4(ref.randn(N * K, 500 + K, 0.02), N, K)
    X = ref.randn(M * K, 501 + M)
    wb, xb = g.upload(b), g.upload(X)
    y, _, ns = gemvM_call(g, wb, xb, M, N, K)
    want, _, _ = ref.gemvM(b, X, M, N, K)
    assert ns == 1
    assert_close(y, want)
    again, _, _ = gemvM_call(g, wb, xb, M, N, K)
    assert np.array_equal(y.view(np.uint32), again.view(np.uint32))


@pytest.mark.parametrize("M", [1, 4])
def test_cluster_down_splits(g, M):
    # the decode chain's down projection: K 8192 in four kPer 2048 partials, each (tile, split) its own unit
    N, K, kPer = 2048, 8192, 2048
    b, _ = ref.pack_q4(ref.randn(N * K, 510, 0.02), N, K)
    X = ref.randn(M * K, 511)
    wb, xb = g.upload(b), g.upload(X)
    y, _, ns = gemvM_call(g, wb, xb, M, N, K, kPer=kPer, nsplit=4)
    want, _, _ = ref.gemvM(b, X, M, N, K, kPer=kPer)
    assert ns == 4
    assert_close(y, want)


@pytest.mark.parametrize("M,N", [(1, 2048), (4, 8192)])
def test_cluster_softcap(g, M, N):
    K = 2048
    b, _ = ref.pack_q4(ref.randn(N * K, 520 + N, 0.02), N, K)
    X = ref.randn(M * K, 521)
    nw = ref.randn(K, 522, 0.1) + 1
    st = np.array([0.8 + 0.03 * m for m in range(M)], np.float32)
    wb, xb = g.upload(b), g.upload(X)
    y, mx, _ = gemvM_call(g, wb, xb, M, N, K, pro="rms", epi="softcap", cap=30.0, norm={"buf": g.upload(nw), "off": 0},
                          stat={"buf": g.upload(st), "off": 0, "ld": 1})
    wy, wmx, _ = ref.gemvM(b, X, M, N, K, pro="rms", epi="softcap", norm=nw, stat=st, stat_off=0, stat_ld=1, cap=30.0)
    assert_close(y, wy)
    NT = N // 64
    for m in range(M):
        check_mx(mx[m * NT * 2:(m + 1) * NT * 2], wmx[m * NT * 2:(m + 1) * NT * 2], wy[m * N:(m + 1) * N], NT)


@pytest.mark.parametrize("M,N,K", [(1, 8192, 2048), (4, 8192, 2048), (8, 64, 2048), (3, 1024, 96)])
def test_cluster_geglu(g, M, N, K):
    # the decode chain's FFN: gate ranks and up ranks of one cluster, combined by rank 0
    b, _ = ref.pack_q4(ref.randn(2 * N * K, 530 + K, 0.02), 2 * N, K)
    X = ref.randn(M * K, 531)
    nw = ref.randn(K, 532, 0.1) + 1
    st = np.array([0.7 + 0.05 * m for m in range(M)], np.float32)
    wb, xb = g.upload(b), g.upload(X)
    yb = nan_buf(g, M * N * 4)
    a = {"w": wview(wb, 2 * N, K), "x": {"buf": xb}, "M": M, "N": N, "K": K, "y": {"buf": yb}, "pro": "rms", "epi": "geglu",
         "norm": {"buf": g.upload(nw), "off": 0}, "stat": {"buf": g.upload(st), "off": 0, "ld": 1}}
    assert p0.gemvM(g, a) == 1
    want, _, _ = ref.gemvM(b, X, M, N, K, pro="rms", epi="geglu", norm=nw, stat=st, stat_off=0, stat_ld=1)
    assert_close(g.read(yb, 0, M * N * 4, np.float32), want)


def test_cluster_gemv_single_token_forms(g):
    # gemv (M = 1, lops.js) through v5: rms with the stat slot, raw with an offset x row
    N, K = 2560, 2048
    b, _ = ref.pack_q4(ref.randn(N * K, 540, 0.02), N, K)
    x = ref.randn(K + 64, 541)
    nw = ref.randn(K, 542, 0.1) + 1
    st = np.array([0, 0.9, 0, 0], np.float32)
    wb = g.upload(b)
    yb = nan_buf(g, N * 4)
    p0.gemv(g, {"w": wview(wb, N, K), "x": {"buf": g.upload(x), "rowB": 64}, "N": N, "K": K, "y": {"buf": yb}, "pro": "rms",
                "norm": {"buf": g.upload(nw), "off": 0}, "stat": {"buf": g.upload(st), "off": 1}})
    want, _, _ = ref.gemv(b, x, N, K, rowB=64, pro="rms", norm=nw, stat_buf=st, stat_off=1)
    assert_close(g.read(yb, 0, N * 4, np.float32), want)
