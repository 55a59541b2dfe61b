"""GPU parity of the stream-K GEMV partition: units (tile, k-split) whose records are split across warps, combined
through the context's workspace by the warp that arrives last. Each case is compared with the CPU oracle
(lops.js:30-106 / lops_spec.js:44-157 restated) and, where it matters, with itself: a repeated call must give the
same bits (the parts are summed in a fixed order, and every arrival counter must be back at zero after a call).
"""
import numpy as np
import pytest

import p0pc0rn_b200 as p0
from oracle import ref

from .test_gpu_parity import assert_close, check_mx, nan_buf, wview

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _prefer_stream_k(monkeypatch):
    # the default dispatch sends many of these shapes to other kernels; here every shape that fits goes to v4
    monkeypatch.setenv("P0MM_GEMV", "v4")


def gemvM_call(g, wb, xb, M, N, K, **a):
    ns_guess = a.pop("nsplit", 1)
    yb = nan_buf(g, ns_guess * M * N * 4)
    args = {"w": wview(wb, N, K), "x": {"buf": xb}, "M": M, "N": N, "K": K, "y": {"buf": yb}}
    mxb = None
    if a.get("epi") == "softcap":
        mxb = nan_buf(g, M * (N // 64) * 8, "mx")
        args["mx"] = {"buf": mxb}
    for k in ("norm", "stat"):
        if k in a:
            args[k] = a.pop(k)
    args.update(a)
    ns = p0.gemvM(g, args)
    y = g.read(yb, 0, ns * M * N * 4, np.float32)
    mx = g.read(mxb, 0, M * (N // 64) * 8, np.float32) if mxb is not None else None
    return y, mx, ns


@pytest.mark.parametrize("M,N,K", [(1, 64, 2048), (8, 64, 2048), (3, 4096, 96), (5, 1024, 416), (2, 192, 1024), (7, 16384, 32)])
def test_streamk_shapes(g, M, N, K):
    # one tile over a whole CTA of warps; odd group counts (G = 3, 13, 1); pairs of records straddling tiles
    b, _ = ref.pack_q4(ref.randn(N * K, 200 + K, 0.02), N, K)
    X = ref.randn(M * K, 201 + M)
    wb, xb = g.upload(b), g.upload(X)
    y, _, ns = gemvM_call(g, wb, xb, M, N, K)
    want, _, _ = ref.gemvM(b, X, M, N, K)
    assert ns == 1
    assert_close(y, want)


@pytest.mark.parametrize("M,kPer", [(1, 96), (4, 160), (8, 1024)])
def test_streamk_splits(g, M, kPer):
    # k-splits whose group counts are odd and whose last split is short: each (tile, split) is its own unit
    N, K = 512, 4096
    b, _ = ref.pack_q4(ref.randn(N * K, 210, 0.02), N, K)
    X = ref.randn(M * K, 211)
    wb, xb = g.upload(b), g.upload(X)
    nsw = -(-K // kPer)
    y, _, ns = gemvM_call(g, wb, xb, M, N, K, kPer=kPer, nsplit=nsw)
    want, _, ns_ref = ref.gemvM(b, X, M, N, K, kPer=kPer)
    assert ns == ns_ref == nsw
    assert_close(y, want)


@pytest.mark.parametrize("M,N", [(1, 128), (3, 1024), (8, 8192)])
def test_streamk_softcap(g, M, N):
    # softcap and the per-tile max / argmax from a unit completed by the last-arriving warp
    K = 2048
    b, _ = ref.pack_q4(ref.randn(N * K, 220 + N, 0.02), N, K)
    X = ref.randn(M * K, 221)
    nw = ref.randn(K, 222, 0.1) + 1
    st = np.array([0.8 + 0.03 * m for m in range(M)], np.float32)
    wb, xb = g.upload(b), g.upload(X)
    y, mx, _ = gemvM_call(g, wb, xb, M, N, K, pro="rms", epi="softcap", cap=30.0, norm={"buf": g.upload(nw), "off": 0},
                          stat={"buf": g.upload(st), "off": 0, "ld": 1})
    wy, wmx, _ = ref.gemvM(b, X, M, N, K, pro="rms", epi="softcap", norm=nw, stat=st, stat_off=0, stat_ld=1, cap=30.0)
    assert_close(y, wy)
    NT = N // 64
    for m in range(M):
        check_mx(mx[m * NT * 2:(m + 1) * NT * 2], wmx[m * NT * 2:(m + 1) * NT * 2], wy[m * N:(m + 1) * N], NT)


def test_streamk_repeat_bit_identical(g):
    # the same call three times, with calls of other partitions in between: identical bits every time
    M, N, K = 4, 4096, 2048
    b, _ = ref.pack_q4(ref.randn(N * K, 230, 0.02), N, K)
    X = ref.randn(M * K, 231)
    wb, xb = g.upload(b), g.upload(X)
    b2, _ = ref.pack_q4(ref.randn(192 * 416, 232, 0.02), 192, 416)
    wb2, xb2 = g.upload(b2), g.upload(ref.randn(3 * 416, 233))
    first, _, _ = gemvM_call(g, wb, xb, M, N, K)
    for _ in range(2):
        gemvM_call(g, wb2, xb2, 3, 192, 416)
        again, _, _ = gemvM_call(g, wb, xb, M, N, K)
        assert np.array_equal(first.view(np.uint32), again.view(np.uint32))
    want, _, _ = ref.gemvM(b, X, M, N, K)
    assert_close(first, want)


def test_streamk_layouts_in_sequence(g):
    # calls whose unit counts differ (32, 128, 64, 128 ...): one call's partial sums must never land on the arrival
    # counters a later call uses
    cases = [(1024, 2048, 1024), (8192, 2048, 0), (2048, 2048, 1024), (2048, 8192, 2048), (256, 4096, 512), (8192, 2048, 0)]
    data = {}
    for N, K, kPer in cases:
        if (N, K, kPer) not in data:
            b, _ = ref.pack_q4(ref.randn(N * K, 240 + N + K, 0.02), N, K)
            x = ref.randn(K, 241)
            data[(N, K, kPer)] = (g.upload(b), g.upload(x), ref.gemv(b, x, N, K, kPer=kPer or None)[0])
    for _ in range(2):
        for N, K, kPer in cases:
            wb, xb, want = data[(N, K, kPer)]
            ns = -(-K // kPer) if kPer else 1
            yb = nan_buf(g, ns * N * 4)
            a = {"w": wview(wb, N, K), "x": {"buf": xb}, "N": N, "K": K, "y": {"buf": yb}}
            if kPer:
                a["kPer"] = kPer
            assert p0.gemv(g, a) == ns
            assert_close(g.read(yb, 0, ns * N * 4, np.float32), want)


@pytest.mark.parametrize("M,s0,s1", [(1, 1, 3), (4, 2, 4)])
def test_streamk_kslice_view(g, M, s0, s1):
    # a rank's share of a k-split down projection (p0pc0rn_b200.shard.kslice_args): the weight view starts at a later
    # group of tile 0 with the full tile stride, x at a later element; its partials are slices s0..s1-1 of the full call
    from p0pc0rn_b200 import shard
    N, K, kPer = 512, 4096, 1024
    b, _ = ref.pack_q4(ref.randn(N * K, 250, 0.02), N, K)
    X = ref.randn(M * K, 251)
    wb, xb = g.upload(b), g.upload(X)
    full = {"w": wview(wb, N, K), "x": {"buf": xb, "ldx": K}, "N": N, "K": K, "M": M}
    a = shard.kslice_args(full, kPer, s0, s1)
    ns = s1 - s0
    yb = nan_buf(g, ns * M * N * 4)
    a["y"] = {"buf": yb}
    assert p0.gemvM(g, a) == ns
    got = g.read(yb, 0, ns * M * N * 4, np.float32)
    want, _, _ = ref.gemvM(b, X, M, N, K, kPer=kPer)
    assert_close(got, want.reshape(K // kPer, M * N)[s0:s1].reshape(-1))


@pytest.mark.parametrize("M,N,K", [(1, 64, 2048), (8, 192, 416), (3, 8192, 2048), (2, 1024, 96)])
def test_streamk_geglu(g, M, N, K):
    # geglu units (the gate tile's records, then the up tile's) split across warps, some at the gate / up boundary
    b, _ = ref.pack_q4(ref.randn(2 * N * K, 260 + K, 0.02), 2 * N, K)
    X = ref.randn(M * K, 261)
    nw = ref.randn(K, 262, 0.1) + 1
    st = np.array([0.7 + 0.05 * m for m in range(M)], np.float32)
    wb, xb = g.upload(b), g.upload(X)
    yb = nan_buf(g, M * N * 4)
    a = {"w": wview(wb, 2 * N, K), "x": {"buf": xb}, "M": M, "N": N, "K": K, "y": {"buf": yb}, "pro": "rms", "epi": "geglu",
         "norm": {"buf": g.upload(nw), "off": 0}, "stat": {"buf": g.upload(st), "off": 0, "ld": 1}}
    assert p0.gemvM(g, a) == 1
    want, _, _ = ref.gemvM(b, X, M, N, K, pro="rms", epi="geglu", norm=nw, stat=st, stat_off=0, stat_ld=1)
    assert_close(g.read(yb, 0, M * N * 4, np.float32), want)
