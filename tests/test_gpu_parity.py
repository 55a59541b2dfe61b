"""GPU parity: the CUDA kernels of libp0mm.so (through the C ABI, via the reference-shaped ops) against the CPU oracle
and the committed fixtures. Tolerances: on fp16-rounded outputs max-abs <= 1e-2 and rel-L2
<= 1e-3; the packer and the GEMM's dequantised weights bit-exact. Outputs are NaN-poisoned before each call
(tune/autotune.js:135) so a kernel that did not write fails.
"""
import json
import math
import os

import numpy as np
import pytest

import p0pc0rn_b200 as p0
from oracle import ref

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
MAXABS, RELL2 = 1e-2, 1e-3


def f16r(a):
    return np.asarray(a, np.float32).astype(np.float16).astype(np.float64)


def assert_close(got, want, maxabs=MAXABS, rel=RELL2):
    g, w = f16r(got), f16r(want)
    assert np.all(np.isfinite(g)), "non-finite output (a slot the kernel did not write?)"
    err = float(np.max(np.abs(g - w))) if g.size else 0.0
    rl2 = float(np.sqrt(np.sum((g - w) ** 2) / max(1e-300, np.sum(w ** 2))))
    assert err <= maxabs and rl2 <= rel, "max-abs %.3g rel-L2 %.3g" % (err, rl2)
    return err, rl2


def nan_buf(g, nbytes, label="y"):
    return g.upload(np.full(nbytes // 4, np.nan, np.float32), label)


def wview(buf, N, K, off=0):
    return {"buf": buf, "off": off, "enc": "q4g32a.t64", "rows": N, "cols": K}


def gold(name, key):
    with open(os.path.join(GOLD, "manifest.json")) as f:
        e = json.load(f)[name][key]
    return np.fromfile(os.path.join(GOLD, e["file"]), dtype=e["dtype"])


# ---------------------------------------------------------------- quantiser and dequantiser: bit-exact
@pytest.mark.parametrize("N,K,seed,scale", [(64, 256, 11, 0.05), (256, 2048, 0, 0.02), (128, 96, 3, 1.0)])
def test_pack_q4_bit_exact(g, N, K, seed, scale):
    W = ref.randn(N * K, seed, scale)
    W[:32] = 0.25                                                   # constant group -> s = 1
    W[K:K + 32] = np.linspace(1.0, 1.0 + 3e-6, 32, dtype=np.float32)  # subnormal fp16 scale
    if N >= 128:
        W[2 * K:2 * K + 32] = np.linspace(-60000, 60000, 32, dtype=np.float32)
    want, _ = ref.pack_q4(W, N, K)
    wb = g.upload(W)
    out = p0.pack_q4(g, wb, N, K)
    got = g.read(out, 0, want.size)
    assert np.array_equal(got, want)


def test_pack_fixture(g):
    W = ref.randn(64 * 256, 11, 0.05)
    out = p0.pack_q4(g, g.upload(W), 64, 256)
    assert np.array_equal(g.read(out, 0, 10240), gold("pack", "bytes"))


@pytest.mark.parametrize("N,K", [(64, 256), (192, 3072)])
def test_dequant_bit_exact(g, N, K):
    b, _ = ref.pack_q4(ref.randn(N * K, 5, 0.02), N, K)
    wb = g.upload(b)
    out = g.buffer(N * K * 2)
    p0.dequant_f16(g, wview(wb, N, K), out)
    assert np.array_equal(g.read(out, 0, N * K * 2, np.uint16), ref.deq16(b, N, K).ravel())


def test_dequant_edge_groups(g):
    # groups whose q*s + mn is not exact in f32 (scale and min far apart in exponent) take the f32 path of the
    # dequantiser, the others its fp16 fma path: both must give f16(f32(q*s + mn)) bit for bit
    N, K = 128, 512
    W = ref.randn(N * K, 9, 0.02).reshape(N, K)
    rng = np.random.default_rng(5)
    for r in range(N):
        for gi in range(K // 32):
            kind = (r * 7 + gi) % 6
            sl = W[r, gi * 32:(gi + 1) * 32]
            if kind == 1:      # large offset, tiny range: Em - Es large
                sl[:] = np.float32(1000.0 + rng.uniform(0, 1e-3, 32))
            elif kind == 2:    # minimum near zero, wide range: Es - Em large
                sl[:] = np.float32(rng.uniform(0, 50.0, 32))
                sl[0] = np.float32(1e-7)
            elif kind == 3:    # negative offset, subnormal scale
                sl[:] = np.float32(-2.0 - rng.uniform(0, 2e-6, 32))
            elif kind == 4:    # huge values near the fp16 limit
                sl[:] = np.float32(rng.uniform(-60000, 60000, 32))
    b, _ = ref.pack_q4(W.ravel(), N, K)
    out = g.buffer(N * K * 2)
    p0.dequant_f16(g, wview(g.upload(b), N, K), out)
    assert np.array_equal(g.read(out, 0, N * K * 2, np.uint16), ref.deq16(b, N, K).ravel())


def test_dequant_fixture(g):
    b = gold("pack", "bytes")
    out = g.buffer(64 * 256 * 2)
    p0.dequant_f16(g, wview(g.upload(b), 64, 256), out)
    assert np.array_equal(g.read(out, 0, 64 * 256 * 2, np.uint16), gold("pack", "deq16"))


# ---------------------------------------------------------------- GEMV
def run_gemv(g, b, x, N, K, y_bytes, mx_bytes=0, extra=None, **a):
    wb, xb = g.upload(b), g.upload(np.ascontiguousarray(x, np.float32))
    yb = nan_buf(g, y_bytes)
    args = {"w": wview(wb, a.pop("rows", N), K), "x": {"buf": xb, "rowB": a.pop("rowB", 0)}, "N": N, "K": K, "y": {"buf": yb}}
    args.update(a)
    mxb = None
    if mx_bytes:
        mxb = g.upload(extra["mx"]) if extra and "mx" in extra else nan_buf(g, mx_bytes, "mx")
        args["mx"] = {"buf": mxb}
    if extra:
        for k in ("norm", "ev", "stat"):
            if k in extra:
                args[k] = {"buf": g.upload(extra[k][0]), "off": extra[k][1]}
    ns = p0.gemv(g, args)
    y = g.read(yb, 0, y_bytes, np.float32)
    mx = g.read(mxb, 0, mx_bytes, np.float32) if mxb is not None else None
    return y, mx, ns


def test_gemv_config1(g):
    # config 1: M=1, K=2048, N=8192, W ~N(0, 0.02) seed 0, x fp16 ~N(0, 1)
    N, K = 8192, 2048
    b, _ = ref.pack_q4(ref.randn(N * K, 0, 0.02), N, K)
    x = ref.round_f16(ref.randn(K, 1))
    y, _, ns = run_gemv(g, b, x, N, K, N * 4)
    want, _, _ = ref.gemv(b, x, N, K)
    assert ns == 1
    assert_close(y, want)


def test_gemv_fixture(g):
    N, K = 256, 2048
    b, _ = ref.pack_q4(ref.randn(N * K, 0, 0.02), N, K)
    y, _, _ = run_gemv(g, b, ref.round_f16(ref.randn(K, 1)), N, K, N * 4)
    assert_close(y, gold("gemv_raw", "y"))


@pytest.mark.parametrize("K,kPer", [(8192, 2048), (4096, 1024), (2048, 0), (3072, 0), (256, 0)])
def test_gemv_splits(g, K, kPer):
    N = 2048
    b, _ = ref.pack_q4(ref.randn(N * K, 40 + K, 0.02), N, K)
    x = ref.randn(K, 41)
    kw = {"kPer": kPer} if kPer else {}
    ns_want = -(-K // kPer) if kPer else 1
    y, _, ns = run_gemv(g, b, x, N, K, ns_want * N * 4, **kw)
    want, _, nsw = ref.gemv(b, x, N, K, kPer=kPer or None)
    assert ns == nsw == ns_want
    assert_close(y, want)


def test_gemv_rms_softcap_head(g):
    # the head's call shape (gemma4.js:505-509): rms prologue reading rstd from the mx buffer past the tile slots
    N, K = 4096, 2048
    b, _ = ref.pack_q4(ref.randn(N * K, 50, 0.02), N, K)
    x = ref.randn(K, 51)
    nw = ref.randn(K, 52, 0.1) + 1
    NT = N // 64
    mx = np.full(NT * 2 + 4, np.nan, np.float32)
    mx[NT * 2] = 0.8
    y, MX, _ = run_gemv(g, b, x, N, K, N * 4, mx_bytes=mx.nbytes, extra={"mx": mx, "norm": (nw, 0)}, pro="rms", epi="softcap",
                        stat={"buf": None, "off": NT * 2}, cap=30.0)
    wy, wmx, _ = ref.gemv(b, x, N, K, pro="rms", epi="softcap", norm=nw, stat_off=NT * 2, mx=mx.copy(), cap=30.0)
    assert_close(y, wy)
    check_mx(MX[:NT * 2], wmx[:NT * 2], wy, NT)


def check_mx(got, want, yref, ntile):
    gu, wu = got.view(np.uint32), want.view(np.uint32)
    for t in range(ntile):
        gi, wi = int(gu[2 * t + 1]), int(wu[2 * t + 1])
        # argmax equal, or tied within 1e-5 (kshipped.js:41)
        assert gi == wi or abs(float(yref[gi]) - float(yref[wi])) <= 1e-5, (t, gi, wi)
        assert abs(float(got[2 * t]) - float(want[2 * t])) <= 1e-2


def test_gemv_fixture_softcap(g):
    N, K = 128, 1536
    b, _ = ref.pack_q4(ref.randn(N * K, 33 + K, 0.05), N, K)
    x = ref.randn(K, 34 + K)
    nw = np.array([0.9 + 0.2 * ((i * 7919) % 100) / 100 for i in range(K)], np.float32)
    mx = np.zeros(N // 64 * 2 + 4, np.float32)
    mx[N // 64 * 2] = 0.75
    y, MX, _ = run_gemv(g, b, x, N, K, N * 4, mx_bytes=mx.nbytes, extra={"mx": mx, "norm": (nw, 0)}, pro="rms", epi="softcap",
                        stat={"off": N // 64 * 2}, cap=30.0)
    assert_close(y, gold("gemv_rms_softcap", "y"))
    check_mx(MX[:4], gold("gemv_rms_softcap", "mx")[:4], gold("gemv_rms_softcap", "y"), 2)


def test_gemv_geglu(g):
    N, K = 2048, 2048
    b, _ = ref.pack_q4(ref.randn(2 * N * K, 60, 0.02), 2 * N, K)
    x = ref.randn(K, 61)
    nw = ref.randn(K, 62, 0.1) + 1
    st = np.array([0, 1.25, 0, 0], np.float32)
    y, _, _ = run_gemv(g, b, x, N, K, N * 4, extra={"norm": (nw, 0), "stat": (st, 1)}, pro="rms", epi="geglu", rows=2 * N)
    want, _, _ = ref.gemv(b, x, N, K, pro="rms", epi="geglu", norm=nw, stat_buf=st, stat_off=1)
    assert_close(y, want)


def test_gemv_fixture_geglu(g):
    N, K = 128, 512
    b, _ = ref.pack_q4(ref.randn(2 * N * K, 5, 0.05), 2 * N, K)
    st = np.array([0, 1.25, 0, 0], np.float32)
    nw = ref.randn(K, 6, 0.1) + 1
    y, _, _ = run_gemv(g, b, ref.randn(K, 7), N, K, N * 4, extra={"norm": (nw, 0), "stat": (st, 1)}, pro="rms", epi="geglu", rows=2 * N)
    assert_close(y, gold("gemv_geglu", "y"))


@pytest.mark.parametrize("pro", ["sum", "pleg"])
def test_gemv_sum_pleg(g, pro):
    # the PLE path (gemma4.js:489-495): K=256, partials summed in the prologue (+ gelu * per-layer vector)
    N, K, nsrc = 2048, 256, 3
    b, _ = ref.pack_q4(ref.randn(N * K, 70, 0.02), N, K)
    X = ref.randn(nsrc * K, 71)
    ev = ref.randn(K + 64, 72, 0.5)
    y, _, _ = run_gemv(g, b, X, N, K, N * 4, extra={"ev": (ev, 64)}, pro=pro, src={"n": nsrc, "ld": K})
    want, _, _ = ref.gemv(b, X, N, K, pro=pro, src=(K, nsrc), ev=ev, ev_off=64)
    assert_close(y, want)


def test_gemv_offsets(g):
    # a weight view inside a larger buffer (off), x at rowB, ldy > N
    N, K = 1024, 1024
    b, _ = ref.pack_q4(ref.randn(N * K, 80, 0.02), N, K)
    pad = np.zeros(4096, np.uint8)
    wb = g.upload(np.concatenate([pad, b]))
    x = ref.randn(K + 100, 81)
    xb = g.upload(x)
    ldy = N + 64
    yb = nan_buf(g, ldy * 4)
    p0.gemv(g, {"w": wview(wb, N, K, off=4096), "x": {"buf": xb, "rowB": 100}, "N": N, "K": K, "y": {"buf": yb}, "ldy": ldy})
    y = g.read(yb, 0, N * 4, np.float32)
    want, _, _ = ref.gemv(b, x, N, K, rowB=100)
    assert_close(y, want)


# ---------------------------------------------------------------- gemvM
def run_gemvM(g, b, X, M, N, K, y_floats, mx_floats=0, extra=None, **a):
    wb, xb = g.upload(b), g.upload(np.ascontiguousarray(X, np.float32))
    yb = nan_buf(g, y_floats * 4)
    args = {"w": wview(wb, a.pop("rows", N), K), "x": {"buf": xb, "ldx": a.pop("ldx", 0), "rowB": a.pop("rowB", 0)}, "M": M, "N": N,
            "K": K, "y": {"buf": yb, "ldm": a.pop("ldm", 0), "ldy": a.pop("ldy", 0)}}
    args.update(a)
    mxb = None
    if mx_floats:
        mxb = nan_buf(g, mx_floats * 4, "mx")
        args["mx"] = {"buf": mxb}
    if extra:
        for k in ("norm", "ev", "stat"):
            if k in extra:
                args[k] = {"buf": g.upload(extra[k][0]), "off": extra[k][1], "ld": extra[k][2] if len(extra[k]) > 2 else 0}
    ns = p0.gemvM(g, args)
    return g.read(yb, 0, y_floats * 4, np.float32), (g.read(mxb, 0, mx_floats * 4, np.float32) if mxb is not None else None), ns


@pytest.mark.parametrize("M", [1, 2, 4, 8])
@pytest.mark.parametrize("N", [2048, 16384])
def test_gemvM_config2(g, M, N):
    K = 2048
    b, _ = ref.pack_q4(ref.randn(N * K, 90, 0.02), N, K)
    X = ref.round_f16(ref.randn(M * K, 91 + M))
    y, _, ns = run_gemvM(g, b, X, M, N, K, M * N)
    want, _, _ = ref.gemvM(b, X, M, N, K)
    assert ns == 1
    assert_close(y, want)


_HEAD = {}


def head_weights(N, K):
    if (N, K) not in _HEAD:
        _HEAD[(N, K)] = ref.pack_q4(ref.randn(N * K, 100, 0.02), N, K)[0]
    return _HEAD[(N, K)]


@pytest.mark.parametrize("M", [1, 2, 4, 8])
def test_gemvM_head_softcap(g, M):
    # the verify head (spec.js:164): rms + softcap over the vocab (config 2's N = 262144), per-row per-tile max/argmax
    N, K = 262144, 2048
    b = head_weights(N, K)
    X = ref.randn(M * K, 101)
    nw = ref.randn(K, 102, 0.1) + 1
    st = np.array([0.9 + 0.05 * m for m in range(M)], np.float32)
    NT = N // 64
    y, MX, _ = run_gemvM(g, b, X, M, N, K, M * N, mx_floats=M * NT * 2, extra={"norm": (nw, 0), "stat": (st, 0, 1)},
                         pro="rms", epi="softcap", cap=30.0)
    wy, wmx, _ = ref.gemvM(b, X, M, N, K, pro="rms", epi="softcap", norm=nw, stat=st, stat_off=0, stat_ld=1, cap=30.0)
    assert_close(y, wy)
    gu, wu = MX.view(np.uint32), wmx.view(np.uint32)
    ties = 0
    for m in range(M):
        gi, wi = gu[1::2][m * NT:(m + 1) * NT].astype(np.int64), wu[1::2][m * NT:(m + 1) * NT].astype(np.int64)
        diff = np.nonzero(gi != wi)[0]
        yr = wy[m * N:(m + 1) * N]
        for t in diff:
            assert abs(float(yr[gi[t]]) - float(yr[wi[t]])) <= 1e-5
        ties += diff.size
    assert ties <= 4


def test_gemvM_split_fixture(g):
    M, N, K = 4, 128, 2048
    b, _ = ref.pack_q4(ref.randn(N * K, 8, 0.02), N, K)
    y, _, ns = run_gemvM(g, b, ref.randn(M * K, 9), M, N, K, 4 * M * N, kPer=512)
    assert ns == 4
    assert_close(y, gold("gemvM_split", "y"))


def test_gemvM_geglu_pleg_ld(g):
    M, N, K = 4, 1024, 1024
    b, _ = ref.pack_q4(ref.randn(2 * N * K, 110, 0.02), 2 * N, K)
    X = ref.randn(M * (K + 32), 111)
    nw = ref.randn(K, 112, 0.1) + 1
    st = np.array([0.7, 0, 0.8, 0, 0.9, 0, 1.0, 0], np.float32)
    y, _, _ = run_gemvM(g, b, X, M, N, K, M * (N + 64), extra={"norm": (nw, 0), "stat": (st, 0, 2)}, pro="rms", epi="geglu",
                        rows=2 * N, ldx=K + 32, ldm=N + 64)
    want, _, _ = ref.gemvM(b, X, M, N, K, pro="rms", epi="geglu", norm=nw, stat=st, stat_ld=2, ldx=K + 32, ldm=N + 64)
    for m in range(M):
        assert_close(y[m * (N + 64):m * (N + 64) + N], want[m * (N + 64):m * (N + 64) + N])
    # pleg with per-row ev
    b2, _ = ref.pack_q4(ref.randn(N * 256, 113, 0.02), N, 256)
    X2 = ref.randn(2 * M * 256, 114)
    ev = ref.randn(M * 256, 115, 0.5)
    y2, _, _ = run_gemvM(g, b2, X2, M, N, 256, M * N, extra={"ev": (ev, 0, 256)}, pro="pleg", src={"n": 2, "ld": M * 256})
    want2, _, _ = ref.gemvM(b2, X2, M, N, 256, pro="pleg", ev=ev, ev_ld=256, src=(M * 256, 2))
    assert_close(y2, want2)


# ---------------------------------------------------------------- GEMM
def run_gemm(g, b, X16, M, N, K, y_init=None, y_bytes=None, **a):
    wb, xb = g.upload(b), g.upload(X16)   # X16: fp16 bits, or f32 for the x prologues
    f32y = a.get("epi") in ("f32", "resadd")
    ldy = a.get("y", {}).get("ld") or (N // 2 if a.get("epi") == "swiglu" else N)
    nb = y_bytes or M * ldy * (4 if f32y else 2)
    yb = g.upload(y_init) if y_init is not None else g.upload(np.full(nb // 2, 0x7E00, np.uint16))
    args = {"w": wview(wb, a.pop("rows", N), a.pop("cols", K)), "x": {"buf": xb, **a.pop("x", {})}, "M": M, "N": N, "K": K,
            "y": {"buf": yb, **a.pop("y", {})}}
    if "enc" in a:
        args["w"]["enc"] = a.pop("enc")
    for k in ("ev", "bv"):
        if k in a:
            v = a.pop(k)
            args[k] = {"buf": g.upload(v[0]), "off": v[1], **({"up": v[2]} if len(v) > 2 else {})}
    a.pop("stats", None)
    a.pop("pv", None)
    if "_stats" in a:   # x prologue inputs: stats (rows of {mean, rstd}) and pv vectors
        v = a.pop("_stats")
        args["stats"] = {"buf": g.upload(v[0]), "off": v[1]}
    if "_pv" in a:
        v = a.pop("_pv")
        args["pv"] = {"buf": g.upload(v[0]), "off": v[1], "stride": v[2]}
    args.update(a)
    fl = p0.gemm(g, args)
    assert fl == 2.0 * M * N * K
    return g.read(yb, 0, nb, np.float32 if f32y else np.uint16)


@pytest.mark.parametrize("M,N,K", [(32, 128, 256), (300, 384, 320), (129, 256, 2048), (1000, 640, 1024), (4, 128, 64)])
def test_gemm_f16(g, M, N, K):
    b, _ = ref.pack_q4(ref.randn(N * K, 120 + M, 0.02), N, K)
    X = ref.f2h(ref.round_f16(ref.randn(M * K, 121)))
    y = run_gemm(g, b, X, M, N, K)
    want = ref.gemm(b, X, M, N, K)
    assert_close(ref.h2f(y), ref.h2f(want))


def test_gemm_fixture(g):
    M, N, K = 32, 128, 256
    b, _ = ref.pack_q4(ref.randn(N * K, 11, 0.05), N, K)
    y = run_gemm(g, b, ref.f2h(ref.round_f16(ref.randn(M * K, 7))), M, N, K)
    assert_close(ref.h2f(y), ref.h2f(gold("gemm_f16", "y")))


def test_gemm_bias_gelu_fixture(g):
    M, N, K = 48, 128, 320
    b, _ = ref.pack_q4(ref.randn(N * K, 12, 0.02), N, K)
    y = run_gemm(g, b, ref.f2h(ref.round_f16(ref.randn(M * K, 14))), M, N, K, epi="bias", ev=(ref.randn(N, 13, 0.01), 0), post_gelu=True)
    assert_close(ref.h2f(y), ref.h2f(gold("gemm_bias_gelu", "y")))


@pytest.mark.parametrize("res", [False, True])
def test_gemm_bias(g, res):
    M, N, K = 200, 256, 512
    b, _ = ref.pack_q4(ref.randn(N * K, 130, 0.02), N, K)
    X = ref.f2h(ref.round_f16(ref.randn(M * K, 131)))
    bias = ref.randn(N + 8, 132, 0.01)
    y0 = ref.f2h(ref.randn(M * N, 133, 0.5))
    y = run_gemm(g, b, X, M, N, K, y_init=y0.copy(), epi="bias", ev=(bias, 8), res=res)
    want = ref.gemm(b, X, M, N, K, epi="bias", ev=bias, ev_off=8, res=res, Y=y0.copy())
    assert_close(ref.h2f(y), ref.h2f(want))


@pytest.mark.parametrize("act", ["silu", "gelu"])
def test_gemm_swiglu(g, act):
    M, N, K = 130, 512, 256
    b, _ = ref.pack_q4(ref.randn(N * K, 140, 0.02), N, K)
    X = ref.f2h(ref.round_f16(ref.randn(M * K, 141)))
    bv = ref.randn(N, 142, 0.01)
    # y.ld defaults to N (the weight-column count, gemm.js:313) even for swiglu: the output rows are N/2 wide here
    y = run_gemm(g, b, X, M, N, K, epi="swiglu", act=act, wr0=0, wr1=N // 2, bv=(bv, 0, N // 2), y={"ld": N // 2})
    want = ref.gemm(b, X, M, N, K, epi="swiglu", act=act, wr0=0, wr1=N // 2, bv=bv, bv_up=N // 2, ldy=N // 2)
    assert_close(ref.h2f(y), ref.h2f(want))


def test_gemm_swiglu_fixture(g):
    M, N, K = 40, 256, 256
    b, _ = ref.pack_q4(ref.randn(N * K, 15, 0.02), N, K)
    y = run_gemm(g, b, ref.f2h(ref.round_f16(ref.randn(M * K, 17))), M, N, K, epi="swiglu", act="gelu", wr0=0, wr1=N // 2,
                 bv=(ref.randn(N, 16, 0.01), 0, N // 2), y={"ld": N // 2})
    assert_close(ref.h2f(y), ref.h2f(gold("gemm_swiglu", "y")))


@pytest.mark.parametrize("store", [False, True])
def test_gemm_resadd_f32(g, store):
    M, N, K = 100, 256, 384
    b, _ = ref.pack_q4(ref.randn(N * K, 150, 0.02), N, K)
    X = ref.f2h(ref.round_f16(ref.randn(M * K, 151)))
    gate, bv = ref.randn(N, 152, 1.0), ref.randn(N, 153, 0.01)
    r0 = ref.randn(M * N, 154)
    y = run_gemm(g, b, X, M, N, K, y_init=r0.copy(), epi="resadd", ev=(gate, 0), bv=(bv, 0), store=store)
    want = ref.gemm(b, X, M, N, K, epi="resadd", ev=gate, bv=bv, store=store, Y=r0.copy())
    assert_close(y, want)
    yf = run_gemm(g, b, X, M, N, K, y_bytes=M * N * 4, epi="f32")
    assert_close(yf, ref.gemm(b, X, M, N, K, epi="f32"))


def test_gemm_subviews(g):
    # wr0 / wk0 / x.k0 / x.ld / y.ld / y.n0: a sub-matrix of a larger weight into a column range of a wider Y
    Nw, Kw, M, N, K = 512, 1024, 96, 256, 512
    b, _ = ref.pack_q4(ref.randn(Nw * Kw, 160, 0.02), Nw, Kw)
    ldx, k0 = Kw + 64, 256
    X = ref.f2h(ref.round_f16(ref.randn(M * ldx, 161)))
    ldy, n0 = N + 128, 64
    y0 = np.zeros(M * ldy, np.uint16)
    y = run_gemm(g, b, X, M, N, K, y_init=y0.copy(), rows=Nw, cols=Kw, wr0=128, wk0=256, x={"ld": ldx, "k0": k0},
                 y={"ld": ldy, "n0": n0})
    want = ref.gemm(b, X, M, N, K, rows=Nw, cols=Kw, wr0=128, wk0=256, ldx=ldx, kx0=k0, ldy=ldy, ny0=n0, Y=y0.copy())
    assert_close(ref.h2f(y), ref.h2f(want))


# every config-3 / config-4 shape of BASELINE.json (bias epilogue; the MLP-up shapes with the fused tanh-GELU)
FULL_SIZE = {"c3_qkv": (4096, 9216, 3072, False), "c3_mlp_up": (4096, 12288, 3072, True), "c3_down": (4096, 3072, 12288, False),
             "c4_qkv": (32760, 6720, 2240, False), "c4_up": (32760, 8960, 2240, True), "c4_down": (32760, 2240, 8960, False)}


@pytest.mark.parametrize("cfg", list(FULL_SIZE))
def test_gemm_full_size_rows(g, cfg):
    # BASELINE shapes at full size, checked on a sample of rows against the oracle (the whole oracle GEMM is minutes)
    M, N, K, gelu = FULL_SIZE[cfg]
    b, _ = ref.pack_q4(ref.randn(N * K, 170, 0.02), N, K)
    X = ref.f2h(ref.round_f16(ref.randn(M * K, 171)))
    bias = ref.randn(N, 172, 0.01)
    y = run_gemm(g, b, X, M, N, K, epi="bias", ev=(bias, 0), post_gelu=gelu, acc="f16")
    rows = np.unique(np.concatenate([np.arange(0, 8), np.linspace(8, M - 9, 16).astype(int), np.arange(M - 8, M)]))
    Xs = X.reshape(M, K)[rows].ravel()
    want = ref.gemm(b, Xs, len(rows), N, K, epi="bias", ev=bias, post_gelu=gelu, threads=0).reshape(len(rows), N)
    assert_close(ref.h2f(y.reshape(M, N)[rows]), ref.h2f(want))


def cosine(a, b):
    a, b = np.asarray(a, np.float64).ravel(), np.asarray(b, np.float64).ravel()
    return float(np.dot(a, b) / max(1e-300, np.linalg.norm(a) * np.linalg.norm(b)))


# acc 'f16' (fp16 partial sums per 32-k tile, gemm.js:172-183) is what every DiT call passes (pocketflux-engine.js:4095).
# The tensor cores accumulate in f32 for both modes: the results meet BASELINE's tolerance against the oracle's f32
# accumulation, and the reference's own device-check bar (kcheck.js:88, cos > 0.9995) against its fp16-partial mode.
@pytest.mark.parametrize("epi", ["f16", "bias", "swiglu", "resadd"])
def test_gemm_acc_f16(g, epi):
    M, N, K = 256, 512, 3072
    b, _ = ref.pack_q4(ref.randn(N * K, 180, 0.02), N, K)
    X = ref.f2h(ref.round_f16(ref.randn(M * K, 181)))
    bias, gate = ref.randn(N, 182, 0.01), ref.randn(N, 183, 1.0)
    kw, ref_kw = {"epi": epi}, {"epi": epi}
    if epi == "bias":
        kw.update(ev=(bias, 0)); ref_kw.update(ev=bias)
    elif epi == "swiglu":
        kw.update(act="gelu", wr0=0, wr1=N // 2, bv=(bias, 0, N // 2), y={"ld": N // 2})
        ref_kw.update(act="gelu", wr0=0, wr1=N // 2, bv=bias, bv_up=N // 2, ldy=N // 2)
    elif epi == "resadd":
        kw.update(ev=(gate, 0), bv=(bias, 0), store=True); ref_kw.update(ev=gate, bv=bias, store=True)
    y = run_gemm(g, b, X, M, N, K, acc="f16", **kw)
    f32y = epi == "resadd"
    got = y if f32y else ref.h2f(y)
    want32 = ref.gemm(b, X, M, N, K, acc="f32", threads=0, **ref_kw)
    want16 = ref.gemm(b, X, M, N, K, acc="f16", threads=0, **ref_kw)
    w32, w16 = (want32, want16) if f32y else (ref.h2f(want32), ref.h2f(want16))
    assert_close(got, w32)
    assert cosine(got, w16) > 0.9995
    # the same call with acc 'f32' gives the same bits: one kernel serves both modes
    y32 = run_gemm(g, b, X, M, N, K, acc="f32", **kw)
    assert np.array_equal(y32, y)


# ---------------------------------------------------------------- errors keep the reference's wording
def test_errors(g):
    b, _ = ref.pack_q4(ref.randn(64 * 256, 1, 0.02), 64, 256)
    wb, xb, yb = g.upload(b), g.upload(np.zeros(4096, np.float32)), g.buffer(1 << 16)
    base = {"w": wview(wb, 64, 256), "x": {"buf": xb}, "K": 256, "y": {"buf": yb}}
    with pytest.raises(p0.P0Error, match="gemv: N % 64"):
        p0.gemv(g, dict(base, N=32))
    with pytest.raises(p0.P0Error, match="gemv: K 4096 needs a kPer"):
        p0.gemv(g, dict(base, N=64, K=4096))
    with pytest.raises(p0.P0Error, match="kPer must be a multiple of 32"):
        p0.gemv(g, dict(base, N=64, kPer=48))
    with pytest.raises(p0.P0Error, match="softcap needs one split"):
        p0.gemv(g, dict(base, N=64, kPer=128, epi="softcap", mx={"buf": yb}))
    with pytest.raises(p0.P0Error, match="gemv: weight offset"):
        p0.gemv(g, dict(base, N=64, w=dict(wview(wb, 64, 256), off=2)))
    with pytest.raises(p0.P0Error, match="exceeds its buffer"):
        p0.gemv(g, dict(base, N=128))   # 2 tiles of weights in a 1-tile buffer
    with pytest.raises(p0.P0Error, match="gemvM: prologue sum"):
        p0.gemvM(g, dict(base, N=64, M=2, pro="sum"))
    with pytest.raises(p0.P0Error, match="gemm: K must be a multiple of 32"):
        p0.gemm(g, {"w": wview(wb, 64, 256), "x": {"buf": xb}, "M": 4, "N": 64, "K": 48, "y": {"buf": yb}})
    with pytest.raises(p0.P0Error, match="gemm: unsupported weight encoding"):
        p0.gemm(g, {"w": dict(wview(wb, 64, 256), enc="q3"), "x": {"buf": xb}, "M": 4, "N": 64, "K": 64, "y": {"buf": yb}})
    g.done()   # the context stays usable after rejected calls
