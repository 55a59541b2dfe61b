"""GPU parity of the decode-path operators around the GEMV, through the C ABI, against the CPU oracle:
  argmax / argmaxM (lops.js:416-436, lops_spec.js:326-348): index and max bits exact, ties to the lowest index, NaN
      never wins; and the head -> argmaxM chain (the verify step's token choice) against the oracle's head;
  embed (lops.js:323-365): rows bit-exact (the kernel rounds each operation as the oracle does), the rstd within 1e-6;
  normadd (lops.js:143-180): both modes, split partials, within the parity tolerance;
  dhead (lops_spec.js:428-482): the per-tile max and argmax row of the selected clusters, values bit-exact."""
import numpy as np
import pytest

import p0pc0rn_b200 as p0
from oracle import ref

from .test_gpu_parity import assert_close, nan_buf, run_gemvM

pytestmark = pytest.mark.gpu
Q4, Q8 = "q4g32a.t64", "q8g64s.t64"


def mx_pairs(M, n, seed):
    rng = np.random.default_rng(seed)
    MX = np.empty((M, n, 2), np.float32)
    MX[:, :, 0] = rng.standard_normal((M, n)).astype(np.float32)
    MX[:, :, 1] = rng.permutation(M * n).astype(np.uint32).reshape(M, n).view(np.float32)
    return MX


@pytest.mark.parametrize("M,n", [(1, 4096), (4, 4096), (8, 37), (3, 100000)])
def test_argmaxM(g, M, n):
    MX = mx_pairs(M, n, 70 + n)
    MX[0, n // 2, 0] = MX[0, n - 1, 0] = 50.0          # a tie: the lower index wins
    MX[0, n // 2, 1], MX[0, n - 1, 1] = np.uint32(9).view(np.float32), np.uint32(3).view(np.float32)
    if M > 1:
        MX[1, 0, 0] = np.nan                            # never wins
    out = g.buffer(M * 8)
    if M == 1:
        p0.argmax(g, {"mx": {"buf": g.upload(MX.ravel())}, "n": n, "out": {"buf": out}})
    else:
        p0.argmaxM(g, {"mx": {"buf": g.upload(MX.ravel())}, "n": n, "M": M, "out": {"buf": out}})
    got = g.read(out, 0, M * 8, np.uint32)
    assert np.array_equal(got, ref.argmaxM(MX.ravel(), n, M))
    assert got[0] == 3


def test_head_then_argmaxM(g):
    # the verify step: the head GEMV's softcap epilogue writes per-tile (max, argmax), argmaxM picks each row's token
    M, N, K = 4, 65536, 2048
    b, _ = ref.pack_q4(ref.randn(N * K, 80, 0.02), N, K)
    X = ref.randn(M * K, 81)
    nw = ref.randn(K, 82, 0.1) + 1
    st = np.array([0.9, 1.0, 1.1, 1.2], np.float32)
    NT = N // 64
    y, mx, _ = run_gemvM(g, b, X, M, N, K, M * N, mx_floats=M * NT * 2, extra={"norm": (nw, 0), "stat": (st, 0, 1)}, pro="rms",
                         epi="softcap", cap=30.0)
    out = g.buffer(M * 8)
    p0.argmaxM(g, {"mx": {"buf": g.upload(mx)}, "n": NT, "M": M, "out": {"buf": out}})
    got = g.read(out, 0, M * 8, np.uint32)
    wy, _, _ = ref.gemvM(b, X, M, N, K, pro="rms", epi="softcap", norm=nw, stat=st, stat_off=0, stat_ld=1, cap=30.0)
    for m in range(M):
        row = wy[m * N:(m + 1) * N]
        best = int(np.argmax(row))
        # the chosen token is the oracle's, or one whose logit is within rounding of it
        assert got[2 * m] == best or abs(float(row[got[2 * m]]) - float(row[best])) <= 1e-5
        assert got[2 * m + 1] == y[m * N + got[2 * m]].view(np.uint32)


@pytest.mark.parametrize("enc,K", [(Q4, 2048), (Q8, 2048), (Q4, 96), (Q8, 640)])
def test_embed(g, enc, K):
    V = 64 * 20
    b, _ = (ref.pack_q4 if enc == Q4 else ref.pack_q8)(ref.randn(V * K, 90 + K, 0.05), V, K)
    ids = np.array([0, 1279, 64, 5, 5, 700], np.uint32)
    n, row_out, st_off = ids.size, 2, 3
    xb, sb = nan_buf(g, (row_out + n) * K * 4), nan_buf(g, (st_off + n) * 4)
    p0.embed(g, {"w": {"buf": g.upload(b), "off": 0, "enc": enc, "rows": V, "cols": K}, "ids": {"buf": g.upload(ids)},
                 "x": {"buf": xb}, "st": {"buf": sb, "off": st_off}, "K": K, "n": n, "scale": 45.25, "rowOut": row_out})
    X, ST = ref.embed(b, ids, K, enc=enc, scale=45.25, st_off=st_off, row_out=row_out)
    gx = g.read(xb, 0, (row_out + n) * K * 4, np.float32)
    assert np.array_equal(gx[row_out * K:], X[row_out * K:])
    assert np.allclose(g.read(sb, 0, (st_off + n) * 4, np.float32)[st_off:], ST[st_off:], rtol=1e-6, atol=0)


def test_embed_out_of_table_id_reads_zeros(g):
    V, K = 128, 256
    b, _ = ref.pack_q4(ref.randn(V * K, 95, 0.05), V, K)
    xb, sb = nan_buf(g, 2 * K * 4), nan_buf(g, 8)
    p0.embed(g, {"w": {"buf": g.upload(b), "off": 0, "enc": Q4, "rows": V, "cols": K}, "ids": {"buf": g.upload(np.array([3, 9999], np.uint32))},
                 "x": {"buf": xb}, "st": {"buf": sb}, "K": K, "n": 2, "scale": 1.0})
    gx = g.read(xb, 0, 2 * K * 4, np.float32)
    assert np.array_equal(gx[:K], ref.embed(b, [3], K, scale=1.0)[0]) and not gx[K:].any()


@pytest.mark.parametrize("mode,nsrc,D,M", [(0, 1, 2048, 1), (0, 4, 2048, 4), (1, 4, 2560, 2), (0, 2, 12288, 3)])
def test_normadd(g, mode, nsrc, D, M):
    T = ref.randn(nsrc * M * D, 100 + D, 1.0)
    W = ref.randn(D + 8, 101, 0.2) + 1
    X0 = ref.randn(M * D, 102)
    xb, sb = g.upload(X0), nan_buf(g, (M + 1) * 4)
    p0.normadd(g, {"t": {"buf": g.upload(T), "n": nsrc, "ld": M * D}, "w": {"buf": g.upload(W), "off": 8}, "x": {"buf": xb},
                   "st": {"buf": sb, "off": 1}, "D": D, "M": M, "mode": mode, "eps": 1e-6, "scale": 0.5})
    X, ST = X0.copy(), np.zeros(M + 1, np.float32)
    ref.normadd(T, nsrc, M * D, W, 8, X, ST, 1, D, M, mode=mode, eps=1e-6, scale=0.5)
    assert_close(g.read(xb, 0, M * D * 4, np.float32), X)
    assert np.allclose(g.read(sb, 0, (M + 1) * 4, np.float32)[1:], ST[1:], rtol=1e-5, atol=0)


@pytest.mark.parametrize("enc,K,tPer", [(Q4, 512, 2), (Q8, 512, 2), (Q4, 256, 1), (Q8, 128, 3)])
def test_dhead(g, enc, K, tPer):
    V = 64 * 48
    b, _ = (ref.pack_q4 if enc == Q4 else ref.pack_q8)(ref.randn(V * K, 110 + K, 0.05), V, K)
    X, NW = ref.randn(K, 111), ref.randn(K + 2, 112, 0.1) + 1
    ST = np.array([0.0, 0.0, 0.75], np.float32)
    nsel = 5
    SEL = np.array([0, 15, 7, 3, 15], np.uint32)[:nsel] % (V // 64 // tPer)
    mxb = nan_buf(g, nsel * tPer * 8)
    p0.dhead(g, {"w": {"buf": g.upload(b), "off": 0, "enc": enc, "rows": V, "cols": K}, "x": {"buf": g.upload(X)},
                 "stat": {"buf": g.upload(ST), "off": 2}, "norm": {"buf": g.upload(NW), "off": 2}, "sel": {"buf": g.upload(SEL)},
                 "mx": {"buf": mxb}, "K": K, "tPer": tPer, "nsel": nsel})
    want = ref.dhead(b, X, ST, NW, SEL, K, tPer, nsel, enc=enc, stat_off=2, norm_off=2)
    got = g.read(mxb, 0, nsel * tPer * 8, np.float32)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_dhead_checks(g):
    b, _ = ref.pack_q4(ref.randn(64 * 1024, 120, 0.05), 64, 1024)
    bb = g.upload(b)
    with pytest.raises(p0.P0Error, match="K > 512"):
        p0.dhead(g, {"w": {"buf": bb, "off": 0, "enc": Q4, "rows": 64, "cols": 1024}, "x": {"buf": bb}, "stat": {"buf": bb},
                     "norm": {"buf": bb}, "sel": {"buf": bb}, "mx": {"buf": bb}, "K": 1024, "tPer": 1, "nsel": 1})
