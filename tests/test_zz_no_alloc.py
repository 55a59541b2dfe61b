"""p0_gemvM_noalloc, the gemvM entry point that allocates no device memory (it has no counterpart in the reference).

It exists for callers that must not allocate in the middle of their work: a latency-bound decode loop cannot afford
the device-wide wait of a workspace re-allocation, and a process whose device memory already belongs to another
allocator may have nothing left to allocate. It runs the stream-K GEMV with its scratch in a fixed device array that
every call shares. Each case calls it twice in a row through the C ABI and compares both outputs with the existing
p0_gemvM and with the CPU oracle on the same inputs, within the tolerance of the other parity tests (per-tile argmax
rows exactly, or a tie within 1e-5), and the two calls with each other bit for bit. This file sorts last so that a run which
stops at its first failure has run every other test before this one; it also passes when run on its own.
"""
import numpy as np
import pytest

import p0pc0rn_b200 as p0
from oracle import ref

from .test_gpu_parity import assert_close, nan_buf, wview

pytestmark = pytest.mark.gpu

CASES = [
    # (M, N, K, kPer, epilogue): units split across warps, a k-split call, the softcap head form, geglu
    (4, 4096, 2048, 0, "store"),
    (1, 512, 4096, 1024, "store"),
    (2, 8192, 2048, 0, "softcap"),
    (3, 1024, 2048, 0, "geglu"),
]


def _call(g, fn, wb, xb, M, N, K, kPer, epi, extra):
    rows = 2 * N if epi == "geglu" else N
    ns = -(-K // kPer) if kPer else 1
    yb = nan_buf(g, ns * M * N * 4)
    a = {"w": wview(wb, rows, K), "x": {"buf": xb}, "M": M, "N": N, "K": K, "y": {"buf": yb}, "epi": epi}
    if kPer:
        a["kPer"] = kPer
    mxb = None
    if epi in ("softcap", "geglu"):
        a.update(pro="rms", norm={"buf": extra["nw"], "off": 0}, stat={"buf": extra["st"], "off": 0, "ld": 1})
    if epi == "softcap":
        mxb = nan_buf(g, M * (N // 64) * 8, "mx")
        a.update(mx={"buf": mxb}, cap=30.0)
    assert fn(g, a) == ns
    y = g.read(yb, 0, ns * M * N * 4, np.float32)
    mx = g.read(mxb, 0, M * (N // 64) * 8, np.float32) if mxb is not None else None
    return y, mx


@pytest.mark.parametrize("M,N,K,kPer,epi", CASES)
def test_noalloc_matches_gemvM_two_calls(g, M, N, K, kPer, epi):
    rows = 2 * N if epi == "geglu" else N
    b, _ = ref.pack_q4(ref.randn(rows * K, 400 + N + K, 0.02), rows, K)
    X = ref.randn(M * K, 401)
    wb, xb = g.upload(b), g.upload(X)
    extra = {"nw": g.upload(ref.randn(K, 402, 0.1) + 1), "st": g.upload(np.array([0.8 + 0.05 * m for m in range(M)], np.float32))}
    want_y, want_mx = _call(g, p0.gemvM, wb, xb, M, N, K, kPer, epi, extra)
    # the CPU oracle's restatement of lgemvM on the same inputs (lops_spec.js:44-157)
    st = np.array([0.8 + 0.05 * m for m in range(M)], np.float32)
    kw = {"pro": "rms", "norm": ref.randn(K, 402, 0.1) + 1, "stat": st, "stat_ld": 1} if epi in ("softcap", "geglu") else {}
    ora_y, ora_mx, _ = ref.gemvM(b, X, M, N, K, kPer=kPer or None, epi=epi, **kw)
    first = None
    for _ in range(2):
        y, mx = _call(g, p0.gemvM_noalloc, wb, xb, M, N, K, kPer, epi, extra)
        assert_close(y, want_y)
        assert_close(y[:ora_y.size], ora_y)
        if epi == "softcap":
            assert_close(mx[0::2], want_mx[0::2])
            assert_close(mx[0::2], ora_mx[0::2])
            # the per-tile argmax rows (bitcast u32): equal, or a tie within 1e-5 of the logits (kshipped.js:41-43)
            for other in (want_mx, ora_mx):
                gi, wi = mx.view(np.uint32)[1::2].astype(np.int64), other.view(np.uint32)[1::2].astype(np.int64)
                for t in np.nonzero(gi != wi)[0]:
                    row = ora_y[(t // (N // 64)) * N:(t // (N // 64) + 1) * N]
                    assert abs(float(row[gi[t]]) - float(row[wi[t]])) <= 1e-5, (t, gi[t], wi[t])
        # the two calls in a row give the same bits (the shared array keeps no state a later call depends on)
        if first is None:
            first = (y.copy(), None if mx is None else mx.copy())
        else:
            assert np.array_equal(y.view(np.uint32), first[0].view(np.uint32))
            if mx is not None:
                assert np.array_equal(mx.view(np.uint32), first[1].view(np.uint32))
    g.done()


def test_noalloc_rejects_calls_beyond_the_fixed_array(g):
    # 16384 tiles at M = 8 need ~38 MB of partial sums: more than the fixed array holds, so the call is refused
    M, N, K = 8, 1048576, 32
    wb = g.buffer(N * K * 5 // 8, "w")
    xb = g.upload(np.zeros(M * K, np.float32))
    yb = g.buffer(M * N * 4)
    with pytest.raises(p0.P0Error, match="fixed array holds"):
        p0.gemvM_noalloc(g, {"w": wview(wb, N, K), "x": {"buf": xb}, "M": M, "N": N, "K": K, "y": {"buf": yb}})
