"""Recorded GEMV chains (p0_chain_*, the DecodeRunner of engine/llm/drunner.js): the calls recorded between
chain_begin and chain_end, run as one persistent kernel, against the same calls launched one by one and against the CPU
oracle chained the same way. The layer's shape follows a decode step (gemma4.js:457-511): rms QKV, O on part of its
output, rms GeGLU, the down projection with kPer split partials, then an rms softcap head with per-tile argmax; every
call reads the previous call's output, so the kernel must order them with grid barriers.
"""
import numpy as np
import pytest

import p0pc0rn_b200 as p0
from oracle import ref

from .test_gpu_parity import assert_close, nan_buf

pytestmark = pytest.mark.gpu

D, QKV, FF, HEAD, KP = 512, 640, 1024, 4096, 256


def wv(buf, rows, cols):
    return {"buf": buf, "off": 0, "enc": "q4g32a.t64", "rows": rows, "cols": cols}


class Layer:
    """weights and buffers of one synthetic decode layer + head, M tokens"""

    def __init__(self, g, M, seed):
        self.g, self.M = g, M
        self.wq = ref.pack_q4(ref.randn(QKV * D, seed, 0.02), QKV, D)[0]
        self.wo = ref.pack_q4(ref.randn(D * D, seed + 1, 0.02), D, D)[0]
        self.wg = ref.pack_q4(ref.randn(2 * FF * D, seed + 2, 0.02), 2 * FF, D)[0]
        self.wd = ref.pack_q4(ref.randn(D * FF, seed + 3, 0.02), D, FF)[0]
        self.wh = ref.pack_q4(ref.randn(HEAD * D, seed + 4, 0.02), HEAD, D)[0]
        self.x0 = ref.randn(M * D, seed + 5)
        self.nw = ref.randn(D, seed + 6, 0.1) + 1
        self.st = np.array([0.9, 1.1, 0.8, 1.0, 0.95, 1.05, 0.85, 1.2][:M], np.float32)
        self.b = {k: g.upload(getattr(self, k)) for k in ("wq", "wo", "wg", "wd", "wh", "x0", "nw", "st")}

    def outputs(self):
        g, M = self.g, self.M
        return {"y1": nan_buf(g, M * QKV * 4), "y2": nan_buf(g, M * D * 4), "y3": nan_buf(g, M * FF * 4),
                "y4": nan_buf(g, (FF // KP) * M * D * 4), "y5": nan_buf(g, M * HEAD * 4), "mx": nan_buf(g, M * (HEAD // 64) * 8)}

    def calls(self, o):
        """the five calls of the layer; each reads the previous one's output"""
        b, M = self.b, self.M
        rms = {"norm": {"buf": b["nw"], "off": 0}, "stat": {"buf": b["st"], "off": 0, "ld": 1}}
        return [
            dict(rms, w=wv(b["wq"], QKV, D), x={"buf": b["x0"], "ldx": D}, M=M, N=QKV, K=D, pro="rms", y={"buf": o["y1"]}),
            dict(w=wv(b["wo"], D, D), x={"buf": o["y1"], "ldx": QKV}, M=M, N=D, K=D, y={"buf": o["y2"]}),
            dict(rms, w=wv(b["wg"], 2 * FF, D), x={"buf": o["y2"], "ldx": D}, M=M, N=FF, K=D, pro="rms", epi="geglu", y={"buf": o["y3"]}),
            dict(w=wv(b["wd"], D, FF), x={"buf": o["y3"], "ldx": FF}, M=M, N=D, K=FF, kPer=KP, y={"buf": o["y4"]}),
            dict(rms, w=wv(b["wh"], HEAD, D), x={"buf": o["y4"], "ldx": D}, M=M, N=HEAD, K=D, pro="rms", epi="softcap", cap=30.0,
                 y={"buf": o["y5"]}, mx={"buf": o["mx"]}),
        ]

    def read(self, o):
        g, M = self.g, self.M
        g.done()
        return {k: g.read(o[k], 0, n, np.float32) for k, n in
                (("y1", M * QKV * 4), ("y2", M * D * 4), ("y3", M * FF * 4), ("y4", (FF // KP) * M * D * 4), ("y5", M * HEAD * 4),
                 ("mx", M * (HEAD // 64) * 8))}

    def oracle(self):
        M = self.M
        kw = {"norm": self.nw, "stat": self.st, "stat_ld": 1}
        y1, _, _ = ref.gemvM(self.wq, self.x0, M, QKV, D, pro="rms", **kw)
        y2, _, _ = ref.gemvM(self.wo, y1, M, D, D, ldx=QKV)
        y3, _, _ = ref.gemvM(self.wg, y2, M, FF, D, pro="rms", epi="geglu", **kw)
        y4, _, _ = ref.gemvM(self.wd, y3, M, D, FF, kPer=KP)
        y5, mx, _ = ref.gemvM(self.wh, y4, M, HEAD, D, pro="rms", epi="softcap", **kw)
        return {"y1": y1, "y2": y2, "y3": y3, "y4": y4, "y5": y5, "mx": mx}


@pytest.mark.parametrize("M", [1, 4])
def test_chain_matches_calls_and_oracle(g, M):
    L = Layer(g, M, 700 + M)
    o_seq = L.outputs()
    for a in L.calls(o_seq):
        p0.gemvM(g, a)
    seq = L.read(o_seq)
    o_ch = L.outputs()
    g.chain_begin()
    for a in L.calls(o_ch):
        assert p0.gemvM(g, a) == (FF // KP if a.get("kPer") else 1)   # recorded: the same return value, nothing launched
    ch = g.chain_end()
    info = ch.info()
    assert info == {"calls": 5, "kernel_calls": 5, "launches": 1, "barriers": 4}, info
    g.done()
    assert np.all(np.isnan(g.read(o_ch["y1"], 0, 16, np.float32)))          # recording ran nothing
    ch.run()
    got = L.read(o_ch)
    want = L.oracle()
    for k in ("y1", "y2", "y3", "y4", "y5"):
        assert_close(got[k], seq[k])
        assert_close(got[k], want[k])
    assert_close(got["mx"][0::2], want["mx"][0::2])
    # argmax rows: equal, or a tie within 1e-5 of the logits (kshipped.js:41-43)
    NT = HEAD // 64
    gi, wi = got["mx"].view(np.uint32)[1::2].astype(np.int64), want["mx"].view(np.uint32)[1::2].astype(np.int64)
    for t in np.nonzero(gi != wi)[0]:
        row = want["y5"][(t // NT) * HEAD:(t // NT + 1) * HEAD]
        assert abs(float(row[gi[t]]) - float(row[wi[t]])) <= 1e-5
    # a second run gives the same bits (counters and barriers reset; partials summed in a fixed order)
    ch.run()
    again = L.read(o_ch)
    for k in got:
        assert np.array_equal(again[k].view(np.uint32), got[k].view(np.uint32)), k
    ch.free()


def test_chain_independent_calls_need_no_barrier(g):
    # three calls that read x0 and write their own outputs: one launch, no grid barrier
    L = Layer(g, 2, 720)
    o = L.outputs()
    calls = L.calls(o)
    indep = [calls[0], dict(calls[2], x={"buf": L.b["x0"], "ldx": D}), dict(calls[4], x={"buf": L.b["x0"], "ldx": D})]
    g.chain_begin()
    for a in indep:
        p0.gemvM(g, a)
    ch = g.chain_end()
    assert ch.info() == {"calls": 3, "kernel_calls": 3, "launches": 1, "barriers": 0}
    ch.run()
    got = L.read(o)
    want = {}
    kw = {"norm": L.nw, "stat": L.st, "stat_ld": 1}
    want["y1"], _, _ = ref.gemvM(L.wq, L.x0, 2, QKV, D, pro="rms", **kw)
    want["y3"], _, _ = ref.gemvM(L.wg, L.x0, 2, FF, D, pro="rms", epi="geglu", **kw)
    want["y5"], _, _ = ref.gemvM(L.wh, L.x0, 2, HEAD, D, pro="rms", epi="softcap", **kw)
    for k in want:
        assert_close(got[k], want[k])
    ch.free()


def test_chain_with_a_wide_call_and_gemv(g):
    # gemv (M = 1) calls; a head wider than the chain kernel takes (1024 tiles > 4 x SMs) runs on its own kernel between
    # two chain launches, still in order
    M, Kw, Nw = 1, 256, 65536
    L = Layer(g, M, 730)
    wide = ref.pack_q4(ref.randn(Nw * Kw, 731, 0.02), Nw, Kw)[0]
    wb = g.upload(wide)
    o = L.outputs()
    yw = nan_buf(g, Nw * 4)
    mxw = g.upload(np.full(Nw // 64 * 2 + 4, 0.9, np.float32))       # rstd slot past the tile pairs (lops.js:125)
    c = L.calls(o)
    seq = [
        dict(c[0], x={"buf": L.b["x0"]}, stat={"buf": L.b["st"], "off": 0}),
        dict(c[1], x={"buf": o["y1"]}),
        {"w": wv(wb, Nw, Kw), "x": {"buf": o["y2"]}, "N": Nw, "K": Kw, "pro": "rms", "epi": "softcap", "cap": 30.0,
         "norm": {"buf": L.b["nw"], "off": 0}, "stat": {"buf": mxw, "off": Nw // 64 * 2}, "mx": {"buf": mxw}, "y": {"buf": yw}},
        dict(c[2], x={"buf": o["y2"]}, stat={"buf": L.b["st"], "off": 0}),
    ]
    for a in seq:
        a.pop("M", None)
        a["x"].pop("ldx", None)
    g.chain_begin()
    for a in seq:
        p0.gemv(g, a)
    ch = g.chain_end()
    assert ch.info() == {"calls": 4, "kernel_calls": 3, "launches": 3, "barriers": 1}
    ch.run()
    got = L.read(o)
    g.done()
    gw = g.read(yw, 0, Nw * 4, np.float32)
    y1, _, _ = ref.gemv(L.wq, L.x0, QKV, D, pro="rms", norm=L.nw, stat_buf=L.st)
    y2, _, _ = ref.gemv(L.wo, y1, D, D)
    mxh = np.full(Nw // 64 * 2 + 4, 0.9, np.float32)
    yh, _, _ = ref.gemv(wide, y2, Nw, Kw, pro="rms", epi="softcap", norm=L.nw, stat_off=Nw // 64 * 2, mx=mxh)
    y3, _, _ = ref.gemv(L.wg, y2, FF, D, pro="rms", epi="geglu", norm=L.nw, stat_buf=L.st)
    assert_close(got["y1"], y1)
    assert_close(got["y2"], y2)
    assert_close(gw, yh)
    assert_close(got["y3"], y3)
    ch.free()


def test_chain_recording_errors(g):
    L = Layer(g, 1, 740)
    o = L.outputs()
    with pytest.raises(p0.P0Error, match="no chain"):
        g.chain_end()
    g.chain_begin()
    with pytest.raises(p0.P0Error, match="already"):
        g.chain_begin()
    bad = dict(L.calls(o)[1], N=100)
    with pytest.raises(p0.P0Error, match="N % 64"):   # checked as the call itself would be, and not recorded
        p0.gemvM(g, bad)
    p0.gemvM(g, L.calls(o)[0])
    ch = g.chain_end()
    assert ch.info()["calls"] == 1
    ch.free()
