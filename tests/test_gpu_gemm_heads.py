"""GPU parity of the GEMM epilogues that reduce over one 128-wide head (engine/ops/gemm.js:212-250), against the CPU
oracle (oracle.c or_gemm_red128 over the accumulators of or_gemm):
  'heads'     QK-RMSNorm + RoPE + head-major q / k / v write, in the caller forms of the reference: the text encoder's
              rotate_half form (pocketflux-engine.js:2313-2314: Hq 32, Hkv 8, rowOff 0) scaled down, and the DiT's
              interleaved form after the lnmod prologue, two calls (text rows, image rows) into one head buffer at
              rowOff 0 and rowOff = text rows (pocketflux-engine.js:2342-2344, 2363-2364);
  'onormgate' the linear-attention read-out (pocketflux-engine.js:3120): one head per call (N = K = 128), y.ld = D,
              y.n0 = h * 128, the gate rows of ld heads.Ltot, eps = 1e-5 / L^2.
Slots a call must not write (other rows of the head buffer, other heads' columns of y) keep their bits."""
import numpy as np
import pytest

import p0pc0rn_b200 as p0
from p0pc0rn_b200 import _lib as plib
from oracle import ref

from .test_gpu_parity import assert_close, wview

pytestmark = pytest.mark.gpu


def rope_table(L, seed):
    """cos / sin pairs per row: 64 angles per row, as the callers' rope buffers hold them (128 f32 per row)"""
    ang = ref.randn(L * 64, seed, 3.0).astype(np.float64).reshape(L, 64)
    t = np.empty((L, 64, 2), np.float32)
    t[:, :, 0], t[:, :, 1] = np.cos(ang), np.sin(ang)
    return t.ravel()


def pattern_f16(n, seed):
    return ref.f2h(ref.round_f16(ref.randn(n, seed)))


def run_heads(g, b, X, M, N, K, ybuf, ev, rp, heads, enc="q4g32a.t64", **extra):
    args = {"w": {**wview(g.upload(b), N, K), "enc": enc}, "x": {"buf": g.upload(X), **extra.pop("x", {})}, "M": M, "N": N, "K": K,
            "epi": "heads", "y": {"buf": ybuf}, "ev": {"buf": g.upload(ev[0]), "off": ev[1]},
            "heads": {**heads, "rope": {"buf": g.upload(rp)}}}
    args.update(extra)
    assert p0.gemm(g, args) == 2.0 * M * N * K


@pytest.mark.parametrize("M,Hq,Hkv,K", [(129, 4, 1, 512), (64, 2, 2, 256), (300, 3, 1, 1024)])
def test_heads_rotate_half(g, M, Hq, Hkv, K):
    N = (Hq + 2 * Hkv) * 128
    b, _ = ref.pack_q4(ref.randn(N * K, 900 + M, 0.02), N, K)
    X = pattern_f16(M * K, 901)
    ev = ref.randn(256 + 8, 902, 0.2) + 1
    rp = rope_table(M, 903)
    heads = {"Ltot": M, "Hq": Hq, "Hkv": Hkv, "rowOff": 0, "eps": 1e-6, "ropeMode": "half"}
    y0 = pattern_f16(N // 128 * M * 128, 904)
    yb = g.upload(y0)
    run_heads(g, b, X, M, N, K, yb, (ev, 8), rp, heads)
    want = ref.gemm(b, X, M, N, K, epi="heads", ev=ev, ev_off=8, heads={**heads, "rope": rp}, Y=y0.copy())
    assert_close(ref.h2f(g.read(yb, 0, y0.size * 2, np.uint16)), ref.h2f(want))


def test_heads_interleaved_joint_rows_after_lnmod(g):
    # DiT double block: text rows then image rows into one head buffer [head][Ltot][128], each call with its own
    # weights, lnmod x prologue from f32 rows and their stats, q heads [0, NH), k [NH, 2NH), v [2NH, 3NH)
    NH, K, Mt, Mi = 2, 256, 40, 200
    N, L = 3 * NH * 128, Mt + Mi
    rp = rope_table(L, 910)
    ev = ref.randn(256, 911, 0.2) + 1
    y0 = pattern_f16(3 * NH * L * 128, 912)
    yb = g.upload(y0)
    want = y0.copy()
    for seg, (M, row0) in enumerate(((Mt, 0), (Mi, Mt))):
        b, _ = ref.pack_q4(ref.randn(N * K, 913 + seg, 0.02), N, K)
        Xf = ref.randn(M * K, 915 + seg)
        st = np.empty(2 * M, np.float32)
        st[0::2], st[1::2] = ref.randn(M, 917 + seg, 0.1), 0.5 + np.abs(ref.randn(M, 919 + seg, 0.2))
        pv = ref.randn(2 * K, 921 + seg, 0.1)
        heads = {"Ltot": L, "Hq": NH, "Hkv": NH, "rowOff": row0, "eps": 1e-6, "ropeMode": "inter"}
        run_heads(g, b, Xf, M, N, K, yb, (ev, 0), rp, heads, x={"mode": "lnmod"}, stats={"buf": g.upload(st), "off": 0},
                  pv={"buf": g.upload(pv), "off": 0, "stride": K})
        X16 = ref.gemm_xpro("lnmod", Xf, M, K, stats=st, pv=pv, pv_stride=K)
        want = ref.gemm(b, X16, M, N, K, epi="heads", ev=ev, heads={**heads, "rope": rp}, Y=want)
    assert_close(ref.h2f(g.read(yb, 0, y0.size * 2, np.uint16)), ref.h2f(want))


def test_heads_q8_and_default_eps(g):
    # q8 weights; eps 0 means the reference's default 1e-6 (`h.eps || 1e-6`); v heads only beyond Hq + Hkv
    M, Hq, Hkv, K = 96, 1, 1, 256
    N = 4 * 128                                  # heads q, k, v, v: the fourth is past Hq + 2 Hkv and still a v head
    b, _ = ref.pack_q8(ref.randn(N * K, 930, 0.02), N, K)
    X = pattern_f16(M * K, 931)
    ev = ref.randn(256, 932, 0.2) + 1
    rp = rope_table(M + 7, 933)
    heads = {"Ltot": M + 7, "Hq": Hq, "Hkv": Hkv, "rowOff": 7, "ropeMode": "half"}
    y0 = pattern_f16(4 * (M + 7) * 128, 934)
    yb = g.upload(y0)
    run_heads(g, b, X, M, N, K, yb, (ev, 0), rp, heads, enc="q8g64s.t64")
    want = ref.gemm(b, X, M, N, K, enc="q8g64s.t64", epi="heads", ev=ev, heads={**heads, "rope": rp}, Y=y0.copy())
    assert_close(ref.h2f(g.read(yb, 0, y0.size * 2, np.uint16)), ref.h2f(want))


@pytest.mark.parametrize("M,h", [(200, 1), (64, 0), (1000, 2)])
def test_onormgate(g, M, h):
    D, LDG, K = 3 * 128, 4 * 128, 128
    b, _ = ref.pack_q4(ref.randn(128 * K, 940 + M, 0.05), 128, K)
    X = pattern_f16(M * K, 941)
    ev = ref.randn(128, 942, 0.2) + 1
    gt = pattern_f16(M * LDG, 943)
    y0 = pattern_f16(M * D, 944)
    yb = g.upload(y0)
    heads = {"Ltot": LDG, "eps": 1e-5 / (M * M)}
    args = {"w": wview(g.upload(b), 128, K), "x": {"buf": g.upload(X)}, "M": M, "N": 128, "K": K, "epi": "onormgate",
            "y": {"buf": yb, "off": 0, "ld": D, "n0": h * 128}, "ev": {"buf": g.upload(ev), "off": 0}, "gt": {"buf": g.upload(gt)},
            "heads": heads}
    assert p0.gemm(g, args) == 2.0 * M * 128 * K
    want = ref.gemm(b, X, M, 128, K, epi="onormgate", ev=ev, ldy=D, ny0=h * 128, heads=heads, gt=gt, Y=y0.copy())
    assert_close(ref.h2f(g.read(yb, 0, y0.size * 2, np.uint16)), ref.h2f(want))


def test_head_epilogue_checks(g):
    # whole heads only; the gate rows must keep vec4 alignment; a rope table too short for the rows is refused
    K = 128
    b, _ = ref.pack_q4(ref.randn(192 * K, 950, 0.05), 192, K)
    wb, xb = g.upload(b), g.upload(pattern_f16(8 * K, 951))
    yb, eb, rb = g.buffer(1 << 20), g.upload(np.ones(256, np.float32)), g.upload(rope_table(8, 952))
    base = {"w": wview(wb, 192, K), "x": {"buf": xb}, "M": 8, "K": K, "y": {"buf": yb}, "ev": {"buf": eb, "off": 0}}
    with pytest.raises(p0.P0Error, match="whole 128-wide heads") as e:
        p0.gemm(g, {**base, "N": 192, "epi": "heads", "heads": {"Ltot": 8, "Hq": 1, "rope": {"buf": rb}}})
    assert e.value.status == plib.P0_EINVAL
    with pytest.raises(p0.P0Error, match="Ltot % 4") as e:
        p0.gemm(g, {**base, "N": 128, "epi": "onormgate", "gt": {"buf": yb}, "heads": {"Ltot": 130}})
    assert e.value.status == plib.P0_EALIGN
    with pytest.raises(p0.P0Error, match="rope range") as e:
        p0.gemm(g, {**base, "N": 128, "epi": "heads", "heads": {"Ltot": 16, "Hq": 1, "rowOff": 4, "rope": {"buf": rb}}})
    assert e.value.status == plib.P0_EINVAL
