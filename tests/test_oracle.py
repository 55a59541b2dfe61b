"""Pins the CPU oracle (oracle/oracle.c) before anything is checked against it.

The reference ships no golden vectors and cannot run here (JavaScript + WebGPU), so the pins are:
  1. hand-derived vectors for f2h (incl. the f64 -> f32 -> f16 double rounding of core/gpu.js:274-289) and rng;
  2. a second, independent transcription of the JS helpers (tests/jsref.py) agreeing bit for bit;
  3. the reference's own known-answer checks: kcheck.js:72-88 (q4 gemm, cos > 0.9995), kcheck.js:129-135 (q4 gemv,
     cos > 0.9999), tune/kshipped.js:17-45 (per-shape gemv, cos > 0.99999 + tile argmax), tune/autotune.js:168-188
     (engine kernel vs f64 dot, rel-L2 <= 2e-5), lops_spec.js:6-7 (gemvM row == gemv row);
  4. the committed fixtures under tests/golden/ (oracle outputs; regenerate with tests/golden/make_golden.py).
"""
import json
import math
import os

import numpy as np
import pytest

from oracle import ref
from tests import jsref

GOLD = os.path.join(os.path.dirname(__file__), "golden")


# ---------------------------------------------------------------- 1. hand-derived vectors
def test_f2h_vectors():
    cases = {
        1.0: 0x3C00, -2.0: 0xC000, 65504.0: 0x7BFF, 65519.0: 0x7BFF, 65520.0: 0x7C00, 1e-8: 0x0000, 6e-8: 0x0001,
        -0.0: 0x8000, 0.1: 0x2E66, float("inf"): 0x7C00, 2.0 ** -14: 0x0400, 2.0 ** -24: 0x0001, 3 * 2.0 ** -25: 0x0002,
        # f64 -> f32 first: 1 + 2^-11 + 2^-40 rounds to the f32 1 + 2^-11, an f16 tie that goes to even (1.0);
        # rounding f64 straight to f16 would give 0x3C01
        1 + 2.0 ** -11 + 2.0 ** -40: 0x3C00,
        1 + 2.0 ** -11 + 2.0 ** -20: 0x3C01,
        1 + 3 * 2.0 ** -11: 0x3C02,   # tie between 0x3C01 and 0x3C02 -> even
    }
    got = ref.f2h(list(cases.keys()))
    assert [int(v) for v in got] == list(cases.values())
    assert int(ref.f2h([float("nan")])[0]) == 0x7E00


def test_f2h_matches_ieee_rne_via_f32():
    x = np.concatenate([ref.randn(20000, 5, 3.0), ref.randn(20000, 6, 1e-5), ref.randn(2000, 7, 3e4)]).astype(np.float64)
    # numpy's f32 -> f16 cast is IEEE round-to-nearest-even, with subnormals and overflow to inf (the 3e4-scale
    # samples reach past 65504 on purpose)
    with np.errstate(over="ignore"):
        want = x.astype(np.float32).astype(np.float16).view(np.uint16)
    assert np.array_equal(ref.f2h(x), want)
    h = np.arange(0, 0x7C00, 7, dtype=np.uint16)
    assert np.array_equal(ref.h2f(h), h.view(np.float16).astype(np.float64))


def test_rng_vectors():
    # xorshift32 with JS's signed `>> 17`: hand-stepped for seed 1 (kcheck.js:10)
    s = 1
    s ^= (s << 13) & 0xFFFFFFFF            # 0x00002001
    s ^= s >> 17                           # positive int32: same as logical
    s ^= (s << 5) & 0xFFFFFFFF             # 0x00042021
    assert s == 0x00042021 and ref.rng_state(1, 0) == 0x00042021
    assert ref.rng_state(0, 0) == ref.rng_state(1, 0)   # seed 0 -> 1 (`seed >>> 0 || 1`)
    # a state with the top bit set exercises the arithmetic shift: compare with the transcription
    r = jsref.rng(0xDEADBEEF)
    for k in range(200):
        v = r()
        assert int(round(v * 4294967296)) == ref.rng_state(0xDEADBEEF, k)


# ---------------------------------------------------------------- 2. second transcription
@pytest.mark.parametrize("seed,scale", [(0, 1.0), (7, 1.0), (11, 0.05), (31, 1.0), (0x80000001, 0.02)])
def test_randn_matches_transcription(seed, scale):
    n = 2001
    assert np.array_equal(ref.randn(n, seed, scale), np.array(jsref.randn(n, seed, scale), np.float32))


def test_f2h_matches_transcription():
    xs = list(ref.randn(3000, 9, 2.0).astype(np.float64)) + [65520.0, 1e-7, 3e-5, -7e-6, 2 ** -15 * 1.5]
    assert [int(v) for v in ref.f2h(xs)] == [jsref.f2h(x) for x in xs]


def test_pack_q4_matches_transcription():
    N, K = 64, 96
    W = ref.randn(N * K, 11, 0.05)
    # edge groups: constant (s == 0 -> 1), a tiny-range group (subnormal fp16 scale), large values
    W[0:32] = 0.25
    W[K:K + 32] = np.linspace(1.0, 1.0 + 3e-6, 32, dtype=np.float32)
    W[2 * K:2 * K + 32] = np.linspace(-60000.0, 60000.0, 32, dtype=np.float32)
    b, deq = ref.pack_q4(W, N, K)
    jb, jdeq = jsref.pack_q4([float(v) for v in W], N, K)
    assert bytes(b) == jb
    assert np.array_equal(deq, np.array(jdeq, np.float32))


def test_pack_q4_layout():
    # one record by hand: row r's 32 codes at bytes r*16.., the (s, mn) word at 1024 + 4r (kcheck.js:32-34)
    N, K = 64, 32
    W = np.zeros(N * K, np.float32)
    W[:32] = np.arange(32, dtype=np.float32) / 31 * 1.5 - 0.5     # row 0: min -0.5, max 1.0
    b, deq = ref.pack_q4(W, N, K)
    mn, s = -0.5, float(np.float16(1.5 / 15))
    sm = int.from_bytes(bytes(b[1024:1028]), "little")
    assert sm & 0xFFFF == int(np.float16(s).view(np.uint16)) and sm >> 16 == int(np.float16(mn).view(np.uint16))
    q = [min(15, max(0, int(np.rint((W[i] - mn) / s)))) for i in range(32)]
    assert list(b[:16]) == [q[2 * j] | (q[2 * j + 1] << 4) for j in range(16)]
    assert np.array_equal(deq[:32], (np.array(q, np.float64) * s + mn).astype(np.float32))
    # row 1: all zero -> s = 1, mn = 0, codes 0
    assert int.from_bytes(bytes(b[1028:1032]), "little") == 0x3C00 and not any(b[16:32])


# ---------------------------------------------------------------- 3. the reference's own known-answer checks
def test_kcheck_gemm_q4():
    # kcheck.js:72-88: M=32, N=128, K=256, X roundF16(randn(M*K, 7)), W randn(N*K, 11, 0.05), cos > 0.9995
    M, N, K = 32, 128, 256
    X = ref.round_f16(ref.randn(M * K, 7))
    b, deq = ref.pack_q4(ref.randn(N * K, 11, 0.05), N, K)
    Y = ref.h2f(ref.gemm(b, ref.f2h(X), M, N, K))
    c = ref.compare(Y, ref.dot64(deq, X.astype(np.float64), M, N, K))
    assert c["cos"] > 0.9995
    for acc in ("f16",):   # the DiT's default fp16 partial sums (gemm.js:172-183) pass the same gate
        c16 = ref.compare(ref.h2f(ref.gemm(b, ref.f2h(X), M, N, K, acc=acc)), ref.dot64(deq, X.astype(np.float64), M, N, K))
        assert c16["cos"] > 0.9995


def test_kcheck_gemv_q4():
    # kcheck.js:129-135: N=256, K=1536, x randn(K, 31), W randn(N*K, 32, 0.05), cos > 0.9999
    N, K = 256, 1536
    x = ref.randn(K, 31)
    b, deq = ref.pack_q4(ref.randn(N * K, 32, 0.05), N, K)
    y, _, ns = ref.gemv(b, x, N, K)
    assert ns == 1
    assert ref.compare(y, ref.dot64(deq, x.astype(np.float64), 1, N, K).ravel())["cos"] > 0.9999


def _gelu64(v):
    return v * 0.5 * (1 + math.tanh(max(-15.0, min(15.0, 0.7978845608028654 * (v + 0.044715 * v * v * v)))))


@pytest.mark.parametrize("pro,epi,K,kPer", [("rms", "softcap", 1536, 0), ("rms", "geglu", 1536, 0), ("raw", "store", 6144, 2048),
                                            ("rms", "store", 2560, 0), ("raw", "store", 2048, 0), ("pleg", "store", 256, 0)])
def test_kshipped_gemv(pro, epi, K, kPer):
    # tune/kshipped.js:17-45: 128 rows, W randn(rows*K, 33+K, 0.05), x randn(K, 34+K), nw 0.9 + 0.2*((i*7919)%100)/100,
    # ev randn(K, 35+K, 0.5); cos > 0.99999 and each tile's argmax equal or tied within 1e-5
    N = 128
    rows = 2 * N if epi == "geglu" else N
    b, deq = ref.pack_q4(ref.randn(rows * K, 33 + K, 0.05), rows, K)
    x = ref.randn(K, 34 + K)
    nw = np.array([0.9 + 0.2 * ((i * 7919) % 100) / 100 for i in range(K)], np.float32)
    ev = ref.randn(K, 35 + K, 0.5)
    ss = float(np.sum(x.astype(np.float64) ** 2))
    rstd = np.float32(1 / math.sqrt(ss / K + 1e-6))
    NT = N // 64
    mxb = np.zeros(NT * 2 + 4, np.float32)
    mxb[NT * 2] = rstd
    stb = np.array([0, rstd, 0, 0], np.float32)
    kw = dict(pro=pro, epi=epi, kPer=kPer or None)
    if pro == "rms":
        kw.update(norm=nw, stat_buf=stb, stat_off=1)
        if epi == "softcap":
            kw.update(stat_off=NT * 2)
    if pro == "pleg":
        kw.update(src=(K, 1), ev=ev)
    if epi == "softcap":
        kw.update(mx=mxb, cap=30.0)
    y, MX, ns = ref.gemv(b, x, N, K, **kw)
    got = y.reshape(ns, -1)[:, :N].sum(0) if epi == "store" else y[:N]
    xp = [float(x[k]) if pro == "raw" else float(x[k]) * float(rstd) * float(nw[k]) if pro == "rms" else _gelu64(float(x[k])) * float(ev[k])
          for k in range(K)]
    dot = ref.dot64(deq, np.array(xp, np.float64), 1, rows, K).ravel()
    want = np.array([_gelu64(dot[n]) * dot[n + N] if epi == "geglu" else 30 * math.tanh(max(-15, min(15, dot[n] / 30)))
                     if epi == "softcap" else dot[n] for n in range(N)])
    assert ref.compare(got, want)["cos"] > 0.99999
    if epi == "softcap":
        mxu = MX.view(np.uint32)
        for t in range(NT):
            best = t * 64 + int(np.argmax(want[t * 64:(t + 1) * 64]))
            i = int(mxu[2 * t + 1])
            assert i == best or abs(want[i] - want[best]) <= 1e-5


def test_autotune_gate_rel_l2():
    # tune/autotune.js:168-188: the engine kernel against an f64 dot product, rel-L2 <= 2e-5 (fill s in [0.006, 0.010],
    # min = -7.5 s, :83 -- here packQ4 of N(0, 0.02) weights)
    N, K = 256, 2048
    b, deq = ref.pack_q4(ref.randn(N * K, 3, 0.02), N, K)
    x = ref.randn(K, 4)
    y, _, _ = ref.gemv(b, x, N, K)
    assert ref.compare(y, ref.dot64(deq, x.astype(np.float64), 1, N, K).ravel())["relL2"] <= 2e-5


@pytest.mark.parametrize("M", [1, 2, 4, 8])
def test_gemvM_rows_equal_gemv(M):
    # lops_spec.js:6-7: each gemvM row is bit-identical to the engine gemv of that row
    N, K = 128, 512
    b, _ = ref.pack_q4(ref.randn(N * K, 21, 0.02), N, K)
    X = ref.randn(M * K, 22)
    Y, _, _ = ref.gemvM(b, X, M, N, K)
    for m in range(M):
        y1, _, _ = ref.gemv(b, X[m * K:(m + 1) * K], N, K)
        assert np.array_equal(y1, Y[m * N:(m + 1) * N])


def test_gemv_host_errors():
    b, _ = ref.pack_q4(ref.randn(64 * 64, 1, 0.02), 64, 64)
    with pytest.raises(ValueError, match="N % 64"):
        ref.gemv(b, np.zeros(64, np.float32), 32, 64)
    with pytest.raises(ValueError, match="needs a kPer"):
        ref.gemv(b, np.zeros(4096, np.float32), 64, 4096)
    with pytest.raises(ValueError, match="softcap needs one split"):
        ref.gemv(b, np.zeros(64, np.float32), 64, 64, kPer=32, epi="softcap", mx=np.zeros(8, np.float32))


# ---------------------------------------------------------------- 4. committed fixtures
def test_golden_fixtures():
    from tests.golden import make_golden
    with open(os.path.join(GOLD, "manifest.json")) as f:
        man = json.load(f)
    cases = make_golden.cases()
    assert sorted(man) == sorted(cases)
    for name, fn in cases.items():
        arrays = fn()
        ent = man[name]
        for k, arr in arrays.items():
            stored = np.fromfile(os.path.join(GOLD, ent[k]["file"]), dtype=ent[k]["dtype"])
            assert np.array_equal(stored, np.ascontiguousarray(arr).ravel().view(stored.dtype)), (name, k)


# ---------------------------------------------------------------- head-reducing GEMM epilogues (gemm.js:212-250)
# The reference's tests hold no vectors for these epilogues, so the restatement is pinned by identities of the math
# it states, checked in f64 from the same accumulators: RMSNorm scaling, the rotation's pair norms, the identity rope,
# the untouched v heads and the sigmoid gate.
def _acc_and_inputs(M, N, K, seed):
    b, _ = ref.pack_q4(ref.randn(N * K, seed, 0.03), N, K)
    X = ref.f2h(ref.round_f16(ref.randn(M * K, seed + 1)))
    A = ref.gemm(b, X, M, N, K, epi="f32").reshape(M, N).astype(np.float64)
    return b, X, A


@pytest.mark.parametrize("mode", ["half", "inter"])
def test_heads_oracle_identities(mode):
    M, K, Hq, Hkv = 6, 128, 1, 1
    N = 3 * 128
    b, X, A = _acc_and_inputs(M, N, K, 960)
    ev = (ref.randn(256, 962, 0.2) + 1).astype(np.float32)
    eps = 1e-6
    inv = 1.0 / np.sqrt(np.stack([(A[:, h * 128:(h + 1) * 128] ** 2).sum(1) / 128 + eps for h in range(3)], 1))   # [M][head]
    # identity rope (cos 1, sin 0): out = a * inv * w
    rp = np.zeros(M * 128, np.float32)
    rp[0::2] = 1.0
    h = {"Ltot": M, "Hq": Hq, "Hkv": Hkv, "rowOff": 0, "eps": eps, "ropeMode": mode, "rope": rp}
    y = ref.h2f(ref.gemm(b, X, M, N, K, epi="heads", ev=ev, heads=h)).reshape(3, M, 128)
    for hd in range(2):
        want = A[:, hd * 128:(hd + 1) * 128] * inv[:, hd:hd + 1] * ev[hd * 128:(hd + 1) * 128]
        assert np.max(np.abs(y[hd] - want)) <= 2e-3 * max(1.0, np.max(np.abs(want)))
    assert np.array_equal(ref.gemm(b, X, M, N, K, epi="heads", ev=ev, heads=h).reshape(3, M, 128)[2],
                          ref.f2h(A[:, 256:384].astype(np.float32).astype(np.float64)))   # v: f16(acc), unnormalised
    # random rope, unit norm weights: each rotated pair keeps its length, sqrt(2) * |normalised pair|
    ang = ref.randn(M * 64, 963, 3.0).astype(np.float64)
    rp = np.empty(M * 128, np.float32)
    rp[0::2], rp[1::2] = np.cos(ang), np.sin(ang)
    y = ref.h2f(ref.gemm(b, X, M, N, K, epi="heads", ev=np.ones(256, np.float32), heads={**h, "rope": rp})).reshape(3, M, 128)
    for hd in range(2):
        v = A[:, hd * 128:(hd + 1) * 128] * inv[:, hd:hd + 1]
        if mode == "half":
            pn_in, pn_out = v[:, :64] ** 2 + v[:, 64:] ** 2, y[hd][:, :64] ** 2 + y[hd][:, 64:] ** 2
            c, s = np.cos(ang).reshape(M, 64), np.sin(ang).reshape(M, 64)
            lo = v[:, :64] * c - v[:, 64:] * s
            assert np.max(np.abs(y[hd][:, :64] - lo)) <= 5e-3
        else:
            pn_in, pn_out = v[:, 0::2] ** 2 + v[:, 1::2] ** 2, y[hd][:, 0::2] ** 2 + y[hd][:, 1::2] ** 2
            c, s = np.cos(ang).reshape(M, 64), np.sin(ang).reshape(M, 64)
            assert np.max(np.abs(y[hd][:, 1::2] - (v[:, 0::2] * s + v[:, 1::2] * c))) <= 5e-3
        assert np.max(np.abs(pn_out - pn_in)) <= 2e-2


def test_onormgate_oracle_identities():
    M, K, LDG = 5, 128, 132
    b, X, A = _acc_and_inputs(M, 128, K, 970)
    ev = (ref.randn(128, 972, 0.2) + 1).astype(np.float32)
    eps = 1e-9
    inv = 1.0 / np.sqrt((A ** 2).sum(1, keepdims=True) / 128 + eps)
    gate = ref.randn(M * LDG, 973, 2.0)
    gt = ref.f2h(ref.round_f16(gate))
    y = ref.gemm(b, X, M, 128, K, epi="onormgate", ev=ev, ldy=256, ny0=4, heads={"Ltot": LDG, "eps": eps}, gt=gt,
                 Y=np.zeros(M * 256, np.uint16))
    y = ref.h2f(y).reshape(M, 256)
    g = ref.h2f(gt).reshape(M, LDG)[:, 4:132]
    want = A * inv * ev / (1 + np.exp(-g))
    assert np.max(np.abs(y[:, 4:132] - want)) <= 2e-3 * max(1.0, np.max(np.abs(want)))
    assert not y[:, :4].any() and not y[:, 132:].any()   # columns outside the head untouched


# ---------------------------------------------------------------- decode-path operators (lops.js, lops_spec.js)
# No reference vectors exist for these; each restatement is pinned against an independent numpy statement of the
# same math.
def test_argmax_oracle_rules():
    rng = np.random.default_rng(5)
    M, n = 3, 1000
    v = rng.standard_normal((M, n)).astype(np.float32)
    idx = rng.permutation(M * n).astype(np.uint32).reshape(M, n)
    v[1, 17] = v[1, 600] = 9.0                 # a tie: the lower index wins
    idx[1, 17], idx[1, 600] = 500, 40
    v[2, 3] = np.nan                           # NaN never wins
    MX = np.empty((M, n, 2), np.float32)
    MX[:, :, 0] = v
    MX[:, :, 1] = idx.view(np.float32)
    out = ref.argmaxM(MX.ravel(), n, M).reshape(M, 2)
    for m in range(M):
        vm = np.where(np.isnan(v[m]), -np.inf, v[m])
        best = vm.max()
        assert out[m, 0] == idx[m][vm == best].min()
        assert out[m, 1] == np.float32(best).view(np.uint32)
    assert out[1, 0] == 40


def _deq_row(b, enc, i, K):
    """row i of a q4 / q8 table dequantised in numpy f32: q * s + mn (q4) or q * s (q8), before any fp16 rounding"""
    raw = np.frombuffer(np.asarray(b, np.uint8).tobytes(), np.uint8)
    t, r = i // 64, i % 64
    if enc == "q4g32a.t64":
        rec = [raw[(t * (K // 32) + g) * 1280:(t * (K // 32) + g + 1) * 1280] for g in range(K // 32)]
        q = np.concatenate([np.stack([rc[r * 16:r * 16 + 16] & 15, rc[r * 16:r * 16 + 16] >> 4], 1).ravel() for rc in rec])
        sm = np.array([rc[1024 + 4 * r:1028 + 4 * r].view(np.uint16) for rc in rec])
        s, mn = np.repeat(ref.h2f(sm[:, 0]), 32).astype(np.float32), np.repeat(ref.h2f(sm[:, 1]), 32).astype(np.float32)
        return q.astype(np.float32) * s + mn
    rec = [raw[(t * (K // 64) + g) * 4224:(t * (K // 64) + g + 1) * 4224] for g in range(K // 64)]
    q = np.concatenate([rc[r * 64:r * 64 + 64].view(np.int8) for rc in rec]).astype(np.float32)
    s = np.repeat(ref.h2f(np.array([rc[4096 + 2 * r:4098 + 2 * r].view(np.uint16)[0] for rc in rec])), 64).astype(np.float32)
    return q * s


@pytest.mark.parametrize("enc", ["q4g32a.t64", "q8g64s.t64"])
def test_embed_oracle_against_dequant(enc):
    V, K = 192, 256
    b, _ = (ref.pack_q4 if enc == "q4g32a.t64" else ref.pack_q8)(ref.randn(V * K, 30, 0.05), V, K)
    ids = np.array([0, 63, 64, 191, 7], np.uint32)
    X, ST = ref.embed(b, ids, K, enc=enc, scale=1.5, eps=1e-6)
    for m, i in enumerate(ids):
        row = _deq_row(b, enc, int(i), K) * np.float32(1.5)
        assert np.array_equal(X[m * K:(m + 1) * K], row)
        want = 1.0 / np.sqrt(np.mean(row.astype(np.float64) ** 2) + 1e-6)
        assert abs(ST[m] - want) <= 1e-5 * want


@pytest.mark.parametrize("mode,nsrc", [(0, 1), (0, 3), (1, 2)])
def test_normadd_oracle(mode, nsrc):
    M, D = 3, 1000
    T = ref.randn(nsrc * M * D, 40, 1.0)
    W = ref.randn(D + 5, 41, 0.2) + 1
    X0 = ref.randn(M * D, 42)
    X, ST = X0.copy(), np.zeros(M + 2, np.float32)
    ref.normadd(T, nsrc, M * D, W, 5, X, ST, 2, D, M, mode=mode, eps=1e-6, scale=0.7)
    t = T.astype(np.float64).reshape(nsrc, M, D).sum(0)
    if mode == 0:
        rs = 1 / np.sqrt((t ** 2).mean(1, keepdims=True) + 1e-6)
        want = (X0.astype(np.float64).reshape(M, D) + t * rs * W[5:]) * 0.7
    else:
        want = t
    assert np.max(np.abs(X.reshape(M, D) - want)) <= 1e-5 * max(1.0, np.abs(want).max())
    assert np.allclose(ST[2:], 1 / np.sqrt((want ** 2).mean(1) + 1e-6), rtol=1e-5)


@pytest.mark.parametrize("enc,K", [("q4g32a.t64", 512), ("q8g64s.t64", 256)])
def test_dhead_oracle(enc, K):
    V = 64 * 12
    b, _ = (ref.pack_q4 if enc == "q4g32a.t64" else ref.pack_q8)(ref.randn(V * K, 50, 0.05), V, K)
    X, NW = ref.randn(K, 51), ref.randn(K + 3, 52, 0.1) + 1
    ST = np.array([0.0, 0.8], np.float32)
    SEL = np.array([4, 1, 3], np.uint32)
    MX = ref.dhead(b, X, ST, NW, SEL, K, 2, 3, enc=enc, stat_off=1, norm_off=3)
    xs = X.astype(np.float64) * 0.8 * NW[3:]
    for wt in range(6):
        tile = SEL[wt // 2] * 2 + wt % 2
        rows = np.array([_deq_row(b, enc, int(tile) * 64 + r, K) for r in range(64)], np.float64)
        dots = rows @ xs
        r = int(np.argmax(dots))
        assert MX[2 * wt + 1].view(np.uint32) == tile * 64 + r
        assert abs(MX[2 * wt] - dots[r]) <= 1e-4 * max(1.0, abs(dots[r]))


def test_qkrope_oracle():
    D, nq, nkv, kv_len, row, pos, npairs = 256, 4, 2, 10, 7, 3, 32
    nh = nq + 2 * nkv
    S = ref.randn(2 * nh * D, 60, 1.0)
    NW = ref.randn(2 * D + 4, 61, 0.2) + 1
    ang = ref.randn(8 * npairs, 62, 2.0).astype(np.float64)
    RP = np.empty(5 + 16 * npairs, np.float32)
    RP[5:5 + 16 * npairs:2], RP[6:5 + 16 * npairs:2] = np.cos(ang), np.sin(ang)
    Q, KC, VC = ref.qkrope(S, 2, nh * D, NW, RP, D, nq, nkv=nkv, pos=pos, qw=4, kw=4 + D, npairs=npairs, rope_off=5, kv_row=row,
                           kv_len=kv_len)
    x = S.astype(np.float64).reshape(2, nh, D).sum(0)
    rs = 1 / np.sqrt((x ** 2).mean(1, keepdims=True) + 1e-6)
    cs, sn = np.ones(D // 2), np.zeros(D // 2)
    cs[:npairs], sn[:npairs] = np.cos(ang[pos * npairs:(pos + 1) * npairs]), np.sin(ang[pos * npairs:(pos + 1) * npairs])
    for h in range(nh):
        if h >= nq + nkv:
            want = x[h] * rs[h]
            got = ref.h2f(VC.reshape(nkv, kv_len, D)[h - nq - nkv, row])
        else:
            w = NW[4:4 + D] if h < nq else NW[4 + D:4 + 2 * D]
            v = x[h] * rs[h] * w
            a, b = v[:D // 2], v[D // 2:]
            want = np.concatenate([a * cs - b * sn, b * cs + a * sn])
            got = Q.reshape(nq, D)[h] if h < nq else ref.h2f(KC.reshape(nkv, kv_len, D)[h - nq, row])
        assert np.max(np.abs(got - want)) <= (1e-5 if h < nq else 2e-3) * max(1.0, np.abs(want).max())


@pytest.mark.parametrize("D,nh,nkv,k0,k1,ring", [(256, 8, 2, 5, 290, 0), (512, 8, 1, 0, 64, 0), (128, 4, 4, 30, 200, 100)])
def test_attn_dec_oracle(D, nh, nkv, k0, k1, ring):
    L = 300
    Q = ref.randn(nh * D, 70, 0.08)
    KC, VC = ref.f2h(ref.round_f16(ref.randn(nkv * L * D, 71))), ref.f2h(ref.round_f16(ref.randn(nkv * L * D, 72)))
    O = ref.attn_dec(Q, KC, VC, D, nh, nkv, L, k0, k1, ring)
    K, V, q = ref.h2f(KC).reshape(nkv, L, D), ref.h2f(VC).reshape(nkv, L, D), Q.reshape(nh, D).astype(np.float64)
    rows = np.array([j % ring if ring else j for j in range(k0, k1)])
    for h in range(nh):
        g = h // (nh // nkv)
        s = K[g, rows] @ q[h]
        p = np.exp(s - s.max())
        assert np.max(np.abs(O[h * D:(h + 1) * D] - (p / p.sum()) @ V[g, rows])) <= 1e-5


# ---------------------------------------------------------------- q8g64s.t64 (kcheck.js:39-52) in the oracle
def test_pack_q8_matches_transcription():
    N, K = 64, 128
    W = ref.randn(N * K, 80, 0.05)
    W[:64] = 0.0                                                   # an all-zero group: s = 1
    W[K:K + 64] = np.linspace(-1e-6, 1e-6, 64, dtype=np.float32)   # a subnormal fp16 scale
    W[2 * K:2 * K + 64] = 0.5 * np.arange(64, dtype=np.float32) / 127.0   # ties for round-half-even
    got, deq = ref.pack_q8(W, N, K)
    want, wdeq = jsref.pack_q8([float(v) for v in W], N, K)
    assert bytes(np.asarray(got, np.uint8)) == want
    assert np.array_equal(np.asarray(deq, np.float32).ravel(), np.asarray(wdeq, np.float32))


def test_q8_gemv_and_gemm_oracle_against_dequantised_weights():
    # the q8 GEMV (f32 x, f32 accumulate) against an f64 dot with q*s; the q8 GEMM against f64 with f16(q*s) tiles
    N, K, M = 128, 256, 3
    W = ref.randn(N * K, 81, 0.05)
    b, deq = ref.pack_q8(W, N, K)
    deq = np.asarray(deq, np.float64).reshape(N, K)
    x = ref.randn(K, 82).astype(np.float64)
    y, _, _ = ref.gemv(b, x.astype(np.float32), N, K, enc="q8g64s.t64")
    assert np.max(np.abs(y - deq @ x)) <= 1e-4 * max(1.0, np.abs(deq @ x).max())
    X16 = ref.f2h(ref.round_f16(ref.randn(M * K, 83)))
    Y = ref.h2f(ref.gemm(b, X16, M, N, K, enc="q8g64s.t64"))
    w16 = ref.h2f(ref.deq16(b, N, K, enc="q8g64s.t64")).reshape(N, K)
    want = ref.h2f(X16).reshape(M, K) @ w16.T
    assert np.max(np.abs(Y.reshape(M, N) - want)) <= 2e-3 * max(1.0, np.abs(want).max())


# ---------------------------------------------------------------- the GEMM epilogues (gemm.js:187-211) on the accumulators
def test_gemm_epilogues_oracle():
    # every epilogue restated in numpy (f64, then the store's rounding) on the same f32 accumulators (the 'f32' store)
    M, N, K = 5, 256, 128
    b, _ = ref.pack_q4(ref.randn(N * K, 90, 0.05), N, K)
    X = ref.f2h(ref.round_f16(ref.randn(M * K, 91)))
    A = ref.gemm(b, X, M, N, K, epi="f32").reshape(M, N).astype(np.float64)
    assert np.array_equal(ref.gemm(b, X, M, N, K), ref.f2h(A.astype(np.float32).astype(np.float64).ravel()))   # 'f16' = f16(acc)
    bias = ref.randn(N, 92, 0.1).astype(np.float64)
    y0 = ref.f2h(ref.round_f16(ref.randn(M * N, 93)))
    got = ref.h2f(ref.gemm(b, X, M, N, K, epi="bias", ev=bias.astype(np.float32), res=True, Y=y0.copy())).reshape(M, N)
    assert np.max(np.abs(got - (A + bias + ref.h2f(y0).reshape(M, N)))) <= 4e-3 * max(1.0, np.abs(got).max())
    gate, cb = ref.randn(N, 94, 0.5).astype(np.float64), ref.randn(N, 95, 0.1).astype(np.float64)
    r0 = ref.randn(M * N, 96)
    got = ref.gemm(b, X, M, N, K, epi="resadd", ev=gate.astype(np.float32), bv=cb.astype(np.float32), Y=r0.copy()).reshape(M, N)
    assert np.max(np.abs(got - (r0.reshape(M, N) + gate * (A + cb)))) <= 1e-5 * max(1.0, np.abs(got).max())
    # swiglu: weight rows [gate 0..N/2) | up [N/2..N), interleaved (gate n, up n) in the accumulator columns
    for act in ("silu", "gelu"):
        got = ref.h2f(ref.gemm(b, X, M, N, K, epi="swiglu", act=act, wr0=0, wr1=N // 2, ldy=N // 2)).reshape(M, N // 2)
        Ar = ref.gemm(b, X, M, N, K, epi="f32").reshape(M, N).astype(np.float64)   # plain rows 0..N-1
        g_, u = Ar[:, :N // 2], Ar[:, N // 2:]
        if act == "silu":
            a = g_ / (1 + np.exp(-g_))
        else:
            a = g_ * 0.5 * (1 + np.tanh(np.clip(0.7978845608 * (g_ + 0.044715 * g_ ** 3), -15, 15)))
        want = a * u
        assert np.max(np.abs(got - want)) <= 4e-3 * max(1.0, np.abs(want).max())


def test_gemm_f16_weights_oracle():
    # fp16 weights with a row stride wider than the columns and a k offset: the oracle reads W[row * ld + wk0 + k]
    M, N, K, ld, wk0 = 4, 96, 128, 200, 40
    W = ref.f2h(ref.round_f16(ref.randn(N * ld, 97, 0.05)))
    X = ref.f2h(ref.round_f16(ref.randn(M * K, 98)))
    got = ref.h2f(ref.gemm(W, X, M, N, K, enc="f16", rows=N, cols=ld, wk0=wk0)).reshape(M, N)
    want = ref.h2f(X).reshape(M, K) @ ref.h2f(W).reshape(N, ld)[:, wk0:wk0 + K].T
    assert np.max(np.abs(got - want)) <= 2e-3 * max(1.0, np.abs(want).max())


@pytest.mark.parametrize("mode", ["lnmod", "rms"])
def test_gemm_xpro_oracle(mode):
    # the f32 x prologues (gemm.js:55-63) against numpy in the WGSL's order of f32 operations, then fp16 rounding
    M, K, ldx, kx0 = 6, 96, 130, 32
    X = ref.randn(M * ldx, 99)
    st = np.empty(2 * (M + 2), np.float32)
    st[0::2], st[1::2] = ref.randn(M + 2, 100, 0.2), 0.5 + np.abs(ref.randn(M + 2, 101, 0.3))
    pv = ref.randn(4 + 2 * 200, 102, 0.2)
    got = ref.gemm_xpro(mode, X, M, K, ldx=ldx, kx0=kx0, stats=st, stat_off=2, pv=pv, pv_off=4, pv_stride=200)
    x = X.reshape(M, ldx)[:, kx0:kx0 + K]
    mean, rstd = st[4::2][:M, None], st[5::2][:M, None]
    f = np.float32
    if mode == "lnmod":
        v = ((x - mean).astype(f) * rstd).astype(f) * (f(1) + pv[4 + kx0:4 + kx0 + K]).astype(f)
        v = (v.astype(f) + pv[204 + kx0:204 + kx0 + K]).astype(f)
    else:
        v = ((x * rstd).astype(f) * pv[4 + kx0:4 + kx0 + K]).astype(f)
    assert np.array_equal(got, ref.f2h(v.astype(np.float64).ravel()))


# ---------------------------------------------------------------- the oracle's kernel arithmetic against a second,
# independent transcription of the WGSL (tests/jsref_kernels.py, numpy), bit for bit on small shapes
from . import jsref_kernels as jk  # noqa: E402


def _bits_equal(a, b):
    a, b = np.asarray(a), np.asarray(b)
    assert a.shape == b.shape
    if a.dtype == np.float32:
        a, b = a.view(np.uint32), b.view(np.uint32)
    diff = np.nonzero(a != b)[0]
    assert diff.size == 0, "%d of %d differ, first at %d: %r vs %r" % (diff.size, a.size, diff[0], a[diff[0]], b[diff[0]])


@pytest.mark.parametrize("enc", ["q4g32a.t64", "q8g64s.t64"])
@pytest.mark.parametrize("pro,epi,kPer", [("raw", "store", None), ("raw", "store", 256), ("rms", "softcap", None), ("rms", "geglu", None),
                                          ("sum", "store", None), ("pleg", "store", None)])
def test_gemv_second_transcription(enc, pro, epi, kPer):
    N, K = 128, 512
    rows = 2 * N if epi == "geglu" else N
    W = ref.randn(rows * K, 900, 0.02)
    b = (ref.pack_q4 if enc == "q4g32a.t64" else ref.pack_q8)(W, rows, K)[0]
    kw = {}
    X = ref.randn(2 * K + 64, 901)
    okw = {}
    if pro == "rms":
        # the rstd slot: in the MX buffer past the tile pairs for softcap (lops.js:125), else the stat buffer
        st = np.zeros(N // 64 * 2 + 4, np.float32)
        st[N // 64 * 2 + 1] = 0.83
        kw.update(stat=st.copy(), stat_off=N // 64 * 2 + 1, norm=ref.randn(K + 16, 902, 0.1) + 1, norm_off=16)
        okw = {"mx": st.copy()} if epi == "softcap" else {"stat_buf": st.copy()}
        okw.update(stat_off=kw["stat_off"], norm=kw["norm"], norm_off=16)
    if pro in ("sum", "pleg"):
        kw.update(src=(K + 32, 2))
    if pro == "pleg":
        kw.update(ev=ref.randn(K + 8, 903, 0.5), ev_off=8)
    if pro in ("sum", "pleg"):
        okw = {k: v for k, v in kw.items()}
    rowB = 32 if pro in ("raw", "rms") else 0
    want_y, want_mx, ns = ref.gemv(b, X, N, K, enc=enc, rowB=rowB, kPer=kPer, pro=pro, epi=epi, **okw)
    got_y, got_mx, ns2 = jk.gemv(b, X, N, K, enc=enc, rowB=rowB, kPer=kPer, pro=pro, epi=epi, **kw)
    assert ns == ns2
    _bits_equal(got_y, want_y[:got_y.size])
    if epi == "softcap":
        _bits_equal(got_mx, want_mx[:got_mx.size])


@pytest.mark.parametrize("M", [2, 3])
@pytest.mark.parametrize("pro,epi,kPer", [("raw", "store", 128), ("rms", "softcap", None), ("rms", "geglu", None), ("pleg", "store", None)])
def test_gemvM_second_transcription(M, pro, epi, kPer):
    N, K = 128, 256
    rows = 2 * N if epi == "geglu" else N
    b, _ = ref.pack_q4(ref.randn(rows * K, 910, 0.02), rows, K)
    ldx = K + 32
    X = ref.randn(2 * M * ldx, 911)
    kw = {}
    if pro == "rms":
        kw.update(stat=np.array([0.7, 0, 0.8, 0, 0.9, 0], np.float32), stat_ld=2, norm=ref.randn(K, 912, 0.1) + 1)
    if pro == "pleg":
        kw.update(src=(M * ldx, 2), ev=ref.randn(M * K, 913, 0.5), ev_ld=K)
    want_y, want_mx, ns = ref.gemvM(b, X, M, N, K, ldx=ldx, kPer=kPer, pro=pro, epi=epi, **kw)
    got_y, got_mx, ns2 = jk.gemvM(b, X, M, N, K, ldx=ldx, kPer=kPer, pro=pro, epi=epi, **kw)
    assert ns == ns2
    _bits_equal(got_y, want_y[:got_y.size])
    if epi == "softcap":
        _bits_equal(got_mx, want_mx)


@pytest.mark.parametrize("enc", ["q4g32a.t64", "q8g64s.t64"])
@pytest.mark.parametrize("acc", ["f32", "f16"])
@pytest.mark.parametrize("epi", ["f16", "f32", "bias", "bias_gelu", "resadd", "swiglu_silu", "swiglu_gelu"])
def test_gemm_second_transcription(enc, acc, epi):
    M, N, K = 6, 128, 128
    W = ref.randn(N * K, 920, 0.02)
    b = (ref.pack_q4 if enc == "q4g32a.t64" else ref.pack_q8)(W, N, K)[0]
    X = ref.f2h(ref.round_f16(ref.randn(M * K, 921)))
    kw = {}
    e = epi
    if epi.startswith("bias"):
        e = "bias"
        kw.update(ev=ref.randn(N + 4, 922, 0.01), ev_off=4, res=True, post_gelu=epi == "bias_gelu",
                  Y=ref.f2h(ref.randn(M * N, 923, 0.5)))
    elif epi == "resadd":
        kw.update(ev=ref.randn(N, 924, 1.0), bv=ref.randn(N, 925, 0.01), Y=ref.randn(M * N, 926))
    elif epi.startswith("swiglu"):
        e = "swiglu"
        kw.update(act=epi.split("_")[1], wr0=0, wr1=N // 2, bv=ref.randn(N, 927, 0.01), bv_up=N // 2)
    want = ref.gemm(b, X, M, N, K, enc=enc, epi=e, acc=acc, **{k: (v.copy() if isinstance(v, np.ndarray) and k == "Y" else v) for k, v in kw.items()})
    got = jk.gemm(b, X, M, N, K, enc=enc, epi=e, acc=acc, **kw)
    _bits_equal(got, want)


@pytest.mark.parametrize("mode", ["lnmod", "rms"])
def test_gemm_x_prologue_second_transcription(mode):
    M, K, ldx, kx0, stat_off, pv_off, pv_stride = 5, 96, 120, 16, 3, 8, 136
    X = ref.randn(M * ldx, 940, 2.0)
    X[7] = 70000.0                     # beyond fp16's range after the prologue: both round to inf alike
    st = ref.randn(2 * (stat_off + M), 941, 0.5)
    st[1::2] = np.abs(st[1::2]) + 0.25
    pv = ref.randn(pv_off + pv_stride + kx0 + K, 942, 0.3)
    want = ref.gemm_xpro(mode, X, M, K, ldx=ldx, kx0=kx0, stats=st, stat_off=stat_off, pv=pv, pv_off=pv_off, pv_stride=pv_stride)
    got = jk.gemm_xpro(mode, X, M, K, ldx=ldx, kx0=kx0, stats=st, stat_off=stat_off, pv=pv, pv_off=pv_off, pv_stride=pv_stride)
    _bits_equal(got, want)


@pytest.mark.parametrize("form", ["heads_half", "heads_inter", "onormgate"])
def test_gemm_red128_second_transcription(form):
    # q, k and v heads (Hq 2, Hkv 1: heads 0-1 q, 2 k, 3 v), rows written at rowOff into a head buffer of Ltot rows; the
    # onormgate form into a column range of a wider Y with its gate rows of ld Ltot
    M, K = 6, 128
    N = 4 * 128 if form != "onormgate" else 128
    b = ref.pack_q4(ref.randn(N * K, 950, 0.02), N, K)[0]
    X = ref.f2h(ref.round_f16(ref.randn(M * K, 951)))
    A = jk.gemm(b, X, M, N, K, epi="f32")
    ev = ref.randn(256 + 8, 952, 0.2) + 1
    if form == "onormgate":
        Ltot, ldy, ny0 = 3 * 128, 2 * 128, 128
        gt = ref.f2h(ref.round_f16(ref.randn(M * Ltot, 953)))
        heads = {"Ltot": Ltot, "eps": 1e-5 / 64.0}
        Y0 = ref.f2h(ref.randn(M * ldy, 954, 0.5))
        want = ref.gemm(b, X, M, N, K, epi="onormgate", ev=ev, ev_off=8, heads=heads, gt=gt, Y=Y0.copy(), ldy=ldy, ny0=ny0)
        got = jk.gemm_red128(A, M, N, epi="onormgate", ev=ev, ev_off=8, heads=heads, gt=gt, Y=Y0, ldy=ldy, ny0=ny0)
    else:
        Ltot, rowOff = M + 5, 3
        ang = ref.randn(Ltot * 64, 955, 3.0).astype(np.float64)
        rope = np.empty(Ltot * 128, np.float32)
        rope[0::2], rope[1::2] = np.cos(ang), np.sin(ang)
        heads = {"Ltot": Ltot, "Hq": 2, "Hkv": 1, "rowOff": rowOff, "eps": 1e-6, "ropeMode": "half" if form == "heads_half" else "inter",
                 "rope": rope}
        Y0 = ref.f2h(ref.randn(4 * Ltot * 128, 956, 0.5))
        want = ref.gemm(b, X, M, N, K, epi="heads", ev=ev, ev_off=8, heads=heads, Y=Y0.copy())
        got = jk.gemm_red128(A, M, N, epi="heads", ev=ev, ev_off=8, heads=heads, Y=Y0)
    _bits_equal(got, want)


@pytest.mark.parametrize("mode,nsrc,D", [(0, 1, 1000), (0, 3, 1152), (1, 2, 640), (0, 2, 200)])
def test_normadd_second_transcription(mode, nsrc, D):
    M = 3
    T = ref.randn(nsrc * M * D, 960, 1.0)
    W = ref.randn(D + 5, 961, 0.2) + 1
    X0, ST0 = ref.randn(M * D, 962), np.zeros(M + 2, np.float32)
    X, ST = ref.normadd(T, nsrc, M * D, W, 5, X0.copy(), ST0.copy(), 2, D, M, mode=mode, eps=1e-6, scale=0.7)
    jX, jST = jk.normadd(T, nsrc, M * D, W, 5, X0, ST0, 2, D, M, mode=mode, eps=1e-6, scale=0.7)
    _bits_equal(jX, X)
    _bits_equal(jST, ST)


@pytest.mark.parametrize("D,nq,nkv,npairs,hasKV", [(256, 4, 2, 32, True), (128, 8, 1, 64, True), (512, 2, 1, 100, False)])
def test_qkrope_second_transcription(D, nq, nkv, npairs, hasKV):
    kv_len, row, pos = 10, 7, 3
    nh = nq + 2 * nkv
    S = ref.randn(2 * nh * D, 963, 1.0)
    NW = ref.randn(2 * D + 4, 964, 0.2) + 1
    ang = ref.randn(8 * npairs, 965, 2.0).astype(np.float64)
    RP = np.empty(5 + 16 * npairs, np.float32)
    RP[5:5 + 16 * npairs:2], RP[6:5 + 16 * npairs:2] = np.cos(ang), np.sin(ang)
    kw = dict(nkv=nkv, hasKV=hasKV, pos=pos, qw=4, kw=4 + D, npairs=npairs, rope_off=5, kv_row=row, kv_len=kv_len)
    KC0 = ref.f2h(ref.randn(nkv * kv_len * D, 966, 0.5))
    VC0 = ref.f2h(ref.randn(nkv * kv_len * D, 967, 0.5))
    Q, KC, VC = ref.qkrope(S, 2, nh * D, NW, RP, D, nq, KC=KC0.copy(), VC=VC0.copy(), **kw)
    jQ, jKC, jVC = jk.qkrope(S, 2, nh * D, NW, RP, D, nq, KC=KC0, VC=VC0, **kw)
    _bits_equal(jQ, Q)
    _bits_equal(jKC, KC)
    _bits_equal(jVC, VC)


@pytest.mark.parametrize("D,nh,nkv,k0,k1,ring", [(128, 8, 2, 5, 150, 0), (256, 4, 1, 0, 64, 0), (128, 4, 4, 30, 200, 100)])
def test_attn_dec_second_transcription(D, nh, nkv, k0, k1, ring):
    L = 210
    Q = ref.randn(nh * D, 968, 0.08)
    KC, VC = ref.f2h(ref.round_f16(ref.randn(nkv * L * D, 969))), ref.f2h(ref.round_f16(ref.randn(nkv * L * D, 970)))
    O = ref.attn_dec(Q, KC, VC, D, nh, nkv, L, k0, k1, ring)
    _bits_equal(jk.attn_dec(Q, KC, VC, D, nh, nkv, L, k0, k1, ring), O)


@pytest.mark.parametrize("enc,K", [("q4g32a.t64", 640), ("q8g64s.t64", 320)])
def test_embed_second_transcription(enc, K):
    V = 64 * 5
    b = (ref.pack_q4 if enc == "q4g32a.t64" else ref.pack_q8)(ref.randn(V * K, 975, 0.05), V, K)[0]
    ids = np.array([7, 300, 64, 0, 129], np.uint32)
    X, ST = ref.embed(b, ids, K, enc=enc, scale=22.6, eps=1e-6, st_off=2, row_out=1)
    jX, jST = jk.embed(b, ids, K, enc=enc, scale=22.6, eps=1e-6, st_off=2, row_out=1)
    _bits_equal(jX, X)
    _bits_equal(jST, ST)


@pytest.mark.parametrize("enc,K", [("q4g32a.t64", 256), ("q8g64s.t64", 128)])
def test_dhead_second_transcription(enc, K):
    V = 64 * 8
    b = (ref.pack_q4 if enc == "q4g32a.t64" else ref.pack_q8)(ref.randn(V * K, 976, 0.05), V, K)[0]
    X, NW = ref.randn(K, 977), ref.randn(K + 3, 978, 0.1) + 1
    ST = np.array([0.0, 0.8], np.float32)
    SEL = np.array([3, 0, 2], np.uint32)
    MX = ref.dhead(b, X, ST, NW, SEL, K, 2, 3, enc=enc, stat_off=1, norm_off=3)
    _bits_equal(jk.dhead(b, X, ST, NW, SEL, K, 2, 3, enc=enc, stat_off=1, norm_off=3), MX)


def test_fast_fp16_fma_equals_definitional():
    # the GEMM's fp16-partial accumulation uses a table / add-and-subtract form of the oracle's fp16 FMA (one rounding of
    # the f64 value a*b + c to fp16, ties to even); it must give the definitional form's bits on every input
    rng = np.random.default_rng(990)
    n = 2_000_000
    a, b, c = (rng.integers(0, 65536, n, dtype=np.uint32).astype(np.uint16) for _ in range(3))
    a[: n // 2] &= 0xBFFF                      # half the products in a moderate range, where rounding ties occur
    b[: n // 2] &= 0xBFFF
    special = np.array([0, 0x8000, 0x0001, 0x8001, 0x03FF, 0x0400, 0x7BFF, 0xFBFF, 0x7C00, 0xFC00, 0x7E00, 0x3C00, 0xBC00], np.uint16)
    sa, sb, sc = (g.ravel() for g in np.meshgrid(special, special, special, indexing="ij"))
    a, b, c = np.concatenate([a, sa]), np.concatenate([b, sb]), np.concatenate([c, sc])
    want, got = np.empty_like(a), np.empty_like(a)
    L = ref.lib()
    L.or_hfma_arr(a, b, c, a.size, want)
    L.or_hfma_d_arr(a, b, c, a.size, got)
    nan = lambda h: ((h & 0x7C00) == 0x7C00) & ((h & 0x3FF) != 0)
    assert np.all((got == want) | (nan(got) & nan(want)))
