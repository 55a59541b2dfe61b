"""GPU parity of the GEMM's forms against the CPU oracle, through ops.gemm. The library picks the form per call
(measured on B200, configs 3 and 4): Cfg7 (one 128-row x 256-token tile per CTA, 128-k stages, dequantised weights in
tensor memory) for q4 records by bulk copy in 256-token tiles; else the persistent form (one CTA per SM walking the
tiles, two tensor-memory accumulators, dequantised weights in shared memory) for q4 records by bulk copy with a store
epilogue when the CTAs get more than one tile and K is at most 96 stages; else Cfg1 (64-k stages: q8 and fp16
weights, gathered rows, tiles of fewer tokens). P0MM_GEMM forces a form: 7 = Cfg7, 6 = persistent, 5 = the CTA pair
(a 2-CTA cluster on one tcgen05.mma.cta_group::2 of 256 weight rows, each CTA loading half of the token tile's X;
about 0.8x Cfg1, never chosen by default), 1 = Cfg1. The cases cover a token count that is not a multiple of 256,
an odd count of 128-row tiles (a pair's odd CTA past the last weight row stores nothing), K with a one-group last
stage, and the bias (+ GELU), f32, resadd, swiglu and heads epilogues (engine/ops/gemm.js:187-250); the many-tile
cases make every persistent CTA walk several tiles, so both accumulators and the ring are reused across tiles."""
import numpy as np
import pytest

from oracle import ref

from .test_gpu_gemm_heads import rope_table, run_heads
from .test_gpu_gemm_xpro import _case as xpro_case
from .test_gpu_parity import assert_close, run_gemm

pytestmark = pytest.mark.gpu


@pytest.fixture(params=["7", "6", "5", "1"], ids=["k128", "persistent", "pair", "cfg1"])
def form(request, monkeypatch):
    monkeypatch.setenv("P0MM_GEMM", request.param)
    return request.param


@pytest.mark.parametrize("M,N,K", [(300, 384, 352), (400, 384, 512), (257, 128, 64)])
def test_form_f16(g, form, M, N, K):
    b, _ = ref.pack_q4(ref.randn(N * K, 190 + M, 0.02), N, K)
    X = ref.f2h(ref.round_f16(ref.randn(M * K, 191)))
    y = run_gemm(g, b, X, M, N, K)
    assert_close(ref.h2f(y), ref.h2f(ref.gemm(b, X, M, N, K)))


def test_form_bias_gelu(g, form):
    M, N, K = 300, 384, 512
    b, _ = ref.pack_q4(ref.randn(N * K, 192, 0.02), N, K)
    X = ref.f2h(ref.round_f16(ref.randn(M * K, 193)))
    bias = ref.randn(N, 194, 0.01)
    y = run_gemm(g, b, X, M, N, K, epi="bias", ev=(bias, 0), post_gelu=True)
    assert_close(ref.h2f(y), ref.h2f(ref.gemm(b, X, M, N, K, epi="bias", ev=bias, post_gelu=True, threads=0)))


def test_form_resadd_f32(g, form):
    M, N, K = 400, 384, 512
    b, _ = ref.pack_q4(ref.randn(N * K, 195, 0.02), N, K)
    X = ref.f2h(ref.round_f16(ref.randn(M * K, 196)))
    gate, bv = ref.randn(N, 197, 1.0), ref.randn(N, 198, 0.01)
    r0 = ref.randn(M * N, 199)
    y = run_gemm(g, b, X, M, N, K, y_init=r0.copy(), epi="resadd", ev=(gate, 0), bv=(bv, 0), store=False)
    assert_close(y, ref.gemm(b, X, M, N, K, epi="resadd", ev=gate, bv=bv, store=False, Y=r0.copy(), threads=0))
    yf = run_gemm(g, b, X, M, N, K, y_bytes=M * N * 4, epi="f32")
    assert_close(yf, ref.gemm(b, X, M, N, K, epi="f32", threads=0))


@pytest.mark.parametrize("act", ["silu", "gelu"])
def test_form_swiglu(g, form, act):
    M, N, K = 300, 768, 512
    b, _ = ref.pack_q4(ref.randn(N * K, 200, 0.02), N, K)
    X = ref.f2h(ref.round_f16(ref.randn(M * K, 201)))
    bv = ref.randn(N, 202, 0.01)
    y = run_gemm(g, b, X, M, N, K, epi="swiglu", act=act, wr0=0, wr1=N // 2, bv=(bv, 0, N // 2), y={"ld": N // 2})
    want = ref.gemm(b, X, M, N, K, epi="swiglu", act=act, wr0=0, wr1=N // 2, bv=bv, bv_up=N // 2, ldy=N // 2, threads=0)
    assert_close(ref.h2f(y), ref.h2f(want))


def test_form_heads(g, form):
    # 3 q heads + 1 k head + 1 v head = 5 row tiles (odd), 300 tokens, rotate_half RoPE
    M, Hq, Hkv, K = 300, 3, 1, 512
    N = (Hq + 2 * Hkv) * 128
    b, _ = ref.pack_q4(ref.randn(N * K, 203, 0.02), N, K)
    X = ref.f2h(ref.round_f16(ref.randn(M * K, 204)))
    ev = ref.randn(256 + 8, 205, 0.2) + 1
    rp = rope_table(M, 206)
    heads = {"Ltot": M, "Hq": Hq, "Hkv": Hkv, "rowOff": 0, "eps": 1e-6, "ropeMode": "half"}
    y0 = ref.f2h(ref.round_f16(ref.randn(N // 128 * M * 128, 207)))
    yb = g.upload(y0)
    run_heads(g, b, X, M, N, K, yb, (ev, 8), rp, heads)
    want = ref.gemm(b, X, M, N, K, epi="heads", ev=ev, ev_off=8, heads={**heads, "rope": rp}, Y=y0.copy(), threads=0)
    assert_close(ref.h2f(g.read(yb, 0, y0.size * 2, np.uint16)), ref.h2f(want))


# ---------------------------------------------------------------- the default (persistent) form over many tiles per CTA
@pytest.mark.parametrize("M,N,K", [(200, 57344, 32), (130, 38400, 96), (100, 40960, 64)])
def test_persistent_many_tiles(g, monkeypatch, M, N, K):
    monkeypatch.setenv("P0MM_GEMM", "6")
    # 300-448 tiles on 148 SMs: every CTA walks two or three, so both accumulators are reused and the ring runs across
    # tiles (one-stage tiles; two stages with a one-group last stage; 128-token tiles)
    b, _ = ref.pack_q4(ref.randn(N * K, 210 + K, 0.02), N, K)
    X = ref.f2h(ref.round_f16(ref.randn(M * K, 211)))
    bias = ref.randn(N, 212, 0.01)
    y = run_gemm(g, b, X, M, N, K, epi="bias", ev=(bias, 0))
    assert_close(ref.h2f(y), ref.h2f(ref.gemm(b, X, M, N, K, epi="bias", ev=bias, threads=0)))


def test_persistent_many_tiles_swiglu_resadd(g, monkeypatch):
    monkeypatch.setenv("P0MM_GEMM", "6")
    M, N, K = 130, 40960, 64
    b, _ = ref.pack_q4(ref.randn(N * K, 213, 0.02), N, K)
    X = ref.f2h(ref.round_f16(ref.randn(M * K, 214)))
    bv = ref.randn(N, 215, 0.01)
    y = run_gemm(g, b, X, M, N, K, epi="swiglu", act="gelu", wr0=0, wr1=N // 2, bv=(bv, 0, N // 2), y={"ld": N // 2})
    want = ref.gemm(b, X, M, N, K, epi="swiglu", act="gelu", wr0=0, wr1=N // 2, bv=bv, bv_up=N // 2, ldy=N // 2, threads=0)
    assert_close(ref.h2f(y), ref.h2f(want))
    gate = ref.randn(N, 216, 1.0)
    r0 = ref.randn(M * N, 217)
    y2 = run_gemm(g, b, X, M, N, K, y_init=r0.copy(), epi="resadd", ev=(gate, 0), bv=(bv, 0), store=False)
    assert_close(y2, ref.gemm(b, X, M, N, K, epi="resadd", ev=gate, bv=bv, store=False, Y=r0.copy(), threads=0))


# ---------------------------------------------------------------- k split (grids that fill at most half the SMs)
@pytest.mark.parametrize("ks", ["auto", "3"])
@pytest.mark.parametrize("gemm_form", ["7", "1"], ids=["k128", "cfg1"])
def test_ksplit_epilogues(g, monkeypatch, gemm_form, ks):
    # 130 tokens x 512 rows = 4 CTAs: the library splits K (2080 = 16.25 x 128: the last split ends on a one-group
    # stage); each split stores f32 partials, a second pass sums them in order and applies the epilogue
    monkeypatch.setenv("P0MM_GEMM", gemm_form)
    if ks != "auto":
        monkeypatch.setenv("P0MM_GEMM_KSPLIT", ks)
    M, N, K = 130, 512, 2080
    b, _ = ref.pack_q4(ref.randn(N * K, 220, 0.02), N, K)
    X = ref.f2h(ref.round_f16(ref.randn(M * K, 221)))
    bias, gate = ref.randn(N, 222, 0.01), ref.randn(N, 223, 1.0)
    y = run_gemm(g, b, X, M, N, K)
    assert_close(ref.h2f(y), ref.h2f(ref.gemm(b, X, M, N, K, threads=0)))
    y0 = ref.f2h(ref.randn(M * N, 224, 0.5))
    y = run_gemm(g, b, X, M, N, K, y_init=y0.copy(), epi="bias", ev=(bias, 0), res=True, post_gelu=True)
    want = ref.gemm(b, X, M, N, K, epi="bias", ev=bias, res=True, post_gelu=True, Y=y0.copy(), threads=0)
    assert_close(ref.h2f(y), ref.h2f(want))
    r0 = ref.randn(M * N, 225)
    y = run_gemm(g, b, X, M, N, K, y_init=r0.copy(), epi="resadd", ev=(gate, 0), bv=(bias, 0), store=False)
    assert_close(y, ref.gemm(b, X, M, N, K, epi="resadd", ev=gate, bv=bias, store=False, Y=r0.copy(), threads=0))
    yf = run_gemm(g, b, X, M, N, K, y_bytes=M * N * 4, epi="f32")
    assert_close(yf, ref.gemm(b, X, M, N, K, epi="f32", threads=0))


def test_ksplit_with_x_prologue(g, monkeypatch):
    # the workspace holds the lnmod prologue's fp16 X and the splits' partials side by side
    monkeypatch.setenv("P0MM_GEMM_KSPLIT", "4")
    M, N, K = 40, 256, 1024
    b, _ = ref.pack_q4(ref.randn(N * K, 226, 0.02), N, K)
    X, st, pv = xpro_case(M, K, 227, K, 0, 0, 0, K)
    y = run_gemm(g, b, X, M, N, K, x={"mode": "lnmod"}, _stats=(st, 0), _pv=(pv, 0, K))
    X16 = ref.gemm_xpro("lnmod", X, M, K, stats=st, pv=pv, pv_stride=K)
    assert_close(ref.h2f(y), ref.h2f(ref.gemm(b, X16, M, N, K, threads=0)))
