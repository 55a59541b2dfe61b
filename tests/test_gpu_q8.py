"""q8g64s.t64 on the GPU: the device packQ8 bit for bit against the oracle (engine/kcheck.js:39-52 restated); the
GEMV / gemvM over q8 weights (the lgemv / lgemvM q8 arithmetic of lops.js:72-81, lops_spec.js restated) within the
parity tolerance, for the forms the reference's 8-bit layers use (raw and rms prologues, store / softcap / geglu
epilogues, k-splits, M up to 8); and the GEMM over q8 weights (gemm.js:150-160): its dequantised weights bit for bit,
its outputs within the tolerance, on whole-tile and gathered row views."""
import numpy as np
import pytest

import p0pc0rn_b200 as p0
from oracle import ref

from .test_gpu_parity import assert_close, check_mx, nan_buf

pytestmark = pytest.mark.gpu
Q8 = "q8g64s.t64"


def q8view(buf, N, K):
    return {"buf": buf, "off": 0, "enc": Q8, "rows": N, "cols": K}


@pytest.mark.parametrize("N,K,seed,scale", [(64, 128, 1, 0.05), (256, 2048, 2, 0.02), (128, 192, 3, 3.0)])
def test_pack_q8_bit_exact(g, N, K, seed, scale):
    W = ref.randn(N * K, seed, scale)
    W[:64] = 0.0                                                     # all-zero group: s = 1
    W[K:K + 64] = np.linspace(-1e-6, 1e-6, 64, dtype=np.float32)     # subnormal fp16 scale
    if N >= 128:
        W[2 * K:2 * K + 64] = np.linspace(-60000, 60000, 64, dtype=np.float32)
        W[3 * K:3 * K + 64] = 0.5 * np.arange(64, dtype=np.float32) / 127.0   # ties for round-half-even
    want, _ = ref.pack_q8(W, N, K)
    out = p0.pack_q8(g, g.upload(W), N, K)
    assert np.array_equal(g.read(out, 0, want.size), want)


def _packed(N, K, seed):
    return ref.pack_q8(ref.randn(N * K, seed, 0.02), N, K)[0]


@pytest.mark.parametrize("N,K,kPer", [(2048, 2048, 0), (2560, 2048, 0), (2048, 8192, 2048), (512, 1024, 256)])
def test_gemv_q8(g, N, K, kPer):
    b = _packed(N, K, 700 + K)
    x = ref.randn(K, 701)
    ns = -(-K // kPer) if kPer else 1
    yb = nan_buf(g, ns * N * 4)
    a = {"w": q8view(g.upload(b), N, K), "x": {"buf": g.upload(x)}, "N": N, "K": K, "y": {"buf": yb}}
    if kPer:
        a["kPer"] = kPer
    assert p0.gemv(g, a) == ns
    want, _, _ = ref.gemv(b, x, N, K, enc=Q8, kPer=kPer or None)
    assert_close(g.read(yb, 0, ns * N * 4, np.float32), want)


@pytest.mark.parametrize("M", [1, 2, 4, 8])
def test_gemvM_q8_rms_store(g, M):
    N, K = 4096, 2048
    b = _packed(N, K, 710)
    X = ref.randn(M * K, 711)
    nw = ref.randn(K, 712, 0.1) + 1
    st = np.array([0.8 + 0.05 * m for m in range(M)], np.float32)
    yb = nan_buf(g, M * N * 4)
    p0.gemvM(g, {"w": q8view(g.upload(b), N, K), "x": {"buf": g.upload(X)}, "M": M, "N": N, "K": K, "y": {"buf": yb}, "pro": "rms",
                 "norm": {"buf": g.upload(nw), "off": 0}, "stat": {"buf": g.upload(st), "off": 0, "ld": 1}})
    want, _, _ = ref.gemvM(b, X, M, N, K, enc=Q8, pro="rms", norm=nw, stat=st, stat_off=0, stat_ld=1)
    assert_close(g.read(yb, 0, M * N * 4, np.float32), want)


@pytest.mark.parametrize("M", [1, 4])
def test_gemvM_q8_softcap(g, M):
    N, K = 8192, 2048
    b = _packed(N, K, 720)
    X = ref.randn(M * K, 721)
    nw = ref.randn(K, 722, 0.1) + 1
    st = np.array([0.9] * M, np.float32)
    NT = N // 64
    yb, mxb = nan_buf(g, M * N * 4), nan_buf(g, M * NT * 8, "mx")
    p0.gemvM(g, {"w": q8view(g.upload(b), N, K), "x": {"buf": g.upload(X)}, "M": M, "N": N, "K": K, "y": {"buf": yb}, "pro": "rms",
                 "epi": "softcap", "cap": 30.0, "mx": {"buf": mxb}, "norm": {"buf": g.upload(nw), "off": 0},
                 "stat": {"buf": g.upload(st), "off": 0, "ld": 1}})
    wy, wmx, _ = ref.gemvM(b, X, M, N, K, enc=Q8, pro="rms", epi="softcap", norm=nw, stat=st, stat_off=0, stat_ld=1, cap=30.0)
    y, mx = g.read(yb, 0, M * N * 4, np.float32), g.read(mxb, 0, M * NT * 8, np.float32)
    assert_close(y, wy)
    for m in range(M):
        check_mx(mx[m * NT * 2:(m + 1) * NT * 2], wmx[m * NT * 2:(m + 1) * NT * 2], wy[m * N:(m + 1) * N], NT)


@pytest.mark.parametrize("M", [1, 3])
def test_gemvM_q8_geglu(g, M):
    N, K = 2048, 2048
    b = _packed(2 * N, K, 730)
    X = ref.randn(M * K, 731)
    nw = ref.randn(K, 732, 0.1) + 1
    st = np.array([0.7] * M, np.float32)
    yb = nan_buf(g, M * N * 4)
    p0.gemvM(g, {"w": q8view(g.upload(b), 2 * N, K), "x": {"buf": g.upload(X)}, "M": M, "N": N, "K": K, "y": {"buf": yb},
                 "pro": "rms", "epi": "geglu", "norm": {"buf": g.upload(nw), "off": 0}, "stat": {"buf": g.upload(st), "off": 0, "ld": 1}})
    want, _, _ = ref.gemvM(b, X, M, N, K, enc=Q8, pro="rms", epi="geglu", norm=nw, stat=st, stat_off=0, stat_ld=1)
    assert_close(g.read(yb, 0, M * N * 4, np.float32), want)


# ---------------------------------------------------------------- GEMM over q8 weights (gemm.js:150-160)
from .test_gpu_parity import run_gemm  # noqa: E402


@pytest.mark.parametrize("N,K", [(64, 128), (192, 1024)])
def test_dequant_q8_bit_exact(g, N, K):
    W = ref.randn(N * K, 740, 0.05)
    W[:64] = 0.0
    W[K:K + 64] = np.linspace(-1e-6, 1e-6, 64, dtype=np.float32)   # subnormal scale: subnormal products
    b, _ = ref.pack_q8(W, N, K)
    out = g.buffer(N * K * 2)
    p0.dequant_f16(g, q8view(g.upload(b), N, K), out)
    assert np.array_equal(g.read(out, 0, N * K * 2, np.uint16), ref.deq16(b, N, K, enc=Q8).ravel())


@pytest.mark.parametrize("M,N,K", [(32, 128, 256), (300, 384, 320), (129, 256, 2048), (4, 128, 64), (64, 256, 96)])
def test_gemm_q8_f16(g, M, N, K):
    Kw = -(-K // 64) * 64                      # the weight's columns cover K in whole 64-k groups
    b, _ = ref.pack_q8(ref.randn(N * Kw, 750 + M, 0.02), N, Kw)
    X = ref.f2h(ref.round_f16(ref.randn(M * K, 751)))
    y = run_gemm(g, b, X, M, N, K, enc=Q8, cols=Kw)
    want = ref.gemm(b, X, M, N, K, enc=Q8, cols=Kw)
    assert_close(ref.h2f(y), ref.h2f(want))


def test_gemm_q8_bias_gelu_and_swiglu(g):
    M, N, K = 200, 512, 1024
    b, _ = ref.pack_q8(ref.randn(N * K, 760, 0.02), N, K)
    X = ref.f2h(ref.round_f16(ref.randn(M * K, 761)))
    bias = ref.randn(N, 762, 0.01)
    y = run_gemm(g, b, X, M, N, K, enc=Q8, epi="bias", ev=(bias, 0), post_gelu=True)
    assert_close(ref.h2f(y), ref.h2f(ref.gemm(b, X, M, N, K, enc=Q8, epi="bias", ev=bias, post_gelu=True)))
    # swiglu: gate rows [0, N/2), up rows [N/2, N), interleaved by the kernel as the reference's wrow() does
    y = run_gemm(g, b, X, M, N, K, enc=Q8, epi="swiglu", act="gelu", wr0=0, wr1=N // 2, y={"ld": N // 2})
    want = ref.gemm(b, X, M, N, K, enc=Q8, epi="swiglu", act="gelu", wr0=0, wr1=N // 2, ldy=N // 2)
    assert_close(ref.h2f(y), ref.h2f(want))


def test_gemm_q8_row_and_k_offsets(g):
    # a weight sub-view: rows from 64 on (whole tiles) and k from 64 on; x from its column 64
    M, N, K, Nw, Kw = 96, 256, 512, 384, 640
    b, _ = ref.pack_q8(ref.randn(Nw * Kw, 770, 0.02), Nw, Kw)
    X = ref.f2h(ref.round_f16(ref.randn(M * Kw, 771)))
    y = run_gemm(g, b, X, M, N, K, enc=Q8, rows=Nw, cols=Kw, wr0=64, wk0=64, x={"ld": Kw, "k0": 64})
    want = ref.gemm(b, X, M, N, K, enc=Q8, rows=Nw, cols=Kw, ldx=Kw, kx0=64, wr0=64, wk0=64)
    assert_close(ref.h2f(y), ref.h2f(want))


def test_gemm_q8_gathered_rows(g):
    # rows from 32 on: not whole 64-row tiles, so the producer gathers each row's codes and scale
    M, N, K, Nw = 70, 128, 256, 256
    b, _ = ref.pack_q8(ref.randn(Nw * K, 780, 0.02), Nw, K)
    X = ref.f2h(ref.round_f16(ref.randn(M * K, 781)))
    y = run_gemm(g, b, X, M, N, K, enc=Q8, rows=Nw, wr0=32)
    assert_close(ref.h2f(y), ref.h2f(ref.gemm(b, X, M, N, K, enc=Q8, rows=Nw, wr0=32)))
