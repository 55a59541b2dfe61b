"""GPU parity of the GEMM over fp16 (unquantised) weights, `w.enc = 'f16'` (engine/ops/gemm.js:162-168: rows of `w.ld`
halves, default the view's columns), against the CPU oracle's gemm (the same fp16 weight tile, f32 accumulation):
whole and partial 64-row tiles, a row stride wider than the columns with a k offset, the bias and swiglu epilogues,
and the alignment the kernel's 16-byte row reads need."""
import numpy as np
import pytest

import p0pc0rn_b200 as p0
from p0pc0rn_b200 import _lib as plib
from oracle import ref

from .test_gpu_parity import assert_close

pytestmark = pytest.mark.gpu


def f16(n, seed, scale=1.0):
    return ref.f2h(ref.round_f16(ref.randn(n, seed, scale)))


def run(g, W16, X16, M, N, K, rows, ld, **a):
    y, x = a.pop("y", {}), a.pop("x", {})
    ldy = y.get("ld") or (N // 2 if a.get("epi") == "swiglu" else N)
    yb = g.upload(np.full(M * ldy, 0x7E00, np.uint16))
    args = {"w": {"buf": g.upload(W16), "off": 0, "enc": "f16", "rows": rows, "cols": a.pop("cols", ld), "ld": ld},
            "x": {"buf": g.upload(X16), **x}, "M": M, "N": N, "K": K, "y": {"buf": yb, **y}}
    for k in ("ev", "bv"):
        if k in a:
            v = a.pop(k)
            args[k] = {"buf": g.upload(v[0]), "off": v[1]}
    args.update(a)
    assert p0.gemm(g, args) == 2.0 * M * N * K
    return g.read(yb, 0, M * ldy * 2, np.uint16)


@pytest.mark.parametrize("M,N,K", [(300, 384, 512), (64, 200, 256), (1000, 128, 1024), (7, 256, 64)])
def test_gemm_f16_weights(g, M, N, K):
    W = f16(N * K, 1000 + N, 0.05)
    X = f16(M * K, 1001)
    y = run(g, W, X, M, N, K, N, K)
    assert_close(ref.h2f(y), ref.h2f(ref.gemm(W, X, M, N, K, enc="f16", rows=N, cols=K)))


def test_gemm_f16_weights_stride_and_k_offset(g):
    # rows of 640 halves, the call's k from 64 to 64 + 512; x from its column 64 as well; bias epilogue
    M, N, K, ld = 130, 192, 512, 640
    W = f16(N * ld, 1010, 0.05)
    X = f16(M * ld, 1011)
    bias = ref.randn(N, 1012, 0.01)
    y = run(g, W, X, M, N, K, N, ld, cols=576, wk0=64, x={"ld": ld, "k0": 64}, epi="bias", ev=(bias, 0))
    want = ref.gemm(W, X, M, N, K, enc="f16", rows=N, cols=ld, ldx=ld, kx0=64, wk0=64, epi="bias", ev=bias)
    assert_close(ref.h2f(y), ref.h2f(want))


def test_gemm_f16_weights_swiglu(g):
    M, N, K, rows = 96, 256, 384, 320
    W = f16(rows * K, 1020, 0.05)
    X = f16(M * K, 1021)
    y = run(g, W, X, M, N, K, rows, K, epi="swiglu", act="gelu", wr0=8, wr1=8 + N // 2, y={"ld": N // 2})
    want = ref.gemm(W, X, M, N, K, enc="f16", rows=rows, cols=K, epi="swiglu", act="gelu", wr0=8, wr1=8 + N // 2, ldy=N // 2)
    assert_close(ref.h2f(y), ref.h2f(want))


def test_gemm_f16_weights_alignment(g):
    W, X = f16(64 * 100, 1030), f16(8 * 96, 1031)
    with pytest.raises(p0.P0Error, match="16-byte boundaries") as e:
        p0.gemm(g, {"w": {"buf": g.upload(W), "off": 0, "enc": "f16", "rows": 64, "cols": 96, "ld": 100}, "x": {"buf": g.upload(X)},
                    "M": 8, "N": 64, "K": 96, "y": {"buf": g.buffer(8 * 64 * 2)}})
    assert e.value.status == plib.P0_EALIGN
