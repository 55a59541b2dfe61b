"""The GEMM's f32 x prologues on the GPU (engine/ops/gemm.js:55-63): 'lnmod' (the DiT's modulated layer norm,
f16(((x - mean) * rstd) * (1 + scale[k]) + shift[k])) and 'rms' (f16((x * rstd) * w[k])), with per-row {mean, rstd} from
a stats buffer (ops/misc.js rowstats rows) and the vectors from a pv buffer. The oracle restates the prologue in the
WGSL's order of operations and feeds the fp16 X to its GEMM; outputs must agree within the parity tolerance."""
import numpy as np
import pytest

from oracle import ref

from .test_gpu_parity import assert_close, run_gemm

pytestmark = pytest.mark.gpu


def _case(M, K, seed, ldx, k0, stat_off, pv_off, pv_stride):
    X = ref.randn(M * ldx, seed)
    rows = stat_off + M
    st = np.empty(rows * 2, np.float32)
    st[0::2] = ref.randn(rows, seed + 1, 0.1)
    st[1::2] = 0.5 + np.abs(ref.randn(rows, seed + 2, 0.3))
    pv = ref.randn(pv_off + pv_stride + k0 + K + 8, seed + 3, 0.2)
    return X, st, pv


@pytest.mark.parametrize("mode", ["lnmod", "rms"])
@pytest.mark.parametrize("enc", ["q4g32a.t64", "q8g64s.t64"])
def test_gemm_x_prologue(g, mode, enc):
    M, N, K, ldx, k0, stat_off, pv_off, pv_stride = 300, 384, 512, 576, 64, 7, 4, 600
    b = (ref.pack_q4 if enc == "q4g32a.t64" else ref.pack_q8)(ref.randn(N * K, 800, 0.02), N, K)[0]
    X, st, pv = _case(M, K, 801, ldx, k0, stat_off, pv_off, pv_stride)
    bias = ref.randn(N, 805, 0.01)
    y = run_gemm(g, b, X, M, N, K, enc=enc, epi="bias", ev=(bias, 0), x={"mode": mode, "ld": ldx, "k0": k0},
                 stats=None, pv=None, _stats=(st, stat_off), _pv=(pv, pv_off, pv_stride))
    X16 = ref.gemm_xpro(mode, X, M, K, ldx=ldx, kx0=k0, stats=st, stat_off=stat_off, pv=pv, pv_off=pv_off, pv_stride=pv_stride)
    want = ref.gemm(b, X16, M, N, K, enc=enc, epi="bias", ev=bias)
    assert_close(ref.h2f(y), ref.h2f(want))


def test_gemm_x_prologue_config3_slice(g):
    # the DiT's lnmod QKV shape (config 3: M 4096, K 3072, N 9216), on a 256-token slice of rows and a 1024-row weight slice
    M, N, K = 256, 1024, 3072
    b = ref.pack_q4(ref.randn(N * K, 810, 0.02), N, K)[0]
    X, st, pv = _case(M, K, 811, K, 0, 0, 0, K)
    y = run_gemm(g, b, X, M, N, K, x={"mode": "lnmod"}, _stats=(st, 0), _pv=(pv, 0, K))
    X16 = ref.gemm_xpro("lnmod", X, M, K, stats=st, pv=pv, pv_stride=K)
    assert_close(ref.h2f(y), ref.h2f(ref.gemm(b, X16, M, N, K)))
