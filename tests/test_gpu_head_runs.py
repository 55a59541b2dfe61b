"""GPU parity of the wide-projection GEMV (the vocabulary-head kernel, whole 64-row tiles per warp from each CTA's
contiguous share) on a shape whose tiles do not divide evenly over the CTAs and warps (2432 tiles: 16-17 per CTA on
148 SMs) with an odd group count (65 groups: a half stage at each tile's end), store and softcap epilogues, against the
CPU oracle (lops.js:30-106, lops_spec.js:44-157 restated). At M = 1 and 2 this is the grouped form (one or two groups
per MMA lane pair), whose last stage of each tile holds one group here; P0MM_V3_G4=0 runs the generic form on the same
cases."""
import numpy as np
import pytest

from oracle import ref

from .test_gpu_parity import assert_close, check_mx, run_gemvM

pytestmark = pytest.mark.gpu

N, K = 155648, 2080          # 2432 tiles: 16.4 per CTA on 148 SMs; 65 groups per tile
_W = {}


def weights():
    if "b" not in _W:
        _W["b"] = ref.pack_q4(ref.randn(N * K, 600, 0.02), N, K)[0]
    return _W["b"]


@pytest.mark.parametrize("M", [1, 2, 3, 8])
def test_wide_store(g, M):
    b = weights()
    X = ref.randn(M * K, 601 + M)
    y, _, ns = run_gemvM(g, b, X, M, N, K, M * N)
    want, _, _ = ref.gemvM(b, X, M, N, K)
    assert ns == 1
    assert_close(y, want)


@pytest.mark.parametrize("M", [1, 2, 5])
def test_wide_softcap(g, M):
    b = weights()
    X = ref.randn(M * K, 611 + M)
    nw = ref.randn(K, 612, 0.1) + 1
    st = np.array([0.8 + 0.04 * m for m in range(M)], np.float32)
    NT = N // 64
    y, mx, _ = run_gemvM(g, b, X, M, N, K, M * N, mx_floats=M * NT * 2, extra={"norm": (nw, 0), "stat": (st, 0, 1)}, pro="rms",
                         epi="softcap", cap=30.0)
    wy, wmx, _ = ref.gemvM(b, X, M, N, K, pro="rms", epi="softcap", norm=nw, stat=st, stat_off=0, stat_ld=1, cap=30.0)
    assert_close(y, wy)
    for m in range(M):
        check_mx(mx[m * NT * 2:(m + 1) * NT * 2], wmx[m * NT * 2:(m + 1) * NT * 2], wy[m * N:(m + 1) * N], NT)


@pytest.mark.parametrize("M", [1, 2, 4])
def test_wide_repeat_bit_identical(g, M):
    # every tile is summed by one warp in a fixed order: the same call gives the same bits
    b = weights()
    X = ref.randn(M * K, 620)
    y0, _, _ = run_gemvM(g, b, X, M, N, K, M * N)
    y1, _, _ = run_gemvM(g, b, X, M, N, K, M * N)
    assert np.array_equal(y0.view(np.uint32), y1.view(np.uint32))
