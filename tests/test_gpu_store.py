"""The pack store on the GPU: a synthetic pocketflux.pack (a q4 and a q8 projection over 16 MiB, so the native reader
runs several double-buffered chunks, and a norm vector) verified, uploaded shard by shard into device buffers, read
back byte for byte, and used through its tensor views by the GEMV and the GEMM, checked against the oracle."""
import numpy as np
import pytest

import p0pc0rn_b200 as p0
from p0pc0rn_b200 import store
from oracle import ref

from .test_gpu_parity import assert_close, nan_buf

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def pack(tmp_path_factory):
    base = str(tmp_path_factory.mktemp("pack"))
    N4, N8, K = 8192, 4096, 4096
    b4, _ = ref.pack_q4(ref.randn(N4 * K, 300, 0.02), N4, K)     # 20 MiB: two chunks
    b8, _ = ref.pack_q8(ref.randn(N8 * K, 301, 0.02), N8, K)     # 16.5 MiB
    nw = ref.randn(K, 302, 0.1) + 1
    store.write_pack(base, {
        "blk0": [("norm", "f32", (K,), nw.tobytes()), ("w4", "q4g32a.t64", (N4, K), bytes(np.asarray(b4, np.uint8)))],
        "blk1": [("w8", "q8g64s.t64", (N8, K), bytes(np.asarray(b8, np.uint8)))],
    })
    return base, b4, b8, nw, K


def test_upload_and_gemv_through_views(g, pack):
    base, b4, b8, nw, K = pack
    st = store.WeightStore(g, base)
    st.open()
    assert st.verify()["complete"]
    h0, h1 = st.upload("blk0"), st.upload("blk1")
    raw = open(base + "/blk0.pfw", "rb").read()
    assert g.read(h0.buf, 0, len(raw)).tobytes() == raw
    w4, w8, nv = h0.t("blk0/w4"), h1.t("blk1/w8"), h0.t("blk0/norm")
    assert w4["off"] % 256 == 0
    x = ref.randn(K, 303)
    stat = np.array([0.9], np.float32)
    for w, b, enc in ((w4, b4, "q4g32a.t64"), (w8, b8, "q8g64s.t64")):
        N = w["rows"]
        yb = nan_buf(g, N * 4 * 2)
        ns = p0.gemv(g, {"w": w, "x": {"buf": g.upload(x)}, "N": N, "K": K, "kPer": 2048, "y": {"buf": yb}, "pro": "rms",
                         "norm": {"buf": nv["buf"], "off": nv["off"] // 4}, "stat": {"buf": g.upload(stat), "off": 0}})
        want, _, _ = ref.gemv(b, x, N, K, enc=enc, kPer=2048, pro="rms", norm=nw, stat_buf=stat, stat_off=0)
        assert_close(g.read(yb, 0, ns * N * 4, np.float32), want)
    st.release(h0)
    st.release(h1)
    st.drainPool()


def test_upload_part_and_gemm(g, pack):
    base, b4, _, _, K = pack
    st = store.WeightStore(g, base)
    st.open()
    part = st.uploadPart("blk0", ["blk0/w4"])
    w = part.t("blk0/w4")
    M, N = 200, w["rows"]
    X = ref.f2h(ref.round_f16(ref.randn(M * K, 310)))
    yb = g.buffer(M * N * 2)
    p0.gemm(g, {"w": w, "x": {"buf": g.upload(X)}, "M": M, "N": N, "K": K, "y": {"buf": yb}})
    rows = slice(0, 8 * N)   # the oracle's GEMM over the first 8 rows of x
    want = ref.gemm(b4, X[:8 * K], 8, N, K)
    assert_close(ref.h2f(g.read(yb, 0, M * N * 2, np.uint16)[rows]), ref.h2f(want))
