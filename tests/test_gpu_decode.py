"""GPU parity of the decode step's attention operators, through the C ABI, against the CPU oracle:
  qkrope (lops.js:183-233): q heads f32, k / v heads into fp16 head-major caches at the token's row, split partials,
      partial rotary (npairs < D/2), GQA;
  attnDec + combine (lops.js:236-321): every query head over its KV head's keys, chunk tails, ring caches, MQA and GQA;
and one decode layer composed from the library's operators as the reference's decode step chains them (embed ->
gemv QKV (rms prologue, k-split partials) -> qkrope -> attnDec -> gemv O -> normadd), against the same chain run
through the oracle."""
import numpy as np
import pytest

import p0pc0rn_b200 as p0
from oracle import ref

from .test_gpu_parity import assert_close, nan_buf

pytestmark = pytest.mark.gpu


def rope_table(rows, npairs, seed, off=0):
    ang = ref.randn(rows * npairs, seed, 2.0).astype(np.float64)
    rp = np.zeros(off + 2 * rows * npairs, np.float32)
    rp[off::2], rp[off + 1::2] = np.cos(ang), np.sin(ang)
    return rp


@pytest.mark.parametrize("D,nq,nkv,nsrc,npairs", [(256, 8, 1, 1, 128), (512, 8, 2, 4, 64), (256, 4, 4, 2, 32)])
def test_qkrope(g, D, nq, nkv, nsrc, npairs):
    nh, kv_len, row, pos = nq + 2 * nkv, 40, 17, 11
    S = ref.randn(nsrc * nh * D, 400 + D, 1.0)
    NW = ref.randn(2 * D + 8, 401, 0.2) + 1
    RP = rope_table(pos + 1, npairs, 402, off=6)
    kc0, vc0 = ref.f2h(ref.round_f16(ref.randn(nkv * kv_len * D, 403))), ref.f2h(ref.round_f16(ref.randn(nkv * kv_len * D, 404)))
    qb, kcb, vcb = nan_buf(g, nq * D * 4), g.upload(kc0), g.upload(vc0)
    p0.qkrope(g, {"s": {"buf": g.upload(S), "n": nsrc, "ld": nh * D}, "norm": {"buf": g.upload(NW)}, "rope": {"buf": g.upload(RP), "off": 6},
                  "q": {"buf": qb}, "kc": {"buf": kcb}, "vc": {"buf": vcb}, "D": D, "nq": nq, "hasKV": True, "pos": pos, "eps": 1e-6,
                  "qw": 8, "kw": 8 + D, "npairs": npairs, "kvRow": row, "nkv": nkv, "kvLen": kv_len})
    Q, KC, VC = ref.qkrope(S, nsrc, nh * D, NW, RP, D, nq, nkv=nkv, pos=pos, qw=8, kw=8 + D, npairs=npairs, rope_off=6, kv_row=row,
                           kv_len=kv_len, KC=kc0.copy(), VC=vc0.copy())
    assert_close(g.read(qb, 0, nq * D * 4, np.float32), Q)
    gk, gv = g.read(kcb, 0, kc0.nbytes, np.uint16), g.read(vcb, 0, vc0.nbytes, np.uint16)
    assert_close(ref.h2f(gk), ref.h2f(KC))
    assert_close(ref.h2f(gv), ref.h2f(VC))
    other = np.ones(nkv * kv_len, bool).reshape(nkv, kv_len)
    other[:, row] = False                      # rows other than the token's keep their bits
    assert np.array_equal(gk.reshape(nkv, kv_len, D)[other], kc0.reshape(nkv, kv_len, D)[other])


@pytest.mark.parametrize("D,nh,nkv,k0,k1,ring,kv_len", [(256, 8, 1, 0, 1000, 0, 1024), (512, 8, 2, 3, 4100, 0, 4100),
                                                        (128, 4, 4, 100, 700, 512, 512), (256, 8, 8, 0, 1, 0, 64)])
def test_attn_dec(g, D, nh, nkv, k0, k1, ring, kv_len):
    Q = ref.randn(nh * D, 410 + D, 0.06)
    KC = ref.f2h(ref.round_f16(ref.randn(nkv * kv_len * D, 411)))
    VC = ref.f2h(ref.round_f16(ref.randn(nkv * kv_len * D, 412)))
    nchunk = -(-(k1 - k0) // 64)
    ob = nan_buf(g, nh * D * 4)
    p0.attnDec(g, {"q": {"buf": g.upload(Q)}, "kc": {"buf": g.upload(KC)}, "vc": {"buf": g.upload(VC)},
                   "part": {"buf": g.buffer(nchunk * nh * (2 + D) * 4)}, "out": {"buf": ob}, "D": D, "nh": nh, "kStart": k0, "kEnd": k1,
                   "ring": ring, "nkv": nkv, "kvLen": kv_len})
    assert_close(g.read(ob, 0, nh * D * 4, np.float32), ref.attn_dec(Q, KC, VC, D, nh, nkv, kv_len, k0, k1, ring))


def test_attn_dec_checks(g):
    b = g.buffer(1 << 20)
    base = {"q": {"buf": b}, "kc": {"buf": b}, "vc": {"buf": b}, "part": {"buf": b}, "out": {"buf": b}, "D": 256, "nh": 8, "kStart": 0,
            "nkv": 1, "kvLen": 20000}
    with pytest.raises(p0.P0Error, match="context too long for one combine"):
        p0.attnDec(g, {**base, "kEnd": 64 * 256 + 1})
    with pytest.raises(p0.P0Error, match="at most 8"):
        p0.attnDec(g, {**base, "kEnd": 64, "nh": 16})


def test_decode_layer_chain(g):
    # one decode token through one attention layer at position pos with pos earlier keys in the cache:
    # embed -> QKV gemv (rms prologue on the embedding's stat, kPer split) -> qkrope -> attnDec -> O gemv -> normadd
    V, D, nq, nkv, hd, pos = 1024, 2048, 8, 1, 256, 37
    nh = nq + 2 * nkv
    NQKV, kv_len, kPer = nh * hd, 64, 1024
    E, _ = ref.pack_q4(ref.randn(V * D, 420, 0.05), V, D)
    Wqkv, _ = ref.pack_q4(ref.randn(NQKV * D, 421, 0.02), NQKV, D)
    Wo, _ = ref.pack_q4(ref.randn(D * nq * hd, 422, 0.02), D, nq * hd)
    nw_in, nw_qk, nw_post = ref.randn(D, 423, 0.1) + 1, ref.randn(2 * hd, 424, 0.1) + 1, ref.randn(D, 425, 0.1) + 1
    RP = rope_table(pos + 1, hd // 2, 426)
    kc0 = ref.f2h(ref.round_f16(ref.randn(nkv * kv_len * hd, 427)))
    vc0 = ref.f2h(ref.round_f16(ref.randn(nkv * kv_len * hd, 428)))
    tok = np.array([777], np.uint32)
    # ---- the oracle's chain
    x0, st0 = ref.embed(E, tok, D, scale=45.25)
    qkv, _, ns = ref.gemv(Wqkv, x0, NQKV, D, kPer=kPer, pro="rms", norm=nw_in, stat_buf=st0, stat_off=0)
    Q, KC, VC = ref.qkrope(qkv, ns, NQKV, nw_qk, RP, hd, nq, nkv=nkv, pos=pos, qw=0, kw=hd, npairs=hd // 2, kv_row=pos, kv_len=kv_len,
                           KC=kc0.copy(), VC=vc0.copy())
    att = ref.attn_dec(Q, KC, VC, hd, nq, nkv, kv_len, 0, pos + 1)
    o, _, _ = ref.gemv(Wo, att, D, nq * hd)
    x_want, st_want = x0.copy(), np.zeros(1, np.float32)
    ref.normadd(o, 1, D, nw_post, 0, x_want, st_want, 0, D, 1, mode=0, eps=1e-6, scale=1.0)
    # ---- the same chain on the GPU through the library
    eb, wq, wo = g.upload(E), g.upload(Wqkv), g.upload(Wo)
    xb, stb = g.buffer(D * 4), g.buffer(16)
    p0.embed(g, {"w": {"buf": eb, "off": 0, "enc": "q4g32a.t64", "rows": V, "cols": D}, "ids": {"buf": g.upload(tok)}, "x": {"buf": xb},
                 "st": {"buf": stb}, "K": D, "n": 1, "scale": 45.25})
    qkvb = g.buffer(ns * NQKV * 4)
    assert p0.gemv(g, {"w": {"buf": wq, "off": 0, "enc": "q4g32a.t64", "rows": NQKV, "cols": D}, "x": {"buf": xb}, "N": NQKV, "K": D,
                       "kPer": kPer, "y": {"buf": qkvb}, "pro": "rms", "norm": {"buf": g.upload(nw_in), "off": 0},
                       "stat": {"buf": stb, "off": 0}}) == ns
    qb, kcb, vcb = g.buffer(nq * hd * 4), g.upload(kc0), g.upload(vc0)
    p0.qkrope(g, {"s": {"buf": qkvb, "n": ns, "ld": NQKV}, "norm": {"buf": g.upload(nw_qk)}, "rope": {"buf": g.upload(RP)}, "q": {"buf": qb},
                  "kc": {"buf": kcb}, "vc": {"buf": vcb}, "D": hd, "nq": nq, "hasKV": True, "pos": pos, "qw": 0, "kw": hd,
                  "npairs": hd // 2, "kvRow": pos, "nkv": nkv, "kvLen": kv_len})
    ab = g.buffer(nq * hd * 4)
    p0.attnDec(g, {"q": {"buf": qb}, "kc": {"buf": kcb}, "vc": {"buf": vcb}, "part": {"buf": g.buffer(nq * (2 + hd) * 4)},
                   "out": {"buf": ab}, "D": hd, "nh": nq, "kStart": 0, "kEnd": pos + 1, "nkv": nkv, "kvLen": kv_len})
    ob = g.buffer(D * 4)
    p0.gemv(g, {"w": {"buf": wo, "off": 0, "enc": "q4g32a.t64", "rows": D, "cols": nq * hd}, "x": {"buf": ab}, "N": D, "K": nq * hd,
                "kPer": nq * hd, "y": {"buf": ob}})
    p0.normadd(g, {"t": {"buf": ob, "n": 1, "ld": D}, "w": {"buf": g.upload(nw_post), "off": 0}, "x": {"buf": xb}, "st": {"buf": stb},
                   "D": D, "M": 1, "eps": 1e-6})
    assert_close(g.read(xb, 0, D * 4, np.float32), x_want)
    assert abs(float(g.read(stb, 0, 4, np.float32)[0]) - float(st_want[0])) <= 1e-4 * abs(float(st_want[0]))
