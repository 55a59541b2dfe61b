"""The Python mirror of the reference's operator surface on CPU (no kernel runs): how gemv / gemvM / gemm and the
decode operators turn the reference's argument objects (engine/llm/lops.js, lops_spec.js, engine/ops/gemm.js) into the
C structs of include/p0mm.h -- defaults, enum names, nested offsets, the rejections made before any call -- checked
against a stand-in library that records the struct each entry point receives. The Python enum tables are checked
against the header's values with a C program compiled against it."""
import ctypes
import os
import shutil
import subprocess

import pytest

from p0pc0rn_b200 import _lib as L
from p0pc0rn_b200 import ops
from p0pc0rn_b200.gpu import P0Error

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


class FakeBuf:
    def __init__(self, i):
        self.id = i

    @property
    def handle(self):
        return L.p0_buf(self.id)


class FakeLib:
    """records (entry point, struct copy or positional arguments); every call succeeds"""

    def __init__(self):
        self.calls = []

    def __getattr__(self, name):
        if not name.startswith("p0_"):
            raise AttributeError(name)

        def entry(ctx, *args):
            rec = []
            for a in args:
                obj = getattr(a, "_obj", None)          # ctypes.byref(struct) keeps the struct in _obj
                if isinstance(obj, ctypes.Structure):
                    cp = type(obj)()
                    ctypes.memmove(ctypes.byref(cp), ctypes.byref(obj), ctypes.sizeof(obj))
                    rec.append(cp)
                else:
                    rec.append(a)
            self.calls.append((name, rec))
            return L.P0_OK
        return entry


class FakeGpu:
    def __init__(self):
        self._lib = FakeLib()
        self.ctx = ctypes.c_void_p(1)

    def _check(self, st):
        assert st == L.P0_OK
        return st

    def last(self):
        return self._lib.calls[-1]


B = {i: FakeBuf(i) for i in range(1, 40)}


def wv(enc="q4g32a.t64", **kw):
    w = {"buf": B[1], "off": 256, "enc": enc, "rows": 4096, "cols": 2048}
    w.update(kw)
    return w


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_enum_tables_match_the_header(tmp_path):
    names = {**{"P0_ENC_" + k.upper().replace(".", "_"): v for k, v in L.ENC.items()},
             **{"P0_PRO_" + k.upper(): v for k, v in L.PRO.items()},
             **{"P0_EPI_" + k.upper(): v for k, v in L.EPI.items()},
             **{"P0_GEPI_" + k.upper(): v for k, v in L.GEPI.items()},
             **{"P0_ACT_" + k.upper(): v for k, v in L.ACT.items()},
             **{"P0_XPRO_" + k.upper(): v for k, v in L.XPRO.items()},
             **{v: k for k, v in L.STATUS.items()},
             "P0_ROPE_INTER": L.P0_ROPE_INTER, "P0_ROPE_HALF": L.P0_ROPE_HALF}
    src = tmp_path / "enums.c"
    src.write_text('#include <stdio.h>\n#include "p0mm.h"\nint main(void) {\n' +
                   "".join('  printf("%s %%d\\n", (int)%s);\n' % (n, n) for n in names) + "  return 0;\n}\n")
    exe = tmp_path / "enums"
    subprocess.run(["gcc", "-std=c11", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    out = dict(line.split() for line in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n") if line)
    assert {n: int(v) for n, v in out.items()} == names


def test_gemv_defaults():
    g = FakeGpu()
    ops.gemv(g, {"w": wv(), "x": {"buf": B[2]}, "N": 4096, "K": 2048, "y": {"buf": B[3]}})
    name, (a, _) = g.last()
    assert name == "p0_gemv"
    assert (a.w.buf.id, a.w.off, a.w.bytes, a.w.enc, a.w.rows, a.w.cols) == (1, 256, 0, 1, 4096, 2048)
    assert (a.x.id, a.x_rowB, a.N, a.K, a.kPer, a.pro, a.epi, a.y.id, a.ldy) == (2, 0, 4096, 2048, 0, 0, 0, 3, 0)
    assert (a.stat.id, a.norm.id, a.ev.id, a.mx.id, a.src_n, a.src_ld, a.cap) == (0, 0, 0, 0, 0, 0, 0.0)


def test_gemv_every_field():
    g = FakeGpu()
    ops.gemv(g, {"w": wv(bytes=1 << 20), "x": {"buf": B[2], "rowB": 64}, "N": 128, "K": 4096, "kPer": 2048, "pro": "pleg",
                 "epi": "store", "y": {"buf": B[3]}, "ldy": 256, "stat": {"buf": B[4], "off": 5}, "norm": {"buf": B[5], "off": 6},
                 "ev": {"buf": B[6], "off": 7}, "src": {"n": 3, "ld": 4096}, "mx": {"buf": B[7]}, "cap": 50.0})
    _, (a, _) = g.last()
    assert (a.w.bytes, a.x_rowB, a.kPer, a.pro, a.epi, a.ldy) == (1 << 20, 64, 2048, L.PRO["pleg"], 0, 256)
    assert (a.stat.id, a.stat_off, a.norm.id, a.norm_off, a.ev.id, a.ev_off) == (4, 5, 5, 6, 6, 7)
    assert (a.src_n, a.src_ld, a.mx.id, a.cap) == (3, 4096, 7, 50.0)


def test_gemv_rejections_in_the_reference_wording():
    g = FakeGpu()
    base = {"w": wv(), "x": {"buf": B[2]}, "N": 64, "K": 64, "y": {"buf": B[3]}}
    with pytest.raises(P0Error, match="^gemv: encoding q2$"):
        ops.gemv(g, {**base, "w": wv(enc="q2")})
    with pytest.raises(P0Error, match="^gemv: prologue bogus$"):
        ops.gemv(g, {**base, "pro": "bogus"})
    with pytest.raises(P0Error, match="^gemvM: epilogue bogus$"):
        ops.gemvM(g, {**base, "M": 2, "epi": "bogus"})
    assert g._lib.calls == []


@pytest.mark.parametrize("entry", ["gemvM", "gemvM_noalloc"])
def test_gemvM_fields(entry):
    g = FakeGpu()
    getattr(ops, entry)(g, {"w": wv(enc="q8g64s.t64"), "x": {"buf": B[2], "rowB": 8, "ldx": 3000}, "M": 4, "N": 512, "K": 2048,
                            "kPer": 1024, "pro": "rms", "epi": "softcap", "y": {"buf": B[3], "ldy": 9000, "ldm": 600},
                            "stat": {"buf": B[4], "off": 2, "ld": 3}, "norm": {"buf": B[5], "off": 1}, "ev": {"buf": B[6], "off": 9, "ld": 10},
                            "src": {"n": 2, "ld": 77}, "mx": {"buf": B[7]}, "cap": 15.0})
    name, (a, _) = g.last()
    assert name == "p0_" + entry
    assert (a.w.enc, a.x.id, a.x_rowB, a.x_ldx, a.M, a.N, a.K, a.kPer) == (2, 2, 8, 3000, 4, 512, 2048, 1024)
    assert (a.pro, a.epi, a.y.id, a.ldy, a.ldm) == (L.PRO["rms"], L.EPI["softcap"], 3, 9000, 600)
    assert (a.stat.id, a.stat_off, a.stat_ld, a.norm.id, a.norm_off) == (4, 2, 3, 5, 1)
    assert (a.ev.id, a.ev_off, a.ev_ld, a.src_n, a.src_ld, a.mx.id, a.cap) == (6, 9, 10, 2, 77, 7, 15.0)


def test_gemm_defaults():
    g = FakeGpu()
    ops.gemm(g, {"w": wv(), "x": {"buf": B[2]}, "M": 256, "N": 4096, "K": 2048, "y": {"buf": B[3]}})
    name, (a, fl) = g.last()
    assert name == "p0_gemm"
    assert (a.x.id, a.x_off, a.x_ld, a.x_k0, a.x_mode, a.M, a.N, a.K) == (2, 0, 0, 0, L.XPRO["f16"], 256, 4096, 2048)
    assert (a.wr0, a.wr1, a.wk0, a.epi, a.act, a.acc) == (0, 0, 0, L.GEPI["f16"], L.ACT["silu"], 0)
    assert (a.y.id, a.y_off, a.y_ld, a.y_n0, a.ev.id, a.bv.id, a.res, a.store, a.post_gelu) == (3, 0, 0, 0, 0, 0, 0, 0, 0)
    assert (a.stats.id, a.pv.id, a.h_Ltot, a.h_Hq, a.h_Hkv, a.h_rowOff, a.h_eps) == (0, 0, 0, 0, 0, 0, 0.0)
    assert (a.h_rope_mode, a.rope.id, a.gt.id) == (L.P0_ROPE_INTER, 0, 0)


def test_gemm_every_field():
    g = FakeGpu()
    ops.gemm(g, {"w": wv(enc="f16", ld=4104), "x": {"buf": B[2], "off": 4096, "ld": 3072, "k0": 64, "mode": "lnmod"},
                 "M": 100, "N": 256, "K": 1024, "wr0": 128, "wr1": 8320, "wk0": 32, "epi": "swiglu", "act": "gelu", "acc": "f16",
                 "y": {"buf": B[3], "off": 512, "ld": 9216, "n0": 128}, "ev": {"buf": B[4], "off": 11}, "bv": {"buf": B[5], "off": 12, "up": 8192},
                 "res": True, "store": 1, "post_gelu": "yes", "stats": {"buf": B[6], "off": 13}, "pv": {"buf": B[7], "off": 14, "stride": 3072},
                 "heads": {"Ltot": 4608, "Hq": 24, "Hkv": 8, "rowOff": 512, "eps": 1e-5, "ropeMode": "half", "rope": {"buf": B[8], "off": 99}},
                 "gt": {"buf": B[9], "off": 7}})
    _, (a, _) = g.last()
    assert (a.w.enc, a.w.ld) == (L.ENC["f16"], 4104)
    assert (a.x_off, a.x_ld, a.x_k0, a.x_mode) == (4096, 3072, 64, L.XPRO["lnmod"])
    assert (a.wr0, a.wr1, a.wk0, a.epi, a.act, a.acc) == (128, 8320, 32, L.GEPI["swiglu"], L.ACT["gelu"], 1)
    assert (a.y_off, a.y_ld, a.y_n0, a.ev.id, a.ev_off, a.bv.id, a.bv_off, a.bv_up) == (512, 9216, 128, 4, 11, 5, 12, 8192)
    assert (a.res, a.store, a.post_gelu, a.stats.id, a.stats_off, a.pv.id, a.pv_off, a.pv_stride) == (1, 1, 1, 6, 13, 7, 14, 3072)
    assert (a.h_Ltot, a.h_Hq, a.h_Hkv, a.h_rowOff, a.h_rope_mode) == (4608, 24, 8, 512, L.P0_ROPE_HALF)
    assert abs(a.h_eps - 1e-5) < 1e-12
    # rope and gt are bound from their buffers' start, as gemm.js:304 binds them (their offsets are not used)
    assert (a.rope.id, a.gt.id) == (8, 9)


@pytest.mark.parametrize("mode", [None, "inter", "interleaved", "HALF"])
def test_gemm_rope_mode_other_than_half_is_interleaved(mode):
    g = FakeGpu()
    h = {"Ltot": 64, "Hq": 1, "Hkv": 1, "rope": {"buf": B[8]}}
    if mode is not None:
        h["ropeMode"] = mode
    ops.gemm(g, {"w": wv(), "x": {"buf": B[2]}, "M": 64, "N": 384, "K": 128, "epi": "heads", "y": {"buf": B[3]}, "heads": h})
    assert g.last()[1][0].h_rope_mode == L.P0_ROPE_INTER


def test_gemm_rejections():
    g = FakeGpu()
    base = {"w": wv(), "x": {"buf": B[2]}, "M": 64, "N": 128, "K": 128, "y": {"buf": B[3]}}
    with pytest.raises(P0Error, match="^gemm: unsupported weight encoding q2$"):
        ops.gemm(g, {**base, "w": wv(enc="q2")})
    with pytest.raises(P0Error, match="^gemm: epilogue gelu2 is not built in this library yet$"):
        ops.gemm(g, {**base, "epi": "gelu2"})
    with pytest.raises(P0Error, match="^gemm: x prologue conv is not built in this library yet$"):
        ops.gemm(g, {**base, "conv": {"Hi": 8, "Wi": 8, "Ci": 16}})
    with pytest.raises(P0Error, match="^gemm: x prologue conv3 is not built in this library yet$"):
        ops.gemm(g, {**base, "x": {"buf": B[2], "mode": "conv3"}})
    assert g._lib.calls == []


def test_decode_operator_defaults():
    g = FakeGpu()
    ops.normadd(g, {"t": {"buf": B[2]}, "x": {"buf": B[3]}, "st": {"buf": B[4]}, "D": 2048})
    a = g.last()[1][0]
    assert (a.t.id, a.t_n, a.t_ld, a.w.id, a.x.id, a.st.id, a.st_off, a.D, a.M, a.mode, a.eps, a.scale) == \
        (2, 1, 0, 0, 3, 4, 0, 2048, 1, 0, 0.0, 1.0)
    ops.normadd(g, {"t": {"buf": B[2], "n": 4, "ld": 8192}, "w": {"buf": B[5], "off": 3}, "x": {"buf": B[3]}, "st": {"buf": B[4], "off": 2},
                    "D": 2048, "M": 3, "mode": 1, "eps": 1e-5, "scale": 0.0})
    a = g.last()[1][0]
    assert (a.t_n, a.t_ld, a.w.id, a.w_off, a.st_off, a.M, a.mode, a.scale) == (4, 8192, 5, 3, 2, 3, 1, 0.0)
    ops.qkrope(g, {"s": {"buf": B[2]}, "norm": {"buf": B[3]}, "rope": {"buf": B[4]}, "q": {"buf": B[5]}, "D": 256, "nq": 8, "npairs": 64})
    a = g.last()[1][0]
    assert (a.s_n, a.nkv, a.hasKV, a.kc.id, a.vc.id, a.pos, a.kvRow, a.eps) == (1, 1, 0, 0, 0, 0, 0, 0.0)
    ops.attnDec(g, {"q": {"buf": B[2]}, "kc": {"buf": B[3]}, "vc": {"buf": B[4]}, "part": {"buf": B[5]}, "out": {"buf": B[6]},
                    "D": 256, "nh": 8, "kStart": 0, "kEnd": 100})
    a = g.last()[1][0]
    assert (a.nkv, a.kvLen, a.kStart, a.kEnd, a.ring) == (1, 0, 0, 100, 0)
    ops.argmax(g, {"mx": {"buf": B[2]}, "n": 4096, "out": {"buf": B[3]}})
    assert g.last()[0] == "p0_argmaxM" and g.last()[1][1:3] == [4096, 1]
    ops.argmaxM(g, {"mx": {"buf": B[2]}, "n": 4096, "M": 5, "out": {"buf": B[3]}})
    assert g.last()[1][1:3] == [4096, 5]


def test_decode_operator_rejections():
    g = FakeGpu()
    with pytest.raises(P0Error, match="^embed: encoding f16$"):
        ops.embed(g, {"w": wv(enc="f16"), "ids": {"buf": B[2]}, "x": {"buf": B[3]}, "st": {"buf": B[4]}, "K": 64, "n": 1, "scale": 1.0})
    dh = {"w": wv(), "x": {"buf": B[2]}, "stat": {"buf": B[3]}, "norm": {"buf": B[4]}, "sel": {"buf": B[5]}, "mx": {"buf": B[6]},
          "tPer": 2, "nsel": 32}
    with pytest.raises(P0Error, match="^dhead: K > 512$"):
        ops.dhead(g, {**dh, "K": 1024})
    with pytest.raises(P0Error, match="^dhead: encoding f16$"):
        ops.dhead(g, {**dh, "w": wv(enc="f16"), "K": 256})
    assert g._lib.calls == []
    ops.dhead(g, {**dh, "K": 512})
    a = g.last()[1][0]
    assert (a.K, a.tPer, a.nsel, a.sel.id, a.mx.id) == (512, 2, 32, 5, 6)
