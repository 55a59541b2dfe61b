"""ctypes + numpy wrapper over oracle.c (TEST INFRASTRUCTURE ONLY; see oracle/__init__.py).

Every function mirrors one reference function:
  randn            engine/kcheck.js:11        pack_q4 / pack_q8   engine/kcheck.js:22-53
  f2h / h2f        engine/core/gpu.js:274-295 compare             engine/kcheck.js:15-20
  gemv             engine/llm/lops.js:30-141 (lgemv, with gemv()'s host checks and defaults)
  gemvM            engine/llm/lops_spec.js:44-191 (lgemvM, with gemvM()'s host checks and defaults)
  gemm             engine/ops/gemm.js:25-322 (x prologue 'f16'; epilogues f16/f32/bias/resadd/swiglu)
"""
import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(dtype=np.uint32, flags="C_CONTIGUOUS")
_vp = ctypes.c_void_p
_i64, _u32, _i = ctypes.c_int64, ctypes.c_uint32, ctypes.c_int


def build():
    """Compile liboracle.so with the Makefile beside this file (idempotent)."""
    src = os.path.join(_HERE, "oracle.c")
    if os.path.exists(_LIB_PATH) and os.path.getmtime(_LIB_PATH) >= os.path.getmtime(src):
        return _LIB_PATH
    subprocess.run(["make", "-C", _HERE, "-s"], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.or_randn.argtypes = [_f32p, _i64, _u32, ctypes.c_double]
        L.or_rng_u32.argtypes = [_u32, _i64]
        L.or_rng_u32.restype = _u32
        L.or_f2h.argtypes = [ctypes.c_double]
        L.or_f2h.restype = ctypes.c_uint16
        L.or_h2f.argtypes = [ctypes.c_uint16]
        L.or_h2f.restype = ctypes.c_double
        L.or_f2h_arr.argtypes = [_f64p, _i64, _u16p]
        L.or_h2f_arr.argtypes = [_u16p, _i64, _f64p]
        L.or_hfma_arr.argtypes = [_u16p, _u16p, _u16p, _i64, _u16p]
        L.or_hfma_d_arr.argtypes = [_u16p, _u16p, _u16p, _i64, _u16p]
        L.or_pack_q4.argtypes = [_f32p, _i64, _i64, _u8p, _vp]
        L.or_pack_q8.argtypes = [_f32p, _i64, _i64, _u8p, _vp]
        L.or_deq16_q4.argtypes = [_u8p, _i64, _i64, _u16p]
        L.or_deq16_q8.argtypes = [_u8p, _i64, _i64, _u16p]
        L.or_gemv.argtypes = [_i, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp] + [_u32] * 11 + [ctypes.c_float] + [_u32] * 4
        L.or_gemvM.argtypes = [_i, _i, _i, _u32, _vp, _vp, _vp, _vp, _vp, _vp, _vp] + [_u32] * 14 + [ctypes.c_float] + [_u32] * 4
        L.or_gemm.argtypes = [_i] * 9 + [_vp] * 5 + [_u32] * 15 + [_i]
        L.or_gemm_xpro.argtypes = [_i, _f32p, _u32, _u32, _u32, _u32, _f32p, _u32, _f32p, _u32, _u32, _u16p]
        L.or_argmaxM.argtypes = [_f32p, _u32, _u32, _u32p]
        L.or_embed.argtypes = [_i, _u32p, _u32p, _u32, _u32, _u32, ctypes.c_float, ctypes.c_float, _u32, _u32, _f32p, _f32p]
        L.or_normadd.argtypes = [_f32p, _u32, _u32, _f32p, _u32, _f32p, _f32p, _u32, _u32, _u32, _u32, ctypes.c_float, ctypes.c_float]
        L.or_dhead.argtypes = [_i, _f32p, _u32p, _f32p, _f32p, _u32p] + [_u32] * 6 + [_f32p]
        L.or_qkrope.argtypes = [_f32p, _u32, _u32, _f32p, _f32p, _f32p, _u16p, _u16p, _u32, _u32, _u32, _i, _u32, ctypes.c_float] + [_u32] * 6
        L.or_attn_dec.argtypes = [_f32p, _u16p, _u16p, _f32p] + [_u32] * 7
        L.or_gemm_red128.argtypes = [_i, _i, _f32p, _u32, _u32, _u16p, _f32p, _u32, _u16p, _f32p] + [_u32] * 6 + [ctypes.c_float]
        L.or_dot64.argtypes = [_f32p, _f64p, _i64, _i64, _i64, _f64p]
        L.or_gemv_cpu_mt.argtypes = [_f32p, _u32p, _f32p, _u32, _u32, _u32, _u32, _i]
        L.or_max_threads.restype = _i
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


# ---------------------------------------------------------------- data + fp16 helpers
def randn(n, seed, scale=1.0):
    o = np.empty(int(n), np.float32)
    if n:
        lib().or_randn(o, int(n), int(seed) & 0xFFFFFFFF, float(scale))
    return o


def rng_state(seed, k):
    """the xorshift state after k+1 draws (kcheck.js:10)"""
    return lib().or_rng_u32(int(seed) & 0xFFFFFFFF, int(k))


def f2h(x):
    a = np.ascontiguousarray(np.asarray(x, dtype=np.float64).ravel())
    o = np.empty(a.size, np.uint16)
    lib().or_f2h_arr(a, a.size, o)
    return o.reshape(np.shape(x))


def h2f(h):
    a = np.ascontiguousarray(np.asarray(h, dtype=np.uint16).ravel())
    o = np.empty(a.size, np.float64)
    lib().or_h2f_arr(a, a.size, o)
    return o.reshape(np.shape(h))


def round_f16(a):
    """roundF16 (kcheck.js:13): f32 values rounded through fp16"""
    return h2f(f2h(a)).astype(np.float32)


# ---------------------------------------------------------------- packers
def pack_q4(W, N, K):
    """packQ4 (kcheck.js:22-38) -> (bytes uint8[N*K*5/8], deq float32[N*K])"""
    if N % 64 or K % 32:
        raise ValueError("packQ4 needs N % 64 == 0 and K % 32 == 0")
    W = np.ascontiguousarray(W, dtype=np.float32).ravel()
    out = np.zeros((N // 64) * (K // 32) * 1280, np.uint8)
    deq = np.empty(N * K, np.float32)
    lib().or_pack_q4(W, N, K, out, _p(deq))
    return out, deq


def pack_q8(W, N, K):
    """packQ8 (kcheck.js:39-52) -> (bytes, deq)"""
    if N % 64 or K % 64:
        raise ValueError("packQ8 needs N % 64 == 0 and K % 64 == 0")
    W = np.ascontiguousarray(W, dtype=np.float32).ravel()
    out = np.zeros((N // 64) * (K // 64) * 4224, np.uint8)
    deq = np.empty(N * K, np.float32)
    lib().or_pack_q8(W, N, K, out, _p(deq))
    return out, deq


def deq16(wbytes, N, K, enc="q4g32a.t64"):
    """the fp16 weight the GEMM tile holds for each (n, k): f16(q*s + mn) (q4) or f16(q*s) (q8)"""
    out = np.empty(N * K, np.uint16)
    wb = np.ascontiguousarray(wbytes, dtype=np.uint8)
    if enc == "q4g32a.t64":
        lib().or_deq16_q4(wb, N, K, out)
    else:
        lib().or_deq16_q8(wb, N, K, out)
    return out.reshape(N, K)


def compare(got, want):
    """compare (kcheck.js:15-20) plus rel-L2 and max-abs: {cos, maxErr, relL2}"""
    g = np.asarray(got, np.float64).ravel()
    w = np.asarray(want, np.float64).ravel()
    dot, ga, wa = float(g @ w), float(g @ g), float(w @ w)
    e = np.abs(g - w)
    me = float(np.inf) if not np.all(np.isfinite(e)) else (float(e.max()) if e.size else 0.0)
    cos = dot / np.sqrt(max(1e-30, ga * wa))
    rel = float(np.sqrt(np.sum((g - w) ** 2) / max(1e-300, wa)))
    return {"cos": cos if np.isfinite(cos) else 0.0, "maxErr": me, "relL2": rel}


# ---------------------------------------------------------------- lgemv / lgemvM / gemm
PRO = {"raw": 0, "rms": 1, "sum": 2, "pleg": 3}
EPI = {"store": 0, "geglu": 1, "softcap": 2}
KCH = 2048


def _f32(a):
    return None if a is None else np.ascontiguousarray(a, dtype=np.float32)


def gemv(W, X, N, K, *, enc="q4g32a.t64", cols=None, woff=0, rowB=0, kPer=None, pro="raw", epi="store", ldy=None,
         Y=None, stat_buf=None, stat_off=0, norm=None, norm_off=0, ev=None, ev_off=0, src=None, mx=None, cap=30.0):
    """lops.js gemv() host logic (:111-141) + lgemv arithmetic. Buffers are numpy arrays standing for the bound
    storage buffers (X f32, W uint8 bytes, norm/ev f32, mx f32 (also the rms stat slot when epi is softcap, as
    lops.js:125 binds it), stat_buf f32). Returns (Y, MX, nsplit); Y and MX are updated in place when given."""
    q8 = enc == "q8g64s.t64"
    if enc not in ("q4g32a.t64", "q8g64s.t64"):
        raise ValueError("gemv: encoding " + str(enc))
    G = 64 if q8 else 32
    kch = (-(-K // 256) * 256) if (not kPer and K > KCH) else KCH
    if kch > 3072:
        raise ValueError("gemv: K %d needs a kPer" % K)
    kp = min(kch, kPer or K)
    if kp % G:
        raise ValueError("gemv: kPer must be a multiple of %d" % G)
    nsplit = -(-K // kp)
    if epi != "store" and nsplit > 1:
        raise ValueError("gemv: %s needs one split" % epi)
    if N % 64:
        raise ValueError("gemv: N % 64")
    if woff % 4:
        raise ValueError("gemv: weight offset")
    cols = cols or K
    wG = cols // G
    ldy = ldy or N
    mxb = mx if epi == "softcap" else stat_buf
    if Y is None:
        Y = np.zeros(nsplit * ldy if epi == "store" else N, np.float32)
    Wu = np.frombuffer(np.ascontiguousarray(W, dtype=np.uint8).tobytes() + b"\0" * 16, dtype=np.uint32)
    Xa = _f32(X)
    dummy = np.zeros(64, np.float32)
    NWa = _f32(norm) if norm is not None else dummy
    EVa = _f32(ev) if ev is not None else dummy
    MXa = mxb if mxb is not None else np.zeros(64, np.float32)
    ldp, nsrc = (src if src else (0, 0))
    lib().or_gemv(int(q8), PRO[pro], EPI[epi], _p(Xa), _p(Wu), _p(Y), _p(NWa), _p(EVa), _p(MXa),
                  N, K, wG, kp, nsplit, ldy, woff // 4, norm_off, stat_off, rowB, ev_off, float(cap), ldp, nsrc, 0, kch)
    return Y, MXa, nsplit


def gemvM(W, X, M, N, K, *, enc="q4g32a.t64", cols=None, woff=0, rowB=0, ldx=None, kPer=None, pro="raw", epi="store",
          ldm=None, ldy=None, Y=None, stat=None, stat_off=0, stat_ld=2, norm=None, norm_off=0, ev=None, ev_off=0,
          ev_ld=0, src=None, mx=None, cap=30.0):
    """lops_spec.js gemvM() host logic (:163-191) + lgemvM arithmetic. Returns (Y, MX, nsplit)."""
    q8 = enc == "q8g64s.t64"
    if enc not in ("q4g32a.t64", "q8g64s.t64"):
        raise ValueError("gemvM: encoding " + str(enc))
    if pro not in ("raw", "rms", "pleg"):
        raise ValueError("gemvM: prologue " + pro)
    G = 64 if q8 else 32
    kp = min(KCH, kPer) if kPer else K
    if kp % G:
        raise ValueError("gemvM: kPer must be a multiple of %d" % G)
    nsplit = -(-K // kp)
    if epi != "store" and nsplit > 1:
        raise ValueError("gemvM: %s needs one split" % epi)
    if N % 64:
        raise ValueError("gemvM: N % 64")
    if woff % 4:
        raise ValueError("gemvM: weight offset")
    cols = cols or K
    wG = cols // G
    ldm = ldm or N
    ldy = ldy or M * ldm
    ldx = ldx or K
    if Y is None:
        Y = np.zeros(nsplit * ldy if epi == "store" else M * ldm, np.float32)
    NT = N // 64
    if mx is None and epi == "softcap":
        mx = np.zeros(M * NT * 2, np.float32)
    Wu = np.frombuffer(np.ascontiguousarray(W, dtype=np.uint8).tobytes() + b"\0" * 16, dtype=np.uint32)
    dummy = np.zeros(64, np.float32)
    ldp, nsrc = (src if src else (0, 1))
    lib().or_gemvM(int(q8), PRO[pro], EPI[epi], M, _p(_f32(X)), _p(Wu), _p(Y),
                   _p(_f32(norm) if norm is not None else dummy), _p(_f32(ev) if ev is not None else dummy),
                   _p(_f32(stat) if stat is not None else dummy), _p(mx if mx is not None else dummy),
                   N, K, wG, kp, ldy, ldm, ldx, woff // 4, norm_off, stat_off, stat_ld, rowB, ev_off, ev_ld, float(cap),
                   nsrc, ldp, 0, NT)
    return Y, mx, nsplit


GEPI = {"f16": 0, "f32": 1, "bias": 2, "resadd": 3, "swiglu": 4}
WENC = {"q4g32a.t64": 0, "q8g64s.t64": 1, "f16": 2}


def gemm(W, X16, M, N, K, *, enc="q4g32a.t64", rows=None, cols=None, ldx=None, kx0=0, wr0=0, wr1=0, wk0=0,
         epi="f16", act="silu", acc="f32", Y=None, ldy=None, ny0=0, ev=None, ev_off=0, bv=None, bv_off=0, bv_up=0,
         res=False, store=False, post_gelu=False, threads=1, heads=None, gt=None):
    """gemm.js gemm() (:264-322) + gemmCode arithmetic for the 'f16' x prologue. X16 is uint16 fp16 bits [M, ldx].
    Y: uint16 (f16/bias/swiglu/heads/onormgate) or float32 (f32/resadd), updated in place when given. Returns Y.
    epi 'heads' / 'onormgate' (gemm.js:212-250): heads = {Ltot, Hq, Hkv, rowOff, eps, ropeMode, rope (f32 array, read
    from element 0 like the reference's whole-buffer binding)}; gt = the onormgate gate, fp16 bits, from element 0."""
    if epi in ("heads", "onormgate"):
        return _gemm_red128(W, X16, M, N, K, enc=enc, rows=rows, cols=cols, ldx=ldx, kx0=kx0, wr0=wr0, wk0=wk0, epi=epi,
                            Y=Y, ldy=ldy, ny0=ny0, ev=ev, ev_off=ev_off, heads=heads or {}, gt=gt, threads=threads)
    if K % 32:
        raise ValueError("gemm: K must be a multiple of 32")
    rows = rows or N
    cols = cols or K
    wG = cols // 32 if enc == "q4g32a.t64" else cols // 64 if enc == "q8g64s.t64" else cols
    ldx = ldx or K
    ldy = ldy or N
    f32y = epi in ("f32", "resadd")
    if Y is None:
        Y = np.zeros(M * ldy, np.float32 if f32y else np.uint16)
    if enc == "f16":
        Wu = np.ascontiguousarray(W, dtype=np.uint16)
    else:
        Wu = np.frombuffer(np.ascontiguousarray(W, dtype=np.uint8).tobytes() + b"\0" * 16, dtype=np.uint32)
    dummy = np.zeros(64, np.float32)
    lib().or_gemm(WENC[enc], GEPI[epi], int(acc == "f16"), int(act == "gelu"), int(res), int(store),
                  int(ev is not None and epi == "resadd"), int(bv is not None), int(post_gelu),
                  _p(np.ascontiguousarray(X16, dtype=np.uint16)), _p(Wu), _p(Y),
                  _p(_f32(ev) if ev is not None else dummy), _p(_f32(bv) if bv is not None else dummy),
                  M, N, K, ldx, kx0, wr0, wr1, wG, wk0, ldy, ny0, rows, ev_off, bv_off, bv_up, int(threads))
    return Y


def _gemm_red128(W, X16, M, N, K, *, enc, rows, cols, ldx, kx0, wr0, wk0, epi, Y, ldy, ny0, ev, ev_off, heads, gt, threads):
    """the f32 accumulators of the call (gemm() with epi 'f32'), then the head-reducing epilogue on them"""
    if N % 128:
        raise ValueError("gemm: the %s epilogue reduces over whole 128-wide heads (N %% 128)" % epi)
    A = gemm(W, X16, M, N, K, enc=enc, rows=rows, cols=cols, ldx=ldx, kx0=kx0, wr0=wr0, wk0=wk0, epi="f32", threads=threads)
    h = heads
    Ltot, Hq, Hkv, rowOff = int(h.get("Ltot") or 0), int(h.get("Hq") or 0), int(h.get("Hkv") or 0), int(h.get("rowOff") or 0)
    eps = float(h.get("eps") or 1e-6)
    ldy = ldy or N
    if Y is None:
        n = ((N // 128 - 1) * Ltot + rowOff + M) * 128 if epi == "heads" else (M - 1) * ldy + ny0 + N
        Y = np.zeros(n, np.uint16)
    dummy = np.zeros(64, np.float32)
    rp = _f32(h["rope"]) if h.get("rope") is not None else dummy
    g16 = np.ascontiguousarray(gt, dtype=np.uint16) if gt is not None else np.zeros(64, np.uint16)
    lib().or_gemm_red128(int(epi == "onormgate"), int(h.get("ropeMode") == "half"), _f32(A), M, N, Y,
                         _f32(ev) if ev is not None else dummy, ev_off, g16, rp, ldy, ny0, rowOff, Ltot, Hq, Hkv, eps)
    return Y


def gemm_xpro(mode, X, M, K, *, ldx=None, kx0=0, stats=None, stat_off=0, pv=None, pv_off=0, pv_stride=0):
    """the fp16 X [M][K] of gemm()'s f32 x prologues (gemm.js:55-63): mode 'lnmod' or 'rms'; stats = ST f32 rows of
    {mean, rstd}; pv = the scale (and, for lnmod, shift at pv_off + pv_stride) vectors. Returns uint16 fp16 bits."""
    out = np.empty(M * K, np.uint16)
    lib().or_gemm_xpro({"lnmod": 1, "rms": 2}[mode], _f32(X), M, K, ldx or K, kx0, _f32(stats), stat_off, _f32(pv), pv_off,
                       pv_stride, out)
    return out


def dot64(deq, x, M, N, K):
    """y[m][n] = sum_k deq[n][k] * x[m][k] in f64"""
    y = np.empty(M * N, np.float64)
    lib().or_dot64(np.ascontiguousarray(deq, np.float32).ravel(), np.ascontiguousarray(x, np.float64).ravel(), M, N, K, y)
    return y.reshape(M, N)


def gemv_cpu_mt(Wbytes, X, M, N, K, threads=0):
    """the timed CPU baseline: lgemvM arithmetic (raw/store, q4), OpenMP over 64-row tiles"""
    Wu = np.frombuffer(np.ascontiguousarray(Wbytes, dtype=np.uint8).tobytes(), dtype=np.uint32)
    Y = np.empty(M * N, np.float32)
    lib().or_gemv_cpu_mt(np.ascontiguousarray(X, np.float32).ravel(), Wu, Y, M, N, K, K // 32, int(threads))
    return Y


def max_threads():
    return lib().or_max_threads()


# ---------------------------------------------------------------- decode-path operators (lops.js, lops_spec.js)
def _words(b):
    return np.frombuffer(np.ascontiguousarray(b, dtype=np.uint8).tobytes() + b"\0" * 16, dtype=np.uint32)


def argmaxM(MX, n, M):
    """argmax / argmaxM (lops.js:416-436, lops_spec.js:326-348): MX f32 [M][n][2] (max, bitcast index) -> uint32 [M][2]
    (index, bits of the max)"""
    out = np.empty(2 * M, np.uint32)
    lib().or_argmaxM(_f32(MX), n, M, out)
    return out


def embed(W, ids, K, *, enc="q4g32a.t64", scale=1.0, eps=1e-6, st_off=0, row_out=0, X=None, ST=None):
    """embed (lops.js:323-365): rows ids of a q4 / q8 table -> X[(row_out + m) * K + k] (dequant * scale), ST[st_off + m]
    = rstd of the row. X / ST updated in place when given; returns (X, ST)."""
    q8 = enc == "q8g64s.t64"
    ids = np.ascontiguousarray(ids, np.uint32)
    n = ids.size
    X = np.zeros((row_out + n) * K, np.float32) if X is None else X
    ST = np.zeros(st_off + n, np.float32) if ST is None else ST
    lib().or_embed(int(q8), _words(W), ids, n, K, K // (64 if q8 else 32), float(scale), float(eps), st_off, row_out, X, ST)
    return X, ST


def normadd(T, nsrc, ldp, W, w_off, X, ST, st_off, D, M, *, mode=0, eps=1e-6, scale=1.0):
    """normadd (lops.js:143-180) on X [M][D] in place; ST[st_off + m] = rstd of the new row"""
    lib().or_normadd(_f32(T), nsrc, ldp, _f32(W) if W is not None else np.zeros(1, np.float32), w_off, X, ST, st_off, D, M, mode,
                     float(eps), float(scale))
    return X, ST


def dhead(W, X, ST, NW, SEL, K, tPer, nsel, *, enc="q4g32a.t64", stat_off=0, norm_off=0):
    """dhead (lops_spec.js:428-482): per selected tile its max and argmax row -> MX f32 [nsel * tPer][2]"""
    q8 = enc == "q8g64s.t64"
    MX = np.empty(2 * nsel * tPer, np.float32)
    lib().or_dhead(int(q8), _f32(X), _words(W), _f32(ST), _f32(NW), np.ascontiguousarray(SEL, np.uint32), stat_off, norm_off, K,
                   K // (64 if q8 else 32), tPer, nsel, MX)
    return MX


def qkrope(S, nsrc, ldp, NW, RP, D, nq, *, nkv=1, hasKV=True, pos=0, eps=1e-6, qw=0, kw=0, npairs=None, rope_off=0, kv_row=0,
           kv_len=0, Q=None, KC=None, VC=None):
    """qkrope (lops.js:183-233): returns (Q f32 [nq][D], KC, VC fp16 bits [nkv][kv_len][D]); arrays updated in place when given"""
    npairs = D // 2 if npairs is None else npairs
    Q = np.zeros(nq * D, np.float32) if Q is None else Q
    KC = np.zeros(max(1, nkv * kv_len * D), np.uint16) if KC is None else KC
    VC = np.zeros(max(1, nkv * kv_len * D), np.uint16) if VC is None else VC
    lib().or_qkrope(_f32(S), nsrc, ldp, _f32(NW), _f32(RP), Q, KC, VC, D, nq, nkv, int(bool(hasKV)), pos, float(eps), qw, kw, npairs,
                    rope_off, kv_row, kv_len)
    return Q, KC, VC


def attn_dec(Q, KC, VC, D, nh, nkv, kv_len, k_start, k_end, ring=0):
    """attnDec + combine (lops.js:236-321): O f32 [nh][D]"""
    O = np.empty(nh * D, np.float32)
    lib().or_attn_dec(_f32(Q), np.ascontiguousarray(KC, np.uint16), np.ascontiguousarray(VC, np.uint16), O, D, nh, nkv, kv_len,
                      k_start, k_end, ring)
    return O
