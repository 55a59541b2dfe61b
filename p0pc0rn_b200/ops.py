"""The three matmul operators with the reference's own argument objects, over the C ABI.

  gemv(g, a)   -> nsplit   engine/llm/lops.js:108-141       (a = {w, x: {buf, rowB}, N, K, kPer, pro, epi, y: {buf},
                                                            ldy, stat: {buf, off}, norm: {buf, off}, ev: {buf, off},
                                                            src: {n, ld}, mx: {buf}, cap})
  gemvM(g, a)  -> nsplit   engine/llm/lops_spec.js:159-191  (adds M, x.ldx, y.ldm / y.ldy, stat.ld, ev.ld)
  gemm(gpu, a) -> flops    engine/ops/gemm.js:255-322       (a = {w, x: {buf, off, ld, k0, mode}, M, N, K, wr0, wr1, wk0,
                                                            epi, act, acc, y: {buf, off, ld, n0}, ev: {buf, off},
                                                            bv: {buf, off, up}, res, store, stats: {buf, off},
                                                            pv: {buf, off, stride}} + post_gelu)
w = {buf, off (bytes), bytes, enc, rows, cols} as WeightStore.t() returns it (core/store.js:249-253).
Every call enqueues one kernel on the context's stream; results are read with g.read() after it. Errors raise
P0Error with the reference's messages. There is no CPU path: these always run the CUDA kernels in libp0mm.so.
"""
import ctypes

from . import _lib as L
from .gpu import P0Error, handle


def _wview(w, op="gemv"):
    enc = w.get("enc")
    if enc not in L.ENC:
        # gemm.js:267 and lops.js:115 / lops_spec.js:166 word it differently
        raise P0Error(L.P0_EINVAL, (op + ": unsupported weight encoding " if op == "gemm" else op + ": encoding ") + str(enc))
    return L.p0_wview(handle(w["buf"]), int(w.get("off") or 0), int(w.get("bytes") or 0), L.ENC[enc], int(w["rows"]),
                      int(w["cols"]), int(w.get("ld") or 0))


def _b(o):
    return handle(o.get("buf")) if o else L.p0_buf(0)


def gemv(g, a):
    """gemv(g, a) -> nsplit (lops.js:111-141)"""
    x, y = a["x"], a["y"]
    stat, norm, ev, src, mx = a.get("stat"), a.get("norm"), a.get("ev"), a.get("src"), a.get("mx")
    pro, epi = a.get("pro") or "raw", a.get("epi") or "store"
    if pro not in L.PRO:
        raise P0Error(L.P0_EINVAL, "gemv: prologue " + str(pro))
    if epi not in L.EPI:
        raise P0Error(L.P0_EINVAL, "gemv: epilogue " + str(epi))
    args = L.p0_gemv_args(
        _wview(a["w"]), handle(x["buf"]), int(x.get("rowB") or 0), int(a["N"]), int(a["K"]), int(a.get("kPer") or 0), L.PRO[pro],
        L.EPI[epi], handle(y["buf"]), int(a.get("ldy") or 0), _b(stat), int((stat or {}).get("off") or 0), _b(norm),
        int((norm or {}).get("off") or 0), _b(ev), int((ev or {}).get("off") or 0), int((src or {}).get("n") or 0),
        int((src or {}).get("ld") or 0), _b(mx), float(a.get("cap") or 0.0))
    ns = ctypes.c_uint32()
    g._check(g._lib.p0_gemv(g.ctx, ctypes.byref(args), ctypes.byref(ns)))
    return ns.value


def gemvM(g, a):
    """gemvM(g, a) -> nsplit (lops_spec.js:163-191)"""
    return _gemvM(g, a, g._lib.p0_gemvM)


def gemvM_noalloc(g, a):
    """gemvM(g, a) -> nsplit without any device allocation during the call (no counterpart in the reference): for
    callers that must not allocate mid-call, e.g. a latency-bound decode loop that cannot afford the device-wide wait
    of a workspace re-allocation, or a process whose device memory belongs to another allocator. Its scratch is a
    fixed 16 MiB device array shared by every call on the device, so calls that overlap on the GPU race; calls that
    need more scratch raise P0Error (include/p0mm.h has the limits)."""
    return _gemvM(g, a, g._lib.p0_gemvM_noalloc)


def _gemvM(g, a, entry):
    x, y = a["x"], a["y"]
    stat, norm, ev, src, mx = a.get("stat"), a.get("norm"), a.get("ev"), a.get("src"), a.get("mx")
    pro, epi = a.get("pro") or "raw", a.get("epi") or "store"
    if pro not in L.PRO:
        raise P0Error(L.P0_EINVAL, "gemvM: prologue " + str(pro))
    if epi not in L.EPI:
        raise P0Error(L.P0_EINVAL, "gemvM: epilogue " + str(epi))
    args = L.p0_gemvM_args(
        _wview(a["w"], "gemvM"), handle(x["buf"]), int(x.get("rowB") or 0), int(x.get("ldx") or 0), int(a["M"]), int(a["N"]), int(a["K"]),
        int(a.get("kPer") or 0), L.PRO[pro], L.EPI[epi], handle(y["buf"]), int(y.get("ldy") or 0), int(y.get("ldm") or 0),
        _b(stat), int((stat or {}).get("off") or 0), int((stat or {}).get("ld") or 0), _b(norm), int((norm or {}).get("off") or 0),
        _b(ev), int((ev or {}).get("off") or 0), int((ev or {}).get("ld") or 0), int((src or {}).get("n") or 0),
        int((src or {}).get("ld") or 0), _b(mx), float(a.get("cap") or 0.0))
    ns = ctypes.c_uint32()
    g._check(entry(g.ctx, ctypes.byref(args), ctypes.byref(ns)))
    return ns.value


def gemm(gpu, a):
    """gemm(gpu, a) -> flops (gemm.js:264-322). x prologues 'f16', 'lnmod', 'rms'; acc 'f32' or 'f16' (both
    accumulate in f32 on the tensor cores); every epilogue of
    gemm.js:187-250 ('f16', 'f32', 'bias', 'resadd', 'swiglu', 'heads', 'onormgate')."""
    x, y = a["x"], a["y"]
    ev, bv = a.get("ev"), a.get("bv")
    epi = a.get("epi") or "f16"
    if epi not in L.GEPI:
        raise P0Error(L.P0_EINVAL, "gemm: epilogue %s is not built in this library yet" % epi)
    xmode = x.get("mode") or "f16"
    if xmode not in L.XPRO or a.get("conv"):
        raise P0Error(L.P0_EINVAL, "gemm: x prologue %s is not built in this library yet" % ("conv" if a.get("conv") else xmode))
    stats, pv = a.get("stats"), a.get("pv")
    acc = a.get("acc") or "f32"
    args = L.p0_gemm_args(
        _wview(a["w"], "gemm"), handle(x["buf"]), int(x.get("off") or 0), int(x.get("ld") or 0), int(x.get("k0") or 0), int(a["M"]),
        int(a["N"]), int(a["K"]), int(a.get("wr0") or 0), int(a.get("wr1") or 0), int(a.get("wk0") or 0), L.GEPI[epi],
        L.ACT[a.get("act") or "silu"], 1 if acc == "f16" else 0, handle(y["buf"]), int(y.get("off") or 0), int(y.get("ld") or 0),
        int(y.get("n0") or 0), _b(ev), int((ev or {}).get("off") or 0), _b(bv), int((bv or {}).get("off") or 0),
        int((bv or {}).get("up") or 0), int(bool(a.get("res"))), int(bool(a.get("store"))), int(bool(a.get("post_gelu"))),
        L.XPRO[xmode], _b(stats), int((stats or {}).get("off") or 0), _b(pv), int((pv or {}).get("off") or 0),
        int((pv or {}).get("stride") or 0))
    h = a.get("heads") or {}
    args.h_Ltot, args.h_Hq, args.h_Hkv, args.h_rowOff = (int(h.get(k) or 0) for k in ("Ltot", "Hq", "Hkv", "rowOff"))
    args.h_eps = float(h.get("eps") or 0.0)
    args.h_rope_mode = L.P0_ROPE_HALF if h.get("ropeMode") == "half" else L.P0_ROPE_INTER
    args.rope, args.gt = _b(h.get("rope")), _b(a.get("gt"))   # bound from the buffer start, as gemm.js:304 binds them
    fl = ctypes.c_double()
    gpu._check(gpu._lib.p0_gemm(gpu.ctx, ctypes.byref(args), ctypes.byref(fl)))
    return fl.value


def dequant_f16(g, w, out):
    """the GEMM's in-kernel dequantisation of a q4 view written to out (rows*cols fp16), for bit-exact checks"""
    wv = _wview(w, "dequant")
    g._check(g._lib.p0_dequant_f16(g.ctx, ctypes.byref(wv), handle(out)))


def pack_q4(g, w_f32, N, K, out=None, w_off=0, ldw=0, out_off=0):
    """packQ4 (engine/kcheck.js:22-38) on the device: a W f32 [N][K] buffer -> q4g32a.t64 records; returns the out buffer"""
    if out is None:
        out = g.buffer(N * K // 32 * 20, "q4")
    g._check(g._lib.p0_pack_q4(g.ctx, handle(w_f32), int(w_off), int(ldw), int(N), int(K), handle(out), int(out_off)))
    return out


def pack_q8(g, w_f32, N, K, out=None, w_off=0, ldw=0, out_off=0):
    """packQ8 (engine/kcheck.js:39-52) on the device: a W f32 [N][K] buffer -> q8g64s.t64 records; returns the out buffer"""
    if out is None:
        out = g.buffer(N * K // 64 * 66, "q8")
    g._check(g._lib.p0_pack_q8(g.ctx, handle(w_f32), int(w_off), int(ldw), int(N), int(K), handle(out), int(out_off)))
    return out


# ---------------------------------------------------------------- decode-path operators (lops.js, lops_spec.js)
def argmax(g, a):
    """argmax(g, a) (lops.js:434-436): a = {mx: {buf}, n, out: {buf}}; out[0] = the index of the largest of the n
    (max, bitcast index) pairs (ties: the lowest index), out[1] = the bits of that max"""
    g._check(g._lib.p0_argmaxM(g.ctx, handle(a["mx"]["buf"]), int(a["n"]), 1, handle(a["out"]["buf"])))


def argmaxM(g, a):
    """argmaxM(g, a) (lops_spec.js:346-348): a = {mx: {buf}, n, M, out: {buf}}; per row m of mx [M][n][2], out[2m] /
    out[2m + 1] as argmax"""
    g._check(g._lib.p0_argmaxM(g.ctx, handle(a["mx"]["buf"]), int(a["n"]), int(a["M"]), handle(a["out"]["buf"])))


def embed(g, a):
    """embed(g, a) (lops.js:352-365): a = {w (q4 / q8 table view), ids: {buf}, x: {buf}, st: {buf, off}, K, n, scale,
    rowOut, eps}; x[(rowOut + m) * K + k] = dequant(w[ids[m]]) * scale, st[off + m] = the row's rstd"""
    w = a["w"]
    enc = w.get("enc") or "q4g32a.t64"
    if enc not in ("q4g32a.t64", "q8g64s.t64"):
        raise P0Error(L.P0_EINVAL, "embed: encoding " + str(enc))
    st = a["st"]
    args = L.p0_embed_args(_wview(w, "embed"), handle(a["ids"]["buf"]), handle(a["x"]["buf"]), handle(st["buf"]),
                           int(st.get("off") or 0), int(a["K"]), int(a["n"]), int(a.get("rowOut") or 0), float(a["scale"]),
                           float(a.get("eps") or 0.0))
    g._check(g._lib.p0_embed(g.ctx, ctypes.byref(args)))


def normadd(g, a):
    """normadd(g, a) (lops.js:174-180): a = {t: {buf, n, ld}, w: {buf, off} (mode 0), x: {buf}, st: {buf, off}, D, M,
    eps, scale (default 1), mode (0: x = (x + rms(t) * w) * scale, 1: x = t)}"""
    t, w, st = a["t"], a.get("w"), a["st"]
    scale = a.get("scale")
    args = L.p0_normadd_args(handle(t["buf"]), int(t.get("n") or 1), int(t.get("ld") or 0), _b(w), int((w or {}).get("off") or 0),
                             handle(a["x"]["buf"]), handle(st["buf"]), int(st.get("off") or 0), int(a["D"]), int(a.get("M") or 1),
                             int(a.get("mode") or 0), float(a.get("eps") or 0.0), 1.0 if scale is None else float(scale))
    g._check(g._lib.p0_normadd(g.ctx, ctypes.byref(args)))


def dhead(g, a):
    """dhead(g, a) (lops_spec.js:475-482): a = {w (q4 / q8 head view), x: {buf}, stat: {buf, off}, norm: {buf, off},
    sel: {buf}, mx: {buf}, K (<= 512), tPer, nsel}; per selected tile its largest row dot and that row's index"""
    w = a["w"]
    enc = w.get("enc") or "q4g32a.t64"
    if enc not in ("q4g32a.t64", "q8g64s.t64"):
        raise P0Error(L.P0_EINVAL, "dhead: encoding " + str(enc))
    if int(a["K"]) > 512:
        raise P0Error(L.P0_EINVAL, "dhead: K > 512")
    stat, norm = a["stat"], a["norm"]
    args = L.p0_dhead_args(_wview(w, "dhead"), handle(a["x"]["buf"]), handle(stat["buf"]), int(stat.get("off") or 0),
                           handle(norm["buf"]), int(norm.get("off") or 0), handle(a["sel"]["buf"]), handle(a["mx"]["buf"]),
                           int(a["K"]), int(a["tPer"]), int(a["nsel"]))
    g._check(g._lib.p0_dhead(g.ctx, ctypes.byref(args)))


def qkrope(g, a):
    """qkrope(g, a) (lops.js:226-233): a = {s: {buf, n, ld}, norm: {buf}, rope: {buf, off}, q: {buf}, kc: {buf}, vc: {buf},
    D, nq, hasKV, pos, eps, qw, kw, npairs, kvRow, nkv, kvLen}; q f32 out, k / v into the fp16 caches at kvRow"""
    s, rope = a["s"], a["rope"]
    kc, vc = a.get("kc"), a.get("vc")
    args = L.p0_qkrope_args(handle(s["buf"]), int(s.get("n") or 1), int(s.get("ld") or 0), handle(a["norm"]["buf"]), int(a.get("qw") or 0),
                            int(a.get("kw") or 0), handle(rope["buf"]), int(rope.get("off") or 0), int(a["npairs"]), int(a.get("pos") or 0),
                            handle(a["q"]["buf"]), _b(kc), _b(vc), int(a["D"]), int(a["nq"]), int(a.get("nkv") or 1),
                            int(bool(a.get("hasKV"))), int(a.get("kvRow") or 0), int(a.get("kvLen") or 0), float(a.get("eps") or 0.0))
    g._check(g._lib.p0_qkrope(g.ctx, ctypes.byref(args)))


def attnDec(g, a):
    """attnDec(g, a) (lops.js:306-321): a = {q: {buf}, kc: {buf}, vc: {buf}, part: {buf}, out: {buf}, D, nh, kStart, kEnd,
    ring, nkv, kvLen}; out f32 [nh][D] = softmax(q . k) . v over the keys (a tuner's `ad` choice is not used)"""
    args = L.p0_attn_dec_args(handle(a["q"]["buf"]), handle(a["kc"]["buf"]), handle(a["vc"]["buf"]), handle(a["part"]["buf"]),
                              handle(a["out"]["buf"]), int(a["D"]), int(a["nh"]), int(a.get("nkv") or 1), int(a.get("kvLen") or 0),
                              int(a["kStart"]), int(a["kEnd"]), int(a.get("ring") or 0))
    g._check(g._lib.p0_attn_dec(g.ctx, ctypes.byref(args)))
