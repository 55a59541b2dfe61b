"""A second, independent transcription of the reference's kernel arithmetic for this path, in numpy, used to pin the C
oracle (oracle/oracle.c) bit for bit on small shapes. It is written from the WGSL the reference generates, not from the
oracle:

  lgemv   engine/llm/lops.js:30-106        (gemvCode: prologues raw / rms / sum / pleg, q4 and q8 records, epilogues
                                            store / geglu / softcap with the per-tile max and lowest argmax)
  lgemvM  engine/llm/lops_spec.js:44-157   (gemvMCode with the default variant: x staged per chunk, same per-row order)
  gemm    engine/ops/gemm.js:131-211       (the 'f16' x path: fp16 X tile, fp16 W tile f16(q*s + mn) / f16(q*s), f32 FMA
                                            accumulation or fp16 partial sums per 32-k tile, epilogues f16 / f32 / bias /
                                            resadd / swiglu)
          engine/ops/gemm.js:55-63         (the f32 x prologues lnmod / rms)
          engine/ops/gemm.js:212-250       (the head-reducing epilogues heads (QK-RMSNorm + RoPE, head-major) and
                                            onormgate)
  decode  engine/llm/lops.js:143-347       (normadd, qkrope, attnDec and its combine, embed: 256-thread strided
                                            sums and the workgroup tree, as the WGSL reduces)
          engine/llm/lops_spec.js:428-473  (dhead: the drafter's head over selected tiles, max and lowest argmax)

Conventions, stated once for every WGSL expression: f32 arithmetic rounds after every operation (numpy float32), with
no contraction of a*b + c unless the WGSL writes fma(); `dot(u, v)` is u.x*v.x + u.y*v.y + u.z*v.z + u.w*v.w added
left to right; `a + b * c + d * e` is (a + b*c) + d*e; tanh is the C library's tanhf (the WGSL leaves its precision to
the implementation). A fused f32 FMA of two fp16 values and an f32 is one f32 addition, since the product of two fp16
values is exact in f32; the fp16 FMA of the 'f16' accumulation rounds the exact f64 value once to fp16. Rows and
quarter lanes are vectorised with numpy; the loops run over k groups in the WGSL's order.
"""
import ctypes
import ctypes.util

import numpy as np

F = np.float32
_libm = ctypes.CDLL(ctypes.util.find_library("m") or "libm.so.6")
_libm.tanhf.restype = ctypes.c_float
_libm.tanhf.argtypes = [ctypes.c_float]
_tanhf_vec = np.frompyfunc(lambda v: _libm.tanhf(float(v)), 1, 1)
_libm.expf.restype = ctypes.c_float
_libm.expf.argtypes = [ctypes.c_float]
_expf_vec = np.frompyfunc(lambda v: _libm.expf(float(v)), 1, 1)

C_GELU1, C_GELU2 = F(0.7978845608028654), F(0.044715)


def tanhf(a):
    a = np.asarray(a, F)
    return np.asarray(_tanhf_vec(a), dtype=np.float64).astype(F).reshape(a.shape)


def expf(a):
    a = np.asarray(a, F)
    return np.asarray(_expf_vec(a), dtype=np.float64).astype(F).reshape(a.shape)


def gelu_lops(v):
    """lops.js:24 GELU(v): (v * 0.5 * (1.0 + tanh(clamp(0.79788.. * (v + 0.044715 * v * v * v), -15, 15))))"""
    v = np.asarray(v, F)
    t = ((C_GELU2 * v) * v) * v
    u = np.clip(C_GELU1 * (v + t), F(-15.0), F(15.0)).astype(F)
    return ((v * F(0.5)) * (F(1.0) + tanhf(u))).astype(F)


def gelu_gemm(g):
    """gemm.js:204 swiglu 'gelu': g * 0.5 * (1 + tanh(clamp(0.7978845608 * (g + 0.044715 * g * g * g), -15, 15)))"""
    g = np.asarray(g, F)
    t = ((F(0.044715) * g) * g) * g
    u = np.clip(F(0.7978845608) * (g + t), F(-15.0), F(15.0)).astype(F)
    return ((g * F(0.5)) * (F(1.0) + tanhf(u))).astype(F)


def silu_gemm(g):
    """gemm.js:204 swiglu 'silu': g / (1 + exp(-g)) (exp: the C library's expf)"""
    g = np.asarray(g, F)
    e = expf(-g)
    return (g / (F(1.0) + e)).astype(F)


def words(b):
    """the weight buffer as u32 words (W: array<u32>)"""
    return np.frombuffer(np.ascontiguousarray(b, dtype=np.uint8).tobytes(), dtype=np.uint32)


def unpack2x16float(w):
    """WGSL unpack2x16float: (low half, high half) as f32"""
    w = np.asarray(w, np.uint32)
    lo = (w & 0xFFFF).astype(np.uint16).view(np.float16).astype(F)
    hi = (w >> 16).astype(np.uint16).view(np.float16).astype(F)
    return lo, hi


def dot4(u, v):
    """dot(u, v) over the last axis of length 4, added left to right"""
    return (((u[..., 0] * v[..., 0]) + (u[..., 1] * v[..., 1])) + (u[..., 2] * v[..., 2])) + (u[..., 3] * v[..., 3])


def _tile_dots(W, xs, k0, k1, tile_rows, wG, wOff, q8):
    """acc for every (row of the given tiles, quarter lane w) over groups [g0, g1): lops.js:63-82 / lops_spec.js:92-112.
    xs: the staged x, f32, indexed from k0. Returns f32 [rows, 4]."""
    rows = np.asarray(tile_rows)
    t, r = rows // 64, rows % 64
    acc = np.zeros((rows.size, 4), F)
    wv = np.arange(4)
    if not q8:
        g0, g1 = k0 // 32, (k1 + 31) // 32
        for g in range(g0, g1):
            rec = wOff + (t * wG + g) * 320
            q = W[rec[:, None] + r[:, None] * 4 + wv[None, :]]                         # [rows, 4]
            s, mn = unpack2x16float(W[rec + 256 + r])
            xb = g * 32 - k0 + wv * 8                                                   # [4]
            a = np.stack([xs[xb + i] for i in range(4)], -1)[None, :, :]                  # [1, 4, 4]
            b = np.stack([xs[xb + 4 + i] for i in range(4)], -1)[None, :, :]
            qa = np.stack([((q >> (4 * i)) & 15) for i in range(4)], -1).astype(F)
            qb = np.stack([((q >> (16 + 4 * i)) & 15) for i in range(4)], -1).astype(F)
            one = np.ones(4, F)
            d1 = dot4(qa, a) + dot4(qb, b)
            d2 = dot4(a, one) + dot4(b, one)
            acc = (acc + s[:, None] * d1) + mn[:, None] * d2
    else:
        g0, g1 = k0 // 64, (k1 + 63) // 64
        for g in range(g0, g1):
            rec = wOff + (t * wG + g) * 1056
            s2x, s2y = unpack2x16float(W[rec + 1024 + (r >> 1)])
            sc = np.where((r & 1) == 1, s2y, s2x).astype(F)
            d = np.zeros((rows.size, 4), F)
            for u in range(4):
                q = W[rec[:, None] + r[:, None] * 16 + wv[None, :] * 4 + u]
                qv = np.stack([((q << (24 - 8 * i)) & 0xFFFFFFFF).astype(np.uint32).view(np.int32) >> 24 for i in range(4)], -1).astype(F)
                xb = g * 64 - k0 + wv * 16 + u * 4
                xv = np.stack([xs[xb + i] for i in range(4)], -1)[None, :, :]
                d = d + dot4(qv, xv)
            acc = acc + sc[:, None] * d
    return acc


def _quarter_sum(acc):
    """red[li] + red[li + 1] + red[li + 2] + red[li + 3] (lops.js:86-88)"""
    return ((acc[:, 0] + acc[:, 1]) + acc[:, 2]) + acc[:, 3]


def _softcap_tiles(tot, cap, ntile_rows):
    """v = cap * tanh(clamp(tot / cap, -15, 15)); per 64-row tile the max and the lowest row holding it"""
    cap = F(cap)
    v = (cap * tanhf(np.clip(tot / cap, F(-15.0), F(15.0)).astype(F))).astype(F)
    vt = v.reshape(-1, 64)
    mx = vt.max(axis=1)
    idx = np.array([int(np.nonzero(vt[i] == mx[i])[0][0]) for i in range(vt.shape[0])], np.int64)
    return v, mx, idx


def gemv(Wbytes, X, N, K, *, enc="q4g32a.t64", cols=None, woff=0, rowB=0, kPer=None, pro="raw", epi="store", ldy=None,
         stat=None, stat_off=0, norm=None, norm_off=0, ev=None, ev_off=0, src=None, cap=30.0, KCH=2048):
    """lgemv for one token. Returns (Y, MX or None, nsplit) with the reference's output layout."""
    q8 = enc == "q8g64s.t64"
    G = 64 if q8 else 32
    W = words(Wbytes)
    wG = (cols or K) // G
    kp = kPer or K
    nsplit = -(-K // kp)
    ldy = ldy or N
    X = np.asarray(X, F)
    NT = N // 64
    Y = np.zeros(nsplit * ldy if epi == "store" else N, F)
    MX = np.zeros(NT * 2, F) if epi == "softcap" else None
    for split in range(nsplit):
        k0, k1 = split * kp, min(K, split * kp + kp)
        k = np.arange(k0, k1)
        if pro == "raw":
            xs = X[rowB + k]
        elif pro == "rms":
            xs = (X[rowB + k] * F(stat[stat_off])) * np.asarray(norm, F)[norm_off + k]
        else:
            ldp, nsrc = src
            s = np.zeros(k.size, F)
            for j in range(nsrc):
                s = s + X[j * ldp + k]
            xs = s if pro == "sum" else gelu_lops(s) * np.asarray(ev, F)[ev_off + k]
        xs = np.asarray(xs, F)
        rows = np.arange(N)
        tot0 = _quarter_sum(_tile_dots(W, xs, k0, k1, rows, wG, woff // 4, q8))
        if epi == "store":
            Y[split * ldy:split * ldy + N] = tot0
        elif epi == "geglu":
            tot1 = _quarter_sum(_tile_dots(W, xs, k0, k1, rows + N, wG, woff // 4, q8))
            Y[:N] = gelu_lops(tot0) * tot1
        else:
            v, mx, idx = _softcap_tiles(tot0, cap, NT)
            Y[:N] = v
            MX[0::2] = mx
            MX[1::2] = (np.arange(NT) * 64 + idx).astype(np.uint32).view(F)
    return Y, MX, nsplit


def gemvM(Wbytes, X, M, N, K, *, enc="q4g32a.t64", cols=None, woff=0, rowB=0, ldx=None, kPer=None, pro="raw", epi="store",
          ldm=None, ldy=None, stat=None, stat_off=0, stat_ld=2, norm=None, norm_off=0, ev=None, ev_off=0, ev_ld=0, src=None,
          cap=30.0):
    """lgemvM: per row m the lgemv order with x from row m (x.ldx), rstd ST[statOff + m*statLd], pleg ev per row.
    Returns (Y, MX or None, nsplit) in lops_spec.js's layout Y[split*ldy + m*ldm + n], MX[(m*ntile + tile)*2]."""
    q8 = enc == "q8g64s.t64"
    G = 64 if q8 else 32
    W = words(Wbytes)
    wG = (cols or K) // G
    kp = kPer or K
    nsplit = -(-K // kp)
    ldx, ldm = ldx or K, ldm or N
    ldy = ldy or M * ldm
    X = np.asarray(X, F)
    NT = N // 64
    Y = np.zeros(nsplit * ldy if epi == "store" else M * ldm, F)
    MX = np.zeros(M * NT * 2, F) if epi == "softcap" else None
    rows = np.arange(N)
    for split in range(nsplit):
        k0, k1 = split * kp, min(K, split * kp + kp)
        k = np.arange(k0, k1)
        for m in range(M):
            if pro == "raw":
                xs = X[m * ldx + rowB + k]
            elif pro == "rms":
                xs = (X[m * ldx + rowB + k] * F(stat[stat_off + m * stat_ld])) * np.asarray(norm, F)[norm_off + k]
            else:
                ldp, nsrc = src
                s = np.zeros(k.size, F)
                for j in range(nsrc):
                    s = s + X[j * ldp + m * ldx + k]
                xs = gelu_lops(s) * np.asarray(ev, F)[ev_off + m * ev_ld + k]
            xs = np.asarray(xs, F)
            tot0 = _quarter_sum(_tile_dots(W, xs, k0, k1, rows, wG, woff // 4, q8))
            if epi == "store":
                Y[split * ldy + m * ldm:split * ldy + m * ldm + N] = tot0
            elif epi == "geglu":
                tot1 = _quarter_sum(_tile_dots(W, xs, k0, k1, rows + N, wG, woff // 4, q8))
                Y[m * ldm:m * ldm + N] = gelu_lops(tot0) * tot1
            else:
                v, mx, idx = _softcap_tiles(tot0, cap, NT)
                Y[m * ldm:m * ldm + N] = v
                MX[m * NT * 2:(m + 1) * NT * 2:2] = mx
                MX[m * NT * 2 + 1:(m + 1) * NT * 2:2] = (np.arange(NT) * 64 + idx).astype(np.uint32).view(F)
    return Y, MX, nsplit


def _h(bits):
    return np.asarray(bits, np.uint16).view(np.float16).astype(F)


def gemm_wtile(Wbytes, rows, k_lo, k_hi, enc, wG, wk0=0):
    """the fp16 W tile values gemm.js:139-160 builds for weight rows `rows` and k in [k_lo, k_hi): q4 f16(q*s + mn),
    q8 f16(q*s), as f32 values [rows, k]"""
    W = words(Wbytes)
    rows = np.asarray(rows)
    out = np.zeros((rows.size, k_hi - k_lo), F)
    rr, tb = rows & 63, rows >> 6
    for kk in range(k_lo, k_hi):
        kw = wk0 + kk
        if enc == "q4g32a.t64":
            rec = (tb * wG + kw // 32) * 320
            q = W[rec + rr * 4 + (kw % 32) // 8]
            cv = ((q >> (4 * (kw % 8))) & 15).astype(F)
            s, mn = unpack2x16float(W[rec + 256 + rr])
            out[:, kk - k_lo] = ((cv * s) + mn).astype(np.float16).astype(F)
        else:
            rec = (tb * wG + kw // 64) * 1056
            q = W[rec + rr * 16 + (kw % 64) // 4]
            cv = ((q << (24 - 8 * (kw % 4))) & 0xFFFFFFFF).astype(np.uint32).view(np.int32) >> 24
            s2x, s2y = unpack2x16float(W[rec + 1024 + (rr >> 1)])
            sc = np.where((rr & 1) == 1, s2y, s2x)
            out[:, kk - k_lo] = (cv.astype(F) * sc).astype(np.float16).astype(F)
    return out


def _f16_round_once(v64):
    """an exact f64 value rounded once to fp16 (round half to even), as f32"""
    return np.asarray(v64, np.float64).astype(np.float16).astype(F)


def gemm(Wbytes, X16, M, N, K, *, enc="q4g32a.t64", rows=None, cols=None, ldx=None, kx0=0, wr0=0, wr1=0, wk0=0, epi="f16",
         act="silu", acc="f32", Y=None, ldy=None, ny0=0, ev=None, ev_off=0, bv=None, bv_off=0, bv_up=0, res=False, store=False,
         post_gelu=False):
    """gemm.js with the 'f16' x path. X16 fp16 bits [M][ldx]. Returns Y (fp16 bits, or f32 for 'f32' / 'resadd')."""
    Nw = rows or N
    G = 64 if enc == "q8g64s.t64" else 32
    wG = (cols or K) // G
    ldx, ldy = ldx or K, ldy or N
    f32y = epi in ("f32", "resadd")
    if Y is None:
        Y = np.zeros(M * ldy, F if f32y else np.uint16)
    Y = Y.copy()
    ncol = N if epi != "swiglu" else N
    cc = np.arange(ncol)
    if epi == "swiglu":
        wrows = np.where((cc & 1) == 0, wr0, wr1) + (cc >> 1)
    else:
        wrows = np.minimum(wr0 + cc, Nw - 1)
    Wt = gemm_wtile(Wbytes, wrows, 0, K, enc, wG, wk0)               # [N, K] fp16 values
    Xv = _h(np.asarray(X16, np.uint16).reshape(M, ldx)[:, kx0:kx0 + K])   # [M, K]
    A = np.zeros((M, ncol), F)
    for k0 in range(0, K, 32):
        if acc == "f16":
            h = np.zeros((M, ncol), F)
            for k in range(k0, k0 + 32):
                h = _f16_round_once(Xv[:, k:k + 1].astype(np.float64) * Wt[None, :, k].astype(np.float64) + h.astype(np.float64))
            A = A + h
        else:
            for k in range(k0, k0 + 32):
                A = A + Xv[:, k:k + 1] * Wt[None, :, k]       # fma: the fp16 x fp16 product is exact in f32
    Yr = Y.reshape(M, ldy)
    if epi == "swiglu":
        gB = np.asarray(bv, F)[bv_off + np.arange(N // 2)] if bv is not None else np.zeros(N // 2, F)
        uB = np.asarray(bv, F)[bv_off + bv_up + np.arange(N // 2)] if bv is not None else np.zeros(N // 2, F)
        g = A[:, 0::2] + gB
        u = A[:, 1::2] + uB
        a = gelu_gemm(g) if act == "gelu" else silu_gemm(g)
        Yr[:, ny0:ny0 + N // 2] = (a * u).astype(np.float16).view(np.uint16)
    elif epi == "f16":
        Yr[:, ny0:ny0 + N] = A.astype(np.float16).view(np.uint16)
    elif epi == "f32":
        Yr[:, ny0:ny0 + N] = A
    elif epi == "bias":
        t = A + np.asarray(ev, F)[ev_off + np.arange(N)]
        if res:
            t = t + _h(Yr[:, ny0:ny0 + N])
        h = t.astype(np.float16)
        if post_gelu:   # misc.js:116 ew 'gelu' on the fp16 result, in f32: 0.5 * x * (1 + tanh(clamp(u, -15, 15)))
            x = h.astype(F)
            uu = np.clip(F(0.7978845608) * (x + ((C_GELU2 * x) * x) * x), F(-15.0), F(15.0)).astype(F)
            h = ((F(0.5) * x) * (F(1.0) + tanhf(uu))).astype(np.float16)
        Yr[:, ny0:ny0 + N] = h.view(np.uint16)
    elif epi == "resadd":
        gte = np.asarray(ev, F)[ev_off + np.arange(N)] if ev is not None else np.ones(N, F)
        c = np.asarray(bv, F)[bv_off + np.arange(N)] if bv is not None else np.zeros(N, F)
        t = gte * (A + c)
        Yr[:, ny0:ny0 + N] = t if store else Yr[:, ny0:ny0 + N] + t
    return Y


def gemm_xpro(mode, X, M, K, *, ldx=None, kx0=0, stats=None, stat_off=0, pv=None, pv_off=0, pv_stride=0):
    """gemm.js:55-63, xload() for the f32 x paths: one fp16 X value per element of the k range [kx0, kx0 + K) of each
    row, with {mean, rstd} = ST[(statOff + row) * 2 ..] and the PV vectors indexed by the x column (kx0 + k):
      lnmod  f16(((x - mean) * rstd) * (1 + PV[pvOff + col]) + PV[pvOff + pvStride + col])
      rms    f16((x * rstd) * PV[pvOff + col])
    Returns fp16 bits [M][K]."""
    ldx = ldx or K
    Xr = np.asarray(X, F).reshape(M, ldx)[:, kx0:kx0 + K]
    st = np.asarray(stats, F).reshape(-1)
    srow = (stat_off + np.arange(M)) * 2
    mean, rstd = st[srow][:, None], st[srow + 1][:, None]
    pvv = np.asarray(pv, F)
    col = kx0 + np.arange(K)
    if mode == "lnmod":
        v = ((Xr - mean) * rstd) * (F(1.0) + pvv[pv_off + col]) + pvv[pv_off + pv_stride + col]
    elif mode == "rms":
        v = (Xr * rstd) * pvv[pv_off + col]
    else:
        raise ValueError(mode)
    return v.astype(F).astype(np.float16).view(np.uint16).ravel()


def gemm_red128(A, M, N, *, epi, ev, ev_off=0, heads=None, gt=None, Y=None, ldy=None, ny0=0):
    """gemm.js:212-250, the epilogues that reduce over one 128-wide head, on the call's f32 accumulators A [M][N], in
    the workgroup-memory form (no subgroup shuffles): thread tx of the head's 16 holds 8 columns (tx*8 .. +7, or for
    rotate_half tx*4 .. +3 and 64 + tx*4 .. +3), its share of the sum of squares is dot(a0, a0) + dot(a1, a1), and the
    row's sum adds the 16 shares in tx order from 0.0; inv = inverseSqrt(s / 128 + eps), taken correctly rounded.
      onormgate  Y[(m*ldy + ny0) & ~3 + n] = f16(((a * inv) * EV[evOff + c]) / (1 + exp(-GT[(m*Ltot + ny0) & ~3 + n])))
      heads      q heads (hd < Hq) / k heads (hd < Hq + Hkv): v = (a * inv) * EV[evOff + (k ? 128 : 0) + c], then RoPE
                 with the (cos, sin) pairs of RP row rowOff + m: rotate_half pairs (d, d + 64) with pair d, interleaved
                 pairs (2p, 2p + 1) with pair p; v heads: a. Y head-major: Y[((hd * Ltot) + rowOff + m) * 128 + c].
    Returns Y (fp16 bits; slots the call does not write keep theirs)."""
    A = np.asarray(A, F).reshape(M, N)
    h = heads or {}
    Ltot, Hq, Hkv, rowOff = int(h.get("Ltot") or 0), int(h.get("Hq") or 0), int(h.get("Hkv") or 0), int(h.get("rowOff") or 0)
    eps = F(h.get("eps") or 1e-6)
    half = epi == "heads" and h.get("ropeMode") == "half"
    ldy = ldy or N
    evv = np.asarray(ev, F)
    Y = np.asarray(Y, np.uint16).copy()
    c = np.arange(128)
    for hd in range(N // 128):
        a = A[:, hd * 128:(hd + 1) * 128]
        s = np.zeros(M, F)
        for tx in range(16):
            i0, i1 = (tx * 4, 64 + tx * 4) if half else (tx * 8, tx * 8 + 4)
            s = s + (dot4(a[:, i0:i0 + 4], a[:, i0:i0 + 4]) + dot4(a[:, i1:i1 + 4], a[:, i1:i1 + 4]))
        inv = (1.0 / np.sqrt((s / F(128.0) + eps).astype(np.float64))).astype(F)[:, None]
        if epi == "onormgate":
            g16 = _h(gt)
            for m in range(M):
                gb, yb = (m * Ltot + ny0) & ~3, (m * ldy + ny0) & ~3
                n = hd * 128 + c
                g = g16[gb + n]
                v = ((a[m] * inv[m]) * evv[ev_off + c]) / (F(1.0) + expf(-g))
                Y[yb + n] = v.astype(F).astype(np.float16).view(np.uint16)
            continue
        sec = 0 if hd < Hq else 1 if hd < Hq + Hkv else 2
        rows = rowOff + np.arange(M)
        out = ((hd * Ltot + rows) * 128)[:, None] + c[None, :]
        if sec == 2:
            Y[out] = a.astype(np.float16).view(np.uint16)
            continue
        v = (a * inv) * evv[ev_off + (128 if sec else 0) + c][None, :]
        rp = np.asarray(h["rope"], F).reshape(-1, 128)[rows]           # (cos, sin) pairs of each row
        cs, sn = rp[:, 0::2], rp[:, 1::2]                               # [M, 64]
        r = np.empty_like(v)
        if half:
            lo, hi = v[:, :64], v[:, 64:]
            r[:, :64] = (lo * cs) - (hi * sn)
            r[:, 64:] = (hi * cs) + (lo * sn)
        else:
            x0, x1 = v[:, 0::2], v[:, 1::2]
            r[:, 0::2] = (x0 * cs) - (x1 * sn)
            r[:, 1::2] = (x0 * sn) + (x1 * cs)
        Y[out] = r.astype(F).astype(np.float16).view(np.uint16)
    return Y


# ---------------------------------------------------------------- decode-path operators (engine/llm/lops.js)
def _inverse_sqrt(v):
    """WGSL inverseSqrt, taken correctly rounded"""
    return F(1.0 / np.sqrt(np.float64(v)))


def _strided_sumsq(v, D):
    """the 256 threads' shares of sum(v * v) over i = t, t + 256, ... (in that order, from 0.0), then the workgroup's
    tree: red[t] += red[t + k] for k = 128, 64, .., 1"""
    red = np.zeros(256, F)
    for i0 in range(0, D, 256):
        n = min(256, D - i0)
        red[:n] = red[:n] + v[i0:i0 + n] * v[i0:i0 + n]
    k = 128
    while k > 0:
        red[:k] = red[:k] + red[k:2 * k]
        k >>= 1
    return red[0]


def _split_sum(S, nsrc, ldp, idx):
    """src(i) = sum of the split partials S[j * ldp + i] for j = 0 .. nsrc - 1, from 0.0"""
    v = np.zeros(len(idx), F)
    for j in range(nsrc):
        v = v + S[j * ldp + idx]
    return v


def normadd(T, nsrc, ldp, W, w_off, X, ST, st_off, D, M, *, mode=0, eps=1e-6, scale=1.0):
    """lops.js:143-178 (NORMADD): per row m, tv = the split partials summed; rs = inverseSqrt(sumsq(tv) / D + eps);
    mode 0: x = (x + (tv * rs) * W[wOff + i]) * scale, mode 1: x = tv; ST[statOff + m] = inverseSqrt(sumsq(x) / D + eps).
    Returns (X, ST) as new arrays."""
    T, X, ST = np.asarray(T, F), np.asarray(X, F).copy(), np.asarray(ST, F).copy()
    Wv = np.asarray(W, F) if W is not None else None
    eps, scale = F(eps), F(scale)
    i = np.arange(D)
    for m in range(M):
        xb = m * D
        tv = _split_sum(T, nsrc, ldp, xb + i)
        rs = _inverse_sqrt(_strided_sumsq(tv, D) / F(D) + eps)
        x = X[xb:xb + D]
        x = (x + (tv * rs) * Wv[w_off + i]) * scale if mode == 0 else tv
        X[xb:xb + D] = x
        ST[st_off + m] = _inverse_sqrt(_strided_sumsq(x, D) / F(D) + eps)
    return X, ST


def qkrope(S, nsrc, ldp, NW, RP, D, nq, *, nkv=1, hasKV=True, pos=0, eps=1e-6, qw=0, kw=0, npairs=None, rope_off=0, kv_row=0,
           kv_len=0, Q=None, KC=None, VC=None):
    """lops.js:181-224 (QKROPE): workgroup h (q heads 0 .. nq - 1, then nkv k heads, then nkv v heads) sums its head's
    split partials hv, rs = inverseSqrt(sumsq(hv) / D + eps); v heads: f16(hv * rs) into VC's row kvRow of the head;
    q / k heads: a = (hv[d] * rs) * NW[w + d], b = (hv[d + D/2] * rs) * NW[w + d + D/2], (cos, sin) from
    RP[ropeOff + (pos * npairs + d) * 2] for d < npairs (else (1, 0)), lo = a*c - b*sn, hi = b*c + a*sn; q heads -> Q,
    k heads -> f16 into KC's row kvRow. Returns (Q, KC, VC) as new arrays (fp16 bits for the caches)."""
    npairs = D // 2 if npairs is None else npairs
    S, NW, RP = np.asarray(S, F), np.asarray(NW, F), np.asarray(RP, F)
    Q = np.zeros(nq * D, F) if Q is None else np.asarray(Q, F).copy()
    KC = np.zeros(max(1, nkv * kv_len * D), np.uint16) if KC is None else np.asarray(KC, np.uint16).copy()
    VC = np.zeros(max(1, nkv * kv_len * D), np.uint16) if VC is None else np.asarray(VC, np.uint16).copy()
    eps, half = F(eps), D // 2
    d = np.arange(half)
    for h in range(nq + (2 * nkv if hasKV else 0)):
        base = h * D
        hv = _split_sum(S, nsrc, ldp, base + np.arange(D))
        rs = _inverse_sqrt(_strided_sumsq(hv, D) / F(D) + eps)
        isv = h >= nq + nkv
        kvh = h - nq - nkv if isv else h - nq
        cb = (kvh * kv_len + kv_row) * D
        if isv:
            VC[cb:cb + D] = (hv * rs).astype(np.float16).view(np.uint16)
            continue
        wo = qw if h < nq else kw
        a = (hv[:half] * rs) * NW[wo + d]
        b = (hv[half:] * rs) * NW[wo + half + d]
        c, sn = np.ones(half, F), np.zeros(half, F)
        rb = rope_off + (pos * npairs + d[:npairs]) * 2
        c[:npairs], sn[:npairs] = RP[rb], RP[rb + 1]
        lo, hi = (a * c) - (b * sn), (b * c) + (a * sn)
        if h < nq:
            Q[base:base + half], Q[base + half:base + D] = lo, hi
        else:
            KC[cb:cb + half], KC[cb + half:cb + D] = lo.astype(np.float16).view(np.uint16), hi.astype(np.float16).view(np.uint16)
    return Q, KC, VC


def attn_dec(Q, KC, VC, D, nh, nkv, kv_len, k_start, k_end, ring=0):
    """lops.js:236-302 (ATTDEC, one workgroup per 64-key chunk) and ATTCOMB: per chunk c and head h, the scores
    s = sum over d of dot(f32(K[4d .. 4d+3]), Q[h][4d ..]) (from 0.0; K of the head's KV group h / (nh / nkv), row
    j or j % ring), m = max over the chunk's keys (from -3e38), p = exp(s - m), l = sum p (from 0.0), acc[h][d] = sum
    over keys of p * f32(V) (from 0.0); the combine: M = max_c m_c, w_c = exp(m_c - M), L = sum_c w_c * l_c, w_c /= L,
    O[h][d] = sum_c w_c * acc_c[h][d] (from 0.0). exp is the C library's expf. Returns O f32 [nh][D]."""
    Qv = np.asarray(Q, F).reshape(nh, D)
    K = _h(KC).reshape(nkv, kv_len, D)
    V = _h(VC).reshape(nkv, kv_len, D)
    hpg = nh // nkv
    nchunk = -(-(k_end - k_start) // 64)
    ms, ls, accs = [], [], []
    for ch in range(nchunk):
        j0 = k_start + ch * 64
        nk = min(64, k_end - j0)
        rows = np.array([(j0 + j) % ring if ring > 0 else j0 + j for j in range(nk)])
        sc = np.zeros((nh, nk), F)
        for hh in range(nh):
            kr = K[hh // hpg, rows]                                     # [nk, D]
            s = np.zeros(nk, F)
            for d4 in range(D // 4):
                s = s + dot4(kr[:, 4 * d4:4 * d4 + 4], np.broadcast_to(Qv[hh, 4 * d4:4 * d4 + 4], (nk, 4)))
            sc[hh] = s
        m = np.full(nh, F(-3.0e38), F)
        for k in range(nk):
            m = np.maximum(m, sc[:, k])
        p = expf(sc - m[:, None])
        l = np.zeros(nh, F)
        for k in range(nk):
            l = l + p[:, k]
        acc = np.zeros((nh, D), F)
        for k in range(nk):
            for hh in range(nh):
                acc[hh] = acc[hh] + p[hh, k] * V[hh // hpg, rows[k]]
        ms.append(m), ls.append(l), accs.append(acc)
    O = np.zeros((nh, D), F)
    for h in range(nh):
        Mx = F(-3.0e38)
        for ch in range(nchunk):
            Mx = max(Mx, ms[ch][h])
        wts, L = [], F(0.0)
        for ch in range(nchunk):
            e = expf(np.array([ms[ch][h] - Mx], F))[0]
            wts.append(e)
            L = F(L + F(e * ls[ch][h]))
        wts = [F(w / L) for w in wts]
        o = np.zeros(D, F)
        for ch in range(nchunk):
            o = o + wts[ch] * accs[ch][h]
        O[h] = o
    return O.ravel()


def embed(Wbytes, ids, K, *, enc="q4g32a.t64", scale=1.0, eps=1e-6, st_off=0, row_out=0, X=None, ST=None):
    """lops.js:324-347 (EMBED): row id of the table (tile id >> 6, row id & 63), v = ((q * s) + mn) * scale (q4) or
    (q * s) * scale (q8, q the sign-extended byte, s the row's fp16 scale); ST[statOff + m] = inverseSqrt(sumsq(v) /
    K + eps) with the 256-thread strided sums and the workgroup tree. Returns (X, ST) as new arrays."""
    W = words(Wbytes)
    ids = np.asarray(ids, np.uint32)
    n = ids.size
    X = np.zeros((row_out + n) * K, F) if X is None else np.asarray(X, F).copy()
    ST = np.zeros(st_off + n, F) if ST is None else np.asarray(ST, F).copy()
    q8 = enc == "q8g64s.t64"
    wG = K // (64 if q8 else 32)
    k = np.arange(K)
    scale, eps = F(scale), F(eps)
    for m in range(n):
        tile, r = int(ids[m]) >> 6, int(ids[m]) & 63
        if q8:
            rec = (tile * wG + (k >> 6)) * 1056
            kk = k & 63
            qb = ((W[rec + r * 16 + (kk >> 2)] >> (8 * (kk & 3))) & 255).astype(np.uint32)
            qs = ((qb << 24).astype(np.uint32).view(np.int32) >> 24).astype(F)
            s2x, s2y = unpack2x16float(W[rec + 1024 + (r >> 1)])
            v = (qs * (s2y if r & 1 else s2x)) * scale
        else:
            rec = (tile * wG + (k >> 5)) * 320
            kk = k & 31
            q = ((W[rec + r * 4 + (kk >> 3)] >> (4 * (kk & 7))) & 15).astype(F)
            s, mn = unpack2x16float(W[rec + 256 + r])
            v = ((q * s) + mn) * scale
        X[(row_out + m) * K:(row_out + m + 1) * K] = v
        ST[st_off + m] = _inverse_sqrt(_strided_sumsq(v.astype(F), K) / F(K) + eps)
    return X, ST


def dhead(Wbytes, X, ST, NW, SEL, K, tPer, nsel, *, enc="q4g32a.t64", stat_off=0, norm_off=0):
    """lops_spec.js:428-473 (DHEAD): for selected tile wt (SEL[wt / tPer] * tPer + wt % tPer), xs = (X * rs) * NW[nOff + k];
    row r's four k-quarter lanes w accumulate over the groups in order, q4: acc + s * (dot(qa, a) + dot(qb, b)) + mn *
    (sum(a) + sum(b)) with a, b the lane's 8 x and qa, qb its 8 codes; q8: acc + s * d, d = sum over the lane's four
    code words of dot(codes, x); the row's total ((w0 + w1) + w2) + w3; the tile's max with the lowest row on ties.
    Returns MX f32 [nsel * tPer][max, bitcast row]."""
    W = words(Wbytes)
    q8 = enc == "q8g64s.t64"
    wG = K // (64 if q8 else 32)
    xs = (np.asarray(X, F)[:K] * F(np.asarray(ST, F)[stat_off])) * np.asarray(NW, F)[norm_off + np.arange(K)]
    SEL = np.asarray(SEL, np.uint32)
    MX = np.empty(2 * nsel * tPer, F)
    one = np.ones(4, F)
    for wt in range(nsel * tPer):
        tile = int(SEL[wt // tPer]) * tPer + wt % tPer
        tot = np.zeros(64, F)
        for r in range(64):
            lanes = []
            for w in range(4):
                acc = F(0.0)
                for g in range(wG):
                    if q8:
                        rec = (tile * wG + g) * 1056
                        s2x, s2y = unpack2x16float(W[rec + 1024 + (r >> 1)])
                        sc = s2y if r & 1 else s2x
                        d = F(0.0)
                        for u in range(4):
                            q = np.uint32(W[rec + r * 16 + w * 4 + u])
                            qv = np.array([(np.uint32(q << sh) & 0xFFFFFFFF) for sh in (24, 16, 8, 0)], np.uint32).view(np.int32) >> 24
                            xb = g * 64 + w * 16 + u * 4
                            d = F(d + dot4(qv.astype(F), xs[xb:xb + 4]))
                        acc = F(acc + F(sc * d))
                    else:
                        rec = (tile * wG + g) * 320
                        q = np.uint32(W[rec + r * 4 + w])
                        s, mn = unpack2x16float(W[rec + 256 + r])
                        xb = g * 32 + w * 8
                        a, b = xs[xb:xb + 4], xs[xb + 4:xb + 8]
                        qa = ((q >> np.array([0, 4, 8, 12], np.uint32)) & 15).astype(F)
                        qb = ((q >> np.array([16, 20, 24, 28], np.uint32)) & 15).astype(F)
                        acc = F(F(acc + F(s * F(dot4(qa, a) + dot4(qb, b)))) + F(mn * F(dot4(a, one) + dot4(b, one))))
                lanes.append(acc)
            tot[r] = F(F(F(lanes[0] + lanes[1]) + lanes[2]) + lanes[3])
        r = int(np.argmax(tot))   # the first of equal maxima: the lowest row
        MX[2 * wt] = tot[r]
        MX[2 * wt + 1] = np.uint32(tile * 64 + r).view(F)
    return MX
