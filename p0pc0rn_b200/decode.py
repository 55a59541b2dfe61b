"""One whole decode token of a Gemma-4-style decoder from the library's operators: the reference's encodeStep
(engine/llm/gemma4.js:526-537) without its per-layer-embedding (PLE) path.

  embed (lops.js:323-365)                      x = E[token] * scale, st = rstd(x)
  per layer, _attnPart (gemma4.js:457-478):    gemv rms QKV -> qkrope (q to f32, k / v into the layer's fp16 caches at
                                               the token's row) -> attnDec over keys [kStart, pos] -> gemv O (kPer 2048)
                                               -> normadd (sums the O partials, adds to x, new rstd)
  per layer, _mlpPart (gemma4.js:479-488):     gemv rms GeGLU -> gemv down (kPer 2048) -> normadd
  head, _headWith (gemma4.js:503-511):         rstd copied into the MX buffer's stat slot, gemv rms softcap over the
                                               vocabulary with per-tile max / argmax, argmax

Every step is a CUDA kernel of libp0mm.so (no host arithmetic), enqueued in order on the context's stream; the result
(argmax index, max logit bits) stays on the device in `s["arg"]` until it is read. The rms prologues read the rstd
normadd (or embed) wrote: the reference recomputes the same value with rowstats (ops/misc.js:33-40) before each part.
Sliding layers (kind "sliding") attend over the last `window` positions of a ring cache of `window` rows
(gemma4.js:97-116, 466); full layers over every position.
"""
import numpy as np

from . import ops

KP = 2048   # the O and down projections' k-split (gemma4.js:475, 485)


def model_sizes(cfg):
    """the per-layer matrix shapes of a config {D, layers, NH, NKV, hd, FF, vocab, window, kinds}"""
    D, NH, NKV, hd = cfg["D"], cfg["NH"], cfg["NKV"], cfg["hd"]
    return {"qkv": (NH * hd + 2 * NKV * hd, D), "o": (D, NH * hd), "gu": (2 * cfg["FF"], D), "down": (D, cfg["FF"]), "head": (cfg["vocab"], D)}


class DecodeState:
    """the scratch buffers of one decode stream and the layers' KV caches (kc / vc fp16 [NKV][len][hd])"""

    def __init__(self, g, cfg, max_pos):
        D, NH, NKV, hd, FF, V = cfg["D"], cfg["NH"], cfg["NKV"], cfg["hd"], cfg["FF"], cfg["vocab"]
        self.g, self.cfg = g, cfg
        nqkv = NH * hd + 2 * NKV * hd
        self.b = {
            "x": g.buffer(D * 4, "x"), "st": g.buffer(64, "st"), "qkvp": g.buffer(nqkv * 4, "qkvp"), "q": g.buffer(NH * hd * 4, "q"),
            "ao": g.buffer(NH * hd * 4, "ao"), "apart": g.buffer(256 * NH * (2 + hd) * 4, "apart"),
            "tpart": g.buffer(max(-(-NH * hd // KP), -(-FF // KP)) * D * 4, "tpart"), "mbuf": g.buffer(FF * 4, "mbuf"),
            "logits": g.buffer(V * 4, "logits"), "mx": g.buffer((V // 64 + 1) * 8, "mx"), "arg": g.buffer(16, "arg"),
            "ids": g.buffer(16, "ids"),
        }
        self.caches = []
        for l in range(cfg["layers"]):
            n = cfg["window"] if cfg["kinds"][l] == "sliding" else max_pos
            self.caches.append({"len": n, "ring": n if cfg["kinds"][l] == "sliding" else 0,
                                "kc": g.buffer(NKV * n * hd * 2, "kc"), "vc": g.buffer(NKV * n * hd * 2, "vc")})

    def row(self, l, pos):
        c = self.caches[l]
        return pos % c["len"] if c["ring"] else pos


def decode_token(g, m, s, pos, token_buf=None):
    """enqueue one decode token at position pos (gemma4.js encodeStep). m: the model's device buffers
    {embed, layers: [{qkv, o, gu, down, in_norm, qk_norm (q at 0, k at hd), post_attn, pre_ff, post_ff}], final_norm,
    rope: {full, sliding} (f32 (cos, sin) pairs per position and pair)}; s: a DecodeState. The token id is read from
    token_buf (a device buffer) or s.b["ids"]. Returns the number of kernels enqueued (the stat copy is not one)."""
    cfg = s.cfg
    D, NH, NKV, hd, FF, V = cfg["D"], cfg["NH"], cfg["NKV"], cfg["hd"], cfg["FF"], cfg["vocab"]
    eps, b = cfg.get("eps", 1e-6), s.b
    nq, nqkv = NH * hd, NH * hd + 2 * NKV * hd
    wv = lambda buf, shape: {"buf": buf, "off": 0, "enc": "q4g32a.t64", "rows": shape[0], "cols": shape[1]}
    sz = model_sizes(cfg)
    n = 0
    ops.embed(g, {"w": wv(m["embed"], sz["head"]), "ids": {"buf": token_buf or b["ids"]}, "x": {"buf": b["x"]}, "st": {"buf": b["st"], "off": 1},
                  "K": D, "n": 1, "scale": float(np.float32(cfg["embed_scale"])), "eps": eps})
    n += 1
    for l, L in enumerate(m["layers"]):
        kind, cache = cfg["kinds"][l], s.caches[l]
        npairs = cfg.get("npairs", hd // 2)
        kStart = 0 if kind == "full" else max(0, pos - cfg["window"] + 1)
        # _attnPart
        ops.gemv(g, {"w": wv(L["qkv"], sz["qkv"]), "x": {"buf": b["x"]}, "N": nqkv, "K": D, "pro": "rms", "stat": {"buf": b["st"], "off": 1},
                     "norm": {"buf": L["in_norm"], "off": 0}, "y": {"buf": b["qkvp"]}})
        ops.qkrope(g, {"s": {"buf": b["qkvp"], "n": 1, "ld": nqkv}, "norm": {"buf": L["qk_norm"]}, "qw": 0, "kw": hd,
                       "rope": {"buf": m["rope"][kind], "off": 0}, "q": {"buf": b["q"]}, "kc": {"buf": cache["kc"]}, "vc": {"buf": cache["vc"]},
                       "D": hd, "nq": NH, "hasKV": True, "pos": pos, "npairs": npairs, "kvRow": s.row(l, pos), "nkv": NKV,
                       "kvLen": cache["len"], "eps": eps})
        ops.attnDec(g, {"q": {"buf": b["q"]}, "kc": {"buf": cache["kc"]}, "vc": {"buf": cache["vc"]}, "part": {"buf": b["apart"]},
                        "out": {"buf": b["ao"]}, "D": hd, "nh": NH, "kStart": kStart, "kEnd": pos + 1, "ring": cache["ring"], "nkv": NKV,
                        "kvLen": cache["len"]})
        ns_o = ops.gemv(g, {"w": wv(L["o"], sz["o"]), "x": {"buf": b["ao"]}, "N": D, "K": nq, "kPer": KP, "y": {"buf": b["tpart"]}})
        ops.normadd(g, {"t": {"buf": b["tpart"], "n": ns_o, "ld": D}, "w": {"buf": L["post_attn"], "off": 0}, "x": {"buf": b["x"]},
                        "st": {"buf": b["st"], "off": 1}, "D": D, "eps": eps, "scale": 1.0})
        # _mlpPart
        ops.gemv(g, {"w": wv(L["gu"], sz["gu"]), "x": {"buf": b["x"]}, "N": FF, "K": D, "pro": "rms", "stat": {"buf": b["st"], "off": 1},
                     "norm": {"buf": L["pre_ff"], "off": 0}, "epi": "geglu", "y": {"buf": b["mbuf"]}})
        ns_d = ops.gemv(g, {"w": wv(L["down"], sz["down"]), "x": {"buf": b["mbuf"]}, "N": D, "K": FF, "kPer": KP, "y": {"buf": b["tpart"]}})
        ops.normadd(g, {"t": {"buf": b["tpart"], "n": ns_d, "ld": D}, "w": {"buf": L["post_ff"], "off": 0}, "x": {"buf": b["x"]},
                        "st": {"buf": b["st"], "off": 1}, "D": D, "eps": eps, "scale": 1.0})
        n += 9   # the two gemv projections, qkrope, attnDec's chunk and combine kernels, two gemv MLP calls, two normadds
    # _headWith: the rms prologue of the softcap head reads its rstd from the MX buffer past the tile slots (lops.js:125)
    stoff = V // 64 * 2
    g.copy(b["st"], 4, b["mx"], stoff * 4, 4)
    ops.gemv(g, {"w": wv(m["embed"], sz["head"]), "x": {"buf": b["x"]}, "N": V, "K": D, "pro": "rms", "stat": {"buf": b["mx"], "off": stoff},
                 "norm": {"buf": m["final_norm"], "off": 0}, "epi": "softcap", "cap": cfg.get("softcap", 30.0), "mx": {"buf": b["mx"]},
                 "y": {"buf": b["logits"]}})
    ops.argmax(g, {"mx": {"buf": b["mx"]}, "out": {"buf": b["arg"]}, "n": V // 64})
    return n + 2
