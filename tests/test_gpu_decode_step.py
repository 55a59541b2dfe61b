"""Whole decode tokens (p0pc0rn_b200.decode.decode_token, the reference's encodeStep, gemma4.js:526-537) through the
library's kernels against the same tokens through the CPU oracle: embed -> per layer [rms QKV gemv -> qkrope into the
layer's KV cache -> attnDec -> O gemv (kPer 2048) -> normadd -> rms GeGLU gemv -> down gemv (kPer 2048) -> normadd] ->
rms softcap head with per-tile argmax -> argmax. A small model with full and sliding-window layers decodes a fixed
token sequence (teacher forcing), so the sliding ring cache wraps; each token's logits must match within the parity
tolerance and its argmax must be the oracle's (or a tie within 1e-5, kshipped.js:41-43)."""
import numpy as np
import pytest

import p0pc0rn_b200 as p0
from oracle import ref
from p0pc0rn_b200 import decode

from .test_gpu_parity import assert_close

pytestmark = pytest.mark.gpu

CFG = {"D": 512, "layers": 3, "NH": 4, "NKV": 1, "hd": 128, "FF": 2304, "vocab": 4096, "window": 8,
       "kinds": ["full", "sliding", "full"], "embed_scale": 22.627417, "softcap": 30.0, "eps": 1e-6}
MAXPOS = 32


def rope_table(npos, npairs, seed):
    ang = ref.randn(npos * npairs, seed, 2.0).astype(np.float64)
    rp = np.zeros(2 * npos * npairs, np.float32)
    rp[0::2], rp[1::2] = np.cos(ang), np.sin(ang)
    return rp


def host_model(cfg, seed):
    sz = decode.model_sizes(cfg)
    pk = lambda shape, s, sc: ref.pack_q4(ref.randn(shape[0] * shape[1], s, sc), shape[0], shape[1])[0]
    m = {"embed": pk(sz["head"], seed, 0.05), "final_norm": ref.randn(cfg["D"], seed + 1, 0.1) + 1,
         "rope": {"full": rope_table(MAXPOS, cfg["hd"] // 2, seed + 2), "sliding": rope_table(MAXPOS, cfg["hd"] // 2, seed + 3)}, "layers": []}
    for l in range(cfg["layers"]):
        s0 = seed + 100 * (l + 1)
        m["layers"].append({"qkv": pk(sz["qkv"], s0, 0.02), "o": pk(sz["o"], s0 + 1, 0.02), "gu": pk(sz["gu"], s0 + 2, 0.02),
                            "down": pk(sz["down"], s0 + 3, 0.02), "in_norm": ref.randn(cfg["D"], s0 + 4, 0.1) + 1,
                            "qk_norm": ref.randn(2 * cfg["hd"], s0 + 5, 0.1) + 1, "post_attn": ref.randn(cfg["D"], s0 + 6, 0.1) + 1,
                            "pre_ff": ref.randn(cfg["D"], s0 + 7, 0.1) + 1, "post_ff": ref.randn(cfg["D"], s0 + 8, 0.1) + 1})
    return m


def upload_model(g, h):
    up = g.upload
    return {"embed": up(h["embed"]), "final_norm": up(h["final_norm"]), "rope": {k: up(v) for k, v in h["rope"].items()},
            "layers": [{k: up(v) for k, v in L.items()} for L in h["layers"]]}


class OracleDecoder:
    """the same step through the oracle's restatements, with its own caches"""

    def __init__(self, cfg, h):
        self.cfg, self.h = cfg, h
        self.caches = []
        for kind in cfg["kinds"]:
            n = cfg["window"] if kind == "sliding" else MAXPOS
            self.caches.append({"len": n, "ring": n if kind == "sliding" else 0, "kc": np.zeros(cfg["NKV"] * n * cfg["hd"], np.uint16),
                                "vc": np.zeros(cfg["NKV"] * n * cfg["hd"], np.uint16)})

    def step(self, tok, pos):
        c, h = self.cfg, self.h
        D, NH, NKV, hd, FF, V, eps = c["D"], c["NH"], c["NKV"], c["hd"], c["FF"], c["vocab"], c["eps"]
        nq, nqkv = NH * hd, NH * hd + 2 * NKV * hd
        x, st = ref.embed(h["embed"], np.array([tok], np.uint32), D, scale=float(np.float32(c["embed_scale"])), eps=eps, st_off=1)
        for l, L in enumerate(h["layers"]):
            cache, kind = self.caches[l], c["kinds"][l]
            row = pos % cache["len"] if cache["ring"] else pos
            qkv, _, _ = ref.gemv(L["qkv"], x, nqkv, D, pro="rms", norm=L["in_norm"], stat_buf=st, stat_off=1)
            Q, _, _ = ref.qkrope(qkv, 1, nqkv, L["qk_norm"], h["rope"][kind], hd, NH, nkv=NKV, pos=pos, eps=eps, qw=0, kw=hd,
                                 npairs=hd // 2, kv_row=row, kv_len=cache["len"], KC=cache["kc"], VC=cache["vc"])
            k0 = 0 if kind == "full" else max(0, pos - c["window"] + 1)
            ao = ref.attn_dec(Q, cache["kc"], cache["vc"], hd, NH, NKV, cache["len"], k0, pos + 1, cache["ring"])
            t, _, ns = ref.gemv(L["o"], ao, D, nq, kPer=decode.KP)
            ref.normadd(t, ns, D, L["post_attn"], 0, x, st, 1, D, 1, eps=eps, scale=1.0)
            mb, _, _ = ref.gemv(L["gu"], x, FF, D, pro="rms", epi="geglu", norm=L["pre_ff"], stat_buf=st, stat_off=1)
            t, _, ns = ref.gemv(L["down"], mb, D, FF, kPer=decode.KP)
            ref.normadd(t, ns, D, L["post_ff"], 0, x, st, 1, D, 1, eps=eps, scale=1.0)
        mx = np.zeros(V // 64 * 2 + 2, np.float32)
        mx[V // 64 * 2] = st[1]
        logits, mx, _ = ref.gemv(h["embed"], x, V, D, pro="rms", epi="softcap", norm=h["final_norm"], stat_off=V // 64 * 2, mx=mx,
                                 cap=c["softcap"])
        return logits, ref.argmaxM(mx[:V // 64 * 2], V // 64, 1), x


def test_decode_tokens_match_oracle(g):
    h = host_model(CFG, 900)
    m = upload_model(g, h)
    s = decode.DecodeState(g, CFG, MAXPOS)
    ora = OracleDecoder(CFG, h)
    toks = [7, 1033, 2048, 5, 4095, 300, 301, 302, 77, 1, 2, 3]          # 12 positions: the window-8 ring wraps
    V = CFG["vocab"]
    for pos, tok in enumerate(toks):
        g.write(s.b["ids"], np.array([tok, 0, 0, 0], np.uint32))
        n = decode.decode_token(g, m, s, pos)
        assert n == 1 + 9 * CFG["layers"] + 2
        g.done()
        logits = g.read(s.b["logits"], 0, V * 4, np.float32)
        arg = g.read(s.b["arg"], 0, 8, np.uint32)
        x = g.read(s.b["x"], 0, CFG["D"] * 4, np.float32)
        want_logits, want_arg, want_x = ora.step(tok, pos)
        assert_close(x, want_x)
        assert_close(logits, want_logits)
        if arg[0] != want_arg[0]:
            assert abs(float(want_logits[arg[0]]) - float(want_logits[want_arg[0]])) <= 1e-5, (pos, arg, want_arg)
        # the device kept the reference's result layout: index, then the bits of the max logit
        assert abs(arg[1:2].view(np.float32)[0] - logits[arg[0]]) == 0.0
