"""Generates the committed fixtures in this folder from the CPU oracle (oracle/oracle.c).

The reference (JavaScript + WGSL) stores no golden vectors and cannot run in this environment, so these fixtures
are oracle outputs on seeded inputs made by the reference's own generator (kcheck.js rng/randn, packQ4). They pin
the oracle against regressions (tests/test_oracle.py) and give the GPU tests fixed vectors to meet.

    python -m tests.golden.make_golden      # rewrites *.bin and manifest.json
"""
import json
import os

import numpy as np

from oracle import ref

HERE = os.path.dirname(os.path.abspath(__file__))


def _x16(n, seed):
    return ref.round_f16(ref.randn(n, seed))


def case_pack():
    b, deq = ref.pack_q4(ref.randn(64 * 256, 11, 0.05), 64, 256)
    return {"bytes": b, "deq16": ref.deq16(b, 64, 256).ravel()}


def case_gemv_raw():
    N, K = 256, 2048
    b, _ = ref.pack_q4(ref.randn(N * K, 0, 0.02), N, K)
    y, _, _ = ref.gemv(b, _x16(K, 1), N, K)
    return {"y": y}


def case_gemv_rms_softcap():
    N, K = 128, 1536
    b, _ = ref.pack_q4(ref.randn(N * K, 33 + K, 0.05), N, K)
    x = ref.randn(K, 34 + K)
    nw = np.array([0.9 + 0.2 * ((i * 7919) % 100) / 100 for i in range(K)], np.float32)
    mx = np.zeros(N // 64 * 2 + 4, np.float32)
    mx[N // 64 * 2] = 0.75
    y, MX, _ = ref.gemv(b, x, N, K, pro="rms", epi="softcap", norm=nw, stat_off=N // 64 * 2, mx=mx, cap=30.0)
    return {"y": y, "mx": MX}


def case_gemv_geglu():
    N, K = 128, 512
    b, _ = ref.pack_q4(ref.randn(2 * N * K, 5, 0.05), 2 * N, K)
    st = np.array([0, 1.25, 0, 0], np.float32)
    nw = ref.randn(K, 6, 0.1) + 1
    y, _, _ = ref.gemv(b, ref.randn(K, 7), N, K, pro="rms", epi="geglu", norm=nw, stat_buf=st, stat_off=1)
    return {"y": y}


def case_gemvM_split():
    M, N, K = 4, 128, 2048
    b, _ = ref.pack_q4(ref.randn(N * K, 8, 0.02), N, K)
    Y, _, ns = ref.gemvM(b, ref.randn(M * K, 9), M, N, K, kPer=512)
    assert ns == 4
    return {"y": Y}


def case_gemm_f16():
    M, N, K = 32, 128, 256
    b, _ = ref.pack_q4(ref.randn(N * K, 11, 0.05), N, K)
    return {"y": ref.gemm(b, ref.f2h(_x16(M * K, 7)), M, N, K)}


def case_gemm_bias_gelu():
    M, N, K = 48, 128, 320
    b, _ = ref.pack_q4(ref.randn(N * K, 12, 0.02), N, K)
    bias = ref.randn(N, 13, 0.01)
    return {"y": ref.gemm(b, ref.f2h(_x16(M * K, 14)), M, N, K, epi="bias", ev=bias, post_gelu=True)}


def case_gemm_swiglu():
    M, N, K = 40, 256, 256
    b, _ = ref.pack_q4(ref.randn(N * K, 15, 0.02), N, K)
    bv = ref.randn(N, 16, 0.01)
    return {"y": ref.gemm(b, ref.f2h(_x16(M * K, 17)), M, N, K, epi="swiglu", act="gelu", wr0=0, wr1=N // 2, bv=bv, bv_up=N // 2,
                          ldy=N // 2)}


def cases():
    return {"pack": case_pack, "gemv_raw": case_gemv_raw, "gemv_rms_softcap": case_gemv_rms_softcap, "gemv_geglu": case_gemv_geglu,
            "gemvM_split": case_gemvM_split, "gemm_f16": case_gemm_f16, "gemm_bias_gelu": case_gemm_bias_gelu,
            "gemm_swiglu": case_gemm_swiglu}


def main():
    man = {}
    for name, fn in cases().items():
        man[name] = {}
        for k, arr in fn().items():
            a = np.ascontiguousarray(arr).ravel()
            fname = "%s.%s.bin" % (name, k)
            a.tofile(os.path.join(HERE, fname))
            man[name][k] = {"file": fname, "dtype": str(a.dtype), "n": int(a.size)}
    with open(os.path.join(HERE, "manifest.json"), "w") as f:
        json.dump(man, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
