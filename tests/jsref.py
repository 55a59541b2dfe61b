"""A second, independent transcription of the reference's JS helpers in plain Python (no C), used to pin the C oracle:
rng / randn (engine/kcheck.js:10-11), f2h / h2f (engine/core/gpu.js:274-295), rhe (kcheck.js:14), packQ4
(kcheck.js:22-38), packQ8 (kcheck.js:39-52). JS numbers are f64; Float32Array stores round to f32 (struct pack 'f'); `>>` is JS's signed shift
of the int32 view. Slow: small sizes only.
"""
import math
import struct


def _i32(x):
    x &= 0xFFFFFFFF
    return x - (1 << 32) if x & 0x80000000 else x


def _u32(x):
    return x & 0xFFFFFFFF


def rng(seed):
    s = _u32(seed) or 1
    state = [s]

    def nxt():
        s = state[0]
        s = _i32(s) ^ _i32(_i32(s) << 13)        # s ^= s << 13 (int32 result)
        s = _u32(s)                              # s >>>= 0
        s = _i32(s) ^ (_i32(s) >> 17)            # s ^= s >> 17 (arithmetic shift of the int32 view)
        s = _i32(s) ^ _i32(_i32(s) << 5)         # s ^= s << 5
        s = _u32(s)                              # s >>>= 0
        state[0] = s
        return s / 4294967296
    return nxt


def f32(v):
    return struct.unpack("<f", struct.pack("<f", v))[0]


def randn(n, seed, scale=1.0):
    r = rng(seed)
    o = [0.0] * n
    for i in range(0, n, 2):
        u = max(1e-9, r())
        v = r()
        m = math.sqrt(-2 * math.log(u)) * scale
        o[i] = f32(m * math.cos(2 * math.pi * v))
        if i + 1 < n:
            o[i + 1] = f32(m * math.sin(2 * math.pi * v))
    return o


def f2h(v):
    x = struct.unpack("<I", struct.pack("<f", v))[0]
    sign = (x >> 16) & 0x8000
    e = (x >> 23) & 0xFF
    m = x & 0x7FFFFF
    if e == 0xFF:
        return sign | 0x7C00 | (0x200 if m else 0)
    ne = e - 112
    if ne >= 0x1F:
        return sign | 0x7C00
    if ne <= 0:
        if ne < -10:
            return sign
        m |= 0x800000
        sh = 14 - ne
        hm = m >> sh
        rem = m & ((1 << sh) - 1)
        half = 1 << (sh - 1)
        if rem > half or (rem == half and (hm & 1)):
            hm += 1
        return sign | hm
    r = sign | (ne << 10) | (m >> 13)
    rem2 = m & 0x1FFF
    if rem2 > 0x1000 or (rem2 == 0x1000 and (r & 1)):
        r += 1
    return r


def h2f(h):
    s = -1 if (h & 0x8000) else 1
    e = (h >> 10) & 0x1F
    m = h & 0x3FF
    if e == 0:
        return s * m * 5.960464477539063e-8
    if e == 31:
        return float("nan") if m else s * float("inf")
    return s * (1 + m / 1024) * math.pow(2, e - 15)


def rf16(x):
    return h2f(f2h(x))


def rhe(x):
    f = math.floor(x)
    d = x - f
    return f + 1 if d > 0.5 else f if d < 0.5 else (f if f % 2 == 0 else f + 1)


def pack_q4(W, N, K):
    NT, G = N // 64, K // 32
    out = bytearray(NT * G * 1280)
    deq = [0.0] * (N * K)
    for t in range(NT):
        for g in range(G):
            rec = (t * G + g) * 1280
            for r in range(64):
                n = t * 64 + r
                base = n * K + g * 32
                mnv, mxv = math.inf, -math.inf
                for i in range(32):
                    v = W[base + i]
                    if v < mnv:
                        mnv = v
                    if v > mxv:
                        mxv = v
                mn = rf16(mnv)
                s = rf16((mxv - mn) / 15)
                if s == 0:
                    s = 1
                for j in range(16):
                    q0 = min(15, max(0, rhe((W[base + 2 * j] - mn) / s)))
                    q1 = min(15, max(0, rhe((W[base + 2 * j + 1] - mn) / s)))
                    out[rec + r * 16 + j] = int(q0) | (int(q1) << 4)
                    deq[base + 2 * j] = f32(q0 * s + mn)
                    deq[base + 2 * j + 1] = f32(q1 * s + mn)
                word = (f2h(s) | (f2h(mn) << 16)) & 0xFFFFFFFF
                out[rec + 1024 + r * 4: rec + 1028 + r * 4] = struct.pack("<I", word)
    return bytes(out), deq


def pack_q8(W, N, K):
    NT, G = N // 64, K // 64
    out = bytearray(NT * G * 4224)
    deq = [0.0] * (N * K)
    for t in range(NT):
        for g in range(G):
            rec = (t * G + g) * 4224
            for r in range(64):
                n = t * 64 + r
                base = n * K + g * 64
                am = 0.0
                for i in range(64):
                    am = max(am, abs(W[base + i]))
                s = rf16(am / 127)
                if s == 0:
                    s = 1
                for i in range(64):
                    q = int(min(127, max(-128, rhe(W[base + i] / s))))
                    out[rec + r * 64 + i] = q & 255
                    deq[base + i] = f32(q * s)
                out[rec + 4096 + r * 2: rec + 4098 + r * 2] = struct.pack("<H", f2h(s))
    return bytes(out), deq
