"""The weight-pack store on CPU (engine/core/store.js): manifest checks, chunk verification, shard upload and buffer
reuse, part uploads and tensor views, through a stand-in for the device that copies the file bytes the native reader
would copy; readRows' dequantisation against an independent statement of the row formats."""
import json
import os

import numpy as np
import pytest

from p0pc0rn_b200 import store
from oracle import ref


class FakeBuf:
    def __init__(self, size, label):
        self.size, self.label, self.data = max(16, -(-size // 16) * 16), label, bytearray(max(16, -(-size // 16) * 16))


class FakeGpu:
    """the device calls the store makes, on host memory"""

    def __init__(self):
        self.bufs, self.allocs, self.freed = set(), 0, 0

    def buffer(self, size, label=""):
        b = FakeBuf(size, label)
        self.bufs.add(b)
        self.allocs += 1
        return b

    def upload_file(self, b, path, file_off=0, nbytes=None, dst_off=0):
        with open(path, "rb") as f:
            f.seek(file_off)
            data = f.read(nbytes)
        assert len(data) == nbytes and dst_off + nbytes <= b.size
        b.data[dst_off:dst_off + nbytes] = data
        return b

    def free(self, b):
        if b in self.bufs:
            self.bufs.discard(b)
            self.freed += 1

    def done(self, timeout_ms=0):
        pass


def q4_rows(W, V, K):
    """q4g32a.rows: per row K/2 code bytes (low nibble = even k) then K/32 (fp16 s, fp16 mn), packQ4's quantisation"""
    b, _ = ref.pack_q4(W, V, K)
    raw = np.frombuffer(np.asarray(b, np.uint8).tobytes(), np.uint8)
    out = bytearray()
    for n in range(V):
        t, r = n // 64, n % 64
        codes, sm = bytearray(), bytearray()
        for g in range(K // 32):
            rec = raw[(t * (K // 32) + g) * 1280:(t * (K // 32) + g + 1) * 1280]
            codes += rec[r * 16:r * 16 + 16].tobytes()
            sm += rec[1024 + 4 * r:1028 + 4 * r].tobytes()
        out += codes + sm
    return bytes(out), b


def q8_rows(W, V, K):
    b, _ = ref.pack_q8(W, V, K)
    raw = np.frombuffer(np.asarray(b, np.uint8).tobytes(), np.uint8)
    out = bytearray()
    for n in range(V):
        t, r = n // 64, n % 64
        codes, sc = bytearray(), bytearray()
        for g in range(K // 64):
            rec = raw[(t * (K // 64) + g) * 4224:(t * (K // 64) + g + 1) * 4224]
            codes += rec[r * 64:r * 64 + 64].tobytes()
            sc += rec[4096 + 2 * r:4098 + 2 * r].tobytes()
        out += codes + sc
    return bytes(out), b


@pytest.fixture
def pack(tmp_path):
    V, K = 128, 128
    W4 = ref.randn(V * K, 1, 0.05)
    rows4, b4 = q4_rows(W4, V, K)
    rows8, b8 = q8_rows(ref.randn(V * K, 2, 0.05), V, K)
    vec = ref.randn(300, 3).tobytes()
    shards = {
        "embed": [("tok.rows", "q4g32a.rows", (V, K), rows4), ("tok8.rows", "q8g64s.rows", (V, K), rows8)],
        "blk0": [("wq", "q4g32a.t64", (V, K), bytes(np.asarray(b4, np.uint8))), ("norm", "f32", (300,), vec)],
        "blk1": [("wq", "q4g32a.t64", (V, K), bytes(np.asarray(b4, np.uint8))), ("norm", "f32", (300,), vec)],
    }
    m = store.write_pack(str(tmp_path), shards, chunk_bytes=4096)
    return str(tmp_path), m, b4, b8


def test_manifest_and_verify(pack):
    base, m, _, _ = pack
    st = store.WeightStore(FakeGpu(), base)
    assert st.open()["format"] == "pocketflux.pack"
    assert st.status()["complete"] is False          # nothing verified yet
    s = st.verify()
    assert s["complete"] and s["have"] == s["total"] == sum(x["bytes"] for x in m["shards"])
    # one flipped byte: that chunk fails, the shard is missing, `have` drops by the chunk
    p = os.path.join(base, "blk1.pfw")
    data = bytearray(open(p, "rb").read())
    data[5000] ^= 1
    open(p, "wb").write(bytes(data))
    s = st.verify(["blk1"])
    assert s["missing"] == ["blk1"] and s["have"] == s["total"] - 4096


def test_bad_format(tmp_path):
    store.write_pack(str(tmp_path), {"a": [("x", "f32", (4,), bytes(16))]})
    mp = os.path.join(str(tmp_path), "manifest.json")
    m = json.load(open(mp))
    m["format_version"] = 2
    json.dump(m, open(mp, "w"))
    with pytest.raises(ValueError, match="unsupported pack format pocketflux.pack/2"):
        store.WeightStore(FakeGpu(), str(tmp_path)).open()


def test_upload_views_and_reuse(pack):
    base, m, b4, _ = pack
    g = FakeGpu()
    st = store.WeightStore(g, base)
    st.open()
    h0 = st.upload("blk0")
    v = h0.t("blk0/wq")
    assert (v["rows"], v["cols"], v["enc"], v["off"]) == (128, 128, "q4g32a.t64", 0)
    assert bytes(h0.buf.data[v["off"]:v["off"] + v["bytes"]]) == bytes(np.asarray(b4, np.uint8))
    n = h0.t("blk0/norm")
    assert n["off"] % 256 == 0 and n["shape"] == [300]
    with pytest.raises(KeyError, match="tensor blk1/wq not in blk0"):
        h0.t("blk1/wq")
    with pytest.raises(KeyError, match="unknown shard"):
        st.upload("nope")
    # equal-size shards: the released buffer is reused (no new allocation); a shard of another size frees it
    buf0 = h0.buf
    st.release(h0)
    h1 = st.upload("blk1")
    assert h1.buf is buf0 and g.allocs == 1
    st.release(h1)
    st.upload("embed")
    assert g.freed == 1 and g.allocs == 2


def test_upload_part(pack):
    base, _, b4, _ = pack
    st = store.WeightStore(FakeGpu(), base)
    st.open()
    part = st.uploadPart("blk0", ["blk0/norm", "blk0/wq"])
    n, w = part.t("blk0/norm"), part.t("blk0/wq")
    assert n["off"] == 0 and w["off"] == 1280          # 300 floats = 1200 bytes, rounded up to 256
    assert bytes(part.buf.data[w["off"]:w["off"] + w["bytes"]]) == bytes(np.asarray(b4, np.uint8))
    with pytest.raises(KeyError):
        part.t("blk0/other")


@pytest.mark.parametrize("name,enc", [("embed/tok.rows", "q4g32a.t64"), ("embed/tok8.rows", "q8g64s.t64")])
def test_read_rows(pack, name, enc):
    base, _, b4, b8 = pack
    st = store.WeightStore(FakeGpu(), base)
    st.open()
    ids = [0, 127, 64, 5, 5]
    got = st.readRows(name, ids)
    # the same rows through the oracle's embed of the tile-layout pack at scale 1 (the same q*s + mn / q*s in f32)
    want, _ = ref.embed(b4 if enc == "q4g32a.t64" else b8, np.array(ids, np.uint32), 128, enc=enc, scale=1.0)
    assert np.array_equal(got.ravel(), want)
