"""The weight-pack store (engine/core/store.js WeightStore) over a local pack directory: a `pocketflux.pack` v1
manifest, per-chunk SHA-256 verification, one device buffer per shard filled straight from the shard file, and the
tensor views the operators take ({buf, off, bytes, enc, shape, rows, cols}, store.js:249-253).

Where the reference downloads into the browser's private file system (OPFS) and keeps a per-chunk bitmap of verified
chunks, this store reads the pack from a directory on local disk and keeps the same bitmap in memory, filled by
`verify()`. Uploads go through the library's native file reader (Gpu.upload_file: 16 MiB chunks, two pinned staging
buffers, disk reads overlapping the PCIe copies). The buffer-reuse rule of `release` / `_reuse` is the reference's: the
last released shard buffer is kept and reused by the next upload of the same size, any other upload frees it first.

`write_pack` builds a pack directory (shards of 256-byte aligned tensors, manifest with chunk hashes) from arrays, for
tests and synthetic benchmarks; the reference's packers (tools/*_pack.py) write the same format.
"""
import hashlib
import json
import os

import numpy as np

FORMAT, FORMAT_VERSION = "pocketflux.pack", 1
CHUNK = 16 * 1024 * 1024   # chunk_bytes of the reference's packers and its download unit
ALIGN = 256                # tensor alignment inside a shard


def _sha(b):
    return hashlib.sha256(b).hexdigest()


def _h2f(u16):
    return np.asarray(u16, np.uint16).view(np.float16).astype(np.float32)


class ShardHandle:
    """an uploaded shard: its device buffer and views of its tensors (store.js:246-253)"""

    def __init__(self, store, name, buf, nbytes):
        self.store, self.name, self.buf, self.bytes = store, name, buf, nbytes

    def t(self, tn):
        x = self.store.m["tensors"].get(tn)
        if not x or x["shard"] != self.name:
            raise KeyError("tensor %s not in %s" % (tn, self.name))
        shape = list(x["shape"])
        return {"buf": self.buf, "off": x["offset"], "bytes": x["bytes"], "enc": x["enc"], "shape": shape, "rows": shape[0],
                "cols": shape[-1]}


class PartHandle:
    """a few tensors of a shard in their own small buffer (store.js:208-220)"""

    def __init__(self, name, buf, nbytes, views):
        self.name, self.buf, self.bytes, self._views = name, buf, nbytes, views

    def t(self, tn):
        if tn not in self._views:
            raise KeyError("tensor %s not in part" % tn)
        return self._views[tn]


class WeightStore:
    """WeightStore(gpu, base): base = the pack directory (manifest.json lives there)."""

    def __init__(self, gpu, base):
        self.gpu, self.base = gpu, base
        self.m, self.shards = None, {}
        self.verified = {}          # shard name -> list of booleans, one per chunk
        self.gpool = []
        self.stats = {"uploadBytes": 0, "uploadMs": 0.0}

    # ------------------------------------------------------------------ manifest and verification
    def open(self):
        path = os.path.join(self.base, "manifest.json")
        if not os.path.exists(path):
            raise FileNotFoundError("pack manifest unavailable (%s)" % path)
        with open(path, "rb") as f:
            m = json.loads(f.read().decode("utf-8"))
        if m.get("format") != FORMAT or m.get("format_version") != FORMAT_VERSION:
            raise ValueError("unsupported pack format %s/%s" % (m.get("format"), m.get("format_version")))
        self.m = m
        self.shards = {s["name"]: s for s in m["shards"]}
        self.verified = {s["name"]: [False] * len(s["chunk_sha256"]) for s in m["shards"]}
        return m

    def _path(self, s):
        return os.path.join(self.base, s["file"])

    def verify(self, names=None, on_progress=None):
        """check every chunk of the named shards (default: all) against the manifest's chunk_sha256; a shard whose file is
        missing or of the wrong size has no good chunk. Returns status()."""
        done, total = 0, sum(self.shards[n]["bytes"] for n in (names or self.shards))
        for name in names or list(self.shards):
            s = self.shards[name]
            bits = [False] * len(s["chunk_sha256"])
            p = self._path(s)
            if os.path.exists(p) and os.path.getsize(p) == s["bytes"]:
                with open(p, "rb") as f:
                    for i, want in enumerate(s["chunk_sha256"]):
                        data = f.read(s["chunk_bytes"])
                        bits[i] = _sha(data) == want
                        done += len(data)
                        if on_progress:
                            on_progress({"have": done, "total": total, "shard": name})
            self.verified[name] = bits
        return self.status()

    def status(self):
        """{have, total, missing, complete} over the verified chunks (store.js:108-118)"""
        have = total = 0
        missing = []
        for s in self.m["shards"]:
            total += s["bytes"]
            bits = self.verified.get(s["name"], [])
            for i, ok in enumerate(bits):
                if ok:
                    have += min(s["chunk_bytes"], s["bytes"] - i * s["chunk_bytes"])
            if not bits or not all(bits):
                missing.append(s["name"])
        return {"have": have, "total": total, "missing": missing, "complete": not missing}

    # ------------------------------------------------------------------ device upload: one buffer per shard
    def upload(self, shard_name):
        """the shard's bytes in a device buffer (a kept buffer of the same size is reused) -> ShardHandle"""
        import time
        s = self.shards.get(shard_name)
        if s is None:
            raise KeyError("unknown shard " + str(shard_name))
        t0 = time.perf_counter()
        buf = self._reuse(s["bytes"]) or self.gpu.buffer(s["bytes"], "shard " + shard_name)
        self.gpu.upload_file(buf, self._path(s), 0, s["bytes"])
        self.stats["uploadBytes"] += s["bytes"]
        self.stats["uploadMs"] += (time.perf_counter() - t0) * 1e3
        return ShardHandle(self, shard_name, buf, s["bytes"])

    def uploadPart(self, shard_name, names):
        """a few tensors of a shard in a NEW buffer, each at a 256-byte aligned offset (store.js:208-220)"""
        s = self.shards.get(shard_name)
        if s is None:
            raise KeyError("unknown shard " + str(shard_name))
        T, lay, tot = self.m["tensors"], [], 0
        for n in names:
            x = T[n]
            lay.append((n, x, tot))
            tot += -(-x["bytes"] // ALIGN) * ALIGN
        buf = self.gpu.buffer(tot, "part " + shard_name)
        for n, x, o in lay:
            self.gpu.upload_file(buf, self._path(s), x["offset"], x["bytes"], dst_off=o)
        views = {n: {"buf": buf, "off": o, "bytes": x["bytes"], "enc": x["enc"], "shape": list(x["shape"]), "rows": x["shape"][0],
                     "cols": x["shape"][-1]} for n, x, o in lay}
        return PartHandle(shard_name + "(part)", buf, tot, views)

    def release(self, h):
        """keep the released shard's buffer for the next upload of the same size; free any kept before (store.js:254-262)"""
        if h is None or h.buf is None:
            return
        b, h.buf = h.buf, None
        if b not in self.gpu.bufs:
            return
        for x in self.gpool:
            self.gpu.free(x)
        self.gpool = [b]

    def _reuse(self, nbytes):
        size = max(16, -(-int(nbytes) // 16) * 16)
        pool, self.gpool = self.gpool, []
        hit = None
        for b in pool:
            if hit is None and b.size == size and b in self.gpu.bufs:
                hit = b
            else:
                self.gpu.free(b)
        if hit is not None:
            self.gpu.done()   # work that still reads the old contents finishes before the new copies
        return hit

    def drainPool(self):
        for b in self.gpool:
            self.gpu.free(b)
        self.gpool = []

    # ------------------------------------------------------------------ host reads
    def readFile(self, shard_name):
        s = self.shards[shard_name]
        with open(self._path(s), "rb") as f:
            return f.read(s["bytes"])

    def readRows(self, tensor_name, ids):
        """gather and dequantise rows of a *.rows tensor -> float32 [len(ids), K] (store.js:270-301): q4g32a.rows rows are
        K/2 code bytes (low nibble first) then K/32 (fp16 s, fp16 mn) pairs, value q*s + mn; q8g64s.rows rows are K int8
        codes then K/64 fp16 scales, value q*s"""
        x = self.m["tensors"][tensor_name]
        s = self.shards[x["shard"]]
        K = x["shape"][1]
        q4 = x["enc"] == "q4g32a.rows"
        if not q4 and x["enc"] != "q8g64s.rows":
            raise ValueError("readRows: " + x["enc"])
        rb = K // 2 + (K // 32) * 4 if q4 else K + (K // 64) * 2
        out = np.empty((len(ids), K), np.float32)
        with open(self._path(s), "rb") as f:
            for i, r in enumerate(ids):
                f.seek(x["offset"] + int(r) * rb)
                row = np.frombuffer(f.read(rb), np.uint8)
                if q4:
                    codes = np.stack([row[:K // 2] & 15, row[:K // 2] >> 4], 1).reshape(K // 32, 32).astype(np.float32)
                    sm = _h2f(row[K // 2:].view(np.uint16).reshape(K // 32, 2))
                    out[i] = (codes * sm[:, :1] + sm[:, 1:]).ravel()
                else:
                    codes = row[:K].view(np.int8).reshape(K // 64, 64).astype(np.float32)
                    out[i] = (codes * _h2f(row[K:].view(np.uint16))[:, None]).ravel()
        return out


def write_pack(out_dir, shards, *, pack_id="synthetic", pack_version="1", model=None, chunk_bytes=CHUNK):
    """write a pocketflux.pack v1 directory: shards = {shard name: [(tensor name, enc, shape, bytes), ...]}; tensors at
    256-byte aligned offsets, tensor names f"{shard}/{name}"; returns the manifest"""
    os.makedirs(out_dir, exist_ok=True)
    tensors, man_shards = {}, []
    for name, parts in shards.items():
        buf = bytearray()
        for tn, enc, shape, b in parts:
            tensors["%s/%s" % (name, tn)] = {"offset": len(buf), "bytes": len(b), "shape": list(shape), "enc": enc, "layout": "rowmajor",
                                            "shard": name}
            buf += bytes(b)
            buf += bytes((-len(buf)) % ALIGN)
        data = bytes(buf)
        fn = name + ".pfw"
        with open(os.path.join(out_dir, fn), "wb") as f:
            f.write(data)
        man_shards.append({"name": name, "file": fn, "kind": "weights", "bytes": len(data), "sha256": _sha(data), "chunk_bytes": chunk_bytes,
                           "chunk_sha256": [_sha(data[i:i + chunk_bytes]) for i in range(0, len(data), chunk_bytes)]})
    m = {"format": FORMAT, "format_version": FORMAT_VERSION, "pack_id": pack_id, "pack_version": pack_version, "model": model or {},
         "shards": man_shards, "tensors": tensors}
    with open(os.path.join(out_dir, "manifest.json"), "w", encoding="utf-8") as f:
        json.dump(m, f, indent=1)
    return m
