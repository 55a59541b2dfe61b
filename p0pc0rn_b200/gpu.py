"""The device context and buffers: the Python face of engine/core/gpu.js (createGpu :18-23, Gpu.buffer :81-88,
free :89-94, upload :98-117, read/_readback :118-140, done :141-147), backed by the C ABI (include/p0mm.h).

Buffers are opaque handles owned by the context, like WebGPU buffers owned by Gpu. Errors raise P0Error with the
library's message, which keeps the reference's wording (e.g. "gemv: N % 64").
"""
import ctypes
import os

import numpy as np

from . import _lib as L


class P0Error(Exception):
    """A failed library call (the reference throws Error / GpuError at the same points)."""

    def __init__(self, status, msg):
        super().__init__(msg)
        self.status = status
        self.code = L.STATUS.get(status, str(status))


class Buffer:
    """A device buffer handle (the WebGPU GPUBuffer of the reference; `_pf` is its rounded size as in gpu.js:85)."""
    __slots__ = ("gpu", "id", "size", "label", "_pf", "external")

    def __init__(self, gpu, bid, size, label, external=False):
        self.gpu, self.id, self.size, self.label, self._pf, self.external = gpu, bid, size, label, size, external

    @property
    def handle(self):
        return L.p0_buf(self.id)

    @property
    def ptr(self):
        v = ctypes.c_uint64()
        self.gpu._check(self.gpu._lib.p0_device_ptr(self.gpu.ctx, self.handle, ctypes.byref(v)))
        return v.value

    def __repr__(self):
        return "Buffer(%d, %d B, %r)" % (self.id, self.size, self.label)


NONE = L.p0_buf(0)


def handle(b):
    return NONE if b is None else b.handle


class Gpu:
    """One device context. createGpu() in the reference; here Gpu(device)."""

    def __init__(self, device=0):
        self._lib = L.load()
        self.ctx = ctypes.c_void_p()
        st = self._lib.p0_init(int(device), ctypes.byref(self.ctx))
        if st != L.P0_OK:
            raise P0Error(st, "p0_init(%d) failed: %s" % (device, L.STATUS.get(st)))
        self.device = device
        self.bufs = set()

    # -------------------------------------------------------------- plumbing
    def _check(self, st):
        if st != L.P0_OK:
            raise P0Error(st, self.last_error())
        return st

    def last_error(self):
        b = ctypes.create_string_buffer(512)
        self._lib.p0_last_error(self.ctx, b, 512)
        return b.value.decode()

    def set_stream(self, stream_ptr):
        """run subsequent work on an external cudaStream_t (an int address; 0 = the context's own stream)"""
        self._check(self._lib.p0_set_stream(self.ctx, ctypes.c_void_p(int(stream_ptr) or None)))

    def set_overlap(self, weights_static=True):
        """let GEMV calls fetch their weights before the call ahead on the stream has finished (p0_set_overlap): the
        caller guarantees that no work in flight writes a weight buffer (weights written once, then synchronised)"""
        self._check(self._lib.p0_set_overlap(self.ctx, 1 if weights_static else 0))

    @property
    def stats(self):
        a, p, d = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint64()
        self._check(self._lib.p0_stats(self.ctx, ctypes.byref(a), ctypes.byref(p), ctypes.byref(d)))
        return {"alive": a.value, "peak": p.value, "dispatches": d.value}

    # -------------------------------------------------------------- buffers (gpu.js:81-147)
    def buffer(self, size, label=""):
        b = L.p0_buf()
        self._check(self._lib.p0_buffer(self.ctx, int(size), label.encode(), ctypes.byref(b)))
        rounded = max(16, -(-int(size) // 16) * 16)
        buf = Buffer(self, b.id, rounded, label)
        self.bufs.add(buf)
        return buf

    def wrap(self, ptr, size, label=""):
        """register caller-owned device memory (e.g. torch_tensor.data_ptr()) as a buffer"""
        b = L.p0_buf()
        self._check(self._lib.p0_wrap(self.ctx, ctypes.c_void_p(int(ptr)), int(size), label.encode(), ctypes.byref(b)))
        buf = Buffer(self, b.id, int(size), label, external=True)
        self.bufs.add(buf)
        return buf

    def upload(self, data, label="", dst=None, dst_off=0):
        """upload host data into a NEW buffer (or into dst at dst_off), as Gpu.upload"""
        a = np.ascontiguousarray(data)
        nbytes = a.nbytes
        b = dst or self.buffer(nbytes, label)
        self._check(self._lib.p0_upload(self.ctx, b.handle, int(dst_off), a.ctypes.data_as(ctypes.c_void_p), nbytes))
        # the copy is stream-ordered; keep the host array alive until it has been consumed
        self._check(self._lib.p0_done(self.ctx, 0))
        return b

    def upload_file(self, b, path, file_off=0, nbytes=None, dst_off=0):
        """nbytes of the file at path (from file_off) into buffer b at dst_off: the native chunked, double-buffered
        disk -> pinned -> device copy (p0_upload_file); the copies are ordered on the stream"""
        if nbytes is None:
            nbytes = os.path.getsize(path) - int(file_off)
        self._check(self._lib.p0_upload_file(self.ctx, b.handle, int(dst_off), os.fsencode(path), int(file_off), int(nbytes)))
        return b

    def write(self, b, data, dst_off=0):
        return self.upload(data, dst=b, dst_off=dst_off)

    def copy(self, src, src_off, dst, dst_off, size):
        """Runner.copy (gpu.js:237): device -> device, ordered on the stream"""
        self._check(self._lib.p0_copy(self.ctx, src.handle, int(src_off), dst.handle, int(dst_off), int(size)))

    def read(self, b, off=0, size=None, dtype=np.uint8):
        """read size bytes at off (flushes), returned as a numpy array of dtype"""
        size = b.size - off if size is None else int(size)
        out = np.empty(size, np.uint8)
        self._check(self._lib.p0_read(self.ctx, b.handle, int(off), size, out.ctypes.data_as(ctypes.c_void_p)))
        return out.view(dtype)

    def free(self, b):
        if b is None or b not in self.bufs:
            return
        self.bufs.discard(b)
        self._check(self._lib.p0_free(self.ctx, b.handle))

    def free_all(self):
        for b in list(self.bufs):
            self.free(b)

    def done(self, timeout_ms=60000):
        """wait for the device with a bound (gpu.js:141-147); raises P0Error(P0_ETIMEOUT) when it runs out"""
        self._check(self._lib.p0_done(self.ctx, int(timeout_ms)))

    def wait_selftest(self, polls=4096):
        """enqueue the failure-path check: a kernel whose bounded in-kernel wait runs out after `polls` tries and
        records its code; the next done() raises P0Error(P0_ETIMEOUT) and the context stays usable"""
        self._check(self._lib.p0_wait_selftest(self.ctx, int(polls)))

    # -------------------------------------------------------------- recorded chains (engine/llm/drunner.js)
    def chain_begin(self):
        """start recording: gemv / gemvM calls on this context are checked and kept, not launched (DecodeRunner.begin)"""
        self._check(self._lib.p0_chain_begin(self.ctx))

    def chain_end(self):
        """stop recording; returns the Chain (its device state is allocated here)"""
        h = ctypes.c_void_p()
        self._check(self._lib.p0_chain_end(self.ctx, ctypes.byref(h)))
        return Chain(self, h)

    def close(self):
        if self.ctx:
            self._lib.p0_destroy(self.ctx)
            self.ctx = ctypes.c_void_p()
            self.bufs.clear()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def createGpu(device=0):
    """createGpu (gpu.js:18-23)"""
    return Gpu(device)


def version():
    return L.load().p0_version().decode()


class Chain:
    """a recorded sequence of gemv / gemvM calls (p0_chain_*): run() enqueues them as one persistent kernel where they fit"""

    def __init__(self, g, h):
        self.g, self.h = g, h

    def run(self):
        self.g._check(self.g._lib.p0_chain_run(self.g.ctx, self.h))

    def info(self):
        v = [ctypes.c_uint32() for _ in range(4)]
        self.g._check(self.g._lib.p0_chain_info(self.g.ctx, self.h, *[ctypes.byref(x) for x in v]))
        return dict(zip(("calls", "kernel_calls", "launches", "barriers"), (x.value for x in v)))

    def free(self):
        if self.h:
            self.g._lib.p0_chain_free(self.g.ctx, self.h)
            self.h = None
