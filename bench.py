#!/usr/bin/env python
"""Benchmark of the 4-bit quantized matmul hot path on B200 (driver contract: one JSON line from rank 0).

Workload ("skinny-M decode / speculative-verify GEMV sweep"): K = 2048, M in {1, 2, 4, 8},
N in {2048, 16384, 262144}; W ~ N(0, 0.02) packed to q4g32a.t64 on the device (the reference's packQ4); x ~ N(0, 1)
fp16 values. N = 262144 is the vocabulary head and runs as the engine runs it (rms prologue, softcap epilogue with
per-tile max/argmax, gemma4.js:503-509); the others run raw/store. M = 1 calls gemv (lops.js), M > 1 gemvM
(lops_spec.js). One step = the 12 calls once. With N GPUs every call is column-split (each rank owns N/ranks rows,
whole 64-row tiles) and the step ends with ONE all-gather of every rank's outputs (NCCL over NVLink).
value = algorithmic bytes of the step (N*K*0.625 + M*K*4 + M*N*4 (+MX) per call) / device time (max over ranks).
Inputs larger than L2: each small-N call cycles through a ring of weight copies totalling >= 2x the 126 MB L2.
Secondary (same line, key "gemm"): config 3 / config 4 W4A16 GEMM TFLOP/s (rows split across ranks, no comm).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

L2_BYTES = 126 * 2 ** 20
K = 2048
MS = (1, 2, 4, 8)
NS = (2048, 16384, 262144)
HEAD_N = 262144
# DRAM bytes (read + write) of one head GEMV launch (N = 262144, K = 2048, M = 1) from an ncu capture
HEAD_TRAFFIC = 340.45e6


def gemv_bytes(M, N, K, head):
    b = N * K * 0.625 + M * K * 4 + M * N * 4
    if head:
        b += M * (N // 64) * 8
    return b


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


# ------------------------------------------------------------------------------------------ clocks sampler
class Clocks:
    """nvidia-smi sampled every 200 ms in the background; stop(t0, t1) summarises the samples taken inside the wall-clock
    window [t0, t1] of the timed region (the nearest samples when the window is shorter than the sampling period)."""
    FIELDS = "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown," \
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"

    def __init__(self, index):
        self.index, self.proc, self.lines = index, None, []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), "--query-gpu=" + self.FIELDS, "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
            t0 = time.time()
            while not self.lines and time.time() - t0 < 3.0:   # the sampler is running before the timed region starts
                time.sleep(0.02)
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def stop(self, t0=None, t1=None):
        if t1 is not None:
            end = time.time() + 0.5
            while time.time() < end and not any(ts >= t1 for ts, _ in self.lines):
                time.sleep(0.02)                               # one sample after the window
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(2)
            except Exception:
                self.proc.kill()
        rows = []
        for ts, ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                rows.append((ts, float(f[1]), float(f[2]), f))
            except ValueError:
                continue
        inside = [r for r in rows if t0 is None or (t0 <= r[0] <= t1)]
        if not inside and rows and t0 is not None:
            mid = (t0 + t1) / 2
            inside = sorted(rows, key=lambda r: abs(r[0] - mid))[:2]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in inside:
            for nm, v in zip(names, r[3][5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        sm = [r[1] for r in inside]
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max([r[2] for r in inside], default=None),
                "reasons": sorted(reasons), "samples": len(inside), "window_s": round(t1 - t0, 4) if t0 is not None else None}


# ------------------------------------------------------------------------------------------ distributed plumbing
def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def init_dist(ws, local):
    import torch
    import torch.distributed as dist
    if ws > 1 and not dist.is_initialized():
        import datetime
        dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=datetime.timedelta(seconds=120))
    return dist if ws > 1 else None


# ------------------------------------------------------------------------------------------ our arm
class Sweep:
    """the config-2 sweep on this rank: weight rings, inputs, outputs, one step = 12 calls"""

    def __init__(self, g, torch, ws, rank, seed=0):
        import p0pc0rn_b200 as p0
        self.p0, self.g, self.torch, self.ws, self.rank = p0, g, torch, ws, rank
        dev = torch.device("cuda", torch.cuda.current_device())
        gen = torch.Generator(device=dev)
        self.calls = []
        self.keep = []
        out_floats = 0
        for N in NS:
            Nr = N // ws                                     # this rank's rows (whole tiles)
            head = N == HEAD_N
            wbytes = Nr * K * 5 // 8
            copies = 1 if wbytes * 1 >= 2 * L2_BYTES else max(2, -(-2 * L2_BYTES // wbytes))
            ring = []
            for c in range(copies):
                gen.manual_seed(seed * 1000003 + N * 31 + c * 7 + rank)
                wf = torch.randn(Nr, K, generator=gen, device=dev, dtype=torch.float32) * 0.02
                wb = g.wrap(wf.data_ptr(), wf.numel() * 4, "wf32")
                q = p0.pack_q4(g, wb, Nr, K)
                g.done()
                g.free(wb)
                del wf
                ring.append(q)
            for M in MS:
                rng = np.random.default_rng(seed + 17 * M + N)
                x = rng.standard_normal(M * K).astype(np.float16).astype(np.float32)
                xb = g.upload(x, "x")
                NT = Nr // 64
                c = {"M": M, "N": Nr, "Nfull": N, "head": head, "ring": ring, "i": 0, "x": x, "xb": xb,
                     "bytes": gemv_bytes(M, Nr, K, head), "out_off": out_floats}
                c["y"] = g.buffer(M * Nr * 4, "y")
                if head:
                    nw = (1.0 + 0.1 * rng.standard_normal(K)).astype(np.float32)
                    c["nw"] = g.upload(nw, "nw")
                    mx = np.zeros(M * NT * 2 + 8, np.float32)
                    c["mxb"] = g.upload(mx, "mx")
                    c["st"] = g.upload(np.full(8, 0.9, np.float32), "st")
                    c["stat_off"] = M * NT * 2              # the rstd slot past the tile slots (gemma4.js:504)
                    g.write(c["mxb"], np.full(1, 0.9, np.float32), dst_off=c["stat_off"] * 4)
                    out_floats += M * NT * 2
                else:
                    out_floats += M * Nr
                self.calls.append(c)
        self.out_floats = out_floats
        self.step_bytes = sum(c["bytes"] for c in self.calls)

    def args(self, c):
        q = c["ring"][c["i"] % len(c["ring"])]
        w = {"buf": q, "off": 0, "enc": "q4g32a.t64", "rows": c["N"], "cols": K}
        a = {"w": w, "x": {"buf": c["xb"]}, "N": c["N"], "K": K, "y": {"buf": c["y"]}}
        if c["head"]:
            a.update(pro="rms", epi="softcap", cap=30.0, norm={"buf": c["nw"], "off": 0}, mx={"buf": c["mxb"]})
            if c["M"] == 1:
                a["stat"] = {"buf": c["mxb"], "off": c["stat_off"]}
            else:
                a["stat"] = {"buf": c["st"], "off": 0, "ld": 1}
        if c["M"] > 1:
            a["M"] = c["M"]
        return a

    def launch(self, c, ev=None):
        a = self.args(c)
        if ev is not None:
            ev[0].record()
        if c["M"] == 1:
            self.p0.gemv(self.g, a)
        else:
            self.p0.gemvM(self.g, a)
        if ev is not None:
            ev[1].record()
        c["i"] += 1

    def step(self, head_events=None):
        n = 0
        for c in self.calls:
            ev = None
            if head_events is not None and c["head"]:
                ev = (self.torch.cuda.Event(enable_timing=True), self.torch.cuda.Event(enable_timing=True))
                head_events.append((c, ev))
            self.launch(c, ev)
            n += 1
        return n


def capture(torch, stream, fn):
    """a CUDA graph of the library launches `fn` issues on `stream` (the library launches on the stream it was given)"""
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr, stream=stream, capture_error_mode="relaxed"):
        fn()
    return gr


def run_ours(args, ws, rank, local):
    import torch
    torch.cuda.set_device(local)
    dist = init_dist(ws, local)
    import p0pc0rn_b200 as p0
    g = p0.Gpu(local)
    # one non-default stream for everything: torch events / copies / NCCL and the library's launches are ordered on it
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    g.set_stream(stream.cuda_stream)
    sw = Sweep(g, torch, ws, rank)
    torch.cuda.synchronize()
    # the weights are packed and synchronised: GEMVs may fetch them while the call ahead finishes (p0_set_overlap)
    g.set_overlap(True)
    # one gather buffer: every call's outputs of this rank, concatenated; one all-gather per step
    gather_src = torch.empty(sw.out_floats, dtype=torch.float32, device="cuda")
    gather_dst = torch.empty(sw.out_floats * ws, dtype=torch.float32, device="cuda")
    outs = []
    for c in sw.calls:
        buf = c["mxb"] if c["head"] else c["y"]
        n = c["M"] * (c["N"] // 64) * 2 if c["head"] else c["M"] * c["N"]
        outs.append((c["out_off"], n, buf.ptr))

    def copies(ptrs=None):
        for i, (off, n, ptr) in enumerate(outs):
            _memcpy_d2d(gather_src.data_ptr() + off * 4, ptrs[i] if ptrs else ptr, n * 4, stream.cuda_stream)

    def gather(ptrs=None):
        """every call's outputs of this rank (at ptrs, default the first buffer set) -> one buffer -> one NCCL
        all-gather (stream-ordered)"""
        if dist is None:
            return
        copies(ptrs)
        dist.all_gather_into_tensor(gather_dst, gather_src)

    # eager warm-up (sizes the library's workspace before any capture), then the step as CUDA graphs: the 8 small-N calls
    # as one graph per weight-ring position, each head call as its own graph (events between graph launches time the
    # head inside the timed region), the gather copies as one graph; the NCCL all-gather stays eager
    for _ in range(args.warmup):
        sw.step()
        gather()
    torch.cuda.synchronize()
    small = [c for c in sw.calls if not c["head"]]
    heads = [c for c in sw.calls if c["head"]]
    R = max(len(c["ring"]) for c in small)
    # the whole step as one graph per ring position (small calls, then the head calls)
    g_step = [capture(torch, stream, lambda: [sw.launch(c) for c in small + heads]) for _ in range(R)]
    # the same step with an event record node before and after each head call (the events bracket the head kernel
    # inside the graph, without graph-launch gaps); NI such graphs, each with its own events, replayed in turn on ~1% of
    # the timed steps, so the events of each hold the timing of its last replay
    NI = 10
    g_inst = []
    for _ in range(NI):
        evs = [(c, torch.cuda.Event(enable_timing=True, external=True), torch.cuda.Event(enable_timing=True, external=True)) for c in heads]

        def body(evs=evs):
            for c in small:
                sw.launch(c)
            for c, e0, e1 in evs:
                e0.record()
                sw.launch(c)
                e1.record()
        g_inst.append((capture(torch, stream, body), evs))
    g_copy = capture(torch, stream, copies) if dist else None

    def step(s, inst=None):
        if inst is None:
            g_step[s % R].replay()
        else:
            g_inst[inst % NI][0].replay()
        if dist:
            g_copy.replay()
            dist.all_gather_into_tensor(gather_dst, gather_src)

    for s in range(max(3, args.warmup)):
        step(s)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clk = Clocks(local)
    clk.start()
    every = max(1, args.steps // 100)   # the instrumented graphs on ~100 of the timed steps
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    w0 = time.time()
    t0.record()
    for s in range(args.steps):
        step(s, s // every if s % every == 0 else None)
    t1.record()
    torch.cuda.synchronize()
    clocks = clk.stop(w0, time.time())
    ms = t0.elapsed_time(t1)
    if dist:
        tt = torch.tensor([ms], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    head_ms = {}
    ninst = len(range(0, args.steps, every))
    for gr, evs in g_inst[:min(NI, ninst)]:
        for c, a, b in evs:
            head_ms.setdefault(c["M"], []).append(a.elapsed_time(b))
    # ---- per-call device time after the timed region: each call launched once per ring copy (cold weights) in one graph
    calls_us = {}
    for c in sw.calls:
        n = len(c["ring"]) if not c["head"] else 8
        gr = capture(torch, stream, lambda c=c, n=n: [sw.launch(c) for _ in range(n)])
        gr.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        gr.replay()
        e1.record()
        torch.cuda.synchronize()
        calls_us["M%d_N%d" % (c["M"], c["Nfull"])] = round(e0.elapsed_time(e1) * 1e3 / n, 2)
        del gr
    del g_step, g_inst, g_copy
    # ---- e2e: host inputs (pinned) -> device, the public API calls, results -> host, every step
    e2e = run_e2e(args, sw, g, torch, dist, gather)
    # ---- secondary: GEMM configs 3 and 4; config 5 decode chain (one GPU)
    gemm = run_gemm_secondary(args, g, torch, ws, rank, dist)
    decode = run_decode_chain(args, g, torch, stream) if ws == 1 else None
    res = None
    if rank == 0:
        hbm, tfl, src = peaks()
        total_bytes = sw.step_bytes * ws * args.steps
        value = total_bytes / (ms / 1e3) / 1e9
        # roofline of the dominant kernel: the vocabulary head GEMV, averaged over its launches in the timed region
        per_m = {M: float(np.mean(v)) for M, v in head_ms.items()}
        head_bytes = sum(c["bytes"] for c in sw.calls if c["head"])
        head_time = sum(per_m.values()) / 1e3
        achieved = head_bytes / head_time / 1e9
        res = {
            "metric": "W4 GEMV GB/s (config 2 sweep: M 1/2/4/8 x N 2048/16384/262144, K 2048)",
            "value": round(value, 1), "unit": "GB/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "q4 weights, f32 x/accumulate", "data": "synthetic (seeded N(0,0.02) weights packed to q4g32a.t64 on device; N(0,1) fp16 x)",
            "config": {"workload": "config2_gemv_sweep", "M": list(MS), "N": list(NS), "K": K, "parallelism": "column-split x%d + all-gather" % ws,
                       "l2": "weight rings >= 2x L2 per small-N call; head 335 MB > L2", "bytes_per_step": sw.step_bytes * ws,
                       "launch": "one CUDA graph per step (the 12 library calls, per weight-ring position); on ~1% of the "
                                 "timed steps the step graph carries event record nodes around each head call, which time the "
                                 "head kernel"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s", "frac": round(achieved / hbm, 4),
                         "traffic": HEAD_TRAFFIC if ws == 1 else None,
                         "traffic_note": "dram__bytes_read.sum + dram__bytes_write.sum of one head launch at M=1 from an ncu "
                                         "capture (335.7 + 4.7 MB); algorithmic 336.6 MB", "kernel": "gemv head (rms+softcap) N=%d/rank K=%d, M=1/2/4/8" % (HEAD_N // ws, K),
                         "per_M_us": {str(k): round(v * 1e3, 2) for k, v in sorted(per_m.items())}, "peak_source": src},
            "e2e": e2e, "gpu_launches": len(sw.calls) * args.steps, "clocks": clocks, "gemm": gemm,
            "calls_us": calls_us, "decode": decode,
        }
        res["cpu_baseline"] = cpu_baseline(args) if ws == 1 else None
    if dist:
        dist.barrier()
    g.close()
    return res


_cudart = None


def _memcpy_d2d(dst, src, nbytes, stream):
    global _cudart
    import ctypes
    if _cudart is None:
        import torch  # noqa: F401  (loads the CUDA runtime into the process)
        for name in ("libcudart.so.12", "libcudart.so"):
            try:
                _cudart = ctypes.CDLL(name)
                break
            except OSError:
                continue
        _cudart.cudaMemcpyAsync.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_void_p]
    r = _cudart.cudaMemcpyAsync(ctypes.c_void_p(dst), ctypes.c_void_p(src), nbytes, 3, ctypes.c_void_p(stream))
    if r != 0:
        raise RuntimeError("cudaMemcpyAsync failed: %d" % r)


def run_e2e(args, sw, g, torch, dist, gather):
    """the same sweep through the public API with host buffers: every step, x from pinned host memory -> device, the
    12 calls, results device -> pinned host; wall-clock over the steps (max over ranks). Run as a serving loop runs it:
    two sets of device inputs / outputs and pinned outputs alternate, the copies go on a second stream (the copy
    engines) so that step s's downloads and step s+1's uploads overlap the kernels, and the host waits for step s-2's
    results before it enqueues step s (two steps in flight). Events order each buffer's reuse: an upload waits for the compute two steps
    back that read its buffer, a compute waits for its upload and for the download two steps back of its outputs."""
    h2d = d2h = 0
    pin_in, pin_out = [], [[], []]
    sets = [[], []]                                  # per parity: (call, x buffer, output buffer, y buffer, mx buffer)
    for c in sw.calls:
        t = torch.from_numpy(c["x"]).pin_memory()
        pin_in.append(t)
        h2d += t.numel() * 4
        n = c["M"] * (c["N"] // 64) * 2 if c["head"] else c["M"] * c["N"]
        d2h += n * 4
        for b in range(2):
            pin_out[b].append(torch.empty(n, dtype=torch.float32).pin_memory())
            if b == 0:
                xb, yb, mxb = c["xb"], c["y"], c.get("mxb")
            else:
                xb, yb = g.buffer(c["xb"].size, "x1"), g.buffer(c["y"].size, "y1")
                mxb = None
                if c["head"]:
                    mxb = g.buffer(c["mxb"].size, "mx1")
                    g.write(mxb, np.full(1, 0.9, np.float32), dst_off=c["stat_off"] * 4)
            sets[b].append((c, xb.ptr, (mxb if c["head"] else yb).ptr, xb, yb, mxb))
    comp = torch.cuda.current_stream()
    cps = torch.cuda.Stream()
    h2d_done = [torch.cuda.Event(), torch.cuda.Event()]
    comp_done = [torch.cuda.Event(), torch.cuda.Event()]
    d2h_done = [torch.cuda.Event(), torch.cuda.Event()]
    for e in h2d_done + comp_done + d2h_done:
        e.record(comp)
    torch.cuda.synchronize()

    def step(s):
        b = s & 1
        d2h_done[b].synchronize()                     # step s - 2's results are on the host (its pinned set is free)
        cps.wait_event(comp_done[b])                 # the compute two steps back has read these inputs
        for (c, xp, _, _, _, _), t in zip(sets[b], pin_in):
            _memcpy_h2d(xp, t.data_ptr(), t.numel() * 4, cps.cuda_stream)
        h2d_done[b].record(cps)
        comp.wait_event(h2d_done[b])
        comp.wait_event(d2h_done[b])                 # the download two steps back has read these outputs
        for c, _, _, xb, yb, mxb in sets[b]:
            c["xb"], c["y"] = xb, yb
            if mxb is not None:
                c["mxb"] = mxb
            sw.launch(c)
        gather([op for _, _, op, _, _, _ in sets[b]])
        comp_done[b].record(comp)
        cps.wait_event(comp_done[b])
        for (c, _, op, _, _, _), o in zip(sets[b], pin_out[b]):
            _memcpy_d2h(o.data_ptr(), op, o.numel() * 4, cps.cuda_stream)
        d2h_done[b].record(cps)

    steps = max(3, args.steps // 2)
    for s in range(4):
        step(s)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for s in range(steps):
        step(s)
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    for c, _, _, xb, yb, mxb in sets[0]:             # the set the rest of the bench uses
        c["xb"], c["y"] = xb, yb
        if mxb is not None:
            c["mxb"] = mxb
    if dist:
        tt = torch.tensor([dt], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        dt = float(tt.item())
    ws = dist.get_world_size() if dist else 1
    val = sw.step_bytes * ws * steps / dt / 1e9
    return {"value": round(val, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_step": round(dt / steps * 1e3, 4),
            "path": "p0pc0rn_b200.gemv/gemvM (ctypes -> libp0mm.so C ABI), pinned host x in, outputs out; copies on a second "
                    "stream, two buffer sets, two steps in flight"}


def _memcpy_h2d(dst, src, nbytes, stream):
    _memcpy_kind(dst, src, nbytes, stream, 1)


def _memcpy_d2h(dst, src, nbytes, stream):
    _memcpy_kind(dst, src, nbytes, stream, 2)


def _memcpy_kind(dst, src, nbytes, stream, kind):
    global _cudart
    import ctypes
    if _cudart is None:
        _memcpy_d2d(0, 0, 0, stream)
    r = _cudart.cudaMemcpyAsync(ctypes.c_void_p(dst), ctypes.c_void_p(src), nbytes, kind, ctypes.c_void_p(stream))
    if r != 0:
        raise RuntimeError("cudaMemcpyAsync failed: %d" % r)


# ------------------------------------------------------------------------------------------ decode chain (secondary)
CHAIN_LAYERS, CHAIN_D, CHAIN_QKV, CHAIN_FF = 26, 2048, 2560, 8192


def run_decode_chain(args, g, torch, stream):
    """config 5: the linear chain of one decode pass of a random-init 26-layer decoder (hidden 2048): per layer QKV
    2560x2048 (rms prologue), O 2048x2048, GeGLU 2x8192x2048 (rms prologue), down 2048x8192 (kPer 2048 -> 4 split
    partials, as gemma4.js runs it), then the head 262144x2048 (rms prologue, softcap + per-tile argmax). Attention,
    norms and residual adds are excluded (as config 5 states): each matmul reads a resident synthetic activation.
    Every weight is its own q4g32a.t64 matrix (1.31 GB per pass > L2). One pass = one CUDA graph of the 105 calls;
    tok/s = M tokens per pass / pass time (M = 1 decode, M = 4 draft-verify)."""
    import p0pc0rn_b200 as p0
    dev = torch.device("cuda", torch.cuda.current_device())
    gen = torch.Generator(device=dev)
    D = CHAIN_D

    def packed(rows, cols, seed):
        gen.manual_seed(seed)
        wf = torch.randn(rows, cols, generator=gen, device=dev) * 0.02
        wb = g.wrap(wf.data_ptr(), wf.numel() * 4, "wf")
        q = p0.pack_q4(g, wb, rows, cols)
        g.done()
        g.free(wb)
        del wf
        return {"buf": q, "off": 0, "enc": "q4g32a.t64", "rows": rows, "cols": cols}

    layers = []
    for l in range(CHAIN_LAYERS):
        layers.append((packed(CHAIN_QKV, D, 7000 + 4 * l), packed(D, D, 7001 + 4 * l), packed(2 * CHAIN_FF, D, 7002 + 4 * l),
                       packed(D, CHAIN_FF, 7003 + 4 * l)))
    head = packed(HEAD_N, D, 7999)
    wbytes = (sum(w["rows"] * w["cols"] for ws_ in layers for w in ws_) + HEAD_N * D) * 0.625
    rng = np.random.default_rng(5)
    out = {}
    for M in (1, 4):
        xd = g.upload(rng.standard_normal(M * CHAIN_FF).astype(np.float32), "x")
        nw = g.upload((1.0 + 0.1 * rng.standard_normal(D)).astype(np.float32), "nw")
        st = g.upload(np.full(8, 0.9, np.float32), "st")
        y = g.buffer(4 * M * 2 * CHAIN_FF * 4, "y")
        mx = g.buffer(M * (HEAD_N // 64) * 8 + 64, "mx")
        yh = g.buffer(M * HEAD_N * 4, "yh")

        def call(w, N, Kk, pro="raw", epi="store", kPer=0, yb=y, extra=None):
            a = {"w": w, "x": {"buf": xd}, "N": N, "K": Kk, "y": {"buf": yb}, "pro": pro, "epi": epi}
            if kPer:
                a["kPer"] = kPer
            if pro == "rms":
                a["norm"] = {"buf": nw, "off": 0}
                a["stat"] = {"buf": st, "off": 0, "ld": 1}
            if extra:
                a.update(extra)
            if M == 1:
                if pro == "rms" and epi != "softcap":
                    a["stat"] = {"buf": st, "off": 0}
                p0.gemv(g, a)
            else:
                p0.gemvM(g, dict(a, M=M))

        def one_pass():
            for wq, wo, wg, wd in layers:
                call(wq, CHAIN_QKV, D, pro="rms")
                call(wo, D, D)
                call(wg, CHAIN_FF, D, pro="rms", epi="geglu")
                call(wd, D, CHAIN_FF, kPer=2048)
            if M == 1:   # the head's rstd is read from the mx buffer past the tile slots (lops.js:125)
                call(head, HEAD_N, D, pro="rms", epi="softcap", yb=yh,
                     extra={"mx": {"buf": mx}, "stat": {"buf": mx, "off": HEAD_N // 64 * 2}, "cap": 30.0})
            else:
                call(head, HEAD_N, D, pro="rms", epi="softcap", yb=yh, extra={"mx": {"buf": mx}, "cap": 30.0})

        one_pass()
        torch.cuda.synchronize()
        gr = capture(torch, stream, one_pass)
        for _ in range(2):
            gr.replay()
        reps = max(3, min(50, args.steps // 40))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            gr.replay()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        # algorithmic bytes: weights + x reads + outputs (down: 4 split partials; head: logits + MX)
        act = (M * D * 4 + M * CHAIN_QKV * 4) + (M * D * 4 * 2) + (M * D * 4 + M * CHAIN_FF * 4) + (M * CHAIN_FF * 4 + 4 * M * D * 4)
        pass_bytes = wbytes + CHAIN_LAYERS * act + M * D * 4 + M * HEAD_N * 4 + M * (HEAD_N // 64) * 8
        out["M%d" % M] = {"ms_per_pass": round(ms, 4), "tok_s": round(M / (ms / 1e3), 1), "GB_s": round(pass_bytes / (ms / 1e3) / 1e9, 1),
                          "calls_per_pass": CHAIN_LAYERS * 4 + 1}
        del gr
        for b in (xd, nw, st, y, mx, yh):
            g.free(b)
    for ws_ in layers:
        for w in ws_:
            g.free(w["buf"])
    g.free(head["buf"])
    hbm, _, _ = peaks()
    return {"metric": "linear-chain decode tok/s (config 5: 26 x [QKV, O, GeGLU, down] + head, attention excluded)",
            "weights_GB": round(wbytes / 1e9, 3), "hbm_peak_gbs": hbm, "passes": out,
            "frac_of_hbm_M1": round(out["M1"]["GB_s"] / hbm, 4), "launch": "one CUDA graph per pass"}


# ------------------------------------------------------------------------------------------ GEMM (secondary)
def run_gemm_secondary(args, g, torch, ws, rank, dist):
    """configs 3 and 4 (bias epilogue; GELU-tanh fused on the MLP-up): TFLOP/s per shape, rows split across ranks"""
    import p0pc0rn_b200 as p0
    shapes = [("c3_qkv", 4096, 9216, 3072, False), ("c3_mlp_up", 4096, 12288, 3072, True), ("c3_down", 4096, 3072, 12288, False),
              ("c4_qkv", 32760, 6720, 2240, False), ("c4_mlp_up", 32760, 8960, 2240, True), ("c4_down", 32760, 2240, 8960, False)]
    out = {}
    dev = torch.device("cuda", torch.cuda.current_device())
    gen = torch.Generator(device=dev)
    reps = 5
    for name, M, N, Kk, gelu in shapes:
        Mr = -(-M // ws)
        m0 = min(M, rank * Mr)
        Mr = max(0, min(M, m0 + Mr) - m0)
        gen.manual_seed(hash(name) & 0xFFFF)
        wf = torch.randn(N, Kk, generator=gen, device=dev) * 0.02
        wb = g.wrap(wf.data_ptr(), wf.numel() * 4, "wf")
        q = p0.pack_q4(g, wb, N, Kk)
        g.done()
        g.free(wb)
        del wf
        # two activation copies (each > L2 at config 4; config 3's X is 25 MB: L2-resident, as in a real DiT block)
        xs = [torch.randn(max(Mr, 1), Kk, generator=gen, device=dev).half() for _ in range(2)]
        bias = torch.randn(N, generator=gen, device=dev) * 0.01
        y = torch.empty(max(Mr, 1), N, device=dev, dtype=torch.float16)
        xbs = [g.wrap(x.data_ptr(), x.numel() * 2, "x") for x in xs]
        bb = g.wrap(bias.data_ptr(), bias.numel() * 4, "bias")
        yb = g.wrap(y.data_ptr(), y.numel() * 2, "y")
        w = {"buf": q, "off": 0, "enc": "q4g32a.t64", "rows": N, "cols": Kk}

        def call(i):
            if Mr:
                p0.gemm(g, {"w": w, "x": {"buf": xbs[i % 2]}, "M": Mr, "N": N, "K": Kk, "epi": "bias", "ev": {"buf": bb, "off": 0},
                            "y": {"buf": yb}, "post_gelu": gelu})
        for i in range(2):
            call(i)
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(reps):
            call(i)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        if dist:
            tt = torch.tensor([ms], device="cuda")
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            ms = float(tt.item())
        out[name] = {"M": M, "N": N, "K": Kk, "ms": round(ms, 4), "tflops": round(2.0 * M * N * Kk / (ms / 1e3) / 1e12, 1)}
        for b in xbs + [bb, yb, q]:
            g.free(b)
        del xs, bias, y
    hbm, tfl, src = peaks()
    tot_fl = sum(2.0 * v["M"] * v["N"] * v["K"] for v in out.values())
    tot_ms = sum(v["ms"] for v in out.values())
    agg = tot_fl / (tot_ms / 1e3) / 1e12
    return {"metric": "W4A16 GEMM TFLOP/s (configs 3+4, bias epilogue, GELU-tanh on MLP-up)", "value": round(agg, 1), "unit": "TFLOP/s",
            "frac_of_bf16_peak": round(agg / tfl, 4), "peak": tfl, "peak_source": src, "shapes": out,
            "parallelism": "row-split x%d, no comm" % ws}


# ------------------------------------------------------------------------------------------ CPU baseline / reference arm
def cpu_baseline(args, budget_s=12.0):
    """The reference's GEMV arithmetic on this host's cores: the oracle's C restatement of lgemv/lgemvM (OpenMP over
    64-row tiles, all threads), on a bounded sample of the workload: the config-2 calls with N cut to a slice."""
    from oracle import ref
    thr = ref.max_threads()
    rng = np.random.default_rng(1)
    Ns = 8192
    W = (rng.standard_normal(Ns * K) * 0.02).astype(np.float32)
    b, _ = ref.pack_q4(W, Ns, K)
    t_total, bytes_total, calls = 0.0, 0.0, 0
    t_start = time.perf_counter()
    while time.perf_counter() - t_start < budget_s:
        for M in MS:
            X = rng.standard_normal(M * K).astype(np.float32)
            t0 = time.perf_counter()
            ref.gemv_cpu_mt(b, X, M, Ns, K, thr)
            t_total += time.perf_counter() - t0
            bytes_total += gemv_bytes(M, Ns, K, False)
            calls += 1
    return {"value": round(bytes_total / t_total / 1e9, 3), "unit": "GB/s", "cores": thr, "kind": "port",
            "sample": "config-2 GEMV calls M=1/2/4/8 at N=8192 rows, K=2048, repeated for ~%.0f s (%d calls)" % (budget_s, calls)}


def run_reference(args, ws, rank):
    if rank != 0:
        return None
    cb = cpu_baseline(args, budget_s=max(5.0, min(60.0, 3.0 * args.steps)))
    return {"impl": "reference", "metric": "W4 GEMV GB/s (config 2 sweep: M 1/2/4/8 x N 2048/16384/262144, K 2048)", "value": cb["value"],
            "unit": "GB/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "q4 weights, f32 x/accumulate", "data": "synthetic",
            "config": {"workload": "config2_gemv_sweep", "M": list(MS), "N": list(NS), "K": K},
            "cpu_baseline": cb, "e2e": {"value": cb["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "the reference is JS + WebGPU (no CPU WebGPU adapter or JS engine on this box): its lgemv/lgemvM arithmetic "
                    "restated in C (oracle/oracle.c) on the host cores"}


def run_case(args):
    """One operator on cuda:0: one warm launch, then `--reps` launches timed with CUDA events (the small cases ncu
    captures; back-to-back launches, so a weight matrix below the L2 size is partly L2-resident).
      --case gemv  --M 1 --N 262144 --K 2048 [--head]   (head: rms prologue + softcap epilogue, as the engine's head)
      --case gemm  --M 4096 --N 9216 --K 3072 [--gelu]  (bias epilogue)"""
    import torch
    import p0pc0rn_b200 as p0
    torch.cuda.set_device(0)
    g = p0.Gpu(0)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    g.set_stream(stream.cuda_stream)
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1)
    M, N, Kk = args.M, args.N, args.K
    wf = torch.randn(N, Kk, generator=gen, device=dev) * 0.02
    q = p0.pack_q4(g, g.wrap(wf.data_ptr(), wf.numel() * 4, "wf"), N, Kk)
    g.done()
    del wf
    w = {"buf": q, "off": 0, "enc": "q4g32a.t64", "rows": N, "cols": Kk}
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    if args.case == "gemv":
        x = g.upload(np.random.default_rng(2).standard_normal(M * Kk).astype(np.float32))
        y = g.buffer(M * N * 4)
        a = {"w": w, "x": {"buf": x}, "N": N, "K": Kk, "y": {"buf": y}}
        if args.head:
            NT = N // 64
            mx = g.upload(np.full(M * NT * 2 + 8, 0.9, np.float32))
            a.update(pro="rms", epi="softcap", cap=30.0, norm={"buf": g.upload(np.ones(Kk, np.float32)), "off": 0}, mx={"buf": mx},
                     stat={"buf": mx, "off": M * NT * 2} if M == 1 else {"buf": g.upload(np.full(8, 0.9, np.float32)), "off": 0, "ld": 1})
        fn, aa = (p0.gemv, a) if M == 1 else (p0.gemvM, dict(a, M=M))
        fn(g, aa)
        ev[0].record()
        for _ in range(args.reps):
            fn(g, aa)
        ev[1].record()
        algo = N * Kk * 0.625 + M * Kk * 4 + M * N * 4
    else:
        x = torch.randn(M, Kk, generator=gen, device=dev).half()
        bias = torch.randn(N, generator=gen, device=dev) * 0.01
        y = torch.empty(M, N, device=dev, dtype=torch.float16)
        a = {"w": w, "x": {"buf": g.wrap(x.data_ptr(), x.numel() * 2, "x")}, "M": M, "N": N, "K": Kk, "epi": "bias",
             "ev": {"buf": g.wrap(bias.data_ptr(), bias.numel() * 4, "b"), "off": 0}, "y": {"buf": g.wrap(y.data_ptr(), y.numel() * 2, "y")},
             "post_gelu": bool(args.gelu)}
        p0.gemm(g, a)
        ev[0].record()
        for _ in range(args.reps):
            p0.gemm(g, a)
        ev[1].record()
        algo = 2.0 * M * N * Kk
    torch.cuda.synchronize()
    g.done()
    us = ev[0].elapsed_time(ev[1]) * 1e3 / args.reps
    rate = algo / (us * 1e-6) / (1e9 if args.case == "gemv" else 1e12)
    g.close()
    print(json.dumps({"case": args.case, "M": M, "N": N, "K": Kk, "reps": args.reps, "us": round(us, 2),
                      ("GB/s" if args.case == "gemv" else "TFLOP/s"): round(rate, 1),
                      "note": "back-to-back launches; weights beyond L2 only when N*K*0.625 > 126 MB"}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--case", default=None, choices=["gemv", "gemm"], help="run one operator (for ncu captures)")
    ap.add_argument("--M", type=int, default=1)
    ap.add_argument("--N", type=int, default=262144)
    ap.add_argument("--K", type=int, default=2048)
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--head", action="store_true")
    ap.add_argument("--gelu", action="store_true")
    args = ap.parse_args()
    if args.case:
        return run_case(args)
    args.warmup = max(3, args.warmup)
    ws, rank, local = dist_env()
    if args.impl == "reference":
        res = run_reference(args, ws, rank)
    else:
        res = run_ours(args, ws, rank, local)
    if rank == 0 and res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
