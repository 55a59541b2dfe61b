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
HEAD_TRAFFIC = 340.01e6


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
        self.index = ",".join(str(i) for i in index) if isinstance(index, (list, tuple)) else str(index)
        self.proc, self.lines = None, []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", self.index, "--query-gpu=" + self.FIELDS, "--format=csv,noheader,nounits",
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
def call_cost_us(M, N, head=False):
    """rough device time of one GEMV call (a fixed ~3 us per call plus its bytes at 4 TB/s), for placing calls on ranks"""
    return 3.0 + gemv_bytes(M, N, K, head) / 4e6


def step_bytes():
    """the whole job's algorithmic bytes of one step: the 12 calls, whatever the split"""
    return sum(gemv_bytes(M, N, K, N == HEAD_N) for N in NS for M in MS)


def head_parts(ws):
    """the parts (runs of whole 64-row tiles) each vocabulary-head call is cut into: one per rank on up to two ranks;
    from four ranks on, ws / 4, so that the four head calls' parts spread one per rank and no rank pays a head call's
    fixed cost (x staging, ring fill and drain, the last tiles' epilogues: ~15 us) more than once per step"""
    return ws if ws <= 2 else max(1, ws // 4)


def plan_calls(ws):
    """The units of a step and where they run. Each vocabulary-head call (N = 262144) is cut into head_parts(ws) row
    ranges (whole 64-row tiles); each small call (N = 2048, 16384) is one unit. Every unit runs whole on one rank:
    largest first, onto the rank with the least estimated time so far (ties: lowest rank); every rank computes the same
    plan. On two ranks each rank runs half of every head call; on four, one whole head call; on eight, one half."""
    P = head_parts(ws)
    units = []
    for N in NS:
        for j, M in enumerate(MS):
            parts = P if N == HEAD_N else 1
            for p in range(parts):
                units.append({"M": M, "Nfull": N, "head": N == HEAD_N, "j": j, "part": p, "rows": N // parts})
    load = [0.0] * ws
    for u in sorted(units, key=lambda u: -call_cost_us(u["M"], u["rows"], u["head"])):
        r = min(range(ws), key=lambda r: (load[r], r))
        u["rank"] = r
        load[r] += call_cost_us(u["M"], u["rows"], u["head"])
    return units


def ring_copies(wbytes):
    """weight copies per matrix so that the copies together are at least 2x the L2 size"""
    return max(1, -(-2 * L2_BYTES // wbytes))


def ring_offset(j, copies):
    """the copy the j-th M call of one matrix starts on: the four M calls of a step read four different copies"""
    return j * (copies // 4) if copies >= 4 else j % copies


class Sweep:
    """the config-2 sweep's calls on this rank: weight rings, inputs, outputs (one step = every rank's calls once)"""

    def __init__(self, g, torch, ws, rank, seed=0):
        import p0pc0rn_b200 as p0
        self.p0, self.g, self.torch, self.ws, self.rank = p0, g, torch, ws, rank
        dev = torch.device("cuda", torch.cuda.current_device())
        gen = torch.Generator(device=dev)
        plan = plan_calls(ws)
        self.total_bytes = step_bytes()   # the whole job's step
        self.parts = head_parts(ws)
        # the graph count every rank uses: the longest ring of any rank (the same number of replays everywhere)
        self.R = max(ring_copies(c["rows"] * K * 5 // 8) for c in plan)
        self.calls, rings = [], {}
        out_floats = 0
        # every call's gathered output (Y, or the head's MX pairs and its rstd slot) is a slice of one per-rank buffer,
        # the all-gather's source: the step needs no copies before the collective. All ranks size it alike.
        per_rank = max(sum((c["M"] * (c["rows"] // 64) * 2 + 8) if c["head"] else c["M"] * c["rows"]
                           for c in plan if c["rank"] == r) for r in range(ws))
        self.gather_src = torch.zeros(per_rank, dtype=torch.float32, device=dev)
        self.per_rank = per_rank
        slice_of = lambda off, n, label: g.wrap(self.gather_src.data_ptr() + off * 4, n * 4, label)
        for pc in plan:
            if pc["rank"] != rank:
                continue
            N, M, head = pc["Nfull"], pc["M"], pc["head"]
            Nr = pc["rows"]                                  # rows this unit runs (whole 64-row tiles)
            if N not in rings:
                wbytes = Nr * K * 5 // 8
                ring = []
                for c in range(ring_copies(wbytes)):
                    gen.manual_seed(seed * 1000003 + N * 31 + c * 7 + rank)
                    wf = torch.randn(Nr, K, generator=gen, device=dev, dtype=torch.float32) * 0.02
                    wb = g.wrap(wf.data_ptr(), wf.numel() * 4, "wf32")
                    q = p0.pack_q4(g, wb, Nr, K)
                    g.done()
                    g.free(wb)
                    del wf
                    ring.append(q)
                rings[N] = ring
            ring = rings[N]
            rng = np.random.default_rng(seed + 17 * M + N)
            x = rng.standard_normal(M * K).astype(np.float16).astype(np.float32)
            xb = g.upload(x, "x")
            NT = Nr // 64
            c = {"M": M, "N": Nr, "Nfull": N, "head": head, "ring": ring, "i": ring_offset(pc["j"], len(ring)), "x": x, "xb": xb,
                 "bytes": gemv_bytes(M, Nr, K, head), "out_off": out_floats}
            if head:
                c["y"] = g.buffer(M * Nr * 4, "y")       # the logits stay on the rank; the MX pairs are gathered
                nw = (1.0 + 0.1 * rng.standard_normal(K)).astype(np.float32)
                c["nw"] = g.upload(nw, "nw")
                c["mxb"] = slice_of(out_floats, M * NT * 2 + 8, "mx")
                c["st"] = g.upload(np.full(8, 0.9, np.float32), "st")
                c["stat_off"] = M * NT * 2              # the rstd slot past the tile slots (gemma4.js:504)
                g.write(c["mxb"], np.full(1, 0.9, np.float32), dst_off=c["stat_off"] * 4)
                out_floats += M * NT * 2 + 8
            else:
                c["y"] = slice_of(out_floats, M * Nr, "y")
                out_floats += M * Nr
            self.calls.append(c)
        self.out_floats = out_floats
        self.step_bytes = sum(c["bytes"] for c in self.calls)    # this rank's share

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

    def launch(self, c):
        a = self.args(c)
        if c["M"] == 1:
            self.p0.gemv(self.g, a)
        else:
            self.p0.gemvM(self.g, a)
        c["i"] += 1


def capture(torch, stream, fn):
    """a CUDA graph of the library launches `fn` issues on `stream` (the library launches on the stream it was given)"""
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr, stream=stream, capture_error_mode="relaxed"):
        fn()
    return gr


def time_graph_us(torch, gr, n):
    """device time per launch of a graph of n launches: one untimed replay, then one timed by CUDA events"""
    gr.replay()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    gr.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1e3 / n


def run_config1(g, torch, stream):
    """BASELINE config 1, one W4 GEMV layer: M = 1, N = 8192, K = 2048 (10,526,720 algorithmic bytes per call), raw /
    store. A graph of 4 launches per ring copy, the copies together >= 2x L2, so every call reads its weights from HBM."""
    import p0pc0rn_b200 as p0
    N = 8192
    dev = torch.device("cuda", torch.cuda.current_device())
    gen = torch.Generator(device=dev)
    ring = []
    for c in range(ring_copies(N * K * 5 // 8)):
        gen.manual_seed(8192 + c)
        wf = torch.randn(N, K, generator=gen, device=dev) * 0.02
        wb = g.wrap(wf.data_ptr(), wf.numel() * 4, "wf")
        ring.append(p0.pack_q4(g, wb, N, K))
        g.done()
        g.free(wb)
        del wf
    xb = g.upload(np.random.default_rng(11).standard_normal(K).astype(np.float16).astype(np.float32), "x")
    yb = g.buffer(N * 4, "y")
    n = 4 * len(ring)

    def body():
        for i in range(n):
            p0.gemv(g, {"w": {"buf": ring[i % len(ring)], "off": 0, "enc": "q4g32a.t64", "rows": N, "cols": K}, "x": {"buf": xb},
                        "N": N, "K": K, "y": {"buf": yb}})
    gr = capture(torch, stream, body)
    us = min(time_graph_us(torch, gr, n) for _ in range(3))
    del gr
    for b in ring + [xb, yb]:
        g.free(b)
    hbm, _, _ = peaks()
    byts = gemv_bytes(1, N, K, False)
    return {"M": 1, "N": N, "K": K, "us_per_call": round(us, 2), "GB_s": round(byts / (us * 1e-6) / 1e9, 1),
            "frac_of_hbm": round(byts / (us * 1e-6) / 1e9 / hbm, 4), "bytes_per_call": byts,
            "launch": "graph of %d back-to-back calls over %d weight copies (%.0f MB > 2x L2)" % (n, len(ring), len(ring) * N * K * 0.625 / 1e6)}


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
    # the all-gather: every rank's output slices (equal sizes) into one buffer per step
    gather_src = sw.gather_src
    gather_dst = torch.empty(sw.per_rank * ws, dtype=torch.float32, device="cuda")
    outs = []
    for c in sw.calls:
        buf = c["mxb"] if c["head"] else c["y"]
        n = c["M"] * (c["N"] // 64) * 2 if c["head"] else c["M"] * c["N"]
        outs.append((c["out_off"], n, buf.ptr))

    def copies(ptrs=None):
        """outputs written elsewhere (the e2e loop's second buffer set) into their slices; the first set writes there"""
        for i, (off, n, ptr) in enumerate(outs):
            src = ptrs[i] if ptrs else ptr
            if src != gather_src.data_ptr() + off * 4:
                _memcpy_d2d(gather_src.data_ptr() + off * 4, src, n * 4, stream.cuda_stream)

    def gather(ptrs=None):
        """every call's outputs of this rank (at ptrs, default the first buffer set) -> one buffer -> one NCCL
        all-gather (stream-ordered)"""
        if dist is None:
            return
        copies(ptrs)
        dist.all_gather_into_tensor(gather_dst, gather_src)

    # eager warm-up (sizes the library's workspace and sets up NCCL before any capture)
    for _ in range(args.warmup):
        for c in sw.calls:
            sw.launch(c)
        gather()
    torch.cuda.synchronize()
    small = [c for c in sw.calls if not c["head"]]
    heads = [c for c in sw.calls if c["head"]]
    # the step as one graph per weight-ring position: this rank's small calls, then its head calls between two event
    # record nodes (they time the head group inside every timed step: the group's time / its launches is the head
    # kernel's average launch duration, the calls chained back to back as in the step), then the gather copies
    steps_g = []
    for _ in range(sw.R):
        e0, e1 = torch.cuda.Event(enable_timing=True, external=True), torch.cuda.Event(enable_timing=True, external=True)

        def body(e0=e0, e1=e1):
            for c in small:
                sw.launch(c)
            e0.record()
            for c in heads:
                sw.launch(c)
            e1.record()
            if dist:
                copies()
        steps_g.append((capture(torch, stream, body), e0, e1))
    # the NCCL all-gather as its own graph (captured once, replayed after every step graph)
    g_gather = None
    if dist:
        g_gather = capture(torch, stream, lambda: dist.all_gather_into_tensor(gather_dst, gather_src))

    def step(s):
        steps_g[s % sw.R][0].replay()
        if g_gather is not None:
            g_gather.replay()

    # every step graph replayed before the timed region (a graph's first launch uploads it)
    for s in range(max(sw.R, args.warmup)):
        step(s)
    torch.cuda.synchronize()
    clk = Clocks(list(range(ws))) if rank == 0 else None
    if clk:
        clk.start()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    w0 = time.time()
    t0.record()
    for s in range(args.steps):
        step(s)
    t1.record()
    torch.cuda.synchronize()
    w1 = time.time()
    ms = t0.elapsed_time(t1)
    rank_ms = [ms]
    if dist:
        tt = torch.zeros(ws, device="cuda")
        tt[rank] = ms
        dist.all_reduce(tt, op=dist.ReduceOp.SUM)
        rank_ms = [float(v) for v in tt.tolist()]
        ms = max(rank_ms)
    clocks = clk.stop(w0, w1) if clk else None
    # the head group of every graph the timed region replayed (each graph's events hold its last replay)
    used = sorted({s % sw.R for s in range(args.steps)})
    head_us = [steps_g[i][1].elapsed_time(steps_g[i][2]) * 1e3 for i in used]
    # ---- per-call device time after the timed region: each call launched once per ring copy (cold weights) in one graph
    calls_us = {}
    for c in sw.calls:
        n = max(4, len(c["ring"]))
        gr = capture(torch, stream, lambda c=c, n=n: [sw.launch(c) for _ in range(n)])
        calls_us["M%d_N%d" % (c["M"], c["Nfull"])] = round(time_graph_us(torch, gr, n), 2)
        del gr
    del steps_g
    if g_gather is not None:
        del g_gather
    torch.cuda.synchronize()
    # ---- e2e: host inputs (pinned) -> device, the public API calls, results -> host, every step
    e2e = run_e2e(args, sw, g, torch, dist, gather)
    # ---- secondary: config 1; GEMM configs 3 and 4; config 5 decode chain
    config1 = run_config1(g, torch, stream) if rank == 0 else None
    gemm = run_gemm_secondary(args, g, torch, ws, rank, dist)
    decode = run_decode_chain(args, g, torch, stream, dist, ws, rank)
    decode_step = run_decode_step(args, g, torch, stream) if rank == 0 else None
    res = None
    if rank == 0:
        hbm, tfl, src = peaks()
        value = sw.total_bytes * args.steps / (ms / 1e3) / 1e9
        # roofline of the dominant kernel: the vocabulary head GEMV (this rank's rows), timed inside the timed steps
        head_bytes = sum(c["bytes"] for c in heads)
        head_launch_us = float(np.mean(head_us)) / len(heads)
        achieved = head_bytes / len(heads) / (head_launch_us * 1e-6) / 1e9
        res = {
            "metric": "W4 GEMV GB/s (config 2 sweep: M 1/2/4/8 x N 2048/16384/262144, K 2048)",
            "value": round(value, 1), "unit": "GB/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "q4 weights (fp16 scale/min), f32 accumulate; x as an fp16 hi+lo pair (~22 significant bits) on the tensor cores",
            "data": "synthetic (seeded N(0,0.02) weights packed to q4g32a.t64 on device; N(0,1) fp16 x)",
            "config": sweep_config(ws),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s", "frac": round(achieved / hbm, 4),
                         "traffic": HEAD_TRAFFIC * heads[0]["N"] / HEAD_N,
                         "traffic_note": "dram__bytes_read.sum + dram__bytes_write.sum of one head launch at M=1 (N=262144) from an ncu "
                                         "capture (335.63 + 4.38 MB; algorithmic 336.6 MB), scaled by the rows of this rank's head calls at N>1",
                         "kernel": "gemv head (rms+softcap) N=%d rows per call K=%d, M=%s on this rank" % (
                             heads[0]["N"], K, "/".join(str(c["M"]) for c in heads)),
                         "launch_us": round(head_launch_us, 2), "launches_timed": len(used) * len(heads),
                         "timing": "event record nodes around this rank's head calls inside every timed step graph; achieved = "
                                   "the head calls' algorithmic bytes / the group's device time", "peak_source": src},
            "e2e": e2e, "gpu_launches": len(sw.calls) * args.steps, "clocks": clocks, "rank_ms": [round(v, 4) for v in rank_ms],
            "config1": config1, "gemm": gemm, "calls_us": calls_us, "decode": decode, "decode_step": decode_step,
        }
        res["cpu_baseline"] = cpu_baseline(args) if ws == 1 else None
    if dist:
        dist.barrier()
    g.close()
    return res


def sweep_config(ws):
    return {"workload": "config2_gemv_sweep", "M": list(MS), "N": list(NS), "K": K,
            "parallelism": ("each head call cut into %d row range(s); head ranges and small calls each run whole on one rank "
                            "(largest first onto the least-loaded rank), one all-gather per step" % head_parts(ws)) if ws > 1 else "one GPU",
            "l2": "every call reads weights from HBM: each matrix has copies totalling >= 2x L2 (or one copy > 2x L2) and the "
                  "four M calls of a matrix read four different copies in a step",
            "bytes_per_step": step_bytes(),
            "launch": "one CUDA graph per step and weight-ring position (every rank's calls; the head group between two event "
                      "record nodes)" + (", then the NCCL all-gather graph" if ws > 1 else "")}


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
    two sets of device inputs / outputs and pinned outputs alternate, uploads and downloads go on two more streams (the
    two copy engines) so that step s's downloads and step s+1's uploads overlap the kernels and neither waits behind
    the other, and the host waits for step s-2's results before it enqueues step s (two steps in flight). Events order each buffer's reuse: an upload waits for the compute two steps
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
    ups, downs = torch.cuda.Stream(), torch.cuda.Stream()   # uploads and downloads on their own copy engines

    def use(b):
        for c, _, _, xb, yb, mxb in sets[b]:
            c["xb"], c["y"] = xb, yb
            if mxb is not None:
                c["mxb"] = mxb
    # the calls a step makes through the public API, recorded as a CUDA graph per step of a cycle of 2R steps (buffer
    # set s & 1; the weight-ring copies advance per step as they do when the calls are launched one by one): one launch
    # per step from the host, as a serving loop runs its decode step
    graphs = []
    for k in range(2 * sw.R):
        use(k & 1)
        graphs.append(capture(torch, comp, lambda: [sw.launch(c) for c in sw.calls]))
    h2d_done = [torch.cuda.Event(), torch.cuda.Event()]
    comp_done = [torch.cuda.Event(), torch.cuda.Event()]
    d2h_done = [torch.cuda.Event(), torch.cuda.Event()]
    for e in h2d_done + comp_done + d2h_done:
        e.record(comp)
    torch.cuda.synchronize()

    def step(s):
        b = s & 1
        d2h_done[b].synchronize()                     # step s - 2's results are on the host (its pinned set is free)
        ups.wait_event(comp_done[b])                 # the compute two steps back has read these inputs
        for (c, xp, _, _, _, _), t in zip(sets[b], pin_in):
            _memcpy_h2d(xp, t.data_ptr(), t.numel() * 4, ups.cuda_stream)
        h2d_done[b].record(ups)
        comp.wait_event(h2d_done[b])
        comp.wait_event(d2h_done[b])                 # the download two steps back has read these outputs
        graphs[s % len(graphs)].replay()
        gather([op for _, _, op, _, _, _ in sets[b]])
        comp_done[b].record(comp)
        downs.wait_event(comp_done[b])
        for (c, _, op, _, _, _), o in zip(sets[b], pin_out[b]):
            _memcpy_d2h(o.data_ptr(), op, o.numel() * 4, downs.cuda_stream)
        d2h_done[b].record(downs)

    steps = max(20, args.steps)
    for s in range(len(graphs) + 4):               # every graph replayed once (its first launch uploads it)
        step(s)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for s in range(steps):
        step(s)
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    use(0)                                           # the set the rest of the bench uses
    del graphs
    if dist:
        tt = torch.tensor([dt], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        dt = float(tt.item())
    val = sw.total_bytes * steps / dt / 1e9
    return {"value": round(val, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_step": round(dt / steps * 1e3, 4),
            "path": "p0pc0rn_b200.gemv/gemvM (ctypes -> libp0mm.so C ABI) recorded as one CUDA graph per step; "
                    "pinned host x in, outputs out every step; uploads and downloads on their own streams, two buffer sets, two steps "
                    "in flight"}


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


def run_decode_chain(args, g, torch, stream, dist=None, ws=1, rank=0):
    """config 5: the linear chain of one decode pass of a random-init 26-layer decoder (hidden 2048): per layer QKV
    2560x2048 (rms prologue), O 2048x2048, GeGLU 2x8192x2048 (rms prologue), down 2048x8192 (kPer 2048 split
    partials, as gemma4.js runs it), then the head 262144x2048 (rms prologue, softcap + per-tile argmax). Attention,
    norms and residual adds are excluded (as config 5 states), but the data dependencies of a real step are kept: each
    call reads the previous call's output (QKV -> O reads the first 2048 of q|k|v, O -> GeGLU, GeGLU -> down, the down
    projection's first split partial -> the next layer's QKV and the head), so no call can start its math before the
    one ahead has finished. Every weight is its own q4g32a.t64 matrix (1.31 GB per pass > L2).
    One GPU, two ways: "graph" = the 105 library calls captured in one CUDA graph (each a kernel launch, chained by
    programmatic dependent launch); "chain" = the same calls recorded with p0_chain_begin / p0_chain_end and run as one
    persistent chain kernel (the 104 layer calls, grid barriers between dependent calls, weights streamed ahead across
    them) plus the head's own kernel, one CUDA graph per pass.
    With ws GPUs the FFN and the head are tensor-parallel: rank r owns 1/ws of the GeGLU's gate and up rows, the
    matching 1/ws k-slice of the down projection (its split partials are all-gathered, so every rank holds the partials
    a one-GPU normadd sums) and 1/ws of the head's rows (their per-tile max / argmax pairs are all-gathered); QKV and O
    run whole on every rank ("graph" form only: the collectives sit between the calls).
    tok/s = M tokens per pass / pass time (max over ranks; M = 1 decode, M = 4 draft-verify)."""
    import p0pc0rn_b200 as p0
    dev = torch.device("cuda", torch.cuda.current_device())
    gen = torch.Generator(device=dev)
    D = CHAIN_D
    FFr, HEADr = CHAIN_FF // ws, HEAD_N // ws
    kp = min(2048, FFr)
    nsp = -(-FFr // kp)

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
        s0 = 7000 + 4 * l + 1000 * rank
        layers.append((packed(CHAIN_QKV, D, s0), packed(D, D, s0 + 1), packed(2 * FFr, D, s0 + 2), packed(D, FFr, s0 + 3)))
    head = packed(HEADr, D, 7999 + rank)
    # the whole job's weight bytes per pass (QKV and O on every rank)
    wbytes = (CHAIN_LAYERS * ((CHAIN_QKV * D + D * D) * ws + 2 * CHAIN_FF * D + D * CHAIN_FF) + HEAD_N * D) * 0.625
    rng = np.random.default_rng(5)
    out = {}
    for M in (1, 4):
        xh = g.upload(rng.standard_normal(M * D).astype(np.float32), "x")
        nw = g.upload((1.0 + 0.1 * rng.standard_normal(D)).astype(np.float32), "nw")
        st = g.upload(np.full(8, 0.9, np.float32), "st")
        yq, yo, yg = g.buffer(M * CHAIN_QKV * 4, "yq"), g.buffer(M * D * 4, "yo"), g.buffer(M * FFr * 4, "yg")
        yd = g.buffer(ws * nsp * M * D * 4, "yd")       # the down partials (all ranks' after the gather)
        mx = g.buffer(M * (HEADr // 64) * 8 + 64, "mx")
        yh = g.buffer(M * HEADr * 4, "yh")
        g.write(mx, np.full(1, 0.9, np.float32), dst_off=HEADr // 64 * 2 * 4)   # the head's rstd slot (lops.js:125)
        coll = None
        if dist:
            part = torch.zeros(nsp * M * D, dtype=torch.float32, device=dev)
            part_all = torch.zeros(ws * nsp * M * D, dtype=torch.float32, device=dev)
            mxt = torch.empty(M * (HEADr // 64) * 2, dtype=torch.float32, device=dev)
            mx_all = torch.empty(ws * mxt.numel(), dtype=torch.float32, device=dev)
            coll = (part, part_all, mxt, mx_all, g.wrap(part.data_ptr(), part.numel() * 4, "part"),
                    g.wrap(mxt.data_ptr(), mxt.numel() * 4, "mxt"), g.wrap(part_all.data_ptr(), part_all.numel() * 4, "part_all"))
        hid = coll[6] if coll else yd                     # the next layer's x: the first split partial, rows of D

        def call(w, N, Kk, x, ldx, yb, pro="raw", epi="store", kPer=0, extra=None):
            a = {"w": w, "x": {"buf": x, "ldx": ldx}, "N": N, "K": Kk, "y": {"buf": yb}, "pro": pro, "epi": epi}
            if kPer:
                a["kPer"] = kPer
            if pro == "rms":
                a["norm"] = {"buf": nw, "off": 0}
                a["stat"] = {"buf": st, "off": 0, "ld": 1}
            if extra:
                a.update(extra)
            if M == 1:
                a["x"].pop("ldx")
                if pro == "rms" and epi != "softcap":
                    a["stat"] = {"buf": st, "off": 0}
                p0.gemv(g, a)
            else:
                p0.gemvM(g, dict(a, M=M))

        def layer_calls(l, x0):
            wq, wo, wg, wd = layers[l]
            call(wq, CHAIN_QKV, D, x0, D, yq, pro="rms")
            call(wo, D, D, yq, CHAIN_QKV, yo)
            call(wg, FFr, D, yo, D, yg, pro="rms", epi="geglu")
            call(wd, D, FFr, yg, FFr, coll[4] if coll else yd, kPer=kp)

        def head_call():
            if M == 1:
                extra = {"mx": {"buf": mx}, "stat": {"buf": mx, "off": HEADr // 64 * 2}, "cap": 30.0}
            else:
                extra = {"mx": {"buf": coll[5] if coll else mx}, "cap": 30.0}
            call(head, HEADr, D, hid, D, yh, pro="rms", epi="softcap", extra=extra)

        def graph_pass():
            for l in range(CHAIN_LAYERS):
                layer_calls(l, xh if l == 0 else hid)
                if coll:
                    dist.all_gather_into_tensor(coll[1], coll[0])
            head_call()
            if coll:
                if M == 1:
                    _memcpy_d2d(coll[2].data_ptr(), mx.ptr, coll[2].numel() * 4, stream.cuda_stream)
                dist.all_gather_into_tensor(coll[3], coll[2])

        def time_pass(fn):
            fn()
            torch.cuda.synchronize()
            gr = capture(torch, stream, fn)
            for _ in range(3):
                gr.replay()
            torch.cuda.synchronize()
            if dist:
                dist.barrier()
                torch.cuda.synchronize()
            reps = max(3, min(50, args.steps // 40))
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                gr.replay()
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / reps
            if dist:
                tt = torch.tensor([ms], device=dev)
                dist.all_reduce(tt, op=dist.ReduceOp.MAX)
                ms = float(tt.item())
            del gr
            return ms

        # algorithmic bytes: weights + x reads + outputs (down: its split partials; head: logits + MX), whole job
        act = (M * D * 4 + M * CHAIN_QKV * 4) * ws + (M * D * 4 * 2) * ws + (M * D * 4 + M * CHAIN_FF * 4) + (M * CHAIN_FF * 4 + 4 * M * D * 4)
        pass_bytes = wbytes + CHAIN_LAYERS * act + M * D * 4 * ws + M * HEAD_N * 4 + M * (HEAD_N // 64) * 8

        def entry(ms, extra=None):
            e = {"ms_per_pass": round(ms, 4), "tok_s": round(M / (ms / 1e3), 1), "GB_s": round(pass_bytes / (ms / 1e3) / 1e9, 1)}
            if extra:
                e.update(extra)
            return e

        res = {"graph": entry(time_pass(graph_pass), {"launches_per_pass": CHAIN_LAYERS * 4 + 1,
                                                      "collectives_per_pass": (CHAIN_LAYERS + 1) if dist else 0})}
        if not dist:
            g.chain_begin()
            for l in range(CHAIN_LAYERS):
                layer_calls(l, xh if l == 0 else hid)
            head_call()
            ch = g.chain_end()
            info = ch.info()
            res["chain"] = entry(time_pass(ch.run), {"recorded_calls": info["calls"], "calls_in_chain_kernel": info["kernel_calls"],
                                                     "launches_per_pass": info["launches"] + 1, "grid_barriers": info["barriers"]})
            torch.cuda.synchronize()
            ch.free()
        out["M%d" % M] = res
        for b in (xh, nw, st, yq, yo, yg, yd, mx, yh):
            g.free(b)
        if coll:
            for b in coll[4:]:
                g.free(b)
            del coll
    for ws_ in layers:
        for w in ws_:
            g.free(w["buf"])
    g.free(head["buf"])
    hbm, _, _ = peaks()
    # the headline form: the faster of the two at M = 1
    best = "chain" if (not dist and out["M1"]["chain"]["ms_per_pass"] < out["M1"]["graph"]["ms_per_pass"]) else "graph"
    return {"metric": "linear-chain decode tok/s (config 5: 26 x [QKV, O, GeGLU, down] + head, attention excluded, each call "
                      "reading the previous call's output)",
            "weights_GB": round(wbytes / 1e9, 3), "hbm_peak_gbs": hbm, "passes": out, "form": best,
            "tok_s_M1": out["M1"][best]["tok_s"], "tok_s_M4": out["M4"][best]["tok_s"],
            "frac_of_hbm_M1": round(out["M1"][best]["GB_s"] / (hbm * ws), 4),
            "parallelism": "one GPU" if ws == 1 else "FFN and head tensor-parallel x%d (NCCL all-gather of the down partials "
                           "and of the head's max/argmax pairs), QKV and O on every rank" % ws,
            "launch": "one CUDA graph per pass"}


# ------------------------------------------------------------------------------------------ whole decode token (secondary)
def run_decode_step(args, g, torch, stream, ctx_len=1024):
    """One whole decode token of a random-init Gemma-4-style decoder with config 5's matmul shapes (hidden 2048, 26
    layers of QKV 2560x2048 / O 2048x2048 / GeGLU 2x8192x2048 / down 2048x8192, the tied 262144x2048 head), 8 query heads
    of 256 over one KV head, every fifth layer full attention and the others a 512-position sliding window, at position
    ctx_len - 1 with the caches holding ctx_len (full) or 512 (sliding) earlier keys: p0pc0rn_b200.decode.decode_token
    (gemma4.js encodeStep without the per-layer embeddings) = embed, per layer QKV -> qkrope -> attnDec -> O -> normadd
    -> GeGLU -> down -> normadd, then the softcap head and argmax, all library kernels, one CUDA graph per token."""
    import p0pc0rn_b200 as p0
    from p0pc0rn_b200 import decode
    cfg = {"D": CHAIN_D, "layers": CHAIN_LAYERS, "NH": 8, "NKV": 1, "hd": 256, "FF": CHAIN_FF, "vocab": HEAD_N, "window": 512,
           "kinds": ["full" if l % 5 == 4 else "sliding" for l in range(CHAIN_LAYERS)], "embed_scale": 45.254834, "softcap": 30.0,
           "eps": 1e-6}
    dev = torch.device("cuda", torch.cuda.current_device())
    gen = torch.Generator(device=dev)
    sz = decode.model_sizes(cfg)

    def packed(shape, seed):
        gen.manual_seed(seed)
        wf = torch.randn(shape[0], shape[1], generator=gen, device=dev) * 0.02
        wb = g.wrap(wf.data_ptr(), wf.numel() * 4, "wf")
        q = p0.pack_q4(g, wb, shape[0], shape[1])
        g.done()
        g.free(wb)
        del wf
        return q

    rng = np.random.default_rng(9)
    vec = lambda n: g.upload((1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32))
    ang = rng.uniform(0, 6.283, ctx_len * 128)
    rope = np.zeros(2 * ctx_len * 128, np.float32)
    rope[0::2], rope[1::2] = np.cos(ang), np.sin(ang)
    rb = g.upload(rope)
    m = {"embed": packed(sz["head"], 8000), "final_norm": vec(CHAIN_D), "rope": {"full": rb, "sliding": rb}, "layers": []}
    for l in range(CHAIN_LAYERS):
        m["layers"].append({"qkv": packed(sz["qkv"], 8100 + 4 * l), "o": packed(sz["o"], 8101 + 4 * l), "gu": packed(sz["gu"], 8102 + 4 * l),
                            "down": packed(sz["down"], 8103 + 4 * l), "in_norm": vec(CHAIN_D), "qk_norm": vec(512), "post_attn": vec(CHAIN_D),
                            "pre_ff": vec(CHAIN_D), "post_ff": vec(CHAIN_D)})
    s = decode.DecodeState(g, cfg, ctx_len)
    kv = []
    for c in s.caches:   # earlier keys and values: random fp16
        for k in ("kc", "vc"):
            t = (torch.randn(c["len"] * 256, generator=gen, device=dev) * 0.5).half()
            g.copy(g.wrap(t.data_ptr(), t.numel() * 2, "kv"), 0, c[k], 0, t.numel() * 2)
            kv.append(t)
    g.write(s.b["ids"], np.array([1234, 0, 0, 0], np.uint32))
    pos = ctx_len - 1
    nk = decode.decode_token(g, m, s, pos)
    g.done()
    gr = capture(torch, stream, lambda: decode.decode_token(g, m, s, pos))
    for _ in range(3):
        gr.replay()
    reps = 20
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        gr.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    arg = g.read(s.b["arg"], 0, 8, np.uint32)
    del gr
    wbytes = (CHAIN_LAYERS * (sum(a * b for a, b in (sz["qkv"], sz["o"], sz["gu"], sz["down"]))) + HEAD_N * CHAIN_D) * 0.625
    kvbytes = sum(2 * min(c["len"], pos + 1) * 256 * 2 for c in s.caches)
    hbm, _, _ = peaks()
    for b in list(s.b.values()) + [c[k] for c in s.caches for k in ("kc", "vc")]:
        g.free(b)
    for L in m["layers"]:
        for b in L.values():
            g.free(b)
    g.free(m["embed"])
    g.free(rb)
    del kv
    return {"ms_per_token": round(ms, 4), "tok_s": round(1e3 / ms, 1), "context": ctx_len, "kernels_per_token": nk,
            "GB_s": round((wbytes + kvbytes) / (ms / 1e3) / 1e9, 1), "frac_of_hbm": round((wbytes + kvbytes) / (ms / 1e3) / 1e9 / hbm, 4),
            "argmax": int(arg[0]), "weights_GB": round(wbytes / 1e9, 3), "kv_MB": round(kvbytes / 1e6, 2),
            "note": "whole decode token (embed, 26 x [attention + MLP], head, argmax) through p0pc0rn_b200.decode; one CUDA graph"}


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
HEAD_SLICE = 8192


def host_cores():
    """the host threads this process may run on (torchrun sets OMP_NUM_THREADS=1 for its ranks; the CPU legs set their
    OpenMP thread count from this instead)"""
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


class CpuSweep:
    """The reference's GEMV arithmetic on the host cores over the sweep's own calls: the oracle's C restatement of
    lgemv / lgemvM (lops.js:30-106, lops_spec.js:44-157; scalar C, no SIMD, OpenMP over 64-row tiles), raw / store.
    The N = 2048 and 16384 calls run whole; the vocabulary head runs on an 8192-row slice (1/32 of its rows, its
    rms / softcap work left out) and its time is scaled by 32. One step = the 12 calls; its time estimates the full
    sweep step."""

    def __init__(self, threads):
        from oracle import ref
        self.ref, self.threads = ref, threads
        rng = np.random.default_rng(1)
        self.w = {}
        for N in (2048, 16384, HEAD_SLICE):
            W = (rng.standard_normal(N * K) * 0.02).astype(np.float32)
            self.w[N] = ref.pack_q4(W, N, K)[0]
        self.x = {M: rng.standard_normal(M * K).astype(np.float16).astype(np.float32) for M in MS}

    def step(self):
        t = 0.0
        for N in NS:
            Nr = HEAD_SLICE if N == HEAD_N else N
            for M in MS:
                t0 = time.perf_counter()
                self.ref.gemv_cpu_mt(self.w[Nr], self.x[M], M, Nr, K, self.threads)
                t += (time.perf_counter() - t0) * (N // Nr)
        return t

    @staticmethod
    def sample(steps):
        return ("the config-2 sweep's 12 calls per step (N=2048 and 16384 whole; the N=262144 head on an %d-row slice, "
                "time x%d), %d steps, scalar C restatement of lgemv/lgemvM with OpenMP" % (HEAD_SLICE, HEAD_N // HEAD_SLICE, steps))


def cpu_baseline(args, budget_s=12.0):
    """the same sweep through the CPU restatement on all host cores, repeated for about budget_s seconds"""
    thr = host_cores()
    cs = CpuSweep(thr)
    cs.step()
    total = step_bytes()
    t, n, t_start = 0.0, 0, time.perf_counter()
    while time.perf_counter() - t_start < budget_s or n < 3:
        t += cs.step()
        n += 1
    return {"value": round(total * n / t / 1e9, 3), "unit": "GB/s", "cores": thr, "kind": "port", "sample": cs.sample(n)}


def run_reference(args, ws, rank):
    """the reference arm: the reference's own GEMV arithmetic for this path on the host cores (the reference is JS +
    WebGPU: no JS engine and no CPU WebGPU adapter here, so the oracle's C restatement stands in, kind "port"); rank 0
    alone at N > 1. W warm-up steps, then K timed steps of the sweep (each a bounded sample: the head on a slice)."""
    if rank != 0:
        return None
    thr = host_cores()
    cs = CpuSweep(thr)
    for _ in range(args.warmup):
        cs.step()
    t = sum(cs.step() for _ in range(args.steps))
    total = step_bytes()
    value = round(total * args.steps / t / 1e9, 3)
    cb = {"value": value, "unit": "GB/s", "cores": thr, "kind": "port", "sample": cs.sample(args.steps)}
    return {"impl": "reference", "metric": "W4 GEMV GB/s (config 2 sweep: M 1/2/4/8 x N 2048/16384/262144, K 2048)", "value": value,
            "unit": "GB/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t / args.steps * 1e3, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "q4 weights (fp16 scale/min), f32 x and accumulate", "data": "synthetic", "config": sweep_config(1),
            "cpu_baseline": cb, "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "the reference is JS + WebGPU (no CPU WebGPU adapter or JS engine on this box): its lgemv/lgemvM arithmetic "
                    "restated in C (oracle/oracle.c) on the host cores, the same calls as the GPU arm"}


def run_case(args):
    """One operator on cuda:0: one warm launch, then `--reps` launches timed with CUDA events (the small cases ncu
    captures; back-to-back launches, so a weight matrix below the L2 size is partly L2-resident).
      --case gemv  --M 1 --N 262144 --K 2048 [--head]   (head: rms prologue + softcap epilogue, as the engine's head)
      --case gemm  --M 4096 --N 9216 --K 3072 [--gelu]  (bias epilogue)
      --case step                                       (one whole decode token, as the line's decode_step key)
      --case chain --M 1                                (config 5 as a recorded chain, as the line's decode key)"""
    import torch
    import p0pc0rn_b200 as p0
    torch.cuda.set_device(0)
    g = p0.Gpu(0)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    g.set_stream(stream.cuda_stream)
    if args.case in ("step", "chain"):
        g.set_overlap(True)
        args.steps = 40 * args.reps
        out = run_decode_step(args, g, torch, stream) if args.case == "step" else run_decode_chain(args, g, torch, stream)
        g.close()
        print(json.dumps({"case": args.case, "result": out}))
        return
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
    ap.add_argument("--case", default=None, choices=["gemv", "gemm", "step", "chain"], help="run one operator or pass (for ncu captures)")
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
