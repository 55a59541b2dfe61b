"""Two CUDA ranks (one process per GPU, NCCL over NVLink): the sharded forms of the reference's calls computed by
libp0mm.so on each rank, exchanged by p0pc0rn_b200.shard, checked against the one-GPU call and the CPU oracle.

  * column split of the vocabulary head (rms prologue, softcap epilogue; gemma4.js:503-509, spec.js:164): each rank
    runs gemvM on its half of the 64-row tiles; the all-gathered per-tile (max, argmax) pairs, rebased to global rows,
    give the one-GPU argmax (tie rule on the global index, lops.js:95-102 / lops_spec.js:144-153);
  * k split of the FFN down projection (gemma4.js:485, kPer 2048): each rank runs the reference's own call on its kPer
    slices; the all-gathered split partials are the one-GPU partials, and their split-order sum is normadd's
    (lops.js:155).
Skipped with fewer than two GPUs. The ranks are spawned processes with a short process-group timeout; the parent
joins them with a bound.
"""
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MAXABS, RELL2 = 1e-2, 1e-3


def _gpus():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _head_inputs():
    from oracle import ref
    M, N, K = 4, 32768, 2048
    b, _ = ref.pack_q4(ref.randn(N * K, 600, 0.02), N, K)
    X = ref.round_f16(ref.randn(M * K, 601))
    nw = ref.randn(K, 602, 0.1) + 1
    st = np.array([0.9, 1.1, 0.8, 1.0], np.float32)
    return M, N, K, b, X, nw, st


def _down_inputs():
    from oracle import ref
    M, N, K, kPer = 2, 2048, 8192, 2048
    b, _ = ref.pack_q4(ref.randn(N * K, 610, 0.02), N, K)
    X = ref.randn(M * K, 611)
    return M, N, K, kPer, b, X


def _worker(rank, world, port, q):
    try:
        import datetime

        import torch
        import torch.distributed as dist

        import p0pc0rn_b200 as p0
        from p0pc0rn_b200 import shard
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                                timeout=datetime.timedelta(seconds=60))
        g = p0.Gpu(rank)
        out = {}
        # ---- column split of the head
        M, N, K, b, X, nw, st = _head_inputs()
        wb = g.upload(b)
        w = {"buf": wb, "off": 0, "enc": "q4g32a.t64", "rows": N, "cols": K}
        n0, n1 = shard.tile_range(N, world, rank)
        Nr = n1 - n0
        xb, nwb, stb = g.upload(X), g.upload(nw), g.upload(st)
        yb, mxb = g.buffer(M * Nr * 4), g.buffer(M * (Nr // 64) * 8)
        p0.gemvM(g, {"w": shard.column_view(w, n0, n1), "x": {"buf": xb}, "M": M, "N": Nr, "K": K, "pro": "rms", "epi": "softcap",
                     "cap": 30.0, "norm": {"buf": nwb, "off": 0}, "stat": {"buf": stb, "off": 0, "ld": 1}, "y": {"buf": yb},
                     "mx": {"buf": mxb}})
        g.done()
        y_loc = g.read(yb, 0, M * Nr * 4, np.float32)
        mx_loc = g.read(mxb, 0, M * (Nr // 64) * 8, np.float32)
        gathered = shard.all_gather_np(dist, mx_loc)
        starts = [shard.tile_range(N, world, r)[0] for r in range(world)]
        out["mx"] = shard.merge_mx(gathered, world, M, Nr // 64, starts)
        out["y"] = shard.all_gather_np(dist, y_loc.reshape(M, Nr))      # [world][M][Nr]
        if rank == 0:   # the one-GPU call on the whole head
            y1, mx1 = g.buffer(M * N * 4), g.buffer(M * (N // 64) * 8)
            p0.gemvM(g, {"w": w, "x": {"buf": xb}, "M": M, "N": N, "K": K, "pro": "rms", "epi": "softcap", "cap": 30.0,
                         "norm": {"buf": nwb, "off": 0}, "stat": {"buf": stb, "off": 0, "ld": 1}, "y": {"buf": y1}, "mx": {"buf": mx1}})
            g.done()
            out["mx1"] = g.read(mx1, 0, M * (N // 64) * 8, np.float32)
            out["y1"] = g.read(y1, 0, M * N * 4, np.float32)
        # ---- k split of the down projection
        M, N, K, kPer, b, X = _down_inputs()
        wb2, xb2 = g.upload(b), g.upload(X)
        nsplit = K // kPer
        s0, s1 = shard.split_range(nsplit, world, rank)
        a = {"w": {"buf": wb2, "off": 0, "enc": "q4g32a.t64", "rows": N, "cols": K}, "x": {"buf": xb2, "ldx": K}, "M": M, "N": N,
             "K": K, "kPer": kPer}
        ak = shard.kslice_args(a, kPer, s0, s1)
        pb = g.buffer((s1 - s0) * M * N * 4)
        ak["y"] = {"buf": pb}
        assert p0.gemvM(g, ak) == s1 - s0
        g.done()
        parts = g.read(pb, 0, (s1 - s0) * M * N * 4, np.float32).reshape(s1 - s0, M * N)
        out["parts"] = shard.all_gather_np(dist, parts).reshape(nsplit, M * N)
        if rank == 0:
            p1 = g.buffer(nsplit * M * N * 4)
            a1 = dict(a, y={"buf": p1})
            assert p0.gemvM(g, a1) == nsplit
            g.done()
            out["parts1"] = g.read(p1, 0, nsplit * M * N * 4, np.float32).reshape(nsplit, M * N)
        dist.barrier()
        g.close()
        dist.destroy_process_group()
        q.put((rank, out))
    except Exception as e:   # report to the parent instead of hanging it
        q.put((rank, repr(e)))


def _run(world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            r, out = q.get(timeout=600)
            res[r] = out
    finally:
        for p in procs:
            p.join(60)
            if p.is_alive():
                p.kill()
    for r in range(world):
        assert isinstance(res.get(r), dict), "rank %d: %r" % (r, res.get(r))
    return res


def _close(got, want):
    g = np.asarray(got, np.float32).astype(np.float16).astype(np.float64)
    w = np.asarray(want, np.float32).astype(np.float16).astype(np.float64)
    err = float(np.max(np.abs(g - w)))
    rl2 = float(np.sqrt(np.sum((g - w) ** 2) / np.sum(w ** 2)))
    assert np.all(np.isfinite(g)) and err <= MAXABS and rl2 <= RELL2, (err, rl2)


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
def test_two_rank_column_split_head_and_k_split_down():
    from oracle import ref
    from p0pc0rn_b200 import shard
    res = _run(2)
    r0 = res[0]
    # head: gathered logits and pairs vs the oracle and vs the one-GPU call
    M, N, K, b, X, nw, st = _head_inputs()
    want_y, want_mx, _ = ref.gemvM(b, X, M, N, K, pro="rms", epi="softcap", norm=nw, stat=st, stat_ld=1)
    y = np.concatenate([r0["y"][r] for r in range(2)], axis=1).reshape(-1)   # [M][N]
    _close(y, want_y)
    _close(y, r0["y1"])
    mx = r0["mx"]
    assert np.array_equal(mx, res[1]["mx"])                  # every rank holds the same merged pairs
    _close(mx[0::2], want_mx[0::2])
    for other in (want_mx, r0["mx1"]):
        gi, wi = mx.view(np.uint32)[1::2].astype(np.int64), other.view(np.uint32)[1::2].astype(np.int64)
        for t in np.nonzero(gi != wi)[0]:
            m = t // (N // 64)
            assert abs(float(want_y[m * N + gi[t]]) - float(want_y[m * N + wi[t]])) <= 1e-5
    am, am1, amo = shard.pick_argmax(mx, M), shard.pick_argmax(r0["mx1"], M), shard.pick_argmax(want_mx, M)
    for m in range(M):
        for other in (am1, amo):
            if am[m, 0] != other[m, 0]:
                assert abs(float(want_y[m * N + am[m, 0]]) - float(want_y[m * N + other[m, 0]])) <= 1e-5
    # down: gathered partials vs the oracle's and the one-GPU call's, and their split-order sum
    M, N, K, kPer, b, X = _down_inputs()
    want_p, _, ns = ref.gemvM(b, X, M, N, K, kPer=kPer)
    want_p = want_p.reshape(ns, M * N)
    parts = r0["parts"]
    assert np.array_equal(parts, res[1]["parts"])
    for s in range(ns):
        _close(parts[s], want_p[s])
        _close(parts[s], r0["parts1"][s])
    _close(shard.sum_splits(parts), shard.sum_splits(want_p))
