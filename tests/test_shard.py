"""Multi-GPU host logic on CPU: two gloo ranks (spawned processes, 127.0.0.1) run the sharded forms of the reference's
calls, each rank's compute done by the CPU oracle (the checker, standing in for the GPU), and the exchange done by
p0pc0rn_b200.shard over torch.distributed. The merged results must equal the one-rank results bit for bit:
  * column split of the softcap head: logits, per-tile (max, argmax) pairs with global indices, the argmax itself;
  * k split of the down projection: the split partials and their split-order sum (normadd's order).
"""
import os
import socket

import numpy as np
import pytest

from p0pc0rn_b200 import shard


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_ranges():
    assert [shard.tile_range(262144, 8, r) for r in (0, 7)] == [(0, 32768), (229376, 262144)]
    with pytest.raises(ValueError):
        shard.tile_range(64 * 3, 2, 0)
    sizes = [shard.row_range(4095 * 8 - 1, 8, r) for r in (0, 7)]
    assert [b - a for a, b in sizes] == [4095, 4094]
    assert shard.split_range(4, 2, 1) == (2, 4)


def test_column_view_offsets():
    w = {"buf": None, "off": 256, "enc": "q4g32a.t64", "rows": 4096, "cols": 2048}
    v = shard.column_view(w, 1024, 2048)
    assert v["off"] == 256 + 16 * 64 * 1280 and v["rows"] == 1024 and v["bytes"] == 16 * 64 * 1280


def test_pick_argmax_tie_rule():
    mx = np.array([1.0, 0, 3.0, 0, 3.0, 0], np.float32)
    mx.view(np.uint32)[1::2] = [5, 70, 9]
    out = shard.pick_argmax(mx, 1)
    assert out[0, 0] == 9 and out[0, 1] == np.float32(3.0).view(np.uint32)


def _head_case():
    from oracle import ref
    M, N, K = 2, 1024, 256
    b, _ = ref.pack_q4(ref.randn(N * K, 300, 0.02), N, K)
    X = ref.randn(M * K, 301)
    nw = ref.randn(K, 302, 0.1) + 1
    st = np.array([0.9, 1.1], np.float32)
    return M, N, K, b, X, nw, st


def _column_worker(rank, world, port, res):
    import torch.distributed as dist
    from oracle import ref
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        M, N, K, b, X, nw, st = _head_case()
        n0, n1 = shard.tile_range(N, world, rank)
        view = shard.column_view({"off": 0, "enc": "q4g32a.t64", "rows": N, "cols": K}, n0, n1)
        wl = b[view["off"]:view["off"] + view["bytes"]]
        y, mx, _ = ref.gemvM(wl, X, M, n1 - n0, K, pro="rms", epi="softcap", norm=nw, stat=st, stat_off=0, stat_ld=1, cap=30.0)
        ys = shard.all_gather_np(dist, y.reshape(M, n1 - n0))
        mxs = shard.all_gather_np(dist, mx[:M * (n1 - n0) // 64 * 2])
        starts = [shard.tile_range(N, world, r)[0] for r in range(world)]
        if rank == 0:
            res["y"] = np.concatenate(list(ys), axis=1).reshape(-1)
            res["mx"] = shard.merge_mx(mxs, world, M, (n1 - n0) // 64, starts)
            res["arg"] = shard.pick_argmax(res["mx"], M)
    finally:
        dist.destroy_process_group()


def _ksplit_worker(rank, world, port, res):
    import torch.distributed as dist
    from oracle import ref
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        N, K, kPer = 512, 4096, 1024
        b, _ = ref.pack_q4(ref.randn(N * K, 310, 0.02), N, K)
        x = ref.randn(K, 311)
        ns = K // kPer
        s0, s1 = shard.split_range(ns, world, rank)
        a = shard.kslice_args({"w": {"off": 0, "enc": "q4g32a.t64", "rows": N, "cols": K}, "x": {"rowB": 0}, "N": N, "K": K},
                              kPer, s0, s1)
        y, _, nsl = ref.gemv(b, x, N, a["K"], cols=a["w"]["cols"], woff=a["w"]["off"], rowB=a["x"]["rowB"], kPer=kPer)
        assert nsl == s1 - s0
        parts = shard.all_gather_np(dist, y.reshape(nsl, N))
        if rank == 0:
            res["parts"] = parts.reshape(ns, N)
            res["sum"] = shard.sum_splits(res["parts"])
    finally:
        dist.destroy_process_group()


def _run(worker, world=2):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    with ctx.Manager() as man:
        res = man.dict()
        mp.start_processes(worker, args=(world, free_port(), res), nprocs=world, start_method="spawn", join=True)
        return dict(res)


def test_column_split_head_gloo():
    from oracle import ref
    got = _run(_column_worker)
    M, N, K, b, X, nw, st = _head_case()
    y, mx, _ = ref.gemvM(b, X, M, N, K, pro="rms", epi="softcap", norm=nw, stat=st, stat_off=0, stat_ld=1, cap=30.0)
    mx = mx[:M * N // 64 * 2]
    assert np.array_equal(got["y"].view(np.uint32), y.view(np.uint32))
    assert np.array_equal(got["mx"].view(np.uint32), mx.view(np.uint32))
    assert np.array_equal(got["arg"], shard.pick_argmax(mx, M))


def test_ksplit_down_gloo():
    from oracle import ref
    got = _run(_ksplit_worker)
    N, K, kPer = 512, 4096, 1024
    b, _ = ref.pack_q4(ref.randn(N * K, 310, 0.02), N, K)
    x = ref.randn(K, 311)
    y, _, ns = ref.gemv(b, x, N, K, kPer=kPer)
    assert np.array_equal(got["parts"].view(np.uint32), y.reshape(ns, N).view(np.uint32))
    assert np.array_equal(got["sum"].view(np.uint32), shard.sum_splits(y.reshape(ns, N)).view(np.uint32))
