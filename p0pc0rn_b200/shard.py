"""Multi-GPU sharding of the matmul path: one process per GPU, torch.distributed (NCCL over NVLink on B200, gloo on
CPU) for the exchange, libp0mm.so for the compute. Nothing here changes the arithmetic of a call, so a sharded result
equals the one-GPU result of the same call.

* Column split (lm_head, FFN gate/up): rank r owns whole 64-row tiles, rows [n0, n1), which are one contiguous run of
  q4g32a.t64 records (engine/kcheck.js:22-38), so its weight is a sub-view of the packed buffer. Each rank writes its
  logits and per-tile (max, argmax) pairs; after an all-gather the argmax indices are rebased to global rows, and the
  argmax is the one-GPU argmax because the tie rule (lowest index, llm/lops.js:95-102) is on the global index.
* K split (FFN down projection): the reference's split-K contract (Y[split*ldy + n], llm/lops.js:93) summed by
  normadd in split order (llm/lops.js:155: v = 0; v += T[j] for j = 0..nsrc-1). Rank r owns whole kPer slices
  [s0, s1); its call is the reference's own gemv with the weight view moved by s0*kPer/32 records and x.rowB moved by
  s0*kPer, so the partials are the one-GPU partials bit for bit, and so is their split-order sum after an all-gather.
* Row split (DiT GEMM): rank r owns token rows [m0, m1) with the weights replicated; no exchange.
"""
import numpy as np

TILE = 64
REC = 1280   # bytes per q4g32a.t64 record (64 rows x 32 k)


def tile_range(N, world, rank):
    """rows [n0, n1) of rank `rank`: equal runs of whole 64-row tiles (all-gathers need equal shards)"""
    if N % TILE or (N // TILE) % world:
        raise ValueError("column split: N %d is not a multiple of 64 x %d ranks" % (N, world))
    per = N // world
    return rank * per, (rank + 1) * per


def row_range(M, world, rank):
    """token rows [m0, m1) of rank `rank` (ceil split; the last ranks may hold fewer or none)"""
    per = -(-M // world)
    m0 = min(M, rank * per)
    return m0, min(M, m0 + per)


def split_range(nsplit, world, rank):
    """k-split slices [s0, s1) of rank `rank` (equal counts; the reference's kPer slices stay whole)"""
    if nsplit % world:
        raise ValueError("k split: %d slices over %d ranks" % (nsplit, world))
    per = nsplit // world
    return rank * per, (rank + 1) * per


def column_view(w, n0, n1):
    """the sub-view of a q4g32a.t64 weight view holding rows [n0, n1) (whole tiles)"""
    if w["enc"] != "q4g32a.t64" or n0 % TILE or n1 % TILE:
        raise ValueError("column view: whole 64-row tiles of a q4g32a.t64 weight")
    G = w["cols"] // 32
    return dict(w, off=w.get("off", 0) + (n0 // TILE) * G * REC, rows=n1 - n0, bytes=(n1 - n0) // TILE * G * REC)


def kslice_args(a, kPer, s0, s1):
    """the gemv / gemvM argument object computing k-split slices [s0, s1) of call `a` (its kPer slices) as slices
    0 .. s1-s0-1 of a call over K' = (s1 - s0) * kPer: the weight view starts s0*kPer/32 records later (its cols, and so
    its tile stride, unchanged) and x starts s0*kPer elements later"""
    K = a["K"]
    k0, k1 = s0 * kPer, min(K, s1 * kPer)
    if kPer % 32 or k0 >= K:
        raise ValueError("k slice: kPer %d, slices [%d, %d) of K %d" % (kPer, s0, s1, K))
    w = dict(a["w"])
    w["off"] = w.get("off", 0) + (k0 // 32) * REC
    w.pop("bytes", None)
    x = dict(a["x"])
    x["rowB"] = x.get("rowB", 0) + k0
    return dict(a, w=w, x=x, K=k1 - k0, kPer=kPer)


def sum_splits(parts):
    """the split partials [nsplit][...] summed in split order in f32, as normadd does (llm/lops.js:155)"""
    parts = np.asarray(parts, np.float32)
    acc = np.zeros(parts.shape[1:], np.float32)
    for p in parts:
        acc = (acc + p).astype(np.float32)
    return acc


def rebase_mx(mx, n0):
    """per-tile (max, bitcast argmax) pairs of a rank's rows [n0, ...) -> global row indices (a copy)"""
    out = np.array(mx, dtype=np.float32, copy=True)
    idx = out.view(np.uint32)
    idx[..., 1::2] += np.uint32(n0)
    return out


def merge_mx(gathered, world, M, nt_local, starts):
    """all-gathered [world][M][nt_local * 2] pairs -> the one-GPU layout MX[(m * ntile + tile) * 2] with global indices"""
    g = np.asarray(gathered, np.float32).reshape(world, M, nt_local * 2)
    parts = [rebase_mx(g[r], starts[r]) for r in range(world)]
    return np.concatenate(parts, axis=1).reshape(-1)


def pick_argmax(mx, M):
    """argmaxM over per-tile pairs (llm/lops_spec.js:346-368): per row m the largest max, ties to the lowest index.
    Returns [M][2] uint32 = (index, bits of the max)."""
    pairs = np.asarray(mx, np.float32).reshape(M, -1, 2)
    out = np.zeros((M, 2), np.uint32)
    for m in range(M):
        v = pairs[m, :, 0]
        i = pairs[m, :, 1].view(np.uint32)
        best = np.max(v)
        out[m, 0] = i[v == best].min()
        out[m, 1] = np.float32(best).view(np.uint32)
    return out


def all_gather_np(dist, arr):
    """all-gather a numpy array through torch.distributed (any backend) -> [world, *arr.shape]"""
    import torch
    t = torch.from_numpy(np.ascontiguousarray(arr))
    if dist.get_backend() == "nccl":
        t = t.to(torch.device("cuda", torch.cuda.current_device()))
    outs = [torch.empty_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(outs, t)
    return np.stack([o.cpu().numpy() for o in outs])
