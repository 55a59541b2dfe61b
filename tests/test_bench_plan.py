"""bench.py's plan of a sweep step over N ranks (CPU only): every call of the step is covered once, the head calls
cut into whole 64-row tiles, the units placed so that no rank pays a head call's fixed cost more than once per step
from four ranks on."""
import collections
import importlib.util
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def load_bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("ws", [1, 2, 3, 4, 8])
def test_plan_covers_every_call_once(ws):
    b = load_bench()
    plan = b.plan_calls(ws)
    rows = collections.Counter()
    for u in plan:
        assert 0 <= u["rank"] < ws
        assert u["rows"] % 64 == 0
        rows[(u["Nfull"], u["M"])] += u["rows"]
    assert set(rows) == {(N, M) for N in b.NS for M in b.MS}
    assert all(rows[(N, M)] == N for N, M in rows)
    # the step's bytes do not depend on the split
    assert b.step_bytes() == sum(b.gemv_bytes(M, N, b.K, N == b.HEAD_N) for N in b.NS for M in b.MS)


def test_plan_head_units_per_rank():
    b = load_bench()
    per = lambda ws: collections.Counter(u["rank"] for u in b.plan_calls(ws) if u["head"])
    # one rank: the four head calls whole; two ranks: half of every head call each; four: one whole head call each;
    # eight: one half each
    assert per(1) == {0: 4}
    assert per(2) == {0: 4, 1: 4} and all(u["rows"] == b.HEAD_N // 2 for u in b.plan_calls(2) if u["head"])
    assert per(4) == {r: 1 for r in range(4)} and all(u["rows"] == b.HEAD_N for u in b.plan_calls(4) if u["head"])
    assert per(8) == {r: 1 for r in range(8)} and all(u["rows"] == b.HEAD_N // 2 for u in b.plan_calls(8) if u["head"])
    # every rank computes the same plan
    assert b.plan_calls(8) == b.plan_calls(8)
