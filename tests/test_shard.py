"""The batch-sharded launcher (decode_b200/shard.py) on the CPU with two worker processes and stand-in
engines (tests/shard_fakes.py): per-step lists concatenated in input order, uneven splits, and the
host-side detection of a worker that raises, exits or stops answering - each turned into an exception
in the caller. No GPU is used."""

import pytest

import shard_fakes as F
from decode_b200 import shard


def _expected(rows, n):
    return [[F.token(r, t) for r in rows] for t in range(n)]


def test_split_rows_is_contiguous_and_even():
    assert shard.split_rows(64, 8) == [(8 * g, 8 * g + 8) for g in range(8)]
    assert shard.split_rows(5, 2) == [(0, 3), (3, 5)]
    assert shard.split_rows(1, 4) == [(0, 1)]
    r = shard.split_rows(37, 4)
    assert r[0][0] == 0 and r[-1][1] == 37 and all(a[1] == b[0] for a, b in zip(r, r[1:]))
    assert max(h - l for l, h in r) - min(h - l for l, h in r) <= 1


def test_two_workers_concatenate_steps_in_input_order():
    rows = [[i, i + 1, 2 * i] for i in range(5)]
    with shard.ShardedEngine("fake", gpus=[0, 1], timeout=60, factory=F.factory) as eng:
        assert list(eng.generate(rows, 6)) == _expected(rows, 6)
        assert list(eng.generate(rows[:1], 3)) == _expected(rows[:1], 3)  # one row: the second worker idles
        assert list(eng.generate(rows, 0)) == []


@pytest.mark.parametrize("fault,match", [("raise", "planted failure in the decode step"),
                                         ("exit", "exit"), ("stall", "sent nothing")])
def test_a_failing_worker_becomes_an_error_in_the_caller(fault, match):
    rows = [[i, 3 * i] for i in range(4)]
    eng = shard.ShardedEngine(f"fake:1:{fault}:2", gpus=[0, 1], timeout=3, factory=F.factory)
    got = []
    with pytest.raises(shard.ShardError, match=match):
        for step in eng.generate(rows, 5):
            got.append(step)
    assert got == _expected(rows, 2)  # the steps before the failure were delivered intact
    assert all(not p.is_alive() for p in eng.procs)
    with pytest.raises(shard.ShardError, match="closed"):
        list(eng.generate(rows, 1))


def test_a_worker_that_fails_to_load_fails_the_constructor():
    with pytest.raises(shard.ShardError, match="loading the checkpoint"):
        shard.ShardedEngine("fake:0:build:0", gpus=[0, 1], timeout=60, factory=F.factory)
