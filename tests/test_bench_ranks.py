"""bench.py's multi-rank host logic on the CPU: the reduction over ranks that the torchrun launch uses
for its timings (max of the per-rank device times; min of the per-rank end-to-end rates), run on two
`gloo` ranks, and the reference arm's rule that only rank 0 works and prints. No GPU is used."""

import argparse
import datetime
import multiprocessing as mp
import os
import socket

import bench


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_worker(rank: int, world: int, port: int, out) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        x = 1.5 + 2.0 * rank  # rank 0: 1.5, rank 1: 3.5
        out.put((rank, bench.rank_reduce(x, "max", "cpu"), bench.rank_reduce(x, "min", "cpu")))
    finally:
        dist.destroy_process_group()


def test_rank_reduce_without_a_process_group_is_the_value_itself():
    assert bench.rank_reduce(2.25, "max", "cpu") == 2.25
    assert bench.rank_reduce(2.25, "min", "cpu") == 2.25


def test_rank_reduce_over_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_worker, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        got = sorted(out.get(timeout=120) for _ in procs)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert got == [(0, 3.5, 1.5), (1, 3.5, 1.5)]  # every rank sees the same max and min
    assert all(p.exitcode == 0 for p in procs)


def test_reference_arm_runs_on_rank_0_only(monkeypatch, capsys):
    monkeypatch.setenv("RANK", "1")
    a = argparse.Namespace(layers=36, batch=1, prompt=128, steps=3, warmup=3, cpu_steps=96, gpus=2)
    assert bench.run_reference(a) is None  # returns before building the model
    assert capsys.readouterr().out == ""
