"""bench.py's host-side contract on the CPU: the reduction over ranks that the torchrun launch uses for
its timings (max of the per-rank device times; min of the per-rank end-to-end rates), run on two
`gloo` ranks; the reference arm's rule that only rank 0 works and prints; and the reference arm's one
JSON line on a one-layer model. No GPU is used."""

import argparse
import datetime
import json
import multiprocessing as mp
import os
import socket
import subprocess
import sys

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


def test_reference_arm_prints_one_contract_line():
    """`bench.py --impl reference` (the host-core arm the driver runs beside ours) on a one-layer model:
    exactly one JSON line with the contract's keys, its cpu_baseline and e2e describing the same run."""
    cmd = [sys.executable, os.path.join(os.path.dirname(bench.__file__), "bench.py"), "--impl", "reference",
           "--layers", "1", "--prompt", "8", "--steps", "2", "--warmup", "1", "--cpu-steps", "2"]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300, env={**os.environ, "RANK": "0"})
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["metric"] == bench.METRIC and d["higher_is_better"] is True
    assert d["steps"] == 2 and d["warmup"] == 1 and d["value"] > 0
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
