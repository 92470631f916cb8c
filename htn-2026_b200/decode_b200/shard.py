"""Batch-sharded decoding over several GPUs of one node, behind the same `generate` contract.

Greedy decode of independent sequences needs no communication between GPUs: each GPU holds a full
replica of the weights and decodes its own rows. `ShardedEngine` starts one worker process per GPU
(CUDA_VISIBLE_DEVICES set to that GPU before the worker imports torch), hands worker g the contiguous
rows [g * B / G, (g + 1) * B / G) of every request, and yields, per step, the workers' token lists
concatenated in input order - exactly what `Engine.generate` yields for the whole batch. There is no
collective and no GPU-to-GPU traffic; the host pipes carry B token ids per step.

Failure handling is on the host. A worker that raises sends the exception text back and the caller's
`generate` raises `ShardError` naming the worker; a worker that exits, or sends nothing for `timeout`
seconds, is detected while the parent waits on its pipe, and `generate` raises `ShardError` as well.
After any failure every worker is stopped (the GPUs are released by the workers' exit), and the
engine refuses further requests.

The reference engine is single-GPU (engine/engine.py:70); this is the multi-GPU form of its contract.
"""

from __future__ import annotations

import multiprocessing as mp
import os
import time
import traceback


class ShardError(RuntimeError):
    """A worker failed (raised, exited or stopped answering); the sharded engine is closed."""


def _build_engine(model_path: str):
    import engine as E

    return E.Engine(model_path, "cuda:0")


def _worker(conn, gpu, model_path, factory):
    """Worker main: build the engine once, then serve requests until told to stop. Messages out:
    ("ready",), ("step", tokens), ("done",), ("error", text)."""
    if gpu is not None:
        os.environ["CUDA_VISIBLE_DEVICES"] = str(gpu)
    try:
        eng = (factory or _build_engine)(model_path)
        conn.send(("ready",))
    except BaseException:
        conn.send(("error", traceback.format_exc(limit=8)))
        return
    while True:
        msg = conn.recv()
        if msg[0] == "stop":
            return
        _, rows, n = msg
        try:
            for step in eng.generate(rows, n):
                conn.send(("step", list(step)))
            conn.send(("done",))
        except BaseException:
            conn.send(("error", traceback.format_exc(limit=8)))
            return


def split_rows(batch: int, shards: int) -> list[tuple[int, int]]:
    """Contiguous row ranges [lo, hi) for `shards` workers, sizes differing by at most one (the first
    batch % shards workers take the extra row); empty ranges are dropped."""
    base, extra = divmod(batch, shards)
    out, lo = [], 0
    for g in range(shards):
        hi = lo + base + (1 if g < extra else 0)
        if hi > lo:
            out.append((lo, hi))
        lo = hi
    return out


class ShardedEngine:
    """`Engine`'s contract over several GPUs: ShardedEngine(model_path, gpus=[0, 1, ...]).generate(ids, n).

    `factory(model_path)` builds the per-worker engine (default: `Engine(model_path, "cuda:0")` inside the
    worker, which sees only its own GPU); it must be a picklable top-level callable. `timeout` bounds
    the wait for any one message from a worker (engine build included), in seconds."""

    def __init__(self, model_path: str, gpus=None, timeout: float = 600.0, factory=None, start_method: str = "spawn"):
        if gpus is None:
            import torch

            gpus = list(range(torch.cuda.device_count()))
        if not gpus:
            raise ValueError("no GPUs to shard over")
        self.gpus, self.timeout = list(gpus), float(timeout)
        ctx = mp.get_context(start_method)
        self.procs, self.conns = [], []
        self.closed = False
        for gpu in self.gpus:
            parent, child = ctx.Pipe()
            p = ctx.Process(target=_worker, args=(child, gpu, model_path, factory), daemon=True)
            p.start()
            child.close()
            self.procs.append(p)
            self.conns.append(parent)
        for g in range(len(self.gpus)):
            self._expect(g, "ready")

    # ------------------------------------------------------------------ plumbing
    def _recv(self, g: int):
        """Next message of worker g; raises ShardError when the worker exits or stays silent too long."""
        conn, proc = self.conns[g], self.procs[g]
        deadline = time.monotonic() + self.timeout
        while True:
            left = deadline - time.monotonic()
            if left <= 0:
                self._fail(f"worker {g} (GPU {self.gpus[g]}) sent nothing for {self.timeout:g} s")
            try:
                if conn.poll(min(left, 0.05)):
                    return conn.recv()
            except (EOFError, OSError):
                self._fail(f"worker {g} (GPU {self.gpus[g]}) closed its pipe (exit code {proc.exitcode})")
            if not proc.is_alive() and not conn.poll(0):
                self._fail(f"worker {g} (GPU {self.gpus[g]}) exited with code {proc.exitcode}")

    def _expect(self, g: int, kind: str):
        msg = self._recv(g)
        if msg[0] == "error":
            self._fail(f"worker {g} (GPU {self.gpus[g]}) raised:\n{msg[1]}")
        if msg[0] != kind:
            self._fail(f"worker {g} (GPU {self.gpus[g]}) sent {msg[0]!r}, expected {kind!r}")
        return msg

    def _fail(self, why: str):
        self.close()
        raise ShardError(why)

    # ------------------------------------------------------------------ API
    def generate(self, input_ids: list[list[int]], max_new_tokens: int):
        if self.closed:
            raise ShardError("sharded engine is closed (a worker failed or close() was called)")
        N = int(max_new_tokens)
        if N <= 0:
            return
        B = len(input_ids)
        if B < 1 or any(len(r) != len(input_ids[0]) for r in input_ids) or not input_ids[0]:
            raise ValueError("input_ids must be a non-empty batch of equal-length rows")
        ranges = split_rows(B, len(self.gpus))
        for g, (lo, hi) in enumerate(ranges):
            self.conns[g].send(("run", [list(r) for r in input_ids[lo:hi]], N))
        for _ in range(N):
            step = []
            for g, (lo, hi) in enumerate(ranges):
                toks = self._expect(g, "step")[1]
                if len(toks) != hi - lo:
                    self._fail(f"worker {g} returned {len(toks)} tokens for {hi - lo} rows")
                step.extend(toks)
            yield step
        for g in range(len(ranges)):
            self._expect(g, "done")

    def close(self) -> None:
        if self.closed:
            return
        self.closed = True
        for conn in self.conns:
            try:
                conn.send(("stop",))
            except (OSError, ValueError):
                pass
        for p in self.procs:
            p.join(timeout=5)
            if p.is_alive():
                p.terminate()
                p.join(timeout=5)
            if p.is_alive():
                p.kill()
                p.join()
        for conn in self.conns:
            conn.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
