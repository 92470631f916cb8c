"""Stand-in engines for the sharded launcher's CPU tests (imported by the spawned worker processes, so
it imports nothing heavy). The model path names the fault to plant: "fake" (none), or
"fake:<gpu>:<fault>:<step>" where the worker on that GPU raises, exits or stalls at that step."""

import os
import time


def token(row, t):
    """Deterministic 'greedy token' of a row at step t (depends on the row's own prompt only)."""
    return (sum(row) * 31 + len(row) * 7 + t * 13) % 151936


class FakeEngine:
    def __init__(self, fault):
        self.fault = fault

    def generate(self, rows, n):
        for t in range(n):
            if self.fault is not None and t == self.fault[1]:
                kind = self.fault[0]
                if kind == "raise":
                    raise RuntimeError("planted failure in the decode step")
                if kind == "exit":
                    os._exit(3)
                if kind == "stall":
                    time.sleep(60)
            yield [token(r, t) for r in rows]


def factory(model_path):
    parts = model_path.split(":")
    gpu = os.environ.get("CUDA_VISIBLE_DEVICES")
    if len(parts) == 4 and parts[1] == gpu:
        if parts[2] == "build":
            raise RuntimeError("planted failure while loading the checkpoint")
        return FakeEngine((parts[2], int(parts[3])))
    return FakeEngine(None)
