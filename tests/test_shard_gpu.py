"""The batch-sharded launcher with real engines on two GPUs (skipped with fewer): one worker process
per GPU decodes its contiguous rows, and the concatenated steps equal, bit for bit, single-GPU runs of
the same row slices (same batch per engine, so the same kernels and the same arithmetic)."""

import pytest
import torch

from conftest import synth_state

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_sharded_engine_matches_per_shard_single_gpu_runs(tmp_path):
    import engine as E
    from decode_b200 import shard, synth

    state, cfg = synth_state(2)
    path = synth.write_checkpoint(str(tmp_path / "ckpt"), cfg, state=state)
    prompt = synth.random_prompt(6, 32, cfg["vocab_size"], seed=12)
    N = 12
    with shard.ShardedEngine(path, gpus=[0, 1], timeout=600) as eng:
        got = list(eng.generate(prompt, N))
    single = E.Engine.from_state_dict(state, cfg, "cuda:0")
    a = list(single.generate(prompt[:3], N))
    b = list(single.generate(prompt[3:], N))
    assert got == [x + y for x, y in zip(a, b)]
