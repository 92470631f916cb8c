"""The drop-in constructor `Engine(model_path)` on the GPU (the platform's call; the reference's load is
engine/engine.py:237-282): a Hugging Face directory written once as a single model.safetensors and
once as two shards with model.safetensors.index.json decodes exactly as the engine built from the same
tensors in memory, and follows the reference's recorded tokens (tests/golden/config0.json) under the
tie rule."""

import pytest

import parity as P
from conftest import load_golden, synth_state

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shards", [1, 2])
def test_engine_from_checkpoint_directory(tmp_path, shards):
    import engine as E
    from decode_b200 import synth

    g = load_golden("config0")
    state, cfg = synth_state(g["spec"]["layers"])
    path = synth.write_checkpoint(str(tmp_path / f"ckpt{shards}"), cfg, state=state, shards=shards)
    eng = E.Engine(path, "cuda:0")
    assert eng.n_layers == 4 and eng.vocab == cfg["vocab_size"]
    N = g["spec"]["new"]
    steps = list(eng.generate(g["prompt"], N))
    ref_eng = E.Engine.from_state_dict(state, cfg, "cuda:0")
    assert steps == list(ref_eng.generate(g["prompt"], N))
    toks = [list(r) for r in zip(*steps)]
    tol = max(P.TOL, 2 * g["self_drift"]["max_logsoftmax_diff"])
    where = P.first_divergence(toks, g["native"]["tokens"])[0]
    if where is not None:
        assert P.golden_token_ok(toks[0][where], g["native"]["steps"][where], 0, tol), where
