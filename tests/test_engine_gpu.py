"""End-to-end parity of the decode engine against the reference, on the GPU.

Parity rule: per-step logits agree within max-abs 5e-2 after softmax
normalisation, and greedy tokens are identical up to any step where the reference's own top-2 gap
is below that tolerance. Logits are compared teacher-forced: the oracle (the reference's tier-1
arithmetic on CPU) is fed this engine's own tokens, so a legitimate near-tie flip does not cascade
(the reference's own check, engine/engine.py:974-996).

Two bounds are checked per step, over all 151,936 entries:
  * softmax probabilities: max-abs <= TOL (5e-2), the north star's rule as written;
  * log-softmax (raw logits minus log-sum-exp): max-abs <= max(TOL, 2 x the reference's own
    self-drift). The reference's cached decode and its own full-forward replay of the same tokens
    already differ by up to 0.0626 on config 0 (recorded in tests/golden/*.json "self_drift" by
    running the reference engine): BF16 logits near 4-8 have a 0.031 ulp, and one rounding flip
    at the LM head moves a logit by that much. 5e-2 on log-softmax is below the reference's own
    noise floor, so the bound is twice that floor.
"""

import pytest
import torch

from conftest import load_golden, synth_state
from oracle import qwen3_cpu as Q

pytestmark = pytest.mark.gpu
TOL = 5e-2


@pytest.fixture(scope="module")
def engines():
    import engine as E

    cache = {}

    def get(n_layers):
        if n_layers not in cache:
            state, cfg = synth_state(n_layers)
            cache[n_layers] = (E.Engine.from_state_dict(state, cfg, "cuda:0"), state, cfg)
        return cache[n_layers]

    return get


def _golden_token_ok(tok, step, row):
    """Tie rule against the golden top-8 of the reference's native run."""
    vals, ids = step["top_vals"][row], step["top_ids"][row]
    best = vals[0]
    if tok in ids and vals[ids.index(tok)] == best:
        return True
    return (best - vals[1]) < TOL and tok in ids and vals[ids.index(tok)] >= best - TOL


@pytest.mark.parametrize("case", ["config0", "b3_s17"])
def test_generate_matches_reference_golden(engines, case):
    g = load_golden(case)
    eng, state, cfg = engines(g["spec"]["layers"])
    steps = list(eng.generate(g["prompt"], g["spec"]["new"]))
    assert len(steps) == g["spec"]["new"] and all(len(s) == len(g["prompt"]) for s in steps)
    toks = [list(r) for r in zip(*steps)]
    ref = g["native"]["tokens"]
    for b in range(len(ref)):
        for t in range(len(ref[b])):
            if toks[b][t] != ref[b][t]:
                # allowed only at a reference near-tie; after a flip the prefixes differ, stop here
                assert _golden_token_ok(toks[b][t], g["native"]["steps"][t], b), (case, b, t)
                break


@pytest.mark.parametrize("case", ["config0", "b3_s17"])
def test_teacher_forced_logits_within_tolerance(engines, case):
    g = load_golden(case)
    eng, state, cfg = engines(g["spec"]["layers"])
    N = g["spec"]["new"]
    toks, logits = eng.generate_with_logits(g["prompt"], N)
    orc = Q.Qwen3Oracle(state, cfg)
    _, ref_logits = orc.generate(g["prompt"], N, forced=toks)
    lsm_bound = max(TOL, 2 * g["self_drift"]["max_logsoftmax_diff"])
    worst_lsm = worst_p = 0.0
    for t in range(N):
        worst_lsm = max(worst_lsm, Q.log_softmax_maxdiff(logits[t], ref_logits[t]))
        worst_p = max(worst_p, Q.softmax_maxdiff(logits[t], ref_logits[t]))
        for b in range(len(toks)):
            assert Q.token_ok(toks[b][t], ref_logits[t][b], TOL), (case, t, b)
    print(f"{case}: max |softmax diff| {worst_p:.2e}, max |log-softmax diff| {worst_lsm:.4f} "
          f"(bound {lsm_bound:.4f}; reference self-drift {g['self_drift']['max_logsoftmax_diff']:.4f})")
    assert worst_p <= TOL
    assert worst_lsm <= lsm_bound, f"max |log_softmax diff| {worst_lsm:.4f} > {lsm_bound:.4f}"


def test_graph_and_eager_paths_agree_and_are_deterministic(engines):
    g = load_golden("config0")
    eng, _, _ = engines(4)
    a = list(eng.generate(g["prompt"], g["spec"]["new"]))
    b = list(eng.generate(g["prompt"], g["spec"]["new"]))
    toks, _ = eng.generate_with_logits(g["prompt"], g["spec"]["new"])
    assert a == b
    assert [list(r) for r in zip(*a)] == toks


def test_consecutive_generates_reset_state(engines):
    """A second prompt of the same shape gives the same tokens as on a fresh state (engine/engine.py:725-727)."""
    from decode_b200 import synth

    eng, _, cfg = engines(2)
    p1 = synth.random_prompt(2, 24, cfg["vocab_size"], seed=21)
    p2 = synth.random_prompt(2, 24, cfg["vocab_size"], seed=22)
    first = list(eng.generate(p2, 6))
    list(eng.generate(p1, 6))
    again = list(eng.generate(p2, 6))
    assert first == again
    eng.state = None
    fresh = list(eng.generate(p2, 6))
    assert fresh == first


def test_poisoned_cache_slots_are_never_read(engines):
    """NaN in every cache slot the step must not read leaves the tokens unchanged."""
    from decode_b200 import synth

    eng, _, cfg = engines(2)
    p = synth.random_prompt(1, 40, cfg["vocab_size"], seed=31)
    ref = list(eng.generate(p, 8))
    st = eng.state
    st.k_all.fill_(float("nan"))
    st.v_all.fill_(float("nan"))
    again = list(eng.generate(p, 8))
    assert again == ref


def test_contract_step_counts(engines):
    from decode_b200 import synth

    eng, _, cfg = engines(2)
    p = synth.random_prompt(1, 8, cfg["vocab_size"], seed=1)
    assert list(eng.generate(p, 0)) == []
    one = list(eng.generate(p, 1))
    assert len(one) == 1 and len(one[0]) == 1
