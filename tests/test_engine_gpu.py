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
The tie rule for tokens uses the same calibrated bound: a token may differ from the reference argmax
only where the reference's own top-2 gap is below it. The oracle runs on the test host's CPU, whose
BF16 matmul kernels can round differently from the machine the golden vectors came from, so the
reference side of the comparison carries that same ulp-level noise.
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


def _golden_token_ok(tok, step, row, tol):
    """Tie rule against the golden top-8 of the reference's native run."""
    vals, ids = step["top_vals"][row], step["top_ids"][row]
    best = vals[0]
    if tok in ids and vals[ids.index(tok)] == best:
        return True
    return (best - vals[1]) < tol and tok in ids and vals[ids.index(tok)] >= best - tol


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
                tol = max(TOL, 2 * g["self_drift"]["max_logsoftmax_diff"])
                assert _golden_token_ok(toks[b][t], g["native"]["steps"][t], b, tol), (case, b, t)
                break


@pytest.mark.parametrize("T", [3, 7])
def test_speculative_generate_matches_reference_golden(engines, T):
    """Exact prompt-lookup speculation (batch 1, verify width T): the emitted tokens follow the
    reference's greedy tokens under the same tie rule as plain decoding."""
    g = load_golden("config0")
    eng, state, cfg = engines(g["spec"]["layers"])
    eng.speculate = T
    try:
        steps = list(eng.generate(g["prompt"], g["spec"]["new"]))
        assert eng.state.verify is not None and eng.state.verify.T == T
    finally:
        eng.speculate = 0
        eng.state = None
    assert len(steps) == g["spec"]["new"] and all(len(s) == 1 for s in steps)
    toks, ref = [s[0] for s in steps], g["native"]["tokens"][0]
    tol = max(TOL, 2 * g["self_drift"]["max_logsoftmax_diff"])
    for t in range(len(ref)):
        if toks[t] != ref[t]:
            assert _golden_token_ok(toks[t], g["native"]["steps"][t], 0, tol), (T, t)
            break


@pytest.mark.parametrize("T", [2, 4, 8])
def test_speculative_matches_plain_greedy(engines, T):
    """Speculation emits the plain greedy tokens of this engine (a repetitive prompt, so drafts get
    accepted): identical up to any step where the plain run's own top-2 logit gap is a near-tie."""
    from decode_b200 import synth

    eng, _, cfg = engines(2)
    base = synth.random_prompt(1, 12, cfg["vocab_size"], seed=5)[0]
    prompt = [base * 4]
    N = 48
    eng.state = None
    plain, logits = eng.generate_with_logits(prompt, N)
    eng.state = None
    eng.speculate = T
    try:
        steps = list(eng.generate(prompt, N))
        verifies = eng.state.spec_stats["verifies"]
    finally:
        eng.speculate = 0
        eng.state = None
    toks = [s[0] for s in steps]
    assert len(toks) == N and 1 <= verifies <= N - 1
    # the verify forward is other kernels (GEMV rows, prompt attention): a flip is allowed only where the
    # plain run's top-2 gap is within the calibrated bound of the golden tests
    tol = max(TOL, 2 * load_golden("config0")["self_drift"]["max_logsoftmax_diff"])
    for t in range(N):
        if toks[t] != plain[0][t]:
            top2 = logits[t][0].float().topk(2).values
            assert float(top2[0] - top2[1]) <= tol, (T, t)
            break


def test_speculation_gate_falls_back_to_plain_steps(engines):
    """On a uniform-random prompt drafts are rarely accepted: the gate hands most tokens to plain decode
    steps on the same cache, and the emitted tokens stay this engine's plain greedy tokens (up to a
    near-tie flip of the plain run)."""
    from decode_b200 import synth

    eng, _, cfg = engines(2)
    prompt = synth.random_prompt(1, 40, cfg["vocab_size"], seed=9)
    N = 96
    eng.state = None
    plain, logits = eng.generate_with_logits(prompt, N)
    eng.state = None
    eng.speculate = 4
    try:
        toks = [s[0] for s in eng.generate(prompt, N)]
        stats = dict(eng.state.spec_stats)
    finally:
        eng.speculate = 0
        eng.state = None
    assert len(toks) == N and stats["verifies"] >= 4
    if stats["verifies"] * 2 > N:  # drafts kept paying: nothing to fall back from
        pytest.skip(f"drafts accepted on this prompt ({stats})")
    assert stats["plain_steps"] > 0
    tol = max(TOL, 2 * load_golden("config0")["self_drift"]["max_logsoftmax_diff"])
    for t in range(N):
        if toks[t] != plain[0][t]:
            top2 = logits[t][0].float().topk(2).values
            assert float(top2[0] - top2[1]) <= tol, t
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
            if not Q.token_ok(toks[b][t], ref_logits[t][b], lsm_bound):
                rv, ri = ref_logits[t][b].float().topk(3)
                ours = logits[t][b].float()
                raise AssertionError(
                    f"{case} step {t} row {b}: token {toks[b][t]} (ref logit "
                    f"{float(ref_logits[t][b][toks[b][t]]):.4f}, ours {float(ours[toks[b][t]]):.4f}); ref top3 "
                    f"{list(zip(ri.tolist(), [round(v, 4) for v in rv.tolist()]))}, ours at those "
                    f"{[round(float(ours[i]), 4) for i in ri.tolist()]}")
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


def test_prefill_row_chunks_are_bit_identical(engines, monkeypatch):
    """A prompt batch over one prefill chunk (at most 16384 tokens per chunk, engine/engine.py:79, :189)
    runs as several chunks of whole sequences. Every prompt kernel is row-independent and deterministic,
    so the first-token logits, the cache and the decoded logits equal the one-chunk run's bit for bit.
    The GEMMs' K split is chosen from the chunk's token count (it changes the fp32 summation order), so
    it is pinned to none here."""
    import engine as E
    from decode_b200 import synth

    monkeypatch.setenv("QD_GEMM_KSPLIT", "1")
    eng, _, cfg = engines(2)
    p = synth.random_prompt(5, 40, cfg["vocab_size"], seed=41)
    eng.state = None
    toks1, lg1 = eng.generate_with_logits(p, 3)
    assert eng.state.chunks == [(0, 5)]
    k1, v1 = eng.state.k_all[:, :, :, :40].clone(), eng.state.v_all[:, :, :, :40].clone()
    monkeypatch.setattr(E, "PREFILL_TOKENS", 100)  # 2 sequences of 40 tokens per chunk: 3 chunks
    eng.state = None
    toks2, lg2 = eng.generate_with_logits(p, 3)
    assert eng.state.chunks == [(0, 2), (2, 4), (4, 5)]
    assert toks1 == toks2
    assert all(torch.equal(a, b) for a, b in zip(lg1, lg2))
    assert torch.equal(k1, eng.state.k_all[:, :, :, :40]) and torch.equal(v1, eng.state.v_all[:, :, :, :40])
    eng.state = None


def test_contract_step_counts(engines):
    from decode_b200 import synth

    eng, _, cfg = engines(2)
    p = synth.random_prompt(1, 8, cfg["vocab_size"], seed=1)
    assert list(eng.generate(p, 0)) == []
    one = list(eng.generate(p, 1))
    assert len(one) == 1 and len(one[0]) == 1


def test_persistent_step_matches_per_op_kernels_bit_exactly():
    """The persistent step kernel runs the per-op kernels' arithmetic with the same partitions: same
    tokens and bit-identical logits."""
    import engine as E

    g = load_golden("config0")
    state, cfg = synth_state(4)
    out = {}
    for mode in ("persistent", "kernels"):
        old = E.STEP_MODE
        E.STEP_MODE = mode
        try:
            eng = E.Engine.from_state_dict(state, cfg, "cuda:0")
            toks, logits = eng.generate_with_logits(g["prompt"], 12)
            steps = list(eng.generate(g["prompt"], 12))
        finally:
            E.STEP_MODE = old
        assert [list(r) for r in zip(*steps)] == toks
        out[mode] = (toks, logits)
        del eng
    assert out["persistent"][0] == out["kernels"][0]
    for a, b in zip(out["persistent"][1], out["kernels"][1]):
        assert torch.equal(a, b)


def test_persistent_step_long_cache_uses_both_attention_teams():
    """A cache long enough that attention has more units than SMs, so the second 4-warp team of each
    CTA runs units too (cap 740 -> 24 splits x 8 KV heads = 192 units): same tokens and logits as
    the per-op kernels."""
    import engine as E
    from decode_b200 import synth

    state, cfg = synth_state(2)
    prompt = synth.random_prompt(1, 100, cfg["vocab_size"], seed=41)
    out = {}
    for mode in ("persistent", "kernels"):
        old = E.STEP_MODE
        E.STEP_MODE = mode
        try:
            eng = E.Engine.from_state_dict(state, cfg, "cuda:0")
            st = eng._build(1, 100, 640)
            if mode == "persistent":
                assert st.step.splits * 8 > eng.sm_count
            toks, logits = eng.generate_with_logits(prompt, 640)
        finally:
            E.STEP_MODE = old
        out[mode] = (toks, logits[-8:])
        del eng
    assert out["persistent"][0] == out["kernels"][0]
    for a, b in zip(out["persistent"][1], out["kernels"][1]):
        assert torch.equal(a, b)
