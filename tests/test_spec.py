"""Host side of exact prompt-lookup speculative decoding (decode_b200/spec.py) on the CPU.

The draft index is checked against a brute-force restatement of the reference's rule
(engine/engine.py:776-808: the continuation of the latest earlier occurrence of the last 3-gram, else
2-gram, padded with the last token), also when the history grows by several tokens between lookups;
the loop against a toy deterministic "model" whose greedy continuation is known: speculation must
emit exactly the greedy tokens, and it must save verifies once the text repeats.
"""

import random
import time

import pytest

from decode_b200 import spec


def _brute_draft(seq, k):
    last, n = seq[-1], len(seq)
    p = None
    for j in range(n - 2, 1, -1):  # n-grams ending at j <= n - 2 (their continuation exists)
        if seq[j - 2:j + 1] == seq[-3:]:
            p = j + 1
            break
    if p is None:
        for j in range(n - 2, 0, -1):
            if seq[j - 1:j + 1] == seq[-2:]:
                p = j + 1
                break
    d = seq[p:p + k] if p is not None else []
    return d + [last] * (k - len(d))


@pytest.mark.parametrize("seed", range(20))
def test_draft_matches_brute_force_as_the_history_grows(seed):
    rnd = random.Random(seed)
    vocab = rnd.choice([3, 5, 12])
    seq = [rnd.randrange(vocab) for _ in range(rnd.randrange(2, 12))]
    drafter = spec.NgramDrafter(seq)
    for _ in range(25):
        k = rnd.randrange(1, 8)
        assert drafter.propose(k) == _brute_draft(seq, k)
        more = [rnd.randrange(vocab) for _ in range(rnd.randrange(1, 5))]
        seq.extend(more)
        drafter.extend(more)
        assert drafter.history == seq


def test_draft_without_history_pads_with_the_last_token():
    assert spec.NgramDrafter([7, 9]).propose(3) == [9, 9, 9]
    assert spec.NgramDrafter([4]).propose(2) == [4, 4]
    # 2-gram (1, 2) occurred: its continuation [3, 1] then padding
    assert spec.NgramDrafter([1, 2, 3, 1, 2]).propose(4) == [3, 1, 2, 2]
    # the 3-gram wins over a later 2-gram occurrence: (5, 1, 2) continues with 8, (1, 2) last with 3
    assert spec.NgramDrafter([5, 1, 2, 8, 1, 2, 3, 5, 1, 2]).propose(2) == [8, 1]


def test_verified_tokens_take_the_agreeing_drafts_and_the_next_greedy_token():
    assert spec.verified_tokens([5, 1, 2, 3], [1, 2, 3, 4]) == [1, 2, 3, 4]  # every draft stands
    assert spec.verified_tokens([5, 1, 2, 3], [1, 9, 3, 4]) == [1, 9]        # second draft rejected
    assert spec.verified_tokens([5, 1, 2, 3], [8, 2, 3, 4]) == [8]           # none stands: one token
    assert spec.verified_tokens([5, 1, 9, 3], [1, 2, 3, 4]) == [1, 2]        # a later match does not count


def _toy_next(prefix):
    """A deterministic 'model': greedy next token from the last two tokens (so the text cycles within
    25 steps)."""
    return (prefix[-1] * 2 + prefix[-2] + 1) % 5 if len(prefix) > 1 else 1


def _toy_verify(history):
    def verify(row, pos0):
        assert len(history) == pos0 + 1 and history[-1] == row[0]  # starts at the last emitted token
        pre = history[:pos0] + [row[0]]
        out = []
        for t in range(len(row)):
            out.append(_toy_next(pre))
            if t + 1 < len(row):
                pre = pre + [row[t + 1]]
        return out
    return verify


@pytest.mark.parametrize("k", [1, 3, 6])
@pytest.mark.parametrize("S,N", [(5, 1), (5, 2), (3, 40), (9, 100)])
def test_stream_emits_exactly_the_greedy_tokens(k, S, N):
    prompt = [(3 * i + 2) % 5 for i in range(S)]
    greedy = list(prompt)
    for _ in range(N):
        greedy.append(_toy_next(greedy))
    seq = prompt + [greedy[S]]
    stats = {}
    out = [greedy[S]] + list(spec.stream(seq, S, N, k, _toy_verify(seq), stats))
    assert out == greedy[S:S + N]
    assert stats["verifies"] <= max(0, N - 1)
    if N >= 100 and k >= 3:  # the toy text cycles: drafts from earlier cycles get accepted
        assert stats["verifies"] < (N - 1) / 2


def _long_next(prefix):
    """A 'model' whose text does not repeat for a long while: drafts (nearly) never match."""
    return (prefix[-1] * 31 + len(prefix) * 17 + 5) % 1009


def _verify_with(next_fn, history):
    def verify(row, pos0):
        assert len(history) == pos0 + 1 and history[-1] == row[0]
        pre, out = history[:pos0] + [row[0]], []
        for t in range(len(row)):
            out.append(next_fn(pre))
            if t + 1 < len(row):
                pre = pre + [row[t + 1]]
        return out
    return verify


def _step_with(next_fn, history):
    def step(tok, pos, n):
        assert len(history) == pos + 1 and history[-1] == tok
        for _ in range(n):
            yield next_fn(history)  # the caller appends each token before asking for the next
    return step


@pytest.mark.parametrize("next_fn,expect_plain", [(_long_next, True), (_toy_next, False)])
def test_gated_stream_falls_back_to_plain_steps_and_stays_exact(next_fn, expect_plain):
    """With the gate, rounds whose drafts keep failing become plain steps (so speculation costs little
    where it cannot help); where the text repeats, speculation keeps running. Either way the emitted
    tokens are the greedy ones."""
    S, N, k = 6, 300, 6
    prompt = [(5 * i + 1) % 5 for i in range(S)]
    greedy = list(prompt)
    for _ in range(N):
        greedy.append(next_fn(greedy))
    seq = prompt + [greedy[S]]
    stats = {}
    gate = spec.Gate(prior_cost=1.4)
    out = [greedy[S]] + list(spec.stream(seq, S, N, k, _verify_with(next_fn, seq), stats,
                                         step=_step_with(next_fn, seq), gate=gate))
    assert out == greedy[S:S + N]
    if expect_plain:
        assert stats["plain_steps"] > 0.8 * N and stats["verifies"] < 0.2 * N
    else:
        assert stats["plain_steps"] == 0


def test_gate_clock_excludes_the_consumers_time():
    """Plain steps are timed only while the step generator produces a token: a slow consumer between
    tokens must not make plain steps look expensive (which would bias the gate toward speculating)."""
    S, N, k = 6, 60, 4
    prompt = [(5 * i + 1) % 5 for i in range(S)]
    greedy = list(prompt)
    for _ in range(N):
        greedy.append(_long_next(greedy))
    seq = prompt + [greedy[S]]
    gate = spec.Gate(window=1, backoff=8, prior_cost=1.4)
    out = [greedy[S]]
    for tok in spec.stream(seq, S, N, k, _verify_with(_long_next, seq), {}, step=_step_with(_long_next, seq),
                           gate=gate):
        out.append(tok)
        time.sleep(0.002)  # the consumer's own work between tokens
    assert out == greedy[S:S + N]
    assert gate.n_step > 0 and gate.t_step / gate.n_step < 1e-3


def test_gate_backoff_doubles_and_resets():
    g = spec.Gate(window=2, backoff=4, max_backoff=16, prior_cost=1.5)
    assert g.verified(1, 1.0) == 0          # window not full yet
    assert g.verified(1, 1.0) == 4          # 1 token per verify < 1.5: four plain steps
    assert g.verified(1, 1.0) == 0
    assert g.verified(1, 1.0) == 8          # doubled
    assert g.verified(1, 1.0) == 0 and g.verified(1, 1.0) == 16 and g.verified(1, 1.0) == 0
    assert g.verified(1, 1.0) == 16         # capped
    assert g.verified(3, 1.0) == 0 and g.verified(3, 1.0) == 0  # pays again: back-off resets
    assert g.backoff == 4
    g.stepped(0.5)                           # measured: one verify = 1.0 / 0.5 = 2 steps
    assert abs(g.cost() - 2.0) < 1e-9
