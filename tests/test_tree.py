"""Host side of exact token-tree speculation (decode_b200/tree.py) on the CPU.

The trie's invariants (shared prefixes reuse nodes, parents precede children, index >= depth, ancestor
masks), the walk that accepts drafts, the K/V compaction order, the drafter's candidate sources, and
the loop against toy deterministic "models": the emitted tokens must be exactly the greedy tokens,
and repetitive text must take fewer verifies than tokens.
"""

import random

import pytest

from decode_b200 import spec, tree as T


def test_insert_shares_prefixes_and_respects_capacity():
    t = T.TokenTree(7, 6)
    a = t.insert([1, 2, 3], 8)
    b = t.insert([1, 2, 4], 8)
    c = t.insert([5, 6, 7, 8], 8)  # only 1 more node fits
    assert a == [1, 2, 3] and b == [1, 2, 4] and c == [5]
    assert len(t) == 6 and t.token == [7, 1, 2, 3, 4, 5]
    assert all(t.parent[i] < i for i in range(1, len(t)))
    assert all(i >= t.depth[i] for i in range(len(t)))
    assert t.insert([1, 2, 3, 9], 3) == [1, 2, 3]  # depth limit
    m = t.masks()
    assert m[0] == 1 and m[3] == 0b1111 and m[4] == 0b10111 and m[5] == 0b100001


def test_padded_rows_are_inert():
    t = T.TokenTree(9, 8)
    t.insert([1, 2], 4)
    tok, dep, masks = t.padded(8)
    assert tok[3:] == [9] * 5 and dep[3:] == [1] * 5
    assert all(masks[i] == 1 | (1 << i) for i in range(3, 8))
    # no walk reaches a padding row, even when the model predicts the root token
    assert t.walk([9, 2, 5] + [0] * 5) == ([9], [])


def test_walk_follows_the_models_choices():
    t = T.TokenTree(0, 16)
    t.insert([1, 2, 3], 8)   # nodes 1, 2, 3
    t.insert([1, 5], 8)      # node 4 under node 1
    t.insert([6], 8)         # node 5
    greedy = [1, 5, 0, 0, 8, 0]  # root -> 1 (node 1) -> 5 (node 4) -> model says 8: stop
    assert t.walk(greedy) == ([1, 5, 8], [1, 4])
    assert t.walk([4, 0, 0, 0, 0, 0]) == ([4], [])


@pytest.mark.parametrize("seed", range(10))
def test_compaction_moves_bring_the_path_to_consecutive_slots(seed):
    rnd = random.Random(seed)
    t = T.TokenTree(0, 32)
    for _ in range(12):
        t.insert([rnd.randrange(4) for _ in range(rnd.randrange(1, 8))], 8)
    greedy = [rnd.randrange(4) for _ in range(len(t))]
    _, path = t.walk(greedy)
    pos0 = 100
    cache = {pos0 + i: ("node", i) for i in range(len(t))}  # the slot of node i holds node i's K/V
    for src, dst in T.compaction_moves(path, pos0):
        cache[dst] = cache[src]
    assert [cache[pos0 + d] for d in range(1, len(path) + 1)] == [("node", n) for n in path]
    assert cache[pos0] == ("node", 0)


def test_drafter_sources():
    d = T.TreeDrafter([1, 2, 3, 9, 1, 2, 3, 8, 1, 2, 4, 1, 2, 3])
    cands = d.candidates(3)
    # the last 3-gram (1, 2, 3) occurred twice before: newest continuation first; then the 2-gram (2, 3)
    assert cands[0] == [8, 1, 2] and cands[1] == [9, 1, 2] and [8, 1, 2] in cands[2:]
    tree, chain = d.build(8, 3)
    assert len(tree) <= 8 and chain == tree.insert(cands[0], 3)
    # the model's predictions become a pool chain and a lookahead window
    greedy = [5] + [7] * (len(tree) - 1)
    emitted, path = tree.walk(greedy)
    d.learn(tree, chain, greedy, path)
    assert d.pool[(2, 3)] == 5 and d.lookahead == [greedy[c] for c in chain]
    d.push(5)
    assert d.candidates(2)[0] == [7, 7]


def _greedy_verify(next_fn, history):
    def verify(tree, pos0):
        assert len(history) == pos0 + 1 and history[-1] == tree.token[0]
        greedy = []
        for i in range(len(tree)):
            ctx, at = [], i
            while at > 0:
                ctx.append(tree.token[at])
                at = tree.parent[at]
            greedy.append(next_fn(history + ctx[::-1]))
        return greedy, (lambda path, p0: None)
    return verify


def _cycle_next(prefix):
    return (prefix[-1] * 2 + prefix[-2] + 1) % 5 if len(prefix) > 1 else 1


def _long_next(prefix):
    return (prefix[-1] * 31 + len(prefix) * 17 + 5) % 1009


def _step_with(next_fn, history):
    def step(tok, pos, n):
        assert len(history) == pos + 1 and history[-1] == tok
        for _ in range(n):
            yield next_fn(history)
    return step


@pytest.mark.parametrize("cap,depth", [(2, 1), (8, 4), (32, 12)])
@pytest.mark.parametrize("S,N", [(5, 1), (5, 2), (3, 60), (9, 150)])
def test_tree_stream_emits_exactly_the_greedy_tokens(cap, depth, S, N):
    prompt = [(3 * i + 2) % 5 for i in range(S)]
    greedy = list(prompt)
    for _ in range(N):
        greedy.append(_cycle_next(greedy))
    seq = prompt + [greedy[S]]
    stats = {}
    out = [greedy[S]] + list(T.stream(seq, S, N, cap, depth, _greedy_verify(_cycle_next, seq), stats))
    assert out == greedy[S:S + N]
    if N >= 150 and cap >= 8:  # the toy text cycles: drafts from earlier cycles are accepted
        assert stats["verifies"] < (N - 1) / 2


def test_gated_tree_stream_falls_back_to_plain_steps_and_stays_exact():
    S, N = 6, 200
    prompt = [(5 * i + 1) % 5 for i in range(S)]
    greedy = list(prompt)
    for _ in range(N):
        greedy.append(_long_next(greedy))
    seq = prompt + [greedy[S]]
    stats = {}
    out = [greedy[S]] + list(T.stream(seq, S, N, 16, 6, _greedy_verify(_long_next, seq), stats,
                                      step=_step_with(_long_next, seq), gate=spec.Gate(prior_cost=1.4)))
    assert out == greedy[S:S + N]
    assert stats["plain_steps"] > 0.8 * N


def _batch_verify(next_fn, seqs, log):
    """verify(trees, pos0s) over B toy sequences: each unfinished tree's root is its sequence's last token
    at position pos0; a finished sequence gets None."""
    def verify(trees, pos0s):
        greedy = []
        for b, tree in enumerate(trees):
            if tree is None:
                greedy.append(None)
                continue
            greedy.append(_greedy_verify(next_fn, seqs[b])(tree, pos0s[b])[0])
        log.append([t is None for t in trees])

        def commit(paths, p0s):
            assert [p is None for p in paths] == [t is None for t in trees] and list(p0s) == list(pos0s)
        return greedy, commit
    return verify


@pytest.mark.parametrize("cap,depth", [(2, 1), (8, 4), (16, 12)])
@pytest.mark.parametrize("B,S,N", [(2, 5, 1), (3, 5, 2), (4, 3, 60), (2, 9, 150)])
def test_batched_tree_stream_yields_every_sequences_greedy_tokens(cap, depth, B, S, N):
    prompts = [[(3 * i + 2 + b) % 5 for i in range(S)] for b in range(B)]
    nexts = [_cycle_next, _long_next]
    fn = lambda p: nexts[p[0] % 2](p)  # noqa: E731  (sequences follow different rules by their first token)
    greedy = []
    for p in prompts:
        g = list(p)
        for _ in range(N + cap):
            g.append(fn(g))
        greedy.append(g)
    seqs = [p + [g[S]] for p, g in zip(prompts, greedy)]
    log, stats = [], {}
    steps = [[s[S] for s in seqs]] + list(T.stream_batch(seqs, S, N, cap, depth, _batch_verify(fn, seqs, log), stats))
    assert len(steps) == N and all(len(st) == B for st in steps)
    for b in range(B):
        assert [st[b] for st in steps] == greedy[b][S:S + N]
        assert seqs[b][:S + N] == greedy[b][:S + N]  # overshoot past N is still the greedy continuation
    assert stats["verifies"] == len(log)
    if N > 1:
        # a sequence drops out of the verifies once it has N tokens, and only then
        for b in range(B):
            col = [row[b] for row in log]
            assert col == sorted(col)
