"""Host side of exact token-tree speculative decoding (the reference's tree speculation: engine/spec.py,
engine/engine.py:830-936).

A round drafts a trie of candidate continuations of the current sequence, rooted at its last emitted
token, and one verify forward runs every node as an activation row: node i sits at position
pos0 + depth(i) and attends to the cached prefix and to its own ancestors. The model's greedy token at
every node is returned; walking from the root along the children whose token equals the model's
choice gives the accepted drafts, and the model's token after the last of them is emitted too - so the
emitted tokens are the model's own greedy tokens whatever was drafted (exact).

Candidate sources (kept from the reference, because they decide what gets proposed): the lookahead
window (the model's predictions at the previous tree's main chain past what was accepted), up to three
recent occurrences of the last 3-gram and of the last 2-gram with their continuations, and a pool of the
model's predictions at every verified node keyed by (token before, token).
"""

from __future__ import annotations

import time
from collections import deque


class TokenTree:
    """A draft trie of at most `capacity` nodes. Node 0 is the root (the last emitted token); nodes are
    numbered in insertion order, so a parent always precedes its children and index >= depth."""

    def __init__(self, root: int, capacity: int):
        if not 1 <= capacity <= 32:
            raise ValueError("a token tree holds 1 to 32 nodes (one bit each in the ancestor masks)")
        self.capacity = capacity
        self.token = [root]
        self.parent = [-1]
        self.depth = [0]
        self.kids: list[dict[int, int]] = [{}]

    def __len__(self) -> int:
        return len(self.token)

    def insert(self, path, max_depth: int) -> list[int]:
        """Add a candidate continuation below the root (shared prefixes are reused); returns the node ids
        along it, as far as the capacity allowed."""
        at, nodes = 0, []
        for tok in list(path)[:max_depth]:
            nxt = self.kids[at].get(tok)
            if nxt is None:
                if len(self.token) == self.capacity:
                    break
                nxt = len(self.token)
                self.token.append(tok)
                self.parent.append(at)
                self.depth.append(self.depth[at] + 1)
                self.kids.append({})
                self.kids[at][tok] = nxt
            nodes.append(nxt)
            at = nxt
        return nodes

    def masks(self) -> list[int]:
        """Per node, the bit set of the node and its ancestors (bit j = node j)."""
        out = []
        for i, p in enumerate(self.parent):
            out.append((1 << i) | (out[p] if p >= 0 else 0))
        return out

    def padded(self, rows: int):
        """(tokens, depths, masks) for a verify of `rows` rows: the tree, then inert rows (the root token,
        attending to the root only) that no walk can reach."""
        masks = self.masks()
        tok, dep = list(self.token), list(self.depth)
        for i in range(len(tok), rows):
            tok.append(self.token[0])
            dep.append(1)
            masks.append(1 | (1 << i))
        return tok, dep, masks

    def walk(self, greedy: list[int]) -> tuple[list[int], list[int]]:
        """(emitted tokens, accepted node ids) given the model's greedy token at every node."""
        emitted, path, at = [greedy[0]], [], 0
        while True:
            nxt = self.kids[at].get(emitted[-1])
            if nxt is None:
                return emitted, path
            path.append(nxt)
            emitted.append(greedy[nxt])
            at = nxt


def compaction_moves(path: list[int], pos0: int) -> list[tuple[int, int]]:
    """Cache moves that bring the accepted nodes' keys / values from their tree slots (pos0 + node id)
    to consecutive slots (pos0 + depth). Applied in order they never overwrite a slot still to be read:
    node ids along a path increase and each is at least its depth."""
    return [(pos0 + n, pos0 + d) for d, n in enumerate(path, start=1) if n != d]


class TreeDrafter:
    """Candidate continuations of one sequence; fed every emitted token (`push`) and every verify's
    results (`learn`)."""

    def __init__(self, history=(), orders=(3, 2), per_gram: int = 3):
        self.orders = tuple(sorted(orders, reverse=True))
        self.per_gram = per_gram
        self.history: list[int] = []
        # order -> {n-gram: continuation starts of its latest occurrences, oldest first}
        self.starts: dict[int, dict[tuple, deque]] = {n: {} for n in self.orders}
        self.pool: dict[tuple[int, int], int] = {}
        self.lookahead: list[int] = []
        for tok in history:
            self.push(tok)

    def push(self, tok: int) -> None:
        h, here = self.history, len(self.history)
        for n in self.orders:
            if here >= n:
                q = self.starts[n].setdefault(tuple(h[here - n:]), deque(maxlen=self.per_gram))
                q.append(here)
        h.append(tok)

    def candidates(self, depth: int) -> list[list[int]]:
        h, out = self.history, []
        if self.lookahead:
            out.append(self.lookahead[:depth])
        for n in self.orders:
            if len(h) >= n:
                for at in reversed(self.starts[n].get(tuple(h[-n:]), ())):
                    out.append(h[at:at + depth])
        if len(h) >= 2:  # follow the model's recorded predictions from the last two tokens
            chain, a, b = [], h[-2], h[-1]
            while len(chain) < depth and (a, b) in self.pool:
                a, b = b, self.pool[(a, b)]
                chain.append(b)
            if chain:
                out.append(chain)
        return [c for c in out if c]

    def build(self, capacity: int, depth: int) -> tuple[TokenTree, list[int]]:
        """The next tree and its main chain (the first candidate's nodes, for the lookahead window)."""
        tree = TokenTree(self.history[-1], capacity)
        cands = self.candidates(depth) or [[self.history[-1]] * depth]
        chain: list[int] = []
        for i, c in enumerate(cands):
            nodes = tree.insert(c, depth)
            if i == 0:
                chain = nodes
            if len(tree) == capacity:
                break
        return tree, chain

    def learn(self, tree: TokenTree, chain: list[int], greedy: list[int], path: list[int]) -> None:
        """Record the model's prediction at every node (its context is the node's ancestry) and keep the
        main chain's predictions past the accepted drafts as the next lookahead window."""
        before = self.history[-2] if len(self.history) >= 2 else None
        for i in range(len(tree)):
            prev = tree.token[tree.parent[i]] if i else before
            if prev is not None:
                self.pool[(prev, tree.token[i])] = greedy[i]
        a = len(path)
        self.lookahead = [greedy[c] for c in chain[a:]] if chain[:a] == path else []


def stream(seq: list[int], S: int, N: int, capacity: int, depth: int, verify, stats: dict | None = None, step=None,
           gate=None):
    """The token-tree loop after the prompt forward (one sequence). `seq` is the prompt (S tokens) plus
    the first generated token; it is extended in place, and generated tokens 2..N are yielded one at a
    time. verify(tree, pos0) runs the tree's nodes at positions pos0 + depth (pos0 = the position of the
    last emitted token) and returns (greedy token per node, a callback that moves the accepted path's
    keys / values given the path). With `step` and a `gate` (decode_b200.spec.Gate), runs of tokens come
    from plain decode steps while trees do not pay, as in decode_b200.spec.stream."""
    drafter = TreeDrafter(seq)
    done = len(seq) - S
    stats = {} if stats is None else stats
    stats["verifies"] = stats["plain_steps"] = stats["accepted"] = 0
    plain_run = 0
    while done < N:
        if plain_run and step is not None:
            n = min(plain_run, N - done)
            plain_run = 0
            tokens = step(seq[-1], len(seq) - 1, n)
            busy = 0.0
            for _ in range(n):
                t0 = time.perf_counter()
                tok = next(tokens)
                busy += time.perf_counter() - t0
                seq.append(tok)
                drafter.push(tok)
                done += 1
                yield tok
            stats["plain_steps"] += n
            if gate is not None:
                gate.stepped(busy, n)
            continue
        tree, chain = drafter.build(capacity, depth)
        pos0 = len(seq) - 1
        t0 = time.perf_counter()
        greedy, commit = verify(tree, pos0)
        emitted, path = tree.walk(greedy)
        commit(path, pos0)
        spent = time.perf_counter() - t0
        drafter.learn(tree, chain, greedy, path)
        stats["verifies"] += 1
        stats["accepted"] += len(path)
        if gate is not None and step is not None:
            plain_run = gate.verified(len(emitted), spent)
        for tok in emitted:
            seq.append(tok)
            drafter.push(tok)
        for tok in emitted[:N - done]:
            done += 1
            yield tok


def stream_batch(seqs: list[list[int]], S: int, N: int, capacity: int, depth: int, verify, stats: dict | None = None):
    """The token-tree loop for B sequences after the prompt forward (the reference's batched tree stream,
    engine/engine.py:830-908). `seqs[b]` is prompt b (S tokens) plus its first generated token; each list
    is extended in place. Every round drafts one tree per unfinished sequence and verifies all of them in
    one forward: verify(trees, pos0s) gets a tree (None for a finished sequence, whose rows are inert) and
    the position of its root per sequence, and returns (greedy tokens per sequence, a callback given the
    accepted paths that moves their keys / values). Sequences accept different numbers of drafts, so step
    t (t = 2..N) is yielded as the list of B tokens once every sequence has its t-th token."""
    B = len(seqs)
    drafters = [TreeDrafter(s) for s in seqs]
    stats = {} if stats is None else stats
    stats["verifies"] = stats["accepted"] = stats["plain_steps"] = 0
    yielded = 1
    while yielded < N:
        trees, chains, pos0s = [], [], []
        for b in range(B):
            if len(seqs[b]) - S >= N:  # finished: its rows go to slots past the prompt, never read again
                trees.append(None)
                chains.append(None)
                pos0s.append(S)
            else:
                tree, chain = drafters[b].build(capacity, depth)
                trees.append(tree)
                chains.append(chain)
                pos0s.append(len(seqs[b]) - 1)
        greedy, commit = verify(trees, pos0s)
        paths = []
        for b in range(B):
            if trees[b] is None:
                paths.append(None)
                continue
            emitted, path = trees[b].walk(greedy[b])
            drafters[b].learn(trees[b], chains[b], greedy[b], path)
            for tok in emitted:
                seqs[b].append(tok)
                drafters[b].push(tok)
            paths.append(path)
            stats["accepted"] += len(path)
        commit(paths, pos0s)
        stats["verifies"] += 1
        while yielded < N and all(len(s) - S > yielded for s in seqs):
            yield [s[S + yielded] for s in seqs]
            yielded += 1
