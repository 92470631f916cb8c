"""Host side of exact prompt-lookup speculative decoding (the reference's `_stream_spec`,
engine/engine.py:759-828).

Drafting rule (kept from the reference, because it decides which tokens get proposed and so how many
verifies a generation takes): the draft after a history is the continuation of the latest earlier
occurrence of its last 3 tokens, else of its last 2, cut to k tokens and padded with the last token
(k copies of it when neither occurred). `NgramDrafter` keeps, per n-gram order, a table from each
n-gram to the index just after its latest occurrence that already has a continuation; it is fed one
token at a time, so a lookup never rescans the history.

A verify forward runs T = k + 1 tokens, [last emitted] + draft, and returns the greedy token after each
prefix of that row. `verified_tokens` keeps the drafts the model agrees with and the model's own token
after them, so what is emitted is always the verify forward's greedy output, whatever was drafted.
"""

from __future__ import annotations

import time
from itertools import takewhile


class NgramDrafter:
    """Draft proposals from a token history, by n-gram lookup (longest order first)."""

    def __init__(self, history=(), orders=(3, 2)):
        self.orders = tuple(sorted(orders, reverse=True))
        self.history: list[int] = []
        # order -> {n-gram: index where its latest continued occurrence's continuation starts}
        self.next_at: dict[int, dict[tuple, int]] = {n: {} for n in self.orders}
        for tok in history:
            self.push(tok)

    def push(self, tok: int) -> None:
        """Append one token. It is the continuation of every n-gram that ends just before it, so
        those n-grams now point here."""
        h = self.history
        here = len(h)
        for n in self.orders:
            if here >= n:
                self.next_at[n][tuple(h[here - n:])] = here
        h.append(tok)

    def extend(self, toks) -> None:
        for tok in toks:
            self.push(tok)

    def propose(self, k: int) -> list[int]:
        """k draft tokens to follow the current history."""
        h = self.history
        for n in self.orders:
            if len(h) < n:
                continue
            at = self.next_at[n].get(tuple(h[-n:]))
            if at is not None:
                cont = h[at:at + k]
                return cont + [h[-1]] * (k - len(cont))
        return [h[-1]] * k


def verified_tokens(row: list[int], greedy: list[int]) -> list[int]:
    """What one verify emits. row = [last emitted] + drafts; greedy[i] = the model's token after
    row[:i + 1]. Draft i + 1 stands only if it equals greedy[i] (the token the model itself would have
    produced at that point) and every draft before it stood; the model's token after the last standing
    draft is emitted too."""
    agreed = sum(1 for _ in takewhile(lambda pair: pair[0] == pair[1], zip(row[1:], greedy)))
    return greedy[:agreed + 1]


class Gate:
    """When speculation pays (a policy of this engine; the reference instead times one warm-up run,
    engine/engine.py:83-85). After every verify it compares the tokens the last few verifies emitted
    with what one verify costs in plain decode steps (measured as the generation runs); while
    speculation does not pay, the next `backoff` tokens come from plain steps, the back-off doubling
    each time (up to `max_backoff`) and resetting once speculation pays again."""

    def __init__(self, window: int = 4, backoff: int = 8, max_backoff: int = 128, prior_cost: float = 1.4):
        self.window, self.min_backoff, self.max_backoff = window, backoff, max_backoff
        self.backoff = backoff
        self.recent: list[int] = []
        self.t_verify, self.n_verify, self.t_step, self.n_step = 0.0, 0, 0.0, 0
        self.prior_cost = prior_cost

    def cost(self) -> float:
        """One verify in plain steps: measured once both have run, the prior before."""
        if self.n_verify and self.n_step and self.t_step > 0:
            return (self.t_verify / self.n_verify) / (self.t_step / self.n_step)
        return self.prior_cost

    def verified(self, emitted: int, seconds: float) -> int:
        """Record one verify; returns how many plain steps to run next (0: keep speculating)."""
        self.t_verify += seconds
        self.n_verify += 1
        self.recent = (self.recent + [emitted])[-self.window:]
        if len(self.recent) < self.window or sum(self.recent) / len(self.recent) >= self.cost():
            if len(self.recent) == self.window:
                self.backoff = self.min_backoff
            return 0
        plain, self.backoff = self.backoff, min(2 * self.backoff, self.max_backoff)
        self.recent = []
        return plain

    def stepped(self, seconds: float, n: int = 1) -> None:
        """Record n plain steps that took `seconds` together."""
        self.t_step += seconds
        self.n_step += n


def stream(seq: list[int], S: int, N: int, k: int, verify, stats: dict | None = None, step=None,
           gate: Gate | None = None):
    """The speculative loop after the prompt forward (one sequence). `seq` is the prompt (S tokens)
    plus the first generated token; it is extended in place with every emitted token, and generated
    tokens 2..N are yielded one at a time.

    verify(row, pos0) returns the greedy token after every prefix of row (k + 1 tokens at positions
    pos0 ..); a verify always starts at the last emitted token, so pos0 + k + 1 <= S + N + k - 1.
    With `step` (plain decode steps: step(token, pos, n) yields the n greedy tokens after `token` at
    `pos`, one at a time) and a `gate`, the runs of tokens the gate hands to plain steps come from
    `step`. Both emit greedy tokens, so the output does not depend on the gate. The gate's clock for
    plain steps runs only while `step` produces a token, not while the caller consumes one."""
    drafter = NgramDrafter(seq)
    done = len(seq) - S  # generated tokens already delivered (the first one came from the prefill)
    stats = {} if stats is None else stats
    stats["verifies"] = stats["plain_steps"] = 0
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
        row = [seq[-1]] + drafter.propose(k)
        t0 = time.perf_counter()
        got = verified_tokens(row, verify(row, len(seq) - 1))
        spent = time.perf_counter() - t0
        stats["verifies"] += 1
        if gate is not None and step is not None:
            plain_run = gate.verified(len(got), spent)
        for tok in got:
            seq.append(tok)
            drafter.push(tok)
        for tok in got[:N - done]:
            done += 1
            yield tok
