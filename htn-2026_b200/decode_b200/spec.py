"""Prompt-lookup drafts for exact speculative decoding (engine/engine.py:759-828, the reference's
`_stream_spec`).

A sequence's history (prompt + generated tokens) is indexed by its 3-grams and 2-grams, each mapped to
the index just after its latest occurrence whose continuation exists. The draft after the history
`seq` is the continuation of the latest earlier occurrence of seq[-3:] (else of seq[-2:]), k tokens
long, padded with seq[-1] when shorter or when neither n-gram occurred. The verify forward runs the T =
k + 1 tokens [seq[-1]] + draft at positions len(seq) - 1 ..; its greedy token after every prefix decides
how many draft tokens are accepted (`accept`), so the emitted tokens are the verify forward's own
greedy tokens whatever the draft was.
"""

from __future__ import annotations


class PromptLookup:
    """n-gram index of one sequence (engine/engine.py:776-787 register, :802-808 the draft)."""

    def __init__(self, seq: list[int]):
        self.seq = seq  # shared with the caller, which extends it
        self.i3: dict[tuple[int, int, int], int] = {}
        self.i2: dict[tuple[int, int], int] = {}
        self.reg = 1  # next n-gram end index to register
        self.register()

    def register(self) -> None:
        """Index the n-grams ending at j for every j whose continuation seq[j + 1] exists."""
        seq, i3, i2 = self.seq, self.i3, self.i2
        for j in range(self.reg, len(seq) - 1):
            i2[(seq[j - 1], seq[j])] = j + 1
            if j >= 2:
                i3[(seq[j - 2], seq[j - 1], seq[j])] = j + 1
        self.reg = max(self.reg, len(seq) - 1)

    def draft(self, k: int) -> list[int]:
        seq = self.seq
        last = seq[-1]
        p = self.i3.get((seq[-3], seq[-2], last)) if len(seq) >= 3 else None
        if p is None and len(seq) >= 2:
            p = self.i2.get((seq[-2], last))
        d = seq[p:p + k] if p is not None else []
        return d + [last] * (k - len(d))


def accept(row: list[int], greedy: list[int]) -> list[int]:
    """Tokens emitted by one verify (engine/engine.py:819-825): row = [last] + draft, greedy[t] = the
    greedy token after row[:t + 1]. The leading drafts that equal the greedy tokens are accepted, then
    the greedy token after them."""
    k = len(row) - 1
    a = 0
    while a < k and row[a + 1] == greedy[a]:
        a += 1
    return greedy[:a + 1]


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
        if self.n_verify and self.n_step:
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
    """The speculative loop after the prompt forward (engine/engine.py:788-828, one sequence): `seq` is
    the prompt (S tokens) plus the first generated token; yields generated tokens 2..N, one at a time.
    verify(row, pos0) returns the greedy token after every prefix of row (k + 1 tokens at positions
    pos0 ..); every verify starts at the last emitted token, so pos0 + k + 1 <= S + N + k - 1. With
    `step` (plain decode steps: step(token, pos, n) yields the n greedy tokens after `token` at `pos`,
    one at a time) and a `gate`, the tokens the gate hands to plain steps come from `step`; both emit
    greedy tokens."""
    import time

    look = PromptLookup(seq)
    yielded = len(seq) - S
    stats = {} if stats is None else stats
    stats["verifies"] = stats["plain_steps"] = 0
    plain = 0
    while yielded < N:
        if plain and step is not None:
            n = min(plain, N - yielded)
            t0 = time.perf_counter()
            for tok in step(seq[-1], len(seq) - 1, n):
                seq.append(tok)
                yield tok
                yielded += 1
            if gate is not None:
                gate.stepped(time.perf_counter() - t0, n)
            stats["plain_steps"] += n
            plain = 0
        else:
            row = [seq[-1]] + look.draft(k)
            t0 = time.perf_counter()
            got = accept(row, verify(row, len(seq) - 1))
            seq.extend(got)
            stats["verifies"] += 1
            if gate is not None and step is not None:
                plain = gate.verified(len(got), time.perf_counter() - t0)
        look.register()
        while yielded < N and len(seq) - S > yielded:
            yield seq[S + yielded]
            yielded += 1
