"""Exact token-tree speculation on the GPU: the tree kernels against the oracle, and the engine's tree
stream against plain greedy decoding.

* qd_tree_attn: every node's output equals the oracle's SDPA (and an fp32 reference) over its sequence's
  cached prefix plus the node's own ancestors, within the 2e-2 of the other attention tests, for one
  and for several sequences with different prefixes; cache slots past each tree hold NaN, so a read of
  any of them shows (a non-ancestor node's slot holds finite values, so the oracle comparison is what
  catches a wrong mask).
* qd_tree_qk_rope: per-node q/k RMSNorm + RoPE at the node's own position equals the oracle's
  qk_norm_rope at that position (one BF16 ulp of each rounded term), K/V written to the node's slot.
* qd_tree_compact: the accepted path's K/V rows land in consecutive slots of every layer and head.
* Engine with trees on, at batch 1 and with one tree per sequence at batch 2-8: the emitted tokens
  follow the plain greedy run (ties excepted) and the reference's recorded tokens; a tree holding the
  model's own continuation is accepted whole, its K/V compacted, and decoding continues from it exactly,
  also when the sequences of a batch accept different numbers of drafts.
"""

import math
import random

import pytest
import torch

from conftest import load_golden, synth_state
from oracle import qwen3_cpu as Q

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16
DEV = "cuda:0"
NQ, NKV, D = 32, 8, 128


def _random_tree(T, seed):
    from decode_b200 import tree as TT

    rnd = random.Random(seed)
    t = TT.TokenTree(0, T)
    while len(t) < T:
        t.insert([rnd.randrange(5) for _ in range(rnd.randrange(1, 6))], 8)
    return t


def _masks_i32(masks):
    return [m - (1 << 32) if m >= 1 << 31 else m for m in masks]


@pytest.mark.parametrize("T,prefixes", [(1, [1]), (8, [37]), (16, [200]), (32, [511]), (32, [0]), (32, [4000]),
                                        (16, [5, 300, 0, 77]), (32, [100, 3]), (8, [9, 1000, 64, 2, 0, 513, 31, 8]),
                                        (2, [7000] + [0] * 31)])
def test_tree_attention_matches_oracle(T, prefixes):
    """B sequences, each with its own prefix length and tree; slots past each sequence's tree are NaN.
    The split-K partition follows each row's prefix on the device: long and short prefixes share a launch
    (the last case: one sequence of 7000 cached keys among 31 empty ones)."""
    from decode_b200 import ops

    B = len(prefixes)
    cap = max(prefixes) + T + 16
    g = torch.Generator().manual_seed(T * 1000 + sum(prefixes))
    trees = [_random_tree(T, T + p + b) for b, p in enumerate(prefixes)]
    masks = [tr.padded(T)[2] for tr in trees]
    kc = torch.full((B, NKV, cap, D), float("nan"), dtype=BF16)
    vc = torch.full((B, NKV, cap, D), float("nan"), dtype=BF16)
    for b, p in enumerate(prefixes):
        kc[b, :, :p + T] = torch.randn((NKV, p + T, D), generator=g).to(BF16)
        vc[b, :, :p + T] = torch.randn((NKV, p + T, D), generator=g).to(BF16)
    q = torch.randn((B * T, NQ * D), generator=g).to(BF16)
    out = torch.full((B * T, NQ * D), float("nan"), dtype=BF16, device=DEV)
    anc = torch.tensor(sum((_masks_i32(m) for m in masks), []), dtype=torch.int32, device=DEV)
    pre = torch.tensor(prefixes, dtype=torch.int32, device=DEV)
    err = torch.zeros((1,), dtype=torch.int32, device=DEV)
    ops.tree_attn(q.to(DEV), B, T, NQ, NKV, kc.to(DEV), vc.to(DEV), pre, anc, out, err=err)
    o = out.float().cpu()
    assert int(err.item()) == 0 and torch.isfinite(o).all()
    worst = 0.0
    for b, prefix in enumerate(prefixes):
        for i in range(T):
            r = b * T + i
            keys = list(range(prefix)) + [prefix + j for j in range(T) if (masks[b][i] >> j) & 1]
            k = kc[b, :, keys][None]
            v = vc[b, :, keys][None]
            ref = Q.attention_decode(q[r].view(1, NQ, D), k, v, len(keys)).float().view(-1)
            qg = q[r].float().view(NKV, 4, D)
            p = torch.softmax(torch.einsum("hgd,hnd->hgn", qg, k[0].float()) / math.sqrt(D), -1)
            ref32 = torch.einsum("hgn,hnd->hgd", p, v[0].float()).reshape(-1)
            worst = max(worst, (o[r] - ref).abs().max().item(), (o[r] - ref32).abs().max().item())
    assert worst < 2e-2, worst


@pytest.mark.parametrize("T,prefix", [(1, 1), (8, 37), (32, 0), (32, 100), (32, 127), (16, 128), (32, 500),
                                      (32, 2000)])
def test_tree_attention_rows_on_tensor_cores_matches_oracle(T, prefix):
    """qd_tree_attn_rows (the prompt attention kernel with the ancestor mask): every node's output against
    the oracle's SDPA and an fp32 reference over the cached prefix plus its ancestors, within 2e-2 (the
    prompt attention's tolerance); trees that straddle a 128-key tile boundary included. Slots past the
    tree hold NaN, so a read of any of them shows."""
    from decode_b200 import ops

    cap = prefix + T + 40
    g = torch.Generator().manual_seed(T * 7 + prefix)
    tree = _random_tree(T, prefix + 3)
    _, _, masks = tree.padded(T)
    kc = torch.full((NKV, cap, D), float("nan"), dtype=BF16)
    vc = torch.full((NKV, cap, D), float("nan"), dtype=BF16)
    kc[:, :prefix + T] = torch.randn((NKV, prefix + T, D), generator=g).to(BF16)
    vc[:, :prefix + T] = torch.randn((NKV, prefix + T, D), generator=g).to(BF16)
    q = torch.randn((T, NQ * D), generator=g).to(BF16)
    out = torch.full((T, NQ * D), float("nan"), dtype=BF16, device=DEV)
    anc = torch.tensor(_masks_i32(masks), dtype=torch.int32, device=DEV)
    err = torch.zeros((1,), dtype=torch.int32, device=DEV)
    ops.tree_attn_rows(q.to(DEV), T, prefix, anc, NQ, NKV, kc.to(DEV), vc.to(DEV), out, err=err)
    o = out.float().cpu()
    assert int(err.item()) == 0 and torch.isfinite(o).all()
    worst = 0.0
    for i in range(T):
        keys = list(range(prefix)) + [prefix + j for j in range(T) if (masks[i] >> j) & 1]
        k = kc[:, keys][None]
        v = vc[:, keys][None]
        ref = Q.attention_decode(q[i].view(1, NQ, D), k, v, len(keys)).float().view(-1)
        qg = q[i].float().view(NKV, 4, D)
        p = torch.softmax(torch.einsum("hgd,hnd->hgn", qg, k[0].float()) / math.sqrt(D), -1)
        ref32 = torch.einsum("hgn,hnd->hgd", p, v[0].float()).reshape(-1)
        worst = max(worst, (o[i] - ref).abs().max().item(), (o[i] - ref32).abs().max().item())
    assert worst < 2e-2, worst


def test_tree_attention_flags_a_tree_past_the_cache():
    """A sequence whose tree would reach past the cache gets zeros and the position error; the other
    sequence is computed as usual (the kernel checks the device-side prefix before any cache read)."""
    from decode_b200 import ops

    T, cap = 8, 64
    kc = torch.randn((2, NKV, cap, D), device=DEV).to(BF16)
    vc = torch.randn((2, NKV, cap, D), device=DEV).to(BF16)
    q = torch.randn((2 * T, NQ * D), device=DEV).to(BF16)
    out = torch.full((2 * T, NQ * D), float("nan"), dtype=BF16, device=DEV)
    anc = torch.tensor([1 | (1 << i) for i in range(T)] * 2, dtype=torch.int32, device=DEV)
    err = torch.zeros((1,), dtype=torch.int32, device=DEV)
    ops.tree_attn(q, 2, T, NQ, NKV, kc, vc, torch.tensor([10, cap - T + 1], dtype=torch.int32, device=DEV), anc, out,
                  err=err)
    assert int(err.item()) & 16  # QD_DEVERR_POS
    assert torch.equal(out[T:].float(), torch.zeros_like(out[T:].float()))
    assert torch.isfinite(out[:T].float()).all()


def test_tree_qk_rope_at_node_positions():
    from decode_b200 import ops
    from engine import rope_tables

    T, cap = 12, 80
    slots = [50, 7, 0]
    B = len(slots)
    g = torch.Generator().manual_seed(3)
    deps = [_random_tree(T, 9 + b).padded(T)[1] for b in range(B)]
    qkv = torch.randn((B * T, (NQ + 2 * NKV) * D), generator=g).to(BF16)
    qn = (1 + 0.1 * torch.randn(D, generator=g)).to(BF16)
    kn = (1 + 0.1 * torch.randn(D, generator=g)).to(BF16)
    cos, sin = rope_tables(cap, D, 5e6)
    kc = torch.full((B, NKV, cap, D), float("nan"), dtype=BF16, device=DEV)
    vc = torch.full((B, NKV, cap, D), float("nan"), dtype=BF16, device=DEV)
    q_out = torch.empty((B * T, NQ * D), dtype=BF16, device=DEV)
    pos = torch.tensor([slots[b] + d for b in range(B) for d in deps[b]], dtype=torch.int32, device=DEV)
    slot0 = torch.tensor(slots, dtype=torch.int32, device=DEV)
    err = torch.zeros((1,), dtype=torch.int32, device=DEV)
    ops.tree_qk_rope(qkv.to(DEV), B, T, slot0, pos, NQ, NKV, qn.to(DEV), kn.to(DEV), 1e-6, cos.to(DEV), sin.to(DEV),
                     q_out, kc, vc, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    for b, slot in enumerate(slots):
        for t in range(T):
            r, p = b * T + t, slot + deps[b][t]
            q, k, v = Q.qk_norm_rope(qkv[r:r + 1], qn, kn, cos[p], sin[p], 1e-6)
            tol = 2 * q.float().abs().max().item() * 2.0 ** -8 + 1e-6
            assert (q_out[r].float().cpu() - q.float().view(-1)).abs().max().item() <= tol
            assert (kc[b, :, slot + t].float().cpu() - k[0].float()).abs().max().item() <= tol
            assert torch.equal(vc[b, :, slot + t].cpu(), v[0])
        assert torch.isnan(kc[b, :, :slot].float()).all() and torch.isnan(kc[b, :, slot + T:].float()).all()


def test_tree_compact_moves_rows_of_every_layer():
    from decode_b200 import ops

    Ly, B, cap = 3, 2, 64
    k = torch.randn((Ly, B, NKV, cap, D), device=DEV).to(BF16)
    v = torch.randn((Ly, B, NKV, cap, D), device=DEV).to(BF16)
    k0, v0 = k.clone(), v.clone()
    moves = {0: [(22, 21), (25, 22), (30, 23)], 1: [(9, 5), (12, 6)]}
    flat = [(b, s_, d) for b in (1, 0) for s_, d in moves[b]]  # sequences interleaved in any order
    m = torch.tensor(flat + [(0, 0, 0)] * 10, dtype=torch.int32, device=DEV)
    ops.tree_compact(k, v, m, len(flat))
    torch.cuda.synchronize()
    for b in range(B):
        for src, dst in moves[b]:
            assert torch.equal(k[:, b, :, dst], k0[:, b, :, src]) and torch.equal(v[:, b, :, dst], v0[:, b, :, src])
        moved = {d for _, d in moves[b]}
        untouched = [s_ for s_ in range(cap) if s_ not in moved]
        assert torch.equal(k[:, b, :, untouched], k0[:, b, :, untouched])
        assert torch.equal(v[:, b, :, untouched], v0[:, b, :, untouched])


@pytest.fixture(scope="module")
def eng2():
    import engine as E

    state, cfg = synth_state(2)
    return E.Engine.from_state_dict(state, cfg, "cuda:0"), cfg


def _tie_ok(toks, plain, logits, tol, b=0):
    for t in range(len(toks)):
        if toks[t] != plain[t]:
            top2 = logits[t][b].float().topk(2).values
            return float(top2[0] - top2[1]) <= tol, t
    return True, None


@pytest.mark.parametrize("T", [8, 32])
def test_tree_generate_matches_plain_greedy(eng2, T):
    """Random-init weights have no reason to continue a pattern, so drafts are rarely accepted here; the
    emitted tokens must still be the plain run's, on a fresh state and on a second request."""
    from decode_b200 import synth

    eng, cfg = eng2
    prompt = synth.random_prompt(1, 36, cfg["vocab_size"], seed=5)
    N = 40
    eng.state = None
    plain, logits = eng.generate_with_logits(prompt, N)
    eng.state = None
    eng.tree = T
    try:
        toks = [s[0] for s in eng.generate(prompt, N)]
        again = [s[0] for s in eng.generate(prompt, N)]
    finally:
        eng.tree = 0
        eng.state = None
    tol = max(5e-2, 2 * load_golden("config0")["self_drift"]["max_logsoftmax_diff"])
    ok, where = _tie_ok(toks, plain[0], logits, tol)
    assert ok, (T, where)
    assert toks == again and len(toks) == N


@pytest.mark.parametrize("T,depth", [(16, 6), (32, 12)])
def test_tree_verify_accepts_the_models_own_continuation(eng2, T, depth):
    """A tree whose main branch is the model's plain greedy continuation (plus distractor branches):
    the verify's greedy token at every branch node is the plain run's next token, the walk accepts the
    whole branch, the compaction moves its K/V into place, and plain decode steps continuing from there
    give the plain run's tokens - over two rounds."""
    import engine as E
    from decode_b200 import synth, tree as TT

    eng, cfg = eng2
    S, N = 40, 2 * depth + 12
    prompt = synth.random_prompt(1, S, cfg["vocab_size"], seed=17)
    eng.state = None
    plain, logits = eng.generate_with_logits(prompt, N)
    P = plain[0]
    eng.state = None
    eng.tree = T
    try:
        st = eng._build(1, S, N)
        tv = st.tree
        with torch.inference_mode():
            eng._upload_prompt(st, prompt)
            eng._enqueue_prefill(st)
        torch.cuda.synchronize()
        assert int(st.tok.item()) == P[0]
        emitted_all = [P[0]]
        rnd = random.Random(T)
        tol = max(5e-2, 2 * load_golden("config0")["self_drift"]["max_logsoftmax_diff"])
        flipped = False
        for _ in range(2):
            pos0 = S + len(emitted_all) - 1  # position of the last emitted token (the root)
            tree = TT.TokenTree(emitted_all[-1], T)
            tree.insert([rnd.randrange(1000) for _ in range(3)], depth)       # a distractor first
            branch = tree.insert(P[len(emitted_all):len(emitted_all) + depth], depth)
            while len(tree) < T:
                tree.insert([rnd.randrange(1000) for _ in range(rnd.randrange(1, depth))], depth)
            greedy, commit = tv(eng, st, [tree], [pos0])
            emitted, path = tree.walk(greedy[0])
            commit([path], [pos0])
            if path != branch:
                # the walk may stop early only at a near tie of the plain run (summation order)
                t = len(emitted_all) + len(path)
                top2 = logits[t][0].float().topk(2).values
                gap = float(top2[0] - top2[1])
                assert path == branch[:len(path)] and gap <= tol, (t, gap, path, branch)
                flipped = True
                break
            emitted_all += emitted
            assert emitted_all == P[:len(emitted_all)], (emitted_all, P[:len(emitted_all)])
        if not flipped:
            # continue with plain decode steps from the compacted cache
            n = N - len(emitted_all)
            rest = list(eng._plain_steps(st, emitted_all[-1], S + len(emitted_all) - 1, n))
            ok, where = _tie_ok(emitted_all + rest, P, logits, tol)
            assert ok, where
        eng.check_device_errors(st)
    finally:
        eng.tree = 0
        eng.state = None


@pytest.mark.parametrize("B", [2, 4, 8])
def test_batched_tree_generate_matches_plain_greedy(eng2, B):
    """Trees for B sequences in one verify (32 // (B / 2) nodes each, at most 64 rows): every sequence's
    tokens are the plain batched run's (ties excepted), on a fresh state and on a second request."""
    from decode_b200 import synth

    eng, cfg = eng2
    prompt = synth.random_prompt(B, 20, cfg["vocab_size"], seed=B)
    N = 30
    eng.state = None
    plain, logits = eng.generate_with_logits(prompt, N)
    eng.state = None
    eng.tree = 32
    try:
        steps = list(eng.generate(prompt, N))
        assert eng.state.tree is not None and eng.state.tree.T == min(32, 64 // B)
        again = list(eng.generate(prompt, N))
        stats = dict(eng.state.spec_stats)
    finally:
        eng.tree = 0
        eng.state = None
    assert len(steps) == N and all(len(x) == B for x in steps) and steps == again
    assert 1 <= stats["verifies"] <= N - 1
    tol = max(5e-2, 2 * load_golden("config0")["self_drift"]["max_logsoftmax_diff"])
    for b in range(B):
        ok, where = _tie_ok([x[b] for x in steps], plain[b], logits, tol, b)
        assert ok, (b, where)


def test_batched_tree_verify_accepts_each_sequences_own_continuation(eng2):
    """Three sequences whose trees hold their own greedy continuations to different depths (one sequence
    sits a round out as finished): each walk accepts exactly its branch, the compaction moves each
    sequence's K/V, and the next rounds - at positions that now differ per sequence - continue with every
    sequence's plain greedy tokens. A walk may stop early only where the plain run's own top-2 gap is
    within the parity bound (a near tie the verify's summation order may flip); that sequence then
    leaves the test."""
    from decode_b200 import synth, tree as TT

    eng, cfg = eng2
    B, S, N = 3, 24, 40
    prompt = synth.random_prompt(B, S, cfg["vocab_size"], seed=23)
    eng.state = None
    plain, logits = eng.generate_with_logits(prompt, N)
    eng.state = None
    eng.tree = 16
    try:
        st = eng._build(B, S, N)
        tv = st.tree
        assert tv.T == 16 and tv.B == B
        with torch.inference_mode():
            eng._upload_prompt(st, prompt)
            eng._enqueue_prefill(st)
        torch.cuda.synchronize()
        assert st.tok.tolist() == [plain[b][0] for b in range(B)]
        out = [[plain[b][0]] for b in range(B)]
        tol = max(5e-2, 2 * load_golden("config0")["self_drift"]["max_logsoftmax_diff"])
        active = [True] * B
        rnd = random.Random(5)
        for rnd_i in range(4):
            trees, pos0s, branches = [], [], []
            for b in range(B):
                if (b == 1 and rnd_i == 1) or not active[b]:
                    # sits this round out at its own root slot: the inert rows write slots that its next
                    # round writes again before any query reads them
                    trees.append(None)
                    pos0s.append(S + len(out[b]) - 1)
                    branches.append(None)
                    continue
                depth = [6, 2, 9][b] if rnd_i % 2 == 0 else [1, 7, 3][b]
                tree = TT.TokenTree(out[b][-1], tv.T)
                tree.insert([rnd.randrange(1000) for _ in range(2)], depth)
                branches.append(tree.insert(plain[b][len(out[b]):len(out[b]) + depth], depth))
                while len(tree) < tv.T:
                    tree.insert([rnd.randrange(1000) for _ in range(rnd.randrange(1, depth + 1))], depth)
                trees.append(tree)
                pos0s.append(S + len(out[b]) - 1)
            greedy, commit = tv(eng, st, trees, pos0s)
            paths = []
            for b in range(B):
                if trees[b] is None:
                    paths.append(None)
                    continue
                emitted, path = trees[b].walk(greedy[b])
                paths.append(path)
                if path != branches[b]:
                    t = len(out[b]) + len(path)  # the plain step whose token the verify did not repeat
                    top2 = logits[t][b].float().topk(2).values
                    gap = float(top2[0] - top2[1])
                    assert path == branches[b][:len(path)] and gap <= tol, (rnd_i, b, t, gap, path, branches[b])
                    active[b] = False
                    continue
                out[b] += emitted
            commit(paths, pos0s)
        assert sum(active) >= 2, active
        for b in range(B):
            if not active[b]:
                continue
            assert len(out[b]) > 12
            ok, where = _tie_ok(out[b], plain[b][:len(out[b])], logits, tol, b)
            assert ok, (b, where)
        eng.check_device_errors(st)
    finally:
        eng.tree = 0
        eng.state = None


def test_tree_generate_follows_reference_golden():
    import engine as E

    g = load_golden("config0")
    state, cfg = synth_state(g["spec"]["layers"])
    eng = E.Engine.from_state_dict(state, cfg, "cuda:0")
    eng.tree = 16
    steps = list(eng.generate(g["prompt"], g["spec"]["new"]))
    assert eng.state.tree is not None and len(steps) == g["spec"]["new"]
    toks, ref = [s[0] for s in steps], g["native"]["tokens"][0]
    tol = max(5e-2, 2 * g["self_drift"]["max_logsoftmax_diff"])
    for t in range(len(ref)):
        if toks[t] != ref[t]:
            step = g["native"]["steps"][t]
            vals, ids = step["top_vals"][0], step["top_ids"][0]
            assert vals[0] - vals[1] < tol and toks[t] in ids, t
            break
