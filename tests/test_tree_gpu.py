"""Exact token-tree speculation on the GPU: the tree kernels against the oracle, and the engine's tree
stream against plain greedy decoding.

* qd_tree_attn: every node's output equals the oracle's SDPA (and an fp32 reference) over the cached
  prefix plus the node's own ancestors, within the 2e-2 of the other attention tests; cache slots of
  non-ancestor nodes and past the tree hold NaN, so a read of any of them shows.
* qd_tree_qk_rope: per-node q/k RMSNorm + RoPE at the node's own position equals the oracle's
  qk_norm_rope at that position (one BF16 ulp of each rounded term), K/V written to the node's slot.
* qd_tree_compact: the accepted path's K/V rows land in consecutive slots of every layer and head.
* Engine with trees on: the emitted tokens follow the plain greedy run (ties excepted) and the
  reference's recorded tokens; a tree holding the model's own continuation is accepted whole, its K/V
  compacted, and plain decoding continues from it exactly.
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


@pytest.mark.parametrize("T,prefix", [(1, 1), (8, 37), (16, 200), (32, 511), (32, 0)])
def test_tree_attention_matches_oracle(T, prefix):
    from decode_b200 import ops

    cap = prefix + T + 16
    g = torch.Generator().manual_seed(T * 1000 + prefix)
    tree = _random_tree(T, T + prefix)
    _, _, masks = tree.padded(T)
    kc = torch.full((NKV, cap, D), float("nan"), dtype=BF16)
    vc = torch.full((NKV, cap, D), float("nan"), dtype=BF16)
    kc[:, :prefix + T] = torch.randn((NKV, prefix + T, D), generator=g).to(BF16)
    vc[:, :prefix + T] = torch.randn((NKV, prefix + T, D), generator=g).to(BF16)
    q = torch.randn((T, NQ * D), generator=g).to(BF16)
    out = torch.full((T, NQ * D), float("nan"), dtype=BF16, device=DEV)
    anc = torch.tensor([m - (1 << 32) if m >= 1 << 31 else m for m in masks], dtype=torch.int32, device=DEV)
    ops.tree_attn(q.to(DEV), T, NQ, NKV, kc.to(DEV), vc.to(DEV), prefix, anc, out)
    o = out.float().cpu()
    assert torch.isfinite(o).all()
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


def test_tree_qk_rope_at_node_positions():
    from decode_b200 import ops
    from engine import rope_tables

    T, slot0, cap = 12, 50, 80
    g = torch.Generator().manual_seed(3)
    tree = _random_tree(T, 9)
    _, dep, _ = tree.padded(T)
    qkv = torch.randn((T, (NQ + 2 * NKV) * D), generator=g).to(BF16)
    qn = (1 + 0.1 * torch.randn(D, generator=g)).to(BF16)
    kn = (1 + 0.1 * torch.randn(D, generator=g)).to(BF16)
    cos, sin = rope_tables(cap, D, 5e6)
    kc = torch.full((NKV, cap, D), float("nan"), dtype=BF16, device=DEV)
    vc = torch.full((NKV, cap, D), float("nan"), dtype=BF16, device=DEV)
    q_out = torch.empty((T, NQ * D), dtype=BF16, device=DEV)
    pos = torch.tensor([slot0 + d for d in dep], dtype=torch.int32, device=DEV)
    err = torch.zeros((1,), dtype=torch.int32, device=DEV)
    ops.tree_qk_rope(qkv.to(DEV), T, slot0, pos, NQ, NKV, qn.to(DEV), kn.to(DEV), 1e-6, cos.to(DEV), sin.to(DEV),
                     q_out, kc, vc, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    for t in range(T):
        p = slot0 + dep[t]
        q, k, v = Q.qk_norm_rope(qkv[t:t + 1], qn, kn, cos[p], sin[p], 1e-6)
        tol = 2 * q.float().abs().max().item() * 2.0 ** -8 + 1e-6
        assert (q_out[t].float().cpu() - q.float().view(-1)).abs().max().item() <= tol
        assert (kc[:, slot0 + t].float().cpu() - k[0].float()).abs().max().item() <= tol
        assert torch.equal(vc[:, slot0 + t].cpu(), v[0])
    assert torch.isnan(kc[:, :slot0].float()).all() and torch.isnan(kc[:, slot0 + T:].float()).all()


def test_tree_compact_moves_rows_of_every_layer():
    from decode_b200 import ops

    L, cap = 3, 64
    k = torch.randn((L, 1, NKV, cap, D), device=DEV).to(BF16)
    v = torch.randn((L, 1, NKV, cap, D), device=DEV).to(BF16)
    k0, v0 = k.clone(), v.clone()
    moves = [(22, 21), (25, 22), (30, 23)]
    m = torch.tensor(moves + [(0, 0)] * 29, dtype=torch.int32, device=DEV)
    ops.tree_compact(k, v, m, len(moves))
    torch.cuda.synchronize()
    for src, dst in moves:
        assert torch.equal(k[:, :, :, dst], k0[:, :, :, src]) and torch.equal(v[:, :, :, dst], v0[:, :, :, src])
    untouched = [s for s in range(cap) if s not in (21, 22, 23)]
    assert torch.equal(k[:, :, :, untouched], k0[:, :, :, untouched])


@pytest.fixture(scope="module")
def eng2():
    import engine as E

    state, cfg = synth_state(2)
    return E.Engine.from_state_dict(state, cfg, "cuda:0"), cfg


def _tie_ok(toks, plain, logits, tol):
    for t in range(len(toks)):
        if toks[t] != plain[t]:
            top2 = logits[t][0].float().topk(2).values
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
        for _ in range(2):
            pos0 = S + len(emitted_all) - 1  # position of the last emitted token (the root)
            tree = TT.TokenTree(emitted_all[-1], T)
            tree.insert([rnd.randrange(1000) for _ in range(3)], depth)       # a distractor first
            branch = tree.insert(P[len(emitted_all):len(emitted_all) + depth], depth)
            while len(tree) < T:
                tree.insert([rnd.randrange(1000) for _ in range(rnd.randrange(1, depth))], depth)
            greedy, commit = tv(eng, st, tree, pos0)
            emitted, path = tree.walk(greedy)
            assert path == branch, (path, branch)
            commit(path, pos0)
            emitted_all += emitted
            assert emitted_all == P[:len(emitted_all)], (emitted_all, P[:len(emitted_all)])
        # continue with plain decode steps from the compacted cache
        n = N - len(emitted_all)
        rest = list(eng._plain_steps(st, emitted_all[-1], S + len(emitted_all) - 1, n))
        tol = max(5e-2, 2 * load_golden("config0")["self_drift"]["max_logsoftmax_diff"])
        ok, where = _tie_ok(emitted_all + rest, P, logits, tol)
        assert ok, where
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
