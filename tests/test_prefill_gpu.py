"""Prompt (prefill) kernels on the GPU, through the C ABI, against CPU / fp64 references.

qd_tc_gemm (tcgen05, tiles of 128 tokens x 128 or 256 weight rows) is checked against an fp64 product
of the same BF16 operands with the same BF16 rounding points, for both tile widths, ragged token
counts (rows past m must stay untouched), an odd number of 128-row weight groups, strided rows, the
residual epilogue in place and the SwiGLU epilogue on the interleaved gate/up matrix. The tensor
cores accumulate in fp32 in their own order, so an output may sit one BF16 ulp away at a rounding
tie. qd_rmsnorm_rows and qd_prefill_qk_rope are checked against the oracle's op restatements
(oracle/qwen3_cpu.py, engine/engine.py:505-509 and :550-592), qd_prefill_attn against the exact
softmax in fp64 and against PyTorch's flash SDPA (the reference's prompt attention).
"""

import pytest
import torch

from oracle import qwen3_cpu as Q

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16
DEV = "cuda:0"
RTOL = 2.0 ** -7


def _ops():
    from decode_b200 import ops

    return ops


def _rand(shape, std, gen):
    return (torch.randn(shape, generator=gen) * std).to(BF16)


def _ref(x, w):
    """fp64 product of the BF16 operands, on the GPU (exact enough to be the rounding reference)."""
    return x.to(DEV).double() @ w.to(DEV).double().T


def _assert_close(ours, ref, extra=None, rtol=RTOL):
    ours, ref = ours.float(), ref.float().to(ours.device)
    tol = rtol * (ref.abs() + (extra.abs().to(ours.device) if extra is not None else 0)) + 1e-3
    bad = (ours - ref).abs() > tol
    assert not bad.any(), f"{int(bad.sum())} mismatches, max diff {float((ours - ref).abs().max()):.4g}"


# (m, n, k): ragged token tiles, an odd group count (n = 384), the model's projection shapes
SHAPES = [(1, 256, 128), (7, 384, 640), (128, 2560, 2560), (129, 6144, 2560), (300, 2560, 4096),
          (2048, 2560, 640), (517, 2560, 9728)]


@pytest.mark.parametrize("bn", ["128", "256"])
@pytest.mark.parametrize("m,n,k", SHAPES)
def test_tc_gemm_store(m, n, k, bn, monkeypatch):
    monkeypatch.setenv("QD_GEMM_BN", bn)
    ops = _ops()
    g = torch.Generator().manual_seed(m * 7 + n + k)
    x, w = _rand((m, k), 1.0, g), _rand((n, k), 0.02, g)
    out = torch.full((m + 5, n), float("nan"), dtype=BF16, device=DEV)  # rows m.. must stay untouched
    ops.tc_gemm(x.to(DEV), ops.pack_matrix(w.to(DEV)), n, out[:m])
    _assert_close(out[:m], _ref(x, w).to(BF16))
    assert torch.isnan(out[m:].float()).all()


def test_tc_gemm_plan_picks_wide_tiles_for_large_prompts():
    ops = _ops()
    sms = ops.sm_count()
    grid, bn, ks, nb = ops.tc_gemm_plan(16384, 19456, 2560)
    assert bn == 256 and grid == sms and ks == 1 and nb == 0
    grid, bn, ks, nb = ops.tc_gemm_plan(128, 2560, 4096)
    assert bn == 128 and ks > 1 and grid == min(sms, 20 * ks) and nb > 0


SPLIT_CASES = [("", 128, 2560, 4096, "res"), ("", 1, 2560, 9728, "res"), ("", 77, 6144, 2560, "store"),
               ("", 128, 19456, 2560, "swiglu"), ("", 300, 2560, 640, "store"),
               # whole waves of whole tiles, then the last wave's tiles split (hybrid)
               ("", 1024, 2560, 9728, "res"), ("", 1000, 2560, 4096, "store"), ("", 1024, 19456, 2560, "swiglu"),
               ("", 1100, 6144, 2560, "store")]
SPLIT_CASES += [(ks, m, n, k, e) for ks in ("2", "3") for (_, m, n, k, e) in SPLIT_CASES[:5]]
# 256-wide tiles over an odd group count: the repeated last group is never stored
SPLIT_CASES += [("2/256", 77, 384, 1280, "store"), ("3/256", 130, 384, 1280, "swiglu")]


@pytest.mark.parametrize("ksplit,m,n,k,epi", SPLIT_CASES)
def test_tc_gemm_split_k(m, n, k, epi, ksplit, monkeypatch):
    """K split across CTAs (the plan's own choice, or forced): the split tiles' fp32 partials summed in
    split order by the second launch, then the same epilogues; deterministic on a reused scratch."""
    if ksplit:
        ks_env, _, bn_env = ksplit.partition("/")
        monkeypatch.setenv("QD_GEMM_KSPLIT", ks_env)
        if bn_env:
            monkeypatch.setenv("QD_GEMM_BN", bn_env)
    ops = _ops()
    g = torch.Generator().manual_seed(m + n + k)
    x, w = _rand((m, k), 1.0, g), _rand((n, k), 0.02, g)
    _, _, ks, nb = ops.tc_gemm_plan(m, n, k)
    scratch = torch.full((max(nb, 1),), 0x7F, dtype=torch.uint8, device=DEV)  # contents do not matter
    xd = x.to(DEV)
    if epi == "swiglu":
        inter = n // 2
        wp = ops.pack_gate_up(w[:inter].to(DEV), w[inter:].to(DEV))
        outs = [torch.empty((m, inter), dtype=BF16, device=DEV) for _ in range(2)]
        for o in outs:
            ops.tc_gemm(xd, wp, n, o, epilogue=ops.Gemv.SWIGLU, scratch=scratch)
        gu = _ref(x, w).to(BF16)
        gv, uv = gu[:, :inter].float().cpu(), gu[:, inter:].float().cpu()
        sv = torch.nn.functional.silu(gv)
        _assert_close(outs[0], Q.swiglu(gu.cpu(), inter), extra=(1.1 * gv.abs() * uv.abs() + sv.abs() * uv.abs()),
                      rtol=2.0 ** -6)
    elif epi == "res":
        wp = ops.pack_matrix(w.to(DEV))
        res = _rand((m, n), 1.0, g).to(DEV)
        outs = [res.clone() for _ in range(2)]
        for o in outs:
            ops.tc_gemm(xd, wp, n, o, res=o, epilogue=ops.Gemv.RES, scratch=scratch)
        y = _ref(x, w).to(BF16).float()
        _assert_close(outs[0], (res.float() + y).to(BF16), extra=y)
    else:
        wp = ops.pack_matrix(w.to(DEV))
        outs = [torch.empty((m, n), dtype=BF16, device=DEV) for _ in range(2)]
        for o in outs:
            ops.tc_gemm(xd, wp, n, o, scratch=scratch)
        _assert_close(outs[0], _ref(x, w).to(BF16))
    assert torch.equal(outs[0], outs[1])


def test_tc_gemm_split_k_scratch_shared_across_shapes():
    """One scratch (arbitrary contents) serves split-K launches of different shapes in stream order, as
    the prompt forward uses it: each gives the bits of a launch on a fresh scratch."""
    ops = _ops()
    g = torch.Generator().manual_seed(11)
    shapes = [(128, 2560, 4096), (128, 6144, 2560), (1, 2560, 9728), (40, 2560, 1280), (128, 2560, 4096)]
    plans = [ops.tc_gemm_plan(*s) for s in shapes]
    assert all(p[2] > 1 for p in plans)
    shared = torch.full((max(p[3] for p in plans),), 0xA5, dtype=torch.uint8, device=DEV)
    for (m, n, k), (_, _, _, nb) in zip(shapes, plans):
        x, w = _rand((m, k), 1.0, g).to(DEV), ops.pack_matrix(_rand((n, k), 0.02, g).to(DEV))
        a = ops.tc_gemm(x, w, n, torch.empty((m, n), dtype=BF16, device=DEV), scratch=shared)
        b = ops.tc_gemm(x, w, n, torch.empty((m, n), dtype=BF16, device=DEV),
                        scratch=torch.zeros((nb,), dtype=torch.uint8, device=DEV))
        assert torch.equal(a, b), (m, n, k)


@pytest.mark.parametrize("bn", ["128", "256"])
@pytest.mark.parametrize("m,n,k", [(300, 2560, 4096), (1100, 2560, 9728), (5, 2560, 4096)])
def test_tc_gemm_residual_in_place_strided(m, n, k, bn, monkeypatch):
    """out = bf16(res + bf16(x W^T)) written over res, with x and res rows strided (every third row of
    a larger buffer, as the last-position rows of a prompt are)."""
    monkeypatch.setenv("QD_GEMM_BN", bn)
    ops = _ops()
    g = torch.Generator().manual_seed(m + 3 * n + k)
    x, w, res = _rand((m, k), 1.0, g), _rand((n, k), 0.02, g), _rand((m, n), 1.0, g)
    xb = torch.zeros((3 * m, k), dtype=BF16, device=DEV)
    xb[::3] = x.to(DEV)
    rb = torch.full((3 * m, n), float("nan"), dtype=BF16, device=DEV)
    rb[::3] = res.to(DEV)
    xr = rb[::3]
    ops.tc_gemm(xb[::3], ops.pack_matrix(w.to(DEV)), n, xr, res=xr, epilogue=ops.Gemv.RES)
    y = _ref(x, w).to(BF16).float()
    ref = (res.to(DEV).float() + y).to(BF16)
    # bf16(y) may round one ulp apart at a tie, and that ulp can carry into the rounded sum
    _assert_close(xr, ref, extra=y)
    assert torch.isnan(rb[1::3].float()).all() and torch.isnan(rb[2::3].float()).all()


@pytest.mark.parametrize("bn", ["128", "256"])
@pytest.mark.parametrize("m", [3, 300, 1500])
def test_tc_gemm_swiglu_gate_up(m, bn, monkeypatch):
    monkeypatch.setenv("QD_GEMM_BN", bn)
    ops = _ops()
    inter, k = 9728, 2560
    g = torch.Generator().manual_seed(inter + m)
    x, gate, up = _rand((m, k), 1.0, g), _rand((inter, k), 0.02, g), _rand((inter, k), 0.02, g)
    out = torch.empty((m, inter), dtype=BF16, device=DEV)
    ops.tc_gemm(x.to(DEV), ops.pack_gate_up(gate.to(DEV), up.to(DEV)), 2 * inter, out, epilogue=ops.Gemv.SWIGLU)
    gu = _ref(x, torch.cat([gate, up])).to(BF16)
    ref = Q.swiglu(gu.cpu(), inter)
    # a one-ulp difference in bf16(g) or bf16(u) at a rounding tie moves the output by up to
    # |u| |silu'(g)| ulp(g) + |silu(g)| ulp(u), with |silu'| < 1.1
    gv, uv = gu[:, :inter].float().cpu(), gu[:, inter:].float().cpu()
    sv = torch.nn.functional.silu(gv)
    _assert_close(out, ref, extra=(1.1 * gv.abs() * uv.abs() + sv.abs() * uv.abs()).to(DEV), rtol=2.0 ** -6)


def test_tc_gemm_deterministic_and_tile_width_independent(monkeypatch):
    """Without a K split each output is one tile's fp32 accumulation in K order: the same bits for either
    tile width and on every run."""
    monkeypatch.setenv("QD_GEMM_KSPLIT", "1")
    ops = _ops()
    g = torch.Generator().manual_seed(5)
    m, n, k = 2000, 6144, 2560
    x, w = _rand((m, k), 1.0, g).to(DEV), ops.pack_matrix(_rand((n, k), 0.02, g).to(DEV))
    outs = []
    for bn in ("256", "128", "256"):
        monkeypatch.setenv("QD_GEMM_BN", bn)
        o = torch.empty((m, n), dtype=BF16, device=DEV)
        ops.tc_gemm(x, w, n, o)
        outs.append(o)
    assert torch.equal(outs[0], outs[2]) and torch.equal(outs[0], outs[1])


def test_tc_gemm_lm_head_shape():
    """The prompt's LM head: 151936 vocabulary rows (1187 groups, odd) for a few last positions."""
    ops = _ops()
    g = torch.Generator().manual_seed(11)
    m, n, k = 4, 151936, 2560
    x, e = _rand((m, k), 1.0, g), _rand((n, k), 0.02, g)
    out = torch.empty((m, n), dtype=BF16, device=DEV)
    ops.tc_gemm(x.to(DEV), ops.pack_matrix(e.to(DEV)), n, out)
    ref = _ref(x, e).to(BF16).float()
    _assert_close(out, ref)
    # our argmax is the reference's, or a reference near-tie within one BF16 ulp of the best
    idx = out.float().argmax(-1)
    best = ref.max(-1).values
    at = ref.gather(1, idx[:, None])[:, 0]
    assert ((best - at) <= RTOL * best.abs() + 1e-3).all()


@pytest.mark.parametrize("m,k", [(1, 2560), (77, 2560), (3000, 2560), (5, 4096)])
def test_rmsnorm_rows(m, k):
    ops = _ops()
    g = torch.Generator().manual_seed(m + k)
    x = _rand((m, k), 1.0, g)
    w = (1.0 + 0.1 * torch.randn(k, generator=g)).to(BF16)
    out = torch.empty((m, k), dtype=BF16, device=DEV)
    ops.rmsnorm_rows(x.to(DEV), w.to(DEV), 1e-6, out)
    # two roundings (bf16(x * rstd), then bf16(w * that)): an fp32-level difference in rstd (sum order,
    # rsqrt vs 1/sqrt) that flips the inner rounding can leave the output two ulps apart
    _assert_close(out, Q.rms_norm(x, w, 1e-6).view(m, k), rtol=2.0 ** -6)


@pytest.mark.parametrize("b,S", [(1, 1), (1, 128), (3, 17), (2, 1024)])
def test_prefill_qk_rope_and_cache(b, S):
    ops = _ops()
    nq, nkv, D, eps = 32, 8, 128, 1e-6
    cap = S + 9
    g = torch.Generator().manual_seed(b * 100 + S)
    qkv = _rand((b * S, (nq + 2 * nkv) * D), 1.0, g)
    qn = (1.0 + 0.1 * torch.randn(D, generator=g)).to(BF16)
    kn = (1.0 + 0.1 * torch.randn(D, generator=g)).to(BF16)
    cos, sin = Q.rope_tables(cap, D, 5e6)
    q = torch.empty((b * S, nq * D), dtype=BF16, device=DEV)
    kc = torch.full((b, nkv, cap, D), float("nan"), dtype=BF16, device=DEV)
    vc = torch.full((b, nkv, cap, D), float("nan"), dtype=BF16, device=DEV)
    ops.prefill_qk_rope(qkv.to(DEV), b, S, nq, nkv, qn.to(DEV), kn.to(DEV), eps, cos.to(DEV), sin.to(DEV), q, kc, vc)
    # oracle: per-head norm, then RoPE at each token's own position s (engine/engine.py:566-572)
    c = cos[:S].repeat(b, 1)[:, None]
    s = sin[:S].repeat(b, 1)[:, None]
    qh = Q.rms_norm(qkv, qn, eps, nq)
    kh = Q.rms_norm(qkv[:, nq * D:], kn, eps, nkv)
    qr = (qh * c) + (Q.rotate_half(qh) * s)
    kr = (kh * c) + (Q.rotate_half(kh) * s)
    vr = qkv[:, (nq + nkv) * D:].view(b * S, nkv, D)

    def rope_tol(y):
        y = y.float()
        return (y * c.float()).abs() + (Q.rotate_half(y) * s.float()).abs()

    _assert_close(q.view(b * S, nq, D), qr, extra=rope_tol(qh))
    kcs = kc[:, :, :S].permute(0, 2, 1, 3).reshape(b * S, nkv, D)
    vcs = vc[:, :, :S].permute(0, 2, 1, 3).reshape(b * S, nkv, D)
    _assert_close(kcs, kr, extra=rope_tol(kh))
    assert torch.equal(vcs.cpu(), vr)
    assert torch.isnan(kc[:, :, S:].float()).all() and torch.isnan(vc[:, :, S:].float()).all()


def _attn_ref(q, kc, vc, b, S, nq, nkv, q_begin):
    """fp64 causal GQA attention of positions q_begin..S-1 (exact softmax), rows i * (S - q_begin) + s."""
    D = 128
    qd = q.to(DEV).double().view(b, S, nq, D).transpose(1, 2)                     # [b, nq, S, D]
    k = kc[:, :, :S].to(DEV).double().repeat_interleave(nq // nkv, dim=1)        # [b, nq, S, D]
    v = vc[:, :, :S].to(DEV).double().repeat_interleave(nq // nkv, dim=1)
    s = (qd @ k.transpose(-1, -2)) / (D ** 0.5)
    mask = torch.ones((S, S), dtype=torch.bool, device=DEV).tril()
    s = s.masked_fill(~mask, float("-inf"))
    o = torch.softmax(s, -1) @ v                                                   # [b, nq, S, D]
    return o[:, :, q_begin:].transpose(1, 2).reshape(b * (S - q_begin), nq * D)


@pytest.mark.parametrize("variant", ["1", "2"])
@pytest.mark.parametrize("b,S", [(1, 1), (1, 127), (1, 128), (3, 17), (2, 300), (1, 1024)])
@pytest.mark.parametrize("q_mode", ["all", "last", "middle"])
def test_prefill_attn_causal_gqa(b, S, q_mode, variant, monkeypatch):
    """Against the exact softmax, with NaN in every cache slot past the prompt (never read): P is
    rounded to BF16 before P.V (as flash attention does), so an output may differ by a few ulp of the
    values it averages (|v| <= ~5 here), hence the absolute term. Variant 2 is the two-query-tile
    kernel with P in tensor memory (QD_PREFILL_ATTN=2)."""
    monkeypatch.setenv("QD_PREFILL_ATTN", variant)
    ops = _ops()
    nq, nkv, D = 32, 8, 128
    cap = S + 40
    g = torch.Generator().manual_seed(b * 1000 + S)
    q = _rand((b * S, nq * D), 1.0, g)
    kc = torch.full((b, nkv, cap, D), float("nan"), dtype=BF16)
    vc = torch.full((b, nkv, cap, D), float("nan"), dtype=BF16)
    kc[:, :, :S] = _rand((b, nkv, S, D), 1.0, g)
    vc[:, :, :S] = _rand((b, nkv, S, D), 1.0, g)
    q0 = {"all": 0, "last": S - 1, "middle": S // 2}[q_mode]
    rows = b * (S - q0)
    out = torch.full((rows + 2, nq * D), float("nan"), dtype=BF16, device=DEV)
    ops.prefill_attn(q.to(DEV), b, S, nq, nkv, kc.to(DEV), vc.to(DEV), out[:rows], q_begin=q0)
    ref = _attn_ref(q, kc, vc, b, S, nq, nkv, q0).float()
    _assert_close(out[:rows], ref, extra=torch.ones_like(ref), rtol=2.0 ** -6)
    assert torch.isnan(out[rows:].float()).all()


@pytest.mark.parametrize("variant", ["1", "2"])
def test_prefill_attn_matches_torch_flash_sdpa(variant, monkeypatch):
    """The same computation as the reference's prompt attention (flash SDPA, enable_gqa), to within
    the BF16 rounding of the probabilities and of the output."""
    monkeypatch.setenv("QD_PREFILL_ATTN", variant)
    ops = _ops()
    b, S, nq, nkv, D = 2, 700, 32, 8, 128
    g = torch.Generator().manual_seed(77)
    q = _rand((b * S, nq * D), 1.0, g).to(DEV)
    kc = _rand((b, nkv, S, D), 1.0, g).to(DEV)
    vc = _rand((b, nkv, S, D), 1.0, g).to(DEV)
    out = torch.empty((b * S, nq * D), dtype=BF16, device=DEV)
    ops.prefill_attn(q, b, S, nq, nkv, kc, vc, out)
    ref = torch.nn.functional.scaled_dot_product_attention(q.view(b, S, nq, D).transpose(1, 2), kc, vc, is_causal=True,
                                                           scale=D ** -0.5, enable_gqa=True)
    ref = ref.transpose(1, 2).reshape(b * S, nq * D).float()
    _assert_close(out, ref, extra=torch.ones_like(ref), rtol=2.0 ** -6)


@pytest.mark.parametrize("variant", ["1", "2"])
def test_prefill_attn_deterministic(variant, monkeypatch):
    monkeypatch.setenv("QD_PREFILL_ATTN", variant)
    ops = _ops()
    b, S, nq, nkv, D = 2, 513, 32, 8, 128
    g = torch.Generator().manual_seed(3)
    q = _rand((b * S, nq * D), 1.0, g).to(DEV)
    kc = _rand((b, nkv, S, D), 1.0, g).to(DEV)
    vc = _rand((b, nkv, S, D), 1.0, g).to(DEV)
    o1 = torch.empty((b * S, nq * D), dtype=BF16, device=DEV)
    o2 = torch.empty_like(o1)
    ops.prefill_attn(q, b, S, nq, nkv, kc, vc, o1)
    ops.prefill_attn(q, b, S, nq, nkv, kc, vc, o2)
    assert torch.equal(o1, o2)


@pytest.mark.parametrize("b,S,T", [(1, 9, 7), (1, 300, 50), (2, 140, 8), (3, 17, 17)])
def test_prefill_qk_rope_at_equals_whole_prompt(b, S, T):
    """Tokens at positions S - T .. S - 1 (qd_prefill_qk_rope_at, the speculative verify's q/k RoPE and
    K/V write) give the bits of the same tokens inside a whole-prompt call, and write no other slot."""
    ops = _ops()
    nq, nkv, D, eps = 32, 8, 128, 1e-6
    cap, pos0 = S + 5, S - T
    g = torch.Generator().manual_seed(b + S + T)
    qkv = _rand((b * S, (nq + 2 * nkv) * D), 1.0, g).to(DEV)
    qn = (1.0 + 0.1 * torch.randn(D, generator=g)).to(BF16).to(DEV)
    kn = (1.0 + 0.1 * torch.randn(D, generator=g)).to(BF16).to(DEV)
    cos, sin = (t.to(DEV) for t in Q.rope_tables(cap, D, 5e6))
    q_all = torch.empty((b * S, nq * D), dtype=BF16, device=DEV)
    kc_all = torch.full((b, nkv, cap, D), float("nan"), dtype=BF16, device=DEV)
    vc_all = torch.full_like(kc_all, float("nan"))
    ops.prefill_qk_rope(qkv, b, S, nq, nkv, qn, kn, eps, cos, sin, q_all, kc_all, vc_all)
    tail = qkv.view(b, S, -1)[:, pos0:].reshape(b * T, -1)
    q_t = torch.empty((b * T, nq * D), dtype=BF16, device=DEV)
    kc = torch.full_like(kc_all, float("nan"))
    vc = torch.full_like(kc_all, float("nan"))
    ops.prefill_qk_rope(tail, b, T, nq, nkv, qn, kn, eps, cos, sin, q_t, kc, vc, pos0=pos0)
    assert torch.equal(q_t, q_all.view(b, S, -1)[:, pos0:].reshape(b * T, -1))
    assert torch.equal(kc[:, :, pos0:S], kc_all[:, :, pos0:S]) and torch.equal(vc[:, :, pos0:S], vc_all[:, :, pos0:S])
    assert torch.isnan(kc[:, :, :pos0].float()).all() and torch.isnan(kc[:, :, S:].float()).all()
    assert torch.isnan(vc[:, :, :pos0].float()).all() and torch.isnan(vc[:, :, S:].float()).all()


@pytest.mark.parametrize("variant", ["1", "2"])
@pytest.mark.parametrize("b,S,q0", [(1, 7, 0), (1, 300, 250), (1, 135, 127), (2, 140, 133), (3, 17, 16),
                                    (1, 1030, 1023)])
def test_prefill_attn_rows(b, S, q0, variant, monkeypatch):
    """q holding only the computed rows (qd_prefill_attn_rows, the speculative verify's attention over the
    cached prefix), including query rows that cross a 128-row tile, against the exact softmax as the
    full-q call is. (Not bit-equal to the full-q call: the rows of a query tile before q_begin read as
    zero here, and a warp's rescale decision is shared by its rows.)"""
    monkeypatch.setenv("QD_PREFILL_ATTN", variant)
    ops = _ops()
    nq, nkv, D = 32, 8, 128
    g = torch.Generator().manual_seed(b * 7 + S + q0)
    q = _rand((b * S, nq * D), 1.0, g).to(DEV)
    kc = _rand((b, nkv, S + 3, D), 1.0, g).to(DEV)
    vc = _rand((b, nkv, S + 3, D), 1.0, g).to(DEV)
    rows = b * (S - q0)
    qr = q.view(b, S, -1)[:, q0:].reshape(rows, -1).clone()
    out = torch.full((rows + 2, nq * D), float("nan"), dtype=BF16, device=DEV)
    ops.prefill_attn(qr, b, S, nq, nkv, kc, vc, out[:rows], q_begin=q0, q_rows=True)
    ref = _attn_ref(q, kc, vc, b, S, nq, nkv, q0).float()
    _assert_close(out[:rows], ref, extra=torch.ones_like(ref), rtol=2.0 ** -6)
    assert torch.isnan(out[rows:].float()).all()
    again = torch.empty((rows, nq * D), dtype=BF16, device=DEV)
    ops.prefill_attn(qr, b, S, nq, nkv, kc, vc, again, q_begin=q0, q_rows=True)
    assert torch.equal(out[:rows], again)
