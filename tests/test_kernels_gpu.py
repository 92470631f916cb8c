"""Per-kernel parity on the GPU, through the C ABI, against CPU references.

The references are the oracle's op restatements (oracle/qwen3_cpu.py, which follow the reference
engine's torch path op by op) or, for the plain projections, an fp64 product of the same BF16
operands with the same BF16 rounding points. Tolerances are stated per test: reduction order on the
GPU differs from the CPU, so an output may sit one BF16 ulp (2^-8 relative) away at a rounding tie.
"""

import math

import pytest
import torch

from packref import gate_up_interleaved, pack_reference
from oracle import qwen3_cpu as Q

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16
DEV = "cuda:0"
RTOL = 2.0 ** -7   # two BF16 ulps relative


def _ops():
    from decode_b200 import ops

    return ops


def _rand(shape, std, gen):
    return (torch.randn(shape, generator=gen) * std).to(BF16)


def _norm_ref(x, w, eps):
    return Q.rms_norm(x, w, eps).view(x.shape[0], -1)


def _assert_bf16_close(ours, ref, scale=1.0, rtol=RTOL):
    ours, ref = ours.float().cpu(), ref.float().cpu()
    tol = rtol * ref.abs() + 1e-3 * scale
    bad = (ours - ref).abs() > tol
    assert not bad.any(), f"{int(bad.sum())} mismatches, max diff {float((ours - ref).abs().max()):.4g}"


# ------------------------------------------------------------------------------------ packing / embed
@pytest.mark.parametrize("n,k", [(256, 128), (6144, 2560), (2560, 9728)])
def test_pack_matches_layout_restatement(n, k):
    ops = _ops()
    g = torch.Generator().manual_seed(n + k)
    w = _rand((n, k), 0.02, g)
    packed = ops.pack_matrix(w.to(DEV))
    assert torch.equal(packed.cpu().view(torch.int16), pack_reference(w).view(torch.int16))


def test_pack_gate_up_interleave():
    ops = _ops()
    g = torch.Generator().manual_seed(3)
    gate, up = _rand((256, 128), 0.02, g), _rand((256, 128), 0.02, g)
    packed = ops.pack_gate_up(gate.to(DEV), up.to(DEV))
    ref = pack_reference(gate_up_interleaved(gate, up))
    assert torch.equal(packed.cpu().view(torch.int16), ref.view(torch.int16))


def test_embed_gathers_rows_bit_exact():
    ops = _ops()
    g = torch.Generator().manual_seed(4)
    E = _rand((1024, 2560), 0.02, g)
    ep = ops.pack_matrix(E.to(DEV))
    tok = torch.tensor([0, 1023, 517, 128, 5], dtype=torch.int64, device=DEV)
    x = torch.empty((5, 2560), dtype=BF16, device=DEV)
    err = torch.zeros((1,), dtype=torch.int32, device=DEV)
    ops.embed(tok, ep, 1024, x, err)
    assert torch.equal(x.cpu(), E[tok.cpu()])
    assert int(err.item()) == 0
    bad = torch.tensor([1024], dtype=torch.int64, device=DEV)       # out of range: clamped + flagged
    ops.embed(bad, ep, 1024, x[:1], err)
    assert int(err.item()) == 8 and torch.equal(x[:1].cpu(), E[1023:1024])


# ------------------------------------------------------------------------------------ GEMV
SHAPES = [(6144, 2560), (2560, 4096), (19456, 2560), (2560, 9728), (256, 128), (384, 192), (1024, 640)]


def _gemv_ref(x, w, norm_w, eps):
    xn = _norm_ref(x, norm_w, eps) if norm_w is not None else x
    return xn.double() @ w.double().T          # exact products of the BF16 operands


@pytest.mark.parametrize("n,k", SHAPES)
@pytest.mark.parametrize("m", [1, 3, 4, 8])
@pytest.mark.parametrize("norm", [False, True])
def test_gemv_store(n, k, m, norm):
    ops = _ops()
    g = torch.Generator().manual_seed(n * 7 + k + m)
    x, w = _rand((m, k), 1.0, g), _rand((n, k), 0.02, g)
    nw = (1.0 + 0.1 * torch.randn(k, generator=g)).to(BF16) if norm else None
    plan = ops.Gemv(m, n, k, ops.Gemv.STORE, DEV)
    out = torch.full((m, n), float("nan"), dtype=BF16, device=DEV)
    plan(x.to(DEV), ops.pack_matrix(w.to(DEV)), out, norm_w=nw.to(DEV) if norm else None)
    ref = _gemv_ref(x, w, nw, 1e-6).to(BF16)
    _assert_bf16_close(out, ref)


@pytest.mark.parametrize("n,k", [(2560, 4096), (2560, 9728), (256, 128)])
@pytest.mark.parametrize("m", [1, 2, 5, 8])
def test_gemv_residual_in_place(n, k, m):
    ops = _ops()
    g = torch.Generator().manual_seed(n + k * 3 + m)
    x, w, res = _rand((m, k), 1.0, g), _rand((n, k), 0.02, g), _rand((m, n), 1.0, g)
    plan = ops.Gemv(m, n, k, ops.Gemv.RES, DEV)
    xr = res.to(DEV).clone()
    plan(x.to(DEV), ops.pack_matrix(w.to(DEV)), xr, res=xr)                 # out aliases res (x += ...)
    y = _gemv_ref(x, w, None, 0).to(BF16).float()
    ref = (res.float() + y).to(BF16)
    # bf16(y) may round one ulp apart at a tie (fp32 against fp64 sums), and that ulp can carry into the
    # rounded sum
    diff = (xr.float().cpu() - ref.float()).abs()
    tol = RTOL * (ref.float().abs() + y.abs()) + 1e-3
    assert not (diff > tol).any(), f"{int((diff > tol).sum())} mismatches, max diff {float(diff.max()):.4g}"


@pytest.mark.parametrize("inter,k", [(9728, 2560), (128, 128), (320, 192)])
@pytest.mark.parametrize("m", [1, 4, 8])
def test_gemv_swiglu_gate_up(inter, k, m):
    ops = _ops()
    g = torch.Generator().manual_seed(inter + k + m)
    x, gate, up = _rand((m, k), 1.0, g), _rand((inter, k), 0.02, g), _rand((inter, k), 0.02, g)
    nw = (1.0 + 0.1 * torch.randn(k, generator=g)).to(BF16)
    plan = ops.Gemv(m, 2 * inter, k, ops.Gemv.SWIGLU, DEV)
    out = torch.empty((m, inter), dtype=BF16, device=DEV)
    plan(x.to(DEV), ops.pack_gate_up(gate.to(DEV), up.to(DEV)), out, norm_w=nw.to(DEV))
    gu = _gemv_ref(x, torch.cat([gate, up]), nw, 1e-6).to(BF16)
    ref = Q.swiglu(gu, inter)
    _assert_bf16_close(out, ref, rtol=2.0 ** -6)


@pytest.mark.parametrize("grid", [1, 7, 148, 300])
def test_gemv_grid_independent_of_partition(grid):
    """Every stream-K partition (one CTA, a few, one per SM, more than SMs) gives the same result up
    to summation order; a fixed partition is bit-reproducible."""
    ops = _ops()
    g = torch.Generator().manual_seed(11)
    m, n, k = 2, 1024, 640
    x, w = _rand((m, k), 1.0, g), _rand((n, k), 0.02, g)
    wp = ops.pack_matrix(w.to(DEV))
    plan = ops.Gemv(m, n, k, ops.Gemv.STORE, DEV, grid=grid)
    a = torch.empty((m, n), dtype=BF16, device=DEV)
    b = torch.empty((m, n), dtype=BF16, device=DEV)
    plan(x.to(DEV), wp, a)
    plan(x.to(DEV), wp, b)
    assert torch.equal(a, b)
    _assert_bf16_close(a, _gemv_ref(x, w, None, 0).to(BF16))


# ------------------------------------------------------------------------------------ QKV + RoPE + append
@pytest.mark.parametrize("m", [1, 3, 8])
@pytest.mark.parametrize("pos", [0, 77, 383])
def test_qkv_rope_append(m, pos):
    ops = _ops()
    H, nq, nkv, D, cap, eps = 2560, 32, 8, 128, 384, 1e-6
    g = torch.Generator().manual_seed(m * 1000 + pos)
    x = _rand((m, H), 1.0, g)
    w = _rand(((nq + 2 * nkv) * D, H), 0.02, g)
    ln = (1.0 + 0.1 * torch.randn(H, generator=g)).to(BF16)
    qn = (1.0 + 0.1 * torch.randn(D, generator=g)).to(BF16)
    kn = (1.0 + 0.1 * torch.randn(D, generator=g)).to(BF16)
    cos, sin = Q.rope_tables(cap, D, 5e6)
    plan = ops.QkvRopeAppend(m, H, nq, nkv, DEV)
    kc = torch.full((m, nkv, cap, D), float("nan"), dtype=BF16, device=DEV)
    vc = torch.full((m, nkv, cap, D), float("nan"), dtype=BF16, device=DEV)
    q = torch.empty((m, nq, D), dtype=BF16, device=DEV)
    raw = torch.empty((m, (nq + 2 * nkv) * D), dtype=BF16, device=DEV)
    posd = torch.tensor([pos], dtype=torch.int64, device=DEV)
    plan(x.to(DEV), ops.pack_matrix(w.to(DEV)), ln.to(DEV), qn.to(DEV), kn.to(DEV), cos.to(DEV), sin.to(DEV), posd,
         q, kc, vc, raw_out=raw)
    # projection: fp64 reference of the same operands
    _assert_bf16_close(raw, _gemv_ref(x, w, ln, eps).to(BF16))
    # epilogue: the oracle's q/k norm + RoPE applied to this kernel's own BF16 projection
    qr, kr, vr = Q.qk_norm_rope(raw.cpu(), qn, kn, cos[pos], sin[pos], eps)
    _assert_bf16_close(q, qr)
    _assert_bf16_close(kc[:, :, pos], kr)
    assert torch.equal(vc[:, :, pos].cpu(), vr)
    # nothing else in the cache was touched
    others = torch.ones(cap, dtype=torch.bool)
    others[pos] = False
    assert torch.isnan(kc[:, :, others].float()).all() and torch.isnan(vc[:, :, others].float()).all()


# ------------------------------------------------------------------------------------ attention
@pytest.mark.parametrize("B,L,cap", [(1, 1, 384), (1, 129, 384), (1, 384, 384), (3, 200, 256), (8, 1000, 1024),
                                     (2, 64, 65), (1, 4096, 8192)])
def test_attention_decode(B, L, cap):
    ops = _ops()
    nq, nkv, D = 32, 8, 128
    g = torch.Generator().manual_seed(B * 10000 + L)
    q = _rand((B, nq, D), 1.0, g)
    kc = torch.full((B, nkv, cap, D), float("nan"), dtype=BF16)     # poisoned beyond the valid length
    vc = torch.full((B, nkv, cap, D), float("nan"), dtype=BF16)
    kc[:, :, :L] = _rand((B, nkv, L, D), 1.0, g)
    vc[:, :, :L] = _rand((B, nkv, L, D), 1.0, g)
    attn = ops.DecodeAttention(B, nq, nkv, cap, DEV)
    out = torch.empty((B, nq, D), dtype=BF16, device=DEV)
    pos = torch.tensor([L - 1], dtype=torch.int64, device=DEV)
    attn(q.to(DEV), kc.to(DEV), vc.to(DEV), pos, out)
    ref = Q.attention_decode(q, kc, vc, L)
    o = out.float().cpu()
    assert torch.isfinite(o).all()
    assert (o - ref.float()).abs().max().item() < 2e-2
    # fp32 math reference (no BF16 rounding of probabilities): same bound
    s = torch.einsum("bhd,bhnd->bhn", q.float(), Q.repeat_kv(kc[:, :, :L]).float()) / math.sqrt(D)
    ref32 = torch.einsum("bhn,bhnd->bhd", torch.softmax(s, -1), Q.repeat_kv(vc[:, :, :L]).float())
    assert (o - ref32).abs().max().item() < 2e-2


def test_attention_deterministic_and_ticket_reset():
    ops = _ops()
    B, nq, nkv, D, cap, L = 2, 32, 8, 128, 512, 300
    g = torch.Generator().manual_seed(5)
    q = _rand((B, nq, D), 1.0, g).to(DEV)
    kc = _rand((B, nkv, cap, D), 1.0, g).to(DEV)
    vc = _rand((B, nkv, cap, D), 1.0, g).to(DEV)
    attn = ops.DecodeAttention(B, nq, nkv, cap, DEV)
    pos = torch.tensor([L - 1], dtype=torch.int64, device=DEV)
    outs = []
    for _ in range(3):
        out = torch.empty((B, nq, D), dtype=BF16, device=DEV)
        attn(q, kc, vc, pos, out)
        outs.append(out)
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])


# ------------------------------------------------------------------------------------ LM head
@pytest.mark.parametrize("m", [1, 2, 8])
def test_lm_head_argmax_and_logits(m):
    ops = _ops()
    V, H, eps = 151936, 2560, 1e-6
    g = torch.Generator().manual_seed(100 + m)
    x = _rand((m, H), 1.0, g)
    E = _rand((V, H), 0.02, g)
    nw = (1.0 + 0.1 * torch.randn(H, generator=g)).to(BF16)
    lm = ops.LmHeadArgmax(m, V, H, DEV)
    tok = torch.full((m,), -1, dtype=torch.int64, device=DEV)
    pos = torch.tensor([41], dtype=torch.int64, device=DEV)
    logits = torch.empty((m, V), dtype=BF16, device=DEV)
    lm(x.to(DEV), ops.pack_matrix(E.to(DEV)), nw.to(DEV), tok, pos, inc_pos=True, logits=logits)
    ref = (_norm_ref(x, nw, eps).float() @ E.float().T).to(BF16)
    _assert_bf16_close(logits, ref)
    lo = logits.cpu()
    for i in range(m):
        t = int(tok[i])
        # exact argmax of the kernel's own BF16 logits, lowest index on ties
        assert t == int(Q.argmax_lowest(lo[i:i + 1]))
        assert Q.token_ok(t, ref[i], 2.0 ** -6 * float(ref[i].float().abs().max()))
    assert int(pos.item()) == 42


def test_lm_head_ties_pick_lowest_index():
    ops = _ops()
    V, H = 1024, 128
    x = torch.zeros((1, H), dtype=BF16)
    x[0, 0] = 1.0
    E = torch.zeros((V, H), dtype=BF16)
    for r in (700, 300, 900):      # three exact ties at the maximum
        E[r, 0] = 2.0
    lm = ops.LmHeadArgmax(1, V, H, DEV)
    tok = torch.empty((1,), dtype=torch.int64, device=DEV)
    lm(x.to(DEV), ops.pack_matrix(E.to(DEV)), torch.ones(H, dtype=BF16, device=DEV), tok)
    assert int(tok.item()) == 300
