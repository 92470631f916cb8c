"""Tensor-core (tcgen05) batch path on the GPU, through the C ABI, against CPU references.

Same references and tolerances as the CUDA-core kernels (test_kernels_gpu.py): an fp64 product of the
same BF16 operands with the same BF16 rounding points, and the oracle's op restatements for the fused
epilogues. The tensor cores accumulate in fp32 in their own order, so an output may sit one BF16 ulp
away at a rounding tie.
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


def _norm_ref(x, w, eps):
    return Q.rms_norm(x, w, eps).view(x.shape[0], -1)


def _gemv_ref(x, w, norm_w, eps):
    xn = _norm_ref(x, norm_w, eps) if norm_w is not None else x
    return xn.double() @ w.double().T


def _assert_bf16_close(ours, ref, scale=1.0, rtol=RTOL):
    ours, ref = ours.float().cpu(), ref.float().cpu()
    tol = rtol * ref.abs() + 1e-3 * scale
    bad = (ours - ref).abs() > tol
    assert not bad.any(), f"{int(bad.sum())} mismatches, max diff {float((ours - ref).abs().max()):.4g}"


def _assert_rope_close(ours, ref, y, c, s):
    """RoPE output y*c + rotate_half(y)*s with each product rounded to BF16: a one-ulp difference in the
    normalised head y (sum-of-squares order at a rounding tie) moves each product by up to one ulp of
    the product, which cancellation in the sum does not shrink."""
    y = y.float()
    yp = torch.cat([y[..., 64:], y[..., :64]], -1)
    terms = (y * c.float()).abs() + (yp * s.float()).abs()
    diff = (ours.float().cpu() - ref.float()).abs()
    tol = RTOL * (ref.float().abs() + terms) + 1e-3
    assert not (diff > tol).any(), f"{int((diff > tol).sum())} mismatches, max diff {float(diff.max()):.4g}"


def _pack_act_reference(xn: torch.Tensor, n_pad: int) -> torch.Tensor:
    """[k/64][n_pad][64] tiles, 16-byte chunk c of row m at chunk c ^ (m & 7), padding rows zero."""
    m, k = xn.shape
    out = torch.zeros((k // 64, n_pad, 8, 8), dtype=BF16)
    src = xn.view(m, k // 64, 8, 8).permute(1, 0, 2, 3)            # [kb][m][chunk][8]
    for r in range(m):
        perm = [c ^ (r & 7) for c in range(8)]
        out[:, r, perm] = src[:, r]
    return out.reshape(-1)


@pytest.mark.parametrize("m,k", [(9, 128), (16, 2560), (33, 640), (64, 9728)])
def test_pack_act_layout(m, k):
    ops = _ops()
    g = torch.Generator().manual_seed(m + k)
    x = _rand((m, k), 1.0, g)
    xp = ops.PackedActivations(m, k, DEV).pack(x.to(DEV))
    assert torch.equal(xp.t.cpu().view(torch.int16), _pack_act_reference(x, xp.n_pad).view(torch.int16))
    nw = (1.0 + 0.1 * torch.randn(k, generator=g)).to(BF16)
    xp.pack(x.to(DEV), norm_w=nw.to(DEV))
    ref = _pack_act_reference(_norm_ref(x, nw, 1e-6), xp.n_pad)
    _assert_bf16_close(xp.t, ref)


SHAPES = [(6144, 2560), (2560, 4096), (19456, 2560), (2560, 9728), (256, 128), (1024, 640)]


@pytest.mark.parametrize("n,k", SHAPES)
@pytest.mark.parametrize("m", [9, 16, 40, 64])
def test_tc_gemv_store(n, k, m):
    ops = _ops()
    g = torch.Generator().manual_seed(n * 5 + k + m)
    x, w = _rand((m, k), 1.0, g), _rand((n, k), 0.02, g)
    nw = (1.0 + 0.1 * torch.randn(k, generator=g)).to(BF16)
    xp = ops.PackedActivations(m, k, DEV).pack(x.to(DEV), norm_w=nw.to(DEV))
    plan = ops.TcGemv(m, n, k, ops.TcGemv.STORE, DEV)
    out = torch.full((m + 3, n), float("nan"), dtype=BF16, device=DEV)   # rows m.. must stay untouched
    plan(xp, ops.pack_matrix(w.to(DEV)), out[:m])
    ref = _gemv_ref(x, w, nw, 1e-6).to(BF16)
    _assert_bf16_close(out[:m], ref)
    assert torch.isnan(out[m:].float()).all()


@pytest.mark.parametrize("n,k", [(2560, 4096), (2560, 9728)])
@pytest.mark.parametrize("m", [12, 32, 64])
def test_tc_gemv_residual_in_place(n, k, m):
    ops = _ops()
    g = torch.Generator().manual_seed(n + 3 * k + m)
    x, w, res = _rand((m, k), 1.0, g), _rand((n, k), 0.02, g), _rand((m, n), 1.0, g)
    xp = ops.PackedActivations(m, k, DEV).pack(x.to(DEV))
    plan = ops.TcGemv(m, n, k, ops.TcGemv.RES, DEV)
    xr = res.to(DEV).clone()
    plan(xp, ops.pack_matrix(w.to(DEV)), xr, res=xr)
    y = _gemv_ref(x, w, None, 0).to(BF16).float()
    ref = (res.float() + y).to(BF16)
    # bf16(y) may round one ulp apart at a tie, and that ulp can carry into the rounded sum
    diff = (xr.float().cpu() - ref.float()).abs()
    tol = RTOL * (ref.float().abs() + y.abs()) + 1e-3
    assert not (diff > tol).any(), f"{int((diff > tol).sum())} mismatches, max diff {float(diff.max()):.4g}"


@pytest.mark.parametrize("m", [16, 48, 64])
def test_tc_gemv_swiglu_gate_up(m):
    ops = _ops()
    inter, k = 9728, 2560
    g = torch.Generator().manual_seed(inter + m)
    x, gate, up = _rand((m, k), 1.0, g), _rand((inter, k), 0.02, g), _rand((inter, k), 0.02, g)
    nw = (1.0 + 0.1 * torch.randn(k, generator=g)).to(BF16)
    xp = ops.PackedActivations(m, k, DEV).pack(x.to(DEV), norm_w=nw.to(DEV))
    plan = ops.TcGemv(m, 2 * inter, k, ops.TcGemv.SWIGLU, DEV)
    out = torch.empty((m, inter), dtype=BF16, device=DEV)
    plan(xp, ops.pack_gate_up(gate.to(DEV), up.to(DEV)), out)
    gu = _gemv_ref(x, torch.cat([gate, up]), nw, 1e-6).to(BF16)
    _assert_bf16_close(out, Q.swiglu(gu, inter), rtol=2.0 ** -6)


@pytest.mark.parametrize("grid", [1, 37, 148])
def test_tc_grid_independent_and_deterministic(grid):
    ops = _ops()
    g = torch.Generator().manual_seed(21)
    m, n, k = 24, 1024, 640
    x, w = _rand((m, k), 1.0, g), _rand((n, k), 0.02, g)
    xp = ops.PackedActivations(m, k, DEV).pack(x.to(DEV))
    wp = ops.pack_matrix(w.to(DEV))
    plan = ops.TcGemv(m, n, k, ops.TcGemv.STORE, DEV, grid=grid)
    a = torch.empty((m, n), dtype=BF16, device=DEV)
    b = torch.empty((m, n), dtype=BF16, device=DEV)
    plan(xp, wp, a)
    plan(xp, wp, b)
    assert torch.equal(a, b)
    _assert_bf16_close(a, _gemv_ref(x, w, None, 0).to(BF16))


def test_tc_matches_cuda_core_gemv_at_eight_rows():
    """The two paths agree (up to summation order) where both apply."""
    ops = _ops()
    g = torch.Generator().manual_seed(8)
    m, n, k = 8, 6144, 2560
    x, w = _rand((m, k), 1.0, g), _rand((n, k), 0.02, g)
    nw = (1.0 + 0.1 * torch.randn(k, generator=g)).to(BF16).to(DEV)
    wp = ops.pack_matrix(w.to(DEV))
    a = torch.empty((m, n), dtype=BF16, device=DEV)
    b = torch.empty((m, n), dtype=BF16, device=DEV)
    ops.Gemv(m, n, k, ops.Gemv.STORE, DEV)(x.to(DEV), wp, a, norm_w=nw)
    ops.TcGemv(m, n, k, ops.TcGemv.STORE, DEV)(ops.PackedActivations(m, k, DEV).pack(x.to(DEV), norm_w=nw), wp, b)
    diff = (a.float() - b.float()).abs()
    assert float(diff.max()) <= 2.0 ** -7 * float(a.float().abs().max())


@pytest.mark.parametrize("m", [16, 64])
@pytest.mark.parametrize("pos", [0, 1100])
def test_tc_qkv_rope_append(m, pos):
    ops = _ops()
    H, nq, nkv, D, cap, eps = 2560, 32, 8, 128, 1536, 1e-6
    g = torch.Generator().manual_seed(m * 1000 + pos)
    x = _rand((m, H), 1.0, g)
    w = _rand(((nq + 2 * nkv) * D, H), 0.02, g)
    ln = (1.0 + 0.1 * torch.randn(H, generator=g)).to(BF16)
    qn = (1.0 + 0.1 * torch.randn(D, generator=g)).to(BF16)
    kn = (1.0 + 0.1 * torch.randn(D, generator=g)).to(BF16)
    cos, sin = Q.rope_tables(cap, D, 5e6)
    xp = ops.PackedActivations(m, H, DEV).pack(x.to(DEV), norm_w=ln.to(DEV))
    plan = ops.TcQkvRopeAppend(m, H, nq, nkv, DEV)
    kc = torch.full((m, nkv, cap, D), float("nan"), dtype=BF16, device=DEV)
    vc = torch.full((m, nkv, cap, D), float("nan"), dtype=BF16, device=DEV)
    q = torch.empty((m, nq, D), dtype=BF16, device=DEV)
    raw = torch.empty((m, (nq + 2 * nkv) * D), dtype=BF16, device=DEV)
    posd = torch.tensor([pos], dtype=torch.int64, device=DEV)
    plan(xp, ops.pack_matrix(w.to(DEV)), qn.to(DEV), kn.to(DEV), cos.to(DEV), sin.to(DEV), posd, q, kc, vc,
         raw_out=raw)
    _assert_bf16_close(raw, _gemv_ref(x, w, ln, eps).to(BF16))
    rc = raw.cpu()
    qr, kr, vr = Q.qk_norm_rope(rc, qn, kn, cos[pos], sin[pos], eps)
    _assert_rope_close(q, qr, Q.rms_norm(rc, qn, eps, nq), cos[pos], sin[pos])
    _assert_rope_close(kc[:, :, pos], kr, Q.rms_norm(rc[:, nq * D:], kn, eps, nkv), cos[pos], sin[pos])
    assert torch.equal(vc[:, :, pos].cpu(), vr)
    others = torch.ones(cap, dtype=torch.bool)
    others[pos] = False
    assert torch.isnan(kc[:, :, others].float()).all() and torch.isnan(vc[:, :, others].float()).all()


@pytest.mark.parametrize("m", [10, 64])
def test_tc_lm_head_argmax_and_logits(m):
    ops = _ops()
    V, H, eps = 151936, 2560, 1e-6
    g = torch.Generator().manual_seed(300 + m)
    x = _rand((m, H), 1.0, g)
    E = _rand((V, H), 0.02, g)
    nw = (1.0 + 0.1 * torch.randn(H, generator=g)).to(BF16)
    xp = ops.PackedActivations(m, H, DEV).pack(x.to(DEV), norm_w=nw.to(DEV))
    lm = ops.TcLmHeadArgmax(m, V, H, DEV)
    tok = torch.full((m,), -1, dtype=torch.int64, device=DEV)
    pos = torch.tensor([7], dtype=torch.int64, device=DEV)
    logits = torch.empty((m, V), dtype=BF16, device=DEV)
    lm(xp, ops.pack_matrix(E.to(DEV)), tok, pos, inc_pos=True, logits=logits)
    ref = (_norm_ref(x, nw, eps).float() @ E.float().T).to(BF16)
    _assert_bf16_close(logits, ref)
    lo = logits.cpu()
    for i in range(m):
        t = int(tok[i])
        assert t == int(Q.argmax_lowest(lo[i:i + 1]))
        assert Q.token_ok(t, ref[i], 2.0 ** -6 * float(ref[i].float().abs().max()))
    assert int(pos.item()) == 8


def test_tc_lm_head_ties_pick_lowest_index():
    ops = _ops()
    V, H, m = 1024, 128, 16
    x = torch.zeros((m, H), dtype=BF16)
    x[:, 0] = 1.0
    E = torch.zeros((V, H), dtype=BF16)
    for r in (700, 300, 900):
        E[r, 0] = 2.0
    xp = ops.PackedActivations(m, H, DEV).pack(x.to(DEV))
    lm = ops.TcLmHeadArgmax(m, V, H, DEV)
    tok = torch.empty((m,), dtype=torch.int64, device=DEV)
    lm(xp, ops.pack_matrix(E.to(DEV)), tok)
    assert (tok.cpu() == 300).all()


@pytest.mark.parametrize("m", [16, 40])
def test_tc_swiglu_packed_output_is_packed_rowmajor(m):
    """SWIGLU_PACKED writes exactly what packing the row-major SwiGLU output would."""
    ops = _ops()
    inter, k = 9728, 2560
    g = torch.Generator().manual_seed(77 + m)
    x, gate, up = _rand((m, k), 1.0, g), _rand((inter, k), 0.02, g), _rand((inter, k), 0.02, g)
    xp = ops.PackedActivations(m, k, DEV).pack(x.to(DEV))
    w = ops.pack_gate_up(gate.to(DEV), up.to(DEV))
    row = torch.empty((m, inter), dtype=BF16, device=DEV)
    ops.TcGemv(m, 2 * inter, k, ops.TcGemv.SWIGLU, DEV)(xp, w, row)
    packed = ops.PackedActivations(m, inter, DEV)
    ops.TcGemv(m, 2 * inter, k, ops.TcGemv.SWIGLU_PACKED, DEV)(xp, w, packed)
    ref = ops.PackedActivations(m, inter, DEV).pack(row)
    assert torch.equal(packed.t.view(torch.int16), ref.t.view(torch.int16))


@pytest.mark.parametrize("n,k", [(2560, 4096), (2560, 9728)])
@pytest.mark.parametrize("m", [13, 32, 64])
def test_tc_gemv_deferred_residual_sums(n, k, m):
    """QD_EPI_RES_SUMS + qd_pack_act_res: the projection's split-K partials go into fixed-point sums, the
    packing adds them to the residual stream (x written back) and clears them; x against the fp64
    reference as in the residual test, the packed operand equal to packing the new x, the sums zero after,
    and a second round on the cleared sums gives the same bytes."""
    ops = _ops()
    g = torch.Generator().manual_seed(n + k + 7 * m)
    x, w, res = _rand((m, k), 1.0, g), _rand((n, k), 0.02, g), _rand((m, n), 1.0, g)
    nw = (1.0 + 0.1 * torch.randn(n, generator=g)).to(BF16).to(DEV)
    xp = ops.PackedActivations(m, k, DEV).pack(x.to(DEV))
    wp = ops.pack_matrix(w.to(DEV))
    plan = ops.TcGemv(m, n, k, ops.TcGemv.RES_SUMS, DEV)
    sums = torch.zeros((m, n), dtype=torch.int64, device=DEV)
    outs = []
    for _ in range(2):
        xr = res.to(DEV).clone()
        plan(xp, wp, sums)
        packed = ops.PackedActivations(m, n, DEV).pack_res(xr, sums, nw)
        torch.cuda.synchronize()
        assert int(sums.abs().sum()) == 0
        outs.append((xr.clone(), packed.t.clone()))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
    xr, pk = outs[0]
    y = _gemv_ref(x, w, None, 0).to(BF16).float()
    ref = (res.float() + y).to(BF16)
    diff = (xr.float().cpu() - ref.float()).abs()
    tol = RTOL * (ref.float().abs() + y.abs()) + 1e-3
    assert not (diff > tol).any(), f"{int((diff > tol).sum())} mismatches, max diff {float(diff.max()):.4g}"
    assert torch.equal(pk, ops.PackedActivations(m, n, DEV).pack(xr, nw).t)


@pytest.mark.parametrize("m", [13, 64])
@pytest.mark.parametrize("pos", [0, 700])
def test_tc_qkv_store_sums_then_rope_epilogue(m, pos):
    """QD_EPI_STORE_SUMS + qd_qkv_rope_sums (the chain's QKV without a split-K last arriver) against the
    fused qd_tc_qkv_rope_append on the same inputs: q, k and v within the rope tolerance (the projection
    sums differ only in summation order, fixed point against fp32), the sums cleared, the rest of the
    cache untouched, and a second round on the cleared sums giving the same bytes."""
    ops = _ops()
    H, nq, nkv, D, cap, eps = 2560, 32, 8, 128, 1024, 1e-6
    g = torch.Generator().manual_seed(m * 31 + pos)
    x = _rand((m, H), 1.0, g)
    w = _rand(((nq + 2 * nkv) * D, H), 0.02, g)
    ln = (1.0 + 0.1 * torch.randn(H, generator=g)).to(BF16).to(DEV)
    qn = (1.0 + 0.1 * torch.randn(D, generator=g)).to(BF16).to(DEV)
    kn = (1.0 + 0.1 * torch.randn(D, generator=g)).to(BF16).to(DEV)
    cos, sin = (t.to(DEV) for t in Q.rope_tables(cap, D, 5e6))
    xp = ops.PackedActivations(m, H, DEV).pack(x.to(DEV), norm_w=ln)
    wp = ops.pack_matrix(w.to(DEV))
    posd = torch.tensor([pos], dtype=torch.int64, device=DEV)

    def caches():
        return (torch.full((m, nkv, cap, D), float("nan"), dtype=BF16, device=DEV),
                torch.full((m, nkv, cap, D), float("nan"), dtype=BF16, device=DEV),
                torch.empty((m, nq, D), dtype=BF16, device=DEV))

    kr, vr, qr = caches()
    raw = torch.empty((m, (nq + 2 * nkv) * D), dtype=BF16, device=DEV)
    ops.TcQkvRopeAppend(m, H, nq, nkv, DEV)(xp, wp, qn, kn, cos, sin, posd, qr, kr, vr, raw_out=raw)
    mm = ops.TcGemv(m, (nq + 2 * nkv) * D, H, ops.TcGemv.STORE_SUMS, DEV)
    sums = torch.zeros((m, (nq + 2 * nkv) * D), dtype=torch.int64, device=DEV)
    outs = []
    for _ in range(2):
        kc, vc, q = caches()
        mm(xp, wp, sums)
        ops.qkv_rope_sums(sums, m, nq, nkv, qn, kn, eps, cos, sin, posd, q, kc, vc)
        torch.cuda.synchronize()
        assert int(sums.abs().sum()) == 0
        outs.append((q.clone(), kc[:, :, pos].clone(), vc[:, :, pos].clone()))
        others = torch.ones(cap, dtype=torch.bool)
        others[pos] = False
        assert torch.isnan(kc[:, :, others].float()).all() and torch.isnan(vc[:, :, others].float()).all()
    for a, b in zip(outs[0], outs[1]):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    rc = raw.cpu()
    y_q = Q.rms_norm(rc, qn.cpu(), eps, nq)
    y_k = Q.rms_norm(rc[:, nq * D:], kn.cpu(), eps, nkv)
    _assert_rope_close(outs[0][0], qr.cpu(), y_q, cos[pos].cpu(), sin[pos].cpu())
    _assert_rope_close(outs[0][1], kr[:, :, pos].cpu(), y_k, cos[pos].cpu(), sin[pos].cpu())
    _assert_bf16_close(outs[0][2], vr[:, :, pos])
