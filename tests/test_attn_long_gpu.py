"""GQA decode attention at the cache lengths of BASELINE config 3 (B in {1, 8, 32}, KV length up to
32768), where the split count and the log-sum-exp merge over many splits matter most.

Kernels: qd_attn_decode (the team kernel; the batch 1-3 persistent step runs the same device code) and
qd_attn_decode_tc (tcgen05; the batch path), plus the CUDA-core streaming kernel on the largest cases.
Each output is checked against the oracle's SDPA restatement (engine/engine.py:633-636, one sequence at
a time to bound host memory) and an fp32 math reference (scores and softmax in fp32, no BF16 rounding
of the probabilities) within 2e-2 absolute, the bound of the other attention tests. Cache slots past
the valid length hold NaN, so a read beyond it shows as a non-finite output. Split-boundary cases put
the valid length one key before, on and after the end of a split (the reference's split/merge:
engine/kernels/decode_attn.py:26-119)."""

import math

import pytest
import torch

from oracle import qwen3_cpu as Q

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16
DEV = "cuda:0"
NQ, NKV, D = 32, 8, 128
TOL = 2e-2


def _inputs(B, L, cap, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn((B, NQ, D), generator=g).to(BF16)
    kc = torch.full((B, NKV, cap, D), float("nan"), dtype=BF16)
    vc = torch.full((B, NKV, cap, D), float("nan"), dtype=BF16)
    kc[:, :, :L] = torch.randn((B, NKV, L, D), generator=g).to(BF16)
    vc[:, :, :L] = torch.randn((B, NKV, L, D), generator=g).to(BF16)
    return q, kc, vc


def _references(q, kc, vc, L):
    """(oracle SDPA, fp32 math) outputs [B, 32, 128] float, sequence by sequence."""
    B = q.shape[0]
    sdpa, f32 = [], []
    for b in range(B):
        sdpa.append(Q.attention_decode(q[b:b + 1], kc[b:b + 1], vc[b:b + 1], L).float())
        qg = q[b].float().view(NKV, NQ // NKV, D)                 # query heads grouped by KV head
        k, v = kc[b, :, :L].float(), vc[b, :, :L].float()          # [8, L, 128]
        p = torch.softmax(torch.einsum("hgd,hnd->hgn", qg, k) / math.sqrt(D), -1)
        f32.append(torch.einsum("hgn,hnd->hgd", p, v).reshape(1, NQ, D))
    return torch.cat(sdpa), torch.cat(f32)


def _run(kind, q, kc, vc, L, cap):
    from decode_b200 import ops

    B = q.shape[0]
    cls = {"team": ops.DecodeAttention, "tc": ops.DecodeAttentionTc, "stream": ops.DecodeAttentionStream}[kind]
    attn = cls(B, NQ, NKV, cap, DEV)
    out = torch.full((B, NQ, D), float("nan"), dtype=BF16, device=DEV)
    err = torch.zeros((1,), dtype=torch.int32, device=DEV)
    pos = torch.tensor([L - 1], dtype=torch.int64, device=DEV)
    kd, vd = kc.to(DEV), vc.to(DEV)
    attn(q.to(DEV), kd, vd, pos, out, err=err)
    again = torch.empty_like(out)
    attn(q.to(DEV), kd, vd, pos, again, err=err)  # same plan, same inputs: bit-identical (tickets reset)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(out, again)
    return attn, out.float().cpu()


def _check(o, q, kc, vc, L, what):
    assert torch.isfinite(o).all(), what
    sdpa, f32 = _references(q, kc, vc, L)
    d1, d2 = (o - sdpa).abs().max().item(), (o - f32).abs().max().item()
    print(f"{what}: max |out - oracle| {d1:.2e}, max |out - fp32| {d2:.2e}")
    assert d1 < TOL and d2 < TOL, (what, d1, d2)


@pytest.mark.parametrize("B,L", [(1, 8192), (1, 32768), (8, 8192), (8, 32768), (32, 8192)])
@pytest.mark.parametrize("kind", ["team", "tc"])
def test_attention_at_config3_lengths(kind, B, L):
    cap = L + 64  # poisoned slots past the valid length
    q, kc, vc = _inputs(B, L, cap, seed=2 + B * 100003 + L)
    _, o = _run(kind, q, kc, vc, L, cap)
    _check(o, q, kc, vc, L, f"{kind} B{B} L{L}")


@pytest.mark.parametrize("B,L", [(32, 32768), (8, 32768)])
def test_streaming_kernel_at_the_longest_caches(B, L):
    cap = L + 64
    q, kc, vc = _inputs(B, L, cap, seed=11 + B + L)
    _, o = _run("stream", q, kc, vc, L, cap)
    _check(o, q, kc, vc, L, f"stream B{B} L{L}")


def test_tc_attention_b32_l32768():
    B, L = 32, 32768
    cap = L
    q, kc, vc = _inputs(B, L, cap, seed=77)
    _, o = _run("tc", q, kc, vc, L, cap)
    _check(o, q, kc, vc, L, f"tc B{B} L{L}")


@pytest.mark.parametrize("B", [1, 8])
@pytest.mark.parametrize("delta", [-1, 0, 1])
def test_team_attention_at_a_split_boundary(B, delta):
    """Valid length one key before, on and one after the end of a middle split of the team kernel's
    plan (the plan splits the capacity into `splits` chunks of `chunk` keys)."""
    from decode_b200 import ops

    cap = 8192
    plan = ops.DecodeAttention(B, NQ, NKV, cap, DEV)
    assert plan.splits >= 2, plan.splits
    L = max(1, plan.splits // 2) * plan.chunk + delta
    q, kc, vc = _inputs(B, L, cap, seed=900 + B * 3 + delta)
    _, o = _run("team", q, kc, vc, L, cap)
    _check(o, q, kc, vc, L, f"team B{B} L{L} (chunk {plan.chunk}, {plan.splits} splits)")


@pytest.mark.parametrize("B", [1, 8])
@pytest.mark.parametrize("delta", [-1, 0, 1])
def test_tc_attention_at_a_chunk_boundary(B, delta):
    """Valid length one key before, on and one after a multiple of the tensor-core kernel's 128-key
    chunk, and at a length whose chunk count divides unevenly over the CTAs."""
    cap = 8192
    L = 128 * 37 + delta
    q, kc, vc = _inputs(B, L, cap, seed=700 + B * 3 + delta)
    _, o = _run("tc", q, kc, vc, L, cap)
    _check(o, q, kc, vc, L, f"tc B{B} L{L}")
