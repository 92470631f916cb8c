"""Streaming split-K GQA flash-decode (qd_attn_decode_stream, CUDA cores, and qd_attn_decode_tc, tcgen05
tensor cores) on the GPU against the oracle's SDPA restatement and an fp32 math reference, through the
C ABI. Grids are varied so that CTAs end one (sequence, KV head) pair and start the next, and pairs are
merged from up to dozens of segments."""

import math

import pytest
import torch

from oracle import qwen3_cpu as Q

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16
DEV = "cuda:0"


def _cls(kind):
    from decode_b200 import ops

    return ops.DecodeAttentionTc if kind == "tc" else ops.DecodeAttentionStream


def _rand(shape, std, gen):
    return (torch.randn(shape, generator=gen) * std).to(BF16)


@pytest.mark.parametrize("B,L,cap,grid", [(1, 1, 384, 0), (1, 33, 384, 0), (1, 384, 384, 0), (3, 200, 256, 0),
                                          (8, 1000, 1024, 0), (2, 64, 65, 0), (1, 4096, 8192, 0),
                                          (64, 1280, 1536, 0), (5, 777, 800, 7), (5, 777, 800, 37),
                                          (16, 300, 320, 1000), (32, 1024, 1024, 0),
                                          # the tensor-core kernel's last chunk in 32-key boxes: exactly
                                          # one box, a box one key short, a box past the capacity
                                          (2, 160, 192, 0), (4, 255, 256, 0), (3, 70, 72, 0)])
@pytest.mark.parametrize("kind", ["stream", "tc"])
def test_stream_attention_matches_oracle(B, L, cap, grid, kind):
    from decode_b200 import ops

    nq, nkv, D = 32, 8, 128
    g = torch.Generator().manual_seed(B * 7919 + L + grid)
    q = _rand((B, nq, D), 1.0, g)
    kc = torch.full((B, nkv, cap, D), float("nan"), dtype=BF16)     # poisoned beyond the valid length
    vc = torch.full((B, nkv, cap, D), float("nan"), dtype=BF16)
    kc[:, :, :L] = _rand((B, nkv, L, D), 1.0, g)
    vc[:, :, :L] = _rand((B, nkv, L, D), 1.0, g)
    attn = _cls(kind)(B, nq, nkv, cap, DEV, grid=grid)
    out = torch.empty((B, nq, D), dtype=BF16, device=DEV)
    err = torch.zeros((1,), dtype=torch.int32, device=DEV)
    pos = torch.tensor([L - 1], dtype=torch.int64, device=DEV)
    attn(q.to(DEV), kc.to(DEV), vc.to(DEV), pos, out, err=err)
    assert int(err.item()) == 0
    o = out.float().cpu()
    assert torch.isfinite(o).all()
    ref = Q.attention_decode(q, kc, vc, L)
    assert (o - ref.float()).abs().max().item() < 2e-2
    s = torch.einsum("bhd,bhnd->bhn", q.float(), Q.repeat_kv(kc[:, :, :L]).float()) / math.sqrt(D)
    ref32 = torch.einsum("bhn,bhnd->bhd", torch.softmax(s, -1), Q.repeat_kv(vc[:, :, :L]).float())
    assert (o - ref32).abs().max().item() < 2e-2


@pytest.mark.parametrize("kind", ["stream", "tc"])
def test_stream_attention_deterministic_across_calls_and_lengths(kind):
    """Fixed grid: bit-identical results on repeated calls (tickets reset themselves), and a shorter
    valid length on the same plan reads only its keys."""
    from decode_b200 import ops

    B, nq, nkv, D, cap = 4, 32, 8, 128, 2048
    g = torch.Generator().manual_seed(3)
    q = _rand((B, nq, D), 1.0, g).to(DEV)
    kc = _rand((B, nkv, cap, D), 1.0, g).to(DEV)
    vc = _rand((B, nkv, cap, D), 1.0, g).to(DEV)
    attn = _cls(kind)(B, nq, nkv, cap, DEV)
    outs = []
    for L in (2000, 2000, 2000, 150, 2000):
        out = torch.empty((B, nq, D), dtype=BF16, device=DEV)
        attn(q, kc, vc, torch.tensor([L - 1], dtype=torch.int64, device=DEV), out)
        outs.append(out)
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2]) and torch.equal(outs[0], outs[4])
    ref = Q.attention_decode(q.cpu(), kc.cpu(), vc.cpu(), 150)
    assert (outs[3].float().cpu() - ref.float()).abs().max().item() < 2e-2


@pytest.mark.parametrize("kind", ["stream", "tc"])
def test_stream_attention_flags_position_outside_cache(kind):
    from decode_b200 import ops

    B, nq, nkv, D, cap = 1, 32, 8, 128, 64
    g = torch.Generator().manual_seed(4)
    q = _rand((B, nq, D), 1.0, g).to(DEV)
    kc = _rand((B, nkv, cap, D), 1.0, g).to(DEV)
    vc = _rand((B, nkv, cap, D), 1.0, g).to(DEV)
    attn = _cls(kind)(B, nq, nkv, cap, DEV)
    out = torch.empty((B, nq, D), dtype=BF16, device=DEV)
    err = torch.zeros((1,), dtype=torch.int32, device=DEV)
    attn(q, kc, vc, torch.tensor([cap + 5], dtype=torch.int64, device=DEV), out, err=err)  # clamped, flagged
    assert int(err.item()) == 16
    ref = Q.attention_decode(q.cpu(), kc.cpu(), vc.cpu(), cap)
    assert (out.float().cpu() - ref.float()).abs().max().item() < 2e-2


@pytest.mark.parametrize("B", [9, 33, 64])
def test_tc_attention_packed_output_is_packed_rowmajor(B):
    """out_npad > 0 writes the O projection's packed operand: bit-equal to packing the [B, 32, 128] output."""
    from decode_b200 import ops

    nq, nkv, D, cap, L = 32, 8, 128, 640, 600
    g = torch.Generator().manual_seed(B)
    q = _rand((B, nq, D), 1.0, g).to(DEV)
    kc = _rand((B, nkv, cap, D), 1.0, g).to(DEV)
    vc = _rand((B, nkv, cap, D), 1.0, g).to(DEV)
    attn = ops.DecodeAttentionTc(B, nq, nkv, cap, DEV)
    pos = torch.tensor([L - 1], dtype=torch.int64, device=DEV)
    row = torch.empty((B, nq, D), dtype=BF16, device=DEV)
    attn(q, kc, vc, pos, row)
    packed = ops.PackedActivations(B, nq * D, DEV)
    attn(q, kc, vc, pos, packed)
    ref = ops.PackedActivations(B, nq * D, DEV).pack(row.view(B, -1))
    assert torch.equal(packed.t.view(torch.int16), ref.t.view(torch.int16))
