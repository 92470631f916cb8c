"""The allocation-free GEMV entry point (qd_gemv_noalloc) against the regular one (qd_gemv).

qd_gemv_noalloc exists for callers that cannot allocate device memory - a host whose device memory
is owned end to end by its own pool allocator, a plugin inside such a host without an allocator
handle, or a latency-critical loop that must not call cudaMalloc because it can synchronize the
device. Its scratch is a fixed 4 MiB array inside the library instead of a caller buffer. This test
calls it through the C ABI (ctypes) several times in a row, including a change of shape (which must
not inherit the previous call's tickets) and a repeat of the first shape after it, and compares every
output with qd_gemv's. Both entry points run the same plan and grid, and the split-K partial sums are
added in a fixed CTA order, so the outputs must be bit-identical: a stale ticket or partial left in the
shared array by an earlier call would show as a difference of even one ulp. Collected last so a
failure here leaves every other result in place; it also passes alone in a fresh process.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16
DEV = "cuda:0"


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _noalloc(lib, x, w, n, k, m, out, res, norm_w, epi):
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    err = torch.zeros((1,), dtype=torch.int32, device=DEV)
    rc = lib.qd_gemv_noalloc(_p(x), x.stride(0), _p(w), n, k, m, _p(out), out.stride(0), _p(res),
                             res.stride(0) if res is not None else 0, _p(norm_w), 1e-6, epi, _p(err), 1, stream)
    assert rc == 0, lib.qd_last_error()
    torch.cuda.synchronize()
    assert int(err.item()) == 0


def _same(a, b, what):
    assert torch.equal(a, b), (what, float((a.float() - b.float()).abs().max()))


def test_noalloc_matches_regular_gemv_on_consecutive_calls():
    from decode_b200 import lib as L
    from decode_b200 import ops

    lib = L.load()
    g = torch.Generator().manual_seed(7)
    cases = [  # (m, n, k, epilogue, norm): gate/up + SwiGLU twice, the O-projection shape with residual,
        # the down-projection shape, and gate/up once more after the shape changes
        (3, 19456, 2560, ops.Gemv.SWIGLU, True),
        (3, 19456, 2560, ops.Gemv.SWIGLU, True),
        (2, 2560, 4096, ops.Gemv.RES, False),
        (1, 2560, 9728, ops.Gemv.RES, False),
        (3, 19456, 2560, ops.Gemv.SWIGLU, True),
    ]
    for i, (m, n, k, epi, norm) in enumerate(cases):
        x = (torch.randn((m, k), generator=g)).to(BF16).to(DEV)
        w = ops.pack_matrix((torch.randn((n, k), generator=g) * 0.02).to(BF16).to(DEV))
        nw = (1.0 + 0.1 * torch.randn(k, generator=g)).to(BF16).to(DEV) if norm else None
        cols = n // 2 if epi == ops.Gemv.SWIGLU else n
        res = (torch.randn((m, cols), generator=g)).to(BF16).to(DEV) if epi == ops.Gemv.RES else None
        ref = torch.empty((m, cols), dtype=BF16, device=DEV)
        if res is not None:
            ref.copy_(res)
        ops.Gemv(m, n, k, epi, DEV)(x, w, ref, res=ref if res is not None else None, norm_w=nw)
        out = torch.full((m, cols), float("nan"), dtype=BF16, device=DEV)
        if res is not None:
            out.copy_(res)
        _noalloc(lib, x, w, n, k, m, out, out if res is not None else None, nw, epi)
        _same(out, ref, (i, m, n, k))


def test_noalloc_rejects_oversized_plans():
    from decode_b200 import lib as L

    lib = L.load()
    x = torch.zeros((8, 2560), dtype=BF16, device=DEV)
    w = torch.zeros((151936 * 2560,), dtype=BF16, device=DEV)
    out = torch.zeros((8, 151936), dtype=BF16, device=DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.qd_gemv_noalloc(_p(x), 2560, _p(w), 151936, 2560, 8, _p(out), 151936, None, 0, None, 1e-6, 0,
                             None, 1, stream)
    assert rc == 4 and b"scratch" in lib.qd_last_error()
